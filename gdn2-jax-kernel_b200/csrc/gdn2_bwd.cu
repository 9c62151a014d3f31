// GDN-2 fused backward: the reverse state pass (B1 with B2's dv_partial,
// gdn2_bwd.py:45-80, 84-96) and three intra-chunk passes (B2's dAqk, B3, B4,
// B5 and the final assembly of gdn2_pipeline.py:117-137).
#include "gdn2_b4_exact.cuh"
#include "gdn2_kernels.cuh"

namespace gdn2 {

constexpr float kFinalClip = 1e4f;   // gdn2_pipeline.py:34

// ---------------------------------------------------------------------------
// Reverse state pass, serial over chunks; each CTA owns NV value columns of
// one (batch, head) dh:
//   dv_partial = san(Aqk^T do)                       (B2, gdn2_bwd.py:93)
//   dv_new     = san(dv_partial + kg dh)             (gdn2_bwd.py:66-68)
//   dh         = san(qg^T (scale do) + e^{gc_last} dh - W^T dv_new)
// dv_new and dh (the dh_pre of each chunk) go to the workspace; dh0 is written
// with the final +-1e4 sanitiser.
// ---------------------------------------------------------------------------
template <int C, int D, int NV>
__global__ void __launch_bounds__(kThreads, 2)
k_bwd_state(Problem p, Workspace ws, const float* __restrict__ dout,
            const float* __restrict__ dh_final, float* __restrict__ dh0, bool only_flagged,
            bool pair) {
  using T1 = typename TileFor<C, NV>::type;
  using T3 = typename TileFor<D, NV>::type;
  constexpr int LDC = C + 4, LDD = D + 4;
  extern __shared__ __align__(16) float sm[];
  float* X = sm;
  float* sdh = X + StateSmem<C, D, NV>::BIG;   // [D][NV]
  float* sdo = sdh + D * NV;                    // [C][NV]
  float* sdv = sdo + C * NV;                    // [C][NV]
  const int v0 = blockIdx.x * NV, h = blockIdx.y, bb = blockIdx.z;
  const size_t bh = (size_t)bb * p.H + h;
  const long rs = p.row_stride();
  // Exact recompute of the (b, h) the tensor-core scan's guard flagged.
  if (only_flagged && ws.bnd[bh * p.nc * 4 + 3] == 0.f) return;

  for (int e = threadIdx.x; e < D * NV; e += kThreads) {
    const int d = e / NV, vv = e % NV;
    sdh[e] = dh_final ? san(dh_final[bh * D * D + d * D + v0 + vv], p.clip) : 0.f;
  }
  // pair: 64-row chunks of the tensor-core workspace, two per 128-row tile;
  // the row-major arrays (kg, dv) line up with 64-row chunks, the transposed
  // tile arrays (Aqk^T, qg^T, W^T) are read at the tile's row stride.
  const long tld = pair ? 2 * C : C;
  for (int c = p.nc - 1; c >= 0; --c) {
    const size_t chunk = bh * p.nc + c;
    const size_t tile = pair ? chunk >> 1 : chunk;
    const int hoff = pair ? (int)(chunk & 1) * C : 0;
    const float* doc = dout + ((long)bb * p.T + (long)c * C) * rs + (long)h * D + v0;
    load_tile<float>(sdo, NV, doc, rs, C, NV);
    load_tile_T<float>(X, LDC, ws.AqkT + tile * tld * tld + hoff * tld + hoff, tld, C, C);   // X[i][j] = Aqk(i,j)
    __syncthreads();
    T1 tp;
    tp.zero();
    tp.mma(X, LDC, sdo, NV, tp.r0, C);
    __syncthreads();
    load_tile_T<float>(X, LDC, ws.kg + chunk * C * D, D, C, D);     // X[d][i] = kg(i,d)
    __syncthreads();
    {
      T1 t;
      t.zero();
      t.mma(X, LDC, sdh, NV, 0, D);
      float* dvo = ws.dv + chunk * C * D;
#pragma unroll
      for (int ii = 0; ii < T1::TM_; ++ii) {
        const int i = t.r0 + ii;
        float o4[T1::TN_];
#pragma unroll
        for (int jj = 0; jj < T1::TN_; ++jj)
          o4[jj] = san(san(tp.acc[ii][jj], p.clip) + t.acc[ii][jj], p.clip);
        store_vec<T1::TN_>(sdv + i * NV + t.c0, o4);
        store_vec<T1::TN_>(dvo + i * D + v0 + t.c0, o4);
      }
    }
    __syncthreads();
    load_tile_T<float>(X, LDD, ws.qgT + tile * tld * D + hoff, tld, D, C);    // X[i][d] = qg(i,d)
    __syncthreads();
    T3 ta;
    ta.zero();
    ta.mma(X, LDD, sdo, NV, 0, C);
    __syncthreads();
    load_tile_T<float>(X, LDD, ws.WT + tile * tld * D + hoff, tld, D, C);     // X[i][d] = W(i,d)
    __syncthreads();
    {
      T3 tb;
      tb.zero();
      tb.mma(X, LDD, sdv, NV, 0, C);
      const float* gl = ws.gcl + chunk * D;
      float* dho = ws.dh + chunk * D * D;
#pragma unroll
      for (int ii = 0; ii < T3::TM_; ++ii) {
        const int d = ta.r0 + ii;
        const float dec = __expf(gl[d]);
        float o4[T3::TN_];
#pragma unroll
        for (int jj = 0; jj < T3::TN_; ++jj) {
          const float cur = sdh[d * NV + ta.c0 + jj];
          o4[jj] = san(p.scale * ta.acc[ii][jj] + dec * cur - tb.acc[ii][jj], p.clip);
        }
        store_vec<T3::TN_>(sdh + d * NV + ta.c0, o4);
        store_vec<T3::TN_>(dho + d * D + v0 + ta.c0, o4);
      }
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < D * NV; e += kThreads)
    dh0[bh * D * D + (e / NV) * D + v0 + e % NV] = san(sdh[e], kFinalClip);
}

// ---------------------------------------------------------------------------
// Intra pass 1 (B2's dAqk and the state-facing half of B3, gdn2_bwd.py:84-96,
// 152-159, 182-201):
//   dqg = scale do h_pre^T, dWp = -dv h_pre^T, dkg = vnew dh_next^T,
//   dAqk = san((do vnew^T) * causal).
// Writes san(dq_B3) to pdq, the raw partial dk (kg branch) to pdk, the raw
// partial dgc (qg and kg branches plus the gc_last row) to pdgc, dWp and
// dAqk^T.
// ---------------------------------------------------------------------------
template <typename T, int C, int D>
__global__ void __launch_bounds__(kThreads, 1)
k_bwd_intra1(const T* __restrict__ q, const T* __restrict__ k, const float* __restrict__ dout,
             const float* __restrict__ dh_final, Problem p, Workspace ws) {
  using TD = typename TileFor<C, D>::type;
  using TC = typename TileFor<C, C>::type;
  constexpr int LDC = C + 4, LDD = D + 4;
  constexpr int P = C > D ? C : D, BIG = P * (P + 4);
  extern __shared__ __align__(16) float sm[];
  float* X1 = sm;
  float* X2 = X1 + BIG;
  float* X3 = X2 + BIG;
  float* colpart = X3 + BIG;  // [C/TM][D] per-row-group column partials
  const int c = blockIdx.x, h = blockIdx.y, bb = blockIdx.z;
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const size_t bh = (size_t)bb * p.H + h, chunk = bh * p.nc + c;
  const T *qc = q + off, *kc = k + off;
  const float* gc = ws.gc + chunk * C * D;
  const float* hpre = ws.hpre + chunk * D * D;
  const float* dhn = (c + 1 < p.nc) ? ws.dh + (chunk + 1) * D * D : dh_final + bh * D * D;
  float *pdq = ws.pdq + chunk * C * D, *pdk = ws.pdk + chunk * C * D,
        *pdgc = ws.pdgc + chunk * C * D;

  load_tile_T<float>(X1, LDC, dout + off, rs, C, D);                // X1[v][i] = do(i,v)
  load_tile_T<float>(X2, LDD, hpre, D, D, D);                       // X2[v][dk] = hpre(dk,v)
  load_tile_T<float>(X3, LDC, ws.dv + chunk * C * D, D, C, D);      // X3[v][i] = dv(i,v)
  __syncthreads();
  {
    TD t;
    t.zero();
    t.mma(X1, LDC, X2, LDD, 0, D);
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      const int i = t.r0 + ii;
      float oq[TD::TN_], og[TD::TN_];
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        const int d = t.c0 + jj;
        const float eg = __expf(gc[i * D + d]);
        const float dqg = p.scale * t.acc[ii][jj];
        oq[jj] = san(dqg * eg, p.clip);
        og[jj] = dqg * (to_f<T>(qc[i * rs + d]) * eg);
      }
      store_vec<TD::TN_>(pdq + i * D + t.c0, oq);
      store_vec<TD::TN_>(pdgc + i * D + t.c0, og);
    }
    t.zero();
    t.mma(X3, LDC, X2, LDD, 0, D);
    float* dwp = ws.dWp + chunk * C * D;
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      float o4[TD::TN_];
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) o4[jj] = -t.acc[ii][jj];
      store_vec<TD::TN_>(dwp + (t.r0 + ii) * D + t.c0, o4);
    }
  }
  __syncthreads();
  load_tile_T<float>(X2, LDC, ws.vnew + chunk * C * D, D, C, D);    // X2[v][j] = vnew(j,v)
  __syncthreads();
  {
    TC t;
    t.zero();
    if (t.c0 <= t.r0) t.mma(X1, LDC, X2, LDC, 0, D);
    float* out = ws.dAqkT + chunk * C * C;
#pragma unroll
    for (int jj = 0; jj < TC::TN_; ++jj) {
      const int j = t.c0 + jj;
      float o4[TC::TM_];
#pragma unroll
      for (int ii = 0; ii < TC::TM_; ++ii)
        o4[ii] = (j <= t.r0 + ii) ? san(t.acc[ii][jj], p.clip) : 0.f;
      store_vec<TC::TM_>(out + j * C + t.r0, o4);
    }
  }
  __syncthreads();
  load_tile_T<float>(X1, LDD, dhn, D, D, D);                        // X1[v][dk] = dhn(dk,v)
  __syncthreads();
  {
    TD t;
    t.zero();
    t.mma(X2, LDC, X1, LDD, 0, D);
    const float* gl = gc + (C - 1) * D;
    float cs[TD::TN_];
#pragma unroll
    for (int jj = 0; jj < TD::TN_; ++jj) cs[jj] = 0.f;
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      const int i = t.r0 + ii;
      float ok[TD::TN_], og[TD::TN_];
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        const int d = t.c0 + jj;
        const float f = __expf(gl[d] - gc[i * D + d]);
        const float dkg = t.acc[ii][jj];
        const float x = dkg * (to_f<T>(kc[i * rs + d]) * f);
        ok[jj] = dkg * f;
        og[jj] = pdgc[i * D + d] - x;
        cs[jj] += x;
      }
      store_vec<TD::TN_>(pdk + i * D + t.c0, ok);
      store_vec<TD::TN_>(pdgc + i * D + t.c0, og);
    }
    store_vec<TD::TN_>(colpart + (t.r0 / TD::TM_) * D + t.c0, cs);
  }
  __syncthreads();
  // gc_last row: sum_i dkg*kg + e^{gc_last} * sum_v dh_next * h_pre (gdn2_bwd.py:185, 196-201)
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float s = 0.f;
    for (int vv = 0; vv < D; ++vv) s = fmaf(dhn[d * D + vv], hpre[d * D + vv], s);
    float cs = 0.f;
    for (int r = 0; r < C / TD::TM_; ++r) cs += colpart[r * D + d];   // fixed order
    const float gl = gc[(C - 1) * D + d];
    pdgc[(C - 1) * D + d] += cs + __expf(gl) * s;
  }
}

// ---------------------------------------------------------------------------
// Intra pass 2 (the WY half of B3, gdn2_bwd.py:161-193):
//   dA = san(dWp kb^T + dv wv^T); tmp = san(dA A^T); dAkk = -(A^T tmp) * strict
//   dkb = A^T dWp; dwv = A^T dv  ->  dk, db, dgc partials; dw, dv final.
// ---------------------------------------------------------------------------
template <typename T, int C, int D, bool GATES>
__global__ void __launch_bounds__(kThreads, 1)
k_bwd_intra2(const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ w,
             const T* __restrict__ b, T* __restrict__ dv_out, T* __restrict__ dw_out, Problem p,
             Workspace ws) {
  using TD = typename TileFor<C, D>::type;
  using TC = typename TileFor<C, C>::type;
  constexpr int LDC = C + 4, LDD = D + 4;
  constexpr int P = C > D ? C : D, BIG = P * (P + 4);
  extern __shared__ __align__(16) float sm[];
  float* X1 = sm;
  float* X2 = X1 + BIG;
  const int c = blockIdx.x, h = blockIdx.y, bb = blockIdx.z;
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const size_t chunk = ((size_t)bb * p.H + h) * p.nc + c;
  const T *kc = k + off, *vc = v + off, *wc = w + off, *bc = b + off;
  const float* gc = ws.gc + chunk * C * D;

  load_tile_T<float>(X1, LDC, ws.dWp + chunk * C * D, D, C, D);     // X1[d][i] = dWp(i,d)
  for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
    const int j = e % C, d = (e / C) * 4;
    const float4 kv = ld4<T>(kc + j * rs + d), bv = ld4_gate<T>(bc + j * rs + d, GATES, kGateB);
    const float* g4 = gc + j * D + d;
    X2[(d + 0) * LDC + j] = bv.x * kv.x * __expf(g4[0]);
    X2[(d + 1) * LDC + j] = bv.y * kv.y * __expf(g4[1]);
    X2[(d + 2) * LDC + j] = bv.z * kv.z * __expf(g4[2]);
    X2[(d + 3) * LDC + j] = bv.w * kv.w * __expf(g4[3]);
  }
  __syncthreads();
  TC ta;
  ta.zero();
  ta.mma(X1, LDC, X2, LDC, 0, D);
  __syncthreads();
  load_tile_T<float>(X1, LDC, ws.dv + chunk * C * D, D, C, D);      // X1[d][i] = dv(i,d)
  for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
    const int j = e % C, d = (e / C) * 4;
    const float4 wv = ld4_gate<T>(wc + j * rs + d, GATES, kGateW), vv = ld4<T>(vc + j * rs + d);
    X2[(d + 0) * LDC + j] = wv.x * vv.x;
    X2[(d + 1) * LDC + j] = wv.y * vv.y;
    X2[(d + 2) * LDC + j] = wv.z * vv.z;
    X2[(d + 3) * LDC + j] = wv.w * vv.w;
  }
  __syncthreads();
  ta.mma(X1, LDC, X2, LDC, 0, D);
  __syncthreads();
  // dA^T into X1, A^T into X2
#pragma unroll
  for (int jj = 0; jj < TC::TN_; ++jj) {
    float o4[TC::TM_];
#pragma unroll
    for (int ii = 0; ii < TC::TM_; ++ii) o4[ii] = san(ta.acc[ii][jj], p.clip);
    store_vec<TC::TM_>(X1 + (ta.c0 + jj) * LDC + ta.r0, o4);
  }
  load_tile<float>(X2, LDC, ws.AT + chunk * C * C, C, C, C);        // X2[k][j] = A(j,k)
  __syncthreads();
  {
    TC t;
    t.zero();
    t.mma(X1, LDC, X2, LDC, 0, min(C, t.c0 + TC::TN_));
    __syncthreads();
#pragma unroll
    for (int ii = 0; ii < TC::TM_; ++ii) {
      float o4[TC::TN_];
#pragma unroll
      for (int jj = 0; jj < TC::TN_; ++jj) o4[jj] = san(t.acc[ii][jj], p.clip);
      store_vec<TC::TN_>(X1 + (t.r0 + ii) * LDC + t.c0, o4);       // tmp row-major
    }
  }
  load_tile_T<float>(X2, LDC, ws.AT + chunk * C * C, C, C, C);      // X2[k][i] = A(k,i)
  __syncthreads();
  {
    TC t;
    t.zero();
    if (t.c0 <= t.r0) t.mma(X2, LDC, X1, LDC, t.r0, C);
    float* out = ws.dAkkT + chunk * C * C;
#pragma unroll
    for (int jj = 0; jj < TC::TN_; ++jj) {
      const int j = t.c0 + jj;
      float o4[TC::TM_];
#pragma unroll
      for (int ii = 0; ii < TC::TM_; ++ii)
        o4[ii] = (j < t.r0 + ii) ? san(-t.acc[ii][jj], p.clip) : 0.f;
      store_vec<TC::TM_>(out + j * C + t.r0, o4);
    }
  }
  __syncthreads();
  load_tile<float>(X1, LDD, ws.dWp + chunk * C * D, D, C, D);       // X1[i][d] = dWp(i,d)
  __syncthreads();
  {
    TD t;
    t.zero();
    t.mma(X2, LDC, X1, LDD, t.r0, C);
    float *pdk = ws.pdk + chunk * C * D, *pdb = ws.pdb + chunk * C * D,
          *pdgc = ws.pdgc + chunk * C * D;
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      const int j = t.r0 + ii;
      float ok[TD::TN_], ob[TD::TN_], og[TD::TN_];
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        const int d = t.c0 + jj;
        const float eg = __expf(gc[j * D + d]);
        const float kk = to_f<T>(kc[j * rs + d]), bv = ld_gate<T>(bc + j * rs + d, GATES, kGateB);
        const float dkb = t.acc[ii][jj];
        ok[jj] = san(pdk[j * D + d] + dkb * eg * bv, p.clip);
        ob[jj] = san(dkb * eg * kk, p.clip);
        og[jj] = san(pdgc[j * D + d] + dkb * (bv * kk * eg), p.clip);
      }
      store_vec<TD::TN_>(pdk + j * D + t.c0, ok);
      store_vec<TD::TN_>(pdb + j * D + t.c0, ob);
      store_vec<TD::TN_>(pdgc + j * D + t.c0, og);
    }
  }
  __syncthreads();
  load_tile<float>(X1, LDD, ws.dv + chunk * C * D, D, C, D);        // X1[i][d] = dv(i,d)
  __syncthreads();
  {
    TD t;
    t.zero();
    t.mma(X2, LDC, X1, LDD, t.r0, C);
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      const int j = t.r0 + ii;
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        const int d = t.c0 + jj;
        const float dwv = t.acc[ii][jj];
        const float wa = ld_gate<T>(wc + j * rs + d, GATES, kGateW);
        const float dwo = san(san(dwv * to_f<T>(vc[j * rs + d]), p.clip), kFinalClip);
        dw_out[off + j * rs + d] = from_f<T>(GATES ? dwo * wa * (1.f - wa) : dwo);
        dv_out[off + j * rs + d] = from_f<T>(san(san(dwv * wa, p.clip), kFinalClip));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Intra pass 3: backward of the chunk scores (B4, gdn2_bwd.py:248-339), the
// in-chunk reverse cumsum (B5, gdn2_bwd.py:32-41) and the final assembly with
// the +-1e4 sanitiser (gdn2_pipeline.py:117-135).  The four pair sums are
// grouped-decay products (see Tile::mma_grouped); the decay derivative is
// dgc_i += L_i * dL_i and dgc_j -= R_j * dR_j, which equals the reference's
// pair sum of the weights.  Chunks with any g > 0 use the exact elementwise
// form with the +-20 clip and its mask.
// ---------------------------------------------------------------------------
template <typename T, int C, int D, bool GATES>
__global__ void __launch_bounds__(kThreads, 1)
k_bwd_intra3(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ b,
             const T* __restrict__ g, T* __restrict__ dq_out, T* __restrict__ dk_out,
             T* __restrict__ db_out, T* __restrict__ dg_out, Problem p, Workspace ws) {
  using TD = typename TileFor<C, D>::type;
  constexpr int GS = TD::TM_, NG = C / GS;
  constexpr int LDC = C + 4, LDD = D + 4;
  constexpr int P = C > D ? C : D, BIG = P * (P + 4);
  extern __shared__ __align__(16) float sm[];
  float* X1 = sm;
  float* X2 = X1 + BIG;
  float* sdg = X2 + BIG;      // [C][D]
  float* gref = sdg + C * D;  // [NG][D]
  float* red = gref + NG * D; // 256
  const int c = blockIdx.x, h = blockIdx.y, bb = blockIdx.z;
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const size_t chunk = ((size_t)bb * p.H + h) * p.nc + c;
  const T *qc = q + off, *kc = k + off, *bc = b + off, *gcp = g + off;
  const float* gc = ws.gc + chunk * C * D;
  const float* pdq = ws.pdq + chunk * C * D;
  const float* pdk = ws.pdk + chunk * C * D;
  const float* pdb = ws.pdb + chunk * C * D;
  const float* pdgc = ws.pdgc + chunk * C * D;
  const float* dAqkT = ws.dAqkT + chunk * C * C;
  const float* dAkkT = ws.dAkkT + chunk * C * C;

  float gpos = -1.f;
  for (int e = threadIdx.x; e < C * D; e += kThreads)
    gpos = fmaxf(gpos, ld_gate<T>(gcp + (e / D) * rs + e % D, GATES, kGateG));
  // positive gates, or sub-blocks that do not hold whole row groups (the
  // clip guard below needs partials per BC block), take the exact path
  const bool exact = block_max(gpos, red) > 0.f || p.bc % GS != 0;
  bool run_exact = exact;

  if (!exact) {
    for (int e = threadIdx.x; e < NG * D; e += kThreads)
      gref[e] = gc[(e / D) * GS * D + e % D];
    load_tile<float>(X1, LDC, dAqkT, C, C, C);                      // X1[j][i] = dAqk(i,j)
    for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
      const int j = e / (D / 4), d = (e % (D / 4)) * 4;
      const float4 kv = ld4<T>(kc + j * rs + d);
      const float* gj = gc + j * D + d;
      const float* gr = gc + (j & ~(GS - 1)) * D + d;
      *reinterpret_cast<float4*>(X2 + j * LDD + d) =
          make_float4(kv.x * __expf(gr[0] - gj[0]), kv.y * __expf(gr[1] - gj[1]),
                      kv.z * __expf(gr[2] - gj[2]), kv.w * __expf(gr[3] - gj[3]));
    }
    __syncthreads();
    TD t;
    const int rg = t.r0 / GS;
    float dka[TD::TM_][TD::TN_];
    // Clip guard.  The reference sanitises its B4 accumulators after every
    // BC-row sub-block pair (_clip_acc, gdn2_bwd.py:26-28); summing all pairs
    // at once gives the same value while the sum of the absolute per-block
    // partials stays below CLIP.  grouped() runs the contraction one BC block
    // at a time and leaves sum |block partial| per element in sab.
    float sab[TD::TM_][TD::TN_];
    const int gpb = p.bc / GS;   // row groups per sub-block
    auto grouped = [&](int g0, int g1) {
      t.zero();
#pragma unroll
      for (int i = 0; i < TD::TM_; ++i)
#pragma unroll
        for (int j = 0; j < TD::TN_; ++j) sab[i][j] = 0.f;
      for (int a0 = g0; a0 < g1;) {
        const int a1 = min(g1, (a0 / gpb + 1) * gpb);
        TD tb;
        tb.zero();
        tb.mma_grouped(X1, LDC, X2, LDD, gref, D, a0, a1, rg);
#pragma unroll
        for (int i = 0; i < TD::TM_; ++i)
#pragma unroll
          for (int j = 0; j < TD::TN_; ++j) {
            t.acc[i][j] += tb.acc[i][j];
            sab[i][j] += fabsf(tb.acc[i][j]);
          }
        a0 = a1;
      }
    };
    float gd_dq = 0.f, gd_dbk = 0.f, gd_dk2 = 0.f, gd_dk3 = 0.f;
    float gg0 = 0.f, gg1 = 0.f, gg2 = 0.f, gg3 = 0.f;
    // dL_qk -> dq and dgc (i role)
    grouped(0, rg + 1);
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      const int i = t.r0 + ii;
      float o4[TD::TN_];
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        const int d = t.c0 + jj;
        const float f = __expf(gc[i * D + d] - gc[t.r0 * D + d]);
        const float dl = t.acc[ii][jj] * f;
        o4[jj] = p.scale * to_f<T>(qc[i * rs + d]) * dl;
        gd_dq = fmaxf(gd_dq, fabsf(p.scale) * sab[ii][jj] * f);
        gg0 = fmaxf(gg0, fabsf(p.scale * to_f<T>(qc[i * rs + d])) * sab[ii][jj] * f);
        const float dq4 = san(p.scale * dl, p.clip);
        dq_out[off + i * rs + d] = from_f<T>(san(pdq[i * D + d] + dq4, kFinalClip));
      }
      store_vec<TD::TN_>(sdg + i * D + t.c0, o4);
    }
    __syncthreads();
    load_tile<float>(X1, LDC, dAkkT, C, C, C);
    __syncthreads();
    // dL_kk = dbk -> db, dk (b branch), dgc (i role)
    grouped(0, rg + 1);
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      const int i = t.r0 + ii;
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        const int d = t.c0 + jj;
        const float f = __expf(gc[i * D + d] - gc[t.r0 * D + d]);
        const float dbk = t.acc[ii][jj] * f;
        const float kk = to_f<T>(kc[i * rs + d]), bv = ld_gate<T>(bc + i * rs + d, GATES, kGateB);
        gd_dbk = fmaxf(gd_dbk, sab[ii][jj] * f);
        gg1 = fmaxf(gg1, fabsf(bv * kk) * sab[ii][jj] * f);
        dka[ii][jj] = dbk * bv;
        sdg[i * D + d] += bv * kk * dbk;
        const float dbo = san(pdb[i * D + d] + san(dbk * kk, p.clip), kFinalClip);
        db_out[off + i * rs + d] = from_f<T>(GATES ? dbo * bv * (1.f - bv) : dbo);
      }
    }
    __syncthreads();
    // dR_qk: X1 = dAqk row-major, X2 = scale q e^{gc_i - gc_rG}
    load_tile_T<float>(X1, LDC, dAqkT, C, C, C);                    // X1[i][j] = dAqk(i,j)
    for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
      const int i = e / (D / 4), d = (e % (D / 4)) * 4;
      const float4 qv = ld4<T>(qc + i * rs + d);
      const float* gi = gc + i * D + d;
      const float* gr = gc + (i & ~(GS - 1)) * D + d;
      *reinterpret_cast<float4*>(X2 + i * LDD + d) = make_float4(
          p.scale * qv.x * __expf(gi[0] - gr[0]), p.scale * qv.y * __expf(gi[1] - gr[1]),
          p.scale * qv.z * __expf(gi[2] - gr[2]), p.scale * qv.w * __expf(gi[3] - gr[3]));
    }
    __syncthreads();
    grouped(rg, NG);
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      const int j = t.r0 + ii;
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        const int d = t.c0 + jj;
        const float fr = __expf(gc[t.r0 * D + d] - gc[j * D + d]);
        const float dr = t.acc[ii][jj] * fr;
        dka[ii][jj] += dr;
        sdg[j * D + d] -= to_f<T>(kc[j * rs + d]) * dr;
        gd_dk2 = fmaxf(gd_dk2, sab[ii][jj] * fr);
        gg2 = fmaxf(gg2, fabsf(to_f<T>(kc[j * rs + d])) * sab[ii][jj] * fr);
      }
    }
    __syncthreads();
    // dR_kk: X1 = dAkk row-major, X2 = b k e^{gc_i - gc_rG}
    load_tile_T<float>(X1, LDC, dAkkT, C, C, C);
    for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
      const int i = e / (D / 4), d = (e % (D / 4)) * 4;
      const float4 kv = ld4<T>(kc + i * rs + d), bv = ld4_gate<T>(bc + i * rs + d, GATES, kGateB);
      const float* gi = gc + i * D + d;
      const float* gr = gc + (i & ~(GS - 1)) * D + d;
      *reinterpret_cast<float4*>(X2 + i * LDD + d) = make_float4(
          bv.x * kv.x * __expf(gi[0] - gr[0]), bv.y * kv.y * __expf(gi[1] - gr[1]),
          bv.z * kv.z * __expf(gi[2] - gr[2]), bv.w * kv.w * __expf(gi[3] - gr[3]));
    }
    __syncthreads();
    grouped(rg, NG);
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      const int j = t.r0 + ii;
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        const int d = t.c0 + jj;
        const float fr = __expf(gc[t.r0 * D + d] - gc[j * D + d]);
        const float dr = t.acc[ii][jj] * fr;
        gd_dk3 = fmaxf(gd_dk3, sab[ii][jj] * fr);
        gg3 = fmaxf(gg3, fabsf(to_f<T>(kc[j * rs + d])) * sab[ii][jj] * fr);
        const float dk4 = san(dka[ii][jj] + dr, p.clip);
        dk_out[off + j * rs + d] = from_f<T>(san(pdk[j * D + d] + dk4, kFinalClip));
        const float x = sdg[j * D + d] - to_f<T>(kc[j * rs + d]) * dr;
        sdg[j * D + d] = pdgc[j * D + d] + san(x, p.clip);
      }
    }
    const float lim = p.clip * (1.f - 1e-5f);   // NaN fails every test below
    run_exact = __syncthreads_or(!(gd_dq < lim && gd_dbk < lim && gd_dk2 + gd_dk3 < lim &&
                                   gg0 + gg1 + gg2 + gg3 < lim));
    if (run_exact && threadIdx.x == 0) atomicOr(ws.status + 4, 1);
  }
  if (run_exact) {
    // the reference's pair order (overwrites the fast path's outputs)
    b4_exact_chunk<T>(C, D, p.bc, qc, kc, bc, rs, gc, D, dAqkT, dAkkT, pdq, pdk, pdb, pdgc,
                      dq_out, dk_out, db_out, off, sdg, p.scale, p.clip, GATES, C);
  }
  __syncthreads();
  column_revcumsum<C, D>(sdg, red);
  for (int e = threadIdx.x; e < C * D; e += kThreads) {
    const int i = e / D, d = e % D;
    float dgo = san(san(sdg[e], p.clip), kFinalClip);
    if (GATES) dgo *= -gate_sig(to_f<T>(gcp[i * rs + d]));   // d(-softplus(g'))/dg'
    dg_out[off + i * rs + d] = from_f<T>(dgo);
  }
}

// ---------------------------------------------------------------------------
template <int C, int D>
cudaError_t launch_bwd_state(const Problem& p, const Workspace& ws, const float* dout,
                             const float* dh_final, float* dh0, cudaStream_t s,
                             bool only_flagged, bool pair) {
  constexpr int NV = 32;
  const size_t smem = StateSmem<C, D, NV>::bytes();
  auto kern = k_bwd_state<C, D, NV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(D / NV, p.H, p.B), kThreads, smem, s>>>(p, ws, dout, dh_final, dh0, only_flagged,
                                                       pair);
  return cudaGetLastError();
}

template <typename T, int C, int D>
cudaError_t launch_bwd_intra(const T* q, const T* k, const T* v, const T* w, const T* b,
                             const T* g, const float* dout, const float* dh_final, T* dq, T* dk,
                             T* dv, T* dw, T* db, T* dg, const Problem& p, const Workspace& ws,
                             cudaStream_t s, const LaunchHook& hook, bool skip12) {
  constexpr int P = C > D ? C : D, BIG = P * (P + 4);
  const dim3 grid(p.nc, p.H, p.B);
  cudaError_t e;
  if (!skip12) {
    hook.begin(kStageBwdIntra1, s);
    using TD = typename TileFor<C, D>::type;
    const size_t smem = (size_t)(3 * BIG + (C / TD::TM_) * D) * sizeof(float);
    auto kern = k_bwd_intra1<T, C, D>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem, s>>>(q, k, dout, dh_final, p, ws);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    hook.end(kStageBwdIntra1, s);
  }
  if (!skip12) {
    hook.begin(kStageBwdIntra2, s);
    const size_t smem = (size_t)(2 * BIG) * sizeof(float);
    auto kern = p.gates ? k_bwd_intra2<T, C, D, true> : k_bwd_intra2<T, C, D, false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem, s>>>(k, v, w, b, dv, dw, p, ws);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    hook.end(kStageBwdIntra2, s);
  }
  {
    hook.begin(kStageBwdIntra3, s);
    using TD = typename TileFor<C, D>::type;
    constexpr int NG = C / TD::TM_;
    const size_t smem = (size_t)(2 * BIG + C * D + NG * D + 256) * sizeof(float);
    auto kern = p.gates ? k_bwd_intra3<T, C, D, true> : k_bwd_intra3<T, C, D, false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem, s>>>(q, k, b, g, dq, dk, db, dg, p, ws);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    hook.end(kStageBwdIntra3, s);
  }
  return cudaSuccess;
}

#define GDN2_INST_BSTATE(C, D)                                                               \
  template cudaError_t launch_bwd_state<C, D>(const Problem&, const Workspace&, const float*, \
                                              const float*, float*, cudaStream_t, bool, bool);
#define GDN2_INST_BINTRA(T, C, D)                                                            \
  template cudaError_t launch_bwd_intra<T, C, D>(                                            \
      const T*, const T*, const T*, const T*, const T*, const T*, const float*, const float*, \
      T*, T*, T*, T*, T*, T*, const Problem&, const Workspace&, cudaStream_t,                \
      const LaunchHook&, bool);
GDN2_FOR_SHAPES(GDN2_INST_BSTATE)
GDN2_FOR_SHAPES_T(GDN2_INST_BINTRA)

}  // namespace gdn2
