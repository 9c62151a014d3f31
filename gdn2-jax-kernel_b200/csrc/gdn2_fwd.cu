// GDN-2 chunked forward: the intra-chunk kernel (reference Kernels A, B, C:
// gdn2_fwd.py:99-139, 173-260, 263-330) and the inter-chunk state kernel
// (Kernel D: gdn2_fwd.py:338-397).
#include "gdn2_kernels.cuh"

namespace gdn2 {

// ---------------------------------------------------------------------------
// Intra-chunk forward.  One CTA per (chunk, head, batch).
//   gc = cumsum(g); Aqk, Akk (Kernel A); A = (I+Akk)^-1 (Kernel B);
//   W = A (b k e^gc), U = A (w v), kg, qg, gc_last (Kernel C).
// Pair decays e^{gc_i - gc_j} are factored about the first row r of each
// GS-row group: e^{gc_i-gc_rG} * e^{gc_rG-gc_rJ} * e^{gc_rJ-gc_j}; for a
// non-increasing gc (g <= 0) every factor is bounded (the last by GS steps),
// so the product is exact to rounding and the reference's exponent clip at
// -20 changes values by < e^-20.  Chunks with any g > 0 take the exact
// elementwise path with the reference's +-20 clip.
// ---------------------------------------------------------------------------
template <typename T, int C, int D, bool DIAG, bool GATES>
__global__ void __launch_bounds__(kThreads, 1)
k_fwd_intra(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
            const T* __restrict__ w, const T* __restrict__ b, const T* __restrict__ g,
            Problem p, Workspace ws) {
  using TC = typename TileFor<C, C>::type;
  using TD = typename TileFor<C, D>::type;
  constexpr int GS = TC::TM_;
  constexpr int LDC = C + 4, LDD = D + 4;
  extern __shared__ __align__(16) float sm[];
  float* sgc = sm;                       // [C][D]
  float* X = sgc + C * D;                // big buffer
  float* Y = X + FwdSmem<C, D>::BIG;     // big buffer
  float* red = Y + FwdSmem<C, D>::BIG;   // scratch (>= 2*D floats)

  const int c = blockIdx.x, h = blockIdx.y, bb = blockIdx.z;
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const size_t chunk = ((size_t)bb * p.H + h) * p.nc + c;
  const T *qc = q + off, *kc = k + off, *vc = v + off, *wc = w + off, *bc = b + off,
          *gcp = g + off;

  // ---- gc = in-chunk cumsum of g (gdn2_fwd.py:105-107)
  load_tile<T>(sgc, D, gcp, rs, C, D);
  __syncthreads();
  if (GATES)   // g = -softplus(g') fused into the load
    for (int e = threadIdx.x; e < C * D; e += kThreads) sgc[e] = gate_act(sgc[e], kGateG);
  __syncthreads();
  float gpos = -1.f;
  for (int e = threadIdx.x; e < C * D; e += kThreads) gpos = fmaxf(gpos, sgc[e]);
  const bool exact = block_max(gpos, red) > 0.f;
  column_cumsum<C, D>(sgc, red);
  {
    float* gco = ws.gc + chunk * C * D;
    for (int e = threadIdx.x * 4; e < C * D; e += kThreads * 4)
      *reinterpret_cast<float4*>(gco + e) = *reinterpret_cast<float4*>(sgc + e);
    for (int d = threadIdx.x; d < D; d += kThreads)
      ws.gcl[chunk * D + d] = san(sgc[(C - 1) * D + d], p.clip);
  }

  float* aqkT = ws.AqkT + chunk * C * C;
  StageDiag dga, dgb;   // stage diagnostics (p.diag only)
  if (!exact) {
    // ---- Kernel A, factored: R^T into Y, L^T into X (contraction index d outer)
    for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
      const int j = e % C, d = (e / C) * 4;
      const float4 kv = ld4<T>(kc + j * rs + d);
      const float4 qv = ld4<T>(qc + j * rs + d);
      const int jr = j & ~(GS - 1);
      const float* gj = sgc + j * D + d;
      const float* gr = sgc + jr * D + d;
      Y[(d + 0) * LDC + j] = kv.x * __expf(gr[0] - gj[0]);
      Y[(d + 1) * LDC + j] = kv.y * __expf(gr[1] - gj[1]);
      Y[(d + 2) * LDC + j] = kv.z * __expf(gr[2] - gj[2]);
      Y[(d + 3) * LDC + j] = kv.w * __expf(gr[3] - gj[3]);
      X[(d + 0) * LDC + j] = qv.x * __expf(gj[0] - gr[0]);
      X[(d + 1) * LDC + j] = qv.y * __expf(gj[1] - gr[1]);
      X[(d + 2) * LDC + j] = qv.z * __expf(gj[2] - gr[2]);
      X[(d + 3) * LDC + j] = qv.w * __expf(gj[3] - gr[3]);
    }
    __syncthreads();
    TC t;
    t.zero();
    t.mma_group_decay(X, LDC, Y, LDC, sgc, D, D);
#pragma unroll
    for (int jj = 0; jj < TC::TN_; ++jj) {
      const int j = t.c0 + jj;
      float o4[TC::TM_];
#pragma unroll
      for (int ii = 0; ii < TC::TM_; ++ii) {
        const int i = t.r0 + ii;
        o4[ii] = (j <= i) ? san(p.scale * t.acc[ii][jj], p.clip) : 0.f;
        if (DIAG) dga.add(o4[ii]);
      }
      store_vec<TC::TM_>(aqkT + j * C + t.r0, o4);
    }
    __syncthreads();
    // L for Akk: b k e^{gc_i - gc_rG}
    for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
      const int j = e % C, d = (e / C) * 4;
      const float4 kv = ld4<T>(kc + j * rs + d);
      const float4 bv = ld4_gate<T>(bc + j * rs + d, GATES, kGateB);
      const int jr = j & ~(GS - 1);
      const float* gj = sgc + j * D + d;
      const float* gr = sgc + jr * D + d;
      X[(d + 0) * LDC + j] = bv.x * kv.x * __expf(gj[0] - gr[0]);
      X[(d + 1) * LDC + j] = bv.y * kv.y * __expf(gj[1] - gr[1]);
      X[(d + 2) * LDC + j] = bv.z * kv.z * __expf(gj[2] - gr[2]);
      X[(d + 3) * LDC + j] = bv.w * kv.w * __expf(gj[3] - gr[3]);
    }
    __syncthreads();
    t.zero();
    t.mma_group_decay(X, LDC, Y, LDC, sgc, D, D);
    __syncthreads();
    // Akk^T into X: X[j*LDC + i] = Akk(i, j), strictly lower
#pragma unroll
    for (int jj = 0; jj < TC::TN_; ++jj) {
      const int j = t.c0 + jj;
      float o4[TC::TM_];
#pragma unroll
      for (int ii = 0; ii < TC::TM_; ++ii) {
        const int i = t.r0 + ii;
        o4[ii] = (j < i) ? san(t.acc[ii][jj], p.clip) : 0.f;
        if (DIAG) dgb.add(o4[ii]);
      }
      store_vec<TC::TM_>(X + j * LDC + t.r0, o4);
    }
  } else {
    // ---- Kernel A, exact elementwise form with the +-20 exponent clip
    for (int e = threadIdx.x; e < C * C; e += kThreads) {
      const int i = e % C, j = e / C;
      float sq = 0.f, sk = 0.f;
      if (j <= i) {
        for (int d = 0; d < D; ++d) {
          const float ed = __expf(fminf(fmaxf(sgc[i * D + d] - sgc[j * D + d], -20.f), 20.f));
          const float kj = to_f<T>(kc[j * rs + d]) * ed;
          sq = fmaf(to_f<T>(qc[i * rs + d]), kj, sq);
          sk = fmaf(ld_gate<T>(bc + i * rs + d, GATES, kGateB) * to_f<T>(kc[i * rs + d]), kj, sk);
        }
      }
      aqkT[j * C + i] = (j <= i) ? san(p.scale * sq, p.clip) : 0.f;
      X[j * LDC + i] = (j < i) ? san(sk, p.clip) : 0.f;
      if (DIAG) {
        dga.add(aqkT[j * C + i]);
        dgb.add(X[j * LDC + i]);
      }
    }
  }
  if (DIAG) {
    dga.flush(ws.status, kDiagAqk);
    dgb.flush(ws.status, kDiagAkk);
  }
  __syncthreads();

  // ---- Kernel B: A = (I + Akk)^-1, computed in place on the transpose.
  wy_inverse_T<C>(X, LDC, Y, p.bc, p.clip);
  {
    float* at = ws.AT + chunk * C * C;
    for (int e = threadIdx.x * 4; e < C * C; e += kThreads * 4) {
      const int r = e / C, cc = e % C;
      const float4 a4 = *reinterpret_cast<const float4*>(X + r * LDC + cc);
      *reinterpret_cast<float4*>(at + e) = a4;
      if (DIAG) dga.add4(a4);
    }
    if (DIAG) dga.flush(ws.status, kDiagA);
  }

  // ---- Kernel C: W = A (b k e^gc), U = A (w v)
  for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
    const int j = e / (D / 4), d = (e % (D / 4)) * 4;
    const float4 kv = ld4<T>(kc + j * rs + d), bv = ld4_gate<T>(bc + j * rs + d, GATES, kGateB);
    const float* gj = sgc + j * D + d;
    float4 o = make_float4(bv.x * kv.x * __expf(gj[0]), bv.y * kv.y * __expf(gj[1]),
                           bv.z * kv.z * __expf(gj[2]), bv.w * kv.w * __expf(gj[3]));
    *reinterpret_cast<float4*>(Y + j * LDD + d) = o;
  }
  __syncthreads();
  {
    TD t;
    t.zero();
    t.mma(X, LDC, Y, LDD, 0, min(C, t.r0 + TD::TM_));
    float* wt = ws.WT + chunk * C * D;
#pragma unroll
    for (int jj = 0; jj < TD::TN_; ++jj) {
      float o4[TD::TM_];
#pragma unroll
      for (int ii = 0; ii < TD::TM_; ++ii) {
        o4[ii] = san(t.acc[ii][jj], p.clip);
        if (DIAG) dga.add(o4[ii]);
      }
      store_vec<TD::TM_>(wt + (t.c0 + jj) * C + t.r0, o4);
    }
    if (DIAG) dga.flush(ws.status, kDiagW);
    __syncthreads();
    for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
      const int j = e / (D / 4), d = (e % (D / 4)) * 4;
      const float4 wv = ld4_gate<T>(wc + j * rs + d, GATES, kGateW), vv = ld4<T>(vc + j * rs + d);
      *reinterpret_cast<float4*>(Y + j * LDD + d) =
          make_float4(wv.x * vv.x, wv.y * vv.y, wv.z * vv.z, wv.w * vv.w);
    }
    __syncthreads();
    t.zero();
    t.mma(X, LDC, Y, LDD, 0, min(C, t.r0 + TD::TM_));
    float* u = ws.U + chunk * C * D;
#pragma unroll
    for (int ii = 0; ii < TD::TM_; ++ii) {
      float o4[TD::TN_];
#pragma unroll
      for (int jj = 0; jj < TD::TN_; ++jj) {
        o4[jj] = san(t.acc[ii][jj], p.clip);
        if (DIAG) dga.add(o4[jj]);
      }
      store_vec<TD::TN_>(u + (t.r0 + ii) * D + t.c0, o4);
    }
    if (DIAG) dga.flush(ws.status, kDiagU);
  }
  // kg = k e^{gc_last - gc} (row-major), qg = q e^{gc} (transposed)
  {
    float* kgo = ws.kg + chunk * C * D;
    float* qgo = ws.qgT + chunk * C * D;
    const float* gl = sgc + (C - 1) * D;
    for (int e = threadIdx.x; e < C * (D / 4); e += kThreads) {
      const int i = e / (D / 4), d = (e % (D / 4)) * 4;
      const float4 kv = ld4<T>(kc + i * rs + d);
      const float* gi = sgc + i * D + d;
      float4 o = make_float4(san(kv.x * __expf(gl[d] - gi[0]), p.clip),
                             san(kv.y * __expf(gl[d + 1] - gi[1]), p.clip),
                             san(kv.z * __expf(gl[d + 2] - gi[2]), p.clip),
                             san(kv.w * __expf(gl[d + 3] - gi[3]), p.clip));
      *reinterpret_cast<float4*>(kgo + i * D + d) = o;
      if (DIAG) dga.add4(o);
    }
    if (DIAG) dga.flush(ws.status, kDiagKg);
    for (int e = threadIdx.x; e < C * D; e += kThreads) {
      const int i = e % C, d = e / C;
      qgo[d * C + i] = san(to_f<T>(qc[i * rs + d]) * __expf(sgc[i * D + d]), p.clip);
      if (DIAG) dga.add(qgo[d * C + i]);
    }
    if (DIAG) dga.flush(ws.status, kDiagQg);
  }
}

// ---------------------------------------------------------------------------
// Inter-chunk state recurrence (Kernel D, gdn2_fwd.py:347-360), serial over
// chunks.  Columns of h are independent, so each CTA owns NV value columns of
// one (batch, head) state and keeps that D x NV slice in shared memory:
//   vnew = U - W h;  o = scale qg h + Aqk vnew;  h <- e^{gc_last} h + kg^T vnew.
// When `save` is set, h entering each chunk and vnew are written for the
// backward (the batch-major residuals of gdn2_fwd.py:369-397).
// ---------------------------------------------------------------------------
template <int C, int D, int NV>
__global__ void __launch_bounds__(kThreads, 2)
k_fwd_state(Problem p, Workspace ws, const float* __restrict__ h0, float* __restrict__ o,
            float* __restrict__ hfinal, int save) {
  using T1 = typename TileFor<C, NV>::type;
  using T3 = typename TileFor<D, NV>::type;
  constexpr int LDC = C + 4, LDD = D + 4;
  extern __shared__ __align__(16) float sm[];
  float* X = sm;                                 // big buffer
  float* sh = X + StateSmem<C, D, NV>::BIG;      // [D][NV]
  float* svn = sh + D * NV;                      // [C][NV]
  const int v0 = blockIdx.x * NV, h = blockIdx.y, bb = blockIdx.z;
  const size_t bh = (size_t)bb * p.H + h;
  const long rs = p.row_stride();

  for (int e = threadIdx.x; e < D * NV; e += kThreads) {
    const int d = e / NV, vv = e % NV;
    sh[e] = h0 ? san(h0[bh * D * D + d * D + v0 + vv], p.clip) : 0.f;
  }
  __syncthreads();
  StageDiag dgo;   // o, then h_final (p.diag only)
  for (int c = 0; c < p.nc; ++c) {
    const size_t chunk = bh * p.nc + c;
    if (save) {
      float* hp = ws.hpre + chunk * D * D;
      for (int e = threadIdx.x; e < D * NV; e += kThreads)
        hp[(e / NV) * D + v0 + e % NV] = sh[e];
    }
    load_tile<float>(X, LDC, ws.WT + chunk * C * D, C, D, C);
    __syncthreads();
    {
      T1 t;
      t.zero();
      t.mma(X, LDC, sh, NV, 0, D);
      const float* u = ws.U + chunk * C * D;
      float* vn = ws.vnew + chunk * C * D;
#pragma unroll
      for (int ii = 0; ii < T1::TM_; ++ii) {
        const int i = t.r0 + ii;
        float o4[T1::TN_];
#pragma unroll
        for (int jj = 0; jj < T1::TN_; ++jj) o4[jj] = u[i * D + v0 + t.c0 + jj] - t.acc[ii][jj];
        store_vec<T1::TN_>(svn + i * NV + t.c0, o4);
        if (save) store_vec<T1::TN_>(vn + i * D + v0 + t.c0, o4);
      }
    }
    __syncthreads();
    if (o) {
    load_tile<float>(X, LDC, ws.qgT + chunk * C * D, C, D, C);
    __syncthreads();
    {
      T1 t;
      t.zero();
      t.mma(X, LDC, sh, NV, 0, D);
#pragma unroll
      for (int ii = 0; ii < T1::TM_; ++ii)
#pragma unroll
        for (int jj = 0; jj < T1::TN_; ++jj) t.acc[ii][jj] *= p.scale;
      __syncthreads();
      load_tile<float>(X, LDC, ws.AqkT + chunk * C * C, C, C, C);
      __syncthreads();
      t.mma(X, LDC, svn, NV, 0, min(C, t.r0 + T1::TM_));
      float* orow = o + ((long)bb * p.T + (long)c * C) * rs + (long)h * D + v0;
#pragma unroll
      for (int ii = 0; ii < T1::TM_; ++ii) {
        float o4[T1::TN_];
#pragma unroll
        for (int jj = 0; jj < T1::TN_; ++jj) {
          o4[jj] = san(t.acc[ii][jj], p.clip);
          if (p.diag) dgo.add(o4[jj]);
        }
        store_vec<T1::TN_>(orow + (t.r0 + ii) * rs + t.c0, o4);
      }
    }
    __syncthreads();
    }
    load_tile<float>(X, LDD, ws.kg + chunk * C * D, D, C, D);
    __syncthreads();
    {
      T3 t;
      t.zero();
      t.mma(X, LDD, svn, NV, 0, C);
      const float* gl = ws.gcl + chunk * D;
#pragma unroll
      for (int ii = 0; ii < T3::TM_; ++ii) {
        const int d = t.r0 + ii;
        const float dec = __expf(gl[d]);
#pragma unroll
        for (int jj = 0; jj < T3::TN_; ++jj) {
          float* hv = sh + d * NV + t.c0 + jj;
          *hv = san(fmaf(dec, *hv, t.acc[ii][jj]), p.clip);
        }
      }
    }
    __syncthreads();
  }
  if (p.diag && o) dgo.flush(ws.status, kDiagO);
  if (hfinal) {
    for (int e = threadIdx.x; e < D * NV; e += kThreads) {
      hfinal[bh * D * D + (e / NV) * D + v0 + e % NV] = sh[e];
      if (p.diag) dgo.add(sh[e]);
    }
    if (p.diag) dgo.flush(ws.status, kDiagHFinal);
  }
}

// ---------------------------------------------------------------------------
template <typename T, int C, int D>
cudaError_t launch_fwd_intra(const T* q, const T* k, const T* v, const T* w, const T* b,
                             const T* g, const Problem& p, const Workspace& ws,
                             cudaStream_t s) {
  const size_t smem = FwdSmem<C, D>::bytes();
  auto kern = p.diag ? (p.gates ? k_fwd_intra<T, C, D, true, true> : k_fwd_intra<T, C, D, true, false>)
                     : (p.gates ? k_fwd_intra<T, C, D, false, true> : k_fwd_intra<T, C, D, false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(p.nc, p.H, p.B), kThreads, smem, s>>>(q, k, v, w, b, g, p, ws);
  return cudaGetLastError();
}

template <int C, int D>
cudaError_t launch_fwd_state(const Problem& p, const Workspace& ws, const float* h0, float* o,
                             float* hfinal, int save, cudaStream_t s) {
  constexpr int NV = 32;
  const size_t smem = StateSmem<C, D, NV>::bytes();
  auto kern = k_fwd_state<C, D, NV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(D / NV, p.H, p.B), kThreads, smem, s>>>(p, ws, h0, o, hfinal, save);
  return cudaGetLastError();
}

#define GDN2_INST_FWD(T, C, D)                                                              \
  template cudaError_t launch_fwd_intra<T, C, D>(const T*, const T*, const T*, const T*,    \
                                                 const T*, const T*, const Problem&,        \
                                                 const Workspace&, cudaStream_t);
#define GDN2_INST_STATE(C, D)                                                               \
  template cudaError_t launch_fwd_state<C, D>(const Problem&, const Workspace&, const float*, \
                                              float*, float*, int, cudaStream_t);
GDN2_FOR_SHAPES_T(GDN2_INST_FWD)
GDN2_FOR_SHAPES(GDN2_INST_STATE)

}  // namespace gdn2
