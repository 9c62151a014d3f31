// The reference's stage functions as separate entry points: Kernels A, B, C
// and D of gdn2_fwd.py and B1-B5 of gdn2_bwd.py, each on the reference's
// chunked layouts ((B, H, nc, BT, .) float32, gc_last (B, H, nc, D)).  The
// fused kernels never call these: they serve code that composes the stages
// itself, and the Python layer runs head dim 256 (which the fused kernels do
// not cover) through them.  CUDA-core kernels, one CTA per chunk (or per
// (b, h) and 32 value columns for the two serial scans), with every
// sanitiser where the reference has it.
#include <cstdio>

#include "../../include/gdn2.h"
#include "gdn2_b4_exact.cuh"
#include "gdn2_kernels.cuh"

namespace gdn2 {
int report_error(int code, const char* msg);   // gdn2_capi.cu

namespace {

constexpr float kPairClip = 20.f;   // exponent clip of the pair decays, gdn2_fwd.py:125
constexpr int kNV = 32;             // value columns per CTA of the serial scans

// gc = in-chunk cumsum of g for the chunk whose first row is g (row stride
// rs), into s[r * D + d]; one thread per column, rows in order.
template <typename T>
__device__ void chunk_cumsum(const T* g, long rs, int BT, int D, float* s) {
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float acc = 0.f;
    for (int r = 0; r < BT; ++r) {
      acc += to_f<T>(g[r * rs + d]);
      s[r * D + d] = acc;
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Kernel A (gdn2_fwd.py:99-139): Aqk(i,j) = san(scale sum_d q_id k_jd e^{clip(gc_id-gc_jd,+-20)})
// for j <= i, Akk(i,j) = san(sum_d b_id k_id k_jd e^{...}) for j < i, zero
// above.  Every entry is one sub-block pair's element, so the per-pair
// sanitiser is per element.  Shared: gc and k of the chunk.
template <typename T>
__global__ void __launch_bounds__(kThreads)
k_stage_scores(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ b,
               const T* __restrict__ g, float* __restrict__ aqk, float* __restrict__ akk, int Tn,
               int H, int D, int BT, float scale, float clip, bool k_resident) {
  extern __shared__ __align__(16) float sm[];
  float* gc = sm;
  float* ks = k_resident ? sm + BT * D : nullptr;   // k of the chunk, when it fits
  const int nc = Tn / BT;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % nc), h = (int)((chunk / nc) % H), bb = (int)(chunk / nc / H);
  const long rs = (long)H * D;
  const long off = ((long)bb * Tn + (long)c * BT) * rs + (long)h * D;
  auto kat = [&](int r, int d) { return ks ? ks[r * D + d] : to_f<T>(k[off + r * rs + d]); };
  if (ks)
    for (int e = threadIdx.x; e < BT * D; e += kThreads) ks[e] = to_f<T>(k[off + (e / D) * rs + e % D]);
  chunk_cumsum(g + off, rs, BT, D, gc);
  float* ao = aqk + chunk * BT * BT;
  float* ko = akk + chunk * BT * BT;
  for (int e = threadIdx.x; e < BT * BT; e += kThreads) {
    const int i = e / BT, j = e % BT;   // a warp shares row i: q, b broadcast
    float sq = 0.f, sk = 0.f;
    if (j <= i) {
      for (int d = 0; d < D; ++d) {
        const float ed = expf(fminf(fmaxf(gc[i * D + d] - gc[j * D + d], -kPairClip), kPairClip));
        const float kj = kat(j, d) * ed;
        sq = fmaf(to_f<T>(q[off + i * rs + d]), kj, sq);
        sk = fmaf(to_f<T>(b[off + i * rs + d]) * kat(i, d), kj, sk);
      }
    }
    ao[e] = j <= i ? san(scale * sq, clip) : 0.f;
    ko[e] = j < i ? san(sk, clip) : 0.f;
  }
}

// ---------------------------------------------------------------------------
// Kernel B (gdn2_fwd.py:173-260): A = (I + Akk)^-1 per chunk, the reference's
// micro solves and block substitution with its sanitisers (any number of BC
// sub-blocks).  Shared: the transposed tile and the solve's scratch.
template <int C>
__global__ void __launch_bounds__(kThreads)
k_stage_wy(const float* __restrict__ akk, float* __restrict__ a, int bc, float clip) {
  extern __shared__ __align__(16) float sm[];
  constexpr int LD = C + 4;
  float* S = sm;
  float* tmp = sm + C * LD;
  const size_t chunk = blockIdx.x;
  const float* src = akk + chunk * C * C;
  for (int e = threadIdx.x; e < C * C; e += kThreads) S[(e % C) * LD + e / C] = src[e];
  __syncthreads();
  wy_inverse_T<C>(S, LD, tmp, bc, clip);
  __syncthreads();
  float* dst = a + chunk * C * C;
  for (int e = threadIdx.x; e < C * C; e += kThreads) dst[e] = S[(e % C) * LD + e / C];
}

// Chunks too large for one shared tile (BT = 256): the BC diagonal blocks are
// solved as above (one CTA per block; the reference's _block_solve), then
// k_stage_wy_compose runs the substitution across the BC sub-blocks in the
// reference's order (its Kernel B for two sub-blocks, gdn2_fwd.py:228-243,
// continued for more), in global memory with one BC x BC scratch per chunk:
//   A_mn = san(-A_mm acc),  acc = san(acc + T_mk A_kn) for k = n .. m-1.
template <int C>
__global__ void __launch_bounds__(kThreads)
k_stage_wy_diag(const float* __restrict__ akk, float* __restrict__ a, int BT, float clip) {
  extern __shared__ __align__(16) float sm[];
  constexpr int LD = C + 4;
  float* S = sm;
  float* tmp = sm + C * LD;
  const int nsub = BT / C;
  const size_t chunk = blockIdx.x / nsub;
  const int m = blockIdx.x % nsub;
  const float* src = akk + chunk * BT * BT + (size_t)m * C * BT + m * C;
  for (int e = threadIdx.x; e < C * C; e += kThreads) S[(e % C) * LD + e / C] = src[(e / C) * BT + e % C];
  __syncthreads();
  wy_inverse_T<C>(S, LD, tmp, C, clip);
  __syncthreads();
  float* dst = a + chunk * BT * BT + (size_t)m * C * BT + m * C;
  for (int e = threadIdx.x; e < C * C; e += kThreads) dst[(e / C) * BT + e % C] = S[(e % C) * LD + e / C];
}

__global__ void __launch_bounds__(kThreads)
k_stage_wy_compose(const float* __restrict__ akk, float* __restrict__ a, float* __restrict__ scr,
                   int BT, int BC, float clip) {
  const size_t chunk = blockIdx.x;
  const float* T = akk + chunk * BT * BT;
  float* A = a + chunk * BT * BT;
  float* acc = scr + chunk * BC * BC;
  const int nsub = BT / BC;
  for (int m = 1; m < nsub; ++m) {
    for (int n = m - 1; n >= 0; --n) {
      for (int e = threadIdx.x; e < BC * BC; e += kThreads) acc[e] = 0.f;
      __syncthreads();
      for (int kk = n; kk < m; ++kk) {
        for (int e = threadIdx.x; e < BC * BC; e += kThreads) {
          const int i = e / BC, j = e % BC;
          float s = 0.f;
          for (int x = 0; x < BC; ++x)
            s = fmaf(T[(size_t)(m * BC + i) * BT + kk * BC + x], A[(size_t)(kk * BC + x) * BT + n * BC + j], s);
          acc[e] = san(acc[e] + s, clip);
        }
        __syncthreads();
      }
      for (int e = threadIdx.x; e < BC * BC; e += kThreads) {
        const int i = e / BC, j = e % BC;
        float s = 0.f;
        for (int x = 0; x < BC; ++x) s = fmaf(A[(size_t)(m * BC + i) * BT + m * BC + x], acc[x * BC + j], s);
        A[(size_t)(m * BC + i) * BT + n * BC + j] = san(-s, clip);
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// Kernel C (gdn2_fwd.py:264-295): W = san(A (b k e^gc)), U = san(A (w v)),
// kg = san(k e^{gc_last - gc}), qg = san(q e^gc), gc_last = san(gc_last).
// Shared: b k e^gc and w v of the chunk.
template <typename T>
__global__ void __launch_bounds__(kThreads)
k_stage_recompute(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                  const T* __restrict__ w, const T* __restrict__ b, const T* __restrict__ g,
                  const float* __restrict__ a, float* __restrict__ wp, float* __restrict__ u,
                  float* __restrict__ kg, float* __restrict__ qg, float* __restrict__ gcl, int Tn,
                  int H, int D, int BT, float clip, bool wv_resident) {
  extern __shared__ __align__(16) float sm[];
  float* gc = sm;                                      // then b k e^gc
  float* wv = wv_resident ? sm + BT * D : nullptr;     // w v, when it fits
  const int nc = Tn / BT;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % nc), h = (int)((chunk / nc) % H), bb = (int)(chunk / nc / H);
  const long rs = (long)H * D;
  const long off = ((long)bb * Tn + (long)c * BT) * rs + (long)h * D;
  chunk_cumsum(g + off, rs, BT, D, gc);
  const size_t co = chunk * BT * D;
  for (int e = threadIdx.x; e < BT * D; e += kThreads) {
    const int i = e / D, d = e % D;
    const float gi = gc[e], gl = gc[(BT - 1) * D + d];
    const long x = off + i * rs + d;
    kg[co + e] = san(to_f<T>(k[x]) * expf(gl - gi), clip);
    qg[co + e] = san(to_f<T>(q[x]) * expf(gi), clip);
    if (wv) wv[e] = to_f<T>(w[x]) * to_f<T>(v[x]);
  }
  for (int d = threadIdx.x; d < D; d += kThreads) gcl[chunk * D + d] = san(gc[(BT - 1) * D + d], clip);
  __syncthreads();
  for (int e = threadIdx.x; e < BT * D; e += kThreads) {
    const int i = e / D, d = e % D;
    gc[e] = to_f<T>(b[off + i * rs + d]) * to_f<T>(k[off + i * rs + d]) * expf(gc[e]);
  }
  __syncthreads();
  const float* ac = a + chunk * BT * BT;
  for (int e = threadIdx.x; e < BT * D; e += kThreads) {
    const int i = e / D, d = e % D;
    float sw = 0.f, su = 0.f;
    for (int j = 0; j < BT; ++j) {
      const float aij = ac[i * BT + j];
      sw = fmaf(aij, gc[j * D + d], sw);
      su = fmaf(aij, wv ? wv[j * D + d] : to_f<T>(w[off + j * rs + d]) * to_f<T>(v[off + j * rs + d]),
                su);
    }
    wp[co + e] = san(sw, clip);
    u[co + e] = san(su, clip);
  }
}

// ---------------------------------------------------------------------------
// Kernel D (gdn2_fwd.py:338-397), serial over the chunks of one (b, h); this
// CTA owns kNV value columns of the state.  Per chunk:
//   vnew = U - W h;  o = san(scale qg h + Aqk vnew);
//   h = san(h e^{gc_last} + kg^T vnew).
// hpre / vnew_all (may be null) are chunk-major, (nc, B, H, .), as the
// reference's scan stacks them.
__global__ void __launch_bounds__(kThreads)
k_stage_combine(const float* __restrict__ aqk, const float* __restrict__ wp,
                const float* __restrict__ u, const float* __restrict__ kg,
                const float* __restrict__ qg, const float* __restrict__ gcl,
                const float* __restrict__ h0, float* __restrict__ o, float* __restrict__ hf,
                float* __restrict__ hpre, float* __restrict__ vall, int B, int H, int nc, int BT,
                int D, float scale, float clip) {
  extern __shared__ __align__(16) float sm[];
  float* hs = sm;             // [D][kNV]
  float* vn = sm + D * kNV;   // [BT][kNV]
  float* hn = vn + BT * kNV;  // [D][kNV] next state
  const int v0 = blockIdx.x * kNV, h = blockIdx.y, bb = blockIdx.z;
  const size_t bh = (size_t)bb * H + h;
  for (int e = threadIdx.x; e < D * kNV; e += kThreads)
    hs[e] = h0 ? san(h0[bh * D * D + (e / kNV) * D + v0 + e % kNV], clip) : 0.f;
  __syncthreads();
  for (int c = 0; c < nc; ++c) {
    const size_t chunk = bh * nc + c;
    const float* W = wp + chunk * BT * D;
    const float* Q = qg + chunk * BT * D;
    const float* K = kg + chunk * BT * D;
    const float* U = u + chunk * BT * D;
    const float* Aq = aqk + chunk * BT * BT;
    if (hpre)
      for (int e = threadIdx.x; e < D * kNV; e += kThreads)
        hpre[(((size_t)c * B + bb) * H + h) * D * D + (e / kNV) * D + v0 + e % kNV] = hs[e];
    for (int e = threadIdx.x; e < BT * kNV; e += kThreads) {
      const int i = e / kNV, vv = e % kNV;
      float s = 0.f;
      for (int d = 0; d < D; ++d) s = fmaf(W[i * D + d], hs[d * kNV + vv], s);
      vn[e] = U[i * D + v0 + vv] - s;
      if (vall) vall[(((size_t)c * B + bb) * H + h) * BT * D + i * D + v0 + vv] = vn[e];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < BT * kNV; e += kThreads) {
      const int i = e / kNV, vv = e % kNV;
      float sq = 0.f, sa = 0.f;
      for (int d = 0; d < D; ++d) sq = fmaf(Q[i * D + d], hs[d * kNV + vv], sq);
      for (int j = 0; j < BT; ++j) sa = fmaf(Aq[i * BT + j], vn[j * kNV + vv], sa);
      o[chunk * BT * D + i * D + v0 + vv] = san(scale * sq + sa, clip);
    }
    for (int e = threadIdx.x; e < D * kNV; e += kThreads) {
      const int d = e / kNV, vv = e % kNV;
      float s = 0.f;
      for (int i = 0; i < BT; ++i) s = fmaf(K[i * D + d], vn[i * kNV + vv], s);
      hn[e] = san(hs[e] * expf(gcl[chunk * D + d]) + s, clip);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < D * kNV; e += kThreads) hs[e] = hn[e];
    __syncthreads();
  }
  for (int e = threadIdx.x; e < D * kNV; e += kThreads)
    hf[bh * D * D + (e / kNV) * D + v0 + e % kNV] = hs[e];
}

// ---------------------------------------------------------------------------
// B1 (gdn2_bwd.py:45-80), serial in reverse over the chunks of one (b, h):
//   dv_new = san(dv_partial + kg dh);
//   dh = san(qg^T (scale do) + dh e^{gc_last} - W^T dv_new).
// dh_all[c] = the dh after chunk c's step (the state gradient entering c).
__global__ void __launch_bounds__(kThreads)
k_stage_dhu(const float* __restrict__ dout, const float* __restrict__ dvp,
            const float* __restrict__ wp, const float* __restrict__ qg,
            const float* __restrict__ kg, const float* __restrict__ gcl,
            const float* __restrict__ dht, float* __restrict__ dh_all, float* __restrict__ dh0,
            float* __restrict__ dv_all, int H, int nc, int BT, int D, float scale, float clip) {
  extern __shared__ __align__(16) float sm[];
  float* dh = sm;              // [D][kNV]
  float* dv = sm + D * kNV;    // [BT][kNV]
  float* dn = dv + BT * kNV;   // [D][kNV]
  const int v0 = blockIdx.x * kNV, h = blockIdx.y, bb = blockIdx.z;
  const size_t bh = (size_t)bb * H + h;
  for (int e = threadIdx.x; e < D * kNV; e += kThreads)
    dh[e] = dht ? san(dht[bh * D * D + (e / kNV) * D + v0 + e % kNV], clip) : 0.f;
  __syncthreads();
  for (int c = nc - 1; c >= 0; --c) {
    const size_t chunk = bh * nc + c;
    const size_t co = chunk * BT * D;
    for (int e = threadIdx.x; e < BT * kNV; e += kThreads) {
      const int i = e / kNV, vv = e % kNV;
      float s = 0.f;
      for (int d = 0; d < D; ++d) s = fmaf(kg[co + i * D + d], dh[d * kNV + vv], s);
      dv[e] = san(dvp[co + i * D + v0 + vv] + s, clip);
      dv_all[co + i * D + v0 + vv] = dv[e];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < D * kNV; e += kThreads) {
      const int d = e / kNV, vv = e % kNV;
      float so = 0.f, sv = 0.f;
      for (int i = 0; i < BT; ++i) {
        so = fmaf(qg[co + i * D + d], scale * dout[co + i * D + v0 + vv], so);
        sv = fmaf(wp[co + i * D + d], dv[i * kNV + vv], sv);
      }
      dn[e] = san(so + dh[e] * expf(gcl[chunk * D + d]) - sv, clip);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < D * kNV; e += kThreads) {
      dh[e] = dn[e];
      dh_all[chunk * D * D + (e / kNV) * D + v0 + e % kNV] = dn[e];
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < D * kNV; e += kThreads)
    dh0[bh * D * D + (e / kNV) * D + v0 + e % kNV] = dh[e];
}

// ---------------------------------------------------------------------------
// B2 (gdn2_bwd.py:84-96): dAqk = san((do vnew^T) * causal), dv = san(Aqk^T do).
__global__ void __launch_bounds__(kThreads)
k_stage_dav(const float* __restrict__ aqk, const float* __restrict__ vnew,
            const float* __restrict__ dout, float* __restrict__ daqk, float* __restrict__ dv,
            int BT, int D, float clip) {
  const size_t chunk = blockIdx.x;
  const size_t co = chunk * BT * D, so = chunk * BT * BT;
  for (int e = threadIdx.x; e < BT * BT; e += kThreads) {
    const int i = e / BT, j = e % BT;
    float s = 0.f;
    if (j <= i)
      for (int x = 0; x < D; ++x) s = fmaf(dout[co + i * D + x], vnew[co + j * D + x], s);
    daqk[so + e] = san(j <= i ? s : 0.f, clip);
  }
  for (int e = threadIdx.x; e < BT * D; e += kThreads) {
    const int j = e / D, x = e % D;
    float s = 0.f;
    for (int i = 0; i < BT; ++i) s = fmaf(aqk[so + i * BT + j], dout[co + i * D + x], s);
    dv[co + e] = san(s, clip);
  }
}

// ---------------------------------------------------------------------------
// B3 (gdn2_bwd.py:126-210) for one chunk.  The output buffers hold the
// intermediates between phases (dqg in dq, dWp in dv_raw, dkg in dk, dkb in
// db, dwv in dw, dA in dAkk); `tmp` is a BT x BT scratch per chunk.
__global__ void __launch_bounds__(kThreads)
k_stage_wy_dqkg(const float* __restrict__ q, const float* __restrict__ k,
                const float* __restrict__ b, const float* __restrict__ w,
                const float* __restrict__ v, const float* __restrict__ gc,
                const float* __restrict__ a, const float* __restrict__ hpre,
                const float* __restrict__ vnew, const float* __restrict__ dout,
                const float* __restrict__ dvn, const float* __restrict__ dhn, float* dq, float* dk,
                float* db, float* dw, float* dvr, float* dgc, float* dakk, float* tmp, int BT,
                int D, float scale, float clip) {
  __shared__ float colsum[256];
  const size_t chunk = blockIdx.x;
  const size_t co = chunk * BT * D, so = chunk * BT * BT, ho = chunk * D * D;
  const float* G = gc + co;
  const float* A = a + so;
  const float* Hp = hpre + ho;
  const float* Dn = dhn + ho;
  auto idx = [&](const float* t, int r, int x) { return t[co + r * D + x]; };
  // phase 1: dqg = scale do h^T, dWp = -dv h^T, dkg = vnew dh_next^T
  for (int e = threadIdx.x; e < BT * D; e += kThreads) {
    const int i = e / D, x = e % D;
    float sq = 0.f, sw = 0.f, sk = 0.f;
    for (int y = 0; y < D; ++y) {
      const float hv = Hp[x * D + y];
      sq = fmaf(idx(dout, i, y), hv, sq);
      sw = fmaf(idx(dvn, i, y), hv, sw);
      sk = fmaf(idx(vnew, i, y), Dn[x * D + y], sk);
    }
    dq[co + e] = scale * sq;
    dvr[co + e] = -sw;
    dk[co + e] = sk;
  }
  __syncthreads();
  // phase 2: dA = san(dWp kb^T + dv wv^T); dkb = A^T dWp; dwv = A^T dv
  for (int e = threadIdx.x; e < BT * BT; e += kThreads) {
    const int i = e / BT, j = e % BT;
    float s = 0.f;
    for (int x = 0; x < D; ++x) {
      const float kb = idx(b, j, x) * idx(k, j, x) * expf(G[j * D + x]);
      s = fmaf(dvr[co + i * D + x], kb, s);
      s = fmaf(idx(dvn, i, x), idx(w, j, x) * idx(v, j, x), s);
    }
    dakk[so + e] = san(s, clip);
  }
  for (int e = threadIdx.x; e < BT * D; e += kThreads) {
    const int j = e / D, x = e % D;
    float s1 = 0.f, s2 = 0.f;
    for (int i = 0; i < BT; ++i) {
      const float aij = A[i * BT + j];
      s1 = fmaf(aij, dvr[co + i * D + x], s1);
      s2 = fmaf(aij, idx(dvn, i, x), s2);
    }
    db[co + e] = s1;
    dw[co + e] = s2;
  }
  __syncthreads();
  // phase 3: tmp = san(dA A^T)
  float* tp = tmp + so;
  for (int e = threadIdx.x; e < BT * BT; e += kThreads) {
    const int i = e / BT, kk = e % BT;
    float s = 0.f;
    for (int j = 0; j < BT; ++j) s = fmaf(dakk[so + i * BT + j], A[kk * BT + j], s);
    tp[e] = san(s, clip);
  }
  __syncthreads();
  // phase 4: dAkk = -(A^T tmp) * strict
  for (int e = threadIdx.x; e < BT * BT; e += kThreads) {
    const int i = e / BT, j = e % BT;
    float s = 0.f;
    if (j < i)
      for (int kk = 0; kk < BT; ++kk) s = fmaf(A[kk * BT + i], tp[kk * BT + j], s);
    dakk[so + e] = san(j < i ? -s : 0.f, clip);
  }
  // phase 5: the gc_last row, sum_i dkg kg + e^{gc_last} sum_v dh_next h_pre
  const float* gl = G + (BT - 1) * D;
  for (int x = threadIdx.x; x < D; x += kThreads) {
    float s = 0.f, r = 0.f;
    for (int i = 0; i < BT; ++i) s += dk[co + i * D + x] * (idx(k, i, x) * expf(gl[x] - G[i * D + x]));
    for (int y = 0; y < D; ++y) r += Dn[x * D + y] * Hp[x * D + y];
    colsum[x] = s + expf(gl[x]) * r;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < BT * D; e += kThreads) {
    const int i = e / D, x = e % D;
    const float eg = expf(G[e]), f = expf(gl[x] - G[e]);
    const float dqg = dq[co + e], dkg = dk[co + e], dkb = db[co + e], dwv = dw[co + e];
    const float kv = idx(k, i, x), bv = idx(b, i, x);
    const float kbd = bv * kv * eg, kgv = kv * f, qgv = idx(q, i, x) * eg;
    float g = dkb * kbd + dqg * qgv - dkg * kgv;
    if (i == BT - 1) g += colsum[x];
    dk[co + e] = san(dkb * eg * bv + dkg * f, clip);
    db[co + e] = san(dkb * eg * kv, clip);
    dq[co + e] = san(dqg * eg, clip);
    dw[co + e] = san(dwv * idx(v, i, x), clip);
    dvr[co + e] = san(dwv * idx(w, i, x), clip);
    dgc[co + e] = san(g, clip);
  }
}

// ---------------------------------------------------------------------------
// B4 (gdn2_bwd.py:248-339): the sub-block pairs in the reference's order
// (b4_exact_chunk) with zero B3 partials and the final sanitiser at CLIP.
// dAqkT / dAkkT are the transposed score gradients (element (i, j) at
// j * BT + i); outputs chunked.
template <typename T>
__global__ void __launch_bounds__(kThreads)
k_stage_intra_bwd(const float* __restrict__ daqkT, const float* __restrict__ dakkT,
                  const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ b,
                  const T* __restrict__ g, const float* __restrict__ zeros, float* dq, float* dk,
                  float* db, float* dgc, int Tn, int H, int D, int BT, int BC, float scale,
                  float clip) {
  extern __shared__ __align__(16) float sm[];
  const int nc = Tn / BT;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % nc), h = (int)((chunk / nc) % H), bb = (int)(chunk / nc / H);
  const long rs = (long)H * D;
  const long off = ((long)bb * Tn + (long)c * BT) * rs + (long)h * D;
  chunk_cumsum(g + off, rs, BT, D, sm);
  const size_t co = chunk * BT * D, so = chunk * BT * BT;
  // zero B3 partials; final sanitiser at CLIP (the stage's own, gdn2_bwd.py:333-336)
  b4_exact_chunk<T, float>(BT, D, BC, q + off, k + off, b + off, rs, sm, D, daqkT + so,
                           dakkT + so, zeros, zeros, zeros, zeros, dq, dk, db, (long)co,
                           dgc + co, scale, clip, 0, BT, D, clip);
}

// ---------------------------------------------------------------------------
// B5 (gdn2_bwd.py:32-41): dg = san(reverse in-chunk cumsum of dgc).
__global__ void __launch_bounds__(kThreads)
k_stage_revcumsum(const float* __restrict__ dgc, float* __restrict__ dg, int BT, int D,
                  float clip) {
  const size_t co = (size_t)blockIdx.x * BT * D;
  for (int x = threadIdx.x; x < D; x += kThreads) {
    float acc = 0.f;
    for (int i = BT - 1; i >= 0; --i) {
      acc += dgc[co + i * D + x];
      dg[co + i * D + x] = san(acc, clip);
    }
  }
}

}  // namespace
}  // namespace gdn2

// ---------------------------------------------------------------------------
// C ABI (include/gdn2.h)
namespace {
using namespace gdn2;

// D = 256 (beyond the reference's D = 128, gdn2_fwd.py:145) with BT <= 128:
// the per-chunk gc tile of 256 x 256 floats would not fit shared memory.
bool shape_ok(int BT, int D) {
  return (BT == 64 || BT == 128 || BT == 256) && (D == 64 || D == 128 || D == 256) &&
         !(D == 256 && BT == 256);
}
constexpr size_t kSmemMax = 200 * 1024;   // resident-tile budget of the stage kernels

int bad(const char* what) { return report_error(GDN2_ERR_INVALID, what); }

int launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return GDN2_OK;
  char msg[256];
  snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
  return report_error(GDN2_ERR_CUDA, msg);
}

template <class K>
int smem_attr(K kern, size_t bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
                 cudaSuccess
             ? GDN2_OK
             : launched("stage smem attribute");
}

int dims_ok(int B, int T, int H, int D, int BT) {
  return B > 0 && T > 0 && H > 0 && shape_ok(BT, D) && T % BT == 0;
}
}  // namespace

extern "C" {

int gdn2_stage_scores(int dtype, const void* q, const void* k, const void* b, const void* g,
                      float* aqk, float* akk, int B, int T, int H, int D, int BT, float scale,
                      float clip, void* stream) {
  if (!dims_ok(B, T, H, D, BT) || !q || !k || !b || !g || !aqk || !akk)
    return bad("gdn2_stage_scores: bad shape or null pointer");
  const bool kres = 2 * (size_t)BT * D * sizeof(float) <= kSmemMax;
  const size_t smem = (kres ? 2 : 1) * (size_t)BT * D * sizeof(float);
  const unsigned n = (unsigned)B * H * (T / BT);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == GDN2_F32) {
    if (int rc = smem_attr(k_stage_scores<float>, smem)) return rc;
    k_stage_scores<float><<<n, kThreads, smem, s>>>(
        (const float*)q, (const float*)k, (const float*)b, (const float*)g, aqk, akk, T, H, D, BT,
        scale, clip, kres);
  } else if (dtype == GDN2_BF16) {
    using bf = __nv_bfloat16;
    if (int rc = smem_attr(k_stage_scores<bf>, smem)) return rc;
    k_stage_scores<bf><<<n, kThreads, smem, s>>>((const bf*)q, (const bf*)k, (const bf*)b,
                                                 (const bf*)g, aqk, akk, T, H, D, BT, scale, clip,
                                                 kres);
  } else {
    return bad("gdn2_stage_scores: dtype");
  }
  return launched("gdn2_stage_scores");
}

int gdn2_stage_wy_solve(const float* akk, float* a, float* scratch, int n_chunks, int BT, int BC,
                        float clip, void* stream) {
  if (!akk || !a || n_chunks <= 0 || (BT != 64 && BT != 128 && BT != 256) || BC <= 0 || BC % 16 ||
      BT % BC || (BT == 256 && (BC > 128 || !scratch)))
    return bad("gdn2_stage_wy_solve: bad shape or null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (BT == 256) {   // diagonal blocks in shared memory, then the cross-block substitution
    if (cudaMemsetAsync(a, 0, (size_t)n_chunks * BT * BT * sizeof(float), s) != cudaSuccess)
      return launched("gdn2_stage_wy_solve");
    const unsigned nb = (unsigned)n_chunks * (BT / BC);
    const size_t smem = ((size_t)BC * (BC + 4) + (size_t)BC * BC / 4) * sizeof(float);
#define GDN2_DIAG(CC)                                                                   \
    if (BC == CC) {                                                                     \
      if (int rc = smem_attr(k_stage_wy_diag<CC>, smem)) return rc;                     \
      k_stage_wy_diag<CC><<<nb, kThreads, smem, s>>>(akk, a, BT, clip);                 \
    }
    GDN2_DIAG(16) GDN2_DIAG(32) GDN2_DIAG(64) GDN2_DIAG(128)
#undef GDN2_DIAG
    if (int rc = launched("gdn2_stage_wy_solve")) return rc;
    k_stage_wy_compose<<<n_chunks, kThreads, 0, s>>>(akk, a, scratch, BT, BC, clip);
    return launched("gdn2_stage_wy_solve");
  }
  const size_t smem = ((size_t)BT * (BT + 4) + (size_t)BT * BT / 4) * sizeof(float);
  if (BT == 64) {
    if (int rc = smem_attr(k_stage_wy<64>, smem)) return rc;
    k_stage_wy<64><<<n_chunks, kThreads, smem, s>>>(akk, a, BC, clip);
  } else {
    if (int rc = smem_attr(k_stage_wy<128>, smem)) return rc;
    k_stage_wy<128><<<n_chunks, kThreads, smem, s>>>(akk, a, BC, clip);
  }
  return launched("gdn2_stage_wy_solve");
}

int gdn2_stage_recompute_wy(int dtype, const void* q, const void* k, const void* v, const void* w,
                            const void* b, const void* g, const float* a, float* w_pseudo,
                            float* u, float* kg, float* qg, float* gc_last, int B, int T, int H,
                            int D, int BT, float clip, void* stream) {
  if (!dims_ok(B, T, H, D, BT) || !q || !k || !v || !w || !b || !g || !a || !w_pseudo || !u ||
      !kg || !qg || !gc_last)
    return bad("gdn2_stage_recompute_wy: bad shape or null pointer");
  const bool wres = 2 * (size_t)BT * D * sizeof(float) <= kSmemMax;
  const size_t smem = (wres ? 2 : 1) * (size_t)BT * D * sizeof(float);
  const unsigned n = (unsigned)B * H * (T / BT);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == GDN2_F32) {
    if (int rc = smem_attr(k_stage_recompute<float>, smem)) return rc;
    k_stage_recompute<float><<<n, kThreads, smem, s>>>(
        (const float*)q, (const float*)k, (const float*)v, (const float*)w, (const float*)b,
        (const float*)g, a, w_pseudo, u, kg, qg, gc_last, T, H, D, BT, clip, wres);
  } else if (dtype == GDN2_BF16) {
    using bf = __nv_bfloat16;
    if (int rc = smem_attr(k_stage_recompute<bf>, smem)) return rc;
    k_stage_recompute<bf><<<n, kThreads, smem, s>>>((const bf*)q, (const bf*)k, (const bf*)v,
                                                    (const bf*)w, (const bf*)b, (const bf*)g, a,
                                                    w_pseudo, u, kg, qg, gc_last, T, H, D, BT,
                                                    clip, wres);
  } else {
    return bad("gdn2_stage_recompute_wy: dtype");
  }
  return launched("gdn2_stage_recompute_wy");
}

int gdn2_stage_combine(const float* aqk, const float* w_pseudo, const float* u, const float* kg,
                       const float* qg, const float* gc_last, const float* h0, float* o,
                       float* h_final, float* h_pre_all, float* v_new_all, int B, int H, int nc,
                       int BT, int D, float scale, float clip, void* stream) {
  if (B <= 0 || H <= 0 || nc <= 0 || !shape_ok(BT, D) || !aqk || !w_pseudo || !u || !kg || !qg ||
      !gc_last || !o || !h_final)
    return bad("gdn2_stage_combine: bad shape or null pointer");
  const size_t smem = (size_t)(2 * D + BT) * kNV * sizeof(float);
  if (int rc = smem_attr(k_stage_combine, smem)) return rc;
  k_stage_combine<<<dim3(D / kNV, H, B), kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      aqk, w_pseudo, u, kg, qg, gc_last, h0, o, h_final, h_pre_all, v_new_all, B, H, nc, BT, D,
      scale, clip);
  return launched("gdn2_stage_combine");
}

int gdn2_stage_dhu(const float* dout, const float* dv_partial, const float* w_pseudo,
                   const float* qg, const float* kg, const float* gc_last, const float* dht,
                   float* dh_all, float* dh0, float* dv_all, int B, int H, int nc, int BT, int D,
                   float scale, float clip, void* stream) {
  if (B <= 0 || H <= 0 || nc <= 0 || !shape_ok(BT, D) || !dout || !dv_partial || !w_pseudo ||
      !qg || !kg || !gc_last || !dh_all || !dh0 || !dv_all)
    return bad("gdn2_stage_dhu: bad shape or null pointer");
  const size_t smem = (size_t)(2 * D + BT) * kNV * sizeof(float);
  if (int rc = smem_attr(k_stage_dhu, smem)) return rc;
  k_stage_dhu<<<dim3(D / kNV, H, B), kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      dout, dv_partial, w_pseudo, qg, kg, gc_last, dht, dh_all, dh0, dv_all, H, nc, BT, D, scale,
      clip);
  return launched("gdn2_stage_dhu");
}

int gdn2_stage_dav(const float* aqk, const float* v_new, const float* dout, float* daqk,
                   float* dv, int n_chunks, int BT, int D, float clip, void* stream) {
  if (n_chunks <= 0 || !shape_ok(BT, D) || !aqk || !v_new || !dout || !daqk || !dv)
    return bad("gdn2_stage_dav: bad shape or null pointer");
  k_stage_dav<<<n_chunks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(aqk, v_new, dout,
                                                                             daqk, dv, BT, D, clip);
  return launched("gdn2_stage_dav");
}

int gdn2_stage_wy_dqkg(const float* q, const float* k, const float* b, const float* w,
                       const float* v, const float* gc, const float* a, const float* h_pre,
                       const float* v_new, const float* dout, const float* dv,
                       const float* dh_next, float* dq, float* dk, float* db, float* dw,
                       float* dv_raw, float* dgc, float* dakk, float* scratch, int n_chunks,
                       int BT, int D, float scale, float clip, void* stream) {
  if (n_chunks <= 0 || !shape_ok(BT, D) || !q || !k || !b || !w || !v || !gc || !a || !h_pre ||
      !v_new || !dout || !dv || !dh_next || !dq || !dk || !db || !dw || !dv_raw || !dgc || !dakk ||
      !scratch)
    return bad("gdn2_stage_wy_dqkg: bad shape or null pointer");
  k_stage_wy_dqkg<<<n_chunks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      q, k, b, w, v, gc, a, h_pre, v_new, dout, dv, dh_next, dq, dk, db, dw, dv_raw, dgc, dakk,
      scratch, BT, D, scale, clip);
  return launched("gdn2_stage_wy_dqkg");
}

int gdn2_stage_intra_bwd(int dtype, const float* daqkT, const float* dakkT, const void* q,
                         const void* k, const void* b, const void* g, const float* zeros,
                         float* dq, float* dk, float* db, float* dgc, int B, int T, int H, int D,
                         int BT, int BC, float scale, float clip, void* stream) {
  if (!dims_ok(B, T, H, D, BT) || BC <= 0 || BC % 16 || BT % BC || !daqkT || !dakkT || !q ||
      !k || !b || !g || !zeros || !dq || !dk || !db || !dgc)
    return bad("gdn2_stage_intra_bwd: bad shape or null pointer");
  const size_t smem = (size_t)BT * D * sizeof(float);
  const unsigned n = (unsigned)B * H * (T / BT);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == GDN2_F32) {
    if (int rc = smem_attr(k_stage_intra_bwd<float>, smem)) return rc;
    k_stage_intra_bwd<float><<<n, kThreads, smem, s>>>(
        daqkT, dakkT, (const float*)q, (const float*)k, (const float*)b, (const float*)g, zeros,
        dq, dk, db, dgc, T, H, D, BT, BC, scale, clip);
  } else if (dtype == GDN2_BF16) {
    using bf = __nv_bfloat16;
    if (int rc = smem_attr(k_stage_intra_bwd<bf>, smem)) return rc;
    k_stage_intra_bwd<bf><<<n, kThreads, smem, s>>>(daqkT, dakkT, (const bf*)q, (const bf*)k,
                                                    (const bf*)b, (const bf*)g, zeros, dq, dk, db,
                                                    dgc, T, H, D, BT, BC, scale, clip);
  } else {
    return bad("gdn2_stage_intra_bwd: dtype");
  }
  return launched("gdn2_stage_intra_bwd");
}

int gdn2_stage_revcumsum(const float* dgc, float* dg, int n_chunks, int BT, int D, float clip,
                         void* stream) {
  if (n_chunks <= 0 || BT <= 0 || D <= 0 || !dgc || !dg)
    return bad("gdn2_stage_revcumsum: bad shape or null pointer");
  k_stage_revcumsum<<<n_chunks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(dgc, dg, BT, D,
                                                                                    clip);
  return launched("gdn2_stage_revcumsum");
}

}  // extern "C"
