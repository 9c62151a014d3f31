// Tensor-core (tcgen05, 3xTF32) kernels of the chunk = head dim = 128 path.
//
// The inter-chunk recurrence (reference Kernel D, gdn2_fwd.py:347-360, and
// B1, gdn2_bwd.py:58-75) is evaluated in affine form.  Substituting
// vnew = U - W h into h' = e^{gc_last} h + kg^T vnew gives
//     h_{c+1} = M_c h_c + Bc_c,   M_c = diag(e^{gc_last}) - kg^T W,  Bc_c = kg^T U,
// and the backward pass dh_c = M_c^T dh_{c+1} + E_c with
//     E_c = scale qg^T do - W^T dv_partial,   dv_partial = san(Aqk^T do).
// M_c, Bc_c and E_c are chunk-parallel products; the serial chain keeps one
// 128 x 128 x 128 product per chunk.  The outputs o = scale qg h + Aqk vnew,
// vnew = U - W h and dv_new = san(dv_partial + kg dh_next) are chunk-parallel
// again.  Sanitisers sit where the reference has them (h and dh after every
// chunk, o, dv_partial, dv_new).
#include "gdn2_kernels.cuh"
#include "gdn2_tc_stage.cuh"

namespace gdn2 {

using namespace tc;

namespace {

struct TcSmem {
  uint64_t bars[2];
  uint64_t done;
  uint32_t tmem;
};

// Barriers + TMEM allocation; returns the TMEM base address.
__device__ __forceinline__ uint32_t tc_setup(TcSmem* s, uint32_t ncols) {
  if ((threadIdx.x >> 5) == 0) tmem_alloc(&s->tmem, ncols);
  if (threadIdx.x == 0) {
    mbar_init(&s->bars[0], 1);
    mbar_init(&s->bars[1], 1);
    mbar_init(&s->done, 1);
    fence_mbar_init();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  return s->tmem;
}

__device__ __forceinline__ void tc_teardown(uint32_t tmem, uint32_t ncols) {
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if ((threadIdx.x >> 5) == 0) tmem_free(tmem, ncols);
}

__device__ __forceinline__ Ring make_ring(float* base, TcSmem* s, int nop) {
  Ring r;
  r.base = base;
  r.bars = s->bars;
  r.phase[0] = r.phase[1] = 0;
  r.nop = nop;
  return r;
}

struct SanT {   // sanitise while staging
  float clip;
  __device__ __forceinline__ float4 operator()(float4 v) const {
    return make_float4(san(v.x, clip), san(v.y, clip), san(v.z, clip), san(v.w, clip));
  }
};

constexpr int C = 128, D = 128;

__device__ __forceinline__ float4 ld4f(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4f(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

}  // namespace

// ---------------------------------------------------------------------------
// M = diag(e^{gc_last}) - kg^T W and Bc = kg^T U, one CTA per chunk.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) k_tc_affine(Problem p, Workspace ws) {
  extern __shared__ __align__(128) float sm[];
  __shared__ TcSmem ts;
  const size_t chunk = blockIdx.x;
  const uint32_t tmem = tc_setup(&ts, 256);
  Ring ring = make_ring(sm, &ts, 3);
  const float* kg = ws.kg + chunk * C * D;
  const float* wt = ws.WT + chunk * C * D;
  const float* u = ws.U + chunk * C * D;
  int g = 0;
  const Src srcs[3] = {trans(kg, D), direct(wt, C), trans(u, D)};   // (d,i)=kg, (d',i)=W, (v,i)=U
  kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
    mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
    mma3(tmem + 128, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
  });
  uint32_t ph = 0;
  drain(&ts.done, ph, ws.status);
  float* mo = ws.M + chunk * D * D;
  float* bo = ws.Bc + chunk * D * D;
  const float* gl = ws.gcl + chunk * D;
  for_acc<128>(tmem, 0, [&](int row, int c, const float* v) {
    const float dec = __expf(gl[row]);
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      float4 o = make_float4(-v[j], -v[j + 1], -v[j + 2], -v[j + 3]);
      if (row == c + j) o.x += dec;
      if (row == c + j + 1) o.y += dec;
      if (row == c + j + 2) o.z += dec;
      if (row == c + j + 3) o.w += dec;
      st4f(mo + row * D + c + j, o);
    }
  });
  for_acc<128>(tmem, 128, [&](int row, int c, const float* v) {
#pragma unroll
    for (int j = 0; j < 16; j += 4)
      st4f(bo + row * D + c + j, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
  });
  tc_teardown(tmem, 256);
}

// ---------------------------------------------------------------------------
// Serial affine scan over the chunks of one (batch, head).  The state is kept
// transposed (rows = value column v, cols = key dim d) as the A operand:
//   forward:  h_{c+1}^T = h_c^T M_c^T + Bc_c^T   (state entering every chunk -> ws.hpre)
//   backward: dh_c^T    = dh_{c+1}^T M_c + E_c^T (dh_pre of every chunk -> ws.dh)
// Each step: 4 K-slices of M staged through a two-buffer ring, one
// 128 x 128 x 128 3xTF32 product into TMEM, then the epilogue adds the
// constant term, sanitises, stores the state and restages it as the A tile.
// ---------------------------------------------------------------------------
// PROD (forward only) instead accumulates the segment map P = M_last ... M_first
// from P = I with no constant term and no sanitiser, writing only P to
// out_final (sequence parallelism).
template <bool BWD, bool PROD = false>
__global__ void __launch_bounds__(kThreads, 1)
k_tc_scan(Problem p, Workspace ws, const float* __restrict__ init, float* __restrict__ out_final) {
  extern __shared__ __align__(128) float sm[];
  __shared__ TcSmem ts;
  const int h = blockIdx.x, bb = blockIdx.y;
  const size_t bh = (size_t)bb * p.H + h;
  const uint32_t tmem = tc_setup(&ts, 128);
  float* S = sm;                                     // 4 slices x (hi, lo) of 128 x 32
  Ring ring = make_ring(sm + 4 * 2 * SLICE_FLOATS, &ts, 1);
  auto s_hi = [&](int s) { return S + s * 2 * SLICE_FLOATS; };
  auto s_lo = [&](int s) { return S + s * 2 * SLICE_FLOATS + SLICE_FLOATS; };

  const float* src0 = init ? init + bh * D * D : nullptr;
  if (PROD) {
    for (int e = threadIdx.x; e < D * D / 4; e += kThreads) {   // identity, transposed = itself
      const int r = e / (D / 4), cc = (e % (D / 4)) * 4;
      float4 v4 = make_float4(r == cc ? 1.f : 0.f, r == cc + 1 ? 1.f : 0.f, r == cc + 2 ? 1.f : 0.f,
                              r == cc + 3 ? 1.f : 0.f);
      st_split4(S + (cc / KS) * 2 * SLICE_FLOATS, S + (cc / KS) * 2 * SLICE_FLOATS + SLICE_FLOATS, r,
                cc % KS, KS, v4);
    }
  } else if (src0) {
    for (int s = 0; s < D / KS; ++s) stage_trans(s_hi(s), s_lo(s), src0, D, s * KS, SanT{p.clip});
  } else {
    for (int e = threadIdx.x; e < 4 * 2 * SLICE_FLOATS / 4; e += kThreads)
      st4f(S + 4 * e, make_float4(0.f, 0.f, 0.f, 0.f));
  }
  if (!BWD && !PROD) {
    float* hp = ws.hpre + (bh * p.nc) * D * D;
    for (int e = threadIdx.x; e < D * D; e += kThreads) hp[e] = src0 ? san(src0[e], p.clip) : 0.f;
  }
  uint32_t ph = 0;
  int g = 0;   // slice counter over the whole scan (ring phases)
  // Register prefetch: this thread's share of the next M (4 slices) and of
  // the constant term it adds in the epilogue (row v, 64 columns d).
  const int warp = threadIdx.x >> 5;
  const int vrow = 32 * (warp & 3) + (threadIdx.x & 31);
  const int dcol0 = (warp >> 2) * 64;
  Frag mf[4];
  float addv[64];
  auto load_m = [&](int c) {
    const float* m = ws.M + (bh * p.nc + c) * D * D;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if (!BWD) load_direct(mf[s], m, D, s * KS);
      else load_trans(mf[s], m, D, s * KS);
    }
  };
  auto load_add = [&](int c) {
    const float* add = (BWD ? ws.E : ws.Bc) + (bh * p.nc + c) * D * D;
#pragma unroll
    for (int j = 0; j < 64; ++j) addv[j] = PROD ? 0.f : __ldg(add + (dcol0 + j) * D + vrow);
  };
  load_m(BWD ? p.nc - 1 : 0);
  for (int it = 0; it < p.nc; ++it) {
    const int c = BWD ? p.nc - 1 - it : it;
    const size_t chunk = bh * p.nc + c;
    load_add(c);
    for (int s = 0; s < D / KS; ++s, ++g) {
      const int buf = g & 1;
      ring_acquire(ring, buf, g >> 1, ws.status);
      if (!BWD) store_direct(ring.hi(buf, 0), ring.lo(buf, 0), mf[s]);   // (d, d') = M
      else store_trans(ring.hi(buf, 0), ring.lo(buf, 0), mf[s]);         // (d', d) = M(d, d')
      slice_publish();
      if (threadIdx.x == 0) {
        mma3(tmem, kmajor(s_hi(s), s_lo(s), KS), ring.op(buf, 0), 128, KS / 8, s > 0);
        commit(&ring.bars[buf]);
      }
    }
    if (it + 1 < p.nc) load_m(BWD ? c - 1 : c + 1);
    drain(&ts.done, ph, ws.status);
    const bool last = it == p.nc - 1;
    float* dst;
    if (PROD) dst = last ? out_final + bh * D * D : nullptr;
    else if (!BWD) dst = last ? (out_final ? out_final + bh * D * D : nullptr) : ws.hpre + (chunk + 1) * D * D;
    else dst = ws.dh + chunk * D * D;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c0 = dcol0 + q * 16;
      float x[16];
      tmem_ld16(lane_quarter_addr(tmem, c0), x);
      float y[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        y[j] = PROD ? x[j] : san(x[j] + addv[q * 16 + j], p.clip);
        if (dst) dst[(c0 + j) * D + vrow] = y[j];
        if (BWD && last && out_final) out_final[bh * D * D + (c0 + j) * D + vrow] = san(y[j], 1e4f);
      }
      const int s = c0 / KS, cc = c0 % KS;
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        st_split4(s_hi(s), s_lo(s), vrow, cc + j, KS, make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]));
    }
  }
  tc_teardown(tmem, 128);
}

// ---------------------------------------------------------------------------
// Chunk outputs from the chunk-entry state h (gdn2_fwd.py:349-359):
//   vnew = U - W h  (-> ws.vnew),   o = san(scale qg h + Aqk vnew)  (-> o)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
k_tc_fwd_out(Problem p, Workspace ws, float* __restrict__ o) {
  extern __shared__ __align__(128) float sm[];
  __shared__ TcSmem ts;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const int h = (int)(bh % p.H), bb = (int)(bh / p.H);
  const uint32_t tmem = tc_setup(&ts, 256);
  Ring ring = make_ring(sm, &ts, 3);
  const float* wt = ws.WT + chunk * C * D;
  const float* qgt = ws.qgT + chunk * C * D;
  const float* hp = ws.hpre + chunk * D * D;
  int g = 0;
  {
    const Src srcs[3] = {trans(wt, C), trans(qgt, C, p.scale), trans(hp, D)};  // W, s qg, h^T
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
      mma3(tmem + 128, ring.op(buf, 1), ring.op(buf, 2), 128, KS / 8, s > 0);
    });
  }
  uint32_t ph = 0;
  drain(&ts.done, ph, ws.status);
  const float* u = ws.U + chunk * C * D;
  float* vn = ws.vnew + chunk * C * D;
  for_acc<128>(tmem, 0, [&](int i, int c0, const float* x) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      const float4 uu = ld4f(u + i * D + c0 + j);
      st4f(vn + i * D + c0 + j,
           make_float4(uu.x - x[j], uu.y - x[j + 1], uu.z - x[j + 2], uu.w - x[j + 3]));
    }
  });
  __syncthreads();   // vnew (global) visible to the whole CTA
  const float* aqkt = ws.AqkT + chunk * C * C;
  {
    const Src srcs[2] = {trans(aqkt, C), trans(vn, D)};   // (i,j) = Aqk, (v,j) = vnew(j,v)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem + 128, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, 1);
    });
  }
  drain(&ts.done, ph, ws.status);
  if (o) {
    const long rs = p.row_stride();
    float* orow = o + ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
    for_acc<128>(tmem, 128, [&](int i, int c0, const float* x) {
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        st4f(orow + i * rs + c0 + j, make_float4(san(x[j], p.clip), san(x[j + 1], p.clip),
                                                 san(x[j + 2], p.clip), san(x[j + 3], p.clip)));
    });
  }
  tc_teardown(tmem, 256);
}

// ---------------------------------------------------------------------------
// Backward chunk-parallel terms of the state pass:
//   dv_partial = san(Aqk^T do)  (B2, gdn2_bwd.py:93)          -> ws.dvp
//   E = scale qg^T do - W^T dv_partial                        -> ws.E
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
k_tc_bwd_prep(Problem p, Workspace ws, const float* __restrict__ dout) {
  extern __shared__ __align__(128) float sm[];
  __shared__ TcSmem ts;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const int h = (int)(bh % p.H), bb = (int)(bh / p.H);
  const uint32_t tmem = tc_setup(&ts, 256);
  Ring ring = make_ring(sm, &ts, 3);
  const long rs = p.row_stride();
  const float* doc = dout + ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const float* aqkt = ws.AqkT + chunk * C * C;
  const float* qgt = ws.qgT + chunk * C * D;
  int g = 0;
  {
    const Src srcs[3] = {direct(aqkt, C), direct(qgt, C, p.scale), trans(doc, rs)};  // (j,i) (d,i) (v,i)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
      mma3(tmem + 128, ring.op(buf, 1), ring.op(buf, 2), 128, KS / 8, s > 0);
    });
  }
  uint32_t ph = 0;
  drain(&ts.done, ph, ws.status);
  float* dvp = ws.dvp + chunk * C * D;
  for_acc<128>(tmem, 0, [&](int j, int c0, const float* x) {
#pragma unroll
    for (int k = 0; k < 16; k += 4)
      st4f(dvp + j * D + c0 + k, make_float4(san(x[k], p.clip), san(x[k + 1], p.clip),
                                             san(x[k + 2], p.clip), san(x[k + 3], p.clip)));
  });
  __syncthreads();
  const float* wt = ws.WT + chunk * C * D;
  {
    const Src srcs[2] = {direct(wt, C, -1.f), trans(dvp, D)};   // (d,j) = -W, (v,j) = dvp
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem + 128, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, 1);
    });
  }
  drain(&ts.done, ph, ws.status);
  float* eo = ws.E + chunk * D * D;
  for_acc<128>(tmem, 128, [&](int d, int c0, const float* x) {
#pragma unroll
    for (int k = 0; k < 16; k += 4) st4f(eo + d * D + c0 + k, make_float4(x[k], x[k + 1], x[k + 2], x[k + 3]));
  });
  tc_teardown(tmem, 256);
}

// ---------------------------------------------------------------------------
// dv_new = san(dv_partial + kg dh_next)  (gdn2_bwd.py:66-68)  -> ws.dv
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
k_tc_bwd_dvn(Problem p, Workspace ws, const float* __restrict__ dh_final) {
  extern __shared__ __align__(128) float sm[];
  __shared__ TcSmem ts;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const uint32_t tmem = tc_setup(&ts, 128);
  Ring ring = make_ring(sm, &ts, 2);
  const float* kg = ws.kg + chunk * C * D;
  const float* dhn = (c + 1 < p.nc) ? ws.dh + (chunk + 1) * D * D : dh_final + bh * D * D;
  int g = 0;
  const Src srcs[2] = {direct(kg, D), trans(dhn, D)};   // (i,d), (v,d)
  kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
    mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
  });
  uint32_t ph = 0;
  drain(&ts.done, ph, ws.status);
  const float* dvp = ws.dvp + chunk * C * D;
  float* dv = ws.dv + chunk * C * D;
  for_acc<128>(tmem, 0, [&](int i, int c0, const float* x) {
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      const float4 a = ld4f(dvp + i * D + c0 + k);
      st4f(dv + i * D + c0 + k, make_float4(san(a.x + x[k], p.clip), san(a.y + x[k + 1], p.clip),
                                            san(a.z + x[k + 2], p.clip), san(a.w + x[k + 3], p.clip)));
    }
  });
  tc_teardown(tmem, 128);
}

// ---------------------------------------------------------------------------
namespace {
template <class K>
cudaError_t prep(K kern, size_t smem) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}
constexpr size_t kRing3 = 2 * 3 * (size_t)SLICE_BYTES;   // 192 KB
constexpr size_t kRing2 = 2 * 2 * (size_t)SLICE_BYTES;   // 128 KB
constexpr size_t kScan = 6 * (size_t)SLICE_BYTES;        // state tile + ring, 192 KB
}  // namespace

cudaError_t launch_tc_fwd(const Problem& p, const Workspace& ws, const float* h0, float* o,
                          float* hfinal, cudaStream_t s, const LaunchHook& hook) {
  cudaError_t e;
  const unsigned nchunks = (unsigned)p.B * p.H * p.nc;
  if ((e = prep(k_tc_affine, kRing3)) != cudaSuccess) return e;
  if ((e = prep(k_tc_scan<false>, kScan)) != cudaSuccess) return e;
  if ((e = prep(k_tc_fwd_out, kRing3)) != cudaSuccess) return e;
  hook.begin(kStageFwdAffine, s);
  k_tc_affine<<<nchunks, kThreads, kRing3, s>>>(p, ws);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageFwdAffine, s);
  hook.begin(kStageFwdScan, s);
  k_tc_scan<false><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, h0, hfinal);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageFwdScan, s);
  hook.begin(kStageFwdOut, s);
  k_tc_fwd_out<<<nchunks, kThreads, kRing3, s>>>(p, ws, o);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageFwdOut, s);
  return cudaSuccess;
}

cudaError_t launch_tc_bwd_state(const Problem& p, const Workspace& ws, const float* dout,
                                const float* dh_final, float* dh0, cudaStream_t s,
                                const LaunchHook& hook) {
  cudaError_t e;
  const unsigned nchunks = (unsigned)p.B * p.H * p.nc;
  if ((e = prep(k_tc_bwd_prep, kRing3)) != cudaSuccess) return e;
  if ((e = prep(k_tc_scan<true>, kScan)) != cudaSuccess) return e;
  if ((e = prep(k_tc_bwd_dvn, kRing2)) != cudaSuccess) return e;
  hook.begin(kStageBwdPrep, s);
  k_tc_bwd_prep<<<nchunks, kThreads, kRing3, s>>>(p, ws, dout);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageBwdPrep, s);
  hook.begin(kStageBwdScan, s);
  k_tc_scan<true><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, dh_final, dh0);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageBwdScan, s);
  hook.begin(kStageBwdDvn, s);
  k_tc_bwd_dvn<<<nchunks, kThreads, kRing2, s>>>(p, ws, dh_final);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageBwdDvn, s);
  return cudaSuccess;
}

}  // namespace gdn2

namespace gdn2 {
cudaError_t launch_tc_sp(int op, const Problem& p, const Workspace& ws, const float* in,
                         float* o, float* out, cudaStream_t s, const LaunchHook& hook) {
  cudaError_t e;
  const unsigned nchunks = (unsigned)p.B * p.H * p.nc;
  if (op == 0) {            // forward segment map P = prod M_c
    if ((e = prep(k_tc_scan<false, true>, kScan)) != cudaSuccess) return e;
    k_tc_scan<false, true><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, nullptr, out);
    return cudaGetLastError();
  }
  if (op == 1) {            // rescan from a given start state + chunk outputs
    if ((e = prep(k_tc_scan<false>, kScan)) != cudaSuccess) return e;
    if ((e = prep(k_tc_fwd_out, kRing3)) != cudaSuccess) return e;
    hook.begin(kStageFwdScan, s);
    k_tc_scan<false><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, in, out);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    hook.end(kStageFwdScan, s);
    hook.begin(kStageFwdOut, s);
    k_tc_fwd_out<<<nchunks, kThreads, kRing3, s>>>(p, ws, o);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    hook.end(kStageFwdOut, s);
    return cudaSuccess;
  }
  // op == 2: backward segment term, zero incoming gradient
  if ((e = prep(k_tc_bwd_prep, kRing3)) != cudaSuccess) return e;
  if ((e = prep(k_tc_scan<true>, kScan)) != cudaSuccess) return e;
  k_tc_bwd_prep<<<nchunks, kThreads, kRing3, s>>>(p, ws, in);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  k_tc_scan<true><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, nullptr, out);
  return cudaGetLastError();
}
}  // namespace gdn2
