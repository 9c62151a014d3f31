// Tensor-core (tcgen05, 3xTF32) backward intra-chunk passes 1 and 2 of the
// chunk = head dim = 128 path.  Same contracts as k_bwd_intra1 / k_bwd_intra2
// in gdn2_bwd.cu (B2's dAqk and B3, gdn2_bwd.py:84-96, 126-210); every
// product runs as a 128 x 128 x 128 3xTF32 MMA into TMEM.
#include "gdn2_kernels.cuh"
#include "gdn2_tc_stage.cuh"

namespace gdn2 {

using namespace tc;

namespace {

constexpr int C = 128, D = 128;
constexpr float kFinalClipTc = 1e4f;   // gdn2_pipeline.py:34

struct TcSmemB {
  float colpart[8][D];   // first member: 16-byte aligned for float4 stores
  uint64_t bars[2];
  uint64_t done;
  uint32_t tmem;
};

__device__ __forceinline__ uint32_t setup(TcSmemB* s) {
  if ((threadIdx.x >> 5) == 0) tmem_alloc(&s->tmem, 512);
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

__device__ __forceinline__ void teardown(uint32_t tmem) {
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if ((threadIdx.x >> 5) == 0) tmem_free(tmem, 512);
}

__device__ __forceinline__ Ring ring_of(float* base, TcSmemB* s, int nop) {
  Ring r;
  r.base = base;
  r.bars = s->bars;
  r.phase[0] = r.phase[1] = 0;
  r.nop = nop;
  return r;
}

__device__ __forceinline__ void st4(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ldg4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 san4(float4 v, float c) {
  return make_float4(san(v.x, c), san(v.y, c), san(v.z, c), san(v.w, c));
}
__device__ __forceinline__ float4 exp4(float4 v) {
  return make_float4(__expf(v.x), __expf(v.y), __expf(v.z), __expf(v.w));
}

}  // namespace

// ---------------------------------------------------------------------------
// dqg = scale do h_pre^T, dWp = -dv h_pre^T, dkg = vnew dh_next^T,
// dAqk = san((do vnew^T) * causal); writes pdq, pdk, pdgc (+ gc_last row),
// dWp and dAqk^T exactly as k_bwd_intra1.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
k_tc_bwd_intra1(const T* __restrict__ q, const T* __restrict__ k, const float* __restrict__ dout,
                const float* __restrict__ dh_final, Problem p, Workspace ws) {
  extern __shared__ __align__(128) float sm[];
  __shared__ __align__(16) TcSmemB ts;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const int h = (int)(bh % p.H), bb = (int)(bh / p.H);
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const T *qc = q + off, *kc = k + off;
  const float* doc = dout + off;
  const float* gc = ws.gc + chunk * C * D;
  const float* hpre = ws.hpre + chunk * D * D;
  const float* dvn = ws.dv + chunk * C * D;
  const float* vnew = ws.vnew + chunk * C * D;
  const float* dhn = (c + 1 < p.nc) ? ws.dh + (chunk + 1) * D * D : dh_final + bh * D * D;
  float *pdq = ws.pdq + chunk * C * D, *pdk = ws.pdk + chunk * C * D,
        *pdgc = ws.pdgc + chunk * C * D;
  const uint32_t tmem = setup(&ts);
  Ring ring = ring_of(sm, &ts, 3);
  int g = 0;
  // contraction over the value dim v for every product
  {
    const Src srcs[3] = {direct(doc, rs), direct(dvn, D, -1.f), direct(hpre, D)};  // (i,v) (i,v) (dk,v)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
      mma3(tmem + 128, ring.op(buf, 1), ring.op(buf, 2), 128, KS / 8, s > 0);
    });
  }
  {
    const Src srcs[3] = {direct(vnew, D), direct(doc, rs), direct(dhn, D)};  // (i|j,v) (i,v) (dk,v)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem + 256, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
      mma3(tmem + 384, ring.op(buf, 1), ring.op(buf, 0), 128, KS / 8, s > 0);
    });
  }
  uint32_t ph = 0;
  drain(&ts.done, ph, ws.status);
  float* t0 = sm;                  // the ring is free: two padded 128 x 128 tiles
  float* t1 = sm + TILE_FLOATS;
  acc_to_smem<false>(tmem, 0, t0);     // dqg / scale
  acc_to_smem<false>(tmem, 128, t1);   // dWp
  __syncthreads();
  float* dwp = ws.dWp + chunk * C * D;
  for_tile([&](int i, int d) {
    const float4 x = lds4(t0 + i * TLD + d);
    const float4 eg = exp4(ldg4(gc + i * D + d));
    const float4 qv = ld4<T>(qc + i * rs + d);
    const float4 dqg = make_float4(p.scale * x.x, p.scale * x.y, p.scale * x.z, p.scale * x.w);
    st4(pdq + i * D + d, san(dqg.x * eg.x, p.clip), san(dqg.y * eg.y, p.clip),
        san(dqg.z * eg.z, p.clip), san(dqg.w * eg.w, p.clip));
    st4(pdgc + i * D + d, dqg.x * (qv.x * eg.x), dqg.y * (qv.y * eg.y), dqg.z * (qv.z * eg.z),
        dqg.w * (qv.w * eg.w));
    *reinterpret_cast<float4*>(dwp + i * D + d) = lds4(t1 + i * TLD + d);
  });
  __syncthreads();
  acc_to_smem<true>(tmem, 384, t0);    // t0[j][i] = dAqk(i, j)
  acc_to_smem<false>(tmem, 256, t1);   // dkg
  __syncthreads();
  float* daqkT = ws.dAqkT + chunk * C * C;
  for_tile([&](int j, int i) {
    const float4 x = lds4(t0 + j * TLD + i);
    st4(daqkT + j * C + i, j <= i ? san(x.x, p.clip) : 0.f, j <= i + 1 ? san(x.y, p.clip) : 0.f,
        j <= i + 2 ? san(x.z, p.clip) : 0.f, j <= i + 3 ? san(x.w, p.clip) : 0.f);
  });
  // dkg -> pdk = dkg e^{gc_last - gc}; pdgc -= dkg kg; column sums of dkg kg
  const float* gl = gc + (C - 1) * D;
  float cs[4] = {0.f, 0.f, 0.f, 0.f};
  for_tile([&](int i, int d) {
    const float4 x = lds4(t1 + i * TLD + d);
    const float4 g4 = ldg4(gc + i * D + d), l4 = ldg4(gl + d);
    const float4 kv = ld4<T>(kc + i * rs + d);
    const float4 f = exp4(make_float4(l4.x - g4.x, l4.y - g4.y, l4.z - g4.z, l4.w - g4.w));
    const float4 xs = make_float4(x.x * (kv.x * f.x), x.y * (kv.y * f.y), x.z * (kv.z * f.z),
                                  x.w * (kv.w * f.w));
    st4(pdk + i * D + d, x.x * f.x, x.y * f.y, x.z * f.z, x.w * f.w);
    const float4 pg = ldg4(pdgc + i * D + d);
    st4(pdgc + i * D + d, pg.x - xs.x, pg.y - xs.y, pg.z - xs.z, pg.w - xs.w);
    cs[0] += xs.x; cs[1] += xs.y; cs[2] += xs.z; cs[3] += xs.w;
  });
  {
    const int d = (threadIdx.x & 31) * 4;
    st4(&ts.colpart[threadIdx.x >> 5][d], cs[0], cs[1], cs[2], cs[3]);
  }
  __syncthreads();
  // gc_last row: sum_i dkg kg + e^{gc_last} sum_v dh_next h_pre (gdn2_bwd.py:185, 196-201)
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
    float sdot = 0.f;
    for (int vv = 0; vv < D; ++vv) sdot = fmaf(dhn[d * D + vv], hpre[d * D + vv], sdot);
    float csum = 0.f;
    for (int r = 0; r < 8; ++r) csum += ts.colpart[r][d];   // fixed order
    pdgc[(C - 1) * D + d] += csum + __expf(gl[d]) * sdot;
  }
  teardown(tmem);
}

// ---------------------------------------------------------------------------
// dA = san(dWp kb^T + dv wv^T); tmp = san(dA A^T); dAkk = -(A^T tmp) * strict;
// dkb = A^T dWp; dwv = A^T dv -> pdk, pdb, pdgc (sanitised B3 totals), dw, dv,
// exactly as k_bwd_intra2.  dA and tmp pass through the workspace tiles dAkkT
// and E of the chunk (both free at this point of the backward).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
k_tc_bwd_intra2(const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ w,
                const T* __restrict__ b, T* __restrict__ dv_out, T* __restrict__ dw_out, Problem p,
                Workspace ws) {
  extern __shared__ __align__(128) float sm[];
  __shared__ __align__(16) TcSmemB ts;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const int h = (int)(bh % p.H), bb = (int)(bh / p.H);
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const T *kc = k + off, *vc = v + off, *wc = w + off, *bc = b + off;
  const float* gc = ws.gc + chunk * C * D;
  const float* dwp = ws.dWp + chunk * C * D;
  const float* dvn = ws.dv + chunk * C * D;
  const float* at = ws.AT + chunk * C * C;   // at[k*C + j] = A(j, k)
  float* dA = ws.dAkkT + chunk * C * C;      // scratch: dA row-major, later dAkk^T
  float* tmp = ws.E + chunk * D * D;         // scratch: tmp row-major
  const uint32_t tmem = setup(&ts);
  Ring ring = ring_of(sm, &ts, 3);
  int g = 0;
  uint32_t ph = 0;
  // dA = dWp kb^T + dv wv^T  (contraction over d)
  {
    const Src srcs[1] = {direct(dwp, D)};   // (i,d)
    kloop_pf(ring, g, ws.status, srcs,
             [&](int buf, int s) {
               stage_direct_f(ring.hi(buf, 1), ring.lo(buf, 1), [&](int j, int cc) {   // (j,d) kb
                 const int d = s * KS + cc;
                 const float4 kv = ld4<T>(kc + j * rs + d), bv = ld4<T>(bc + j * rs + d);
                 const float4 g4 = *reinterpret_cast<const float4*>(gc + j * D + d);
                 return make_float4(bv.x * kv.x * __expf(g4.x), bv.y * kv.y * __expf(g4.y),
                                    bv.z * kv.z * __expf(g4.z), bv.w * kv.w * __expf(g4.w));
               });
             },
             [&](int buf, int s) { mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0); });
  }
  {
    const Src srcs[1] = {direct(dvn, D)};   // (i,d)
    kloop_pf(ring, g, ws.status, srcs,
             [&](int buf, int s) {
               stage_direct_f(ring.hi(buf, 1), ring.lo(buf, 1), [&](int j, int cc) {   // (j,d) wv
                 const int d = s * KS + cc;
                 const float4 wv = ld4<T>(wc + j * rs + d), vv = ld4<T>(vc + j * rs + d);
                 return make_float4(wv.x * vv.x, wv.y * vv.y, wv.z * vv.z, wv.w * vv.w);
               });
             },
             [&](int buf, int s) { mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, 1); });
  }
  drain(&ts.done, ph, ws.status);
  float* t0 = sm;
  float* t1 = sm + TILE_FLOATS;
  acc_to_smem<false>(tmem, 0, t0);
  __syncthreads();
  for_tile([&](int i, int c4) {
    *reinterpret_cast<float4*>(dA + i * C + c4) = san4(lds4(t0 + i * TLD + c4), p.clip);
  });
  __syncthreads();
  // tmp = san(dA A^T)  (contraction over k)
  {
    const Src srcs[2] = {direct(dA, C), trans(at, C)};   // (i,k) = dA, (j,k) = A(j,k)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem + 128, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  acc_to_smem<false>(tmem, 128, t0);
  __syncthreads();
  for_tile([&](int i, int c4) {
    *reinterpret_cast<float4*>(tmp + i * C + c4) = san4(lds4(t0 + i * TLD + c4), p.clip);
  });
  __syncthreads();
  // dAkk = -(A^T tmp): (i, j) = sum_k A(k, i) tmp(k, j)
  {
    const Src srcs[2] = {direct(at, C), trans(tmp, C)};   // (i,k) = A(k,i), (j,k) = tmp(k,j)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem + 256, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
    });
  }
  // dkb = A^T dWp, dwv = A^T dv: (j, d) = sum_i A(i, j) X(i, d)
  {
    const Src srcs[3] = {direct(at, C), trans(dwp, D), trans(dvn, D)};   // (j,i) (d,i) (d,i)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem + 384, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  float* dAkkT = ws.dAkkT + chunk * C * C;
  acc_to_smem<true>(tmem, 256, t0);    // t0[j][i] = acc(i, j)
  acc_to_smem<false>(tmem, 384, t1);   // dkb (j, d)
  __syncthreads();
  for_tile([&](int j, int i) {
    const float4 x = lds4(t0 + j * TLD + i);
    st4(dAkkT + j * C + i, j < i ? san(-x.x, p.clip) : 0.f, j < i + 1 ? san(-x.y, p.clip) : 0.f,
        j < i + 2 ? san(-x.z, p.clip) : 0.f, j < i + 3 ? san(-x.w, p.clip) : 0.f);
  });
  float *pdk = ws.pdk + chunk * C * D, *pdb = ws.pdb + chunk * C * D,
        *pdgc = ws.pdgc + chunk * C * D;
  for_tile([&](int j, int d) {
    const float4 x = lds4(t1 + j * TLD + d);
    const float4 eg = exp4(ldg4(gc + j * D + d));
    const float4 kv = ld4<T>(kc + j * rs + d), bv = ld4<T>(bc + j * rs + d);
    const float4 pk = ldg4(pdk + j * D + d), pg = ldg4(pdgc + j * D + d);
    st4(pdk + j * D + d, san(pk.x + x.x * eg.x * bv.x, p.clip), san(pk.y + x.y * eg.y * bv.y, p.clip),
        san(pk.z + x.z * eg.z * bv.z, p.clip), san(pk.w + x.w * eg.w * bv.w, p.clip));
    st4(pdb + j * D + d, san(x.x * eg.x * kv.x, p.clip), san(x.y * eg.y * kv.y, p.clip),
        san(x.z * eg.z * kv.z, p.clip), san(x.w * eg.w * kv.w, p.clip));
    st4(pdgc + j * D + d, san(pg.x + x.x * (bv.x * kv.x * eg.x), p.clip),
        san(pg.y + x.y * (bv.y * kv.y * eg.y), p.clip), san(pg.z + x.z * (bv.z * kv.z * eg.z), p.clip),
        san(pg.w + x.w * (bv.w * kv.w * eg.w), p.clip));
  });
  __syncthreads();
  acc_to_smem<false>(tmem, 0, t0);     // dwv (j, d)
  __syncthreads();
  for_tile([&](int j, int d) {
    const float4 x = lds4(t0 + j * TLD + d);
    const float4 vv = ld4<T>(vc + j * rs + d), wv = ld4<T>(wc + j * rs + d);
    const float4 dw = make_float4(x.x * vv.x, x.y * vv.y, x.z * vv.z, x.w * vv.w);
    const float4 dvv = make_float4(x.x * wv.x, x.y * wv.y, x.z * wv.z, x.w * wv.w);
    st4<T>(dw_out + off + j * rs + d, san4(san4(dw, p.clip), kFinalClipTc));
    st4<T>(dv_out + off + j * rs + d, san4(san4(dvv, p.clip), kFinalClipTc));
  });
  teardown(tmem);
}

// ---------------------------------------------------------------------------
template <typename T>
cudaError_t launch_tc_bwd_intra12(const T* q, const T* k, const T* v, const T* w, const T* b,
                                  const float* dout, const float* dh_final, T* dv_out, T* dw_out,
                                  const Problem& p, const Workspace& ws, cudaStream_t s,
                                  const LaunchHook& hook) {
  constexpr size_t smem = 2 * 3 * (size_t)SLICE_BYTES;
  const unsigned nchunks = (unsigned)p.B * p.H * p.nc;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(k_tc_bwd_intra1<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem)) != cudaSuccess)
    return e;
  if ((e = cudaFuncSetAttribute(k_tc_bwd_intra2<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem)) != cudaSuccess)
    return e;
  hook.begin(kStageBwdIntra1, s);
  k_tc_bwd_intra1<T><<<nchunks, kThreads, smem, s>>>(q, k, dout, dh_final, p, ws);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageBwdIntra1, s);
  hook.begin(kStageBwdIntra2, s);
  k_tc_bwd_intra2<T><<<nchunks, kThreads, smem, s>>>(k, v, w, b, dv_out, dw_out, p, ws);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageBwdIntra2, s);
  return cudaSuccess;
}

template cudaError_t launch_tc_bwd_intra12<float>(const float*, const float*, const float*,
                                                  const float*, const float*, const float*,
                                                  const float*, float*, float*, const Problem&,
                                                  const Workspace&, cudaStream_t,
                                                  const LaunchHook&);
template cudaError_t launch_tc_bwd_intra12<__nv_bfloat16>(
    const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
    const __nv_bfloat16*, const float*, const float*, __nv_bfloat16*, __nv_bfloat16*,
    const Problem&, const Workspace&, cudaStream_t, const LaunchHook&);

}  // namespace gdn2
