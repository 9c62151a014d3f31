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
  uint64_t bars[2];
  uint64_t done;
  uint32_t tmem;
  float colpart[4][D];
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
  __shared__ TcSmemB ts;
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
  kloop(ring, g, ws.status,
        [&](int buf, int s) {
          stage_direct(ring.hi(buf, 0), ring.lo(buf, 0), doc, rs, s * KS, Ident{});      // (i,v)
          stage_direct(ring.hi(buf, 1), ring.lo(buf, 1), dvn, D, s * KS, Scale{-1.f});    // (i,v)
          stage_direct(ring.hi(buf, 2), ring.lo(buf, 2), hpre, D, s * KS, Ident{});      // (dk,v)
        },
        [&](int buf, int s) {
          mma3(tmem, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
          mma3(tmem + 128, ring.op(buf, 1), ring.op(buf, 2), 128, KS / 8, s > 0);
        });
  kloop(ring, g, ws.status,
        [&](int buf, int s) {
          stage_direct(ring.hi(buf, 0), ring.lo(buf, 0), vnew, D, s * KS, Ident{});      // (i|j,v)
          stage_direct(ring.hi(buf, 1), ring.lo(buf, 1), doc, rs, s * KS, Ident{});      // (i,v)
          stage_direct(ring.hi(buf, 2), ring.lo(buf, 2), dhn, D, s * KS, Ident{});       // (dk,v)
        },
        [&](int buf, int s) {
          mma3(tmem + 256, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
          mma3(tmem + 384, ring.op(buf, 1), ring.op(buf, 0), 128, KS / 8, s > 0);
        });
  uint32_t ph = 0;
  drain(&ts.done, ph, ws.status);
  // dqg -> pdq = san(dqg e^gc), pdgc = dqg qg
  for_acc<128>(tmem, 0, [&](int i, int c0, const float* x) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      float oq[4], og[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int d = c0 + j + t;
        const float eg = __expf(gc[i * D + d]);
        const float dqg = p.scale * x[j + t];
        oq[t] = san(dqg * eg, p.clip);
        og[t] = dqg * (to_f<T>(qc[i * rs + d]) * eg);
      }
      st4(pdq + i * D + c0 + j, oq[0], oq[1], oq[2], oq[3]);
      st4(pdgc + i * D + c0 + j, og[0], og[1], og[2], og[3]);
    }
  });
  float* dwp = ws.dWp + chunk * C * D;
  for_acc<128>(tmem, 128, [&](int i, int c0, const float* x) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) st4(dwp + i * D + c0 + j, x[j], x[j + 1], x[j + 2], x[j + 3]);
  });
  float* daqkT = ws.dAqkT + chunk * C * C;
  for_acc<128>(tmem, 384, [&](int i, int c0, const float* x) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int jj = c0 + j;
      daqkT[jj * C + i] = (jj <= i) ? san(x[j], p.clip) : 0.f;
    }
  });
  // dkg -> pdk = dkg e^{gc_last - gc}; pdgc -= dkg kg; column sums of dkg kg
  const float* gl = gc + (C - 1) * D;
  const int warp = threadIdx.x >> 5;
  for_acc<128>(tmem, 256, [&](int i, int c0, const float* x) {
    float ok[16], og[16], xs[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = c0 + j;
      const float f = __expf(gl[d] - gc[i * D + d]);
      xs[j] = x[j] * (to_f<T>(kc[i * rs + d]) * f);
      ok[j] = x[j] * f;
      og[j] = pdgc[i * D + d] - xs[j];
    }
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      st4(pdk + i * D + c0 + j, ok[j], ok[j + 1], ok[j + 2], ok[j + 3]);
      st4(pdgc + i * D + c0 + j, og[j], og[j + 1], og[j + 2], og[j + 3]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v = xs[j];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if ((threadIdx.x & 31) == 0) ts.colpart[warp & 3][c0 + j] = v;
    }
  });
  __syncthreads();
  // gc_last row: sum_i dkg kg + e^{gc_last} sum_v dh_next h_pre (gdn2_bwd.py:185, 196-201)
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
    float s = 0.f;
    for (int vv = 0; vv < D; ++vv) s = fmaf(dhn[d * D + vv], hpre[d * D + vv], s);
    const float cs = ((ts.colpart[0][d] + ts.colpart[1][d]) + ts.colpart[2][d]) + ts.colpart[3][d];
    pdgc[(C - 1) * D + d] += cs + __expf(gl[d]) * s;
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
  __shared__ TcSmemB ts;
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
  kloop(ring, g, ws.status,
        [&](int buf, int s) {
          stage_direct(ring.hi(buf, 0), ring.lo(buf, 0), dwp, D, s * KS, Ident{});       // (i,d)
          stage_direct_f(ring.hi(buf, 1), ring.lo(buf, 1), [&](int j, int cc) {          // (j,d) kb
            const int d = s * KS + cc;
            const float4 kv = ld4<T>(kc + j * rs + d), bv = ld4<T>(bc + j * rs + d);
            const float4 g4 = *reinterpret_cast<const float4*>(gc + j * D + d);
            return make_float4(bv.x * kv.x * __expf(g4.x), bv.y * kv.y * __expf(g4.y),
                               bv.z * kv.z * __expf(g4.z), bv.w * kv.w * __expf(g4.w));
          });
        },
        [&](int buf, int s) { mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0); });
  kloop(ring, g, ws.status,
        [&](int buf, int s) {
          stage_direct(ring.hi(buf, 0), ring.lo(buf, 0), dvn, D, s * KS, Ident{});       // (i,d)
          stage_direct_f(ring.hi(buf, 1), ring.lo(buf, 1), [&](int j, int cc) {          // (j,d) wv
            const int d = s * KS + cc;
            const float4 wv = ld4<T>(wc + j * rs + d), vv = ld4<T>(vc + j * rs + d);
            return make_float4(wv.x * vv.x, wv.y * vv.y, wv.z * vv.z, wv.w * vv.w);
          });
        },
        [&](int buf, int s) { mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, 1); });
  drain(&ts.done, ph, ws.status);
  for_acc<128>(tmem, 0, [&](int i, int c0, const float* x) {
#pragma unroll
    for (int j = 0; j < 16; j += 4)
      st4(dA + i * C + c0 + j, san(x[j], p.clip), san(x[j + 1], p.clip), san(x[j + 2], p.clip),
          san(x[j + 3], p.clip));
  });
  __syncthreads();
  // tmp = san(dA A^T)  (contraction over k)
  kloop(ring, g, ws.status,
        [&](int buf, int s) {
          stage_direct(ring.hi(buf, 0), ring.lo(buf, 0), dA, C, s * KS, Ident{});       // (i,k)
          stage_trans(ring.hi(buf, 1), ring.lo(buf, 1), at, C, s * KS, Ident{});         // (j,k)=A(j,k)
        },
        [&](int buf, int s) { mma3(tmem + 128, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0); });
  drain(&ts.done, ph, ws.status);
  for_acc<128>(tmem, 128, [&](int i, int c0, const float* x) {
#pragma unroll
    for (int j = 0; j < 16; j += 4)
      st4(tmp + i * C + c0 + j, san(x[j], p.clip), san(x[j + 1], p.clip), san(x[j + 2], p.clip),
          san(x[j + 3], p.clip));
  });
  __syncthreads();
  // dAkk = -(A^T tmp): (i, j) = sum_k A(k, i) tmp(k, j)
  kloop(ring, g, ws.status,
        [&](int buf, int s) {
          stage_direct(ring.hi(buf, 0), ring.lo(buf, 0), at, C, s * KS, Ident{});       // (i,k)=A(k,i)
          stage_trans(ring.hi(buf, 1), ring.lo(buf, 1), tmp, C, s * KS, Ident{});       // (j,k)=tmp(k,j)
        },
        [&](int buf, int s) { mma3(tmem + 256, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0); });
  // dkb = A^T dWp, dwv = A^T dv: (j, d) = sum_i A(i, j) X(i, d)
  kloop(ring, g, ws.status,
        [&](int buf, int s) {
          stage_direct(ring.hi(buf, 0), ring.lo(buf, 0), at, C, s * KS, Ident{});       // (j,i)=A(i,j)
          stage_trans(ring.hi(buf, 1), ring.lo(buf, 1), dwp, D, s * KS, Ident{});       // (d,i)
          stage_trans(ring.hi(buf, 2), ring.lo(buf, 2), dvn, D, s * KS, Ident{});       // (d,i)
        },
        [&](int buf, int s) {
          mma3(tmem + 384, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
          mma3(tmem, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
        });
  drain(&ts.done, ph, ws.status);
  float* dAkkT = ws.dAkkT + chunk * C * C;
  for_acc<128>(tmem, 256, [&](int i, int c0, const float* x) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int jj = c0 + j;
      dAkkT[jj * C + i] = (jj < i) ? san(-x[j], p.clip) : 0.f;
    }
  });
  float *pdk = ws.pdk + chunk * C * D, *pdb = ws.pdb + chunk * C * D,
        *pdgc = ws.pdgc + chunk * C * D;
  for_acc<128>(tmem, 384, [&](int j, int c0, const float* x) {
#pragma unroll
    for (int t = 0; t < 16; t += 4) {
      float ok[4], ob[4], og[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = c0 + t + u;
        const float eg = __expf(gc[j * D + d]);
        const float kk = to_f<T>(kc[j * rs + d]), bv = to_f<T>(bc[j * rs + d]);
        const float dkb = x[t + u];
        ok[u] = san(pdk[j * D + d] + dkb * eg * bv, p.clip);
        ob[u] = san(dkb * eg * kk, p.clip);
        og[u] = san(pdgc[j * D + d] + dkb * (bv * kk * eg), p.clip);
      }
      st4(pdk + j * D + c0 + t, ok[0], ok[1], ok[2], ok[3]);
      st4(pdb + j * D + c0 + t, ob[0], ob[1], ob[2], ob[3]);
      st4(pdgc + j * D + c0 + t, og[0], og[1], og[2], og[3]);
    }
  });
  for_acc<128>(tmem, 0, [&](int j, int c0, const float* x) {
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const int d = c0 + t;
      dw_out[off + j * rs + d] =
          from_f<T>(san(san(x[t] * to_f<T>(vc[j * rs + d]), p.clip), kFinalClipTc));
      dv_out[off + j * rs + d] =
          from_f<T>(san(san(x[t] * to_f<T>(wc[j * rs + d]), p.clip), kFinalClipTc));
    }
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
