// Tensor-core (tcgen05, 3xTF32) backward intra-chunk passes 1 and 2 of the
// chunk = head dim = 128 path.  Same contracts as k_bwd_intra1 / k_bwd_intra2
// in gdn2_bwd.cu (B2's dAqk and B3, gdn2_bwd.py:84-96, 126-210); every
// product runs as a 128 x 128 x 128 3xTF32 MMA into TMEM.
#include "gdn2_b4_exact.cuh"
#include "gdn2_kernels.cuh"
#include "gdn2_tc_stage.cuh"

// Optional per-phase cycle counts of one CTA (build with -DGDN2_PHASE_TIMING;
// the counts are printed by that CTA).  Compiled out otherwise.
#ifdef GDN2_PHASE_TIMING
#include <cstdio>
#define GDN2_TMARK(i) \
  do { if (blockIdx.x == gridDim.x / 2 && threadIdx.x == 0) tmark[i] = clock64(); } while (0)
#define GDN2_TPRINT(name, n)                                                         \
  do {                                                                               \
    if (blockIdx.x == gridDim.x / 2 && threadIdx.x == 0) {                           \
      printf("%s phases:", name);                                                    \
      for (int i_ = 1; i_ < n; ++i_) printf(" %lld", tmark[i_] - tmark[i_ - 1]);     \
      printf("\n");                                                                 \
    }                                                                                \
  } while (0)
#define GDN2_TDECL long long tmark[16]; long long tsub[4] = {0, 0, 0, 0}, tsub0 = 0
#define GDN2_TSUB(i)                                                                   \
  do {                                                                                 \
    if (blockIdx.x == gridDim.x / 2 && threadIdx.x == 0) {                             \
      const long long t_ = clock64();                                                  \
      if (i > 0) tsub[i - 1] += t_ - tsub0;                                            \
      tsub0 = t_;                                                                      \
    }                                                                                  \
  } while (0)
#define GDN2_TSUBPRINT(name)                                                           \
  do {                                                                                 \
    if (blockIdx.x == gridDim.x / 2 && threadIdx.x == 0)                               \
      printf("%s slices: %lld %lld %lld %lld\n", name, tsub[0], tsub[1], tsub[2], tsub[3]); \
  } while (0)
#else
#define GDN2_TSUB(i) do { } while (0)
#define GDN2_TSUBPRINT(name) do { } while (0)
#define GDN2_TMARK(i) do { } while (0)
#define GDN2_TPRINT(name, n) do { } while (0)
#define GDN2_TDECL
#endif

namespace gdn2 {

using namespace tc;

namespace {

constexpr int C = 128, D = 128;
constexpr float kFinalClipTc = 1e4f;   // gdn2_pipeline.py:34

struct TcSmemB {
  float colpart[8][D];   // first member: 16-byte aligned for float4 stores
  float colpart1[8][D];  // the second chunk's sums (paired tiles)
  float rowdot[D];
  float rowdot1[D];
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
// dv = san(dv_partial + kg dh_next) (B1's dv_new, gdn2_bwd.py:66-68, -> ws.dv),
// then dqg = scale do h_pre^T, dWp = -dv h_pre^T, dkg = vnew dh_next^T,
// dAqk = san((do vnew^T) * causal); writes pdq, pdk, pdgc (+ gc_last row),
// dWp and dAqk^T exactly as k_bwd_intra1.  dv stays in TMEM as the A operand
// of dWp.
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
  const float* vnew = ws.vnew + chunk * C * D;
  const float* dhn = (c + 1 < p.nc) ? ws.dh + (chunk + 1) * D * D : dh_final + bh * D * D;
  float *pdq = ws.pdq + chunk * C * D, *pdk = ws.pdk + chunk * C * D,
        *pdgc = ws.pdgc + chunk * C * D;
  GDN2_TDECL;
  GDN2_TMARK(0);
  const uint32_t tmem = setup(&ts);
  Ring ring = ring_of(sm, &ts, 2);
  int g = 0;
  uint32_t ph = 0;
  // dv = san(dvp + kg dh_next)  (TMEM 0, contraction over d).  B1 carries
  // the sanitised dh_final into the last chunk (gdn2_bwd.py:53), while B3's
  // dh_next is the raw dh_final (gdn2_pipeline.py:52-56): only this product
  // sees it clipped.
  {
    const float dclip = (c + 1 < p.nc) ? 0.f : p.clip;
    const Src srcs[2] = {direct(ws.kg + chunk * C * D, D), trans(dhn, D, 1.f, dclip)};   // (i,d), (v,d)
    kloop_pf<false>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  GDN2_TMARK(1);
  {
    const float* dvp = ws.dvp + chunk * C * D;
    float* dv = ws.dv + chunk * C * D;
    // every dv_partial load of this thread (its row, 64 columns) before the
    // first dv store, which the compiler must assume may alias them
    const int warp = threadIdx.x >> 5;
    const int row = 32 * (warp & 3) + (threadIdx.x & 31), cb = (warp >> 2) * 64;
    float4 avs[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) avs[k] = *reinterpret_cast<const float4*>(dvp + row * D + cb + 4 * k);
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      const int i = row, c0 = cb + 16 * grp;
      float x[16];
      tmem_ld16(lane_quarter_addr(tmem, c0), x);
      float hv[16], lv[16];
#pragma unroll
      for (int k = 0; k < 16; k += 4) {
        const float4 a = avs[grp * 4 + k / 4];
        const float4 y = make_float4(san(a.x + x[k], p.clip), san(a.y + x[k + 1], p.clip),
                                     san(a.z + x[k + 2], p.clip), san(a.w + x[k + 3], p.clip));
        *reinterpret_cast<float4*>(dv + i * D + c0 + k) = y;
        split(-y.x, hv[k], lv[k]);
        split(-y.y, hv[k + 1], lv[k + 1]);
        split(-y.z, hv[k + 2], lv[k + 2]);
        split(-y.w, hv[k + 3], lv[k + 3]);
      }
      tmem_st16(lane_quarter_addr(tmem, 256 + c0), hv);   // -dv: A operand (rows i, K = v)
      tmem_st16(lane_quarter_addr(tmem, 384 + c0), lv);
    }
    tmem_st_wait();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  GDN2_TMARK(2);
  // contraction over the value dim v for every product
  {
    const Src srcs[2] = {direct(doc, rs), direct(hpre, D)};  // (i,v) (dk,v)
    kloop_pf<false>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
      mma3_ta(tmem + 128, tmem + 256 + s * KS, tmem + 384 + s * KS, ring.op(buf, 1), 128, KS / 8,
              s > 0);
    });
  }
  drain(&ts.done, ph, ws.status);   // TMEM 256..511 free again
  GDN2_TMARK(3);
  ring.nop = 3;
  {
    const Src srcs[3] = {direct(vnew, D), direct(doc, rs), direct(dhn, D)};  // (i|j,v) (i,v) (dk,v)
    kloop_pf<false>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem + 256, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
      mma3(tmem + 384, ring.op(buf, 1), ring.op(buf, 0), 128, KS / 8, s > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  GDN2_TMARK(4);
  float* t0 = sm;                  // the ring is free: two padded 128 x 128 tiles
  float* t1 = sm + TILE_FLOATS;
  float* dwp = ws.dWp + chunk * C * D;
  for_acc<128>(tmem, 128, [&](int i, int c0, const float* x) {   // dWp straight out
#pragma unroll
    for (int j = 0; j < 16; j += 4) st4(dwp + i * D + c0 + j, x[j], x[j + 1], x[j + 2], x[j + 3]);
  });
  acc_to_smem<false>(tmem, 0, t0);     // dqg / scale
  acc_to_smem<false>(tmem, 256, t1);   // dkg
  __syncthreads();
  GDN2_TMARK(5);
  // pdq = dqg e^gc; pdk = dkg e^{gc_last - gc}; pdgc = dqg q e^gc - dkg kg;
  // column sums of dkg kg
  const float* gl = gc + (C - 1) * D;
  float cs[4] = {0.f, 0.f, 0.f, 0.f};
  // the for_tile walk (row i = warp + 8 it, columns d = 4 lane), four rows at
  // a time with all their global loads issued before any store: the stores
  // may alias the loads for the compiler, which would otherwise serialise
  // one memory latency per row
  {
    const int d = (threadIdx.x & 31) * 4;
    const float4 l4 = ldg4(gl + d);
#pragma unroll 1
    for (int it0 = 0; it0 < 16; it0 += 4) {
      float4 g4[4], qv[4], kv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = (threadIdx.x >> 5) + 8 * (it0 + u);
        g4[u] = ldg4(gc + i * D + d);
        qv[u] = ld4<T>(qc + i * rs + d);
        kv[u] = ld4<T>(kc + i * rs + d);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = (threadIdx.x >> 5) + 8 * (it0 + u);
        const float4 x = lds4(t0 + i * TLD + d), y = lds4(t1 + i * TLD + d);
        const float4 eg = exp4(g4[u]);
        const float4 dqg = make_float4(p.scale * x.x, p.scale * x.y, p.scale * x.z, p.scale * x.w);
        st4(pdq + i * D + d, san(dqg.x * eg.x, p.clip), san(dqg.y * eg.y, p.clip),
            san(dqg.z * eg.z, p.clip), san(dqg.w * eg.w, p.clip));
        const float4 q4 = qv[u], k4 = kv[u], gg = g4[u];
        const float4 pg = make_float4(dqg.x * (q4.x * eg.x), dqg.y * (q4.y * eg.y),
                                      dqg.z * (q4.z * eg.z), dqg.w * (q4.w * eg.w));
        const float4 f = exp4(make_float4(l4.x - gg.x, l4.y - gg.y, l4.z - gg.z, l4.w - gg.w));
        const float4 xs = make_float4(y.x * (k4.x * f.x), y.y * (k4.y * f.y), y.z * (k4.z * f.z),
                                      y.w * (k4.w * f.w));
        st4(pdk + i * D + d, y.x * f.x, y.y * f.y, y.z * f.z, y.w * f.w);
        st4(pdgc + i * D + d, pg.x - xs.x, pg.y - xs.y, pg.z - xs.z, pg.w - xs.w);
        cs[0] += xs.x; cs[1] += xs.y; cs[2] += xs.z; cs[3] += xs.w;
      }
    }
  }
  GDN2_TMARK(6);
  float* daqkT = ws.dAqkT + chunk * C * C;
  for_acc<128>(tmem, 384, [&](int i, int c, const float* v) {   // dAqk^T, coalesced per column
#pragma unroll
    for (int t = 0; t < 16; ++t) daqkT[(c + t) * C + i] = c + t <= i ? san(v[t], p.clip) : 0.f;
  });
  {
    const int d = (threadIdx.x & 31) * 4;
    st4(&ts.colpart[threadIdx.x >> 5][d], cs[0], cs[1], cs[2], cs[3]);
  }
  // rowdot[d] = sum_v dh_next(d, v) h_pre(d, v): one warp per 16 rows, a lane
  // per 4 columns, fixed-order shuffle reduction
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll 4
    for (int rr = 0; rr < D / 8; ++rr) {
      const int d = warp * (D / 8) + rr;
      const float4 a = *reinterpret_cast<const float4*>(dhn + d * D + lane * 4);
      const float4 h4 = *reinterpret_cast<const float4*>(hpre + d * D + lane * 4);
      float v = a.x * h4.x + a.y * h4.y + a.z * h4.z + a.w * h4.w;
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) ts.rowdot[d] = v;
    }
  }
  __syncthreads();
  // gc_last row: sum_i dkg kg + e^{gc_last} sum_v dh_next h_pre (gdn2_bwd.py:185, 196-201)
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
    const float sdot = ts.rowdot[d];
    float csum = 0.f;
    for (int r = 0; r < 8; ++r) csum += ts.colpart[r][d];   // fixed order
    pdgc[(C - 1) * D + d] += csum + __expf(gl[d]) * sdot;
  }
  GDN2_TMARK(7);
  teardown(tmem);
  GDN2_TMARK(8);
  GDN2_TPRINT("bwd_intra1", 9);
}

// ---------------------------------------------------------------------------
// k_tc_bwd_intra1 for a tile of two 64-row chunks (BT = 64).  Every product
// that meets a state (h_pre or dh_next of the chunk) runs as one K loop per
// chunk with the other chunk's rows masked, accumulating in TMEM; dWp is
// formed transposed, (dk, i) = h_pre (-dv)^T, because the A operand of the
// single-chunk form (-dv in TMEM) cannot be row-masked.  gc_last, the column
// sums and the state row dots are per chunk; dAqk is block-diagonal.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
k_tc_bwd_intra1_pair(const T* __restrict__ q, const T* __restrict__ k,
                     const float* __restrict__ dout, const float* __restrict__ dh_final,
                     Problem p, Workspace ws) {
  extern __shared__ __align__(128) float sm[];
  __shared__ __align__(16) TcSmemB ts;
  constexpr int R = C / 2;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const int h = (int)(bh % p.H), bb = (int)(bh / p.H);
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const T *qc = q + off, *kc = k + off;
  const float* doc = dout + off;
  const float* gc = ws.gc + chunk * C * D;
  const float* vnew = ws.vnew + chunk * C * D;
  const size_t sc0 = chunk * 2;   // first reference chunk of the tile
  const float* hp[2] = {ws.hpre + sc0 * D * D, ws.hpre + (sc0 + 1) * D * D};
  const bool last_tile = c + 1 == p.nc;
  const float* dhn[2] = {ws.dh + (sc0 + 1) * D * D,
                         last_tile ? dh_final + bh * D * D : ws.dh + (sc0 + 2) * D * D};
  float *pdq = ws.pdq + chunk * C * D, *pdk = ws.pdk + chunk * C * D,
        *pdgc = ws.pdgc + chunk * C * D;
  float* dv = ws.dv + chunk * C * D;
  const uint32_t tmem = setup(&ts);
  Ring ring = ring_of(sm, &ts, 2);
  int g = 0;
  uint32_t ph = 0;
  // dv = san(dvp + kg dh_next)  (TMEM 0); only the last chunk of the
  // sequence sees dh_final, sanitised (gdn2_bwd.py:53)
#pragma unroll 1
  for (int hf = 0; hf < 2; ++hf) {
    const float dclip = (hf == 1 && last_tile) ? p.clip : 0.f;
    const Src srcs[2] = {rows(direct(ws.kg + chunk * C * D, D), hf * R, hf * R + R),
                         trans(dhn[hf], D, 1.f, dclip)};   // (i,d), (v,d)
    kloop_pf<false, 4, true>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0 || hf > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  {
    // every dv_partial load of this thread before the first dv store
    const float* dvp = ws.dvp + chunk * C * D;
    const int warp = threadIdx.x >> 5;
    const int i = 32 * (warp & 3) + (threadIdx.x & 31), cb = (warp >> 2) * 64;
    float4 avs[16];
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) avs[kk] = *reinterpret_cast<const float4*>(dvp + i * D + cb + 4 * kk);
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      const int c0 = cb + 16 * grp;
      float x[16];
      tmem_ld16(lane_quarter_addr(tmem, c0), x);
#pragma unroll
      for (int kk = 0; kk < 16; kk += 4) {
        const float4 a = avs[grp * 4 + kk / 4];
        *reinterpret_cast<float4*>(dv + i * D + c0 + kk) =
            make_float4(san(a.x + x[kk], p.clip), san(a.y + x[kk + 1], p.clip),
                        san(a.z + x[kk + 2], p.clip), san(a.w + x[kk + 3], p.clip));
      }
    }
  }
  fence_before_sync();
  __syncthreads();   // dv in global memory for the staging below; TMEM 0 free
  fence_after_sync();
  // dqg = do h_pre^T (i, dk) at TMEM 0; dWp^T = h_pre (-dv)^T (dk, i) at 128
  ring.nop = 3;
#pragma unroll 1
  for (int hf = 0; hf < 2; ++hf) {
    const Src srcs[3] = {rows(direct(doc, rs), hf * R, hf * R + R), direct(hp[hf], D),
                         rows(direct(dv, D, -1.f), hf * R, hf * R + R)};   // (i,v) (dk,v) (i,v)
    kloop_pf<false, 4, true>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0 || hf > 0);
      mma3(tmem + 128, ring.op(buf, 1), ring.op(buf, 2), 128, KS / 8, s > 0 || hf > 0);
    });
  }
  // dkg = vnew dh_next^T (j, dk) at TMEM 256 (B3's raw dh_next,
  // gdn2_pipeline.py:52-56); do vnew^T (i, j) at 384
#pragma unroll 1
  for (int hf = 0; hf < 2; ++hf) {
    const Src srcs[3] = {rows(direct(vnew, D), hf * R, hf * R + R), direct(doc, rs),
                         direct(dhn[hf], D)};   // (j,v) (i,v) (dk,v)
    kloop_pf<false, 4, true>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem + 256, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0 || hf > 0);
      mma3(tmem + 384, ring.op(buf, 1), ring.op(buf, 0), 128, KS / 8, s > 0 || hf > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  float* t0 = sm;                  // the ring is free: two padded 128 x 128 tiles
  float* t1 = sm + TILE_FLOATS;
  float* dwp = ws.dWp + chunk * C * D;
  for_acc<128>(tmem, 128, [&](int dk, int i0, const float* x) {   // dWp(i, dk), coalesced over dk
#pragma unroll
    for (int j = 0; j < 16; ++j) dwp[(i0 + j) * D + dk] = x[j];
  });
  acc_to_smem<false>(tmem, 0, t0);     // dqg / scale
  acc_to_smem<false>(tmem, 256, t1);   // dkg
  __syncthreads();
  float4 cs0 = make_float4(0.f, 0.f, 0.f, 0.f), cs1 = cs0;   // column sums per chunk
  // the for_tile walk (row i = warp + 8 it, columns d = 4 lane), four rows at
  // a time with their global loads before any store (see k_tc_bwd_intra1)
  const int d = (threadIdx.x & 31) * 4;
  const float4 l4a = ldg4(gc + (R - 1) * D + d), l4b = ldg4(gc + (2 * R - 1) * D + d);
#pragma unroll 1
  for (int it0 = 0; it0 < 16; it0 += 4) {
  float4 g4v[4], qvv[4], kvv[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = (threadIdx.x >> 5) + 8 * (it0 + u);
    g4v[u] = ldg4(gc + i * D + d);
    qvv[u] = ld4<T>(qc + i * rs + d);
    kvv[u] = ld4<T>(kc + i * rs + d);
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = (threadIdx.x >> 5) + 8 * (it0 + u);
    const bool hf = i >= R;   // the tile's second chunk
    const float4 x = lds4(t0 + i * TLD + d), y = lds4(t1 + i * TLD + d);
    const float4 g4 = g4v[u], l4 = hf ? l4b : l4a;
    const float4 eg = exp4(g4);
    const float4 qv = qvv[u], kv = kvv[u];
    const float4 dqg = make_float4(p.scale * x.x, p.scale * x.y, p.scale * x.z, p.scale * x.w);
    st4(pdq + i * D + d, san(dqg.x * eg.x, p.clip), san(dqg.y * eg.y, p.clip),
        san(dqg.z * eg.z, p.clip), san(dqg.w * eg.w, p.clip));
    const float4 pg = make_float4(dqg.x * (qv.x * eg.x), dqg.y * (qv.y * eg.y),
                                  dqg.z * (qv.z * eg.z), dqg.w * (qv.w * eg.w));
    const float4 f = exp4(make_float4(l4.x - g4.x, l4.y - g4.y, l4.z - g4.z, l4.w - g4.w));
    const float4 xs = make_float4(y.x * (kv.x * f.x), y.y * (kv.y * f.y), y.z * (kv.z * f.z),
                                  y.w * (kv.w * f.w));
    st4(pdk + i * D + d, y.x * f.x, y.y * f.y, y.z * f.z, y.w * f.w);
    st4(pdgc + i * D + d, pg.x - xs.x, pg.y - xs.y, pg.z - xs.z, pg.w - xs.w);
    if (hf) { cs1.x += xs.x; cs1.y += xs.y; cs1.z += xs.z; cs1.w += xs.w; }
    else { cs0.x += xs.x; cs0.y += xs.y; cs0.z += xs.z; cs0.w += xs.w; }
  }
  }
  float* daqkT = ws.dAqkT + chunk * C * C;
  for_acc<128>(tmem, 384, [&](int i, int c0, const float* v) {   // dAqk^T, coalesced per column
#pragma unroll
    for (int t = 0; t < 16; ++t)
      daqkT[(c0 + t) * C + i] = (c0 + t <= i && (c0 + t) / R == i / R) ? san(v[t], p.clip) : 0.f;
  });
  st4(&ts.colpart[threadIdx.x >> 5][d], cs0.x, cs0.y, cs0.z, cs0.w);
  st4(&ts.colpart1[threadIdx.x >> 5][d], cs1.x, cs1.y, cs1.z, cs1.w);
  // rowdot[d] = sum_v dh_next(d, v) h_pre(d, v) of each chunk
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll 1
    for (int hf = 0; hf < 2; ++hf) {
#pragma unroll 4
      for (int rr = 0; rr < D / 8; ++rr) {
        const int d = warp * (D / 8) + rr;
        const float4 a = *reinterpret_cast<const float4*>(dhn[hf] + d * D + lane * 4);
        const float4 h4 = *reinterpret_cast<const float4*>(hp[hf] + d * D + lane * 4);
        float v = a.x * h4.x + a.y * h4.y + a.z * h4.z + a.w * h4.w;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) (hf ? ts.rowdot1 : ts.rowdot)[d] = v;
      }
    }
  }
  __syncthreads();
  // gc_last row of each chunk: sum_i dkg kg + e^{gc_last} sum_v dh_next h_pre
  // (gdn2_bwd.py:185, 196-201)
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
#pragma unroll 1
    for (int hf = 0; hf < 2; ++hf) {
      float csum = 0.f;
      for (int r = 0; r < 8; ++r) csum += (hf ? ts.colpart1 : ts.colpart)[r][d];   // fixed order
      const int lr = hf * R + R - 1;
      pdgc[lr * D + d] += csum + __expf(gc[lr * D + d]) * (hf ? ts.rowdot1 : ts.rowdot)[d];
    }
  }
  teardown(tmem);
}

// ---------------------------------------------------------------------------
// dA = san(dWp kb^T + dv wv^T); tmp = san(dA A^T); dAkk = -(A^T tmp) * strict;
// dkb = A^T dWp; dwv = A^T dv -> pdk, pdb, pdgc (sanitised B3 totals), dw, dv,
// exactly as k_bwd_intra2.  dkb/dwv run first (inputs only); dA then goes from
// TMEM into resident shared-memory B tiles, and tmp is formed transposed so
// that its accumulator is already the TMEM A operand of dAkk^T.
// ---------------------------------------------------------------------------
template <typename T, bool GATES>
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
  const uint32_t tmem = setup(&ts);
  // one ring (its mbarrier phases carry across the K loops); base and operand
  // count change between loops
  Ring ring = ring_of(sm, &ts, 3);
  int g = 0;
  uint32_t ph = 0;
  const int warp = threadIdx.x >> 5;
  float* t0 = sm;
  float* t1 = sm + TILE_FLOATS;
  // ---- dkb = A^T dWp (TMEM 0), dwv = A^T dv (TMEM 128): (j, d) = sum_i A(i, j) X(i, d)
  {
    const Src srcs[3] = {direct(at, C), trans(dwp, D), trans(dvn, D)};   // (j,i) (d,i) (d,i)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);
      mma3(tmem + 128, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  acc_to_smem<false>(tmem, 0, t0);     // dkb (j, d)
  acc_to_smem<false>(tmem, 128, t1);   // dwv (j, d)
  __syncthreads();
  float *pdk = ws.pdk + chunk * C * D, *pdb = ws.pdb + chunk * C * D,
        *pdgc = ws.pdgc + chunk * C * D;
  // the for_tile walk (row j = warp + 8 it, columns d = 4 lane), two rows at
  // a time with all their global loads issued before any store (the stores
  // may alias the loads for the compiler, which would otherwise serialise
  // the latencies); dwv -> dw, dv in the same pass
  {
    const int d = (threadIdx.x & 31) * 4;
#pragma unroll 1
    for (int it0 = 0; it0 < 16; it0 += 2) {
      float4 gx[2], kx[2], bx[2], pkx[2], pgx[2], vx[2], wx[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = (threadIdx.x >> 5) + 8 * (it0 + u);
        gx[u] = ldg4(gc + j * D + d);
        kx[u] = ld4<T>(kc + j * rs + d);
        bx[u] = ld4_gate<T>(bc + j * rs + d, GATES, kGateB);
        pkx[u] = ldg4(pdk + j * D + d);
        pgx[u] = ldg4(pdgc + j * D + d);
        vx[u] = ld4<T>(vc + j * rs + d);
        wx[u] = ld4_gate<T>(wc + j * rs + d, GATES, kGateW);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = (threadIdx.x >> 5) + 8 * (it0 + u);
        const float4 x = lds4(t0 + j * TLD + d);
        const float4 eg = exp4(gx[u]);
        const float4 kv = kx[u], bv = bx[u], pk = pkx[u], pg = pgx[u];
        st4(pdk + j * D + d, san(pk.x + x.x * eg.x * bv.x, p.clip), san(pk.y + x.y * eg.y * bv.y, p.clip),
            san(pk.z + x.z * eg.z * bv.z, p.clip), san(pk.w + x.w * eg.w * bv.w, p.clip));
        st4(pdb + j * D + d, san(x.x * eg.x * kv.x, p.clip), san(x.y * eg.y * kv.y, p.clip),
            san(x.z * eg.z * kv.z, p.clip), san(x.w * eg.w * kv.w, p.clip));
        st4(pdgc + j * D + d, san(pg.x + x.x * (bv.x * kv.x * eg.x), p.clip),
            san(pg.y + x.y * (bv.y * kv.y * eg.y), p.clip), san(pg.z + x.z * (bv.z * kv.z * eg.z), p.clip),
            san(pg.w + x.w * (bv.w * kv.w * eg.w), p.clip));
        const float4 y = lds4(t1 + j * TLD + d);
        const float4 vv = vx[u], wv = wx[u];
        const float4 dw = make_float4(y.x * vv.x, y.y * vv.y, y.z * vv.z, y.w * vv.w);
        const float4 dvv = make_float4(y.x * wv.x, y.y * wv.y, y.z * wv.z, y.w * wv.w);
        const float4 dwo = san4(san4(dw, p.clip), kFinalClipTc);
        st4<T>(dw_out + off + j * rs + d, GATES ? mul4(dwo, sig_grad4(wv)) : dwo);
        st4<T>(dv_out + off + j * rs + d, san4(san4(dvv, p.clip), kFinalClipTc));
      }
    }
  }
  fence_before_sync();
  __syncthreads();   // staging tiles and TMEM 0..255 free again
  fence_after_sync();

  // ---- dA = dWp kb^T + dv wv^T  (TMEM 0, contraction over d)
  {
    ring.base = sm;
    ring.nop = 2;
    // the computed operands (kb, then wv) are loaded a slice ahead in
    // registers, in the thread -> (row, column) map of store_direct
    auto rc = [&](int it, int& r, int& cc) {
      const int e = threadIdx.x + it * kThreads, lane = e & 31, w = e >> 5;
      r = (w & 15) * 8 + (lane & 7);
      cc = ((w >> 4) * 4 + (lane >> 3)) * 4;
    };
    Frag fx, fy, fz;
    auto ld_kb = [&](int sl) {
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        int j, cc;
        rc(it, j, cc);
        const int d = sl * KS + cc;
        fx.v[it] = ld4<T>(kc + j * rs + d);
        fy.v[it] = ld4_gate<T>(bc + j * rs + d, GATES, kGateB);
        fz.v[it] = ldg4(gc + j * D + d);
      }
    };
    auto ld_wv = [&](int sl) {
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        int j, cc;
        rc(it, j, cc);
        const int d = sl * KS + cc;
        fx.v[it] = ld4_gate<T>(wc + j * rs + d, GATES, kGateW);
        fy.v[it] = ld4<T>(vc + j * rs + d);
      }
    };
    ld_kb(0);
    {
      const Src srcs[1] = {direct(dwp, D)};   // (i,d)
      kloop_pf(ring, g, ws.status, srcs,
               [&](int buf, int s) {
                 Frag kb;   // (j,d) = b k e^gc
#pragma unroll
                 for (int it = 0; it < 4; ++it) {
                   const float4 kv = fx.v[it], bv = fy.v[it], g4 = fz.v[it];
                   kb.v[it] = make_float4(bv.x * kv.x * __expf(g4.x), bv.y * kv.y * __expf(g4.y),
                                          bv.z * kv.z * __expf(g4.z), bv.w * kv.w * __expf(g4.w));
                 }
                 if (s + 1 < D / KS) ld_kb(s + 1);
                 else ld_wv(0);
                 store_direct(ring.hi(buf, 1), ring.lo(buf, 1), kb);
               },
               [&](int buf, int s) { mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0); });
    }
    {
      const Src srcs[1] = {direct(dvn, D)};   // (i,d)
      kloop_pf(ring, g, ws.status, srcs,
               [&](int buf, int s) {
                 Frag wv;   // (j,d) = w v
#pragma unroll
                 for (int it = 0; it < 4; ++it) {
                   const float4 a = fx.v[it], b4 = fy.v[it];
                   wv.v[it] = make_float4(a.x * b4.x, a.y * b4.y, a.z * b4.z, a.w * b4.w);
                 }
                 if (s + 1 < D / KS) ld_wv(s + 1);
                 store_direct(ring.hi(buf, 1), ring.lo(buf, 1), wv);
               },
               [&](int buf, int s) { mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, 1); });
    }
  }
  drain(&ts.done, ph, ws.status);
  // dA = san(acc) straight into four resident K-slices (rows i, K = k) in
  // shared memory: the B operand of the next product.
  float* dAt = sm;                          // 4 x (hi, lo) x 128 x 32
  for_acc<128>(tmem, 0, [&](int row, int c, const float* v) {
    float* hi = dAt + (c / KS) * 2 * SLICE_FLOATS;
#pragma unroll
    for (int j = 0; j < 16; j += 4)
      st_split4(hi, hi + SLICE_FLOATS, row, c % KS + j, KS,
                make_float4(san(v[j], p.clip), san(v[j + 1], p.clip), san(v[j + 2], p.clip),
                            san(v[j + 3], p.clip)));
  });
  // ---- tmp^T = (dA A^T)^T: (j, i) = sum_k A(j, k) dA(i, k)  (TMEM 128)
  {
    ring.base = sm + 4 * 2 * SLICE_FLOATS;
    ring.nop = 1;
    const Src srcs[1] = {trans(at, C)};   // (j,k) = A(j,k)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      float* hi = dAt + s * 2 * SLICE_FLOATS;
      mma3(tmem + 128, ring.op(buf, 0), kmajor(hi, hi + SLICE_FLOATS, KS), 128, KS / 8, s > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  // tmp^T = san(acc) split into hi (TMEM 256..383) and lo (384..511): the A
  // operand (rows j, K = k) of the next product.
  for_acc<128>(tmem, 128, [&](int row, int c, const float* v) {
    float hv[16], lv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) split(san(v[j], p.clip), hv[j], lv[j]);
    tmem_st16(lane_quarter_addr(tmem, 256 + c), hv);
    tmem_st16(lane_quarter_addr(tmem, 384 + c), lv);
  });
  tmem_st_wait();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  // ---- dAkk^T: (j, i) = -sum_k tmp(k, j) A(k, i)  (TMEM 0)
  {
    ring.base = sm;
    ring.nop = 1;
    const Src srcs[1] = {direct(at, C)};   // (i,k) = A(k,i)
    kloop_pf(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3_ta(tmem, tmem + 256 + s * KS, tmem + 384 + s * KS, ring.op(buf, 0), 128, KS / 8, s > 0);
    });
  }
  drain(&ts.done, ph, ws.status);
  (void)warp;
  float* dAkkT = ws.dAkkT + chunk * C * C;
  acc_to_smem<false>(tmem, 0, t0);    // t0[j][i] = acc(j, i)
  __syncthreads();
  // strictly lower and, for a tile of two chunks, block-diagonal (the 4
  // columns i of one store lie in one chunk)
  const int cm = p.sub == 2 ? C / 2 : 0;   // chunk bit of a row index
  for_tile([&](int j, int i) {
    const float4 x = lds4(t0 + j * TLD + i);
    const bool same = ((j ^ i) & cm) == 0;
    st4(dAkkT + j * C + i, same && j < i ? san(-x.x, p.clip) : 0.f,
        same && j < i + 1 ? san(-x.y, p.clip) : 0.f, same && j < i + 2 ? san(-x.z, p.clip) : 0.f,
        same && j < i + 3 ? san(-x.w, p.clip) : 0.f);
  });
  teardown(tmem);
}

// Statistics of the order-free B4 guard from one staged slice: fm holds
// dM(i = d0 + comp, j = j0 + jj) (left passes: row and column L1 of dAqk in
// pass 0, of dAkk in pass 1); fx the raw k (pass 0), q (pass 2) or k (pass 3,
// fb its gate) at rows j0 + jj, columns d0 + comp: column maxima.  gst rows
// as k_tc_bwd_intra3's enum.
__device__ __forceinline__ void gather_stats(int pass, int j0, int d0, const Frag& fm,
                                             const Frag& fx, const Frag& fb, float scale,
                                             float* gst) {
  // lane bits: 0-2 pick the row block (d0), 3-4 the column block (j0); the
  // sums over lanes sharing a row (or column) block are formed with shuffles
  // first, so one lane per group does the shared-memory atomic
  const int lane = threadIdx.x & 31;
  auto amax = [](float* a, float v) {   // v >= 0 (or NaN, which the guard test rejects)
    atomicMax(reinterpret_cast<int*>(a), __float_as_int(v));
  };
  if (pass < 2) {
    float* rowl = gst + (pass == 0 ? 0 : 1) * 128;
    float* coll = gst + (pass == 0 ? 2 : 3) * 128;
    float r[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = fm.v[j];
      const float a = fabsf(v.x), b2 = fabsf(v.y), c2 = fabsf(v.z), d2 = fabsf(v.w);
      r[0] += a; r[1] += b2; r[2] += c2; r[3] += d2;
      float cs = a + b2 + c2 + d2;   // column j0 + j: the 8 lanes of this column block
      cs += __shfl_xor_sync(0xffffffffu, cs, 1);
      cs += __shfl_xor_sync(0xffffffffu, cs, 2);
      cs += __shfl_xor_sync(0xffffffffu, cs, 4);
      if ((lane & 7) == 0) atomicAdd(coll + j0 + j, cs);
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {   // row d0 + t: the 4 lanes of this row block
      r[t] += __shfl_xor_sync(0xffffffffu, r[t], 8);
      r[t] += __shfl_xor_sync(0xffffffffu, r[t], 16);
      if ((lane & 24) == 0) atomicAdd(rowl + d0 + t, r[t]);
    }
  }
  if (pass == 1) return;
  float m[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float4 v = fx.v[j];
    if (pass == 2) v = make_float4(scale * v.x, scale * v.y, scale * v.z, scale * v.w);
    if (pass == 3) v = make_float4(fb.v[j].x * v.x, fb.v[j].y * v.y, fb.v[j].z * v.z, fb.v[j].w * v.w);
    m[0] = fmaxf(m[0], fabsf(v.x)); m[1] = fmaxf(m[1], fabsf(v.y));
    m[2] = fmaxf(m[2], fabsf(v.z)); m[3] = fmaxf(m[3], fabsf(v.w));
  }
  float* mx = gst + (pass == 0 ? 4 : (pass == 2 ? 5 : 6)) * 128;
#pragma unroll
  for (int t = 0; t < 4; ++t) {   // column d0 + t: the 4 lanes of this row block
    // a NaN must survive the reduction (fmaxf would drop it): compare instead
    float o = __shfl_xor_sync(0xffffffffu, m[t], 8);
    m[t] = (o > m[t] || o != o) ? o : m[t];
    o = __shfl_xor_sync(0xffffffffu, m[t], 16);
    m[t] = (o > m[t] || o != o) ? o : m[t];
    if ((lane & 24) == 0) amax(mx + d0 + t, m[t]);
  }
}

// ---------------------------------------------------------------------------
// Backward of the chunk scores (B4, gdn2_bwd.py:248-339), the in-chunk
// reverse cumsum (B5, gdn2_bwd.py:32-41) and the final assembly with the
// +-1e4 sanitiser (gdn2_pipeline.py:117-135); same contract as k_bwd_intra3.
// The four pair sums run as three passes of products 128 x 128 x JW (the two
// dR sums accumulate in one), one per JW-wide block with its own reference
// row r (JW = 64, or 32 when a 64-row spread of gc exceeds 80):
//   dL_i = sum_J e^{gc_i - gc_rJ} sum_{j in J} dM_ij (k_j e^{gc_rJ - gc_j})
//   dR_j = sum_I e^{gc_rI - gc_j} sum_{i in I} dM_ij (L_i e^{gc_i - gc_rI})
// (every factor bounded for g <= 0 and a 32-row gc spread <= 80, otherwise
// the exact elementwise form with the +-20 clip runs).  The decay derivative
// is dgc_i += L_i dL_i, dgc_j -= k_j dR_j.  The dk and dgc partials stay in
// registers (thread = TMEM row) across the passes.
// ---------------------------------------------------------------------------
template <typename T, bool GATES, bool CRUDE>
__global__ void __launch_bounds__(kThreads, 1)
k_tc_bwd_intra3(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ b,
                const T* __restrict__ g, T* __restrict__ dq_out, T* __restrict__ dk_out,
                T* __restrict__ db_out, T* __restrict__ dg_out, Problem p, Workspace ws) {
  extern __shared__ __align__(128) float sm[];
  __shared__ __align__(16) TcSmemB ts;
  // statistics of the order-free guard (BC < JW): row / column L1 of dAqk,
  // dAkk; column maxima of |k|, |scale q|, |b k|
  __shared__ float gstat[7][128];
  enum { kRowQ = 0, kRowK, kColQ, kColK, kKmax, kLqmax, kLkmax };
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const int h = (int)(bh % p.H), bb = (int)(bh / p.H);
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const T *qc = q + off, *kc = k + off, *bc = b + off, *gcp = g + off;
  const float* gcg = ws.gc + chunk * C * D;
  const float* pdq = ws.pdq + chunk * C * D;
  const float* pdk = ws.pdk + chunk * C * D;
  const float* pdb = ws.pdb + chunk * C * D;
  const float* pdgc = ws.pdgc + chunk * C * D;
  const float* dAqkT = ws.dAqkT + chunk * C * C;
  const float* dAkkT = ws.dAkkT + chunk * C * C;
  float* red = &ts.colpart[0][0];
  float* sdg = sm;   // [C][D] after the products (ring area)
  GDN2_TDECL;
  GDN2_TMARK(0);

  const uint32_t tmem = setup(&ts);
  // gc tile resident in shared memory after the ring: read by every operand
  // staging and epilogue below
  // (row stride GLD: per-row reads of consecutive rows hit distinct banks)
  constexpr int GLD = D + 4;
  float* sgc = sm + 2 * 2 * 2 * SLICE_FLOATS;
#pragma unroll 4
  for (int e = threadIdx.x; e < C * D / 4; e += kThreads)
    *reinterpret_cast<float4*>(sgc + (e >> 5) * GLD + (e & 31) * 4) =
        *reinterpret_cast<const float4*>(gcg + 4 * e);
  __syncthreads();
  const float* gc = sgc;
  float gpos = -1.f;
#pragma unroll 8
  for (int it = 0; it < C * D / 4 / kThreads; ++it) {
    const int e = threadIdx.x + it * kThreads;
    const float4 g4 = ld4_gate<T>(gcp + (e >> 5) * rs + (e & 31) * 4, GATES, kGateG);
    gpos = fmaxf(gpos, fmaxf(fmaxf(g4.x, g4.y), fmaxf(g4.z, g4.w)));
  }
  const float gmax = block_max(gpos, red);
  float spread = 0.f, spread64 = 0.f;
  for (int e = threadIdx.x; e < 4 * D; e += kThreads) {
    const int J = e / D, d = e % D;
    spread = fmaxf(spread, fabsf(gc[(32 * J) * GLD + d] - gc[(32 * J + 31) * GLD + d]));
    if (J < 2) spread64 = fmaxf(spread64, fabsf(gc[(64 * J) * GLD + d] - gc[(64 * J + 63) * GLD + d]));
  }
  const bool exact = gmax > 0.f || block_max(spread, red) > 80.f || spread != spread;
  const int JW = (block_max(spread64, red) <= 80.f && p.bc % 64 == 0) ? 64 : 32;
  // The block guard below needs the JW-column blocks to nest inside the
  // reference's BC-row sub-blocks.  For BC < JW the fast path is guarded
  // instead by sums of absolute terms, which bound every prefix of the
  // reference's pair sequence whatever its order (with g <= 0 every decay
  // factor e^{gc_i - gc_j}, j <= i, is at most 1):
  //   |dq|  <= |scale| rowL1(dAqk)_i kmax_d      |dbk| <= rowL1(dAkk)_i kmax_d
  //   |dk|  <= colL1(dAqk)_j lqmax_d + colL1(dAkk)_j lkmax_d
  //   |dgc| <= (lqmax rowL1(dAqk) + lkmax rowL1(dAkk)) kmax + kmax |dk bound|
  // with kmax_d = max_i |k_id|, lqmax_d = max_i |scale q_id|,
  // lkmax_d = max_i |b_i k_id| over the tile.  The staging gathers them.
  // (JW >= 32 always, and 64 only for BC a multiple of 64: BC < JW iff
  // BC < 32, which the launch resolves into the CRUDE instance)
  constexpr bool crude = CRUDE;
  float* gst = &gstat[0][0];
  if (crude) {
    for (int e = threadIdx.x; e < 7 * 128; e += kThreads) gst[e] = 0.f;
    __syncthreads();
  }
  bool run_exact = exact;
  const int R = C / p.sub;   // rows of one reference chunk
  const int cm = p.sub == 2 ? C / 2 : 0;   // rows x, r share a chunk iff ((x ^ r) & cm) == 0
  GDN2_TMARK(1);

  if (!exact) {
    Ring ring = ring_of(sm, &ts, 2);
    int gs = 0;
    uint32_t ph = 0;
    const int warp = threadIdx.x >> 5;
    const int x = 32 * (warp & 3) + (threadIdx.x & 31);   // this thread's TMEM row
    const int cb = (warp >> 2) * 64;                       // its first column
    float dkr[64], dgr[64];
#pragma unroll
    for (int t = 0; t < 64; ++t) dkr[t] = dgr[t] = 0.f;
    // Clip guard.  The reference sanitises its B4 accumulators after every
    // BC-row sub-block pair (_clip_acc); summing all pairs at once gives the
    // same value while no prefix of that sequence reaches CLIP, which holds
    // when the sum of the absolute block partials stays below CLIP (the JW
    // blocks nest in the BC blocks, so every reference prefix is a sum of
    // them).  Per thread: the largest such sum of each accumulator.
    // Three passes: dL of the q scores, dL of the k scores, and the two dR
    // sums in one accumulation (slices 0-3 from dAqk with scale q, 4-7 from
    // dAkk with b k): only dRq + dRk is ever used, and the reference adds
    // exactly that sum to dk per pair (gdn2_bwd.py:326), so the guard on the
    // combined partials bounds its prefixes too.
    float gq_dq = 0.f, gq_dbk = 0.f, gq_dk = 0.f;
    float gg0 = 0.f, gg1 = 0.f, gg2 = 0.f;   // dgc terms of each pass
#pragma unroll 1
    for (int pass = 0; pass < 3; ++pass) {
      if (pass > 0) GDN2_TMARK(1 + 2 * pass);
      const bool left = pass < 2;                          // dL (row i) or dR (row j)
      // Every global load of a slice is issued first (one memory latency per
      // slice), and the MMAs of slice sl are issued during slice sl+1 while
      // its loads are in flight: the issuing thread blocks for about as long
      // as the tensor core takes, and that wait overlaps the load latency
      // instead of delaying its warp's staging.  (Loading slice sl+1 during
      // slice sl needs registers the dk / dgc accumulators hold.)
      const int e = threadIdx.x;
      const int rb = (e & 7) + ((e >> 5) & 3) * 8, kb = ((e >> 3) & 3) + (e >> 7) * 4;
      const int d0 = rb * 4;   // this thread's 4 x 4 block of the second operand
      // kpart: this slice belongs to the k scores (pass 1, second half of 2)
      auto load_slice = [&](int k0, bool kpart, Frag& fm, Frag& fx) {
        const float* MT = kpart ? dAkkT : dAqkT;
        if (left) {
          load_trans(fm, MT, C, k0);                      // (i, jj) = dM(i, k0+jj)
#pragma unroll
          for (int j = 0; j < 4; ++j) fx.v[j] = ld4<T>(kc + (k0 + kb * 4 + j) * rs + d0);
        } else {
          load_direct(fm, MT, C, k0);                     // (j, ii) = dM(k0+ii, j)
          const T* src = kpart ? kc : qc;
#pragma unroll
          for (int j = 0; j < 4; ++j) fx.v[j] = ld4<T>(src + (k0 + kb * 4 + j) * rs + d0);
        }
      };
      Frag fm, fx;
      int pend_buf = -1, pend_J = 0;
      bool pend_acc = false;
      const int nsl = left ? 4 : 8;
#pragma unroll 1
      for (int sl = 0; sl < nsl; ++sl, ++gs) {
        const int sl4 = sl & 3;
        const bool kpart = pass == 1 || sl >= 4;
        const int J = sl4 * 32 / JW, r = JW * J, k0 = 32 * sl4;   // K slice k0 of block J
        const int buf = gs & 1;
        GDN2_TSUB(0);
        ring_acquire(ring, buf, gs >> 1, ws.status);
        GDN2_TSUB(1);
        load_slice(k0, kpart, fm, fx);
        Frag fb;   // the gate of the right pass's k part
        if (!left && kpart) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            fb.v[j] = ld4_gate<T>(bc + (k0 + kb * 4 + j) * rs + d0, GATES, kGateB);
        }
        if (crude) gather_stats(left ? pass : (kpart ? 3 : 2), k0 + kb * 4, d0, fm, fx, fb, p.scale, gst);
        if (threadIdx.x == 0 && pend_buf >= 0) {
          mma3(tmem + 128 * pend_J, ring.op(pend_buf, 0), ring.op(pend_buf, 1), 128, KS / 8, pend_acc);
          commit(&ring.bars[pend_buf]);
        }
        const float4 gr = ldg4(gc + r * GLD + d0);
        if (left) {
          store_trans(ring.hi(buf, 0), ring.lo(buf, 0), fm);
#pragma unroll
          for (int j = 0; j < 4; ++j) {   // (d, jj) = R = k_j e^{gc_r - gc_j}
            const float4 gj = ldg4(gc + (k0 + kb * 4 + j) * GLD + d0);
            const float4 kv = fx.v[j];
            fx.v[j] = make_float4(kv.x * __expf(gr.x - gj.x), kv.y * __expf(gr.y - gj.y),
                                  kv.z * __expf(gr.z - gj.z), kv.w * __expf(gr.w - gj.w));
          }
        } else {
          store_direct(ring.hi(buf, 0), ring.lo(buf, 0), fm);
#pragma unroll
          for (int j = 0; j < 4; ++j) {   // (d, ii) = L = l_i e^{gc_i - gc_r}
            const float4 gi = ldg4(gc + (k0 + kb * 4 + j) * GLD + d0);
            float4 lv = fx.v[j];
            if (!kpart) {
              lv = scl(lv, p.scale);
            } else {
              const float4 bv = fb.v[j];
              lv = make_float4(bv.x * lv.x, bv.y * lv.y, bv.z * lv.z, bv.w * lv.w);
            }
            fx.v[j] = make_float4(lv.x * __expf(gi.x - gr.x), lv.y * __expf(gi.y - gr.y),
                                  lv.z * __expf(gi.z - gr.z), lv.w * __expf(gi.w - gr.w));
          }
        }
        store_trans(ring.hi(buf, 1), ring.lo(buf, 1), fx);
        GDN2_TSUB(2);
        slice_publish();
        GDN2_TSUB(3);
        pend_buf = buf;
        pend_J = J;
        pend_acc = k0 > r || sl >= 4;   // the k part adds onto the q part's blocks
      }
      if (threadIdx.x == 0) {
        mma3(tmem + 128 * pend_J, ring.op(pend_buf, 0), ring.op(pend_buf, 1), 128, KS / 8, pend_acc);
        commit(&ring.bars[pend_buf]);
      }
      drain(&ts.done, ph, ws.status);
      GDN2_TMARK(2 + 2 * pass);
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        const int c0 = cb + qd * 16;
        float val[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) val[t] = 0.f;
        float gx[16], sab[16];
#pragma unroll
        for (int t = 0; t < 16; t += 4) {
          const float4 v4 = ldg4(gc + x * GLD + c0 + t);
          gx[t] = v4.x; gx[t + 1] = v4.y; gx[t + 2] = v4.z; gx[t + 3] = v4.w;
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) sab[t] = 0.f;
#pragma unroll
        for (int J = 0; J < 4; ++J) {
          if (J >= C / JW) break;
          float a[16];
          tmem_ld16(lane_quarter_addr(tmem, 128 * J + c0), a);
          const int r = JW * J;
          // same chunk only (paired tiles): across chunks the gc are of
          // different chunks and the factor below is meaningless
          const bool use = (left ? (x >= r) : (x < r + JW)) && ((x ^ r) & cm) == 0;
          if (use) {
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              const float gr = gc[r * GLD + c0 + t];
              const float part = a[t] * __expf(left ? gx[t] - gr : gr - gx[t]);
              val[t] += part;
              sab[t] += fabsf(part);
            }
          }
        }
        float4 xa[4], xb[4];
        if (pass == 0) {
#pragma unroll
          for (int t = 0; t < 16; t += 4) xa[t / 4] = ld4<T>(qc + x * rs + c0 + t);
          float4 pqv[4];   // loads before the aliasing gradient stores
#pragma unroll
          for (int t = 0; t < 4; ++t) pqv[t] = ldg4(pdq + x * D + c0 + 4 * t);
#pragma unroll
          for (int t = 0; t < 16; t += 4) {
            const float4 pq = pqv[t / 4];
            const float* qv = &xa[t / 4].x;
            const float* pv = &pq.x;
            float o[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              o[u] = san(pv[u] + san(p.scale * val[t + u], p.clip), kFinalClipTc);
              dgr[qd * 16 + t + u] += p.scale * qv[u] * val[t + u];
              gq_dq = fmaxf(gq_dq, fabsf(p.scale) * sab[t + u]);
              gg0 = fmaxf(gg0, fabsf(p.scale * qv[u]) * sab[t + u]);
            }
            st4<T>(dq_out + off + x * rs + c0 + t, make_float4(o[0], o[1], o[2], o[3]));
          }
        } else if (pass == 1) {
#pragma unroll
          for (int t = 0; t < 16; t += 4) {
            xa[t / 4] = ld4<T>(kc + x * rs + c0 + t);
            xb[t / 4] = ld4_gate<T>(bc + x * rs + c0 + t, GATES, kGateB);
          }
          float4 pbv[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) pbv[t] = ldg4(pdb + x * D + c0 + 4 * t);
#pragma unroll
          for (int t = 0; t < 16; t += 4) {
            const float4 pb = pbv[t / 4];
            const float* kv = &xa[t / 4].x;
            const float* bv = &xb[t / 4].x;
            const float* pv = &pb.x;
            float o[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float dbk = val[t + u];
              o[u] = san(pv[u] + san(dbk * kv[u], p.clip), kFinalClipTc);
              if (GATES) o[u] *= bv[u] * (1.f - bv[u]);
              dkr[qd * 16 + t + u] = dbk * bv[u];
              dgr[qd * 16 + t + u] += bv[u] * kv[u] * dbk;
              gq_dbk = fmaxf(gq_dbk, sab[t + u]);
              gg1 = fmaxf(gg1, fabsf(bv[u] * kv[u]) * sab[t + u]);
            }
            st4<T>(db_out + off + x * rs + c0 + t, make_float4(o[0], o[1], o[2], o[3]));
          }
        } else {
#pragma unroll
          for (int t = 0; t < 16; t += 4) xa[t / 4] = ld4<T>(kc + x * rs + c0 + t);
#pragma unroll
          for (int t = 0; t < 16; t += 4) {
            const float* kv = &xa[t / 4].x;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              dkr[qd * 16 + t + u] += val[t + u];
              dgr[qd * 16 + t + u] -= kv[u] * val[t + u];
              gq_dk = fmaxf(gq_dk, sab[t + u]);
              gg2 = fmaxf(gg2, fabsf(kv[u]) * sab[t + u]);
            }
          }
          {
            float4 pkv[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) pkv[t] = ldg4(pdk + x * D + c0 + 4 * t);
#pragma unroll
            for (int t = 0; t < 16; t += 4) {
              const float4 pk = pkv[t / 4];
              const float* pv = &pk.x;
              float o[4];
#pragma unroll
              for (int u = 0; u < 4; ++u)
                o[u] = san(pv[u] + san(dkr[qd * 16 + t + u], p.clip), kFinalClipTc);
              st4<T>(dk_out + off + x * rs + c0 + t, make_float4(o[0], o[1], o[2], o[3]));
            }
          }
        }
      }
    }
    const float lim = p.clip * (1.f - 1e-5f);   // NaN fails every test below
    GDN2_TMARK(9);
    bool bad;
    if (!crude) {
      bad = !(gq_dq < lim && gq_dbk < lim && gq_dk < lim && gg0 + gg1 + gg2 < lim);
    } else {
      __syncthreads();   // the statistics of every thread are in
      const float rq = gstat[kRowQ][x], rk = gstat[kRowK][x];
      const float cq = gstat[kColQ][x], ck = gstat[kColK][x];
      bad = false;
#pragma unroll 4
      for (int d = cb; d < cb + 64; ++d) {
        const float km = gstat[kKmax][d], lq = gstat[kLqmax][d], lk = gstat[kLkmax][d];
        const float bdk = cq * lq + ck * lk;
        const float bdg = (lq * rq + lk * rk) * km + km * bdk;
        bad |= !(fabsf(p.scale) * rq * km < lim && rk * km < lim && bdk < lim && bdg < lim);
      }
    }
    run_exact = __syncthreads_or(bad);
    // dgc total into shared memory (ring is idle after the last drain)
    if (!run_exact) {
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) {
      const int c0 = cb + qd * 16;
#pragma unroll
      for (int t = 0; t < 16; t += 4) {
        const float4 pg = ldg4(pdgc + x * D + c0 + t);
        st4(sdg + x * D + c0 + t, pg.x + san(dgr[qd * 16 + t], p.clip),
            pg.y + san(dgr[qd * 16 + t + 1], p.clip), pg.z + san(dgr[qd * 16 + t + 2], p.clip),
            pg.w + san(dgr[qd * 16 + t + 3], p.clip));
      }
    }
    }
    if (run_exact && threadIdx.x == 0) atomicOr(ws.status + 4, 1);
  }
  if (run_exact) {
    // the reference's pair order: positive gates, wide gate spreads, BC < 32,
    // or a chunk whose guard failed (its fast-path outputs are overwritten)
    b4_exact_chunk<T>(C, D, p.bc, qc, kc, bc, rs, gc, GLD, dAqkT, dAkkT, pdq, pdk, pdb, pdgc, dq_out,
                      dk_out, db_out, off, sdg, p.scale, p.clip, GATES, R);
  }
  GDN2_TMARK(10);
  __syncthreads();
  column_revcumsum<C, D>(sdg, red, p.sub == 2);
  for_tile([&](int i, int d) {
    const float4 v4 = ldg4(sdg + i * D + d);
    float4 dgo = san4(san4(v4, p.clip), kFinalClipTc);
    if (GATES) {   // d(-softplus(g'))/dg' = -sigmoid(g')
      const float4 gr = ld4<T>(gcp + i * rs + d);
      dgo = make_float4(-dgo.x * gate_sig(gr.x), -dgo.y * gate_sig(gr.y), -dgo.z * gate_sig(gr.z),
                        -dgo.w * gate_sig(gr.w));
    }
    st4<T>(dg_out + off + i * rs + d, dgo);
  });
  teardown(tmem);
  GDN2_TMARK(11);
  GDN2_TPRINT("bwd_intra3", 12);
  GDN2_TSUBPRINT("bwd_intra3");
}

template <typename T>
cudaError_t launch_tc_bwd_intra3(const T* q, const T* k, const T* b, const T* g, T* dq, T* dk,
                                 T* db, T* dg, const Problem& p, const Workspace& ws,
                                 cudaStream_t s, const LaunchHook& hook) {
  // ring (also the C x D dgc tile at the end), then the gc tile
  constexpr size_t smem = 2 * 2 * (size_t)SLICE_BYTES + (size_t)C * (D + 4) * sizeof(float);
  auto kern = p.bc < 32 ? (p.gates ? k_tc_bwd_intra3<T, true, true> : k_tc_bwd_intra3<T, false, true>)
                        : (p.gates ? k_tc_bwd_intra3<T, true, false> : k_tc_bwd_intra3<T, false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  hook.begin(kStageBwdIntra3, s);
  kern<<<(unsigned)p.B * p.H * p.nc, kThreads, smem, s>>>(q, k, b, g, dq, dk, db, dg, p, ws);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageBwdIntra3, s);
  return cudaSuccess;
}

template cudaError_t launch_tc_bwd_intra3<float>(const float*, const float*, const float*,
                                                 const float*, float*, float*, float*, float*,
                                                 const Problem&, const Workspace&, cudaStream_t,
                                                 const LaunchHook&);
template cudaError_t launch_tc_bwd_intra3<__nv_bfloat16>(
    const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
    __nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16*, const Problem&,
    const Workspace&, cudaStream_t, const LaunchHook&);

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
  auto kern2 = p.gates ? k_tc_bwd_intra2<T, true> : k_tc_bwd_intra2<T, false>;
  if ((e = cudaFuncSetAttribute(kern2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
      cudaSuccess)
    return e;
  if ((e = cudaFuncSetAttribute(k_tc_bwd_intra1_pair<T>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
    return e;
  hook.begin(kStageBwdIntra1, s);
  if (p.sub == 2) k_tc_bwd_intra1_pair<T><<<nchunks, kThreads, smem, s>>>(q, k, dout, dh_final, p, ws);
  else k_tc_bwd_intra1<T><<<nchunks, kThreads, smem, s>>>(q, k, dout, dh_final, p, ws);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageBwdIntra1, s);
  hook.begin(kStageBwdIntra2, s);
  kern2<<<nchunks, kThreads, smem, s>>>(k, v, w, b, dv_out, dw_out, p, ws);
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
