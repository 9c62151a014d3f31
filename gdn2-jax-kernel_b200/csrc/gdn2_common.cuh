// Shared device helpers for the GDN-2 sm_100a kernels.
//
// Layout conventions used by every kernel in this library:
//   * user tensors q,k,v,w,b,g,do and the gradients are (B, T, H, D) row-major;
//     a chunk tile for (b, h, c) is BT rows of D contiguous elements with a row
//     stride of H*D elements — read in place, never transposed in HBM;
//   * h0 / h_final / dh_final / dh0 are (B, H, D, D) float32 (row = key dim);
//   * per-chunk intermediates live in a workspace laid out [B][H][nc][tile].
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace gdn2 {

constexpr int kThreads = 256;   // every CTA of this library runs 8 warps

// nan -> 0, +-inf -> +-clip, clip to [-clip, clip]: the stage sanitiser of the
// reference (gdn2_fwd.py:42-44).
__device__ __forceinline__ float san(float x, float clip) {
  if (x != x) return 0.f;
  return fminf(fmaxf(x, -clip), clip);
}

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Load 4 consecutive elements as float4 (16-byte aligned for float, 8 for bf16).
template <typename T> __device__ __forceinline__ float4 ld4(const T* p);
template <> __device__ __forceinline__ float4 ld4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <> __device__ __forceinline__ float4 ld4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
template <typename T> __device__ __forceinline__ void st4(T* p, float4 v);
template <> __device__ __forceinline__ void st4<float>(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
}
template <> __device__ __forceinline__ void st4<__nv_bfloat16>(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// Copy a rows x cols tile (cols % 4 == 0) from global (row stride lds elements)
// into shared memory (row stride ldd floats), converting to float.
template <typename T>
__device__ __forceinline__ void load_tile(float* dst, int ldd, const T* src, long lds,
                                          int rows, int cols) {
  const int c4 = cols >> 2;
  for (int e = threadIdx.x; e < rows * c4; e += kThreads) {
    int r = e / c4, c = (e - r * c4) << 2;
    float4 v = ld4<T>(src + r * lds + c);
    *reinterpret_cast<float4*>(dst + r * ldd + c) = v;
  }
}

// Same, but stores the transpose: dst[c*ldd + r] = src[r*lds + c].
template <typename T>
__device__ __forceinline__ void load_tile_T(float* dst, int ldd, const T* src, long lds,
                                            int rows, int cols) {
  const int c4 = cols >> 2;
  for (int e = threadIdx.x; e < rows * c4; e += kThreads) {
    int r = e % rows, c = (e / rows) << 2;
    float4 v = ld4<T>(src + r * lds + c);
    dst[(c + 0) * ldd + r] = v.x;
    dst[(c + 1) * ldd + r] = v.y;
    dst[(c + 2) * ldd + r] = v.z;
    dst[(c + 3) * ldd + r] = v.w;
  }
}

// Register-tiled CTA matrix product on shared-memory operands stored with the
// contraction index outermost:  acc(m, n) += sum_k As[k*lda + m] * Bs[k*ldb + n].
// 256 threads as a (M/TM) x (N/TN) grid, each owning a TM x TN block at rows
// ty*TM.., cols tx*TN...  lda/ldb must keep TM/TN-float vectors aligned.
template <int M, int N, int TM, int TN>
struct Tile {
  static constexpr int TX = N / TN;
  static constexpr int TY = M / TM;
  static constexpr int TM_ = TM, TN_ = TN;
  static_assert(TX * TY == kThreads, "tile must map onto 256 threads");
  static_assert(TM % 2 == 0 && TN % 2 == 0, "vector widths");
  float acc[TM][TN];
  int r0, c0;

  __device__ __forceinline__ Tile() {
    int t = threadIdx.x;
    r0 = (t / TX) * TM;
    c0 = (t % TX) * TN;
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
  }
  template <int W>
  __device__ __forceinline__ static void ldv(float* r, const float* p) {
    if constexpr (W % 4 == 0) {
#pragma unroll
      for (int i = 0; i < W; i += 4) {
        float4 v = *reinterpret_cast<const float4*>(p + i);
        r[i] = v.x; r[i + 1] = v.y; r[i + 2] = v.z; r[i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < W; i += 2) {
        float2 v = *reinterpret_cast<const float2*>(p + i);
        r[i] = v.x; r[i + 1] = v.y;
      }
    }
  }
  // k in [k0, k1)
  __device__ __forceinline__ void mma(const float* As, int lda, const float* Bs, int ldb,
                                      int k0, int k1) {
#pragma unroll 4
    for (int k = k0; k < k1; ++k) {
      float a[TM], b[TN];
      ldv<TM>(a, As + k * lda + r0);
      ldv<TN>(b, Bs + k * ldb + c0);
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
  }

  // Square-group variant for the intra-chunk score products: contraction over
  // the head dim d (k index), with the inter-group decay
  // gamma(d) = exp(gc[r0][d] - gc[c0][d]) folded into B.  Row/column groups are
  // TM == TN wide and start at r0 / c0; groups above the diagonal are skipped.
  __device__ __forceinline__ void mma_group_decay(const float* As, int lda, const float* Bs,
                                                  int ldb, const float* gc, int ldg, int K) {
    static_assert(TM == TN, "square groups");
    if (c0 > r0) return;
    const bool diag = (c0 == r0);
    const float* gr = gc + r0 * ldg;
    const float* gq = gc + c0 * ldg;
#pragma unroll 2
    for (int k = 0; k < K; ++k) {
      float a[TM], b[TN];
      ldv<TM>(a, As + k * lda + r0);
      ldv<TN>(b, Bs + k * ldb + c0);
      const float gm = diag ? 1.f : __expf(gr[k] - gq[k]);
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] *= gm;
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
  }

  // Grouped-decay variant for the score backward: contraction index k runs
  // over groups kg in [kg0, kg1) of GS = TM rows; every B row of group kg is
  // scaled per output column n by exp(gref[hi][n] - gref[lo][n]) with
  // hi = max(kg, rg), lo = min(kg, rg) (1 on the diagonal group).  gref holds
  // gc at the first row of each group (ld = ldg).
  __device__ __forceinline__ void mma_grouped(const float* As, int lda, const float* Bs, int ldb,
                                              const float* gref, int ldg, int kg0, int kg1,
                                              int rg) {
    for (int kg = kg0; kg < kg1; ++kg) {
      float gm[TN];
      if (kg == rg) {
#pragma unroll
        for (int j = 0; j < TN; ++j) gm[j] = 1.f;
      } else {
        const float* ghi = gref + (kg > rg ? kg : rg) * ldg + c0;
        const float* glo = gref + (kg > rg ? rg : kg) * ldg + c0;
#pragma unroll
        for (int j = 0; j < TN; ++j) gm[j] = __expf(ghi[j] - glo[j]);
      }
#pragma unroll
      for (int kk = 0; kk < TM; ++kk) {
        const int k = kg * TM + kk;
        float a[TM], b[TN];
        ldv<TM>(a, As + k * lda + r0);
        ldv<TN>(b, Bs + k * ldb + c0);
#pragma unroll
        for (int j = 0; j < TN; ++j) b[j] *= gm[j];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
    }
  }
};

// Pick a 256-thread register tile for an M x N output.
template <int M, int N> struct TileFor;
template <> struct TileFor<128, 128> { using type = Tile<128, 128, 8, 8>; };
template <> struct TileFor<128, 64>  { using type = Tile<128, 64, 8, 4>; };
template <> struct TileFor<64, 128>  { using type = Tile<64, 128, 4, 8>; };
template <> struct TileFor<64, 64>   { using type = Tile<64, 64, 4, 4>; };
template <> struct TileFor<128, 32>  { using type = Tile<128, 32, 4, 4>; };
template <> struct TileFor<64, 32>   { using type = Tile<64, 32, 4, 2>; };

// Block-wide reductions over 256 threads (scratch: 8 floats of shared memory).
__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

// Gate activations fused into the loads (GDN2_GATES_RAW): the caller passes
// the pre-activations, and the kernels read w = sigmoid(w'), b = sigmoid(b'),
// g = -softplus(g') (the activations the reference leaves to its caller,
// README.md:60-68).  Gradients leave with the chain rule applied:
// dw' = dw w (1 - w), db' = db b (1 - b), dg' = -dg sigmoid(g').
enum Gate { kGateW = 0, kGateB, kGateG };
__device__ __forceinline__ float gate_sig(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float gate_act(float x, int gate) {
  return gate == kGateG ? -(fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)))) : gate_sig(x);
}
__device__ __forceinline__ float4 gate_act4(float4 v, int gate) {
  return make_float4(gate_act(v.x, gate), gate_act(v.y, gate), gate_act(v.z, gate),
                     gate_act(v.w, gate));
}
template <typename T>
__device__ __forceinline__ float4 ld4_gate(const T* p, int raw, int gate) {
  const float4 v = ld4<T>(p);
  return raw ? gate_act4(v, gate) : v;
}
template <typename T>
__device__ __forceinline__ float ld_gate(const T* p, int raw, int gate) {
  const float x = to_f<T>(*p);
  return raw ? gate_act(x, gate) : x;
}
// d(sigmoid)/dx from the activated value s
__device__ __forceinline__ float4 sig_grad4(float4 s) {
  return make_float4(s.x * (1.f - s.x), s.y * (1.f - s.y), s.z * (1.f - s.z), s.w * (1.f - s.w));
}
__device__ __forceinline__ float4 mul4(float4 a, float4 b) {
  return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w);
}

// Per-stage diagnostics (the reference's _stage_diag, gdn2_fwd.py:47-76):
// non-finite count and largest finite |x| of a stage output, accumulated per
// thread and merged per warp into the workspace status header (ints
// kDiagBase + 2 s, kDiagBase + 2 s + 1 for stage s; the header is cleared by
// every call).  Only used when Problem::diag is set.
enum DiagStage {
  kDiagAqk = 0, kDiagAkk, kDiagA, kDiagW, kDiagU, kDiagKg, kDiagQg, kDiagO, kDiagHFinal,
  kNumDiag
};
constexpr int kDiagBase = 16;   // ints: byte offset 64 of the status header
struct StageDiag {
  float mx = 0.f;
  int nf = 0;
  __device__ __forceinline__ void add(float x) {
    if (isfinite(x)) mx = fmaxf(mx, fabsf(x));
    else ++nf;
  }
  __device__ __forceinline__ void add4(float4 v) { add(v.x); add(v.y); add(v.z); add(v.w); }
  // every lane of the warp calls this
  __device__ __forceinline__ void flush(int* hdr, int stage) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      nf += __shfl_xor_sync(0xffffffffu, nf, o);
    }
    if ((threadIdx.x & 31) == 0) {
      if (nf) atomicAdd(hdr + kDiagBase + 2 * stage, nf);
      atomicMax(hdr + kDiagBase + 2 * stage + 1, __float_as_int(mx));   // mx >= 0
    }
    mx = 0.f;
    nf = 0;
  }
};

}  // namespace gdn2
