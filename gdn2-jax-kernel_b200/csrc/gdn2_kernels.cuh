// Kernel-side declarations and the device building blocks shared by the
// forward and backward translation units.
#pragma once
#ifdef GDN2_PHASE_TIMING
#include <cstdio>
#endif
#include "gdn2_common.cuh"
#include "gdn2_ws.cuh"

namespace gdn2 {

// Supported (chunk, head-dim) shapes.
#define GDN2_FOR_SHAPES(X) X(64, 64) X(64, 128) X(128, 64) X(128, 128)
#define GDN2_FOR_SHAPES_T(X)                                                                 \
  X(float, 64, 64) X(float, 64, 128) X(float, 128, 64) X(float, 128, 128)                  \
  X(__nv_bfloat16, 64, 64) X(__nv_bfloat16, 64, 128) X(__nv_bfloat16, 128, 64)             \
  X(__nv_bfloat16, 128, 128)

template <int W>
__device__ __forceinline__ void store_vec(float* p, const float* v) {
  if constexpr (W % 4 == 0) {
#pragma unroll
    for (int i = 0; i < W; i += 4)
      *reinterpret_cast<float4*>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < W; i += 2) *reinterpret_cast<float2*>(p + i) = make_float2(v[i], v[i + 1]);
  }
}

template <int C, int D> struct FwdSmem {
  static constexpr int P = C > D ? C : D;
  static constexpr int BIG = P * (P + 4);
  static size_t bytes() { return (size_t)(C * D + 2 * BIG + 256 + 8) * sizeof(float); }
};
template <int C, int D, int NV> struct StateSmem {
  static constexpr int P = C > D ? C : D;
  static constexpr int BIG = P * (P + 4);
  static size_t bytes() { return (size_t)(BIG + D * NV + 2 * C * NV) * sizeof(float); }
};

// Block forward substitution of (I + T)^-1 in the reference's order
// (_block_solve, gdn2_fwd.py:192-222; Kernel B's sub-block step,
// gdn2_fwd.py:225-243, generalised from two sub-blocks to nb): within every
// group of nb diagonal blocks of size blk whose diagonal blocks already hold
// their inverses,
//     for m = 1 .. nb-1, n = m-1 .. 0:
//         acc = 0;  for k = n .. m-1:  acc = san(acc + T_mk A_kn)
//         A_mn = san(-A_mm acc)
// S is transposed (S[j*ld + i] = M(i, j)), holding T below the processed
// rows and A elsewhere.  `tmp` needs (nb-1) * BLK^2 * (C / (BLK*nb)) floats.
// Each thread owns a 4 x 4 tile of one output block: a float4 of four
// consecutive rows of S per contraction step (S is transposed, so rows are
// contiguous) against four columns, 16 FMAs per 5 shared loads.  ld must keep
// float4 rows 16-byte aligned (ld % 4 == 0).
template <int BLK>
__device__ __forceinline__ void wy_compose_seq(float* S, int ld, int C, int nb, float* tmp,
                                               float clip) {
  constexpr int per = BLK * BLK, TPB = (BLK / 4) * (BLK / 4);   // 4 x 4 tiles per block
  const int groups = C / (BLK * nb);
  for (int m = 1; m < nb; ++m) {
    const int tiles = groups * m * TPB;
    for (int e = threadIdx.x; e < tiles; e += kThreads) {   // acc_n of every block (m, n)
      const int gi = e / (m * TPB), rem = e - gi * (m * TPB), n = rem / TPB, tt = rem % TPB;
      const int ti = tt % (BLK / 4), tj = tt / (BLK / 4), o = gi * BLK * nb;
      const int row0 = o + m * BLK + 4 * ti, col0 = o + n * BLK + 4 * tj;
      float acc[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
      for (int k = n; k < m; ++k) {
        float sm4[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) sm4[r][c] = 0.f;
        const int x0 = o + k * BLK;
#pragma unroll 4
        for (int t = 0; t < BLK; ++t) {
          const float4 tv = *reinterpret_cast<const float4*>(S + (x0 + t) * ld + row0);  // T(row0+r, x)
          float av[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) av[c] = S[(col0 + c) * ld + x0 + t];             // A(x, col0+c)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            sm4[0][c] = fmaf(tv.x, av[c], sm4[0][c]);
            sm4[1][c] = fmaf(tv.y, av[c], sm4[1][c]);
            sm4[2][c] = fmaf(tv.z, av[c], sm4[2][c]);
            sm4[3][c] = fmaf(tv.w, av[c], sm4[3][c]);
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[r][c] = san(acc[r][c] + sm4[r][c], clip);
      }
      float* tb = tmp + (gi * (nb - 1) + n) * per;   // tb[j * BLK + i] = acc(i, j)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<float4*>(tb + (4 * tj + c) * BLK + 4 * ti) =
            make_float4(acc[0][c], acc[1][c], acc[2][c], acc[3][c]);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < tiles; e += kThreads) {   // A_mn = san(-A_mm acc_n)
      const int gi = e / (m * TPB), rem = e - gi * (m * TPB), n = rem / TPB, tt = rem % TPB;
      const int ti = tt % (BLK / 4), tj = tt / (BLK / 4), o = gi * BLK * nb;
      const int row0 = o + m * BLK + 4 * ti, col0 = o + n * BLK + 4 * tj;
      const float* tb = tmp + (gi * (nb - 1) + n) * per;
      const int xm = o + m * BLK;
      float sm4[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) sm4[r][c] = 0.f;
#pragma unroll 4
      for (int t = 0; t < BLK; ++t) {
        const float4 av = *reinterpret_cast<const float4*>(S + (xm + t) * ld + row0);   // A_mm(row0+r, t)
        float bv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) bv[c] = tb[(4 * tj + c) * BLK + t];                // acc(t, col0+c)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          sm4[0][c] = fmaf(av.x, bv[c], sm4[0][c]);
          sm4[1][c] = fmaf(av.y, bv[c], sm4[1][c]);
          sm4[2][c] = fmaf(av.z, bv[c], sm4[2][c]);
          sm4[3][c] = fmaf(av.w, bv[c], sm4[3][c]);
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<float4*>(S + (col0 + c) * ld + row0) =
            make_float4(san(-sm4[0][c], clip), san(-sm4[1][c], clip), san(-sm4[2][c], clip),
                        san(-sm4[3][c], clip));
    }
    __syncthreads();
  }
}

// Sub-block level of the substitution with blocks of bc rows (runtime size,
// a multiple of 16), dispatched to the unrolled forms.
__device__ __forceinline__ void wy_compose_blocks(float* S, int ld, int C, int bc, int nb,
                                                  float* tmp, float clip) {
  if (bc == 16) wy_compose_seq<16>(S, ld, C, nb, tmp, clip);
  else if (bc == 32) wy_compose_seq<32>(S, ld, C, nb, tmp, clip);
  else if (bc == 64) wy_compose_seq<64>(S, ld, C, nb, tmp, clip);
}

// Row-by-row forward substitution of every 16 x 16 diagonal block
// (_micro_forward_substitution, gdn2_fwd.py:174-189), in place on the
// transposed S; one warp per block, one lane per column of A.
template <int C>
__device__ __forceinline__ void wy_micro_solves(float* S, int ld, float clip) {
  constexpr int MBK = 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int blkid = warp; blkid < C / MBK; blkid += kThreads / 32) {
    if (lane < MBK) {
      const int o = blkid * MBK, jj = lane;
      float x[MBK];
#pragma unroll
      for (int r = 0; r < MBK; ++r) {
        float s = 0.f;
#pragma unroll
        for (int t = 0; t < r; ++t) s = fmaf(S[(o + t) * ld + o + r], x[t], s);
        x[r] = (r < jj) ? 0.f : (r == jj ? san(1.f - s, clip) : san(-s, clip));
      }
      __syncwarp(0x0000ffffu);
#pragma unroll
      for (int r = 0; r < MBK; ++r) S[(o + jj) * ld + o + r] = x[r];
    }
  }
  __syncthreads();
}

// In-place A = (I + T)^-1 for a strictly lower-triangular C x C matrix held
// transposed in shared memory (on entry S[j*ld + i] = T(i, j), on exit
// S[j*ld + i] = A(i, j)), in the reference's order: 16 x 16 micro solves,
// the block substitution of the 16-row blocks inside every BC sub-block
// (_block_solve), then of the BC sub-blocks (Kernel B).  Every product is
// sanitised where the reference sanitises it, so the result matches it also
// when CLIP acts.  BC is a multiple of 16 dividing C.  `tmp` needs C*C/4 floats.
template <int C>
__device__ __forceinline__ void wy_inverse_T(float* S, int ld, float* tmp, int bc, float clip) {
  wy_micro_solves<C>(S, ld, clip);
  if (bc > 16) wy_compose_seq<16>(S, ld, C, bc / 16, tmp, clip);
  if (C > bc) wy_compose_blocks(S, ld, C, bc, C / bc, tmp, clip);
}

// Column-wise inclusive prefix sum of a C x D tile held row-major in shared
// memory (ld = D).  256 threads: each column split into 256/D row segments.
// restart = true: each RS-row segment is summed on its own (two 64-row
// chunks per 128-row tile).
template <int C, int D, int LD = D>
__device__ __forceinline__ void column_cumsum(float* s, float* tot, bool restart = false) {
  constexpr int NSEG = kThreads / D;
  constexpr int RS = C / NSEG;
  const int d = threadIdx.x % D, seg = threadIdx.x / D;
  float acc = 0.f;
#pragma unroll 8
  for (int r = seg * RS; r < (seg + 1) * RS; ++r) acc += s[r * LD + d];
  tot[seg * D + d] = acc;
  __syncthreads();
  float off = 0.f;
  if (!restart)
    for (int sg = 0; sg < seg; ++sg) off += tot[sg * D + d];
#pragma unroll 8
  for (int r = seg * RS; r < (seg + 1) * RS; ++r) {
    off += s[r * LD + d];
    s[r * LD + d] = off;
  }
  __syncthreads();
}

// One doubling level of wy_inverse_T128 (blocks of 2*HALF, A10 = -A11 (T10
// A00)) on register tiles: each block's HALF x HALF outputs go to
// HALF*HALF/(TM*TN) threads with TM x TN outputs each.  The sums run over the
// full K range; the operands' upper-triangle entries are exact zeros in S, so
// the result equals the triangular sums bit for bit.
template <int HALF, int TM, int TN>
__device__ __forceinline__ void wy_level_tiled(float* S, int ld, float* tmp, float clip) {
  constexpr int P = HALF * HALF / (TM * TN);      // threads per block
  constexpr int TXI = HALF / TM;                  // lanes along i: contiguous rows
  static_assert(P * (128 / (2 * HALF)) == kThreads, "one pass over the blocks");
  const int beta = threadIdx.x / P, u = threadIdx.x % P;
  const int i0 = (u % TXI) * TM, j0 = (u / TXI) * TN, o = beta * 2 * HALF;
  float* tb = tmp + beta * HALF * HALF;           // tb[j * HALF + i] = tmp(i, j)
  float acc[TM][TN];
#pragma unroll
  for (int a = 0; a < TM; ++a)
#pragma unroll
    for (int b = 0; b < TN; ++b) acc[a][b] = 0.f;
#pragma unroll 4
  for (int kk = 0; kk < HALF; ++kk) {             // tmp = T10 A00
    float av[TM], bv[TN];
#pragma unroll
    for (int a = 0; a < TM; ++a) av[a] = S[(o + kk) * ld + o + HALF + i0 + a];
#pragma unroll
    for (int b = 0; b < TN; ++b) bv[b] = S[(o + j0 + b) * ld + o + kk];
#pragma unroll
    for (int a = 0; a < TM; ++a)
#pragma unroll
      for (int b = 0; b < TN; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
  }
#pragma unroll
  for (int a = 0; a < TM; ++a)
#pragma unroll
    for (int b = 0; b < TN; ++b) tb[(j0 + b) * HALF + i0 + a] = san(acc[a][b], clip);
  __syncthreads();
#pragma unroll
  for (int a = 0; a < TM; ++a)
#pragma unroll
    for (int b = 0; b < TN; ++b) acc[a][b] = 0.f;
#pragma unroll 4
  for (int kk = 0; kk < HALF; ++kk) {             // A10 = -A11 tmp
    float av[TM], bv[TN];
#pragma unroll
    for (int a = 0; a < TM; ++a) av[a] = S[(o + HALF + kk) * ld + o + HALF + i0 + a];
#pragma unroll
    for (int b = 0; b < TN; ++b) bv[b] = tb[(j0 + b) * HALF + kk];
#pragma unroll
    for (int a = 0; a < TM; ++a)
#pragma unroll
      for (int b = 0; b < TN; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
  }
#pragma unroll
  for (int a = 0; a < TM; ++a)
#pragma unroll
    for (int b = 0; b < TN; ++b) S[(o + j0 + b) * ld + o + HALF + i0 + a] = san(-acc[a][b], clip);
  __syncthreads();
}

// wy_inverse_T for C = 128.  For BC = 64 (two sub-blocks) the sub-block
// step is the two 64 x 64 x 64 products tmp = san(T10 A00),
// A10 = san(-A11 tmp) on register tiles; for BC = 32 the 16-row step inside a
// sub-block is one register-tiled level.  Other BC take the generic
// substitution.  `tmp` needs 4096 floats, `scr` 2 * 64 * 68.
// `span` = rows of one reference chunk: 128, or 64 when the tile holds two
// chunks (block-diagonal T; the two 64-row groups are solved independently).
__device__ __forceinline__ void wy_inverse_T128(float* S, int ld, float* tmp, float* scr, int bc,
                                                float clip, int span = 128) {
  constexpr int C = 128, H = 64, LY = 68;
#ifdef GDN2_PHASE_TIMING
  long long t0 = clock64();
  long long wy_t[2];
  (void)wy_t;
#endif
  wy_micro_solves<C>(S, ld, clip);
#ifdef GDN2_PHASE_TIMING
  long long t1 = clock64();
#endif
  if (bc == 32) wy_level_tiled<16, 2, 2>(S, ld, tmp, clip);            // two 16-row blocks
  else if (bc > 16) wy_compose_seq<16>(S, ld, C, bc / 16, tmp, clip);   // inside each sub-block
#ifdef GDN2_PHASE_TIMING
  long long t2 = clock64();
  if (blockIdx.x == gridDim.x / 2 && threadIdx.x == 0) wy_t[0] = t1 - t0, wy_t[1] = t2 - t1;
#endif
  if (bc != 64 || span != C) {
    if (span > bc) wy_compose_blocks(S, ld, C, bc, span / bc, tmp, clip);
    return;
  }
  // last level: T10 = M(64.., 0..63), A00 = A(0..63, 0..63), A11 = A(64.., 64..)
  float* y = scr;             // y[k][j] = A00(k, j)   (row-major copy)
  float* t = scr + H * LY;    // t[k][j] = tmp(k, j)
  for (int e = threadIdx.x; e < H * H; e += kThreads) {
    const int j = e / H, kk = e % H;
    y[kk * LY + j] = S[j * ld + kk];
  }
  __syncthreads();
  using T64 = Tile<64, 64, 4, 4>;
  {
    T64 tt;
    tt.zero();
    tt.mma(S + H, ld, y, LY, 0, H);             // X(i,k) = S[k*ld + 64 + i] = T10(i,k)
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      float o4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) o4[q] = san(tt.acc[ii][q], clip);
      store_vec<4>(t + (tt.r0 + ii) * LY + tt.c0, o4);
    }
  }
  __syncthreads();
  {
    T64 tt;
    tt.zero();
    tt.mma(S + H * ld + H, ld, t, LY, 0, H);    // X(i,k) = A11(i,k)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float o4[4];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) o4[ii] = san(-tt.acc[ii][q], clip);
      store_vec<4>(S + (tt.c0 + q) * ld + H + tt.r0, o4);
    }
  }
  __syncthreads();
#ifdef GDN2_PHASE_TIMING
  if (blockIdx.x == gridDim.x / 2 && threadIdx.x == 0)
    printf("wy phases: micro %lld in-block %lld last %lld\n", wy_t[0], wy_t[1], clock64() - t2);
#endif
}

// Reverse (suffix) column sum of a C x D tile in shared memory (ld = D),
// the in-chunk reverse cumsum of gdn2_bwd.py:32-41.  `tot` >= 256 floats.
template <int C, int D>
__device__ __forceinline__ void column_revcumsum(float* s, float* tot, bool restart = false) {
  constexpr int NSEG = kThreads / D;
  constexpr int RS = C / NSEG;
  const int d = threadIdx.x % D, seg = threadIdx.x / D;
  float acc = 0.f;
  for (int r = seg * RS; r < (seg + 1) * RS; ++r) acc += s[r * D + d];
  tot[seg * D + d] = acc;
  __syncthreads();
  float off = 0.f;
  if (!restart)
    for (int sg = seg + 1; sg < NSEG; ++sg) off += tot[sg * D + d];
  for (int r = (seg + 1) * RS - 1; r >= seg * RS; --r) {
    off += s[r * D + d];
    s[r * D + d] = off;
  }
  __syncthreads();
}

// Stage ids for the optional per-launch CUDA-event profiler of the C ABI.
enum Stage {
  kStageFwdIntra = 0, kStageFwdState, kStageBwdState, kStageBwdIntra1, kStageBwdIntra2,
  kStageBwdIntra3, kStageFwdAffine, kStageFwdScan, kStageFwdOut, kStageBwdPrep, kStageBwdScan,
  kStageBwdExact, kNumStages
};

// Called around every kernel launch of a multi-kernel launcher (no-op unless
// the C ABI's profiler is on).
struct LaunchHook {
  void (*fn)(int stage, int end, cudaStream_t s) = nullptr;
  void begin(int st, cudaStream_t s) const { if (fn) fn(st, 0, s); }
  void end(int st, cudaStream_t s) const { if (fn) fn(st, 1, s); }
};

// Launchers (defined in gdn2_fwd.cu / gdn2_bwd.cu).
template <typename T, int C, int D>
cudaError_t launch_fwd_intra(const T* q, const T* k, const T* v, const T* w, const T* b,
                             const T* g, const Problem& p, const Workspace& ws, cudaStream_t s);
template <int C, int D>
cudaError_t launch_fwd_state(const Problem& p, const Workspace& ws, const float* h0, float* o,
                             float* hfinal, int save, cudaStream_t s);
template <int C, int D>
cudaError_t launch_bwd_state(const Problem& p, const Workspace& ws, const float* dout,
                             const float* dh_final, float* dh0, cudaStream_t s,
                             bool only_flagged = false, bool pair = false);
template <typename T, int C, int D>
cudaError_t launch_bwd_intra(const T* q, const T* k, const T* v, const T* w, const T* b,
                             const T* g, const float* dout, const float* dh_final, T* dq, T* dk,
                             T* dv, T* dw, T* db, T* dg, const Problem& p, const Workspace& ws,
                             cudaStream_t s, const LaunchHook& hook, bool skip12 = false);
template <typename T>
cudaError_t launch_tc_bwd_intra3(const T* q, const T* k, const T* b, const T* g, T* dq, T* dk,
                                 T* db, T* dg, const Problem& p, const Workspace& ws,
                                 cudaStream_t s, const LaunchHook& hook);
template <typename T>
cudaError_t launch_tc_fwd_intra(const T* q, const T* k, const T* v, const T* w, const T* b,
                                const T* g, const Problem& p, const Workspace& ws, cudaStream_t s);
template <typename T>
cudaError_t launch_tc_bwd_intra12(const T* q, const T* k, const T* v, const T* w, const T* b,
                                  const float* dout, const float* dh_final, T* dv_out, T* dw_out,
                                  const Problem& p, const Workspace& ws, cudaStream_t s,
                                  const LaunchHook& hook);

// Sequence-parallel pieces (tensor-core path): op 0 segment map P = prod M_c,
// op 1 rescan from the start state `in` + chunk outputs, op 2 backward
// segment term from dout = `in` with zero incoming gradient.
cudaError_t launch_tc_sp(int op, const Problem& p, const Workspace& ws, const float* in, float* o,
                         float* out, cudaStream_t s, const LaunchHook& hook);
// Tensor-core path (chunk = head dim = 128, float32 workspace), gdn2_tc_kernels.cu.
// outputs = false: no k_tc_fwd_out (o and the vnew residual are left to a
// later rescan); with_prep = false: the k_tc_bwd_prep terms are in place.
cudaError_t launch_tc_fwd(const Problem& p, const Workspace& ws, const float* h0, float* o,
                          float* hfinal, cudaStream_t s, const LaunchHook& hook,
                          bool outputs = true);
cudaError_t launch_tc_bwd_state(const Problem& p, const Workspace& ws, const float* dout,
                                const float* dh_final, float* dh0, cudaStream_t s,
                                const LaunchHook& hook, bool with_prep = true);

}  // namespace gdn2
