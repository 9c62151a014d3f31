// Self-test of the tcgen05 3xTF32 building blocks (gdn2_tc.cuh): a batched
// 128 x N x K float32 product through canonical shared-memory tiles and a
// TMEM accumulator.  Exposed through the C ABI so the tests can check the
// descriptor encodings on the GPU.  trans_a / trans_b stage the operand from a
// transposed source through the register transpose the kernels use.
#include "../../include/gdn2.h"
#include "gdn2_common.cuh"
#include "gdn2_tc.cuh"

namespace gdn2 {

// D[b] = A[b] (128 x K, row-major) * B[b] (K x N, row-major), float32.
// Both operands are staged K-major; trans_a / trans_b pick gathered loads or
// 4x4 register-transposed loads for the staging.
__global__ void __launch_bounds__(kThreads, 1)
k_selftest_gemm(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ D,
                int K, int N, int trans_a, int trans_b, int* err) {
  constexpr int KS = 32;
  __shared__ __align__(16) float a_hi[128 * KS], a_lo[128 * KS];
  extern __shared__ __align__(16) float dyn[];   // b_hi, b_lo: N*KS each
  float* b_hi = dyn;
  float* b_lo = dyn + N * KS;
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5;
  const float* Ab = A + (size_t)blockIdx.x * 128 * K;
  const float* Bb = B + (size_t)blockIdx.x * K * N;
  float* Db = D + (size_t)blockIdx.x * 128 * N;
  const uint32_t ncols = N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
  if (warp == 0) tc::tmem_alloc(&tmem_slot, ncols);
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  uint32_t phase = 0;
  for (int k0 = 0; k0 < K; k0 += KS) {
    // A slice: 128 rows (m) x KS cols (k)
    for (int e = tid; e < 128 * KS / 4; e += kThreads) {
      const int m = e / (KS / 4), kk = (e % (KS / 4)) * 4;
      const float* p = Ab + (size_t)m * K + k0 + kk;
      const float4 v = trans_a ? make_float4(p[0], p[1], p[2], p[3])
                               : *reinterpret_cast<const float4*>(p);
      tc::st_split4(a_hi, a_lo, m, kk, KS, v);
    }
    if (!trans_b) {
      for (int e = tid; e < N * KS / 4; e += kThreads) {   // tile rows = n, cols = k
        const int n = e / (KS / 4), kk = (e % (KS / 4)) * 4;
        float4 v = make_float4(Bb[(size_t)(k0 + kk) * N + n], Bb[(size_t)(k0 + kk + 1) * N + n],
                               Bb[(size_t)(k0 + kk + 2) * N + n], Bb[(size_t)(k0 + kk + 3) * N + n]);
        tc::st_split4(b_hi, b_lo, n, kk, KS, v);
      }
    } else {
      for (int e = tid; e < (N / 4) * (KS / 4); e += kThreads) {   // 4x4 blocks
        const int n = (e % (N / 4)) * 4, kk = (e / (N / 4)) * 4;
        const float* p = Bb + (size_t)(k0 + kk) * N + n;
        tc::st_split4x4T(b_hi, b_lo, n, kk, KS, *reinterpret_cast<const float4*>(p),
                         *reinterpret_cast<const float4*>(p + N),
                         *reinterpret_cast<const float4*>(p + 2 * N),
                         *reinterpret_cast<const float4*>(p + 3 * N));
      }
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0) {
      const tc::Opnd Ao = tc::kmajor(a_hi, a_lo, KS);
      const tc::Opnd Bo = tc::kmajor(b_hi, b_lo, KS);
      tc::mma3(tmem, Ao, Bo, N, KS / 8, k0 > 0);
      tc::commit(&bar);
    }
    tc::mbar_wait(&bar, phase, err);
    phase ^= 1;
    tc::fence_after_sync();
  }
  // epilogue: warp w reads lanes 32*(w%4).., columns [half*N/2, (half+1)*N/2)
  const int row = 32 * (warp & 3) + (tid & 31);
  const int half = warp >> 2;
  for (int c = half * (N / 2); c < (half + 1) * (N / 2); c += 16) {
    float v[16];
    tc::tmem_ld16(tc::lane_quarter_addr(tmem, c), v);
#pragma unroll
    for (int j = 0; j < 16; ++j) Db[(size_t)row * N + c + j] = v[j];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_free(tmem, ncols);
}

// One warp waits on an mbarrier that nothing ever arrives on, with a short
// poll limit: the wait gives up, records kErrWaitTimeout in *status and the
// kernel returns.  No TMEM, no MMA and no copy is in flight.
__global__ void k_selftest_wait_timeout(int* status, long long polls) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  tc::mbar_wait(&bar, 0, status, polls);
}

}  // namespace gdn2

size_t gdn2_status_offset(const void* workspace);

extern "C" int gdn2_selftest_wait_timeout(void* workspace, size_t workspace_bytes, int polls,
                                          void* stream) {
  if (!workspace || workspace_bytes < 512 || polls <= 0) return GDN2_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = reinterpret_cast<int*>(static_cast<char*>(workspace) + gdn2_status_offset(workspace));
  if (cudaMemsetAsync(status, 0, 256, s) != cudaSuccess) return GDN2_ERR_CUDA;
  gdn2::k_selftest_wait_timeout<<<1, 32, 0, s>>>(status, polls);
  return cudaGetLastError() == cudaSuccess ? GDN2_OK : GDN2_ERR_CUDA;
}

extern "C" int gdn2_selftest_gemm_tf32x3(const float* A, const float* B, float* D, int batch,
                                         int K, int N, int trans_a, int trans_b, int* status,
                                         void* stream) {
  if (batch <= 0 || K <= 0 || K % 32 || N < 32 || N > 256 || N % 32) return GDN2_ERR_INVALID;
  const size_t smem = (size_t)2 * N * 32 * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(gdn2::k_selftest_gemm,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return GDN2_ERR_CUDA;
  gdn2::k_selftest_gemm<<<batch, gdn2::kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      A, B, D, K, N, trans_a, trans_b, status);
  return cudaGetLastError() == cudaSuccess ? GDN2_OK : GDN2_ERR_CUDA;
}
