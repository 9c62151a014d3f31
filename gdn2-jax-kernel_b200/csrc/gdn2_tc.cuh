// Blackwell (sm_100a) tensor-core building blocks: tcgen05.mma kind::tf32
// with TMEM accumulators, used as 3xTF32 (a = hi + lo; D += hi*hi + hi*lo +
// lo*hi) for float32-accurate products.
//
// Shared-memory operand layout ("canonical tile"): an R x K float tile is a
// grid of core matrices of 8 rows x 16 bytes (4 floats), stored row-group
// major with the 4-column chunks fastest:
//   byte(r, c) = ((r/8) * (K/4) + c/4) * 128 + (r%8) * 16 + (c%4) * 4.
// Operands are always K-major: the contraction index runs along the columns
// of the stored tile (no-swizzle layout, 16-byte aligned).  Measured on B200
// (tests/test_gpu_tc.py): an MN-major (transposed) kind::tf32 operand yields
// an all-zero product, so a transposed operand is transposed while it is
// staged instead.
//
// Every wait on an mbarrier is bounded; on expiry the kernel records an error
// code in a caller-provided device status word and proceeds (its results are
// then invalid; the C ABI reports the word through gdn2_workspace_status).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn2 {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t canon_off(int r, int c, int K) {
  return (uint32_t)((((r >> 3) * (K >> 2)) + (c >> 2)) * 128 + (r & 7) * 16 + (c & 3) * 4);
}

// Split x into a tf32-exact head (low 13 mantissa bits cleared) and the rest.
__device__ __forceinline__ void split(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  lo = x - hi;
}
__device__ __forceinline__ void split4(float4 v, float4& h, float4& l) {
  split(v.x, h.x, l.x); split(v.y, h.y, l.y); split(v.z, h.z, l.z); split(v.w, h.w, l.w);
}

// Store 4 consecutive columns (c % 4 == 0) of row r of an R x K canonical tile
// pair (hi plane, lo plane).
__device__ __forceinline__ void st_split4(float* hi, float* lo, int r, int c, int K, float4 v) {
  float4 h, l;
  split4(v, h, l);
  const uint32_t o = canon_off(r, c, K) >> 2;
  *reinterpret_cast<float4*>(hi + o) = h;
  *reinterpret_cast<float4*>(lo + o) = l;
}

// Rows r0..r0+3 of a 4x4 block given as 4 float4 rows of the transposed
// source (src row j = tile column c + j, columns = tile rows r0..r0+3):
// transpose in registers and store 4 tile rows of 4 columns each.
__device__ __forceinline__ void st_split4x4T(float* hi, float* lo, int r0, int c, int K, float4 s0,
                                             float4 s1, float4 s2, float4 s3) {
  st_split4(hi, lo, r0 + 0, c, K, make_float4(s0.x, s1.x, s2.x, s3.x));
  st_split4(hi, lo, r0 + 1, c, K, make_float4(s0.y, s1.y, s2.y, s3.y));
  st_split4(hi, lo, r0 + 2, c, K, make_float4(s0.z, s1.z, s2.z, s3.z));
  st_split4(hi, lo, r0 + 3, c, K, make_float4(s0.w, s1.w, s2.w, s3.w));
}

// --------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (no swizzle): start >> 4 at [0,14),
// leading byte offset >> 4 at [16,30), stride byte offset >> 4 at [32,46),
// descriptor version 1 at [46,48), layout type 0 (none) at [61,64).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3fff) | ((uint64_t)((lbo >> 4) & 0x3fff) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fff) << 32) | (1ull << 46);
}

// K-major operand view of a canonical tile (rows = M or N, cols = K):
// LBO = 128 (the two 16-byte K chunks of one k-step), SBO = (cols/4)*128
// (between 8-row groups); one k-step (8 columns) advances 256 bytes.
struct Opnd {
  uint32_t hi, lo;      // shared addresses of the two planes
  uint32_t lbo, sbo, step;
  uint32_t mn_major;
};
__device__ __forceinline__ Opnd kmajor(const float* hi, const float* lo, int cols) {
  return Opnd{smem_u32(hi), smem_u32(lo), 128u, (uint32_t)(cols / 4) * 128u, 256u, 0u};
}
__device__ __forceinline__ Opnd advance(Opnd o, int ksteps) {
  o.hi += o.step * ksteps;
  o.lo += o.step * ksteps;
  return o;
}

// Instruction descriptor, kind::tf32, f32 accumulate: c_format F32 (1) at
// [4,6), a/b format TF32 (2) at [7,10) / [10,13), a/b major at bits 15/16,
// N >> 3 at [17,23), M >> 4 at [24,29).
__device__ __forceinline__ uint32_t idesc_tf32(int M, int N, uint32_t a_mn, uint32_t b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (a_mn << 15) | (b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// D[128 x N] (+)= A[128 x 8*ksteps] * B[N x 8*ksteps]^T in 3xTF32.  Issued by
// one thread.  `accumulate` = 0 overwrites D on the first product.
__device__ __forceinline__ void mma3(uint32_t d_tmem, const Opnd& A, const Opnd& B, int N,
                                     int ksteps, uint32_t accumulate) {
  const uint32_t id = idesc_tf32(128, N, A.mn_major, B.mn_major);
  for (int s = 0; s < ksteps; ++s) {
    const uint64_t ah = sdesc(A.hi + s * A.step, A.lbo, A.sbo);
    const uint64_t al = sdesc(A.lo + s * A.step, A.lbo, A.sbo);
    const uint64_t bh = sdesc(B.hi + s * B.step, B.lbo, B.sbo);
    const uint64_t bl = sdesc(B.lo + s * B.step, B.lbo, B.sbo);
    mma_tf32(d_tmem, al, bh, id, (s > 0 || accumulate) ? 1u : 0u);
    mma_tf32(d_tmem, ah, bl, id, 1u);
    mma_tf32(d_tmem, ah, bh, id, 1u);
  }
}

// A operand in TMEM (lane = row m, one 32-bit column per k; the tensor core
// reads a float32 word as its tf32 head, the low 13 mantissa bits ignored).
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

// mma3 with the A planes in TMEM: a_hi / a_lo are the TMEM addresses of the
// first k column of the slice (hi and lo planes, 8 columns per k-step).
__device__ __forceinline__ void mma3_ta(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo,
                                        const Opnd& B, int N, int ksteps, uint32_t accumulate) {
  const uint32_t id = idesc_tf32(128, N, 0, B.mn_major);
  for (int s = 0; s < ksteps; ++s) {
    const uint64_t bh = sdesc(B.hi + s * B.step, B.lbo, B.sbo);
    const uint64_t bl = sdesc(B.lo + s * B.step, B.lbo, B.sbo);
    mma_tf32_ta(d_tmem, a_lo + 8 * s, bh, id, (s > 0 || accumulate) ? 1u : 0u);
    mma_tf32_ta(d_tmem, a_hi + 8 * s, bl, id, 1u);
    mma_tf32_ta(d_tmem, a_hi + 8 * s, bh, id, 1u);
  }
}

// ------------------------------------------------------------------ barriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Status word written on a timed-out wait (a device int the caller provides).
constexpr int kErrWaitTimeout = 1;
constexpr long long kWaitLimit = 1ll << 22;

// Wait for the phase with parity `parity` of `bar` to complete; bounded.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          long long limit = kWaitLimit) {
  const uint32_t a = smem_u32(bar);
  for (long long it = 0; it < limit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  if (err) atomicExch(err, kErrWaitTimeout);
  return false;
}

// Bulk (non-tensor) copy global -> this CTA's shared memory, completing
// `bytes` of transaction count on `bar`; both addresses 16-byte aligned, bytes
// a multiple of 16.  The expecting arrival is mbar_arrive_expect_tx.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Arrive on `bar` when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Generic-proxy shared-memory writes -> visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// -------------------------------------------------------------------- TMEM
// Allocate `ncols` (power of two >= 32) TMEM columns; called by one full warp.
// The base address is written to *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols)
               : "memory");
}

// Load 16 consecutive f32 columns of this thread's TMEM lane.  `taddr` must
// carry the warp's lane quarter in bits [16, 32): (32 * (warp % 4)) << 16.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Load 64 consecutive f32 columns of this thread's TMEM lane (address rule as
// tmem_ld16): four loads in flight, one wait.  The wait names the 64
// registers so that no use of them is scheduled before it.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr + 0));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr + 16));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47])
      : "r"(taddr + 32));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr + 48));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]), "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]), "+r"(r[36]), "+r"(r[37]), "+r"(r[38]), "+r"(r[39]), "+r"(r[40]), "+r"(r[41]), "+r"(r[42]), "+r"(r[43]), "+r"(r[44]), "+r"(r[45]), "+r"(r[46]), "+r"(r[47]), "+r"(r[48]), "+r"(r[49]), "+r"(r[50]), "+r"(r[51]), "+r"(r[52]), "+r"(r[53]), "+r"(r[54]), "+r"(r[55]), "+r"(r[56]), "+r"(r[57]), "+r"(r[58]), "+r"(r[59]), "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive f32 columns of this thread's TMEM lane (same address
// rule as tmem_ld16); completion needs tmem_st_wait().
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
      "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t lane_quarter_addr(uint32_t tmem_base, int col) {
  const int warp = threadIdx.x >> 5;
  return tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)col;
}

}  // namespace tc
}  // namespace gdn2
