// Staging of 128 x 32 K-slices of float32 operands from global memory into
// canonical 3xTF32 shared-memory tiles (see gdn2_tc.cuh), with a per-element
// transform, and the double-buffered slice loop around tcgen05.mma.
#pragma once
#include "gdn2_common.cuh"
#include "gdn2_tc.cuh"

namespace gdn2 {
namespace tc {

constexpr int KS = 32;                               // K-slice width
constexpr int SLICE_FLOATS = 128 * KS;               // one plane of one slice
constexpr int SLICE_BYTES = 2 * SLICE_FLOATS * 4;    // hi + lo planes

struct Ident {
  __device__ __forceinline__ float4 operator()(float4 v) const { return v; }
};
struct Scale {
  float s;
  __device__ __forceinline__ float4 operator()(float4 v) const {
    return make_float4(s * v.x, s * v.y, s * v.z, s * v.w);
  }
};

// tile(r, k) = src[r * ld + k0 + k], r < 128, k < 32.  A warp covers 8 rows x
// 4 column chunks, so its 16-byte shared stores span all 8 bank quads.
template <class F>
__device__ __forceinline__ void stage_direct(float* hi, float* lo, const float* src,
                                             long ld, int k0, F f) {
#pragma unroll
  for (int it = 0; it < 1024 / kThreads; ++it) {
    const int e = threadIdx.x + it * kThreads;
    const int lane = e & 31, w = e >> 5;
    const int r = (w & 15) * 8 + (lane & 7);
    const int c = ((w >> 4) * 4 + (lane >> 3)) * 4;
    const float4 v = *reinterpret_cast<const float4*>(src + r * ld + k0 + c);
    st_split4(hi, lo, r, c, KS, f(v));
  }
}

// tile(r, k) = src[(k0 + k) * ld + r]: 4 x 4 blocks read as 4 float4 rows of
// the source and transposed in registers.  The store order of the 4 tile rows
// is rotated by lane so the 8 lanes of each quarter-warp (one 16-byte store
// phase) hit 8 distinct bank quads.
template <class F>
__device__ __forceinline__ void stage_trans(float* hi, float* lo, const float* src,
                                            long ld, int k0, F f) {
  const int e = threadIdx.x;                       // 256 blocks of 4 x 4
  const int rb = (e & 7) + ((e >> 5) & 3) * 8;     // 32 row blocks
  const int kb = ((e >> 3) & 3) + (e >> 7) * 4;    // 8 column blocks
  const int r0 = rb * 4, c0 = kb * 4;
  const float* p = src + (long)(k0 + c0) * ld + r0;
  const float4 s0 = *reinterpret_cast<const float4*>(p);
  const float4 s1 = *reinterpret_cast<const float4*>(p + ld);
  const float4 s2 = *reinterpret_cast<const float4*>(p + 2 * ld);
  const float4 s3 = *reinterpret_cast<const float4*>(p + 3 * ld);
  const float4 t0 = make_float4(s0.x, s1.x, s2.x, s3.x), t1 = make_float4(s0.y, s1.y, s2.y, s3.y);
  const float4 t2 = make_float4(s0.z, s1.z, s2.z, s3.z), t3 = make_float4(s0.w, s1.w, s2.w, s3.w);
  const int rot = (e >> 1) & 3;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int j = (t + rot) & 3;
    const float4 v = j == 0 ? t0 : (j == 1 ? t1 : (j == 2 ? t2 : t3));
    st_split4(hi, lo, r0 + j, c0, KS, f(v));
  }
}

// Split forms of the two staging patterns: load a thread's share of a slice
// into registers (so the load can be issued early), store it later.
struct Frag {
  float4 v[4];
};
__device__ __forceinline__ void load_direct(Frag& f, const float* src, long ld, int k0) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int e = threadIdx.x + it * kThreads;
    const int lane = e & 31, w = e >> 5;
    const int r = (w & 15) * 8 + (lane & 7);
    const int c = ((w >> 4) * 4 + (lane >> 3)) * 4;
    f.v[it] = *reinterpret_cast<const float4*>(src + r * ld + k0 + c);
  }
}
__device__ __forceinline__ float4 scl(float4 v, float s) {
  return make_float4(s * v.x, s * v.y, s * v.z, s * v.w);
}
__device__ __forceinline__ void store_direct(float* hi, float* lo, const Frag& f, float sc = 1.f) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int e = threadIdx.x + it * kThreads;
    const int lane = e & 31, w = e >> 5;
    const int r = (w & 15) * 8 + (lane & 7);
    const int c = ((w >> 4) * 4 + (lane >> 3)) * 4;
    st_split4(hi, lo, r, c, KS, scl(f.v[it], sc));
  }
}
__device__ __forceinline__ void load_trans(Frag& f, const float* src, long ld, int k0) {
  const int e = threadIdx.x;
  const int rb = (e & 7) + ((e >> 5) & 3) * 8;
  const int kb = ((e >> 3) & 3) + (e >> 7) * 4;
  const float* p = src + (long)(k0 + kb * 4) * ld + rb * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) f.v[j] = *reinterpret_cast<const float4*>(p + j * ld);
}
__device__ __forceinline__ void store_trans(float* hi, float* lo, const Frag& f, float sc = 1.f) {
  const int e = threadIdx.x;
  const int rb = (e & 7) + ((e >> 5) & 3) * 8;
  const int kb = ((e >> 3) & 3) + (e >> 7) * 4;
  const int r0 = rb * 4, c0 = kb * 4;
  const float4 s0 = f.v[0], s1 = f.v[1], s2 = f.v[2], s3 = f.v[3];
  const float4 t0 = make_float4(s0.x, s1.x, s2.x, s3.x), t1 = make_float4(s0.y, s1.y, s2.y, s3.y);
  const float4 t2 = make_float4(s0.z, s1.z, s2.z, s3.z), t3 = make_float4(s0.w, s1.w, s2.w, s3.w);
  const int rot = (e >> 1) & 3;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int j = (t + rot) & 3;
    st_split4(hi, lo, r0 + j, c0, KS, scl(j == 0 ? t0 : (j == 1 ? t1 : (j == 2 ? t2 : t3)), sc));
  }
}

// Loader forms: ld(r, c) returns tile(r, c..c+3) (direct), or ld(kk, r0)
// returns tile(r0..r0+3, kk), i.e. one float4 row of the transposed source.
template <class L>
__device__ __forceinline__ void stage_direct_f(float* hi, float* lo, L ld) {
#pragma unroll
  for (int it = 0; it < 1024 / kThreads; ++it) {
    const int e = threadIdx.x + it * kThreads;
    const int lane = e & 31, w = e >> 5;
    const int r = (w & 15) * 8 + (lane & 7);
    const int c = ((w >> 4) * 4 + (lane >> 3)) * 4;
    st_split4(hi, lo, r, c, KS, ld(r, c));
  }
}
template <class L>
__device__ __forceinline__ void stage_trans_f(float* hi, float* lo, L ld) {
  const int e = threadIdx.x;
  const int rb = (e & 7) + ((e >> 5) & 3) * 8;
  const int kb = ((e >> 3) & 3) + (e >> 7) * 4;
  Frag f;
#pragma unroll
  for (int j = 0; j < 4; ++j) f.v[j] = ld(kb * 4 + j, rb * 4);
  store_trans(hi, lo, f);
}

// Slice ring of two buffers, each holding NOP operand slices.
struct Ring {
  float* base;          // 2 * nop * SLICE_BYTES bytes
  uint64_t* bars;       // 2 mbarriers (one per buffer)
  uint32_t phase[2];
  int nop;
  __device__ __forceinline__ float* hi(int buf, int op) const {
    return base + (size_t)(buf * nop + op) * 2 * SLICE_FLOATS;
  }
  __device__ __forceinline__ float* lo(int buf, int op) const { return hi(buf, op) + SLICE_FLOATS; }
  __device__ __forceinline__ Opnd op(int buf, int o) const {
    return kmajor(hi(buf, o), lo(buf, o), KS);
  }
};

// Make the staged slices visible to the tensor core and to the issuing thread.
__device__ __forceinline__ void slice_publish() {
  fence_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
}

// Wait until the MMAs that last read buffer `buf` completed (no-op for the
// first use of each buffer).
__device__ __forceinline__ void ring_acquire(Ring& r, int buf, int uses, int* err) {
  if (uses > 0) {
    mbar_wait(&r.bars[buf], r.phase[buf], err);
    r.phase[buf] ^= 1;
  }
}

// One K = 128 pass in four 32-wide slices: stage(buf, s) fills the buffer,
// issue(buf, s) (thread 0) issues the MMAs that read it.
template <class St, class Is>
__device__ __forceinline__ void kloop(Ring& ring, int& g, int* err, St stage, Is issue) {
  for (int s = 0; s < 128 / KS; ++s, ++g) {
    const int buf = g & 1;
    ring_acquire(ring, buf, g >> 1, err);
    stage(buf, s);
    slice_publish();
    if (threadIdx.x == 0) {
      issue(buf, s);
      commit(&ring.bars[buf]);
    }
  }
}

// A float32 operand source for the prefetching K loop: tile(r, k) =
// sc * p[r*ld + k] (trans = false) or sc * p[k*ld + r] (trans = true).
struct Src {
  const float* p;
  long ld;
  float sc;
  bool trans;
  float clip;     // > 0: the staged values are sanitised to +-clip (after scaling)
  int rlo, rhi;   // tile rows outside [rlo, rhi) are staged as zeros (not loaded)
};
__device__ __forceinline__ Src direct(const float* p, long ld, float sc = 1.f) {
  return Src{p, ld, sc, false, 0.f, 0, 128};
}
__device__ __forceinline__ Src trans(const float* p, long ld, float sc = 1.f, float clip = 0.f) {
  return Src{p, ld, sc, true, clip, 0, 128};
}
// Only tile rows [lo, hi) (multiples of 8) of the source (one chunk of a
// paired tile).
__device__ __forceinline__ Src rows(Src s, int lo, int hi) {
  s.rlo = lo;
  s.rhi = hi;
  return s;
}
// MASK = false: the row range is ignored (every source of the one-chunk
// kernels); MASK = true honours it.
template <bool MASK = false>
__device__ __forceinline__ void src_load(const Src& s, int k0, Frag& f) {
  if (!MASK) {
    if (s.trans) load_trans(f, s.p, s.ld, k0);
    else load_direct(f, s.p, s.ld, k0);
    return;
  }
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  const int e = threadIdx.x;
  if (s.trans) {   // the thread's 4 tile rows rb*4 .. rb*4+3
    const int rb = (e & 7) + ((e >> 5) & 3) * 8;
    const int kb = ((e >> 3) & 3) + (e >> 7) * 4;
    const bool in = rb * 4 >= s.rlo && rb * 4 < s.rhi;
    const float* p = s.p + (long)(k0 + kb * 4) * s.ld + rb * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) f.v[j] = in ? *reinterpret_cast<const float4*>(p + j * s.ld) : z;
  } else {
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int x = e + it * kThreads;
      const int lane = x & 31, w = x >> 5;
      const int r = (w & 15) * 8 + (lane & 7);
      const int c = ((w >> 4) * 4 + (lane >> 3)) * 4;
      f.v[it] = (r >= s.rlo && r < s.rhi) ? *reinterpret_cast<const float4*>(s.p + r * s.ld + k0 + c) : z;
    }
  }
}
__device__ __forceinline__ void src_store(const Src& s, float* hi, float* lo, const Frag& f) {
  Frag g = f;
  if (s.clip > 0.f) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      g.v[i] = make_float4(san(s.sc * f.v[i].x, s.clip), san(s.sc * f.v[i].y, s.clip),
                           san(s.sc * f.v[i].z, s.clip), san(s.sc * f.v[i].w, s.clip));
    if (s.trans) store_trans(hi, lo, g, 1.f);
    else store_direct(hi, lo, g, 1.f);
    return;
  }
  if (s.trans) store_trans(hi, lo, g, s.sc);
  else store_direct(hi, lo, g, s.sc);
}

// K = 128 pass over NOP float32 sources with register double-buffering: the
// loads of slice s+1 are in flight while slice s is split, stored and issued.
// Operand slot o of the ring holds source o; extra(buf, s) may stage more
// slots synchronously (e.g. products of several input tensors).
// The slice loop is rolled (one copy of its body: the kernels run each K loop
// once per chunk, so unrolled copies cost instruction-cache misses); the
// register double buffer advances by copying the prefetched slice.
template <int NS, bool MASK, int NOP, class Ex, class Is>
__device__ __forceinline__ void kloop_pf_unrolled(Ring& ring, int& g, int* err,
                                                  const Src (&src)[NOP], Ex extra, Is issue) {
  Frag fa[NOP], fb[NOP];
#pragma unroll
  for (int o = 0; o < NOP; ++o) src_load<MASK>(src[o], 0, fa[o]);
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    Frag* cur = (s & 1) ? fb : fa;
    Frag* nxt = (s & 1) ? fa : fb;
    if (s + 1 < NS) {
#pragma unroll
      for (int o = 0; o < NOP; ++o) src_load<MASK>(src[o], (s + 1) * KS, nxt[o]);
    }
    const int buf = g & 1;
    ring_acquire(ring, buf, g >> 1, err);
#pragma unroll
    for (int o = 0; o < NOP; ++o) src_store(src[o], ring.hi(buf, o), ring.lo(buf, o), cur[o]);
    extra(buf, s);
    slice_publish();
    if (threadIdx.x == 0) {
      issue(buf, s);
      commit(&ring.bars[buf]);
    }
    ++g;
  }
}

// ROLL = false: the slice loop fully unrolled (measured faster for the short
// kernels whose K loops carry few operands: affine, fwd_out, bwd_prep, and the
// dv / dqg loops of bwd_intra1).  NS: 32-wide K slices (4 = K of 128; 2 = one
// 64-row chunk of a paired tile), MASK: honour the sources' row ranges (both
// unrolled form only).
template <bool ROLL = true, int NS = 128 / KS, bool MASK = false, int NOP, class Ex, class Is>
__device__ __forceinline__ void kloop_pf(Ring& ring, int& g, int* err, const Src (&src)[NOP],
                                         Ex extra, Is issue) {
  static_assert((NS == 128 / KS && !MASK) || !ROLL, "partial or masked K loops are unrolled");
  if (!ROLL) {
    kloop_pf_unrolled<NS, MASK>(ring, g, err, src, extra, issue);
    return;
  }
  Frag cur[NOP], nxt[NOP];
#pragma unroll
  for (int o = 0; o < NOP; ++o) src_load(src[o], 0, cur[o]);
#pragma unroll 1
  for (int s = 0; s < 128 / KS; ++s) {
    if (s + 1 < 128 / KS) {
#pragma unroll
      for (int o = 0; o < NOP; ++o) src_load(src[o], (s + 1) * KS, nxt[o]);
    }
    const int buf = g & 1;
    ring_acquire(ring, buf, g >> 1, err);
#pragma unroll
    for (int o = 0; o < NOP; ++o) src_store(src[o], ring.hi(buf, o), ring.lo(buf, o), cur[o]);
    extra(buf, s);
    slice_publish();
    if (threadIdx.x == 0) {
      issue(buf, s);
      commit(&ring.bars[buf]);
    }
    ++g;
#pragma unroll
    for (int o = 0; o < NOP; ++o) cur[o] = nxt[o];
  }
}
// kloop_pf with the MMA issue split over NISS issuing threads (lane 0 of
// warps 0 .. NISS-1): issue(buf, s, who) issues issuer `who`'s share, which
// that thread then commits.  The ring's barriers need arrival count NISS.
template <int NISS, int NOP, class Ex, class Is>
__device__ __forceinline__ void kloop_pf_n(Ring& ring, int& g, int* err, const Src (&src)[NOP],
                                           Ex extra, Is issue) {
  Frag fa[NOP], fb[NOP];
#pragma unroll
  for (int o = 0; o < NOP; ++o) src_load(src[o], 0, fa[o]);
#pragma unroll
  for (int s = 0; s < 128 / KS; ++s) {
    Frag* cur = (s & 1) ? fb : fa;
    Frag* nxt = (s & 1) ? fa : fb;
    if (s + 1 < 128 / KS) {
#pragma unroll
      for (int o = 0; o < NOP; ++o) src_load(src[o], (s + 1) * KS, nxt[o]);
    }
    const int buf = g & 1;
    ring_acquire(ring, buf, g >> 1, err);
#pragma unroll
    for (int o = 0; o < NOP; ++o) src_store(src[o], ring.hi(buf, o), ring.lo(buf, o), cur[o]);
    extra(buf, s);
    slice_publish();
    if ((threadIdx.x & 31) == 0 && (threadIdx.x >> 5) < NISS) {
      issue(buf, s, (int)(threadIdx.x >> 5));
      commit(&ring.bars[buf]);
    }
    ++g;
  }
}

// K = 128 pass whose slices are all staged by stage(buf, s) (no prefetched
// sources), with the issue split as in kloop_pf_n.
template <int NISS, class St, class Is>
__device__ __forceinline__ void kloop_n(Ring& ring, int& g, int* err, St stage, Is issue) {
#pragma unroll 1
  for (int s = 0; s < 128 / KS; ++s) {
    const int buf = g & 1;
    ring_acquire(ring, buf, g >> 1, err);
    stage(buf, s);
    slice_publish();
    if ((threadIdx.x & 31) == 0 && (threadIdx.x >> 5) < NISS) {
      issue(buf, s, (int)(threadIdx.x >> 5));
      commit(&ring.bars[buf]);
    }
    ++g;
  }
}

// drain for NISS issuing threads (the barrier has arrival count NISS).
template <int NISS>
__device__ __forceinline__ void drain_n(uint64_t* bar, uint32_t& phase, int* err) {
  if ((threadIdx.x & 31) == 0 && (threadIdx.x >> 5) < NISS) commit(bar);
  mbar_wait(bar, phase, err);
  phase ^= 1;
  fence_after_sync();
}

struct NoExtra {
  __device__ __forceinline__ void operator()(int, int) const {}
};

// Wait for every MMA issued so far (commit to `bar`, then all threads wait).
__device__ __forceinline__ void drain(uint64_t* bar, uint32_t& phase, int* err) {
  if (threadIdx.x == 0) commit(bar);
  mbar_wait(bar, phase, err);
  phase ^= 1;
  fence_after_sync();
}

// This thread's share of a 128 x N accumulator: warp w owns lanes 32*(w%4)..
// and the column half w/4.  fn(row, col, v[16]) for each 16 columns.
template <int N, class Fn>
__device__ __forceinline__ void for_acc(uint32_t tmem, int col0, Fn fn) {
  const int warp = threadIdx.x >> 5;
  const int row = 32 * (warp & 3) + (threadIdx.x & 31);
  const int half = warp >> 2;
#pragma unroll 1
  for (int c = half * (N / 2); c < (half + 1) * (N / 2); c += 16) {
    float v[16];
    tmem_ld16(lane_quarter_addr(tmem, col0 + c), v);
    fn(row, c, v);
  }
}

// Epilogue staging through shared memory: a 128 x 128 accumulator copied
// to a padded row-major tile (ld = TLD) so the global reads and writes of the
// epilogue can be coalesced.  TRANS stores the transpose (tile[c][r]).
constexpr int TLD = 132;
constexpr int TILE_FLOATS = 128 * TLD;
template <bool TRANS>
__device__ __forceinline__ void acc_to_smem(uint32_t tmem, int col0, float* t) {
  for_acc<128>(tmem, col0, [&](int row, int c, const float* v) {
    if (!TRANS) {
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(t + row * TLD + c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) t[(c + j) * TLD + row] = v[j];
    }
  });
}
// fn(r, c) for every row r < 128 and column group c = 0, 4, ..., 124; a warp
// covers one row, so global accesses at (r, c..c+3) are coalesced.
template <class F>
__device__ __forceinline__ void for_tile(F fn) {
#pragma unroll 4
  for (int it = 0; it < 128 * 32 / kThreads; ++it) {
    const int e = threadIdx.x + it * kThreads;
    fn(e >> 5, (e & 31) * 4);
  }
}

}  // namespace tc
}  // namespace gdn2
