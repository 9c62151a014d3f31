// Tensor-core (tcgen05, 3xTF32) intra-chunk forward of the chunk = head dim =
// 128 path: reference Kernels A, B, C (gdn2_fwd.py:99-139, 173-260, 263-330).
// Same workspace contract as k_fwd_intra (gdn2_fwd.cu).
//
// Chunk scores.  Aqk(i,j) = scale sum_d q_id k_jd e^{gc_id - gc_jd} for j <= i
// (Akk likewise with b k on the left, j < i).  For the column block J of JW
// columns (JW = 64, or 32 when a 64-row spread of gc exceeds 80) with first
// row r = JW J:
//     e^{gc_i - gc_j} = e^{gc_i - gc_r} e^{gc_r - gc_j},
// so block J is one product of A_J(i) = x_i e^{gc_i - gc_r} (rows i >= r, every
// factor <= 1 for g <= 0) and B_J(j) = k_j e^{gc_r - gc_j} (j inside block J,
// factor <= e^{spread of the block}).  A chunk whose g has a positive entry,
// or whose 32-row spread of gc exceeds 80 (the factor could leave the float
// range), takes the exact elementwise form with the reference's +-20 clip; for
// g <= 0 the clip at -20 changes a term by < e^-20.
#include "gdn2_kernels.cuh"
#include "gdn2_tc_stage.cuh"

// Optional per-phase cycle counts of one CTA (build with -DGDN2_PHASE_TIMING;
// the counts are printed by that CTA).  Compiled out otherwise.
#ifdef GDN2_PHASE_TIMING
#include <cstdio>
#define GDN2_TMARK(i) \
  do { if (blockIdx.x == gridDim.x / 2 && threadIdx.x == 0) tmark[i] = clock64(); } while (0)
#else
#define GDN2_TMARK(i) do { } while (0)
#endif

namespace gdn2 {

using namespace tc;

namespace {

constexpr int C = 128, D = 128;
constexpr int GLD = D + 4;   // row stride of the resident gc tile (conflict-free row reads)
// threads issuing MMAs: lane 0 of warps 0 .. kIss-1, one accumulator each
#ifndef GDN2_FWD_ISS
#define GDN2_FWD_ISS 2
#endif
constexpr int kIss = GDN2_FWD_ISS;

struct TcSmemF {
  float rowl1[C];   // sum_d |kg(i, d)| per row i
  uint64_t bars[2];
  uint64_t done;
  uint32_t tmem;
};

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void sts4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

}  // namespace

template <typename T, bool DIAG, bool GATES>
__global__ void __launch_bounds__(kThreads, 1)
k_tc_fwd_intra(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               const T* __restrict__ w, const T* __restrict__ b, const T* __restrict__ g,
               Problem p, Workspace ws) {
  extern __shared__ __align__(128) float sm[];
  __shared__ __align__(16) TcSmemF ts;
#ifdef GDN2_PHASE_TIMING
  long long tmark[16];
#endif
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const int h = (int)(bh % p.H), bb = (int)(bh / p.H);
  const long rs = p.row_stride();
  const long off = ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const T *qc = q + off, *kc = k + off, *vc = v + off, *wc = w + off, *bc = b + off,
          *gcp = g + off;
  // shared memory plan (floats): gc stays in [0, C * GLD) through phase 3; the
  // score ring, then the transposed score tiles and the solve, follow it;
  // phase 3 puts its ring after gc (A itself moves to TMEM).
  float* sgc = sm;                                 // [C][GLD]
  float* red = sm + C * GLD;                       // phase-0 reduction scratch (256 floats)
  float* ringA = sm + C * GLD;                     // 2 buffers x 2 operands x slice
  float* bsl = ringA + 2 * 2 * 2 * SLICE_FLOATS;   // 2 buffers x (hi, lo) x 64 x 32
  float* t0 = sm + C * GLD;                        // after the score products
  float* S = t0 + TILE_FLOATS;
  float* tmp = S + TILE_FLOATS;                    // 4096 floats

  if ((threadIdx.x >> 5) == 0) tmem_alloc(&ts.tmem, 512);
  if (threadIdx.x < C) ts.rowl1[threadIdx.x] = 0.f;
  if (threadIdx.x == 0) {
    mbar_init(&ts.bars[0], kIss);
    mbar_init(&ts.bars[1], kIss);
    mbar_init(&ts.done, kIss);
    fence_mbar_init();
  }

  GDN2_TMARK(0);
  StageDiag dkg, dqg, dsc;   // stage diagnostics (p.diag only)
  // ---- phase 0: gc = in-chunk cumsum of g (gdn2_fwd.py:105-107), kg, qg
#pragma unroll 8
  for (int it = 0; it < C * D / 4 / kThreads; ++it) {
    const int e = threadIdx.x + it * kThreads;
    const int r = e >> 5, cc = (e & 31) * 4;
    sts4(sgc + r * GLD + cc, ld4_gate<T>(gcp + r * rs + cc, GATES, kGateG));
  }
  // k and q for the kg / qg pass, four iterations per batch: the first batch
  // is in flight during the cumsum, each later one during the batch before
  auto kq_at = [&](int it, int& i, int& d) {
    const int e = threadIdx.x + it * kThreads;
    const int l = e & 31, wq = e >> 5;
    i = (wq & 31) * 4 + (l >> 3);
    d = ((wq >> 5) * 8 + (l & 7)) * 4;
  };
  float4 kcur[4], qcur[4], knx[4], qnx[4];
  auto ld_kq = [&](int bt, float4* kx, float4* qx) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      int i, d;
      kq_at(4 * bt + u, i, d);
      kx[u] = ld4<T>(kc + i * rs + d);
      qx[u] = ld4<T>(qc + i * rs + d);
    }
  };
  ld_kq(0, kcur, qcur);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  GDN2_TMARK(8);
  const uint32_t tmem = ts.tmem;
  float gpos = -1.f;
  for (int e = threadIdx.x; e < C * D; e += kThreads) gpos = fmaxf(gpos, sgc[(e / D) * GLD + e % D]);
  const float gmax = block_max(gpos, red);
  GDN2_TMARK(9);
  // chunk-local gc: with two 64-row chunks per tile the cumsum restarts at row 64
  column_cumsum<C, D, GLD>(sgc, red, p.sub == 2);
  const int R = C / p.sub;   // rows of one reference chunk
  // bit tests instead of divisions by R: rows i, j are in one chunk iff
  // ((i ^ j) & cm) == 0, and i | lm is the last row of i's chunk
  const int cm = p.sub == 2 ? 64 : 0, lm = R - 1;
  GDN2_TMARK(10);
  // largest decay-block width (64 or 32 rows) whose in-block gc spread keeps
  // every factor e^{gc_r - gc_j} inside the float range
  float spread = 0.f, spread64 = 0.f;
  for (int e = threadIdx.x; e < 4 * D; e += kThreads) {
    const int J = e / D, d = e % D;
    spread = fmaxf(spread, fabsf(sgc[(32 * J) * GLD + d] - sgc[(32 * J + 31) * GLD + d]));
    if (J < 2) spread64 = fmaxf(spread64, fabsf(sgc[(64 * J) * GLD + d] - sgc[(64 * J + 63) * GLD + d]));
  }
  const bool exact = gmax > 0.f || block_max(spread, red) > 80.f || spread != spread;
  const int JW = block_max(spread64, red) <= 80.f ? 64 : 32;
  GDN2_TMARK(11);
  {
    float* gco = ws.gc + chunk * C * D;
    for (int e = threadIdx.x * 4; e < C * D; e += kThreads * 4)
      sts4(gco + e, lds4(sgc + (e / D) * GLD + e % D));
    GDN2_TMARK(12);
    for (int e = threadIdx.x; e < p.sub * D; e += kThreads)
      ws.gcl[chunk * p.sub * D + e] = san(sgc[((e / D) * R + R - 1) * GLD + e % D], p.clip);
    float* kgo = ws.kg + chunk * C * D;
    // qg is staged transposed with an odd row stride; a warp covers 4 rows x 32
    // columns, so the transposed scalar stores hit 32 distinct banks and the
    // global rows are read in 128-byte pieces.
    constexpr int QLD = C + 1;
    float* tq = sm + C * GLD;   // free until the score products start
#pragma unroll 1
    for (int bt = 0; bt < C * D / 16 / kThreads; ++bt) {
    if (bt + 1 < C * D / 16 / kThreads) ld_kq(bt + 1, knx, qnx);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int l = threadIdx.x & 31;
      int i, d;
      kq_at(4 * bt + u, i, d);
      const float4 kv = kcur[u], qv = qcur[u];
      const float4 gi = lds4(sgc + i * GLD + d), l4 = lds4(sgc + (i | lm) * GLD + d);
      const float4 kg4 = make_float4(san(kv.x * __expf(l4.x - gi.x), p.clip),
                                     san(kv.y * __expf(l4.y - gi.y), p.clip),
                                     san(kv.z * __expf(l4.z - gi.z), p.clip),
                                     san(kv.w * __expf(l4.w - gi.w), p.clip));
      sts4(kgo + i * D + d, kg4);
      if (DIAG) dkg.add4(kg4);
      // row L1 norm of kg: the 8 lanes sharing row i cover 32 columns
      float l1 = fabsf(kg4.x) + fabsf(kg4.y) + fabsf(kg4.z) + fabsf(kg4.w);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 4);
      if ((l & 7) == 0) atomicAdd(&ts.rowl1[i], l1);
      tq[(d + 0) * QLD + i] = san(qv.x * __expf(gi.x), p.clip);
      tq[(d + 1) * QLD + i] = san(qv.y * __expf(gi.y), p.clip);
      tq[(d + 2) * QLD + i] = san(qv.z * __expf(gi.z), p.clip);
      tq[(d + 3) * QLD + i] = san(qv.w * __expf(gi.w), p.clip);
      if (DIAG)
        dqg.add4(make_float4(tq[(d + 0) * QLD + i], tq[(d + 1) * QLD + i], tq[(d + 2) * QLD + i],
                             tq[(d + 3) * QLD + i]));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      kcur[u] = knx[u];
      qcur[u] = qnx[u];
    }
    }
    __syncthreads();
    GDN2_TMARK(13);
    float* qgo = ws.qgT + chunk * C * D;
#pragma unroll 8
    for (int it = 0; it < C * D / kThreads; ++it) {
      const int e = threadIdx.x + it * kThreads;
      qgo[e] = tq[(e >> 7) * QLD + (e & 127)];
    }
    __syncthreads();
    if (DIAG) {
      dkg.flush(ws.status, kDiagKg);
      dqg.flush(ws.status, kDiagQg);
    }
    // max_i ||kg_i||_1, the gain of dv_new's kg dh term (backward guard)
    for (int hf = 0; hf < p.sub; ++hf) {
      const bool mine = threadIdx.x >= hf * R && threadIdx.x < (hf + 1) * R;
      const float kl1 = block_max(mine ? ts.rowl1[threadIdx.x] : 0.f, red);
      if (threadIdx.x == 0) ws.bnd[(chunk * p.sub + hf) * 4] = kl1;
    }
  }

  GDN2_TMARK(1);
  Ring ring;
  ring.base = ringA;
  ring.bars = ts.bars;
  ring.phase[0] = ring.phase[1] = 0;
  ring.nop = 2;
  int gs = 0;
  uint32_t ph = 0;
  float* aqkT = ws.AqkT + chunk * C * C;
  if (!exact) {
    // ---- phase 1: scores.  Outer loop over 32-wide slices of d (q, k, b of
    // the slice held in registers, the next slice prefetched), inner loop
    // over the column blocks J of width JW (N = JW products: one tcgen05.mma
    // costs about the same pipe time for N = 32 and 64, so wider blocks
    // halve both the MMAs and the staging of the row operands).
    float4 qa[4], ka[4], ba[4], qn[4], kn[4], bn[4];
    auto rc_of = [&](int it, int& i, int& cc) {
      const int e = threadIdx.x + it * kThreads;
      const int lane = e & 31, wq = e >> 5;
      i = (wq & 15) * 8 + (lane & 7);
      cc = ((wq >> 4) * 4 + (lane >> 3)) * 4;
    };
    auto load_qkb = [&](int s, float4* qx, float4* kx, float4* bx) {
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        int i, cc;
        rc_of(it, i, cc);
        const int d = s * KS + cc;
        qx[it] = ld4<T>(qc + i * rs + d);
        kx[it] = ld4<T>(kc + i * rs + d);
        bx[it] = ld4_gate<T>(bc + i * rs + d, GATES, kGateB);
      }
    };
    load_qkb(0, qa, ka, ba);
    // rolled slice loop (instruction-cache friendly); the prefetched slice is
    // copied into the current registers at the end of each step
#pragma unroll 1
    for (int s = 0; s < D / KS; ++s) {
      const float4* qx = qa;
      const float4* kx = ka;
      const float4* bx = ba;
      if (s + 1 < D / KS) load_qkb(s + 1, qn, kn, bn);
#pragma unroll 1
      for (int J = 0; J < C / JW; ++J, ++gs) {
        const int r = JW * J;
        const int buf = gs & 1;
        ring_acquire(ring, buf, gs >> 1, ws.status);
        float* bhi = bsl + buf * 2 * 64 * KS;
        float* blo = bhi + 64 * KS;
        // Both operands from the slice already in registers: the row operands
        // for rows i >= r, and the column operand B_J(i - r) = k_i e^{gc_r - gc_i}
        // for the rows i of block J (the same elements, so no second load).
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          int i, cc;
          rc_of(it, i, cc);
          const int d = s * KS + cc;
          float4 aq = make_float4(0.f, 0.f, 0.f, 0.f), ak = aq;
          // rows of the column block's own chunk only (block-diagonal when
          // the tile holds two chunks)
          if (i >= r && ((i ^ r) & cm) == 0) {
            const float4 gi = lds4(sgc + i * GLD + d), gr = lds4(sgc + r * GLD + d);
            const float e0 = __expf(gi.x - gr.x), e1 = __expf(gi.y - gr.y),
                        e2 = __expf(gi.z - gr.z), e3 = __expf(gi.w - gr.w);
            const float4 qv = qx[it], kv = kx[it], bv = bx[it];
            aq = make_float4(qv.x * e0, qv.y * e1, qv.z * e2, qv.w * e3);
            ak = make_float4(bv.x * kv.x * e0, bv.y * kv.y * e1, bv.z * kv.z * e2, bv.w * kv.w * e3);
            if (i < r + JW)
              st_split4(bhi, blo, i - r, cc, KS,
                        make_float4(kv.x * __expf(gr.x - gi.x), kv.y * __expf(gr.y - gi.y),
                                    kv.z * __expf(gr.z - gi.z), kv.w * __expf(gr.w - gi.w)));
          }
          st_split4(ring.hi(buf, 0), ring.lo(buf, 0), i, cc, KS, aq);
          st_split4(ring.hi(buf, 1), ring.lo(buf, 1), i, cc, KS, ak);
        }
        slice_publish();
        if ((threadIdx.x & 31) == 0 && (threadIdx.x >> 5) < kIss) {
          const Opnd B = kmajor(bhi, blo, KS);
          const int who = threadIdx.x >> 5;
          if (who == 0) mma3(tmem + r, ring.op(buf, 0), B, JW, KS / 8, s > 0);
          if (who == kIss - 1) mma3(tmem + 128 + r, ring.op(buf, 1), B, JW, KS / 8, s > 0);
          commit(&ring.bars[buf]);
        }
      }
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        qa[it] = qn[it];
        ka[it] = kn[it];
        ba[it] = bn[it];
      }
    }
  GDN2_TMARK(2);
    drain_n<kIss>(&ts.done, ph, ws.status);
    // straight from TMEM (lane = row i): for each column j a warp's stores are
    // 32 consecutive i, coalesced in global memory and conflict-free in S
    for_acc<128>(tmem, 0, [&](int i, int c, const float* v) {   // Aqk / scale
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        aqkT[(c + t) * C + i] = c + t <= i && (((c + t) ^ i) & cm) == 0 ? san(p.scale * v[t], p.clip) : 0.f;
        if (DIAG) dsc.add(aqkT[(c + t) * C + i]);
      }
    });
    if (DIAG) dsc.flush(ws.status, kDiagAqk);
    for_acc<128>(tmem, 128, [&](int i, int c, const float* v) {   // S[j][i] = Akk(i, j)
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        S[(c + t) * TLD + i] = c + t < i && (((c + t) ^ i) & cm) == 0 ? san(v[t], p.clip) : 0.f;
        if (DIAG) dsc.add(S[(c + t) * TLD + i]);
      }
    });
    if (DIAG) dsc.flush(ws.status, kDiagAkk);
  } else {
    // exact elementwise form with the +-20 exponent clip (gdn2_fwd.py:124-139)
    for (int e = threadIdx.x; e < C * C; e += kThreads) {
      const int i = e % C, j = e / C;
      const bool pair = j <= i && ((j ^ i) & cm) == 0;   // same chunk, causal
      float sq = 0.f, sk = 0.f;
      if (pair) {
        for (int d = 0; d < D; ++d) {
          const float ed = __expf(fminf(fmaxf(sgc[i * GLD + d] - sgc[j * GLD + d], -20.f), 20.f));
          const float kj = to_f<T>(kc[j * rs + d]) * ed;
          sq = fmaf(to_f<T>(qc[i * rs + d]), kj, sq);
          sk = fmaf(ld_gate<T>(bc + i * rs + d, GATES, kGateB) * to_f<T>(kc[i * rs + d]), kj, sk);
        }
      }
      aqkT[j * C + i] = pair ? san(p.scale * sq, p.clip) : 0.f;
      S[j * TLD + i] = (pair && j < i) ? san(sk, p.clip) : 0.f;
      if (DIAG) {
        dsc.add(aqkT[j * C + i]);
        dqg.add(S[j * TLD + i]);   // (dqg reused as the Akk accumulator here)
      }
    }
    if (DIAG) {
      dsc.flush(ws.status, kDiagAqk);
      dqg.flush(ws.status, kDiagAkk);
    }
  }
  __syncthreads();

  GDN2_TMARK(3);
  // ---- phase 2: A = (I + Akk)^-1 on the transpose (gdn2_fwd.py:173-260)
  wy_inverse_T128(S, TLD, tmp, t0, p.bc, p.clip, R);
  GDN2_TMARK(4);
  float* at = ws.AT + chunk * C * C;
  for_tile([&](int j, int i) {
    const float4 a4 = lds4(S + j * TLD + i);
    sts4(at + j * C + i, a4);
    if (DIAG) dsc.add4(a4);
  });
  if (DIAG) dsc.flush(ws.status, kDiagA);
  {
    // A (rows i, K = j) split into hi (TMEM 256..383) and lo (384..511): the A
    // operand of phase 3.  S[j * TLD + i] = A(i, j), one TMEM lane per row i.
    const int warp = threadIdx.x >> 5;
    const int row = 32 * (warp & 3) + (threadIdx.x & 31), half = warp >> 2;
#pragma unroll 1
    for (int c = half * 64; c < half * 64 + 64; c += 16) {
      float hv[16], lv[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) split(S[(c + t) * TLD + row], hv[t], lv[t]);
      tmem_st16(lane_quarter_addr(tmem, 256 + c), hv);
      tmem_st16(lane_quarter_addr(tmem, 384 + c), lv);
    }
    tmem_st_wait();
  }
  fence_before_sync();
  __syncthreads();   // A in TMEM; smem past the gc tile reusable
  fence_after_sync();

  GDN2_TMARK(5);
  // ---- phase 3: W = A (b k e^gc), U = A (w v)  (gdn2_fwd.py:278-282)
  ring.base = sm + C * GLD;   // after the gc tile
  ring.nop = 2;
  {
    // b, k, w, v rows of the next slice are loaded while the current slice is
    // stored and issued.
    Frag fb, fk, fw, fv;
    const int rb = (threadIdx.x & 7) + ((threadIdx.x >> 5) & 3) * 8;
    const int kb4 = ((threadIdx.x >> 3) & 3) + (threadIdx.x >> 7) * 4;
    auto ld_rows = [&](int sl) {
#pragma unroll
      for (int jr = 0; jr < 4; ++jr) {
        const int j = sl * KS + kb4 * 4 + jr, d = rb * 4;
        fb.v[jr] = ld4_gate<T>(bc + j * rs + d, GATES, kGateB);
        fk.v[jr] = ld4<T>(kc + j * rs + d);
        fw.v[jr] = ld4_gate<T>(wc + j * rs + d, GATES, kGateW);
        fv.v[jr] = ld4<T>(vc + j * rs + d);
      }
    };
    ld_rows(0);
    kloop_n<kIss>(ring, gs, ws.status,
             [&](int buf, int s) {
               Frag kbf, wv;
#pragma unroll
               for (int jr = 0; jr < 4; ++jr) {
                 const int j = s * KS + kb4 * 4 + jr;
                 const float4 bv = fb.v[jr], kv = fk.v[jr], g4 = lds4(sgc + j * GLD + rb * 4),
                              w4 = fw.v[jr], v4 = fv.v[jr];
                 kbf.v[jr] = make_float4(bv.x * kv.x * __expf(g4.x), bv.y * kv.y * __expf(g4.y),
                                         bv.z * kv.z * __expf(g4.z), bv.w * kv.w * __expf(g4.w));
                 wv.v[jr] = make_float4(w4.x * v4.x, w4.y * v4.y, w4.z * v4.z, w4.w * v4.w);
               }
               if (s + 1 < C / KS) ld_rows(s + 1);
               store_trans(ring.hi(buf, 0), ring.lo(buf, 0), kbf);  // (d, j) = kb(j, d)
               store_trans(ring.hi(buf, 1), ring.lo(buf, 1), wv);   // (v, j) = wv(j, v)
             },
             [&](int buf, int s, int who) {
               const uint32_t ah = tmem + 256 + s * KS, al = tmem + 384 + s * KS;
               if (who == 0) mma3_ta(tmem, ah, al, ring.op(buf, 0), 128, KS / 8, s > 0);
               if (who == kIss - 1) mma3_ta(tmem + 128, ah, al, ring.op(buf, 1), 128, KS / 8, s > 0);
             });
  }
  GDN2_TMARK(6);
  drain_n<kIss>(&ts.done, ph, ws.status);
  float* wt = ws.WT + chunk * C * D;
  float* uo = ws.U + chunk * C * D;
  for_acc<128>(tmem, 0, [&](int i, int c, const float* v) {     // W^T, coalesced per column
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      wt[(c + t) * C + i] = san(v[t], p.clip);
      if (DIAG) dsc.add(san(v[t], p.clip));
    }
  });
  if (DIAG) dsc.flush(ws.status, kDiagW);
  for_acc<128>(tmem, 128, [&](int i, int c, const float* v) {   // U, one row per lane
#pragma unroll
    for (int t = 0; t < 16; t += 4) {
      const float4 u4 = make_float4(san(v[t], p.clip), san(v[t + 1], p.clip),
                                    san(v[t + 2], p.clip), san(v[t + 3], p.clip));
      sts4(uo + i * D + c + t, u4);
      if (DIAG) dsc.add4(u4);
    }
  });
  if (DIAG) dsc.flush(ws.status, kDiagU);
  GDN2_TMARK(7);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if ((threadIdx.x >> 5) == 0) tmem_free(tmem, 512);
#ifdef GDN2_PHASE_TIMING
  if (blockIdx.x == gridDim.x / 2 && threadIdx.x == 0)
    printf("fwd_intra phases: %lld %lld %lld %lld %lld %lld %lld | p0: %lld %lld %lld %lld %lld %lld %lld\n",
           tmark[1] - tmark[0], tmark[2] - tmark[1], tmark[3] - tmark[2], tmark[4] - tmark[3],
           tmark[5] - tmark[4], tmark[6] - tmark[5], tmark[7] - tmark[6], tmark[8] - tmark[0],
           tmark[9] - tmark[8], tmark[10] - tmark[9], tmark[11] - tmark[10],
           tmark[12] - tmark[11], tmark[13] - tmark[12], tmark[1] - tmark[13]);
#endif
}

template <typename T>
cudaError_t launch_tc_fwd_intra(const T* q, const T* k, const T* v, const T* w, const T* b,
                                const T* g, const Problem& p, const Workspace& ws, cudaStream_t s) {
  constexpr size_t smem_rest = (size_t)(C * GLD + 2 * TILE_FLOATS + 4096) * sizeof(float);
  constexpr size_t smem_scores = (size_t)(C * GLD + 4 * SLICE_FLOATS * 2 + 4 * 64 * KS) * sizeof(float);
  constexpr size_t smem = smem_rest > smem_scores ? smem_rest : smem_scores;
  static_assert(smem >= (size_t)(C * GLD + 4 * SLICE_FLOATS * 2 + 4 * 64 * KS) * sizeof(float),
                "score ring fits");
  static_assert(smem >= (size_t)C * GLD * sizeof(float) + 2 * 2 * (size_t)SLICE_BYTES,
                "phase-3 ring fits after the gc tile");
  // per-stage diagnostics are compiled into a second instance of the kernel
  auto kern = p.diag ? (p.gates ? k_tc_fwd_intra<T, true, true> : k_tc_fwd_intra<T, true, false>)
                     : (p.gates ? k_tc_fwd_intra<T, false, true> : k_tc_fwd_intra<T, false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)p.B * p.H * p.nc, kThreads, smem, s>>>(q, k, v, w, b, g, p, ws);
  return cudaGetLastError();
}

template cudaError_t launch_tc_fwd_intra<float>(const float*, const float*, const float*,
                                                const float*, const float*, const float*,
                                                const Problem&, const Workspace&, cudaStream_t);
template cudaError_t launch_tc_fwd_intra<__nv_bfloat16>(
    const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
    const __nv_bfloat16*, const __nv_bfloat16*, const Problem&, const Workspace&, cudaStream_t);

}  // namespace gdn2
