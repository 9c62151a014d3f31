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
// vnew = U - W h and dv_new = san(dv_partial + kg dh_next) (formed in the
// backward intra kernel) are chunk-parallel again.  Sanitisers sit where the
// reference has them (h and dh after every chunk, o, dv_partial, dv_new).
#include "gdn2_kernels.cuh"
#include "gdn2_tc_stage.cuh"

namespace gdn2 {

using namespace tc;

namespace {

struct TcSmem {
  float red[8];
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
template <int SUB>   // reference chunks per tile (p.sub)
__global__ void __launch_bounds__(kThreads, 1) k_tc_affine(Problem p, Workspace ws) {
  extern __shared__ __align__(128) float sm[];
  __shared__ TcSmem ts;
  const size_t chunk = blockIdx.x;
  const uint32_t tmem = tc_setup(&ts, 512);
  Ring ring = make_ring(sm, &ts, 3);
  const float* kg = ws.kg + chunk * C * D;
  const float* wt = ws.WT + chunk * C * D;
  const float* u = ws.U + chunk * C * D;
  int g = 0;
  uint32_t ph = 0;
  // one map per reference chunk: K = its rows (all 128, or 64 per chunk of a
  // paired tile)
  constexpr int R = C / SUB;
#pragma unroll 1
  for (int hf = 0; hf < SUB; ++hf) {
    const int r0 = hf * R;
    const Src srcs[3] = {trans(kg + r0 * D, D), direct(wt + r0, C), trans(u + r0 * D, D)};   // (d,i)=kg, (d',i)=W, (v,i)=U
    auto issue = [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 0), ring.op(buf, 1), 128, KS / 8, s > 0);         // kg^T W
      mma3(tmem + 128, ring.op(buf, 0), ring.op(buf, 2), 128, KS / 8, s > 0);   // kg^T U
      mma3(tmem + 256, ring.op(buf, 1), ring.op(buf, 0), 128, KS / 8, s > 0);   // (kg^T W)^T
    };
    kloop_pf<false, 4 / SUB>(ring, g, ws.status, srcs, NoExtra{}, issue);
    drain(&ts.done, ph, ws.status);
    // M and M^T leave TMEM row by row as the canonical K-slices the scan
    // streams with bulk copies (row = TMEM lane, K = column); the scan forms
    // the lo planes itself (the tensor core reads a float32 word as its tf32
    // head).
    const size_t sc = chunk * SUB + hf;   // reference chunk
    float* bo = ws.Bc + sc * D * D;
    const float* gl = ws.gcl + sc * D;
#pragma unroll 1
    for (int orient = 0; orient < 2; ++orient) {
      float* mo = ws.M + sc * 2 * D * D + (size_t)orient * D * D;
      for_acc<128>(tmem, orient ? 256 : 0, [&](int row, int c, const float* v) {
        const float dec = __expf(gl[row]);
        float* sl = mo + (c / KS) * SLICE_FLOATS;
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
          float4 o = make_float4(-v[j], -v[j + 1], -v[j + 2], -v[j + 3]);
          if (row == c + j) o.x += dec;
          if (row == c + j + 1) o.y += dec;
          if (row == c + j + 2) o.z += dec;
          if (row == c + j + 3) o.w += dec;
          st4f(sl + canon_off(row, c % KS + j, KS) / 4, o);
        }
      });
    }
    for_acc<128>(tmem, 128, [&](int row, int c, const float* v) {
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        st4f(bo + row * D + c + j, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
    });
    if (hf + 1 < SUB) {   // every thread's TMEM reads complete before the next chunk's MMAs
      fence_before_sync();
      __syncthreads();
      fence_after_sync();
    }
  }
  tc_teardown(tmem, 512);
}

// ---------------------------------------------------------------------------
// Serial affine scan over the chunks of one (batch, head).  The state is kept
// transposed (rows = value column v, cols = key dim d) in TMEM as the A operand:
//   forward:  h_{c+1}^T = h_c^T M_c^T + Bc_c^T   (state entering every chunk -> ws.hpre)
//   backward: dh_c^T    = dh_{c+1}^T M_c + E_c^T (dh_pre of every chunk -> ws.dh)
// The B operand (M, or M^T backward) arrives from k_tc_affine as four 16 KB
// canonical K-slices per chunk, streamed by bulk copies through a ring of
// kScanSlots slots (1.5 chunks ahead); the constant term (Bc, or E backward)
// lands in shared memory by one bulk copy a step ahead of its use.  The raw
// float32 slice is the hi plane; each step first forms the four lo planes (x - tf32(x)) in shared memory, then
// issues one 128 x 128 x 128 3xTF32 product; the epilogue adds the constant
// term, sanitises, stores the state and writes it back to TMEM as hi / lo.
// ---------------------------------------------------------------------------
// PROD (forward only) instead accumulates the segment map P = M_last ... M_first
// from P = I with no constant term and no sanitiser, writing only P to
// out_final (sequence parallelism).
constexpr int kScanSlots = 6;
constexpr int kScanSliceBytes = SLICE_FLOATS * 4;   // one plane of one slice
struct ScanSmem {
  float wmax[2][8];   // per-warp max |state|, double-buffered by step parity
  uint64_t full[kScanSlots];
  uint64_t addfull;    // the step's constant term landed in shared memory
  uint64_t done;
  uint32_t tmem;
};

template <bool BWD, bool PROD = false>
__global__ void __launch_bounds__(kThreads, 1)
k_tc_scan(Problem p, Workspace ws, const float* __restrict__ init, float* __restrict__ out_final) {
  // shared memory: kScanSlots raw slices, the 4 lo planes of the step, the
  // step's constant term
  extern __shared__ __align__(128) float sm[];
  __shared__ ScanSmem ts;
  float* lo = sm + kScanSlots * SLICE_FLOATS;
  float* addt = lo + 4 * SLICE_FLOATS;   // the step's constant term (Bc or E), D x D
  const int h = blockIdx.x, bb = blockIdx.y;
  const size_t bh = (size_t)bb * p.H + h;
  // TMEM: accumulator [0, 128), state hi [128, 256), state lo [256, 384)
  if ((threadIdx.x >> 5) == 0) tmem_alloc(&ts.tmem, 512);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kScanSlots; ++i) mbar_init(&ts.full[i], 1);
    mbar_init(&ts.addfull, 1);
    mbar_init(&ts.done, 1);
    fence_mbar_init();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = ts.tmem;
  const int ncs = p.ncs();          // state steps: one per reference chunk
  const int nt = ncs * (D / KS);   // slices over the whole scan
  auto issue = [&](int t) {          // thread 0 only
    const int it = t / (D / KS), s = t % (D / KS);
    const int c = BWD ? ncs - 1 - it : it;
    const float* src = ws.M + (bh * ncs + c) * 2 * D * D + (BWD ? D * D : 0) + s * SLICE_FLOATS;
    const int slot = t % kScanSlots;
    mbar_arrive_expect_tx(&ts.full[slot], kScanSliceBytes);
    bulk_g2s(sm + slot * SLICE_FLOATS, src, kScanSliceBytes, &ts.full[slot]);
  };
  // the constant term of step `it`, one bulk copy a step ahead of its use
  auto issue_add = [&](int it) {   // thread 0 only
    const int c = BWD ? ncs - 1 - it : it;
    mbar_arrive_expect_tx(&ts.addfull, D * D * 4);
    bulk_g2s(addt, (BWD ? ws.E : ws.Bc) + (bh * ncs + c) * D * D, D * D * 4, &ts.addfull);
  };
  if (threadIdx.x == 0) {
    for (int t = 0; t < kScanSlots && t < nt; ++t) issue(t);
    if (!PROD) issue_add(0);
  }

  const int warp = threadIdx.x >> 5;
  const int vrow = 32 * (warp & 3) + (threadIdx.x & 31);
  const int dcol0 = (warp >> 2) * 64;
  // initial state (transposed): PROD -> I, else san(init) or 0
  const float* src0 = init ? init + bh * D * D : nullptr;
  if (!BWD && !PROD) {
    float* hp = ws.hpre + (bh * ncs) * D * D;
    for (int e = threadIdx.x; e < D * D; e += kThreads) hp[e] = src0 ? san(src0[e], p.clip) : 0.f;
  }
  // Backward guard.  The affine step replaces the reference's
  // dv_new = san(dv_partial + kg dh) by the unclipped sum, which is the same
  // value while |dv_partial + kg dh| <= CLIP.  That holds whenever
  // max|dv_partial| + max_i ||kg_i||_1 max|dh| < CLIP (ws.bnd); a (b, h) whose
  // chain fails the test anywhere is flagged and recomputed by the exact
  // reference step (k_bwd_state).  smax = this thread's max |state|.
  constexpr bool kGuard = BWD && !PROD;
  float smax = 0.f;
  bool flagged = false;
  bool clipped = false;   // the state sanitiser acted (reported for sequence parallelism)
  StageDiag dhf;          // h_final diagnostics (forward, p.diag only)
#pragma unroll 1
  for (int q = 0; q < 4; ++q) {
    const int c0 = dcol0 + q * 16;
    float hv[16], lv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float x = PROD ? (vrow == c0 + j ? 1.f : 0.f)
                           : (src0 ? san(src0[(c0 + j) * D + vrow], p.clip) : 0.f);
      smax = fmaxf(smax, fabsf(x));
      split(x, hv[j], lv[j]);
    }
    tmem_st16(lane_quarter_addr(tmem, 128 + c0), hv);
    tmem_st16(lane_quarter_addr(tmem, 256 + c0), lv);
  }
  tmem_st_wait();
  auto publish_max = [&](int parity) {
    float m = smax;
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) ts.wmax[parity][warp] = m;
  };
  if (kGuard) publish_max(0);

  uint32_t ph = 0;
  float addv[64];
  for (int it = 0; it < ncs; ++it) {
    const int c = BWD ? ncs - 1 - it : it;
    const size_t chunk = bh * ncs + c;
    if (!PROD) {   // this thread's share of the constant term (row v, 64 columns d)
      mbar_wait(&ts.addfull, (uint32_t)(it & 1), ws.status);
#pragma unroll
      for (int j = 0; j < 64; ++j) addv[j] = addt[(dcol0 + j) * D + vrow];
    }
    // lo planes of this step's four slices
#pragma unroll 1
    for (int s = 0; s < D / KS; ++s) {
      const int t = it * (D / KS) + s, slot = t % kScanSlots;
      mbar_wait(&ts.full[slot], (uint32_t)((t / kScanSlots) & 1), ws.status);
      const float4* raw = reinterpret_cast<const float4*>(sm + slot * SLICE_FLOATS);
      float4* lp = reinterpret_cast<float4*>(lo + s * SLICE_FLOATS);
#pragma unroll
      for (int e = threadIdx.x; e < SLICE_FLOATS / 4; e += kThreads) {
        float4 hv, lv;
        split4(raw[e], hv, lv);
        lp[e] = lv;
      }
    }
    fence_async_smem();
    fence_before_sync();
    __syncthreads();   // lo planes and the state in TMEM ready for the MMAs
    fence_after_sync();
    if (threadIdx.x == 0) {
      for (int s = 0; s < D / KS; ++s) {
        const int slot = (it * (D / KS) + s) % kScanSlots;
        const Opnd B = kmajor(sm + slot * SLICE_FLOATS, lo + s * SLICE_FLOATS, KS);
        mma3_ta(tmem, tmem + 128 + s * KS, tmem + 256 + s * KS, B, 128, KS / 8, s > 0);
      }
      commit(&ts.done);
      // every thread read its constant term before the barrier above: the
      // next step's tile may land
      if (!PROD && it + 1 < ncs) {
        fence_async_smem();
        issue_add(it + 1);
      }
    }
    // the guard test of this step runs while its MMAs do (its bound loads are
    // off the issue path)
    if (kGuard) {
      float m = ts.wmax[it & 1][0];
#pragma unroll
      for (int w = 1; w < 8; ++w) m = fmaxf(m, ts.wmax[it & 1][w]);
      float* bd = ws.bnd + chunk * 4;
      // NaN anywhere fails the comparison and flags the chunk
      const bool ok = bd[1] + bd[0] * m < p.clip * (1.f - 1e-5f);
      flagged |= !ok;
      if (threadIdx.x == 0) bd[2] = ok ? 0.f : 1.f;
    }
    mbar_wait(&ts.done, ph, ws.status);
    ph ^= 1;
    fence_after_sync();
    // every MMA of this step is complete: its raw slots can be refilled
    if (threadIdx.x == 0)
      for (int s = 0; s < D / KS; ++s) {
        const int t = it * (D / KS) + s + kScanSlots;
        if (t < nt) issue(t);
      }
    const bool last = it == ncs - 1;
    smax = 0.f;
    float* dst;
    if (PROD) dst = last ? out_final + bh * D * D : nullptr;
    else if (!BWD) dst = last ? (out_final ? out_final + bh * D * D : nullptr) : ws.hpre + (chunk + 1) * D * D;
    else dst = ws.dh + chunk * D * D;
    float xa[64];   // the thread's 64 accumulator columns, one wait
    tmem_ld64(lane_quarter_addr(tmem, dcol0), xa);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c0 = dcol0 + q * 16;
      const float* x = xa + q * 16;
      float hv[16], lv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float pre = x[j] + addv[q * 16 + j];
        const float y = PROD ? x[j] : san(pre, p.clip);
        if (!PROD && !(fabsf(pre) <= p.clip)) clipped = true;
        if (kGuard) smax = fmaxf(smax, fabsf(y));
        if (dst) dst[(c0 + j) * D + vrow] = y;
        if (!BWD && !PROD && last && p.diag) dhf.add(y);
        if (BWD && last && out_final) out_final[bh * D * D + (c0 + j) * D + vrow] = san(y, 1e4f);
        split(y, hv[j], lv[j]);
      }
      tmem_st16(lane_quarter_addr(tmem, 128 + c0), hv);
      tmem_st16(lane_quarter_addr(tmem, 256 + c0), lv);
    }
    tmem_st_wait();
    if (kGuard) publish_max((it + 1) & 1);
  }
  if (kGuard && threadIdx.x == 0) ws.bnd[bh * ncs * 4 + 3] = flagged ? 1.f : 0.f;
  if (clipped) atomicOr(ws.status + (BWD ? 2 : 1), 1);
  if (!BWD && !PROD && p.diag && out_final) dhf.flush(ws.status, kDiagHFinal);
  if (kGuard && flagged && threadIdx.x == 0) atomicOr(ws.status + 3, 1);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if ((threadIdx.x >> 5) == 0) tmem_free(tmem, 512);
}

// ---------------------------------------------------------------------------
// Chunk outputs from the chunk-entry state h (gdn2_fwd.py:349-359):
//   vnew = U - W h  (-> ws.vnew),   o = san(scale qg h + Aqk vnew)  (-> o)
// ---------------------------------------------------------------------------
template <int SUB>
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
  int g = 0;
  // one K loop per reference chunk of the tile, each with that chunk's entry
  // state and the other chunk's rows of W and qg masked (paired tiles)
  constexpr int R = C / SUB;
#pragma unroll 1
  for (int hf = 0; hf < SUB; ++hf) {
    const float* hp = ws.hpre + (chunk * SUB + hf) * D * D;
    const int lo = hf * R, hi = lo + R;
    const Src srcs[3] = {rows(trans(wt, C), lo, hi), rows(trans(qgt, C, p.scale), lo, hi),
                         trans(hp, D)};  // W, s qg, h^T
    auto issue = [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 2), ring.op(buf, 0), 128, KS / 8, s > 0 || hf > 0);        // (W h)^T: (v, i)
      mma3(tmem + 128, ring.op(buf, 1), ring.op(buf, 2), 128, KS / 8, s > 0 || hf > 0);  // scale qg h: (i, v)
    };
    kloop_pf<false, 4, (SUB > 1)>(ring, g, ws.status, srcs, NoExtra{}, issue);
  }
  uint32_t ph = 0;
  drain(&ts.done, ph, ws.status);
  // vnew^T = U^T - (W h)^T, one TMEM lane per value column v: written to
  // ws.vnew (coalesced per column i) and kept as four resident K-slices (rows
  // v, K = i) in shared memory, the B operand of Aqk vnew.
  const float* u = ws.U + chunk * C * D;
  float* vn = ws.vnew + chunk * C * D;
  float* vt = sm;
  {
    // all 64 U loads of this thread (its value column v, 64 rows i) before
    // the first vnew store, which the compiler must assume may alias them
    const int warp = threadIdx.x >> 5;
    const int v = 32 * (warp & 3) + (threadIdx.x & 31), cb = (warp >> 2) * 64;
    float uu[64];
#pragma unroll
    for (int t = 0; t < 64; ++t) uu[t] = u[(cb + t) * D + v];
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      const int c0 = cb + 16 * grp;
      float x[16];
      tmem_ld16(lane_quarter_addr(tmem, c0), x);
      float* hi = vt + (c0 / KS) * 2 * SLICE_FLOATS;
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        float y[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          y[t] = uu[16 * grp + j + t] - x[j + t];
          vn[(c0 + j + t) * D + v] = y[t];
        }
        st_split4(hi, hi + SLICE_FLOATS, v, c0 % KS + j, KS, make_float4(y[0], y[1], y[2], y[3]));
      }
    }
  }
  const float* aqkt = ws.AqkT + chunk * C * C;
  ring.base = sm + 4 * 2 * SLICE_FLOATS;
  ring.nop = 1;
  {
    const Src srcs[1] = {trans(aqkt, C)};   // (i,j) = Aqk
    kloop_pf<false>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      float* hi = vt + s * 2 * SLICE_FLOATS;
      mma3(tmem + 128, ring.op(buf, 0), kmajor(hi, hi + SLICE_FLOATS, KS), 128, KS / 8, 1);
    });
  }
  drain(&ts.done, ph, ws.status);
  if (o) {
    const long rs = p.row_stride();
    float* orow = o + ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
    StageDiag dg;
    for_acc<128>(tmem, 128, [&](int i, int c0, const float* x) {
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 o4 = make_float4(san(x[j], p.clip), san(x[j + 1], p.clip),
                                      san(x[j + 2], p.clip), san(x[j + 3], p.clip));
        st4f(orow + i * rs + c0 + j, o4);
        if (p.diag) dg.add4(o4);
      }
    });
    if (p.diag) dg.flush(ws.status, kDiagO);
  }
  tc_teardown(tmem, 256);
}

// ---------------------------------------------------------------------------
// Backward chunk-parallel terms of the state pass:
//   dv_partial = san(Aqk^T do)  (B2, gdn2_bwd.py:93)          -> ws.dvp
//   E = scale qg^T do - W^T dv_partial                        -> ws.E
// ---------------------------------------------------------------------------
template <int SUB>
__global__ void __launch_bounds__(kThreads, 1)
k_tc_bwd_prep(Problem p, Workspace ws, const float* __restrict__ dout) {
  extern __shared__ __align__(128) float sm[];
  __shared__ TcSmem ts;
  const size_t chunk = blockIdx.x;
  const int c = (int)(chunk % p.nc);
  const size_t bh = chunk / p.nc;
  const int h = (int)(bh % p.H), bb = (int)(bh / p.H);
  constexpr uint32_t kCols = SUB == 1 ? 256 : 512;
  const uint32_t tmem = tc_setup(&ts, kCols);
  // E of reference chunk hf accumulates at TMEM 128 + 128 hf; its K rows are
  // the slices [hf * NSC, (hf + 1) * NSC)
  constexpr int NSC = 4 / SUB;
  Ring ring = make_ring(sm, &ts, 3);
  const long rs = p.row_stride();
  const float* doc = dout + ((long)bb * p.T + (long)c * C) * rs + (long)h * D;
  const float* aqkt = ws.AqkT + chunk * C * C;
  const float* qgt = ws.qgT + chunk * C * D;
  int g = 0;
  {
    const Src srcs[3] = {direct(aqkt, C), direct(qgt, C, p.scale), trans(doc, rs)};  // (j,i) (d,i) (v,i)
    kloop_pf<false>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      mma3(tmem, ring.op(buf, 2), ring.op(buf, 0), 128, KS / 8, s > 0);        // dvp^T: (v, j)
      mma3(tmem + 128 + 128 * (s / NSC), ring.op(buf, 1), ring.op(buf, 2), 128, KS / 8,
           s % NSC > 0);                                                         // scale qg^T do
    });
  }
  uint32_t ph = 0;
  drain(&ts.done, ph, ws.status);
  // dvp = san(Aqk^T do), one TMEM lane per value column v: written to ws.dvp
  // (coalesced per column j) and kept as four resident K-slices (rows v,
  // K = j) in shared memory, the B operand of -W^T dvp.
  float* dvp = ws.dvp + chunk * C * D;
  float* dt = sm;
  float amax0 = 0.f, amax1 = 0.f;   // per reference chunk (column j's chunk)
  constexpr int R = C / SUB;
  for_acc<128>(tmem, 0, [&](int v, int c0, const float* x) {
    float* hi = dt + (c0 / KS) * 2 * SLICE_FLOATS;
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      float y[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        y[t] = san(x[k + t], p.clip);
        if (SUB == 1 || c0 < R) amax0 = fmaxf(amax0, fabsf(y[t]));
        else amax1 = fmaxf(amax1, fabsf(y[t]));
        dvp[(c0 + k + t) * D + v] = y[t];
      }
      st_split4(hi, hi + SLICE_FLOATS, v, c0 % KS + k, KS, make_float4(y[0], y[1], y[2], y[3]));
    }
  });
  // max |dv_partial|: the constant part of the backward guard
  for (int hf = 0; hf < SUB; ++hf) {
    const float m = block_max(hf ? amax1 : amax0, ts.red);
    if (threadIdx.x == 0) ws.bnd[(chunk * SUB + hf) * 4 + 1] = m;
  }
  const float* wt = ws.WT + chunk * C * D;
  ring.base = sm + 4 * 2 * SLICE_FLOATS;
  ring.nop = 1;
  {
    const Src srcs[1] = {direct(wt, C, -1.f)};   // (d,j) = -W
    kloop_pf<false>(ring, g, ws.status, srcs, NoExtra{}, [&](int buf, int s) {
      float* hi = dt + s * 2 * SLICE_FLOATS;
      mma3(tmem + 128 + 128 * (s / NSC), ring.op(buf, 0), kmajor(hi, hi + SLICE_FLOATS, KS), 128,
           KS / 8, 1);
    });
  }
  drain(&ts.done, ph, ws.status);
#pragma unroll 1
  for (int hf = 0; hf < SUB; ++hf) {
    float* eo = ws.E + (chunk * SUB + hf) * D * D;
    for_acc<128>(tmem, 128 + 128 * hf, [&](int d, int c0, const float* x) {
#pragma unroll
      for (int k = 0; k < 16; k += 4) st4f(eo + d * D + c0 + k, make_float4(x[k], x[k + 1], x[k + 2], x[k + 3]));
    });
  }
  tc_teardown(tmem, kCols);
}


// ---------------------------------------------------------------------------
namespace {
template <class K>
cudaError_t prep(K kern, size_t smem) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}
constexpr size_t kRing3 = 2 * 3 * (size_t)SLICE_BYTES;   // 192 KB
constexpr size_t kScan = (kScanSlots + 8) * (size_t)kScanSliceBytes;   // raw ring + lo + constant term, 224 KB
}  // namespace

cudaError_t launch_tc_fwd(const Problem& p, const Workspace& ws, const float* h0, float* o,
                          float* hfinal, cudaStream_t s, const LaunchHook& hook, bool outputs) {
  cudaError_t e;
  const unsigned nchunks = (unsigned)p.B * p.H * p.nc;
  auto affine = p.sub == 2 ? k_tc_affine<2> : k_tc_affine<1>;
  auto fwd_out = p.sub == 2 ? k_tc_fwd_out<2> : k_tc_fwd_out<1>;
  if ((e = prep(affine, kRing3)) != cudaSuccess) return e;
  if ((e = prep(k_tc_scan<false>, kScan)) != cudaSuccess) return e;
  if ((e = prep(fwd_out, kRing3)) != cudaSuccess) return e;
  hook.begin(kStageFwdAffine, s);
  affine<<<nchunks, kThreads, kRing3, s>>>(p, ws);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageFwdAffine, s);
  hook.begin(kStageFwdScan, s);
  k_tc_scan<false><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, h0, hfinal);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageFwdScan, s);
  if (!outputs) return cudaSuccess;
  hook.begin(kStageFwdOut, s);
  fwd_out<<<nchunks, kThreads, kRing3, s>>>(p, ws, o);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageFwdOut, s);
  return cudaSuccess;
}

cudaError_t launch_tc_bwd_state(const Problem& p, const Workspace& ws, const float* dout,
                                const float* dh_final, float* dh0, cudaStream_t s,
                                const LaunchHook& hook, bool with_prep) {
  cudaError_t e;
  const unsigned nchunks = (unsigned)p.B * p.H * p.nc;
  auto bwd_prep = p.sub == 2 ? k_tc_bwd_prep<2> : k_tc_bwd_prep<1>;
  if ((e = prep(bwd_prep, kRing3)) != cudaSuccess) return e;
  if ((e = prep(k_tc_scan<true>, kScan)) != cudaSuccess) return e;
  if (with_prep) {
    hook.begin(kStageBwdPrep, s);
    bwd_prep<<<nchunks, kThreads, kRing3, s>>>(p, ws, dout);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    hook.end(kStageBwdPrep, s);
  }
  hook.begin(kStageBwdScan, s);
  k_tc_scan<true><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, dh_final, dh0);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  hook.end(kStageBwdScan, s);
  // The (b, h) whose guard failed rerun the reference's three-product step
  // (the CTAs of every other (b, h) return at once).
  hook.begin(kStageBwdExact, s);
  if (p.sub == 1) {
    if ((e = launch_bwd_state<C, D>(p, ws, dout, dh_final, dh0, s, true)) != cudaSuccess) return e;
  } else {   // paired tiles: the 64-row step over the reference chunks
    Problem p64 = p;
    p64.C = C / 2;
    p64.nc = p.ncs();
    p64.sub = 1;
    if ((e = launch_bwd_state<C / 2, D>(p64, ws, dout, dh_final, dh0, s, true, true)) != cudaSuccess)
      return e;
  }
  hook.end(kStageBwdExact, s);
  // dv_new is formed by the first product of k_tc_bwd_intra1
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
    if ((e = prep(k_tc_fwd_out<1>, kRing3)) != cudaSuccess) return e;
    hook.begin(kStageFwdScan, s);
    k_tc_scan<false><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, in, out);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    hook.end(kStageFwdScan, s);
    hook.begin(kStageFwdOut, s);
    k_tc_fwd_out<1><<<nchunks, kThreads, kRing3, s>>>(p, ws, o);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    hook.end(kStageFwdOut, s);
    return cudaSuccess;
  }
  // op == 2: backward segment term, zero incoming gradient
  if ((e = prep(k_tc_bwd_prep<1>, kRing3)) != cudaSuccess) return e;
  if ((e = prep(k_tc_scan<true>, kScan)) != cudaSuccess) return e;
  k_tc_bwd_prep<1><<<nchunks, kThreads, kRing3, s>>>(p, ws, in);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  k_tc_scan<true><<<dim3(p.H, p.B), kThreads, kScan, s>>>(p, ws, nullptr, out);
  return cudaGetLastError();
}
}  // namespace gdn2
