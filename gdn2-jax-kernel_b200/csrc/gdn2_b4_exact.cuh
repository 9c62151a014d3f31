// Exact B4 (backward of the chunk scores, gdn2_bwd.py:248-339) for one chunk,
// in the reference's sub-block pair order.
//
// The reference loops over the BC-row sub-block pairs (si, sj), sj <= si, and
// after every pair sanitises each accumulator it touched (_clip_acc,
// gdn2_bwd.py:26-28, 316-328):
//     dq[I]  = clip(dq[I]  + dLq scale)        dbk[I] = clip(dbk[I] + dLk)
//     dk[J]  = clip(dk[J]  + dRq + dRk)
//     dgc[I] = clip(dgc[I] + wq.sum(-2) + wk.sum(-2))
//     dgc[J] = clip(dgc[J] - wq.sum(-3) - wk.sum(-3))
// with the pair decay e^{clip(gc_i - gc_j, +-20)} and the mask cm zeroing the
// dgc terms of clipped pairs.  The fast kernels sum every pair in one product
// and agree with this only while no accumulator reaches CLIP; this routine is
// the reference order itself, used for chunks whose gates are positive or
// whose guard says a clip could act.  One thread per (row x, column d); a
// warp covers 32 consecutive d of one row.
#pragma once
#include "gdn2_common.cuh"

namespace gdn2 {

constexpr float kB4FinalClip = 1e4f;   // gdn2_pipeline.py:34

// gc: chunk-local cumulative gates, gc[x * gld + d].  dAqkT / dAkkT: element
// (i, j) at j * C + i.  pd*: the sanitised B3 partials of this chunk
// ([C][D]).  Writes dq, dk, db (with the final +-1e4 sanitiser) and
// sdg[x * D + d] = pdgc + clip(dgc) (the input of the B5 reverse cumsum).
template <typename T, typename TO = T>   // input / output element types
__device__ void b4_exact_chunk(int C, int D, int BC, const T* __restrict__ qc,
                               const T* __restrict__ kc, const T* __restrict__ bc, long rs,
                               const float* gc, int gld, const float* __restrict__ dAqkT,
                               const float* __restrict__ dAkkT, const float* pdq, const float* pdk,
                               const float* pdb, const float* pdgc, TO* dq_out, TO* dk_out,
                               TO* db_out, long off, float* sdg, float scale, float clip,
                               int gates, int span, long ors = -1,
                               float final_clip = kB4FinalClip) {
  // ors: row stride of the outputs (default: rs, the inputs' layout)
  if (ors < 0) ors = rs;
  // span: rows of one reference chunk (C, or C / 2 for a tile of two chunks);
  // the pairs stay inside the chunk of row x
  const int nsc = span / BC;
  for (int e = threadIdx.x; e < C * D; e += kThreads) {
    const int x = e / D, d = e % D, X = x / BC, X0 = (X / nsc) * nsc;
    const float kx = to_f<T>(kc[x * rs + d]), bx = ld_gate<T>(bc + x * rs + d, gates, kGateB);
    const float lqx = scale * to_f<T>(qc[x * rs + d]), lkx = bx * kx;
    const float gx = gc[x * gld + d];
    float dq = 0.f, dbk = 0.f, dk = 0.f, dgc = 0.f;
    for (int si = X; si < X0 + nsc; ++si) {
      for (int sj = X0; sj <= si; ++sj) {
        if (si != X && sj != X) continue;
        float dlq = 0.f, dlk = 0.f, wqi = 0.f, wki = 0.f;
        float drq = 0.f, drk = 0.f, wqj = 0.f, wkj = 0.f;
        if (si == X) {   // x is a row i of the pair: columns j of block sj
          for (int y = sj * BC; y < (sj + 1) * BC; ++y) {
            const float dd = gx - gc[y * gld + d];
            const float ed = expf(fminf(fmaxf(dd, -20.f), 20.f));
            const float cm = (dd >= -20.f && dd <= 20.f) ? 1.f : 0.f;
            // stored dAqk is causal and dAkk strictly lower: the diagonal
            // pair's masks are already in the zeros
            const float mq = dAqkT[y * C + x], mk = dAkkT[y * C + x];
            const float r = to_f<T>(kc[y * rs + d]) * ed;
            dlq = fmaf(mq, r, dlq);
            dlk = fmaf(mk, r, dlk);
            wqi = fmaf(mq * lqx, r * cm, wqi);
            wki = fmaf(mk * lkx, r * cm, wki);
          }
        }
        if (sj == X) {   // x is a column j of the pair: rows i of block si
          for (int y = si * BC; y < (si + 1) * BC; ++y) {
            const float dd = gc[y * gld + d] - gx;
            const float ed = expf(fminf(fmaxf(dd, -20.f), 20.f));
            const float cm = (dd >= -20.f && dd <= 20.f) ? 1.f : 0.f;
            const float mq = dAqkT[x * C + y], mk = dAkkT[x * C + y];
            const float lqy = scale * to_f<T>(qc[y * rs + d]) * ed;
            const float lky = ld_gate<T>(bc + y * rs + d, gates, kGateB) * to_f<T>(kc[y * rs + d]) * ed;
            drq = fmaf(mq, lqy, drq);
            drk = fmaf(mk, lky, drk);
            wqj = fmaf(mq * lqy, kx * cm, wqj);
            wkj = fmaf(mk * lky, kx * cm, wkj);
          }
        }
        // the reference's statement order for one pair (gdn2_bwd.py:324-328)
        if (si == X) {
          dq = san(dq + dlq * scale, clip);
          dbk = san(dbk + dlk, clip);
        }
        if (sj == X) dk = san(dk + drq + drk, clip);
        if (si == X) dgc = san(dgc + wqi + wki, clip);
        if (sj == X) dgc = san(dgc - wqj - wkj, clip);
      }
    }
    // _kernel_b4_body's final sanitisers, then the pipeline's sum with B3
    // and the +-1e4 clip (gdn2_bwd.py:333-336, gdn2_pipeline.py:117-135)
    const long o = off + x * ors + d;
    dq_out[o] = from_f<TO>(san(pdq[e] + san(dq, clip), final_clip));
    dk_out[o] = from_f<TO>(san(pdk[e] + san(dk + dbk * bx, clip), final_clip));
    const float dbo = san(pdb[e] + san(dbk * kx, clip), final_clip);
    db_out[o] = from_f<TO>(gates ? dbo * bx * (1.f - bx) : dbo);
    sdg[e] = pdgc[e] + san(dgc, clip);
  }
}

}  // namespace gdn2
