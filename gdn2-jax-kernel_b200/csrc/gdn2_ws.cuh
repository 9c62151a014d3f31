// Workspace layout shared by the forward and backward kernels.
//
// Every per-chunk tile is stored contiguously at offset
// chunk_id * tile_elems, chunk_id = (b*H + h)*nc + c, in float32.  Tiles are
// stored in the orientation their consumer streams into shared memory.
// Arrays of the state recurrence (gcl, hpre, M, Bc, bnd, E, dh) hold one
// entry per reference chunk: index chunk_id * sub + half when a tile carries
// sub = 2 chunks of 64 rows.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace gdn2 {

struct Problem {
  int B, T, H, D, C, nc;   // C = kernel tile rows, nc = T / C
  int sub;                 // reference chunks per tile: 1, or 2 (two BT = 64 chunks
                           // stacked in one 128-row tensor-core tile)
  int bc;                  // the reference's sub-block BC (clip granularity of B4)
  int diag;                // 1: accumulate per-stage diagnostics in the status header
  int gates;               // 1: w, b, g are pre-activations (GDN2_GATES_RAW)
  float scale, clip;
  __host__ __device__ long row_stride() const { return (long)H * D; }
  __host__ __device__ int ncs() const { return nc * sub; }   // reference chunks per (b, h)
};

// Float offsets (per chunk multiples) of every workspace array.
struct Workspace {
  float* base;
  // forward intermediates
  float* AqkT;   // [C][C]  Aqk transposed: element (i,j) at j*C + i
  float* AT;     // [C][C]  A = (I+Akk)^-1 transposed
  float* WT;     // [D][C]  W transposed
  float* U;      // [C][D]
  float* kg;     // [C][D]
  float* qgT;    // [D][C]
  float* gc;     // [C][D]  in-chunk cumulative log decay
  float* gcl;    // [D]     sanitised gc of the last row
  // forward residuals kept for the backward
  float* hpre;   // [D][D]  state entering each chunk
  float* vnew;   // [C][D]
  // backward intermediates
  float* dv;     // [C][D]  dv_new from the reverse state pass
  float* dh;     // [D][D]  dh_pre of each chunk (dh_all)
  float* dAqkT;  // [C][C]
  float* dAkkT;  // [C][C]
  float* dWp;    // [C][D]
  float* pdq;    // [C][D]  partial dq  (B3)
  float* pdk;    // [C][D]  partial dk  (B3, then B4 scratch)
  float* pdb;    // [C][D]  partial db  (B3)
  float* pdgc;   // [C][D]  partial dgc (B3)
  // affine form of the state recurrence (tensor-core path)
  float* M;      // [2][D][D] M = diag(e^{gc_last}) - kg^T W as scan operands:
                 //   [0, D^2): M as 4 K-slices, canonical 128 x 32 tiles (rows =
                 //   row of M, K = column); [D^2, 2 D^2): the same for M^T
  float* Bc;     // [D][D]  kg^T U
  float* bnd;    // [4] per chunk, the exactness guard of the affine backward chain:
                 //   [0] max_i sum_d |kg(i,d)|   (forward intra kernel)
                 //   [1] max |dv_partial|        (backward prep kernel)
                 //   [2] 1 if this chunk's step could clip dv_new (backward scan)
                 //   [3] on the first chunk of each (b,h): 1 if any of its chunks could
  float* E;      // [D][D]  scale qg^T do - W^T dv_partial
  float* dvp;    // [C][D]  dv_partial = san(Aqk^T do)
  int* status;   // device status word (1 = a bounded wait timed out), zeroed by every entry point
  size_t bytes;

  static size_t per_chunk_floats(int C, int D, bool bwd, int sub = 1) {
    const size_t S = (size_t)sub;
    size_t f = 2 * (size_t)C * C + 5 * (size_t)C * D + S * D;   // forward
    f += S * D * D + (size_t)C * D;                              // residuals
    f += S * 3 * D * D;                                          // M (both ways), Bc
    f += S * 4;                                                  // bnd
    if (bwd) f += 2 * (size_t)C * C + 7 * (size_t)C * D + S * 2 * D * D;
    return f;
  }
  static size_t required_bytes(int B, int H, int nc, int C, int D, bool bwd, int sub = 1) {
    return per_chunk_floats(C, D, bwd, sub) * (size_t)B * H * nc * sizeof(float) + 512;
  }
  static Workspace carve(void* p, int B, int H, int nc, int C, int D, bool bwd, int sub = 1) {
    Workspace w{};
    size_t n = (size_t)B * H * nc;
    float* f = reinterpret_cast<float*>(((uintptr_t)p + 255) & ~(uintptr_t)255);
    w.status = reinterpret_cast<int*>(f);   // first 256 bytes: status word
    f += 64;
    w.base = f;
    auto take = [&](size_t per) { float* r = f; f += per * n; return r; };
    w.AqkT = take((size_t)C * C);
    w.AT = take((size_t)C * C);
    w.WT = take((size_t)C * D);
    w.U = take((size_t)C * D);
    w.kg = take((size_t)C * D);
    w.qgT = take((size_t)C * D);
    w.gc = take((size_t)C * D);
    const size_t S = (size_t)sub;
    w.gcl = take(S * D);
    w.hpre = take(S * D * D);
    w.vnew = take((size_t)C * D);
    w.M = take(S * 2 * D * D);
    w.Bc = take(S * D * D);
    w.bnd = take(S * 4);
    if (bwd) {
      w.dv = take((size_t)C * D);
      w.dh = take(S * D * D);
      w.dAqkT = take((size_t)C * C);
      w.dAkkT = take((size_t)C * C);
      w.dWp = take((size_t)C * D);
      w.pdq = take((size_t)C * D);
      w.pdk = take((size_t)C * D);
      w.pdb = take((size_t)C * D);
      w.pdgc = take((size_t)C * D);
      w.E = take(S * D * D);
      w.dvp = take((size_t)C * D);
    }
    w.bytes = required_bytes(B, H, nc, C, D, bwd, sub);
    return w;
  }
};

}  // namespace gdn2
