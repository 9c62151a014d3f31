// fp32 C++/OpenMP restatement of the reference GDN-2 chunked forward and
// fused backward (Akseleu-J/gdn2-jax-kernel: gdn2_fwd.py, gdn2_bwd.py,
// gdn2_pipeline.py), for the timed CPU baseline of bench.py.
//
// TEST AND BENCHMARK INFRASTRUCTURE: nothing in the product path loads this
// library.  It follows oracle/gdn2_oracle.py (the float64 restatement pinned
// to the reference's own outputs) step by step, in float32, one (batch, head)
// per OpenMP task:
//   forward   chunk scores (gdn2_fwd.py:99-139), WY solve (174-243),
//             Kernel C (264-295), Kernel D (347-360);
//   backward  B2 (gdn2_bwd.py:84-96), B1 (45-80), B3 (126-210),
//             B4 (248-339), B5 (32-41), assembly (gdn2_pipeline.py:70-137).
//
// Build: python oracle/gdn2_cpu.py (g++ -O3 -fopenmp, into oracle/_build/).
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

namespace {

constexpr float kPairClip = 20.f;     // gdn2_fwd.py:120
constexpr float kFinalClip = 1e4f;    // gdn2_pipeline.py:34
constexpr int kMB = 16;               // gdn2_fwd.py:32

inline float san(float x, float c) {  // gdn2_fwd.py:42-44
  if (x != x) return 0.f;
  return std::min(std::max(x, -c), c);
}

using Mat = std::vector<float>;       // row-major

// C (m x n) = A (m x k) * B (k x n); strides given
void mm(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int m, int k, int n,
        bool acc = false) {
  for (int i = 0; i < m; ++i) {
    float* c = C + (size_t)i * ldc;
    if (!acc) std::fill(c, c + n, 0.f);
    for (int t = 0; t < k; ++t) {
      const float a = A[(size_t)i * lda + t];
      if (a == 0.f) continue;
      const float* b = B + (size_t)t * ldb;
      for (int j = 0; j < n; ++j) c[j] += a * b[j];
    }
  }
}
Mat tr(const float* A, int m, int n) {   // n x m
  Mat R((size_t)m * n);
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) R[(size_t)j * m + i] = A[(size_t)i * n + j];
  return R;
}

// A = (I + T)^-1 of a strictly lower n x n T (ld n), the reference's block
// substitution (gdn2_fwd.py:174-222): blocks of `blk`, diag solved by `diag`.
template <class Diag>
void compose(const float* T, float* A, int n, int blk, float clip, Diag diag) {
  const int nb = n / blk;
  std::fill(A, A + (size_t)n * n, 0.f);
  Mat Tb((size_t)blk * blk), Ab((size_t)blk * blk), acc((size_t)blk * blk), pr((size_t)blk * blk);
  auto get = [&](const float* M, int bi, int bj, float* out) {
    for (int i = 0; i < blk; ++i)
      std::memcpy(out + (size_t)i * blk, M + (size_t)(bi * blk + i) * n + bj * blk, blk * 4);
  };
  auto put = [&](float* M, int bi, int bj, const float* in) {
    for (int i = 0; i < blk; ++i)
      std::memcpy(M + (size_t)(bi * blk + i) * n + bj * blk, in + (size_t)i * blk, blk * 4);
  };
  Mat Amm((size_t)blk * blk);
  for (int m = 0; m < nb; ++m) {
    get(T, m, m, Tb.data());
    diag(Tb.data(), Amm.data());
    for (auto& x : Amm) x = san(x, clip);
    put(A, m, m, Amm.data());
    for (int nn = m - 1; nn >= 0; --nn) {
      std::fill(acc.begin(), acc.end(), 0.f);
      for (int k = nn; k < m; ++k) {
        get(T, m, k, Tb.data());
        get(A, k, nn, Ab.data());
        mm(Tb.data(), blk, Ab.data(), blk, pr.data(), blk, blk, blk, blk);
        for (size_t e = 0; e < acc.size(); ++e) acc[e] = san(acc[e] + pr[e], clip);
      }
      mm(Amm.data(), blk, acc.data(), blk, pr.data(), blk, blk, blk, blk);
      for (auto& x : pr) x = san(-x, clip);
      put(A, m, nn, pr.data());
    }
  }
}

void micro_solve(const float* T, float* A, int n, float clip) {   // gdn2_fwd.py:174-189
  std::fill(A, A + (size_t)n * n, 0.f);
  for (int i = 0; i < n; ++i)
    for (int c = 0; c < n; ++c) {
      float s = 0.f;
      for (int r = 0; r < i; ++r) s += T[(size_t)i * n + r] * A[(size_t)r * n + c];
      A[(size_t)i * n + c] = san((i == c ? 1.f : 0.f) - s, clip);
    }
}

struct Slice {   // one (batch, head): pointers with row stride rs
  const float *q, *k, *v, *w, *b, *g, *dout;
  long rs;
};

struct Fwd {     // per-chunk residuals of one (b, h)
  int C, D, nc;
  std::vector<Mat> Aqk, A, W, U, kg, qg, gc, hpre, vnew;
  std::vector<std::vector<float>> gcl;   // sanitised gc_last
};

void forward(const Slice& s, const float* h0, float* o, float* hf, int T, int D, int C, int BC,
             float scale, float clip, Fwd& R) {
  const int nc = T / C;
  R.C = C; R.D = D; R.nc = nc;
  for (auto* v : {&R.Aqk, &R.A, &R.W, &R.U, &R.kg, &R.qg, &R.gc, &R.hpre, &R.vnew}) v->resize(nc);
  R.gcl.resize(nc);
  Mat h((size_t)D * D, 0.f);
  if (h0)
    for (size_t e = 0; e < h.size(); ++e) h[e] = san(h0[e], clip);
  Mat Akk((size_t)C * C), tmp((size_t)C * D), kb((size_t)C * D), wv((size_t)C * D);
  const int mb = std::min(kMB, BC);
  for (int c = 0; c < nc; ++c) {
    auto at = [&](const float* x, int i, int d) { return x[((long)c * C + i) * s.rs + d]; };
    Mat& gc = R.gc[c];
    gc.assign((size_t)C * D, 0.f);
    for (int d = 0; d < D; ++d) {
      float a = 0.f;
      for (int i = 0; i < C; ++i) gc[(size_t)i * D + d] = (a += at(s.g, i, d));
    }
    // chunk scores (gdn2_fwd.py:99-139)
    Mat& Aqk = R.Aqk[c];
    Aqk.assign((size_t)C * C, 0.f);
    std::fill(Akk.begin(), Akk.end(), 0.f);
    for (int i = 0; i < C; ++i)
      for (int j = 0; j <= i; ++j) {
        float sq = 0.f, sk = 0.f;
        for (int d = 0; d < D; ++d) {
          const float ed = std::exp(std::min(std::max(gc[(size_t)i * D + d] - gc[(size_t)j * D + d],
                                                      -kPairClip), kPairClip));
          const float kj = at(s.k, j, d) * ed;
          sq += at(s.q, i, d) * kj;
          sk += at(s.b, i, d) * at(s.k, i, d) * kj;
        }
        Aqk[(size_t)i * C + j] = san(scale * sq, clip);
        if (j < i) Akk[(size_t)i * C + j] = san(sk, clip);
      }
    // WY solve (gdn2_fwd.py:174-243, sub-blocks generalised as the oracle does)
    Mat& A = R.A[c];
    A.assign((size_t)C * C, 0.f);
    compose(Akk.data(), A.data(), C, BC, clip, [&](const float* Tb, float* Ab) {
      compose(Tb, Ab, BC, mb, clip, [&](const float* Tm, float* Am) { micro_solve(Tm, Am, mb, clip); });
    });
    // Kernel C (gdn2_fwd.py:264-295)
    for (int i = 0; i < C; ++i)
      for (int d = 0; d < D; ++d) {
        kb[(size_t)i * D + d] = at(s.b, i, d) * at(s.k, i, d) * std::exp(gc[(size_t)i * D + d]);
        wv[(size_t)i * D + d] = at(s.w, i, d) * at(s.v, i, d);
      }
    Mat &W = R.W[c], &U = R.U[c], &kg = R.kg[c], &qg = R.qg[c];
    W.resize((size_t)C * D); U.resize((size_t)C * D); kg.resize((size_t)C * D); qg.resize((size_t)C * D);
    mm(A.data(), C, kb.data(), D, W.data(), D, C, C, D);
    mm(A.data(), C, wv.data(), D, U.data(), D, C, C, D);
    R.gcl[c].resize(D);
    for (int i = 0; i < C; ++i)
      for (int d = 0; d < D; ++d) {
        const size_t e = (size_t)i * D + d;
        W[e] = san(W[e], clip);
        U[e] = san(U[e], clip);
        kg[e] = san(at(s.k, i, d) * std::exp(gc[(size_t)(C - 1) * D + d] - gc[e]), clip);
        qg[e] = san(at(s.q, i, d) * std::exp(gc[e]), clip);
      }
    for (int d = 0; d < D; ++d) R.gcl[c][d] = san(gc[(size_t)(C - 1) * D + d], clip);
    // Kernel D (gdn2_fwd.py:347-360)
    R.hpre[c] = h;
    Mat& vn = R.vnew[c];
    vn.resize((size_t)C * D);
    mm(W.data(), D, h.data(), D, tmp.data(), D, C, D, D);
    for (size_t e = 0; e < vn.size(); ++e) vn[e] = U[e] - tmp[e];
    Mat oc((size_t)C * D);
    mm(qg.data(), D, h.data(), D, oc.data(), D, C, D, D);
    for (auto& x : oc) x *= scale;
    mm(Aqk.data(), C, vn.data(), D, oc.data(), D, C, C, D, true);
    if (o)
      for (int i = 0; i < C; ++i)
        for (int d = 0; d < D; ++d) o[((long)c * C + i) * s.rs + d] = san(oc[(size_t)i * D + d], clip);
    Mat kgT = tr(kg.data(), C, D), wr((size_t)D * D);
    mm(kgT.data(), C, vn.data(), D, wr.data(), D, D, C, D);
    for (int d = 0; d < D; ++d) {
      const float dec = std::exp(R.gcl[c][d]);
      for (int v = 0; v < D; ++v) {
        const size_t e = (size_t)d * D + v;
        h[e] = san(h[e] * dec + wr[e], clip);
      }
    }
  }
  if (hf) std::memcpy(hf, h.data(), h.size() * 4);
}

// B4 in the reference's sub-block pair order (gdn2_bwd.py:248-339)
void intra_backward(const Slice& s, int c, const Mat& gc, const Mat& dAqk, const Mat& dAkk, int C,
                    int D, int BC, float scale, float clip, Mat& dq, Mat& dk, Mat& db, Mat& dgc) {
  auto at = [&](const float* x, int i, int d) { return x[((long)c * C + i) * s.rs + d]; };
  Mat q4((size_t)C * D, 0.f), k4((size_t)C * D, 0.f), dbk((size_t)C * D, 0.f), g4((size_t)C * D, 0.f);
  const int ns = C / BC;
  std::vector<float> dLq(D), dLk(D), dRq(D), dRk(D), wi(D), wj(D);
  for (int si = 0; si < ns; ++si)
    for (int sj = 0; sj <= si; ++sj) {
      // per row i of block si: dL and the I-side dgc weights
      for (int i = si * BC; i < (si + 1) * BC; ++i) {
        std::fill(dLq.begin(), dLq.end(), 0.f); std::fill(dLk.begin(), dLk.end(), 0.f);
        for (int j = sj * BC; j < (sj + 1) * BC; ++j) {
          const float mq = (si == sj && j > i) ? 0.f : dAqk[(size_t)i * C + j];
          const float mk = (si == sj && j >= i) ? 0.f : dAkk[(size_t)i * C + j];
          if (mq == 0.f && mk == 0.f) continue;
          for (int d = 0; d < D; ++d) {
            const float dd = gc[(size_t)i * D + d] - gc[(size_t)j * D + d];
            const float ed = std::exp(std::min(std::max(dd, -kPairClip), kPairClip));
            const float cm = (dd >= -kPairClip && dd <= kPairClip) ? 1.f : 0.f;
            (void)cm;
            const float r = at(s.k, j, d) * ed;
            dLq[d] += mq * r;
            dLk[d] += mk * r;
          }
        }
        for (int d = 0; d < D; ++d) {
          const size_t e = (size_t)i * D + d;
          q4[e] = san(q4[e] + dLq[d] * scale, clip);
          dbk[e] = san(dbk[e] + dLk[d], clip);
        }
      }
      // per column j of block sj: dR and the J-side weights
      for (int j = sj * BC; j < (sj + 1) * BC; ++j) {
        std::fill(dRq.begin(), dRq.end(), 0.f); std::fill(dRk.begin(), dRk.end(), 0.f);
        for (int i = si * BC; i < (si + 1) * BC; ++i) {
          const float mq = (si == sj && j > i) ? 0.f : dAqk[(size_t)i * C + j];
          const float mk = (si == sj && j >= i) ? 0.f : dAkk[(size_t)i * C + j];
          if (mq == 0.f && mk == 0.f) continue;
          for (int d = 0; d < D; ++d) {
            const float dd = gc[(size_t)i * D + d] - gc[(size_t)j * D + d];
            const float ed = std::exp(std::min(std::max(dd, -kPairClip), kPairClip));
            const float cm = (dd >= -kPairClip && dd <= kPairClip) ? 1.f : 0.f;
            const float lq = scale * at(s.q, i, d) * ed, lk = at(s.b, i, d) * at(s.k, i, d) * ed;
            (void)cm;
            dRq[d] += mq * lq;
            dRk[d] += mk * lk;
          }
        }
        for (int d = 0; d < D; ++d) {
          const size_t e = (size_t)j * D + d;
          k4[e] = san(k4[e] + dRq[d] + dRk[d], clip);
        }
      }
      // dgc: the I rows first, then the J rows (gdn2_bwd.py:327-328)
      for (int i = si * BC; i < (si + 1) * BC; ++i) {
        std::fill(wi.begin(), wi.end(), 0.f);
        for (int j = sj * BC; j < (sj + 1) * BC; ++j) {
          const float mq = (si == sj && j > i) ? 0.f : dAqk[(size_t)i * C + j];
          const float mk = (si == sj && j >= i) ? 0.f : dAkk[(size_t)i * C + j];
          if (mq == 0.f && mk == 0.f) continue;
          for (int d = 0; d < D; ++d) {
            const float dd = gc[(size_t)i * D + d] - gc[(size_t)j * D + d];
            const float ed = std::exp(std::min(std::max(dd, -kPairClip), kPairClip));
            const float cm = (dd >= -kPairClip && dd <= kPairClip) ? 1.f : 0.f;
            wi[d] += (mq * scale * at(s.q, i, d) + mk * at(s.b, i, d) * at(s.k, i, d)) *
                     at(s.k, j, d) * ed * cm;
          }
        }
        for (int d = 0; d < D; ++d) {
          const size_t e = (size_t)i * D + d;
          g4[e] = san(g4[e] + wi[d], clip);
        }
      }
      for (int j = sj * BC; j < (sj + 1) * BC; ++j) {
        std::fill(wj.begin(), wj.end(), 0.f);
        for (int i = si * BC; i < (si + 1) * BC; ++i) {
          const float mq = (si == sj && j > i) ? 0.f : dAqk[(size_t)i * C + j];
          const float mk = (si == sj && j >= i) ? 0.f : dAkk[(size_t)i * C + j];
          if (mq == 0.f && mk == 0.f) continue;
          for (int d = 0; d < D; ++d) {
            const float dd = gc[(size_t)i * D + d] - gc[(size_t)j * D + d];
            const float ed = std::exp(std::min(std::max(dd, -kPairClip), kPairClip));
            const float cm = (dd >= -kPairClip && dd <= kPairClip) ? 1.f : 0.f;
            wj[d] += (mq * scale * at(s.q, i, d) + mk * at(s.b, i, d) * at(s.k, i, d)) * ed *
                     at(s.k, j, d) * cm;
          }
        }
        for (int d = 0; d < D; ++d) {
          const size_t e = (size_t)j * D + d;
          g4[e] = san(g4[e] - wj[d], clip);
        }
      }
    }
  dq.resize((size_t)C * D); dk.resize((size_t)C * D); db.resize((size_t)C * D); dgc.resize((size_t)C * D);
  for (int i = 0; i < C; ++i)
    for (int d = 0; d < D; ++d) {
      const size_t e = (size_t)i * D + d;
      dq[e] = san(q4[e], clip);
      dk[e] = san(k4[e] + dbk[e] * at(s.b, i, d), clip);
      db[e] = san(dbk[e] * at(s.k, i, d), clip);
      dgc[e] = san(g4[e], clip);
    }
}

void backward(const Slice& s, const float* h0, const float* dhf, float* const* g, float* dh0,
              int T, int D, int C, int BC, float scale, float clip) {
  Fwd R;
  forward(s, h0, nullptr, nullptr, T, D, C, BC, scale, clip, R);
  const int nc = R.nc;
  auto at = [&](const float* x, int c, int i, int d) { return x[((long)c * C + i) * s.rs + d]; };
  // B2 (gdn2_bwd.py:84-96)
  std::vector<Mat> dAqk(nc), dvp(nc), dh_all(nc), dv_all(nc);
  for (int c = 0; c < nc; ++c) {
    Mat doc((size_t)C * D);
    for (int i = 0; i < C; ++i)
      for (int d = 0; d < D; ++d) doc[(size_t)i * D + d] = at(s.dout, c, i, d);
    Mat vT = tr(R.vnew[c].data(), C, D);
    dAqk[c].resize((size_t)C * C);
    mm(doc.data(), D, vT.data(), C, dAqk[c].data(), C, C, D, C);
    for (int i = 0; i < C; ++i)
      for (int j = 0; j < C; ++j) {
        float& x = dAqk[c][(size_t)i * C + j];
        x = j <= i ? san(x, clip) : 0.f;
      }
    Mat AT = tr(R.Aqk[c].data(), C, C);
    dvp[c].resize((size_t)C * D);
    mm(AT.data(), C, doc.data(), D, dvp[c].data(), D, C, C, D);
    for (auto& x : dvp[c]) x = san(x, clip);
  }
  // B1 (gdn2_bwd.py:45-80)
  Mat dh((size_t)D * D);
  for (size_t e = 0; e < dh.size(); ++e) dh[e] = san(dhf[e], clip);
  for (int c = nc - 1; c >= 0; --c) {
    Mat dvn((size_t)C * D);
    mm(R.kg[c].data(), D, dh.data(), D, dvn.data(), D, C, D, D);
    for (size_t e = 0; e < dvn.size(); ++e) dvn[e] = san(dvp[c][e] + dvn[e], clip);
    Mat qgT = tr(R.qg[c].data(), C, D), WT = tr(R.W[c].data(), C, D), doc((size_t)C * D);
    for (int i = 0; i < C; ++i)
      for (int d = 0; d < D; ++d) doc[(size_t)i * D + d] = scale * at(s.dout, c, i, d);
    Mat dhp((size_t)D * D), wt((size_t)D * D);
    mm(qgT.data(), C, doc.data(), D, dhp.data(), D, D, C, D);
    mm(WT.data(), C, dvn.data(), D, wt.data(), D, D, C, D);
    for (int d = 0; d < D; ++d) {
      const float dec = std::exp(R.gcl[c][d]);
      for (int v = 0; v < D; ++v) {
        const size_t e = (size_t)d * D + v;
        dh[e] = san(dhp[e] + dh[e] * dec - wt[e], clip);
      }
    }
    dh_all[c] = dh;
    dv_all[c] = dvn;
  }
  for (size_t e = 0; e < dh.size(); ++e) dh0[e] = san(dh[e], kFinalClip);
  // B3, B4, B5 and the assembly per chunk
  for (int c = 0; c < nc; ++c) {
    const Mat& dhn = (c + 1 < nc) ? dh_all[c + 1] : Mat(dhf, dhf + (size_t)D * D);
    const Mat& gc = R.gc[c];
    const Mat& hp = R.hpre[c];
    Mat eg((size_t)C * D), kbd((size_t)C * D), kgr((size_t)C * D), qgr((size_t)C * D),
        wvv((size_t)C * D), e2((size_t)C * D);
    for (int i = 0; i < C; ++i)
      for (int d = 0; d < D; ++d) {
        const size_t e = (size_t)i * D + d;
        eg[e] = std::exp(gc[e]);
        kbd[e] = at(s.b, c, i, d) * at(s.k, c, i, d) * eg[e];
        e2[e] = std::exp(gc[(size_t)(C - 1) * D + d] - gc[e]);
        kgr[e] = at(s.k, c, i, d) * e2[e];
        qgr[e] = at(s.q, c, i, d) * eg[e];
        wvv[e] = at(s.w, c, i, d) * at(s.v, c, i, d);
      }
    Mat doS((size_t)C * D), dvm((size_t)C * D);
    for (int i = 0; i < C; ++i)
      for (int d = 0; d < D; ++d) {
        doS[(size_t)i * D + d] = scale * at(s.dout, c, i, d);
        dvm[(size_t)i * D + d] = -dv_all[c][(size_t)i * D + d];
      }
    Mat hT = tr(hp.data(), D, D), dhT = tr(dhn.data(), D, D);
    Mat dqg((size_t)C * D), dWp((size_t)C * D), dkg((size_t)C * D);
    mm(doS.data(), D, hT.data(), D, dqg.data(), D, C, D, D);
    mm(dvm.data(), D, hT.data(), D, dWp.data(), D, C, D, D);
    mm(R.vnew[c].data(), D, dhT.data(), D, dkg.data(), D, C, D, D);
    Mat kbT = tr(kbd.data(), C, D), wvT = tr(wvv.data(), C, D), dA((size_t)C * C);
    mm(dWp.data(), D, kbT.data(), C, dA.data(), C, C, D, C);
    mm(dv_all[c].data(), D, wvT.data(), C, dA.data(), C, C, D, C, true);
    for (auto& x : dA) x = san(x, clip);
    const Mat& A = R.A[c];
    Mat AT = tr(A.data(), C, C), dkb((size_t)C * D), dwv((size_t)C * D), tmp((size_t)C * C),
        dAkk((size_t)C * C);
    mm(AT.data(), C, dWp.data(), D, dkb.data(), D, C, C, D);
    mm(AT.data(), C, dv_all[c].data(), D, dwv.data(), D, C, C, D);
    mm(dA.data(), C, AT.data(), C, tmp.data(), C, C, C, C);
    for (auto& x : tmp) x = san(x, clip);
    mm(AT.data(), C, tmp.data(), C, dAkk.data(), C, C, C, C);
    for (int i = 0; i < C; ++i)
      for (int j = 0; j < C; ++j) {
        float& x = dAkk[(size_t)i * C + j];
        x = j < i ? san(-x, clip) : 0.f;
      }
    Mat b3q((size_t)C * D), b3k((size_t)C * D), b3b((size_t)C * D), b3w((size_t)C * D),
        b3v((size_t)C * D), b3g((size_t)C * D);
    std::vector<float> dxs(D, 0.f), rowdot(D, 0.f);
    for (int d = 0; d < D; ++d)
      for (int v = 0; v < D; ++v) rowdot[d] += dhn[(size_t)d * D + v] * hp[(size_t)d * D + v];
    for (int i = 0; i < C; ++i)
      for (int d = 0; d < D; ++d) {
        const size_t e = (size_t)i * D + d;
        const float dx = dkg[e] * kgr[e];
        dxs[d] += dx;
        b3k[e] = dkb[e] * eg[e] * at(s.b, c, i, d) + dkg[e] * e2[e];
        b3b[e] = dkb[e] * eg[e] * at(s.k, c, i, d);
        b3g[e] = dkb[e] * kbd[e] + dqg[e] * qgr[e] - dx;
        b3q[e] = dqg[e] * eg[e];
        b3w[e] = dwv[e] * at(s.v, c, i, d);
        b3v[e] = dwv[e] * at(s.w, c, i, d);
      }
    for (int d = 0; d < D; ++d)
      b3g[(size_t)(C - 1) * D + d] += dxs[d] + std::exp(gc[(size_t)(C - 1) * D + d]) * rowdot[d];
    for (auto* m : {&b3q, &b3k, &b3b, &b3w, &b3v, &b3g})
      for (auto& x : *m) x = san(x, clip);
    Mat q4, k4, b4, g4;
    intra_backward(s, c, gc, dAqk[c], dAkk, C, D, BC, scale, clip, q4, k4, b4, g4);
    // B5 and the final sum (gdn2_bwd.py:32-41, gdn2_pipeline.py:117-135)
    std::vector<float> run(D, 0.f);
    for (int i = C - 1; i >= 0; --i)
      for (int d = 0; d < D; ++d) {
        const size_t e = (size_t)i * D + d;
        run[d] += b3g[e] + g4[e];
        g[5][((long)c * C + i) * s.rs + d] = san(san(run[d], clip), kFinalClip);
      }
    for (int i = 0; i < C; ++i)
      for (int d = 0; d < D; ++d) {
        const size_t e = (size_t)i * D + d;
        const long o = ((long)c * C + i) * s.rs + d;
        g[0][o] = san(b3q[e] + q4[e], kFinalClip);
        g[1][o] = san(b3k[e] + k4[e], kFinalClip);
        g[2][o] = san(b3v[e], kFinalClip);
        g[3][o] = san(b3w[e], kFinalClip);
        g[4][o] = san(b3b[e] + b4[e], kFinalClip);
      }
  }
}

}  // namespace

extern "C" {

// Forward (o, h_final) and, when dout != NULL, the backward (dq, dk, dv, dw,
// db, dg, dh0) of (B, T, H, D) float32 tensors; h0 may be NULL.  One OpenMP
// task per (batch, head); `threads` <= 0 uses the OpenMP default.
int gdn2_cpu_fwd_bwd(const float* q, const float* k, const float* v, const float* w,
                     const float* b, const float* g, const float* h0, const float* dout,
                     const float* dh_final, float* o, float* h_final, float* dq, float* dk,
                     float* dv, float* dw, float* db, float* dg, float* dh0, int B, int T, int H,
                     int D, int BT, int BC, float scale, float clip, int threads) {
  if (!q || !k || !v || !w || !b || !g || !o || !h_final) return -1;
  if (dout && (!dh_final || !dq || !dk || !dv || !dw || !db || !dg || !dh0)) return -1;
  if (B <= 0 || T <= 0 || H <= 0 || D <= 0 || BT <= 0 || T % BT || BC <= 0 || BT % BC) return -1;
  const long rs = (long)H * D;
  const int nt = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
  for (int bh = 0; bh < B * H; ++bh) {
    const int bb = bh / H, hh = bh % H;
    const long off = (long)bb * T * rs + (long)hh * D;
    const size_t so = (size_t)bh * D * D;
    Slice s{q + off, k + off, v + off, w + off, b + off, g + off, dout ? dout + off : nullptr, rs};
    Fwd R;
    forward(s, h0 ? h0 + so : nullptr, o + off, h_final + so, T, D, BT, BC, scale, clip, R);
    if (dout) {
      float* gp[6] = {dq + off, dk + off, dv + off, dw + off, db + off, dg + off};
      backward(s, h0 ? h0 + so : nullptr, dh_final + so, gp, dh0 + so, T, D, BT, BC, scale, clip);
    }
  }
  return 0;
}

}  // extern "C"
