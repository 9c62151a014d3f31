// C-ABI entry points of libgdn2 (declared in include/gdn2.h).
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "../../include/gdn2.h"
#include "gdn2_kernels.cuh"

using namespace gdn2;

namespace {

thread_local char g_err[512] = "";

// Optional per-launch timing: when enabled, every kernel launch is bracketed by
// CUDA events recorded on its own stream; gdn2_profile_read() resolves them.
struct Profiler {
  bool on = false;
  struct Rec { int stage; cudaEvent_t a, b; };
  std::vector<Rec> recs;
  cudaEvent_t pending[kNumStages] = {};
  double total_ms[kNumStages] = {};
  long count[kNumStages] = {};
};
Profiler g_prof;
std::mutex g_prof_mu;
int g_diag = 0;   // per-stage diagnostics on (gdn2_diag_enable)
std::atomic<int> g_pair64{1};  // BT = 64 chunks paired into 128-row tiles (gdn2_pair64_enable)

void prof_hook(int stage, int end, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_prof.on) return;
  cudaEvent_t ev;
  if (cudaEventCreate(&ev) != cudaSuccess) return;
  cudaEventRecord(ev, s);
  if (!end) {
    g_prof.pending[stage] = ev;
  } else if (g_prof.pending[stage]) {
    g_prof.recs.push_back({stage, g_prof.pending[stage], ev});
    g_prof.pending[stage] = nullptr;
  } else {
    cudaEventDestroy(ev);
  }
}

LaunchHook hook() {
  LaunchHook h;
  h.fn = prof_hook;
  return h;
}

int fail(int code, const char* fmt, const char* a = "", long x = 0, long y = 0) {
  snprintf(g_err, sizeof(g_err), fmt, a, x, y);
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  snprintf(g_err, sizeof(g_err), "%s: %s", where, cudaGetErrorString(e));
  return GDN2_ERR_CUDA;
}

int validate(int dtype, int B, int T, int H, int D, int BT, int BC, float scale, float clip) {
  dtype &= ~(GDN2_GATES_RAW | GDN2_NO_PAIR | GDN2_NO_OUT);
  if (dtype != GDN2_F32 && dtype != GDN2_BF16)
    return fail(GDN2_ERR_INVALID, "unsupported dtype code %s%ld", "", dtype);
  if (B <= 0 || T <= 0 || H <= 0)
    return fail(GDN2_ERR_INVALID, "%sempty problem B*T*H (T=%ld, H=%ld)", "", T, H);
  if (D != 64 && D != 128)
    return fail(GDN2_ERR_INVALID, "%shead dim D=%ld unsupported (64 or 128)", "", D);
  if (BT != 64 && BT != 128)
    return fail(GDN2_ERR_INVALID, "%schunk BT=%ld unsupported (64 or 128)", "", BT);
  if (T % BT != 0)
    return fail(GDN2_ERR_INVALID, "%sT=%ld must be divisible by BT=%ld", "", T, BT);
  if (BC <= 0 || BT % BC != 0)
    return fail(GDN2_ERR_INVALID, "%ssub-block BC=%ld must divide BT=%ld", "", BC, BT);
  // the reference's block solve runs MB = 16 micro-blocks inside each BC
  // sub-block (gdn2_fwd.py:32, 194)
  if (BC % 16 != 0)
    return fail(GDN2_ERR_INVALID, "%ssub-block BC=%ld must be a multiple of MB=16", "", BC);
  if (!(clip > 0.f)) return fail(GDN2_ERR_INVALID, "%sclip must be positive");
  if (scale != scale) return fail(GDN2_ERR_INVALID, "%sscale is NaN");
  return GDN2_OK;
}

template <typename T>
int run_fwd_intra(int BT, int D, const void* q, const void* k, const void* v, const void* w,
                  const void* b, const void* g, const Problem& p, const Workspace& ws,
                  cudaStream_t s) {
  auto c = [](const void* x) { return static_cast<const T*>(x); };
  cudaError_t e;
  hook().begin(kStageFwdIntra, s);
  if (BT == 128 && D == 128) {
    e = launch_tc_fwd_intra<T>(c(q), c(k), c(v), c(w), c(b), c(g), p, ws, s);
    hook().end(kStageFwdIntra, s);
    return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "tc_fwd_intra");
  }
#define GDN2_CASE(CC, DD)                                                                  \
  if (BT == CC && D == DD)                                                                  \
    e = launch_fwd_intra<T, CC, DD>(c(q), c(k), c(v), c(w), c(b), c(g), p, ws, s);          \
  else
  GDN2_FOR_SHAPES(GDN2_CASE) return fail(GDN2_ERR_INVALID, "%sno kernel for this shape");
#undef GDN2_CASE
  hook().end(kStageFwdIntra, s);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "fwd_intra");
}

int run_fwd_state(int BT, int D, const Problem& p, const Workspace& ws, const float* h0, float* o,
                  float* hf, int save, cudaStream_t s) {
  cudaError_t e;
  hook().begin(kStageFwdState, s);
#define GDN2_CASE(CC, DD)                                                                  \
  if (BT == CC && D == DD) e = launch_fwd_state<CC, DD>(p, ws, h0, o, hf, save, s); else
  GDN2_FOR_SHAPES(GDN2_CASE) return fail(GDN2_ERR_INVALID, "%sno kernel for this shape");
#undef GDN2_CASE
  hook().end(kStageFwdState, s);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "fwd_state");
}

int run_bwd_state(int BT, int D, const Problem& p, const Workspace& ws, const float* dout,
                  const float* dhf, float* dh0, cudaStream_t s) {
  cudaError_t e;
  hook().begin(kStageBwdState, s);
#define GDN2_CASE(CC, DD)                                                                  \
  if (BT == CC && D == DD) e = launch_bwd_state<CC, DD>(p, ws, dout, dhf, dh0, s); else
  GDN2_FOR_SHAPES(GDN2_CASE) return fail(GDN2_ERR_INVALID, "%sno kernel for this shape");
#undef GDN2_CASE
  hook().end(kStageBwdState, s);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "bwd_state");
}

template <typename T>
int run_bwd_intra(int BT, int D, const void* q, const void* k, const void* v, const void* w,
                  const void* b, const void* g, const float* dout, const float* dhf, void* dq,
                  void* dk, void* dv, void* dw, void* db, void* dg, const Problem& p,
                  const Workspace& ws, cudaStream_t s) {
  auto c = [](const void* x) { return static_cast<const T*>(x); };
  auto m = [](void* x) { return static_cast<T*>(x); };
  cudaError_t e;
  const bool tc = BT == 128 && D == 128;
  if (tc) {
    e = launch_tc_bwd_intra12<T>(c(q), c(k), c(v), c(w), c(b), dout, dhf, m(dv), m(dw), p, ws,
                                 s, hook());
    if (e != cudaSuccess) return cuda_fail(e, "tc_bwd_intra");
    e = launch_tc_bwd_intra3<T>(c(q), c(k), c(b), c(g), m(dq), m(dk), m(db), m(dg), p, ws, s,
                                hook());
    return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "tc_bwd_intra3");
  }
#define GDN2_CASE(CC, DD)                                                                  \
  if (BT == CC && D == DD)                                                                  \
    e = launch_bwd_intra<T, CC, DD>(c(q), c(k), c(v), c(w), c(b), c(g), dout, dhf, m(dq),   \
                                    m(dk), m(dv), m(dw), m(db), m(dg), p, ws, s, hook(),    \
                                    tc);                                                    \
  else
  GDN2_FOR_SHAPES(GDN2_CASE) return fail(GDN2_ERR_INVALID, "%sno kernel for this shape");
#undef GDN2_CASE
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "bwd_intra");
}

// Chunk = head dim = 128 runs the inter-chunk recurrence on the tensor cores
// (affine scan, gdn2_tc_kernels.cu); other shapes use the CUDA-core kernels.
bool use_tc(int BT, int D) { return BT == 128 && D == 128; }
// BT = 64 with D = 128 runs on the tensor-core kernels with two chunks per
// 128-row tile (block-diagonal scores and solve, per-chunk gates, a state
// step per chunk) when T is a multiple of 128.
bool use_pair64(int T, int D, int BT) { return g_pair64 && BT == 64 && D == 128 && T % 128 == 0; }

// Every entry point clears the status header of its workspace first, so the
// word gdn2_workspace_status() reads belongs to the latest call.
int clear_status(const Workspace& ws, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(ws.status, 0, 256, s);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "status reset");
}

Problem make_problem(int B, int T, int H, int D, int BT, int BC, float scale, float clip) {
  Problem p;
  p.B = B; p.T = T; p.H = H; p.D = D; p.C = BT; p.nc = T / BT; p.bc = BC;
  p.diag = g_diag;
  p.gates = 0;
  p.sub = 1;
  p.scale = scale; p.clip = clip;
  return p;
}

}  // namespace

namespace gdn2 {
// Lets other translation units of the library report a message through
// gdn2_last_error().
int report_error(int code, const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}
}  // namespace gdn2

// Byte offset of the status header inside a caller workspace (the first
// 256-byte boundary at or after its start, as Workspace::carve places it).
size_t gdn2_status_offset(const void* workspace) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(workspace);
  return (size_t)(((a + 255) & ~(uintptr_t)255) - a);
}

extern "C" {

int gdn2_diag_enable(int on) {
  g_diag = on != 0;
  return GDN2_OK;
}

int gdn2_pair64_enable(int on) {
  return g_pair64.exchange(on != 0 ? 1 : 0);
}

int gdn2_diag_read(const void* workspace, size_t workspace_bytes, void* stream, int n,
                   int* nonfinite, float* maxabs) {
  if (!workspace || workspace_bytes < 512 || n < 0 || n > kNumDiag)
    return fail(GDN2_ERR_INVALID, "%sgdn2_diag_read: bad workspace or stage count");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int* hdr = reinterpret_cast<const int*>(static_cast<const char*>(workspace) +
                                                gdn2_status_offset(workspace));
  int host[2 * kNumDiag];
  cudaError_t e = cudaMemcpyAsync(host, hdr + kDiagBase, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "gdn2_diag_read");
  for (int i = 0; i < n; ++i) {
    if (nonfinite) nonfinite[i] = host[2 * i];
    if (maxabs) {
      int bits = host[2 * i + 1];
      memcpy(&maxabs[i], &bits, sizeof(float));
    }
  }
  return kNumDiag;
}

int gdn2_workspace_status(const void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < 512)
    return fail(GDN2_ERR_INVALID, "%sgdn2_workspace_status: null or undersized workspace");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int* st = reinterpret_cast<const int*>(static_cast<const char*>(workspace) +
                                               gdn2_status_offset(workspace));
  int host[5] = {0, 0, 0, 0, 0};
  cudaError_t e = cudaMemcpyAsync(host, st, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "gdn2_workspace_status");
  return (host[0] ? GDN2_STATUS_WAIT_TIMEOUT : 0) | (host[1] ? GDN2_STATUS_FWD_STATE_CLIPPED : 0) |
         (host[2] ? GDN2_STATUS_BWD_STATE_CLIPPED : 0) | (host[3] ? GDN2_STATUS_EXACT_RECOMPUTE : 0) |
         (host[4] ? GDN2_STATUS_B4_EXACT : 0);
}

int gdn2_copy_heads(void* host, void* dev, long rows, int H, int h0, int Hs, size_t head_bytes,
                    int to_device, void* stream) {
  if (!host || !dev || rows < 0 || H <= 0 || Hs <= 0 || h0 < 0 || h0 + Hs > H || head_bytes == 0)
    return fail(GDN2_ERR_INVALID, "%sgdn2_copy_heads: bad pointers or head range");
  if (rows == 0) return GDN2_OK;
  char* hp = static_cast<char*>(host) + (size_t)h0 * head_bytes;
  const size_t hpitch = (size_t)H * head_bytes, dpitch = (size_t)Hs * head_bytes;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      to_device ? cudaMemcpy2DAsync(dev, dpitch, hp, hpitch, dpitch, (size_t)rows,
                                    cudaMemcpyHostToDevice, s)
                : cudaMemcpy2DAsync(hp, hpitch, dev, dpitch, dpitch, (size_t)rows,
                                    cudaMemcpyDeviceToHost, s);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_copy_heads");
}

int gdn2_abi_version(void) { return GDN2_ABI_VERSION; }

int gdn2_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof.on = on != 0;
  return GDN2_OK;
}

int gdn2_profile_read(int n, double* total_ms, long* launches, int reset) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto& r : g_prof.recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      g_prof.total_ms[r.stage] += ms;
      g_prof.count[r.stage] += 1;
    }
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  g_prof.recs.clear();
  for (int i = 0; i < n && i < kNumStages; ++i) {
    if (total_ms) total_ms[i] = g_prof.total_ms[i];
    if (launches) launches[i] = g_prof.count[i];
  }
  if (reset)
    for (int i = 0; i < kNumStages; ++i) { g_prof.total_ms[i] = 0; g_prof.count[i] = 0; }
  return kNumStages;
}

const char* gdn2_last_error(void) { return g_err; }

size_t gdn2_workspace_bytes(int B, int T, int H, int D, int BT, int with_backward) {
  if (B <= 0 || T <= 0 || H <= 0 || D <= 0 || BT <= 0 || T % BT) return 0;
  size_t n = Workspace::required_bytes(B, H, T / BT, BT, D, with_backward != 0);
  // BT = 64, D = 128: enough for either kernel family, so the answer does
  // not depend on gdn2_pair64_enable
  if (BT == 64 && D == 128 && T % 128 == 0) {
    const size_t m = Workspace::required_bytes(B, H, T / 128, 128, D, with_backward != 0, 2);
    if (m > n) n = m;
  }
  return n;
}

int gdn2_fwd(int dtype, const void* q, const void* k, const void* v, const void* w,
             const void* b, const void* g, const float* h0, float* o, float* h_final,
             void* workspace, size_t workspace_bytes, int save_residuals, int B, int T, int H,
             int D, int BT, int BC, float scale, float clip, void* stream) {
  int rc = validate(dtype, B, T, H, D, BT, BC, scale, clip);
  if (rc) return rc;
  const bool no_out = (dtype & GDN2_NO_OUT) != 0;
  if (!q || !k || !v || !w || !b || !g || (!o && !no_out) || !h_final || !workspace)
    return fail(GDN2_ERR_INVALID, "%snull buffer pointer");
  if (no_out && (!use_tc(BT, D) || !save_residuals))
    return fail(GDN2_ERR_INVALID, "%sGDN2_NO_OUT needs BT = D = 128 and save_residuals");
  const size_t need = gdn2_workspace_bytes(B, T, H, D, BT, 0);
  if (workspace_bytes < need)
    return fail(GDN2_ERR_WORKSPACE, "%sworkspace too small: need %ld bytes, got %ld", "",
                (long)need, (long)workspace_bytes);
  const bool pair = use_pair64(T, D, BT) && !(dtype & GDN2_NO_PAIR);
  const int KT = pair ? 128 : BT;   // kernel tile rows
  Problem p = make_problem(B, T, H, D, KT, BC, scale, clip);
  p.sub = pair ? 2 : 1;
  p.gates = (dtype & GDN2_GATES_RAW) != 0;
  dtype &= ~(GDN2_GATES_RAW | GDN2_NO_PAIR | GDN2_NO_OUT);
  const Workspace ws = Workspace::carve(workspace, B, H, p.nc, KT, D, false, p.sub);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = clear_status(ws, s))) return rc;
  rc = dtype == GDN2_F32
           ? run_fwd_intra<float>(KT, D, q, k, v, w, b, g, p, ws, s)
           : run_fwd_intra<__nv_bfloat16>(KT, D, q, k, v, w, b, g, p, ws, s);
  if (rc) return rc;
  if (use_tc(KT, D)) {
    cudaError_t e = launch_tc_fwd(p, ws, h0, o, h_final, s, hook(), !no_out);
    return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "tc_fwd");
  }
  return run_fwd_state(BT, D, p, ws, h0, o, h_final, save_residuals, s);
}

int gdn2_bwd(int dtype, const void* q, const void* k, const void* v, const void* w,
             const void* b, const void* g, const float* h0, const float* dout,
             const float* dh_final, void* dq, void* dk, void* dv, void* dw, void* db, void* dg,
             float* dh0, void* workspace, size_t workspace_bytes, int residuals_valid, int B,
             int T, int H, int D, int BT, int BC, float scale, float clip, void* stream) {
  int rc = validate(dtype, B, T, H, D, BT, BC, scale, clip);
  if (rc) return rc;
  if (!q || !k || !v || !w || !b || !g || !dout || !dh_final || !dq || !dk || !dv || !dw || !db || !dg ||
      !dh0 || !workspace)
    return fail(GDN2_ERR_INVALID, "%snull buffer pointer");
  const size_t need = gdn2_workspace_bytes(B, T, H, D, BT, 1);
  if (workspace_bytes < need)
    return fail(GDN2_ERR_WORKSPACE, "%sworkspace too small: need %ld bytes, got %ld", "",
                (long)need, (long)workspace_bytes);
  // the same kernel family as the forward that left the residuals
  const bool pair = use_pair64(T, D, BT) && !(dtype & GDN2_NO_PAIR);
  const int KT = pair ? 128 : BT;   // kernel tile rows
  Problem p = make_problem(B, T, H, D, KT, BC, scale, clip);
  p.sub = pair ? 2 : 1;
  p.gates = (dtype & GDN2_GATES_RAW) != 0;
  dtype &= ~(GDN2_GATES_RAW | GDN2_NO_PAIR);
  const Workspace ws = Workspace::carve(workspace, B, H, p.nc, KT, D, true, p.sub);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = clear_status(ws, s))) return rc;
  if (!residuals_valid) {
    // The reference's custom_vjp keeps only the inputs and recomputes the
    // forward in the backward (gdn2_pipeline.py:64-83); o is not needed.
    rc = dtype == GDN2_F32
             ? run_fwd_intra<float>(KT, D, q, k, v, w, b, g, p, ws, s)
             : run_fwd_intra<__nv_bfloat16>(KT, D, q, k, v, w, b, g, p, ws, s);
    if (rc) return rc;
    if (use_tc(KT, D)) {
      cudaError_t e = launch_tc_fwd(p, ws, h0, nullptr, nullptr, s, hook());
      if (e != cudaSuccess) return cuda_fail(e, "tc_fwd");
    } else {
      rc = run_fwd_state(KT, D, p, ws, h0, nullptr, nullptr, 1, s);
      if (rc) return rc;
    }
  }
  if (use_tc(KT, D)) {
    // residuals_valid == 2: the bwd_prep terms of this dout are in place
    // (gdn2_sp_segment op 2 formed them from the same residuals)
    cudaError_t e = launch_tc_bwd_state(p, ws, dout, dh_final, dh0, s, hook(),
                                        residuals_valid != 2 || p.sub != 1);
    if (e != cudaSuccess) return cuda_fail(e, "tc_bwd_state");
  } else {
    rc = run_bwd_state(KT, D, p, ws, dout, dh_final, dh0, s);
    if (rc) return rc;
  }
  return dtype == GDN2_F32
             ? run_bwd_intra<float>(KT, D, q, k, v, w, b, g, dout, dh_final, dq, dk, dv, dw,
                                    db, dg, p, ws, s)
             : run_bwd_intra<__nv_bfloat16>(KT, D, q, k, v, w, b, g, dout, dh_final, dq, dk,
                                            dv, dw, db, dg, p, ws, s);
}

int gdn2_sp_segment(int op, void* workspace, size_t workspace_bytes, const float* in, float* o,
                    float* out, int B, int T, int H, int D, int BT, int BC, float scale,
                    float clip, void* stream) {
  int rc = validate(GDN2_F32, B, T, H, D, BT, BC, scale, clip);
  if (rc) return rc;
  if (!use_tc(BT, D))
    return fail(GDN2_ERR_INVALID, "%ssequence parallelism needs BT = D = 128");
  if (op < 0 || op > 2) return fail(GDN2_ERR_INVALID, "%sunknown segment op %ld", "", op);
  if (!workspace || !out || (op == 2 && !in))
    return fail(GDN2_ERR_INVALID, "%snull buffer pointer");
  const bool bwd = op == 2;
  const size_t need = gdn2_workspace_bytes(B, T, H, D, BT, bwd ? 1 : 0);
  if (workspace_bytes < need)
    return fail(GDN2_ERR_WORKSPACE, "%sworkspace too small: need %ld bytes, got %ld", "",
                (long)need, (long)workspace_bytes);
  const Problem p = make_problem(B, T, H, D, BT, BC, scale, clip);
  const Workspace ws = Workspace::carve(workspace, B, H, p.nc, BT, D, bwd);
  if ((rc = clear_status(ws, static_cast<cudaStream_t>(stream)))) return rc;
  cudaError_t e = launch_tc_sp(op, p, ws, in, o, out, static_cast<cudaStream_t>(stream), hook());
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "sp_segment");
}

}  // extern "C"
