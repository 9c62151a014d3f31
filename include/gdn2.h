/* libgdn2 — C ABI of the B200 (sm_100a) Gated DeltaNet-2 chunked kernels.
 *
 * Plain pointers and sizes only; every device buffer is owned by the caller
 * (the library never allocates or synchronises).  All entry points are
 * asynchronous on `stream` (a cudaStream_t, NULL = legacy default stream) and
 * return 0 on success or a negative GDN2_ERR_* code; gdn2_last_error() then
 * holds a one-line message for the calling thread.
 *
 * Tensor conventions (the reference's, Akseleu-J/gdn2-jax-kernel):
 *   q, k, v, w, b, g        (B, T, H, D) row-major, dtype GDN2_F32 or GDN2_BF16
 *   h0, h_final             (B, H, D, D) float32, row index = key dim
 *   o                       (B, T, H, D) float32          (gdn2_fwd.py:164-165)
 *   dout                    (B, T, H, D) float32 cotangent of o
 *   dh_final                (B, H, D, D) float32 cotangent of h_final
 *   dq, dk, dv, dw, db, dg  (B, T, H, D) in the input dtype (gdn2_pipeline.py:129-134)
 *   dh0                     (B, H, D, D) float32
 * BT is the chunk length (64 or 128), BC the reference's sub-block (a
 * multiple of MB = 16 dividing BT; it sets where the sanitisers of the WY
 * solve and of B4's accumulators act, so results depend on it only when CLIP
 * acts), D the head dim (64 or 128), clip the stage sanitiser bound CLIP
 * (gdn2_fwd.py:33, 42-44).
 */
#ifndef GDN2_H_
#define GDN2_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN2_ABI_VERSION 1

enum { GDN2_F32 = 0, GDN2_BF16 = 1 };
/* OR-ed into the dtype argument of gdn2_fwd / gdn2_bwd / gdn2_fwd_noalloc /
 * gdn2_decode: w, b, g are pre-activations and the kernels apply
 * w = sigmoid(w), b = sigmoid(b), g = -softplus(g) as they load them (the
 * activations the reference leaves to its caller, README.md:60-68).
 * gdn2_bwd then returns dw, db, dg with respect to the pre-activations.  The
 * same flag must be given to the forward and the backward of one step. */
#define GDN2_GATES_RAW 0x100
/* OR-ed into the dtype argument of gdn2_fwd / gdn2_bwd / gdn2_fwd_noalloc:
 * this call runs BT = 64 on the CUDA-core kernels even where
 * gdn2_pair64_enable() would pair chunks on the tensor cores (the forward
 * and the backward of one step must agree). */
#define GDN2_NO_PAIR 0x200
/* OR-ed into the dtype argument of gdn2_fwd (BT = D = 128 only, with
 * save_residuals = 1): the call forms the residuals and h_final but not the
 * chunk outputs, and `o` may be NULL.  For a segment whose outputs a
 * gdn2_sp_segment op 1 rescan forms afterwards (sequence parallelism, the
 * chunk-parallel scan on one GPU), which rewrites them in full. */
#define GDN2_NO_OUT 0x400
enum {
  GDN2_OK = 0,
  GDN2_ERR_INVALID = -1,   /* bad shape / argument (reference: AssertionError, gdn2_fwd.py:145-146) */
  GDN2_ERR_WORKSPACE = -2, /* workspace smaller than gdn2_workspace_bytes() */
  GDN2_ERR_CUDA = -3       /* a CUDA launch failed */
};

int gdn2_abi_version(void);
const char* gdn2_last_error(void);

/* Bytes of scratch the caller must provide.  with_backward = 0 sizes a plain
 * forward; with_backward = 1 sizes a forward that keeps residuals plus the
 * backward (one buffer serves both calls).  Returns 0 for invalid sizes. */
size_t gdn2_workspace_bytes(int B, int T, int H, int D, int BT, int with_backward);

/* Forward: replaces gdn2_pallas_forward(q,k,v,w,b,g,scale,h0) -> (o, h_final)
 * (gdn2_fwd.py:400-424; Kernels A-D at gdn2_fwd.py:142, 246, 298, 338).
 * h0 may be NULL (zero state, gdn2_fwd.py:403-404).  With save_residuals = 1
 * the per-chunk state and v_new stay in `workspace` (which must then be sized
 * with with_backward = 1) so gdn2_bwd can skip the forward recompute. */
int gdn2_fwd(int dtype, const void* q, const void* k, const void* v, const void* w,
             const void* b, const void* g, const float* h0, float* o, float* h_final,
             void* workspace, size_t workspace_bytes, int save_residuals, int B, int T, int H,
             int D, int BT, int BC, float scale, float clip, void* stream);

/* Backward of the custom_vjp: replaces _gdn2_core_bwd (gdn2_pipeline.py:70-137;
 * B1-B5 at gdn2_bwd.py:32, 45, 99, 213, 342).  residuals_valid = 0 recomputes
 * the forward from the inputs exactly as the reference does; 1 reuses the
 * residuals a gdn2_fwd(save_residuals=1) call left in the same workspace; 2
 * (BT = D = 128) also reuses the per-chunk backward terms of this same dout
 * that a gdn2_sp_segment op 2 call left there after those residuals.
 * h0 may be NULL; dh_final must be given (zeros for no cotangent). */
int gdn2_bwd(int dtype, const void* q, const void* k, const void* v, const void* w,
             const void* b, const void* g, const float* h0, const float* dout,
             const float* dh_final, void* dq, void* dk, void* dv, void* dw, void* db, void* dg,
             float* dh0, void* workspace, size_t workspace_bytes, int residuals_valid, int B,
             int T, int H, int D, int BT, int BC, float scale, float clip, void* stream);

/* Sequence-parallel building blocks (no single counterpart in the reference,
 * whose scan is serial over the whole sequence, gdn2_fwd.py:362): a rank that
 * owns a contiguous time segment uses them on the workspace of its segment.
 * Requires BT = D = 128.
 *   op 0: after gdn2_fwd(save_residuals = 1), out (B,H,D,D) = the segment map
 *         P = M_last ... M_first, where h_out = P h_in + c and c is the h_final
 *         of the segment run from a zero state;
 *   op 1: rescan the segment from start state `in` (B,H,D,D): rewrites the
 *         per-chunk residual states, o (may be NULL) and out = h_final;
 *   op 2: (backward workspace) out (B,H,D,D) = the gradient at the segment
 *         start for a zero incoming gradient, given dout = `in`.
 * The incoming gradient of a segment maps as g_start = P^T g_end + out. */
int gdn2_sp_segment(int op, void* workspace, size_t workspace_bytes, const float* in, float* o,
                    float* out, int B, int T, int H, int D, int BT, int BC, float scale,
                    float clip, void* stream);

/* Device status of the latest call on a workspace (no counterpart in the
 * reference, whose kernels have no device-side waits).  Every entry point
 * that takes a workspace clears its status header on `stream` before its
 * kernels run.  This call copies the header to the host, synchronizes
 * `stream` and returns a bit set, or a negative GDN2_ERR_* code:
 *   GDN2_STATUS_WAIT_TIMEOUT       a bounded barrier wait inside a kernel ran
 *                                  out of polls; the call's outputs are invalid;
 *   GDN2_STATUS_FWD_STATE_CLIPPED  the CLIP sanitiser acted on the state h in
 *                                  the tensor-core scan (exact for a whole
 *                                  sequence; breaks the linear segment maps of
 *                                  gdn2_sp_segment);
 *   GDN2_STATUS_BWD_STATE_CLIPPED  the same for the state gradient dh;
 *   GDN2_STATUS_EXACT_RECOMPUTE    some (b, h) could clip dv_new inside the
 *                                  backward chain and were recomputed with the
 *                                  reference's exact step (breaks the segment
 *                                  maps of gdn2_sp_segment; otherwise information);
 *   GDN2_STATUS_B4_EXACT           some chunk's B4 accumulators could reach CLIP
 *                                  and it ran the reference's sub-block pair
 *                                  order (information only). */
#define GDN2_STATUS_WAIT_TIMEOUT 1
#define GDN2_STATUS_FWD_STATE_CLIPPED 2
#define GDN2_STATUS_BWD_STATE_CLIPPED 4
#define GDN2_STATUS_EXACT_RECOMPUTE 8
#define GDN2_STATUS_B4_EXACT 16
int gdn2_workspace_status(const void* workspace, size_t workspace_bytes, void* stream);

/* Per-stage diagnostics of the forward (the reference's _stage_diag,
 * gdn2_fwd.py:47-76, enabled there by GDN2_FWD_DIAG=1).  While enabled
 * (process-wide), every forward kernel reduces, for each stage output, the
 * number of non-finite values and the largest finite |x| into the status
 * header of its workspace.  gdn2_diag_read() copies them to the host
 * (synchronizing `stream`) for stages 0 kernel_A_Aqk, 1 kernel_A_Akk,
 * 2 kernel_B_wy_inverse_A, 3 kernel_C_w_pseudo, 4 kernel_C_u, 5 kernel_C_kg,
 * 6 kernel_C_qg, 7 kernel_D_o, 8 kernel_D_h_final and returns the number of
 * stages (9).  Values describe the latest call on that workspace. */
int gdn2_diag_enable(int on);
/* BT = 64 with D = 128 on the tensor-core kernels: two chunks per 128-row
 * tile (block-diagonal chunk scores and WY solve, gates and gc_last per
 * chunk, one state step per chunk), the same function as the BT = 64
 * CUDA-core kernels.  Needs T % 128 == 0 (otherwise the CUDA-core kernels
 * run).  On by default; per call, GDN2_NO_PAIR opts out.  Process-wide: a
 * forward that kept residuals and its backward must run under the same
 * setting, so change it only between steps.  Returns the previous setting. */
int gdn2_pair64_enable(int on);
int gdn2_diag_read(const void* workspace, size_t workspace_bytes, void* stream, int n,
                   int* nonfinite, float* maxabs);

/* Forward for callers that cannot allocate device memory (no counterpart in
 * the reference).  Same arguments and results as gdn2_fwd without the
 * workspace: the scratch lives in a fixed device array of
 * GDN2_NOALLOC_SCRATCH_BYTES inside the library, present on every GPU that
 * loads it until the process exits.  Problems whose forward workspace
 * (gdn2_workspace_bytes(..., 0)) exceeds that size are rejected with
 * GDN2_ERR_WORKSPACE.  The first call on a device looks up the array's device
 * address (make that first call before any stream capture).  All calls share
 * the one array, so calls that overlap on the GPU (different streams or
 * threads without ordering) race with each other. */
#define GDN2_NOALLOC_SCRATCH_BYTES (64u << 20)
int gdn2_fwd_noalloc(int dtype, const void* q, const void* k, const void* v, const void* w,
                     const void* b, const void* g, const float* h0, float* o, float* h_final,
                     int B, int T, int H, int D, int BT, int BC, float scale, float clip,
                     void* stream);
/* gdn2_workspace_status() of the built-in scratch array on the current device:
 * the status of the latest gdn2_fwd_noalloc call there (synchronizes `stream`). */
int gdn2_noalloc_status(void* stream);

/* Copies one head group of a host batch shard to or from the device with a
 * single pitched DMA (the streamed host path, gdn2_fwd_bwd in the Python
 * package).  `host` points at row 0 of the shard in the caller's layout
 * [rows][H][head_bytes] (e.g. rows = batch rows x T for (B,T,H,D) tensors,
 * head_bytes = D x element size; rows = batch rows, head_bytes = D x D x 4
 * for (B,H,D,D) states); `dev` is the packed [rows][Hs][head_bytes] device
 * buffer of heads h0 .. h0+Hs-1.  to_device = 1 copies host -> dev, 0 copies
 * dev -> host.  Asynchronous on `stream` (pinned host memory for overlap). */
int gdn2_copy_heads(void* host, void* dev, long rows, int H, int h0, int Hs, size_t head_bytes,
                    int to_device, void* stream);

/* The reference's stage functions as separate entry points, on its chunked
 * layouts: (B, H, nc, BT, .) float32 tiles, gc_last (B, H, nc, D), inputs
 * q..g (B, T, H, D) of `dtype` where named; BT 64, 128 or 256; D 64, 128 or
 * 256 (D = 256 with BT <= 128).  The fused gdn2_fwd / gdn2_bwd never call
 * them.  Each replaces the reference function of the same name:
 *   gdn2_stage_scores        build_chunk_scores_pallas (gdn2_fwd.py:142-170)
 *   gdn2_stage_wy_solve      wy_solve_pallas (gdn2_fwd.py:246-260), any BC;
 *                            BT = 256 needs BC <= 128 and n_chunks*BC*BC
 *                            floats of scratch (NULL otherwise)
 *   gdn2_stage_recompute_wy  recompute_wy_pallas (gdn2_fwd.py:298-330)
 *   gdn2_stage_combine       gdn2_inter_chunk_combine(_with_state)
 *                            (gdn2_fwd.py:338-397); h_pre_all (nc,B,H,D,D) and
 *                            v_new_all (nc,B,H,BT,D) chunk-major, may be NULL
 *   gdn2_stage_dhu           gdn2_dhu_backward (gdn2_bwd.py:45-80)
 *   gdn2_stage_dav           dav_backward_pallas (gdn2_bwd.py:84-122)
 *   gdn2_stage_wy_dqkg       wy_dqkg_backward_pallas (gdn2_bwd.py:126-244);
 *                            scratch: n_chunks * BT * BT floats
 *   gdn2_stage_intra_bwd     intra_backward_pallas (gdn2_bwd.py:248-375);
 *                            dAqk / dAkk given transposed per chunk, zeros:
 *                            BT * D zero floats
 *   gdn2_stage_revcumsum     reverse_cumsum_bwd (gdn2_bwd.py:32-41) */
int gdn2_stage_scores(int dtype, const void* q, const void* k, const void* b, const void* g,
                      float* aqk, float* akk, int B, int T, int H, int D, int BT, float scale,
                      float clip, void* stream);
int gdn2_stage_wy_solve(const float* akk, float* a, float* scratch, int n_chunks, int BT, int BC,
                        float clip, void* stream);
int gdn2_stage_recompute_wy(int dtype, const void* q, const void* k, const void* v, const void* w,
                            const void* b, const void* g, const float* a, float* w_pseudo,
                            float* u, float* kg, float* qg, float* gc_last, int B, int T, int H,
                            int D, int BT, float clip, void* stream);
int gdn2_stage_combine(const float* aqk, const float* w_pseudo, const float* u, const float* kg,
                       const float* qg, const float* gc_last, const float* h0, float* o,
                       float* h_final, float* h_pre_all, float* v_new_all, int B, int H, int nc,
                       int BT, int D, float scale, float clip, void* stream);
int gdn2_stage_dhu(const float* dout, const float* dv_partial, const float* w_pseudo,
                   const float* qg, const float* kg, const float* gc_last, const float* dht,
                   float* dh_all, float* dh0, float* dv_all, int B, int H, int nc, int BT, int D,
                   float scale, float clip, void* stream);
int gdn2_stage_dav(const float* aqk, const float* v_new, const float* dout, float* daqk,
                   float* dv, int n_chunks, int BT, int D, float clip, void* stream);
int gdn2_stage_wy_dqkg(const float* q, const float* k, const float* b, const float* w,
                       const float* v, const float* gc, const float* a, const float* h_pre,
                       const float* v_new, const float* dout, const float* dv,
                       const float* dh_next, float* dq, float* dk, float* db, float* dw,
                       float* dv_raw, float* dgc, float* dakk, float* scratch, int n_chunks,
                       int BT, int D, float scale, float clip, void* stream);
int gdn2_stage_intra_bwd(int dtype, const float* daqkT, const float* dakkT, const void* q,
                         const void* k, const void* b, const void* g, const float* zeros,
                         float* dq, float* dk, float* db, float* dgc, int B, int T, int H, int D,
                         int BT, int BC, float scale, float clip, void* stream);
int gdn2_stage_revcumsum(const float* dgc, float* dg, int n_chunks, int BT, int D, float clip,
                         void* stream);

/* Token-by-token decode of a short segment (B, T, H, D), carrying the state
 * h0 (B,H,D,D, may be NULL = zero) to h_final: the recurrence of
 * gdn2_pallas_forward (gdn2_fwd.py:338-362, state API gdn2_fwd.py:400-404)
 * with chunks of one token, the CLIP sanitiser applied to o and to the state
 * after every token.  One CTA per (batch, head), no workspace; the cost is
 * linear in T with no chunk parallelism, so long prompts belong to gdn2_fwd. */
int gdn2_decode(int dtype, const void* q, const void* k, const void* v, const void* w,
                const void* b, const void* g, const float* h0, float* o, float* h_final, int B,
                int T, int H, int D, float scale, float clip, void* stream);

/* Per-launch device timing (test and benchmark support; no counterpart in the
 * reference).  When enabled, every kernel launch of gdn2_fwd / gdn2_bwd is
 * bracketed by CUDA events on its stream.  gdn2_profile_read() waits for the
 * recorded events and fills, per stage, the accumulated milliseconds and the
 * launch count (stages: 0 fwd_intra, 1 fwd_state, 2 bwd_state, 3 bwd_intra1,
 * 4 bwd_intra2, 5 bwd_intra3, 6 fwd_affine, 7 fwd_scan, 8 fwd_out, 9 bwd_prep,
 * 10 bwd_scan, 11 bwd_exact); it returns the number of stages. */
int gdn2_profile_enable(int on);
int gdn2_profile_read(int n, double* total_ms, long* launches, int reset);

/* Self-test of the tensor-core building block (no counterpart in the
 * reference): D[b] = A[b] (128 x K) * B[b] (K x N), float32 row-major device
 * arrays, computed with tcgen05 kind::tf32 in 3xTF32 form.  trans_a / trans_b pick
 * how each operand is staged (1 = through a 4x4 register transpose).
 * K % 32 == 0, N in {32, 64, ..., 256}.  *status (device int) receives 1 if a
 * barrier wait timed out. */
int gdn2_selftest_gemm_tf32x3(const float* A, const float* B, float* D, int batch, int K, int N,
                              int trans_a, int trans_b, int* status, void* stream);

/* Self-test of the failure path (no counterpart in the reference): clears the
 * status header of `workspace`, then one warp waits on a barrier that nothing
 * completes, giving up after `polls` polls.  The wait records its timeout in
 * the status word (read it with gdn2_workspace_status) and the kernel returns;
 * nothing else is in flight, so the context stays usable. */
int gdn2_selftest_wait_timeout(void* workspace, size_t workspace_bytes, int polls, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GDN2_H_ */
