// gdn2_fwd_noalloc: the forward for callers that must not allocate device
// memory themselves — e.g. code running inside a framework that owns every
// allocation (a custom-call handler that was not given a scratch buffer), or
// a caller whose allocator is unavailable at that point.  The workspace the
// forward needs comes from one fixed-size device array compiled into the
// library instead of from the caller.
#include <stdio.h>


#include "../../include/gdn2.h"

namespace gdn2 {
int report_error(int code, const char* msg);
}

namespace {

constexpr size_t kScratchBytes = GDN2_NOALLOC_SCRATCH_BYTES;

// The scratch: one per device, kept for the life of the process.  Host code
// must not pass this name to a kernel (on the host it is only a stand-in);
// its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// Device address of the scratch on the current device.  Looked up on every
// call (cheap), so the address stays valid across a cudaDeviceReset or a new
// context on the device.
int scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p) {
    char msg[256];
    snprintf(msg, sizeof(msg), "gdn2_fwd_noalloc: cudaGetSymbolAddress failed: %s",
             cudaGetErrorString(e));
    return gdn2::report_error(GDN2_ERR_CUDA, msg);
  }
  *out = p;
  return GDN2_OK;
}

}  // namespace

extern "C" int gdn2_fwd_noalloc(int dtype, const void* q, const void* k, const void* v,
                                const void* w, const void* b, const void* g, const float* h0,
                                float* o, float* h_final, int B, int T, int H, int D, int BT,
                                int BC, float scale, float clip, void* stream) {
  const size_t need = gdn2_workspace_bytes(B, T, H, D, BT, 0);
  if (need == 0)
    return gdn2::report_error(GDN2_ERR_INVALID, "gdn2_fwd_noalloc: invalid problem sizes");
  if (need > kScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "gdn2_fwd_noalloc: problem needs %zu bytes of scratch, the built-in limit is %zu "
             "(use gdn2_fwd with a caller workspace)", need, kScratchBytes);
    return gdn2::report_error(GDN2_ERR_WORKSPACE, msg);
  }
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  // The forward writes every workspace tile before reading it, and gdn2_fwd
  // clears the status header first, so the previous call's contents need no
  // other clearing.
  return gdn2_fwd(dtype, q, k, v, w, b, g, h0, o, h_final, scratch, kScratchBytes,
                  /*save_residuals=*/0, B, T, H, D, BT, BC, scale, clip, stream);
}

extern "C" int gdn2_noalloc_status(void* stream) {
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  return gdn2_workspace_status(scratch, kScratchBytes, stream);
}
