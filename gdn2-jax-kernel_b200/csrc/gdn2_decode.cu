// Token-by-token decode of short segments: the recurrence of the chunked
// forward (gdn2_fwd.py:338-362) with chunks of one token, for inference that
// carries a state h0 -> h_final across calls (the state API of
// gdn2_fwd.py:400-404).  With a single-token chunk the WY form reduces to
//     S~ = diag(e^{g_t}) S,   vnew = w_t v_t - S~^T (b_t k_t),
//     S  = san(S~ + k_t vnew^T),   o_t = san(scale S_unsanitised^T q_t),
// the sanitiser acting after every token as it acts after every chunk.
//
// Every value column of S evolves independently, so one CTA per (batch,
// head) runs one thread per column with that column of S in registers; the
// token vectors q, b k, e^g go through shared memory.  No workspace.
#include "../../include/gdn2.h"
#include "gdn2_kernels.cuh"

namespace gdn2 {
int report_error(int code, const char* msg);

namespace {

template <typename T, int D>
__global__ void __launch_bounds__(D)
k_decode(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
         const T* __restrict__ w, const T* __restrict__ b, const T* __restrict__ g,
         const float* __restrict__ h0, float* __restrict__ o, float* __restrict__ hf, int T_,
         int H, float scale, float clip) {
  __shared__ float sq[D], sk[D], sbk[D], seg[D];
  const int bh = blockIdx.x, h = bh % H, bb = bh / H, col = threadIdx.x;
  float s[D];   // S[:, col]
  const float* hs = h0 ? h0 + (size_t)bh * D * D : nullptr;
#pragma unroll
  for (int d = 0; d < D; ++d) s[d] = hs ? san(hs[d * D + col], clip) : 0.f;
  for (int t = 0; t < T_; ++t) {
    const size_t off = (((size_t)bb * T_ + t) * H + h) * D;
    const float kv = to_f<T>(k[off + col]);
    sq[col] = to_f<T>(q[off + col]);
    sk[col] = kv;
    sbk[col] = to_f<T>(b[off + col]) * kv;
    seg[col] = __expf(to_f<T>(g[off + col]));
    const float wv = to_f<T>(w[off + col]) * to_f<T>(v[off + col]);
    __syncthreads();
    // four partial sums per dot product: shorter dependency chains
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int d = 0; d < D; d += 4) {
      s[d] *= seg[d];
      s[d + 1] *= seg[d + 1];
      s[d + 2] *= seg[d + 2];
      s[d + 3] *= seg[d + 3];
      a0 = fmaf(sbk[d], s[d], a0);
      a1 = fmaf(sbk[d + 1], s[d + 1], a1);
      a2 = fmaf(sbk[d + 2], s[d + 2], a2);
      a3 = fmaf(sbk[d + 3], s[d + 3], a3);
    }
    const float vn = wv - ((a0 + a1) + (a2 + a3));
    a0 = a1 = a2 = a3 = 0.f;
#pragma unroll
    for (int d = 0; d < D; d += 4) {
      s[d] = fmaf(sk[d], vn, s[d]);
      s[d + 1] = fmaf(sk[d + 1], vn, s[d + 1]);
      s[d + 2] = fmaf(sk[d + 2], vn, s[d + 2]);
      s[d + 3] = fmaf(sk[d + 3], vn, s[d + 3]);
      a0 = fmaf(sq[d], s[d], a0);
      a1 = fmaf(sq[d + 1], s[d + 1], a1);
      a2 = fmaf(sq[d + 2], s[d + 2], a2);
      a3 = fmaf(sq[d + 3], s[d + 3], a3);
    }
    o[off + col] = san(scale * ((a0 + a1) + (a2 + a3)), clip);
#pragma unroll
    for (int d = 0; d < D; ++d) s[d] = san(s[d], clip);
    __syncthreads();   // token vectors are rewritten next iteration
  }
  float* out = hf + (size_t)bh * D * D;
#pragma unroll
  for (int d = 0; d < D; ++d) out[d * D + col] = s[d];
}

template <typename T, int D>
cudaError_t launch(const void* q, const void* k, const void* v, const void* w, const void* b,
                   const void* g, const float* h0, float* o, float* hf, int B, int T_, int H,
                   float scale, float clip, cudaStream_t s) {
  auto c = [](const void* x) { return static_cast<const T*>(x); };
  k_decode<T, D><<<(unsigned)(B * H), D, 0, s>>>(c(q), c(k), c(v), c(w), c(b), c(g), h0, o, hf,
                                                  T_, H, scale, clip);
  return cudaGetLastError();
}

}  // namespace
}  // namespace gdn2

extern "C" int gdn2_decode(int dtype, const void* q, const void* k, const void* v, const void* w,
                           const void* b, const void* g, const float* h0, float* o,
                           float* h_final, int B, int T, int H, int D, float scale, float clip,
                           void* stream) {
  using namespace gdn2;
  if (dtype != GDN2_F32 && dtype != GDN2_BF16)
    return report_error(GDN2_ERR_INVALID, "gdn2_decode: unsupported dtype code");
  if (B <= 0 || T <= 0 || H <= 0)
    return report_error(GDN2_ERR_INVALID, "gdn2_decode: empty problem B*T*H");
  if (D != 64 && D != 128)
    return report_error(GDN2_ERR_INVALID, "gdn2_decode: head dim D unsupported (64 or 128)");
  if (!(clip > 0.f) || scale != scale)
    return report_error(GDN2_ERR_INVALID, "gdn2_decode: clip must be positive, scale finite");
  if (!q || !k || !v || !w || !b || !g || !o || !h_final)
    return report_error(GDN2_ERR_INVALID, "gdn2_decode: null buffer pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == GDN2_F32)
    e = D == 128 ? launch<float, 128>(q, k, v, w, b, g, h0, o, h_final, B, T, H, scale, clip, s)
                 : launch<float, 64>(q, k, v, w, b, g, h0, o, h_final, B, T, H, scale, clip, s);
  else
    e = D == 128
            ? launch<__nv_bfloat16, 128>(q, k, v, w, b, g, h0, o, h_final, B, T, H, scale, clip, s)
            : launch<__nv_bfloat16, 64>(q, k, v, w, b, g, h0, o, h_final, B, T, H, scale, clip, s);
  if (e != cudaSuccess) return report_error(GDN2_ERR_CUDA, cudaGetErrorString(e));
  return GDN2_OK;
}
