// Token-by-token decode of short segments: the chunked forward
// (gdn2_fwd.py:264-362) with chunks of one token, for inference that carries a
// state h0 -> h_final across calls (the state API of gdn2_fwd.py:400-404).
// With a single-token chunk the WY form reduces to A = san(1), gc = gc_last = g
// and W = san(A b k e^g), U = san(A w v), kg = san(k), qg = san(q e^g),
//     Aqk = san(scale q . k),  vnew = U - W^T h,
//     o = san(scale qg^T h + Aqk vnew),  h <- san(e^{san(g)} h + kg vnew),
// every sanitiser where the chunked kernels apply it (Kernels A, C, D).
//
// Every value column of h evolves independently, so one CTA per (batch,
// head) runs one thread per column with that column of h in registers; the
// token vectors W, qg, kg, e^{gc_last} go through shared memory.  No workspace.
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
         int H, float scale, float clip, int gates) {
  __shared__ float sW[D], sqg[D], skg[D], sdec[D], red[D / 32];
  const int bh = blockIdx.x, h = bh % H, bb = bh / H, col = threadIdx.x;
  const int lane = col & 31, warp = col >> 5;
  const float a1 = san(1.f, clip);   // A = (I + Akk)^-1 of a one-token chunk, sanitised
  float s[D];   // h[:, col]
  const float* hs = h0 ? h0 + (size_t)bh * D * D : nullptr;
#pragma unroll
  for (int d = 0; d < D; ++d) s[d] = hs ? san(hs[d * D + col], clip) : 0.f;
  for (int t = 0; t < T_; ++t) {
    const size_t off = (((size_t)bb * T_ + t) * H + h) * D;
    const float qv = to_f<T>(q[off + col]), kv = to_f<T>(k[off + col]);
    const float gv = ld_gate<T>(g + off + col, gates, kGateG);
    const float eg = expf(gv);
    sW[col] = san(a1 * (ld_gate<T>(b + off + col, gates, kGateB) * kv * eg), clip);
    sqg[col] = san(qv * eg, clip);
    skg[col] = san(kv, clip);
    sdec[col] = expf(san(gv, clip));
    const float u = san(a1 * (ld_gate<T>(w + off + col, gates, kGateW) * to_f<T>(v[off + col])), clip);
    // Aqk = san(scale q . k): block reduction in a fixed order
    float qk = qv * kv;
#pragma unroll
    for (int o_ = 16; o_; o_ >>= 1) qk += __shfl_xor_sync(0xffffffffu, qk, o_);
    if (lane == 0) red[warp] = qk;
    __syncthreads();
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) dot += red[i];
    const float aqk = san(scale * dot, clip);
    // four partial sums per dot product: shorter dependency chains
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
    for (int d = 0; d < D; d += 4) {
      a0 = fmaf(sW[d], s[d], a0);
      a1 = fmaf(sW[d + 1], s[d + 1], a1);
      a2 = fmaf(sW[d + 2], s[d + 2], a2);
      a3 = fmaf(sW[d + 3], s[d + 3], a3);
      c0 = fmaf(sqg[d], s[d], c0);
      c1 = fmaf(sqg[d + 1], s[d + 1], c1);
      c2 = fmaf(sqg[d + 2], s[d + 2], c2);
      c3 = fmaf(sqg[d + 3], s[d + 3], c3);
    }
    const float vn = u - ((a0 + a1) + (a2 + a3));
    o[off + col] = san(scale * ((c0 + c1) + (c2 + c3)) + aqk * vn, clip);
#pragma unroll
    for (int d = 0; d < D; ++d) s[d] = san(fmaf(sdec[d], s[d], skg[d] * vn), clip);
    __syncthreads();   // token vectors are rewritten next iteration
  }
  float* out = hf + (size_t)bh * D * D;
#pragma unroll
  for (int d = 0; d < D; ++d) out[d * D + col] = s[d];
}

template <typename T, int D>
cudaError_t launch(const void* q, const void* k, const void* v, const void* w, const void* b,
                   const void* g, const float* h0, float* o, float* hf, int B, int T_, int H,
                   float scale, float clip, int gates, cudaStream_t s) {
  auto c = [](const void* x) { return static_cast<const T*>(x); };
  k_decode<T, D><<<(unsigned)(B * H), D, 0, s>>>(c(q), c(k), c(v), c(w), c(b), c(g), h0, o, hf,
                                                  T_, H, scale, clip, gates);
  return cudaGetLastError();
}

}  // namespace
}  // namespace gdn2

extern "C" int gdn2_decode(int dtype, const void* q, const void* k, const void* v, const void* w,
                           const void* b, const void* g, const float* h0, float* o,
                           float* h_final, int B, int T, int H, int D, float scale, float clip,
                           void* stream) {
  using namespace gdn2;
  const int gates = (dtype & GDN2_GATES_RAW) != 0;
  dtype &= ~GDN2_GATES_RAW;
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
    e = D == 128 ? launch<float, 128>(q, k, v, w, b, g, h0, o, h_final, B, T, H, scale, clip, gates, s)
                 : launch<float, 64>(q, k, v, w, b, g, h0, o, h_final, B, T, H, scale, clip, gates, s);
  else
    e = D == 128
            ? launch<__nv_bfloat16, 128>(q, k, v, w, b, g, h0, o, h_final, B, T, H, scale, clip,
                                          gates, s)
            : launch<__nv_bfloat16, 64>(q, k, v, w, b, g, h0, o, h_final, B, T, H, scale, clip,
                                         gates, s);
  if (e != cudaSuccess) return report_error(GDN2_ERR_CUDA, cudaGetErrorString(e));
  return GDN2_OK;
}
