// wx_rope.cu — RoPE tables and the position primitives they are built from
// (model/minimax h3/H3Layout.swift):
//  * axisFromSqrtArea (:188-194), videoTSpan / videoTGrid (:197-210) and
//    writeFrameGrid (:683-694): host-side position ids of a packed layout;
//  * buildRope (:725-740): angles = concat(t·inv, h·inv, w·inv) over the
//    checkpoint's inverse frequencies, cos / sin rounded to bf16, on the GPU.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "wx_internal.h"

namespace wx {

// one thread per (row, axis, frequency): ang = float(pos) * inv in fp32, as the
// reference multiplies its fp32 position array by the fp32 inv_freq
__global__ void build_rope_kernel(const float* __restrict__ pos, int64_t S, const float* __restrict__ inv, int nf,
                                  __nv_bfloat16* __restrict__ cos_t, __nv_bfloat16* __restrict__ sin_t) {
  const int half = 3 * nf;
  const int64_t total = S * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i / half;
    const int c = (int)(i % half);
    const int a = c / nf, f = c % nf;
    const float ang = pos[s * 3 + a] * inv[f];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    cos_t[i] = __float2bfloat16_rn(cs);
    sin_t[i] = __float2bfloat16_rn(sn);
  }
}

}  // namespace wx

using namespace wx;

extern "C" {

int wx_axis_from_sqrt_area(uint32_t dim, uint32_t patch, double sqrt_area, double* out, int cap) {
  if (patch == 0 || !(sqrt_area > 0.0)) return WX_ERR_INVALID;
  const int n = (int)(dim / patch);
  if (!out) return n;
  if (cap < n) return WX_ERR_INVALID;
  const double ratio = (double)dim / sqrt_area;
  const double step = ratio / (double)n;
  const double start = (1.0 - ratio) / 2.0;
  for (int i = 0; i < n; ++i) out[i] = ((double)i * step + start) * 32.0;
  return n;
}

double wx_video_t_span(int k) {
  // H3Const.frameRescale (5/3) x framePerToken[k % 5] ([1, 4, 4, 4, 4]), H3Common.swift:22-23
  static const uint32_t per_token[5] = {1, 4, 4, 4, 4};
  return (5.0 / 3.0) * (double)per_token[((k % 5) + 5) % 5];
}

int wx_video_t_grid(uint32_t n, double origin, double* out) {
  if (!out && n) return WX_ERR_INVALID;
  double acc = origin;
  for (uint32_t i = 0; i < n; ++i) {
    out[i] = acc;
    acc += wx_video_t_span((int)i);
  }
  return WX_OK;
}

int wx_write_frame_grid(double* pos, int64_t row, double t, const double* h_axis, int nh, const double* w_axis,
                        int nw) {
  if (!pos || row < 0 || nh < 0 || nw < 0 || (nh && !h_axis) || (nw && !w_axis)) return WX_ERR_INVALID;
  int64_t i = row;
  for (int a = 0; a < nh; ++a)
    for (int b = 0; b < nw; ++b, ++i) {
      pos[i * 3 + 0] = t;
      pos[i * 3 + 1] = h_axis[a];
      pos[i * 3 + 2] = w_axis[b];
    }
  return WX_OK;
}

int wx_build_rope(wx_ctx* ctx, const float* pos, int64_t S, const float* inv_freq, int nf, void* cos_t,
                  void* sin_t) {
  WX_CHECK_ARG(ctx, ctx && pos && inv_freq && cos_t && sin_t && S >= 0 && nf > 0 && nf <= 1024);
  if (!S) return WX_OK;
  const int64_t total = S * 3 * nf;
  const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)ctx->num_sms * 16);
  build_rope_kernel<<<grid, 256, 0, ctx->stream>>>(pos, S, inv_freq, nf, static_cast<__nv_bfloat16*>(cos_t),
                                                  static_cast<__nv_bfloat16*>(sin_t));
  return launch_status(ctx, "build_rope");
}

}  // extern "C"
