// wx_lora.cu — LoRA adapters of the quantized linears (LoraRef / loraDelta,
// model/minimax h3/H3Common.swift:407-433; applied in MfLinear.forward :369-375).
//
// The reference adds sum_i scale_i * ((x A_i) B_i) after the quantized product.
// Here the adapters of one linear are packed once into the operands of a K
// extension of the main GEMM: at [R, k] holds scale_i * A_i^T (rows stacked over
// adapters), bt [n, R] holds B_i^T (columns side by side), R = sum r_i padded to
// a multiple of 64 with zeros. Per call, t = x at^T ([m, R]) is one small GEMM,
// and the main GEMM accumulates x W^T and t bt^T into the same fp32 accumulator
// before its epilogue.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

// at[(off + j) * k + c] = bf16(scale * a[c * r + j]) for j < r, c < k
__global__ void lora_pack_a_kernel(const __nv_bfloat16* __restrict__ a, int64_t k, int r, float scale, int64_t off,
                                   __nv_bfloat16* __restrict__ at) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= k * r) return;
  const int64_t j = i / k, c = i % k;
  at[(off + j) * k + c] = __float2bfloat16_rn(scale * __bfloat162float(a[c * r + j]));
}

// bt[nn * R + off + j] = b[j * n + nn] for j < r, nn < n
__global__ void lora_pack_b_kernel(const __nv_bfloat16* __restrict__ b, int64_t n, int r, int64_t R, int64_t off,
                                   __nv_bfloat16* __restrict__ bt) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n * r) return;
  const int64_t nn = i / r, j = i % r;
  bt[nn * R + off + j] = b[j * n + nn];
}

}  // namespace wx

using namespace wx;

extern "C" {

int wx_lora_pack_bytes(int64_t n, int64_t k, const wx_lora* l, int count, int64_t* R, size_t* at_bytes,
                       size_t* bt_bytes) {
  if (!l || count <= 0 || n <= 0 || k <= 0 || !R || !at_bytes || !bt_bytes) return WX_ERR_INVALID;
  int64_t sum = 0;
  for (int i = 0; i < count; ++i) {
    if (l[i].r <= 0) return WX_ERR_INVALID;
    sum += l[i].r;
  }
  *R = (sum + 63) / 64 * 64;
  *at_bytes = (size_t)*R * k * 2;
  *bt_bytes = (size_t)n * *R * 2;
  return WX_OK;
}

int wx_lora_pack_build(wx_ctx* ctx, int64_t n, int64_t k, const wx_lora* l, int count, wx_lora_pack* out) {
  WX_CHECK_ARG(ctx, ctx && l && count > 0 && out && out->at && out->bt && n > 0 && k > 0);
  WX_CHECK_ARG(ctx, aligned16(out->at) && aligned16(out->bt) && k % 64 == 0 && n % 64 == 0);
  int64_t R = 0;
  size_t ab = 0, bb = 0;
  if (wx_lora_pack_bytes(n, k, l, count, &R, &ab, &bb) != WX_OK)
    return set_error(ctx, WX_ERR_INVALID, "lora: every adapter needs r > 0");
  for (int i = 0; i < count; ++i) WX_CHECK_ARG(ctx, l[i].a && l[i].b);
  cudaError_t e = cudaMemsetAsync(out->at, 0, ab, ctx->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(out->bt, 0, bb, ctx->stream);
  if (e != cudaSuccess) return set_error(ctx, WX_ERR_CUDA, "lora pack memset: %s", cudaGetErrorString(e));
  int64_t off = 0;
  auto* at = static_cast<__nv_bfloat16*>(out->at);
  auto* bt = static_cast<__nv_bfloat16*>(out->bt);
  for (int i = 0; i < count; ++i) {
    const int r = l[i].r;
    lora_pack_a_kernel<<<(unsigned)((k * r + 255) / 256), 256, 0, ctx->stream>>>(
        static_cast<const __nv_bfloat16*>(l[i].a), k, r, l[i].scale, off, at);
    lora_pack_b_kernel<<<(unsigned)((n * r + 255) / 256), 256, 0, ctx->stream>>>(
        static_cast<const __nv_bfloat16*>(l[i].b), n, r, R, off, bt);
    int st = launch_status(ctx, "lora_pack", 2);
    if (st) return st;
    off += r;
  }
  out->R = R;
  out->n = n;
  out->k = k;
  return WX_OK;
}

}  // extern "C"
