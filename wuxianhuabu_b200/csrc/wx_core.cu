// wx_core.cu — context lifetime, status/error plumbing, workspace arena, TMA
// map encoding, the PAB / sigma / sparse-policy schedules (host logic of the
// sampler loop) and the small fp32 islands of the step.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>

#include <algorithm>
#include <mutex>
#include <map>
#include <utility>

#include <nvtx3/nvToolsExt.h>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

int set_error(wx_ctx* ctx, int status, const char* fmt, ...) {
  if (!ctx) return status;
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  ctx->last_error = buf;
  return status;
}

void* workspace(wx_ctx* ctx, size_t bytes, int* status) {
  *status = WX_OK;
  if (bytes <= ctx->ws_bytes) return ctx->ws;
  if (ctx->ws) {
    // the arena may still be read by work queued on the stream
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  size_t want = (bytes + (size_t(1) << 20) - 1) & ~((size_t(1) << 20) - 1);
  cudaError_t e = cudaMalloc(&ctx->ws, want);
  if (e != cudaSuccess) {
    ctx->ws = nullptr;
    *status = set_error(ctx, WX_ERR_NOMEM, "workspace of %zu bytes: %s", want, cudaGetErrorString(e));
    return nullptr;
  }
  ctx->ws_bytes = want;
  return ctx->ws;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_bf16_2d(wx_ctx* ctx, CUtensorMap* map, const void* base, uint64_t rows,
                      uint64_t cols, uint64_t ld, uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(ctx, WX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (!aligned16(base) || (ld * 2) % 16 != 0)
    return set_error(ctx, WX_ERR_INVALID, "TMA operand needs 16-byte aligned base and row pitch");
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride,
                  box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ctx, WX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): rows=%llu cols=%llu ld=%llu",
                     (int)r, (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)ld);
  return WX_OK;
}

int make_tmap_u32_2d(wx_ctx* ctx, CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(ctx, WX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (!aligned16(base) || (ld * 4) % 16 != 0 || (box_cols * 4) % 16 != 0)
    return set_error(ctx, WX_ERR_INVALID, "TMA operand needs 16-byte aligned base, row pitch and box width");
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {ld * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ctx, WX_ERR_CUDA, "cuTensorMapEncodeTiled (u32) failed (%d): rows=%llu cols=%llu ld=%llu", (int)r,
                     (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)ld);
  return WX_OK;
}

int launch_status(wx_ctx* ctx, const char* what, int n) {
  ctx->launches += n;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(ctx, WX_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return WX_OK;
}

int ensure_smem_attr(wx_ctx* ctx, const void* fn, int bytes, const char* what) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> limit set so far
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(ctx, WX_ERR_CUDA, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(fn, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return WX_OK;  // the limit only ever grows
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return set_error(ctx, WX_ERR_CUDA, "%s shared-memory attribute (%d bytes, device %d): %s", what, bytes, dev,
                     cudaGetErrorString(e));
  done[key] = bytes;
  return WX_OK;
}

static cudaEvent_t pool_event(wx_ctx* c) {
  if (!c->prof_pool.empty()) {
    cudaEvent_t e = c->prof_pool.back();
    c->prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

ProfScope::ProfScope(wx_ctx* ctx, int kind) : c(ctx) {
  if (!c || !c->prof) return;
  wx_ctx::ProfRec r{kind, pool_event(c), pool_event(c)};
  cudaEventRecord(r.a, c->stream);
  c->prof_recs.push_back(r);
  idx = (int)c->prof_recs.size() - 1;
}

ProfScope::~ProfScope() {
  if (idx >= 0) cudaEventRecord(c->prof_recs[idx].b, c->stream);
}

static const char* const kTraceNames[WX_TRACE_PHASES] = {"wx.norm1", "wx.qkv", "wx.rope", "wx.attn", "wx.out",
                                                         "wx.mlp"};

LayerTrace::LayerTrace(wx_ctx* ctx, int mode) : c(ctx) {
  if (!c || !c->trace) return;
  wx_ctx::TraceRec r{};
  r.layer = c->trace_layer++;
  r.mode = mode;
  r.n = 1;
  r.mark[0] = pool_event(c);
  cudaEventRecord(r.mark[0], c->stream);
  c->trace_recs.push_back(r);
  idx = (int)c->trace_recs.size() - 1;
  nvtxRangePushA("wx.block");
}

void LayerTrace::begin(int phase) {
  if (idx < 0 || phase < 0 || phase >= WX_TRACE_PHASES) return;
  wx_ctx::TraceRec& r = c->trace_recs[idx];
  if (open > 0 && r.n <= WX_TRACE_PHASES) {  // end the open phase here
    r.mark[r.n] = pool_event(c);
    r.phase_of[r.n] = open - 1;
    cudaEventRecord(r.mark[r.n], c->stream);
    ++r.n;
    nvtxRangePop();
  }
  open = phase + 1;
  nvtxRangePushA(kTraceNames[phase]);
}

static void trace_release(wx_ctx* ctx) {
  for (auto& r : ctx->trace_recs)
    for (int i = 0; i < r.n; ++i) ctx->prof_pool.push_back(r.mark[i]);
  ctx->trace_recs.clear();
  ctx->trace_layer = 0;
}

LayerTrace::~LayerTrace() {
  if (idx < 0) return;
  wx_ctx::TraceRec& r = c->trace_recs[idx];
  if (open > 0) {
    if (r.n <= WX_TRACE_PHASES) {
      r.mark[r.n] = pool_event(c);
      r.phase_of[r.n] = open - 1;
      cudaEventRecord(r.mark[r.n], c->stream);
      ++r.n;
    }
    nvtxRangePop();
  }
  nvtxRangePop();
}

// ------------------------------------------------------------ fp32 islands
__global__ void dense_f32_kernel(const float* __restrict__ x, int64_t m, int64_t k,
                                 const float* __restrict__ w, int64_t n, const float* __restrict__ b,
                                 float* __restrict__ y) {
  // 64 rows x 32 columns per 256-thread block; x tile staged through shared memory
  __shared__ float xs[64][33];
  __shared__ float ws[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 row groups
  const int64_t r0 = (int64_t)blockIdx.x * 64, c0 = (int64_t)blockIdx.y * 32;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int64_t k0 = 0; k0 < k; k0 += 32) {
    for (int i = threadIdx.x; i < 64 * 32; i += 256) {
      int rr = i >> 5, kk = i & 31;
      int64_t gr = r0 + rr, gk = k0 + kk;
      xs[rr][kk] = (gr < m && gk < k) ? x[gr * k + gk] : 0.f;
    }
    for (int i = threadIdx.x; i < 32 * 32; i += 256) {
      int kk = i >> 5, cc = i & 31;
      int64_t gk = k0 + kk, gc = c0 + cc;
      ws[kk][cc] = (gk < k && gc < n) ? w[gk * n + gc] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < 32; ++kk) {
      float wv = ws[kk][tx];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(xs[ty * 8 + i][kk], wv, acc[i]);
    }
    __syncthreads();
  }
  const int64_t c = c0 + tx;
  if (c < n) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int64_t r = r0 + ty * 8 + i;
      if (r < m) y[r * n + c] = acc[i] + (b ? b[c] : 0.f);
    }
  }
}

__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ x, int64_t n, float* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, int64_t n, __nv_bfloat16* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

__global__ void euler_kernel(float* __restrict__ x, const float* __restrict__ v, int64_t n, float dsigma) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = x[i] + (-v[i]) * dsigma;
}

// runs `fn` with the context's device current, then restores the caller's current device
template <class F>
static int on_ctx_device(wx_ctx* ctx, F fn) {
  int prev = 0;
  WX_CUDA_TRY(ctx, cudaGetDevice(&prev));
  if (prev != ctx->device) WX_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  const int st = fn();
  if (prev != ctx->device) cudaSetDevice(prev);
  return st;
}

}  // namespace wx

using namespace wx;

extern "C" {

int wx_version(void) { return 1; }

int wx_ctx_create(int device, wx_ctx** out) {
  if (!out) return WX_ERR_INVALID;
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return WX_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return WX_ERR_CUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return WX_ERR_CUDA;
  if (prop.major != 10) return WX_ERR_UNSUPPORTED;  // sm_100a kernels only
  wx_ctx* c = new wx_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  if (cudaMalloc(&c->dev_err, sizeof(int) * 4) != cudaSuccess) {
    delete c;
    return WX_ERR_NOMEM;
  }
  cudaMemset(c->dev_err, 0, sizeof(int) * 4);
  *out = c;
  return WX_OK;
}

int wx_ctx_destroy(wx_ctx* ctx) {
  if (!ctx) return WX_OK;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  sp_p2p_release(ctx);
  if (ctx->p2p_counters) cudaFree(ctx->p2p_counters);
  sp_destroy_comm(ctx);
  for (auto& r : ctx->prof_recs) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  trace_release(ctx);
  for (auto e : ctx->prof_pool) cudaEventDestroy(e);
  if (ctx->aux) cudaStreamDestroy(ctx->aux);
  if (ctx->fork) cudaEventDestroy(ctx->fork);
  if (ctx->join) cudaEventDestroy(ctx->join);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->dev_err) cudaFree(ctx->dev_err);
  delete ctx;
  return WX_OK;
}

int wx_ctx_set_stream(wx_ctx* ctx, void* stream) {
  if (!ctx) return WX_ERR_INVALID;
  ctx->stream = static_cast<cudaStream_t>(stream);
  return WX_OK;
}

const char* wx_last_error(wx_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int wx_alloc(wx_ctx* ctx, size_t bytes, void** out) {
  WX_CHECK_ARG(ctx, ctx && out);
  *out = nullptr;
  if (bytes == 0) return WX_OK;
  return on_ctx_device(ctx, [&]() -> int {
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess)
      return set_error(ctx, WX_ERR_NOMEM, "wx_alloc of %zu bytes on device %d: %s", bytes, ctx->device,
                       cudaGetErrorString(e));
    *out = p;
    return WX_OK;
  });
}

int wx_free(wx_ctx* ctx, void* p) {
  WX_CHECK_ARG(ctx, ctx);
  if (!p) return WX_OK;
  return on_ctx_device(ctx, [&]() -> int {
    WX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));  // no queued work may still use it
    WX_CUDA_TRY(ctx, cudaFree(p));
    return WX_OK;
  });
}

int wx_upload(wx_ctx* ctx, void* dst, const void* src_host, size_t bytes) {
  WX_CHECK_ARG(ctx, ctx && (bytes == 0 || (dst && src_host)));
  if (bytes == 0) return WX_OK;
  WX_CUDA_TRY(ctx, cudaMemcpyAsync(dst, src_host, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return WX_OK;
}

int wx_download(wx_ctx* ctx, void* dst_host, const void* src, size_t bytes) {
  WX_CHECK_ARG(ctx, ctx && (bytes == 0 || (dst_host && src)));
  if (bytes == 0) return WX_OK;
  WX_CUDA_TRY(ctx, cudaMemcpyAsync(dst_host, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return WX_OK;
}

int wx_ctx_synchronize(wx_ctx* ctx) {
  if (!ctx) return WX_ERR_INVALID;
  WX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  return WX_OK;
}

size_t wx_ctx_workspace_bytes(wx_ctx* ctx) { return ctx ? ctx->ws_bytes : 0; }

int64_t wx_ctx_launch_count(wx_ctx* ctx) { return ctx ? ctx->launches : -1; }

int wx_ctx_profile_enable(wx_ctx* ctx, int enable) {
  if (!ctx) return WX_ERR_INVALID;
  for (auto& r : ctx->prof_recs) {
    ctx->prof_pool.push_back(r.a);
    ctx->prof_pool.push_back(r.b);
  }
  ctx->prof_recs.clear();
  ctx->prof = enable != 0;
  return WX_OK;
}

int wx_ctx_profile_read(wx_ctx* ctx, double* ms, int64_t* launches, int nkinds) {
  if (!ctx || !ms || !launches || nkinds <= 0) return WX_ERR_INVALID;
  WX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  for (int k = 0; k < nkinds; ++k) {
    ms[k] = 0.0;
    launches[k] = 0;
  }
  for (auto& r : ctx->prof_recs) {
    float t = 0.f;
    if (r.kind < nkinds && cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess) {
      ms[r.kind] += t;
      launches[r.kind] += 1;
    }
    ctx->prof_pool.push_back(r.a);
    ctx->prof_pool.push_back(r.b);
  }
  ctx->prof_recs.clear();
  return WX_OK;
}

int wx_ctx_trace_enable(wx_ctx* ctx, int enable) {
  if (!ctx) return WX_ERR_INVALID;
  trace_release(ctx);
  ctx->trace = enable != 0;
  return WX_OK;
}

int wx_ctx_trace_read(wx_ctx* ctx, double* records, int max_records, int* count) {
  if (!ctx || !count || max_records < 0 || (max_records > 0 && !records)) return WX_ERR_INVALID;
  *count = 0;
  WX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  int k = 0;
  for (auto& r : ctx->trace_recs) {
    if (k >= max_records) break;
    double* o = records + (size_t)k * WX_TRACE_FIELDS;
    for (int f = 0; f < WX_TRACE_FIELDS; ++f) o[f] = 0.0;
    o[0] = r.layer;
    o[1] = r.mode;
    for (int i = 1; i < r.n; ++i) {
      float t = 0.f;
      if (cudaEventElapsedTime(&t, r.mark[i - 1], r.mark[i]) == cudaSuccess) o[2 + r.phase_of[i]] += t;
    }
    float tot = 0.f;
    if (r.n > 1 && cudaEventElapsedTime(&tot, r.mark[0], r.mark[r.n - 1]) == cudaSuccess)
      o[2 + WX_TRACE_PHASES] = tot;
    ++k;
  }
  *count = k;
  trace_release(ctx);
  return WX_OK;
}

int wx_ctx_check_device(wx_ctx* ctx) {
  if (!ctx) return WX_ERR_INVALID;
  WX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  int h[4] = {0, 0, 0, 0};
  WX_CUDA_TRY(ctx, cudaMemcpy(h, ctx->dev_err, sizeof(h), cudaMemcpyDeviceToHost));
  if (h[0] != 0) {
    cudaMemset(ctx->dev_err, 0, sizeof(int) * 4);
    return set_error(ctx, WX_ERR_DEVICE, "device error word %d (bounded wait expired in a kernel)", h[0]);
  }
  return WX_OK;
}

// --------------------------------------------------------------- schedules
static int scaled_gate(uint32_t steps, uint32_t at30) {
  long v = (long)steps * (long)at30 / 30;
  if (v > (long)at30) v = at30;
  if (v < 1) v = 1;
  return (int)v;
}

int wx_pab_refresh(int i, uint32_t steps, uint32_t k) {
  if (k <= 1) return 1;
  const int warm = scaled_gate(steps, 4);
  if (i < warm) return 1;
  if (i + scaled_gate(steps, 2) >= (int)steps) return 1;
  return ((i - warm) % (int)k) == 0;
}

int wx_pab_must_refresh(double cached_sigma, double sigma, double max_stale) {
  // !(|sigma - cached| <= max_stale): an empty cache (+inf) always refreshes
  return !(fabs(sigma - cached_sigma) <= max_stale);
}

int wx_pab_plan(const double* sigmas, int nsigmas, uint32_t k, double max_stale, uint8_t* out) {
  const int nfe = nsigmas > 1 ? nsigmas - 1 : 0;
  double cached = INFINITY;
  for (int i = 0; i < nfe; ++i) {
    int refresh = wx_pab_refresh(i, (uint32_t)nfe, k) || wx_pab_must_refresh(cached, sigmas[i], max_stale);
    if (refresh) cached = sigmas[i];
    if (out) out[i] = (uint8_t)refresh;
  }
  return nfe;
}

int wx_sigma_schedule(uint32_t steps, double shift, double* out) {
  if (!out || steps == 0) return WX_ERR_INVALID;
  for (uint32_t i = 0; i <= steps; ++i) {
    const double base = 1.0 - (double)i / (double)steps;
    // timeShiftSigma(base, from 1, to shift): the base-grid value of `base` under shift 1 is base
    const double b = base / (1.0 + base * (1.0 - 1.0));
    out[i] = shift * b / (1.0 + (shift - 1.0) * b);
  }
  return WX_OK;
}

int wx_sparse_mode_for_layer(int layer, int nlayers, int policy) {
  switch (policy) {
    case 0: return 0;
    case 2: return 1;
    case 3: return 2;
    case 1: {
      const int mid = nlayers / 2;
      if (layer < 2 || layer + 2 >= nlayers || layer == mid || layer == mid + 1) return 0;
      return (layer % 2 == 0) ? 1 : 2;
    }
    default: return 0;
  }
}

int wx_build_row_mod_map(const wx_mod_run* runs, int nruns, int64_t count, uint32_t* map_out) {
  if (!map_out || count < 0 || (nruns > 0 && !runs)) return WX_ERR_INVALID;
  for (int64_t i = 0; i < count; ++i) map_out[i] = 0;
  for (int r = 0; r < nruns; ++r) {
    int64_t s = runs[r].start, e = runs[r].end;
    if (s < 0) s = 0;
    if (s > count) s = count;
    if (e < 0) e = 0;
    if (e > count) e = count;
    for (int64_t i = s; i < e; ++i) map_out[i] = runs[r].mod_row;
  }
  return WX_OK;
}

// ------------------------------------------------------------ fp32 islands
int wx_dense_f32(wx_ctx* ctx, const float* x, int64_t m, int64_t k, const float* w, int64_t n,
                 const float* b, float* y) {
  WX_CHECK_ARG(ctx, ctx && x && w && y && m >= 0 && k > 0 && n > 0);
  if (m == 0) return WX_OK;
  dim3 grid((unsigned)((m + 63) / 64), (unsigned)((n + 31) / 32));
  dense_f32_kernel<<<grid, 256, 0, ctx->stream>>>(x, m, k, w, n, b, y);
  return launch_status(ctx, "dense_f32");
}

int wx_bf16_to_f32(wx_ctx* ctx, const void* x, int64_t n, float* y) {
  WX_CHECK_ARG(ctx, ctx && x && y && n >= 0);
  if (!n) return WX_OK;
  bf16_to_f32_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 65536), 256, 0, ctx->stream>>>(
      static_cast<const __nv_bfloat16*>(x), n, y);
  return launch_status(ctx, "bf16_to_f32");
}

int wx_f32_to_bf16(wx_ctx* ctx, const float* x, int64_t n, void* y) {
  WX_CHECK_ARG(ctx, ctx && x && y && n >= 0);
  if (!n) return WX_OK;
  f32_to_bf16_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 65536), 256, 0, ctx->stream>>>(
      x, n, static_cast<__nv_bfloat16*>(y));
  return launch_status(ctx, "f32_to_bf16");
}

int wx_euler_update(wx_ctx* ctx, float* x, const float* v, int64_t n, float dsigma) {
  WX_CHECK_ARG(ctx, ctx && x && v && n >= 0);
  if (!n) return WX_OK;
  euler_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 65536), 256, 0, ctx->stream>>>(x, v, n, dsigma);
  return launch_status(ctx, "euler");
}

}  // extern "C"
