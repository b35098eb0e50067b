// wx_noalloc.cu — the quantized linear layer for callers that cannot allocate
// device memory.
//
// wx_qlinear expands the 6-bit weight into a bf16 copy held in the context's
// workspace, which the context grows with cudaMalloc. Some hosts cannot make
// that call at the point where they run a layer: code running under a
// restricted allocator or inside an engine that owns every device allocation,
// or a plugin handed only a stream and tensors it does not own. For them this
// file keeps the expanded weight in one file-scope static device array whose
// size is fixed when the library is built (kNoAllocScratchBytes). Each GPU that
// loads this module holds its own copy until the process exits; with CUDA's
// lazy module loading (the default) the module, and with it the 64 MiB, is
// loaded on a device at the first call there, so make that first call while
// allocation is still allowed (at set-up), and before any stream capture.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress (that device current) and caches it. In host code
// the array's name is only a host-side stand-in, so kernels are always handed
// the looked-up device pointer.
//
// All calls share the one array and it keeps whatever the last call left in
// it. Every element a call reads is first written by the same call, so
// nothing needs clearing; calls whose work overlaps on the GPU (different
// streams without ordering) race on the array.
//
// Errors: argument and launch failures come back as the call's status, with
// the message in a per-thread string (wx_qlinear_noalloc_last_error). A kernel
// whose bounded wait expires records the fact in a per-device error word that
// the call cannot see without synchronising; wx_qlinear_noalloc_check reads and
// clears it.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>
#include <string>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

int launch_dequant(wx_ctx* ctx, const wx_qweight* w, void* out);
int gemm_bf16(wx_ctx* ctx, const void* x, int64_t M, int64_t lda, const void* wd, int64_t N, int64_t K,
              const void* bias, int epi, const void* gate, const void* resid, const uint32_t* rowmap, void* y,
              int64_t ldy, void* y_raw);
bool qweight_ok(const wx_qweight* w);

// 64 MiB: room for an expanded bf16 weight of up to 33,554,432 elements (n*k),
// e.g. a 9216 x 3072 qkv projection.
constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
// where the kernels launched from this path record a bounded-wait expiry (first
// code wins); read and cleared by wx_qlinear_noalloc_check
static __device__ __align__(16) int g_noalloc_err[4];

// message of the last failed call on this thread
static thread_local std::string g_noalloc_msg;

namespace {
constexpr int kMaxDevices = 64;
struct DeviceSlot {
  void* scratch = nullptr;
  int* err = nullptr;
  int num_sms = 0;
  bool ready = false;
};
std::mutex g_mu;
DeviceSlot g_slots[kMaxDevices];

int setup_device(int dev, DeviceSlot*& out) {
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceSlot& s = g_slots[dev];
  if (!s.ready) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return WX_ERR_CUDA;
    void* e = nullptr;
    if (cudaGetSymbolAddress(&e, g_noalloc_err) != cudaSuccess || !e) return WX_ERR_CUDA;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return WX_ERR_CUDA;
    s.scratch = p;
    s.err = static_cast<int*>(e);
    s.num_sms = sms;
    s.ready = true;
  }
  out = &s;
  return WX_OK;
}
}  // namespace

}  // namespace wx

using namespace wx;

static int fail(int status, const char* msg) {
  g_noalloc_msg = msg;
  return status;
}

extern "C" int wx_qlinear_noalloc(void* stream, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                                  int epilogue, const void* gate, const void* resid, const uint32_t* rowmap,
                                  void* y, int64_t ldy, void* y_raw) {
  if (!x || !y || !qweight_ok(w) || m < 0 || lda < w->k) return fail(WX_ERR_INVALID, "invalid argument");
  if (epilogue != WX_EPI_NONE && epilogue != WX_EPI_GELU && epilogue != WX_EPI_GATE_RESID)
    return fail(WX_ERR_UNSUPPORTED, "epilogue not offered without allocation (WX_EPI_SWIGLU needs a temporary)");
  if (epilogue == WX_EPI_GATE_RESID && (!gate || !resid)) return fail(WX_ERR_INVALID, "gate and resid required");
  if (ldy < w->n) return fail(WX_ERR_INVALID, "ldy < n");
  // the expanded weight must fit the static scratch array
  if ((uint64_t)w->n * (uint64_t)w->k * 2u > kNoAllocScratchBytes)
    return fail(WX_ERR_INVALID, "n * k exceeds the 33,554,432 elements of the static scratch");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return fail(WX_ERR_CUDA, "cudaGetDevice");
  DeviceSlot* slot = nullptr;
  int st = setup_device(dev, slot);
  if (st) return fail(st, "cudaGetSymbolAddress of the static scratch failed");
  // a stack context: no workspace, no error-word allocation, no profiling
  wx_ctx local;
  local.device = dev;
  local.num_sms = slot->num_sms;
  local.stream = static_cast<cudaStream_t>(stream);
  local.dev_err = slot->err;
  if (!(st = launch_dequant(&local, w, slot->scratch)))
    st = gemm_bf16(&local, x, m, lda, slot->scratch, w->n, w->k, w->bias, epilogue, gate, resid, rowmap, y, ldy,
                   y_raw);
  if (st) g_noalloc_msg = local.last_error;
  return st;
}

extern "C" int wx_qlinear_noalloc_check(void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return fail(WX_ERR_CUDA, "cudaGetDevice");
  DeviceSlot* slot = nullptr;
  int st = setup_device(dev, slot);
  if (st) return fail(st, "cudaGetSymbolAddress of the error word failed");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  int h = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&h, slot->err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(WX_ERR_CUDA, cudaGetErrorString(e));
  if (h == 0) return WX_OK;
  const int zero = 0;
  cudaMemcpy(slot->err, &zero, sizeof(int), cudaMemcpyHostToDevice);
  char buf[96];
  snprintf(buf, sizeof(buf), "device error word %d (a bounded wait expired in a kernel)", h);
  return fail(WX_ERR_DEVICE, buf);
}

extern "C" const char* wx_qlinear_noalloc_last_error(void) { return g_noalloc_msg.c_str(); }
