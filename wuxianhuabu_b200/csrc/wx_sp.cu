// wx_sp.cu — Ulysses sequence parallelism for the DiT block over NCCL.
//
// Rows of the packed sequence are split evenly over the P ranks; every GEMM,
// row kernel and PAB slot stays row-local. Attention needs the whole sequence,
// so around it the q|k|v of each rank's rows are exchanged head-wise with one
// all-to-all (afterwards every rank holds the full sequence for H/P heads, in
// the packed qkv layout the flash kernel reads directly) and the attention
// output comes back with a second all-to-all. SOL / top-k routing is per head,
// so each rank routes its heads exactly as one GPU would. PAB reuse steps skip
// the attention branch and therefore all communication.
//
// NCCL is resolved at run time with dlopen: a copy already loaded into the
// process (e.g. by torch) is reused, otherwise libnccl.so.2 is loaded. The
// collectives are grouped point-to-point send/recv on the context stream.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

int launch_qk_norm_rope(wx_ctx* ctx, const void* x, int64_t x_stride, void* out, int64_t out_stride,
                        int64_t part_off, int nparts, int64_t S, int H, int hd, const void* w0, const void* w1,
                        const void* cos_t, const void* sin_t, int rot, float eps);
int launch_norm_modscale(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w, const void* shift,
                         const void* scale, const uint32_t* rowmap, float eps, void* out);
int launch_mod_gate(wx_ctx* ctx, const void* x, const void* other, const void* gate, const uint32_t* rowmap,
                    int64_t S, int64_t hidden, void* out);
int qlinear_with_scratch(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w, int epilogue,
                         const void* gate, const void* resid, const uint32_t* rowmap, void* y, int64_t ldy,
                         void* y_raw, void* wd, void* swiglu_tmp);
bool qweight_ok(const wx_qweight* w);
size_t attention_scratch_bytes(int64_t S, int H, int hd, const wx_sparse_spec* spec);
int attention_with_scratch(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, int64_t S, int H,
                           int hd, const wx_sparse_spec* spec, float scale, void* out, int64_t os, void* scratch);

// ------------------------------------------------------------------ NCCL api
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  bool ok = false;
};

static NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](const char* n) { return dlsym(h, n); };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(sym("ncclCommAbort"));
    api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
    api.Send = reinterpret_cast<decltype(api.Send)>(sym("ncclSend"));
    api.Recv = reinterpret_cast<decltype(api.Recv)>(sym("ncclRecv"));
    api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
    api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));  // optional (peer setup)
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommAbort && api.CommGetAsyncError &&
             api.Send && api.Recv && api.GroupStart && api.GroupEnd && api.GetErrorString;
  });
  return api;
}

#define WX_NCCL_TRY(ctx, expr)                                                                    \
  do {                                                                                            \
    ncclResult_t r__ = (expr);                                                                    \
    if (r__ != ncclSuccess)                                                                       \
      return ::wx::set_error((ctx), WX_ERR_CUDA, "%s failed: %s", #expr, nccl().GetErrorString(r__)); \
  } while (0)

// all-to-all of P equal chunks of `chunk_bytes` (chunk r of send goes to rank r,
// chunk r of recv comes from rank r)
static int all_to_all(wx_ctx* ctx, const void* send, void* recv, size_t chunk_bytes) {
  NcclApi& api = nccl();
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
  const uint8_t* s = static_cast<const uint8_t*>(send);
  uint8_t* d = static_cast<uint8_t*>(recv);
  ProfScope prof(ctx, kProfOther);
  WX_NCCL_TRY(ctx, api.GroupStart());
  for (int r = 0; r < ctx->sp_size; ++r) {
    WX_NCCL_TRY(ctx, api.Send(s + (size_t)r * chunk_bytes, chunk_bytes, ncclUint8, r, comm, ctx->stream));
    WX_NCCL_TRY(ctx, api.Recv(d + (size_t)r * chunk_bytes, chunk_bytes, ncclUint8, r, comm, ctx->stream));
  }
  WX_NCCL_TRY(ctx, api.GroupEnd());
  return WX_OK;
}

// --------------------------------------------------------------- pack/unpack
// send[r][row][part][c] = qkv[row][part*H*hd + (r*Hl)*hd + c], c < Hl*hd (16-byte units)
__global__ void sp_pack_qkv_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t rows, int P, int H, int Hl,
                                   int hd, __nv_bfloat16* __restrict__ send) {
  const int64_t per_part = (int64_t)Hl * hd / 8;
  const int64_t per_row = 3 * per_part;
  const int64_t total = (int64_t)P * rows * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (rows * per_row);
    const int64_t rem = i % (rows * per_row);
    const int64_t row = rem / per_row;
    const int64_t u = rem % per_row;
    const int64_t part = u / per_part, c = u % per_part;
    const uint4 v = *reinterpret_cast<const uint4*>(qkv + row * 3 * H * hd + part * H * hd + r * Hl * hd + c * 8);
    *reinterpret_cast<uint4*>(send + ((r * rows + row) * 3 + part) * Hl * hd + c * 8) = v;
  }
}

// att[row][r*Hl*hd + c] = recv[r][row][c]
__global__ void sp_unpack_out_kernel(const __nv_bfloat16* __restrict__ recv, int64_t rows, int P, int Hl, int hd,
                                     __nv_bfloat16* __restrict__ att) {
  const int64_t per_row = (int64_t)Hl * hd / 8;
  const int64_t total = (int64_t)P * rows * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (rows * per_row);
    const int64_t rem = i % (rows * per_row);
    const int64_t row = rem / per_row, c = rem % per_row;
    const uint4 v = *reinterpret_cast<const uint4*>(recv + (r * rows + row) * Hl * hd + c * 8);
    *reinterpret_cast<uint4*>(att + row * (int64_t)P * Hl * hd + r * Hl * hd + c * 8) = v;
  }
}

// ------------------------------------------------------ exchange over peer memory
// Instead of the two all-to-alls, each rank writes its rows of q|k|v (after
// QK-norm + RoPE, in the same kernel) straight into the exchange buffer of the
// rank that owns each head, and the attention kernels write each output row
// straight into the out-projection operand of the rank that owns the row; NVLink
// carries the stores, no staging copies, no collective launches. Each rank's
// buffer: flags of exchange 1 [8] | flags of exchange 2 [8] | attention rows
// [rows, H*128] | q|k|v of its heads for the whole sequence [S, 3*Hl*128].
int launch_qkv_to_peers(wx_ctx* ctx, const void* qkv, int64_t rows, int64_t row0, int H, int Hl,
                        void* const* peers, int P, const void* w0, const void* w1, const void* cos_t,
                        const void* sin_t, int rot, float eps, PeerSignal sig);
bool qkv_to_peers_ok(int hd, int rot);

// waits (bounded by limit_ns) until every flags[r], r < n, holds `epoch` or later
// (wrap-around order); one warp, each lane polling flags lane, lane + 32, ...
__global__ void sp_wait_flags_kernel(const uint32_t* flags, int n, uint32_t epoch, int* err, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int r = threadIdx.x; r < n; r += blockDim.x) {
    while ((int32_t)(ld_acquire_sys_u32(flags + r) - epoch) < 0) {
      if (globaltimer_ns() - t0 > limit_ns) {
        set_dev_error(err, kDevTimeoutPeer);
        return;
      }
      __nanosleep(200);
    }
  }
}

// stores `epoch` into flags[r], r < n, with release semantics at system scope, after
// every earlier write of this stream is visible (stream order + system fence)
__global__ void sp_signal_flags_kernel(uint32_t* flags, int n, uint32_t epoch) {
  __threadfence_system();
  for (int r = threadIdx.x; r < n; r += blockDim.x) st_release_sys_u32(flags + r, epoch);
}

struct P2PLayout {
  size_t flags1 = 0, flags2 = 64, att = 256, qkv = 0, total = 0;
};

static size_t al(size_t b);

static P2PLayout p2p_layout(int64_t S, int64_t rows, int64_t inner, int Hl, int hd) {
  P2PLayout L;
  L.qkv = L.att + al((size_t)rows * inner * 2);
  L.total = L.qkv + al((size_t)S * 3 * Hl * hd * 2);
  return L;
}

static bool sp_p2p_env() {
  static int v = [] {
    const char* e = getenv("WX_SP_P2P");
    return e ? atoi(e) : 1;
  }();
  return v != 0;
}

void sp_p2p_release(wx_ctx* ctx) {
  if (!ctx) return;
  if (ctx->p2p_buf) {
    cudaStreamSynchronize(ctx->stream);
    if (ctx->aux) cudaStreamSynchronize(ctx->aux);
    for (int r = 0; r < kSpMaxPeers; ++r)
      if (ctx->p2p_peer[r] && ctx->p2p_peer[r] != ctx->p2p_buf) cudaIpcCloseMemHandle(ctx->p2p_peer[r]);
    cudaFree(ctx->p2p_buf);
  }
  for (int r = 0; r < kSpMaxPeers; ++r) ctx->p2p_peer[r] = nullptr;
  ctx->p2p_buf = nullptr;
  ctx->p2p_bytes = 0;
  ctx->p2p_epoch = 0;
}

// one record per rank in the all-gather: the IPC handle and whether the rank can take part
struct P2PRecord {
  cudaIpcMemHandle_t handle;
  int32_t ok;
  int32_t pad[15];
};

// all-gather of one record per rank over the context's communicator (blocking)
static int p2p_all_gather(wx_ctx* ctx, const P2PRecord& mine, P2PRecord* all) {
  const int P = ctx->sp_size;
  void* dev = nullptr;
  WX_CUDA_TRY(ctx, cudaMalloc(&dev, sizeof(P2PRecord) * (P + 1)));
  auto* d = static_cast<uint8_t*>(dev);
  cudaError_t e = cudaMemcpyAsync(d, &mine, sizeof(P2PRecord), cudaMemcpyHostToDevice, ctx->stream);
  ncclResult_t nr = ncclSuccess;
  if (e == cudaSuccess)
    nr = nccl().AllGather(d, d + sizeof(P2PRecord), sizeof(P2PRecord), ncclUint8,
                          static_cast<ncclComm_t>(ctx->comm), ctx->stream);
  if (e == cudaSuccess && nr == ncclSuccess)
    e = cudaMemcpyAsync(all, d + sizeof(P2PRecord), sizeof(P2PRecord) * P, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  cudaFree(dev);
  if (nr != ncclSuccess) return set_error(ctx, WX_ERR_CUDA, "peer setup all-gather: %s", nccl().GetErrorString(nr));
  if (e != cudaSuccess) return set_error(ctx, WX_ERR_CUDA, "peer setup: %s", cudaGetErrorString(e));
  return WX_OK;
}

// Collective (every rank calls it at the same point with the same size): makes
// sure the exchange buffers of `bytes` exist and are opened by every rank.
// Returns 1 when the peer path is on, 0 when the ranks use the all-to-alls.
static int p2p_ensure(wx_ctx* ctx, size_t bytes, int hd, int rot, int* status) {
  *status = WX_OK;
  if (ctx->p2p_state == 0) return 0;
  if (ctx->p2p_state == 1 && ctx->p2p_bytes >= bytes) return 1;
  const int P = ctx->sp_size, rank = ctx->sp_rank;
  sp_p2p_release(ctx);
  P2PRecord mine{};
  mine.ok = sp_p2p_env() && nccl().AllGather && P <= kSpMaxPeers && attn_peer_path_ok() && qkv_to_peers_ok(hd, rot);
  if (mine.ok && !ctx->p2p_counters) {
    if (cudaMalloc(&ctx->p2p_counters, 2 * sizeof(int)) != cudaSuccess ||
        cudaMemset(ctx->p2p_counters, 0, 2 * sizeof(int)) != cudaSuccess)
      mine.ok = 0;
  }
  if (mine.ok) {
    if (cudaMalloc(&ctx->p2p_buf, bytes) != cudaSuccess) {
      ctx->p2p_buf = nullptr;
      mine.ok = 0;
    } else if (cudaMemset(ctx->p2p_buf, 0, bytes) != cudaSuccess ||
               cudaIpcGetMemHandle(&mine.handle, ctx->p2p_buf) != cudaSuccess) {
      mine.ok = 0;
    }
    cudaGetLastError();
  }
  if (!nccl().AllGather) {  // cannot even agree: every rank sees the same library, so all fall back
    ctx->p2p_state = 0;
    sp_p2p_release(ctx);
    return 0;
  }
  P2PRecord all[kSpMaxPeers + 1];
  P2PRecord* recs = P <= kSpMaxPeers ? all : nullptr;
  std::vector<P2PRecord> big;
  if (!recs) {
    big.resize(P);
    recs = big.data();
  }
  if ((*status = p2p_all_gather(ctx, mine, recs))) return 0;
  bool all_ok = true;
  for (int r = 0; r < P; ++r) all_ok = all_ok && recs[r].ok;
  P2PRecord opened{};
  opened.ok = all_ok;
  if (all_ok) {
    for (int r = 0; r < P; ++r) {
      if (r == rank) {
        ctx->p2p_peer[r] = ctx->p2p_buf;
        continue;
      }
      void* ptr = nullptr;
      if (cudaIpcOpenMemHandle(&ptr, recs[r].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        opened.ok = 0;
        break;
      }
      ctx->p2p_peer[r] = ptr;
    }
  }
  // every rank must agree that every rank opened every buffer
  if ((*status = p2p_all_gather(ctx, opened, recs))) return 0;
  bool open_all = all_ok;
  for (int r = 0; r < P; ++r) open_all = open_all && recs[r].ok;
  if (!open_all) {
    sp_p2p_release(ctx);
    ctx->p2p_state = 0;
    return 0;
  }
  ctx->p2p_bytes = bytes;
  ctx->p2p_epoch = 0;
  ctx->p2p_state = 1;
  return 1;
}

static unsigned grid_units(wx_ctx* ctx, int64_t total) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)ctx->num_sms * 16));
}

struct SpLayout {
  size_t m, qkv, send, recv, attf, ret, att, at, ha, f1, wd, sw, lt, attn, total;
};

static size_t al(size_t b) { return (b + 255) & ~size_t(255); }

static SpLayout sp_layout(const wx_dit_config* c, int64_t S, int P) {
  SpLayout L{};
  const int64_t rows = S / P;
  const int Hl = c->heads / P;
  const size_t inner = (size_t)c->heads * c->head_dim;
  const size_t fc1_n = c->mlp_kind == WX_MLP_SWIGLU ? 2 * (size_t)c->ffn : (size_t)c->ffn;
  size_t off = 0;
  L.m = off; off += al((size_t)rows * c->hidden * 2);
  L.qkv = off; off += al((size_t)rows * 3 * inner * 2);
  L.send = off; off += al((size_t)rows * 3 * inner * 2);
  L.recv = off; off += al((size_t)S * 3 * Hl * c->head_dim * 2);
  L.attf = off; off += al((size_t)S * Hl * c->head_dim * 2);
  L.ret = off; off += al((size_t)rows * inner * 2);
  L.att = off; off += al((size_t)rows * inner * 2);
  L.at = off; off += al((size_t)rows * c->hidden * 2);
  L.ha = off; off += al((size_t)rows * c->hidden * 2);
  L.f1 = off; off += al((size_t)rows * c->ffn * 2);
  size_t wmax = std::max(std::max(3 * inner * (size_t)c->hidden, inner * (size_t)c->hidden),
                         std::max(fc1_n * (size_t)c->hidden, (size_t)c->ffn * c->hidden));
  // expanded weight of the two-pass GEMM, or the fp32 split-K accumulator of the small-M path
  const size_t nmax = std::max(std::max(3 * inner, (size_t)c->hidden), fc1_n);
  L.wd = off; off += al(std::max(wmax * 2, qlinear_ws_need(rows, (int64_t)nmax, 1)));
  L.sw = off; off += c->mlp_kind == WX_MLP_SWIGLU ? al((size_t)rows * fc1_n * 2) : 0;
  L.lt = off; off += al((size_t)rows * (size_t)std::max(0, c->lora_rank) * 2);  // x at^T of a LoRA pack
  wx_sparse_spec sol{};
  sol.mode = WX_SPARSE_SOL;
  sol.block = 64;
  wx_sparse_spec topk = sol;
  topk.mode = WX_SPARSE_TOPK;
  topk.block = 128;
  size_t a = std::max(attention_scratch_bytes(S, Hl, c->head_dim, &sol),
                      std::max(attention_scratch_bytes(S, Hl, c->head_dim, &topk),
                               attention_scratch_bytes(S, Hl, c->head_dim, nullptr)));
  L.attn = off; off += al(a);
  L.total = off;
  return L;
}

void sp_destroy_comm(wx_ctx* ctx) {
  if (ctx && ctx->comm && nccl().ok) nccl().CommDestroy(static_cast<ncclComm_t>(ctx->comm));
  if (ctx) ctx->comm = nullptr;
}

}  // namespace wx

using namespace wx;

extern "C" {

int wx_sp_make_plan(int64_t S, int H, int head_dim, int P, int rank, wx_sp_plan* out) {
  if (!out || S <= 0 || H <= 0 || head_dim <= 0 || P <= 0 || rank < 0 || rank >= P) return WX_ERR_INVALID;
  if (S % P || H % P) return WX_ERR_INVALID;
  out->S = S;
  out->P = P;
  out->rank = rank;
  out->rows = S / P;
  out->row0 = (int64_t)rank * out->rows;
  out->H = H;
  out->heads = H / P;
  out->head0 = rank * out->heads;
  out->head_dim = head_dim;
  out->qkv_chunk = out->rows * 3 * (int64_t)out->heads * head_dim;
  out->out_chunk = out->rows * (int64_t)out->heads * head_dim;
  return WX_OK;
}

int wx_comm_unique_id(void* id128) {
  if (!id128) return WX_ERR_INVALID;
  NcclApi& api = nccl();
  if (!api.ok) return WX_ERR_UNSUPPORTED;
  ncclUniqueId id;
  if (api.GetUniqueId(&id) != ncclSuccess) return WX_ERR_CUDA;
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
  memcpy(id128, &id, sizeof(id));
  return WX_OK;
}

int wx_ctx_init_comm(wx_ctx* ctx, int nranks, int rank, const void* id128) {
  WX_CHECK_ARG(ctx, ctx && id128 && nranks >= 1 && rank >= 0 && rank < nranks);
  NcclApi& api = nccl();
  if (!api.ok) return set_error(ctx, WX_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) could not be loaded");
  if (ctx->comm) {
    api.CommDestroy(static_cast<ncclComm_t>(ctx->comm));
    ctx->comm = nullptr;
  }
  sp_p2p_release(ctx);  // a new group decides the exchange path again
  ctx->p2p_state = -1;
  ncclUniqueId id;
  memcpy(&id, id128, sizeof(id));
  ncclComm_t comm = nullptr;
  WX_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  WX_NCCL_TRY(ctx, api.CommInitRank(&comm, nranks, id, rank));
  ctx->comm = comm;
  ctx->sp_size = nranks;
  ctx->sp_rank = rank;
  return WX_OK;
}

int wx_ctx_comm_check(wx_ctx* ctx) {
  if (!ctx) return WX_ERR_INVALID;
  if (!ctx->comm) return WX_OK;
  ncclResult_t e = ncclSuccess;
  WX_NCCL_TRY(ctx, nccl().CommGetAsyncError(static_cast<ncclComm_t>(ctx->comm), &e));
  if (e != ncclSuccess && e != ncclInProgress)
    return set_error(ctx, WX_ERR_CUDA, "NCCL asynchronous error: %s", nccl().GetErrorString(e));
  return WX_OK;
}

int wx_ctx_sp_exchange(wx_ctx* ctx) { return ctx ? ctx->p2p_state : WX_ERR_INVALID; }

int wx_ctx_set_peer_wait_limit(wx_ctx* ctx, double seconds) {
  WX_CHECK_ARG(ctx, ctx && seconds > 0.0 && seconds <= 600.0);
  ctx->peer_wait_ns = (uint64_t)(seconds * 1e9);
  return WX_OK;
}

int wx_ctx_signal_flags(wx_ctx* ctx, uint32_t* flags, int n, uint32_t epoch) {
  WX_CHECK_ARG(ctx, ctx && flags && n > 0 && ((uintptr_t)flags & 3) == 0);
  sp_signal_flags_kernel<<<1, 32, 0, ctx->stream>>>(flags, n, epoch);
  return launch_status(ctx, "signal_flags");
}

int wx_ctx_wait_flags(wx_ctx* ctx, const uint32_t* flags, int n, uint32_t epoch) {
  WX_CHECK_ARG(ctx, ctx && flags && n > 0 && ((uintptr_t)flags & 3) == 0);
  ProfScope prof(ctx, kProfPeerWait);
  sp_wait_flags_kernel<<<1, 32, 0, ctx->stream>>>(flags, n, epoch, ctx->dev_err, ctx->peer_wait_ns);
  return launch_status(ctx, "wait_flags");
}

int wx_ctx_comm_abort(wx_ctx* ctx) {
  if (!ctx) return WX_ERR_INVALID;
  if (ctx->comm) nccl().CommAbort(static_cast<ncclComm_t>(ctx->comm));
  ctx->comm = nullptr;
  sp_p2p_release(ctx);
  ctx->p2p_state = -1;
  ctx->sp_size = 1;
  ctx->sp_rank = 0;
  return WX_OK;
}

int64_t wx_dit_block_sp_scratch_bytes(const wx_dit_config* cfg, int64_t S, int P) {
  if (!cfg || S <= 0 || P <= 0 || S % P || cfg->heads % P) return 0;
  return (int64_t)sp_layout(cfg, S, P).total;
}

int wx_dit_block_forward_sp(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w,
                            const wx_block_mods* mods, const uint32_t* rowmap, void* h, int64_t S, const void* cos_t,
                            const void* sin_t, const wx_sparse_spec* spec, void* pab_slot, int refresh,
                            void* scratch) {
  WX_CHECK_ARG(ctx, ctx && cfg && w && mods && h && scratch && S > 0);
  const int P = ctx->sp_size;
  if (P == 1 || !ctx->comm)
    return wx_dit_block_forward(ctx, cfg, w, mods, rowmap, h, S, cos_t, sin_t, spec, pab_slot, refresh, scratch);
  WX_CHECK_ARG(ctx, S % P == 0 && cfg->heads % P == 0 && cfg->head_dim == 128);
  const int64_t inner = (int64_t)cfg->heads * cfg->head_dim;
  const int64_t fc1_n = cfg->mlp_kind == WX_MLP_SWIGLU ? 2 * cfg->ffn : cfg->ffn;
  WX_CHECK_ARG(ctx, qweight_ok(&w->qkv) && w->qkv.k == cfg->hidden && w->qkv.n == 3 * inner);
  WX_CHECK_ARG(ctx, qweight_ok(&w->out) && w->out.k == inner && w->out.n == cfg->hidden);
  WX_CHECK_ARG(ctx, qweight_ok(&w->fc1) && w->fc1.k == cfg->hidden && w->fc1.n == fc1_n);
  WX_CHECK_ARG(ctx, qweight_ok(&w->fc2) && w->fc2.k == cfg->ffn && w->fc2.n == cfg->hidden);
  WX_CHECK_ARG(ctx, pab_slot || refresh);
  WX_CHECK_ARG(ctx, lora_packs_ok(cfg, w));
  const int64_t rows = S / P;
  const int Hl = cfg->heads / P;
  const int hd = cfg->head_dim;
  const SpLayout L = sp_layout(cfg, S, P);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  void* m = base + L.m;
  void* ha = base + L.ha;
  void* f1 = base + L.f1;
  void* wd = base + L.wd;
  void* lt = base + L.lt;
  int st;
  const bool full_fwd = refresh || !pab_slot;
  LayerTrace tr(ctx, !full_fwd ? WX_TRACE_REUSE
                               : (spec && spec->mode != WX_SPARSE_DENSE) ? WX_TRACE_SPARSE : WX_TRACE_DENSE);
  if (full_fwd) {
    void* qkv = base + L.qkv;
    auto* send = reinterpret_cast<__nv_bfloat16*>(base + L.send);
    auto* recv = reinterpret_cast<__nv_bfloat16*>(base + L.recv);
    auto* attf = reinterpret_cast<__nv_bfloat16*>(base + L.attf);
    auto* ret = reinterpret_cast<__nv_bfloat16*>(base + L.ret);
    auto* att = reinterpret_cast<__nv_bfloat16*>(base + L.att);
    tr.begin(WX_TRACE_NORM1);
    if ((st = launch_norm_modscale(ctx, h, rows, cfg->hidden, w->norm1, mods->shift_msa, mods->scale_msa, rowmap,
                                   cfg->eps, m)))
      return st;
    const float scale = 1.0f / sqrtf((float)hd);
    const P2PLayout PL = p2p_layout(S, rows, inner, Hl, hd);
    const int peer = p2p_ensure(ctx, PL.total, hd, cfg->rot, &st);
    if (st) return st;
    // QK-norm + RoPE in the q|k|v GEMM's epilogue where the geometry allows
    const bool fused = qkv_rope_fusable(&w->qkv, rows, w->lora[0] != nullptr, peer != 0, hd, cfg->rot, w->q_norm,
                                        w->k_norm, cos_t, sin_t);
    tr.begin(WX_TRACE_QKV);
    if (!(peer && fused)) {
      if (fused) {
        if ((st = qkv_rope_with_scratch(ctx, m, rows, cfg->hidden, &w->qkv, w->lora[0], hd, qkv, 3 * inner,
                                        w->q_norm, w->k_norm, cos_t, sin_t, cfg->rot, cfg->eps, wd, lt, nullptr)))
          return st;
      } else if ((st = qlinear_lora_with_scratch(ctx, m, rows, cfg->hidden, &w->qkv, w->lora[0], WX_EPI_NONE,
                                                 nullptr, nullptr, nullptr, qkv, 3 * inner, nullptr, wd, lt,
                                                 nullptr))) {
        return st;
      }
    }
    if (peer) {
      // exchange 1: QK-norm + RoPE (and v) of this rank's rows straight into the owners'
      // buffers; exchange 2: attention rows straight into the owners' out-proj operand
      const uint32_t ep = ++ctx->p2p_epoch;
      const int rank = ctx->sp_rank;
      void* qkv_dst[kSpMaxPeers] = {};
      SpPeerOut po{};
      PeerSignal sig1{};
      for (int r = 0; r < P; ++r) {
        uint8_t* b = static_cast<uint8_t*>(ctx->p2p_peer[r]);
        qkv_dst[r] = b + PL.qkv;
        po.out_peer[r] = b + PL.att;
        po.flags[r] = reinterpret_cast<uint32_t*>(b + PL.flags2);
        sig1.flags[r] = reinterpret_cast<uint32_t*>(b + PL.flags1);
      }
      sig1.counter = ctx->p2p_counters;
      sig1.P = P;
      sig1.rank = rank;
      sig1.epoch = ep;
      uint8_t* mine = static_cast<uint8_t*>(ctx->p2p_buf);
      if (fused) {
        // the GEMM's epilogue stores q|k|v rows straight into the owners' buffers
        QkvPeerOut po1{};
        for (int r = 0; r < P; ++r) po1.base[r] = qkv_dst[r];
        po1.row0 = (int64_t)rank * rows;
        po1.rows_total = S;
        po1.Hl = Hl;
        po1.sig = sig1;
        if ((st = qkv_rope_with_scratch(ctx, m, rows, cfg->hidden, &w->qkv, w->lora[0], hd, qkv, 3 * inner,
                                        w->q_norm, w->k_norm, cos_t, sin_t, cfg->rot, cfg->eps, wd, lt, &po1)))
          return st;
        tr.begin(WX_TRACE_ROPE);
      } else {
        tr.begin(WX_TRACE_ROPE);
        if ((st = launch_qkv_to_peers(ctx, qkv, rows, (int64_t)rank * rows, cfg->heads, Hl, qkv_dst, P, w->q_norm,
                                      w->k_norm, cos_t, sin_t, cfg->rot, cfg->eps, sig1)))
          return st;
      }
      {
        ProfScope wprof(ctx, kProfPeerWait);
        sp_wait_flags_kernel<<<1, 32, 0, ctx->stream>>>(reinterpret_cast<const uint32_t*>(mine + PL.flags1), P, ep,
                                                       ctx->dev_err, ctx->peer_wait_ns);
      }
      if ((st = launch_status(ctx, "sp_wait_qkv"))) return st;
      po.rows = rows;
      po.col = rank * Hl * hd;
      po.counter = ctx->p2p_counters + 1;
      po.P = P;
      po.rank = rank;
      po.epoch = ep;
      auto* full = reinterpret_cast<__nv_bfloat16*>(mine + PL.qkv);
      void* att_mine = mine + PL.att;
      const int64_t rs = 3 * (int64_t)Hl * hd;
      tr.begin(WX_TRACE_ATTN);
      if ((st = attention_with_scratch_peer(ctx, full, full + (int64_t)Hl * hd, full + 2 * (int64_t)Hl * hd, rs, S,
                                            Hl, hd, spec, scale, att_mine, inner, base + L.attn, &po)))
        return st;
      {
        ProfScope wprof(ctx, kProfPeerWait);
        sp_wait_flags_kernel<<<1, 32, 0, ctx->stream>>>(reinterpret_cast<const uint32_t*>(mine + PL.flags2), P, ep,
                                                       ctx->dev_err, ctx->peer_wait_ns);
      }
      if ((st = launch_status(ctx, "sp_wait_att"))) return st;
      void* at_dst = pab_slot ? pab_slot : base + L.at;
      tr.begin(WX_TRACE_OUT);
      if ((st = qlinear_lora_with_scratch(ctx, att_mine, rows, inner, &w->out, w->lora[1], WX_EPI_GATE_RESID,
                                          mods->gate_msa, h, rowmap, ha, cfg->hidden, at_dst, wd, lt, nullptr)))
        return st;
    }
    if (!peer) {
      tr.begin(WX_TRACE_ROPE);
      if (!fused && (st = launch_qk_norm_rope(ctx, qkv, 3 * inner, qkv, 3 * inner, inner, 2, rows, cfg->heads, hd,
                                              w->q_norm, w->k_norm, cos_t, sin_t, cfg->rot, cfg->eps)))
        return st;
      // q|k|v of this rank's rows, grouped by destination head block
      const int64_t pack_units = (int64_t)P * rows * 3 * Hl * hd / 8;
      sp_pack_qkv_kernel<<<grid_units(ctx, pack_units), 256, 0, ctx->stream>>>(
          static_cast<const __nv_bfloat16*>(qkv), rows, P, cfg->heads, Hl, hd, send);
      if ((st = launch_status(ctx, "sp_pack_qkv"))) return st;
      if ((st = all_to_all(ctx, send, recv, (size_t)rows * 3 * Hl * hd * 2))) return st;
      // attention over the whole sequence for heads [rank*Hl, rank*Hl + Hl)
      const int64_t rs = 3 * (int64_t)Hl * hd;
      tr.begin(WX_TRACE_ATTN);
      if ((st = attention_with_scratch(ctx, recv, recv + (int64_t)Hl * hd, recv + 2 * (int64_t)Hl * hd, rs, S, Hl,
                                       hd, spec, scale, attf, (int64_t)Hl * hd, base + L.attn)))
        return st;
      // rows of rank r go back to r; gather this rank's rows of every head
      if ((st = all_to_all(ctx, attf, ret, (size_t)rows * Hl * hd * 2))) return st;
      const int64_t un_units = (int64_t)P * rows * Hl * hd / 8;
      sp_unpack_out_kernel<<<grid_units(ctx, un_units), 256, 0, ctx->stream>>>(ret, rows, P, Hl, hd, att);
      if ((st = launch_status(ctx, "sp_unpack_out"))) return st;
      void* at_dst = pab_slot ? pab_slot : base + L.at;
      tr.begin(WX_TRACE_OUT);
      if ((st = qlinear_lora_with_scratch(ctx, att, rows, inner, &w->out, w->lora[1], WX_EPI_GATE_RESID,
                                          mods->gate_msa, h, rowmap, ha, cfg->hidden, at_dst, wd, lt, nullptr)))
        return st;
    }
  } else {
    tr.begin(WX_TRACE_OUT);
    if ((st = launch_mod_gate(ctx, h, pab_slot, mods->gate_msa, rowmap, rows, cfg->hidden, ha))) return st;
  }
  tr.begin(WX_TRACE_MLP);
  if ((st = launch_norm_modscale(ctx, ha, rows, cfg->hidden, w->norm2, mods->shift_mlp, mods->scale_mlp, rowmap,
                                 cfg->eps, m)))
    return st;
  const int act = cfg->mlp_kind == WX_MLP_SWIGLU ? WX_EPI_SWIGLU : WX_EPI_GELU;
  if ((st = qlinear_lora_with_scratch(ctx, m, rows, cfg->hidden, &w->fc1, w->lora[2], act, nullptr, nullptr,
                                      nullptr, f1, cfg->ffn, nullptr, wd, lt, base + L.sw)))
    return st;
  return qlinear_lora_with_scratch(ctx, f1, rows, cfg->ffn, &w->fc2, w->lora[3], WX_EPI_GATE_RESID, mods->gate_mlp, ha, rowmap, h,
                              cfg->hidden, nullptr, wd, lt, nullptr);
}

}  // extern "C"
