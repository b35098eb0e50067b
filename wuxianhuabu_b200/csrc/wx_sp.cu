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

int wx_ctx_comm_abort(wx_ctx* ctx) {
  if (!ctx) return WX_ERR_INVALID;
  if (ctx->comm) nccl().CommAbort(static_cast<ncclComm_t>(ctx->comm));
  ctx->comm = nullptr;
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
  if (refresh || !pab_slot) {
    void* qkv = base + L.qkv;
    auto* send = reinterpret_cast<__nv_bfloat16*>(base + L.send);
    auto* recv = reinterpret_cast<__nv_bfloat16*>(base + L.recv);
    auto* attf = reinterpret_cast<__nv_bfloat16*>(base + L.attf);
    auto* ret = reinterpret_cast<__nv_bfloat16*>(base + L.ret);
    auto* att = reinterpret_cast<__nv_bfloat16*>(base + L.att);
    if ((st = launch_norm_modscale(ctx, h, rows, cfg->hidden, w->norm1, mods->shift_msa, mods->scale_msa, rowmap,
                                   cfg->eps, m)))
      return st;
    if ((st = qlinear_lora_with_scratch(ctx, m, rows, cfg->hidden, &w->qkv, w->lora[0], WX_EPI_NONE, nullptr, nullptr, nullptr, qkv,
                                   3 * inner, nullptr, wd, lt, nullptr)))
      return st;
    if ((st = launch_qk_norm_rope(ctx, qkv, 3 * inner, qkv, 3 * inner, inner, 2, rows, cfg->heads, hd, w->q_norm,
                                  w->k_norm, cos_t, sin_t, cfg->rot, cfg->eps)))
      return st;
    // q|k|v of this rank's rows, grouped by destination head block
    const int64_t pack_units = (int64_t)P * rows * 3 * Hl * hd / 8;
    sp_pack_qkv_kernel<<<grid_units(ctx, pack_units), 256, 0, ctx->stream>>>(
        static_cast<const __nv_bfloat16*>(qkv), rows, P, cfg->heads, Hl, hd, send);
    if ((st = launch_status(ctx, "sp_pack_qkv"))) return st;
    if ((st = all_to_all(ctx, send, recv, (size_t)rows * 3 * Hl * hd * 2))) return st;
    // attention over the whole sequence for heads [rank*Hl, rank*Hl + Hl)
    const float scale = 1.0f / sqrtf((float)hd);
    const int64_t rs = 3 * (int64_t)Hl * hd;
    if ((st = attention_with_scratch(ctx, recv, recv + (int64_t)Hl * hd, recv + 2 * (int64_t)Hl * hd, rs, S, Hl, hd,
                                     spec, scale, attf, (int64_t)Hl * hd, base + L.attn)))
      return st;
    // rows of rank r go back to r; gather this rank's rows of every head
    if ((st = all_to_all(ctx, attf, ret, (size_t)rows * Hl * hd * 2))) return st;
    const int64_t un_units = (int64_t)P * rows * Hl * hd / 8;
    sp_unpack_out_kernel<<<grid_units(ctx, un_units), 256, 0, ctx->stream>>>(ret, rows, P, Hl, hd, att);
    if ((st = launch_status(ctx, "sp_unpack_out"))) return st;
    void* at_dst = pab_slot ? pab_slot : base + L.at;
    if ((st = qlinear_lora_with_scratch(ctx, att, rows, inner, &w->out, w->lora[1], WX_EPI_GATE_RESID, mods->gate_msa, h, rowmap, ha,
                                   cfg->hidden, at_dst, wd, lt, nullptr)))
      return st;
  } else {
    if ((st = launch_mod_gate(ctx, h, pab_slot, mods->gate_msa, rowmap, rows, cfg->hidden, ha))) return st;
  }
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
