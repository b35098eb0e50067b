// wx_internal.h — host-side context, status plumbing and TMA map encoding
// shared by the translation units of libwx.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/wx_api.h"

struct wx_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  int* dev_err = nullptr;         // device error word (wx::DevErr)
  void* ws = nullptr;             // workspace arena
  size_t ws_bytes = 0;
  std::string last_error;
  int64_t launches = 0;  // kernels launched through this context
  // sequence-parallel group (Ulysses): NCCL communicator, size, rank
  void* comm = nullptr;
  int sp_size = 1;
  int sp_rank = 0;
  // per-kernel-class device timing (wx_ctx_profile_enable / _read)
  bool prof = false;
  struct ProfRec {
    int kind;
    cudaEvent_t a, b;
  };
  std::vector<ProfRec> prof_recs;
  std::vector<cudaEvent_t> prof_pool;
  // per-layer phase trace (wx_ctx_trace_enable / _read): one record per block
  // forward, mark[0] its start and mark[i] (i >= 1) the end of phase phase_of[i]
  bool trace = false;
  int trace_layer = 0;
  struct TraceRec {
    int layer, mode, n;
    cudaEvent_t mark[WX_TRACE_PHASES + 1];
    int phase_of[WX_TRACE_PHASES + 1];
  };
  std::vector<TraceRec> trace_recs;
  // side stream for independent kernels that run concurrently with the context
  // stream (forked and joined with the two events); created on first use
  cudaStream_t aux = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  // sequence parallelism over NVLink peer memory (wx_sp.cu): this rank's exchange
  // buffer (flags | attention rows | full-sequence q|k|v of its heads), exported by
  // CUDA IPC and opened by every other rank; the peers' buffers; two CTA counters
  int p2p_state = -1;  // -1 not decided, 0 off (NCCL all-to-alls), 1 on
  void* p2p_buf = nullptr;
  size_t p2p_bytes = 0;
  void* p2p_peer[8] = {};
  int* p2p_counters = nullptr;
  uint32_t p2p_epoch = 0;
  // limit of the cross-GPU flag waits (sequence-parallel exchange, wx_ctx_wait_flags)
  uint64_t peer_wait_ns = 10000000000ull;
};

namespace wx {

int set_error(wx_ctx* ctx, int status, const char* fmt, ...);

#define WX_CUDA_TRY(ctx, expr)                                                              \
  do {                                                                                      \
    cudaError_t e__ = (expr);                                                               \
    if (e__ != cudaSuccess)                                                                 \
      return ::wx::set_error((ctx), WX_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,            \
                             cudaGetErrorString(e__), __FILE__, __LINE__);                  \
  } while (0)

#define WX_CHECK_ARG(ctx, cond)                                                             \
  do {                                                                                      \
    if (!(cond)) return ::wx::set_error((ctx), WX_ERR_INVALID, "invalid argument: %s", #cond); \
  } while (0)

// Returns a device buffer of at least `bytes` from the context arena (grown on
// demand; contents undefined; valid until the next call that grows it).
void* workspace(wx_ctx* ctx, size_t bytes, int* status);

// Carves 256-byte-aligned sub-buffers out of one arena request.
struct Carve {
  size_t off = 0;
  size_t take(size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  }
};

// 2-D bf16 tensor map: `rows` x `cols` elements, row pitch `ld` elements,
// box `box_cols` x `box_rows`, 128-byte swizzle, zero fill out of bounds.
int make_tmap_bf16_2d(wx_ctx* ctx, CUtensorMap* map, const void* base, uint64_t rows,
                      uint64_t cols, uint64_t ld, uint32_t box_cols, uint32_t box_rows);

// 2-D uint32 tensor map (no swizzle): `rows` x `cols` words, row pitch `ld` words,
// box `box_cols` x `box_rows`, zero fill out of bounds.
int make_tmap_u32_2d(wx_ctx* ctx, CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_cols, uint32_t box_rows);

// releases the NCCL communicator of a context (no-op without one)
void sp_destroy_comm(wx_ctx* ctx);
// releases the peer exchange buffers of a context (closes the peers' mappings first)
void sp_p2p_release(wx_ctx* ctx);

// checks the last launch(es) and counts `n` kernel launches on the context
int launch_status(wx_ctx* ctx, const char* what, int n = 1);

// Raises kernel `fn`'s dynamic shared-memory limit to at least `bytes` on the CURRENT
// device (the limit only grows; set once per kernel and device): cudaFuncSetAttribute acts
// on one device only, so a process that drives several GPUs needs it on each.
// Thread-safe. WX_OK or a status set on ctx.
int ensure_smem_attr(wx_ctx* ctx, const void* fn, int bytes, const char* what);

enum ProfKind { kProfGemm = 0, kProfAttn = 1, kProfRoute = 2, kProfRow = 3, kProfDequant = 4, kProfOther = 5,
                kProfNormRope = 6, kProfNormMod = 7, kProfExchange = 8, kProfPeerWait = 9, kProfKinds = 10 };

// Records CUDA events around the launches of one kernel class on the
// context stream while profiling is enabled (no-op otherwise).
struct ProfScope {
  wx_ctx* c;
  int idx = -1;
  ProfScope(wx_ctx* ctx, int kind);
  ~ProfScope();
};

// Phase trace of one block forward (the reference's NA_H3PROF per-layer timers):
// the constructor marks the block's start, begin(p) ends the open phase and opens
// phase p (a wx_trace_phase), the destructor ends the last one. While tracing is
// enabled each mark is a CUDA event on the context stream and the block and each
// phase are NVTX ranges ("wx.block", "wx.<phase>"); otherwise nothing is recorded.
struct LayerTrace {
  wx_ctx* c;
  int idx = -1;
  int open = 0;
  LayerTrace(wx_ctx* ctx, int mode);
  void begin(int phase);
  ~LayerTrace();
};

// Scratch of one quantized linear: the expanded bf16 weight of the two-pass GEMM
// (the small-M path, at most 512 rows, expands in shared memory and needs none).
inline size_t qlinear_ws_need(int64_t /*m*/, int64_t n, int64_t k) { return (size_t)n * k * 2; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Quantized linear with an optional LoRA pack (nullptr = none): `wd` holds the
// expanded weight (qlinear_ws_need bytes), `t` the [m, lora->R] bf16 product
// x at^T, `swiglu_tmp` the [m, n] pre-activation of WX_EPI_SWIGLU.
int qlinear_lora_with_scratch(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                              const wx_lora_pack* lora, int epilogue, const void* gate, const void* resid,
                              const uint32_t* rowmap, void* y, int64_t ldy, void* y_raw, void* wd, void* t,
                              void* swiglu_tmp);
bool lora_pack_ok(const wx_lora_pack* l, const wx_qweight* w);

// The q|k|v projection with QK-RMSNorm + RoPE in its GEMM epilogue (wx_gemm.cu).
// qkv_rope_fusable: whether a block takes that path (the geometry the epilogue
// supports; not where the small-M kernel serves the projection, unless `peer`: the
// sequence-parallel exchange, head_dim 128). qkv_rope_with_scratch: dequant into `wd`,
// the LoRA product into `t`, then the GEMM; peers == nullptr writes y in place,
// otherwise the owners' exchange buffers (QkvPeerOut, wx_ptx.cuh) and their signal.
struct QkvPeerOut;
bool qkv_rope_fusable(const wx_qweight* w, int64_t m, bool has_lora, bool peer, int head_dim, int rot,
                      const void* q_norm, const void* k_norm, const void* cos_t, const void* sin_t);
int qkv_rope_with_scratch(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                          const wx_lora_pack* lora, int head_dim, void* y, int64_t ldy, const void* q_norm,
                          const void* k_norm, const void* cos_t, const void* sin_t, int rot, float eps, void* wd,
                          void* t, const QkvPeerOut* peers);

// Attention output delivered straight into other ranks' memory (sequence
// parallelism): query row s goes to rank s / rows at out_peer[r] + (s % rows) *
// out_stride + col + head*128, and the last CTA stores `epoch` into flags[r][rank]
// of every rank r.
constexpr int kSpMaxPeers = 8;
struct SpPeerOut {
  void* out_peer[kSpMaxPeers];
  int64_t rows;
  int col;
  int* counter;
  uint32_t* flags[kSpMaxPeers];
  int P, rank;
  uint32_t epoch;
};
// true when the attention call takes the paired / duo kernels, the only ones that
// write to peers
bool attn_peer_path_ok();
int attention_with_scratch_peer(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, int64_t S,
                                int H, int hd, const wx_sparse_spec* spec, float scale, void* out, int64_t os,
                                void* scratch, const SpPeerOut* po);
bool lora_packs_ok(const wx_dit_config* cfg, const wx_block_weights* w);

}  // namespace wx
