/*
 * wx_api.h — C ABI of libwx, the B200 (sm_100a) implementation of the
 * MiniMax-H3 video-DiT denoising step of HuaChayu/wuxianhuabu.
 *
 * The reference is Swift over MLX; every entry point below names the Swift
 * interface it replaces (file:line within the reference project). Callers pass
 * device pointers they own; tensors are row-major, bf16 values are raw 16-bit
 * patterns. Calls are ordered on the context's stream and never abort the
 * process: each returns WX_OK or a negative wx_status, and wx_last_error()
 * gives the message. A context is not thread-safe; use one per thread/GPU.
 */
#ifndef WX_API_H
#define WX_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct wx_ctx wx_ctx;

enum wx_status {
  WX_OK = 0,
  WX_ERR_INVALID = -1,     /* bad shape, pointer, alignment or option */
  WX_ERR_CUDA = -2,        /* a CUDA runtime/driver call failed */
  WX_ERR_NOMEM = -3,       /* workspace allocation failed */
  WX_ERR_DEVICE = -4,      /* a kernel reported a device-side error (bounded wait expired) */
  WX_ERR_UNSUPPORTED = -5, /* geometry not supported by this build */
};

/* fused GEMM epilogues (applied to t = bf16(bf16(acc) + bias)) */
enum wx_epilogue {
  WX_EPI_NONE = 0,       /* y = t */
  WX_EPI_GELU = 1,       /* y = bf16(gelu_tanh(t)) */
  WX_EPI_GATE_RESID = 2, /* y = bf16(resid + t * gate[rowmap[m]]); y_raw = t (optional) */
  WX_EPI_SWIGLU = 3,     /* fc1 emits [gate | up]: y[:, j] = bf16(silu(t[:, j]) * t[:, F + j]) */
};

enum wx_sparse_mode {
  WX_SPARSE_DENSE = 0, /* SDPA over every key */
  WX_SPARSE_SOL = 1,   /* SOL tau routing + tail pooled term */
  WX_SPARSE_TOPK = 2,  /* diagonal + top-k fraction of key blocks */
};

enum wx_mlp_kind { WX_MLP_GELU = 0, WX_MLP_SWIGLU = 1 };

/* 6-bit (2..8-bit) MLX-affine group-quantized weight of a linear layer:
 * wq [n, k*bits/32] uint32, scales/biases [n, k/group] bf16, bias [n] bf16 or NULL.
 * Mirrors MfLinear's quantized fields (model/minimax h3/H3Common.swift:283-338). */
typedef struct wx_qweight {
  const uint32_t* wq;
  const void* scales;
  const void* biases;
  const void* bias;
  int64_t n;
  int64_t k;
  int32_t group;
  int32_t bits;
} wx_qweight;

/* H3SolAttnConfig + SparseSpec (网络算子-稀疏注意力-SOL通用.swift:79-98;
 * model/minimax h3/H3Layout.swift:909-920). */
typedef struct wx_sparse_spec {
  int32_t mode;       /* wx_sparse_mode */
  int32_t block;      /* key/query block rows: 64 (SOL) or 128 (top-k) */
  int64_t g;          /* strip rows [0, g) = SparseSpec.videoStart */
  float tau;          /* SOL threshold multiplier (default 1.3) */
  float density;      /* top-k kept fraction of off-diagonal blocks (0.25) */
  int32_t sink_start; /* always-exact video blocks [sink_start, sink_end) */
  int32_t sink_end;
  int32_t tail;       /* 1: unselected blocks add the pooled tail term */
  int32_t reserved;
} wx_sparse_spec;

/* one DiT block's weights (H3BlockW / H3AttnW / H3MlpW, H3Transformer.swift:405-660) */
/* One LoRA adapter of a linear (LoraRef, H3Common.swift:407-411): the layer adds
 * scale * ((x A) B) (loraDelta, H3Common.swift:424-433). a [k, r] and b [r, n] bf16,
 * row-major (the reference's [in, r] and [r, out]). */
typedef struct wx_lora {
  const void* a;
  const void* b;
  int32_t r;
  float scale;
} wx_lora;

/* The adapters of one linear packed as an extension of the GEMM's K dimension:
 * y = x W^T + t bt^T with t = x at^T ([m, R] bf16, computed per call), so the
 * delta accumulates in the same fp32 accumulator as the base product.
 * at [R, k] = scale_i * A_i^T stacked over adapters; bt [n, R] = B_i^T side by side;
 * R = sum r_i rounded up to 64 (zero padding). Built by wx_lora_pack_build. */
typedef struct wx_lora_pack {
  void* at;
  void* bt;
  int64_t R;
  int64_t n;
  int64_t k;
} wx_lora_pack;

typedef struct wx_block_weights {
  wx_qweight qkv; /* hidden -> 3*inner */
  wx_qweight out; /* inner -> hidden */
  wx_qweight fc1; /* hidden -> ffn (GELU) or 2*ffn (SwiGLU) */
  wx_qweight fc2; /* ffn -> hidden */
  const void* q_norm; /* [head_dim] bf16 */
  const void* k_norm;
  const void* norm1; /* [hidden] bf16 */
  const void* norm2;
  /* LoRA of qkv / out / fc1 / fc2 (H3LoraFile entries, H3Common.swift:436-496;
   * attached in production, H3Pipeline.swift:680-687); NULL = none. Each pack's
   * R must not exceed wx_dit_config.lora_rank. */
  const wx_lora_pack* lora[4];
} wx_block_weights;

/* model geometry (H3Config, H3Common.swift:78-139) */
typedef struct wx_dit_config {
  int64_t hidden;
  int32_t heads;
  int32_t head_dim;
  int64_t ffn;
  int32_t mlp_kind; /* wx_mlp_kind */
  int32_t rot;      /* rotated dims (rotHalf*2); dims [rot, head_dim) pass through */
  float eps;        /* RMSNorm epsilon */
  int32_t lora_rank; /* largest packed LoRA rank R of any linear (0 = no LoRA); sizes scratch */
} wx_dit_config;

/* AdaLN modulation tables of one block, each [num_mod_rows, hidden] bf16:
 * shift/scale/gate for attention (MSA) and MLP (H3Transformer.swift:1083-1107) */
typedef struct wx_block_mods {
  const void* shift_msa;
  const void* scale_msa;
  const void* gate_msa;
  const void* shift_mlp;
  const void* scale_mlp;
  const void* gate_mlp;
} wx_block_mods;

/* ModRun (H3Layout.swift:744-753) */
typedef struct wx_mod_run {
  uint32_t start;
  uint32_t end;
  uint32_t mod_row;
} wx_mod_run;

/* ------------------------------------------------------------- context */
int wx_ctx_create(int device, wx_ctx** out);
int wx_ctx_destroy(wx_ctx* ctx);
/* stream: a cudaStream_t (NULL = legacy default stream) */
int wx_ctx_set_stream(wx_ctx* ctx, void* stream);
const char* wx_last_error(wx_ctx* ctx);
/* synchronises the stream and returns WX_ERR_DEVICE if a kernel set the
 * device error word since the last call (the word is cleared) */
int wx_ctx_check_device(wx_ctx* ctx);
/* bytes currently held by the context workspace arena */
size_t wx_ctx_workspace_bytes(wx_ctx* ctx);
/* number of kernels this context has launched so far */
int64_t wx_ctx_launch_count(wx_ctx* ctx);
int wx_version(void);

/* Device memory for hosts that do not link the CUDA runtime themselves (the Swift
 * wrapper; MLXArray's role in the reference): buffers on the context's device, 256-byte
 * aligned, and host <-> device copies ordered on the context stream (host memory pinned
 * or pageable; a copy from pageable memory returns once the source may be reused).
 * The caller's current CUDA device is left as it was. wx_ctx_synchronize waits for
 * everything queued on the context stream. */
int wx_alloc(wx_ctx* ctx, size_t bytes, void** out);
int wx_free(wx_ctx* ctx, void* p);
int wx_upload(wx_ctx* ctx, void* dst, const void* src_host, size_t bytes);
int wx_download(wx_ctx* ctx, void* dst_host, const void* src, size_t bytes);
int wx_ctx_synchronize(wx_ctx* ctx);
/* Device timing by kernel class (0 qGEMM, 1 flash attention, 2 routing + list
 * build, 3 other row kernels (gated residual, RMSNorm, conversions), 4 weight
 * dequant, 5 other (NCCL all-to-alls, pack/unpack), 6 QK-RMSNorm + RoPE,
 * 7 RMSNorm + modulation, 8 QK-RMSNorm + RoPE storing into other ranks' memory
 * (the fused sequence-parallel exchange), 9 waits for other ranks' signals):
 * while enabled, CUDA events bracket each launch on the context stream.
 * enable(…, 0/1) clears the record; read() synchronises, returns the summed
 * milliseconds and launch counts of the first nkinds classes since the last
 * enable/read, and clears the record. */
int wx_ctx_profile_enable(wx_ctx* ctx, int enable);
int wx_ctx_profile_read(wx_ctx* ctx, double* ms, int64_t* launches, int nkinds);

/* Per-layer phase trace: the NA_H3PROF timers of the attention forward
 * (model/minimax h3/H3Transformer.swift:445-450, 575-597: qkv, ropeN, attn, out,
 * tot per layer), extended to the whole block. While enabled, every block
 * forward (wx_dit_block_forward, _sp, and the blocks of the step functions)
 * records CUDA events on the context stream at its phase boundaries and opens
 * NVTX ranges "wx.block" and "wx.<phase>" on the calling thread (visible to any
 * NVTX-aware tool; free without one). enable(…, 0/1) clears the record and the
 * layer counter. read() synchronises and writes up to max_records records of
 * WX_TRACE_FIELDS doubles:
 *   [0] layer (block forwards counted from 0 since enable/read)
 *   [1] mode (WX_TRACE_DENSE, WX_TRACE_SPARSE, WX_TRACE_REUSE)
 *   [2 + p] milliseconds of phase p (wx_trace_phase), 0 when the phase did not run
 *   [2 + WX_TRACE_PHASES] milliseconds of the whole block
 * sets *count to the number written and clears the record (records beyond
 * max_records are dropped). */
enum wx_trace_phase {
  WX_TRACE_NORM1 = 0, /* RMSNorm + modulation before attention */
  WX_TRACE_QKV = 1,   /* fused q|k|v projection */
  WX_TRACE_ROPE = 2,  /* QK-RMSNorm + RoPE (+ the sequence-parallel exchange and its waits) */
  WX_TRACE_ATTN = 3,  /* routing + flash attention (+ the return exchange) */
  WX_TRACE_OUT = 4,   /* out projection + gated residual (PAB reuse: the cached gated residual) */
  WX_TRACE_MLP = 5,   /* RMSNorm + modulation, fc1 + activation, fc2 + gated residual */
  WX_TRACE_PHASES = 6
};
enum { WX_TRACE_DENSE = 0, WX_TRACE_SPARSE = 1, WX_TRACE_REUSE = 2 };
#define WX_TRACE_FIELDS 9
int wx_ctx_trace_enable(wx_ctx* ctx, int enable);
int wx_ctx_trace_read(wx_ctx* ctx, double* records, int max_records, int* count);

/* ---------------------------------------------------- quantized linear */
/* Affine group quantization of fp32 w [n, k] (the offline step of
 * model/minimax h3/tools/quantize_h3_g64.py:92-99, done on the GPU). */
int wx_quantize_affine(wx_ctx* ctx, const float* w, int64_t n, int64_t k, int group, int bits,
                       uint32_t* wq, void* scales, void* biases);
/* MfLinear.dequantizedWeight (H3Common.swift:379-401): w_out[n][k] =
 * bf16(q*scale + bias) computed in fp32. */
int wx_dequantize_affine(wx_ctx* ctx, const wx_qweight* w, void* w_out);
/* MfLinear.forward quantized branch (H3Common.swift:341-377; quantizedMM
 * :358-359, +bias :366-368) with a fused epilogue (wx_epilogue).
 * x [m, k] row pitch lda; y [m, n] (SWIGLU: [m, n/2]) row pitch ldy;
 * gate [num_mod_rows, n] and resid [m, n] (pitch ldy) for WX_EPI_GATE_RESID. */
int wx_qlinear(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
               int epilogue, const void* gate, const void* resid, const uint32_t* rowmap,
               void* y, int64_t ldy, void* y_raw);

/* Bytes of the packed LoRA operands of a linear [n, k] with `count` adapters:
 * *R = sum r_i rounded up to 64, *at_bytes = R*k*2, *bt_bytes = n*R*2. */
int wx_lora_pack_bytes(int64_t n, int64_t k, const wx_lora* l, int count, int64_t* R, size_t* at_bytes,
                       size_t* bt_bytes);
/* Build the packed operands (device buffers at, bt of wx_lora_pack_bytes' sizes)
 * from adapters in device memory; at = bf16(scale_i * A_i^T), bt = B_i^T. */
int wx_lora_pack_build(wx_ctx* ctx, int64_t n, int64_t k, const wx_lora* l, int count, wx_lora_pack* out);
/* wx_qlinear plus the LoRA delta (MfLinear.forward with lora.hasAdapters,
 * H3Common.swift:369-375): two MMA passes into one accumulator, then the epilogue.
 * lora NULL = wx_qlinear. WX_EPI_SWIGLU is supported. */
int wx_qlinear_lora(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                    const wx_lora_pack* lora, int epilogue, const void* gate, const void* resid,
                    const uint32_t* rowmap, void* y, int64_t ldy, void* y_raw);

/* No counterpart in the reference. wx_qlinear for callers that cannot allocate
 * device memory (a host whose engine or restricted allocator owns every device
 * allocation, or a plugin handed only a stream and tensors): it takes a
 * cudaStream_t instead of a context and allocates nothing. The expanded bf16
 * weight lives in a 64 MiB static device array inside libwx, created on every
 * GPU that loads the library and held until exit, so w->n * w->k may be at
 * most 33,554,432; larger weights, and WX_EPI_SWIGLU, are rejected
 * (WX_ERR_INVALID / WX_ERR_UNSUPPORTED). With CUDA's lazy module loading (the
 * default) the array is reserved on a device at the first call there, and that
 * call also looks up its address (cudaGetSymbolAddress): make the first call on
 * each device during set-up, before any stream capture. All calls share the
 * array: calls that overlap on the GPU race. Other arguments and results are
 * those of wx_qlinear; a failure's message is in wx_qlinear_noalloc_last_error. */
int wx_qlinear_noalloc(void* stream, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                       int epilogue, const void* gate, const void* resid, const uint32_t* rowmap,
                       void* y, int64_t ldy, void* y_raw);
/* No counterpart in the reference. Device-side status of the wx_qlinear_noalloc
 * calls on the current device: synchronises `stream`, reads the error word their
 * kernels write when a bounded wait expires, clears it, and returns WX_ERR_DEVICE
 * if it was set (WX_OK otherwise). Allocates nothing. */
int wx_qlinear_noalloc_check(void* stream);
/* No counterpart in the reference. Message of the last failed wx_qlinear_noalloc
 * or wx_qlinear_noalloc_check call on this thread. */
const char* wx_qlinear_noalloc_last_error(void);

/* ------------------------------------------------------ checkpoints */
/* Safetensors container (H3Weights, H3Common.swift:180-261): the file is mapped
 * read-only, the header parsed once, tensors copied to device memory on demand. */
typedef struct wx_st_file wx_st_file;
typedef struct wx_st_info {
  char dtype[8];      /* safetensors dtype name: "BF16", "F32", "U32", ... */
  int32_t ndim;
  int64_t shape[8];
  uint64_t offset;    /* byte offset in the file */
  uint64_t nbytes;
  const void* host;   /* the bytes in the mapping (valid until wx_st_close) */
} wx_st_info;
int wx_st_open(const char* path, wx_st_file** out);
int wx_st_close(wx_st_file* f);
/* message of the last wx_st_* failure of this thread */
const char* wx_st_last_error(void);
int64_t wx_st_count(const wx_st_file* f);
/* name of tensor i, 0 <= i < wx_st_count (valid until wx_st_close) */
const char* wx_st_name(const wx_st_file* f, int64_t i);
/* WX_ERR_INVALID when the name is absent (H3Weights.get returning nil) */
int wx_st_find(const wx_st_file* f, const char* name, wx_st_info* out);
/* copy a tensor's bytes to device memory on the context stream (returns when done) */
int wx_st_upload(wx_ctx* ctx, const wx_st_file* f, const char* name, void* dst, uint64_t dst_bytes);
/* H3Weights.getQuantized + MfLinear.load geometry (H3Common.swift:243-258, 311-338):
 * prefix.weight (U32 [n, k*bits/32]) with prefix.scales/.biases or
 * prefix.weight.scales/.weight.biases ([n, k/group]); bits = 32*w_cols/in_features,
 * group = in_features/s_cols; bias->dtype[0] == 0 when prefix.bias is absent. */
int wx_st_find_qlinear(const wx_st_file* f, const char* prefix, int64_t in_features, wx_st_info* wq,
                       wx_st_info* scales, wx_st_info* biases, wx_st_info* bias, int32_t* bits, int32_t* group);

/* ------------------------------------------------------ fused row ops */
/* H3FusedKernels.fusedRmsnormRope (网络算子-融合-RMSNormRoPE-通用.swift:111-129):
 * rows (s, h) of head_dim at x[s*x_stride + h*head_dim]; cos/sin [S, rot/2] bf16;
 * out may alias x. */
int wx_qk_norm_rope(wx_ctx* ctx, const void* x, int64_t x_stride, int64_t S, int H, int head_dim,
                    const void* w, const void* cos_t, const void* sin_t, int rot, float eps,
                    void* out, int64_t out_stride);
/* q and k of a packed qkv buffer [S, 3*H*head_dim] normalised + rotated in place
 * in one launch (the two fusedRmsnormRope calls of H3AttnW.forward, H3Transformer.swift:454-475) */
int wx_qk_norm_rope_qkv(wx_ctx* ctx, void* qkv, int64_t S, int H, int head_dim, const void* q_w,
                        const void* k_w, const void* cos_t, const void* sin_t, int rot, float eps);
/* The q|k|v projection of H3AttnW.forward together with its two fusedRmsnormRope calls
 * (H3Transformer.swift:451-475): y = MfLinear(x) ([m, 3*H*head_dim] bf16, pitch ldy; with the
 * LoRA delta when lora != NULL), then q and k normalised (q_w / k_w) and rotated per head.
 * head_dim 128 with rot % 16 == 0 runs as ONE GEMM whose epilogue does the norm and the
 * rotation, bit-identical to the two-pass wx_qlinear (M > 512) followed by
 * wx_qk_norm_rope_qkv; other geometries run those two calls. */
int wx_qkv_norm_rope(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                     const wx_lora_pack* lora, int H, int head_dim, const void* q_w, const void* k_w,
                     const void* cos_t, const void* sin_t, int rot, float eps, void* y, int64_t ldy);
/* H3FusedKernels.fusedNormModscale (fused:262-283); rowmap NULL = fusedNormModscaleRow (:295-315) */
int wx_norm_modscale(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w,
                     const void* shift, const void* scale, const uint32_t* rowmap, float eps,
                     void* out);
/* H3FusedKernels.fusedModGate (fused:324-343): out = bf16(x + other*gate[map[r]]) */
int wx_mod_gate(wx_ctx* ctx, const void* x, const void* other, const void* gate,
                const uint32_t* rowmap, int64_t S, int64_t hidden, void* out);
/* H3FusedKernels.buildRowModMap (fused:238-250), host memory in and out */
int wx_build_row_mod_map(const wx_mod_run* runs, int nruns, int64_t count, uint32_t* map_out);

/* ----------------------------------------------------------- attention */
/* Routing tables of H3SolAttn.forward (SOL:455-497), for inspection/tests.
 * q/k/v rows at base + s*row_stride + h*head_dim; nb = ceil((S-g)/block).
 * sel [H,nb,nb] u8, thr [H,nb] f32, cm [H,nb,nb] bf16, vsum [H,nb,hd] bf16, lens [nb] f32 */
int wx_sol_route(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t row_stride,
                 int64_t S, int H, int head_dim, const wx_sparse_spec* spec, float scale,
                 uint8_t* sel, float* thr, void* cm, void* vsum, float* lens);
/* top-k router (benchmark mode); scores [H,nb,nb] f32, other outputs as above */
int wx_topk_route(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t row_stride,
                  int64_t S, int H, int head_dim, const wx_sparse_spec* spec, float scale,
                  uint8_t* sel, float* scores, void* cm, void* vsum, float* lens);
/* H3SolAttn.forward (SOL:388-532) / scaledDotProductAttention for dense layers:
 * routing + tcgen05 flash attention; out rows at out + s*out_stride + h*head_dim.
 * head_dim 128 or 64; q/k/v rows 16-byte aligned. */
int wx_sparse_attention(wx_ctx* ctx, const void* q, const void* k, const void* v,
                        int64_t row_stride, int64_t S, int H, int head_dim,
                        const wx_sparse_spec* spec, float scale, void* out, int64_t out_stride);
/* the flash kernel alone with a caller-provided selection sel [H,nb,nb] (device);
 * cm/vsum/lens are needed only when spec->tail is set */
int wx_attention_from_sel(wx_ctx* ctx, const void* q, const void* k, const void* v,
                          int64_t row_stride, int64_t S, int H, int head_dim,
                          const wx_sparse_spec* spec, float scale, const uint8_t* sel,
                          const void* cm, const void* vsum, const float* lens, void* out,
                          int64_t out_stride);

/* --------------------------------------------------- PAB + schedules (host) */
/* attnBroadcastRefresh (网络算子-注意力跨步缓存-通用.swift:73-79) */
int wx_pab_refresh(int i, uint32_t steps, uint32_t k);
/* attnBroadcastMustRefresh (:85-87) */
int wx_pab_must_refresh(double cached_sigma, double sigma, double max_stale);
/* attnBroadcastPlan (:92-105): out[nfe] = 1 refresh / 0 reuse; returns nfe */
int wx_pab_plan(const double* sigmas, int nsigmas, uint32_t k, double max_stale, uint8_t* out);
/* sigmaSchedule (model/minimax h3/H3Layout.swift:175-182): out[steps+1] */
int wx_sigma_schedule(uint32_t steps, double shift, double* out);
/* sparseModeForLayer (H3Layout.swift:896-906); policy 0 off, 1 mix, 2 spatial, 3 temporal;
 * returns 0 dense, 1 spatial, 2 temporal */
int wx_sparse_mode_for_layer(int layer, int nlayers, int policy);

/* ------------------------------------------------------------ DiT block */
/* Byte size of the scratch buffer wx_dit_block_forward needs for S rows. */
int64_t wx_dit_block_scratch_bytes(const wx_dit_config* cfg, int64_t S);
/* One iteration of the block loop of H3DiT.forward (H3Transformer.swift:1078-1159):
 *   refresh (or pab_slot == NULL): m1 = norm_modscale(h); at = attn(m1) [-> pab_slot]
 *   reuse: at = pab_slot
 *   hAttn = h + at*gateMSA; m2 = norm_modscale(hAttn); h = hAttn + mlp(m2)*gateMLP
 * h [S, hidden] bf16 is updated in place. cos/sin [S, rot/2] bf16.
 * scratch: wx_dit_block_scratch_bytes(cfg, S) bytes of device memory. */
int wx_dit_block_forward(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w,
                         const wx_block_mods* mods, const uint32_t* rowmap, void* h, int64_t S,
                         const void* cos_t, const void* sin_t, const wx_sparse_spec* spec,
                         void* pab_slot, int refresh, void* scratch);

/* The same block forward as a CUDA graph: captured once (on a private stream, nothing
 * runs), replayed on the context stream by wx_graph_launch. Every pointer and scalar of
 * the call is baked in; the caller refreshes the buffers' contents between replays
 * (h is updated in place by each replay, as by wx_dit_block_forward). Cuts the gaps
 * between the block's ~12-20 dependent launches where they matter (small S).
 * Single-GPU contexts only (WX_ERR_UNSUPPORTED after wx_ctx_init_comm with > 1 rank). */
typedef struct wx_graph wx_graph;
int wx_dit_block_graph_create(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w,
                              const wx_block_mods* mods, const uint32_t* rowmap, void* h, int64_t S,
                              const void* cos_t, const void* sin_t, const wx_sparse_spec* spec, void* pab_slot,
                              int refresh, void* scratch, wx_graph** out);
int wx_graph_launch(wx_ctx* ctx, wx_graph* g);
/* libwx kernels one replay launches */
int64_t wx_graph_kernels(const wx_graph* g);
int wx_graph_destroy(wx_graph* g);

/* ------------------------------------------- Ulysses sequence parallelism */
/* No counterpart in the reference (it runs on a single device, with no
 * DP/TP/SP). Rank `rank` of P owns rows [row0, row0 + rows) of the packed
 * sequence (S/P each) for every row-local op, and heads [head0, head0 + heads)
 * (H/P each) for attention over the whole sequence. Before attention each rank
 * sends peer r a chunk of qkv_chunk elements = [rows][3][heads*head_dim] (q|k|v
 * of r's heads for the sender's rows) and receives [S][3*heads*head_dim], the
 * packed q|k|v of its own heads; after attention it sends peer r the rows of r
 * ([rows][heads*head_dim], out_chunk elements) and gathers its rows of every
 * head. S % P == 0 and H % P == 0 are required. */
typedef struct wx_sp_plan {
  int64_t S;
  int64_t rows;
  int64_t row0;
  int32_t P;
  int32_t rank;
  int32_t H;
  int32_t heads;
  int32_t head0;
  int32_t head_dim;
  int64_t qkv_chunk;
  int64_t out_chunk;
} wx_sp_plan;
int wx_sp_make_plan(int64_t S, int H, int head_dim, int P, int rank, wx_sp_plan* out);
/* NCCL bootstrap: rank 0 creates the 128-byte id, every rank passes it to
 * wx_ctx_init_comm (NCCL is loaded at run time, reusing a copy already loaded
 * into the process). */
int wx_comm_unique_id(void* id128);
int wx_ctx_init_comm(wx_ctx* ctx, int nranks, int rank, const void* id128);
/* WX_ERR_CUDA if NCCL reported an asynchronous error on the communicator */
int wx_ctx_comm_check(wx_ctx* ctx);
/* aborts the communicator (pending collectives return); the context keeps working on one GPU */
int wx_ctx_comm_abort(wx_ctx* ctx);
/* exchange path of the sequence-parallel block: 1 = NVLink peer memory (the
 * QK-norm/RoPE kernel and the attention kernels store straight into the other
 * ranks' buffers, opened through CUDA IPC; WX_SP_P2P=0 turns it off), 0 = NCCL
 * all-to-alls, -1 = not decided yet (decided collectively at the first refreshed
 * block of a group) */
int wx_ctx_sp_exchange(wx_ctx* ctx);
/* No counterpart in the reference (it has no multi-GPU path). Limit of every wait for
 * another GPU's signal (the exchange flags of wx_dit_block_forward_sp, and
 * wx_ctx_wait_flags): a waiting kernel that sees no signal within `seconds` records
 * a device error (wx_ctx_check_device then returns WX_ERR_DEVICE) and returns, so a
 * rank that never signals turns into an error on the others instead of a hang; the
 * context stays usable. Default 10 s; 0 < seconds <= 600. */
int wx_ctx_set_peer_wait_limit(wx_ctx* ctx, double seconds);
/* No counterpart in the reference. Cross-GPU signalling on the context stream, the
 * mechanism of the peer-memory exchange: signal stores `epoch` into flags[0..n) with
 * release semantics at system scope once this stream's earlier writes are visible
 * (flags may be another GPU's memory opened in this process); wait holds the stream
 * until every flags[i] has reached `epoch` (acquire, wrap-around order), bounded by
 * the peer wait limit. flags 4-byte aligned, n > 0. */
int wx_ctx_signal_flags(wx_ctx* ctx, uint32_t* flags, int n, uint32_t epoch);
int wx_ctx_wait_flags(wx_ctx* ctx, const uint32_t* flags, int n, uint32_t epoch);
int64_t wx_dit_block_sp_scratch_bytes(const wx_dit_config* cfg, int64_t S, int P);
/* wx_dit_block_forward on this rank's rows of an S-row sequence (the context's
 * communicator decides P and the rank): h/rowmap/cos/sin/pab_slot are the
 * local rows; spec->g counts strip rows of the whole sequence. Refresh steps
 * run two all-to-alls around attention; reuse steps communicate nothing. */
int wx_dit_block_forward_sp(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w,
                            const wx_block_mods* mods, const uint32_t* rowmap, void* h, int64_t S,
                            const void* cos_t, const void* sin_t, const wx_sparse_spec* spec,
                            void* pab_slot, int refresh, void* scratch);

/* ------------------------------------------------------- sampler step */
/* Weights of the DiT around the blocks (H3DiT, H3Transformer.swift:1022-1203). */
typedef struct wx_dit_model {
  const wx_dit_config* cfg;
  int32_t n_blocks;
  int32_t patch_dim;           /* latent features per packed row (96) */
  const wx_block_weights* blocks; /* [n_blocks] */
  const wx_block_mods* mods;      /* [n_blocks] AdaLN tables (precomputeAdaln output) */
  const float* embed_w;        /* [patch_dim, hidden] fp32 patch embed */
  const float* embed_b;        /* [hidden] */
  const void* final_norm;      /* [hidden] bf16 */
  const float* out_w;          /* [hidden, patch_dim] fp32 final projection */
  const float* out_b;          /* [patch_dim] */
  /* audio stream (H3DiT audioPatchW/B, audioOutW/B; H3Transformer.swift:1036-1041,
   * 1176-1188); audio_dim 0 = no audio weights */
  int32_t audio_dim;           /* latent features per audio row (32) */
  const float* audio_embed_w;  /* [audio_dim, hidden] */
  const float* audio_embed_b;  /* [hidden] */
  const float* audio_out_w;    /* [hidden, audio_dim] */
  const float* audio_out_b;    /* [audio_dim] */
} wx_dit_model;

/* One sampler step (the loop body of H3Pipeline.swift:1398-1445): packed rows
 * [0, text_rows) are text states, rows [text_rows, S) come from the patch embed
 * of `latents` ([S - text_rows, patch_dim] fp32: reference/cond rows, then the
 * video latent; audio rows, when given, from the audio embed, see below),
 * rows [video_start, S) are denoised: final head, negated
 * velocity, and latents[video rows] += -v * dsigma in place. Layers follow
 * sparse_mode_for_layer(policy); `spec` is used on the sparse layers. PAB:
 * pab_slots[bi] ([rows, hidden] each, or pab_slots NULL) are written when
 * `refresh` and read otherwise. Under sequence parallelism the context's rank
 * handles rows [rank*S/P, (rank+1)*S/P): rowmap/cos/sin/pab slots are those
 * rows, text_states and latents are whole. */
typedef struct wx_dit_step_args {
  int64_t S;
  int64_t text_rows;
  int64_t video_start;
  const void* text_states;     /* [text_rows, hidden] bf16 */
  float* latents;              /* [S - text_rows, patch_dim] fp32 */
  const uint32_t* rowmap;      /* [rows] */
  const void* cos_t;           /* [rows, rot/2] bf16 */
  const void* sin_t;
  const void* final_shift;     /* [hidden] bf16, this step's row of the final AdaLN table */
  const void* final_scale;
  const wx_sparse_spec* spec;
  int32_t policy;              /* 0 off (all dense), 1 mix, 2 spatial, 3 temporal */
  int32_t refresh;
  void* const* pab_slots;
  float dsigma;
  int32_t reserved;
  void* scratch;               /* wx_dit_step_scratch_bytes */
  /* Audio rows (refAudio and audio segments of the PackedLayout): packed rows
   * [audio_segs[2i], audio_segs[2i+1]) (host array, ascending, inside
   * [text_rows, video_start)) take their embeddings from audio_latents
   * ([sum of segment rows, audio_dim] fp32, segments in order) and every other
   * row after the text from `latents` in order (so `latents` then holds
   * S - text_rows - audio rows). Segment audio_target (-1 = none) is denoised:
   * final head with audio_final_shift/scale (the audio t row of the final
   * tables), then audio_latents += (aout * audio_vscale) * audio_dsigma
   * (H3DiT.forward's -slope and the pipeline's dσa/slope, H3Pipeline.swift:1436-1443). */
  const int64_t* audio_segs;
  int32_t n_audio_segs;
  int32_t audio_target;
  float* audio_latents;
  const void* audio_final_shift;
  const void* audio_final_scale;
  float audio_vscale;
  float audio_dsigma;
} wx_dit_step_args;
int64_t wx_dit_step_scratch_bytes(wx_ctx* ctx, const wx_dit_model* m, int64_t S);
int wx_dit_step(wx_ctx* ctx, const wx_dit_model* m, const wx_dit_step_args* a);

/* Classifier-free guidance of the SelfLift sampler step (SelfLiftH3-(h3专属).swift:826-845):
 * the forward runs on the positive condition (a->text_states, with the PAB slots and
 * a->refresh as in wx_dit_step) and, when text_states_neg is given, again on the negative
 * condition with attention computed fresh and no PAB slot read or written; the video output
 * is v = v_neg + cfg_scale * (v_pos - v_neg) in fp32 (audio takes the positive branch).
 * update = 1 applies the Euler update of wx_dit_step with that output; update = 0 leaves the
 * latents as they are. velocity_out, when not NULL, receives the video output
 * ([this rank's video rows, patch_dim] fp32, the forward's negated velocity, the `out.video`
 * the sampler adds times dsigma). text_states_neg NULL: a single forward (a velocity-out
 * mode of wx_dit_step). Scratch: wx_dit_step_guided_scratch_bytes bytes in a->scratch. */
typedef struct wx_dit_guidance {
  const void* text_states_neg; /* [text_rows, hidden] bf16, padded to the positive's text_rows; NULL = no CFG */
  float cfg_scale;
  int32_t update;              /* 1: Euler update of the latents; 0: none */
  float* velocity_out;         /* NULL or [video rows of this rank, patch_dim] fp32 */
} wx_dit_guidance;
int64_t wx_dit_step_guided_scratch_bytes(wx_ctx* ctx, const wx_dit_model* m, int64_t S);
int wx_dit_step_guided(wx_ctx* ctx, const wx_dit_model* m, const wx_dit_step_args* a, const wx_dit_guidance* g);

/* fp32 dense linear y = x*w + b (H3TensorOps.denseLinear: patch embed and final
 * head islands, H3Transformer.swift:1036-1039, 1192-1203); w [k, n] fp32. */
int wx_dense_f32(wx_ctx* ctx, const float* x, int64_t m, int64_t k, const float* w, int64_t n,
                 const float* b, float* y);
/* bf16 -> fp32 copy of rows (the .asType(.float32) before the final head) */
int wx_bf16_to_f32(wx_ctx* ctx, const void* x, int64_t n, float* y);
/* fp32 -> bf16 (embedding cast) */
int wx_f32_to_bf16(wx_ctx* ctx, const float* x, int64_t n, void* y);
/* Euler update of the sampler loop (H3Pipeline.swift:1436-1443) with the
 * negated velocity of H3DiT.forward (:1188): x[i] += (-v[i]) * dsigma */
int wx_euler_update(wx_ctx* ctx, float* x, const float* v, int64_t n, float dsigma);

/* ---------------------------------------------- RoPE tables (per generation) */
/* axisFromSqrtArea (H3Layout.swift:188-194): n = dim/patch coordinates
 * (i*ratio/n + (1-ratio)/2)*32, ratio = dim/sqrt_area, written to out (cap
 * values); returns n (out NULL: only n) or a negative status. */
int wx_axis_from_sqrt_area(uint32_t dim, uint32_t patch, double sqrt_area, double* out, int cap);
/* videoTSpan (H3Layout.swift:197-200): 5/3 * [1,4,4,4,4][k % 5] */
double wx_video_t_span(int k);
/* videoTGrid (H3Layout.swift:202-210): out[i] = origin + sum_{j<i} span(j) */
int wx_video_t_grid(uint32_t n, double origin, double* out);
/* writeFrameGrid (H3Layout.swift:683-694): rows [row, row + nh*nw) of pos [S,3]
 * (host doubles) get (t, h_axis[a], w_axis[b]), b fastest. */
int wx_write_frame_grid(double* pos, int64_t row, double t, const double* h_axis, int nh, const double* w_axis,
                        int nw);
/* buildRope (H3Layout.swift:725-740): pos [S,3] fp32 and inv_freq [nf] fp32 on
 * the device -> cos_t / sin_t [S, 3*nf] bf16, column a*nf + f = pos[s][a]*inv[f]. */
int wx_build_rope(wx_ctx* ctx, const float* pos, int64_t S, const float* inv_freq, int nf, void* cos_t,
                  void* sin_t);

/* ------------------------------------------------ conditioning (per generation) */
/* Dense MfLinear (H3Common.swift:304-308, 361-366): w [k, n] bf16 stored
 * pre-transposed; y = bf16(bf16(x w) + bias). */
typedef struct wx_dense_bf16 {
  const void* w;    /* [k, n] bf16 */
  const void* bias; /* [n] bf16 or NULL */
  int64_t k;
  int64_t n;
} wx_dense_bf16;
/* y [m, n] = the dense linear of x [m, k]; for the few rows of an AdaLN table */
int wx_linear_bf16(wx_ctx* ctx, const void* x, int64_t m, const wx_dense_bf16* w, void* y);
/* H3TimeEmbedder.forward (H3Transformer.swift:287-302): ts (host, m <= 64) ->
 * temb [m, dim] fp32 = dense(silu(dense(sinusoid(ts), w_in [freq_dim, dim], b_in)),
 * w_out [dim, dim], b_out); sinusoid row = [cos(t f_j) | sin(t f_j)],
 * f_j = exp(-ln(10000) j / (freq_dim/2)). */
int wx_time_embed(wx_ctx* ctx, const double* ts, int m, int freq_dim, const float* w_in, const float* b_in,
                  int64_t dim, const float* w_out, const float* b_out, float* temb);
/* H3AdalnLUT.coeffs (H3Transformer.swift:338-349): row round(t (n_rows-1))
 * (ties away from zero, clamped) of t_table [n_rows, rank] fp32, as bf16 [m, rank]. */
int wx_adaln_lut_coeffs(wx_ctx* ctx, const double* ts, int m, const float* t_table, int64_t n_rows, int rank,
                        void* coeffs);
/* MLX silu on a bf16 array: y = bf16(x * bf16(sigmoid(x))) */
int wx_silu_bf16(wx_ctx* ctx, const void* x, int64_t n, void* y);
/* H3AdalnW.forward (H3Transformer.swift:392-403) of one block (expand 6,
 * modalities 3) or of the final layer (expand 2, modalities 1): temb [m, k]
 * bf16 (SiLU applied first when apply_silu) through the adaln_proj linear,
 * quantized `qw` (+ optional LoRA pack) or dense `dw` (exactly one), then split:
 * tables[e] [m*modalities, hidden] bf16, row t*modalities + tag
 * = y[t, (tag*expand + e)*hidden : +hidden]. Block tables feed wx_block_mods
 * (shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = tables[0..5]);
 * final tables are [shift, scale]. */
int wx_adaln_tables(wx_ctx* ctx, const void* temb, int64_t m, int64_t k, int apply_silu, const wx_qweight* qw,
                    const wx_lora_pack* lora, const wx_dense_bf16* dw, int expand, int modalities,
                    void* const* tables);
/* rmsNormLast (H3Common.swift:502-508): out = bf16(x * rsqrt(mean(x^2) + eps) * w) */
int wx_rms_norm(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w, float eps, void* out);
/* One token-refiner block (H3DiT.refineText loop body, H3Transformer.swift:1003-1010;
 * weights H3RefinerBlockW :676-700, in a wx_block_weights): h [L, hidden] in place,
 * h += attn(rmsNorm(h, norm1)) with per-head q/k RMSNorm, no RoPE and dense
 * attention; h += mlp(rmsNorm(h, norm2)) (cfg->mlp_kind). */
int64_t wx_refiner_scratch_bytes(const wx_dit_config* cfg, int64_t L);
int wx_refiner_block_forward(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w, void* h, int64_t L,
                             void* scratch);
/* H3DiT.refineText (H3Transformer.swift:993-1016): text [L, text_dim] bf16 ->
 * out [L, hidden]; identity copy when text_dim == hidden; else condition_proj
 * (+ LoRA), the n_blocks refiner blocks, and the final RMSNorm when final_norm. */
int64_t wx_refine_text_scratch_bytes(const wx_dit_config* cfg, int64_t L, int64_t text_dim);
int wx_refine_text(wx_ctx* ctx, const wx_dit_config* cfg, const wx_qweight* condition_proj,
                   const wx_lora_pack* condition_lora, const wx_block_weights* blocks, int n_blocks,
                   const void* final_norm, const void* text, int64_t L, int64_t text_dim, void* out, void* scratch);

#ifdef __cplusplus
}
#endif
#endif /* WX_API_H */
