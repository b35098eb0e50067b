// wx_cond.cu — the conditioning around the DiT blocks of H3DiT
// (model/minimax h3/H3Transformer.swift):
//  * the timestep embedder (H3TimeEmbedder.forward, :287-302, an fp32 island):
//    sinusoid [cos | sin] of t times 10000^(-j/half) → dense → SiLU → dense;
//  * the AdaLN table precompute (H3DiT.precomputeAdaln, :957-988, with
//    H3AdalnW.forward :392-403 and the lookup variant H3AdalnLUT :319-350):
//    SiLU(bf16 t-embedding) → the block's adaln_proj linear (quantized, or dense
//    for the folded LUT checkpoints) → `expand` tables of [t·modalities, hidden];
//  * the text refiner (H3DiT.refineText, :993-1016, with H3RefinerBlockW
//    :676-700): condition_proj, then per block h += attn(rmsNorm(h)) and
//    h += mlp(rmsNorm(h)) with dense attention and no RoPE, then a final RMSNorm.
// All of it runs once per generation (tables) or once per prompt (refiner);
// none of it is on the per-step path, so the kernels here are simple.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

int launch_qk_norm_rope(wx_ctx* ctx, const void* x, int64_t x_stride, void* out, int64_t out_stride,
                        int64_t part_off, int nparts, int64_t S, int H, int hd, const void* w0, const void* w1,
                        const void* cos_t, const void* sin_t, int rot, float eps);
int launch_norm_modscale(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w, const void* shift,
                         const void* scale, const uint32_t* rowmap, float eps, void* out);
bool qweight_ok(const wx_qweight* w);
size_t attention_scratch_bytes(int64_t S, int H, int hd, const wx_sparse_spec* spec);
int attention_with_scratch(wx_ctx* ctx, const void* q, const void* k, const void* v, int64_t rs, int64_t S, int H,
                           int hd, const wx_sparse_spec* spec, float scale, void* out, int64_t os, void* scratch);

constexpr int kMaxTs = 64;      // timesteps per call (a plan holds a handful)
constexpr int kMaxTables = 8;   // AdaLN `expand` (6 per block, 2 for the final layer)

struct TsArg {
  double t[kMaxTs];
};
struct IdxArg {
  int32_t i[kMaxTs];
};
struct TablePtrs {
  __nv_bfloat16* p[kMaxTables];
};

// emb[r, j] = cos(t_r f_j), emb[r, half + j] = sin(t_r f_j), f_j = exp(-ln(10000) j / half),
// evaluated in double and rounded to fp32 as the reference's host loop does (:291-299)
__global__ void timestep_sinusoid_kernel(TsArg ts, int m, int dim, float* __restrict__ out) {
  const int half = dim / 2;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m * half) return;
  const int r = i / half, j = i % half;
  const double freq = exp(-log(10000.0) * (double)j / (double)half);
  const double arg = ts.t[r] * freq;
  out[(int64_t)r * dim + j] = (float)cos(arg);
  out[(int64_t)r * dim + half + j] = (float)sin(arg);
}

// MLX sigmoid: y = 1 / (1 + exp(-|x|)), mirrored for x < 0; silu(x) = x * sigmoid(x)
__device__ __forceinline__ float sigmoid_mlx(float x) {
  const float y = 1.0f / (1.0f + expf(-fabsf(x)));
  return x < 0.0f ? 1.0f - y : y;
}

// fp32 SiLU in place (the time embedder's fp32 island)
__global__ void silu_f32_kernel(float* __restrict__ x, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = x[i] * sigmoid_mlx(x[i]);
}

// bf16 SiLU as MLX composes it on a bf16 array: s = bf16(sigmoid(x)), y = bf16(x * s)
__global__ void silu_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t n, __nv_bfloat16* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = __bfloat162float(x[i]);
    const float s = round_bf16(sigmoid_mlx(v));
    y[i] = __float2bfloat16_rn(v * s);
  }
}

// H3AdalnLUT.coeffs (:338-349) + .asType(bf16): out[r, c] = bf16(table[idx_r, c])
__global__ void lut_gather_kernel(const float* __restrict__ table, int rank, IdxArg idx, int m,
                                  __nv_bfloat16* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m * rank) return;
  const int r = i / rank, c = i % rank;
  out[i] = __float2bfloat16_rn(table[(int64_t)idx.i[r] * rank + c]);
}

// The dense MfLinear branch (H3Common.swift:361-366): y = bf16(bf16(x w) + b), w [k, n]
// pre-transposed; fp32 accumulation in k order. One thread per output column, up
// to 8 rows per thread (blockIdx.y walks the row groups): w is read once per group,
// coalesced across the warp. Sized for the few timestep rows of an AdaLN table.
__global__ void linear_bf16_small_kernel(const __nv_bfloat16* __restrict__ x, int64_t m, int64_t k,
                                         const __nv_bfloat16* __restrict__ w, int64_t n,
                                         const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ y) {
  const int64_t col = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * 8;
  if (col >= n) return;
  const int rows = (int)std::min<int64_t>(8, m - r0);
  float acc[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) acc[r] = 0.0f;
  for (int64_t kk = 0; kk < k; ++kk) {
    const float wv = __bfloat162float(w[kk * n + col]);
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < rows) acc[r] = fmaf(__bfloat162float(x[(r0 + r) * k + kk]), wv, acc[r]);
  }
  const float b = bias ? __bfloat162float(bias[col]) : 0.0f;
#pragma unroll
  for (int r = 0; r < 8; ++r)
    if (r < rows) {
      float v = round_bf16(acc[r]);
      if (bias) v = v + b;
      y[(r0 + r) * n + col] = __float2bfloat16_rn(v);
    }
}

// H3AdalnW.forward's reshape + splitEqual (:395-403): y [m, modalities·expand·hidden]
// with column (tag·expand + e)·hidden + c → table e, row t·modalities + tag, column c.
// 8 bf16 per thread (hidden % 8 == 0).
__global__ void adaln_split_kernel(const __nv_bfloat16* __restrict__ y, int64_t m, int expand, int modalities,
                                   int64_t hidden, TablePtrs tabs) {
  const int64_t hv = hidden / 8;
  const int64_t total = m * modalities * expand * hv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c8 = i % hv;
    const int64_t rest = i / hv;
    const int e = (int)(rest % expand);
    const int64_t row = rest / expand;  // t * modalities + tag
    const int64_t t = row / modalities, tag = row % modalities;
    const uint4 v = *reinterpret_cast<const uint4*>(y + t * modalities * expand * hidden +
                                                    (tag * expand + e) * hidden + c8 * 8);
    *reinterpret_cast<uint4*>(tabs.p[e] + row * hidden + c8 * 8) = v;
  }
}

__global__ void fill_bf16_kernel(__nv_bfloat16* __restrict__ p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = __float2bfloat16_rn(v);
}

static unsigned grid_1d(int64_t n, int threads, int sms) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, (int64_t)sms * 8));
}

static size_t al(size_t b) { return (b + 255) & ~size_t(255); }

// Scratch of one refiner block over L rows (offsets into one buffer).
struct RefinerLayout {
  size_t n, qkv, att, ha, f1, ones, wd, sw, lt, attn, h, total;
};

// text_dim > 0 also sizes the condition_proj's scratch and the projected rows `h`
static RefinerLayout refiner_layout(const wx_dit_config* c, int64_t L, int64_t text_dim = 0) {
  RefinerLayout R{};
  const size_t inner = (size_t)c->heads * c->head_dim;
  const size_t fc1_n = c->mlp_kind == WX_MLP_SWIGLU ? 2 * (size_t)c->ffn : (size_t)c->ffn;
  size_t off = 0;
  R.n = off; off += al((size_t)L * c->hidden * 2);
  R.qkv = off; off += al((size_t)L * 3 * inner * 2);
  R.att = off; off += al((size_t)L * inner * 2);
  R.ha = off; off += al((size_t)L * c->hidden * 2);
  R.f1 = off; off += al((size_t)L * c->ffn * 2);
  R.ones = off; off += al((size_t)c->hidden * 2);
  const size_t wmax = std::max(std::max(std::max(3 * inner * (size_t)c->hidden, inner * (size_t)c->hidden),
                                        std::max(fc1_n * (size_t)c->hidden, (size_t)c->ffn * c->hidden)),
                               (size_t)std::max<int64_t>(text_dim, 0) * c->hidden);
  const size_t nmax = std::max(std::max(3 * inner, (size_t)c->hidden), fc1_n);
  R.wd = off; off += al(std::max(wmax * 2, qlinear_ws_need(L, (int64_t)nmax, 1)));
  R.sw = off; off += c->mlp_kind == WX_MLP_SWIGLU ? al((size_t)L * fc1_n * 2) : 0;
  R.lt = off; off += al((size_t)L * (size_t)std::max(0, c->lora_rank) * 2);
  R.attn = off; off += al(attention_scratch_bytes(L, c->heads, c->head_dim, nullptr));
  R.h = off; off += text_dim > 0 ? al((size_t)L * c->hidden * 2) : 0;
  R.total = off;
  return R;
}

static int refiner_block(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w, void* h, int64_t L,
                         uint8_t* base, const RefinerLayout& R) {
  const int64_t inner = (int64_t)cfg->heads * cfg->head_dim;
  void* n = base + R.n;
  void* qkv = base + R.qkv;
  void* att = base + R.att;
  void* ha = base + R.ha;
  void* f1 = base + R.f1;
  const void* ones = base + R.ones;
  void* wd = base + R.wd;
  void* sw = base + R.sw;
  void* lt = base + R.lt;
  int st;
  // n1 = rmsNorm(h, norm1)
  if ((st = launch_norm_modscale(ctx, h, L, cfg->hidden, w->norm1, nullptr, nullptr, nullptr, cfg->eps, n)))
    return st;
  // at = H3AttnW.forward(n1, rope: nil, sparse: nil): qkv, per-head RMSNorm of q and k
  // (no rotation), dense attention, out-projection; h + at through the residual
  // epilogue with a gate of ones (exact: bf16(h + bf16(at)))
  if ((st = qlinear_lora_with_scratch(ctx, n, L, cfg->hidden, &w->qkv, w->lora[0], WX_EPI_NONE, nullptr, nullptr,
                                      nullptr, qkv, 3 * inner, nullptr, wd, lt, nullptr)))
    return st;
  if ((st = launch_qk_norm_rope(ctx, qkv, 3 * inner, qkv, 3 * inner, inner, 2, L, cfg->heads, cfg->head_dim,
                                w->q_norm, w->k_norm, nullptr, nullptr, 0, cfg->eps)))
    return st;
  const uint8_t* qb = static_cast<const uint8_t*>(qkv);
  const float scale = (float)(1.0 / sqrt((double)cfg->head_dim));
  if ((st = attention_with_scratch(ctx, qb, qb + inner * 2, qb + 2 * inner * 2, 3 * inner, L, cfg->heads,
                                   cfg->head_dim, nullptr, scale, att, inner, base + R.attn)))
    return st;
  if ((st = qlinear_lora_with_scratch(ctx, att, L, inner, &w->out, w->lora[1], WX_EPI_GATE_RESID, ones, h, nullptr,
                                      ha, cfg->hidden, nullptr, wd, lt, nullptr)))
    return st;
  // h = hAttn + mlp(rmsNorm(hAttn, norm2))
  if ((st = launch_norm_modscale(ctx, ha, L, cfg->hidden, w->norm2, nullptr, nullptr, nullptr, cfg->eps, n)))
    return st;
  const int act = cfg->mlp_kind == WX_MLP_SWIGLU ? WX_EPI_SWIGLU : WX_EPI_GELU;
  if ((st = qlinear_lora_with_scratch(ctx, n, L, cfg->hidden, &w->fc1, w->lora[2], act, nullptr, nullptr, nullptr,
                                      f1, cfg->ffn, nullptr, wd, lt, sw)))
    return st;
  return qlinear_lora_with_scratch(ctx, f1, L, cfg->ffn, &w->fc2, w->lora[3], WX_EPI_GATE_RESID, ones, ha, nullptr, h,
                                   cfg->hidden, nullptr, wd, lt, nullptr);
}

static int check_refiner_block(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w) {
  WX_CHECK_ARG(ctx, w);
  const int64_t inner = (int64_t)cfg->heads * cfg->head_dim;
  const int64_t fc1_n = cfg->mlp_kind == WX_MLP_SWIGLU ? 2 * cfg->ffn : cfg->ffn;
  WX_CHECK_ARG(ctx, qweight_ok(&w->qkv) && w->qkv.k == cfg->hidden && w->qkv.n == 3 * inner);
  WX_CHECK_ARG(ctx, qweight_ok(&w->out) && w->out.k == inner && w->out.n == cfg->hidden);
  WX_CHECK_ARG(ctx, qweight_ok(&w->fc1) && w->fc1.k == cfg->hidden && w->fc1.n == fc1_n);
  WX_CHECK_ARG(ctx, qweight_ok(&w->fc2) && w->fc2.k == cfg->ffn && w->fc2.n == cfg->hidden);
  WX_CHECK_ARG(ctx, w->q_norm && w->k_norm && w->norm1 && w->norm2);
  WX_CHECK_ARG(ctx, lora_packs_ok(cfg, w));
  return WX_OK;
}

}  // namespace wx

using namespace wx;

extern "C" {

int wx_time_embed(wx_ctx* ctx, const double* ts, int m, int freq_dim, const float* w_in, const float* b_in,
                  int64_t dim, const float* w_out, const float* b_out, float* temb) {
  WX_CHECK_ARG(ctx, ctx && ts && w_in && w_out && temb && m > 0 && m <= kMaxTs);
  WX_CHECK_ARG(ctx, freq_dim > 0 && freq_dim % 2 == 0 && dim > 0);
  TsArg a{};
  for (int i = 0; i < m; ++i) a.t[i] = ts[i];
  int st = WX_OK;
  const size_t b_emb = al((size_t)m * freq_dim * 4);
  void* ws = workspace(ctx, b_emb + al((size_t)m * dim * 4), &st);
  if (!ws) return st;
  float* emb = static_cast<float*>(ws);
  float* h1 = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + b_emb);
  const int half = freq_dim / 2;
  timestep_sinusoid_kernel<<<(m * half + 255) / 256, 256, 0, ctx->stream>>>(a, m, freq_dim, emb);
  if ((st = launch_status(ctx, "timestep_sinusoid"))) return st;
  if ((st = wx_dense_f32(ctx, emb, m, freq_dim, w_in, dim, b_in, h1))) return st;
  silu_f32_kernel<<<grid_1d((int64_t)m * dim, 256, ctx->num_sms), 256, 0, ctx->stream>>>(h1, (int64_t)m * dim);
  if ((st = launch_status(ctx, "silu_f32"))) return st;
  return wx_dense_f32(ctx, h1, m, dim, w_out, dim, b_out, temb);
}

int wx_adaln_lut_coeffs(wx_ctx* ctx, const double* ts, int m, const float* t_table, int64_t n_rows, int rank,
                        void* coeffs) {
  WX_CHECK_ARG(ctx, ctx && ts && t_table && coeffs && m > 0 && m <= kMaxTs && n_rows > 0 && rank > 0);
  IdxArg idx{};
  for (int i = 0; i < m; ++i) {
    // Swift Double.rounded(): to nearest, ties away from zero; clamped to the table
    const double x = ts[i] * (double)(n_rows - 1);
    const double r = x < 0 ? -floor(-x + 0.5) : floor(x + 0.5);
    idx.i[i] = (int32_t)std::min<double>(std::max<double>(r, 0.0), (double)(n_rows - 1));
  }
  lut_gather_kernel<<<(m * rank + 255) / 256, 256, 0, ctx->stream>>>(t_table, rank, idx, m,
                                                                      static_cast<__nv_bfloat16*>(coeffs));
  return launch_status(ctx, "adaln_lut_gather");
}

int wx_silu_bf16(wx_ctx* ctx, const void* x, int64_t n, void* y) {
  WX_CHECK_ARG(ctx, ctx && x && y && n >= 0);
  if (!n) return WX_OK;
  silu_bf16_kernel<<<grid_1d(n, 256, ctx->num_sms), 256, 0, ctx->stream>>>(static_cast<const __nv_bfloat16*>(x), n,
                                                                           static_cast<__nv_bfloat16*>(y));
  return launch_status(ctx, "silu_bf16");
}

int wx_linear_bf16(wx_ctx* ctx, const void* x, int64_t m, const wx_dense_bf16* w, void* y) {
  WX_CHECK_ARG(ctx, ctx && x && y && w && w->w && w->k > 0 && w->n > 0 && m >= 0);
  if (!m) return WX_OK;
  dim3 grid((unsigned)((w->n + 127) / 128), (unsigned)((m + 7) / 8));
  WX_CHECK_ARG(ctx, grid.y <= 65535);
  linear_bf16_small_kernel<<<grid, 128, 0, ctx->stream>>>(
      static_cast<const __nv_bfloat16*>(x), m, w->k, static_cast<const __nv_bfloat16*>(w->w), w->n,
      static_cast<const __nv_bfloat16*>(w->bias), static_cast<__nv_bfloat16*>(y));
  return launch_status(ctx, "linear_bf16");
}

int wx_adaln_tables(wx_ctx* ctx, const void* temb, int64_t m, int64_t k, int apply_silu, const wx_qweight* qw,
                    const wx_lora_pack* lora, const wx_dense_bf16* dw, int expand, int modalities,
                    void* const* tables) {
  WX_CHECK_ARG(ctx, ctx && temb && tables && m > 0 && k > 0);
  WX_CHECK_ARG(ctx, (qw != nullptr) != (dw != nullptr));
  WX_CHECK_ARG(ctx, expand > 0 && expand <= kMaxTables && modalities > 0);
  WX_CHECK_ARG(ctx, !qw || (qweight_ok(qw) && qw->k == k));
  WX_CHECK_ARG(ctx, !dw || (dw->w && dw->k == k && dw->n > 0));
  WX_CHECK_ARG(ctx, !lora || (qw && lora_pack_ok(lora, qw)));
  const int64_t n = qw ? qw->n : dw->n;
  WX_CHECK_ARG(ctx, n % ((int64_t)expand * modalities) == 0);
  const int64_t hidden = n / ((int64_t)expand * modalities);
  WX_CHECK_ARG(ctx, hidden % 8 == 0);
  TablePtrs tabs{};
  for (int e = 0; e < expand; ++e) {
    WX_CHECK_ARG(ctx, tables[e] && aligned16(tables[e]));
    tabs.p[e] = static_cast<__nv_bfloat16*>(tables[e]);
  }
  // scratch: SiLU input, linear output, and the quantized linear's own scratch
  const size_t b_in = al((size_t)m * k * 2), b_y = al((size_t)m * n * 2);
  const size_t b_wd = qw ? al(qlinear_ws_need(m, n, k)) : 0;
  const size_t b_t = lora ? al((size_t)m * lora->R * 2) : 0;
  int st = WX_OK;
  void* ws = workspace(ctx, b_in + b_y + b_wd + b_t, &st);
  if (!ws) return st;
  uint8_t* base = static_cast<uint8_t*>(ws);
  const void* x = temb;
  if (apply_silu) {
    silu_bf16_kernel<<<grid_1d(m * k, 256, ctx->num_sms), 256, 0, ctx->stream>>>(
        static_cast<const __nv_bfloat16*>(temb), m * k, reinterpret_cast<__nv_bfloat16*>(base));
    if ((st = launch_status(ctx, "silu_bf16"))) return st;
    x = base;
  }
  void* y = base + b_in;
  if (qw)
    st = qlinear_lora_with_scratch(ctx, x, m, k, qw, lora, WX_EPI_NONE, nullptr, nullptr, nullptr, y, n, nullptr,
                                   base + b_in + b_y, base + b_in + b_y + b_wd, nullptr);
  else
    st = wx_linear_bf16(ctx, x, m, dw, y);
  if (st) return st;
  adaln_split_kernel<<<grid_1d(m * n / 8, 256, ctx->num_sms), 256, 0, ctx->stream>>>(
      static_cast<const __nv_bfloat16*>(y), m, expand, modalities, hidden, tabs);
  return launch_status(ctx, "adaln_split");
}

int64_t wx_refiner_scratch_bytes(const wx_dit_config* cfg, int64_t L) {
  if (!cfg || L <= 0) return 0;
  return (int64_t)refiner_layout(cfg, L).total;
}

int wx_refiner_block_forward(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w, void* h, int64_t L,
                             void* scratch) {
  WX_CHECK_ARG(ctx, ctx && cfg && h && scratch && L > 0);
  WX_CHECK_ARG(ctx, (cfg->head_dim == 128 || cfg->head_dim == 64) && cfg->heads > 0 && cfg->hidden > 0 &&
                        cfg->ffn > 0);
  int st = check_refiner_block(ctx, cfg, w);
  if (st) return st;
  const RefinerLayout R = refiner_layout(cfg, L);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  fill_bf16_kernel<<<1, 256, 0, ctx->stream>>>(reinterpret_cast<__nv_bfloat16*>(base + R.ones), cfg->hidden, 1.0f);
  if ((st = launch_status(ctx, "fill_bf16"))) return st;
  return refiner_block(ctx, cfg, w, h, L, base, R);
}

int wx_refine_text(wx_ctx* ctx, const wx_dit_config* cfg, const wx_qweight* condition_proj,
                   const wx_lora_pack* condition_lora, const wx_block_weights* blocks, int n_blocks,
                   const void* final_norm, const void* text, int64_t L, int64_t text_dim, void* out, void* scratch) {
  WX_CHECK_ARG(ctx, ctx && cfg && text && out && scratch && L > 0 && text_dim > 0 && n_blocks >= 0);
  WX_CHECK_ARG(ctx, n_blocks == 0 || blocks);
  const size_t row_bytes = (size_t)cfg->hidden * 2;
  if (text_dim == cfg->hidden) {
    // refineText returns the states unchanged when their width already matches (:996)
    WX_CUDA_TRY(ctx, cudaMemcpyAsync(out, text, (size_t)L * row_bytes, cudaMemcpyDeviceToDevice, ctx->stream));
    return WX_OK;
  }
  WX_CHECK_ARG(ctx, condition_proj || text_dim == cfg->hidden);
  WX_CHECK_ARG(ctx, qweight_ok(condition_proj) && condition_proj->k == text_dim &&
                        condition_proj->n == cfg->hidden);
  WX_CHECK_ARG(ctx, !condition_lora || lora_pack_ok(condition_lora, condition_proj));
  WX_CHECK_ARG(ctx, !condition_lora || condition_lora->R <= cfg->lora_rank);
  WX_CHECK_ARG(ctx, (cfg->head_dim == 128 || cfg->head_dim == 64) && cfg->heads > 0 && cfg->hidden > 0 &&
                        cfg->ffn > 0);
  int st;
  for (int b = 0; b < n_blocks; ++b)
    if ((st = check_refiner_block(ctx, cfg, &blocks[b]))) return st;
  const RefinerLayout R = refiner_layout(cfg, L, text_dim);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  // condition_proj: [L, text_dim] -> h [L, hidden] (bias inside the linear, added once)
  void* h = final_norm ? (void*)(base + R.h) : out;
  if ((st = qlinear_lora_with_scratch(ctx, text, L, text_dim, condition_proj, condition_lora, WX_EPI_NONE, nullptr,
                                      nullptr, nullptr, h, cfg->hidden, nullptr, base + R.wd, base + R.lt,
                                      nullptr)))
    return st;
  if (n_blocks > 0) {
    fill_bf16_kernel<<<1, 256, 0, ctx->stream>>>(reinterpret_cast<__nv_bfloat16*>(base + R.ones), cfg->hidden,
                                                 1.0f);
    if ((st = launch_status(ctx, "fill_bf16"))) return st;
  }
  for (int b = 0; b < n_blocks; ++b)
    if ((st = refiner_block(ctx, cfg, &blocks[b], h, L, base, R))) return st;
  if (final_norm)
    return launch_norm_modscale(ctx, h, L, cfg->hidden, final_norm, nullptr, nullptr, nullptr, cfg->eps, out);
  return WX_OK;
}

int64_t wx_refine_text_scratch_bytes(const wx_dit_config* cfg, int64_t L, int64_t text_dim) {
  if (!cfg || L <= 0 || text_dim <= 0) return 0;
  return (int64_t)refiner_layout(cfg, L, text_dim).total;
}

}  // extern "C"
