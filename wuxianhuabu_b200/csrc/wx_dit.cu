// wx_dit.cu — one DiT block of H3DiT.forward (H3Transformer.swift:1078-1159)
// composed from the kernels of this library, with the PAB cross-step cache
// (网络算子-注意力跨步缓存-通用.swift:36-112) as a caller-owned slot per block:
// on a refresh step the out-projection epilogue writes the attention branch
// output `at` straight into the slot while it also forms hAttn = h + at*gate;
// on a reuse step the slot is read back by the gated-residual kernel and the
// whole attention branch (norm1, qkv, norm+RoPE, attention, out-proj) is skipped.
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "wx_internal.h"

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

struct BlockLayout {
  size_t m, qkv, att, at, ha, f1, wd, sw, lt, attn, total;
};

static size_t al(size_t b) { return (b + 255) & ~size_t(255); }

static BlockLayout block_layout(const wx_dit_config* c, int64_t S) {
  BlockLayout L{};
  const size_t inner = (size_t)c->heads * c->head_dim;
  const size_t fc1_n = c->mlp_kind == WX_MLP_SWIGLU ? 2 * (size_t)c->ffn : (size_t)c->ffn;
  size_t off = 0;
  L.m = off; off += al((size_t)S * c->hidden * 2);
  L.qkv = off; off += al((size_t)S * 3 * inner * 2);
  L.att = off; off += al((size_t)S * inner * 2);
  L.at = off; off += al((size_t)S * c->hidden * 2);
  L.ha = off; off += al((size_t)S * c->hidden * 2);
  L.f1 = off; off += al((size_t)S * c->ffn * 2);
  size_t wmax = std::max(std::max(3 * inner * (size_t)c->hidden, inner * (size_t)c->hidden),
                         std::max(fc1_n * (size_t)c->hidden, (size_t)c->ffn * c->hidden));
  // expanded weight of the two-pass GEMM, or the fp32 split-K accumulator of the small-M path
  const size_t nmax = std::max(std::max(3 * inner, (size_t)c->hidden), fc1_n);
  L.wd = off; off += al(std::max(wmax * 2, qlinear_ws_need(S, (int64_t)nmax, 1)));
  L.sw = off; off += c->mlp_kind == WX_MLP_SWIGLU ? al((size_t)S * fc1_n * 2) : 0;
  L.lt = off; off += al((size_t)S * (size_t)std::max(0, c->lora_rank) * 2);  // x at^T of a LoRA pack
  // the widest attention plan this geometry can need (SOL 64-blocks with g = 0)
  wx_sparse_spec sol{};
  sol.mode = WX_SPARSE_SOL;
  sol.block = 64;
  sol.g = 0;
  wx_sparse_spec topk = sol;
  topk.mode = WX_SPARSE_TOPK;
  topk.block = 128;
  size_t a1 = attention_scratch_bytes(S, c->heads, c->head_dim, &sol);
  size_t a2 = attention_scratch_bytes(S, c->heads, c->head_dim, &topk);
  size_t a3 = attention_scratch_bytes(S, c->heads, c->head_dim, nullptr);
  L.attn = off; off += al(std::max(a1, std::max(a2, a3)));
  L.total = off;
  return L;
}

// every attached LoRA pack matches its linear and fits the scratch sized by cfg->lora_rank
bool lora_packs_ok(const wx_dit_config* cfg, const wx_block_weights* w) {
  const wx_qweight* q[4] = {&w->qkv, &w->out, &w->fc1, &w->fc2};
  for (int i = 0; i < 4; ++i)
    if (w->lora[i] && (!lora_pack_ok(w->lora[i], q[i]) || w->lora[i]->R > cfg->lora_rank)) return false;
  return true;
}

}  // namespace wx

using namespace wx;

extern "C" {

int64_t wx_dit_block_scratch_bytes(const wx_dit_config* cfg, int64_t S) {
  if (!cfg || S <= 0) return 0;
  return (int64_t)block_layout(cfg, S).total;
}

int wx_dit_block_forward(wx_ctx* ctx, const wx_dit_config* cfg, const wx_block_weights* w,
                         const wx_block_mods* mods, const uint32_t* rowmap, void* h, int64_t S, const void* cos_t,
                         const void* sin_t, const wx_sparse_spec* spec, void* pab_slot, int refresh, void* scratch) {
  WX_CHECK_ARG(ctx, ctx && cfg && w && mods && h && scratch && S > 0);
  WX_CHECK_ARG(ctx, (cfg->head_dim == 128 || cfg->head_dim == 64) && cfg->heads > 0 && cfg->hidden > 0 &&
                        cfg->ffn > 0);
  const int64_t inner = (int64_t)cfg->heads * cfg->head_dim;
  const int64_t fc1_n = cfg->mlp_kind == WX_MLP_SWIGLU ? 2 * cfg->ffn : cfg->ffn;
  WX_CHECK_ARG(ctx, qweight_ok(&w->qkv) && w->qkv.k == cfg->hidden && w->qkv.n == 3 * inner);
  WX_CHECK_ARG(ctx, qweight_ok(&w->out) && w->out.k == inner && w->out.n == cfg->hidden);
  WX_CHECK_ARG(ctx, qweight_ok(&w->fc1) && w->fc1.k == cfg->hidden && w->fc1.n == fc1_n);
  WX_CHECK_ARG(ctx, qweight_ok(&w->fc2) && w->fc2.k == cfg->ffn && w->fc2.n == cfg->hidden);
  WX_CHECK_ARG(ctx, w->q_norm && w->k_norm && w->norm1 && w->norm2);
  WX_CHECK_ARG(ctx, mods->shift_msa && mods->scale_msa && mods->gate_msa && mods->shift_mlp && mods->scale_mlp &&
                        mods->gate_mlp);
  WX_CHECK_ARG(ctx, cfg->rot >= 0 && cfg->rot <= cfg->head_dim && (cfg->rot == 0 || (cos_t && sin_t)));
  WX_CHECK_ARG(ctx, pab_slot || refresh);
  WX_CHECK_ARG(ctx, lora_packs_ok(cfg, w));
  const BlockLayout L = block_layout(cfg, S);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  void* m = base + L.m;
  void* qkv = base + L.qkv;
  void* att = base + L.att;
  void* ha = base + L.ha;
  void* f1 = base + L.f1;
  void* wd = base + L.wd;
  void* sw = base + L.sw;
  void* lt = base + L.lt;
  int st;
  const bool full = refresh || !pab_slot;
  LayerTrace tr(ctx, !full ? WX_TRACE_REUSE : (spec && spec->mode != WX_SPARSE_DENSE) ? WX_TRACE_SPARSE
                                                                                       : WX_TRACE_DENSE);
  if (full) {
    // m1 = norm1(h) * (scaleMSA + 1) + shiftMSA
    tr.begin(WX_TRACE_NORM1);
    if ((st = launch_norm_modscale(ctx, h, S, cfg->hidden, w->norm1, mods->shift_msa, mods->scale_msa, rowmap,
                                   cfg->eps, m)))
      return st;
    // qkv = qkv_proj(m1); per-head RMSNorm + RoPE of q and k (in the GEMM's epilogue
    // where the geometry allows, else as a separate kernel, in place)
    tr.begin(WX_TRACE_QKV);
    if (qkv_rope_fusable(&w->qkv, S, w->lora[0] != nullptr, false, cfg->head_dim, cfg->rot, w->q_norm, w->k_norm,
                         cos_t, sin_t)) {
      if ((st = qkv_rope_with_scratch(ctx, m, S, cfg->hidden, &w->qkv, w->lora[0], cfg->head_dim, qkv, 3 * inner,
                                      w->q_norm, w->k_norm, cos_t, sin_t, cfg->rot, cfg->eps, wd, lt, nullptr)))
        return st;
    } else {
      if ((st = qlinear_lora_with_scratch(ctx, m, S, cfg->hidden, &w->qkv, w->lora[0], WX_EPI_NONE, nullptr,
                                          nullptr, nullptr, qkv, 3 * inner, nullptr, wd, lt, nullptr)))
        return st;
      tr.begin(WX_TRACE_ROPE);
      if ((st = launch_qk_norm_rope(ctx, qkv, 3 * inner, qkv, 3 * inner, inner, 2, S, cfg->heads, cfg->head_dim,
                                    w->q_norm, w->k_norm, cos_t, sin_t, cfg->rot, cfg->eps)))
        return st;
    }
    // attention over the packed sequence
    const uint8_t* qb = static_cast<const uint8_t*>(qkv);
    const float scale = 1.0f / sqrtf((float)cfg->head_dim);
    tr.begin(WX_TRACE_ATTN);
    if ((st = attention_with_scratch(ctx, qb, qb + inner * 2, qb + 2 * inner * 2, 3 * inner, S, cfg->heads,
                                     cfg->head_dim, spec, scale, att, inner, base + L.attn)))
      return st;
    // at = out_proj(att) (-> PAB slot); hAttn = h + at * gateMSA
    void* at_dst = pab_slot ? pab_slot : base + L.at;
    tr.begin(WX_TRACE_OUT);
    if ((st = qlinear_lora_with_scratch(ctx, att, S, inner, &w->out, w->lora[1], WX_EPI_GATE_RESID, mods->gate_msa, h, rowmap, ha,
                                   cfg->hidden, at_dst, wd, lt, nullptr)))
      return st;
  } else {
    // PAB reuse: at = cache[bi]; hAttn = h + at * gateMSA (current step's gate)
    tr.begin(WX_TRACE_OUT);
    if ((st = launch_mod_gate(ctx, h, pab_slot, mods->gate_msa, rowmap, S, cfg->hidden, ha))) return st;
  }
  // m2 = norm2(hAttn) * (scaleMLP + 1) + shiftMLP
  tr.begin(WX_TRACE_MLP);
  if ((st = launch_norm_modscale(ctx, ha, S, cfg->hidden, w->norm2, mods->shift_mlp, mods->scale_mlp, rowmap,
                                 cfg->eps, m)))
    return st;
  // fc1 + activation
  const int act = cfg->mlp_kind == WX_MLP_SWIGLU ? WX_EPI_SWIGLU : WX_EPI_GELU;
  if ((st = qlinear_lora_with_scratch(ctx, m, S, cfg->hidden, &w->fc1, w->lora[2], act, nullptr, nullptr, nullptr, f1, cfg->ffn,
                                 nullptr, wd, lt, sw)))
    return st;
  // h = hAttn + fc2(f1) * gateMLP
  return qlinear_lora_with_scratch(ctx, f1, S, cfg->ffn, &w->fc2, w->lora[3], WX_EPI_GATE_RESID, mods->gate_mlp, ha, rowmap, h,
                              cfg->hidden, nullptr, wd, lt, nullptr);
}

}  // extern "C"
