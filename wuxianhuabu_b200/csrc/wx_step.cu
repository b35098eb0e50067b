// wx_step.cu — one sampler step of the H3 pipeline as a single native call:
// patch embed (fp32 island) -> packed bf16 stream -> every DiT block with the
// layer's attention mode and the PAB decision -> final norm/modulation, fp32
// projection, negated velocity -> Euler update of the video latent
// (H3Pipeline.swift:1398-1445 around H3DiT.forward, H3Transformer.swift:1022-1203).
// Under sequence parallelism each rank runs its rows; the blocks exchange
// attention data through the context's communicator.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "wx_internal.h"

namespace wx {

int launch_norm_modscale(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w, const void* shift,
                         const void* scale, const uint32_t* rowmap, float eps, void* out);

struct StepLayout {
  size_t h, f32, h16, vel, blk, total;
};

static size_t al(size_t b) { return (b + 255) & ~size_t(255); }

static StepLayout step_layout(wx_ctx* ctx, const wx_dit_model* m, int64_t S) {
  StepLayout L{};
  const int P = ctx ? ctx->sp_size : 1;
  const int64_t rows = S / P;
  const size_t hid = (size_t)m->cfg->hidden;
  size_t off = 0;
  L.h = off; off += al((size_t)rows * hid * 2);
  L.f32 = off; off += al((size_t)rows * hid * 4);
  L.h16 = off; off += al((size_t)rows * hid * 2);
  L.vel = off; off += al((size_t)rows * m->patch_dim * 4);
  const int64_t blk = P == 1 ? wx_dit_block_scratch_bytes(m->cfg, S) : wx_dit_block_sp_scratch_bytes(m->cfg, S, P);
  L.blk = off; off += al((size_t)std::max<int64_t>(blk, 0));
  L.total = off;
  return L;
}

}  // namespace wx

using namespace wx;

extern "C" {

int64_t wx_dit_step_scratch_bytes(wx_ctx* ctx, const wx_dit_model* m, int64_t S) {
  if (!m || !m->cfg || S <= 0) return 0;
  const int P = ctx ? ctx->sp_size : 1;
  if (S % P) return 0;
  return (int64_t)step_layout(ctx, m, S).total;
}

int wx_dit_step(wx_ctx* ctx, const wx_dit_model* m, const wx_dit_step_args* a) {
  WX_CHECK_ARG(ctx, ctx && m && a && m->cfg && m->blocks && m->mods && m->n_blocks > 0);
  WX_CHECK_ARG(ctx, m->embed_w && m->embed_b && m->final_norm && m->out_w && m->out_b && m->patch_dim > 0);
  WX_CHECK_ARG(ctx, a->S > 0 && a->text_rows >= 0 && a->text_rows <= a->video_start && a->video_start < a->S);
  WX_CHECK_ARG(ctx, a->latents && a->rowmap && a->final_shift && a->final_scale && a->scratch);
  WX_CHECK_ARG(ctx, a->text_rows == 0 || a->text_states);
  WX_CHECK_ARG(ctx, a->refresh || a->pab_slots);
  const int P = ctx->sp_size;
  WX_CHECK_ARG(ctx, a->S % P == 0);
  const wx_dit_config* cfg = m->cfg;
  const int64_t hid = cfg->hidden, pd = m->patch_dim, text = a->text_rows, S = a->S;
  const int64_t rows = S / P, row0 = (int64_t)ctx->sp_rank * rows, row1 = row0 + rows;
  const StepLayout L = step_layout(ctx, m, S);
  uint8_t* base = static_cast<uint8_t*>(a->scratch);
  auto* h = reinterpret_cast<__nv_bfloat16*>(base + L.h);
  float* f32 = reinterpret_cast<float*>(base + L.f32);
  auto* h16 = reinterpret_cast<__nv_bfloat16*>(base + L.h16);
  float* vel = reinterpret_cast<float*>(base + L.vel);
  int st;
  // packed stream: text states, then the patch embed of the latent rows
  const int64_t t1 = std::min(row1, text);
  if (t1 > row0)
    WX_CUDA_TRY(ctx, cudaMemcpyAsync(h, static_cast<const __nv_bfloat16*>(a->text_states) + row0 * hid,
                                     (size_t)(t1 - row0) * hid * 2, cudaMemcpyDeviceToDevice, ctx->stream));
  const int64_t e0 = std::max(row0, text), ne = row1 - e0;
  if (ne > 0) {
    if ((st = wx_dense_f32(ctx, a->latents + (e0 - text) * pd, ne, pd, m->embed_w, hid, m->embed_b, f32))) return st;
    if ((st = wx_f32_to_bf16(ctx, f32, ne * hid, h + (e0 - row0) * hid))) return st;
  }
  // blocks
  wx_sparse_spec dense{};
  dense.mode = WX_SPARSE_DENSE;
  dense.block = 128;
  for (int bi = 0; bi < m->n_blocks; ++bi) {
    const int mode = a->spec ? wx_sparse_mode_for_layer(bi, m->n_blocks, a->policy) : 0;
    const wx_sparse_spec* spec = (mode != 0 && a->spec) ? a->spec : &dense;
    void* slot = a->pab_slots ? a->pab_slots[bi] : nullptr;
    const int refresh = a->refresh || !slot;
    st = P == 1 ? wx_dit_block_forward(ctx, cfg, &m->blocks[bi], &m->mods[bi], a->rowmap, h, rows, a->cos_t,
                                       a->sin_t, spec, slot, refresh, base + L.blk)
                : wx_dit_block_forward_sp(ctx, cfg, &m->blocks[bi], &m->mods[bi], a->rowmap, h, S, a->cos_t,
                                          a->sin_t, spec, slot, refresh, base + L.blk);
    if (st) return st;
  }
  // final head on the video rows + Euler update of their latents
  const int64_t v0 = std::max(row0, a->video_start), nv = row1 - v0;
  if (nv > 0) {
    if ((st = launch_norm_modscale(ctx, h + (v0 - row0) * hid, nv, hid, m->final_norm, a->final_shift,
                                   a->final_scale, nullptr, cfg->eps, h16)))
      return st;
    if ((st = wx_bf16_to_f32(ctx, h16, nv * hid, f32))) return st;
    if ((st = wx_dense_f32(ctx, f32, nv, hid, m->out_w, pd, m->out_b, vel))) return st;
    if ((st = wx_euler_update(ctx, a->latents + (v0 - text) * pd, vel, nv * pd, a->dsigma))) return st;
  }
  return WX_OK;
}

}  // extern "C"
