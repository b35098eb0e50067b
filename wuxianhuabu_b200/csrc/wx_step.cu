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
#include <vector>

#include "wx_internal.h"

namespace wx {

int launch_norm_modscale(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w, const void* shift,
                         const void* scale, const uint32_t* rowmap, float eps, void* out);

// audio update of the pipeline: x += (aout * vscale) * dsigma (fp32, in that order)
__global__ void scaled_update_kernel(float* __restrict__ x, const float* __restrict__ v, int64_t n, float vscale,
                                     float dsigma) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = x[i] + (v[i] * vscale) * dsigma;
}

struct StepLayout {
  size_t h, f32, h16, vel, vel2, aout, blk, total;
};

// guidance combine of the two velocities (SelfLift CFG, fp32 in this order):
// vneg[i] = vneg[i] + (vpos[i] - vneg[i]) * scale
__global__ void cfg_combine_kernel(float* __restrict__ vneg, const float* __restrict__ vpos, int64_t n,
                                   float scale) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    vneg[i] = vneg[i] + (vpos[i] - vneg[i]) * scale;
}

// out[i] = -v[i]: the negated velocity the DiT forward returns as its video output
__global__ void negate_kernel(float* __restrict__ out, const float* __restrict__ v, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = -v[i];
}

// One run of packed rows [start, end) whose embeddings come from one latent array
// starting at row `lat` of it.
struct Piece {
  int64_t start, end, lat;
  bool audio;
};

// Splits [text, S) into runs of audio rows (the segments, in order) and video
// rows (everything else after the text), with each run's first latent row.
static std::vector<Piece> latent_pieces(int64_t text, int64_t S, const int64_t* segs, int nsegs) {
  std::vector<Piece> out;
  int64_t p = text, a_lat = 0, v_lat = 0;
  for (int i = 0; i < nsegs; ++i) {
    const int64_t s0 = segs[2 * i], s1 = segs[2 * i + 1];
    if (s0 > p) {
      out.push_back({p, s0, v_lat, false});
      v_lat += s0 - p;
    }
    out.push_back({s0, s1, a_lat, true});
    a_lat += s1 - s0;
    p = s1;
  }
  if (S > p) out.push_back({p, S, v_lat, false});
  return out;
}

static size_t al(size_t b) { return (b + 255) & ~size_t(255); }

static StepLayout step_layout(wx_ctx* ctx, const wx_dit_model* m, int64_t S, bool guided) {
  StepLayout L{};
  const int P = ctx ? ctx->sp_size : 1;
  const int64_t rows = S / P;
  const size_t hid = (size_t)m->cfg->hidden;
  size_t off = 0;
  L.h = off; off += al((size_t)rows * hid * 2);
  L.f32 = off; off += al((size_t)rows * hid * 4);
  L.h16 = off; off += al((size_t)rows * hid * 2);
  L.vel = off; off += al((size_t)rows * m->patch_dim * 4);
  L.vel2 = off; off += guided ? al((size_t)rows * m->patch_dim * 4) : 0;
  L.aout = off; off += al((size_t)rows * std::max(m->audio_dim, 0) * 4);
  const int64_t blk = P == 1 ? wx_dit_block_scratch_bytes(m->cfg, S) : wx_dit_block_sp_scratch_bytes(m->cfg, S, P);
  L.blk = off; off += al((size_t)std::max<int64_t>(blk, 0));
  L.total = off;
  return L;
}

static int check_step_args(wx_ctx* ctx, const wx_dit_model* m, const wx_dit_step_args* a) {
  WX_CHECK_ARG(ctx, ctx && m && a && m->cfg && m->blocks && m->mods && m->n_blocks > 0);
  WX_CHECK_ARG(ctx, m->embed_w && m->embed_b && m->final_norm && m->out_w && m->out_b && m->patch_dim > 0);
  WX_CHECK_ARG(ctx, a->S > 0 && a->text_rows >= 0 && a->text_rows <= a->video_start && a->video_start < a->S);
  WX_CHECK_ARG(ctx, a->latents && a->rowmap && a->final_shift && a->final_scale && a->scratch);
  WX_CHECK_ARG(ctx, a->text_rows == 0 || a->text_states);
  WX_CHECK_ARG(ctx, a->refresh || a->pab_slots);
  WX_CHECK_ARG(ctx, a->S % ctx->sp_size == 0);
  WX_CHECK_ARG(ctx, a->n_audio_segs >= 0 && (a->n_audio_segs == 0 || (a->audio_segs && a->audio_latents)));
  WX_CHECK_ARG(ctx, a->n_audio_segs == 0 || (m->audio_dim > 0 && m->audio_embed_w && m->audio_embed_b));
  WX_CHECK_ARG(ctx, a->audio_target >= -1 && a->audio_target < a->n_audio_segs);
  WX_CHECK_ARG(ctx, a->audio_target < 0 || (m->audio_out_w && m->audio_out_b && a->audio_final_shift &&
                                            a->audio_final_scale));
  for (int i = 0; i < a->n_audio_segs; ++i) {
    const int64_t s0 = a->audio_segs[2 * i], s1 = a->audio_segs[2 * i + 1];
    const int64_t prev = i ? a->audio_segs[2 * i - 1] : a->text_rows;
    WX_CHECK_ARG(ctx, s0 >= prev && s1 > s0 && s1 <= a->video_start);
  }
  return WX_OK;
}

// One forward of the DiT over this rank's rows (H3DiT.forward): the packed stream
// (text_states, then the patch embed of the latent rows), every block with its
// attention mode and PAB decision, then the final head. vel [local video rows,
// patch_dim] receives the velocity v of the video rows (the forward's video output
// is -v); aout [target audio rows, audio_dim] the audio head's output when a
// target audio segment is given.
static int dit_forward(wx_ctx* ctx, const wx_dit_model* m, const wx_dit_step_args* a, const void* text_states,
                       void* const* pab_slots, int refresh, const StepLayout& L, uint8_t* base, float* vel,
                       float* aout) {
  const wx_dit_config* cfg = m->cfg;
  const int P = ctx->sp_size;
  const int64_t hid = cfg->hidden, pd = m->patch_dim, text = a->text_rows, S = a->S;
  const int64_t rows = S / P, row0 = (int64_t)ctx->sp_rank * rows, row1 = row0 + rows;
  auto* h = reinterpret_cast<__nv_bfloat16*>(base + L.h);
  float* f32 = reinterpret_cast<float*>(base + L.f32);
  auto* h16 = reinterpret_cast<__nv_bfloat16*>(base + L.h16);
  int st;
  // packed stream: text states, then the patch embed of the latent rows
  const int64_t t1 = std::min(row1, text);
  if (t1 > row0)
    WX_CUDA_TRY(ctx, cudaMemcpyAsync(h, static_cast<const __nv_bfloat16*>(text_states) + row0 * hid,
                                     (size_t)(t1 - row0) * hid * 2, cudaMemcpyDeviceToDevice, ctx->stream));
  const std::vector<Piece> pieces = latent_pieces(text, S, a->audio_segs, a->n_audio_segs);
  for (const Piece& pc : pieces) {
    const int64_t e0 = std::max(row0, pc.start), e1 = std::min(row1, pc.end), ne = e1 - e0;
    if (ne <= 0) continue;
    const int64_t lat = pc.lat + (e0 - pc.start);
    if (pc.audio) {
      const int64_t ad = m->audio_dim;
      if ((st = wx_dense_f32(ctx, a->audio_latents + lat * ad, ne, ad, m->audio_embed_w, hid, m->audio_embed_b, f32)))
        return st;
    } else if ((st = wx_dense_f32(ctx, a->latents + lat * pd, ne, pd, m->embed_w, hid, m->embed_b, f32))) {
      return st;
    }
    if ((st = wx_f32_to_bf16(ctx, f32, ne * hid, h + (e0 - row0) * hid))) return st;
  }
  // blocks
  wx_sparse_spec dense{};
  dense.mode = WX_SPARSE_DENSE;
  dense.block = 128;
  for (int bi = 0; bi < m->n_blocks; ++bi) {
    const int mode = a->spec ? wx_sparse_mode_for_layer(bi, m->n_blocks, a->policy) : 0;
    const wx_sparse_spec* spec = (mode != 0 && a->spec) ? a->spec : &dense;
    void* slot = pab_slots ? pab_slots[bi] : nullptr;
    const int rf = refresh || !slot;
    st = P == 1 ? wx_dit_block_forward(ctx, cfg, &m->blocks[bi], &m->mods[bi], a->rowmap, h, rows, a->cos_t,
                                       a->sin_t, spec, slot, rf, base + L.blk)
                : wx_dit_block_forward_sp(ctx, cfg, &m->blocks[bi], &m->mods[bi], a->rowmap, h, S, a->cos_t,
                                          a->sin_t, spec, slot, rf, base + L.blk);
    if (st) return st;
  }
  // final head on the video rows
  const int64_t v0 = std::max(row0, a->video_start), nv = row1 - v0;
  if (nv > 0) {
    if ((st = launch_norm_modscale(ctx, h + (v0 - row0) * hid, nv, hid, m->final_norm, a->final_shift,
                                   a->final_scale, nullptr, cfg->eps, h16)))
      return st;
    if ((st = wx_bf16_to_f32(ctx, h16, nv * hid, f32))) return st;
    if ((st = wx_dense_f32(ctx, f32, nv, hid, m->out_w, pd, m->out_b, vel))) return st;
  }
  // final head on the target audio rows (finalHead with the audio t row); the negative
  // branch of a guided step passes aout = nullptr (audio takes the positive branch only)
  if (a->audio_target >= 0 && aout) {
    const int64_t s0 = a->audio_segs[2 * a->audio_target], s1 = a->audio_segs[2 * a->audio_target + 1];
    const int64_t b0 = std::max(row0, s0), b1 = std::min(row1, s1), nb = b1 - b0;
    if (nb > 0) {
      if ((st = launch_norm_modscale(ctx, h + (b0 - row0) * hid, nb, hid, m->final_norm, a->audio_final_shift,
                                     a->audio_final_scale, nullptr, cfg->eps, h16)))
        return st;
      if ((st = wx_bf16_to_f32(ctx, h16, nb * hid, f32))) return st;
      if ((st = wx_dense_f32(ctx, f32, nb, hid, m->audio_out_w, m->audio_dim, m->audio_out_b, aout))) return st;
    }
  }
  return WX_OK;
}

// The sampler's updates after the forward(s): Euler update of the video latents with the
// negated velocity (H3Pipeline.swift:1436-1443), and the audio update of the target segment.
static int step_updates(wx_ctx* ctx, const wx_dit_model* m, const wx_dit_step_args* a, const float* vel,
                        const float* aout, bool video_update) {
  const int P = ctx->sp_size;
  const int64_t pd = m->patch_dim, text = a->text_rows, S = a->S;
  const int64_t rows = S / P, row0 = (int64_t)ctx->sp_rank * rows, row1 = row0 + rows;
  const std::vector<Piece> pieces = latent_pieces(text, S, a->audio_segs, a->n_audio_segs);
  int st;
  // video rows are the last run, so their latent rows are the last ones
  const int64_t v0 = std::max(row0, a->video_start), nv = row1 - v0;
  if (video_update && nv > 0) {
    const int64_t vlat = pieces.back().lat + (v0 - pieces.back().start);
    if ((st = wx_euler_update(ctx, a->latents + vlat * pd, vel, nv * pd, a->dsigma))) return st;
  }
  if (a->audio_target >= 0) {
    const int64_t s0 = a->audio_segs[2 * a->audio_target], s1 = a->audio_segs[2 * a->audio_target + 1];
    const int64_t b0 = std::max(row0, s0), b1 = std::min(row1, s1), nb = b1 - b0;
    if (nb > 0) {
      int64_t lat = 0;
      for (const Piece& pc : pieces)
        if (pc.audio && pc.start == s0) lat = pc.lat + (b0 - s0);
      const int64_t ad = m->audio_dim, n = nb * ad;
      scaled_update_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 65536), 256, 0, ctx->stream>>>(
          a->audio_latents + lat * ad, aout, n, a->audio_vscale, a->audio_dsigma);
      if ((st = launch_status(ctx, "audio_update"))) return st;
    }
  }
  return WX_OK;
}

}  // namespace wx

using namespace wx;

extern "C" {

int64_t wx_dit_step_scratch_bytes(wx_ctx* ctx, const wx_dit_model* m, int64_t S) {
  if (!m || !m->cfg || S <= 0) return 0;
  const int P = ctx ? ctx->sp_size : 1;
  if (S % P) return 0;
  return (int64_t)step_layout(ctx, m, S, false).total;
}

int64_t wx_dit_step_guided_scratch_bytes(wx_ctx* ctx, const wx_dit_model* m, int64_t S) {
  if (!m || !m->cfg || S <= 0) return 0;
  const int P = ctx ? ctx->sp_size : 1;
  if (S % P) return 0;
  return (int64_t)step_layout(ctx, m, S, true).total;
}

int wx_dit_step(wx_ctx* ctx, const wx_dit_model* m, const wx_dit_step_args* a) {
  int st = check_step_args(ctx, m, a);
  if (st) return st;
  const StepLayout L = step_layout(ctx, m, a->S, false);
  uint8_t* base = static_cast<uint8_t*>(a->scratch);
  float* vel = reinterpret_cast<float*>(base + L.vel);
  float* aout = reinterpret_cast<float*>(base + L.aout);
  if ((st = dit_forward(ctx, m, a, a->text_states, a->pab_slots, a->refresh, L, base, vel, aout))) return st;
  return step_updates(ctx, m, a, vel, aout, true);
}

int wx_dit_step_guided(wx_ctx* ctx, const wx_dit_model* m, const wx_dit_step_args* a, const wx_dit_guidance* g) {
  int st = check_step_args(ctx, m, a);
  if (st) return st;
  WX_CHECK_ARG(ctx, g && (g->text_states_neg == nullptr || a->text_rows > 0));
  WX_CHECK_ARG(ctx, g->update == 0 || g->update == 1);
  WX_CHECK_ARG(ctx, g->update || g->velocity_out);
  const StepLayout L = step_layout(ctx, m, a->S, true);
  uint8_t* base = static_cast<uint8_t*>(a->scratch);
  float* vel = reinterpret_cast<float*>(base + L.vel);
  float* vel_pos = reinterpret_cast<float*>(base + L.vel2);
  float* aout = reinterpret_cast<float*>(base + L.aout);
  const int P = ctx->sp_size;
  const int64_t rows = a->S / P, row0 = (int64_t)ctx->sp_rank * rows;
  const int64_t nv = row0 + rows - std::max(row0, a->video_start);
  const int64_t n = std::max<int64_t>(nv, 0) * m->patch_dim;
  if (g->text_states_neg) {
    // positive condition with the PAB cache, then the negative condition with attention
    // computed fresh and no cache read or written (SelfLiftH3-(h3专属).swift:826-845)
    if ((st = dit_forward(ctx, m, a, a->text_states, a->pab_slots, a->refresh, L, base, vel_pos, aout))) return st;
    if ((st = dit_forward(ctx, m, a, g->text_states_neg, nullptr, 1, L, base, vel, nullptr))) return st;
    if (n > 0) {
      cfg_combine_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 65536), 256, 0, ctx->stream>>>(
          vel, vel_pos, n, g->cfg_scale);
      if ((st = launch_status(ctx, "cfg_combine"))) return st;
    }
  } else if ((st = dit_forward(ctx, m, a, a->text_states, a->pab_slots, a->refresh, L, base, vel, aout))) {
    return st;
  }
  if (g->velocity_out && n > 0) {
    negate_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 65536), 256, 0, ctx->stream>>>(g->velocity_out,
                                                                                                vel, n);
    if ((st = launch_status(ctx, "velocity_out"))) return st;
  }
  return step_updates(ctx, m, a, vel, aout, g->update != 0);
}

}  // extern "C"
