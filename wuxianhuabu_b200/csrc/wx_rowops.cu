// wx_rowops.cu — HBM-bound row kernels of the block: fused QK-RMSNorm+RoPE,
// RMSNorm + AdaLN scale/shift, gated residual, SwiGLU, and the affine
// 6-bit group quantizer / dequantizer.
//
// All of them are one warp per row (or per 8-element vector), 16-byte
// vector loads/stores where the geometry allows, fp32 arithmetic and one
// bf16 rounding at the points where the reference rounds.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ----------------------------------------------------------------- K3
// h3_fused_rmsnorm_rope (网络算子-融合-RMSNormRoPE-通用.swift:41-94): one warp per
// (s, h) row. nv = bf16(x*rstd*w); split-half rotation of pairs (j, j+rh)
// for j < rh; dims >= rot pass through. Rows are located by (s, part, h):
// x + s*x_stride + part*part_off + h*hd, output likewise with out_stride.
// The rotation's products are rounded separately (no contraction into FMAs) and
// the sum of squares uses explicit FMAs, so the q|k|v GEMM's fused epilogue
// (wx_gemm.cu) reproduces these bits.
template <int HD>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t x_stride, __nv_bfloat16* __restrict__ out,
    int64_t out_stride, int64_t part_off, int nparts, int64_t S, int H,
    const __nv_bfloat16* __restrict__ w0, const __nv_bfloat16* __restrict__ w1,
    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t, int rot,
    float eps) {
  constexpr int E = HD / 32;  // elements per lane (4 for hd 128, 2 for hd 64)
  __shared__ float nv_s[8][HD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  const int64_t nrows = S * nparts * H;
  if (row >= nrows) return;
  const int h = (int)(row % H);
  const int part = (int)((row / H) % nparts);
  const int64_t s = row / ((int64_t)H * nparts);
  const __nv_bfloat16* xr = x + s * x_stride + part * part_off + (int64_t)h * HD;
  __nv_bfloat16* orow = out + s * out_stride + part * part_off + (int64_t)h * HD;
  const __nv_bfloat16* w = part == 0 ? w0 : w1;

  float xv[E];
  if constexpr (E == 4) {
    uint2 raw = *reinterpret_cast<const uint2*>(xr + lane * 4);
    xv[0] = bf16_lo(raw.x); xv[1] = bf16_hi(raw.x); xv[2] = bf16_lo(raw.y); xv[3] = bf16_hi(raw.y);
  } else {
    uint32_t raw = *reinterpret_cast<const uint32_t*>(xr + lane * 2);
    xv[0] = bf16_lo(raw); xv[1] = bf16_hi(raw);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) ss = __fmaf_rn(xv[i], xv[i], ss);
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)HD + eps);
#pragma unroll
  for (int i = 0; i < E; ++i) {
    const int j = lane * E + i;
    nv_s[warp][j] = round_bf16(xv[i] * rstd * __bfloat162float(w[j]));
  }
  __syncwarp();
  const int rh = rot >> 1;
  float o[E];
#pragma unroll
  for (int i = 0; i < E; ++i) {
    const int j = lane * E + i;
    const float nv = nv_s[warp][j];
    if (j < rh) {
      const float c = __bfloat162float(cos_t[s * rh + j]);
      const float sn = __bfloat162float(sin_t[s * rh + j]);
      o[i] = __fsub_rn(__fmul_rn(nv, c), __fmul_rn(nv_s[warp][j + rh], sn));
    } else if (j < rot) {
      const float c = __bfloat162float(cos_t[s * rh + j - rh]);
      const float sn = __bfloat162float(sin_t[s * rh + j - rh]);
      o[i] = __fadd_rn(__fmul_rn(nv, c), __fmul_rn(nv_s[warp][j - rh], sn));
    } else {
      o[i] = nv;
    }
  }
  if constexpr (E == 4) {
    uint2 st;
    st.x = pack_bf16x2(o[0], o[1]);
    st.y = pack_bf16x2(o[2], o[3]);
    *reinterpret_cast<uint2*>(orow + lane * 4) = st;
  } else {
    *reinterpret_cast<uint32_t*>(orow + lane * 2) = pack_bf16x2(o[0], o[1]);
  }
}

// Same operation for head_dim 128 with rot/2 a multiple of 4, sized for HBM:
// one warp per (s, part, group of up to 8 heads). Every load of the group
// (8 rows x 256 B, plus the position's cos/sin) is issued before any use, so a
// warp keeps ~2.5 KB in flight instead of one 256-B row, and the rotation
// partner (j +- rot/2) comes from lane +- rot/8 by shuffle.
constexpr int kRopeHeads = 8;

// where row (s, part, head h) of the result goes
struct RopeLocalDst {  // the same packed layout, in place or into `out`
  __nv_bfloat16* out;
  int64_t out_stride, part_off;
  __device__ __forceinline__ __nv_bfloat16* operator()(int64_t s, int part, int h) const {
    return out + s * out_stride + part * part_off + (int64_t)h * 128;
  }
};
struct RopePeerDst {  // sequence parallelism: the exchange buffer of the rank owning head h,
                      // full-sequence row row0 + s, layout [S][3][Hl][128]
  __nv_bfloat16* base[kMaxPeers];
  int64_t row0;
  int Hl;
  __device__ __forceinline__ __nv_bfloat16* operator()(int64_t s, int part, int h) const {
    const int r = h / Hl;
    __nv_bfloat16* b = base[0];
#pragma unroll
    for (int i = 1; i < kMaxPeers; ++i)
      if (r == i) b = base[i];
    return b + ((row0 + s) * 3 + part) * (int64_t)Hl * 128 + (int64_t)(h - r * Hl) * 128;
  }
};

// PEER: nparts = 3 and the third part (v) is copied unchanged; every row goes to the
// owner of its head in another GPU's memory, and the last CTA signals the ranks.
template <class Dst, bool PEER>
__global__ void __launch_bounds__(256) qk_norm_rope_vec_kernel(
    const __nv_bfloat16* x, int64_t x_stride, Dst dst, int64_t part_off, int nparts, int64_t S, int H, int n_groups,
    const __nv_bfloat16* __restrict__ w0, const __nv_bfloat16* __restrict__ w1,
    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t, int rot, float eps,
    PeerSignal sig) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t task = (int64_t)blockIdx.x * 8 + warp;
  if (task < S * nparts * n_groups) {
    const int g = (int)(task % n_groups);
    const int part = (int)((task / n_groups) % nparts);
    const int64_t s = task / ((int64_t)n_groups * nparts);
    const int h0 = g * kRopeHeads;
    const int nh = min(kRopeHeads, H - h0);
    const int64_t xoff = s * x_stride + part * part_off + (int64_t)h0 * 128 + lane * 4;
    uint2 raw[kRopeHeads];
#pragma unroll
    for (int i = 0; i < kRopeHeads; ++i)
      if (i < nh) raw[i] = *reinterpret_cast<const uint2*>(x + xoff + i * 128);  // may alias the output (in place)
    if (PEER && part == 2) {
#pragma unroll
      for (int i = 0; i < kRopeHeads; ++i)
        if (i < nh) *reinterpret_cast<uint2*>(dst(s, 2, h0 + i) + lane * 4) = raw[i];
    } else {
      const int rh = rot >> 1;
      const int j0 = lane * 4;
      const bool rotated = j0 < rot;
      const bool first = j0 < rh;
      uint2 cr = make_uint2(0, 0), sr = make_uint2(0, 0);
      if (rotated) {
        const int64_t t = s * rh + (first ? j0 : j0 - rh);
        cr = __ldg(reinterpret_cast<const uint2*>(cos_t + t));
        sr = __ldg(reinterpret_cast<const uint2*>(sin_t + t));
      }
      const uint2 wr = __ldg(reinterpret_cast<const uint2*>((part == 0 ? w0 : w1) + j0));
      const float wv[4] = {bf16_lo(wr.x), bf16_hi(wr.x), bf16_lo(wr.y), bf16_hi(wr.y)};
      const float c[4] = {bf16_lo(cr.x), bf16_hi(cr.x), bf16_lo(cr.y), bf16_hi(cr.y)};
      const float sn[4] = {bf16_lo(sr.x), bf16_hi(sr.x), bf16_lo(sr.y), bf16_hi(sr.y)};
      const int partner = first ? lane + (rh >> 2) : lane - (rh >> 2);
      const int src = rotated ? partner : lane;
#pragma unroll
      for (int i = 0; i < kRopeHeads; ++i) {
        if (i >= nh) break;
        const float xv[4] = {bf16_lo(raw[i].x), bf16_hi(raw[i].x), bf16_lo(raw[i].y), bf16_hi(raw[i].y)};
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) ss = __fmaf_rn(xv[e], xv[e], ss);
        ss = warp_sum(ss);
        const float rstd = rsqrtf(ss / 128.f + eps);
        float nv[4], o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) nv[e] = round_bf16(xv[e] * rstd * wv[e]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float pv = __shfl_sync(0xffffffffu, nv[e], src);
          if (!rotated)
            o[e] = nv[e];
          else if (first)
            o[e] = __fsub_rn(__fmul_rn(nv[e], c[e]), __fmul_rn(pv, sn[e]));
          else
            o[e] = __fadd_rn(__fmul_rn(nv[e], c[e]), __fmul_rn(pv, sn[e]));
        }
        *reinterpret_cast<uint2*>(dst(s, part, h0 + i) + lane * 4) =
            make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
      }
    }
  }
  if constexpr (PEER) peer_signal_cta_done(sig);
}

// ----------------------------------------------------------------- K4
// h3_fused_norm_modscale (fused:133-168): one warp per row, two passes over
// the row (the second pass hits L1). MOD = false is rmsNormLast
// (H3Common.swift:502-508): bf16(x * rstd * w) with no modulation tables.
template <bool MOD>
__global__ void __launch_bounds__(256) norm_modscale_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t S, int hidden, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ shift, const __nv_bfloat16* __restrict__ scale,
    const uint32_t* __restrict__ rowmap, float eps, __nv_bfloat16* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= S) return;
  const __nv_bfloat16* xr = x + r * hidden;
  const int64_t mr = rowmap ? (int64_t)rowmap[r] : 0;
  const __nv_bfloat16* sh = MOD ? shift + mr * hidden : nullptr;
  const __nv_bfloat16* sc = MOD ? scale + mr * hidden : nullptr;
  __nv_bfloat16* orow = out + r * hidden;
  const bool vec = (hidden % 256) == 0;
  float ss = 0.f;
  if (vec) {
    for (int j = lane * 8; j < hidden; j += 256) {
      uint4 v = *reinterpret_cast<const uint4*>(xr + j);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float a = bf16_lo(u[q]), b = bf16_hi(u[q]);
        ss += a * a + b * b;
      }
    }
  } else {
    for (int j = lane; j < hidden; j += 32) {
      float a = __bfloat162float(xr[j]);
      ss += a * a;
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)hidden + eps);
  if (vec) {
    for (int j = lane * 8; j < hidden; j += 256) {
      uint4 xv = *reinterpret_cast<const uint4*>(xr + j);
      uint4 wv = *reinterpret_cast<const uint4*>(w + j);
      const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w}, wu[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t ou[4];
      if constexpr (MOD) {
        uint4 hv = *reinterpret_cast<const uint4*>(sh + j);
        uint4 cv = *reinterpret_cast<const uint4*>(sc + j);
        const uint32_t hu[4] = {hv.x, hv.y, hv.z, hv.w}, cu[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float n0 = round_bf16(bf16_lo(xu[q]) * rstd * bf16_lo(wu[q]));
          float n1 = round_bf16(bf16_hi(xu[q]) * rstd * bf16_hi(wu[q]));
          float o0 = n0 * (bf16_lo(cu[q]) + 1.0f) + bf16_lo(hu[q]);
          float o1 = n1 * (bf16_hi(cu[q]) + 1.0f) + bf16_hi(hu[q]);
          ou[q] = pack_bf16x2(o0, o1);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          ou[q] = pack_bf16x2(bf16_lo(xu[q]) * rstd * bf16_lo(wu[q]), bf16_hi(xu[q]) * rstd * bf16_hi(wu[q]));
      }
      *reinterpret_cast<uint4*>(orow + j) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
    }
  } else {
    for (int j = lane; j < hidden; j += 32) {
      float nv = round_bf16(__bfloat162float(xr[j]) * rstd * __bfloat162float(w[j]));
      if constexpr (MOD) nv = nv * (__bfloat162float(sc[j]) + 1.0f) + __bfloat162float(sh[j]);
      orow[j] = __float2bfloat16_rn(nv);
    }
  }
}

// ----------------------------------------------------------------- K5
// h3_fused_mod_gate (fused:179-196): out = bf16(x + other*gate[map[r]]),
// 8 elements per thread when hidden % 8 == 0.
__global__ void mod_gate_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ other,
                                const __nv_bfloat16* __restrict__ gate, const uint32_t* __restrict__ rowmap,
                                int64_t S, int hidden, __nv_bfloat16* __restrict__ out) {
  const bool vec = (hidden % 8) == 0;
  const int64_t per_row = vec ? hidden / 8 : hidden;
  const int64_t total = S * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row;
    const int64_t mr = rowmap ? (int64_t)rowmap[r] : 0;
    if (vec) {
      const int64_t c = (i % per_row) * 8;
      uint4 xv = *reinterpret_cast<const uint4*>(x + r * hidden + c);
      uint4 ov = *reinterpret_cast<const uint4*>(other + r * hidden + c);
      uint4 gv = *reinterpret_cast<const uint4*>(gate + mr * hidden + c);
      const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w}, ou[4] = {ov.x, ov.y, ov.z, ov.w};
      const uint32_t gu[4] = {gv.x, gv.y, gv.z, gv.w};
      uint32_t res[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        res[q] = pack_bf16x2(bf16_lo(xu[q]) + bf16_lo(ou[q]) * bf16_lo(gu[q]),
                             bf16_hi(xu[q]) + bf16_hi(ou[q]) * bf16_hi(gu[q]));
      *reinterpret_cast<uint4*>(out + r * hidden + c) = make_uint4(res[0], res[1], res[2], res[3]);
    } else {
      const int64_t c = i % per_row;
      out[r * hidden + c] = __float2bfloat16_rn(__bfloat162float(x[r * hidden + c]) +
                                                __bfloat162float(other[r * hidden + c]) *
                                                    __bfloat162float(gate[mr * hidden + c]));
    }
  }
}

// SwiGLU of a [m, 2F] fc1 output: y[:, j] = bf16(silu(t[:, j]) * t[:, F+j])
__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ t, int64_t m, int64_t F, int64_t ldt,
                              __nv_bfloat16* __restrict__ y, int64_t ldy) {
  const int64_t total = m * F;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, j = i % F;
    const float g = __bfloat162float(t[r * ldt + j]);
    const float u = __bfloat162float(t[r * ldt + F + j]);
    const float silu = g / (1.0f + expf(-g));
    y[r * ldy + j] = __float2bfloat16_rn(silu * u);
  }
}

// ---------------------------------------------------------- quantization
// One thread per group: min/max, scale = max((max-min)/nbins, 1e-7) and
// bias = min rounded to bf16, q = clamp(rint((w-bias)/scale)); the group's
// 2*bits words are written whole (group*bits is a multiple of 32).
__global__ void quantize_kernel(const float* __restrict__ w, int64_t n, int64_t k, int group, int bits,
                                uint32_t* __restrict__ wq, __nv_bfloat16* __restrict__ scales,
                                __nv_bfloat16* __restrict__ biases) {
  const int64_t groups = k / group;
  const int64_t total = n * groups;
  const int nbins = (1 << bits) - 1;
  const int64_t words_per_row = k * bits / 32;
  const int words_per_group = group * bits / 32;
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < total;
       gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = gi / groups, g = gi % groups;
    const float* src = w + r * k + g * group;
    float mn = src[0], mx = src[0];
    for (int j = 1; j < group; ++j) {
      mn = fminf(mn, src[j]);
      mx = fmaxf(mx, src[j]);
    }
    float sc = __fdiv_rn(__fsub_rn(mx, mn), (float)nbins);
    if (sc < 1e-7f) sc = 1e-7f;
    const __nv_bfloat16 sb = __float2bfloat16_rn(sc), bb = __float2bfloat16_rn(mn);
    scales[gi] = sb;
    biases[gi] = bb;
    const float s = __bfloat162float(sb), b = __bfloat162float(bb);
    uint32_t* dst = wq + r * words_per_row + g * words_per_group;
    uint32_t cur = 0;
    int filled = 0, wi = 0;
    for (int j = 0; j < group; ++j) {
      float qf = rintf(__fdiv_rn(__fsub_rn(src[j], b), s));
      int q = qf < 0.f ? 0 : (qf > (float)nbins ? nbins : (int)qf);
      cur |= (uint32_t)q << filled;
      if (filled + bits >= 32) {
        dst[wi++] = cur;
        const int used = 32 - filled;
        cur = used < bits ? ((uint32_t)q >> used) : 0u;
        filled = filled + bits - 32;
      } else {
        filled += bits;
      }
    }
  }
}

// w_out[n][k] = bf16(float(q)*scale + bias): 8 values (one 16-byte store) per thread.
__global__ void dequant_kernel(const uint32_t* __restrict__ wq, const __nv_bfloat16* __restrict__ scales,
                               const __nv_bfloat16* __restrict__ biases, int64_t n, int64_t k, int group,
                               int bits, __nv_bfloat16* __restrict__ out) {
  const int64_t per_row = k / 8;
  const int64_t total = n * per_row;
  const int64_t words_per_row = k * bits / 32;
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row;
    const int64_t c0 = (i % per_row) * 8;
    const uint32_t* row = wq + r * words_per_row;
    const int64_t gidx = r * (k / group) + c0 / group;
    const float s = __bfloat162float(scales[gidx]);
    const float b = __bfloat162float(biases[gidx]);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t bit = (c0 + e) * bits;
      const int64_t wi = bit >> 5;
      const int off = (int)(bit & 31);
      uint32_t q = __ldg(row + wi) >> off;
      if (off + bits > 32) q |= __ldg(row + wi + 1) << (32 - off);
      v[e] = __fmaf_rn((float)(q & mask), s, b);  // q*s is exact: one rounding, as fp32 mul+add
    }
    uint4 st = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                          pack_bf16x2(v[6], v[7]));
    *reinterpret_cast<uint4*>(out + r * k + c0) = st;
  }
}

// 6-bit value j (0..15) of a 16-value bundle of three packed words (value j at bit 6j of the
// 96-bit little-endian bundle, as dequant_kernel reads it)
__device__ __forceinline__ uint32_t q6_at(uint32_t w0, uint32_t w1, uint32_t w2, int j) {
  const int bit = 6 * j, wi = bit >> 5, off = bit & 31;
  const uint32_t lo = wi == 0 ? w0 : (wi == 1 ? w1 : w2);
  const uint32_t hi = wi == 0 ? w1 : w2;
  return (off + 6 > 32 ? __funnelshift_r(lo, hi, off) : (lo >> off)) & 63u;
}

// The 6-bit weight expansion (group a multiple of 16): one thread per 16-value bundle, i.e.
// three packed words (a warp reads 384 contiguous bytes) and two 16-byte stores, instead of
// dequant_kernel's per-value word loads. Same arithmetic (q*s exact, one rounding of q*s + b),
// so the output is bit-identical to dequant_kernel's. Bundle i of the matrix starts at word
// 3i and its values land at element 16i (rows are 3k/16 words and k elements).
__global__ void dequant6_kernel(const uint32_t* __restrict__ wq, const __nv_bfloat16* __restrict__ scales,
                                const __nv_bfloat16* __restrict__ biases, int64_t n, int64_t k, int group,
                                __nv_bfloat16* __restrict__ out) {
  const int64_t per_row = k / 16;
  const int64_t total = n * per_row;
  const int64_t groups = k / group;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = i % per_row;
    const uint32_t w0 = __ldg(wq + 3 * i), w1 = __ldg(wq + 3 * i + 1), w2 = __ldg(wq + 3 * i + 2);
    const int64_t gidx = r * groups + (c * 16) / group;
    const float s = __bfloat162float(scales[gidx]);
    const float b = __bfloat162float(biases[gidx]);
    uint32_t pk[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      pk[e] = pack_bf16x2(__fmaf_rn((float)q6_at(w0, w1, w2, 2 * e), s, b),
                          __fmaf_rn((float)q6_at(w0, w1, w2, 2 * e + 1), s, b));
    uint4* dst = reinterpret_cast<uint4*>(out + 16 * i);
    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  }
}

static unsigned grid_for(int64_t total, int threads, int num_sms) {
  int64_t b = (total + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms * 32;
  return (unsigned)std::max<int64_t>(1, std::min(b, cap));
}

int launch_swiglu(wx_ctx* ctx, const void* t, int64_t m, int64_t F, int64_t ldt, void* y, int64_t ldy) {
  swiglu_kernel<<<grid_for(m * F, 256, ctx->num_sms), 256, 0, ctx->stream>>>(
      static_cast<const __nv_bfloat16*>(t), m, F, ldt, static_cast<__nv_bfloat16*>(y), ldy);
  return launch_status(ctx, "swiglu");
}

int launch_dequant(wx_ctx* ctx, const wx_qweight* w, void* out) {
  ProfScope prof(ctx, kProfDequant);
  if (w->bits == 6 && w->group % 16 == 0 && aligned16(out)) {
    dequant6_kernel<<<grid_for(w->n * (w->k / 16), 256, ctx->num_sms), 256, 0, ctx->stream>>>(
        w->wq, static_cast<const __nv_bfloat16*>(w->scales), static_cast<const __nv_bfloat16*>(w->biases), w->n,
        w->k, w->group, static_cast<__nv_bfloat16*>(out));
    return launch_status(ctx, "dequant6");
  }
  dequant_kernel<<<grid_for(w->n * (w->k / 8), 256, ctx->num_sms), 256, 0, ctx->stream>>>(
      w->wq, static_cast<const __nv_bfloat16*>(w->scales), static_cast<const __nv_bfloat16*>(w->biases),
      w->n, w->k, w->group, w->bits, static_cast<__nv_bfloat16*>(out));
  return launch_status(ctx, "dequant");
}

bool qweight_ok(const wx_qweight* w) {
  if (!w || !w->wq || !w->scales || !w->biases) return false;
  if (w->bits < 2 || w->bits > 8 || w->group <= 0 || w->n <= 0 || w->k <= 0) return false;
  if (w->k % w->group || w->k % 8 || (w->k * w->bits) % 32 || (w->group * w->bits) % 32) return false;
  return true;
}

int launch_qk_norm_rope(wx_ctx* ctx, const void* x, int64_t x_stride, void* out, int64_t out_stride,
                        int64_t part_off, int nparts, int64_t S, int H, int hd, const void* w0,
                        const void* w1, const void* cos_t, const void* sin_t, int rot, float eps) {
  const int64_t rows = S * nparts * H;
  if (rows == 0) return WX_OK;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  ProfScope prof(ctx, kProfNormRope);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto O = static_cast<__nv_bfloat16*>(out);
  auto W0 = static_cast<const __nv_bfloat16*>(w0);
  auto W1 = static_cast<const __nv_bfloat16*>(w1);
  auto C = static_cast<const __nv_bfloat16*>(cos_t);
  auto Sn = static_cast<const __nv_bfloat16*>(sin_t);
  const int rh = rot >> 1;
  const bool vec_ok = hd == 128 && rh % 4 == 0 && x_stride % 4 == 0 && out_stride % 4 == 0 && part_off % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(x) & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0 &&
                      (reinterpret_cast<uintptr_t>(w0) & 7) == 0 && (nparts < 2 || (reinterpret_cast<uintptr_t>(w1) & 7) == 0) &&
                      (rot == 0 || ((reinterpret_cast<uintptr_t>(cos_t) & 7) == 0 && (reinterpret_cast<uintptr_t>(sin_t) & 7) == 0));
  if (vec_ok) {
    const int n_groups = (H + kRopeHeads - 1) / kRopeHeads;
    const int64_t tasks = S * nparts * n_groups;
    qk_norm_rope_vec_kernel<RopeLocalDst, false><<<(unsigned)((tasks + 7) / 8), 256, 0, ctx->stream>>>(
        X, x_stride, RopeLocalDst{O, out_stride, part_off}, part_off, nparts, S, H, n_groups, W0, W1, C, Sn, rot,
        eps, PeerSignal{});
    return launch_status(ctx, "qk_norm_rope");
  }
  if (hd == 128)
    qk_norm_rope_kernel<128><<<grid, 256, 0, ctx->stream>>>(X, x_stride, O, out_stride, part_off, nparts, S,
                                                             H, W0, W1, C, Sn, rot, eps);
  else
    qk_norm_rope_kernel<64><<<grid, 256, 0, ctx->stream>>>(X, x_stride, O, out_stride, part_off, nparts, S,
                                                            H, W0, W1, C, Sn, rot, eps);
  return launch_status(ctx, "qk_norm_rope");
}

bool qkv_to_peers_ok(int hd, int rot) { return hd == 128 && (rot >> 1) % 4 == 0; }

// Sequence parallelism: QK-RMSNorm + RoPE of this rank's rows of the packed qkv
// ([rows, 3*H*128]) and the copy of v, each head's row written into the exchange
// buffer of the rank that owns the head (peers[r], layout [S][3][Hl][128], rows
// row0 + s); the last CTA signals every rank through `sig` (sig.total is set here).
int launch_qkv_to_peers(wx_ctx* ctx, const void* qkv, int64_t rows, int64_t row0, int H, int Hl,
                        void* const* peers, int P, const void* w0, const void* w1, const void* cos_t,
                        const void* sin_t, int rot, float eps, PeerSignal sig) {
  if (!qkv_to_peers_ok(128, rot) || P < 1 || P > kMaxPeers || Hl * P != H)
    return set_error(ctx, WX_ERR_UNSUPPORTED, "qkv to peers: head_dim 128, rot/2 %% 4 == 0, H = P*Hl");
  RopePeerDst d{};
  for (int r = 0; r < kMaxPeers; ++r) d.base[r] = r < P ? static_cast<__nv_bfloat16*>(peers[r]) : nullptr;
  d.row0 = row0;
  d.Hl = Hl;
  const int64_t inner = (int64_t)H * 128;
  const int n_groups = (H + kRopeHeads - 1) / kRopeHeads;
  const int64_t tasks = rows * 3 * n_groups;
  const unsigned grid = (unsigned)std::max<int64_t>(1, (tasks + 7) / 8);
  sig.total = (int)grid;
  ProfScope prof(ctx, kProfExchange);
  qk_norm_rope_vec_kernel<RopePeerDst, true><<<grid, 256, 0, ctx->stream>>>(
      static_cast<const __nv_bfloat16*>(qkv), 3 * inner, d, inner, 3, rows, H, n_groups,
      static_cast<const __nv_bfloat16*>(w0), static_cast<const __nv_bfloat16*>(w1),
      static_cast<const __nv_bfloat16*>(cos_t), static_cast<const __nv_bfloat16*>(sin_t), rot, eps, sig);
  return launch_status(ctx, "qkv_to_peers");
}

int launch_norm_modscale(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w,
                         const void* shift, const void* scale, const uint32_t* rowmap, float eps, void* out) {
  if (S == 0) return WX_OK;
  ProfScope prof(ctx, kProfNormMod);
  auto kern = shift ? norm_modscale_kernel<true> : norm_modscale_kernel<false>;
  kern<<<(unsigned)((S + 7) / 8), 256, 0, ctx->stream>>>(
      static_cast<const __nv_bfloat16*>(x), S, (int)hidden, static_cast<const __nv_bfloat16*>(w),
      static_cast<const __nv_bfloat16*>(shift), static_cast<const __nv_bfloat16*>(scale), rowmap, eps,
      static_cast<__nv_bfloat16*>(out));
  return launch_status(ctx, "norm_modscale");
}

int launch_mod_gate(wx_ctx* ctx, const void* x, const void* other, const void* gate, const uint32_t* rowmap,
                    int64_t S, int64_t hidden, void* out) {
  if (S == 0) return WX_OK;
  const int64_t total = (hidden % 8 == 0) ? S * hidden / 8 : S * hidden;
  ProfScope prof(ctx, kProfRow);
  mod_gate_kernel<<<grid_for(total, 256, ctx->num_sms), 256, 0, ctx->stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(other),
      static_cast<const __nv_bfloat16*>(gate), rowmap, S, (int)hidden, static_cast<__nv_bfloat16*>(out));
  return launch_status(ctx, "mod_gate");
}

}  // namespace wx

using namespace wx;

extern "C" {

int wx_quantize_affine(wx_ctx* ctx, const float* w, int64_t n, int64_t k, int group, int bits, uint32_t* wq,
                       void* scales, void* biases) {
  WX_CHECK_ARG(ctx, ctx && w && wq && scales && biases && n > 0 && k > 0);
  WX_CHECK_ARG(ctx, bits >= 2 && bits <= 8 && group > 0 && k % group == 0 && (group * bits) % 32 == 0);
  quantize_kernel<<<grid_for(n * (k / group), 128, ctx->num_sms), 128, 0, ctx->stream>>>(
      w, n, k, group, bits, wq, static_cast<__nv_bfloat16*>(scales), static_cast<__nv_bfloat16*>(biases));
  return launch_status(ctx, "quantize");
}

int wx_dequantize_affine(wx_ctx* ctx, const wx_qweight* w, void* w_out) {
  WX_CHECK_ARG(ctx, ctx && qweight_ok(w) && w_out && aligned16(w_out));
  return launch_dequant(ctx, w, w_out);
}

int wx_qk_norm_rope(wx_ctx* ctx, const void* x, int64_t x_stride, int64_t S, int H, int head_dim, const void* w,
                    const void* cos_t, const void* sin_t, int rot, float eps, void* out, int64_t out_stride) {
  WX_CHECK_ARG(ctx, ctx && x && w && out && S >= 0 && H > 0);
  WX_CHECK_ARG(ctx, head_dim == 128 || head_dim == 64);
  WX_CHECK_ARG(ctx, rot >= 0 && rot <= head_dim && rot % 2 == 0 && (rot == 0 || (cos_t && sin_t)));
  WX_CHECK_ARG(ctx, x_stride >= (int64_t)H * head_dim && out_stride >= (int64_t)H * head_dim);
  WX_CHECK_ARG(ctx, x_stride % 4 == 0 && out_stride % 4 == 0 && aligned16(x) && aligned16(out));
  return launch_qk_norm_rope(ctx, x, x_stride, out, out_stride, 0, 1, S, H, head_dim, w, w, cos_t, sin_t, rot,
                             eps);
}

int wx_qk_norm_rope_qkv(wx_ctx* ctx, void* qkv, int64_t S, int H, int head_dim, const void* q_w,
                        const void* k_w, const void* cos_t, const void* sin_t, int rot, float eps) {
  WX_CHECK_ARG(ctx, ctx && qkv && q_w && k_w && S >= 0 && H > 0);
  WX_CHECK_ARG(ctx, head_dim == 128 || head_dim == 64);
  WX_CHECK_ARG(ctx, rot >= 0 && rot <= head_dim && rot % 2 == 0 && (rot == 0 || (cos_t && sin_t)));
  WX_CHECK_ARG(ctx, aligned16(qkv));
  const int64_t inner = (int64_t)H * head_dim;
  return launch_qk_norm_rope(ctx, qkv, 3 * inner, qkv, 3 * inner, inner, 2, S, H, head_dim, q_w, k_w, cos_t,
                             sin_t, rot, eps);
}

int wx_norm_modscale(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w, const void* shift,
                     const void* scale, const uint32_t* rowmap, float eps, void* out) {
  WX_CHECK_ARG(ctx, ctx && x && w && shift && scale && out && S >= 0 && hidden > 0 && hidden < (1 << 30));
  WX_CHECK_ARG(ctx, hidden % 256 != 0 || (aligned16(x) && aligned16(w) && aligned16(shift) &&
                                          aligned16(scale) && aligned16(out)));
  return launch_norm_modscale(ctx, x, S, hidden, w, shift, scale, rowmap, eps, out);
}

int wx_rms_norm(wx_ctx* ctx, const void* x, int64_t S, int64_t hidden, const void* w, float eps, void* out) {
  WX_CHECK_ARG(ctx, ctx && x && w && out && S >= 0 && hidden > 0 && hidden < (1 << 30));
  WX_CHECK_ARG(ctx, hidden % 256 != 0 || (aligned16(x) && aligned16(w) && aligned16(out)));
  return launch_norm_modscale(ctx, x, S, hidden, w, nullptr, nullptr, nullptr, eps, out);
}

int wx_mod_gate(wx_ctx* ctx, const void* x, const void* other, const void* gate, const uint32_t* rowmap,
                int64_t S, int64_t hidden, void* out) {
  WX_CHECK_ARG(ctx, ctx && x && other && gate && out && S >= 0 && hidden > 0 && hidden < (1 << 30));
  WX_CHECK_ARG(ctx, hidden % 8 != 0 || (aligned16(x) && aligned16(other) && aligned16(gate) && aligned16(out)));
  return launch_mod_gate(ctx, x, other, gate, rowmap, S, hidden, out);
}

}  // extern "C"
