// wx_gemm.cu — the quantized linear layer (MfLinear.forward, H3Common.swift:341-377)
// on sm_100a tensor cores.
//
// Y[M,N] = X[M,K] · deq(Wq)[N,K]^T with fused epilogues. The 6-bit weight is
// expanded to bf16 by the dequant kernel into context scratch, then this
// persistent warp-specialised kernel streams 128xBK A tiles and BNxBK B tiles
// with TMA (128-byte swizzle) through a 4-stage mbarrier ring, issues
// tcgen05.mma (kind::f16, M=128, N=BN, K=16) from one thread into a
// double-buffered TMEM accumulator, and 4 epilogue warps drain TMEM with
// tcgen05.ld, apply bias / GELU / gate+residual and store bf16.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer + TMEM
// owner, warps 2-5 epilogue (warp w reads TMEM lanes 32*(w%4)..+31).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

int launch_dequant(wx_ctx* ctx, const wx_qweight* w, void* out);
bool fused_eligible(const wx_qweight* w, int64_t M, int epilogue);
int qlinear_fused(wx_ctx* ctx, const void* x, int64_t M, int64_t lda, const wx_qweight* w, int epilogue,
                  const void* gate, const void* resid, const uint32_t* rowmap, void* y, int64_t ldy, void* y_raw,
                  void* scratch);
// WX_QGEMM_TWO_PASS=1 disables the fused small-M path (A/B measurements), read once
static bool force_two_pass() {
  static bool v = [] {
    const char* e = getenv("WX_QGEMM_TWO_PASS");
    return e && atoi(e) != 0;
  }();
  return v;
}
int launch_swiglu(wx_ctx* ctx, const void* t, int64_t m, int64_t F, int64_t ldt, void* y, int64_t ldy);
bool qweight_ok(const wx_qweight* w);

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;
constexpr int kGroupM = 16;

// q|k|v projection epilogue with QK-RMSNorm + RoPE fused (gemm_bf16_tc_kernel<BN, HD>):
// columns [0, inner) are q heads, [inner, 2 inner) k heads, [2 inner, 3 inner) v heads,
// head_dim 128. base[0] == nullptr: the result goes in place into y; otherwise head h of
// row m goes to the exchange buffer of rank h / Hl (layout [S][3][Hl][128], row row0 + m)
// and the last CTA raises sig (sequence parallelism over peer memory).
struct QkRopeEpi {
  const __nv_bfloat16* w0;  // q_norm [128]
  const __nv_bfloat16* w1;  // k_norm [128]
  const __nv_bfloat16* cos_t;
  const __nv_bfloat16* sin_t;  // [M, rot/2]
  int rot;
  float eps;
  int inner;
  int hd;  // head_dim: 128 or 64
  __nv_bfloat16* base[kMaxPeers];
  int64_t row0;
  int64_t rows_total;  // rows of each destination buffer (peer mode)
  int Hl;
  PeerSignal sig;
};

static bool qkv_rope_fused_enabled() {  // WX_QKV_ROPE_FUSED=0: separate kernels (A/B), read once
  static bool v = [] {
    const char* e = getenv("WX_QKV_ROPE_FUSED");
    return !(e && atoi(e) == 0);
  }();
  return v;
}

struct GemmParams {
  int M, N, K;
  int K2;  // extra K columns read through the second operand pair (LoRA: t [M,K2], bt [N,K2]); 0 = none
  int tiles_m, tiles_n, num_tiles;
  __nv_bfloat16* y;
  int64_t ldy;
  const __nv_bfloat16* bias;
  int epi;
  const __nv_bfloat16* gate;
  const __nv_bfloat16* resid;
  const uint32_t* rowmap;
  __nv_bfloat16* y_raw;
  int* err;
  QkRopeEpi qk;
};

// QKR adds a 32-row x 256-byte staging buffer per epilogue warp (the rows of one
// head, re-read in 512-byte coalesced pieces for the stores)
template <int BN, bool QKR = false>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOutOffset = kGemmStages * kStageBytes;
  static constexpr int kOutBytes = QKR ? 4 * 32 * 256 : 0;
  static constexpr int kBarOffset = kOutOffset + kOutBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;  // barriers + alignment slack
  static_assert(kBytes <= 227 * 1024, "GEMM shared memory exceeds the per-CTA limit");
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  const int per_group = kGroupM * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int gsize = min(tiles_m - first_m, kGroupM);
  const int in_group = tile % per_group;
  mb = first_m + in_group % gsize;
  nb = in_group / gsize;
}

__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

// Epilogue of 32 accumulator values of output row m, columns n0..n0+31: bf16(acc)
// (+ bias, rounded again), then GELU, or gate + residual (mr = the row's mod row), or
// nothing; bf16 stores (and the raw pre-gate values when y_raw is set).
__device__ __forceinline__ void gemm_epilogue32(const GemmParams& p, float (&v)[32], int64_t m, int64_t mr,
                                                int64_t n0) {
  if (!WX_IN_BOUNDS(p.err, m >= 0 && m < p.M && n0 >= 0 && n0 + 32 <= p.N)) return;
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = round_bf16(v[i]);
  if (p.bias) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      uint4 bv = *reinterpret_cast<const uint4*>(p.bias + n0 + i);
      const uint32_t bu[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[i + 2 * q] = round_bf16(v[i + 2 * q] + bf16_lo(bu[q]));
        v[i + 2 * q + 1] = round_bf16(v[i + 2 * q + 1] + bf16_hi(bu[q]));
      }
    }
  }
  __nv_bfloat16* yrow = p.y + m * p.ldy + n0;
  if (p.epi == WX_EPI_GATE_RESID) {
    const __nv_bfloat16* rrow = p.resid + m * p.ldy + n0;
    const __nv_bfloat16* grow = p.gate + mr * (int64_t)p.N + n0;
    if (p.y_raw) {
      __nv_bfloat16* raw = p.y_raw + m * p.ldy + n0;
#pragma unroll
      for (int i = 0; i < 32; i += 8)
        *reinterpret_cast<uint4*>(raw + i) =
            make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                       pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
    }
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      uint4 rv = *reinterpret_cast<const uint4*>(rrow + i);
      uint4 gv = *reinterpret_cast<const uint4*>(grow + i);
      const uint32_t ru[4] = {rv.x, rv.y, rv.z, rv.w}, gu[4] = {gv.x, gv.y, gv.z, gv.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o[q] = pack_bf16x2(bf16_lo(ru[q]) + v[i + 2 * q] * bf16_lo(gu[q]),
                           bf16_hi(ru[q]) + v[i + 2 * q + 1] * bf16_hi(gu[q]));
      *reinterpret_cast<uint4*>(yrow + i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    if (p.epi == WX_EPI_GELU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_f(v[i]);
    }
#pragma unroll
    for (int i = 0; i < 32; i += 8)
      *reinterpret_cast<uint4*>(yrow + i) =
          make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]),
                     pack_bf16x2(v[i + 4], v[i + 5]), pack_bf16x2(v[i + 6], v[i + 7]));
  }
}

// 16-byte chunk c of staging row r (HD / 8 chunks of a head row): XOR-swizzled so that
// the row-per-thread writes and the multi-row reads of the copy-out are both free of
// bank conflicts
template <int HD>
__device__ __forceinline__ uint4* stage_chunk(uint8_t* buf, int r, int c) {
  constexpr int NC = HD / 8;
  return reinterpret_cast<uint4*>(buf + r * (HD * 2) + ((c ^ (r & (NC - 1))) << 4));
}

// One HD-column head (HD = 128 or 64) of output row m for the q|k|v projection (one
// thread per row, v = the fp32 accumulators): the GEMM's bf16 result (+ bias, rounded
// again); for q and k heads then nv = bf16(x * rstd * w) and the split-half rotation of
// pairs (j, j + rot/2) of h3_fused_rmsnorm_rope (网络算子-融合-RMSNormRoPE-通用.swift:41-94);
// v heads pass through. The result goes as bf16 into the thread's staging row `lane`. The
// sum of squares is formed in the order of the warp-per-row kernels (qk_norm_rope_vec_kernel,
// qk_norm_rope_kernel<64>: partials over HD / 32 consecutive elements, combined as their
// xor butterfly combines lanes) and the rotation with the same explicit roundings, so the
// fused and the separate path give identical bits.
template <int HD>
__device__ __forceinline__ void qk_rope_head(const GemmParams& p, float (&v)[HD / 32][32], int64_t m, int64_t n0,
                                             int part, uint8_t* buf, int lane) {
  constexpr int NCH = HD / 32, E = HD / 32;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 32; ++i) v[c][i] = round_bf16(v[c][i]);
  if (p.bias) {
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        const uint4 bv = __ldg(reinterpret_cast<const uint4*>(p.bias + n0 + c * 32 + i));
        const uint32_t bu[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v[c][i + 2 * q] = round_bf16(v[c][i + 2 * q] + bf16_lo(bu[q]));
          v[c][i + 2 * q + 1] = round_bf16(v[c][i + 2 * q + 1] + bf16_hi(bu[q]));
        }
      }
  }
  if (part < 2) {
    float t[32];
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int c = (l * E) >> 5, i = (l * E) & 31;
      float a = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) a = __fmaf_rn(v[c][i + e], v[c][i + e], a);
      t[l] = a;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int l = 0; l < o; ++l) t[l] = __fadd_rn(t[l], t[l + o]);
    const float rstd = rsqrtf(t[0] / (float)HD + p.qk.eps);
    const __nv_bfloat16* w = part == 0 ? p.qk.w0 : p.qk.w1;
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + c * 32 + i));
        const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v[c][i + 2 * q] = round_bf16(v[c][i + 2 * q] * rstd * bf16_lo(wu[q]));
          v[c][i + 2 * q + 1] = round_bf16(v[c][i + 2 * q + 1] * rstd * bf16_hi(wu[q]));
        }
      }
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 32; i += 8)
      *stage_chunk<HD>(buf, lane, c * 4 + i / 8) =
          make_uint4(pack_bf16x2(v[c][i], v[c][i + 1]), pack_bf16x2(v[c][i + 2], v[c][i + 3]),
                     pack_bf16x2(v[c][i + 4], v[c][i + 5]), pack_bf16x2(v[c][i + 6], v[c][i + 7]));
  if (part < 2 && p.qk.rot > 0) {
    const int rc = p.qk.rot >> 4;  // chunks of 8 in rot/2
    const int64_t rh = p.qk.rot >> 1;
    const __nv_bfloat16* cr = p.qk.cos_t + m * rh;
    const __nv_bfloat16* sr = p.qk.sin_t + m * rh;
#pragma unroll 1
    for (int ch = 0; ch < rc; ++ch) {
      uint4* pa = stage_chunk<HD>(buf, lane, ch);
      uint4* pb = stage_chunk<HD>(buf, lane, ch + rc);
      const uint4 av = *pa, bv = *pb;
      const uint4 cv = __ldg(reinterpret_cast<const uint4*>(cr + ch * 8));
      const uint4 sv = __ldg(reinterpret_cast<const uint4*>(sr + ch * 8));
      const uint32_t au[4] = {av.x, av.y, av.z, av.w}, bu[4] = {bv.x, bv.y, bv.z, bv.w};
      const uint32_t cu[4] = {cv.x, cv.y, cv.z, cv.w}, su[4] = {sv.x, sv.y, sv.z, sv.w};
      uint32_t oa[4], ob[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a0 = bf16_lo(au[q]), a1 = bf16_hi(au[q]), b0 = bf16_lo(bu[q]), b1 = bf16_hi(bu[q]);
        const float c0 = bf16_lo(cu[q]), c1 = bf16_hi(cu[q]), s0 = bf16_lo(su[q]), s1 = bf16_hi(su[q]);
        oa[q] = pack_bf16x2(__fsub_rn(__fmul_rn(a0, c0), __fmul_rn(b0, s0)),
                            __fsub_rn(__fmul_rn(a1, c1), __fmul_rn(b1, s1)));
        ob[q] = pack_bf16x2(__fadd_rn(__fmul_rn(b0, c0), __fmul_rn(a0, s0)),
                            __fadd_rn(__fmul_rn(b1, c1), __fmul_rn(a1, s1)));
      }
      *pa = make_uint4(oa[0], oa[1], oa[2], oa[3]);
      *pb = make_uint4(ob[0], ob[1], ob[2], ob[3]);
    }
  }
}

// QKR: 0 = the plain epilogues; 128 / 64 = the q|k|v projection with QK-RMSNorm + RoPE
// of heads of that many columns
template <int BN, int QKR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                        GemmParams p) {
  using L = GemmSmem<BN, (QKR > 0)>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  // bars: full[4] empty[4] acc_full[2] acc_empty[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kGemmStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + kGemmStages + s); };
  auto accf_bar = [&](int a) { return smem_u32(bars + 2 * kGemmStages + a); };
  auto acce_bar = [&](int a) { return smem_u32(bars + 2 * kGemmStages + 2 + a); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf_bar(a), 1);
      mbar_init(acce_bar(a), 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (p.K2 > 0) {
      prefetch_tmap(&tmA2);
      prefetch_tmap(&tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // K blocks of the main operands, then of the extension pair (same stage layout)
  const int kblocks1 = p.K / kGemmBK;
  const int kblocks = kblocks1 + p.K2 / kGemmBK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p.tiles_m, p.tiles_n, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), L::kStageBytes);
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          if (kb < kblocks1) {
            tma_load_2d(sa, &tmA, full_bar(stage), kb * kGemmBK, mb * kGemmBM);
            tma_load_2d(sa + L::kABytes, &tmB, full_bar(stage), kb * kGemmBK, nb * BN);
          } else {
            tma_load_2d(sa, &tmA2, full_bar(stage), (kb - kblocks1) * kGemmBK, mb * kGemmBM);
            tma_load_2d(sa + L::kABytes, &tmB2, full_bar(stage), (kb - kblocks1) * kGemmBK, nb * BN);
          }
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kGemmBM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(acce_bar(acc), acc_phase ^ 1u, p.err, kDevTimeoutAcc, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, p.err, kDevTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(sb + kk * 32, 16, 1024);
            umma_bf16(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(accf_bar(acc));
      }
    }
  } else if constexpr (QKR > 0) {
    // epilogue of the q|k|v projection: QK-RMSNorm + RoPE per head, rows staged in
    // shared memory and stored in 512-byte pieces (in place, or into the owners' buffers)
    constexpr int HD = QKR, RPI = 512 / (HD * 2), NC = HD / 8;  // rows per store instruction
    const int quarter = warp & 3;
    uint8_t* buf = smem + L::kOutOffset + quarter * 32 * 256;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(accf_bar(acc), acc_phase, p.err, kDevTimeoutAcc, abort_flag)) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(tile, p.tiles_m, p.tiles_n, mb, nb);
      const int64_t row_base = (int64_t)mb * kGemmBM + quarter * 32;
      const int64_t m = row_base + lane;
#pragma unroll 1
      for (int hh = 0; hh < BN / HD; ++hh) {
        float v[HD / 32][32];
#pragma unroll
        for (int c = 0; c < HD / 32; ++c)
          tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + hh * HD + c * 32, v[c]);
        tmem_wait_ld();
        const int64_t n0 = (int64_t)nb * BN + hh * HD;
        const int part = (int)(n0 / p.qk.inner);
        const int head = (int)((n0 - (int64_t)part * p.qk.inner) / HD);
        if (m < p.M) qk_rope_head<HD>(p, v, m, n0, part, buf, lane);
        __syncwarp();
        __nv_bfloat16* dst;
        int64_t dst_stride;
        bool dst_ok = true;  // (bounds-checked build) the destination rows and owner exist
        if (p.qk.base[0] == nullptr) {
          dst = p.y + row_base * p.ldy + n0;
          dst_stride = p.ldy;
          dst_ok = WX_IN_BOUNDS(p.err, n0 + HD <= p.N);
        } else {
          const int owner = head / p.qk.Hl;
          dst_ok = WX_IN_BOUNDS(p.err, owner < kMaxPeers && p.qk.base[owner < kMaxPeers ? owner : 0] != nullptr);
          __nv_bfloat16* b = p.qk.base[0];
#pragma unroll
          for (int r = 1; r < kMaxPeers; ++r)
            if (owner == r) b = p.qk.base[r];
          dst_stride = 3 * (int64_t)p.qk.Hl * HD;
          dst = b + (p.qk.row0 + row_base) * dst_stride + (int64_t)part * p.qk.Hl * HD +
                (int64_t)(head - owner * p.qk.Hl) * HD;
        }
#pragma unroll 4
        for (int i = 0; i < 32 / RPI; ++i) {
          const int r = RPI * i + lane / NC, ch = lane % NC;
          const uint4 val = *stage_chunk<HD>(buf, r, ch);
          if (row_base + r < p.M && dst_ok &&
              WX_IN_BOUNDS(p.err, p.qk.base[0] == nullptr || p.qk.row0 + row_base + r < p.qk.rows_total))
            *reinterpret_cast<uint4*>(dst + r * dst_stride + ch * 8) = val;
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive(acce_bar(acc));
    }
  } else {
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(accf_bar(acc), acc_phase, p.err, kDevTimeoutAcc, abort_flag)) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(tile, p.tiles_m, p.tiles_n, mb, nb);
      const int64_t m = (int64_t)mb * kGemmBM + row_in_tile;
      const bool row_ok = m < p.M;
      const int64_t mr = (p.epi == WX_EPI_GATE_RESID && row_ok && p.rowmap) ? (int64_t)p.rowmap[m] : 0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + c * 32, v);
        tmem_wait_ld();
        if (!row_ok) continue;
        const int64_t n0 = (int64_t)nb * BN + c * 32;
        gemm_epilogue32(p, v, m, mr, n0);
      }
      tc_fence_before();
      mbar_arrive(acce_bar(acc));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
  if constexpr (QKR > 0) {
    if (p.qk.sig.counter) peer_signal_cta_done(p.qk.sig);  // after every store of this CTA
  }
}

template <int BN, int QKR = 0>
static int launch_gemm_bn(wx_ctx* ctx, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2,
                          const CUtensorMap& tb2, GemmParams& p) {
  using L = GemmSmem<BN, (QKR > 0)>;
  int st = ensure_smem_attr(ctx, (const void*)gemm_bf16_tc_kernel<BN, QKR>, L::kBytes,
                            QKR ? "gemm_bf16_tc (qk-norm/rope epilogue)" : "gemm_bf16_tc");
  if (st) return st;
  p.tiles_m = (p.M + kGemmBM - 1) / kGemmBM;
  p.tiles_n = p.N / BN;
  p.num_tiles = p.tiles_m * p.tiles_n;
  const int grid = std::min(p.num_tiles, ctx->num_sms);
  if (QKR > 0) p.qk.sig.total = grid;  // every CTA of the launch counts once
  ProfScope prof(ctx, kProfGemm);
  gemm_bf16_tc_kernel<BN, QKR><<<grid, kGemmThreads, L::kBytes, ctx->stream>>>(ta, tb, ta2, tb2, p);
  return launch_status(ctx, "gemm_bf16_tc");
}

// bf16 GEMM core: Y = X · Wd^T (+ T · Bt^T when k2 > 0) with X [M,K] (pitch lda),
// Wd [N,K] (pitch K), T [M,k2] (pitch k2), Bt [N,k2] (pitch k2)
int gemm_bf16_ext(wx_ctx* ctx, const void* x, int64_t M, int64_t lda, const void* wd, int64_t N, int64_t K,
                  const void* t, const void* bt, int64_t k2, const void* bias, int epi, const void* gate,
                  const void* resid, const uint32_t* rowmap, void* y, int64_t ldy, void* y_raw,
                  const QkRopeEpi* qk = nullptr) {
  if (M == 0) return WX_OK;  // (the q|k|v epilogue is only used with M > 0)
  if (K % kGemmBK != 0 || k2 % kGemmBK != 0 || N % 64 != 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX ||
      k2 > INT32_MAX)
    return set_error(ctx, WX_ERR_UNSUPPORTED, "gemm needs K %% 64 == 0 and N %% 64 == 0 (M=%lld N=%lld K=%lld)",
                     (long long)M, (long long)N, (long long)K);
  if (!aligned16(y) || ldy % 8 != 0 || (bias && !aligned16(bias)) ||
      (epi == WX_EPI_GATE_RESID && (!aligned16(gate) || !aligned16(resid) || (y_raw && !aligned16(y_raw)))))
    return set_error(ctx, WX_ERR_INVALID, "gemm outputs/epilogue operands need 16-byte alignment");
  const int BN = (N % 256 == 0) ? 256 : (N % 128 == 0 ? 128 : 64);
  CUtensorMap ta, tb, ta2, tb2;
  int st = make_tmap_bf16_2d(ctx, &ta, x, (uint64_t)M, (uint64_t)K, (uint64_t)lda, kGemmBK, kGemmBM);
  if (st) return st;
  st = make_tmap_bf16_2d(ctx, &tb, wd, (uint64_t)N, (uint64_t)K, (uint64_t)K, kGemmBK, BN);
  if (st) return st;
  if (k2 > 0) {
    if ((st = make_tmap_bf16_2d(ctx, &ta2, t, (uint64_t)M, (uint64_t)k2, (uint64_t)k2, kGemmBK, kGemmBM))) return st;
    if ((st = make_tmap_bf16_2d(ctx, &tb2, bt, (uint64_t)N, (uint64_t)k2, (uint64_t)k2, kGemmBK, BN))) return st;
  } else {
    ta2 = ta;
    tb2 = tb;
  }
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.K2 = (int)k2;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.epi = epi;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.resid = static_cast<const __nv_bfloat16*>(resid);
  p.rowmap = rowmap;
  p.y_raw = static_cast<__nv_bfloat16*>(y_raw);
  p.err = ctx->dev_err;
  if (qk) {
    if (epi != WX_EPI_NONE || BN < 128 || (qk->hd != 128 && qk->hd != 64) || qk->inner % qk->hd != 0 ||
        N != 3 * (int64_t)qk->inner)
      return set_error(ctx, WX_ERR_UNSUPPORTED, "qk-norm/rope epilogue: q|k|v of 128- or 64-wide heads, N %% 128 == 0");
    p.qk = *qk;
    if (qk->hd == 64)
      return BN == 256 ? launch_gemm_bn<256, 64>(ctx, ta, tb, ta2, tb2, p) : launch_gemm_bn<128, 64>(ctx, ta, tb, ta2, tb2, p);
    return BN == 256 ? launch_gemm_bn<256, 128>(ctx, ta, tb, ta2, tb2, p) : launch_gemm_bn<128, 128>(ctx, ta, tb, ta2, tb2, p);
  }
  if (BN == 256) return launch_gemm_bn<256>(ctx, ta, tb, ta2, tb2, p);
  if (BN == 128) return launch_gemm_bn<128>(ctx, ta, tb, ta2, tb2, p);
  return launch_gemm_bn<64>(ctx, ta, tb, ta2, tb2, p);
}

int gemm_bf16(wx_ctx* ctx, const void* x, int64_t M, int64_t lda, const void* wd, int64_t N, int64_t K,
              const void* bias, int epi, const void* gate, const void* resid, const uint32_t* rowmap, void* y,
              int64_t ldy, void* y_raw) {
  return gemm_bf16_ext(ctx, x, M, lda, wd, N, K, nullptr, nullptr, 0, bias, epi, gate, resid, rowmap, y, ldy,
                       y_raw);
}

bool lora_pack_ok(const wx_lora_pack* l, const wx_qweight* w) {
  return l && l->at && l->bt && l->R > 0 && l->R % 64 == 0 && l->n == w->n && l->k == w->k && aligned16(l->at) &&
         aligned16(l->bt);
}

// Full quantized linear: dequant into scratch `wd` (N*K bf16), then GEMM; with a
// LoRA pack, t = x at^T first and the GEMM runs R extra K columns over (t, bt).
int qlinear_lora_with_scratch(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                              const wx_lora_pack* lora, int epilogue, const void* gate, const void* resid,
                              const uint32_t* rowmap, void* y, int64_t ldy, void* y_raw, void* wd, void* t,
                              void* swiglu_tmp) {
  // small M is weight-bandwidth bound: expand the weights in shared memory instead
  if (!lora && fused_eligible(w, m, epilogue) && !force_two_pass())
    return qlinear_fused(ctx, x, m, lda, w, epilogue, gate, resid, rowmap, y, ldy, y_raw, wd);
  int st = launch_dequant(ctx, w, wd);
  if (st) return st;
  const int64_t R = lora ? lora->R : 0;
  if (R > 0) {
    // t = x (scale A)^T-packed: [m, R], the A operand of the extension columns
    if ((st = gemm_bf16(ctx, x, m, lda, lora->at, R, w->k, nullptr, WX_EPI_NONE, nullptr, nullptr, nullptr, t, R,
                        nullptr)))
      return st;
  }
  const void* bt = R > 0 ? lora->bt : nullptr;
  if (epilogue == WX_EPI_SWIGLU) {
    st = gemm_bf16_ext(ctx, x, m, lda, wd, w->n, w->k, t, bt, R, w->bias, WX_EPI_NONE, nullptr, nullptr, nullptr,
                       swiglu_tmp, w->n, nullptr);
    if (st) return st;
    return launch_swiglu(ctx, swiglu_tmp, m, w->n / 2, w->n, y, ldy);
  }
  return gemm_bf16_ext(ctx, x, m, lda, wd, w->n, w->k, t, bt, R, w->bias, epilogue, gate, resid, rowmap, y, ldy,
                       y_raw);
}

// The fused epilogue runs on the two-pass GEMM; where the small-M kernel would serve the
// projection (M <= 512, no LoRA) the separate path is kept, except for the peer-memory
// exchange (peer = true), which the fused epilogue replaces whatever M is.
// geometry the epilogue takes: heads of 128 or 64 columns, rot/2 a multiple of 8, N % 128 == 0
static bool qkv_rope_geometry_ok(const wx_qweight* w, int head_dim, int rot, const void* q_norm, const void* k_norm,
                                 const void* cos_t, const void* sin_t) {
  return (head_dim == 128 || head_dim == 64) && rot >= 0 && rot <= head_dim && rot % 16 == 0 && aligned16(q_norm) &&
         aligned16(k_norm) && (rot == 0 || (aligned16(cos_t) && aligned16(sin_t))) &&
         w->n % (3 * head_dim) == 0 && w->n % 128 == 0;
}

bool qkv_rope_fusable(const wx_qweight* w, int64_t m, bool has_lora, bool peer, int head_dim, int rot,
                      const void* q_norm, const void* k_norm, const void* cos_t, const void* sin_t) {
  if (!qkv_rope_fused_enabled() || (peer && head_dim != 128) ||
      !qkv_rope_geometry_ok(w, head_dim, rot, q_norm, k_norm, cos_t, sin_t))
    return false;
  const bool small_m = !has_lora && fused_eligible(w, m, WX_EPI_NONE) && !force_two_pass();
  return peer || !small_m;
}

// The q|k|v projection with QK-RMSNorm + RoPE in the GEMM's epilogue: dequant into `wd`,
// (LoRA: t = x at^T), then one GEMM whose epilogue normalises and rotates q and k per
// head. peers == nullptr: the result goes in place into y (pitch ldy); otherwise into
// the owners' exchange buffers, and the launch's last CTA raises peers->sig.
int qkv_rope_with_scratch(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                          const wx_lora_pack* lora, int head_dim, void* y, int64_t ldy, const void* q_norm,
                          const void* k_norm, const void* cos_t, const void* sin_t, int rot, float eps, void* wd,
                          void* t, const QkvPeerOut* peers) {
  if (m <= 0 || !qkv_rope_geometry_ok(w, head_dim, rot, q_norm, k_norm, cos_t, sin_t) || (peers && head_dim != 128))
    return set_error(ctx, WX_ERR_UNSUPPORTED,
                     "qkv rope epilogue: n = 3 * heads * head_dim (128 or 64, 128 with peers), rot %% 16 == 0");
  int st = launch_dequant(ctx, w, wd);
  if (st) return st;
  const int64_t R = lora ? lora->R : 0;
  if (R > 0 && (st = gemm_bf16(ctx, x, m, lda, lora->at, R, w->k, nullptr, WX_EPI_NONE, nullptr, nullptr, nullptr,
                               t, R, nullptr)))
    return st;
  QkRopeEpi e{};
  e.w0 = static_cast<const __nv_bfloat16*>(q_norm);
  e.w1 = static_cast<const __nv_bfloat16*>(k_norm);
  e.cos_t = static_cast<const __nv_bfloat16*>(cos_t);
  e.sin_t = static_cast<const __nv_bfloat16*>(sin_t);
  e.rot = rot;
  e.eps = eps;
  e.inner = (int)(w->n / 3);
  e.hd = head_dim;
  if (peers) {
    for (int r = 0; r < kMaxPeers; ++r) e.base[r] = static_cast<__nv_bfloat16*>(peers->base[r]);
    e.row0 = peers->row0;
    e.rows_total = peers->rows_total;
    e.Hl = peers->Hl;
    e.sig = peers->sig;
  }
  return gemm_bf16_ext(ctx, x, m, lda, wd, w->n, w->k, t, R > 0 ? lora->bt : nullptr, R, w->bias, WX_EPI_NONE,
                       nullptr, nullptr, nullptr, y, ldy, nullptr, &e);
}

int qlinear_with_scratch(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w, int epilogue,
                         const void* gate, const void* resid, const uint32_t* rowmap, void* y, int64_t ldy,
                         void* y_raw, void* wd, void* swiglu_tmp) {
  return qlinear_lora_with_scratch(ctx, x, m, lda, w, nullptr, epilogue, gate, resid, rowmap, y, ldy, y_raw, wd,
                                   nullptr, swiglu_tmp);
}

size_t qlinear_scratch_bytes(const wx_qweight* w, int64_t m, int epilogue) {
  size_t b = qlinear_ws_need(m, w->n, w->k);
  b = (b + 255) & ~size_t(255);
  if (epilogue == WX_EPI_SWIGLU) b += ((size_t)m * w->n * 2 + 255) & ~size_t(255);
  return b;
}

}  // namespace wx

using namespace wx;

extern "C" int wx_qlinear_lora(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                               const wx_lora_pack* lora, int epilogue, const void* gate, const void* resid,
                               const uint32_t* rowmap, void* y, int64_t ldy, void* y_raw) {
  if (!lora) return wx_qlinear(ctx, x, m, lda, w, epilogue, gate, resid, rowmap, y, ldy, y_raw);
  WX_CHECK_ARG(ctx, ctx && x && y && qweight_ok(w) && m >= 0 && lda >= w->k);
  WX_CHECK_ARG(ctx, lora_pack_ok(lora, w));
  WX_CHECK_ARG(ctx, epilogue >= WX_EPI_NONE && epilogue <= WX_EPI_SWIGLU);
  WX_CHECK_ARG(ctx, epilogue != WX_EPI_GATE_RESID || (gate && resid));
  WX_CHECK_ARG(ctx, epilogue != WX_EPI_SWIGLU || w->n % 2 == 0);
  WX_CHECK_ARG(ctx, ldy >= (epilogue == WX_EPI_SWIGLU ? w->n / 2 : w->n));
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t b_wd = al((size_t)w->n * w->k * 2), b_t = al((size_t)m * lora->R * 2);
  const size_t b_sw = epilogue == WX_EPI_SWIGLU ? al((size_t)m * w->n * 2) : 0;
  int st = WX_OK;
  void* ws = workspace(ctx, b_wd + b_t + b_sw, &st);
  if (!ws) return st;
  uint8_t* base = static_cast<uint8_t*>(ws);
  return qlinear_lora_with_scratch(ctx, x, m, lda, w, lora, epilogue, gate, resid, rowmap, y, ldy, y_raw, base,
                                   base + b_wd, base + b_wd + b_t);
}

namespace wx {
int launch_qk_norm_rope(wx_ctx* ctx, const void* x, int64_t x_stride, void* out, int64_t out_stride,
                        int64_t part_off, int nparts, int64_t S, int H, int hd, const void* w0, const void* w1,
                        const void* cos_t, const void* sin_t, int rot, float eps);
}

extern "C" int wx_qkv_norm_rope(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w,
                                const wx_lora_pack* lora, int H, int head_dim, const void* q_w, const void* k_w,
                                const void* cos_t, const void* sin_t, int rot, float eps, void* y, int64_t ldy) {
  WX_CHECK_ARG(ctx, ctx && x && y && qweight_ok(w) && m >= 0 && lda >= w->k && q_w && k_w);
  WX_CHECK_ARG(ctx, H > 0 && (head_dim == 128 || head_dim == 64) && w->n == 3 * (int64_t)H * head_dim);
  WX_CHECK_ARG(ctx, rot >= 0 && rot <= head_dim && rot % 2 == 0 && (rot == 0 || (cos_t && sin_t)));
  WX_CHECK_ARG(ctx, ldy >= w->n && (!lora || lora_pack_ok(lora, w)));
  if (m == 0) return WX_OK;
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t b_wd = al((size_t)w->n * w->k * 2), b_t = lora ? al((size_t)m * lora->R * 2) : 0;
  int st = WX_OK;
  void* ws = workspace(ctx, b_wd + b_t, &st);
  if (!ws) return st;
  uint8_t* base = static_cast<uint8_t*>(ws);
  if (qkv_rope_fused_enabled() && qkv_rope_geometry_ok(w, head_dim, rot, q_w, k_w, cos_t, sin_t))
    return qkv_rope_with_scratch(ctx, x, m, lda, w, lora, head_dim, y, ldy, q_w, k_w, cos_t, sin_t, rot, eps, base,
                                 base + b_wd, nullptr);
  if ((st = qlinear_lora_with_scratch(ctx, x, m, lda, w, lora, WX_EPI_NONE, nullptr, nullptr, nullptr, y, ldy,
                                      nullptr, base, base + b_wd, nullptr)))
    return st;
  const int64_t inner = (int64_t)H * head_dim;
  return launch_qk_norm_rope(ctx, y, ldy, y, ldy, inner, 2, m, H, head_dim, q_w, k_w, cos_t, sin_t, rot, eps);
}

extern "C" int wx_qlinear(wx_ctx* ctx, const void* x, int64_t m, int64_t lda, const wx_qweight* w, int epilogue,
                          const void* gate, const void* resid, const uint32_t* rowmap, void* y, int64_t ldy,
                          void* y_raw) {
  WX_CHECK_ARG(ctx, ctx && x && y && qweight_ok(w) && m >= 0 && lda >= w->k);
  WX_CHECK_ARG(ctx, epilogue >= WX_EPI_NONE && epilogue <= WX_EPI_SWIGLU);
  WX_CHECK_ARG(ctx, epilogue != WX_EPI_GATE_RESID || (gate && resid));
  WX_CHECK_ARG(ctx, epilogue != WX_EPI_SWIGLU || w->n % 2 == 0);
  WX_CHECK_ARG(ctx, ldy >= (epilogue == WX_EPI_SWIGLU ? w->n / 2 : w->n));
  int st = WX_OK;
  void* ws = workspace(ctx, qlinear_scratch_bytes(w, m, epilogue), &st);
  if (!ws) return st;
  uint8_t* base = static_cast<uint8_t*>(ws);
  void* wd = base;
  void* tmp = base + ((qlinear_ws_need(m, w->n, w->k) + 255) & ~size_t(255));
  return qlinear_with_scratch(ctx, x, m, lda, w, epilogue, gate, resid, rowmap, y, ldy, y_raw, wd, tmp);
}
