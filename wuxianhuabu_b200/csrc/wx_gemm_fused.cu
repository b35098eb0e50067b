// wx_gemm_fused.cu — 6-bit quantized linear for small M (weight-bandwidth bound):
// the packed weights are unpacked and dequantised in shared memory and fed to
// tcgen05.mma without an expanded copy in global memory.
//
// Tiling: a CTA owns a 64-column slice of N, up to 2 x 128 rows of M and a
// K range (split-K over CTAs so that small-M problems still fill 148 SMs).
// Per 64-wide K block (= one quantization group):
//   warp 0      TMA-loads the activation tiles (128x64 bf16, SW128) of every M tile
//   warps 6..7  each thread loads its weight row's 12 words + scale/bias, expands
//               the 64 values with fp32 q*scale+bias -> bf16 (bit-identical to
//               the reference dequant) and stores them in the SW128 K-major
//               layout the MMA reads; fence.proxy.async; arrive
//   warp 1      issues tcgen05.mma (M=128, N=64, K=16) per M tile into TMEM
// after the last K block warps 2..5 store the fp32 partial tile of this K split;
// a second kernel sums the splits in a fixed order (deterministic) and applies
// the epilogue (bf16 rounding, bias, GELU or gate + residual) exactly as the main
// GEMM does.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

bool qweight_ok(const wx_qweight* w);

constexpr int kFBN = 64;            // columns per CTA
constexpr int kFMaxSplits = 4;      // K splits (bounded: the partials live in scratch)
constexpr int kFBK = 64;            // K per stage (one quantization group)
constexpr int kFStages = 4;
constexpr int kFMaxMT = 2;          // M tiles per CTA
constexpr int kFThreads = 256;      // 8 warps: TMA, MMA, 4 epilogue, 2 dequant (one thread per weight row)
constexpr int kFABytes = 128 * kFBK * 2;   // one activation tile
constexpr int kFBBytes = kFBN * kFBK * 2;  // the expanded weight tile
constexpr int kFStageBytes = kFMaxMT * kFABytes + kFBBytes;
constexpr int kFBarOffset = kFStages * kFStageBytes;
constexpr int kFSmem = kFBarOffset + 256 + 1024;

struct FusedParams {
  int M, N, K, mt;            // mt = M tiles this CTA computes (rows m_base .. m_base + 128*mt)
  int kb_per_split;
  const uint32_t* wq;
  const __nv_bfloat16* scales;
  const __nv_bfloat16* biases;
  int64_t words_per_row;
  int groups_per_row;
  float* part;                // [splits][M][N] fp32 partial sums
  int* err;
};

// 6-bit value i (0..15) of a 3-word bundle
__device__ __forceinline__ uint32_t q6(uint32_t w0, uint32_t w1, uint32_t w2, int i) {
  switch (i) {
    case 0: return w0 & 63u;
    case 1: return (w0 >> 6) & 63u;
    case 2: return (w0 >> 12) & 63u;
    case 3: return (w0 >> 18) & 63u;
    case 4: return (w0 >> 24) & 63u;
    case 5: return __funnelshift_r(w0, w1, 30) & 63u;
    case 6: return (w1 >> 4) & 63u;
    case 7: return (w1 >> 10) & 63u;
    case 8: return (w1 >> 16) & 63u;
    case 9: return (w1 >> 22) & 63u;
    case 10: return __funnelshift_r(w1, w2, 28) & 63u;
    case 11: return (w2 >> 2) & 63u;
    case 12: return (w2 >> 8) & 63u;
    case 13: return (w2 >> 14) & 63u;
    case 14: return (w2 >> 20) & 63u;
    default: return w2 >> 26;
  }
}

// float(q) exactly, by placing q in the low mantissa bits of 2^23
__device__ __forceinline__ float q_to_f(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }

__global__ void __launch_bounds__(kFThreads, 1)
    gemm_q6_fused_kernel(const __grid_constant__ CUtensorMap tmA, FusedParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kFBarOffset);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kFStages + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + kFStages + s); };
  const uint32_t done_bar = smem_u32(bars + 2 * kFStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kFBN;
  const int m_base = blockIdx.z * kFMaxMT * 128;
  const int kb0 = blockIdx.y * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, p.K / kFBK);
  const int nkb = kb1 - kb0;
  const int mt = p.mt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(full_bar(s), 1 + kFBN);  // A producer (with tx bytes) + one dequant thread per weight row
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kFMaxMT * kFBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % kFStages;
        if (!mbar_wait(empty_bar(s), ((i / kFStages) & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(full_bar(s), mt * kFABytes);
        const uint32_t sa = smem_u32(smem + s * kFStageBytes);
        for (int t = 0; t < mt; ++t)
          tma_load_2d(sa + t * kFABytes, &tmA, full_bar(s), (kb0 + i) * kFBK, m_base + t * 128);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, kFBN, false, false);
      bool ok = true;
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % kFStages;
        if (!mbar_wait(full_bar(s), (i / kFStages) & 1, p.err, kDevTimeoutFull, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * kFStageBytes);
        const uint32_t sb = sa + kFMaxMT * kFABytes;
        for (int t = 0; t < mt; ++t) {
#pragma unroll
          for (int kk = 0; kk < kFBK / 16; ++kk)
            umma_bf16(tmem + t * kFBN, smem_desc_sw128(sa + t * kFABytes + kk * 32, 16, 1024),
                      smem_desc_sw128(sb + kk * 32, 16, 1024), idesc, (i | kk) != 0 ? 1u : 0u);
        }
        umma_commit(empty_bar(s));
      }
      if (ok) umma_commit(done_bar);
    }
  } else if (warp >= 6) {
    // dequant producers: thread t expands weight row n0 + t
    const int t = threadIdx.x - 6 * 32;
    const int64_t n = n0 + t;
    const uint32_t* wrow = p.wq + n * p.words_per_row;
    const __nv_bfloat16* srow = p.scales + n * p.groups_per_row;
    const __nv_bfloat16* brow = p.biases + n * p.groups_per_row;
    // three K blocks of packed words in flight (register ring, statically indexed)
    constexpr int kDepth = 3;
    uint4 ra[kDepth], rb[kDepth], rc[kDepth];
    float rs[kDepth], rbi[kDepth];
    auto fetch = [&](int slot, int kb) {
      const uint4* src = reinterpret_cast<const uint4*>(wrow + (int64_t)kb * 12);
      ra[slot] = __ldg(src);
      rb[slot] = __ldg(src + 1);
      rc[slot] = __ldg(src + 2);
      rs[slot] = __bfloat162float(srow[kb]);
      rbi[slot] = __bfloat162float(brow[kb]);
    };
#pragma unroll
    for (int d = 0; d < kDepth; ++d)
      if (d < nkb) fetch(d, kb0 + d);
    bool ok = true;
    auto expand = [&](int i, int slot) {
      const int s = i % kFStages;
      const uint32_t w[12] = {ra[slot].x, ra[slot].y, ra[slot].z, ra[slot].w, rb[slot].x, rb[slot].y,
                              rb[slot].z, rb[slot].w, rc[slot].x, rc[slot].y, rc[slot].z, rc[slot].w};
      const float2 s2 = make_float2(rs[slot], rs[slot]), b2 = make_float2(rbi[slot], rbi[slot]);
      if (i + kDepth < nkb) fetch(slot, kb0 + i + kDepth);
      if (!mbar_wait(empty_bar(s), ((i / kFStages) & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) {
        ok = false;
        return;
      }
      const uint32_t rowaddr = smem_u32(smem + s * kFStageBytes + kFMaxMT * kFABytes) + t * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {  // 8 values per 16-byte chunk; 16 values per 3 words
        const int bundle = ch >> 1, half = ch & 1;
        const uint32_t w0 = w[bundle * 3], w1 = w[bundle * 3 + 1], w2 = w[bundle * 3 + 2];
        uint32_t packed[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i0 = half * 8 + 2 * e;
          const float2 q = make_float2(q_to_f(q6(w0, w1, w2, i0)), q_to_f(q6(w0, w1, w2, i0 + 1)));
          const float2 v = __ffma2_rn(q, s2, b2);  // one rounding, as fp32 q*s + b (q*s exact)
          packed[e] = pack_bf16x2(v.x, v.y);
        }
        const uint32_t addr = rowaddr + ((ch ^ (t & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(packed[0]), "r"(packed[1]),
                     "r"(packed[2]), "r"(packed[3])
                     : "memory");
      }
      fence_proxy_async_smem();
      mbar_arrive(full_bar(s));
    };
    for (int i = 0; i < nkb && ok; i += kDepth) {
#pragma unroll
      for (int d = 0; d < kDepth; ++d)
        if (ok && i + d < nkb) expand(i + d, d);
    }
  } else {
    // warps 2..5: store this split's fp32 partial tile
    const int quarter = warp & 3;
    const bool ok = nkb > 0 && mbar_wait(done_bar, 0, p.err, kDevTimeoutAcc, abort_flag);
    tc_fence_after();
    for (int tt = 0; tt < mt; ++tt) {
      const int64_t m = m_base + tt * 128 + quarter * 32 + lane;
#pragma unroll 1
      for (int cc = 0; cc < kFBN / 32; ++cc) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + tt * kFBN + cc * 32, v);
        tmem_wait_ld();
        if (!ok || m >= p.M) continue;
        float* dst = p.part + ((int64_t)blockIdx.y * p.M + m) * p.N + n0 + cc * 32;
#pragma unroll
        for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kFMaxMT * kFBN);
  }
}

// epilogue of the split-K path: same rounding sequence as the main GEMM epilogue
__global__ void fused_epilogue_kernel(const float* __restrict__ part, int splits, int64_t M, int N,
                                      const __nv_bfloat16* __restrict__ bias, int epi,
                                      const __nv_bfloat16* __restrict__ gate, const __nv_bfloat16* __restrict__ resid,
                                      const uint32_t* __restrict__ rowmap, __nv_bfloat16* __restrict__ y, int64_t ldy,
                                      __nv_bfloat16* __restrict__ y_raw) {
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N;
    const int n = (int)(i % N);
    float a = part[i];
    for (int sp = 1; sp < splits; ++sp) a += part[(int64_t)sp * total + i];
    float t = round_bf16(a);
    if (bias) t = round_bf16(t + __bfloat162float(bias[n]));
    float o = t;
    if (epi == WX_EPI_GELU) {
      const float cst = 0.7978845608028654f;
      o = 0.5f * t * (1.0f + tanhf(cst * (t + 0.044715f * t * t * t)));
    } else if (epi == WX_EPI_GATE_RESID) {
      const int64_t mr = rowmap ? (int64_t)rowmap[m] : 0;
      o = __bfloat162float(resid[m * ldy + n]) + t * __bfloat162float(gate[mr * N + n]);
      if (y_raw) y_raw[m * ldy + n] = __float2bfloat16_rn(t);
    }
    y[m * ldy + n] = __float2bfloat16_rn(o);
  }
}

size_t fused_scratch_bytes(int64_t M, int64_t N) { return ((size_t)kFMaxSplits * M * N * 4 + 255) & ~size_t(255); }

// eligible: 6-bit, group 64, N % 128 == 0, small M (handled in blocks of 256 rows)
bool fused_eligible(const wx_qweight* w, int64_t M, int epilogue) {
  // beyond one wave of N tiles (148 x 64 columns) every CTA streams all of K and
  // the two-pass GEMM measured faster (M=256, N=12288: 111 vs 130 us)
  return w->bits == 6 && w->group == kFBK && w->n % kFBN == 0 && w->k % kFBK == 0 && M > 0 && M <= 512 &&
         w->n <= 148 * kFBN && epilogue != WX_EPI_SWIGLU && (w->k * 6 / 32) % 4 == 0;
}

int qlinear_fused(wx_ctx* ctx, const void* x, int64_t M, int64_t lda, const wx_qweight* w, int epilogue,
                  const void* gate, const void* resid, const uint32_t* rowmap, void* y, int64_t ldy, void* y_raw,
                  void* scratch) {
  int st = ensure_smem_attr(ctx, (const void*)gemm_q6_fused_kernel, kFSmem, "gemm_q6_fused");
  if (st) return st;
  CUtensorMap ta;
  st = make_tmap_bf16_2d(ctx, &ta, x, (uint64_t)M, (uint64_t)w->k, (uint64_t)lda, kFBK, 128);
  if (st) return st;
  float* part = static_cast<float*>(scratch);
  const int n_tiles = (int)(w->n / kFBN);
  const int m_groups = (int)((M + kFMaxMT * 128 - 1) / (kFMaxMT * 128));
  const int kbs = (int)(w->k / kFBK);
  int splits = std::max(1, ctx->num_sms / std::max(1, n_tiles * m_groups));
  splits = std::min(std::min(splits, kFMaxSplits), std::max(1, kbs / 4));  // >= 4 K blocks per CTA
  const int kb_per = (kbs + splits - 1) / splits;
  splits = (kbs + kb_per - 1) / kb_per;
  FusedParams p{};
  p.M = (int)M;
  p.N = (int)w->n;
  p.K = (int)w->k;
  p.mt = (int)std::min<int64_t>(kFMaxMT, (M + 127) / 128);
  p.kb_per_split = kb_per;
  p.wq = w->wq;
  p.scales = static_cast<const __nv_bfloat16*>(w->scales);
  p.biases = static_cast<const __nv_bfloat16*>(w->biases);
  p.words_per_row = w->k * 6 / 32;
  p.groups_per_row = (int)(w->k / kFBK);
  p.part = part;
  p.err = ctx->dev_err;
  {
    ProfScope prof(ctx, kProfGemm);
    // rows past M in the last group read zero-filled activation tiles and are not stored
    dim3 grid(n_tiles, splits, m_groups);
    gemm_q6_fused_kernel<<<grid, kFThreads, kFSmem, ctx->stream>>>(ta, p);
    if ((st = launch_status(ctx, "gemm_q6_fused"))) return st;
    const int64_t total = M * w->n;
    const unsigned g = (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, ctx->num_sms * 8));
    fused_epilogue_kernel<<<g, 256, 0, ctx->stream>>>(part, splits, M, (int)w->n, static_cast<const __nv_bfloat16*>(w->bias),
                                                      epilogue, static_cast<const __nv_bfloat16*>(gate),
                                                      static_cast<const __nv_bfloat16*>(resid), rowmap,
                                                      static_cast<__nv_bfloat16*>(y), ldy,
                                                      static_cast<__nv_bfloat16*>(y_raw));
  }
  return launch_status(ctx, "fused_epilogue");
}

}  // namespace wx
