// wx_gemm_fused.cu — 6-bit quantized linear for small M (M <= 512: AdaLN tables,
// condition_proj, the text refiner, the small-M points of the GEMM sweep): the packed
// weights are expanded in shared memory and fed to tcgen05.mma, with no bf16 copy of
// the weight in global memory and no second launch.
//
// Operand roles are swapped: D^T[n, m] = W[n, :] . X[m, :], so 128 weight rows are the
// MMA's M and the tokens (up to 256 per CTA) its N; one CTA owns A x 128 output columns
// (A = 1 or 2 accumulators in TMEM), a tile of up to 256 rows and a K range. Per 64-wide
// K block (one quantization group):
//   warp 0      TMA: the activation tile X [Mt x 64] bf16 (SW128) and the packed
//               weight words [A*128 rows x 12 u32] of the block
//   warps 2..   T = 2 or 4 threads per weight row (row n0 + t/T, part t%T): 64/T six-bit
//               values each -> fp32 q*scale+bias (one rounding, as the reference's
//               dequant) -> bf16, stored in the SW128 K-major layout the MMA reads;
//               scales and biases come from a 4-deep register ring of plain loads
//   warp 1      4 x A tcgen05.mma (M=128, N=Mt, K=16) into TMEM [128 lanes x Mt] per
//               accumulator; both accumulators read the same activation tile
// At M = 256 the activation tile (32 KB per K block) outweighs the packed weights (6 KB
// per 128 rows) that each CTA brings in, and the tile is read again for every 128 (A = 1)
// or 256 (A = 2) weight rows: two accumulators cut the shared-memory fill from L2 by ~1.7x.
// K is split over the CTAs of a thread-block cluster (up to 8) so that small-M
// problems fill the SMs; the split count (and A) is chosen so that every cluster of the
// launch is resident at once (cudaOccupancyMaxActiveClusters). After the last MMA each
// CTA copies one accumulator's fp32 partial tile to its own shared memory (transposed,
// [Mt][128]); after a cluster barrier CTA r sums columns [r*Mt/s, (r+1)*Mt/s) of every
// CTA's partial through distributed shared memory, in split order 0, 1, ... (deterministic;
// four columns' loads in flight per thread), and applies the epilogue of the main GEMM
// (bf16 rounding, bias, GELU or gate + residual); a second cluster barrier keeps every
// partial alive until all CTAs have read it. With A = 2 this runs once per accumulator.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "wx_internal.h"
#include "wx_ptx.cuh"

namespace wx {

bool qweight_ok(const wx_qweight* w);

constexpr int kQRows = 128;          // weight rows of one accumulator (the MMA's M)
constexpr int kQBK = 64;             // K per stage (one quantization group)
constexpr int kQWords = 12;          // packed words of 64 six-bit values
constexpr int kQMaxMt = 256;         // tokens per CTA (the MMA's N)
constexpr int kQMaxSplits = 8;       // K splits = cluster size (portable limit)

// Shared-memory plan of the kernel with A accumulators (A * 128 weight rows per CTA, all
// sharing one activation tile per K block) and T expansion threads per weight row. Ring 1 holds what TMA brings per K block (the
// activation tile and the packed words of the CTA's rows), ring 2 the expanded weight tiles;
// the fp32 partial tile of one accumulator ([Mt][128]) reuses ring 1 after the last MMA.
//   A = 1: 4 x (32 + 6) KB + 4 x 16 KB  (216 KB)
//   A = 2: 3 x (32 + 12) KB + 2 x 32 KB (196 KB): the activation tile is read from L2 once
//          per 256 weight rows instead of once per 128
template <int A, int T>
struct Q6Cfg {
  static constexpr int kStages = A == 1 ? 4 : 3;     // ring 1 (TMA)
  static constexpr int kWStages = A == 1 ? 4 : 2;    // ring 2 (expanded weights)
  static constexpr int kRows = kQRows * A;           // weight rows per CTA
  static constexpr int kDequantWarps = 4 * A * T;    // T threads per weight row
  static constexpr int kThreads = 64 + 32 * kDequantWarps;  // warp 0 TMA, warp 1 MMA
  static constexpr int kXBytes = kQMaxMt * kQBK * 2;        // activation tile (32 KB)
  static constexpr int kPBytes = kRows * kQWords * 4;       // packed weight words
  static constexpr int kStageBytes = kXBytes + kPBytes;
  static constexpr int kWBytes = kRows * kQBK * 2;          // expanded weight tile(s)
  static constexpr int kWOff = kStages * kStageBytes;
  static constexpr int kBarOff = kWOff + kWStages * kWBytes;
  static constexpr int kSmem = kBarOff + 256 + 1024;
  static_assert(kStageBytes % 1024 == 0 && kWBytes % 1024 == 0, "SW128 tiles need 1024-byte alignment");
  static_assert(kQMaxMt * kQRows * 4 <= kWOff, "one accumulator's partial tile reuses ring 1");
  static_assert((2 * kStages + 2 * kWStages + 1) * 8 + 8 <= 256, "barriers, TMEM slot and abort flag");
  static_assert(kSmem <= 232448, "227 KB of dynamic shared memory per CTA");
};

struct Q6Params {
  int M, N, K;
  int Mt;            // tokens per CTA tile (multiple of 16, <= 256)
  int kb_per_split;  // K blocks per split
  int splits;        // = cluster size
  const __nv_bfloat16* scales;
  const __nv_bfloat16* biases;
  int groups;        // K / 64
  const __nv_bfloat16* bias;
  int epi;
  const __nv_bfloat16* gate;
  const __nv_bfloat16* resid;
  const uint32_t* rowmap;
  __nv_bfloat16* y;
  int64_t ldy;
  __nv_bfloat16* y_raw;
  int* err;
};

// 6-bit value i (0..15) of a 3-word bundle, OR-ed into the mantissa of 2^23 (so that
// float(result) - 2^23 = q exactly)
__device__ __forceinline__ uint32_t q6_bits(uint32_t w0, uint32_t w1, uint32_t w2, int i) {
  uint32_t q;
  switch (i) {
    case 0: q = w0; break;
    case 1: q = w0 >> 6; break;
    case 2: q = w0 >> 12; break;
    case 3: q = w0 >> 18; break;
    case 4: q = w0 >> 24; break;
    case 5: q = __funnelshift_r(w0, w1, 30); break;
    case 6: q = w1 >> 4; break;
    case 7: q = w1 >> 10; break;
    case 8: q = w1 >> 16; break;
    case 9: q = w1 >> 22; break;
    case 10: q = __funnelshift_r(w1, w2, 28); break;
    case 11: q = w2 >> 2; break;
    case 12: q = w2 >> 8; break;
    case 13: q = w2 >> 14; break;
    case 14: q = w2 >> 20; break;
    default: q = w2 >> 26; break;
  }
  return (q & 63u) | 0x4B000000u;
}

__device__ __forceinline__ float gelu_tanh_q(float x) {
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

template <int A, int T>
__global__ void __launch_bounds__(Q6Cfg<A, T>::kThreads, 1)
    gemm_q6_fused_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                         Q6Params p) {
  using L = Q6Cfg<A, T>;
  constexpr int S1 = L::kStages, S2 = L::kWStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  auto full_bar = [&](int s) { return smem_u32(bars + s); };                   // X + packed words landed
  auto empty_bar = [&](int s) { return smem_u32(bars + S1 + s); };             // MMAs reading ring-1 stage s done
  auto wfull_bar = [&](int w) { return smem_u32(bars + 2 * S1 + w); };         // weight tile w expanded
  auto wempty_bar = [&](int w) { return smem_u32(bars + 2 * S1 + S2 + w); };   // MMAs reading weight tile w done
  const uint32_t done_bar = smem_u32(bars + 2 * S1 + 2 * S2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S1 + 2 * S2 + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto sX = [&](int s) { return smem_u32(smem + s * L::kStageBytes); };
  auto sP = [&](int s) { return smem_u32(smem + s * L::kStageBytes + L::kXBytes); };
  auto sW = [&](int w) { return smem_u32(smem + L::kWOff + w * L::kWBytes); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * L::kRows;
  const int split = (int)cluster_ctarank();
  const int m0 = blockIdx.z * p.Mt;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, p.groups);
  const int nkb = max(0, kb1 - kb0);
  // TMEM columns of one accumulator; accumulator a (weight rows n0 + 128 a ...) at column a * tcols
  const uint32_t tcols = p.Mt <= 32 ? 32u : (p.Mt <= 64 ? 64u : (p.Mt <= 128 ? 128u : 256u));

  if (threadIdx.x == 0) {
    for (int s = 0; s < S1; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int w = 0; w < S2; ++w) {
      mbar_init(wfull_bar(w), L::kDequantWarps);  // one arrival per dequant warp
      mbar_init(wempty_bar(w), 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), tcols * A);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;  // (dequant warps) every K block of this split was expanded

  if (warp == 0) {
    if (lane == 0 && nkb > 0) {
      prefetch_tmap(&tmX);
      prefetch_tmap(&tmW);
      const uint32_t bytes = (uint32_t)p.Mt * kQBK * 2 + L::kPBytes;
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S1;
        if (!mbar_wait(empty_bar(s), ((i / S1) & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(full_bar(s), bytes);
        tma_load_2d(sX(s), &tmX, full_bar(s), (kb0 + i) * kQBK, m0);
        tma_load_2d(sP(s), &tmW, full_bar(s), (kb0 + i) * kQWords, n0);
        issued = i + 1;
      }
      if (issued < nkb)  // aborted: let the copies in flight land before the buffers are reused
        for (int j = max(0, issued - S1); j < issued; ++j) mbar_drain(full_bar(j % S1), (j / S1) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0 && nkb > 0) {
      const uint32_t idesc = idesc_bf16_f32(128, p.Mt, false, false);
      bool mok = true;
      for (int i = 0; i < nkb && mok; ++i) {
        const int s = i % S1, w = i % S2;
        if (!mbar_wait(full_bar(s), (i / S1) & 1, p.err, kDevTimeoutFull, abort_flag) ||
            !mbar_wait(wfull_bar(w), (i / S2) & 1, p.err, kDevTimeoutFull, abort_flag)) {
          mok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int a = 0; a < A; ++a)
#pragma unroll
          for (int kk = 0; kk < kQBK / 16; ++kk)
            umma_bf16(tmem + (uint32_t)a * tcols, smem_desc_sw128(sW(w) + a * kQRows * 128 + kk * 32, 16, 1024),
                      smem_desc_sw128(sX(s) + kk * 32, 16, 1024), idesc, (i | kk) != 0 ? 1u : 0u);
        umma_commit(empty_bar(s));
        umma_commit(wempty_bar(w));
      }
      if (mok) umma_commit(done_bar);
    }
  } else {
    // ---------------------------------------------------------------- dequant
    constexpr int V = kQBK / T;        // values of the K block per thread (32 or 16)
    constexpr int NW = 3 * (V / 16);   // their packed words (3 per 16 values)
    const int t = threadIdx.x - 64;    // 0 .. 128 A T - 1
    const int row = t / T, sub = t % T;  // weight row n0 + row, values [V sub, V sub + V) of the block
    const int64_t n = n0 + row;
    const __nv_bfloat16* srow = p.scales + n * p.groups;
    const __nv_bfloat16* brow = p.biases + n * p.groups;
    constexpr int kDepth = 4;  // scale/bias of the next K blocks in flight
    const unsigned short* srow16 = reinterpret_cast<const unsigned short*>(srow);
    const unsigned short* brow16 = reinterpret_cast<const unsigned short*>(brow);
    unsigned short rs[kDepth], rb[kDepth];
#pragma unroll
    for (int d = 0; d < kDepth; ++d) {
      rs[d] = d < nkb ? __ldg(srow16 + kb0 + d) : (unsigned short)0;
      rb[d] = d < nkb ? __ldg(brow16 + kb0 + d) : (unsigned short)0;
    }
    for (int i0 = 0; i0 < nkb && ok; i0 += kDepth) {
#pragma unroll
      for (int d = 0; d < kDepth; ++d) {
        const int i = i0 + d;
        if (!ok || i >= nkb) break;
        const int s = i % S1, w = i % S2;
        if (!mbar_wait(full_bar(s), (i / S1) & 1, p.err, kDevTimeoutFull, abort_flag) ||
            !mbar_wait(wempty_bar(w), ((i / S2) & 1) ^ 1u, p.err, kDevTimeoutEmpty, abort_flag)) {
          ok = false;
          break;
        }
        uint32_t wd[NW];  // 3-word bundles of 16 values
        const uint32_t pa = sP(s) + row * (kQWords * 4) + sub * (NW * 4);
        if constexpr (NW % 2 == 0) {
#pragma unroll
          for (int q = 0; q < NW / 2; ++q)
            asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(wd[2 * q]), "=r"(wd[2 * q + 1]) : "r"(pa + q * 8));
        } else {
#pragma unroll
          for (int q = 0; q < NW; ++q) asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wd[q]) : "r"(pa + q * 4));
        }
        const float sv = __uint_as_float((uint32_t)rs[d] << 16), bvv = __uint_as_float((uint32_t)rb[d] << 16);
        const float2 s2 = make_float2(sv, sv), b2 = make_float2(bvv, bvv);
        if (i + kDepth < nkb) {
          rs[d] = __ldg(srow16 + kb0 + i + kDepth);
          rb[d] = __ldg(brow16 + kb0 + i + kDepth);
        }
        const uint32_t rowaddr = sW(w) + row * 128;  // rows >= 128 land in the second 16 KB tile
        const float2 magic = make_float2(-8388608.0f, -8388608.0f);
#pragma unroll
        for (int c4 = 0; c4 < V / 8; ++c4) {  // 8 values per 16-byte chunk; 16 values per 3 words
          const int ch = sub * (V / 8) + c4;
          const int bundle = c4 >> 1, half = c4 & 1;
          const uint32_t w0 = wd[bundle * 3], w1 = wd[bundle * 3 + 1], w2 = wd[bundle * 3 + 2];
          uint32_t packed[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i0v = half * 8 + 2 * e;
            float2 q = make_float2(__uint_as_float(q6_bits(w0, w1, w2, i0v)),
                                   __uint_as_float(q6_bits(w0, w1, w2, i0v + 1)));
            q = __fadd2_rn(q, magic);                 // exact: the integer q in [0, 63]
            const float2 v = __ffma2_rn(q, s2, b2);   // one rounding, as fp32 q*s + b (q*s exact)
            packed[e] = pack_bf16x2(v.x, v.y);
          }
          const uint32_t addr = rowaddr + ((ch ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(packed[0]), "r"(packed[1]),
                       "r"(packed[2]), "r"(packed[3])
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(wfull_bar(w));
      }
    }
  }
  // ---------------------------------------- per accumulator: partial tile, cluster reduction
  // Every CTA copies accumulator a's fp32 partial to its own shared memory (transposed,
  // [Mt][128], over ring 1: every MMA has completed, so the stage buffers are free); after a
  // cluster barrier CTA r sums columns [r*Mt/s, (r+1)*Mt/s) of every CTA's partial through
  // distributed shared memory in split order 0, 1, ... (deterministic) and applies the
  // epilogue; a second barrier keeps the partials alive until every CTA has read them.
  bool acc_ok = false;  // (epilogue warps) the accumulators hold this split's sums
  if (warp >= 2) {
    acc_ok = ok && nkb > 0 && mbar_wait(done_bar, 0, p.err, kDevTimeoutAcc, abort_flag);
    tc_fence_after();
  }
  constexpr int G = L::kDequantWarps / 4;  // column groups of the epilogue warps
  constexpr int U = 4;      // columns reduced per iteration (all their loads in flight at once)
  float* part = reinterpret_cast<float*>(smem);
  const int q4 = warp & 3;                // TMEM lane quarter of this warp
  const int cg = (warp - 2) >> 2;         // column group (epilogue warps)
  const int r = q4 * 32 + lane;           // row of the accumulator
#pragma unroll 1
  for (int a = 0; a < A; ++a) {
    if (warp >= 2) {
      for (int c0 = cg * 32; c0 < p.Mt; c0 += 32 * G) {
        float v[32];
        if (acc_ok) {
          tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)a * tcols + c0, v);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < p.Mt) part[(c0 + i) * kQRows + r] = v[i];
      }
    }
    __syncwarp();
    cluster_sync_all();  // every CTA's partial of accumulator a is in its shared memory
    if (warp >= 2) {
      const int64_t n = n0 + a * kQRows + r;
      const int per = (p.Mt + p.splits - 1) / p.splits;
      const int c_lo = split * per, c_hi = min(p.Mt, c_lo + per);
      const uint32_t base = smem_u32(smem) + (uint32_t)r * 4;
      uint32_t peer[kQMaxSplits];
#pragma unroll
      for (int j = 0; j < kQMaxSplits; ++j) peer[j] = j < p.splits ? mapa_shared(base, (uint32_t)j) : 0u;
      const float bv = p.bias ? __bfloat162float(p.bias[n]) : 0.f;
      for (int c = c_lo + cg; c < c_hi; c += G * U) {
        uint32_t off[U];
#pragma unroll
        for (int u = 0; u < U; ++u) off[u] = (uint32_t)min(c + G * u, c_hi - 1) * kQRows * 4;  // in range
        float pv[kQMaxSplits][U];
#pragma unroll
        for (int j = 0; j < kQMaxSplits; ++j)
#pragma unroll
          for (int u = 0; u < U; ++u) pv[j][u] = j < p.splits ? ld_shared_cluster_f32(peer[j] + off[u]) : 0.f;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int cu = c + G * u;
          const int64_t m = m0 + cu;
          if (cu >= c_hi || m >= p.M) break;
          if (!WX_IN_BOUNDS(p.err, n < p.N)) break;
          float acc = pv[0][u];
#pragma unroll
          for (int j = 1; j < kQMaxSplits; ++j)
            if (j < p.splits) acc += pv[j][u];
          float tv = round_bf16(acc);
          if (p.bias) tv = round_bf16(tv + bv);
          float o = tv;
          if (p.epi == WX_EPI_GATE_RESID) {
            const int64_t mr = p.rowmap ? (int64_t)p.rowmap[m] : 0;
            if (p.y_raw) p.y_raw[m * p.ldy + n] = __float2bfloat16_rn(tv);
            o = __bfloat162float(p.resid[m * p.ldy + n]) + tv * __bfloat162float(p.gate[mr * (int64_t)p.N + n]);
          } else if (p.epi == WX_EPI_GELU) {
            o = gelu_tanh_q(tv);
          }
          p.y[m * p.ldy + n] = __float2bfloat16_rn(o);
        }
      }
    }
    __syncwarp();
    cluster_sync_all();  // no CTA overwrites or leaves while another still reads its partial
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols * A);
  }
}

size_t fused_scratch_bytes(int64_t, int64_t) { return 0; }

// eligible: 6-bit, group 64, N % 128 == 0, M <= 512 (tiles of <= 256 rows), not SwiGLU
bool fused_eligible(const wx_qweight* w, int64_t M, int epilogue) {
  return w->bits == 6 && w->group == kQBK && w->n % kQRows == 0 && w->k % kQBK == 0 && M > 0 && M <= 512 &&
         epilogue != WX_EPI_SWIGLU && w->n <= INT32_MAX && w->k <= INT32_MAX;
}

// clusters of `size` CTAs of gemm_q6_fused_kernel<A, T> the current device holds at once
// (cached per device)
template <int A, int T>
static int max_active_clusters(int size) {
  using L = Q6Cfg<A, T>;
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, size});
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1, (unsigned)size, 1);
  cfg.blockDim = dim3(L::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)size;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (const void*)gemm_q6_fused_kernel<A, T>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[{dev, size}] = n;
  return n;
}

// WX_QGEMM_ROWS=128 or 256 forces the weight rows per CTA of the small-M kernel (A/B
// measurements and tests; 256 needs N % 256 == 0); unset or 0: chosen per call
static int forced_rows() {
  const char* e = getenv("WX_QGEMM_ROWS");
  return e ? atoi(e) : 0;
}
// WX_QGEMM_TPR=2 or 4 forces the expansion threads per weight row of the 128-row CTA (A/B
// measurements and tests); unset or 0: chosen per call
static int forced_tpr() {
  const char* e = getenv("WX_QGEMM_TPR");
  const int v = e ? atoi(e) : 0;
  return v == 2 || v == 4 ? v : 0;
}

struct Q6Plan {
  int A = 1, T = 2, splits = 1;
  double cost = 1e30;
};

// Relative cost of one K block of a CTA with A accumulators (A = 1 is the unit). The
// two-accumulator CTA does twice the MMA and expansion work per K block but reads the
// activation tile once for both. Fitted on B200: with 1.45 the plan picks the faster of the
// two shapes at each of ten measured small-M GEMMs (M 8-512, K 704-12288, N 768-32256);
// 256 rows win where 128-row CTAs need more than one wave or few K splits (large N).
template <int A>
constexpr double kQBlockCost = A == 1 ? 1.0 : 1.45;

// K splits (= cluster size, <= 8) for CTAs of A * 128 weight rows: the fewest waves of
// clusters (at most the number of clusters of that size the device holds at once) times
// the K blocks per CTA, plus a fixed cost per reduction pass and a small one per split
template <int A, int T>
static int plan_q6(wx_ctx* ctx, int64_t N, int zt, int kbs, Q6Plan* best) {
  const int st =
      ensure_smem_attr(ctx, (const void*)gemm_q6_fused_kernel<A, T>, Q6Cfg<A, T>::kSmem, "gemm_q6_fused");
  if (st) return st;
  const int64_t clusters = N / Q6Cfg<A, T>::kRows * zt;
  for (int s = 1; s <= kQMaxSplits && s <= kbs; ++s) {
    const int active = max_active_clusters<A, T>(s);
    if (active <= 0) continue;
    const double waves = (double)((clusters + active - 1) / active);
    const double cost = waves * (((kbs + s - 1) / s) * kQBlockCost<A> + 3.0 * A) + 0.25 * s * A;
    if (cost < best->cost - 1e-9) {
      best->cost = cost;
      best->A = A;
      best->T = T;
      best->splits = s;
    }
  }
  return WX_OK;
}

template <int A, int T>
static int launch_q6(wx_ctx* ctx, const CUtensorMap& tx, const CUtensorMap& tw, const Q6Params& p, int64_t N,
                     int zt) {
  using L = Q6Cfg<A, T>;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(N / L::kRows), (unsigned)p.splits, (unsigned)zt);
  cfg.blockDim = dim3(L::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)p.splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ProfScope prof(ctx, kProfGemm);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_q6_fused_kernel<A, T>, tx, tw, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, WX_ERR_CUDA, "gemm_q6_fused<%d> launch (cluster of %d): %s", A, p.splits,
                     cudaGetErrorString(e));
  }
  return launch_status(ctx, "gemm_q6_fused");
}

int qlinear_fused(wx_ctx* ctx, const void* x, int64_t M, int64_t lda, const wx_qweight* w, int epilogue,
                  const void* gate, const void* resid, const uint32_t* rowmap, void* y, int64_t ldy, void* y_raw,
                  void* /*scratch*/) {
  if (!aligned16(x) || lda % 8 != 0)
    return set_error(ctx, WX_ERR_INVALID, "fused qlinear: x needs 16-byte aligned rows");
  // token tiles of Mt rows (balanced, a multiple of 16, at most 256)
  const int zt = (int)((M + kQMaxMt - 1) / kQMaxMt);
  const int Mt = (int)((((M + zt - 1) / zt) + 15) / 16 * 16);
  const int kbs = (int)(w->k / kQBK);
  const int forced = forced_rows();
  const bool two_ok = w->n % (2 * kQRows) == 0;
  Q6Plan plan;
  int st;
  // (both thread counts of the 128-row CTA hold one CTA per SM: the same cluster occupancy)
  if ((forced != 256 || !two_ok) && (st = plan_q6<1, 2>(ctx, w->n, zt, kbs, &plan))) return st;
  if (forced != 128 && two_ok && (st = plan_q6<2, 2>(ctx, w->n, zt, kbs, &plan))) return st;
  if (plan.cost >= 1e30) return set_error(ctx, WX_ERR_CUDA, "gemm_q6_fused: no cluster size fits the device");
  const int kb_per = (kbs + plan.splits - 1) / plan.splits;
  if (plan.A == 1) {
    // four expansion threads per weight row (16 warps, 16 values each) shorten the expansion
    // of a K block; measured faster with full 256-token tiles and short K ranges per CTA
    // (the pipeline start dominates), slower with small token tiles or long K ranges
    const int tpr = forced_tpr();
    plan.T = tpr ? tpr : (Mt == kQMaxMt && kb_per <= 32 ? 4 : 2);
    if (plan.T == 4 &&
        (st = ensure_smem_attr(ctx, (const void*)gemm_q6_fused_kernel<1, 4>, Q6Cfg<1, 4>::kSmem, "gemm_q6_fused")))
      return st;
  }
  CUtensorMap tx, tw;
  if ((st = make_tmap_bf16_2d(ctx, &tx, x, (uint64_t)M, (uint64_t)w->k, (uint64_t)lda, kQBK, (uint32_t)Mt))) return st;
  const int64_t words = w->k * 6 / 32;
  if ((st = make_tmap_u32_2d(ctx, &tw, w->wq, (uint64_t)w->n, (uint64_t)words, (uint64_t)words, kQWords,
                             (uint32_t)(kQRows * plan.A))))
    return st;
  Q6Params p{};
  p.M = (int)M;
  p.N = (int)w->n;
  p.K = (int)w->k;
  p.Mt = Mt;
  p.kb_per_split = kb_per;
  p.splits = plan.splits;
  p.scales = static_cast<const __nv_bfloat16*>(w->scales);
  p.biases = static_cast<const __nv_bfloat16*>(w->biases);
  p.groups = kbs;
  p.bias = static_cast<const __nv_bfloat16*>(w->bias);
  p.epi = epilogue;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.resid = static_cast<const __nv_bfloat16*>(resid);
  p.rowmap = rowmap;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  p.y_raw = static_cast<__nv_bfloat16*>(y_raw);
  p.err = ctx->dev_err;
  if (plan.A == 2) return launch_q6<2, 2>(ctx, tx, tw, p, w->n, zt);
  return plan.T == 4 ? launch_q6<1, 4>(ctx, tx, tw, p, w->n, zt) : launch_q6<1, 2>(ctx, tx, tw, p, w->n, zt);
}

}  // namespace wx
