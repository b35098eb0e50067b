// Probe: tensor-pipe, MMA-issue and softmax rates for the flash-attention tile shapes
// (128x128x128 S = Q K^T as an SS tcgen05.mma, O += P V as a TS tcgen05.mma, the softmax of
// one 128x128 tile out of TMEM), one CTA per SM on garbage operands. Modes: 0-3 MMA streams,
// 4-6 softmax only, 7-9 MMA with concurrent softmax warps, 10-16 MMA with commits / mbarrier
// waits per group, 17-21 MMA issue rate at small N, 22-23 two issuing threads.
// Every wait is bounded (2 s) and records an error code instead of hanging.
#include <cstdio>
#include <cstdlib>
#include <cuda_runtime.h>
#include "../csrc/wx_ptx.cuh"
using namespace wx;

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

constexpr int kTile = 32768;

template <int MODE>
__global__ void __launch_bounds__(384, 1) mb_kernel(int T, long long* cyc, float* sink) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem), sK = sQ + kTile, sV = sQ + 2 * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * kTile);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 6);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 3 * kTile / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0x3c003c00u, 0x3c003c00u, 0, 0);
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bars), 1);
    mbar_init(smem_u32(bars + 1), 1);
    mbar_init(smem_u32(bars + 2), 1);
    mbar_init(smem_u32(bars + 3), 1);
    mbar_init(smem_u32(bars + 4), 1);
    fence_mbar_init();
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(smem_u32(tslot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  long long t0 = clock64();
  if (MODE <= 3 || MODE >= 7) {
    static_assert(true, "");
    if (MODE == 13) { if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 80;"); else asm volatile("setmaxnreg.inc.sync.aligned.u32 200;"); }
    if ((warp == 1 || (MODE >= 22 && warp == 2)) && lane == 0) {
      const uint32_t tmw = tmem + (warp == 2 ? 256 : 0);
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_s256 = idesc_bf16_f32(128, 256, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128, false, true);
      uint64_t ad[8], bd[8];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
        ad[kk] = smem_desc_sw128(sQ + off, 16, 1024);
        bd[kk] = smem_desc_sw128(sK + off, 16, 1024);
      }
      for (int t = 0; t < T; ++t) {
        if (MODE == 0 || MODE == 2 || (MODE >= 7 && MODE <= 16)) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_bf16(tmem + (t & 1) * 128, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(sK + off, 16, 1024),
                      idesc_s, kk > 0 ? 1u : 0u);
          }
          if (MODE >= 10 && MODE != 14 && MODE != 16) {
            umma_commit(smem_u32(bars + 1));
            umma_commit(smem_u32(bars + 2));
          }
          if (MODE == 14) mbar_wait(smem_u32(bars + 3), 1, reinterpret_cast<int*>(sink), 1, nullptr);
          if (MODE == 15 || MODE == 16) {
            uint32_t okv;
            asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                         : "=r"(okv) : "r"(smem_u32(bars + 3)), "r"(1u) : "memory");
            if (!okv) sink[0] = 1.f;
          }
          if (MODE == 11 || MODE == 13) mbar_wait(smem_u32(bars + 3), 1, reinterpret_cast<int*>(sink), 1, nullptr);
          if (MODE == 12 && t > 0) mbar_wait(smem_u32(bars + 1), (t - 1) & 1, reinterpret_cast<int*>(sink), 1, nullptr);
        }
        if (MODE == 1 || MODE == 2 || (MODE >= 7 && MODE <= 16)) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ts(tmem + 256, tmem + 384 + kk * 8, smem_desc_sw128(sV + kk * 2048, 16384, 1024), idesc_o, 1u);
        }
        if (MODE == 17 || MODE == 18 || MODE == 19) {
          constexpr uint32_t idn = idesc_bf16_f32(128, MODE == 17 ? 64 : (MODE == 18 ? 256 : 32), false, false);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_bf16(tmem, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(sK + off, 16, 1024), idn,
                      kk > 0 ? 1u : 0u);
          }
        }
        if (MODE == 22 || MODE == 23) {
          constexpr uint32_t idn = idesc_bf16_f32(128, MODE == 22 ? 32 : 128, false, false);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;" ::"r"(tmw), "l"(ad[kk]), "l"(bd[kk]), "r"(idn) : "memory");
        }
        if (MODE == 20 || MODE == 21) {
          constexpr uint32_t idn = idesc_bf16_f32(128, 32, false, false);
          if (MODE == 20) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;" ::"r"(tmem), "l"(ad[kk]), "l"(bd[kk]), "r"(idn) : "memory");
          } else {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem), "l"(ad[kk]), "l"(bd[kk]), "r"(idn), "r"(kk) : "memory");
          }
        }
        if (MODE == 3 && (t & 1) == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            // B = 256 rows: K tile followed by V tile region (rows 0-127 K, 128-255 V) as one K-major operand
            umma_bf16(tmem, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(sK + off, 16, 1024), idesc_s256,
                      kk > 0 ? 1u : 0u);
          }
        }
      }
      const uint32_t endbar = smem_u32(bars + (warp == 2 ? 4 : 0));
      umma_commit(endbar);
      mbar_wait(endbar, 0, reinterpret_cast<int*>(sink), 1, nullptr);
    }
  }
  if (MODE >= 4 && MODE < 10) {
    // softmax roles: MODE 4: warps 4-7; MODE 5: warps 4-11; MODE 6: MUFU only (warps 4-7)
    const bool act = (MODE == 5 || MODE == 7 || MODE == 8) ? warp >= 4 : (warp >= 4 && warp < 8);
    if (act) {
      const int X = (warp - 4) >> 2;
      const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
      const uint32_t tS = tmem + lane_addr + X * 128;
      float acc = 0.f;
      for (int t = 0; t < T; ++t) {
        float v[128];
        if (MODE != 6 && MODE != 8) {
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<float(*)[32]>(v + c * 32));
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i) v[i] = acc * (float)i;
        }
        float mx[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
#pragma unroll
        for (int i = 0; i < 128; i += 8) {
          mx[0] = max3f(mx[0], v[i], v[i + 1]);
          mx[1] = max3f(mx[1], v[i + 2], v[i + 3]);
          mx[2] = max3f(mx[2], v[i + 4], v[i + 5]);
          mx[3] = max3f(mx[3], v[i + 6], v[i + 7]);
        }
        const float m = max3f(fmaxf(mx[0], mx[1]), mx[2], mx[3]);
        const float2 sc = make_float2(0.127f, 0.127f), nm = make_float2(-m, -m);
        float2 rs[4] = {};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 a = __ffma2_rn(make_float2(v[32 * c + 2 * i], v[32 * c + 2 * i + 1]), sc, nm);
            const float2 pv = make_float2(ex2f(a.x), ex2f(a.y));
            rs[i & 3] = __fadd2_rn(rs[i & 3], pv);
            pk[i] = pack_bf16x2(pv.x, pv.y);
          }
          if (MODE != 6 && MODE != 8) tmem_st16(tS + c * 16, pk);
          else acc += __uint_as_float(pk[0] ^ pk[15]);
        }
        if (MODE != 6 && MODE != 8) tmem_wait_st();
        acc += rs[0].x + rs[1].y + rs[2].x + rs[3].y;
      }
      if (acc == 12345.f) sink[threadIdx.x] = acc;
    }
  }
  long long t1 = clock64();
  if (((MODE <= 3 || MODE >= 7) && threadIdx.x == 32) || (MODE > 3 && MODE < 7 && threadIdx.x == 128))
    cyc[blockIdx.x] = t1 - t0;
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int MODE>
void run(int T, const char* name) {
  long long* cyc;
  float* sink;
  cudaMalloc(&cyc, 148 * 8);
  cudaMalloc(&sink, 4096);
  const int smem = 3 * kTile + 1024 + 1024;
  cudaFuncSetAttribute(mb_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  mb_kernel<MODE><<<148, 384, smem>>>(T, cyc, sink);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0);
  mb_kernel<MODE><<<148, 384, smem>>>(T, cyc, sink);
  cudaEventRecord(e1);
  cudaError_t err = cudaDeviceSynchronize();
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  long long h[148];
  cudaMemcpy(h, cyc, sizeof(h), cudaMemcpyDeviceToHost);
  double avg = 0;
  for (int i = 0; i < 148; ++i) avg += h[i];
  avg /= 148;
  printf("%-34s err=%d  %.3f ms  %.0f clk/tile  (clk %.2f GHz)\n", name, (int)err, ms, avg / T, avg / (ms * 1e6));
  cudaFree(cyc);
  cudaFree(sink);
}

int main() {
  const int T = 4000;
  run<0>(T, "S only (SS 128x128x128)");
  run<1>(T, "PV only (TS 128x128x128)");
  run<2>(T, "S + PV");
  run<3>(T, "SS 128x256x128 per 2 tiles");
  run<4>(T, "softmax 4 warps (TMEM ld/st)");
  run<5>(T, "softmax 8 warps (two slots)");
  run<6>(T, "softmax math only 4 warps");
  run<7>(T, "MMA S+PV | 8 softmax warps TMEM");
  run<8>(T, "MMA S+PV | 8 softmax warps math");
  run<9>(T, "MMA S+PV | 4 softmax warps TMEM");
  run<10>(T, "S+PV, 2 commits per S group");
  run<11>(T, "+ wait on complete barrier");
  run<12>(T, "+ wait previous S group done");
  run<13>(T, "mode 11 + setmaxnreg 80/200");
  run<14>(T, "wait on complete barrier, no commits");
  run<15>(T, "commits + test_wait");
  run<16>(T, "test_wait, no commits");
  run<17>(T, "8 MMAs N=64 per iter");
  run<18>(T, "8 MMAs N=256 per iter");
  run<19>(T, "8 MMAs N=32 per iter");
  run<20>(T, "8 MMAs N=32 precomputed, acc=1");
  run<21>(T, "8 MMAs N=32 precomputed, setp");
  run<22>(T, "2 threads x 8 MMAs N=32");
  run<23>(T, "2 threads x 8 MMAs N=128");
  return 0;
}
