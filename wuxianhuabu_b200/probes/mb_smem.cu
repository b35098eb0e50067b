// Probe: does TMA traffic into shared memory slow the tcgen05 MMAs (shared-memory
// bandwidth)? An S+PV MMA stream with and without a concurrent 2-stage TMA tile stream.
// Every wait is bounded (2 s) and records an error code instead of hanging.
#include <cstdio>
#include <cuda.h>
#include <cuda_runtime.h>
#include "../csrc/wx_ptx.cuh"
using namespace wx;
constexpr int kTile = 32768;

// MODE 0: MMA S+PV only; 1: MMA + TMA stream; 2: TMA stream only; 3: MMA S(TS: A from TMEM)+PV + TMA
template <int MODE>
__global__ void __launch_bounds__(128, 1) mb(const __grid_constant__ CUtensorMap tm, int T, int nt, long long* cyc,
                                             int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem), sK = sQ + kTile, sV = sQ + 2 * kTile, sR = sQ + 3 * kTile;  // ring 2 x 32K
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 5 * kTile);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* stop = reinterpret_cast<volatile int*>(bars + 9);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 3 * kTile / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0x3c003c00u, 0x3c003c00u, 0, 0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(smem_u32(bars + i), 1);
    *stop = 0;
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
  if (warp == 1 && lane == 0) {
    long long t0 = clock64();
    if (MODE != 2) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128, false, true);
      for (int t = 0; t < T; ++t) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          if (MODE == 3)
            umma_bf16_ts(tmem + (t & 1) * 128, tmem + 448 + kk * 8, smem_desc_sw128(sK + off, 16, 1024), idesc_s,
                         kk > 0 ? 1u : 0u);
          else
            umma_bf16(tmem + (t & 1) * 128, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(sK + off, 16, 1024),
                      idesc_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ts(tmem + 256, tmem + 384 + kk * 8, smem_desc_sw128(sV + kk * 2048, 16384, 1024), idesc_o, 1u);
      }
      umma_commit(smem_u32(bars + 4));
      mbar_wait(smem_u32(bars + 4), 0, err, 1, nullptr);
      cyc[blockIdx.x] = clock64() - t0;
      *stop = 1;
    }
  }
  if (warp == 0 && lane == 0 && MODE != 0) {
    // TMA stream: 2-stage ring, consumed immediately (wait full, re-issue)
    uint32_t x = 12345u + blockIdx.x * 7919u;
    long long t0 = clock64();
    int t = 0;
    const int TT = (MODE == 2) ? T : 1 << 30;
    for (; t < TT; ++t) {
      const int st = t & 1;
      if (t >= 2 && !mbar_wait(smem_u32(bars + st), ((t - 2) >> 1) & 1, err, 2, nullptr)) break;
      if (MODE != 2 && *stop) break;
      x = x * 1664525u + 1013904223u;
      const int row = (int)((x >> 8) % (uint32_t)nt) * 128;
      const uint32_t b = smem_u32(bars + st);
      mbar_arrive_expect_tx(b, kTile);
      for (int ch = 0; ch < 2; ++ch) {
        tma_load_2d(sR + st * kTile + ch * 16384, &tm, b, (t & 1) * 3072 + ch * 64, row);
        tma_load_2d(sR + st * kTile + ch * 16384 + 8192, &tm, b, (t & 1) * 3072 + ch * 64, row + 64);
      }
    }
    // drain
    for (int i = t - 2; i < t; ++i)
      if (i >= 0) mbar_wait(smem_u32(bars + (i & 1)), (i >> 1) & 1, err, 3, nullptr);
    if (MODE == 2) cyc[blockIdx.x] = clock64() - t0;
    else cyc[148 + blockIdx.x] = t;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
template <int MODE>
void run(const CUtensorMap& tm, int T, const char* name) {
  long long* cyc;
  int* err;
  cudaMalloc(&cyc, 2 * 148 * 8);
  cudaMalloc(&err, 4);
  cudaMemset(err, 0, 4);
  cudaMemset(cyc, 0, 2 * 148 * 8);
  const int smem = 5 * kTile + 2048;
  cudaFuncSetAttribute(mb<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  mb<MODE><<<148, 128, smem>>>(tm, T, 222, cyc, err);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0);
  mb<MODE><<<148, 128, smem>>>(tm, T, 222, cyc, err);
  cudaEventRecord(e1);
  cudaError_t e = cudaDeviceSynchronize();
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  long long h[296];
  int herr = 0;
  cudaMemcpy(h, cyc, sizeof(h), cudaMemcpyDeviceToHost);
  cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
  double avg = 0, tiles = 0;
  for (int i = 0; i < 148; ++i) avg += h[i], tiles += h[148 + i];
  avg /= 148;
  tiles /= 148;
  printf("%-36s err=%d/%d %.3f ms %.0f clk/tile; TMA tiles during MMA %.0f (%.1f B/clk)\n", name, (int)e, herr, ms,
         avg / T, tiles, tiles * kTile / avg);
  cudaFree(cyc);
  cudaFree(err);
}

int main() {
  const long rows = 28544, cols = 9216;
  void* buf;
  cudaMalloc(&buf, rows * cols * 2);
  cudaMemset(buf, 0, rows * cols * 2);
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
  EncodeFn fn = (EncodeFn)p;
  CUtensorMap tm;
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t es[2] = {1, 1};
  fn(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, buf, gdim, gstride, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  const int T = 3000;
  run<0>(tm, T, "MMA S(SS)+PV only");
  run<2>(tm, T, "TMA stream only (clk per 32K tile)");
  run<1>(tm, T, "MMA S(SS)+PV with TMA stream");
  run<3>(tm, T, "MMA S(TS)+PV with TMA stream");
  return 0;
}
