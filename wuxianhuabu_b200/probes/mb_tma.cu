// Probe: TMA feed rate of 128x128 bf16 tiles (4 boxes of 64x64, SW128, as the flash
// kernels load K and V) into shared memory, NS-stage ring, from one head's K/V columns of a
// packed qkv buffer (L2-resident, heads=1) or from all 24 heads (mostly HBM, heads=24).
// Every wait is bounded (2 s) and records an error code instead of hanging.
#include <cstdio>
#include <cstdlib>
#include <cuda.h>
#include <cuda_runtime.h>
#include "../csrc/wx_ptx.cuh"
using namespace wx;

constexpr int kTile = 32768;

template <int NS>
__global__ void __launch_bounds__(128, 1) mb_tma(const __grid_constant__ CUtensorMap tm, int T, int ntiles,
                                                 long long* cyc, int* err, int heads) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NS * kTile);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(smem_u32(bars + i), 1);
      mbar_init(smem_u32(bars + NS + i), 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  long long t0 = clock64();
  if (warp == 0 && lane == 0) {
    uint32_t x = 12345u + blockIdx.x * 7919u;
    for (int t = 0; t < T; ++t) {
      const int st = t % NS;
      const uint32_t ph = (t / NS) & 1;
      if (!mbar_wait(smem_u32(bars + NS + st), ph ^ 1u, err, 2, nullptr)) break;
      x = x * 1664525u + 1013904223u;
      const int row = (int)((x >> 8) % (uint32_t)ntiles) * 128;
      int col = (t & 1) ? 3072 : 0;  // "K" then "V" region of the packed qkv row
      if (heads > 1) col += (int)((x >> 3) % (uint32_t)heads) * 128;
      const uint32_t b = smem_u32(bars + st);
      mbar_arrive_expect_tx(b, kTile);
      for (int ch = 0; ch < 2; ++ch) {
        tma_load_2d(s0 + st * kTile + ch * 16384, &tm, b, col + ch * 64, row);
        tma_load_2d(s0 + st * kTile + ch * 16384 + 8192, &tm, b, col + ch * 64, row + 64);
      }
    }
  } else if (warp == 1 && lane == 0) {
    for (int t = 0; t < T; ++t) {
      const int st = t % NS;
      const uint32_t ph = (t / NS) & 1;
      if (!mbar_wait(smem_u32(bars + st), ph, err, 1, nullptr)) break;
      mbar_arrive(smem_u32(bars + NS + st));
    }
  }
  long long t1 = clock64();
  if (threadIdx.x == 32) cyc[blockIdx.x] = t1 - t0;
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

template <int NS>
void run(const CUtensorMap& tm, int T, int ntiles, int grid, int heads = 1) {
  long long* cyc;
  int* err;
  cudaMalloc(&cyc, 148 * 8);
  cudaMalloc(&err, 4);
  cudaMemset(err, 0, 4);
  const int smem = NS * kTile + 1024 + 1024;
  cudaFuncSetAttribute(mb_tma<NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  mb_tma<NS><<<grid, 128, smem>>>(tm, T, ntiles, cyc, err, heads);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0);
  mb_tma<NS><<<grid, 128, smem>>>(tm, T, ntiles, cyc, err, heads);
  cudaEventRecord(e1);
  cudaError_t e = cudaDeviceSynchronize();
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  long long h[148];
  int herr = 0;
  cudaMemcpy(h, cyc, grid * 8, cudaMemcpyDeviceToHost);
  cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
  double avg = 0;
  for (int i = 0; i < grid; ++i) avg += h[i];
  avg /= grid;
  const double bytes = (double)grid * T * kTile;
  printf("heads=%2d NS=%d grid=%3d ntiles=%5d err=%d/%d  %.3f ms  %.1f TB/s total  %.1f B/clk/SM  %.0f clk/tile\n", heads,
         NS, grid, ntiles, (int)e, herr, ms, bytes / (ms * 1e9), (double)T * kTile / avg, avg / T);
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
  CUresult r = fn(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, buf, gdim, gstride, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    printf("encode failed %d\n", (int)r);
    return 1;
  }
  const int T = 3000, nt = 222;  // one head's K and V columns over 28416 rows: 14.6 MB
  run<1>(tm, T, nt, 148);
  run<2>(tm, T, nt, 148);
  run<3>(tm, T, nt, 148);
  run<4>(tm, T, nt, 148);
  run<6>(tm, T, nt, 148);
  run<1>(tm, T, nt, 148, 24);
  run<2>(tm, T, nt, 148, 24);
  run<4>(tm, T, nt, 148, 24);
  run<6>(tm, T, nt, 148, 24);
  return 0;
}
