// Probe: MUFU ex2 throughput, f32 vs bf16x2 vs f16x2 (all SMs, 8 warps per SM).
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

template <int MODE>
__global__ void __launch_bounds__(256, 1) k(int iters, float* out, long long* cyc) {
  float a0 = threadIdx.x * 1e-3f - 3.f, a1 = a0 - 0.5f, a2 = a0 - 1.f, a3 = a0 - 1.5f;
  uint32_t b0 = 0x3f00bf00u ^ threadIdx.x, b1 = b0 + 7, b2 = b0 + 13, b3 = b0 + 29;
  long long t0 = clock64();
  for (int i = 0; i < iters; ++i) {
    if (MODE == 0) {
      asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(a0));
      asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(a1));
      asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(a2));
      asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(a3));
    } else if (MODE == 1) {
      asm volatile("ex2.approx.ftz.bf16x2 %0, %0;" : "+r"(b0));
      asm volatile("ex2.approx.ftz.bf16x2 %0, %0;" : "+r"(b1));
      asm volatile("ex2.approx.ftz.bf16x2 %0, %0;" : "+r"(b2));
      asm volatile("ex2.approx.ftz.bf16x2 %0, %0;" : "+r"(b3));
    } else {
      asm volatile("ex2.approx.f16x2 %0, %0;" : "+r"(b0));
      asm volatile("ex2.approx.f16x2 %0, %0;" : "+r"(b1));
      asm volatile("ex2.approx.f16x2 %0, %0;" : "+r"(b2));
      asm volatile("ex2.approx.f16x2 %0, %0;" : "+r"(b3));
    }
  }
  long long t1 = clock64();
  if (threadIdx.x == 0) cyc[blockIdx.x] = t1 - t0;
  if (a0 + a1 + a2 + a3 == 1234.5f || (b0 ^ b1 ^ b2 ^ b3) == 0x12345678u) out[threadIdx.x] = a0 + (float)b0;
}

template <int MODE>
void run(const char* name) {
  float* out;
  long long* cyc;
  cudaMalloc(&out, 4096);
  cudaMalloc(&cyc, 148 * 8);
  const int iters = 20000;
  k<MODE><<<148, 256>>>(iters, out, cyc);
  cudaDeviceSynchronize();
  long long h[148];
  cudaMemcpy(h, cyc, sizeof(h), cudaMemcpyDeviceToHost);
  double avg = 0;
  for (int i = 0; i < 148; ++i) avg += h[i];
  avg /= 148;
  // per SM: 8 warps x iters x 4 instructions
  const double instr = 8.0 * iters * 4;
  const double elems = instr * 32 * (MODE == 0 ? 1 : 2);
  printf("%-10s err=%d  %.2f clk per warp-instr per SM, %.1f results/clk/SM\n", name, (int)cudaGetLastError(),
         avg / instr, elems / avg);
  cudaFree(out);
  cudaFree(cyc);
}

int main() {
  run<0>("f32");
  run<1>("bf16x2");
  run<2>("f16x2");
  return 0;
}
