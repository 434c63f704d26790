// Microbenchmark of the CUDA-core INT32 multiply-add rate, the roofline of
// the i32 GEMM (NVIDIA publishes no INT32 IMAD figure for B200). Built into
// its own library (lib/libb200probe.so); used by bench.py --configs only.
//
// Each thread runs 8 independent chains acc_j = acc_j * x + y (32-bit
// multiply-add, wrap-around), so the dependency latency is hidden and the
// issue rate of the integer pipe is measured. The results are stored so
// the work cannot be removed.
#include <cuda_runtime.h>
#include <cstdint>

__global__ void __launch_bounds__(256) imad_chains(uint32_t x, uint32_t y, int iters,
                                                   uint32_t* out) {
  uint32_t a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = threadIdx.x + j * 7919u + blockIdx.x;
#pragma unroll 1
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int r = 0; r < 16; ++r) {
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = a[j] * x + y;
    }
  }
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) s ^= a[j];
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// Launches `blocks` x 256 threads, each doing iters * 128 multiply-adds;
// returns the elapsed milliseconds (CUDA events) or a negative value on error.
extern "C" float b200_probe_imad(int blocks, int iters, uint32_t* out) {
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) return -1.0f;
  imad_chains<<<blocks, 256>>>(3u, 1u, iters, out);  // warm-up
  cudaEventRecord(e0);
  imad_chains<<<blocks, 256>>>(3u, 1u, iters, out);
  cudaEventRecord(e1);
  cudaEventSynchronize(e1);
  float ms = -1.0f;
  if (cudaGetLastError() == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return ms;
}
