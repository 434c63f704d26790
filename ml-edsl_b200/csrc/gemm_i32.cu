// i32 GEMM on the CUDA cores with wrap-around (mod 2^32) arithmetic.
//
// Reference semantics: linalg.fill(0) + linalg.matmul on i32 tensors lower to
// arith.muli / arith.addi, which wrap modulo 2^32
// (cpp/src/builders/LinalgBuilder.cpp:106-139; tested exactly at
// tests/linalg/test_matmul_execution.py:93-103). The products and sums are
// done on uint32_t so that wrap-around is defined behaviour; the bits equal
// the signed two's-complement result.
//
// Tiling: 128 x 128 output tile per 256-thread CTA, 16-deep k-slabs double
// buffered in shared memory, 8 x 8 outputs per thread (two 4-row by two
// 4-column quadrants so shared-memory reads are 16-byte vectors).
#include <cuda_runtime.h>
#include <cstdint>
#include "kernels.h"

namespace b200 {

constexpr int kIBM = 128, kIBN = 128, kIBK = 16;

__global__ void __launch_bounds__(256, 2)  // two CTAs per SM (<= 128 registers)
    gemm_i32_kernel(const int32_t* __restrict__ A, int64_t lda, const int32_t* __restrict__ B,
                    int64_t ldb, int32_t* __restrict__ C, int64_t ldc, int64_t M, int64_t N,
                    int64_t K, const int32_t* __restrict__ bias) {
  __shared__ __align__(16) uint32_t As[2][kIBK][kIBM];
  __shared__ __align__(16) uint32_t Bs[2][kIBK][kIBN];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * kIBM;
  const int64_t n0 = (int64_t)blockIdx.x * kIBN;

  // Global -> register staging: A tile 128x16 (8 per thread: row tid/2, 8
  // consecutive k), B tile 16x128 (8 per thread: k row tid/16, 8 consecutive n).
  const int a_row = tid >> 1, a_k = (tid & 1) * 8;
  const int b_k = tid >> 4, b_col = (tid & 15) * 8;
  uint32_t ra[8], rb[8];

  // 16-byte global loads when the rows are 16-byte aligned and in range.
  const bool vec_a = ((lda & 3) == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0);
  const bool vec_b = ((ldb & 3) == 0) && ((reinterpret_cast<uintptr_t>(B) & 15) == 0);
  auto load_tiles = [&](int64_t k0) {
    const int64_t gm = m0 + a_row;
    const int64_t ga = k0 + a_k;
    if (vec_a && gm < M && ga + 8 <= K) {
      const uint4 u0 = __ldg(reinterpret_cast<const uint4*>(A + gm * lda + ga));
      const uint4 u1 = __ldg(reinterpret_cast<const uint4*>(A + gm * lda + ga + 4));
      ra[0] = u0.x; ra[1] = u0.y; ra[2] = u0.z; ra[3] = u0.w;
      ra[4] = u1.x; ra[5] = u1.y; ra[6] = u1.z; ra[7] = u1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t gk = ga + j;
        ra[j] = (gm < M && gk < K) ? (uint32_t)__ldg(A + gm * lda + gk) : 0u;
      }
    }
    const int64_t gk = k0 + b_k;
    const int64_t gn0 = n0 + b_col;
    if (vec_b && gk < K && gn0 + 8 <= N) {
      const uint4 u0 = __ldg(reinterpret_cast<const uint4*>(B + gk * ldb + gn0));
      const uint4 u1 = __ldg(reinterpret_cast<const uint4*>(B + gk * ldb + gn0 + 4));
      rb[0] = u0.x; rb[1] = u0.y; rb[2] = u0.z; rb[3] = u0.w;
      rb[4] = u1.x; rb[5] = u1.y; rb[6] = u1.z; rb[7] = u1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t gn = gn0 + j;
        rb[j] = (gk < K && gn < N) ? (uint32_t)__ldg(B + gk * ldb + gn) : 0u;
      }
    }
  };
  auto store_tiles = [&](int buf) {
#pragma unroll
    for (int j = 0; j < 8; ++j) As[buf][a_k + j][a_row] = ra[j];
    *reinterpret_cast<uint4*>(&Bs[buf][b_k][b_col]) = make_uint4(rb[0], rb[1], rb[2], rb[3]);
    *reinterpret_cast<uint4*>(&Bs[buf][b_k][b_col + 4]) = make_uint4(rb[4], rb[5], rb[6], rb[7]);
  };

  uint32_t acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0u;

  const int64_t nk = (K + kIBK - 1) / kIBK;
  load_tiles(0);
  store_tiles(0);
  __syncthreads();
  for (int64_t t = 0; t < nk; ++t) {
    const int buf = (int)(t & 1);
    if (t + 1 < nk) load_tiles((t + 1) * kIBK);
#pragma unroll
    for (int k = 0; k < kIBK; ++k) {
      uint32_t a[8], b[8];
      const uint4 a0 = *reinterpret_cast<const uint4*>(&As[buf][k][ty * 4]);
      const uint4 a1 = *reinterpret_cast<const uint4*>(&As[buf][k][64 + ty * 4]);
      const uint4 b0 = *reinterpret_cast<const uint4*>(&Bs[buf][k][tx * 4]);
      const uint4 b1 = *reinterpret_cast<const uint4*>(&Bs[buf][k][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] += a[i] * b[j];
    }
    if (t + 1 < nk) {
      store_tiles(buf ^ 1);
      __syncthreads();
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn < N) {
        uint32_t v = acc[i][j];
        if (bias) v += (uint32_t)bias[gn];
        C[gm * ldc + gn] = (int32_t)v;
      }
    }
  }
}

int gemm_i32(const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb, int32_t* C,
             int64_t ldc, int64_t M, int64_t N, int64_t K, const int32_t* bias,
             cudaStream_t stream) {
  dim3 grid((unsigned)((N + kIBN - 1) / kIBN), (unsigned)((M + kIBM - 1) / kIBM));
  gemm_i32_kernel<<<grid, 256, 0, stream>>>(A, lda, B, ldb, C, ldc, M, N, K, bias);
  count_launch();
  return launch_result();
}

}  // namespace b200
