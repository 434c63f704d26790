// HBM-bound elementwise kernels for the unfused uses of the dense-layer ops:
//   bias add  Y[m,n] = X[m,n] + b[n]           (reference: linalg.generic
//             "bias_add", cpp/src/builders/LinalgBuilder.cpp:301-339)
//   relu      arith.maximumf(x, 0)             (:213-215)
//   leaky     maximumf(x,0) + alpha*minimumf(x,0)  (:216-225)
// and the K = 0 case of the dense layer (output = act(bias)).
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>
#include "kernels.h"

namespace b200 {

__device__ __forceinline__ float ew_act(float x, int act, float alpha) {
  if (act == kActRelu) return (x > 0.0f || x != x) ? x : 0.0f;
  if (act == kActLeakyRelu) {
    const float pos = (x > 0.0f || x != x) ? x : 0.0f;
    const float neg = (x < 0.0f || x != x) ? x : 0.0f;
    return pos + neg * alpha;
  }
  return x;
}

static int grid_for(int64_t work) {
  int64_t b = (work + 255) / 256;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, 148 * 32));
}

// One thread per 4 consecutive columns when rows are 16-byte aligned.
__global__ void bias_act_f32_vec_kernel(const float* __restrict__ X, int64_t ldx,
                                        const float* __restrict__ b, float* __restrict__ Y,
                                        int64_t ldy, int64_t M, int64_t N, int act, float alpha) {
  const int64_t q = N >> 2;
  const int64_t total = M * q;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / q, n = (i - m * q) << 2;
    float4 x = __ldg(reinterpret_cast<const float4*>(X + m * ldx + n));
    if (b) {
      const float4 bb = __ldg(reinterpret_cast<const float4*>(b + n));
      x.x += bb.x; x.y += bb.y; x.z += bb.z; x.w += bb.w;
    }
    x.x = ew_act(x.x, act, alpha);
    x.y = ew_act(x.y, act, alpha);
    x.z = ew_act(x.z, act, alpha);
    x.w = ew_act(x.w, act, alpha);
    *reinterpret_cast<float4*>(Y + m * ldy + n) = x;
  }
}

__global__ void bias_act_f32_kernel(const float* __restrict__ X, int64_t ldx,
                                    const float* __restrict__ b, float* __restrict__ Y,
                                    int64_t ldy, int64_t M, int64_t N, int act, float alpha) {
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float x = X ? X[m * ldx + n] : 0.0f;
    if (b) x += b[n];
    Y[m * ldy + n] = ew_act(x, act, alpha);
  }
}

__global__ void act_f32_kernel(const float* __restrict__ X, float* __restrict__ Y, int64_t count,
                               int act, float alpha, int vec) {
  if (vec) {
    const int64_t q = count >> 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < q;
         i += (int64_t)gridDim.x * blockDim.x) {
      float4 x = __ldg(reinterpret_cast<const float4*>(X) + i);
      x.x = ew_act(x.x, act, alpha);
      x.y = ew_act(x.y, act, alpha);
      x.z = ew_act(x.z, act, alpha);
      x.w = ew_act(x.w, act, alpha);
      reinterpret_cast<float4*>(Y)[i] = x;
    }
    // tail
    for (int64_t i = (q << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x)
      Y[i] = ew_act(X[i], act, alpha);
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x)
      Y[i] = ew_act(X[i], act, alpha);
  }
}

__global__ void bias_add_i32_kernel(const int32_t* __restrict__ X, int64_t ldx,
                                    const int32_t* __restrict__ b, int32_t* __restrict__ Y,
                                    int64_t ldy, int64_t M, int64_t N) {
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    Y[m * ldy + n] = (int32_t)((uint32_t)X[m * ldx + n] + (uint32_t)b[n]);
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int bias_act_f32(const float* X, int64_t ldx, const float* b, float* Y, int64_t ldy, int64_t M,
                 int64_t N, int act, float alpha, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return kOk;
  const bool vec = X && (N % 4 == 0) && (ldx % 4 == 0) && (ldy % 4 == 0) && al16(X) && al16(Y) &&
                   (!b || al16(b));
  if (vec)
    bias_act_f32_vec_kernel<<<grid_for(M * N / 4), 256, 0, stream>>>(X, ldx, b, Y, ldy, M, N, act,
                                                                     alpha);
  else
    bias_act_f32_kernel<<<grid_for(M * N), 256, 0, stream>>>(X, ldx, b, Y, ldy, M, N, act, alpha);
  count_launch();
  return launch_result();
}

int fill_bias_act_f32(const float* b, float* Y, int64_t ldy, int64_t M, int64_t N, int act,
                      float alpha, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return kOk;
  bias_act_f32_kernel<<<grid_for(M * N), 256, 0, stream>>>(nullptr, 0, b, Y, ldy, M, N, act,
                                                           alpha);
  count_launch();
  return launch_result();
}

int act_f32(const float* X, float* Y, int64_t count, int act, float alpha, cudaStream_t stream) {
  if (count <= 0) return kOk;
  const int vec = al16(X) && al16(Y);
  act_f32_kernel<<<grid_for(vec ? count / 4 + 1 : count), 256, 0, stream>>>(X, Y, count, act,
                                                                            alpha, vec);
  count_launch();
  return launch_result();
}

int bias_add_i32(const int32_t* X, int64_t ldx, const int32_t* b, int32_t* Y, int64_t ldy,
                 int64_t M, int64_t N, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return kOk;
  bias_add_i32_kernel<<<grid_for(M * N), 256, 0, stream>>>(X, ldx, b, Y, ldy, M, N);
  count_launch();
  return launch_result();
}

}  // namespace b200
