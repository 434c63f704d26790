// 1-D reductions and dot products (HBM-bound).
//
// Reference semantics:
//   linalg.dot: 0-D accumulator filled with 0, then sum of a[i]*b[i]
//     (cpp/src/builders/LinalgBuilder.cpp:66-104);
//   linalg.reduce with a user body, folded from a user init
//     (cpp/src/builders/LinalgBuilder.cpp:241-279); the library's bodies are
//     tensor_sum (acc + elem, init 0), tensor_max / tensor_min
//     (If(elem > acc, elem, acc) / If(elem < acc, elem, acc), init -inf/+inf)
//     (mlir_edsl/ops/linalg.py:104-175) and a product body (acc * elem).
//
// Two passes, deterministic: pass 1 has each of up to kMaxBlocks blocks fold a
// contiguous range of the input (16-byte loads, 4 in flight) into one
// partial; pass 2 (one block) folds the partials in block order and finally
// combines the init as the first operand, as the sequential fold does. The
// max/min combine keeps the left (earlier) operand unless the right one is
// strictly greater/smaller, so NaN elements never win and the result equals
// the sequential fold's (up to the sign of a zero when +0 and -0 tie).
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>
#include <cstring>
#include "kernels.h"

namespace b200 {

constexpr int kRedThreads = 256;
constexpr int kMaxBlocks = 148 * 8;

template <class T>
struct Ops;

template <>
struct Ops<float> {
  static __device__ __forceinline__ float identity(int op) {
    const float inf = __int_as_float(0x7f800000);
    return op == kRedSum ? 0.0f : op == kRedProd ? 1.0f : op == kRedMax ? -inf : inf;
  }
  // acc is the earlier operand
  static __device__ __forceinline__ float mul(float a, float b) { return a * b; }
  static __device__ __forceinline__ float combine(int op, float acc, float x) {
    switch (op) {
      case kRedSum: return acc + x;
      case kRedProd: return acc * x;
      case kRedMax: return x > acc ? x : acc;
      default: return x < acc ? x : acc;
    }
  }
};

template <>
struct Ops<int32_t> {
  static __device__ __forceinline__ int32_t identity(int op) {
    return op == kRedSum ? 0 : op == kRedProd ? 1 : op == kRedMax ? INT32_MIN : INT32_MAX;
  }
  static __device__ __forceinline__ int32_t mul(int32_t a, int32_t b) {
    return (int32_t)((uint32_t)a * (uint32_t)b);
  }
  static __device__ __forceinline__ int32_t combine(int op, int32_t acc, int32_t x) {
    switch (op) {  // sums and products wrap modulo 2^32
      case kRedSum: return (int32_t)((uint32_t)acc + (uint32_t)x);
      case kRedProd: return (int32_t)((uint32_t)acc * (uint32_t)x);
      case kRedMax: return x > acc ? x : acc;
      default: return x < acc ? x : acc;
    }
  }
};

// Block-wide ordered tree: value of lane/thread i is combined as the left
// operand with that of i + offset.
template <class T>
__device__ __forceinline__ T block_fold(int op, T v) {
  __shared__ T sh[kRedThreads / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const T o = __shfl_down_sync(0xffffffffu, v, off);
    if (lane + off < 32) v = Ops<T>::combine(op, v, o);
  }
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  if (wid == 0) {
    v = lane < kRedThreads / 32 ? sh[lane] : Ops<T>::identity(op);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const T o = __shfl_down_sync(0xffffffffu, v, off);
      if (lane + off < 32) v = Ops<T>::combine(op, v, o);
    }
  }
  return v;
}

// Pass 1. Block b folds elements [b*chunk, min(n, (b+1)*chunk)). Inside the
// block, each thread folds its elements in index order: with 16-byte aligned
// inputs and chunk a multiple of 4, thread t takes 4-element groups t,
// t+256, ... (four 16-byte loads in flight per iteration), then the ragged
// tail element-wise. With `y` non-null the element is x[i]*y[i] (dot, sum).
template <class T>
__device__ __forceinline__ T fold4(int op, T acc, const T (&v)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) acc = Ops<T>::combine(op, acc, v[j]);
  return acc;
}

template <class T>
__global__ void __launch_bounds__(kRedThreads)
    reduce_pass1(const T* __restrict__ x, const T* __restrict__ y, int64_t n, int64_t chunk,
                 int op, int vec, T* __restrict__ partials) {
  const int64_t lo = (int64_t)blockIdx.x * chunk;
  const int64_t hi = min(n, lo + chunk);
  T acc = Ops<T>::identity(op);
  int64_t tail = lo;
  if (vec) {
    using V = int4;  // 16 bytes of T
    const int64_t ng = (hi - lo) >> 2;  // whole groups of 4
    const V* xv = reinterpret_cast<const V*>(x + lo);
    const V* yv = y ? reinterpret_cast<const V*>(y + lo) : nullptr;
    int64_t g = threadIdx.x;
    for (; g + 3 * kRedThreads < ng; g += 4 * kRedThreads) {
      V a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = __ldg(xv + g + u * kRedThreads);
      if (yv) {
#pragma unroll
        for (int u = 0; u < 4; ++u) b[u] = __ldg(yv + g + u * kRedThreads);
      }
      // fold groups g, g+256, g+512, g+768: this thread's groups in index order
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        T v[4];
        memcpy(v, &a[u], 16);
        if (yv) {
          T w[4];
          memcpy(w, &b[u], 16);
#pragma unroll
          for (int j = 0; j < 4; ++j) v[j] = Ops<T>::mul(v[j], w[j]);
        }
        acc = fold4<T>(op, acc, v);
      }
    }
    for (; g < ng; g += kRedThreads) {
      T v[4];
      const V a = __ldg(xv + g);
      memcpy(v, &a, 16);
      if (yv) {
        T w[4];
        const V b = __ldg(yv + g);
        memcpy(w, &b, 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = Ops<T>::mul(v[j], w[j]);
      }
      acc = fold4<T>(op, acc, v);
    }
    tail = lo + (ng << 2);
  }
  for (int64_t i = tail + threadIdx.x; i < hi; i += kRedThreads) {
    T v = __ldg(x + i);
    if (y) v = Ops<T>::mul(v, __ldg(y + i));  // rounded product, then the add
    acc = Ops<T>::combine(op, acc, v);
  }
  acc = block_fold<T>(op, acc);
  if (threadIdx.x == 0) partials[blockIdx.x] = acc;
}

// Pass 2 (one block): fold the partials in order, then out = init (op) total.
template <class T>
__global__ void __launch_bounds__(kRedThreads)
    reduce_pass2(const T* __restrict__ partials, int nparts, int op, T init, T* __restrict__ out) {
  // Thread t folds a contiguous run of partials so the order is preserved.
  const int per = (nparts + kRedThreads - 1) / kRedThreads;
  const int lo = threadIdx.x * per, hi = min(nparts, lo + per);
  T acc = Ops<T>::identity(op);
  for (int i = lo; i < hi; ++i) acc = Ops<T>::combine(op, acc, partials[i]);
  acc = block_fold<T>(op, acc);
  if (threadIdx.x == 0) out[0] = Ops<T>::combine(op, init, acc);
}

int64_t reduce_scratch_bytes() { return (int64_t)kMaxBlocks * 8; }

template <class T>
static int reduce_impl(const T* x, const T* y, int64_t n, int op, T init, T* out, void* scratch,
                       cudaStream_t st) {
  int64_t blocks = std::min<int64_t>(kMaxBlocks, std::max<int64_t>(1, (n + 4095) / 4096));
  int64_t chunk = std::max<int64_t>(1, (n + blocks - 1) / blocks);
  const int vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (vec) chunk = (chunk + 3) & ~int64_t(3);  // groups of 4 never straddle blocks
  blocks = std::max<int64_t>(1, (n + chunk - 1) / chunk);
  T* partials = static_cast<T*>(scratch);
  reduce_pass1<T><<<(unsigned)blocks, kRedThreads, 0, st>>>(x, y, n, chunk, op, vec, partials);
  count_launch();
  reduce_pass2<T><<<1, kRedThreads, 0, st>>>(partials, (int)blocks, op, init, out);
  count_launch();
  return launch_result();
}

int reduce_f32(const float* x, const float* y, int64_t n, int op, float init, float* out,
               void* scratch, cudaStream_t st) {
  return reduce_impl<float>(x, y, n, op, init, out, scratch, st);
}

int reduce_i32(const int32_t* x, const int32_t* y, int64_t n, int op, int32_t init, int32_t* out,
               void* scratch, cudaStream_t st) {
  return reduce_impl<int32_t>(x, y, n, op, init, out, scratch, st);
}

}  // namespace b200
