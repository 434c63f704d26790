// Allocation-free variant of the f32 dense layer (b200_dense_f32_noalloc).
//
// The regular entry points take the scratch for the tf32 hi/lo operand split
// from cudaMalloc'd buffers. Some callers must not allocate device memory
// while they run: a serving process whose deep-learning framework's caching
// allocator has already reserved nearly all of HBM (a direct cudaMalloc then
// fails or forces that allocator to give back its cache), or a latency-bound
// loop that cannot absorb the device-wide synchronisation cudaMalloc/cudaFree
// imply. For them this file provides the same computation with its scratch in
// a fixed, file-scope device array, so the call itself allocates nothing.
//
// Cost and limits:
//   * every GPU that loads this library holds kNoAllocScratchBytes (64 MiB)
//     of device memory for the array until the process exits;
//   * a problem fits when 8 * (M + N) * roundup(K, 8) bytes (plus 256-byte
//     alignment of the four split regions) is at most 64 MiB, e.g.
//     M = N = K = 2040; larger problems are rejected with B200_ERR_TOO_LARGE;
//   * all calls on a device share the one array and it keeps the last
//     call's contents, so calls that overlap on the GPU (two host threads, or
//     two streams) race and corrupt each other's results. The entry point
//     synchronises its stream before returning, which serialises calls made
//     from one host thread.
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress with that device current); make that first call
//     before any stream capture.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include "../../include/b200_edsl.h"
#include "kernels.h"

namespace b200 {
namespace {

constexpr int64_t kNoAllocScratchBytes = (int64_t)64 << 20;  // 64 MiB per device

// Scratch for the four split operands (X hi/lo, W^T hi/lo) and the status
// word the GEMM kernel sets when a bounded wait gives up. In host code these
// names are host-side stand-ins, not device addresses: the device addresses
// come from cudaGetSymbolAddress in setup_device().
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ int g_noalloc_status;

struct DeviceAddrs {
  unsigned char* scratch = nullptr;
  int* status = nullptr;
};

std::mutex g_setup_mu;
DeviceAddrs g_addrs[64];

// Once per device, with that device current: resolve the device addresses.
int setup_device(int dev, DeviceAddrs* out) {
  if (dev < 0 || dev >= 64) return report_error(kErrInvalidArg, "device index out of range");
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_addrs[dev].scratch == nullptr) {
    void* scratch = nullptr;
    void* status = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      char buf[160];
      snprintf(buf, sizeof buf, "cudaGetSymbolAddress(scratch) on device %d: %s", dev,
               cudaGetErrorString(e));
      return report_error(kErrCuda, buf);
    }
    e = cudaGetSymbolAddress(&status, g_noalloc_status);
    if (e != cudaSuccess) {
      cudaGetLastError();
      char buf[160];
      snprintf(buf, sizeof buf, "cudaGetSymbolAddress(status) on device %d: %s", dev,
               cudaGetErrorString(e));
      return report_error(kErrCuda, buf);
    }
    g_addrs[dev].scratch = static_cast<unsigned char*>(scratch);
    g_addrs[dev].status = static_cast<int*>(status);
  }
  *out = g_addrs[dev];
  return kOk;
}

int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

int cuda_error(cudaError_t e, const char* what) {
  cudaGetLastError();
  char buf[200];
  snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
  return report_error(kErrCuda, buf);
}

// A launch step failed: its own status and message. Steps queued before it
// may still be using the shared array, so the stream is drained first (the
// array is free again when the call returns, on every path).
int step_error(int rc, const char* step, cudaStream_t st) {
  char buf[240];
  snprintf(buf, sizeof buf, "b200_dense_f32_noalloc: %s: %s", step, launch_error_text());
  cudaStreamSynchronize(st);
  cudaGetLastError();
  return report_error(rc, buf);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_dense_f32_noalloc(const float* X, int64_t ldx, const float* W, int64_t ldw,
                                      const float* b, float* Y, int64_t ldy, int64_t M, int64_t N,
                                      int64_t K, int act, float alpha, void* stream) {
  if (M < 0 || N < 0 || K < 0) return report_error(kErrInvalidArg, "negative dimension");
  if (act < kActNone || act > kActLeakyRelu)
    return report_error(kErrInvalidArg, "unknown activation");
  if (M == 0 || N == 0) return report_ok();
  if (!Y || ldy < N) return report_error(kErrInvalidArg, "null output or ldy < N");
  if (K > 0 && (!X || !W || ldx < K || ldw < N))
    return report_error(kErrInvalidArg, "null input or pitch too small");
  if (M > ((int64_t)1 << 31) || N > ((int64_t)1 << 31) || K > ((int64_t)1 << 31))
    return report_error(kErrTooLarge, "dimension exceeds 2^31");

  int n_dev = 0;
  if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0) {
    cudaGetLastError();
    return report_error(kErrNoDevice, "no CUDA device available");
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  DeviceAddrs addr;
  int rc = setup_device(dev, &addr);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  if (K > 0) {
    const int64_t Kp = split_pitch(K);
    const int64_t need = dense_f32_workspace_bytes(M, N, K);
    if (need > kNoAllocScratchBytes) {
      char buf[240];
      snprintf(buf, sizeof buf,
               "b200_dense_f32_noalloc: %lld x %lld x %lld needs %lld bytes of scratch, more than "
               "the fixed %lld-byte array; use b200_dense_f32 or b200_dense_f32_ws",
               (long long)M, (long long)N, (long long)K, (long long)need,
               (long long)kNoAllocScratchBytes);
      return report_error(kErrTooLarge, buf);
    }
    // Carve the four split operands; each region starts 256-byte aligned.
    unsigned char* p = addr.scratch;
    float* xhi = reinterpret_cast<float*>(p);
    p += align256(M * Kp * 4);
    float* xlo = reinterpret_cast<float*>(p);
    p += align256(M * Kp * 4);
    float* whi = reinterpret_cast<float*>(p);
    p += align256(N * Kp * 4);
    float* wlo = reinterpret_cast<float*>(p);
    // The status word must start at zero; the split regions are fully
    // rewritten (padding columns included) before the GEMM reads them.
    e = cudaMemsetAsync(addr.status, 0, sizeof(int), st);
    if (e != cudaSuccess) return cuda_error(e, "clear status");
    const char* step = "split of W";
    rc = split_w_f32(W, ldw, K, N, whi, wlo, st);
    if (rc == kOk) {
      step = "split of X";
      rc = split_x_f32(X, ldx, M, K, xhi, xlo, st);
    }
    if (rc == kOk) {
      step = "GEMM";
      rc = gemm_tf32x3_presplit(xhi, xlo, whi, wlo, M, N, K, b, Y, ldy, act, alpha, addr.status,
                                st);
    }
    if (rc) return step_error(rc, step, st);
  } else {
    rc = fill_bias_act_f32(b, Y, ldy, M, N, act, alpha, st);
    if (rc) return step_error(rc, "bias fill", st);
  }

  // Synchronous: the shared scratch is free again when the call returns.
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_error(e, "stream synchronize");
  if (K > 0) {
    int h = 0;
    e = cudaMemcpyAsync(&h, addr.status, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_error(e, "status read");
    if (h != 0)
      return report_error(kErrDeviceTimeout,
                          "b200_dense_f32_noalloc: a kernel gave up a bounded wait; results are "
                          "invalid");
  }
  return report_ok();
}
