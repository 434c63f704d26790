// Host runtime behind include/b200_edsl.h.
//
// Owns, per device: three streams (compute, host->device, device->host), a
// device status word that kernels set when a bounded wait gives up, grow-only
// device buffers for host-pointer calls, and per-stream scratch for the
// device-pointer calls. Replaces the reference's GPU executor, which
// allocated, copied, launched with a full context synchronize after every
// kernel, copied back and freed on each call
// (reference: cpp/src/MLIRExecutor.cpp:187-238, cpp/src/MLIRCompiler.cpp:352-461).
#include <cuda_runtime.h>
#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>
#include "../../include/b200_edsl.h"
#include "kernels.h"

namespace b200 {

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {

thread_local std::string t_err;
thread_local int t_status = 0;

int fail(int code, const std::string& msg) {
  t_err = msg;
  t_status = code;
  return code;
}
int fail_cuda(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear the non-sticky error
  std::string m = std::string(what) + ": " + cudaGetErrorString(e);
  return fail(e == cudaErrorMemoryAllocation ? kErrOutOfMemory : kErrCuda, m);
}
int succeed() {
  t_status = kOk;
  return kOk;
}

#define B200_CUDA(call, what)                    \
  do {                                           \
    cudaError_t e_ = (call);                     \
    if (e_ != cudaSuccess) return fail_cuda(e_, what); \
  } while (0)

// Host-side fault injection: when > 0, the n-th next device allocation made
// by the runtime fails with cudaErrorMemoryAllocation (b200_debug_fail_alloc).
std::atomic<int> g_fail_alloc_in{0};

struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  // Ensures capacity >= need. The caller guarantees no in-flight work uses it.
  cudaError_t reserve(size_t need) {
    if (need <= n) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    const int k = g_fail_alloc_in.load();
    if (k > 0 && g_fail_alloc_in.fetch_sub(1) == 1) return cudaErrorMemoryAllocation;
    cudaError_t e = cudaMalloc(&p, need);
    if (e == cudaSuccess) n = need;
    return e;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
};

constexpr int kRing = 3;  // slab buffers in flight per device

// Scratch of the device-pointer calls on one (device, stream). Its mutex is
// held from the size check until the call has queued every kernel that uses
// the buffer, so a second host thread on the same stream can neither free it
// (growth) nor hand it out while the first is still enqueueing.
struct StreamScratch {
  std::mutex mu;
  DevBuf buf;
};

// Grow-only page-locked host buffer (staging for pageable user memory).
struct PinnedBuf {
  void* p = nullptr;
  size_t n = 0;
  cudaError_t reserve(size_t need) {
    if (need <= n) return cudaSuccess;
    if (p) cudaFreeHost(p);
    p = nullptr;
    n = 0;
    cudaError_t e = cudaHostAlloc(&p, need, cudaHostAllocPortable);
    if (e == cudaSuccess) n = need;
    return e;
  }
  void release() {
    if (p) cudaFreeHost(p);
    p = nullptr;
    n = 0;
  }
};

// Small persistent pool of host threads for parallel row copies between
// pageable user memory and the pinned staging buffers.
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool pool;
    return pool;
  }
  // Runs fn(t) for t in [0, nthreads()) and waits for all of them. Calls
  // from several host threads (one per device) take turns: one job at a time.
  template <class Fn>
  void run(Fn fn) {
    std::lock_guard<std::mutex> one_job(run_mu_);
    std::unique_lock<std::mutex> lk(mu_);
    job_ = [&fn](int t) { fn(t); };
    pending_ = (int)workers_.size();
    ++gen_;
    cv_.notify_all();
    lk.unlock();
    fn((int)workers_.size());  // the caller is the last participant
    lk.lock();
    done_cv_.wait(lk, [&] { return pending_ == 0; });
  }
  int nthreads() const { return (int)workers_.size() + 1; }

 private:
  CopyPool() {
    // B200_COPY_THREADS overrides the thread count (default: half the
    // hardware threads, at most 8).
    unsigned hw = std::thread::hardware_concurrency();
    int want = (int)std::max(1u, std::min(8u, hw / 2));
    if (const char* e = getenv("B200_COPY_THREADS")) want = std::max(1, std::min(64, atoi(e)));
    const int n = want - 1;
    for (int i = 0; i < n; ++i) workers_.emplace_back([this, i] { loop(i); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  void loop(int id) {
    uint64_t seen = 0;
    while (true) {
      std::function<void(int)> job;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        if (stop_) return;
        job = job_;
      }
      job(id);
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_cv_.notify_all();
    }
  }
  std::vector<std::thread> workers_;
  std::mutex run_mu_;  // serialises run()
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::function<void(int)> job_;
  int pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

// rows x row_bytes copy between two pitched host buffers, split over the pool.
void par_copy_rows(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t row_bytes,
                   int64_t rows) {
  CopyPool& pool = CopyPool::get();
  const int T = pool.nthreads();
  pool.run([&](int t) {
    const int64_t r0 = rows * t / T, r1 = rows * (t + 1) / T;
    char* d = static_cast<char*>(dst) + r0 * dpitch;
    const char* sp = static_cast<const char*>(src) + r0 * spitch;
    if (dpitch == row_bytes && spitch == row_bytes) {
      memcpy(d, sp, (size_t)((r1 - r0) * row_bytes));
    } else {
      for (int64_t r = r0; r < r1; ++r, d += dpitch, sp += spitch) memcpy(d, sp, row_bytes);
    }
  });
}

// True for ordinary (not page-locked, not device) host memory.
bool is_pageable(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type == cudaMemoryTypeUnregistered;
}

struct DeviceCtx {
  int dev = -1;
  std::mutex mu;  // one host-pointer call per device at a time
  bool ready = false;
  cudaStream_t s_comp = nullptr, s_h2d = nullptr, s_d2h = nullptr;
  int* status = nullptr;  // device word written by timed-out kernels
  // host-pointer call buffers
  DevBuf w, whi, wlo, bias;
  DevBuf x[kRing], xhi[kRing], xlo[kRing], y[kRing], part[kRing];
  PinnedBuf sx[kRing], sy[kRing];  // staging for pageable X / Y slabs
  PinnedBuf sc[2];                 // chunk staging for other pageable copies
  cudaEvent_t ev_h2d[kRing], ev_comp[kRing], ev_d2h[kRing], ev_sc[2];
  // device-pointer call scratch, keyed by stream (entries are never erased:
  // a lease may hold a pointer to one while another thread releases buffers)
  std::map<cudaStream_t, std::unique_ptr<StreamScratch>> scratch;
};

std::mutex g_mu;
DeviceCtx g_dev[64];
int g_default_devices = -1;

int device_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Returns the initialised context of `dev` (caller holds no lock).
int get_ctx(int dev, DeviceCtx** out) {
  if (dev < 0 || dev >= 64) return fail(kErrInvalidArg, "device index out of range");
  DeviceCtx& c = g_dev[dev];
  std::lock_guard<std::mutex> lk(g_mu);
  if (!c.ready) {
    int prev = 0;
    cudaGetDevice(&prev);
    B200_CUDA(cudaSetDevice(dev), "cudaSetDevice");
    B200_CUDA(cudaStreamCreateWithFlags(&c.s_comp, cudaStreamNonBlocking), "cudaStreamCreate");
    B200_CUDA(cudaStreamCreateWithFlags(&c.s_h2d, cudaStreamNonBlocking), "cudaStreamCreate");
    B200_CUDA(cudaStreamCreateWithFlags(&c.s_d2h, cudaStreamNonBlocking), "cudaStreamCreate");
    B200_CUDA(cudaMalloc(&c.status, sizeof(int)), "cudaMalloc(status)");
    B200_CUDA(cudaMemset(c.status, 0, sizeof(int)), "cudaMemset(status)");
    for (int i = 0; i < kRing; ++i) {
      B200_CUDA(cudaEventCreateWithFlags(&c.ev_h2d[i], cudaEventDisableTiming), "event");
      B200_CUDA(cudaEventCreateWithFlags(&c.ev_comp[i], cudaEventDisableTiming), "event");
      B200_CUDA(cudaEventCreateWithFlags(&c.ev_d2h[i], cudaEventDisableTiming), "event");
      if (i < 2) B200_CUDA(cudaEventCreateWithFlags(&c.ev_sc[i], cudaEventDisableTiming), "event");
    }
    c.dev = dev;
    c.ready = true;
    cudaSetDevice(prev);
  }
  *out = &c;
  return kOk;
}

int current_ctx(DeviceCtx** out) {
  if (device_count() == 0) return fail(kErrNoDevice, "no CUDA device available");
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  return get_ctx(dev, out);
}

// Exclusive use of the (device, stream) scratch, at least `need` bytes,
// until the lease goes out of scope. Growing first drains the stream: work
// queued by earlier leases may still read the old buffer.
class ScratchLease {
 public:
  int acquire(DeviceCtx* c, cudaStream_t st, size_t need) {
    StreamScratch* e = nullptr;
    {
      std::lock_guard<std::mutex> g(g_mu);
      auto& slot = c->scratch[st];
      if (!slot) slot.reset(new StreamScratch);
      e = slot.get();
    }
    lk_ = std::unique_lock<std::mutex>(e->mu);
    if (e->buf.n < need) {
      B200_CUDA(cudaStreamSynchronize(st), "sync before scratch growth");
      B200_CUDA(e->buf.reserve(need), "alloc scratch");
    }
    p = e->buf.p;
    return kOk;
  }
  void* p = nullptr;

 private:
  std::unique_lock<std::mutex> lk_;
};

// Pageable copies at least this large go through the pinned staging chunks.
constexpr int64_t kStageMin = (int64_t)16 << 20;
constexpr int64_t kStageChunk = (int64_t)32 << 20;

// rows x row_bytes from pitched host memory to pitched device memory on `st`.
// Pageable sources of kStageMin bytes or more are copied chunk-wise through
// two pinned buffers: the host copy of chunk j (several threads) overlaps the
// DMA of chunk j-1. Returns once the source may be reused; the device copy
// completes in stream order. The caller holds c->mu.
int h2d_rows(DeviceCtx* c, void* dst, int64_t dpitch, const void* src, int64_t spitch,
             int64_t row_bytes, int64_t rows, cudaStream_t st) {
  if (rows <= 0 || row_bytes <= 0) return kOk;
  if (rows * row_bytes < kStageMin || !is_pageable(src)) {
    B200_CUDA(cudaMemcpy2DAsync(dst, dpitch, src, spitch, row_bytes, rows,
                                cudaMemcpyHostToDevice, st),
              "H2D");
    return kOk;
  }
  const int64_t per = std::max<int64_t>(1, kStageChunk / row_bytes);
  for (int i = 0; i < 2; ++i) B200_CUDA(c->sc[i].reserve(per * row_bytes), "pinned staging");
  for (int64_t r0 = 0, j = 0; r0 < rows; r0 += per, ++j) {
    const int slot = (int)(j & 1);
    const int64_t n = std::min(per, rows - r0);
    if (j >= 2) B200_CUDA(cudaEventSynchronize(c->ev_sc[slot]), "staging wait");
    par_copy_rows(c->sc[slot].p, row_bytes, static_cast<const char*>(src) + r0 * spitch, spitch,
                  row_bytes, n);
    B200_CUDA(cudaMemcpy2DAsync(static_cast<char*>(dst) + r0 * dpitch, dpitch, c->sc[slot].p,
                                row_bytes, row_bytes, n, cudaMemcpyHostToDevice, st),
              "H2D");
    B200_CUDA(cudaEventRecord(c->ev_sc[slot], st), "record");
  }
  // both staging buffers must be free before the next staged copy reuses them
  const int64_t nchunk = (rows + per - 1) / per;
  for (int i = 0; i < 2 && i < nchunk; ++i)
    B200_CUDA(cudaEventSynchronize(c->ev_sc[i]), "staging wait");
  return kOk;
}

// The device-to-host counterpart; returns after the host data is complete.
int d2h_rows(DeviceCtx* c, void* dst, int64_t dpitch, const void* src, int64_t spitch,
             int64_t row_bytes, int64_t rows, cudaStream_t st) {
  if (rows <= 0 || row_bytes <= 0) return kOk;
  if (rows * row_bytes < kStageMin || !is_pageable(dst)) {
    B200_CUDA(cudaMemcpy2DAsync(dst, dpitch, src, spitch, row_bytes, rows,
                                cudaMemcpyDeviceToHost, st),
              "D2H");
    B200_CUDA(cudaStreamSynchronize(st), "sync");
    return kOk;
  }
  const int64_t per = std::max<int64_t>(1, kStageChunk / row_bytes);
  for (int i = 0; i < 2; ++i) B200_CUDA(c->sc[i].reserve(per * row_bytes), "pinned staging");
  auto unstage = [&](int64_t j) -> int {
    const int slot = (int)(j & 1);
    const int64_t r0 = j * per, n = std::min(per, rows - r0);
    B200_CUDA(cudaEventSynchronize(c->ev_sc[slot]), "staging wait");
    par_copy_rows(static_cast<char*>(dst) + r0 * dpitch, dpitch, c->sc[slot].p, row_bytes,
                  row_bytes, n);
    return kOk;
  };
  const int64_t nchunk = (rows + per - 1) / per;
  for (int64_t j = 0; j < nchunk; ++j) {
    const int slot = (int)(j & 1);
    const int64_t r0 = j * per, n = std::min(per, rows - r0);
    B200_CUDA(cudaMemcpy2DAsync(c->sc[slot].p, row_bytes,
                                static_cast<const char*>(src) + r0 * spitch, spitch, row_bytes, n,
                                cudaMemcpyDeviceToHost, st),
              "D2H");
    B200_CUDA(cudaEventRecord(c->ev_sc[slot], st), "record");
    if (j >= 1) {
      int rc = unstage(j - 1);
      if (rc) return rc;
    }
  }
  return unstage(nchunk - 1);
}

// Contiguous copies, viewed as rows of one staging chunk plus a tail row.
int h2d_flat(DeviceCtx* c, void* dst, const void* src, int64_t bytes, cudaStream_t st) {
  const int64_t rb = kStageChunk, full = bytes / rb, tail = bytes - full * rb;
  int rc = full ? h2d_rows(c, dst, rb, src, rb, rb, full, st) : kOk;
  if (rc == kOk && tail)
    rc = h2d_rows(c, static_cast<char*>(dst) + full * rb, tail,
                  static_cast<const char*>(src) + full * rb, tail, tail, 1, st);
  return rc;
}
int d2h_flat(DeviceCtx* c, void* dst, const void* src, int64_t bytes, cudaStream_t st) {
  const int64_t rb = kStageChunk, full = bytes / rb, tail = bytes - full * rb;
  int rc = full ? d2h_rows(c, dst, rb, src, rb, rb, full, st) : kOk;
  if (rc == kOk && tail)
    rc = d2h_rows(c, static_cast<char*>(dst) + full * rb, tail,
                  static_cast<const char*>(src) + full * rb, tail, tail, 1, st);
  return rc;
}

// Reads and clears the device status word after the stream has drained.
int check_device_status(DeviceCtx* c) {
  int h = 0;
  B200_CUDA(cudaMemcpy(&h, c->status, sizeof(int), cudaMemcpyDeviceToHost), "status read");
  if (h != 0) {
    cudaMemset(c->status, 0, sizeof(int));
    char buf[160];
    snprintf(buf, sizeof buf,
             "device %d: a kernel gave up a bounded wait (code %d); results are invalid",
             c->dev, h);
    return fail(kErrDeviceTimeout, buf);
  }
  return kOk;
}

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// ------------------------------------------------------------ weight cache
// Registered weights (b200_weights_register): a host W[K, N] the caller
// declares unchanged until it registers it again (with a new version) or
// releases it. On each device a call runs on, the runtime keeps W's device
// copy (rows of N floats, pitch N) and, made on first need, the tf32 split
// the GEMM reads: the row-major lo part for the MN-major B path, or the
// transposed hi / lo parts for the K-major one. Calls that find their W here
// copy and split neither; device-pointer calls are recognised by the device
// copy's address (b200_weights_device).
struct PreSplitW {
  const float* lo_mn = nullptr;  // row-major lo, pitch roundup(N, 4)
  const float* hiT = nullptr;    // K-major hi / lo, pitch split_pitch(K)
  const float* loT = nullptr;
};

struct WeightCopy {
  DevBuf w, lo_mn, hiT, loT;
  bool up = false, have_mn = false, have_k = false;
};

struct WeightEntry {
  int64_t ldw = 0, K = 0, N = 0;
  uint64_t version = 0;
  WeightCopy dev[64];
};

std::mutex g_w_mu;
std::map<const float*, std::unique_ptr<WeightEntry>> g_weights;  // by host address

// The entry registered for host W with this shape and pitch (caller holds g_w_mu).
WeightEntry* find_host_weights(const float* W, int64_t ldw, int64_t K, int64_t N) {
  auto it = g_weights.find(W);
  if (it == g_weights.end()) return nullptr;
  WeightEntry* e = it->second.get();
  return (e->ldw == ldw && e->K == K && e->N == N) ? e : nullptr;
}

// The entry whose copy on device `dev` starts at W (caller holds g_w_mu).
WeightEntry* find_device_weights(int dev, const float* W) {
  for (auto& kv : g_weights)
    if (kv.second->dev[dev].up && kv.second->dev[dev].w.p == W) return kv.second.get();
  return nullptr;
}

// Uploads W to device c->dev if needed and makes the split the call needs
// (MN-major lo when `mn`, else the K-major hi / lo pair). Synchronous on the
// device's compute stream, so the copies are complete for every stream.
// Caller holds g_w_mu.
int weights_ready(DeviceCtx* c, const float* Whost, WeightEntry* e, bool mn, PreSplitW* out,
                  const float** dW) {
  WeightCopy& d = e->dev[c->dev];
  const int64_t K = e->K, N = e->N;
  B200_CUDA(cudaSetDevice(c->dev), "cudaSetDevice");
  if (!d.up) {
    B200_CUDA(d.w.reserve((size_t)std::max<int64_t>(K * N, 1) * 4), "alloc registered W");
    int rc = h2d_rows(c, d.w.p, N * 4, Whost, e->ldw * 4, N * 4, K, c->s_comp);
    if (rc) return rc;
    B200_CUDA(cudaStreamSynchronize(c->s_comp), "sync");
    d.up = true;
  }
  float* w = static_cast<float*>(d.w.p);
  if (mn && !d.have_mn) {
    B200_CUDA(d.lo_mn.reserve((size_t)w_lo_mn_bytes(K, N)), "alloc registered W split");
    int rc = split_lo_xw_f32(nullptr, 0, 0, K, nullptr, nullptr, w, N, N,
                             static_cast<float*>(d.lo_mn.p), c->s_comp);
    if (rc) return fail(rc, std::string("split of registered W: ") + launch_error_text());
    B200_CUDA(cudaStreamSynchronize(c->s_comp), "sync");
    d.have_mn = true;
  }
  if (!mn && !d.have_k) {
    const size_t bytes = (size_t)N * split_pitch(K) * 4;
    B200_CUDA(d.hiT.reserve(bytes), "alloc registered W split");
    B200_CUDA(d.loT.reserve(bytes), "alloc registered W split");
    int rc = split_w_f32(w, N, K, N, static_cast<float*>(d.hiT.p), static_cast<float*>(d.loT.p),
                         c->s_comp);
    if (rc) return fail(rc, std::string("split of registered W: ") + launch_error_text());
    B200_CUDA(cudaStreamSynchronize(c->s_comp), "sync");
    d.have_k = true;
  }
  if (mn) {
    out->lo_mn = static_cast<const float*>(d.lo_mn.p);
  } else {
    out->hiT = static_cast<const float*>(d.hiT.p);
    out->loT = static_cast<const float*>(d.loT.p);
  }
  if (dW) *dW = w;
  return kOk;
}

void release_weight_copy(WeightCopy& d) {
  d.w.release();
  d.lo_mn.release();
  d.hiT.release();
  d.loT.release();
  d.up = d.have_mn = d.have_k = false;
}


bool bad_dims(int64_t M, int64_t N, int64_t K) { return M < 0 || N < 0 || K < 0; }

// Scratch layout inside one workspace block.
struct SplitBufs {
  float *xhi, *xlo, *whi, *wlo;
  float* partials;  // split-K partial sums (only when choose_splits() > 1)
};

// Scratch of the dense device path: split operands + split-K partials.
int64_t dense_scratch_bytes(int64_t M, int64_t N, int64_t K) {
  return dense_f32_workspace_bytes(M, N, K) + splitk_partials_bytes(M, N, K);
}
SplitBufs carve(void* ws, int64_t M, int64_t N, int64_t K) {
  const int64_t Kp = split_pitch(K);
  auto al = [](int64_t b) { return round_up(b, 256); };
  char* p = static_cast<char*>(ws);
  SplitBufs s;
  s.xhi = reinterpret_cast<float*>(p);
  p += al(M * Kp * 4);
  s.xlo = reinterpret_cast<float*>(p);
  p += al(M * Kp * 4);
  s.whi = reinterpret_cast<float*>(p);
  p += al(N * Kp * 4);
  s.wlo = reinterpret_cast<float*>(p);
  p += al(N * Kp * 4);
  s.partials = reinterpret_cast<float*>(p);
  return s;
}

// xlo_in (optional): X's tf32 lo part, pitch split_pitch(K), from the previous
// layer's epilogue (X rows must then be 16-byte aligned: X itself is A_hi),
// so X is not split again. ylo (optional, pitch ldylo): the epilogue also
// writes the lo part of Y for the next layer.
int dense_device(DeviceCtx* c, const float* X, int64_t ldx, const float* W, int64_t ldw,
                 const float* b, float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act,
                 float alpha, void* ws, cudaStream_t st, const float* xlo_in = nullptr,
                 float* ylo = nullptr, int64_t ldylo = 0) {
  if (M == 0 || N == 0) return kOk;
  if (K == 0) return fill_bias_act_f32(b, Y, ldy, M, N, act, alpha, st);
  SplitBufs s = carve(ws, M, N, K);
  const int splits = choose_splits(M, N, K);
  const int64_t Kp = split_pitch(K);
  float* xlo = xlo_in ? const_cast<float*>(xlo_in) : s.xlo;
  const bool xraw = x_raw_ok(X, ldx);
  // W is a registered weight's device copy: its split is kept, only X is split
  const bool mn = w_mn_ok(W, ldw, M, N);
  PreSplitW pre;
  bool have_pre = false;
  {
    std::lock_guard<std::mutex> g(g_w_mu);
    WeightEntry* e = g_weights.empty() ? nullptr : find_device_weights(c->dev, W);
    if (e && e->K == K && e->N == N && ldw == N) {
      const int rc = weights_ready(c, nullptr, e, mn, &pre, nullptr);
      if (rc) return rc;
      have_pre = true;
    }
  }
  auto split_x_only = [&]() -> int {
    if (xlo_in) return kOk;
    return xraw ? split_x_lo_f32(X, ldx, M, K, s.xlo, st)
                : split_x_f32(X, ldx, M, K, s.xhi, s.xlo, st);
  };
  int rc;
  if (mn && (have_pre || w_lo_mn_bytes(K, N) <= reinterpret_cast<char*>(s.partials) -
                                                          reinterpret_cast<char*>(s.whi))) {
    // W is read as-is (MN-major B_hi); its row-major lo part goes into the
    // W split region (or is the registered weight's). X likewise when its
    // rows are 16-byte aligned.
    const float* wlo = have_pre ? pre.lo_mn : s.whi;
    if (have_pre)
      rc = split_x_only();
    else if (xlo_in)  // X is pre-split: W alone
      rc = split_lo_xw_f32(nullptr, 0, 0, K, nullptr, nullptr, W, ldw, N, s.whi, st);
    else
      rc = split_lo_xw_f32(X, ldx, M, K, xraw ? nullptr : s.xhi, s.xlo, W, ldw, N, s.whi, st);
    if (rc == kOk)
      rc = gemm_tf32x3_wmn(xraw ? X : s.xhi, xlo, xraw ? ldx : Kp, W, ldw, wlo, M, N, K, b, Y,
                           ldy, act, alpha, splits, s.partials, c->status, st, ylo, ldylo);
  } else if (xraw) {  // X is the hi part; only lo is written
    const float* whi = have_pre ? pre.hiT : s.whi;
    const float* wlo = have_pre ? pre.loT : s.wlo;
    if (have_pre)
      rc = split_x_only();
    else
      rc = xlo_in ? split_w_f32(W, ldw, K, N, s.whi, s.wlo, st)
                  : split_xw_f32(X, ldx, M, W, ldw, K, N, nullptr, s.xlo, s.whi, s.wlo, st);
    if (rc == kOk)
      rc = gemm_tf32x3_xraw(X, ldx, xlo, whi, wlo, M, N, K, b, Y, ldy, act, alpha, splits,
                            s.partials, c->status, st, ylo, ldylo);
  } else {
    if (xlo_in) return fail(kErrInvalidArg, "a pre-split X needs 16-byte aligned X rows");
    rc = have_pre ? split_x_only()
                  : split_xw_f32(X, ldx, M, W, ldw, K, N, s.xhi, s.xlo, s.whi, s.wlo, st);
    if (rc == kOk)
      rc = gemm_tf32x3_splitk(s.xhi, s.xlo, have_pre ? pre.hiT : s.whi,
                              have_pre ? pre.loT : s.wlo, M, N, K, b, Y, ldy, act, alpha, splits,
                              s.partials, c->status, st, ylo, ldylo);
  }
  if (rc != kOk) return fail(rc, std::string("dense_f32: ") + launch_error_text());
  return kOk;
}

int validate_dense(const void* X, int64_t ldx, const void* W, int64_t ldw, const void* Y,
                   int64_t ldy, int64_t M, int64_t N, int64_t K, int act) {
  if (bad_dims(M, N, K)) return fail(kErrInvalidArg, "negative dimension");
  if (act < kActNone || act > kActLeakyRelu) return fail(kErrInvalidArg, "unknown activation");
  if (M > 0 && N > 0) {
    if (!Y) return fail(kErrInvalidArg, "null output");
    if (ldy < N) return fail(kErrInvalidArg, "ldy < N");
    if (K > 0) {
      if (!X || !W) return fail(kErrInvalidArg, "null input");
      if (ldx < K) return fail(kErrInvalidArg, "ldx < K");
      if (ldw < N) return fail(kErrInvalidArg, "ldw < N");
    }
  }
  if (M > (int64_t)1 << 31 || N > (int64_t)1 << 31 || K > (int64_t)1 << 31)
    return fail(kErrTooLarge, "dimension exceeds 2^31");
  return kOk;
}

// One device's share of a host-pointer dense call: rows [0, M) of the given
// host views, processed in row slabs through a kRing-slot ring of device
// buffers on three streams, so the copy-in of slab i+1, the compute of slab i
// and the copy-out of slab i-1 overlap.
int dense_host_on_device(int dev, const float* X, int64_t ldx, const float* W, int64_t ldw,
                         const float* b, float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                         int act, float alpha) {
  DeviceCtx* c = nullptr;
  int rc = get_ctx(dev, &c);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(c->mu);
  B200_CUDA(cudaSetDevice(dev), "cudaSetDevice");
  if (M == 0 || N == 0) return kOk;
  const int64_t Kp = split_pitch(std::max<int64_t>(K, 1));

  // Slab size: one slab for small calls, else B200_HOST_SLABS (default 16)
  // slabs of >= 512 rows, so the first copy-in and the last copy-out that
  // cannot overlap anything are short.
  int64_t slab = M;
  if (M * K * 4 >= ((int64_t)32 << 20) && M >= 1024) {
    static const int64_t nslabs_cfg = [] {
      const char* e = getenv("B200_HOST_SLABS");
      return (int64_t)((e && atoi(e) > 0) ? atoi(e) : 16);
    }();
    slab = std::max<int64_t>(512, round_up((M + nslabs_cfg - 1) / nslabs_cfg, 128));
  }
  const int64_t nslab = (M + slab - 1) / slab;
  // Pageable X / Y (e.g. plain numpy arrays) are staged through pinned slab
  // buffers with a multi-threaded host copy that overlaps the DMA of other
  // slabs; the driver's own staging of pageable copies is much slower.
  const bool stage_x = K > 0 && M * K * 4 >= ((int64_t)16 << 20) && is_pageable(X);
  const bool stage_y = M * N * 4 >= ((int64_t)16 << 20) && is_pageable(Y);

  // Weights (replicated): a registered W's device copy and split are kept
  // (b200_weights_register); any other W is uploaded and split once per call
  // on the compute stream.
  PreSplitW pre;
  const float* regW = nullptr;
  bool have_pre = false;
  if (K > 0) {
    std::lock_guard<std::mutex> g(g_w_mu);
    WeightEntry* e = g_weights.empty() ? nullptr : find_host_weights(W, ldw, K, N);
    if (e) {
      // a registered copy is cudaMalloc'd (aligned), pitch N
      const bool mn = w_mn_ok(reinterpret_cast<const float*>(256), N, M, N);
      if ((rc = weights_ready(c, W, e, mn, &pre, &regW))) return rc;
      have_pre = true;
    }
  }
  B200_CUDA(c->bias.reserve(std::max<int64_t>(N, 1) * 4), "alloc bias");
  if (K > 0 && !have_pre) {
    B200_CUDA(c->w.reserve(K * N * 4), "alloc W");
    B200_CUDA(c->whi.reserve(std::max(N * Kp * 4, w_lo_mn_bytes(K, N))), "alloc W split");
    B200_CUDA(c->wlo.reserve(N * Kp * 4), "alloc W split");
  }
  const int64_t last_rows = M - (nslab - 1) * slab;
  const int64_t part_bytes = K > 0 ? std::max(splitk_partials_bytes(slab, N, K),
                                              splitk_partials_bytes(last_rows, N, K))
                                   : 0;
  for (int i = 0; i < kRing && i < nslab; ++i) {
    if (stage_x) B200_CUDA(c->sx[i].reserve(slab * K * 4), "pinned X staging");
    if (stage_y) B200_CUDA(c->sy[i].reserve(slab * N * 4), "pinned Y staging");
    B200_CUDA(c->y[i].reserve(slab * N * 4), "alloc Y slab");
    if (part_bytes) B200_CUDA(c->part[i].reserve(part_bytes), "alloc split-K partials");
    if (K > 0) {
      B200_CUDA(c->x[i].reserve(slab * K * 4), "alloc X slab");
      B200_CUDA(c->xhi[i].reserve(slab * Kp * 4), "alloc X split");
      B200_CUDA(c->xlo[i].reserve(slab * Kp * 4), "alloc X split");
    }
  }
  float* dW = have_pre ? const_cast<float*>(regW) : static_cast<float*>(c->w.p);
  float* dWhi = have_pre ? const_cast<float*>(pre.hiT) : static_cast<float*>(c->whi.p);
  float* dWlo = have_pre ? const_cast<float*>(pre.loT) : static_cast<float*>(c->wlo.p);
  float* db = b ? static_cast<float*>(c->bias.p) : nullptr;
  // MN-major B (W read as-is, row-major lo part in dWhi) when W qualifies.
  const bool wmn = K > 0 && w_mn_ok(dW, N, M, N);
  if (b) B200_CUDA(cudaMemcpyAsync(db, b, N * 4, cudaMemcpyHostToDevice, c->s_comp), "H2D b");
  if (K > 0 && !have_pre) {
    if ((rc = h2d_rows(c, dW, N * 4, W, ldw * 4, N * 4, K, c->s_comp))) return rc;
    // A single-slab call splits W together with X (one launch) below.
    if (nslab > 1 && wmn) {
      rc = split_lo_xw_f32(nullptr, 0, 0, K, nullptr, nullptr, dW, N, N, dWhi, c->s_comp);
      if (rc) return fail(rc, "split W launch failed");
    } else if (!wmn && nslab > 1) {
      rc = split_w_f32(dW, N, K, N, dWhi, dWlo, c->s_comp);
      if (rc) return fail(rc, "split W launch failed");
    }
  }
  // W and its split are ready: slabs split X only
  const bool w_split = have_pre || nslab > 1;

  for (int64_t i = 0; i < nslab; ++i) {
    const int slot = (int)(i % kRing);
    const int64_t r0 = i * slab;
    const int64_t rows = std::min(slab, M - r0);
    float* dX = static_cast<float*>(c->x[slot].p);
    float* dY = static_cast<float*>(c->y[slot].p);
    // Slot reuse: the copy-in may overwrite X once slab i-kRing's compute has
    // read it; the compute may overwrite Y once slab i-kRing's copy-out is done.
    if (i >= kRing) B200_CUDA(cudaStreamWaitEvent(c->s_h2d, c->ev_comp[slot], 0), "wait");
    if (K > 0 && stage_x) {
      // staging slot free once slab i-kRing's copy from it has finished
      if (i >= kRing) B200_CUDA(cudaEventSynchronize(c->ev_h2d[slot]), "staging wait");
      par_copy_rows(c->sx[slot].p, K * 4, X + r0 * ldx, ldx * 4, K * 4, rows);
      B200_CUDA(cudaMemcpyAsync(dX, c->sx[slot].p, rows * K * 4, cudaMemcpyHostToDevice,
                                c->s_h2d),
                "H2D X");
    } else if (K > 0) {
      B200_CUDA(cudaMemcpy2DAsync(dX, K * 4, X + r0 * ldx, ldx * 4, K * 4, rows,
                                  cudaMemcpyHostToDevice, c->s_h2d),
                "H2D X");
    }
    B200_CUDA(cudaEventRecord(c->ev_h2d[slot], c->s_h2d), "record");
    B200_CUDA(cudaStreamWaitEvent(c->s_comp, c->ev_h2d[slot], 0), "wait");
    if (i >= kRing) B200_CUDA(cudaStreamWaitEvent(c->s_comp, c->ev_d2h[slot], 0), "wait");
    if (K == 0) {
      rc = fill_bias_act_f32(db, dY, N, rows, N, act, alpha, c->s_comp);
    } else {
      float* part = static_cast<float*>(c->part[slot].p);
      const int splits = choose_splits(rows, N, K);
      if (wmn) {
        float* xhi = static_cast<float*>(c->xhi[slot].p);
        float* xlo = static_cast<float*>(c->xlo[slot].p);
        const bool xraw = x_raw_ok(dX, K);
        float* wlo = have_pre ? const_cast<float*>(pre.lo_mn) : dWhi;
        if (!w_split)
          rc = split_lo_xw_f32(dX, K, rows, K, xraw ? nullptr : xhi, xlo, dW, N, N, wlo,
                               c->s_comp);
        else
          rc = xraw ? split_x_lo_f32(dX, K, rows, K, xlo, c->s_comp)
                    : split_x_f32(dX, K, rows, K, xhi, xlo, c->s_comp);
        if (rc == kOk)
          rc = gemm_tf32x3_wmn(xraw ? dX : xhi, xlo, xraw ? K : Kp, dW, N, wlo, rows, N, K, db,
                               dY, N, act, alpha, splits, part, c->status, c->s_comp);
      } else if (x_raw_ok(dX, K)) {
        float* xlo = static_cast<float*>(c->xlo[slot].p);
        rc = !w_split ? split_xw_f32(dX, K, rows, dW, N, K, N, nullptr, xlo, dWhi, dWlo, c->s_comp)
                      : split_x_lo_f32(dX, K, rows, K, xlo, c->s_comp);
        if (rc == kOk)
          rc = gemm_tf32x3_xraw(dX, K, xlo, dWhi, dWlo, rows, N, K, db, dY, N, act, alpha, splits,
                                part, c->status, c->s_comp);
      } else {
        float* xhi = static_cast<float*>(c->xhi[slot].p);
        float* xlo = static_cast<float*>(c->xlo[slot].p);
        rc = !w_split ? split_xw_f32(dX, K, rows, dW, N, K, N, xhi, xlo, dWhi, dWlo, c->s_comp)
                      : split_x_f32(dX, K, rows, K, xhi, xlo, c->s_comp);
        if (rc == kOk)
          rc = gemm_tf32x3_splitk(xhi, xlo, dWhi, dWlo, rows, N, K, db, dY, N, act, alpha,
                                  splits, part, c->status, c->s_comp);
      }
    }
    if (rc) return fail(rc, std::string("dense kernel launch failed: ") + launch_error_text());
    B200_CUDA(cudaEventRecord(c->ev_comp[slot], c->s_comp), "record");
    B200_CUDA(cudaStreamWaitEvent(c->s_d2h, c->ev_comp[slot], 0), "wait");
    if (stage_y) {
      B200_CUDA(cudaMemcpyAsync(c->sy[slot].p, dY, rows * N * 4, cudaMemcpyDeviceToHost,
                                c->s_d2h),
                "D2H Y");
    } else {
      B200_CUDA(cudaMemcpy2DAsync(Y + r0 * ldy, ldy * 4, dY, N * 4, N * 4, rows,
                                  cudaMemcpyDeviceToHost, c->s_d2h),
                "D2H Y");
    }
    B200_CUDA(cudaEventRecord(c->ev_d2h[slot], c->s_d2h), "record");
    if (stage_y && i >= 1) {  // unstage the previous slab while this one computes
      const int ps = (int)((i - 1) % kRing);
      const int64_t pr0 = (i - 1) * slab;
      B200_CUDA(cudaEventSynchronize(c->ev_d2h[ps]), "unstage wait");
      par_copy_rows(Y + pr0 * ldy, ldy * 4, c->sy[ps].p, N * 4, N * 4, std::min(slab, M - pr0));
    }
  }
  if (stage_y) {
    const int64_t li = nslab - 1;
    const int ls = (int)(li % kRing);
    B200_CUDA(cudaEventSynchronize(c->ev_d2h[ls]), "unstage wait");
    par_copy_rows(Y + li * slab * ldy, ldy * 4, c->sy[ls].p, N * 4, N * 4, M - li * slab);
  }
  B200_CUDA(cudaStreamSynchronize(c->s_d2h), "sync");
  B200_CUDA(cudaStreamSynchronize(c->s_comp), "sync");
  return check_device_status(c);
}

int resolve_ndev(int ndev) {
  if (ndev <= 0) ndev = b200_get_default_devices();
  return ndev;
}

// Splits rows [0, M) into `ndev` contiguous shards and runs fn(dev, r0, rows)
// on one host thread per device.
template <class Fn>
int run_sharded(int ndev, int64_t M, Fn fn) {
  const int avail = device_count();
  if (avail == 0) return fail(kErrNoDevice, "no CUDA device available");
  if (ndev > avail) {
    char buf[96];
    snprintf(buf, sizeof buf, "requested %d devices, %d available", ndev, avail);
    return fail(kErrInvalidArg, buf);
  }
  if (ndev == 1) {
    int cur = 0;
    B200_CUDA(cudaGetDevice(&cur), "cudaGetDevice");
    return fn(cur, 0, M);
  }
  std::vector<int> rcs(ndev, kOk);
  std::vector<std::string> errs(ndev);
  std::vector<std::thread> th;
  const int64_t base = M / ndev, rem = M % ndev;
  int64_t r0 = 0;
  for (int d = 0; d < ndev; ++d) {
    const int64_t rows = base + (d < rem ? 1 : 0);
    th.emplace_back([&, d, r0, rows] {
      rcs[d] = fn(d, r0, rows);
      if (rcs[d]) errs[d] = t_err;
    });
    r0 += rows;
  }
  for (auto& t : th) t.join();
  for (int d = 0; d < ndev; ++d)
    if (rcs[d]) return fail(rcs[d], "device " + std::to_string(d) + ": " + errs[d]);
  return kOk;
}

// C = A B (+ bias) mod 2^32 on the current device: the tensor-core kernel
// (byte-sliced int8 MMAs; ws >= gemm_i32_tc_workspace_bytes) unless K == 0
// or B200_I32_TC=0, then the CUDA-core kernel.
int matmul_i32_device(DeviceCtx* c, const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb,
                      const int32_t* bias, int32_t* C, int64_t ldc, int64_t M, int64_t N,
                      int64_t K, void* ws, cudaStream_t st) {
  if (K > 0 && ws && i32_tensor_core_enabled())
    return gemm_i32_tc(A, lda, B, ldb, bias, C, ldc, M, N, K, ws, c->status, st);
  return gemm_i32(A, lda, B, ldb, C, ldc, M, N, K, bias, st);
}

int simple_host_i32_matmul(int dev, const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb,
                           const int32_t* bias, int32_t* C, int64_t ldc, int64_t M, int64_t N,
                           int64_t K) {
  DeviceCtx* c = nullptr;
  int rc = get_ctx(dev, &c);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(c->mu);
  B200_CUDA(cudaSetDevice(dev), "cudaSetDevice");
  if (M == 0 || N == 0) return kOk;
  B200_CUDA(c->x[0].reserve(std::max<int64_t>(M * K, 1) * 4), "alloc A");
  B200_CUDA(c->w.reserve(std::max<int64_t>(K * N, 1) * 4), "alloc B");
  B200_CUDA(c->y[0].reserve(M * N * 4), "alloc C");
  B200_CUDA(c->bias.reserve(std::max<int64_t>(N, 1) * 4), "alloc bias");
  const int64_t ws_bytes = gemm_i32_tc_workspace_bytes(M, N, K);
  if (ws_bytes) B200_CUDA(c->xhi[0].reserve(ws_bytes), "alloc i32 workspace");
  int32_t* dA = static_cast<int32_t*>(c->x[0].p);
  int32_t* dB = static_cast<int32_t*>(c->w.p);
  int32_t* dC = static_cast<int32_t*>(c->y[0].p);
  int32_t* db = bias ? static_cast<int32_t*>(c->bias.p) : nullptr;
  cudaStream_t s = c->s_comp;
  if (K > 0) {
    if ((rc = h2d_rows(c, dA, K * 4, A, lda * 4, K * 4, M, s))) return rc;
    if ((rc = h2d_rows(c, dB, N * 4, B, ldb * 4, N * 4, K, s))) return rc;
  }
  if (bias) B200_CUDA(cudaMemcpyAsync(db, bias, N * 4, cudaMemcpyHostToDevice, s), "H2D bias");
  rc = matmul_i32_device(c, dA, K, dB, N, db, dC, N, M, N, K, ws_bytes ? c->xhi[0].p : nullptr,
                         s);
  if (rc) return fail(rc, std::string("i32 matmul launch failed: ") + launch_error_text());
  if ((rc = d2h_rows(c, C, ldc * 4, dC, N * 4, N * 4, M, s))) return rc;
  return kOk;
}

// Host wrapper for the elementwise kernels: one device, whole-buffer copies.
template <class Launch>
int elementwise_host(size_t in_bytes_x, const void* X, size_t in_bytes_b, const void* b,
                     size_t out_bytes, void* Y, Launch launch) {
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(c->mu);
  if (out_bytes == 0) return kOk;
  B200_CUDA(c->x[0].reserve(std::max<size_t>(in_bytes_x, 4)), "alloc X");
  B200_CUDA(c->bias.reserve(std::max<size_t>(in_bytes_b, 4)), "alloc b");
  B200_CUDA(c->y[0].reserve(out_bytes), "alloc Y");
  cudaStream_t s = c->s_comp;
  if ((rc = h2d_flat(c, c->x[0].p, X, (int64_t)in_bytes_x, s))) return rc;
  if (b) B200_CUDA(cudaMemcpyAsync(c->bias.p, b, in_bytes_b, cudaMemcpyHostToDevice, s), "H2D b");
  rc = launch(c->x[0].p, b ? c->bias.p : nullptr, c->y[0].p, s);
  if (rc) return fail(rc, std::string("elementwise launch failed: ") + launch_error_text());
  return d2h_flat(c, Y, c->y[0].p, (int64_t)out_bytes, s);
}


// Host-pointer reduction / dot on the current device: copy in, two-pass
// reduce into a device scalar, copy the scalar out.
template <class T>
int reduce_host_impl(const T* x, const T* y, int64_t n, int op, T init, T* result) {
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(c->mu);
  const size_t bytes = (size_t)std::max<int64_t>(n, 1) * sizeof(T);
  B200_CUDA(c->x[0].reserve(bytes), "alloc x");
  if (y) B200_CUDA(c->w.reserve(bytes), "alloc y");
  B200_CUDA(c->y[0].reserve((size_t)reduce_scratch_bytes() + 256), "alloc partials");
  cudaStream_t s = c->s_comp;
  if (n && (rc = h2d_flat(c, c->x[0].p, x, n * (int64_t)sizeof(T), s))) return rc;
  if (y && n && (rc = h2d_flat(c, c->w.p, y, n * (int64_t)sizeof(T), s))) return rc;
  char* scratch = static_cast<char*>(c->y[0].p);
  T* dout = reinterpret_cast<T*>(scratch + reduce_scratch_bytes());
  if constexpr (std::is_same<T, float>::value)
    rc = reduce_f32(static_cast<const float*>(c->x[0].p), y ? static_cast<const float*>(c->w.p) : nullptr,
                    n, op, init, dout, scratch, s);
  else
    rc = reduce_i32(static_cast<const int32_t*>(c->x[0].p),
                    y ? static_cast<const int32_t*>(c->w.p) : nullptr, n, op, init, dout, scratch, s);
  if (rc) return fail(rc, std::string("reduction launch failed: ") + launch_error_text());
  B200_CUDA(cudaMemcpyAsync(result, dout, sizeof(T), cudaMemcpyDeviceToHost, s), "D2H result");
  B200_CUDA(cudaStreamSynchronize(s), "sync");
  return kOk;
}

// Device-pointer reduction: partials in the per-(device, stream) scratch.
template <class T>
int reduce_device_impl(const T* x, const T* y, int64_t n, int op, T init, T* out, void* stream) {
  if (n < 0 || op < kRedSum || op > kRedMin) return fail(kErrInvalidArg, "bad reduction arguments");
  if (!out || (n > 0 && !x)) return fail(kErrInvalidArg, "null buffer");
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ScratchLease lease;  // held until the reduction is queued
  if ((rc = lease.acquire(c, st, (size_t)reduce_scratch_bytes()))) return rc;
  void* ws = lease.p;
  if constexpr (std::is_same<T, float>::value)
    rc = reduce_f32(x, y, n, op, init, out, ws, st);
  else
    rc = reduce_i32(x, y, n, op, init, out, ws, st);
  return rc ? fail(rc, std::string("reduction launch failed: ") + launch_error_text()) : kOk;
}
}  // namespace

int report_error(int code, const char* msg) { return fail(code, msg); }
int report_ok() { return succeed(); }

namespace {
thread_local std::string t_launch_err;
}
int launch_result(cudaError_t e) {
  if (e == cudaSuccess) return kOk;
  cudaGetLastError();  // clear the non-sticky error
  t_launch_err = std::string("kernel launch: ") + cudaGetErrorString(e);
  return kErrCuda;
}
int driver_failure(const char* what, int code) {
  t_launch_err = std::string(what) + " failed (CUresult " + std::to_string(code) + ")";
  return kErrDriver;
}
const char* launch_error_text() { return t_launch_err.c_str(); }

}  // namespace b200

using namespace b200;

template <class T>
static T* at(void* aligned, int64_t off) {
  return static_cast<T*>(aligned) + off;
}

// =========================================================================
extern "C" {

const char* b200_version(void) { return "b200-edsl 0.1 (sm_100a, tcgen05 3xTF32)"; }
const char* b200_last_error(void) { return t_err.c_str(); }
int b200_last_status(void) { return t_status; }
int b200_device_count(void) { return device_count(); }
long long b200_launch_count(void) { return g_launches.load(); }

int b200_set_default_devices(int ndev) {
  if (ndev < 1) return fail(kErrInvalidArg, "ndev must be >= 1");
  g_default_devices = ndev;
  return succeed();
}

int b200_get_default_devices(void) {
  if (g_default_devices < 1) {
    const char* e = getenv("B200_DEVICES");
    g_default_devices = (e && atoi(e) > 0) ? atoi(e) : 1;
  }
  return g_default_devices;
}

int b200_release(void) {
  // The loop visits every initialised device; the caller's current device is
  // restored afterwards, so its later device-pointer calls stay on it.
  int prev = 0;
  const bool have_prev = cudaGetDevice(&prev) == cudaSuccess;
  for (int d = 0; d < 64; ++d) {
    DeviceCtx& c = g_dev[d];
    std::lock_guard<std::mutex> lk(c.mu);
    if (!c.ready) continue;
    cudaSetDevice(d);
    cudaDeviceSynchronize();
    c.w.release(); c.whi.release(); c.wlo.release(); c.bias.release();
    for (int i = 0; i < kRing; ++i) {
      c.x[i].release(); c.xhi[i].release(); c.xlo[i].release(); c.y[i].release();
      c.part[i].release();
      if (i < 2) c.sc[i].release();
      c.sx[i].release();
      c.sy[i].release();
    }
    {
      std::lock_guard<std::mutex> g(g_w_mu);
      for (auto& kv : g_weights) release_weight_copy(kv.second->dev[d]);
    }
    std::vector<StreamScratch*> entries;
    {
      std::lock_guard<std::mutex> g(g_mu);
      for (auto& kv : c.scratch) entries.push_back(kv.second.get());
    }
    for (StreamScratch* e : entries) {
      std::lock_guard<std::mutex> el(e->mu);
      e->buf.release();
    }
  }
  if (have_prev) cudaSetDevice(prev);
  return succeed();
}

// ---------------------------------------------------------------- weight cache
int b200_weights_register(const float* W, int64_t ldw, int64_t K, int64_t N, uint64_t version) {
  if (!W || K <= 0 || N <= 0 || ldw < N)
    return fail(kErrInvalidArg, "weights: non-null W, K > 0, N > 0 and ldw >= N are required");
  if (K > (int64_t)1 << 31 || N > (int64_t)1 << 31)
    return fail(kErrTooLarge, "dimension exceeds 2^31");
  std::lock_guard<std::mutex> g(g_w_mu);
  auto& slot = g_weights[W];
  if (slot && slot->ldw == ldw && slot->K == K && slot->N == N && slot->version == version)
    return succeed();  // unchanged: keep the device copies
  if (slot) {
    // new contents or shape: drop the old copies (after work that may read them)
    int prev = 0;
    const bool have_prev = cudaGetDevice(&prev) == cudaSuccess;
    for (int d = 0; d < 64; ++d)
      if (slot->dev[d].w.p || slot->dev[d].lo_mn.p || slot->dev[d].hiT.p) {
        cudaSetDevice(d);
        cudaDeviceSynchronize();
        release_weight_copy(slot->dev[d]);
      }
    if (have_prev) cudaSetDevice(prev);
  } else {
    slot.reset(new WeightEntry);
  }
  slot->ldw = ldw;
  slot->K = K;
  slot->N = N;
  slot->version = version;
  return succeed();
}

int b200_weights_release(const float* W) {
  int prev = 0;
  const bool have_prev = cudaGetDevice(&prev) == cudaSuccess;
  std::lock_guard<std::mutex> g(g_w_mu);
  auto it = g_weights.find(W);
  if (it == g_weights.end()) return fail(kErrInvalidArg, "weights: W is not registered");
  for (int d = 0; d < 64; ++d) {
    WeightCopy& wc = it->second->dev[d];
    if (wc.w.p || wc.lo_mn.p || wc.hiT.p) {
      cudaSetDevice(d);
      cudaDeviceSynchronize();  // work queued on any stream may still read them
      release_weight_copy(wc);
    }
  }
  g_weights.erase(it);
  if (have_prev) cudaSetDevice(prev);
  return succeed();
}

int b200_weights_device(const float* W, const float** dW) {
  if (!W || !dW) return fail(kErrInvalidArg, "weights: null argument");
  *dW = nullptr;
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(c->mu);  // the staging buffers of h2d_rows
  std::lock_guard<std::mutex> g(g_w_mu);
  auto it = g_weights.find(W);
  if (it == g_weights.end()) return fail(kErrInvalidArg, "weights: W is not registered");
  WeightEntry* e = it->second.get();
  WeightCopy& d = e->dev[c->dev];
  if (!d.up) {
    B200_CUDA(d.w.reserve((size_t)e->K * e->N * 4), "alloc registered W");
    if ((rc = h2d_rows(c, d.w.p, e->N * 4, W, e->ldw * 4, e->N * 4, e->K, c->s_comp)))
      return rc;
    B200_CUDA(cudaStreamSynchronize(c->s_comp), "sync");
    d.up = true;
  }
  *dW = static_cast<const float*>(d.w.p);
  return succeed();
}

// ---------------------------------------------------------------- device API
int64_t b200_dense_f32_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (bad_dims(M, N, K)) return -1;
  return dense_scratch_bytes(M, N, std::max<int64_t>(K, 1));
}

int b200_dense_f32_launches(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) return -1;
  if (M == 0 || N == 0) return 0;
  if (K == 0) return 1;  // the bias / activation fill
  return 1 + gemm_f32_launches(M, N, K);  // the split pass, the GEMM (+ reduction)
}

int b200_dense_f32_splits(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 1;
  return choose_splits(M, N, K);
}

int b200_dense_f32_ws(const float* X, int64_t ldx, const float* W, int64_t ldw, const float* b,
                      float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act,
                      float alpha, void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = validate_dense(X, ldx, W, ldw, Y, ldy, M, N, K, act);
  if (rc) return rc;
  const int64_t need = dense_scratch_bytes(M, N, std::max<int64_t>(K, 1));
  if (K > 0 && M > 0 && N > 0) {
    if (!workspace || workspace_bytes < need)
      return fail(kErrInvalidArg, "workspace missing or smaller than "
                                  "b200_dense_f32_workspace_bytes()");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
      return fail(kErrInvalidArg, "workspace must be 256-byte aligned");
  }
  DeviceCtx* c = nullptr;
  if ((rc = current_ctx(&c))) return rc;
  rc = dense_device(c, X, ldx, W, ldw, b, Y, ldy, M, N, K, act, alpha, workspace,
                    static_cast<cudaStream_t>(stream));
  return rc ? rc : succeed();
}

int b200_dense_f32(const float* X, int64_t ldx, const float* W, int64_t ldw, const float* b,
                   float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act, float alpha,
                   void* stream) {
  int rc = validate_dense(X, ldx, W, ldw, Y, ldy, M, N, K, act);
  if (rc) return rc;
  DeviceCtx* c = nullptr;
  if ((rc = current_ctx(&c))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  ScratchLease lease;  // held until the kernels that use ws are queued
  if (M > 0 && N > 0 && K > 0) {
    const size_t need = (size_t)dense_scratch_bytes(M, N, K);
    if ((rc = lease.acquire(c, st, need))) return rc;
    ws = lease.p;
  }
  rc = dense_device(c, X, ldx, W, ldw, b, Y, ldy, M, N, K, act, alpha, ws, st);
  return rc ? rc : succeed();
}

int b200_dense_f32_peers(const float* X, int64_t ldx, const float* W, int64_t ldw,
                         const float* b, float* Y, int64_t ldy, float* const* peer_y, int npeers,
                         int64_t M, int64_t N, int64_t K, int act, float alpha, void* stream) {
  int rc = validate_dense(X, ldx, W, ldw, Y, ldy, M, N, K, act);
  if (rc) return rc;
  if (npeers < 0 || npeers > kMaxEpiloguePeers || (npeers > 0 && peer_y == nullptr))
    return fail(kErrInvalidArg, "npeers must be 0..7, with that many peer output pointers");
  for (int i = 0; i < npeers; ++i)
    if (peer_y[i] == nullptr) return fail(kErrInvalidArg, "null peer output");
  DeviceCtx* c = nullptr;
  if ((rc = current_ctx(&c))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  ScratchLease lease;  // held until the kernels that use ws are queued
  if (M > 0 && N > 0 && K > 0) {
    const size_t need = (size_t)dense_scratch_bytes(M, N, K);
    if ((rc = lease.acquire(c, st, need))) return rc;
    ws = lease.p;
  }
  {
    const EpiloguePeersScope peers(peer_y, npeers);
    rc = dense_device(c, X, ldx, W, ldw, b, Y, ldy, M, N, K, act, alpha, ws, st);
  }
  // K == 0 fills Y with act(b) by a separate kernel: fill the peers the same way
  for (int i = 0; rc == kOk && K == 0 && i < npeers; ++i)
    if (fill_bias_act_f32(b, peer_y[i], ldy, M, N, act, alpha, st) != kOk)
      rc = fail(kErrCuda, std::string("peer fill launch failed: ") + launch_error_text());
  return rc ? rc : succeed();
}

int b200_dense_f32_multicast(const float* X, int64_t ldx, const float* W, int64_t ldw,
                             const float* b, float* Y, int64_t ldy, float* mc_y, int64_t M,
                             int64_t N, int64_t K, int act, float alpha, void* stream) {
  int rc = validate_dense(X, ldx, W, ldw, Y, ldy, M, N, K, act);
  if (rc) return rc;
  if (!mc_y) return fail(kErrInvalidArg, "null multicast output");
  if (M > 0 && N > 0 && K == 0)
    return fail(kErrInvalidArg, "the multicast entry point needs K > 0");
  DeviceCtx* c = nullptr;
  if ((rc = current_ctx(&c))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  ScratchLease lease;  // held until the kernels that use ws are queued
  if (M > 0 && N > 0) {
    const size_t need = (size_t)dense_scratch_bytes(M, N, K);
    if ((rc = lease.acquire(c, st, need))) return rc;
    ws = lease.p;
  }
  {
    const EpiloguePeersScope peers(nullptr, 0, mc_y);
    rc = dense_device(c, X, ldx, W, ldw, b, Y, ldy, M, N, K, act, alpha, ws, st);
  }
  return rc ? rc : succeed();
}

int b200_dense_f32_chain(const float* X, int64_t ldx, const float* Xlo, const float* W,
                         int64_t ldw, const float* b, float* Y, int64_t ldy, float* Ylo,
                         int64_t ldylo, int64_t M, int64_t N, int64_t K, int act, float alpha,
                         void* stream) {
  int rc = validate_dense(X, ldx, W, ldw, Y, ldy, M, N, K, act);
  if (rc) return rc;
  if (Xlo && (!x_raw_ok(X, ldx) || (reinterpret_cast<uintptr_t>(Xlo) & 15) != 0))
    return fail(kErrInvalidArg, "a pre-split X needs 16-byte aligned X and Xlo rows");
  if (Ylo && ldylo < N) return fail(kErrInvalidArg, "Ylo pitch < N");
  if (Ylo && K == 0) return fail(kErrInvalidArg, "Ylo needs K > 0");
  DeviceCtx* c = nullptr;
  if ((rc = current_ctx(&c))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  ScratchLease lease;  // held until the kernels that use ws are queued
  if (M > 0 && N > 0 && K > 0) {
    const size_t need = (size_t)dense_scratch_bytes(M, N, K);
    if ((rc = lease.acquire(c, st, need))) return rc;
    ws = lease.p;
  }
  rc = dense_device(c, X, ldx, W, ldw, b, Y, ldy, M, N, K, act, alpha, ws, st, Xlo, Ylo, ldylo);
  return rc ? rc : succeed();
}

int b200_matmul_i32(const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb,
                    const int32_t* bias, int32_t* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                    void* stream) {
  int rc = validate_dense(A, lda, B, ldb, C, ldc, M, N, K, kActNone);
  if (rc) return rc;
  if (M == 0 || N == 0) return succeed();
  DeviceCtx* c = nullptr;
  if ((rc = current_ctx(&c))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  ScratchLease lease;  // held until the kernels that use ws are queued
  const size_t need = (size_t)gemm_i32_tc_workspace_bytes(M, N, K);
  if (need && i32_tensor_core_enabled()) {
    if ((rc = lease.acquire(c, st, need))) return rc;
    ws = lease.p;
  }
  rc = matmul_i32_device(c, A, lda, B, ldb, bias, C, ldc, M, N, K, ws, st);
  return rc ? fail(rc, std::string("i32 matmul launch failed: ") + launch_error_text()) : succeed();
}

int b200_bias_act_f32(const float* X, int64_t ldx, const float* b, float* Y, int64_t ldy,
                      int64_t M, int64_t N, int act, float alpha, void* stream) {
  if (M < 0 || N < 0 || act < 0 || act > 2) return fail(kErrInvalidArg, "bad arguments");
  if (M > 0 && N > 0 && (!X || !Y || ldx < N || ldy < N))
    return fail(kErrInvalidArg, "null buffer or pitch < N");
  int rc = bias_act_f32(X, ldx, b, Y, ldy, M, N, act, alpha, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, std::string("bias/activation launch failed: ") + launch_error_text()) : succeed();
}

int b200_act_f32(const float* X, float* Y, int64_t count, int act, float alpha, void* stream) {
  if (count < 0 || act < 0 || act > 2) return fail(kErrInvalidArg, "bad arguments");
  if (count > 0 && (!X || !Y)) return fail(kErrInvalidArg, "null buffer");
  int rc = act_f32(X, Y, count, act, alpha, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, std::string("activation launch failed: ") + launch_error_text()) : succeed();
}

int b200_bias_add_i32(const int32_t* X, int64_t ldx, const int32_t* b, int32_t* Y, int64_t ldy,
                      int64_t M, int64_t N, void* stream) {
  if (M < 0 || N < 0) return fail(kErrInvalidArg, "negative dimension");
  if (M > 0 && N > 0 && (!X || !b || !Y || ldx < N || ldy < N))
    return fail(kErrInvalidArg, "null buffer or pitch < N");
  int rc = bias_add_i32(X, ldx, b, Y, ldy, M, N, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, std::string("bias add launch failed: ") + launch_error_text()) : succeed();
}

int b200_stream_sync(void* stream) {
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  B200_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "stream sync");
  rc = check_device_status(c);
  return rc ? rc : succeed();
}

// ---------------------------------------------------------------- split / presplit
int b200_tf32_split_rows(const float* X, int64_t ldx, int64_t M, int64_t K, float* hi, float* lo,
                         void* stream) {
  if (M < 0 || K < 0 || (M > 0 && K > 0 && (!X || !hi || !lo || ldx < K)))
    return fail(kErrInvalidArg, "bad split_rows arguments");
  if (M == 0 || K == 0) return succeed();
  int rc = split_x_f32(X, ldx, M, K, hi, lo, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, std::string("split_rows launch failed: ") + launch_error_text()) : succeed();
}

int b200_tf32_split_transpose(const float* W, int64_t ldw, int64_t K, int64_t N, float* hiT,
                              float* loT, void* stream) {
  if (N < 0 || K < 0 || (N > 0 && K > 0 && (!W || !hiT || !loT || ldw < N)))
    return fail(kErrInvalidArg, "bad split_transpose arguments");
  if (N == 0 || K == 0) return succeed();
  int rc = split_w_f32(W, ldw, K, N, hiT, loT, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, std::string("split_transpose launch failed: ") + launch_error_text()) : succeed();
}

int b200_gemm_tf32x3_presplit(const float* xhi, const float* xlo, const float* whiT,
                              const float* wloT, const float* b, float* Y, int64_t ldy, int64_t M,
                              int64_t N, int64_t K, int act, float alpha, void* stream) {
  int rc = validate_dense(xhi, K, whiT, N, Y, ldy, M, N, K, act);
  if (rc) return rc;
  if (M > 0 && N > 0 && K > 0 && (!xlo || !wloT)) return fail(kErrInvalidArg, "null lo operand");
  for (const void* p : {(const void*)xhi, (const void*)xlo, (const void*)whiT, (const void*)wloT})
    if (reinterpret_cast<uintptr_t>(p) & 15)
      return fail(kErrInvalidArg, "split operands must be 16-byte aligned");
  DeviceCtx* c = nullptr;
  if ((rc = current_ctx(&c))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) return succeed();
  if (K == 0) rc = fill_bias_act_f32(b, Y, ldy, M, N, act, alpha, st);
  else rc = gemm_tf32x3_presplit(xhi, xlo, whiT, wloT, M, N, K, b, Y, ldy, act, alpha, c->status, st);
  return rc ? fail(rc, std::string("gemm launch failed: ") + launch_error_text()) : succeed();
}

int b200_dense_f32_wsplit(const float* X, int64_t ldx, const float* whiT, const float* wloT,
                          const float* b, float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                          int act, float alpha, void* stream) {
  int rc = validate_dense(X, ldx, whiT, N, Y, ldy, M, N, K, act);
  if (rc) return rc;
  if (M > 0 && N > 0 && K > 0) {
    if (!wloT) return fail(kErrInvalidArg, "null lo operand");
    if ((reinterpret_cast<uintptr_t>(whiT) | reinterpret_cast<uintptr_t>(wloT)) & 15)
      return fail(kErrInvalidArg, "split operands must be 16-byte aligned");
  }
  DeviceCtx* c = nullptr;
  if ((rc = current_ctx(&c))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) return succeed();
  if (K == 0) {
    rc = fill_bias_act_f32(b, Y, ldy, M, N, act, alpha, st);
    return rc ? fail(rc, std::string("launch failed: ") + launch_error_text()) : succeed();
  }
  const int splits = choose_splits(M, N, K);
  // Scratch: [X hi | X lo] (separate split pass) then the split-K partials.
  const int64_t Kp = split_pitch(K);
  const int64_t xsplit = 2 * round_up(M * Kp * 4, 256);
  void* ws = nullptr;
  ScratchLease lease;  // held until the kernels that use ws are queued
  {
    const size_t need = (size_t)(xsplit + splitk_partials_bytes(M, N, K)) + 256;
    if ((rc = lease.acquire(c, st, need))) return rc;
    ws = lease.p;
  }
  float* part = reinterpret_cast<float*>(static_cast<char*>(ws) + xsplit);
  if (x_raw_ok(X, ldx)) {
    float* xlo = reinterpret_cast<float*>(static_cast<char*>(ws) + xsplit / 2);
    rc = split_x_lo_f32(X, ldx, M, K, xlo, st);
    if (rc == kOk)
      rc = gemm_tf32x3_xraw(X, ldx, xlo, whiT, wloT, M, N, K, b, Y, ldy, act, alpha, splits, part,
                            c->status, st);
  } else {
    float* xhi = static_cast<float*>(ws);
    float* xlo = reinterpret_cast<float*>(static_cast<char*>(ws) + xsplit / 2);
    rc = split_x_f32(X, ldx, M, K, xhi, xlo, st);
    if (rc == kOk)
      rc = gemm_tf32x3_splitk(xhi, xlo, whiT, wloT, M, N, K, b, Y, ldy, act, alpha, splits, part,
                              c->status, st);
  }
  return rc ? fail(rc, std::string("gemm launch failed: ") + launch_error_text()) : succeed();
}

// ---------------------------------------------------------------- device buffers
// Device buffers come from the device's stream-ordered memory pool with its
// release threshold raised, so freed blocks stay cached for the next call
// instead of returning to the driver (cudaFree would synchronise the device).
static int pool_ready(int dev) {
  static std::atomic<uint64_t> done{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load() & bit) return kOk;
  cudaMemPool_t pool;
  B200_CUDA(cudaDeviceGetDefaultMemPool(&pool, dev), "cudaDeviceGetDefaultMemPool");
  uint64_t threshold = UINT64_MAX;
  B200_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold),
            "cudaMemPoolSetAttribute");
  done.fetch_or(bit);
  return kOk;
}

int b200_malloc(void** ptr, int64_t bytes) {
  if (!ptr || bytes < 0) return fail(kErrInvalidArg, "bad malloc arguments");
  *ptr = nullptr;
  if (bytes == 0) return succeed();
  if (device_count() == 0) return fail(kErrNoDevice, "no CUDA device available");
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  int rc = pool_ready(dev);
  if (rc) return rc;
  B200_CUDA(cudaMallocAsync(ptr, (size_t)bytes, nullptr), "cudaMallocAsync");
  return succeed();
}

int b200_free(void* ptr) {
  if (ptr) B200_CUDA(cudaFreeAsync(ptr, nullptr), "cudaFreeAsync");
  return succeed();
}

// Large pageable host buffers are staged through the runtime's pinned chunks
// (parallel host copies overlapping the DMA); everything else is one copy.
// Both calls are synchronous with respect to the host buffer.
int b200_memcpy_h2d(void* dst, const void* src, int64_t bytes) {
  if (bytes < 0) return fail(kErrInvalidArg, "negative size");
  if (!bytes) return succeed();
  if (bytes < kStageMin) {
    B200_CUDA(cudaMemcpy(dst, src, (size_t)bytes, cudaMemcpyHostToDevice), "H2D");
    return succeed();
  }
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(c->mu);
  // cudaMemcpy's ordering: after the work queued on the legacy default stream
  B200_CUDA(cudaStreamSynchronize(nullptr), "sync");
  if ((rc = h2d_flat(c, dst, src, bytes, c->s_h2d))) return rc;
  B200_CUDA(cudaStreamSynchronize(c->s_h2d), "sync");
  return succeed();
}

int b200_memcpy_d2h(void* dst, const void* src, int64_t bytes) {
  if (bytes < 0) return fail(kErrInvalidArg, "negative size");
  if (!bytes) return succeed();
  if (bytes < kStageMin) {
    B200_CUDA(cudaMemcpy(dst, src, (size_t)bytes, cudaMemcpyDeviceToHost), "D2H");
    return succeed();
  }
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(c->mu);
  B200_CUDA(cudaStreamSynchronize(nullptr), "sync");
  if ((rc = d2h_flat(c, dst, src, bytes, c->s_d2h))) return rc;
  return succeed();
}


// ---------------------------------------------------------------- reductions / dot
int b200_reduce_f32(const float* x, int64_t n, int op, float init, float* out, void* stream) {
  int rc = reduce_device_impl<float>(x, nullptr, n, op, init, out, stream);
  return rc ? rc : succeed();
}
int b200_reduce_i32(const int32_t* x, int64_t n, int op, int32_t init, int32_t* out,
                    void* stream) {
  int rc = reduce_device_impl<int32_t>(x, nullptr, n, op, init, out, stream);
  return rc ? rc : succeed();
}
int b200_dot_f32(const float* a, const float* b, int64_t n, float* out, void* stream) {
  if (n > 0 && !b) return fail(kErrInvalidArg, "null buffer");
  int rc = reduce_device_impl<float>(a, b, n, kRedSum, 0.0f, out, stream);
  return rc ? rc : succeed();
}
int b200_dot_i32(const int32_t* a, const int32_t* b, int64_t n, int32_t* out, void* stream) {
  if (n > 0 && !b) return fail(kErrInvalidArg, "null buffer");
  int rc = reduce_device_impl<int32_t>(a, b, n, kRedSum, 0, out, stream);
  return rc ? rc : succeed();
}
int b200_reduce_f32_host(const float* x, int64_t n, int op, float init, float* result) {
  if (n < 0 || op < kRedSum || op > kRedMin || !result || (n > 0 && !x))
    return fail(kErrInvalidArg, "bad reduction arguments");
  int rc = reduce_host_impl<float>(x, nullptr, n, op, init, result);
  return rc ? rc : succeed();
}
int b200_reduce_i32_host(const int32_t* x, int64_t n, int op, int32_t init, int32_t* result) {
  if (n < 0 || op < kRedSum || op > kRedMin || !result || (n > 0 && !x))
    return fail(kErrInvalidArg, "bad reduction arguments");
  int rc = reduce_host_impl<int32_t>(x, nullptr, n, op, init, result);
  return rc ? rc : succeed();
}
int b200_dot_f32_host(const float* a, const float* b, int64_t n, float* result) {
  if (n < 0 || !result || (n > 0 && (!a || !b))) return fail(kErrInvalidArg, "bad dot arguments");
  int rc = reduce_host_impl<float>(a, b, n, kRedSum, 0.0f, result);
  return rc ? rc : succeed();
}
int b200_dot_i32_host(const int32_t* a, const int32_t* b, int64_t n, int32_t* result) {
  if (n < 0 || !result || (n > 0 && (!a || !b))) return fail(kErrInvalidArg, "bad dot arguments");
  int rc = reduce_host_impl<int32_t>(a, b, n, kRedSum, 0, result);
  return rc ? rc : succeed();
}

// ---------------------------------------------------------------- pinned host pool
// Page-locked host blocks for results returned to Python: device-to-host
// copies into them run at full PCIe speed and never fault pages in. Freed
// blocks are kept (bucketed by size rounded up to 2 MiB, at most
// kPinnedCacheBytes in total) and handed out again.
namespace {
constexpr size_t kPinnedBucket = (size_t)2 << 20;
constexpr size_t kPinnedCacheBytes = (size_t)16 << 30;
std::mutex g_pin_mu;
std::multimap<size_t, void*> g_pin_free;   // bucketed size -> block
std::map<void*, size_t> g_pin_size;        // live and cached blocks
size_t g_pin_cached = 0;
}  // namespace

int b200_host_alloc(void** ptr, int64_t bytes) {
  if (!ptr || bytes < 0) return fail(kErrInvalidArg, "bad host_alloc arguments");
  *ptr = nullptr;
  if (bytes == 0) return succeed();
  if (device_count() == 0) return fail(kErrNoDevice, "no CUDA device available");
  const size_t sz = ((size_t)bytes + kPinnedBucket - 1) / kPinnedBucket * kPinnedBucket;
  {
    std::lock_guard<std::mutex> lk(g_pin_mu);
    auto it = g_pin_free.find(sz);
    if (it != g_pin_free.end()) {
      *ptr = it->second;
      g_pin_free.erase(it);
      g_pin_cached -= sz;
      return succeed();
    }
  }
  B200_CUDA(cudaHostAlloc(ptr, sz, cudaHostAllocPortable), "cudaHostAlloc");
  std::lock_guard<std::mutex> lk(g_pin_mu);
  g_pin_size[*ptr] = sz;
  return succeed();
}

int b200_host_free(void* ptr) {
  if (!ptr) return succeed();
  std::lock_guard<std::mutex> lk(g_pin_mu);
  auto it = g_pin_size.find(ptr);
  if (it == g_pin_size.end()) return fail(kErrInvalidArg, "pointer not from b200_host_alloc");
  const size_t sz = it->second;
  if (g_pin_cached + sz <= kPinnedCacheBytes) {
    g_pin_free.emplace(sz, ptr);
    g_pin_cached += sz;
  } else {
    g_pin_size.erase(it);
    cudaFreeHost(ptr);
  }
  return succeed();
}

// ---------------------------------------------------------------- failure detection
int b200_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  if (limit_ns <= 0) return fail(kErrInvalidArg, "limit_ns must be positive");
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  rc = wait_timeout_selftest((uint64_t)limit_ns, c->status, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, "self-test launch failed") : succeed();
}

// ---------------------------------------------------------------- IPC buffers
// Device buffers another process (another GPU's rank) can map: a rank pushes
// its finished row slabs straight into its peers' output buffers with
// cudaMemcpyAsync, i.e. the copy engines over NVLink, so the transfer needs no
// SMs and overlaps the next slab's GEMM.
int b200_ipc_alloc(void** ptr, int64_t bytes, void* handle_out) {
  if (!ptr || !handle_out || bytes <= 0) return fail(kErrInvalidArg, "bad IPC allocation");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return fail_cuda(e, "cudaMalloc (IPC buffer)");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail_cuda(e, "cudaIpcGetMemHandle");
  }
  memcpy(handle_out, &h, sizeof h);
  *ptr = p;
  return succeed();
}

int b200_ipc_free(void* ptr) {
  if (ptr) B200_CUDA(cudaFree(ptr), "cudaFree (IPC buffer)");
  return succeed();
}

int b200_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(kErrInvalidArg, "bad IPC handle");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  B200_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return succeed();
}

int b200_ipc_close(void* ptr) {
  if (ptr) B200_CUDA(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
  return succeed();
}

// Asynchronous device-to-device copy on `stream`; src and dst may be on
// different GPUs (an IPC-mapped peer buffer), which runs as a peer DMA.
int b200_memcpy_d2d_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes < 0 || (bytes > 0 && (!dst || !src))) return fail(kErrInvalidArg, "bad copy");
  if (bytes)
    B200_CUDA(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice,
                              static_cast<cudaStream_t>(stream)),
              "cudaMemcpyAsync D2D");
  return succeed();
}

int b200_peer_barrier(uint32_t* const* flags, int world, int rank, uint32_t epoch,
                      int64_t timeout_ns, void* stream) {
  if (!flags || world < 1 || world > kMaxPeerRanks || rank < 0 || rank >= world ||
      timeout_ns <= 0)
    return fail(kErrInvalidArg, "peer barrier: flags, 1 <= world <= 8, 0 <= rank < world and "
                                "a positive timeout are required");
  PeerFlags f = {};
  for (int r = 0; r < world; ++r) {
    if (!flags[r]) return fail(kErrInvalidArg, "peer barrier: null flag array");
    f.flags[r] = flags[r];
  }
  f.world = world;
  f.rank = rank;
  DeviceCtx* c = nullptr;
  int rc = current_ctx(&c);
  if (rc) return rc;
  rc = peer_barrier(f, epoch, (uint64_t)timeout_ns, c->status, static_cast<cudaStream_t>(stream));
  return rc ? fail(rc, std::string("peer barrier launch failed: ") + launch_error_text())
            : succeed();
}

int b200_set_gemm_sm_limit(int n) {
  if (n < 0) {
    fail(kErrInvalidArg, "negative SM limit");
    return -1;
  }
  return set_gemm_sm_limit(n);
}

int b200_debug_schedule(int kind, int64_t M, int64_t N, int64_t K, int64_t* out) {
  if ((kind != 0 && kind != 1) || M <= 0 || N <= 0 || K <= 0 || !out)
    return fail(kErrInvalidArg, "bad schedule query");
  if (kind == 0)
    sched_query_f32(M, N, K, out);
  else
    sched_query_i32(M, N, K, out);
  return succeed();
}

int b200_debug_fail_alloc(int n) {
  if (n < 0) return fail(kErrInvalidArg, "n must be >= 0");
  g_fail_alloc_in.store(n);
  return succeed();
}

// ---------------------------------------------------------------- host API
int b200_dense_f32_host(const float* X, int64_t ldx, const float* W, int64_t ldw, const float* b,
                        float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act,
                        float alpha, int ndev) {
  int rc = validate_dense(X, ldx, W, ldw, Y, ldy, M, N, K, act);
  if (rc) return rc;
  ndev = resolve_ndev(ndev);
  if (M < ndev) ndev = M > 0 ? (int)M : 1;
  rc = run_sharded(ndev, M, [&](int dev, int64_t r0, int64_t rows) {
    return dense_host_on_device(dev, X + r0 * ldx, ldx, W, ldw, b, Y + r0 * ldy, ldy, rows, N, K,
                                act, alpha);
  });
  return rc ? rc : succeed();
}

int b200_matmul_i32_host(const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb,
                         const int32_t* bias, int32_t* C, int64_t ldc, int64_t M, int64_t N,
                         int64_t K, int ndev) {
  int rc = validate_dense(A, lda, B, ldb, C, ldc, M, N, K, kActNone);
  if (rc) return rc;
  ndev = resolve_ndev(ndev);
  if (M < ndev) ndev = M > 0 ? (int)M : 1;
  rc = run_sharded(ndev, M, [&](int dev, int64_t r0, int64_t rows) {
    return simple_host_i32_matmul(dev, A + r0 * lda, lda, B, ldb, bias, C + r0 * ldc, ldc, rows,
                                  N, K);
  });
  return rc ? rc : succeed();
}

int b200_bias_act_f32_host(const float* X, int64_t ldx, const float* b, float* Y, int64_t ldy,
                           int64_t M, int64_t N, int act, float alpha) {
  if (M < 0 || N < 0 || act < 0 || act > 2) return fail(kErrInvalidArg, "bad arguments");
  if (M == 0 || N == 0) return succeed();
  if (!X || !Y || ldx < N || ldy < N) return fail(kErrInvalidArg, "null buffer or pitch < N");
  if (device_count() == 0) return fail(kErrNoDevice, "no CUDA device available");
  // Device copies are dense (pitch N); host pitches are honoured by 2-D copies.
  std::vector<float> xs, ys;
  const float* xin = X;
  if (ldx != N) {
    xs.resize(M * N);
    for (int64_t i = 0; i < M; ++i) memcpy(&xs[i * N], X + i * ldx, N * 4);
    xin = xs.data();
  }
  float* yout = Y;
  if (ldy != N) {
    ys.resize(M * N);
    yout = ys.data();
  }
  int rc = elementwise_host(M * N * 4, xin, b ? N * 4 : 0, b, M * N * 4, yout,
                            [&](void* dx, void* dbias, void* dy, cudaStream_t s) {
                              return bias_act_f32(static_cast<float*>(dx), N,
                                                  static_cast<float*>(dbias),
                                                  static_cast<float*>(dy), N, M, N, act, alpha, s);
                            });
  if (rc) return rc;
  if (ldy != N)
    for (int64_t i = 0; i < M; ++i) memcpy(Y + i * ldy, &ys[i * N], N * 4);
  return succeed();
}

int b200_bias_add_i32_host(const int32_t* X, int64_t ldx, const int32_t* b, int32_t* Y,
                           int64_t ldy, int64_t M, int64_t N) {
  if (M < 0 || N < 0) return fail(kErrInvalidArg, "negative dimension");
  if (M == 0 || N == 0) return succeed();
  if (!X || !b || !Y || ldx != N || ldy != N)
    return fail(kErrInvalidArg, "null buffer or non-contiguous rows");
  if (device_count() == 0) return fail(kErrNoDevice, "no CUDA device available");
  int rc = elementwise_host(M * N * 4, X, N * 4, b, M * N * 4, Y,
                            [&](void* dx, void* dbias, void* dy, cudaStream_t s) {
                              return bias_add_i32(static_cast<int32_t*>(dx), N,
                                                  static_cast<int32_t*>(dbias),
                                                  static_cast<int32_t*>(dy), N, M, N, s);
                            });
  return rc ? rc : succeed();
}

int b200_act_f32_host(const float* X, float* Y, int64_t count, int act, float alpha) {
  if (count < 0 || act < 0 || act > 2) return fail(kErrInvalidArg, "bad arguments");
  if (count == 0) return succeed();
  if (!X || !Y) return fail(kErrInvalidArg, "null buffer");
  if (device_count() == 0) return fail(kErrNoDevice, "no CUDA device available");
  int rc = elementwise_host(count * 4, X, 0, nullptr, count * 4, Y,
                            [&](void* dx, void*, void* dy, cudaStream_t s) {
                              return act_f32(static_cast<float*>(dx), static_cast<float*>(dy),
                                             count, act, alpha, s);
                            });
  return rc ? rc : succeed();
}

// ---------------------------------------------------------------- memref ABI
#define M2(n) n##_aligned, n##_off, n##_s0, n##_s1, n##_st0, n##_st1
#define M1(n) n##_aligned, n##_off, n##_s0, n##_st0

static bool memref2_ok(const char* name, void* aligned, int64_t s1, int64_t st0, int64_t st1) {
  if (!aligned) return fail(kErrInvalidArg, std::string(name) + ": null memref"), false;
  if (st1 != 1) return fail(kErrInvalidArg, std::string(name) + ": innermost stride != 1"), false;
  if (st0 < s1) return fail(kErrInvalidArg, std::string(name) + ": row stride < row length"), false;
  return true;
}
static bool memref1_ok(const char* name, void* aligned, int64_t st0) {
  if (!aligned) return fail(kErrInvalidArg, std::string(name) + ": null memref"), false;
  if (st0 != 1) return fail(kErrInvalidArg, std::string(name) + ": stride != 1"), false;
  return true;
}

static void memref_dense_f32(void* x_al, int64_t x_off, int64_t x_s0, int64_t x_s1,
                             int64_t x_st0, int64_t x_st1, void* w_al, int64_t w_off,
                             int64_t w_s0, int64_t w_s1, int64_t w_st0, int64_t w_st1,
                             void* b_al, int64_t b_off, int64_t b_s0, int64_t b_st0, bool has_b,
                             void* y_al, int64_t y_off, int64_t y_s0, int64_t y_s1, int64_t y_st0,
                             int64_t y_st1, int act) {
  if (!memref2_ok("lhs", x_al, x_s1, x_st0, x_st1) || !memref2_ok("rhs", w_al, w_s1, w_st0, w_st1) ||
      !memref2_ok("out", y_al, y_s1, y_st0, y_st1))
    return;
  if (has_b && !memref1_ok("bias", b_al, b_st0)) return;
  if (x_s1 != w_s0 || y_s0 != x_s0 || y_s1 != w_s1 || (has_b && b_s0 != w_s1)) {
    fail(kErrInvalidArg, "memref shapes do not form [M,K]x[K,N]->[M,N]");
    return;
  }
  b200_dense_f32_host(at<float>(x_al, x_off), x_st0, at<float>(w_al, w_off), w_st0,
                      has_b ? at<float>(b_al, b_off) : nullptr, at<float>(y_al, y_off), y_st0,
                      x_s0, w_s1, x_s1, act, 0.0f, 0);
}

void b200_memref_matmul_f32(B200_MEMREF2(A), B200_MEMREF2(B), B200_MEMREF2(C)) {
  memref_dense_f32(M2(A), M2(B), nullptr, 0, 0, 1, false, M2(C), kActNone);
}
void b200_memref_matmul_relu_f32(B200_MEMREF2(A), B200_MEMREF2(B), B200_MEMREF2(C)) {
  memref_dense_f32(M2(A), M2(B), nullptr, 0, 0, 1, false, M2(C), kActRelu);
}
void b200_memref_dense_f32(B200_MEMREF2(X), B200_MEMREF2(W), B200_MEMREF1(b), B200_MEMREF2(Y)) {
  memref_dense_f32(M2(X), M2(W), M1(b), true, M2(Y), kActNone);
}
void b200_memref_dense_relu_f32(B200_MEMREF2(X), B200_MEMREF2(W), B200_MEMREF1(b),
                                B200_MEMREF2(Y)) {
  memref_dense_f32(M2(X), M2(W), M1(b), true, M2(Y), kActRelu);
}

static void memref_i32(void* x_al, int64_t x_off, int64_t x_s0, int64_t x_s1, int64_t x_st0,
                       int64_t x_st1, void* w_al, int64_t w_off, int64_t w_s0, int64_t w_s1,
                       int64_t w_st0, int64_t w_st1, void* b_al, int64_t b_off, int64_t b_s0,
                       int64_t b_st0, bool has_b, void* y_al, int64_t y_off, int64_t y_s0,
                       int64_t y_s1, int64_t y_st0, int64_t y_st1) {
  if (!memref2_ok("lhs", x_al, x_s1, x_st0, x_st1) || !memref2_ok("rhs", w_al, w_s1, w_st0, w_st1) ||
      !memref2_ok("out", y_al, y_s1, y_st0, y_st1))
    return;
  if (has_b && !memref1_ok("bias", b_al, b_st0)) return;
  if (x_s1 != w_s0 || y_s0 != x_s0 || y_s1 != w_s1 || (has_b && b_s0 != w_s1)) {
    fail(kErrInvalidArg, "memref shapes do not form [M,K]x[K,N]->[M,N]");
    return;
  }
  b200_matmul_i32_host(at<int32_t>(x_al, x_off), x_st0, at<int32_t>(w_al, w_off), w_st0,
                       has_b ? at<int32_t>(b_al, b_off) : nullptr, at<int32_t>(y_al, y_off),
                       y_st0, x_s0, w_s1, x_s1, 0);
}

void b200_memref_matmul_i32(B200_MEMREF2(A), B200_MEMREF2(B), B200_MEMREF2(C)) {
  memref_i32(M2(A), M2(B), nullptr, 0, 0, 1, false, M2(C));
}
void b200_memref_dense_i32(B200_MEMREF2(X), B200_MEMREF2(W), B200_MEMREF1(b), B200_MEMREF2(Y)) {
  memref_i32(M2(X), M2(W), M1(b), true, M2(Y));
}

static void memref_bias_act(void* x_al, int64_t x_off, int64_t x_s0, int64_t x_s1, int64_t x_st0,
                            int64_t x_st1, void* b_al, int64_t b_off, int64_t b_s0, int64_t b_st0,
                            bool has_b, void* y_al, int64_t y_off, int64_t y_s0, int64_t y_s1,
                            int64_t y_st0, int64_t y_st1, int act) {
  if (!memref2_ok("input", x_al, x_s1, x_st0, x_st1) || !memref2_ok("out", y_al, y_s1, y_st0, y_st1))
    return;
  if (has_b && !memref1_ok("bias", b_al, b_st0)) return;
  if (y_s0 != x_s0 || y_s1 != x_s1 || (has_b && b_s0 != x_s1)) {
    fail(kErrInvalidArg, "memref shapes do not match");
    return;
  }
  b200_bias_act_f32_host(at<float>(x_al, x_off), x_st0, has_b ? at<float>(b_al, b_off) : nullptr,
                         at<float>(y_al, y_off), y_st0, x_s0, x_s1, act, 0.0f);
}

void b200_memref_bias_add_f32(B200_MEMREF2(X), B200_MEMREF1(b), B200_MEMREF2(Y)) {
  memref_bias_act(M2(X), M1(b), true, M2(Y), kActNone);
}
void b200_memref_bias_relu_f32(B200_MEMREF2(X), B200_MEMREF1(b), B200_MEMREF2(Y)) {
  memref_bias_act(M2(X), M1(b), true, M2(Y), kActRelu);
}
void b200_memref_relu_f32(B200_MEMREF2(X), B200_MEMREF2(Y)) {
  memref_bias_act(M2(X), nullptr, 0, 0, 1, false, M2(Y), kActRelu);
}

// Scalar-returning memref entry points (rank-1 descriptors: alloc, aligned,
// offset, size, stride). On failure they return 0 and set b200_last_status().
static bool memref1_view(const char* name, void* aligned, int64_t st0) {
  return memref1_ok(name, aligned, st0);
}
float b200_memref_dot_f32(B200_MEMREF1(a), B200_MEMREF1(b)) {
  float r = 0.0f;
  if (!memref1_view("lhs", a_aligned, a_st0) || !memref1_view("rhs", b_aligned, b_st0)) return r;
  if (a_s0 != b_s0) return fail(kErrInvalidArg, "dot operands differ in length"), r;
  b200_dot_f32_host(at<float>(a_aligned, a_off), at<float>(b_aligned, b_off), a_s0, &r);
  return r;
}
int32_t b200_memref_dot_i32(B200_MEMREF1(a), B200_MEMREF1(b)) {
  int32_t r = 0;
  if (!memref1_view("lhs", a_aligned, a_st0) || !memref1_view("rhs", b_aligned, b_st0)) return r;
  if (a_s0 != b_s0) return fail(kErrInvalidArg, "dot operands differ in length"), r;
  b200_dot_i32_host(at<int32_t>(a_aligned, a_off), at<int32_t>(b_aligned, b_off), a_s0, &r);
  return r;
}
static float memref_reduce_f32(void* al, int64_t off, int64_t n, int64_t st0, int op,
                               float init) {
  float r = 0.0f;
  if (!memref1_view("input", al, st0)) return r;
  b200_reduce_f32_host(at<float>(al, off), n, op, init, &r);
  return r;
}
float b200_memref_sum_f32(B200_MEMREF1(a)) {
  return memref_reduce_f32(a_aligned, a_off, a_s0, a_st0, kRedSum, 0.0f);
}
float b200_memref_max_f32(B200_MEMREF1(a)) {
  return memref_reduce_f32(a_aligned, a_off, a_s0, a_st0, kRedMax, -INFINITY);
}
float b200_memref_min_f32(B200_MEMREF1(a)) {
  return memref_reduce_f32(a_aligned, a_off, a_s0, a_st0, kRedMin, INFINITY);
}

}  // extern "C"
