/*
 * b200_edsl.h — C ABI of libb200edsl.so, the B200 (sm_100a) implementation of
 * ml-edsl's dense-layer hot path: linalg.matmul and relu(X @ W + b).
 *
 * All entry points are plain C: pointers, sizes and strides in elements, no
 * C++ or torch types. They never throw. Functions returning int return 0
 * (B200_OK) on success or one of the B200_ERR_* codes; the message of the
 * last failure on the calling thread is b200_last_error().
 *
 * Three families:
 *   1. memref-descriptor entry points (b200_memref_*): the exact flattened
 *      signature ml-edsl's JIT'd functions have, so the reference's ctypes
 *      call path (reference: mlir_edsl/backend.py:70-102 builds the
 *      descriptors, :184-191 appends the output descriptor last and calls
 *      ctypes.CFUNCTYPE(None, *types)(ptr)) can call them unchanged. Host
 *      buffers; synchronous; void return — read b200_last_status().
 *   2. host-pointer entry points (*_host): host buffers in and out,
 *      host<->device copies pipelined with compute inside the call, rows
 *      sharded over `ndev` GPUs. Replaces the reference's GPU executor path
 *      (reference: cpp/src/MLIRCompiler.cpp:352-461 executeGPUFunction).
 *   3. device-pointer entry points: device buffers, asynchronous on the given
 *      cudaStream_t (passed as void*, NULL = legacy default stream).
 *
 * Element order is row-major. ld* arguments are row pitches in elements.
 * Activation codes: B200_ACT_NONE, B200_ACT_RELU (arith.maximumf(x, 0):
 * NaN propagates, -0 becomes +0), B200_ACT_LEAKY_RELU (maximumf(x,0) +
 * alpha*minimumf(x,0)) — reference: cpp/src/builders/LinalgBuilder.cpp:207-225.
 */
#ifndef B200_EDSL_H
#define B200_EDSL_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_OK 0
#define B200_ERR_INVALID_ARG 1
#define B200_ERR_CUDA 2
#define B200_ERR_DRIVER 3
#define B200_ERR_NO_DEVICE 4
#define B200_ERR_DEVICE_TIMEOUT 5
#define B200_ERR_OUT_OF_MEMORY 6
#define B200_ERR_TOO_LARGE 7

#define B200_ACT_NONE 0
#define B200_ACT_RELU 1
#define B200_ACT_LEAKY_RELU 2

#define B200_REDUCE_SUM 0  /* acc + x, the tensor_sum body */
#define B200_REDUCE_PROD 1 /* acc * x */
#define B200_REDUCE_MAX 2  /* x > acc ? x : acc, the tensor_max body */
#define B200_REDUCE_MIN 3  /* x < acc ? x : acc, the tensor_min body */

/* ---------------------------------------------------------------- runtime */

/* Library version string. */
const char* b200_version(void);

/* Message of the last failing call on this thread ("" if none). Replaces the
 * reference's std::runtime_error / checkCU messages
 * (reference: cpp/src/MLIRExecutor.cpp:160-167). */
const char* b200_last_error(void);

/* Status code of the last call on this thread; the only error channel of the
 * void b200_memref_* entry points. */
int b200_last_status(void);

/* Number of CUDA devices visible (0 without a GPU or driver). */
int b200_device_count(void);

/* Number of kernels this library has launched in this process. */
long long b200_launch_count(void);

/* Default device count used by the b200_memref_* entry points (1 initially;
 * the B200_DEVICES environment variable overrides the initial value). */
int b200_set_default_devices(int ndev);
int b200_get_default_devices(void);

/* Frees every device buffer and stream the runtime caches. */
int b200_release(void);

/* ------------------------------------------------- device-pointer entry points */

/* Y = act(X @ W + b) in f32 with 3xTF32 tensor-core arithmetic.
 * X[M,K] (pitch ldx), W[K,N] (pitch ldw), b[N] or NULL, Y[M,N] (pitch ldy).
 * Scratch for the tf32 hi/lo operand split (and, for problems with too few
 * 128x256 output tiles to fill the GPU, the split-K partial sums) comes from a
 * buffer the runtime caches per (device, stream).
 * Replaces: linalg.fill+matmul (reference: cpp/src/builders/LinalgBuilder.cpp:106-139),
 * bias generic (:301-339), activation generic (:180-239). */
int b200_dense_f32(const float* X, int64_t ldx, const float* W, int64_t ldw, const float* b,
                   float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act, float alpha,
                   void* stream);

/* Number of K splits b200_dense_f32 uses for an M x N x K problem (1 = no
 * split; otherwise the GEMM writes partial sums and one extra HBM-bound kernel
 * adds them in fixed order, so results are deterministic). */
int b200_dense_f32_splits(int64_t M, int64_t N, int64_t K);

/* Kernel launches of one b200_dense_f32 call: the operand split, the GEMM,
 * and the cut-tile reduction when the problem is split (0 for an empty
 * output, 1 for K == 0; -1 for negative sizes). No counterpart in the reference (its GPU path always launches fill,
 * matmul and bias+relu: cpp/src/MLIRLowering.cpp:495-718). */
int b200_dense_f32_launches(int64_t M, int64_t N, int64_t K);

/* Same as b200_dense_f32 with caller-provided scratch of at least
 * b200_dense_f32_workspace_bytes(M, N, K) bytes (256-byte aligned). */
int64_t b200_dense_f32_workspace_bytes(int64_t M, int64_t N, int64_t K);
int b200_dense_f32_ws(const float* X, int64_t ldx, const float* W, int64_t ldw, const float* b,
                      float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act,
                      float alpha, void* workspace, int64_t workspace_bytes, void* stream);

/* Weight cache. b200_weights_register declares the f32 weight matrix
 * W[K,N] (row pitch ldw floats) at host address W unchanged until it is
 * registered again with another `version` (or shape) or released. The
 * host-buffer entry points (b200_dense_f32_host and the memref entry points)
 * that get this W with this shape and pitch then keep its device copy and
 * its tf32 split on each GPU they run on, made at first use, instead of
 * copying and splitting W in every call as the reference's GPU path does
 * (reference: cpp/src/MLIRCompiler.cpp:368-376, cuMemAlloc + cuMemcpyHtoD
 * of every argument per call). Registering the same (W, ldw, K, N, version)
 * again is a no-op; a new version drops the device copies after the GPUs
 * have finished the work queued so far. b200_weights_release frees them on
 * every GPU (same wait) and forgets W; neither may overlap a call that uses
 * W on another thread. b200_weights_device returns the current device's copy
 * (rows of N floats, pitch N), uploading it if needed; b200_dense_f32 and its
 * device-pointer siblings given that address as W reuse the kept split. */
int b200_weights_register(const float* W, int64_t ldw, int64_t K, int64_t N, uint64_t version);
int b200_weights_release(const float* W);
int b200_weights_device(const float* W, const float** dW);

/* Y = act(X @ W + b) like b200_dense_f32, for callers that must not
 * allocate device memory while they run (for example a serving process whose
 * framework allocator already holds nearly all of HBM, or a latency-bound loop
 * that cannot absorb cudaMalloc/cudaFree synchronisation). This entry point
 * has no counterpart in the reference.
 * The call allocates nothing: its scratch is a fixed 64 MiB device array that
 * every GPU loading this library holds until the process exits. Problems
 * needing more than that (8 * (M + N) * roundup(K, 8) bytes plus alignment)
 * fail with B200_ERR_TOO_LARGE. All calls on a device share the array, so
 * calls that overlap on the GPU race; the call synchronises `stream` before
 * it returns. The first call on a device resolves the array's device address
 * (cudaGetSymbolAddress with that device current); make that first call
 * before any stream capture. */
int b200_dense_f32_noalloc(const float* X, int64_t ldx, const float* W, int64_t ldw,
                           const float* b, float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                           int act, float alpha, void* stream);

/* C = A @ B (+ bias) in i32, wrapping modulo 2^32 (arith.muli/addi).
 * Replaces: linalg.matmul on i32 (reference: cpp/src/builders/LinalgBuilder.cpp:106-139). */
int b200_matmul_i32(const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb,
                    const int32_t* bias, int32_t* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                    void* stream);

/* Y = act(X + b) (b may be NULL). Replaces the unfused bias_add / relu /
 * leaky_relu generics (reference: cpp/src/builders/LinalgBuilder.cpp:180-239,301-339). */
int b200_bias_act_f32(const float* X, int64_t ldx, const float* b, float* Y, int64_t ldy,
                      int64_t M, int64_t N, int act, float alpha, void* stream);

/* Y[i] = act(X[i]) over `count` contiguous elements (any rank). */
int b200_act_f32(const float* X, float* Y, int64_t count, int act, float alpha, void* stream);

/* Y = X + b in i32 (wrapping). */
int b200_bias_add_i32(const int32_t* X, int64_t ldx, const int32_t* b, int32_t* Y, int64_t ldy,
                      int64_t M, int64_t N, void* stream);

/* Synchronizes `stream` and returns B200_ERR_DEVICE_TIMEOUT if a kernel of
 * this library gave up a bounded wait since the last check, else B200_OK or
 * B200_ERR_CUDA. */
int b200_stream_sync(void* stream);

/* tf32 operand split used by the dense kernel, exposed so that a weight
 * matrix can be split once and reused across calls:
 *   b200_tf32_split_rows:      X[M,K] -> hi[M,Kp], lo[M,Kp]
 *   b200_tf32_split_transpose: W[K,N] -> hiT[N,Kp], loT[N,Kp] (K-major)
 * with Kp = K rounded up to a multiple of 8 (32-byte rows; pad columns zero).
 * hi and lo are exact tf32 values: hi is x with its low 13 mantissa bits
 * cleared, lo the remainder truncated to tf32, so hi + lo is x to 2^-21
 * relative (Inf/NaN travel in hi). Outputs must be 16-byte aligned. */
int b200_tf32_split_rows(const float* X, int64_t ldx, int64_t M, int64_t K, float* hi, float* lo,
                         void* stream);
int b200_tf32_split_transpose(const float* W, int64_t ldw, int64_t K, int64_t N, float* hiT,
                              float* loT, void* stream);

/* Y = act(Xhi/Xlo @ WhiT/WloT^T + b) on pre-split operands (the tcgen05
 * kernel alone). Same arithmetic as b200_dense_f32. */
int b200_gemm_tf32x3_presplit(const float* xhi, const float* xlo, const float* whiT,
                              const float* wloT, const float* b, float* Y, int64_t ldy, int64_t M,
                              int64_t N, int64_t K, int act, float alpha, void* stream);

/* Y = act(X @ W + b) with W given pre-split (b200_tf32_split_transpose):
 * the weight-stationary form of b200_dense_f32, which skips the W split on
 * every call. X is split by the HBM-bound split pass into runtime scratch
 * (or, with B200_FUSE_A=1 and 16-byte aligned X rows, inside the GEMM);
 * few-tile problems add a split-K reduction. */
int b200_dense_f32_wsplit(const float* X, int64_t ldx, const float* whiT, const float* wloT,
                          const float* b, float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                          int act, float alpha, void* stream);

/* Device buffers on the current device, from its stream-ordered memory pool
 * (allocation and release are ordered on the legacy default stream; freed
 * blocks stay cached in the pool). Copies are synchronous. */
int b200_malloc(void** ptr, int64_t bytes);
int b200_free(void* ptr);
int b200_memcpy_h2d(void* dst, const void* src, int64_t bytes);
int b200_memcpy_d2h(void* dst, const void* src, int64_t bytes);

/* 1-D reductions and dot products, result in one device element `out`:
 *   out = init (op) x[0] (op) x[1] ... ; dot: out = sum_i a[i]*b[i].
 * Two-pass and deterministic. f32 sums/products/dots are tree-ordered (not
 * the sequential order); max/min equal the sequential fold with the
 * reference's bodies (NaN elements never win). i32 sums/products wrap.
 * Replaces: linalg.dot (reference: cpp/src/builders/LinalgBuilder.cpp:66-104)
 * and linalg.reduce with the tensor_sum / tensor_max / tensor_min bodies
 * (cpp/src/builders/LinalgBuilder.cpp:241-279, mlir_edsl/ops/linalg.py:104-175). */
int b200_reduce_f32(const float* x, int64_t n, int op, float init, float* out, void* stream);
int b200_reduce_i32(const int32_t* x, int64_t n, int op, int32_t init, int32_t* out,
                    void* stream);
int b200_dot_f32(const float* a, const float* b, int64_t n, float* out, void* stream);
int b200_dot_i32(const int32_t* a, const int32_t* b, int64_t n, int32_t* out, void* stream);

/* Failure detection without a GPU fault. Every wait inside this library's
 * kernels is bounded; one that runs out records a code in the device status
 * word and the kernel returns, so the context stays usable and the next
 * b200_stream_sync() reports B200_ERR_DEVICE_TIMEOUT (the reference has no
 * device-side detection; its checkCU turns CUDA errors into exceptions,
 * reference: cpp/src/MLIRExecutor.cpp:160-167).
 * b200_selftest_wait_timeout launches one kernel whose wait can never be
 * satisfied, with a limit of limit_ns, to exercise that path.
 * b200_debug_fail_alloc(n): the n-th next device allocation of the runtime
 * fails with B200_ERR_OUT_OF_MEMORY (0 disables), host-side fault injection
 * (the reference's analogue is inject_test_failure,
 * reference: cpp/src/MLIRCompiler.cpp:331-348). */
int b200_selftest_wait_timeout(int64_t limit_ns, void* stream);
int b200_debug_fail_alloc(int n);

/* b200_dense_f32_chain: b200_dense_f32 for stacked layers kept on the
 * device. Xlo (optional): X's tf32 lo part with row pitch roundup(K, 8), as
 * the previous layer wrote it to its Ylo, so that X is not split again (X and
 * Xlo rows 16-byte aligned). Ylo (optional, pitch ldylo >= N): the epilogue
 * also stores the tf32 lo part of Y (after bias and activation) for the next
 * layer. The results equal b200_dense_f32's bit for bit. Replaces the
 * reference's per-layer host round trips of stacked dense nets
 * (tests/linalg/test_binary_op_execution.py:223-268); no direct counterpart. */
int b200_dense_f32_chain(const float* X, int64_t ldx, const float* Xlo, const float* W,
                         int64_t ldw, const float* b, float* Y, int64_t ldy, float* Ylo,
                         int64_t ldylo, int64_t M, int64_t N, int64_t K, int act, float alpha,
                         void* stream);

/* b200_dense_f32_peers: b200_dense_f32 that also stores every final value
 * of Y into npeers (0..7) other output buffers, at the same element offsets
 * with the same pitch ldy: peer_y is a host array of device addresses, in
 * practice the rows of this call inside other GPUs' output buffers mapped
 * with b200_ipc_open. The GEMM epilogue (and the cut-tile reduction) write
 * them with ordinary stores over NVLink as tiles finish, so a row-sharded
 * layer assembles its full result on every GPU during the GEMM itself. The
 * writes are complete when the call's work on `stream` is; the caller orders
 * them against the peers, on the stream with b200_peer_barrier before and
 * after the call. No counterpart in the reference, whose results never leave
 * one device. */
int b200_dense_f32_peers(const float* X, int64_t ldx, const float* W, int64_t ldw,
                         const float* b, float* Y, int64_t ldy, float* const* peer_y, int npeers,
                         int64_t M, int64_t N, int64_t K, int act, float alpha, void* stream);

/* b200_dense_f32_multicast: the gathered dense layer through NVSwitch
 * multicast (NVLS). mc_y is the multicast address of this call's Y rows (a
 * multicast object every rank's output buffer is bound to, at the same
 * offsets and pitch ldy); the GEMM epilogue (and the cut-tile reduction)
 * stores every final value once with multimem.st and the switch writes it
 * into every GPU's copy, so each value crosses this GPU's NVLink ports once
 * whatever the number of peers. K must be > 0. Ordering against the peers as
 * for b200_dense_f32_peers. No counterpart in the reference. */
int b200_dense_f32_multicast(const float* X, int64_t ldx, const float* W, int64_t ldw,
                             const float* b, float* Y, int64_t ldy, float* mc_y, int64_t M,
                             int64_t N, int64_t K, int act, float alpha, void* stream);

/* Stream-ordered barrier of the `world` GPUs (<= 8) of a gathered call, as
 * one small kernel on `stream`: rank `rank` stores `epoch` into its slot of
 * every peer's flag array (after a system-scope fence, so its earlier stores
 * into peer memory land first) and waits until every peer has stored `epoch`
 * (or a later epoch, modulo 2^32) into its own flag array. flags[r] is rank
 * r's array of `world` 32-bit slots as addressed from this device (its own,
 * or a peer's mapped with b200_ipc_open), zero before the first barrier;
 * every rank passes the same epoch sequence. A wait longer than timeout_ns
 * gives up: b200_stream_sync then returns B200_ERR_DEVICE_TIMEOUT and the
 * context stays usable. No counterpart in the reference. */
int b200_peer_barrier(uint32_t* const* flags, int world, int rank, uint32_t epoch,
                      int64_t timeout_ns, void* stream);

/* Cross-process device buffers for the all-gather of a row-sharded result:
 * b200_ipc_alloc allocates `bytes` on the current device and writes its
 * 64-byte CUDA IPC handle to handle_out; another rank maps it with
 * b200_ipc_open and unmaps it with b200_ipc_close; b200_ipc_free releases it.
 * b200_memcpy_d2d_async copies on `stream`, also into a mapped peer buffer
 * (a peer DMA over NVLink on the copy engines). These have no counterpart in
 * the reference, whose results never leave one device. */
int b200_ipc_alloc(void** ptr, int64_t bytes, void* handle_out);
int b200_ipc_free(void* ptr);
int b200_ipc_open(const void* handle, void** ptr);
int b200_ipc_close(void* ptr);
int b200_memcpy_d2d_async(void* dst, const void* src, int64_t bytes, void* stream);

/* b200_set_gemm_sm_limit(n): the f32 GEMM's persistent grid (and its work
 * schedule) uses at most n SMs from the next call on, leaving the rest free for
 * concurrent kernels such as an NCCL all-gather of finished row slabs; 0 = all
 * SMs. Returns the previous limit (process-wide), or -1 with
 * B200_ERR_INVALID_ARG recorded for n < 0. No counterpart in the reference. */
int b200_set_gemm_sm_limit(int n);

/* b200_debug_schedule(kind, M, N, K, out): the work schedule the persistent
 * GEMM would use on the current device (148 SMs without one); kind 0 = the
 * f32 dense layer, 1 = the i32 matmul. out[0..7] = tiles_m, tiles_n, whole
 * (tiles over all of K), rest (tiles cut into K pieces), pieces, k-blocks per
 * tile, k-blocks per piece, work units. Returns B200_OK, or
 * B200_ERR_INVALID_ARG for a bad kind or non-positive dimensions. Test and
 * tuning aid with no counterpart in the reference. */
int b200_debug_schedule(int kind, int64_t M, int64_t N, int64_t K, int64_t* out);

/* Page-locked host memory from a runtime pool (blocks are cached after
 * b200_host_free and reused). Results copied back into such buffers move at
 * full PCIe speed; the Python frontend returns its arrays in them. */
int b200_host_alloc(void** ptr, int64_t bytes);
int b200_host_free(void* ptr);

/* --------------------------------------------------- host-pointer entry points */

/* Host buffers; synchronous. Rows of X/Y are sharded over `ndev` devices
 * (0 = default device count; 1 = the calling thread's current device,
 * otherwise devices 0..ndev-1); W and b are replicated. Within a device the
 * rows are processed in slabs so host->device copies, compute and
 * device->host copies overlap. */
int b200_dense_f32_host(const float* X, int64_t ldx, const float* W, int64_t ldw, const float* b,
                        float* Y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act,
                        float alpha, int ndev);

int b200_matmul_i32_host(const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb,
                         const int32_t* bias, int32_t* C, int64_t ldc, int64_t M, int64_t N,
                         int64_t K, int ndev);

int b200_bias_act_f32_host(const float* X, int64_t ldx, const float* b, float* Y, int64_t ldy,
                           int64_t M, int64_t N, int act, float alpha);

int b200_bias_add_i32_host(const int32_t* X, int64_t ldx, const int32_t* b, int32_t* Y,
                           int64_t ldy, int64_t M, int64_t N);

int b200_act_f32_host(const float* X, float* Y, int64_t count, int act, float alpha);

/* Host buffers in, host scalar `*result` out (synchronous). */
int b200_reduce_f32_host(const float* x, int64_t n, int op, float init, float* result);
int b200_reduce_i32_host(const int32_t* x, int64_t n, int op, int32_t init, int32_t* result);
int b200_dot_f32_host(const float* a, const float* b, int64_t n, float* result);
int b200_dot_i32_host(const int32_t* a, const int32_t* b, int64_t n, int32_t* result);

/* ------------------------------------------------- memref-descriptor entry points
 * A rank-2 memref is passed as 7 arguments
 *   (void* allocated, void* aligned, int64 offset, int64 size0, int64 size1,
 *    int64 stride0, int64 stride1)
 * and a rank-1 memref as 5: (allocated, aligned, offset, size0, stride0).
 * The output memref comes last and must be fully allocated by the caller
 * (reference: mlir_edsl/backend.py:37-63 _make_output_descriptor). The
 * innermost stride must be 1. Rows are sharded over b200_get_default_devices().
 */
#define B200_MEMREF2(n) \
  void *n##_alloc, void *n##_aligned, int64_t n##_off, int64_t n##_s0, int64_t n##_s1, \
      int64_t n##_st0, int64_t n##_st1
#define B200_MEMREF1(n) \
  void *n##_alloc, void *n##_aligned, int64_t n##_off, int64_t n##_s0, int64_t n##_st0

/* C = A @ B, f32 (21 arguments). */
void b200_memref_matmul_f32(B200_MEMREF2(A), B200_MEMREF2(B), B200_MEMREF2(C));
/* C = relu(A @ B), f32. */
void b200_memref_matmul_relu_f32(B200_MEMREF2(A), B200_MEMREF2(B), B200_MEMREF2(C));
/* Y = X @ W + b, f32 (26 arguments). */
void b200_memref_dense_f32(B200_MEMREF2(X), B200_MEMREF2(W), B200_MEMREF1(b), B200_MEMREF2(Y));
/* Y = relu(X @ W + b), f32 (26 arguments). */
void b200_memref_dense_relu_f32(B200_MEMREF2(X), B200_MEMREF2(W), B200_MEMREF1(b),
                                B200_MEMREF2(Y));
/* C = A @ B, i32 wrapping. */
void b200_memref_matmul_i32(B200_MEMREF2(A), B200_MEMREF2(B), B200_MEMREF2(C));
/* Y = X @ W + b, i32 wrapping. */
void b200_memref_dense_i32(B200_MEMREF2(X), B200_MEMREF2(W), B200_MEMREF1(b), B200_MEMREF2(Y));
/* Y = X + b, f32 (reference library_call "bias_add"). */
void b200_memref_bias_add_f32(B200_MEMREF2(X), B200_MEMREF1(b), B200_MEMREF2(Y));
/* Y = relu(X + b), f32 (the fused bias_add+relu generic). */
void b200_memref_bias_relu_f32(B200_MEMREF2(X), B200_MEMREF1(b), B200_MEMREF2(Y));
/* Y = relu(X), f32 rank 2 (reference library_call "relu"). */
void b200_memref_relu_f32(B200_MEMREF2(X), B200_MEMREF2(Y));

/* Scalar-returning functions (a JIT'd `-> f32` / `-> i32` function returns
 * its scalar; reference: mlir_edsl/backend.py:192-194): dot(a, b) with two
 * rank-1 descriptors (10 arguments), tensor_sum / tensor_max / tensor_min
 * with one (5 arguments). On failure they return 0; see b200_last_status(). */
float b200_memref_dot_f32(B200_MEMREF1(a), B200_MEMREF1(b));
int32_t b200_memref_dot_i32(B200_MEMREF1(a), B200_MEMREF1(b));
float b200_memref_sum_f32(B200_MEMREF1(a));
float b200_memref_max_f32(B200_MEMREF1(a));
float b200_memref_min_f32(B200_MEMREF1(a));

#ifdef __cplusplus
}
#endif

#endif /* B200_EDSL_H */
