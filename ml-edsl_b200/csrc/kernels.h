// Internal interface between the CUDA kernel files and the host runtime.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

// Status codes shared with the public C-ABI (include/b200_edsl.h).
enum Status : int {
  kOk = 0,
  kErrInvalidArg = 1,
  kErrCuda = 2,
  kErrDriver = 3,
  kErrNoDevice = 4,
  kErrDeviceTimeout = 5,
  kErrOutOfMemory = 6,
  kErrTooLarge = 7,
};

enum Act : int { kActNone = 0, kActRelu = 1, kActLeakyRelu = 2 };
enum RedOp : int { kRedSum = 0, kRedProd = 1, kRedMax = 2, kRedMin = 3 };

// Number of kernels this library has launched (process-wide).
void count_launch();

// Records an error for b200_last_error()/b200_last_status() on this thread
// and returns `code`; report_ok() records success and returns kOk.
int report_error(int code, const char* msg);
int report_ok();

// Status of the kernel launch just queued on this thread: kOk, or kErrCuda
// with the CUDA error's text kept for launch_error_text() (the error is
// cleared). driver_failure() keeps the text of a failed driver call (tensor
// map encoding) the same way and returns kErrDriver.
int launch_result(cudaError_t e = cudaGetLastError());
int driver_failure(const char* what, int code);
const char* launch_error_text();

// ---- peer-GPU barrier of gathered calls (peer.cu)
// flags[r]: rank r's flag array (world 32-bit slots) as addressed from this
// device (its own array, or a peer's through a CUDA IPC mapping).
constexpr int kMaxPeerRanks = 8;
struct PeerFlags {
  uint32_t* flags[kMaxPeerRanks];
  int world;
  int rank;
};
int peer_barrier(const PeerFlags& f, uint32_t epoch, uint64_t limit_ns, int* status,
                 cudaStream_t stream);

// ---- 3xTF32 GEMM (gemm_tf32x3.cu)
// Row pitch (floats) of every tf32 hi/lo split buffer of K columns: K
// rounded up to 8, so that every row starts on a 32-byte L2 sector and each
// 64-byte TMA row segment of a K-major operand covers exactly two sectors
// (with a pitch of 4 mod 8 floats, every other row straddles three).
inline int64_t split_pitch(int64_t K) { return (K + 7) & ~int64_t(7); }
// Gathered dense results: the f32 epilogue can also store every final value
// into up to kMaxEpiloguePeers other GPUs' output buffers. The peer bases
// (device addresses valid on the launching device, same element offsets and
// pitch as Y) apply to the dense launches this thread makes while an
// EpiloguePeersScope is alive.
constexpr int kMaxEpiloguePeers = 7;
// With `mc` (the NVSwitch multicast address of Y) set instead, every final
// value is stored once with multimem.st and reaches Y and all peers' copies.
void set_epilogue_peers(float* const* peers, int n, float* mc = nullptr);
struct EpiloguePeersScope {
  EpiloguePeersScope(float* const* peers, int n, float* mc = nullptr) {
    set_epilogue_peers(peers, n, mc);
  }
  ~EpiloguePeersScope() { set_epilogue_peers(nullptr, 0, nullptr); }
  EpiloguePeersScope(const EpiloguePeersScope&) = delete;
  EpiloguePeersScope& operator=(const EpiloguePeersScope&) = delete;
};
int64_t dense_f32_workspace_bytes(int64_t M, int64_t N, int64_t K);
int split_x_f32(const float* X, int64_t ldx, int64_t M, int64_t K, float* xhi, float* xlo,
                cudaStream_t stream);
int split_w_f32(const float* W, int64_t ldw, int64_t K, int64_t N, float* whiT, float* wloT,
                cudaStream_t stream);
// Split-K (few-tile problems): splits chosen by a wave-count cost model;
// partials scratch of splitk_partials_bytes() (0 when splits == 1).
int choose_splits(int64_t M, int64_t N, int64_t K);
// Kernel launches of one f32 GEMM call (1, or 2 with the cut-tile reduction).
int gemm_f32_launches(int64_t M, int64_t N, int64_t K);
// Cap on the SMs the f32 GEMM's persistent grid occupies (0: all); returns the
// previous cap.
int set_gemm_sm_limit(int n);
// Schedule of the persistent GEMMs (tiles_m, tiles_n, whole, rest, pieces,
// kb, kbp, units) for b200_debug_schedule.
void sched_query_f32(int64_t M, int64_t N, int64_t K, int64_t* out);
void sched_query_i32(int64_t M, int64_t N, int64_t K, int64_t* out);
int64_t splitk_partials_bytes(int64_t M, int64_t N, int64_t K);
int gemm_tf32x3_splitk(const float* xhi, const float* xlo, const float* whiT, const float* wloT,
                       int64_t M, int64_t N, int64_t K, const float* bias, float* Y, int64_t ldy,
                       int act, float alpha, int splits, float* partials, int* status,
                       cudaStream_t stream, float* ylo = nullptr, int64_t ldylo = 0);
// Both splits in one launch: X -> (xhi,) xlo (xhi == nullptr: lo only) and
// W -> whiT, wloT.
int split_xw_f32(const float* X, int64_t ldx, int64_t M, const float* W, int64_t ldw,
                 int64_t K, int64_t N, float* xhi, float* xlo, float* whiT, float* wloT,
                 cudaStream_t stream);

// Raw-X A operand (X rows 16-byte aligned: x_raw_ok): the split pass
// writes only the lo part [M, Kp]; the GEMM reads X itself as the hi part.
int split_x_lo_f32(const float* X, int64_t ldx, int64_t M, int64_t K, float* xlo,
                   cudaStream_t stream);
// ylo (optional, pitch ldylo): the epilogue also stores the tf32 lo part of
// every final value, i.e. the next layer's pre-split A_lo.
int gemm_tf32x3_xraw(const float* X, int64_t ldx, const float* xlo, const float* whiT,
                     const float* wloT, int64_t M, int64_t N, int64_t K, const float* bias,
                     float* Y, int64_t ldy, int act, float alpha, int splits, float* partials,
                     int* status, cudaStream_t stream, float* ylo = nullptr,
                     int64_t ldylo = 0);

// MN-major B operand: the GEMM reads the row-major W itself as B_hi and a
// row-major lo part W_lo [K, Np] (Np = roundup(N, 4)) as B_lo. w_mn_ok:
// W rows 16-byte aligned, N % 32 == 0, M <= 4096 and B200_W_MN not 0. split_lo_xw_f32 writes X's lo (and hi when
// xhi != nullptr; X may be null for W alone) and W_lo in one launch.
bool w_mn_ok(const float* W, int64_t ldw, int64_t M, int64_t N);
int64_t w_lo_mn_bytes(int64_t K, int64_t N);
int split_lo_xw_f32(const float* X, int64_t ldx, int64_t M, int64_t K, float* xhi, float* xlo,
                    const float* W, int64_t ldw, int64_t N, float* wlo, cudaStream_t stream);
// xa: raw X (pitch ldx) or its pre-split hi part (pitch Kp); xlo pitch Kp.
int gemm_tf32x3_wmn(const float* xa, const float* xlo, int64_t ldx, const float* W, int64_t ldw,
                    const float* wlo, int64_t M, int64_t N, int64_t K, const float* bias,
                    float* Y, int64_t ldy, int act, float alpha, int splits, float* partials,
                    int* status, cudaStream_t stream, float* ylo = nullptr,
                    int64_t ldylo = 0);

// True when X (pitch ldx) can be read as the raw tf32 hi operand: 16-byte
// aligned rows (TMA strides).
bool x_raw_ok(const float* X, int64_t ldx);
int gemm_tf32x3_presplit(const float* xhi, const float* xlo, const float* whiT,
                         const float* wloT, int64_t M, int64_t N, int64_t K, const float* bias,
                         float* Y, int64_t ldy, int act, float alpha, int* status,
                         cudaStream_t stream);

// Failure-detection self-test (a bounded wait that always runs out).
int wait_timeout_selftest(uint64_t limit_ns, int* status, cudaStream_t stream);

// ---- i32 GEMM (gemm_i32.cu): C = A*B mod 2^32
int gemm_i32(const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb, int32_t* C,
             int64_t ldc, int64_t M, int64_t N, int64_t K, const int32_t* bias,
             cudaStream_t stream);

// ---- i32 GEMM on the tensor cores (gemm_i32_tc.cu): byte-sliced
// tcgen05.mma.kind::i8 products, exact modulo 2^32. ws: at least
// gemm_i32_tc_workspace_bytes(M, N, K) bytes, 256-byte aligned. K > 0.
// B200_I32_TC=0 selects the CUDA-core kernel (i32_tensor_core_enabled).
bool i32_tensor_core_enabled();
int choose_splits_i32(int64_t M, int64_t N, int64_t K);
int64_t gemm_i32_tc_workspace_bytes(int64_t M, int64_t N, int64_t K);
int gemm_i32_tc(const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb,
                const int32_t* bias, int32_t* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                void* ws, int* status, cudaStream_t stream);

// ---- elementwise (elementwise.cu)
int bias_act_f32(const float* X, int64_t ldx, const float* b, float* Y, int64_t ldy, int64_t M,
                 int64_t N, int act, float alpha, cudaStream_t stream);
int act_f32(const float* X, float* Y, int64_t count, int act, float alpha, cudaStream_t stream);
int bias_add_i32(const int32_t* X, int64_t ldx, const int32_t* b, int32_t* Y, int64_t ldy,
                 int64_t M, int64_t N, cudaStream_t stream);
int fill_bias_act_f32(const float* b, float* Y, int64_t ldy, int64_t M, int64_t N, int act,
                      float alpha, cudaStream_t stream);

// ---- 1-D reductions / dot (reduce.cu). `y` non-null: dot product (op = sum).
// `scratch` holds reduce_scratch_bytes(); `out` is one device element.
int64_t reduce_scratch_bytes();
int reduce_f32(const float* x, const float* y, int64_t n, int op, float init, float* out,
               void* scratch, cudaStream_t st);
int reduce_i32(const int32_t* x, const int32_t* y, int64_t n, int op, int32_t init, int32_t* out,
               void* scratch, cudaStream_t st);

}  // namespace b200
