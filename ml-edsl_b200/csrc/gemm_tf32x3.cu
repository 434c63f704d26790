// f32 GEMM with fused bias + activation epilogue on the sm_100a tensor cores.
//
//   Y[M,N] = act( sum_k X[m,k] * W[k,n]  (+ b[n]) )
//
// This is the B200 implementation of the reference's
//   linalg.fill(0) -> linalg.matmul -> linalg.generic{bias_add} -> linalg.generic{relu}
// chain (reference: cpp/src/builders/LinalgBuilder.cpp:106-139 matmul with
// zero init, :301-339 bias broadcast generic, :180-239 relu/leaky_relu
// generic; fused into one pass by linalg-fuse-elementwise-ops,
// cpp/src/MLIRLowering.cpp:355).
//
// Precision: "3xTF32". Each f32 operand x is split into two tf32-exact parts
// x = hi + lo (hi = x with the low 13 mantissa bits cleared, lo = the
// remainder truncated the same way). The tensor core then accumulates
// hi*hi + hi*lo + lo*hi in f32 (the lo*lo term is below f32 resolution).
// The split runs in two HBM-bound pre-pass kernels that also
//   * transpose W to K-major (both UMMA operands are K-major), and
//   * pad the row pitch to a multiple of 8 floats (TMA needs 16-byte strides;
//     32-byte rows keep each 64-byte row segment within two L2 sectors),
// which is how ragged shapes such as K=1001 reach the TMA path.
//
// Accumulation: the tensor core adds into its f32 accumulator with
// round-toward-zero, so a single TMEM accumulator over all of K drifts
// linearly in K (measured 3.3e-3 at K=4096 for |x| <= 1, against ~1e-5 for
// round-to-nearest). The kernel therefore accumulates each 256-wide slice of
// K in TMEM ("chunk") and promotes it into f32 registers with ordinary
// round-to-nearest adds; two TMEM chunk buffers let the MMAs of chunk c+1 run
// while the epilogue warps drain chunk c.
//
// Main kernel (persistent: one CTA per SM walks 128 x 256 output tiles, or
// (tile, K-split) units, in a grouped raster; 320 threads):
//   warp 0      TMA producer: 4 tiles (A_hi, A_lo, B_hi, B_lo) per k-block
//               into a shared-memory ring: 4 stages of 48 KB (BK = 16,
//               64-byte swizzle).
//   warp 1      allocates 512 TMEM columns (2 chunk buffers); lane 0 issues 3
//               tcgen05.mma per 8-wide k-step and frees ring stages and chunk
//               buffers with tcgen05.commit.
//   warps 2-9   epilogue: each thread owns one row x 128 columns of the tile
//               in registers, adds every chunk (tcgen05.ld), then applies
//               bias and activation (arith.maximumf semantics: NaN
//               propagates, -0 -> +0) and stores.
#include <cuda.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <atomic>
#include <type_traits>
#include <utility>
#include <cstdlib>
#include <cstring>
#include <cstdint>
#include "ptx.cuh"
#include "sched.cuh"
#include "kernels.h"

namespace b200 {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kEpiWarps = 8;  // 2 warps per TMEM lane quarter, one per column half
constexpr int kTmemCols = 2 * kBN;  // two chunk accumulators of 128 x 256 f32
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kGroupM = 16;  // tile raster: 16 M-tiles share each N sweep
// K per TMEM partial-sum chunk (compile-time; -DB200_CHUNK_K=128 builds the
// narrower variant). 256 lets the next tile's MMAs run further ahead of the
// epilogue; the error stays below that of a sequential f32 FMA loop.
#ifndef B200_CHUNK_K
#define B200_CHUNK_K 256
#endif
constexpr int kChunkK = B200_CHUNK_K;

// Shared-memory ring configuration. BK floats of K per stage; the rows of
// each operand tile are BK*4 bytes, which selects the TMA / UMMA swizzle:
// 128 B rows -> SWIZZLE_128B (UMMA layout 2), 64 B rows -> SWIZZLE_64B (4).
// Layout: [Stages x (A_hi, A_lo, B_hi, B_lo)][barriers/flags][bias tile],
// base aligned to 1 KB.
template <int BK_, int STAGES_>
struct RingCfg {
  static constexpr int BK = BK_;
  static constexpr int Stages = STAGES_;
  static constexpr int ATileBytes = kBM * BK * 4;
  static constexpr int BTileBytes = kBN * BK * 4;
  static constexpr int StageBytes = 2 * ATileBytes + 2 * BTileBytes;
  static constexpr int ChunkKB = kChunkK / BK;  // k-blocks per TMEM chunk
  static constexpr uint32_t UmmaLayout = BK == 32 ? 2u : 4u;
  static constexpr uint32_t SBO = 8 * BK * 4;  // 8-row core-matrix group stride
  static constexpr int BarOffset = Stages * StageBytes;
  static constexpr int BiasOffset = BarOffset + 256;
  // epilogue store staging: 4 KB (32 rows x 32 floats) per epilogue warp
  static constexpr int StoreStageOffset = BiasOffset + kBN * 4;
  static constexpr int SmemBytes = StoreStageOffset + kEpiWarps * 4096 + 1024;  // + align slack
  static_assert(BK == 32 || BK == 16, "BK must be 32 (SW128) or 16 (SW64)");
  static_assert(SmemBytes <= 232448, "shared memory over the sm_100 limit");
};
using Cfg = RingCfg<16, 4>;  // 4 stages of 48 KB

// x -> hi (tf32: low 13 mantissa bits cleared) + lo (the rest, truncated to
// tf32). The products hi*hi + hi*lo + lo*hi approximate x*y to f32 level.
//
// Non-finite operands. Inf and NaN travel in hi. A zero lo would turn the
// cross term Inf * lo into Inf * 0 = NaN where f32 gives +-Inf (Inf times an
// exactly representable partner such as 1.0, or Inf * Inf). So the lo of a
// non-zero value is never zero: when the exact lo is 0 (x representable in
// tf32, or x = +-Inf), lo = +-FLT_MIN with x's sign. Then Inf * y = +-Inf and
// Inf * 0 = NaN as in f32, and a finite product gains at most
// FLT_MIN * |partner| (about 1e-38), below f32 resolution of any result not
// within ~1e-35 of zero. Zero keeps lo = 0 (exact zeros stay exact); NaN keeps
// lo = 0 (NaN propagates through hi).
__device__ __forceinline__ void tf32_split(float x, float& h, float& l) {
  const uint32_t u = __float_as_uint(x);
  const float tiny = __uint_as_float((u & 0x80000000u) | 0x00800000u);  // +-FLT_MIN
  if ((u & 0x7F800000u) == 0x7F800000u) {  // Inf / NaN travel in the hi part
    h = x;
    l = (u & 0x007FFFFFu) ? 0.0f : tiny;
    return;
  }
  h = __uint_as_float(u & 0xFFFFE000u);
  const float r = x - h;  // exact: r holds the 13 cleared mantissa bits
  l = __uint_as_float(__float_as_uint(r) & 0xFFFFE000u);
  if ((__float_as_uint(l) & 0x7FFFFFFFu) == 0u && (u & 0x7FFFFFFFu) != 0u) l = tiny;
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ void split_quad_store(const float (&v)[4], float* __restrict__ hi,
                                                 float* __restrict__ lo, int64_t off) {
  float4 h, l;
  tf32_split(v[0], h.x, l.x);
  tf32_split(v[1], h.y, l.y);
  tf32_split(v[2], h.z, l.z);
  tf32_split(v[3], h.w, l.w);
  if (hi) *reinterpret_cast<float4*>(hi + off) = h;
  *reinterpret_cast<float4*>(lo + off) = l;
}

// Splits src [rows, cols] (pitch ld) into hi/lo [rows, pc] (pc = cols rounded
// up to 4, zero padded), one 4-float quad per thread and iteration of a
// grid-stride loop. Four quads are loaded before any is split so that each
// thread keeps four 16-byte loads in flight (the pass is HBM-bound).
__device__ __forceinline__ void split_quads(const float* __restrict__ src, int64_t ld,
                                            int64_t rows, int64_t cols, int64_t pc,
                                            float* __restrict__ hi, float* __restrict__ lo,
                                            int64_t i0, int64_t step) {
  constexpr int kU = 4;
  const int64_t q_per_row = pc >> 2;
  const int64_t total = rows * q_per_row;
  const int vec_in = ((ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
  if (vec_in && ld == cols && cols == pc) {
    // contiguous rows without padding: a flat array of quads
    const float4* s4 = reinterpret_cast<const float4*>(src);
    int64_t i = i0;
    for (; i + (kU - 1) * step < total; i += kU * step) {
      float4 t[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) t[u] = __ldg(s4 + i + u * step);
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const float v[4] = {t[u].x, t[u].y, t[u].z, t[u].w};
        split_quad_store(v, hi, lo, (i + u * step) << 2);
      }
    }
    for (; i < total; i += step) {
      const float4 t = __ldg(s4 + i);
      const float v[4] = {t.x, t.y, t.z, t.w};
      split_quad_store(v, hi, lo, i << 2);
    }
    return;
  }
  for (int64_t i = i0; i < total; i += step) {
    const int64_t r = i / q_per_row;
    const int64_t c = (i - r * q_per_row) << 2;
    float v[4];
    if (vec_in && c + 4 <= cols) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(src + r * ld + c));
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (c + j < cols) ? __ldg(src + r * ld + c + j) : 0.0f;
    }
    split_quad_store(v, hi, lo, r * pc + c);
  }
}

// Pre-pass 1: X[M,K] (row pitch ldx) -> hi[M,Kp], lo[M,Kp]; pad columns zero.
__global__ void split_rows_kernel(const float* __restrict__ X, int64_t ldx, int64_t M, int64_t K,
                                  int64_t Kp, float* __restrict__ hi, float* __restrict__ lo) {
  // The GEMM that follows may start its prologue once every CTA is done.
  const PdlTriggerOnExit pdl_trigger_on_exit;
  split_quads(X, ldx, M, K, Kp, hi, lo, blockIdx.x * (int64_t)blockDim.x + threadIdx.x,
              (int64_t)gridDim.x * blockDim.x);
}

// Pre-pass 1b: lo part only, lo[M,Kp]. The GEMM then reads X itself as the
// hi operand: the tensor core reads a tf32 operand from f32 bits by dropping
// the low 13 mantissa bits, which is exactly the hi of tf32_split (for Inf
// and NaN too), so the products are bit-identical to the full split's.
__global__ void split_rows_lo_kernel(const float* __restrict__ X, int64_t ldx, int64_t M,
                                     int64_t K, int64_t Kp, float* __restrict__ lo) {
  // The GEMM that follows may start its prologue once every CTA is done.
  const PdlTriggerOnExit pdl_trigger_on_exit;
  split_quads(X, ldx, M, K, Kp, nullptr, lo, blockIdx.x * (int64_t)blockDim.x + threadIdx.x,
              (int64_t)gridDim.x * blockDim.x);
}

// Pre-pass 2: W[K,N] (row pitch ldw) -> hiT[N,Kp], loT[N,Kp] (K-major).
__global__ void split_transpose_kernel(const float* __restrict__ W, int64_t ldw, int64_t K,
                                       int64_t N, int64_t Kp, float* __restrict__ hiT,
                                       float* __restrict__ loT) {
  // The GEMM that follows may start its prologue once every CTA is done.
  const PdlTriggerOnExit pdl_trigger_on_exit;
  __shared__ float th[32][33];
  __shared__ float tl[32][33];
  const int64_t n0 = (int64_t)blockIdx.x * 32;
  const int64_t k0 = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t k = k0 + ty + 8 * j, n = n0 + tx;
    const float x = (k < K && n < N) ? __ldg(W + k * ldw + n) : 0.0f;
    float h, l;
    tf32_split(x, h, l);
    th[ty + 8 * j][tx] = h;
    tl[ty + 8 * j][tx] = l;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t n = n0 + ty + 8 * j, k = k0 + tx;
    if (n < N && k < Kp) {
      hiT[n * Kp + k] = th[tx][ty + 8 * j];
      loT[n * Kp + k] = tl[tx][ty + 8 * j];
    }
  }
}

// Pre-pass 3: both splits in one launch (fewer launches for small layers).
// Blocks [0, x_blocks) split X (lo only when hi == nullptr, full otherwise);
// the rest split-transpose W, one 32 x 32 tile per block. 256 threads.
__global__ void __launch_bounds__(256)
    split_xw_kernel(const float* __restrict__ X, int64_t ldx, int64_t M, int x_blocks,
                    float* __restrict__ xhi, float* __restrict__ xlo,
                    const float* __restrict__ W, int64_t ldw, int64_t K, int64_t N, int64_t Kp,
                    int tiles_n, float* __restrict__ whiT, float* __restrict__ wloT) {
  // The GEMM that follows may start its prologue once every CTA is done.
  const PdlTriggerOnExit pdl_trigger_on_exit;
  if ((int)blockIdx.x < x_blocks) {
    split_quads(X, ldx, M, K, Kp, xhi, xlo, blockIdx.x * 256ll + threadIdx.x,
                (int64_t)x_blocks * 256);
    return;
  }
  __shared__ float th[32][33];
  __shared__ float tl[32][33];
  const int t = blockIdx.x - x_blocks;
  const int64_t n0 = (int64_t)(t % tiles_n) * 32;
  const int64_t k0 = (int64_t)(t / tiles_n) * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t k = k0 + ty + 8 * j, n = n0 + tx;
    const float x = (k < K && n < N) ? __ldg(W + k * ldw + n) : 0.0f;
    float h, l;
    tf32_split(x, h, l);
    th[ty + 8 * j][tx] = h;
    tl[ty + 8 * j][tx] = l;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t n = n0 + ty + 8 * j, k = k0 + tx;
    if (n < N && k < Kp) {
      whiT[n * Kp + k] = th[tx][ty + 8 * j];
      wloT[n * Kp + k] = tl[tx][ty + 8 * j];
    }
  }
}

// Rows of a row-major [rows, cols] matrix (pitch ld) -> lo (and hi when
// non-null) with pitch pc = roundup(cols, 4); pad columns zero. Quads
// i0, i0 + step, ... of the rows * pc / 4 output quads.
// Pre-pass 4, for the MN-major B operand: X -> X_lo [M, Kp] (and X_hi when
// xhi is non-null) and W [K, N] -> W_lo [K, Np] (row-major, not transposed)
// in one launch; the GEMM reads the raw W as B_hi. Blocks [0, x_blocks)
// take X, the rest W. 256 threads.
__global__ void __launch_bounds__(256)
    split_lo_xw_kernel(const float* __restrict__ X, int64_t ldx, int64_t M, int64_t K,
                       int64_t Kp, int x_blocks, float* __restrict__ xhi,
                       float* __restrict__ xlo, const float* __restrict__ W, int64_t ldw,
                       int64_t N, int64_t Np, float* __restrict__ wlo) {
  // The GEMM that follows may start its prologue once every CTA is done.
  const PdlTriggerOnExit pdl_trigger_on_exit;
  if ((int)blockIdx.x < x_blocks)
    split_quads(X, ldx, M, K, Kp, xhi, xlo, blockIdx.x * 256ll + threadIdx.x,
                (int64_t)x_blocks * 256);
  else
    split_quads(W, ldw, K, N, Np, nullptr, wlo, (blockIdx.x - x_blocks) * 256ll + threadIdx.x,
                (int64_t)(gridDim.x - x_blocks) * 256);
}

// ---------------------------------------------------------------------------
__device__ __forceinline__ float apply_act(float x, int act, float alpha) {
  if (act == kActRelu) {
    // arith.maximumf(x, 0): NaN propagates, max(-0, +0) = +0
    return (x > 0.0f || x != x) ? x : 0.0f;
  }
  if (act == kActLeakyRelu) {
    // max(x,0) + alpha*min(x,0), both with maximumf/minimumf semantics
    const float pos = (x > 0.0f || x != x) ? x : 0.0f;
    const float neg = (x < 0.0f || x != x) ? x : 0.0f;
    return pos + neg * alpha;
  }
  return x;
}

struct Epilogue {
  float* Y;
  int64_t ldy;
  const float* bias;  // may be null
  int64_t M, N;
  int act;
  float alpha;
  int vec_out;  // Y base 16-byte aligned and ldy % 4 == 0
  float* part;  // cut tiles: raw partial sums, tile-local [piece][r][BM][kBN]
  float* Ylo;   // optional: the tf32 lo part of each final value (the next
  int64_t ldylo;  // layer's pre-split A_lo), pitch ldylo
  int stage_store;  // 1: coalesce the epilogue's stores through shared memory
  int bias_vec;     // bias non-null and 16-byte aligned: float4 bias loads
  // Gathered result: every final value is also stored at the same element
  // offset from each peer base (another GPU's output rows, mapped through
  // CUDA IPC), with ordinary stores that travel over NVLink as tiles finish.
  int npeers;
  float* peer[kMaxEpiloguePeers];
  // Gathered result through NVSwitch multicast: the multicast address of Y
  // (same element offsets); every final value is written once with
  // multimem.st and lands in Y and in every peer's copy. Replaces Y / peers.
  float* mc;
};

// Final values: Y and every peer copy (one multicast store when ep.mc is set).
__device__ __forceinline__ void store_final4(const Epilogue& ep, int64_t off, float4 v) {
  if (ep.mc) {
    multimem_st_v4(ep.mc + off, v);
    return;
  }
  *reinterpret_cast<float4*>(ep.Y + off) = v;
#pragma unroll 1
  for (int p = 0; p < ep.npeers; ++p) *reinterpret_cast<float4*>(ep.peer[p] + off) = v;
}
__device__ __forceinline__ void store_final1(const Epilogue& ep, int64_t off, float v) {
  if (ep.mc) {
    multimem_st(ep.mc + off, v);
    return;
  }
  ep.Y[off] = v;
#pragma unroll 1
  for (int p = 0; p < ep.npeers; ++p) ep.peer[p][off] = v;
}

// Bias of columns c .. c+3 (c a multiple of 4 from a 16-byte aligned tile
// origin), zeros without bias. Every lane of a warp loads the same values.
__device__ __forceinline__ float4 bias4(const Epilogue& ep, int64_t c) {
  if (ep.bias_vec) return __ldg(reinterpret_cast<const float4*>(ep.bias + c));
  if (ep.bias == nullptr) return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  return make_float4(c < ep.N ? __ldg(ep.bias + c) : 0.0f,
                     c + 1 < ep.N ? __ldg(ep.bias + c + 1) : 0.0f,
                     c + 2 < ep.N ? __ldg(ep.bias + c + 2) : 0.0f,
                     c + 3 < ep.N ? __ldg(ep.bias + c + 3) : 0.0f);
}

// Final values v[0..3] at (row, col..col+3): Y, and when requested the lo
// part that the next layer's GEMM reads as A_lo.
__device__ __forceinline__ void store_lo4(const Epilogue& ep, int64_t row, int64_t col,
                                          const float (&v)[4]) {
  float lo[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float h;
    tf32_split(v[q], h, lo[q]);
  }
  float* d = ep.Ylo + row * ep.ldylo + col;
  if ((ep.ldylo & 3) == 0 && ((reinterpret_cast<uintptr_t>(ep.Ylo) & 15) == 0) &&
      col + 4 <= ep.N) {
    *reinterpret_cast<float4*>(d) = make_float4(lo[0], lo[1], lo[2], lo[3]);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (col + q < ep.N) d[q] = lo[q];
  }
}

// Stores one epilogue thread's 128 consecutive accumulator columns of a unit:
// tile-local row `lr`, columns [lc0, lc0 + 128). A whole tile's row gets bias,
// activation and the M / N bounds and goes to Y; a piece's raw sums go to its
// tile-local partial buffer.
//
// Coalescing. A thread owns one row, so a direct float4 store per thread
// scatters each warp instruction over 32 rows (16 bytes each). With `stage`
// (4 KB of shared memory per warp) the warp instead passes 32 x 32 blocks
// through shared memory: every thread writes its row's 32 values (16-byte
// chunks XOR-swizzled by row, conflict-free both ways), then the warp reads
// them back transposed so that each store instruction writes four whole
// 128-byte row segments. A warp whose 32 x 128 region is cut by the M / N
// edges, unaligned Y and the Ylo output keep the per-thread stores.
template <int kTileM>
__device__ __forceinline__ void store_tile_row(const Epilogue& ep, const Unit& w, int rest,
                                               int lr, int lc0, const float (&acc)[128],
                                               float* stage, int lane) {
  const int lr0 = lr - lane;  // the warp's first row
  if (w.piece >= 0) {
    float* tile = ep.part + (int64_t)(w.piece * rest + w.r) * kTileM * kBN;
    if (stage) {
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
          *reinterpret_cast<float4*>(stage + lane * 32 + ((ch ^ (lane & 7)) << 2)) =
              make_float4(acc[cb * 32 + ch * 4], acc[cb * 32 + ch * 4 + 1],
                          acc[cb * 32 + ch * 4 + 2], acc[cb * 32 + ch * 4 + 3]);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = k * 4 + (lane >> 3), ch = lane & 7;
          *reinterpret_cast<float4*>(tile + (int64_t)(lr0 + r) * kBN + lc0 + cb * 32 + ch * 4) =
              *reinterpret_cast<const float4*>(stage + r * 32 + ((ch ^ (r & 7)) << 2));
        }
        __syncwarp();
      }
      return;
    }
    float* dst = tile + (int64_t)lr * kBN + lc0;
#pragma unroll
    for (int j = 0; j < 128; j += 4)
      *reinterpret_cast<float4*>(dst + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
    return;
  }
  const int64_t row = (int64_t)w.m0 + lr;
  const int64_t row0 = (int64_t)w.m0 + lr0;
  const int64_t col0 = (int64_t)w.n0 + lc0;
  // warp-uniform: the warp's whole 32 x 128 region lies inside Y
  if (stage != nullptr && ep.vec_out && ep.Ylo == nullptr && row0 + 32 <= ep.M &&
      col0 + 128 <= ep.N) {
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int c = cb * 32 + ch * 4;
        const float4 bv = bias4(ep, col0 + c);
        *reinterpret_cast<float4*>(stage + lane * 32 + ((ch ^ (lane & 7)) << 2)) =
            make_float4(apply_act(acc[c] + bv.x, ep.act, ep.alpha),
                        apply_act(acc[c + 1] + bv.y, ep.act, ep.alpha),
                        apply_act(acc[c + 2] + bv.z, ep.act, ep.alpha),
                        apply_act(acc[c + 3] + bv.w, ep.act, ep.alpha));
      }
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = k * 4 + (lane >> 3), ch = lane & 7;
        store_final4(ep, (row0 + r) * ep.ldy + col0 + cb * 32 + ch * 4,
                     *reinterpret_cast<const float4*>(stage + r * 32 + ((ch ^ (r & 7)) << 2)));
      }
      __syncwarp();
    }
    return;
  }
  if (row >= ep.M) return;
  const int64_t base = row * ep.ldy + col0;
#pragma unroll
  for (int j = 0; j < 128; j += 4) {
    float4 bv;
    if (ep.bias_vec && col0 + j + 4 <= ep.N) {
      bv = bias4(ep, col0 + j);
    } else {
      bv.x = (ep.bias != nullptr && col0 + j < ep.N) ? __ldg(ep.bias + col0 + j) : 0.0f;
      bv.y = (ep.bias != nullptr && col0 + j + 1 < ep.N) ? __ldg(ep.bias + col0 + j + 1) : 0.0f;
      bv.z = (ep.bias != nullptr && col0 + j + 2 < ep.N) ? __ldg(ep.bias + col0 + j + 2) : 0.0f;
      bv.w = (ep.bias != nullptr && col0 + j + 3 < ep.N) ? __ldg(ep.bias + col0 + j + 3) : 0.0f;
    }
    const float v0 = apply_act(acc[j] + bv.x, ep.act, ep.alpha);
    const float v1 = apply_act(acc[j + 1] + bv.y, ep.act, ep.alpha);
    const float v2 = apply_act(acc[j + 2] + bv.z, ep.act, ep.alpha);
    const float v3 = apply_act(acc[j + 3] + bv.w, ep.act, ep.alpha);
    if (ep.vec_out && col0 + j + 4 <= ep.N) {
      store_final4(ep, base + j, make_float4(v0, v1, v2, v3));
    } else {
      if (col0 + j < ep.N) store_final1(ep, base + j, v0);
      if (col0 + j + 1 < ep.N) store_final1(ep, base + j + 1, v1);
      if (col0 + j + 2 < ep.N) store_final1(ep, base + j + 2, v2);
      if (col0 + j + 3 < ep.N) store_final1(ep, base + j + 3, v3);
    }
    if (ep.Ylo && col0 + j < ep.N) {
      const float v[4] = {v0, v1, v2, v3};
      store_lo4(ep, row, col0 + j, v);
    }
  }
}

// UMMA shared-memory descriptors of the four operand tiles of stage base `st`
// at k-step k (8 tf32 = 32 bytes along the row).
template <class Cfg>
struct UmmaDesc {
  static __device__ __forceinline__ uint64_t at(uint32_t addr) {
    return umma_desc_k<Cfg::UmmaLayout, Cfg::SBO>(addr);
  }
  static __device__ __forceinline__ uint64_t a_hi(uint32_t st, int k) { return at(st + k * 32); }
  static __device__ __forceinline__ uint64_t a_lo(uint32_t st, int k) {
    return at(st + Cfg::ATileBytes + k * 32);
  }
  static __device__ __forceinline__ uint64_t b_hi(uint32_t st, int k) {
    return at(st + 2 * Cfg::ATileBytes + k * 32);
  }
  static __device__ __forceinline__ uint64_t b_lo(uint32_t st, int k) {
    return at(st + 2 * Cfg::ATileBytes + Cfg::BTileBytes + k * 32);
  }
};

// B tiles stored MN-major (the raw row-major W[K, N] and its lo part): each
// B tile is 8 blocks of BK K-rows x 128 bytes (32 columns), one TMA box
// each, in the 32-byte-atom 128-byte swizzle; k-step k (8 rows) starts
// 1 KB into every block, and its two 4-row groups are 512 bytes apart.
template <class Cfg>
struct UmmaDescBMn {
  static constexpr uint32_t kAtomBytes = Cfg::BK * 128;
  static __device__ __forceinline__ uint64_t b_hi(uint32_t st, int k) {
    return umma_desc_mn_sw128_32b<kAtomBytes, 512>(st + 2 * Cfg::ATileBytes + k * 1024);
  }
  static __device__ __forceinline__ uint64_t b_lo(uint32_t st, int k) {
    return umma_desc_mn_sw128_32b<kAtomBytes, 512>(st + 2 * Cfg::ATileBytes +
                                                     Cfg::BTileBytes + k * 1024);
  }
};

// kBMn: B_hi is the raw f32 W (row-major [K, N], read as an MN-major tf32
// operand: the tensor core drops the low 13 mantissa bits, which is the hi
// part) and B_lo the row-major lo part, so W needs neither a transpose nor a
// hi copy. The producer warp's lanes issue the two B tiles and two A tiles of a
// stage from separate lanes.
template <class Cfg, bool kBMn>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmAhi,
                       const __grid_constant__ CUtensorMap tmAlo,
                       const __grid_constant__ CUtensorMap tmBhi,
                       const __grid_constant__ CUtensorMap tmBlo, Sched sc, Epilogue ep,
                       int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BarOffset);  // TMA -> MMA
  uint64_t* empty = full + Cfg::Stages;                                   // MMA -> TMA
  uint64_t* tfull = empty + Cfg::Stages;   // MMA -> epilogue: chunk accumulator ready
  uint64_t* tempty = tfull + 2;        // epilogue -> MMA: chunk accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Work units (whole tiles, then pieces of cut tiles) of the schedule `sc`.
  auto unit_of = [&](int u) { return unit_at(sc, u, kBM, kBN); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmAhi);
    tma_prefetch_desc(&tmAlo);
    tma_prefetch_desc(&tmBhi);
    tma_prefetch_desc(&tmBlo);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched as a programmatic dependent of the split pass: everything above
  // overlaps its tail; operands are read only after it has completed.
  pdl_wait();

  // Ring stages and TMEM chunk buffers are counted across all units of the
  // CTA, so their mbarrier phases run on from one tile to the next.
  if (warp == 0 && kBMn) {
    // ------------------------------------------------ TMA producer (MN-major B)
    // Lane 0 waits for the stage and posts the byte count; the decision is
    // broadcast so that the whole warp leaves the loop together.
    int it = 0;
    for (int u = blockIdx.x; u < sc.units; u += gridDim.x) {
      int go = lane == 0 ? !*abort_flag : 0;
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      const Unit w = unit_of(u);
      bool ok = true;
      for (int kb = 0; kb < w.nkb; ++kb, ++it) {
        const int s = it % Cfg::Stages;
        const int round = it / Cfg::Stages;
        go = 1;
        if (lane == 0) {
          if (round > 0 &&
              !mbar_wait(&empty[s], (round - 1) & 1, status, kDevTimeoutEmpty, abort_flag))
            go = 0;
          else
            mbar_arrive_expect_tx(&full[s], Cfg::StageBytes);
        }
        if (!__shfl_sync(0xffffffffu, go, 0)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * Cfg::StageBytes;
        const int kx = (w.kb0 + kb) * Cfg::BK;
        if (lane < 2) {  // whole 256-column B tile: {0, kx, n0 / 32}
          tma_load_3d(st + 2 * Cfg::ATileBytes + lane * Cfg::BTileBytes,
                      lane == 0 ? &tmBhi : &tmBlo, &full[s], 0, kx, w.n0 / 32);
        } else if (lane == 2) {
          tma_load_2d(st, &tmAhi, &full[s], kx, w.m0);
        } else if (lane == 3) {
          tma_load_2d(st + Cfg::ATileBytes, &tmAlo, &full[s], kx, w.m0);
        }
      }
      if (!ok) break;
    }
  } else if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      for (int u = blockIdx.x; u < sc.units && !*abort_flag; u += gridDim.x) {
        const Unit w = unit_of(u);
        for (int kb = 0; kb < w.nkb; ++kb, ++it) {
          const int s = it % Cfg::Stages;
          const int round = it / Cfg::Stages;
          if (round > 0 &&
              !mbar_wait(&empty[s], (round - 1) & 1, status, kDevTimeoutEmpty, abort_flag))
            break;
          uint8_t* st = smem + s * Cfg::StageBytes;
          const int kx = (w.kb0 + kb) * Cfg::BK;
          mbar_arrive_expect_tx(&full[s], Cfg::StageBytes);
          tma_load_2d(st, &tmAhi, &full[s], kx, w.m0);
          tma_load_2d(st + Cfg::ATileBytes, &tmAlo, &full[s], kx, w.m0);
          tma_load_2d(st + 2 * Cfg::ATileBytes, &tmBhi, &full[s], kx, w.n0);
          tma_load_2d(st + 2 * Cfg::ATileBytes + Cfg::BTileBytes, &tmBlo, &full[s], kx, w.n0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = kBMn ? idesc_tf32_f32_bmn(kBM, kBN) : idesc_tf32_f32(kBM, kBN);
      using D = UmmaDesc<Cfg>;
      using DB = typename std::conditional<kBMn, UmmaDescBMn<Cfg>, UmmaDesc<Cfg>>::type;
      int it = 0, cc = 0;  // k-blocks and TMEM chunks issued by this CTA
      bool ok = true;
      for (int u = blockIdx.x; u < sc.units && ok; u += gridDim.x) {
        const Unit w = unit_of(u);
        for (int kb = 0; kb < w.nkb; ++kb, ++it) {
          const int s = it % Cfg::Stages;
          const int round = it / Cfg::Stages;
          const int buf = cc & 1;
          const bool chunk_start = (kb % Cfg::ChunkKB) == 0;
          const bool chunk_end = (kb % Cfg::ChunkKB) == Cfg::ChunkKB - 1 || kb == w.nkb - 1;
          if (chunk_start && cc >= 2) {
            if (!mbar_wait(&tempty[buf], ((cc >> 1) - 1) & 1, status, kDevTimeoutAccum,
                           abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if (!mbar_wait(&full[s], round & 1, status, kDevTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * kBN;
          const uint32_t st = smem_u32(smem + s * Cfg::StageBytes);
#pragma unroll
          for (int k = 0; k < Cfg::BK / 8; ++k) {  // tf32 UMMA consumes K = 8
            umma_tf32(d_tmem, D::a_lo(st, k), DB::b_hi(st, k), idesc,
                      (chunk_start && k == 0) ? 0u : 1u);
            umma_tf32(d_tmem, D::a_hi(st, k), DB::b_lo(st, k), idesc, 1u);
            umma_tf32(d_tmem, D::a_hi(st, k), DB::b_hi(st, k), idesc, 1u);
          }
          umma_commit(&empty[s]);  // stage s may be refilled once these MMAs finish
          if (chunk_end) {
            umma_commit(&tfull[buf]);
            ++cc;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------ epilogue (8 warps)
    // Warp w reads TMEM lane quarter w % 4 and column half (w - 2) / 4.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float acc[128];
    bool ok = true;
    int ce = 0;  // TMEM chunks drained by this CTA
    // Adds the next chunk's partial sums (TMEM buffer ce % 2) into acc, frees it.
    auto drain = [&]() -> bool {
      const int buf = ce & 1;
      if (!mbar_wait(&tfull[buf], (ce >> 1) & 1, status, kDevTimeoutAccum, abort_flag))
        return false;
      tc_fence_after();
      const uint32_t taddr = tmem_base + lane_off + buf * kBN + half * 128;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + g * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[g * 32 + j] += __uint_as_float(r[j]);  // RN add
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      ++ce;
      return true;
    };
#pragma unroll 1
    for (int u = blockIdx.x; u < sc.units && ok && !*abort_flag; u += gridDim.x) {
      const Unit w = unit_of(u);
      const int num_chunks = (w.nkb + Cfg::ChunkKB - 1) / Cfg::ChunkKB;
#pragma unroll
      for (int j = 0; j < 128; ++j) acc[j] = 0.0f;
#pragma unroll 1
      for (int c = 0; c < num_chunks && ok; ++c) ok = drain();
      if (!ok || *abort_flag) break;
      // The MMAs of the next unit proceed into the two TMEM buffers while
      // this tile is stored.
      store_tile_row<kBM>(
          ep, w, sc.rest, quarter * 32 + lane, half * 128, acc,
          ep.stage_store
              ? reinterpret_cast<float*>(smem + Cfg::StoreStageOffset + (warp - 2) * 4096)
              : nullptr,
          lane);
    }
  }

  pdl_trigger();  // a following split-K reduction may launch (it waits for completion)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Failure-detection self-test: one thread waits, with the GEMM's bounded
// wait, on an mbarrier that nothing ever arrives on. After `limit_ns` the
// wait gives up and records kDevTimeoutSelfTest in the status word, exactly
// as a stalled GEMM role would; the kernel then returns normally.
__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns, int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    mbar_wait_for(&bar, 0, status, kDevTimeoutSelfTest, &abort_flag, limit_ns);
}

int wait_timeout_selftest(uint64_t limit_ns, int* status, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns, status);
  count_launch();
  return launch_result();
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Most SMs the f32 GEMM's persistent grid may occupy (0: all). A caller that
// runs a collective concurrently (the slab-pipelined all-gather of a sharded
// result) leaves SMs free for its kernels.
static std::atomic<int> g_gemm_sm_limit{0};
int set_gemm_sm_limit(int n) { return g_gemm_sm_limit.exchange(n > 0 ? n : 0); }

static int device_sm_count();
// SMs the GEMM's schedule and persistent grid use: the device's, capped by
// set_gemm_sm_limit.
static int sm_count() {
  const int n = device_sm_count();
  const int lim = g_gemm_sm_limit.load();
  return lim > 0 && lim < n ? lim : n;
}

// SMs of the current device (cached per device); without a device (host-side
// workspace and schedule queries) the B200's 148.
static int device_sm_count() {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;
  }
  if (sms[dev & 63] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return 148;
    }
    sms[dev & 63] = n;
  }
  return sms[dev & 63];
}

// 2-D f32 tensor map: `rows` rows of `cols` valid floats, row pitch `pitch`
// floats (multiple of 4), box = box_rows x bk floats, swizzle matching the
// bk*4-byte row. Coordinates beyond `cols` / `rows` read as zero.
static int make_tmap(CUtensorMap* map, const float* base, int64_t cols, int64_t rows,
                     int64_t pitch, int box_rows, int bk) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return driver_failure("cuTensorMapEncodeTiled entry point", 0);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)pitch * 4};
  cuuint32_t box[2] = {(cuuint32_t)bk, (cuuint32_t)box_rows};
  const CUtensorMapSwizzle swz = bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : driver_failure("cuTensorMapEncodeTiled", (int)r);
}

// Tensor map of a row-major [rows = K, cols = N] operand read MN-major, N a
// multiple of 32: viewed as 3-D {32 columns, K rows, N/32 column blocks} so
// that one box {32, bk, 8} brings a whole 256-column B tile, stored
// block-major ([8][bk][32]), in the 128-byte swizzle with 32-byte atomicity
// (the only MN-major layout the tensor core takes for 32-bit operands).
// Column blocks past N/32 read as zero.
static int make_tmap_mn(CUtensorMap* map, const float* base, int64_t cols, int64_t rows,
                        int64_t pitch, int bk) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return driver_failure("cuTensorMapEncodeTiled entry point", 0);
  if (cols % 32) return kErrInvalidArg;
  cuuint64_t dims[3] = {32, (cuuint64_t)rows, (cuuint64_t)(cols / 32)};
  cuuint64_t strides[2] = {(cuuint64_t)pitch * 4, 128};
  cuuint32_t box[3] = {32, (cuuint32_t)bk, kBN / 32};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : driver_failure("cuTensorMapEncodeTiled", (int)r);
}

// The B operand of one GEMM: K-major split W^T (hi, lo with pitch Kp), or
// MN-major raw W (hi, pitch ldw) with its row-major lo part (pitch ld_lo).
struct BOp {
  const float* hi;
  const float* lo;
  int64_t ld_hi, ld_lo;
  bool mn;
};
static BOp bop_k(const float* whiT, const float* wloT, int64_t K) {
  const int64_t Kp = split_pitch(K);
  return BOp{whiT, wloT, Kp, Kp, false};
}

int64_t dense_f32_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  const int64_t Kp = split_pitch(K);
  // hi + lo of X (M x Kp) and of W^T (N x Kp), each region 256-byte aligned
  auto al = [](int64_t b) { return (b + 255) & ~int64_t(255); };
  return 2 * al(M * Kp * 4) + 2 * al(N * Kp * 4);
}

int split_w_f32(const float* W, int64_t ldw, int64_t K, int64_t N, float* whiT, float* wloT,
                cudaStream_t stream) {
  const int64_t Kp = split_pitch(K);
  dim3 grid((unsigned)((N + 31) / 32), (unsigned)((Kp + 31) / 32));
  split_transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(W, ldw, K, N, Kp, whiT, wloT);
  count_launch();
  return launch_result();
}

int split_x_f32(const float* X, int64_t ldx, int64_t M, int64_t K, float* xhi, float* xlo,
                cudaStream_t stream) {
  const int64_t Kp = split_pitch(K);
  const int64_t total = M * (Kp / 4);
  int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  if (blocks < 1) blocks = 1;
  split_rows_kernel<<<blocks, 256, 0, stream>>>(X, ldx, M, K, Kp, xhi, xlo);
  count_launch();
  return launch_result();
}

// Programmatic dependent launch (see pdl_wait) for problems of at most 2^33
// multiply-adds (2048^3): there the launch and prologue latency it hides is
// 10-20% of a call (dense 1024^3: 31.0 -> 26.9 us; 256^3: 22.7 -> 18.6 us);
// for long GEMMs it gained nothing measurable. B200_PDL=0 turns it off.
static bool pdl_enabled(int64_t M, int64_t N, int64_t K);

// The epilogue's stores go through shared memory (store_tile_row) unless
// B200_STORE_STAGE=0 (per-thread row stores, for A/B measurements).
static bool store_staging_enabled() {
  static const bool on = [] {
    const char* e = getenv("B200_STORE_STAGE");
    return !(e && e[0] == '0');
  }();
  return on;
}

static bool pdl_enabled(int64_t M, int64_t N, int64_t K) {
  static const bool on = [] {
    const char* e = getenv("B200_PDL");
    return !(e && e[0] == '0');
  }();
  return on && (double)M * (double)N * (double)K <= 8589934592.0;
}

template <class... KArgs, class... Args>
static cudaError_t launch_dependent(bool pdl, void (*kernel)(KArgs...), unsigned grid,
                                    unsigned block, size_t smem, cudaStream_t stream,
                                    Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <class Cfg, bool kBMn>
static int launch_gemm(const CUtensorMap& ta_hi, const CUtensorMap& ta_lo,
                       const CUtensorMap& tb_hi, const CUtensorMap& tb_lo, int64_t M, int64_t N,
                       int64_t K, const Sched& sc, const Epilogue& ep, int* status,
                       cudaStream_t stream) {
  // The dynamic shared-memory opt-in is made once per device (thread-safe).
  static std::atomic<uint64_t> attr_done{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return launch_result();
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_done.load() & bit)) {
    if (cudaFuncSetAttribute(gemm_tf32x3_kernel<Cfg, kBMn>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg::SmemBytes) != cudaSuccess)
      return launch_result();
    attr_done.fetch_or(bit);
  }
  // Persistent: one CTA per SM (the shared-memory ring admits one) walks the
  // work units with stride gridDim.x.
  const int sms = sm_count();
  if (sms <= 0) return kErrCuda;
  const int grid = std::min(sc.units, sms);
  const cudaError_t e =
      launch_dependent(pdl_enabled(M, N, K), gemm_tf32x3_kernel<Cfg, kBMn>, (unsigned)grid,
                       kThreads, Cfg::SmemBytes, stream, ta_hi, ta_lo, tb_hi, tb_lo, sc, ep,
                       status);
  count_launch();
  return launch_result(e);
}

// A operand: hi from `xa` with row pitch ldx (the pre-split xhi with pitch
// Kp, or raw X), lo from xlo (pitch Kp).
static int dispatch_gemm(const float* xa, const float* xlo, int64_t ldx, const BOp& b, int64_t M,
                         int64_t N, int64_t K, const Sched& sc, const Epilogue& ep, int* status,
                         cudaStream_t stream) {
  const int64_t Kp = split_pitch(K);
  CUtensorMap ta_hi, ta_lo, tb_hi, tb_lo;
  int rc = make_tmap(&ta_hi, xa, K, M, ldx, kBM, Cfg::BK);
  if (rc == kOk) rc = make_tmap(&ta_lo, xlo, K, M, Kp, kBM, Cfg::BK);
  if (b.mn) {
    if (rc == kOk) rc = make_tmap_mn(&tb_hi, b.hi, N, K, b.ld_hi, Cfg::BK);
    if (rc == kOk) rc = make_tmap_mn(&tb_lo, b.lo, N, K, b.ld_lo, Cfg::BK);
    if (rc != kOk) return rc;
    return launch_gemm<Cfg, true>(ta_hi, ta_lo, tb_hi, tb_lo, M, N, K, sc, ep, status, stream);
  }
  if (rc == kOk) rc = make_tmap(&tb_hi, b.hi, K, N, b.ld_hi, kBN, Cfg::BK);
  if (rc == kOk) rc = make_tmap(&tb_lo, b.lo, K, N, b.ld_lo, kBN, Cfg::BK);
  if (rc != kOk) return rc;
  return launch_gemm<Cfg, false>(ta_hi, ta_lo, tb_hi, tb_lo, M, N, K, sc, ep, status, stream);
}

namespace {
thread_local int tl_npeers = 0;
thread_local float* tl_peers[kMaxEpiloguePeers] = {};
thread_local float* tl_mc = nullptr;
}  // namespace

void set_epilogue_peers(float* const* peers, int n, float* mc) {
  tl_npeers = (peers != nullptr && n > 0) ? std::min(n, kMaxEpiloguePeers) : 0;
  for (int i = 0; i < kMaxEpiloguePeers; ++i) tl_peers[i] = i < tl_npeers ? peers[i] : nullptr;
  tl_mc = mc;
}

static int gemm_with_splits(const float* xa, const float* xlo, int64_t ldx,
                            const BOp& bop, int64_t M, int64_t N, int64_t K, const float* bias,
                            float* Y, int64_t ldy, int act, float alpha, int splits,
                            float* partials, int* status, cudaStream_t stream,
                            float* ylo = nullptr, int64_t ldylo = 0);

int gemm_tf32x3_presplit(const float* xhi, const float* xlo, const float* whiT,
                         const float* wloT, int64_t M, int64_t N, int64_t K, const float* bias,
                         float* Y, int64_t ldy, int act, float alpha, int* status,
                         cudaStream_t stream) {
  return gemm_with_splits(xhi, xlo, split_pitch(K), bop_k(whiT, wloT, K), M, N, K,
                          bias, Y, ldy, act, alpha, 1, nullptr, status, stream);
}

// ---------------------------------------------------------------------------
// Schedules (see sched.cuh). One 128 x 256 tile over all of K takes
// 2 * BM * 256 * K / 1.65e12 s per SM at the measured 3xTF32 rate; a piece
// spans at least 128 of K (half a TMEM promotion chunk: a piece may end
// mid-chunk). Cut tiles arise when the last wave is partial: the 1024^3
// layer (32 tiles), the MLP's layers (172 and 64 tiles), 4096^3 (512 tiles =
// 3.46 waves).
static Sched sched_f32(int64_t M, int64_t N, int64_t K, bool allow_cut) {
  const int sms = std::max(1, sm_count());
  const double t_tile = 2.0 * kBM * kBN * (double)K / 1.65e12;
  return make_sched(M, N, K, kBM, kBN, Cfg::BK, sms, t_tile, 4, 0, allow_cut ? 16 : 1,
                    128 / Cfg::BK /* pieces may end mid-chunk */, kGroupM);
}

void sched_query_f32(int64_t M, int64_t N, int64_t K, int64_t* out) {
  const Sched sc = sched_f32(M, N, K, true);
  const int64_t v[8] = {sc.tiles_m, sc.tiles_n, sc.whole, sc.rest, sc.pieces, sc.kb, sc.kbp,
                        sc.units};
  for (int i = 0; i < 8; ++i) out[i] = v[i];
}

int choose_splits(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 1;
  const Sched sc = sched_f32(M, N, K, true);
  return sc.rest > 0 ? sc.pieces : 1;
}

int gemm_f32_launches(int64_t M, int64_t N, int64_t K) {
  return choose_splits(M, N, K) > 1 ? 2 : 1;
}

__global__ void __launch_bounds__(256)
    piece_reduce_kernel(const float* __restrict__ part, Sched sc, int tile_m, int64_t M,
                        int64_t N, const float* __restrict__ bias, int act, float alpha,
                        float* __restrict__ Y, int64_t ldy, int vec, Epilogue lo_ep) {
  pdl_wait();  // launched as a programmatic dependent of the GEMM
  const int64_t tile_elems = (int64_t)tile_m * kBN;
  const int64_t quads_per_tile = tile_elems / 4;
  const int64_t total = (int64_t)sc.rest * quads_per_tile;
  const int64_t piece_stride = (int64_t)sc.rest * tile_elems;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / quads_per_tile);
    const int64_t e = (i - r * quads_per_tile) * 4;  // element offset in the tile
    const int lr = (int)(e / kBN), lc = (int)(e - (int64_t)lr * kBN);
    int mt, nt;
    tile_coords(sc, sc.whole + r, mt, nt);
    const int64_t row = (int64_t)mt * tile_m + lr, col = (int64_t)nt * kBN + lc;
    if (row >= M || col >= N) continue;
    const float* src = part + (int64_t)r * tile_elems + e;
    float4 a = __ldg(reinterpret_cast<const float4*>(src));
    for (int p = 1; p < sc.pieces; ++p) {  // fixed order: deterministic
      const float4 t = __ldg(reinterpret_cast<const float4*>(src + p * piece_stride));
      a.x += t.x; a.y += t.y; a.z += t.z; a.w += t.w;
    }
    float v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (bias && col + q < N) v[q] += bias[col + q];
      v[q] = apply_act(v[q], act, alpha);
    }
    // lo_ep carries Y, ldy and the peer copies of this call
    const int64_t off = row * lo_ep.ldy + col;
    if (vec && col + 4 <= N) {
      store_final4(lo_ep, off, make_float4(v[0], v[1], v[2], v[3]));
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (col + q < N) store_final1(lo_ep, off + q, v[q]);
    }
    if (lo_ep.Ylo) store_lo4(lo_ep, row, col, v);
  }
}

// Bytes of cut-tile partial sums for a call of choose_splits(M, N, K) > 1.
int64_t splitk_partials_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const Sched sc = sched_f32(M, N, K, true);
  const int64_t b = sc.rest > 0 ? (int64_t)sc.pieces * sc.rest * kBM * kBN * 4 : 0;
  return b ? (b + 255) & ~int64_t(255) : 0;
}

// One GEMM call: `splits` > 1 (with `partials` sized by splitk_partials_bytes)
// lets the schedule cut the tiles of a partial last wave into K pieces;
// otherwise every tile runs over all of K.
static int gemm_with_splits(const float* xa, const float* xlo, int64_t ldx,
                            const BOp& bop, int64_t M, int64_t N, int64_t K, const float* bias,
                            float* Y, int64_t ldy, int act, float alpha, int splits,
                            float* partials, int* status, cudaStream_t stream, float* ylo,
                            int64_t ldylo) {
  const Sched sc = sched_f32(M, N, K, splits > 1 && partials != nullptr);
  Epilogue ep;
  ep.Y = Y;
  ep.ldy = ldy;
  ep.bias = bias;
  ep.M = M;
  ep.N = N;
  ep.act = act;
  ep.alpha = alpha;
  ep.vec_out = ((ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(Y) & 15) == 0);
  ep.part = partials;
  ep.Ylo = ylo;
  ep.ldylo = ldylo;
  ep.stage_store = store_staging_enabled() ? 1 : 0;
  ep.bias_vec = (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 15) == 0) ? 1 : 0;
  ep.npeers = tl_npeers;
  for (int i = 0; i < kMaxEpiloguePeers; ++i) {
    ep.peer[i] = tl_peers[i];
    if (i < ep.npeers && (reinterpret_cast<uintptr_t>(tl_peers[i]) & 15) != 0) ep.vec_out = 0;
  }
  ep.mc = tl_mc;
  if (ep.mc && (reinterpret_cast<uintptr_t>(ep.mc) & 15) != 0) ep.vec_out = 0;
  int rc = dispatch_gemm(xa, xlo, ldx, bop, M, N, K, sc, ep, status, stream);
  if (rc != kOk || sc.rest == 0) return rc;
  const int tile_m = kBM;
  const int64_t quads = (int64_t)sc.rest * tile_m * (kBN / 4);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((quads + 255) / 256, 148 * 16));
  const cudaError_t e = launch_dependent(pdl_enabled(M, N, K), piece_reduce_kernel,
                                         (unsigned)blocks, 256, 0, stream,
                                         static_cast<const float*>(partials), sc, tile_m, M, N,
                                         bias, act, alpha, Y, ldy, ep.vec_out, ep);
  count_launch();
  return launch_result(e);
}

int gemm_tf32x3_splitk(const float* xhi, const float* xlo, const float* whiT, const float* wloT,
                       int64_t M, int64_t N, int64_t K, const float* bias, float* Y, int64_t ldy,
                       int act, float alpha, int splits, float* partials, int* status,
                       cudaStream_t stream, float* ylo, int64_t ldylo) {
  return gemm_with_splits(xhi, xlo, split_pitch(K), bop_k(whiT, wloT, K), M, N, K,
                          bias, Y, ldy, act, alpha, splits, partials, status, stream, ylo, ldylo);
}

int split_xw_f32(const float* X, int64_t ldx, int64_t M, const float* W, int64_t ldw,
                 int64_t K, int64_t N, float* xhi, float* xlo, float* whiT, float* wloT,
                 cudaStream_t stream) {
  const int64_t Kp = split_pitch(K);
  const int64_t xq = M * (Kp / 4);
  const int x_blocks = (int)std::max<int64_t>(1, std::min<int64_t>((xq + 255) / 256, 148 * 16));
  const int tiles_n = (int)((N + 31) / 32);
  const int64_t w_blocks = (int64_t)tiles_n * ((Kp + 31) / 32);
  split_xw_kernel<<<(unsigned)(x_blocks + w_blocks), 256, 0, stream>>>(
      X, ldx, M, x_blocks, xhi, xlo, W, ldw, K, N, Kp, tiles_n, whiT, wloT);
  count_launch();
  return launch_result();
}

int split_x_lo_f32(const float* X, int64_t ldx, int64_t M, int64_t K, float* xlo,
                   cudaStream_t stream) {
  const int64_t Kp = split_pitch(K);
  const int64_t total = M * (Kp / 4);
  int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  if (blocks < 1) blocks = 1;
  split_rows_lo_kernel<<<blocks, 256, 0, stream>>>(X, ldx, M, K, Kp, xlo);
  count_launch();
  return launch_result();
}

int gemm_tf32x3_xraw(const float* X, int64_t ldx, const float* xlo, const float* whiT,
                     const float* wloT, int64_t M, int64_t N, int64_t K, const float* bias,
                     float* Y, int64_t ldy, int act, float alpha, int splits, float* partials,
                     int* status, cudaStream_t stream, float* ylo, int64_t ldylo) {
  if (!x_raw_ok(X, ldx)) return kErrInvalidArg;
  return gemm_with_splits(X, xlo, ldx, bop_k(whiT, wloT, K), M, N, K, bias, Y, ldy, act,
                          alpha, splits, partials, status, stream, ylo, ldylo);
}

bool x_raw_ok(const float* X, int64_t ldx) {
  return ((ldx & 3) == 0) && ((reinterpret_cast<uintptr_t>(X) & 15) == 0);
}

// ---------------------------------------------------------------------------
// MN-major B: the GEMM reads W itself as B_hi and W_lo [K, Np] as B_lo.
// Selected for M <= 4096 rows: there the transposing W split costs up to
// ~35% of a call (512-row MLP layers: 115 us of split per 200 us of GEMM),
// while the MN-major GEMM itself measured ~2-3% slower than the K-major one
// at M >= 8192 (same-box A/B at 8192^3 and 65536 x 4096 x 4096).
bool w_mn_ok(const float* W, int64_t ldw, int64_t M, int64_t N) {
  static const bool enabled = [] {
    const char* e = getenv("B200_W_MN");
    return !(e && e[0] == '0');
  }();
  return enabled && M <= 4096 && (N % 32) == 0 && ((ldw & 3) == 0) &&
         ((reinterpret_cast<uintptr_t>(W) & 15) == 0);
}

int64_t w_lo_mn_bytes(int64_t K, int64_t N) { return K * ((N + 3) & ~int64_t(3)) * 4; }

int split_lo_xw_f32(const float* X, int64_t ldx, int64_t M, int64_t K, float* xhi, float* xlo,
                    const float* W, int64_t ldw, int64_t N, float* wlo, cudaStream_t stream) {
  const int64_t Kp = split_pitch(K), Np = (N + 3) & ~int64_t(3);
  const int64_t xq = X ? M * (Kp / 4) : 0, wq = K * (Np / 4);
  // blocks in proportion to each part's quads, together about 16 per SM
  const int64_t cap = 148 * 16;
  const int x_blocks = xq ? (int)std::max<int64_t>(
                                1, std::min<int64_t>((xq + 255) / 256, cap * xq / (xq + wq) + 1))
                          : 0;
  const int w_blocks =
      (int)std::max<int64_t>(1, std::min<int64_t>((wq + 255) / 256, cap * wq / (xq + wq) + 1));
  split_lo_xw_kernel<<<(unsigned)(x_blocks + w_blocks), 256, 0, stream>>>(
      X, ldx, M, K, Kp, x_blocks, xhi, xlo, W, ldw, N, Np, wlo);
  count_launch();
  return launch_result();
}

int gemm_tf32x3_wmn(const float* xa, const float* xlo, int64_t ldx, const float* W, int64_t ldw,
                    const float* wlo, int64_t M, int64_t N, int64_t K, const float* bias,
                    float* Y, int64_t ldy, int act, float alpha, int splits, float* partials,
                    int* status, cudaStream_t stream, float* ylo, int64_t ldylo) {
  if (!x_raw_ok(xa, ldx) || !w_mn_ok(W, ldw, M, N)) return kErrInvalidArg;
  const BOp b{W, wlo, ldw, (N + 3) & ~int64_t(3), true};
  return gemm_with_splits(xa, xlo, ldx, b, M, N, K, bias, Y, ldy, act, alpha, splits,
                          partials, status, stream, ylo, ldylo);
}

}  // namespace b200
