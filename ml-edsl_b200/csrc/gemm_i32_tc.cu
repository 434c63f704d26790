// i32 GEMM on the tensor cores, exact modulo 2^32.
//
// Reference semantics: linalg.fill(0) + linalg.matmul on i32 tensors lower to
// arith.muli / arith.addi, which wrap modulo 2^32
// (cpp/src/builders/LinalgBuilder.cpp:106-139; tested exactly at
// tests/linalg/test_matmul_execution.py:93-103); the dense form adds an i32
// bias with arith.addi (cpp/src/builders/LinalgBuilder.cpp:301-339).
//
// Byte-sliced products. Each i32 is read as its 32-bit two's-complement
// pattern u = sum_p u_p 256^p with unsigned bytes u_p (p = 0..3). Then
//   (A B)[m][n] mod 2^32 = sum_{s=0..3} 256^s S_s[m][n] mod 2^32,
//   S_s = sum_{i+j=s} sum_k A_i[m][k] B_j[k][n],
// because every byte product with i + j >= 4 is a multiple of 2^32. The ten
// products A_i B_j (i + j <= 3) run as tcgen05.mma.kind::i8 (u8 x u8 -> s32)
// into four TMEM accumulators, one per shift s; the epilogue forms
// sum_s S_s << 8s with wrapping 32-bit adds and adds the bias the same way.
// An accumulator sums at most 4 * Kr * 255^2 with Kr <= 8192 (the K range of
// one work unit; longer K is split and the partial sums added modulo 2^32), which
// is below 2^31: the s32 accumulators never overflow.
//
// Layout: A's bytes as four planes [4][M][Kp] and B's as four transposed
// planes [4][N][Kp] (K-major, Kp = roundup(K, 32), pad bytes zero), written by
// one HBM pass. Per stage the producer loads all four planes of a 128 x 64-byte
// A tile and of a 128 x 64-byte B tile with one 3-D TMA each (64-byte swizzle).
// Roles as in the f32 kernel: warp 0 TMA, warp 1 TMEM allocation + MMA issue,
// warps 2-9 epilogue; persistent over (tile, K-split) units.
#include <cuda.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include "ptx.cuh"
#include "sched.cuh"
#include "kernels.h"

namespace b200 {

namespace {

constexpr int kQBM = 128, kQBN = 128;  // output tile
constexpr int kQBK = 64;               // K bytes per stage: 64-byte rows, 64-byte swizzle
constexpr int kQStages = 3;
constexpr int kQPlaneA = kQBM * kQBK;  // 8 KB
constexpr int kQPlaneB = kQBN * kQBK;  // 8 KB
constexpr int kQStageBytes = 4 * kQPlaneA + 4 * kQPlaneB;  // 64 KB
constexpr int kQBarOffset = kQStages * kQStageBytes;
constexpr int kQStoreStage = kQBarOffset + 256;  // 4 KB per epilogue warp (store staging)
constexpr int kQSmemBytes = kQStoreStage + 8 * 4096 + 1024;  // + alignment slack
constexpr int kQEpiWarps = 8;
constexpr int kQThreads = 64 + 32 * kQEpiWarps;
constexpr int kQTmemCols = 4 * kQBN;  // one 128 x 128 s32 accumulator per shift
constexpr int kQMaxKr = 8192;         // K per unit: 4 * 8192 * 255^2 < 2^31
constexpr int kQGroupM = 16;
static_assert(kQSmemBytes <= 232448, "shared memory over the sm_100 limit");

struct QEpilogue {
  int32_t* C;
  int64_t ldc;
  const int32_t* bias;  // may be null
  int64_t M, N;
  int vec_out;   // C 16-byte aligned and ldc % 4 == 0
  int32_t* part; // cut tiles: raw partial sums, tile-local [piece][r][128][128]
};

// K-major operand tile with 64-byte rows (64 bytes of K), 8-row groups 512 B
// apart; k-step kk (32 bytes of K) starts 32 * kk bytes into the row.
__device__ __forceinline__ uint64_t qdesc(uint32_t addr) { return umma_desc_k<4, 512>(addr); }

}  // namespace

__global__ void __launch_bounds__(kQThreads, 1)
    gemm_i32_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB, Sched sc, QEpilogue ep,
                       int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kQBarOffset);  // TMA -> MMA
  uint64_t* empty = full + kQStages;                                  // MMA -> TMA
  uint64_t* tfull = empty + kQStages;  // MMA -> epilogue: accumulators complete
  uint64_t* tempty = tfull + 1;        // epilogue -> MMA: accumulators read out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Work units (whole tiles, then pieces of cut tiles) of the schedule `sc`.
  auto unit_of = [&](int u) { return unit_at(sc, u, kQBM, kQBN); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, kQEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kQTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched as a programmatic dependent of the planes pass: the prologue
  // above overlaps its tail; the planes are read only after it has completed.
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      for (int u = blockIdx.x; u < sc.units && !*abort_flag; u += gridDim.x) {
        const Unit w = unit_of(u);
        bool ok = true;
        for (int kb = 0; kb < w.nkb; ++kb, ++it) {
          const int s = it % kQStages;
          const int round = it / kQStages;
          if (round > 0 &&
              !mbar_wait(&empty[s], (round - 1) & 1, status, kDevTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kQStageBytes;
          const int kx = (w.kb0 + kb) * kQBK;
          mbar_arrive_expect_tx(&full[s], kQStageBytes);
          tma_load_3d(st, &tmA, &full[s], kx, w.m0, 0);                 // 4 planes of A
          tma_load_3d(st + 4 * kQPlaneA, &tmB, &full[s], kx, w.n0, 0);  // 4 planes of B^T
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_u8_s32(kQBM, kQBN);
      int it = 0, tu = 0;  // k-blocks and units issued by this CTA
      bool ok = true;
      for (int u = blockIdx.x; u < sc.units && ok; u += gridDim.x) {
        const Unit w = unit_of(u);
        if (tu > 0) {  // the previous unit's accumulators must have been read out
          if (!mbar_wait(tempty, (tu - 1) & 1, status, kDevTimeoutAccum, abort_flag)) break;
          tc_fence_after();
        }
        for (int kb = 0; kb < w.nkb; ++kb, ++it) {
          const int s = it % kQStages;
          if (!mbar_wait(&full[s], (it / kQStages) & 1, status, kDevTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * kQStageBytes);
#pragma unroll
          for (int kk = 0; kk < kQBK / 32; ++kk) {
#pragma unroll
            for (int sh = 0; sh < 4; ++sh) {
#pragma unroll
              for (int i = 0; i <= sh; ++i) {
                const int j = sh - i;
                const uint32_t first = (kb == 0 && kk == 0 && i == 0) ? 0u : 1u;
                umma_i8(tmem_base + sh * kQBN, qdesc(st + i * kQPlaneA + kk * 32),
                        qdesc(st + 4 * kQPlaneA + j * kQPlaneB + kk * 32), idesc, first);
              }
            }
          }
          umma_commit(&empty[s]);  // stage s may be refilled once these MMAs finish
        }
        if (!ok) break;
        umma_commit(tfull);
        ++tu;
      }
    }
  } else {
    // ------------------------------------------------ epilogue (8 warps)
    // Warp w reads TMEM lane quarter w % 4 and column half (w - 2) / 4.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    int tu = 0;
#pragma unroll 1
    for (int u = blockIdx.x; u < sc.units && !*abort_flag; u += gridDim.x) {
      const Unit w = unit_of(u);
      if (!mbar_wait(tfull, tu & 1, status, kDevTimeoutAccum, abort_flag)) break;
      tc_fence_after();
      uint32_t acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0u;
#pragma unroll
      for (int sh = 0; sh < 4; ++sh) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + lane_off + sh * kQBN + half * 64 + g * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[g * 32 + j] += r[j] << (8 * sh);  // mod 2^32
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);  // the next unit's MMAs may start
      ++tu;
      const int lr = quarter * 32 + lane, lc0 = half * 64;
      if (w.piece >= 0) {  // raw sums of a piece, tile-local, whole rows
        int32_t* dst = ep.part + ((int64_t)(w.piece * sc.rest + w.r) * kQBM + lr) * kQBN + lc0;
#pragma unroll
        for (int j = 0; j < 64; j += 4)
          *reinterpret_cast<int4*>(dst + j) =
              make_int4((int)acc[j], (int)acc[j + 1], (int)acc[j + 2], (int)acc[j + 3]);
        continue;
      }
      const int64_t row = (int64_t)w.m0 + lr;
      const int64_t col0 = (int64_t)w.n0 + lc0;
      const int64_t row0 = row - lane;
      // The warp's whole 32 x 64 region inside C: pass it through shared
      // memory in 32 x 32 blocks (16-byte chunks XOR-swizzled by row) so that
      // each store instruction writes four whole 128-byte row segments
      // instead of 32 scattered 16-byte pieces.
      if (ep.vec_out && row0 + 32 <= ep.M && col0 + 64 <= ep.N) {
        uint32_t* stage = reinterpret_cast<uint32_t*>(smem + kQStoreStage + (warp - 2) * 4096);
        const bool bvec = ep.bias != nullptr && (reinterpret_cast<uintptr_t>(ep.bias) & 15) == 0;
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const int c = cb * 32 + ch * 4;
            uint4 bv = make_uint4(0u, 0u, 0u, 0u);
            if (bvec) {
              bv = __ldg(reinterpret_cast<const uint4*>(ep.bias + col0 + c));
            } else if (ep.bias != nullptr) {
              bv = make_uint4((uint32_t)__ldg(ep.bias + col0 + c),
                              (uint32_t)__ldg(ep.bias + col0 + c + 1),
                              (uint32_t)__ldg(ep.bias + col0 + c + 2),
                              (uint32_t)__ldg(ep.bias + col0 + c + 3));
            }
            *reinterpret_cast<uint4*>(stage + lane * 32 + ((ch ^ (lane & 7)) << 2)) =
                make_uint4(acc[c] + bv.x, acc[c + 1] + bv.y, acc[c + 2] + bv.z,
                           acc[c + 3] + bv.w);  // modulo 2^32
          }
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int r = k * 4 + (lane >> 3), ch = lane & 7;
            *reinterpret_cast<uint4*>(ep.C + (row0 + r) * ep.ldc + col0 + cb * 32 + ch * 4) =
                *reinterpret_cast<const uint4*>(stage + r * 32 + ((ch ^ (r & 7)) << 2));
          }
          __syncwarp();
        }
        continue;
      }
      if (row < ep.M) {
        int32_t* dst = ep.C + row * ep.ldc + col0;
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
          uint32_t v[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int64_t c = col0 + j + q;
            v[q] = acc[j + q] +
                   ((ep.bias != nullptr && c < ep.N) ? (uint32_t)__ldg(ep.bias + c) : 0u);
          }
          if (ep.vec_out && col0 + j + 4 <= ep.N) {
            *reinterpret_cast<int4*>(dst + j) =
                make_int4((int)v[0], (int)v[1], (int)v[2], (int)v[3]);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (col0 + j + q < ep.N) dst[j + q] = (int32_t)v[q];
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kQTmemCols);
  }
}

// One HBM pass: A [M, K] -> byte planes Ap [4][M][Kp]; B [K, N] -> transposed
// byte planes Bp [4][N][Kp]; pad bytes (k >= K) zero. Blocks [0, a_blocks)
// take A (4 consecutive k per thread, grid-stride). The others take B in
// 32 (k) x 32 (n) tiles, one per warp: lane n reads its column's 32 values
// (each a coalesced 128-byte warp load), packs them by byte in registers and
// writes 32 bytes (two 16-byte stores) to each plane's row n. 256 threads.
__global__ void __launch_bounds__(256)
    i32_planes_kernel(const int32_t* __restrict__ A, int64_t lda, int64_t M,
                      const int32_t* __restrict__ B, int64_t ldb, int64_t N, int64_t K,
                      int64_t Kp, int a_blocks, int tiles_n, int64_t b_tiles,
                      uint8_t* __restrict__ Ap, uint8_t* __restrict__ Bp) {
  // The GEMM that follows may start its prologue once every CTA is done.
  const PdlTriggerOnExit pdl_trigger_on_exit;
  if ((int)blockIdx.x < a_blocks) {
    const int64_t q_per_row = Kp >> 2;
    const int64_t total = M * q_per_row;
    const int vec = ((lda & 3) == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0);
    for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < total; i += (int64_t)a_blocks * 256) {
      const int64_t m = i / q_per_row;
      const int64_t k = (i - m * q_per_row) << 2;
      uint32_t v[4];
      if (vec && k + 4 <= K) {
        const int4 t = __ldg(reinterpret_cast<const int4*>(A + m * lda + k));
        v[0] = (uint32_t)t.x; v[1] = (uint32_t)t.y; v[2] = (uint32_t)t.z; v[3] = (uint32_t)t.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = (k + j < K) ? (uint32_t)__ldg(A + m * lda + k + j) : 0u;
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint32_t packed = ((v[0] >> (8 * p)) & 0xFFu) | (((v[1] >> (8 * p)) & 0xFFu) << 8) |
                                (((v[2] >> (8 * p)) & 0xFFu) << 16) |
                                (((v[3] >> (8 * p)) & 0xFFu) << 24);
        *reinterpret_cast<uint32_t*>(Ap + (p * M + m) * Kp + k) = packed;
      }
    }
    return;
  }
  const int64_t tile = (int64_t)(blockIdx.x - a_blocks) * 8 + (threadIdx.x >> 5);
  if (tile >= b_tiles) return;
  const int64_t n = (tile % tiles_n) * 32 + (threadIdx.x & 31);
  const int64_t k0 = (tile / tiles_n) * 32;
  if (n >= N) return;
  uint32_t w[4][8];  // [plane][4-byte word of the 32 k]
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    uint32_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + 4 * g + j;
      v[j] = k < K ? (uint32_t)__ldg(B + k * ldb + n) : 0u;
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
      w[p][g] = ((v[0] >> (8 * p)) & 0xFFu) | (((v[1] >> (8 * p)) & 0xFFu) << 8) |
                (((v[2] >> (8 * p)) & 0xFFu) << 16) | (((v[3] >> (8 * p)) & 0xFFu) << 24);
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    uint8_t* row = Bp + (p * N + n) * Kp + k0;
    *reinterpret_cast<uint4*>(row) = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
    if (k0 + 16 < Kp)  // Kp is a multiple of 16 (of 32 today): each half is in or out whole
      *reinterpret_cast<uint4*>(row + 16) = make_uint4(w[p][4], w[p][5], w[p][6], w[p][7]);
  }
}

// Cut tiles: C = sum over pieces of part[piece][r] (+ bias), modulo 2^32.
__global__ void __launch_bounds__(256)
    piece_reduce_i32_kernel(const int32_t* __restrict__ part, Sched sc, int64_t M, int64_t N,
                            const int32_t* __restrict__ bias, int32_t* __restrict__ C,
                            int64_t ldc) {
  const int64_t tile_elems = (int64_t)kQBM * kQBN;
  const int64_t total = (int64_t)sc.rest * tile_elems;
  const int64_t piece_stride = (int64_t)sc.rest * tile_elems;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / tile_elems);
    const int64_t e = i - r * tile_elems;
    const int lr = (int)(e / kQBN), lc = (int)(e - (int64_t)lr * kQBN);
    int mt, nt;
    tile_coords(sc, sc.whole + r, mt, nt);
    const int64_t row = (int64_t)mt * kQBM + lr, col = (int64_t)nt * kQBN + lc;
    if (row >= M || col >= N) continue;
    uint32_t acc = 0;
    for (int p = 0; p < sc.pieces; ++p) acc += (uint32_t)part[p * piece_stride + i];
    if (bias) acc += (uint32_t)bias[col];
    C[row * ldc + col] = (int32_t)acc;
  }
}

namespace {

typedef CUresult (*EncodeTiledFnQ)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnQ encode_fn() {
  static EncodeTiledFnQ fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnQ>(p);
  }
  return fn;
}

// Byte planes [4][rows][Kp] as a 3-D u8 tensor {Kp, rows, 4}; box {64, 128, 4}.
int make_plane_map(CUtensorMap* map, const uint8_t* base, int64_t rows, int64_t Kp) {
  EncodeTiledFnQ enc = encode_fn();
  if (!enc) return driver_failure("cuTensorMapEncodeTiled entry point", 0);
  cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)rows, 4};
  cuuint64_t strides[2] = {(cuuint64_t)Kp, (cuuint64_t)(rows * Kp)};
  cuuint32_t box[3] = {kQBK, 128, 4};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : driver_failure("cuTensorMapEncodeTiled", (int)r);
}

int64_t al256(int64_t b) { return (b + 255) & ~int64_t(255); }
// Row pitch (bytes) of the byte planes: K rounded up to 32, so every row
// starts on a 32-byte L2 sector and each 64-byte TMA row segment covers
// exactly two sectors (a pitch of 16 mod 32 makes every other row straddle
// three).
int64_t kp_of(int64_t K) { return (K + 31) & ~int64_t(31); }

int sm_count_i32() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;  // host-side queries without a device
  }
  return n;
}

// Schedule (sched.cuh): 128 x 128 tiles; one tile over all of K costs ten
// 128 x 128 x 32 int8 MMAs (64 clocks each at the dense int8 rate) per 32
// bytes of K; no unit spans more than 8192 bytes of K (kQMaxKr), so a longer
// K cuts every tile.
Sched sched_i32(int64_t M, int64_t N, int64_t K) {
  const double t_tile = (double)((K + 31) / 32) * 10 * 64 / 1.5e9;
  return make_sched(M, N, K, kQBM, kQBN, kQBK, sm_count_i32(), t_tile, 4, kQMaxKr / kQBK, 16,
                    1, kQGroupM);
}

}  // namespace

void sched_query_i32(int64_t M, int64_t N, int64_t K, int64_t* out) {
  const Sched sc = sched_i32(M, N, K);
  const int64_t v[8] = {sc.tiles_m, sc.tiles_n, sc.whole, sc.rest, sc.pieces, sc.kb, sc.kbp,
                        sc.units};
  for (int i = 0; i < 8; ++i) out[i] = v[i];
}

int choose_splits_i32(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 1;
  const Sched sc = sched_i32(M, N, K);
  return sc.rest > 0 ? sc.pieces : 1;
}

int64_t gemm_i32_tc_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int64_t Kp = kp_of(K);
  const Sched sc = sched_i32(M, N, K);
  const int64_t part = sc.rest > 0 ? al256((int64_t)sc.pieces * sc.rest * kQBM * kQBN * 4) : 0;
  return al256(4 * M * Kp) + al256(4 * N * Kp) + part;
}

bool i32_tensor_core_enabled() {
  static const bool on = [] {
    const char* e = getenv("B200_I32_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

int gemm_i32_tc(const int32_t* A, int64_t lda, const int32_t* B, int64_t ldb,
                const int32_t* bias, int32_t* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                void* ws, int* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return kOk;
  if (K <= 0) return kErrInvalidArg;  // the caller fills bias / zeros for K == 0
  static std::atomic<uint64_t> attr_done{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_done.load() & bit)) {
    if (cudaFuncSetAttribute(gemm_i32_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kQSmemBytes) != cudaSuccess)
      return launch_result();
    attr_done.fetch_or(bit);
  }
  static int sms[64] = {0};
  if (sms[dev & 63] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return kErrCuda;
    sms[dev & 63] = n;
  }
  const int64_t Kp = kp_of(K);
  uint8_t* Ap = static_cast<uint8_t*>(ws);
  uint8_t* Bp = Ap + al256(4 * M * Kp);
  int32_t* part = reinterpret_cast<int32_t*>(Bp + al256(4 * N * Kp));

  // byte planes
  const int64_t aq = M * (Kp / 4);
  const int a_blocks = (int)std::max<int64_t>(1, std::min<int64_t>((aq + 255) / 256, 148 * 8));
  const int tiles_n32 = (int)((N + 31) / 32);
  const int64_t b_tiles = (int64_t)tiles_n32 * ((Kp + 31) / 32);
  const int64_t b_blocks = (b_tiles + 7) / 8;
  i32_planes_kernel<<<(unsigned)(a_blocks + b_blocks), 256, 0, stream>>>(
      A, lda, M, B, ldb, N, K, Kp, a_blocks, tiles_n32, b_tiles, Ap, Bp);
  count_launch();
  if (const int lr = launch_result()) return lr;

  CUtensorMap ta, tb;
  int rc = make_plane_map(&ta, Ap, M, Kp);
  if (rc == kOk) rc = make_plane_map(&tb, Bp, N, Kp);
  if (rc != kOk) return rc;

  const Sched sc = sched_i32(M, N, K);
  const int units = sc.units;
  QEpilogue ep;
  ep.M = M;
  ep.N = N;
  ep.C = C;
  ep.ldc = ldc;
  ep.bias = bias;
  ep.vec_out = ((ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
  ep.part = part;
  const int grid = std::min(units, sms[dev & 63]);  // persistent
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = kQSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_i32_tc_kernel, ta, tb, sc, ep, status);
  count_launch();
  if (const int lr = launch_result(e)) return lr;
  if (sc.rest > 0) {
    const int64_t elems = (int64_t)sc.rest * kQBM * kQBN;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((elems + 255) / 256, 148 * 16));
    piece_reduce_i32_kernel<<<blocks, 256, 0, stream>>>(part, sc, M, N, bias, C, ldc);
    count_launch();
    if (const int lr = launch_result()) return lr;
  }
  return kOk;
}

}  // namespace b200
