// Thin inline-PTX wrappers for the sm_100a features the GEMM kernels use:
// mbarriers, TMA tile loads, TMEM allocation, tcgen05.mma / commit / ld.
//
// Every spin-wait here is bounded by wall-clock (%globaltimer): a wait that
// exceeds B200_WAIT_NS records an error code in the kernel's status word and
// returns false, so a protocol bug ends the kernel instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#ifndef B200_WAIT_NS
#define B200_WAIT_NS 2000000000ull  // 2 s; a legitimate wait is microseconds
#endif

namespace b200 {

// Status codes written by device code into the status word.
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,     // consumer waited too long for a TMA stage
  kDevTimeoutEmpty = 2,    // producer waited too long for a free stage
  kDevTimeoutAccum = 3,    // epilogue waited too long for the accumulator
  kDevTimeoutSelfTest = 4, // the self-test wait (nothing ever arrives) ran out
  kDevTimeoutPeer = 5,     // a peer-GPU barrier waited too long for another rank
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on `bar` reaching phase `parity`. Returns false on timeout
// (after recording `code` in *status); also returns false early when another
// role of the CTA has already recorded a failure (*abort_flag != 0).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* status,
                                              int code, volatile int* abort_flag,
                                              uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit_ns) {
      if (status) atomicCAS(status, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          volatile int* abort_flag) {
  return mbar_wait_for(bar, parity, status, code, abort_flag, B200_WAIT_NS);
}

// ---------------------------------------------------------------- multicast
// Stores through an NVSwitch multicast address: one store reaches the same
// offset in every GPU's memory bound to the multicast object (NVLS).
__device__ __forceinline__ void multimem_st_v4(float* mc, float4 v) {
  asm volatile("multimem.st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void multimem_st(float* mc, float v) {
  asm volatile("multimem.st.global.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialization attribute may begin once every CTA of its predecessor
// in the stream has executed pdl_trigger() or exited; pdl_wait() then blocks
// until the predecessor has completed and its memory writes are visible (it
// returns at once when there is no such predecessor).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Triggers when the CTA's thread leaves the kernel, whatever the exit path.
struct PdlTriggerOnExit {
  __device__ ~PdlTriggerOnExit() { pdl_trigger(); }
};

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------- TMEM
// Warp-collective: allocates `ncols` TMEM columns, writes the base address
// into *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to later
// async-proxy readers (the tensor core reading operands written by threads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- UMMA
// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with a 128- or 64-byte swizzle (rows of 128 B or 64 B; 8-row core groups
// SBO bytes apart). Bit layout (sm_100 "version 1" descriptor): [0,14)
// start>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version=1, [49,52) base
// offset, [61,64) layout (2 = SWIZZLE_128B, 4 = SWIZZLE_64B). Within a row,
// successive K-steps are addressed by advancing the start address.
template <uint32_t kLayout, uint32_t kSBO>
__device__ __forceinline__ uint64_t umma_desc_k(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // LBO (unused for swizzled K-major)
  d |= (uint64_t)(kSBO >> 4) << 32;       // SBO: 8 rows
  d |= (uint64_t)1 << 46;                 // descriptor version for sm_100
  d |= (uint64_t)kLayout << 61;
  return d;
}

// Shared-memory descriptor of an MN-major tf32 operand. For 32-bit MN-major
// operands the only layout is the 128-byte swizzle with 32-byte atomicity
// (layout type 1): K-rows of 128 bytes (32 elements along M/N), grouped by
// four, with the 32-byte chunks of a row XOR-ed by the row index mod 4 (what
// TMA writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B). kLBO is the byte
// stride between 32-element blocks along M/N, kSBO between 4-row groups
// along K.
template <uint32_t kLBO, uint32_t kSBO>
__device__ __forceinline__ uint64_t umma_desc_mn_sw128_32b(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((kLBO >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((kSBO >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)1 << 61;  // SWIZZLE_128B_BASE32B
  return d;
}

// Instruction descriptor for kind::tf32 with f32 accumulation, both operands
// K-major, tile M x N.  Fields: [4,6) D format (1=f32), [7,10) A format
// (2=tf32), [10,13) B format, [15] A major, [16] B major, [17,23) N>>3,
// [24,29) M>>4.
__host__ __device__ constexpr uint32_t idesc_tf32_f32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// The same with B MN-major (bit 16), A K-major.
__host__ __device__ constexpr uint32_t idesc_tf32_f32_bmn(int M, int N) {
  return idesc_tf32_f32(M, N) | (1u << 16);
}

// D[tmem] (+)= A[smem] * B[smem]; issued by a single thread.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for kind::i8 with unsigned 8-bit A and B (format
// 0), s32 accumulation (D format 2), both operands K-major, tile M x N.
__host__ __device__ constexpr uint32_t idesc_u8_s32(int M, int N) {
  return (2u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem] on 8-bit integers (K = 32 per instruction).
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Warp-collective TMEM load: 32 lanes x 32 consecutive 32-bit columns.
// Thread t of the warp receives row (lane base + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace b200
