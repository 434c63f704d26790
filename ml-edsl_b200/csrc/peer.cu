// Stream-ordered barrier among the GPUs of a gathered (single-device result)
// dense call. Each rank's output buffer is mapped into every other rank, and
// next to it sits a flag array of one 32-bit slot per rank. A barrier of epoch
// e: rank r stores e into slot r of every peer's flags (a system-scope
// release, after a system-scope fence, so that every store this GPU made to
// peer memory before the barrier, e.g. the GEMM epilogue's, is visible
// first), then waits until every peer has stored e into its own flags
// (system-scope acquire). The wait is bounded: when it runs out the kernel
// records kDevTimeoutPeer in the status word and returns, and the host reads
// B200_ERR_DEVICE_TIMEOUT at the next b200_stream_sync; the context stays
// usable.
//
// Because the barrier is a kernel on the caller's stream, a gathered call
// needs no host synchronisation: "ready" (every peer's earlier work on its
// stream, which may still read its output buffer, is done) before the GEMM
// stores into the peers, "done" (every peer's stores into this buffer have
// landed) after it.
#include <cuda_runtime.h>
#include <cstdint>
#include "ptx.cuh"
#include "kernels.h"

namespace b200 {

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread per rank t: signal peer t, then wait for peer t's signal.
__global__ void peer_barrier_kernel(PeerFlags f, uint32_t epoch, uint64_t limit_ns,
                                    int* status) {
  const int t = threadIdx.x;
  if (t >= f.world || t == f.rank) return;
  __threadfence_system();  // this GPU's earlier stores to peer memory first
  st_release_sys(f.flags[t] + f.rank, epoch);
  const uint32_t* mine = f.flags[f.rank] + t;
  const uint64_t t0 = globaltimer();
  // epochs wrap modulo 2^32: "reached" is a non-negative signed difference
  while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
    if (globaltimer() - t0 > limit_ns) {
      if (status) atomicCAS(status, 0, kDevTimeoutPeer);
      return;
    }
  }
}

}  // namespace

int peer_barrier(const PeerFlags& f, uint32_t epoch, uint64_t limit_ns, int* status,
                 cudaStream_t stream) {
  peer_barrier_kernel<<<1, 32, 0, stream>>>(f, epoch, limit_ns, status);
  count_launch();
  return launch_result();
}

}  // namespace b200
