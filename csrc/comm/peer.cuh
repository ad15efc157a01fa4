// Cross-GPU flag barrier over peer memory (shared by the comm kernels).
//
// Each rank owns int flags[world].  Arriving at barrier e stores e into slot [me] of
// every peer's array (release, system scope); the barrier is passed once every slot
// of the rank's own array is >= e (acquire, system scope).  Waits are bounded by
// %globaltimer and by the library's status word: a timeout records
// XTU_ERR_PEER_TIMEOUT with the missing peer's rank and returns false.
#pragma once
#include "../cuda/ptx.cuh"

namespace xtu {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Arrive at barrier `e` and wait for all peers (threads 0..world-1 of the calling block
// take part; the caller syncs the block around it).  Returns false on timeout.
__device__ __forceinline__ bool peer_barrier(int* const* peer_flags, int rank, int world, int e, XtuStatus* st, uint32_t where,
                             uint64_t timeout_ns) {
  const int s = threadIdx.x;
  bool ok = true;
  if (s < world) {
    fence_acq_rel_sys();                       // order this rank's earlier stores before the flag
    st_release_sys(peer_flags[s] + rank, e);
    const int* mine = peer_flags[rank] + s;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_sys(mine) < e) {
      if ((++spins & 63u) == 0u) {
        if (globaltimer_ns() - t0 > timeout_ns) {
          report_error(st, XTU_ERR_PEER_TIMEOUT, where, (uint32_t)s);
          ok = false;
          break;
        }
        if (st && *reinterpret_cast<volatile uint32_t*>(&st->code) != 0u) { ok = false; break; }
      }
    }
  }
  return __syncthreads_and(ok);
}

}  // namespace xtu
