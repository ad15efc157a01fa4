// Sequence-number handshake between a GPU stream and a host worker thread, the
// asynchronous form of the CPU-expert bridge (the reference's XIAOTU_MOE_ASYNC path,
// xiaotu_moe/csrc/python_binding/binding.cpp:339-430 with cuStreamWriteValue32 /
// cuStreamWaitValue32; here the device side is a pair of kernels that poll mapped host
// memory with a time bound instead of stream memory operations).
//
// State:
//   host control block (pinned, mapped into the device's address space)
//     req   requests published by the device   (written by the device, read by the worker)
//     done  requests finished by the worker     (written by the worker, read by the device)
//     meta[slot] = {M, lo, hi, engine} of the request in that slot (written by the device)
//   device counters (device memory, survive CUDA-graph replays)
//     posted, consumed: requests posted / whose result the device has read back
//
// Request n lives in slot n % S.  The device may post n only when n - S has been
// consumed (its slot is free); it posts by writing the slot's inputs, a system-scope
// fence, then req = n + 1.  The worker computes request `done` whenever req > done and
// publishes done + 1 after its output is written.  The device consumes n by waiting
// (bounded) for done > n, copying the slot's output, then consumed = n + 1.  With
// expert deferral the device posts layer L before it consumes layer L - 1, so S = 2
// is the smallest ring that never stalls.
//
// Everything in this header is plain index arithmetic and the worker's poll step, so
// the device kernels (csrc/cuda/host_bridge.cu), the real worker (cpu_bridge.cpp) and
// the three-thread protocol simulator (tests/cpp/seq_protocol_sim.cpp) share one
// definition.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define XTU_SEQ_HD __host__ __device__ __forceinline__
#else
#define XTU_SEQ_HD inline
#endif

namespace xtu {
namespace seq {

constexpr int kMaxSlots = 8;

struct SlotMeta {
  int32_t m, lo, hi, eng;   // rows, expert range [lo, hi), engine (layer) index
};

// 64-byte separated so the device's and the worker's words never share a line
struct alignas(64) Ctl {
  uint32_t req;
  uint32_t pad0[15];
  uint32_t done;
  uint32_t pad1[15];
  SlotMeta meta[kMaxSlots];
};

// device-memory counters of one bridge
struct DevCounters {
  uint32_t posted;
  uint32_t consumed;
  uint32_t post_arrive;   // CTAs of the current post kernel that finished their rows
  uint32_t wait_arrive;   // CTAs of the current wait kernel that finished their rows
};

XTU_SEQ_HD int slot_of(uint32_t n, int slots) { return (int)(n % (uint32_t)slots); }

// may request n be posted, given `consumed` requests read back?
XTU_SEQ_HD bool slot_free(uint32_t n, uint32_t consumed, int slots) { return n < consumed + (uint32_t)slots; }

// is there a posted request the device has not read back?
XTU_SEQ_HD bool has_pending(uint32_t posted, uint32_t consumed) { return consumed < posted; }

// has the worker finished request n?
XTU_SEQ_HD bool finished(uint32_t done, uint32_t n) { return done > n; }

#if !defined(__CUDA_ARCH__)
// One poll of the worker: if the device has published a request the worker has not
// computed, run `compute(slot, meta)` on it and publish it as done.  Returns true when
// it did work.  `done_local` is the worker's own count (the published `done`).
template <class Compute>
inline bool worker_poll(Ctl* c, uint32_t& done_local, int slots, Compute&& compute) {
  const uint32_t r = __atomic_load_n(&c->req, __ATOMIC_ACQUIRE);
  if (r == done_local) return false;
  const int s = slot_of(done_local, slots);
  SlotMeta m;
  m.m = __atomic_load_n(&c->meta[s].m, __ATOMIC_RELAXED);
  m.lo = __atomic_load_n(&c->meta[s].lo, __ATOMIC_RELAXED);
  m.hi = __atomic_load_n(&c->meta[s].hi, __ATOMIC_RELAXED);
  m.eng = __atomic_load_n(&c->meta[s].eng, __ATOMIC_RELAXED);
  compute(s, m);
  ++done_local;
  __atomic_store_n(&c->done, done_local, __ATOMIC_RELEASE);
  return true;
}
#endif

}  // namespace seq
}  // namespace xtu
