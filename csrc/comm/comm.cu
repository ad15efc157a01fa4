// Intra-node GPU communication over NVLink / NVSwitch peer memory (sm_100a).
//
// * IPC plumbing: export a device allocation (handle + offset from its base), map a
//   peer's export into this process.  Every rank then holds the same table of peer
//   pointers ("symmetric buffers"), and kernels read and write peer memory directly
//   with ordinary loads and stores (never TMA: a peer address never reaches a tensor
//   map).
// * Flag barrier: each rank owns an int array flags[world]; arriving at barrier e
//   means storing e into slot [me] of every peer's array (release, system scope) and
//   waiting until every slot of its own array is >= e (acquire, system scope).  The
//   epoch lives in device memory and is advanced by the barrier kernel itself, so the
//   same launch can be replayed from a CUDA graph.  Every wait is bounded by
//   %globaltimer; a wait that runs out records XTU_ERR_PEER_TIMEOUT (with the peer's
//   rank) in the status word and returns, so a missing peer never hangs the GPU.
// * One-shot all-reduce for decode-sized tensors: after a barrier, every rank reads
//   all peers' inputs and sums them in fp32 (each rank produces the full result);
//   a closing barrier keeps the inputs alive until every peer has read them.
//
// These replace the reference's TP all-reduce sites (vLLM custom all-reduce / NCCL,
// vllm_xiaotu_moe/hybrid_model.py:1987,2041,2196,2238) for the paths that keep the
// collective in this library.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstring>
#include "../cuda/ptx.cuh"
#include "peer.cuh"

namespace xtu {

// one block: epoch = ++*epoch_ptr (same sequence on every rank), then the barrier
__global__ void barrier_kernel(int* const* peer_flags, int* epoch_ptr, int rank, int world, XtuStatus* st,
                               uint64_t timeout_ns) {
  __shared__ int e;
  if (threadIdx.x == 0) e = *epoch_ptr + 1;
  __syncthreads();
  peer_barrier(peer_flags, rank, world, e, st, 200, timeout_ns);
  if (threadIdx.x == 0) *epoch_ptr = e;
}

// out[i] = sum_r peer_in[r][i]  (bf16 or fp32 in, same type out; fp32 accumulation,
// ranks summed in rank order so every rank computes bit-identical results)
template <typename T>
__global__ void allreduce_sum_kernel(const void* const* peer_in, T* out, int64_t n, int world) {
  const int64_t n8 = n / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < world; ++r) {
      const T* src = reinterpret_cast<const T*>(peer_in[r]) + i * 8;
      if constexpr (sizeof(T) == 2) {
        const uint4 v = *reinterpret_cast<const uint4*>(src);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[2 * j] += bf16_lo(w[j]);
          acc[2 * j + 1] += bf16_hi(w[j]);
        }
      } else {
        const float4 a = *reinterpret_cast<const float4*>(src);
        const float4 b = *reinterpret_cast<const float4*>(src + 4);
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
      }
    }
    T* dst = out + i * 8;
    if constexpr (sizeof(T) == 2) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                                  pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
    } else {
      *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

// Two-shot all-reduce: rank r sums slice r of every rank's input (reads over NVLink) and
// stores the sum into slice r of every rank's output (writes over NVLink), so each byte
// crosses the links twice instead of W-1 times (large tensors, e.g. prefill activations).
template <typename T>
__global__ void allreduce_twoshot_kernel(const void* const* peer_in, void* const* peer_out, int64_t n, int rank,
                                         int world) {
  const int64_t n8 = n / 8;
  const int64_t per = (n8 + world - 1) / world;
  const int64_t lo = per * rank, hi = min(n8, lo + per);
  for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < world; ++r) {
      const T* src = reinterpret_cast<const T*>(peer_in[r]) + i * 8;
      if constexpr (sizeof(T) == 2) {
        const uint4 v = *reinterpret_cast<const uint4*>(src);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[2 * j] += bf16_lo(w[j]);
          acc[2 * j + 1] += bf16_hi(w[j]);
        }
      } else {
        const float4 a = *reinterpret_cast<const float4*>(src);
        const float4 b = *reinterpret_cast<const float4*>(src + 4);
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
      }
    }
    for (int r = 0; r < world; ++r) {
      const int dst_rank = (rank + r) % world;     // stagger the destinations across ranks
      T* dst = reinterpret_cast<T*>(peer_out[dst_rank]) + i * 8;
      if constexpr (sizeof(T) == 2) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                                    pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
      } else {
        *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
      }
    }
  }
}

}  // namespace xtu

using namespace xtu;

extern "C" {

// Export: handle (64 bytes) of the allocation containing ptr, and ptr's offset in it.
typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  }
  return fn;
}

int xtu_ipc_handle(const void* ptr, void* handle_out, long long* offset_out) {
  AddrRangeFn range = addr_range_fn();
  if (!range) return -999;
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult cr = range(&base, &size, (CUdeviceptr)ptr);
  if (cr != CUDA_SUCCESS) return -1000 - (int)cr;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, (void*)base);
  if (e != cudaSuccess) { cudaGetLastError(); return -(int)e; }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (long long)((CUdeviceptr)ptr - base);
  return 0;
}

int xtu_ipc_handle_size() { return (int)sizeof(cudaIpcMemHandle_t); }

// Import: map a peer's export; *ptr_out = mapped base + offset, *base_out = what to close.
int xtu_ipc_open(const void* handle, long long offset, void** ptr_out, void** base_out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) { cudaGetLastError(); return -(int)e; }
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return 0;
}

int xtu_ipc_close(void* base) {
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) { cudaGetLastError(); return -(int)e; }
  return 0;
}

// peer_flags: device array [world] of int* (each rank's flags[world]); epoch: device int
int xtu_peer_barrier(void* const* peer_flags, int* epoch, int rank, int world, void* status, long long timeout_ns,
                     cudaStream_t s) {
  if (world > 1024) return -2;
  barrier_kernel<<<1, world <= 32 ? 32 : ((world + 31) / 32) * 32, 0, s>>>(
      reinterpret_cast<int* const*>(peer_flags), epoch, rank, world, reinterpret_cast<XtuStatus*>(status),
      (uint64_t)timeout_ns);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// peer_in: device array [world] of each rank's symmetric input (this rank's input must
// already be in its own slot); out: local.  dtype 0 = bf16, 1 = fp32; n % 8 == 0.
int xtu_allreduce_oneshot(void* const* peer_in, void* out, long long n, int dtype, void* const* peer_flags,
                          int* epoch, int rank, int world, void* status, long long timeout_ns, cudaStream_t s) {
  if (n <= 0) return 0;
  if (n % 8) return -2;
  int rc = xtu_peer_barrier(peer_flags, epoch, rank, world, status, timeout_ns, s);
  if (rc < 0) return rc;
  const int64_t n8 = n / 8;
  int blocks = (int)((n8 + 255) / 256);
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (dtype == 0)
    allreduce_sum_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(reinterpret_cast<const void* const*>(peer_in),
                                                               (__nv_bfloat16*)out, n, world);
  else
    allreduce_sum_kernel<float><<<blocks, 256, 0, s>>>(reinterpret_cast<const void* const*>(peer_in), (float*)out,
                                                       n, world);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return -(int)e;
  rc = xtu_peer_barrier(peer_flags, epoch, rank, world, status, timeout_ns, s);
  return rc < 0 ? rc : 3;
}

// peer_in / peer_out: device arrays [world] of each rank's symmetric input / output; this
// rank's input already written.  On return (in stream order) every rank's output holds the sum.
int xtu_allreduce_twoshot(void* const* peer_in, void* const* peer_out, long long n, int dtype,
                          void* const* peer_flags, int* epoch, int rank, int world, void* status, long long timeout_ns,
                          cudaStream_t s) {
  if (n <= 0) return 0;
  if (n % 8) return -2;
  int rc = xtu_peer_barrier(peer_flags, epoch, rank, world, status, timeout_ns, s);
  if (rc < 0) return rc;
  const int64_t slice8 = (n / 8 + world - 1) / world;
  int blocks = (int)((slice8 + 255) / 256);
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  if (dtype == 0)
    allreduce_twoshot_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(reinterpret_cast<const void* const*>(peer_in),
                                                                   peer_out, n, rank, world);
  else
    allreduce_twoshot_kernel<float><<<blocks, 256, 0, s>>>(reinterpret_cast<const void* const*>(peer_in), peer_out, n,
                                                           rank, world);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return -(int)e;
  rc = xtu_peer_barrier(peer_flags, epoch, rank, world, status, timeout_ns, s);
  return rc < 0 ? rc : 3;
}

}  // extern "C"
