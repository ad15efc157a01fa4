// Device side of the asynchronous CPU-expert bridge (protocol: csrc/cpu/seq_protocol.hpp).
//
// bridge_post_kernel  writes one request's inputs -- activations (bf16 [M, H]), expert
//                     ids and routing weights ([M, K]) -- straight into the request's
//                     slot of pinned, mapped host buffers, then publishes it: a
//                     system-scope fence and a release store of the request counter that
//                     the host worker polls.  No copy engine, no host-function node.
// bridge_wait_kernel  waits (bounded by %globaltimer) until the worker has finished the
//                     oldest unread request, then copies or adds its fp32 output [M, H]
//                     from host memory into a device buffer.
//
// The request numbers live in device memory (DevCounters) and are advanced by the
// kernels themselves, so a captured post/wait pair replays correctly from a CUDA graph.
// A wait that runs out of time records XTU_ERR_HOST_TIMEOUT and returns; posting into a
// slot whose result was not read back, or reading back with nothing posted, records
// XTU_ERR_PROTOCOL.  After either, the host pauses the worker and resets both sides.
//
// Replaces the reference's cuStreamWriteValue32 / cuStreamWaitValue32 handshake and its
// D2H/H2D copies (xiaotu_moe/csrc/python_binding/binding.cpp:993-1130).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "../cpu/seq_protocol.hpp"
#include "ptx.cuh"

namespace xtu {
namespace {

constexpr int kBridgeThreads = 256;
constexpr int kWaitChunkBytes = 8192;   // fp32 output bytes per CTA of the wait kernel

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Rows of x (bf16, row stride x_stride) go to hx; block 0 also copies ids and weights.
// The last block to finish publishes the request.
__global__ void __launch_bounds__(kBridgeThreads) bridge_post_kernel(
    const __nv_bfloat16* __restrict__ x, int x_stride, const int* __restrict__ ids, const float* __restrict__ w,
    int M, int H, int K, int lo, int hi, int eng, seq::Ctl* ctl, uint16_t* hx, int* hids, float* hw, int slots,
    int max_tokens, seq::DevCounters* dc, XtuStatus* st) {
  const uint32_t n = *reinterpret_cast<volatile uint32_t*>(&dc->posted);
  const uint32_t consumed = *reinterpret_cast<volatile uint32_t*>(&dc->consumed);
  if (!seq::slot_free(n, consumed, slots)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report_error(st, XTU_ERR_PROTOCOL, 1, n);
    return;
  }
  const int s = seq::slot_of(n, slots);
  const size_t base = (size_t)s * max_tokens;
  const int vec_per_row = H / 8;                       // 16-byte vectors of 8 bf16
  for (int r = blockIdx.x; r < M; r += gridDim.x) {
    const int4* src = reinterpret_cast<const int4*>(x + (size_t)r * x_stride);
    int4* dst = reinterpret_cast<int4*>(hx + (base + r) * H);
    for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x) dst[v] = src[v];
  }
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
      hids[base * K + i] = ids[i];
      hw[base * K + i] = w[i];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&dc->post_arrive, 1u);
    if (prev == gridDim.x - 1) {             // last block: every row is out
      __threadfence_system();
      volatile int32_t* meta = reinterpret_cast<volatile int32_t*>(&ctl->meta[s]);
      meta[0] = M;
      meta[1] = lo;
      meta[2] = hi;
      meta[3] = eng;
      __threadfence_system();
      st_release_sys_u32(&ctl->req, n + 1);
      dc->post_arrive = 0;
      dc->posted = n + 1;
    }
  }
}

__global__ void __launch_bounds__(kBridgeThreads) bridge_wait_kernel(
    const seq::Ctl* ctl, const float* hout, int slots, int max_tokens, int H, float* __restrict__ out,
    int out_stride, int M, int accumulate, seq::DevCounters* dc, long long timeout_ns, XtuStatus* st) {
  __shared__ int ok;
  const uint32_t n = *reinterpret_cast<volatile uint32_t*>(&dc->consumed);
  const uint32_t posted = *reinterpret_cast<volatile uint32_t*>(&dc->posted);
  if (!seq::has_pending(posted, n)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report_error(st, XTU_ERR_PROTOCOL, 2, n);
    return;
  }
  if (threadIdx.x == 0) {
    int good = 0;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if (seq::finished(ld_acquire_sys_u32(&ctl->done), n)) {
        good = 1;
        break;
      }
      if ((it & 15u) == 15u) {
        if (status_failed(st)) break;
        if (globaltimer_ns() - t0 > (uint64_t)timeout_ns) {
          report_error(st, XTU_ERR_HOST_TIMEOUT, 3, n);
          break;
        }
      }
      __nanosleep(256);
    }
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  // this CTA's chunk of the flattened [M, H] output, 16-byte vectors, 4 in flight per thread
  const int s = seq::slot_of(n, slots);
  const float* src = hout + (size_t)s * max_tokens * H;
  const int total4 = M * H / 4;
  const int per_cta = kWaitChunkBytes / 16;
  const int v0 = blockIdx.x * per_cta, v1 = min(total4, v0 + per_cta);
  const int vec_per_row = H / 4;
  for (int v = v0 + threadIdx.x; v < v1; v += 4 * blockDim.x) {
    float4 a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int vi = v + u * blockDim.x;
      if (vi < v1) a[u] = __ldcv(reinterpret_cast<const float4*>(src) + vi);   // uncached: new data each replay
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int vi = v + u * blockDim.x;
      if (vi >= v1) continue;
      const int r = vi / vec_per_row, c = (vi - r * vec_per_row) * 4;
      float4* d = reinterpret_cast<float4*>(out + (size_t)r * out_stride + c);
      if (accumulate) {
        float4 o = *d;
        o.x += a[u].x;
        o.y += a[u].y;
        o.z += a[u].z;
        o.w += a[u].w;
        *d = o;
      } else {
        *d = a[u];
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&dc->wait_arrive, 1u);
    if (prev == gridDim.x - 1) {
      dc->wait_arrive = 0;
      dc->consumed = n + 1;
    }
  }
}

}  // namespace
}  // namespace xtu

using namespace xtu;

extern "C" {

// Post one request for engine `eng`: x [M, H] bf16 (row stride x_stride), ids / w [M, K]
// contiguous, experts [lo, hi).
// H must be a multiple of 8 and x 16-byte aligned; M <= max_tokens.
int xtu_bridge_post(const void* x, int x_stride, const int* ids, const float* w, int M, int H, int K, int lo, int hi,
                    int eng, void* ctl, void* hx, void* hids, void* hw, int slots, int max_tokens, void* dev_counters,
                    void* status, cudaStream_t stream) {
  if (M < 0 || M > max_tokens || H % 8 != 0 || x_stride % 8 != 0 || slots < 1 || slots > seq::kMaxSlots) return -1;
  const int grid = M < 1 ? 1 : (M > 148 ? 148 : M);
  bridge_post_kernel<<<grid, kBridgeThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), x_stride, ids, w, M, H, K, lo, hi, eng, static_cast<seq::Ctl*>(ctl),
      static_cast<uint16_t*>(hx), static_cast<int*>(hids), static_cast<float*>(hw), slots, max_tokens,
      static_cast<seq::DevCounters*>(dev_counters), static_cast<XtuStatus*>(status));
  return cudaGetLastError() == cudaSuccess ? 1 : -2;   // one kernel launched
}

// Read back the oldest unread request: out [M, H] fp32 (row stride out_stride) = or +=
// the worker's result.  H and out_stride must be multiples of 4.
int xtu_bridge_wait(const void* ctl, const void* hout, int slots, int max_tokens, int H, float* out, int out_stride,
                    int M, int accumulate, void* dev_counters, long long timeout_ns, void* status,
                    cudaStream_t stream) {
  if (M < 0 || M > max_tokens || H % 4 != 0 || out_stride % 4 != 0 || slots < 1 || slots > seq::kMaxSlots)
    return -1;
  const long long bytes = (long long)M * H * 4;
  int grid = (int)((bytes + kWaitChunkBytes - 1) / kWaitChunkBytes);
  if (grid < 1) grid = 1;
  if (grid > 1024) return -1;                 // 8 MiB: far above any decode-sized request
  bridge_wait_kernel<<<grid, kBridgeThreads, 0, stream>>>(
      static_cast<const seq::Ctl*>(ctl), static_cast<const float*>(hout), slots, max_tokens, H, out, out_stride, M,
      accumulate, static_cast<seq::DevCounters*>(dev_counters), timeout_ns, static_cast<XtuStatus*>(status));
  return cudaGetLastError() == cudaSuccess ? 1 : -2;   // one kernel launched
}

}  // extern "C"
