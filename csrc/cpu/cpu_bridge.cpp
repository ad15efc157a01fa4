// Host <-> device bridge for the CPU expert tier, capturable in CUDA graphs.
//
// enqueue() records, on one stream: D2H copies of the step's activations (bf16), expert
// ids and routing weights into pinned staging buffers, a host-function node that runs
// the CPU engine on them, and an H2D copy of the engine's fp32 partial output.  The
// caller runs this on a side stream forked from the main stream after routing, computes
// the GPU-resident experts meanwhile, and joins before the combine, which adds the CPU
// partial -- so CPU and GPU experts run concurrently in decode and prefill.
// Each enqueue gets its own immutable parameter block from a ring (the reference fixed
// cross-request pollution the same way: xiaotu_moe/csrc/python_binding/binding.cpp:1160-1176);
// under graph replay the captured block is reused, which is correct because the captured
// shapes are fixed.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>

extern "C" int xtu_cpu_engine_forward(void* eng, int M, int K, const int* ids, const float* wts, const uint16_t* x,
                                      float* out, int lo, int hi);

namespace {

struct Bridge;

struct Call {
  Bridge* b;
  int M, lo, hi;
};

constexpr int kRing = 256;

struct Bridge {
  void* eng;
  int H, K, max_tokens;
  uint16_t* hx = nullptr;
  int* hids = nullptr;
  float* hw = nullptr;
  float* hout = nullptr;
  Call calls[kRing];
  std::atomic<int> next{0};
  std::atomic<long long> runs{0};
  std::atomic<long long> pairs{0};
};

void CUDART_CB host_forward(void* p) {
  Call* c = static_cast<Call*>(p);
  Bridge* b = c->b;
  const int n = xtu_cpu_engine_forward(b->eng, c->M, b->K, b->hids, b->hw, b->hx, b->hout, c->lo, c->hi);
  b->runs.fetch_add(1);
  if (n > 0) b->pairs.fetch_add(n);
}

}  // namespace

extern "C" {

void* xtu_cpu_bridge_create(void* eng, int H, int K, int max_tokens) {
  Bridge* b = new Bridge();
  b->eng = eng;
  b->H = H;
  b->K = K;
  b->max_tokens = max_tokens;
  const size_t nx = (size_t)max_tokens * H;
  if (cudaHostAlloc((void**)&b->hx, nx * 2, cudaHostAllocPortable) != cudaSuccess ||
      cudaHostAlloc((void**)&b->hids, (size_t)max_tokens * K * 4, cudaHostAllocPortable) != cudaSuccess ||
      cudaHostAlloc((void**)&b->hw, (size_t)max_tokens * K * 4, cudaHostAllocPortable) != cudaSuccess ||
      cudaHostAlloc((void**)&b->hout, nx * 4, cudaHostAllocPortable) != cudaSuccess) {
    delete b;
    return nullptr;
  }
  return b;
}

// x_dev [M, H] bf16 (row stride x_stride elements), ids/w [M, K], out_dev [M, H] fp32
int xtu_cpu_bridge_enqueue(void* bridge, cudaStream_t s, int M, const void* x_dev, int x_stride, const int* ids_dev,
                           const float* w_dev, float* out_dev, int lo, int hi) {
  Bridge* b = static_cast<Bridge*>(bridge);
  if (!b || M > b->max_tokens) return -1;
  if (M <= 0) return 0;
  cudaError_t e;
  if (x_stride == b->H)
    e = cudaMemcpyAsync(b->hx, x_dev, (size_t)M * b->H * 2, cudaMemcpyDeviceToHost, s);
  else
    e = cudaMemcpy2DAsync(b->hx, (size_t)b->H * 2, x_dev, (size_t)x_stride * 2, (size_t)b->H * 2, M,
                          cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return -(int)e;
  if ((e = cudaMemcpyAsync(b->hids, ids_dev, (size_t)M * b->K * 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return -(int)e;
  if ((e = cudaMemcpyAsync(b->hw, w_dev, (size_t)M * b->K * 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return -(int)e;
  Call* c = &b->calls[b->next.fetch_add(1) % kRing];
  c->b = b;
  c->M = M;
  c->lo = lo;
  c->hi = hi;
  if ((e = cudaLaunchHostFunc(s, host_forward, c)) != cudaSuccess) return -(int)e;
  if ((e = cudaMemcpyAsync(out_dev, b->hout, (size_t)M * b->H * 4, cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return -(int)e;
  return 0;
}

int xtu_cpu_bridge_stats(void* bridge, long long* out) {
  Bridge* b = static_cast<Bridge*>(bridge);
  if (!b) return -1;
  out[0] = b->runs.load();
  out[1] = b->pairs.load();
  return 0;
}

void xtu_cpu_bridge_destroy(void* bridge) {
  Bridge* b = static_cast<Bridge*>(bridge);
  if (!b) return;
  cudaFreeHost(b->hx);
  cudaFreeHost(b->hids);
  cudaFreeHost(b->hw);
  cudaFreeHost(b->hout);
  delete b;
}

}  // extern "C"

extern "C" {

// Page-lock host memory (e.g. the engine's weight shards) for full-speed DMA.
int xtu_host_register(void* p, long long bytes) {
  if (!p || bytes <= 0) return 0;
  cudaError_t e = cudaHostRegister(p, (size_t)bytes, cudaHostRegisterPortable);
  if (e != cudaSuccess) cudaGetLastError();  // not sticky: keep it from surfacing at an unrelated later call
  return e == cudaSuccess ? 0 : -(int)e;
}

int xtu_host_unregister(void* p) {
  if (!p) return 0;
  if (cudaHostUnregister(p) == cudaSuccess) return 0;
  cudaGetLastError();
  return -1;
}

}  // extern "C"

extern "C" {

// one host->device copy on `s` (used by the prefill ring and the pool swap-in)
int xtu_memcpy_h2d_async(void* dst, const void* src, long long bytes, cudaStream_t s) {
  if (bytes <= 0) return 0;
  cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyHostToDevice, s);
  return e == cudaSuccess ? 0 : -(int)e;
}

}  // extern "C"
