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

#include <immintrin.h>
#include <time.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <thread>

#include "seq_protocol.hpp"

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

// ---------------------------------------------------------------------------
// Asynchronous bridge: a worker thread polls a mapped control block that the device
// writes (seq_protocol.hpp), so no host-function node sits in the stream.  The device
// posts a request (inputs written straight into pinned slot buffers by a kernel), runs
// on, and later reads the slot's output back with a bounded wait.  That is what lets a
// layer's CPU experts overlap the next layer's attention (expert deferral).
// ---------------------------------------------------------------------------
namespace {

constexpr int kMaxEngines = 1024;

struct AsyncBridge {
  void* engines[kMaxEngines] = {};   // one CPU engine per tiered layer; requests name theirs
  std::atomic<int> n_engines{0};
  int H = 0, K = 0, max_tokens = 0, slots = 2, spin_idle_us = 50;
  xtu::seq::Ctl* ctl = nullptr;   // pinned + mapped
  uint16_t* hx = nullptr;         // [slots][max_tokens][H] bf16
  int* hids = nullptr;            // [slots][max_tokens][K]
  float* hw = nullptr;            // [slots][max_tokens][K]
  float* hout = nullptr;          // [slots][max_tokens][H] fp32
  std::thread worker;
  std::atomic<bool> stop{false};
  std::atomic<bool> paused{false};
  std::atomic<bool> idle{true};   // worker is parked (paused) or between polls
  uint32_t done_local = 0;
  std::atomic<long long> runs{0}, pairs{0}, busy_ns{0};

  void loop() {
    auto last = std::chrono::steady_clock::now();
    while (!stop.load(std::memory_order_relaxed)) {
      if (paused.load()) {
        idle.store(true);
        std::this_thread::sleep_for(std::chrono::microseconds(100));
        continue;
      }
      idle.store(false);            // announce, then re-check: with pause()'s store-then-load
      if (paused.load()) continue;  // (all seq_cst) one of the two sides always sees the other
      const bool did = xtu::seq::worker_poll(ctl, done_local, slots, [&](int s, const xtu::seq::SlotMeta& m) {
        const auto t0 = std::chrono::steady_clock::now();
        const size_t xo = (size_t)s * max_tokens;
        const int mm = m.m < 0 ? 0 : (m.m > max_tokens ? max_tokens : m.m);
        const bool known = m.eng >= 0 && m.eng < n_engines.load(std::memory_order_acquire);
        int n = 0;
        if (mm > 0 && known)
          n = xtu_cpu_engine_forward(engines[m.eng], mm, K, hids + xo * K, hw + xo * K, hx + xo * H,
                                     hout + xo * H, m.lo, m.hi);
        else if (mm > 0)
          std::memset(hout + xo * H, 0, (size_t)mm * H * sizeof(float));   // unknown engine: contributes 0
        runs.fetch_add(1, std::memory_order_relaxed);
        if (n > 0) pairs.fetch_add(n, std::memory_order_relaxed);
        busy_ns.fetch_add(
            std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count(),
            std::memory_order_relaxed);
      });
      const auto now = std::chrono::steady_clock::now();
      if (did) {
        last = now;
      } else if (now - last > std::chrono::microseconds(spin_idle_us)) {
        idle.store(true);
        std::this_thread::sleep_for(std::chrono::microseconds(20));   // parked after spin_idle_us of no work
      } else {
        _mm_pause();
      }
    }
    idle.store(true);
  }
};

template <class T>
bool alloc_mapped(T** p, size_t bytes) {
  void* v = nullptr;
  if (cudaHostAlloc(&v, bytes, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  std::memset(v, 0, bytes);
  *p = static_cast<T*>(v);
  return true;
}

void free_async(AsyncBridge* b) {
  if (b->ctl) cudaFreeHost(b->ctl);
  if (b->hx) cudaFreeHost(b->hx);
  if (b->hids) cudaFreeHost(b->hids);
  if (b->hw) cudaFreeHost(b->hw);
  if (b->hout) cudaFreeHost(b->hout);
  delete b;
}

}  // namespace

extern "C" {

// slots in [1, 8]; the worker starts at once.  `eng` (may be null) becomes engine 0;
// more engines are added with xtu_async_bridge_add_engine.  Pointers (host addresses of mapped memory,
// valid on the device under unified addressing) come from xtu_async_bridge_ptrs.
void* xtu_async_bridge_create(void* eng, int H, int K, int max_tokens, int slots, int spin_idle_us) {
  if (slots < 1 || slots > xtu::seq::kMaxSlots || H <= 0 || K <= 0 || max_tokens <= 0) return nullptr;
  AsyncBridge* b = new AsyncBridge();
  b->engines[0] = eng;
  b->n_engines.store(eng ? 1 : 0);
  b->H = H;
  b->K = K;
  b->max_tokens = max_tokens;
  b->slots = slots;
  b->spin_idle_us = spin_idle_us < 0 ? 0 : spin_idle_us;
  const size_t rows = (size_t)slots * max_tokens;
  if (!alloc_mapped(&b->ctl, sizeof(xtu::seq::Ctl)) || !alloc_mapped(&b->hx, rows * H * 2) ||
      !alloc_mapped(&b->hids, rows * K * 4) || !alloc_mapped(&b->hw, rows * K * 4) ||
      !alloc_mapped(&b->hout, rows * H * 4)) {
    free_async(b);
    return nullptr;
  }
  b->worker = std::thread([b] { b->loop(); });
  return b;
}

// Register another engine; returns its index (requests name it), or -1 when full.
int xtu_async_bridge_add_engine(void* bridge, void* eng) {
  AsyncBridge* b = static_cast<AsyncBridge*>(bridge);
  if (!b || !eng) return -1;
  const int i = b->n_engines.load();
  if (i >= kMaxEngines) return -1;
  b->engines[i] = eng;
  b->n_engines.store(i + 1, std::memory_order_release);
  return i;
}

// out = {ctl, hx, hids, hw, hout}
int xtu_async_bridge_ptrs(void* bridge, void** out) {
  AsyncBridge* b = static_cast<AsyncBridge*>(bridge);
  if (!b) return -1;
  out[0] = b->ctl;
  out[1] = b->hx;
  out[2] = b->hids;
  out[3] = b->hw;
  out[4] = b->hout;
  return 0;
}

// out = {runs, pairs, busy_ns, req, done}
int xtu_async_bridge_stats(void* bridge, long long* out) {
  AsyncBridge* b = static_cast<AsyncBridge*>(bridge);
  if (!b) return -1;
  out[0] = b->runs.load();
  out[1] = b->pairs.load();
  out[2] = b->busy_ns.load();
  out[3] = __atomic_load_n(&b->ctl->req, __ATOMIC_ACQUIRE);
  out[4] = __atomic_load_n(&b->ctl->done, __ATOMIC_ACQUIRE);
  return 0;
}

// Stop (1) or restart (0) consuming requests; pausing waits (up to 1 s) until the
// worker is parked.  Used to recover after a device wait ran out of time and by tests.
int xtu_async_bridge_pause(void* bridge, int paused) {
  AsyncBridge* b = static_cast<AsyncBridge*>(bridge);
  if (!b) return -1;
  b->paused.store(paused != 0);
  if (!paused) return 0;
  for (int i = 0; i < 10000; ++i) {
    if (b->idle.load()) return 0;
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
  return -2;
}

// Forget all requests (host side).  Call with the worker paused and the device idle;
// the device counters are zeroed by the caller.
int xtu_async_bridge_reset(void* bridge) {
  AsyncBridge* b = static_cast<AsyncBridge*>(bridge);
  if (!b) return -1;
  if (!b->paused.load() || !b->idle.load()) return -2;
  b->done_local = 0;
  __atomic_store_n(&b->ctl->req, 0u, __ATOMIC_RELEASE);
  __atomic_store_n(&b->ctl->done, 0u, __ATOMIC_RELEASE);
  return 0;
}

void xtu_async_bridge_destroy(void* bridge) {
  AsyncBridge* b = static_cast<AsyncBridge*>(bridge);
  if (!b) return;
  b->stop.store(true);
  if (b->worker.joinable()) b->worker.join();
  free_async(b);
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
