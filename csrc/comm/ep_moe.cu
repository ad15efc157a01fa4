// Expert-parallel MoE dispatch over NVLink peer memory (sm_100a).
//
// World W ranks, E experts, rank o owns experts [o*El, (o+1)*El).  One layer call:
//
//   ep_route     (1 block)  histogram of this rank's (token, k) pairs per global expert;
//                           the row is stored into cnt[me][:] of EVERY rank (P2P), then a
//                           flag barrier; every rank now holds the same count matrix C[s][e]
//                           and derives, identically on every rank, the receive layout of
//                           each owner: rows sorted by (local expert, source rank).  Output:
//                           send_base[e] (where this rank's rows for e start in e's owner),
//                           seg[El+1] (this rank's receive segments), cursor[] zeroed.
//   ep_dispatch  (warp per pair)  row x[t] -> owner's receive buffer at send_base[e] + n
//                           (16-byte P2P stores), with (source rank * pair_cap + pair, weight)
//                           in the owner's receive metadata.
//   flag barrier            every owner has all of its rows.
//   grouped GEMMs (gemm_tc.cu, local TMA reads only): gate/up + SwiGLU, then down with the
//                           top-k weight in the epilogue and a P2P store of each output row
//                           into the SOURCE rank's slot buffer (xtu_grouped_gemm_ex).
//   flag barrier, then the usual per-token combine on each source rank.
//
// No tensor map ever covers peer memory: rows cross NVLink only through these stores.
// Replaces the reference's expert-parallel paths (CPU-expert EP with /dev/shm reduction,
// vllm_xiaotu_moe/hybrid_model.py:254-326; GPU-prefill EP + NCCL all-reduce, :2019-2044).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include "../cuda/ptx.cuh"
#include "peer.cuh"

namespace xtu {

constexpr int kRouteThreads = 1024;

// cnt_peers[r] -> rank r's count matrix [W][E] (int32); counts row of this rank = C[me]
__global__ void __launch_bounds__(kRouteThreads) ep_route_kernel(
    const int* __restrict__ ids, int n, int E, int El, int rank, int world, int* const* cnt_peers,
    int* const* peer_flags, int* epoch_ptr, int* __restrict__ send_base, int* __restrict__ cursor,
    int* __restrict__ seg, XtuStatus* st, uint64_t timeout_ns) {
  extern __shared__ int sm[];
  int* hist = sm;             // [E]
  int* tot = sm + E;          // [E]
  __shared__ int e_sh;
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  if (threadIdx.x == 0) e_sh = *epoch_ptr + 1;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  // all-gather of the count rows: row `rank` of every peer's matrix
  for (int r = 0; r < world; ++r) {
    int* dst = cnt_peers[r] + (size_t)rank * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) dst[e] = hist[e];
  }
  __syncthreads();
  const int ep = e_sh;
  if (!peer_barrier(peer_flags, rank, world, ep, st, 210, timeout_ns)) {
    if (threadIdx.x == 0) *epoch_ptr = ep;
    return;
  }
  const int* C = cnt_peers[rank];          // this rank's copy, [W][E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0;
    for (int s = 0; s < world; ++s) t += C[(size_t)s * E + e];
    tot[e] = t;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int o = e / El, le = e - o * El;
    int base = 0;
    for (int j = 0; j < le; ++j) base += tot[o * El + j];
    for (int s = 0; s < rank; ++s) base += C[(size_t)s * E + e];
    send_base[e] = base;
    cursor[e] = 0;
  }
  for (int le = threadIdx.x; le <= El; le += blockDim.x) {
    int base = 0;
    for (int j = 0; j < le; ++j) base += tot[rank * El + j];
    seg[le] = base;
  }
  if (threadIdx.x == 0) *epoch_ptr = ep;
}

// one warp per (token, k) pair
__global__ void ep_dispatch_kernel(const int* __restrict__ ids, const float* __restrict__ weights, int n, int K,
                                   int El, int E, int rank, const __nv_bfloat16* __restrict__ x, int H, int x_stride,
                                   const int* __restrict__ send_base, int* __restrict__ cursor,
                                   void* const* xp_peers, int* const* src_peers, float* const* w_peers, int pair_cap) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= n) return;
  const int e = ids[gw];
  if (e < 0 || e >= E) return;     // not routed (the combine skips it too)
  const int o = e / El;
  int pos = 0;
  if (lane == 0) pos = send_base[e] + atomicAdd(&cursor[e], 1);
  pos = __shfl_sync(0xffffffffu, pos, 0);
  if (lane == 0) {
    src_peers[o][pos] = rank * pair_cap + gw;
    w_peers[o][pos] = weights[gw];
  }
  const int t = gw / K;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * x_stride);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(xp_peers[o]) + (size_t)pos * H);
  for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
}

}  // namespace xtu

using namespace xtu;

extern "C" {

int xtu_ep_route(const int* ids, int n, int E, int El, int rank, int world, void* const* cnt_peers,
                 void* const* peer_flags, int* epoch, int* send_base, int* cursor, int* seg, void* status,
                 long long timeout_ns, cudaStream_t s) {
  if (E > 4096 || world > kRouteThreads || E != El * world) return -2;
  const size_t smem = 2 * (size_t)E * sizeof(int);
  ep_route_kernel<<<1, kRouteThreads, smem, s>>>(ids, n, E, El, rank, world,
                                                 reinterpret_cast<int* const*>(cnt_peers),
                                                 reinterpret_cast<int* const*>(peer_flags), epoch, send_base, cursor,
                                                 seg, reinterpret_cast<XtuStatus*>(status), (uint64_t)timeout_ns);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

int xtu_ep_dispatch(const int* ids, const float* weights, int T, int K, int El, int E, int rank, const void* x,
                    int H, int x_stride, const int* send_base, int* cursor, void* const* xp_peers,
                    void* const* src_peers, void* const* w_peers, int pair_cap, cudaStream_t s) {
  const int n = T * K;
  if (n <= 0) return 0;
  if (H % 8 || x_stride % 8 || n > pair_cap) return -2;
  ep_dispatch_kernel<<<(n * 32 + 255) / 256, 256, 0, s>>>(
      ids, weights, n, K, El, E, rank, (const __nv_bfloat16*)x, H, x_stride, send_base, cursor, xp_peers,
      reinterpret_cast<int* const*>(src_peers), reinterpret_cast<float* const*>(w_peers), pair_cap);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

}  // extern "C"
