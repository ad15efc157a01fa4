// DeepSeek sparse attention (DSA, DeepSeek-V3.2-style MLA) for sm_100a: the lightning
// indexer and the per-query token selection.
//
//   dsa_index_score_kernel  I[t, j] = sum_h w[t, h] relu(q[t, h] . k[j])  for every context
//                           token j <= pos[t] of the query's sequence: one CTA per (64-key
//                           page, query); the query's <= 64 index heads and the page's 64
//                           index keys (128 wide, bf16) sit in shared memory and four warps
//                           form the 64 x 64 head-by-key products with mma.sync m16n8k16
//                           (ldmatrix fragments), then ReLU, weight and reduce over heads.
//                           w already carries n_heads^-1/2 and the softmax scale.
//   dsa_topk_kernel         the top-K positions of one query's scores (radix select over the
//                           order-preserving integer image of the fp32 scores: four 8-bit
//                           digit passes with a shared histogram), written in position order
//                           by block-wide scans (deterministic), as flat rows of the paged
//                           latent cache; fewer than K context tokens: all of them.
//   dsa_gather_kernel       the selected latent rows of every query into a contiguous block
//                           run, so the MLA latent decode kernel attends over them as one
//                           pseudo-sequence per query.
//
// The reference serves these layers through vLLM's sparse-MLA backends (its SM80 port:
// patches/upstream/pr3_body.md "Algorithm notes": per query, gather the top-k selected KV
// slots, then online-softmax attention over them); the indexer's fp8 quantisation and
// Hadamard rotation are not reproduced: the rotation leaves q . k unchanged, and the scores
// are computed in bf16 with fp32 accumulation.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cfloat>
#include "ptx.cuh"

namespace xtu {

constexpr int DSA_KEYS = 64;     // keys per page (the paged cache's block size)
constexpr int DSA_D = 128;       // index head dim
constexpr int DSA_LD = DSA_D + 8;  // padded bf16 row (272 bytes: conflict-free ldmatrix)

__device__ __forceinline__ void dsa_ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void dsa_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// grid (ceil(Lmax / 64), T); block 128.  q [T, nh, 128] bf16 (row stride q_stride elements),
// w [T, nh] fp32, kc [num_blocks * 64, 128] bf16 (the paged index-key cache, flat rows),
// seq [T] sequence of each query, pos [T] its last visible position; scores [T, ld] fp32:
// entries j <= pos[t] written (the top-k pass reads no others).
__global__ void __launch_bounds__(128) dsa_index_score_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride, int nh, const float* __restrict__ w,
    const __nv_bfloat16* __restrict__ kc, const int* __restrict__ bt, int bt_stride, const int* __restrict__ seq,
    const int* __restrict__ pos, int num_blocks, float* __restrict__ scores, long long ld, XtuStatus* st) {
  __shared__ __align__(16) __nv_bfloat16 sq[64 * DSA_LD];
  __shared__ __align__(16) __nv_bfloat16 sk[DSA_KEYS * DSA_LD];
  __shared__ float sw[64];
  __shared__ float part[4][DSA_KEYS];
  const int t = blockIdx.y, j0 = blockIdx.x * DSA_KEYS;
  const int p = pos[t];
  if (j0 > p) return;
  const int b = seq[t];
  const int page = bt[(size_t)b * bt_stride + j0 / DSA_KEYS];
  if (!XTU_IN_BOUNDS(page >= 0 && page < num_blocks, st, 240, page) || page < 0 || page >= num_blocks) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // stage: 16-byte chunks, 16 per 128-wide row
  for (int i = tid; i < 64 * 16; i += 128) {
    const int r = i >> 4, c = (i & 15) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < nh) v = *reinterpret_cast<const uint4*>(q + (size_t)t * q_stride + (size_t)r * DSA_D + c);
    *reinterpret_cast<uint4*>(sq + r * DSA_LD + c) = v;
    *reinterpret_cast<uint4*>(sk + r * DSA_LD + c) =
        *reinterpret_cast<const uint4*>(kc + ((size_t)page * DSA_KEYS + r) * DSA_D + c);
  }
  if (tid < 64) sw[tid] = tid < nh ? w[(size_t)t * nh + tid] : 0.f;
  __syncthreads();
  // warp w: heads 16 w .. 16 w + 15 against all 64 keys (8 n-tiles), 8 k-steps of 16
  float acc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  const uint32_t qa = smem_u32(sq), ka = smem_u32(sk);
#pragma unroll
  for (int k0 = 0; k0 < DSA_D; k0 += 16) {
    uint32_t a0, a1, a2, a3;
    dsa_ldsm_x4(qa + (((16 * warp + (lane & 15)) * DSA_LD + k0 + (lane >> 4) * 8) << 1), a0, a1, a2, a3);
#pragma unroll
    for (int n = 0; n < 8; n += 2) {
      uint32_t b0, b1, b2, b3;
      const int row = 8 * n + (lane & 7) + ((lane >> 4) << 3);
      dsa_ldsm_x4(ka + ((row * DSA_LD + k0 + ((lane >> 3) & 1) * 8) << 1), b0, b1, b2, b3);
      dsa_mma(acc[n], a0, a1, a2, a3, b0, b1);
      dsa_mma(acc[n + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  // relu, head weight, sum over this warp's 16 heads (rows g and g + 8 per lane, then the 8 g's)
  const int g = lane >> 2, tq = lane & 3;
  const float w0 = sw[16 * warp + g], w1 = sw[16 * warp + g + 8];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float v = fmaxf(acc[n][e], 0.f) * w0 + fmaxf(acc[n][2 + e], 0.f) * w1;
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (g == 0) part[warp][8 * n + 2 * tq + e] = v;
    }
  __syncthreads();
  if (tid < DSA_KEYS && j0 + tid <= p)
    scores[(size_t)t * ld + j0 + tid] = part[0][tid] + part[1][tid] + part[2][tid] + part[3][tid];
}

// order-preserving unsigned image of an fp32 score (NaN sorts lowest)
__device__ __forceinline__ uint32_t dsa_key(float f) {
  if (f != f) return 0u;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// block-wide exclusive scan of one int per thread (blockDim = 1024); returns the total
__device__ __forceinline__ int dsa_block_scan(int v, int& excl, int* wsum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    wsum[lane] = s;             // inclusive prefix over warps
  }
  __syncthreads();
  const int total = wsum[31];
  excl = x - v + (warp > 0 ? wsum[warp - 1] : 0);
  __syncthreads();              // wsum is reused by the next scan
  return total;
}

// grid T; block 1024.  The K best of scores[t][0 .. pos[t]] (all of them when fewer) ->
// out_rows[t][0 .. n) flat cache rows (bt[seq][j / 64] * 64 + j % 64) in position order,
// out_len[t] = n.
__global__ void __launch_bounds__(1024) dsa_topk_kernel(const float* __restrict__ scores, long long ld,
                                                        const int* __restrict__ pos, const int* __restrict__ seq,
                                                        const int* __restrict__ bt, int bt_stride, int K,
                                                        int* __restrict__ out_rows, int* __restrict__ out_len) {
  __shared__ int hist[256];
  __shared__ int wsum[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  const int t = blockIdx.x, tid = threadIdx.x;
  const int len = pos[t] + 1;
  const int* btr = bt + (size_t)seq[t] * bt_stride;
  int* orow = out_rows + (size_t)t * K;
  auto flat = [&](int j) { return btr[j / DSA_KEYS] * DSA_KEYS + (j % DSA_KEYS); };
  if (len <= K) {
    for (int j = tid; j < len; j += blockDim.x) orow[j] = flat(j);
    if (tid == 0) out_len[t] = len;
    return;
  }
  const float* sr = scores + (size_t)t * ld;
  uint32_t prefix = 0u, mask = 0u;
  int remaining = K;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int j = tid; j < len; j += blockDim.x) {
      const uint32_t k = dsa_key(sr[j]);
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1);
    }
    __syncthreads();
    if (tid == 0) {
      int cum = 0, d = 255;
      for (; d > 0; --d) {
        if (cum + hist[d] >= remaining) break;
        cum += hist[d];
      }
      s_prefix = prefix | ((uint32_t)d << shift);
      s_remaining = remaining - cum;
    }
    __syncthreads();
    prefix = s_prefix;
    remaining = s_remaining;
    mask |= 255u << shift;
  }
  // prefix: the K-th largest key; take every key above it and the first `remaining` equal ones
  int eq_base = 0, out_base = 0;
  for (int c0 = 0; c0 < len; c0 += blockDim.x) {
    const int j = c0 + tid;
    const uint32_t k = j < len ? dsa_key(sr[j]) : 0u;
    const bool gt = j < len && k > prefix, eq = j < len && k == prefix;
    int eq_ex;
    const int eq_tot = dsa_block_scan(eq ? 1 : 0, eq_ex, wsum);
    const bool take = gt || (eq && eq_base + eq_ex < remaining);
    int o_ex;
    const int o_tot = dsa_block_scan(take ? 1 : 0, o_ex, wsum);
    if (take) orow[out_base + o_ex] = flat(j);
    eq_base += eq_tot;
    out_base += o_tot;
  }
  if (tid == 0) out_len[t] = K;
}

// grid (ceil(K / 8), T); block 256 (a warp per row).  dst [T * kpad, D] <- src rows
// rows[t][i] (i < len[t]) at dst row t * kpad + i; D * 2 a multiple of 16 bytes.
__global__ void __launch_bounds__(256) dsa_gather_kernel(const uint4* __restrict__ src, int d16,
                                                         const int* __restrict__ rows, const int* __restrict__ lens,
                                                         int K, int kpad, long long num_rows, uint4* __restrict__ dst,
                                                         XtuStatus* st) {
  const int t = blockIdx.y;
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (i >= lens[t]) return;
  const int r = rows[(size_t)t * K + i];
  if (!XTU_IN_BOUNDS(r >= 0 && r < num_rows, st, 241, r) || r < 0 || r >= num_rows) return;
  const uint4* s = src + (size_t)r * d16;
  uint4* d = dst + ((size_t)t * kpad + i) * d16;
  for (int c = lane; c < d16; c += 32) d[c] = s[c];
}

}  // namespace xtu

using namespace xtu;

extern "C" {

// Lightning-indexer scores (see dsa_index_score_kernel): q [T, nh <= 64, 128] bf16 with row
// stride q_stride, w [T, nh] fp32, kc the index-key cache [num_blocks, 1, 64, 128] bf16,
// block_table [B, bt_stride], seq / pos [T]; scores [T, ld] fp32 (ld >= max pos + 1).
int xtu_dsa_index_scores(const void* q, int q_stride, int nh, const float* w, const void* kc,
                         const int* block_table, int bt_stride, const int* seq, const int* pos, int T, int max_len,
                         int num_blocks, float* scores, long long ld, void* status, cudaStream_t s) {
  if (T <= 0 || max_len <= 0) return 0;
  if (nh <= 0 || nh > 64 || q_stride % 8 != 0) return -2;
  dsa_index_score_kernel<<<dim3((max_len + DSA_KEYS - 1) / DSA_KEYS, T), 128, 0, s>>>(
      (const __nv_bfloat16*)q, q_stride, nh, w, (const __nv_bfloat16*)kc, block_table, bt_stride, seq, pos,
      num_blocks, scores, ld, reinterpret_cast<XtuStatus*>(status));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// Top-K selection per query row (see dsa_topk_kernel); out_rows [T, K] int32, out_len [T].
int xtu_dsa_topk(const float* scores, long long ld, const int* pos, const int* seq, const int* block_table,
                 int bt_stride, int T, int K, int* out_rows, int* out_len, cudaStream_t s) {
  if (T <= 0) return 0;
  if (K <= 0) return -2;
  dsa_topk_kernel<<<T, 1024, 0, s>>>(scores, ld, pos, seq, block_table, bt_stride, K, out_rows, out_len);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// Selected rows of the flat latent cache src [num_rows, D] bf16 -> dst [T * kpad, D].
int xtu_dsa_gather(const void* src, int D, long long num_rows, const int* rows, const int* lens, int T, int K,
                   int kpad, void* dst, void* status, cudaStream_t s) {
  if (T <= 0 || K <= 0) return 0;
  if ((D * 2) % 16 != 0 || kpad < K) return -2;
  dsa_gather_kernel<<<dim3((K + 7) / 8, T), 256, 0, s>>>((const uint4*)src, D * 2 / 16, rows, lens, K, kpad,
                                                         num_rows, (uint4*)dst, reinterpret_cast<XtuStatus*>(status));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

}  // extern "C"
