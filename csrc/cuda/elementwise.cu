// Memory-bound hot ops around the tensor-core GEMMs (sm_100a):
//   * RMSNorm with fused residual add (W15)
//   * RoPE (full / partial, NeoX or interleaved) + optional per-head q/k RMSNorm,
//     fused with the paged KV-cache write (W16)
//   * router: softmax / sigmoid scoring, correction bias, group-limited top-k,
//     renormalisation and scaling, one warp per token (W8; replaces vLLM's
//     fused_topk_bias used at vllm_xiaotu_moe/hybrid_model.py:1877-1890)
//   * MoE routing permute: histogram -> prefix sum -> scatter + row gather (W3;
//     replaces the torch argsort/scatter/cumsum of gpu_prefill.py:800-883),
//     with an id filter that sends pairs of other tiers (CPU / remote) nowhere (W7)
//   * MoE combine: deterministic per-token sum of the top-k slot rows (+ shared
//     expert, + optional extra partial), no global atomics (W2)
//   * greedy argmax and embedding gather
// All kernels vectorise to 16-byte accesses where the row length allows.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cfloat>
#include "ptx.cuh"
#include "launch.cuh"
#include "../comm/peer.cuh"
#include "xtu_argmax_static.h"
#include <mutex>

namespace xtu {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = l < NT / 32 ? sh[l] : 0.f;
    t = warp_sum(t);
    if (l == 0) sh[0] = t;
  }
  __syncthreads();
  const float r = sh[0];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------
// RMSNorm:  r = x (+ residual);  residual_out = r;  y = r * rsqrt(mean(r^2) + eps) * (w [+ 1])
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                     const __nv_bfloat16* __restrict__ residual,
                                                     __nv_bfloat16* __restrict__ residual_out,
                                                     const __nv_bfloat16* __restrict__ w,
                                                     __nv_bfloat16* __restrict__ y, int H, float eps, int add_one,
                                                     int x_stride, int y_stride, uint4* __restrict__ y16) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  extern __shared__ float row[];  // H floats
  __shared__ float sh[32];
  const int t = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)t * x_stride;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += NT * 8) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + i);
    const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) { v[2 * j] = bf16_lo(xs[j]); v[2 * j + 1] = bf16_hi(xs[j]); }
    if (residual) {
      const uint4 rv = *reinterpret_cast<const uint4*>(residual + (size_t)t * H + i);
      const uint32_t rs[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) { v[2 * j] += bf16_lo(rs[j]); v[2 * j + 1] += bf16_hi(rs[j]); }
      uint4 o;
      o.x = pack_bf16x2(v[0], v[1]); o.y = pack_bf16x2(v[2], v[3]);
      o.z = pack_bf16x2(v[4], v[5]); o.w = pack_bf16x2(v[6], v[7]);
      *reinterpret_cast<uint4*>(residual_out + (size_t)t * H + i) = o;
      // normalise the bf16-rounded sum, as an unfused add-then-norm would
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t pj = j == 0 ? o.x : j == 1 ? o.y : j == 2 ? o.z : o.w;
        v[2 * j] = bf16_lo(pj); v[2 * j + 1] = bf16_hi(pj);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) { row[i + j] = v[j]; ss += v[j] * v[j]; }
  }
  const float tot = block_sum<NT>(ss, sh);
  const float inv = rsqrtf(tot / (float)H + eps);
  __nv_bfloat16* yr = y + (size_t)t * y_stride;
  for (int i = threadIdx.x * 8; i < H; i += NT * 8) {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + i);
    const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float w0 = bf16_lo(ws[j]), w1 = bf16_hi(ws[j]);
      if (add_one) { w0 += 1.f; w1 += 1.f; }
      o[j] = pack_bf16x2(row[i + 2 * j] * inv * w0, row[i + 2 * j + 1] * inv * w1);
    }
    *reinterpret_cast<uint4*>(yr + i) = make_uint4(o[0], o[1], o[2], o[3]);
    // the fp8-weight GEMVs' activation form (f16 x 2^-8) of the same bf16 values
    if (y16) y16[((size_t)t * H + i) >> 3] = bf16x8_f16x8_s8(make_uint4(o[0], o[1], o[2], o[3]));
  }
}

// Tensor-parallel sum + residual add + RMSNorm (the consumer of xtu_gemv_tp): waits
// (bounded) until every rank's partial rows have landed in this rank's receive buffer,
// sums them in rank order in fp32, rounds to bf16 (the all-reduce result), then adds
// the residual and normalises exactly as rmsnorm_kernel.  One CTA per token; the CTA
// that finishes last publishes the epoch for the next producer.
template <int NT>
__global__ void __launch_bounds__(NT) tp_sum_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ recv, long long slot, int world, int H, const int* flags, const int* ep_p,
    int* ep_c, int* done, const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ residual_out,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y, float eps, int add_one, XtuStatus* st,
    long long timeout_ns) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  extern __shared__ float row[];  // H floats
  __shared__ float sh[32];
  const int t = blockIdx.x;
  const int e = *ep_p, par = e & 1;
  bool ok = true;
  if ((int)threadIdx.x < world) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_sys(flags + threadIdx.x) < e) {
      if ((++spins & 63u) == 0u) {
        if (globaltimer_ns() - t0 > (uint64_t)timeout_ns) {
          report_error(st, XTU_ERR_PEER_TIMEOUT, 210, threadIdx.x);
          ok = false;
          break;
        }
        if (status_failed(st)) { ok = false; break; }
      }
    }
  }
  if (!__syncthreads_and(ok)) return;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += NT * 8) {
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < world; ++p) {
      const uint4 pv = __ldcg(reinterpret_cast<const uint4*>(recv + (size_t)(par * world + p) * slot +
                                                             (size_t)t * H + i));
      const uint32_t ps[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) { v[2 * j] += bf16_lo(ps[j]); v[2 * j + 1] += bf16_hi(ps[j]); }
    }
    uint4 xs4;   // the all-reduce result in bf16, as the unfused path would hold it
    xs4.x = pack_bf16x2(v[0], v[1]); xs4.y = pack_bf16x2(v[2], v[3]);
    xs4.z = pack_bf16x2(v[4], v[5]); xs4.w = pack_bf16x2(v[6], v[7]);
    const uint32_t xs[4] = {xs4.x, xs4.y, xs4.z, xs4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) { v[2 * j] = bf16_lo(xs[j]); v[2 * j + 1] = bf16_hi(xs[j]); }
    const uint4 rv = *reinterpret_cast<const uint4*>(residual + (size_t)t * H + i);
    const uint32_t rs[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) { v[2 * j] += bf16_lo(rs[j]); v[2 * j + 1] += bf16_hi(rs[j]); }
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]); o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]); o.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(residual_out + (size_t)t * H + i) = o;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t pj = j == 0 ? o.x : j == 1 ? o.y : j == 2 ? o.z : o.w;
      v[2 * j] = bf16_lo(pj); v[2 * j + 1] = bf16_hi(pj);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) { row[i + j] = v[j]; ss += v[j] * v[j]; }
  }
  const float tot = block_sum<NT>(ss, sh);
  const float inv = rsqrtf(tot / (float)H + eps);
  __nv_bfloat16* yr = y + (size_t)t * H;
  for (int i = threadIdx.x * 8; i < H; i += NT * 8) {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + i);
    const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float w0 = bf16_lo(ws[j]), w1 = bf16_hi(ws[j]);
      if (add_one) { w0 += 1.f; w1 += 1.f; }
      o[j] = pack_bf16x2(row[i + 2 * j] * inv * w0, row[i + 2 * j + 1] * inv * w1);
    }
    *reinterpret_cast<uint4*>(yr + i) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(done, 1) == (int)gridDim.x - 1) {
    *done = 0;
    *ep_c = e;
  }
}

// ---------------------------------------------------------------------------
// RoPE + optional per-head RMSNorm on q/k + paged KV-cache write.
// q [T, Hq, D] (row stride q_stride), k [T, Hk, D], v [T, Hk, Dv] (strides given)
// cos_sin [max_pos, rot] fp32: first rot/2 = cos, next rot/2 = sin.
// Cache layout: [num_blocks, Hk, block_size, D] bf16; slot = block*block_size + offset.
// kv_fp8: e4m3 caches (saturating), K [num_blocks, Hk, block_size, D] times k_inv and V
// stored transposed per block, [num_blocks, Hk, Dv, block_size], times v_inv.
// One warp per (token, head); heads [0,Hq) are q, [Hq, Hq+Hk) are k (+v copy).
// ---------------------------------------------------------------------------
__global__ void rope_kv_kernel(__nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                               const __nv_bfloat16* __restrict__ v, const int* __restrict__ positions,
                               const float* __restrict__ cos_sin, int T, int Hq, int Hk, int D, int Dv, int rot,
                               int neox, int q_stride, int k_stride, int v_stride,
                               const __nv_bfloat16* __restrict__ q_norm_w, const __nv_bfloat16* __restrict__ k_norm_w,
                               float norm_eps, int norm_add_one, const int* __restrict__ slot_mapping,
                               void* __restrict__ k_cache, void* __restrict__ v_cache,
                               int block_size, long long num_slots, XtuStatus* st, int kv_fp8, float k_inv,
                               float v_inv) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int H = Hq + Hk;
  if (gw >= T * H) return;
  const int t = gw / H;
  const int h = gw - t * H;
  const bool is_q = h < Hq;
  __nv_bfloat16* ptr = is_q ? q + (size_t)t * q_stride + (size_t)h * D : k + (size_t)t * k_stride + (size_t)(h - Hq) * D;
  const __nv_bfloat16* nw = is_q ? q_norm_w : k_norm_w;
  // load the head (D <= 512): each lane holds D/32 values
  float vals[16];
  const int per = D / 32;
  for (int j = 0; j < per; ++j) vals[j] = __bfloat162float(ptr[lane + 32 * j]);
  if (nw) {
    float ss = 0.f;
    for (int j = 0; j < per; ++j) ss += vals[j] * vals[j];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)D + norm_eps);
    for (int j = 0; j < per; ++j) {
      float wv = __bfloat162float(nw[lane + 32 * j]);
      if (norm_add_one) wv += 1.f;
      // round like an unfused bf16 norm output
      vals[j] = __bfloat162float(__float2bfloat16(vals[j] * inv * wv));
    }
  }
  // write back normalised values, then rotate in place through global memory
  for (int j = 0; j < per; ++j) ptr[lane + 32 * j] = __float2bfloat16(vals[j]);
  __syncwarp();
  const int pos = positions[t];
  const float* cs = cos_sin + (size_t)pos * rot;
  const int half = rot / 2;
  // each lane rotates pairs i in [lane, half) step 32
  for (int i = lane; i < half; i += 32) {
    int i0, i1;
    if (neox) { i0 = i; i1 = i + half; } else { i0 = 2 * i; i1 = 2 * i + 1; }
    const float x0 = __bfloat162float(ptr[i0]);
    const float x1 = __bfloat162float(ptr[i1]);
    const float c = cs[i], s = cs[half + i];
    ptr[i0] = __float2bfloat16(x0 * c - x1 * s);
    ptr[i1] = __float2bfloat16(x1 * c + x0 * s);
  }
  __syncwarp();
  if (!is_q && k_cache) {
    const int slot = slot_mapping[t];
    // slots past the cache are skipped always, and reported by the bounds-check build
    if (slot >= 0 && XTU_IN_BOUNDS(slot < num_slots, st, 220, slot) && slot < num_slots) {
      const int hk = h - Hq;
      const int blk = slot / block_size, off = slot - blk * block_size;
      const __nv_bfloat16* vr = v + (size_t)t * v_stride + (size_t)hk * Dv;
      if (kv_fp8) {
        uint8_t* kc = static_cast<uint8_t*>(k_cache) + (((size_t)blk * Hk + hk) * block_size + off) * D;
        for (int j = lane; j < D; j += 32)
          kc[j] = __nv_cvt_float_to_fp8(__bfloat162float(ptr[j]) * k_inv, __NV_SATFINITE, __NV_E4M3);
        uint8_t* vc = static_cast<uint8_t*>(v_cache) + ((size_t)blk * Hk + hk) * Dv * block_size + off;
        for (int j = lane; j < Dv; j += 32)
          vc[(size_t)j * block_size] = __nv_cvt_float_to_fp8(__bfloat162float(vr[j]) * v_inv, __NV_SATFINITE, __NV_E4M3);
      } else {
        __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(k_cache) + (((size_t)blk * Hk + hk) * block_size + off) * D;
        for (int j = lane; j < D; j += 32) kc[j] = ptr[j];
        __nv_bfloat16* vc = static_cast<__nv_bfloat16*>(v_cache) + (((size_t)blk * Hk + hk) * block_size + off) * Dv;
        for (int j = lane; j < Dv; j += 32) vc[j] = vr[j];
      }
    }
  }
}

// plain paged KV write (no rope), e.g. for layers without positional rotation
__global__ void kv_write_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v, int T,
                                int Hk, int D, int Dv, int k_stride, int v_stride, const int* __restrict__ slot_mapping,
                                __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                                int block_size, long long num_slots, XtuStatus* st) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= T * Hk) return;
  const int t = gw / Hk, h = gw - t * Hk;
  const int slot = slot_mapping[t];
  if (slot < 0) return;
  if (!XTU_IN_BOUNDS(slot < num_slots, st, 221, slot) || slot >= num_slots) return;
  const int blk = slot / block_size, off = slot - blk * block_size;
  __nv_bfloat16* kc = k_cache + (((size_t)blk * Hk + h) * block_size + off) * D;
  __nv_bfloat16* vc = v_cache + (((size_t)blk * Hk + h) * block_size + off) * Dv;
  for (int j = lane; j < D; j += 32) kc[j] = k[(size_t)t * k_stride + (size_t)h * D + j];
  for (int j = lane; j < Dv; j += 32) vc[j] = v[(size_t)t * v_stride + (size_t)h * Dv + j];
}

// ---------------------------------------------------------------------------
// router top-k, one warp per token, E <= 1024 (32 scores per lane)
// scoring: 0 softmax, 1 sigmoid, 2 sqrt(softplus)
// selection uses score + bias; weights use the unbiased score.
// n_group > 1: group score = sum of the top-2 biased scores of the group;
// keep the best topk_group groups (DeepSeek-V3 "noaux_tc").
// ---------------------------------------------------------------------------
// One warp: token gw's scores -> its K expert ids / weights (out_ids / out_w rows gw).
// gscore: 64 floats of shared memory private to the warp (group scores).
template <int PER>
__device__ __forceinline__ void router_topk_warp(const float* __restrict__ lg, const float* __restrict__ bias,
                                                 int gw, int E, int K, int scoring, int n_group, int topk_group,
                                                 int renorm, float scale, int* __restrict__ out_ids,
                                                 float* __restrict__ out_w, float* gscore) {
  const int lane = threadIdx.x & 31;
  float sc[PER], sel[PER];   // PER = compile-time scores per lane, so these stay in registers
  float mx = -FLT_MAX;
  #pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    sc[j] = e < E ? lg[e] : -FLT_MAX;
    mx = fmaxf(mx, sc[j]);
  }
  if (scoring == 0) {
    mx = warp_max(mx);
    float s = 0.f;
    #pragma unroll
  for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      sc[j] = e < E ? __expf(sc[j] - mx) : 0.f;
      s += sc[j];
    }
    s = warp_sum(s);
    const float inv = 1.f / s;
    #pragma unroll
  for (int j = 0; j < PER; ++j) sc[j] *= inv;
  } else if (scoring == 1) {
    #pragma unroll
  for (int j = 0; j < PER; ++j) sc[j] = 1.f / (1.f + __expf(-sc[j]));
  } else {
    #pragma unroll
  for (int j = 0; j < PER; ++j) {
      const float x = sc[j];
      const float sp = x > 20.f ? x : log1pf(__expf(x));
      sc[j] = sqrtf(sp);
    }
  }
  // selection keys: experts past E and experts already taken are -inf; experts of groups
  // that were not kept are -FLT_MAX (below every real score, above the taken ones), so that
  // a K larger than the kept groups' experts still yields K distinct experts (index order)
  #pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    sel[j] = e < E ? sc[j] + (bias ? bias[e] : 0.f) : -INFINITY;
  }
  if (n_group > 1 && topk_group < n_group) {
    // group g covers experts [g*gs, (g+1)*gs); experts of lane l, slot j: e = l + 32 j
    const int gs = E / n_group;
    for (int g = 0; g < n_group; ++g) {
      // top-2 within group g
      float b1 = -FLT_MAX, b2 = -FLT_MAX;
      #pragma unroll
  for (int j = 0; j < PER; ++j) {
        const int e = lane + 32 * j;
        if (e < E && e / gs == g) {
          const float v = sel[j];
          if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) b2 = v;
        }
      }
      // warp reduce top-2
      for (int o = 16; o > 0; o >>= 1) {
        const float o1 = __shfl_xor_sync(0xffffffffu, b1, o);
        const float o2 = __shfl_xor_sync(0xffffffffu, b2, o);
        float n1 = fmaxf(b1, o1);
        float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
        b1 = n1; b2 = n2;
      }
      if (lane == 0) gscore[g] = b1 + b2;
    }
    __syncwarp();
    // pick topk_group groups
    unsigned long long keep = 0ull;
    for (int r = 0; r < topk_group; ++r) {
      int best = -1; float bv = -FLT_MAX;
      for (int g = 0; g < n_group; ++g)
        if (!((keep >> g) & 1ull) && gscore[g] > bv) { bv = gscore[g]; best = g; }
      if (best >= 0) keep |= 1ull << best;
    }
    #pragma unroll
  for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((keep >> (e / gs)) & 1ull)) sel[j] = -FLT_MAX;
    }
  }
  float wsum = 0.f;
  float myw = 0.f;
  int myid = -1;
  for (int r = 0; r < K; ++r) {
    float bv = -FLT_MAX; int bi = 0x7fffffff;
    #pragma unroll
  for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (sel[j] > bv || (sel[j] == bv && e < bi)) { bv = sel[j]; bi = e; }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    // owner lane knocks the winner out and reports its unbiased score
    float w = 0.f;
    if ((bi & 31) == lane) {
      const int j = bi >> 5;
      for (int jj = 0; jj < PER; ++jj) if (jj == j) { w = sc[jj]; sel[jj] = -INFINITY; }
    }
    w = __shfl_sync(0xffffffffu, w, bi & 31);
    wsum += w;
    if (lane == r) { myw = w; myid = bi; }
  }
  if (lane < K) {
    float w = myw;
    if (renorm) w = w / (wsum > 0.f ? wsum : 1.f);
    out_ids[(size_t)gw * K + lane] = myid;
    out_w[(size_t)gw * K + lane] = w * scale;
  }
}

template <int PER>
__global__ void router_topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int T, int E,
                                   int K, int scoring, int n_group, int topk_group, int renorm, float scale,
                                   int* __restrict__ out_ids, float* __restrict__ out_w, int logits_stride) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  __shared__ float gscore_sh[8][64];
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= T) return;
  router_topk_warp<PER>(logits + (size_t)gw * logits_stride, bias, gw, E, K, scoring, n_group, topk_group, renorm,
                        scale, out_ids, out_w, gscore_sh[(threadIdx.x >> 5) & 7]);
}

// ---------------------------------------------------------------------------
// MoE permute.  Pairs p = t*K + k with id in [lo, hi) are local; id - lo is the
// local expert.  Everything else (other EP ranks, CPU tier, masked) is skipped.
// ---------------------------------------------------------------------------
__global__ void moe_count_kernel(const int* __restrict__ ids, int n, int lo, int hi, int* __restrict__ counts) {
  extern __shared__ int hist[];
  const int E = hi - lo;
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int id = ids[i];
    if (id >= lo && id < hi) atomicAdd(&hist[id - lo], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (hist[e]) atomicAdd(&counts[e], hist[e]);
}

// single block: seg[0..E] = exclusive scan of counts; cursor = seg; counts zeroed for reuse
__global__ void moe_scan_kernel(int* __restrict__ counts, int E, int* __restrict__ seg, int* __restrict__ cursor) {
  __shared__ int sh[1024];
  const int tid = threadIdx.x;
  const int per = (E + blockDim.x - 1) / blockDim.x;
  int local = 0;
  for (int j = 0; j < per; ++j) {
    const int e = tid * per + j;
    if (e < E) local += counts[e];
  }
  sh[tid] = local;
  __syncthreads();
  for (int off = 1; off < blockDim.x; off <<= 1) {
    const int v = tid >= off ? sh[tid - off] : 0;
    __syncthreads();
    sh[tid] += v;
    __syncthreads();
  }
  int run = sh[tid] - local;
  for (int j = 0; j < per; ++j) {
    const int e = tid * per + j;
    if (e < E) {
      seg[e] = run;
      cursor[e] = run;
      run += counts[e];
      counts[e] = 0;
    }
  }
  if (tid == blockDim.x - 1) seg[E] = sh[tid];
}

// one warp per pair: claim a row, record its source token / slot / weight, copy the row
__global__ void moe_scatter_gather_kernel(const int* __restrict__ ids, const float* __restrict__ weights, int n,
                                          int K, int lo, int hi, int* __restrict__ cursor,
                                          int* __restrict__ perm_slot, float* __restrict__ perm_w,
                                          const __nv_bfloat16* __restrict__ x, int H, int x_stride,
                                          __nv_bfloat16* __restrict__ xp, int xp_f16s) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= n) return;
  const int id = ids[gw];
  if (id < lo || id >= hi) return;
  int p = 0;
  if (lane == 0) p = atomicAdd(&cursor[id - lo], 1);
  p = __shfl_sync(0xffffffffu, p, 0);
  if (lane == 0) {
    perm_slot[p] = gw;
    perm_w[p] = weights ? weights[gw] : 1.f;
  }
  if (xp) {
    const int t = gw / K;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * x_stride);
    uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)p * H);
    if (xp_f16s)   // the fp8-weight decode GEMV reads f16 x 2^-8 activations
      for (int i = lane; i < H / 8; i += 32) dst[i] = bf16x8_f16x8_s8(src[i]);
    else
      for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
  }
}

// Row gather after the decode permute, for steps of more tokens than the token-direct
// GEMV takes (speculative verification): warp w < n copies the token of permuted row w
// (perm_slot[w] / K) into xp row w if w < seg_end[0] (the local pairs); warps n .. n + sh_rows
// copy token w - n into xp row w (the rows a shared expert fused into the grouped GEMV reads).
// xp_f16s: f16 x 2^-8 rows (the fp8-weight GEMV's input form) instead of bf16.
__global__ void moe_gather_rows_kernel(const __nv_bfloat16* __restrict__ x, int x_stride, int K, int H,
                                       const int* __restrict__ perm_slot, const int* __restrict__ seg_end, int n,
                                       int sh_rows, __nv_bfloat16* __restrict__ xp, int xp_f16s) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= n + sh_rows) return;
  int t;
  if (w < n) {
    if (w >= __ldg(seg_end)) return;
    t = __ldg(perm_slot + w) / K;
  } else {
    t = w - n;
  }
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * x_stride);
  uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)w * H);
  if (xp_f16s)
    for (int i = lane; i < H / 8; i += 32) dst[i] = bf16x8_f16x8_s8(src[i]);
  else
    for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
}

// Decode-size permute (one CTA, E <= 1024 local experts): per-expert counts, seg, the
// (row -> pair) permutation, the list of experts that have rows, and for the token-direct
// gate/up GEMV the map tokrow[a * 16 + t] = row of token t's pair with active expert a
// (-1 if none; t < 16).  Rows within an expert follow arrival order (atomics); each row's
// result is computed independently, so the order does not change any value.
// the body, for a block of exactly 512 threads (also the tail of the fused decode router)
__device__ __forceinline__ void permute_decode_block(const int* __restrict__ ids, const float* __restrict__ weights,
                                                     int n, int K, int lo, int hi, int* __restrict__ seg,
                                                     int* __restrict__ perm_slot, float* __restrict__ perm_w,
                                                     int* __restrict__ active, int* __restrict__ tokrow) {
  __shared__ int cnt[1024], cur[1024], apos[1024];
  __shared__ int wc[16], wa[16], nact;
  const int E = hi - lo, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < 1024; e += 512) cnt[e] = 0;
  __syncthreads();
  for (int p = tid; p < n; p += 512) {
    const int id = ids[p];
    if (id >= lo && id < hi) atomicAdd(&cnt[id - lo], 1);
  }
  __syncthreads();
  // exclusive scans of the counts and of the "has rows" flags; thread tid owns entries 2tid, 2tid+1
  const int e0 = 2 * tid;
  const int c0 = cnt[e0], c1 = cnt[e0 + 1];
  const int a0 = c0 > 0, a1 = c1 > 0;
  int sc = c0 + c1, sa = a0 + a1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, sc, o), va = __shfl_up_sync(0xffffffffu, sa, o);
    if (lane >= o) {
      sc += v;
      sa += va;
    }
  }
  if (lane == 31) {
    wc[warp] = sc;
    wa[warp] = sa;
  }
  __syncthreads();
  if (warp == 0) {
    int v = lane < 16 ? wc[lane] : 0, va = lane < 16 ? wa[lane] : 0;
    const int v0 = v, va0 = va;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, v, o), ta = __shfl_up_sync(0xffffffffu, va, o);
      if (lane >= o) {
        v += t;
        va += ta;
      }
    }
    if (lane < 16) {
      wc[lane] = v - v0;
      wa[lane] = va - va0;
    }
    if (lane == 15) nact = va;
  }
  __syncthreads();
  const int exc = sc - (c0 + c1) + wc[warp], exa = sa - (a0 + a1) + wa[warp];
  if (e0 < E) {
    seg[e0] = exc;
    cur[e0] = exc;
    apos[e0] = exa;
    if (a0) active[1 + exa] = e0;
  }
  if (e0 + 1 < E) {
    seg[e0 + 1] = exc + c0;
    cur[e0 + 1] = exc + c0;
    apos[e0 + 1] = exa + a0;
    if (a1) active[1 + exa + a0] = e0 + 1;
  }
  if (tid == 511) seg[E] = exc + c0 + c1;
  if (tid == 0) active[0] = nact;
  if (tokrow)
    for (int i = tid; i < nact * 16; i += 512) tokrow[i] = -1;
  __syncthreads();
  for (int p = tid; p < n; p += 512) {
    const int id = ids[p];
    if (id < lo || id >= hi) continue;
    const int row = atomicAdd(&cur[id - lo], 1);
    perm_slot[row] = p;
    perm_w[row] = weights ? weights[p] : 1.f;
    if (tokrow) tokrow[apos[id - lo] * 16 + p / K] = row;
  }
}

__global__ void __launch_bounds__(512) moe_permute_decode_kernel(const int* __restrict__ ids,
                                                                 const float* __restrict__ weights, int n, int K,
                                                                 int lo, int hi, int* __restrict__ seg,
                                                                 int* __restrict__ perm_slot,
                                                                 float* __restrict__ perm_w, int* __restrict__ active,
                                                                 int* __restrict__ tokrow) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  permute_decode_block(ids, weights, n, K, lo, hi, seg, perm_slot, perm_w, active, tokrow);
}

// Decode router in one launch (T <= TT tokens, TT = 16 or 32; E <= 1024 experts): CTA e
// computes the fp32 logits of expert e for all tokens (bf16 gate weights [E, H]), the CTA
// that finishes last (counter, re-zeroed) then runs the top-k of every token and the
// decode permute.
template <int PER, int TT>
__global__ void __launch_bounds__(512) moe_route_decode_kernel(
    const __nv_bfloat16* __restrict__ x, int x_stride, int T, const __nv_bfloat16* __restrict__ gate, int E, int H,
    const float* __restrict__ bias, int K, int scoring, int n_group, int topk_group, int renorm, float scale,
    float* __restrict__ logits, int* __restrict__ counter, int* __restrict__ out_ids, float* __restrict__ out_w,
    int lo, int hi, int* __restrict__ seg, int* __restrict__ perm_slot, float* __restrict__ perm_w,
    int* __restrict__ active, int* __restrict__ tokrow) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // one expert row per CTA, its 16 warps each a sixteenth of H, so that E CTAs share the
  // multiply-adds (four experts per CTA left 32 SMs issuing every token's products for a
  // quarter of H: 20 us of a 40 us call at 20 tokens)
  __shared__ float part[16][TT];
  const int gw = blockIdx.x;
  float acc[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) acc[t] = 0.f;
  {
    const int kq = ((H / 8 + 15) / 16) * 8;          // this warp's [k0, k1)
    const int k0 = warp * kq, k1 = min(H, k0 + kq);
    const __nv_bfloat16* g = gate + (size_t)gw * H;
#pragma unroll 2
    for (int k = k0 + lane * 8; k < k1; k += 256) {
      const uint4 gv = *reinterpret_cast<const uint4*>(g + k);
      const uint32_t gs[4] = {gv.x, gv.y, gv.z, gv.w};
      // every token's load is issued unconditionally (rows past T re-read row T - 1 and are
      // never stored), so the loads of one k step are independent and overlap: a break at
      // T made each wait for the previous token's multiply-add (one L2 latency per token)
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        const int tr = t < T ? t : T - 1;
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)tr * x_stride + k));
        const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[t] += bf16_lo(gs[j]) * bf16_lo(xs[j]) + bf16_hi(gs[j]) * bf16_hi(xs[j]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    const float v = warp_sum(acc[t]);
    if (lane == 0) part[warp][t] = v;
  }
  __syncthreads();
  if (threadIdx.x < TT && threadIdx.x < T) {   // token t of this expert: the 16 slices in order
    const int t = threadIdx.x;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < 16; ++w) v += part[w][t];
    logits[(size_t)t * E + gw] = v;
  }
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(counter, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  __shared__ float gscore_sh[16][64];
  for (int t = warp; t < T; t += 16)
    router_topk_warp<PER>(logits + (size_t)t * E, bias, t, E, K, scoring, n_group, topk_group, renorm, scale,
                          out_ids, out_w, gscore_sh[warp]);
  __syncthreads();
  permute_decode_block(out_ids, out_w, T * K, K, lo, hi, seg, perm_slot, perm_w, active, tokrow);
  if (threadIdx.x == 0) *counter = 0;
}

// out[t] = sum_k slot[t*K+k] (local pairs only) + shared[t] + extra[t]
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ slots, const int* __restrict__ ids, int T,
                                   int K, int H, int lo, int hi, const __nv_bfloat16* __restrict__ shared,
                                   const float* __restrict__ extra, __nv_bfloat16* __restrict__ out,
                                   float* __restrict__ out_f32) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  const int t = blockIdx.x;
  // grid.y splits the hidden dimension so that decode-sized T still fills the GPU
  const int span = (H / 8 + gridDim.y - 1) / gridDim.y * 8;
  const int h0 = blockIdx.y * span, h1 = min(H, h0 + span);
  // which of the token's pairs are local, read once per block (K <= 64), so the slot
  // loads below do not each wait on an id load
  __shared__ unsigned long long local_mask;
  if (threadIdx.x < 32) {
    unsigned long long m = 0ull;
    for (int k = threadIdx.x; k < K && k < 64; k += 32) {
      const int id = ids[(size_t)t * K + k];
      if (id >= lo && id < hi) m |= 1ull << k;
    }
    for (int o = 16; o > 0; o >>= 1) m |= __shfl_xor_sync(0xffffffffu, m, o);
    if (threadIdx.x == 0) local_mask = m;
  }
  __syncthreads();
  const unsigned long long lm = local_mask;
  for (int i = h0 + threadIdx.x * 8; i < h1; i += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 8
    for (int k = 0; k < K; ++k) {
      if (!((lm >> k) & 1ull)) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(slots + ((size_t)t * K + k) * H + i);
      const uint32_t vs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) { acc[2 * j] += bf16_lo(vs[j]); acc[2 * j + 1] += bf16_hi(vs[j]); }
    }
    if (shared) {
      const uint4 v = *reinterpret_cast<const uint4*>(shared + (size_t)t * H + i);
      const uint32_t vs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) { acc[2 * j] += bf16_lo(vs[j]); acc[2 * j + 1] += bf16_hi(vs[j]); }
    }
    if (extra) {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += extra[(size_t)t * H + i + j];
    }
    if (out_f32) {
#pragma unroll
      for (int j = 0; j < 8; ++j) out_f32[(size_t)t * H + i + j] = acc[j];
    } else {
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]); o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]); o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(out + (size_t)t * H + i) = o;
    }
  }
}

// ---------------------------------------------------------------------------
// Tier split of routed pairs (W7; replaces the reference's PIN mask kernel,
// vllm_xiaotu_moe/pin_mask_triton.py:52-72).  slotmap[e - lo] >= 0: expert e is in the
// GPU pool at that slot; -1: it is served by the CPU tier.  Writes the pool-slot id (or
// -1) and the CPU expert id (or -1) of every pair, and counts routed hits per expert for
// the swap policy (device side, graph-capturable).
// ---------------------------------------------------------------------------
__global__ void route_split_kernel(const int* __restrict__ ids, int n, int lo, int E, const int* __restrict__ slotmap,
                                   int* __restrict__ gpu_ids, int* __restrict__ cpu_ids, int* __restrict__ hits) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int id = ids[i];
    const int e = id - lo;
    int g = -1, c = -1;
    if (e >= 0 && e < E) {
      const int slot = slotmap[e];
      if (slot >= 0) g = slot; else c = id;
      if (hits) atomicAdd(&hits[e], 1);
    }
    gpu_ids[i] = g;
    cpu_ids[i] = c;
  }
}

// ---------------------------------------------------------------------------
// greedy argmax over rows (fp32 or bf16 logits); ties -> lowest index; NaN entries never win, and a
// row with nothing above -FLT_MAX (all -inf / NaN) returns index 0
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float ld_f(const T* p, size_t i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, size_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) { return __bfloat162float(p[i]); }

// grid (parts, rows): block (p, r) reduces its slice of row r to (value, index) in part_v/part_i
// (or straight to out when parts == 1); argmax_final_kernel folds the parts.
template <typename T>
__global__ void argmax_kernel(const T* __restrict__ logits, int V, int stride, int* __restrict__ out,
                              float* __restrict__ out_val, float* __restrict__ part_v, int* __restrict__ part_i) {
  const T* row = logits + (size_t)blockIdx.y * stride;
  const int parts = gridDim.x;
  const int per = (V + parts - 1) / parts;
  const int lo = blockIdx.x * per, hi = min(V, lo + per);
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = ld_f<T>(row, i);
    if (v > bv) { bv = v; bi = i; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    bv = l < nw ? sv[l] : -FLT_MAX;
    bi = l < nw ? si[l] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (l == 0) {
      // no element beat -FLT_MAX (the slice is all -inf or NaN): its first index stands in,
      // so a row always yields a valid token id (NaN entries never win)
      if (bi == 0x7fffffff && lo < hi) bi = lo;
      if (parts == 1) {
        out[blockIdx.y] = bi;
        if (out_val) out_val[blockIdx.y] = bv;
      } else {
        part_v[blockIdx.y * parts + blockIdx.x] = bv;
        part_i[blockIdx.y * parts + blockIdx.x] = bi;
      }
    }
  }
}

__global__ void argmax_final_kernel(const float* __restrict__ part_v, const int* __restrict__ part_i, int parts,
                                    int* __restrict__ out, float* __restrict__ out_val) {
  const int r = blockIdx.x, l = threadIdx.x;
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = l; i < parts; i += 32) {
    const float v = part_v[r * parts + i];
    const int id = part_i[r * parts + i];
    if (v > bv || (v == bv && id < bi)) { bv = v; bi = id; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if (l == 0) {
    out[r] = bi;
    if (out_val) out_val[r] = bv;
  }
}

__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table, int T, int H,
                             int vocab, __nv_bfloat16* __restrict__ out, XtuStatus* st) {
  const int t = blockIdx.x;
  int id = ids[t];
  if (threadIdx.x == 0) (void)XTU_IN_BOUNDS(id >= 0 && id < vocab, st, 222, id);
  if (id < 0 || id >= vocab) id = 0;
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// SiLU(gate) * up for [T, 2I] rows (gate first), optional clamp; bf16 out [T, I]
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ x, int T, int I, float limit, float alpha,
                                float beta, __nv_bfloat16* __restrict__ out) {
  const size_t n = (size_t)T * I;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / I, j = i - t * I;
    float g = __bfloat162float(x[t * 2 * I + j]);
    float u = __bfloat162float(x[t * 2 * I + I + j]);
    if (limit > 0.f) { g = fminf(g, limit); u = fminf(fmaxf(u, -limit), limit); }
    out[i] = __float2bfloat16((g / (1.f + __expf(-alpha * g))) * (u + beta));
  }
}

}  // namespace xtu

using namespace xtu;

// returns `launched` (kernels enqueued) on success, a negative CUDA error otherwise
static inline int rc_last(int launched = 1) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? launched : -(int)e;
}

// ---------------------------------------------------------------------------
// sigmoid gates
//   gate_mul:    y[t, h, d] *= sigmoid(g[t, h, d])   (gated-GQA output gate; y and g strided)
//   shared_gate: y[t, :]    *= sigmoid(x[t, :] . w)  (Qwen3-Next shared-expert gate, w [H])
// ---------------------------------------------------------------------------
__global__ void gate_mul_kernel(__nv_bfloat16* __restrict__ y, int y_tok, int y_head,
                                const __nv_bfloat16* __restrict__ g, int g_tok, int g_head, int nh, int D) {
  const int t = blockIdx.x / nh, h = blockIdx.x - (blockIdx.x / nh) * nh;
  __nv_bfloat16* yr = y + (size_t)t * y_tok + (size_t)h * y_head;
  const __nv_bfloat16* gr = g + (size_t)t * g_tok + (size_t)h * g_head;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float gv = __bfloat162float(gr[d]);
    yr[d] = __float2bfloat16(__bfloat162float(yr[d]) / (1.f + __expf(-gv)));
  }
}

// one warp per token
__global__ void shared_gate_kernel(__nv_bfloat16* __restrict__ y, int y_stride, const __nv_bfloat16* __restrict__ x,
                                   int x_stride, const __nv_bfloat16* __restrict__ w, int T, int H) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (t >= T) return;
  const __nv_bfloat16* xr = x + (size_t)t * x_stride;
  float acc = 0.f;
  for (int i = lane * 2; i < H; i += 64) {
    const __nv_bfloat162 xv = *reinterpret_cast<const __nv_bfloat162*>(xr + i);
    const __nv_bfloat162 wv = *reinterpret_cast<const __nv_bfloat162*>(w + i);
    acc = fmaf(__low2float(xv), __low2float(wv), acc);
    acc = fmaf(__high2float(xv), __high2float(wv), acc);
  }
  acc = warp_sum(acc);
  const float s = 1.f / (1.f + __expf(-acc));
  __nv_bfloat16* yr = y + (size_t)t * y_stride;
  for (int i = lane; i < H; i += 32) yr[i] = __float2bfloat16(__bfloat162float(yr[i]) * s);
}

extern "C" {

// y16 (nullable): also write y as f16 x 2^-8 rows [T, H] (the fp8-weight GEMVs' input form)
int xtu_rmsnorm(const void* x, const void* residual, void* residual_out, const void* w, void* y, int T, int H,
                float eps, int add_one, int x_stride, int y_stride, void* y16, cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 8 != 0) return -2;
  const size_t sm = (size_t)H * sizeof(float);
  if (sm > 48 * 1024) {
    cudaFuncSetAttribute(rmsnorm_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  }
  launch_pdl(rmsnorm_kernel<256>, dim3(T), dim3(256), sm, s, (const __nv_bfloat16*)x,
             (const __nv_bfloat16*)residual, (__nv_bfloat16*)residual_out, (const __nv_bfloat16*)w,
             (__nv_bfloat16*)y, H, eps, add_one, x_stride, y_stride, reinterpret_cast<uint4*>(y16));
  return rc_last();
}

// consumer of xtu_gemv_tp; recv: this rank's receive buffer (2 * world slots of `slot`
// elements); flags: this rank's flag array; ep_p / ep_c / done as xtu_gemv_tp's.
int xtu_tp_sum_rmsnorm(const void* recv, long long slot, int world, int T, int H, const int* flags, const int* ep_p,
                       int* ep_c, int* done, const void* residual, void* residual_out, const void* w, void* y,
                       float eps, int add_one, void* status, long long timeout_ns, cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 8 != 0 || world > 256 || (long long)T * H > slot) return -2;
  const size_t sm = (size_t)H * sizeof(float);
  if (sm > 48 * 1024) cudaFuncSetAttribute(tp_sum_rmsnorm_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)sm);
  launch_pdl(tp_sum_rmsnorm_kernel<256>, dim3(T), dim3(256), sm, s, (const __nv_bfloat16*)recv, slot, world, H, flags,
             ep_p, ep_c, done, (const __nv_bfloat16*)residual, (__nv_bfloat16*)residual_out,
             (const __nv_bfloat16*)w, (__nv_bfloat16*)y, eps, add_one, reinterpret_cast<XtuStatus*>(status),
             timeout_ns);
  return rc_last();
}

int xtu_rope_kv(void* q, void* k, const void* v, const int* positions, const float* cos_sin, int T, int Hq, int Hk,
                int D, int Dv, int rot, int neox, int q_stride, int k_stride, int v_stride, const void* q_norm_w,
                const void* k_norm_w, float norm_eps, int norm_add_one, const int* slot_mapping, void* k_cache,
                void* v_cache, int block_size, long long num_slots, void* status, int kv_fp8, float k_inv,
                float v_inv, cudaStream_t s) {
  if (T <= 0) return 0;
  if (D % 32 != 0 || D > 512 || rot > D) return -2;
  const int warps = T * (Hq + Hk);
  const int threads = 256;
  const int blocks = (warps * 32 + threads - 1) / threads;
  launch_pdl(rope_kv_kernel, dim3(blocks), dim3(threads), 0, s, (__nv_bfloat16*)q, (__nv_bfloat16*)k,
             (const __nv_bfloat16*)v, positions, cos_sin, T, Hq, Hk, D, Dv, rot, neox, q_stride, k_stride, v_stride,
             (const __nv_bfloat16*)q_norm_w, (const __nv_bfloat16*)k_norm_w, norm_eps, norm_add_one, slot_mapping,
             k_cache, v_cache, block_size, num_slots, reinterpret_cast<XtuStatus*>(status), kv_fp8, k_inv, v_inv);
  return rc_last();
}

int xtu_kv_write(const void* k, const void* v, int T, int Hk, int D, int Dv, int k_stride, int v_stride,
                 const int* slot_mapping, void* k_cache, void* v_cache, int block_size, long long num_slots,
                 void* status, cudaStream_t s) {
  if (T <= 0) return 0;
  const int warps = T * Hk;
  kv_write_kernel<<<(warps * 32 + 255) / 256, 256, 0, s>>>((const __nv_bfloat16*)k, (const __nv_bfloat16*)v, T, Hk, D,
                                                           Dv, k_stride, v_stride, slot_mapping,
                                                           (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache,
                                                           block_size, num_slots,
                                                           reinterpret_cast<XtuStatus*>(status));
  return rc_last();
}

int xtu_router_topk(const float* logits, const float* bias, int T, int E, int K, int scoring, int n_group,
                    int topk_group, int renorm, float scale, int* out_ids, float* out_w, int logits_stride,
                    cudaStream_t s) {
  if (T <= 0) return 0;
  if (E > 1024 || K > 32 || n_group > 64) return -2;
  const int per = (E + 31) / 32;
#define XTU_TOPK(P)                                                                                          \
  launch_pdl(router_topk_kernel<P>, dim3((T * 32 + 255) / 256), dim3(256), 0, s, logits, bias, T, E, K, scoring,  \
             n_group, topk_group, renorm, scale, out_ids, out_w, logits_stride)
  if (per <= 1) XTU_TOPK(1);
  else if (per <= 2) XTU_TOPK(2);
  else if (per <= 4) XTU_TOPK(4);
  else if (per <= 8) XTU_TOPK(8);
  else if (per <= 16) XTU_TOPK(16);
  else XTU_TOPK(32);
#undef XTU_TOPK
  return rc_last();
}

// counts must be zero on entry (the scan leaves it zeroed for the next call).
// xp_f16s: write the gathered rows as f16 x 2^-8 instead of bf16.
int xtu_moe_permute(const int* ids, const float* weights, int T, int K, int lo, int hi, int* counts, int* seg,
                    int* cursor, int* perm_slot, float* perm_w, const void* x, int H, int x_stride, void* xp,
                    int xp_f16s, cudaStream_t s) {
  const int n = T * K;
  const int E = hi - lo;
  if (E <= 0 || E > 65536) return -2;
  if (n > 0) {
    const int blocks = (n + 1023) / 1024 < 132 ? (n + 1023) / 1024 : 132;
    moe_count_kernel<<<blocks, 1024, E * sizeof(int), s>>>(ids, n, lo, hi, counts);
  }
  moe_scan_kernel<<<1, 1024, 0, s>>>(counts, E, seg, cursor);
  if (n > 0) {
    if (xp && H % 8 != 0) return -3;
    moe_scatter_gather_kernel<<<(n * 32 + 255) / 256, 256, 0, s>>>(ids, weights, n, K, lo, hi, cursor, perm_slot,
                                                                   perm_w, (const __nv_bfloat16*)x, H, x_stride,
                                                                   (__nv_bfloat16*)xp, xp_f16s);
  }
  return rc_last(n > 0 ? 3 : 1);
}

// decode permute without the activation gather (see moe_permute_decode_kernel): E <= 1024,
// tokrow (nullable) needs n / K <= 16 tokens and n_active * 16 ints.
int xtu_moe_permute_decode(const int* ids, const float* weights, int T, int K, int lo, int hi, int* seg,
                           int* perm_slot, float* perm_w, int* active, int* tokrow, cudaStream_t s) {
  const int E = hi - lo;
  if (E <= 0 || E > 1024 || (tokrow && T > 16)) return -2;
  launch_pdl(moe_permute_decode_kernel, dim3(1), dim3(512), 0, s, ids, weights, T * K, K, lo, hi, seg, perm_slot,
             perm_w, active, tokrow);
  return rc_last();
}

// rows of the decode permute gathered into xp (see moe_gather_rows_kernel): n permuted
// rows (seg_end: device int, the local pair count), then sh_rows token rows; x rows and H
// 16-byte aligned.
int xtu_moe_gather_rows(const void* x, int x_stride, int K, int H, const int* perm_slot, const int* seg_end, int n,
                        int sh_rows, void* xp, int xp_f16s, cudaStream_t s) {
  if (n + sh_rows <= 0) return 0;
  if (H % 8 != 0 || x_stride % 8 != 0 || K <= 0) return -2;
  const int warps = n + sh_rows;
  launch_pdl(moe_gather_rows_kernel, dim3((warps * 32 + 255) / 256), dim3(256), 0, s, (const __nv_bfloat16*)x,
             x_stride, K, H, perm_slot, seg_end, n, sh_rows, (__nv_bfloat16*)xp, xp_f16s);
  return rc_last();
}

// decode router + permute in one launch (see moe_route_decode_kernel).  x [T <= 32, H] bf16
// (rows 16-byte aligned), gate [E, H] bf16; logits: T * E fp32 scratch; counter: one zeroed
// int (left zeroed).  Outputs as xtu_router_topk + xtu_moe_permute_decode (tokrow, the
// token-direct map, only for T <= 16; null otherwise).
int xtu_moe_route_decode(const void* x, int x_stride, int T, const void* gate, int E, int H, const float* bias, int K,
                         int scoring, int n_group, int topk_group, int renorm, float scale, float* logits,
                         int* counter, int* out_ids, float* out_w, int lo, int hi, int* seg, int* perm_slot,
                         float* perm_w, int* active, int* tokrow, cudaStream_t s) {
  if (T <= 0) return 0;
  if (T > 32 || (tokrow && T > 16) || E > 1024 || K > 32 || n_group > 64 || H % 8 != 0 || hi - lo <= 0 ||
      hi - lo > 1024)
    return -2;
  const int per = (E + 31) / 32;
  const dim3 grid(E);
#define XTU_ROUTE_T(P, TTV)                                                                                  \
  launch_pdl(moe_route_decode_kernel<P, TTV>, grid, dim3(512), 0, s, (const __nv_bfloat16*)x, x_stride, T,   \
             (const __nv_bfloat16*)gate, E, H, bias, K, scoring, n_group, topk_group, renorm, scale, logits,   \
             counter, out_ids, out_w, lo, hi, seg, perm_slot, perm_w, active, tokrow)
#define XTU_ROUTE(P)                      \
  do {                                    \
    if (T <= 16) XTU_ROUTE_T(P, 16);      \
    else XTU_ROUTE_T(P, 32);              \
  } while (0)
  if (per <= 1) XTU_ROUTE(1);
  else if (per <= 2) XTU_ROUTE(2);
  else if (per <= 4) XTU_ROUTE(4);
  else if (per <= 8) XTU_ROUTE(8);
  else if (per <= 16) XTU_ROUTE(16);
  else XTU_ROUTE(32);
#undef XTU_ROUTE
#undef XTU_ROUTE_T
  return rc_last();
}

int xtu_moe_combine(const void* slots, const int* ids, int T, int K, int H, int lo, int hi, const void* shared,
                    const float* extra, void* out, float* out_f32, cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 8 != 0 || K > 64) return -2;
  const int threads = H / 8 < 128 ? ((H / 8 + 31) / 32) * 32 : 128;
  int ysplit = (H / 8 + threads - 1) / threads;          // one 8-wide vector per thread
  if (T * ysplit > 2048) ysplit = (2048 + T - 1) / T;
  if (ysplit < 1) ysplit = 1;
  launch_pdl(moe_combine_kernel, dim3(T, ysplit), dim3(threads), 0, s, (const __nv_bfloat16*)slots, ids, T, K, H, lo,
             hi, (const __nv_bfloat16*)shared, extra, (__nv_bfloat16*)out, out_f32);
  return rc_last();
}

// ws: scratch of >= T * 64 * 8 bytes when V is large (nullable: single block per row)
int xtu_argmax(const void* logits, int is_bf16, int T, int V, int stride, int* out, float* out_val, void* ws,
               cudaStream_t s) {
  if (T <= 0) return 0;
  int parts = ws ? (V + 8191) / 8192 : 1;
  if (parts > 64) parts = 64;
  float* pv = reinterpret_cast<float*>(ws);
  int* pi = ws ? reinterpret_cast<int*>(pv + (size_t)T * 64) : nullptr;
  const dim3 grid(parts, T);
  if (is_bf16)
    argmax_kernel<__nv_bfloat16><<<grid, 512, 0, s>>>((const __nv_bfloat16*)logits, V, stride, out, out_val, pv, pi);
  else
    argmax_kernel<float><<<grid, 512, 0, s>>>((const float*)logits, V, stride, out, out_val, pv, pi);
  if (parts > 1) argmax_final_kernel<<<T, 32, 0, s>>>(pv, pi, parts, out, out_val);
  return rc_last(parts > 1 ? 2 : 1);
}

int xtu_route_split(const int* ids, int n, int lo, int E, const int* slotmap, int* gpu_ids, int* cpu_ids, int* hits,
                    cudaStream_t s) {
  if (n <= 0) return 0;
  int blocks = (n + 255) / 256;
  if (blocks > 1024) blocks = 1024;
  route_split_kernel<<<blocks, 256, 0, s>>>(ids, n, lo, E, slotmap, gpu_ids, cpu_ids, hits);
  return rc_last();
}

int xtu_embed(const int* ids, const void* table, int T, int H, int vocab, void* out, void* status,
              cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 8 != 0) return -2;
  embed_kernel<<<T, 256, 0, s>>>(ids, (const __nv_bfloat16*)table, T, H, vocab, (__nv_bfloat16*)out,
                                 reinterpret_cast<XtuStatus*>(status));
  return rc_last();
}

// The same lookup from a table in pinned host memory: the device reads the rows over the
// host link through the table's mapped address (large tables kept off HBM, e.g. the
// reference's per-layer-embedding offload).  Returns -3 if the table is not pinned.
int xtu_embed_host(const int* ids, const void* host_table, int T, int H, int vocab, void* out, void* status,
                   cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 8 != 0) return -2;
  void* dtab = nullptr;
  if (cudaHostGetDevicePointer(&dtab, const_cast<void*>(host_table), 0) != cudaSuccess || dtab == nullptr) {
    cudaGetLastError();
    return -3;
  }
  embed_kernel<<<T, 256, 0, s>>>(ids, (const __nv_bfloat16*)dtab, T, H, vocab, (__nv_bfloat16*)out,
                                 reinterpret_cast<XtuStatus*>(status));
  return rc_last();
}

int xtu_gate_mul(void* y, int y_tok, int y_head, const void* g, int g_tok, int g_head, int T, int nh, int D,
                 cudaStream_t s) {
  if (T <= 0) return 0;
  gate_mul_kernel<<<T * nh, D >= 128 ? 128 : 64, 0, s>>>((__nv_bfloat16*)y, y_tok, y_head, (const __nv_bfloat16*)g,
                                                         g_tok, g_head, nh, D);
  return rc_last();
}

int xtu_shared_gate(void* y, int y_stride, const void* x, int x_stride, const void* w, int T, int H, cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 2 != 0) return -2;
  shared_gate_kernel<<<(T * 32 + 255) / 256, 256, 0, s>>>((__nv_bfloat16*)y, y_stride, (const __nv_bfloat16*)x,
                                                          x_stride, (const __nv_bfloat16*)w, T, H);
  return rc_last();
}

int xtu_silu_mul(const void* x, int T, int I, float limit, float alpha, float beta, void* out, cudaStream_t s) {
  if (T <= 0) return 0;
  const size_t n = (size_t)T * I;
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  silu_mul_kernel<<<blocks, 256, 0, s>>>((const __nv_bfloat16*)x, T, I, limit, alpha, beta, (__nv_bfloat16*)out);
  return rc_last();
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Argmax without allocation (declared in xtu_argmax_static.h).
//
// Who needs it: callers that must not allocate device memory while they run.  A
// serving process sizes its KV cache to take the HBM that is left after start-up,
// so a later cudaMalloc can fail for lack of memory, and cudaMalloc / cudaFree
// synchronise the device, which would stall the streams of a decode loop that
// is in flight.  Such callers (a C or C++ decode loop without PyTorch's caching
// allocator, for instance) cannot hand xtu_argmax its workspace.
//
// How: the per-row partial results live in one file-scope device array of fixed
// size.  The first call on a device, with that device current, looks up the
// array's address there with cudaGetSymbolAddress and keeps it; later calls on that
// device reuse it.  Make that first call before any stream capture begins.
// Nothing in the array needs to start at zero: every slot that the second kernel
// reads is written by the first kernel of the same call.  All calls on one device
// share the array, so two calls whose kernels can overlap (different streams, or
// different host threads without ordering between them) race on it and may return
// wrong indices: order such calls on one stream.
// ---------------------------------------------------------------------------
namespace {
constexpr int kArgmaxStaticParts = 64;  // same split limit as xtu_argmax
constexpr size_t kArgmaxStaticBytes = (size_t)XTU_ARGMAX_STATIC_MAX_ROWS * kArgmaxStaticParts *
                                      (sizeof(float) + sizeof(int));
constexpr int kArgmaxStaticMaxDevices = 64;
std::mutex g_argmax_static_mu;
void* g_argmax_static_ptr[kArgmaxStaticMaxDevices] = {};
}  // namespace

static __device__ __align__(256) unsigned char g_argmax_scratch[kArgmaxStaticBytes];

extern "C" int xtu_argmax_static(const void* logits, int is_bf16, int T, int V, int stride, int* out,
                                 float* out_val, cudaStream_t s) {
  if (T == 0) return 0;
  if (T < 0 || V < 1 || stride < V) return XTU_ARGMAX_STATIC_ERR_BAD_SIZE;
  if (T > XTU_ARGMAX_STATIC_MAX_ROWS) return XTU_ARGMAX_STATIC_ERR_TOO_MANY_ROWS;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return -(int)e;
  if (dev < 0 || dev >= kArgmaxStaticMaxDevices) return XTU_ARGMAX_STATIC_ERR_DEVICE;
  void* ws;
  {
    std::lock_guard<std::mutex> g(g_argmax_static_mu);
    ws = g_argmax_static_ptr[dev];
    if (!ws) {
      e = cudaGetSymbolAddress(&ws, g_argmax_scratch);
      if (e != cudaSuccess) return -(int)e;
      g_argmax_static_ptr[dev] = ws;
    }
  }
  int parts = (V + 8191) / 8192;
  if (parts > kArgmaxStaticParts) parts = kArgmaxStaticParts;
  float* pv = reinterpret_cast<float*>(ws);
  int* pi = reinterpret_cast<int*>(pv + (size_t)T * kArgmaxStaticParts);
  const dim3 grid(parts, T);
  if (is_bf16)
    argmax_kernel<__nv_bfloat16><<<grid, 512, 0, s>>>((const __nv_bfloat16*)logits, V, stride, out, out_val, pv, pi);
  else
    argmax_kernel<float><<<grid, 512, 0, s>>>((const float*)logits, V, stride, out, out_val, pv, pi);
  if (parts > 1) argmax_final_kernel<<<T, 32, 0, s>>>(pv, pi, parts, out, out_val);
  return rc_last(parts > 1 ? 2 : 1);
}

