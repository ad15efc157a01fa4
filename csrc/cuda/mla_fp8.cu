// fp8 (e4m3) MLA latent cache for sm_100a: half the bytes per cached token (576 instead
// of 1152 for DeepSeek-V3's 512 latent + 64 RoPE dims), so twice the context fits in HBM.
//
//   mla_latent_write_fp8     one step's latent rows (bf16, RMSNorm'd latent + RoPE'd key)
//                            -> e4m3 rows of the paged cache at their slots, x / scale
//                            rounded to nearest and saturated at +-448
//   mla_latent_dequant_gather the blocks of a step's sequences -> a bf16 scratch cache in
//                            sequence order (block j of sequence b at b * maxb + j), x scale,
//                            which the bf16 latent attention kernels then read
//
// The reference serves its MLA models with vLLM's fp8 latent KV layout (per-token scales);
// this cache keeps one scale per layer, the form the GQA fp8 cache of this library uses.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include "ptx.cuh"
#include "launch.cuh"

namespace xtu {

// grid (T), block D / 8: thread i converts 8 consecutive values of row t
__global__ void mla_latent_write_fp8_kernel(const __nv_bfloat16* __restrict__ x, int x_stride, int D,
                                            const int* __restrict__ slots, long long num_slots,
                                            uint8_t* __restrict__ cache, float inv_scale, XtuStatus* st) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  const int t = blockIdx.x, i = threadIdx.x;
  const int slot = slots[t];
  if (slot < 0 || 8 * i >= D) return;
  if (!XTU_IN_BOUNDS(slot < num_slots, st, 250, slot) || slot >= num_slots) return;
  const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)t * x_stride + 8 * i);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint16_t q[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = make_float2(bf16_lo(w[j]) * inv_scale, bf16_hi(w[j]) * inv_scale);
    q[j] = (uint16_t)__nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
  }
  uint2 o;
  o.x = (uint32_t)q[0] | ((uint32_t)q[1] << 16);
  o.y = (uint32_t)q[2] | ((uint32_t)q[3] << 16);
  *reinterpret_cast<uint2*>(cache + (size_t)slot * D + 8 * i) = o;
}

// grid (maxb, B), block 256: block j of sequence b (if the sequence has it) -> dst block
// b * maxb + j, bf16, times scale.  A block is 64 rows of D bytes.
__global__ void __launch_bounds__(256) mla_latent_dequant_gather_kernel(
    const uint8_t* __restrict__ src, int D, const int* __restrict__ block_table, int bt_stride,
    const int* __restrict__ kv_len, int maxb, int num_blocks, float scale, __nv_bfloat16* __restrict__ dst,
    XtuStatus* st) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  const int j = blockIdx.x, b = blockIdx.y;
  const int nb = (kv_len[b] + 63) / 64;
  if (j >= nb) return;
  const int blk = block_table[(size_t)b * bt_stride + j];
  if (!XTU_IN_BOUNDS(blk >= 0 && blk < num_blocks, st, 251, blk) || blk < 0 || blk >= num_blocks) return;
  const uint2* s = reinterpret_cast<const uint2*>(src + (size_t)blk * 64 * D);
  uint4* d = reinterpret_cast<uint4*>(dst + ((size_t)b * maxb + j) * 64 * D);
  const int n8 = 64 * D / 8;
  for (int i = threadIdx.x; i < n8; i += 256) {
    const uint2 v = s[i];
    const uint32_t w[2] = {v.x, v.y};
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[h] >> (16 * k)), __NV_E4M3);
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
        o[2 * h + k] = pack_bf16x2(f.x * scale, f.y * scale);
      }
    }
    d[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace xtu

using namespace xtu;

extern "C" {

// x [T, D] bf16 (row stride x_stride elements, rows 16-byte aligned), D % 8 == 0, D <= 8192;
// cache e4m3 [num_slots, D]; rows with slot < 0 are skipped.
int xtu_mla_latent_write_fp8(const void* x, int x_stride, int T, int D, const int* slots, long long num_slots,
                             void* cache, float inv_scale, void* status, cudaStream_t s) {
  if (T <= 0) return 0;
  if (D % 8 != 0 || D > 8192 || x_stride % 8 != 0) return -2;
  launch_pdl(mla_latent_write_fp8_kernel, dim3(T), dim3(D / 8), 0, s, (const __nv_bfloat16*)x, x_stride, D, slots,
             num_slots, (uint8_t*)cache, inv_scale, reinterpret_cast<XtuStatus*>(status));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// src e4m3 [num_blocks, 64, D]; block_table [B, bt_stride]; dst bf16 [B * maxb, 64, D].
int xtu_mla_latent_dequant_gather(const void* src, int D, const int* block_table, int bt_stride, const int* kv_len,
                                  int B, int maxb, int num_blocks, float scale, void* dst, void* status,
                                  cudaStream_t s) {
  if (B <= 0 || maxb <= 0) return 0;
  if (D % 8 != 0) return -2;
  launch_pdl(mla_latent_dequant_gather_kernel, dim3(maxb, B), dim3(256), 0, s, (const uint8_t*)src, D, block_table,
             bt_stride, kv_len, maxb, num_blocks, scale, (__nv_bfloat16*)dst, reinterpret_cast<XtuStatus*>(status));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

}  // extern "C"
