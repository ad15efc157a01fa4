// Small-M (decode) GEMV / grouped-GEMV kernels for sm_100a, weight-streaming bound.
//
//   y[m, n] = sum_k x[m, k] * W[n, k]     (m < M <= 16, W bf16 or e4m3 + 128x128 fp32 scales)
//
// At decode the GEMMs see 1..16 rows, so the job is to stream the weights at HBM
// bandwidth.  A SIMT dot product spends ~5-12 instructions per weight byte on
// conversions and FMAs and ends up issue-bound; here the multiply-adds go to the
// tensor cores through warp-level mma.sync m16n8k16 instead:
//   * A = 16 weight rows x 16 k, B = 16 k x 8 tokens, D = 16 rows x 8 tokens (fp32).
//   * The order of k inside each MMA is permuted (a dot product does not care) so that
//     lane t's A fragment comes from ONE contiguous 16-byte load of row (t/4) and one of
//     row (t/4 + 8): lane t owns physical k = 16*(t%4) + [0, 16) of a 64-k chunk (fp8)
//     and feeds MMA g in 0..3 with k = 16*(t%4) + 4g + {0,1 | 2,3}.  Its B fragment is
//     the same k slice of token t/4, so A and B agree on the permutation.
//   * fp8: e4m3 pairs -> f16 pairs with one cvt each (exact), activations -> f16 scaled
//     by 2^-8 (keeps x * 448 inside fp16 range; the scale and 2^8 are restored in fp32
//     with the block scale, once per 64-k chunk).  bf16 weights use the bf16 MMA with
//     no conversion at all.
//   * Each warp streams two 16-row tiles with the next chunk's loads issued before the
//     current chunk's MMAs.  Warps are persistent and stride over row slices.
// Grouped (MoE) forms take the routing permutation of moe_permute: expert e owns rows
// seg[e]..seg[e+1] of the permuted activations.
//   * gate/up: the two row tiles are 16 gate rows and the matching 16 up rows (W13 rows
//     interleaved in 256-row blocks), so SwiGLU is applied in registers and the
//     [T*K, 2I] intermediate never exists.
//   * down: rows scaled by the pair's routing weight and written to the pair's slot row.
// Replaces the reference's SIMT small-M MXFP4 kernel (xiaotu_moe/csrc/moe4_smallm.cu,
// sm_80 FP32 FMA, split-K atomics) and the FP8 pair-centric Triton decode kernels
// (vllm_xiaotu_moe/decode_moe_fp8.py:23-138).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "ptx.cuh"

namespace xtu {

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// two e4m3 (low 16 bits) -> f16x2 (exact)
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(v & 0xFFFFu), __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

// bf16 pair -> f16 pair scaled by 2^-8
__device__ __forceinline__ uint32_t bf16x2_f16x2_s8(uint32_t v) {
  const float lo = __uint_as_float(v << 16) * 0.00390625f;
  const float hi = __uint_as_float(v & 0xFFFF0000u) * 0.00390625f;
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t u4w(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

constexpr int GEMV_WARPS = 8;

// One warp: two 16-row weight tiles (base rows rb[0], rb[1]; row pitch K elements) times
// the activation rows x_row0 .. x_row0 + mcount (mcount <= 8*NT).
// Out: acc[tile][nt][4] = D fragments (row g4 / g4+8, tokens nt*8 + 2*tq + {0,1}).
template <bool FP8, int NT, bool PX = false>
__device__ __forceinline__ void warp_mma_gemv(const uint8_t* __restrict__ W, const float* __restrict__ wscale,
                                              int sk, int N, int K, const int (&rb)[2],
                                              const __nv_bfloat16* __restrict__ x, int x_row0, int x_stride,
                                              int mcount, int c_begin, int c_end, float (&acc)[2][NT][4]) {
  constexpr int CK = FP8 ? 64 : 32;          // k per chunk (a lane loads 16 bytes of each of its rows)
  constexpr int LK = FP8 ? 16 : 8;           // k per lane per chunk
  constexpr int EB = FP8 ? 1 : 2;
  const int lane = threadIdx.x & 31;
  const int g4 = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][n][i] = 0.f;
  // the two rows of each tile this lane loads (clamped for loads; writes are masked by the caller)
  size_t roff[2][2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    roff[t][0] = (size_t)min(rb[t] + g4, N - 1) * K;
    roff[t][1] = (size_t)min(rb[t] + g4 + 8, N - 1) * K;
  }
  if (c_begin >= c_end) return;
  // raw activations of token (nt*8 + g4) for the lane's k slice (LK bf16 = LK/8 uint4)
  auto load_x = [&](int k, uint4 (&xr)[NT][LK / 8]) {
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int tok = n * 8 + g4;
      const bool ok = tok < mcount && k < K;
      const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)(x_row0 + (ok ? tok : 0)) * x_stride + (ok ? k : 0));
#pragma unroll
      for (int q = 0; q < LK / 8; ++q) xr[n][q] = ok ? __ldg(xp + q) : make_uint4(0, 0, 0, 0);
    }
  };
  uint4 w[2][2], wn[2][2];
  uint4 xr[NT][LK / 8], xn[NT][LK / 8];
  {
    const int k = c_begin * CK + tq * LK;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        w[t][h] = k < K ? __ldg(reinterpret_cast<const uint4*>(W + (roff[t][h] + k) * EB)) : make_uint4(0, 0, 0, 0);
    load_x(k, xr);
  }
  for (int c = c_begin; c < c_end; ++c) {
    const int k = c * CK + tq * LK;
    if (c + 1 < c_end) {
      const int kn = k + CK;
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          wn[t][h] = kn < K ? __ldg(reinterpret_cast<const uint4*>(W + (roff[t][h] + kn) * EB))
                            : make_uint4(0, 0, 0, 0);
      if (PX) load_x(kn, xn);
    }
    if (!PX && c != c_begin) load_x(k, xr);
    uint32_t b[NT][LK / 2];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int q = 0; q < LK / 8; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i) b[n][4 * q + i] = FP8 ? bf16x2_f16x2_s8(u4w(xr[n][q], i)) : u4w(xr[n][q], i);
    float d[2][NT][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) d[t][n][i] = 0.f;
#pragma unroll
    for (int g = 0; g < LK / 4; ++g) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        uint32_t a0, a1, a2, a3;
        if (FP8) {
          const uint32_t wa = u4w(w[t][0], g), wb = u4w(w[t][1], g);
          a0 = e4m3x2_f16x2(wa);          // row g4,   k 4g, 4g+1
          a1 = e4m3x2_f16x2(wb);          // row g4+8
          a2 = e4m3x2_f16x2(wa >> 16);    // row g4,   k 4g+2, 4g+3
          a3 = e4m3x2_f16x2(wb >> 16);    // row g4+8
        } else {
          a0 = u4w(w[t][0], 2 * g);
          a1 = u4w(w[t][1], 2 * g);
          a2 = u4w(w[t][0], 2 * g + 1);
          a3 = u4w(w[t][1], 2 * g + 1);
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if (FP8) mma_f16_16816(d[t][n], a0, a1, a2, a3, b[n][2 * g], b[n][2 * g + 1]);
          else mma_bf16_16816(d[t][n], a0, a1, a2, a3, b[n][2 * g], b[n][2 * g + 1]);
        }
      }
    }
    // fp8: block scale of (tile rows, this chunk) and the 2^8 activation pre-scale
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      float sc = 1.f;
      if (FP8) sc = 256.f * __ldg(wscale + (size_t)(min(rb[t], N - 1) >> 7) * sk + ((c * CK) >> 7));
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[t][n][i] = fmaf(d[t][n][i], sc, acc[t][n][i]);
    }
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h) w[t][h] = wn[t][h];
    if (PX) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int q = 0; q < LK / 8; ++q) xr[n][q] = xn[n][q];
    }
  }
}

// The 8 warps of a CTA split the k chunks of one slice; this sums their D fragments
// through shared memory.  On return warp 0 holds the totals (other warps: undefined).
template <int NT>
__device__ __forceinline__ void cta_reduce(float (&acc)[2][NT][4], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int V = 2 * NT * 4;
  float* mine = red + ((size_t)warp * 32 + lane) * V;
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) mine[(t * NT + n) * 4 + i] = acc[t][n][i];
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < GEMV_WARPS; ++w) {
      const float* o = red + ((size_t)w * 32 + lane) * V;
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[t][n][i] += o[(t * NT + n) * 4 + i];
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void chunk_split(int nchunks, int& c0, int& c1) {
  const int warp = threadIdx.x >> 5;
  const int per = (nchunks + GEMV_WARPS - 1) / GEMV_WARPS;
  c0 = min(nchunks, warp * per);
  c1 = min(nchunks, c0 + per);
}

// ---------------------------------------------------------------------------
// dense: y[M, N] = x[M, K] W^T (+ bias); a CTA = one 32-row slice (two 16-row tiles),
// its warps split K
// ---------------------------------------------------------------------------
template <bool FP8, int NT>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_dense_kernel(
    const uint8_t* __restrict__ W, const float* __restrict__ wscale, int N, int K, const __nv_bfloat16* __restrict__ x,
    int x_stride, int M, const __nv_bfloat16* __restrict__ bias, void* __restrict__ y, int y_stride, int y_f32) {
  __shared__ float red[GEMV_WARPS * 32 * 2 * NT * 4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g4 = lane >> 2, tq = lane & 3;
  const int sk = (K + 127) >> 7;
  constexpr int CK = FP8 ? 64 : 32;
  int c0, c1;
  chunk_split((K + CK - 1) / CK, c0, c1);
  {
    const int sl = blockIdx.x;
    const int rb[2] = {sl * 32, sl * 32 + 16};
    float acc[2][NT][4];
    warp_mma_gemv<FP8, NT, true>(W, wscale, sk, N, K, rb, x, 0, x_stride, M, c0, c1, acc);
    cta_reduce<NT>(acc, red);
    if (warp != 0) return;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = rb[t] + g4 + (i >> 1) * 8;
          const int tok = n * 8 + 2 * tq + (i & 1);
          if (row < N && tok < M) {
            float v = acc[t][n][i];
            if (bias) v += __bfloat162float(bias[row]);
            if (y_f32) reinterpret_cast<float*>(y)[(size_t)tok * y_stride + row] = v;
            else reinterpret_cast<__nv_bfloat16*>(y)[(size_t)tok * y_stride + row] = __float2bfloat16(v);
          }
        }
  }
}

// ---------------------------------------------------------------------------
// grouped gate/up + SwiGLU: grid (ctas_per_expert, E).  W13 [E, 2I, K] in 256-row
// blocks (128 gate, 128 up); a warp slice = 16 output columns: 16 gate + 16 up rows.
// ---------------------------------------------------------------------------
template <bool FP8, int NT>
__global__ void __launch_bounds__(GEMV_WARPS * 32) moe_gemv_gate_up_kernel(
    const uint8_t* __restrict__ W, const float* __restrict__ wscale, int I, int K,
    const __nv_bfloat16* __restrict__ xp, const int* __restrict__ seg, __nv_bfloat16* __restrict__ h, float limit,
    float alpha, float beta) {
  const int e = blockIdx.y;
  const int s0 = seg[e], cnt = seg[e + 1] - s0;
  if (cnt <= 0) return;
  const size_t eoff = (size_t)e * 2 * I * K * (FP8 ? 1 : 2);
  const int sk = (K + 127) >> 7;
  const float* esc = FP8 ? wscale + (size_t)e * ((2 * I + 127) >> 7) * sk : nullptr;
  __shared__ float red[GEMV_WARPS * 32 * 2 * NT * 4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g4 = lane >> 2, tq = lane & 3;
  constexpr int CK = FP8 ? 64 : 32;
  int c0, c1;
  chunk_split((K + CK - 1) / CK, c0, c1);
  {
    const int sl = blockIdx.x;
    const int j0 = sl * 16;
    const int grow = (j0 >> 7) * 256 + (j0 & 127);
    const int rb[2] = {grow, grow + 128};
    for (int mb = 0; mb < cnt; mb += 8 * NT) {
      const int mc = min(8 * NT, cnt - mb);
      float acc[2][NT][4];
      warp_mma_gemv<FP8, NT>(W + eoff, esc, sk, 2 * I, K, rb, xp, s0 + mb, K, mc, c0, c1, acc);
      cta_reduce<NT>(acc, red);
      if (warp != 0) continue;
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = j0 + g4 + (i >> 1) * 8;
          const int tok = n * 8 + 2 * tq + (i & 1);
          if (tok < mc) {
            float g = acc[0][n][i], u = acc[1][n][i];
            if (limit > 0.f) { g = fminf(g, limit); u = fminf(fmaxf(u, -limit), limit); }
            const float v = (g / (1.f + __expf(-alpha * g))) * (u + beta);
            h[(size_t)(s0 + mb + tok) * I + j] = __float2bfloat16(v);
          }
        }
    }
  }
}

// ---------------------------------------------------------------------------
// grouped down: out[slot[row]] = w[row] * (h[row] W2[e]^T); grid (ctas_per_expert, E)
// ---------------------------------------------------------------------------
template <bool FP8, int NT>
__global__ void __launch_bounds__(GEMV_WARPS * 32) moe_gemv_down_kernel(
    const uint8_t* __restrict__ W, const float* __restrict__ wscale, int H, int I, const __nv_bfloat16* __restrict__ hp,
    const int* __restrict__ seg, const int* __restrict__ perm_slot, const float* __restrict__ perm_w,
    __nv_bfloat16* __restrict__ out) {
  const int e = blockIdx.y;
  const int s0 = seg[e], cnt = seg[e + 1] - s0;
  if (cnt <= 0) return;
  const size_t eoff = (size_t)e * H * I * (FP8 ? 1 : 2);
  const int sk = (I + 127) >> 7;
  const float* esc = FP8 ? wscale + (size_t)e * ((H + 127) >> 7) * sk : nullptr;
  __shared__ float red[GEMV_WARPS * 32 * 2 * NT * 4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g4 = lane >> 2, tq = lane & 3;
  constexpr int CK = FP8 ? 64 : 32;
  int c0, c1;
  chunk_split((I + CK - 1) / CK, c0, c1);
  {
    const int sl = blockIdx.x;
    const int rb[2] = {sl * 32, sl * 32 + 16};
    for (int mb = 0; mb < cnt; mb += 8 * NT) {
      const int mc = min(8 * NT, cnt - mb);
      float acc[2][NT][4];
      warp_mma_gemv<FP8, NT>(W + eoff, esc, sk, H, I, rb, hp, s0 + mb, I, mc, c0, c1, acc);
      cta_reduce<NT>(acc, red);
      if (warp != 0) continue;
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int row = rb[t] + g4 + (i >> 1) * 8;
            const int tok = n * 8 + 2 * tq + (i & 1);
            if (row < H && tok < mc) {
              const int pr = s0 + mb + tok;
              out[(size_t)perm_slot[pr] * H + row] = __float2bfloat16(acc[t][n][i] * perm_w[pr]);
            }
          }
    }
  }
}

}  // namespace xtu

using namespace xtu;

static int gemv_num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

extern "C" {

// y[M, N] = x[M, K] W^T (+ bias). fp8: W e4m3 [N, K] + scales [ceil(N/128), ceil(K/128)]; else W bf16.
int xtu_gemv(const void* W, const float* wscale, int fp8, int N, int K, const void* x, int x_stride, int M,
             const void* bias, void* y, int y_stride, int y_f32, cudaStream_t s) {
  if (M <= 0 || N <= 0) return 0;
  if (M > 16 || K % 16 != 0) return -2;
  const int grid = (N + 31) / 32;     // one 32-row slice per CTA
  const int nt = M > 8 ? 2 : 1;
#define XTU_GEMV_LAUNCH(F, NTV)                                                                              \
  gemv_dense_kernel<F, NTV><<<grid, GEMV_WARPS * 32, 0, s>>>((const uint8_t*)W, wscale, N, K,               \
                                                             (const __nv_bfloat16*)x, x_stride, M,         \
                                                             (const __nv_bfloat16*)bias, y, y_stride, y_f32)
  if (fp8) {
    if (nt == 1) XTU_GEMV_LAUNCH(true, 1); else XTU_GEMV_LAUNCH(true, 2);
  } else {
    if (nt == 1) XTU_GEMV_LAUNCH(false, 1); else XTU_GEMV_LAUNCH(false, 2);
  }
#undef XTU_GEMV_LAUNCH
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// grouped decode MoE: gate/up+SwiGLU then down+weight+scatter.  mmax bounds the rows
// of any one expert (<= tokens); at most mmax * top_k (<= 16 * mmax) experts have rows.
int xtu_moe_gemv(const void* W13, const float* s13, const void* W2, const float* s2, int fp8, int E, int H, int I,
                 const void* xp, const int* seg, const int* perm_slot, const float* perm_w, void* h, void* slots,
                 int mmax, float limit, float alpha, float beta, cudaStream_t s) {
  if (mmax <= 0) return 0;
  if (H % 32 != 0 || I % 128 != 0) return -2;
  const dim3 g1(I / 16, E), g2((H + 31) / 32, E);   // one slice per CTA; experts without rows exit
  const int nt = mmax > 8 ? 2 : 1;
#define XTU_MOE_GEMV_LAUNCH(F, NTV)                                                                          \
  moe_gemv_gate_up_kernel<F, NTV><<<g1, GEMV_WARPS * 32, 0, s>>>((const uint8_t*)W13, s13, I, H,            \
                                                                 (const __nv_bfloat16*)xp, seg,             \
                                                                 (__nv_bfloat16*)h, limit, alpha, beta);    \
  moe_gemv_down_kernel<F, NTV><<<g2, GEMV_WARPS * 32, 0, s>>>((const uint8_t*)W2, s2, H, I,                 \
                                                              (const __nv_bfloat16*)h, seg, perm_slot,      \
                                                              perm_w, (__nv_bfloat16*)slots)
  if (fp8) {
    if (nt == 1) { XTU_MOE_GEMV_LAUNCH(true, 1); } else { XTU_MOE_GEMV_LAUNCH(true, 2); }
  } else {
    if (nt == 1) { XTU_MOE_GEMV_LAUNCH(false, 1); } else { XTU_MOE_GEMV_LAUNCH(false, 2); }
  }
#undef XTU_MOE_GEMV_LAUNCH
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 2 : -(int)e;
}

}  // extern "C"
