// Gated DeltaNet linear attention (Qwen3-Next "linear_attention" layers), sm_100a.
//
//   gdn_conv_kernel    causal depthwise conv (kernel kw, SiLU) over the q|k|v channels,
//                      gathered straight from the in_proj_qkvz output (per key head:
//                      [q dk | k dk | v r*dv | z r*dv]); earlier inputs of the sequence
//                      come from the slot's conv state.  One warp per (token, head unit);
//                      q and k heads are L2-normalised in the same warp (q also scaled by
//                      1/sqrt(dk)).  Output fp32 q, k [T, nk, dk], v [T, nv, dv].
//   gdn_conv_state_kernel   the slot's conv state <- last kw-1 inputs (after the conv read it).
//   gdn_recurrent_kernel    the gated delta rule, token by token, per (sequence, value head,
//                      32-column slice of the state):
//                          S <- exp(g_t) S + k_t (beta_t (v_t - exp(g_t) S^T k_t))^T,  o_t = S^T q_t
//                      The state slice [dk, 32] lives in registers (4 lanes per column, 32
//                      rows each); the decay is carried as one scalar c (S = c * S_stored),
//                      so a token costs three 32-term dot products and one 32-term update
//                      per lane; c is folded back into the registers before it underflows.
//                      CH = true is the channel-wise form (Kimi Delta Attention): g_t is a
//                      vector over the key dims, S <- Diag(exp(g_t)) S before the same delta
//                      update; exp(g_t) is taken once per (token, channel) while staging, and
//                      each lane scales its 32 rows (one more multiply per row and token).
//
// The in-projection row is either interleaved per key head [q dk | k dk | v r*dv | z r*dv]
// (Qwen3-Next's in_proj_qkvz, z feeding its output gate) or blocked [Q | K | V] with no z
// (KDA: its q, k, v projections concatenated; the output gate has its own projection).
//
// Replaces the FLA chunked kernels the reference's vLLM patches run for these layers;
// the numerics oracle is models/deltanet.py:_delta_rule_ref.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cmath>
#include "ptx.cuh"

namespace xtu {

struct GdnShape {
  int nk, nv, dk, dv, kw;
  int qkvz_stride;     // elements between tokens of the in_proj output
  int blocked;         // 1: the row is [Q | K | V] (conv channel order), 0: per key head with z
};

__device__ __forceinline__ int seq_of(const int* __restrict__ q_start, int B, int t) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (q_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// channel c of the conv input (q | k | v order) -> column of the qkvz row
__device__ __forceinline__ int qkvz_col(const GdnShape& s, int c) {
  if (s.blocked) return c;
  const int r = s.nv / s.nk;
  const int W = 2 * s.dk + 2 * r * s.dv;
  const int nq = s.nk * s.dk;
  if (c < nq) return (c / s.dk) * W + (c % s.dk);
  c -= nq;
  if (c < nq) return (c / s.dk) * W + s.dk + (c % s.dk);
  c -= nq;
  const int vh = c / s.dv, d = c % s.dv;
  return (vh / r) * W + 2 * s.dk + (vh % r) * s.dv + d;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }

// grid: (T, units = 2*nk + nv); block 32 (one warp)
__global__ void gdn_conv_kernel(const __nv_bfloat16* __restrict__ qkvz, GdnShape s, const float* __restrict__ conv_w,
                                const __nv_bfloat16* __restrict__ conv_state, const int* __restrict__ q_start,
                                const int* __restrict__ slots, const int* __restrict__ fresh, int B,
                                float* __restrict__ qo, float* __restrict__ ko, float* __restrict__ vo) {
  const int t = blockIdx.x, u = blockIdx.y, lane = threadIdx.x;
  const int b = seq_of(q_start, B, t);
  const int t0 = q_start[b];
  const int slot = slots[b];
  // slot < 0: a padding sequence of a captured decode graph -- no state, read as fresh
  const bool is_fresh = slot < 0 || (fresh != nullptr && fresh[b] != 0);
  const int nq = s.nk * s.dk;
  const int ch = 2 * nq + s.nv * s.dv;
  int c0, width;
  if (u < s.nk) { c0 = u * s.dk; width = s.dk; }
  else if (u < 2 * s.nk) { c0 = nq + (u - s.nk) * s.dk; width = s.dk; }
  else { c0 = 2 * nq + (u - 2 * s.nk) * s.dv; width = s.dv; }
  float vals[8];
  float ss = 0.f;
  const int per = (width + 31) / 32;   // <= 8 (head dims up to 256)
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    vals[i] = 0.f;
    if (i >= per) continue;
    const int d = lane + 32 * i;
    if (d >= width) continue;
    const int c = c0 + d;
    const int col = qkvz_col(s, c);
    float acc = 0.f;
    for (int j = 0; j < s.kw; ++j) {
      const int tt = t - (s.kw - 1) + j;   // input position of tap j
      float x;
      if (tt >= t0) {
        x = __bfloat162float(qkvz[(size_t)tt * s.qkvz_stride + col]);
      } else {
        const int back = t0 - tt;            // 1 .. kw-1 steps before the chunk
        x = is_fresh ? 0.f : __bfloat162float(conv_state[((size_t)slot * ch + c) * (s.kw - 1) + (s.kw - 1 - back)]);
      }
      acc += x * conv_w[(size_t)c * s.kw + j];
    }
    const float y = silu_f(acc);
    vals[i] = y;
    ss += y * y;
  }
  if (u < 2 * s.nk) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    float inv = 1.f / fmaxf(sqrtf(ss), 1e-12f);   // x / max(||x||, 1e-12), as F.normalize
    if (u < s.nk) inv *= rsqrtf((float)s.dk);
    float* dst = (u < s.nk ? qo + ((size_t)t * s.nk + u) * s.dk : ko + ((size_t)t * s.nk + (u - s.nk)) * s.dk);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (i < per && d < width) dst[d] = vals[i] * inv;
    }
  } else {
    float* dst = vo + ((size_t)t * s.nv + (u - 2 * s.nk)) * s.dv;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (i < per && d < width) dst[d] = vals[i];
    }
  }
}

// grid: (B, ceil(ch / 256)); the new state of each channel = its last kw-1 inputs
__global__ void gdn_conv_state_kernel(const __nv_bfloat16* __restrict__ qkvz, GdnShape s,
                                      __nv_bfloat16* __restrict__ conv_state, const int* __restrict__ q_start,
                                      const int* __restrict__ slots, const int* __restrict__ fresh) {
  const int b = blockIdx.x;
  const int nq = s.nk * s.dk;
  const int ch = 2 * nq + s.nv * s.dv;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= ch) return;
  const int t0 = q_start[b], t1 = q_start[b + 1];
  const int L = t1 - t0;
  if (L <= 0) return;
  const int slot = slots[b];
  if (slot < 0) return;                    // padding sequence: it owns no state
  const bool is_fresh = fresh != nullptr && fresh[b] != 0;
  const int col = qkvz_col(s, c);
  __nv_bfloat16* st = conv_state + ((size_t)slot * ch + c) * (s.kw - 1);
  __nv_bfloat16 nw[8];
  for (int j = 0; j < s.kw - 1; ++j) {
    const int pos = L - (s.kw - 1) + j;    // index in [old state ++ chunk] relative to chunk start
    if (pos >= 0) nw[j] = qkvz[(size_t)(t0 + pos) * s.qkvz_stride + col];
    else nw[j] = is_fresh ? __float2bfloat16(0.f) : st[(s.kw - 1) + pos];
  }
  for (int j = 0; j < s.kw - 1; ++j) st[j] = nw[j];
}

constexpr int GDN_COLS = 32;       // state columns per CTA
constexpr int GDN_TB = 16;         // tokens staged in shared memory at a time

// grid: (B, nv, dv / 32); block 128: lane = col8 * 4 + rq (8 columns x 4 row quarters per warp)
template <int DK, bool CH>
__global__ void __launch_bounds__(128) gdn_recurrent_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, const int* __restrict__ q_start, const int* __restrict__ slots,
    const int* __restrict__ fresh, float* __restrict__ ssm, float* __restrict__ out, int nk, int nv, int dv) {
  constexpr int RPT = DK / 4;                 // state rows per thread
  __shared__ float sq[GDN_TB][DK], sk[GDN_TB][DK];
  __shared__ float sv[GDN_TB][GDN_COLS], sg[GDN_TB], sb[GDN_TB];
  __shared__ float sa[CH ? GDN_TB : 1][CH ? DK : 1];   // CH: exp(g) per (token, key dim)
  const int b = blockIdx.x, h = blockIdx.y, cg = blockIdx.z;
  const int t0 = q_start[b], t1 = q_start[b + 1];
  if (t1 <= t0) return;
  const int kh = h / (nv / nk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cl = warp * 8 + (lane >> 2);      // column within the slice
  const int rq = lane & 3;
  const int col = cg * GDN_COLS + cl;
  const int slot = slots[b];
  // slot < 0: a padding sequence of a captured decode graph; it starts from a zero state
  // and writes none back
  float* S_g = slot < 0 ? nullptr : ssm + (((size_t)slot * nv + h) * DK) * dv;
  float S[RPT];
  const bool is_fresh = slot < 0 || (fresh != nullptr && fresh[b] != 0);
#pragma unroll
  // lane rq holds rows 4i + rq (interleaved, so the four row groups of a warp read four
  // different banks of the staged q / k vectors)
  for (int i = 0; i < RPT; ++i) S[i] = is_fresh ? 0.f : S_g[(size_t)(4 * i + rq) * dv + col];
  float c = 1.f;
  for (int tb = t0; tb < t1; tb += GDN_TB) {
    const int n = min(GDN_TB, t1 - tb);
    __syncthreads();
    for (int i = threadIdx.x; i < n * DK; i += 128) {
      const int tt = i / DK, d = i % DK;
      sq[tt][d] = q[((size_t)(tb + tt) * nk + kh) * DK + d];
      sk[tt][d] = k[((size_t)(tb + tt) * nk + kh) * DK + d];
    }
    for (int i = threadIdx.x; i < n * GDN_COLS; i += 128) {
      const int tt = i / GDN_COLS, d = i % GDN_COLS;
      sv[tt][d] = v[((size_t)(tb + tt) * nv + h) * dv + cg * GDN_COLS + d];
    }
    if (CH) {
      for (int i = threadIdx.x; i < n * DK; i += 128) {
        const int tt = i / DK, d = i % DK;
        sa[tt][d] = __expf(g[((size_t)(tb + tt) * nv + h) * DK + d]);
      }
    }
    if (threadIdx.x < n) {
      if (!CH) sg[threadIdx.x] = g[(size_t)(tb + threadIdx.x) * nv + h];
      sb[threadIdx.x] = beta[(size_t)(tb + threadIdx.x) * nv + h];
    }
    __syncthreads();
    for (int tt = 0; tt < n; ++tt) {
      const float* kt = &sk[tt][rq];
      const float* qt = &sq[tt][rq];
      if (CH) {
        const float* at = &sa[tt][rq];
#pragma unroll
        for (int i = 0; i < RPT; ++i) S[i] *= at[4 * i];
      }
      float a = 0.f, bq = 0.f, kq = 0.f;
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        a = fmaf(S[i], kt[4 * i], a);
        bq = fmaf(S[i], qt[4 * i], bq);
        kq = fmaf(kt[4 * i], qt[4 * i], kq);
      }
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        bq += __shfl_xor_sync(0xffffffffu, bq, o);
        kq += __shfl_xor_sync(0xffffffffu, kq, o);
      }
      if (!CH) c *= __expf(sg[tt]);
      const float delta = sb[tt] * (sv[tt][cl] - c * a);
      if (rq == 0) out[((size_t)(tb + tt) * nv + h) * dv + col] = c * bq + delta * kq;
      const float dc = delta / c;
#pragma unroll
      for (int i = 0; i < RPT; ++i) S[i] = fmaf(kt[4 * i], dc, S[i]);
      if (c < 1e-20f) {                        // fold the decay back before it underflows
#pragma unroll
        for (int i = 0; i < RPT; ++i) S[i] *= c;
        c = 1.f;
      }
    }
  }
  if (S_g == nullptr) return;
#pragma unroll
  for (int i = 0; i < RPT; ++i) S_g[(size_t)(4 * i + rq) * dv + col] = S[i] * c;
}

}  // namespace xtu

using namespace xtu;

extern "C" {

// qkvz: in_proj output [T, qkvz_stride] bf16; conv_w fp32 [ch, kw]; conv_state bf16 [slots, ch, kw-1];
// ssm fp32 [slots, nv, dk, dv] (a sequence whose slot is < 0 is computed from a zero state and
// leaves every state untouched); g fp32 [T, nv] (g_channels = 0) or [T, nv, dk] (channel-wise
// decay, g_channels = 1); beta fp32 [T, nv]; blocked: qkvz rows are [Q | K | V] (else per key
// head [q | k | v | z]); scratch q/k fp32 [T, nk, dk], v fp32 [T, nv, dv]; out fp32 [T, nv, dv].
// Returns kernels launched or a negative error.
int xtu_deltanet_fwd(const void* qkvz, int qkvz_stride, int T, int B, const int* q_start, const int* slots,
                     const int* fresh, int nk, int nv, int dk, int dv, int kw, const float* conv_w, void* conv_state,
                     float* ssm, const float* g, const float* beta, float* qs, float* ks, float* vs, float* out,
                     int blocked, int g_channels, cudaStream_t stream) {
  if (T <= 0 || B <= 0) return 0;
  if (dk != 128 || dv % GDN_COLS != 0 || dv > 256 || kw < 2 || kw > 9 || nv % nk != 0) return -2;
  GdnShape s{nk, nv, dk, dv, kw, qkvz_stride, blocked ? 1 : 0};
  const int ch = 2 * nk * dk + nv * dv;
  gdn_conv_kernel<<<dim3(T, 2 * nk + nv), 32, 0, stream>>>((const __nv_bfloat16*)qkvz, s, conv_w,
                                                          (const __nv_bfloat16*)conv_state, q_start, slots, fresh, B,
                                                          qs, ks, vs);
  gdn_conv_state_kernel<<<dim3(B, (ch + 255) / 256), 256, 0, stream>>>((const __nv_bfloat16*)qkvz, s,
                                                                        (__nv_bfloat16*)conv_state, q_start, slots,
                                                                        fresh);
  if (g_channels)
    gdn_recurrent_kernel<128, true><<<dim3(B, nv, dv / GDN_COLS), 128, 0, stream>>>(qs, ks, vs, g, beta, q_start,
                                                                                  slots, fresh, ssm, out, nk, nv, dv);
  else
    gdn_recurrent_kernel<128, false><<<dim3(B, nv, dv / GDN_COLS), 128, 0, stream>>>(qs, ks, vs, g, beta, q_start,
                                                                                   slots, fresh, ssm, out, nk, nv, dv);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 3 : -(int)e;
}

}  // extern "C"
