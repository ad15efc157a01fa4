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

// fp32 -> tf32 (round to nearest, ties away), as a 32-bit pattern
__device__ __forceinline__ uint32_t f2tf(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

constexpr int GDN_CONV_TPW = 4;        // tokens per warp of the conv kernel
constexpr int GDN_CONV_WARPS = 8;

// Gates of the scalar-decay form from the in_proj_ba row (per key head [b r | a r]):
//   beta = sigmoid(b),  g = -exp(A_log) softplus(a + dt_bias)
struct GdnGates {
  const __nv_bfloat16* ba;   // nullptr: g and beta are inputs
  int ba_stride;
  const float* A_log;        // [nv]
  const float* dt_bias;      // [nv]
  float* g;                  // [T, nv] out
  float* beta;               // [T, nv] out
};

// grid: (ceil(T / (8 * 4)), units = 2*nk + nv); block 256: warp w handles 4 consecutive
// tokens of one head unit.  A unit's channels are contiguous columns of the qkvz row, so
// a lane's column, its KW conv taps and the KW - 1 + 4 inputs the four tokens share are
// read once; taps before a token's sequence start come from the slot's conv state.
// round_tf32: q and k are stored rounded to tf32 (the chunked form's tensor-core operands).
// PER: head-dim elements per lane (4: head dims <= 128, 8: <= 256).
template <int KW, int PER>
__global__ void __launch_bounds__(GDN_CONV_WARPS * 32) gdn_conv_kernel(
    const __nv_bfloat16* __restrict__ qkvz, GdnShape s, const float* __restrict__ conv_w,
    const __nv_bfloat16* __restrict__ conv_state, const int* __restrict__ q_start, const int* __restrict__ slots,
    const int* __restrict__ fresh, int B, int T, float* __restrict__ qo, float* __restrict__ ko,
    float* __restrict__ vo, GdnGates gt, int round_tf32) {
  constexpr int TPW = GDN_CONV_TPW;
  const int u = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tb = (blockIdx.x * GDN_CONV_WARPS + warp) * TPW;
  if (tb >= T) return;
  const int nq = s.nk * s.dk;
  const int ch = 2 * nq + s.nv * s.dv;
  const int r = s.nv / s.nk;
  const int Wrow = 2 * s.dk + 2 * r * s.dv;   // per-key-head group width of the interleaved row
  int c0, width, colbase;
  if (u < s.nk) {
    c0 = u * s.dk; width = s.dk; colbase = s.blocked ? c0 : u * Wrow;
  } else if (u < 2 * s.nk) {
    c0 = nq + (u - s.nk) * s.dk; width = s.dk; colbase = s.blocked ? c0 : (u - s.nk) * Wrow + s.dk;
  } else {
    const int vh = u - 2 * s.nk;
    c0 = 2 * nq + vh * s.dv; width = s.dv; colbase = s.blocked ? c0 : (vh / r) * Wrow + 2 * s.dk + (vh % r) * s.dv;
  }
  int t0s[TPW], slot_s[TPW];
  bool fr[TPW];
#pragma unroll
  for (int tt = 0; tt < TPW; ++tt) {
    const int t = min(tb + tt, T - 1);
    const int b = seq_of(q_start, B, t);
    t0s[tt] = q_start[b];
    slot_s[tt] = slots[b];
    // slot < 0: a padding sequence of a captured decode graph -- no state, read as fresh
    fr[tt] = slot_s[tt] < 0 || (fresh != nullptr && fresh[b] != 0);
  }
  const int per = (width + 31) / 32;   // <= PER
  float vals[PER][TPW];
  float ss[TPW];
#pragma unroll
  for (int tt = 0; tt < TPW; ++tt) ss[tt] = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
#pragma unroll
    for (int tt = 0; tt < TPW; ++tt) vals[i][tt] = 0.f;
    const int d = lane + 32 * i;
    if (i >= per || d >= width) continue;
    const int c = c0 + d;
    float w[KW];
#pragma unroll
    for (int j = 0; j < KW; ++j) w[j] = conv_w[(size_t)c * KW + j];
    float xs[TPW + KW - 1];             // inputs at tb - (KW - 1) .. tb + TPW - 1
#pragma unroll
    for (int p = 0; p < TPW + KW - 1; ++p) {
      const int tp = tb - (KW - 1) + p;
      xs[p] = (tp >= 0 && tp < T) ? __bfloat162float(qkvz[(size_t)tp * s.qkvz_stride + colbase + d]) : 0.f;
    }
#pragma unroll
    for (int tt = 0; tt < TPW; ++tt) {
      const int t = tb + tt;
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < KW; ++j) {
        const int tp = t - (KW - 1) + j;   // input position of tap j
        float x = xs[tt + j];
        if (tp < t0s[tt]) {               // before the sequence: the slot's conv state
          const int back = t0s[tt] - tp;  // 1 .. KW-1 steps before the chunk
          x = fr[tt] ? 0.f
                     : __bfloat162float(conv_state[((size_t)slot_s[tt] * ch + c) * (KW - 1) + (KW - 1 - back)]);
        }
        acc = fmaf(x, w[j], acc);
      }
      const float y = silu_f(acc);
      vals[i][tt] = y;
      ss[tt] = fmaf(y, y, ss[tt]);
    }
  }
#pragma unroll
  for (int tt = 0; tt < TPW; ++tt) {
    const int t = tb + tt;
    if (t >= T) break;
    if (u < 2 * s.nk) {
      float sq = ss[tt];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      float inv = 1.f / fmaxf(sqrtf(sq), 1e-12f);   // x / max(||x||, 1e-12), as F.normalize
      if (u < s.nk) inv *= rsqrtf((float)s.dk);
      float* dst = (u < s.nk ? qo + ((size_t)t * s.nk + u) * s.dk : ko + ((size_t)t * s.nk + (u - s.nk)) * s.dk);
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int d = lane + 32 * i;
        if (i < per && d < width) {
          float y = vals[i][tt] * inv;
          if (round_tf32) y = __uint_as_float(f2tf(y));
          dst[d] = y;
        }
      }
    } else {
      const int vh = u - 2 * s.nk;
      float* dst = vo + ((size_t)t * s.nv + vh) * s.dv;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int d = lane + 32 * i;
        if (i < per && d < width) dst[d] = vals[i][tt];
      }
      if (gt.ba != nullptr && lane == 0) {
        const __nv_bfloat16* row = gt.ba + (size_t)t * gt.ba_stride + (vh / r) * 2 * r;
        const float bb = __bfloat162float(row[vh % r]);
        const float aa = __bfloat162float(row[r + vh % r]) + gt.dt_bias[vh];
        const float sp = aa > 20.f ? aa : log1pf(__expf(aa));   // softplus, threshold 20
        gt.beta[(size_t)t * s.nv + vh] = 1.f / (1.f + __expf(-bb));
        gt.g[(size_t)t * s.nv + vh] = -__expf(gt.A_log[vh]) * sp;
      }
    }
  }
}

// Gated RMSNorm of the recurrence output, one warp per (token, value head):
//   y = o / sqrt(mean(o^2) + eps) * w * act(gate),  act = silu (z of the in_proj_qkvz row,
//   gate_mode 0) or sigmoid (a [T, nv*dv] gate tensor, gate_mode 1); y bf16 [T, nv*dv].
__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(const float* __restrict__ o,
                                                             const __nv_bfloat16* __restrict__ gate, int gate_stride,
                                                             int gate_mode, GdnShape s, const float* __restrict__ w,
                                                             float eps, __nv_bfloat16* __restrict__ y, int T) {
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (item >= T * s.nv) return;
  const int t = item / s.nv, vh = item % s.nv;
  const int per = s.dv / 32;                 // dv in {32, 64, ..., 256}
  const float* src = o + ((size_t)t * s.nv + vh) * s.dv;
  float x[8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    x[i] = i < per ? src[lane + 32 * i] : 0.f;
    ss += x[i] * x[i];
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  const float inv = rsqrtf(ss / (float)s.dv + eps);
  const __nv_bfloat16* gr;
  if (gate_mode == 0) {
    const int r = s.nv / s.nk;
    gr = gate + (size_t)t * gate_stride + (vh / r) * (2 * s.dk + 2 * r * s.dv) + 2 * s.dk + r * s.dv + (vh % r) * s.dv;
  } else {
    gr = gate + (size_t)t * gate_stride + vh * s.dv;
  }
  __nv_bfloat16* dst = y + ((size_t)t * s.nv + vh) * s.dv;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i >= per) continue;
    const int d = lane + 32 * i;
    const float z = __bfloat162float(gr[d]);
    const float act = gate_mode == 0 ? silu_f(z) : 1.f / (1.f + __expf(-z));
    dst[d] = __float2bfloat16(x[i] * inv * w[d] * act);
  }
}

// grid: (B, ceil(ch / 256)); the new state of each channel = its last kw-1 inputs.
// spec_conv (speculative verification steps of at most spec_n tokens per sequence): also
// the state after each token j of the step, spec_conv [slots, spec_n, ch, kw-1].
__global__ void gdn_conv_state_kernel(const __nv_bfloat16* __restrict__ qkvz, GdnShape s,
                                      __nv_bfloat16* __restrict__ conv_state, const int* __restrict__ q_start,
                                      const int* __restrict__ slots, const int* __restrict__ fresh,
                                      __nv_bfloat16* __restrict__ spec_conv, int spec_n) {
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
  // input at position pos of [old state ++ step] (pos < 0: the old state)
  auto input = [&](int pos) -> __nv_bfloat16 {
    if (pos >= 0) return qkvz[(size_t)(t0 + pos) * s.qkvz_stride + col];
    return is_fresh ? __float2bfloat16(0.f) : st[(s.kw - 1) + pos];
  };
  if (spec_conv != nullptr) {
    for (int j = 0; j < L && j < spec_n; ++j) {
      __nv_bfloat16* dst = spec_conv + (((size_t)slot * spec_n + j) * ch + c) * (s.kw - 1);
      for (int i = 0; i < s.kw - 1; ++i) dst[i] = input(j - (s.kw - 2) + i);
    }
  }
  __nv_bfloat16 nw[8];
  for (int j = 0; j < s.kw - 1; ++j) nw[j] = input(L - (s.kw - 1) + j);
  for (int j = 0; j < s.kw - 1; ++j) st[j] = nw[j];
}

// Speculative verification: per sequence b, the states after its accepted position
// acc[b] (of the step's spec_n) become the slot's states.  grid (B, 64); block 256.
__global__ void gdn_spec_commit_kernel(const int* __restrict__ acc, const int* __restrict__ slots, int spec_n,
                                       const float4* __restrict__ spec_ssm, float4* __restrict__ ssm,
                                       long long ssm_vec, const __nv_bfloat16* __restrict__ spec_conv,
                                       __nv_bfloat16* __restrict__ conv, long long conv_elems) {
  const int b = blockIdx.x;
  const int slot = slots[b];
  if (slot < 0) return;
  const int a = min(max(acc[b], 0), spec_n - 1);
  const float4* src = spec_ssm + ((size_t)slot * spec_n + a) * ssm_vec;
  float4* dst = ssm + (size_t)slot * ssm_vec;
  for (long long i = (long long)blockIdx.y * blockDim.x + threadIdx.x; i < ssm_vec; i += (long long)gridDim.y * blockDim.x)
    dst[i] = src[i];
  const __nv_bfloat16* cs = spec_conv + ((size_t)slot * spec_n + a) * conv_elems;
  __nv_bfloat16* cd = conv + (size_t)slot * conv_elems;
  for (long long i = (long long)blockIdx.y * blockDim.x + threadIdx.x; i < conv_elems;
       i += (long long)gridDim.y * blockDim.x)
    cd[i] = cs[i];
}

constexpr int GDN_COLS = 32;       // state columns per CTA
constexpr int GDN_TB = 16;         // tokens staged in shared memory at a time

// grid: (B, nv, dv / 32); block 128: lane = col8 * 4 + rq (8 columns x 4 row quarters per warp)
// spec_ssm (speculative verification): also the state after each token j of the step,
// spec_ssm [slots, spec_n, nv, DK, dv].
template <int DK, bool CH>
__global__ void __launch_bounds__(128) gdn_recurrent_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, const int* __restrict__ q_start, const int* __restrict__ slots,
    const int* __restrict__ fresh, float* __restrict__ ssm, float* __restrict__ out, int nk, int nv, int dv,
    float* __restrict__ spec_ssm, int spec_n) {
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
      if (spec_ssm != nullptr && S_g != nullptr && tb + tt - t0 < spec_n) {
        float* sp = spec_ssm + ((((size_t)slot * spec_n + (tb + tt - t0)) * nv + h) * DK) * dv;
#pragma unroll
        for (int i = 0; i < RPT; ++i) sp[(size_t)(4 * i + rq) * dv + col] = S[i] * c;
      }
    }
  }
  if (S_g == nullptr) return;
#pragma unroll
  for (int i = 0; i < RPT; ++i) S_g[(size_t)(4 * i + rq) * dv + col] = S[i] * c;
}

// ---------------------------------------------------------------------------
// Chunked gated delta rule (prefill), on the tensor cores.  Per chunk of C = 64 tokens
// with cumulative log-decay gamma_i (Gam_i = exp(gamma_i)) and the state S0 it starts
// from, the recurrence above unrolls to (rows = tokens; the UT / WY form):
//     (I + A) U = R,  A_ij = beta_i exp(gamma_i - gamma_j) (k_i . k_j)    (j < i),
//                     R_i = beta_i (v_i - Gam_i (K S0)_i)
//     O = diag(Gam) (Q S0) + P U,  P_ij = exp(gamma_i - gamma_j) (q_i . k_j)  (j <= i)
//     S_C = Gam_C S0 + Kt^T U,     Kt_j = exp(gamma_C - gamma_j) k_j
// With T = (I + A)^-1 the delta terms split into a state-free part and a state term:
//     U = U0 - W S0,   U0 = T diag(beta) V,   W = T diag(beta Gam) K
// so everything but the three products with S0 is independent across chunks:
//   gdn_chunk_prep_kernel   one CTA per (chunk, value head), all chunks at once: P, T (by
//                           column-parallel forward substitution), W and U0 (U0 over v
//                           in place), the in-chunk cumulative log decay.
//   gdn_chunk_state_kernel  one CTA per (sequence, value head, 32-column slice of dv; the
//                           state's dv columns are independent) walks the chunks:
//                           [W; Q] S0 -> U, O = diag(Gam) Q S0 + P U, S <- Gam_C S0 + K^T diag(Gk) U;
//                           the next chunk's operands stream in by cp.async meanwhile.
// Every product is a warp-tiled tf32 mma.sync m16n8k8 with fp32 accumulation; the state
// stays fp32 in shared memory.  dk = dv = 128, scalar decay per token (Qwen3-Next GDN).
// ---------------------------------------------------------------------------
constexpr int GC = 64;                 // tokens per chunk
constexpr int GD = 128;                // dk = dv
constexpr int LD128 = GD + 4;          // padded fp32 row strides (conflict-free A fragments)
constexpr int LD64 = GC + 4;
constexpr int LDK = GD + 8;            // K read as a transposed A operand
constexpr int SC = 32;                 // state columns per CTA of the state kernel
constexpr int LDS = SC + 8;            // row-major B operands [k][n]
constexpr int GDN_PREP_THREADS = 256;
constexpr int GDN_PREP_SMEM = (2 * GC * LD128 + 2 * GC * LD64 + 2 * GC) * 4;
constexpr int GDN_ST_THREADS = 512;
constexpr int GDN_ST_SMEM = (2 * GD * LDS + 2 * GC * LD128 + GC * LDK + GC * LD64 + 4 * GC * LDS + GC) * 4;

__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16-byte / 4-byte asynchronous copies global -> shared; src_bytes 0 fills zeros
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int src_bytes) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// acc[j][4] += A[m0 .. m0+16) x B[.., n0 + 8j .. +8) over k in [0, K):
//   A(i, k) = AT ? a[k * lda + i] : a[i * lda + k]
//   B(k, n) = BT ? b[n * ldb + k] : b[k * ldb + n]
// CA / CB false: that operand is already held as tf32-rounded fp32 patterns
template <int NJ, bool AT, bool BT, bool CA = true, bool CB = true>
__device__ __forceinline__ void warp_mma(float (&acc)[NJ][4], const float* a, int lda, const float* b, int ldb,
                                         int m0, int n0, int K) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  auto ta = [](float x) -> uint32_t { return CA ? f2tf(x) : __float_as_uint(x); };
  auto tb = [](float x) -> uint32_t { return CB ? f2tf(x) : __float_as_uint(x); };
  for (int k = 0; k < K; k += 8) {
    const int r0 = m0 + g, r1 = m0 + g + 8, c0 = k + t, c1 = k + t + 4;
    uint32_t a0, a1, a2, a3;
    if (AT) {
      a0 = ta(a[c0 * lda + r0]); a1 = ta(a[c0 * lda + r1]);
      a2 = ta(a[c1 * lda + r0]); a3 = ta(a[c1 * lda + r1]);
    } else {
      a0 = ta(a[r0 * lda + c0]); a1 = ta(a[r1 * lda + c0]);
      a2 = ta(a[r0 * lda + c1]); a3 = ta(a[r1 * lda + c1]);
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int n = n0 + 8 * j + g;
      const uint32_t b0 = tb(BT ? b[n * ldb + c0] : b[c0 * ldb + n]);
      const uint32_t b1 = tb(BT ? b[n * ldb + c1] : b[c1 * ldb + n]);
      mma_tf32(acc[j], a0, a1, a2, a3, b0, b1);
    }
  }
}

// MT m-tiles (m0 + 16 mt) sharing the B fragments; B row-major [k][n], columns n0 .. n0 + 8 NJ.
// CA / CB false: that operand is already tf32-rounded.  The k loop runs two independent
// accumulator chains (even / odd k steps) that are added at the end, halving the chain of
// dependent MMAs.
template <int MT, int NJ, bool AT, int K, bool CA = true, bool CB = true>
__device__ __forceinline__ void warp_mma_mt(float (&acc)[MT][NJ][4], const float* a, int lda, const float* b, int ldb,
                                            int m0, int n0 = 0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  auto ta = [](float x) -> uint32_t { return CA ? f2tf(x) : __float_as_uint(x); };
  auto tb = [](float x) -> uint32_t { return CB ? f2tf(x) : __float_as_uint(x); };
  float acc2[MT][NJ][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc2[mt][j][e] = 0.f;
  auto step = [&](int k, float (&ac)[MT][NJ][4]) {
    const int c0 = k + t, c1 = k + t + 4;
    uint32_t bf[NJ][2];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      bf[j][0] = tb(b[c0 * ldb + n0 + 8 * j + g]);
      bf[j][1] = tb(b[c1 * ldb + n0 + 8 * j + g]);
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int r0 = m0 + 16 * mt + g, r1 = r0 + 8;
      uint32_t a0, a1, a2, a3;
      if (AT) {
        a0 = ta(a[c0 * lda + r0]); a1 = ta(a[c0 * lda + r1]);
        a2 = ta(a[c1 * lda + r0]); a3 = ta(a[c1 * lda + r1]);
      } else {
        a0 = ta(a[r0 * lda + c0]); a1 = ta(a[r1 * lda + c0]);
        a2 = ta(a[r0 * lda + c1]); a3 = ta(a[r1 * lda + c1]);
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) mma_tf32(ac[mt][j], a0, a1, a2, a3, bf[j][0], bf[j][1]);
    }
  };
  static_assert(K % 16 == 0, "two k steps per iteration");
#pragma unroll 2
  for (int k = 0; k < K; k += 16) {
    step(k, acc);
    step(k + 8, acc2);
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][j][e] += acc2[mt][j][e];
}

// chunk j of the step (sequences' chunks in order) -> sequence b, first token c0, length n;
// warp-cooperative, every lane gets the answer; false past the last chunk
__device__ __forceinline__ bool chunk_of(const int* __restrict__ q_start, int B, int j, int& b_out, int& c0, int& n) {
  const int lane = threadIdx.x & 31;
  int base = 0;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    int nc = 0;
    if (b < B) nc = (q_start[b + 1] - q_start[b] + GC - 1) / GC;
    int incl = nc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (j < base + total) {
      const bool mine = nc > 0 && j >= base + incl - nc && j < base + incl;
      const int src = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
      const int first = __shfl_sync(0xffffffffu, base + incl - nc, src);
      b_out = b0 + src;
      c0 = q_start[b_out] + (j - first) * GC;
      n = min(GC, q_start[b_out + 1] - c0);
      return true;
    }
    base += total;
  }
  return false;
}

// grid (ceil(T / 64) + B, nv); block 256.  q, k fp32 [T, nk, 128] (q pre-scaled), v fp32
// [T, nv, 128] (<- U0), g, beta fp32 [T, nv]; ws_w fp32 [T, nv, 128] (<- W), ws_p fp32
// [T, nv, 64] (<- P rows), ws_g fp32 [T, nv] (<- in-chunk cumulative log decay).
__global__ void __launch_bounds__(GDN_PREP_THREADS, 2) gdn_chunk_prep_kernel(
    const float* __restrict__ q, const float* __restrict__ k, float* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, const int* __restrict__ q_start, int B, float* __restrict__ ws_w,
    float* __restrict__ ws_p, float* __restrict__ ws_g, int nk, int nv) {
  extern __shared__ float gsm[];
  float* Kc = gsm;                      // [64][LD128]  k, then diag(beta Gam) k
  float* QV = Kc + GC * LD128;          // [64][LD128]  q, then diag(beta) v
  float* Tm = QV + GC * LD128;          // [64][LD64]   A
  float* Ti = Tm + GC * LD64;           // [64][LD64]   T = (I + A)^-1
  float* gam = Ti + GC * LD64;          // [64] cumulative log decay
  float* bet = gam + GC;                // [64]
  const int h = blockIdx.y;
  int b, c0, n;
  if (!chunk_of(q_start, B, blockIdx.x, b, c0, n)) return;
  const int kh = h / (nv / nk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  // ---- stage q, k (rows past n are zero: they neither read nor write the state)
  for (int i = tid; i < GC * (GD / 4); i += GDN_PREP_THREADS) {
    const int r = i / (GD / 4), c4 = (i % (GD / 4)) * 4;
    const size_t tok = c0 + min(r, n - 1);
    cp_async16(QV + r * LD128 + c4, q + (tok * nk + kh) * GD + c4, r < n ? 16 : 0);
    cp_async16(Kc + r * LD128 + c4, k + (tok * nk + kh) * GD + c4, r < n ? 16 : 0);
  }
  cp_async_commit();
  if (warp == 0) {           // inclusive scan of g over the chunk (two tokens per lane)
    const float g0 = lane * 2 < n ? g[(size_t)(c0 + lane * 2) * nv + h] : 0.f;
    const float g1 = lane * 2 + 1 < n ? g[(size_t)(c0 + lane * 2 + 1) * nv + h] : 0.f;
    float s = g0 + g1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    const float ex = s - g0 - g1;          // exclusive prefix of the pair
    gam[lane * 2] = ex + g0;
    gam[lane * 2 + 1] = ex + g0 + g1;
    bet[lane * 2] = lane * 2 < n ? beta[(size_t)(c0 + lane * 2) * nv + h] : 0.f;
    bet[lane * 2 + 1] = lane * 2 + 1 < n ? beta[(size_t)(c0 + lane * 2 + 1) * nv + h] : 0.f;
  }
  cp_async_wait<0>();
  __syncthreads();
  if (tid < n) ws_g[(size_t)(c0 + tid) * nv + h] = gam[tid];
  // ---- A = beta_i d_ij k_i.k_j (j < i) into Tm; P = d_ij q_i.k_j (j <= i) straight to ws_p
  {
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
    float aa[4][4] = {}, pp[4][4] = {};
    // q and k arrive tf32-rounded from the conv kernel
    warp_mma<4, false, true, false, false>(aa, Kc, LD128, Kc, LD128, m0, n0, GD);
    warp_mma<4, false, true, false, false>(pp, QV, LD128, Kc, LD128, m0, n0, GD);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = m0 + gq + hh * 8, c = n0 + 8 * j + 2 * tq;
        float av[2], pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float d = (c + e <= i) ? __expf(gam[i] - gam[c + e]) : 0.f;
          av[e] = c + e < i ? bet[i] * d * aa[j][2 * hh + e] : 0.f;
          pv[e] = d * pp[j][2 * hh + e];
          Tm[i * LD64 + c + e] = av[e];
        }
        if (i < n)      // stored tf32-rounded: the state kernel's tensor-core operand
          *reinterpret_cast<float2*>(ws_p + ((size_t)(c0 + i) * nv + h) * GC + c) =
              make_float2(__uint_as_float(f2tf(pv[0])), __uint_as_float(f2tf(pv[1])));
      }
  }
  __syncthreads();                         // A complete; q no longer needed
  // ---- stage v over q while T forms
  for (int i = tid; i < GC * (GD / 4); i += GDN_PREP_THREADS) {
    const int r = i / (GD / 4), c4 = (i % (GD / 4)) * 4;
    const size_t tok = c0 + min(r, n - 1);
    cp_async16(QV + r * LD128 + c4, v + (tok * nv + h) * GD + c4, r < n ? 16 : 0);
  }
  cp_async_commit();
  // ---- T = (I + A)^-1 by 16 x 16 blocks (A is unit-free strictly lower triangular):
  //   T_II = (I + A_II)^-1  by forward substitution, column c of a block by four lanes;
  //   T_IJ = -T_II sum_{K=J..I-1} A_IK T_KJ  (I > J), by block distance I - J = 1, 2, 3,
  //   each 16 x 8 piece one warp's two tf32 products (the sum, then -T_II times it)
  {
    const int c = tid >> 2, r4 = tid & 3;      // column 0..63, lane of four
    const int blk = c >> 4, cb = c & 15;        // block of the column, column within it
    const float* Ab = Tm + (blk * 16) * LD64 + blk * 16;
    float xc[4];                                // this lane's x_j, j = 4 jj + r4 (block rows)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) xc[jj] = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = 4 * jj + r4;
        if (j < i) s = fmaf(Ab[i * LD64 + j], xc[jj], s);
      }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      const float xi = i < cb ? 0.f : (i == cb ? 1.f : -s);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        if (4 * jj + r4 == i) xc[jj] = xi;
    }
    // the full column of T: its block's rows from xc, zeros above; rows below follow.  T is
    // kept tf32-rounded: every later use is a tensor-core operand
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) Ti[(blk * 16 + 4 * jj + r4) * LD64 + c] = __uint_as_float(f2tf(xc[jj]));
    for (int rr = r4; rr < blk * 16; rr += 4) Ti[rr * LD64 + c] = 0.f;
  }
  __syncthreads();
#pragma unroll 1
  for (int dist = 1; dist < 4; ++dist) {
    const int items = 2 * (4 - dist);           // (block row I, 8-column half of block J)
    if (warp < items) {
      const int J = warp >> 1, I = J + dist, n0 = J * 16 + (warp & 1) * 8;
      float m[1][1][4] = {};
      for (int K = J; K < I; ++K)               // sum_K A_IK T_KJ
        warp_mma_mt<1, 1, false, 16, true, false>(m, Tm + K * 16, LD64, Ti + (K * 16) * LD64, LD64, I * 16, n0);
      // M into T_IJ's place (no other piece of this distance reads it), then T_IJ = -T_II M
#pragma unroll
      for (int e = 0; e < 4; ++e)
        Ti[(I * 16 + gq + (e >> 1) * 8) * LD64 + n0 + 2 * tq + (e & 1)] = __uint_as_float(f2tf(m[0][0][e]));
      __syncwarp();
      float tt[1][1][4] = {};
      warp_mma_mt<1, 1, false, 16, false, false>(tt, Ti + I * 16, LD64, Ti + (I * 16) * LD64, LD64, I * 16, n0);
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 4; ++e)
        Ti[(I * 16 + gq + (e >> 1) * 8) * LD64 + n0 + 2 * tq + (e & 1)] = __uint_as_float(f2tf(-tt[0][0][e]));
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  __syncthreads();
  // ---- k <- diag(beta Gam) k, v <- diag(beta) v (tf32-rounded: tensor-core operands)
  for (int i = tid; i < GC * GD; i += GDN_PREP_THREADS) {
    const int r = i / GD, c = i % GD;
    Kc[r * LD128 + c] = __uint_as_float(f2tf(Kc[r * LD128 + c] * (bet[r] * __expf(gam[r]))));
    QV[r * LD128 + c] = __uint_as_float(f2tf(QV[r * LD128 + c] * bet[r]));
  }
  __syncthreads();
  // ---- W = T diag(beta Gam) K -> ws_w, U0 = T diag(beta) V -> v (this CTA's rows only)
  const int om0 = (warp & 3) * 16, on0 = (warp >> 2) * 64;
#pragma unroll 1
  for (int part = 0; part < 2; ++part) {
    float acc[8][4] = {};
    warp_mma<8, false, false, false, false>(acc, Ti, LD64, part ? QV : Kc, LD128, om0, on0, GC);
    float* dst = part ? v : ws_w;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = om0 + gq + hh * 8, c = on0 + 8 * j + 2 * tq;
        float2 val = make_float2(acc[j][2 * hh], acc[j][2 * hh + 1]);
        if (!part) val = make_float2(__uint_as_float(f2tf(val.x)), __uint_as_float(f2tf(val.y)));   // W: tf32
        if (i < n) *reinterpret_cast<float2*>(dst + ((size_t)(c0 + i) * nv + h) * GD + c) = val;
      }
  }
}

// grid (B, nv, 128 / 32); block 512 (16 warps).  Walks sequence b's chunks for value head h
// and state columns [32 z, 32 z + 32); ssm fp32 [slots, nv, 128, 128]; out fp32 [T, nv, 128].
__global__ void __launch_bounds__(GDN_ST_THREADS, 1) gdn_chunk_state_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ u0,
    const float* __restrict__ ws_w, const float* __restrict__ ws_p, const float* __restrict__ ws_g,
    const int* __restrict__ q_start, const int* __restrict__ slots, const int* __restrict__ fresh,
    float* __restrict__ ssm, float* __restrict__ out, int nk, int nv) {
  extern __shared__ float gsm[];
  float* S = gsm;                       // [128][LDS]   state columns of this CTA (fp32)
  float* Sr = S + GD * LDS;             // [128][LDS]   the same, tf32-rounded (tensor-core operand)
  float* Wc = Sr + GD * LDS;            // [64][LD128]
  float* Qc = Wc + GC * LD128;          // [64][LD128]
  float* Kc = Qc + GC * LD128;          // [64][LDK]
  float* Pc = Kc + GC * LDK;            // [64][LD64]
  float* U0 = Pc + GC * LD64;           // [64][LDS]
  float* Uc = U0 + GC * LDS;            // [64][LDS]    U
  float* Ut = Uc + GC * LDS;            // [64][LDS]    diag(Gk) U
  float* O1 = Ut + GC * LDS;            // [64][LDS]    diag(Gam) Q S0
  float* gam = O1 + GC * LDS;           // [64]
  const int b = blockIdx.x, h = blockIdx.y, z = blockIdx.z;
  const int t0 = q_start[b], t1 = q_start[b + 1];
  if (t1 <= t0) return;
  const int kh = h / (nv / nk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int slot = slots[b];
  const bool is_fresh = slot < 0 || (fresh != nullptr && fresh[b] != 0);
  float* S_g = slot < 0 ? nullptr : ssm + ((size_t)slot * nv + h) * GD * GD;
  for (int i = tid; i < GD * SC; i += GDN_ST_THREADS) {
    const int r = i / SC, c = i % SC;
    const float v0 = is_fresh ? 0.f : S_g[(size_t)r * GD + z * SC + c];
    S[r * LDS + c] = v0;
    Sr[r * LDS + c] = __uint_as_float(f2tf(v0));
  }
  // operands of chunk c0: group 1 = W, Q, U0 slice, gamma (products with S0, U);
  // group 2 = K, P (output and state update)
  auto load1 = [&](int c0) {
    if (c0 < t1) {
      const int n = min(GC, t1 - c0);
      for (int i = tid; i < GC * (GD / 4); i += GDN_ST_THREADS) {
        const int r = i / (GD / 4), c4 = (i % (GD / 4)) * 4;
        const size_t tok = c0 + min(r, n - 1);
        const int sz = r < n ? 16 : 0;
        cp_async16(Wc + r * LD128 + c4, ws_w + (tok * nv + h) * GD + c4, sz);
        cp_async16(Qc + r * LD128 + c4, q + (tok * nk + kh) * GD + c4, sz);
      }
      for (int i = tid; i < GC * (SC / 4); i += GDN_ST_THREADS) {
        const int r = i / (SC / 4), c4 = (i % (SC / 4)) * 4;
        const size_t tok = c0 + min(r, n - 1);
        cp_async16(U0 + r * LDS + c4, u0 + (tok * nv + h) * GD + z * SC + c4, r < n ? 16 : 0);
      }
      if (tid < GC) cp_async4(gam + tid, ws_g + (size_t)(c0 + min(tid, n - 1)) * nv + h, tid < n ? 4 : 0);
    }
    cp_async_commit();                  // an empty group past the last chunk keeps the count
  };
  auto load2 = [&](int c0) {
    if (c0 < t1) {
      const int n = min(GC, t1 - c0);
      for (int i = tid; i < GC * (GD / 4); i += GDN_ST_THREADS) {
        const int r = i / (GD / 4), c4 = (i % (GD / 4)) * 4;
        const size_t tok = c0 + min(r, n - 1);
        cp_async16(Kc + r * LDK + c4, k + (tok * nk + kh) * GD + c4, r < n ? 16 : 0);
      }
      for (int i = tid; i < GC * (GC / 4); i += GDN_ST_THREADS) {
        const int r = i / (GC / 4), c4 = (i % (GC / 4)) * 4;
        const size_t tok = c0 + min(r, n - 1);
        cp_async16(Pc + r * LD64 + c4, ws_p + (tok * nv + h) * GC + c4, r < n ? 16 : 0);
      }
    }
    cp_async_commit();
  };
  load1(t0);
  load2(t0);
  for (int c0 = t0; c0 < t1; c0 += GC) {
    const int n = min(GC, t1 - c0);
    cp_async_wait<1>();                 // group 1 of this chunk
    __syncthreads();
    // ---- X = [W; Q] S0: warp w owns rows 16 (w & 7) .. + 15 (W for (w & 7) < 4, Q after),
    // columns 16 (w >> 3) .. + 15
    float gl;
    {
      float x[1][2][4] = {};
      const int mw = warp & 7, n0 = (warp >> 3) * 16;
      const float* A = mw < 4 ? Wc : Qc;
      const int m0 = (mw & 3) * 16;
      warp_mma_mt<1, 2, false, GD, false, false>(x, A, LD128, Sr, LDS, m0, n0);
      const float glast = gam[n - 1];
      gl = __expf(glast);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = m0 + gq + hh * 8, c = n0 + 8 * j + 2 * tq;
          if (mw < 4) {
            const float gk = i < n ? __expf(glast - gam[i]) : 0.f;
            const float ua = U0[i * LDS + c] - x[0][j][2 * hh], ub = U0[i * LDS + c + 1] - x[0][j][2 * hh + 1];
            *reinterpret_cast<float2*>(Uc + i * LDS + c) =
                make_float2(__uint_as_float(f2tf(ua)), __uint_as_float(f2tf(ub)));
            *reinterpret_cast<float2*>(Ut + i * LDS + c) =
                make_float2(__uint_as_float(f2tf(gk * ua)), __uint_as_float(f2tf(gk * ub)));
          } else {
            const float gm = __expf(gam[i]);
            *reinterpret_cast<float2*>(O1 + i * LDS + c) = make_float2(gm * x[0][j][2 * hh], gm * x[0][j][2 * hh + 1]);
          }
        }
    }
    __syncthreads();                    // W, Q, U0, gamma consumed
    load1(c0 + GC);
    cp_async_wait<1>();                 // group 2 of this chunk
    __syncthreads();
    // ---- O = O1 + P U: warp w owns output rows 16 (w & 3) .. + 15, columns 8 (w >> 2) .. + 7
    {
      float o[1][1][4];
      const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 8;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[0][0][e] = O1[(m0 + gq + (e >> 1) * 8) * LDS + n0 + 2 * tq + (e & 1)];
      warp_mma_mt<1, 1, false, GC, false, false>(o, Pc, LD64, Uc, LDS, m0, n0);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = m0 + gq + hh * 8, c = n0 + 2 * tq;
        if (i < n)
          *reinterpret_cast<float2*>(out + ((size_t)(c0 + i) * nv + h) * GD + z * SC + c) =
              make_float2(o[0][0][2 * hh], o[0][0][2 * hh + 1]);
      }
    }
    // ---- S <- Gam_C S0 + K^T diag(Gk) U: warp w owns state rows 16 (w & 7) .. + 15,
    // columns 16 (w >> 3) .. + 15
    {
      float s[1][2][4];
      const int m0 = (warp & 7) * 16, n0 = (warp >> 3) * 16;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          s[0][j][e] = gl * S[(m0 + gq + (e >> 1) * 8) * LDS + n0 + 8 * j + 2 * tq + (e & 1)];
      warp_mma_mt<1, 2, true, GC, false, false>(s, Kc, LDK, Ut, LDS, m0, n0);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = m0 + gq + hh * 8, c = n0 + 8 * j + 2 * tq;
          *reinterpret_cast<float2*>(S + i * LDS + c) = make_float2(s[0][j][2 * hh], s[0][j][2 * hh + 1]);
          *reinterpret_cast<float2*>(Sr + i * LDS + c) =
              make_float2(__uint_as_float(f2tf(s[0][j][2 * hh])), __uint_as_float(f2tf(s[0][j][2 * hh + 1])));
        }
    }
    __syncthreads();                    // K, P, U, O1 consumed; S complete
    load2(c0 + GC);
  }
  cp_async_wait<0>();
  if (S_g == nullptr) return;
  for (int i = tid; i < GD * SC; i += GDN_ST_THREADS) {
    const int r = i / SC, c = i % SC;
    S_g[(size_t)r * GD + z * SC + c] = S[r * LDS + c];
  }
}

}  // namespace xtu

using namespace xtu;

extern "C" {

// qkvz: in_proj output [T, qkvz_stride] bf16; conv_w fp32 [ch, kw]; conv_state bf16 [slots, ch, kw-1];
// ssm fp32 [slots, nv, dk, dv] (a sequence whose slot is < 0 is computed from a zero state and
// leaves every state untouched); g fp32 [T, nv] (g_channels = 0) or [T, nv, dk] (channel-wise
// decay, g_channels = 1); beta fp32 [T, nv]; blocked: qkvz rows are [Q | K | V] (else per key
// head [q | k | v | z]); scratch q/k fp32 [T, nk, dk], v fp32 [T, nv, dv]; out fp32 [T, nv, dv];
// chunked: the scalar-decay rule in chunks of 64 tokens on the tensor cores (dk = dv = 128;
// prefill), with chunk_ws fp32 scratch of T * nv * (128 + 64 + 1) floats (vs is overwritten).
// ba != nullptr (scalar decay): g and beta are outputs, computed by the conv kernel from the
// in_proj_ba rows [T, ba_stride] bf16 (per key head [b r | a r]) with A_log, dt_bias fp32 [nv].
// y != nullptr: y bf16 [T, nv*dv] <- gated RMSNorm of out with weight norm_w fp32 [dv]; the
// gate is silu(z) of the qkvz rows (gate_mode 0; gate = qkvz) or sigmoid of a bf16
// [T, gate_stride] tensor (gate_mode 1).
// spec_ssm / spec_conv (speculative verification, at most spec_n tokens per sequence): the
// recurrent and conv states after every token of the step, [slots, spec_n, ...] each (the
// final states are written to ssm / conv_state as usual); xtu_deltanet_spec_commit then
// installs the ones of each sequence's accepted position.
// Returns kernels launched or a negative error.
int xtu_deltanet_fwd(const void* qkvz, int qkvz_stride, int T, int B, const int* q_start, const int* slots,
                     const int* fresh, int nk, int nv, int dk, int dv, int kw, const float* conv_w, void* conv_state,
                     float* ssm, float* g, float* beta, float* qs, float* ks, float* vs, float* out,
                     int blocked, int g_channels, int chunked, float* chunk_ws, const void* ba, int ba_stride,
                     const float* A_log, const float* dt_bias, const void* gate, int gate_stride, int gate_mode,
                     const float* norm_w, float eps, void* y, float* spec_ssm, void* spec_conv, int spec_n,
                     cudaStream_t stream) {
  if (T <= 0 || B <= 0) return 0;
  if (dk != 128 || dv % GDN_COLS != 0 || dv > 256 || kw < 2 || kw > 9 || nv % nk != 0) return -2;
  if (ba != nullptr && (g_channels || blocked || A_log == nullptr || dt_bias == nullptr)) return -2;
  if (y != nullptr && (norm_w == nullptr || gate == nullptr || (gate_mode == 0 && blocked))) return -2;
  GdnShape s{nk, nv, dk, dv, kw, qkvz_stride, blocked ? 1 : 0};
  const int ch = 2 * nk * dk + nv * dv;
  GdnGates gt{(const __nv_bfloat16*)ba, ba_stride, A_log, dt_bias, g, beta};
  int launched = 2;
  // speculative verification steps keep per-token states: token-serial kernel only
  const bool use_chunks = chunked && chunk_ws != nullptr && !g_channels && dv == GD && spec_ssm == nullptr;
  const int tok_per_cta = GDN_CONV_WARPS * GDN_CONV_TPW;
  const dim3 cgrid((T + tok_per_cta - 1) / tok_per_cta, 2 * nk + nv);
#define XTU_GDN_CONV(KWV)                                                                                        \
  if (dv <= 128)                                                                                                 \
    gdn_conv_kernel<KWV, 4><<<cgrid, GDN_CONV_WARPS * 32, 0, stream>>>(                                           \
        (const __nv_bfloat16*)qkvz, s, conv_w, (const __nv_bfloat16*)conv_state, q_start, slots, fresh, B, T, qs,   \
        ks, vs, gt, use_chunks);                                                                                 \
  else                                                                                                           \
    gdn_conv_kernel<KWV, 8><<<cgrid, GDN_CONV_WARPS * 32, 0, stream>>>(                                           \
        (const __nv_bfloat16*)qkvz, s, conv_w, (const __nv_bfloat16*)conv_state, q_start, slots, fresh, B, T, qs,   \
        ks, vs, gt, use_chunks)
  switch (kw) {
    case 2: XTU_GDN_CONV(2); break;
    case 3: XTU_GDN_CONV(3); break;
    case 4: XTU_GDN_CONV(4); break;
    case 5: XTU_GDN_CONV(5); break;
    case 6: XTU_GDN_CONV(6); break;
    case 7: XTU_GDN_CONV(7); break;
    case 8: XTU_GDN_CONV(8); break;
    default: XTU_GDN_CONV(9); break;
  }
#undef XTU_GDN_CONV
  gdn_conv_state_kernel<<<dim3(B, (ch + 255) / 256), 256, 0, stream>>>(
      (const __nv_bfloat16*)qkvz, s, (__nv_bfloat16*)conv_state, q_start, slots, fresh,
      (__nv_bfloat16*)spec_conv, spec_n);
  if (use_chunks) {
    cudaError_t ea = cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          GDN_PREP_SMEM);
    if (ea == cudaSuccess)
      ea = cudaFuncSetAttribute(gdn_chunk_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_ST_SMEM);
    if (ea != cudaSuccess) return -(int)ea;
    float* ws_w = chunk_ws;
    float* ws_p = ws_w + (size_t)T * nv * GD;
    float* ws_g = ws_p + (size_t)T * nv * GC;
    gdn_chunk_prep_kernel<<<dim3((T + GC - 1) / GC + B, nv), GDN_PREP_THREADS, GDN_PREP_SMEM, stream>>>(
        qs, ks, vs, g, beta, q_start, B, ws_w, ws_p, ws_g, nk, nv);
    gdn_chunk_state_kernel<<<dim3(B, nv, GD / SC), GDN_ST_THREADS, GDN_ST_SMEM, stream>>>(
        qs, ks, vs, ws_w, ws_p, ws_g, q_start, slots, fresh, ssm, out, nk, nv);
    launched += 2;
  } else if (g_channels) {
    gdn_recurrent_kernel<128, true><<<dim3(B, nv, dv / GDN_COLS), 128, 0, stream>>>(
        qs, ks, vs, g, beta, q_start, slots, fresh, ssm, out, nk, nv, dv, spec_ssm, spec_n);
    launched += 1;
  } else {
    gdn_recurrent_kernel<128, false><<<dim3(B, nv, dv / GDN_COLS), 128, 0, stream>>>(
        qs, ks, vs, g, beta, q_start, slots, fresh, ssm, out, nk, nv, dv, spec_ssm, spec_n);
    launched += 1;
  }
  if (y != nullptr) {
    gdn_gated_norm_kernel<<<(T * nv + 7) / 8, 256, 0, stream>>>(out, (const __nv_bfloat16*)gate, gate_stride,
                                                                 gate_mode, s, norm_w, eps, (__nv_bfloat16*)y, T);
    launched += 1;
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? launched : -(int)e;
}

// acc [B]: the accepted position of each sequence (0 .. spec_n - 1); slots [B] (< 0 skipped);
// ssm fp32 [slots, ssm_elems], conv bf16 [slots, conv_elems] <- their spec_n-way copies.
int xtu_deltanet_spec_commit(const int* acc, const int* slots, int B, int spec_n, const float* spec_ssm, float* ssm,
                             long long ssm_elems, const void* spec_conv, void* conv, long long conv_elems,
                             cudaStream_t stream) {
  if (B <= 0) return 0;
  if (ssm_elems % 4 != 0) return -2;
  gdn_spec_commit_kernel<<<dim3(B, 64), 256, 0, stream>>>(acc, slots, spec_n, (const float4*)spec_ssm, (float4*)ssm,
                                                          ssm_elems / 4, (const __nv_bfloat16*)spec_conv,
                                                          (__nv_bfloat16*)conv, conv_elems);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

}  // extern "C"
