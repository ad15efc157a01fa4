// GQA decode attention for sm_100a: KV-bandwidth bound, so built to keep HBM busy.
//
// A decode step has 1 (or, with speculative tokens, a few) query positions per
// sequence, so the G = Hq / Hkv heads that share a KV head give 12..32 query rows per
// (sequence, kv head).  One CTA = one (kv split, kv head, sequence):
//   warp 0     producer: the split's page ids (read 32 at a time by the whole warp),
//              then one elected thread streams each 64-key page of K and V through a
//              3-deep shared-memory ring with TMA (128-byte swizzled 64 x 64 boxes).
//   warps 1-4  consumers: warp w takes m-tile (w % MT) of 16 query rows and key
//              subset (w / MT) of every page (16 keys when MT = 1, 32 when MT = 2):
//                S = Q K^T      mma.sync m16n8k16 bf16, Q in registers, K by ldmatrix
//                online softmax in the exp2 domain (quad shuffles for the row max),
//                O += P V       P re-used from the S registers as the A fragment,
//                               V by ldmatrix.trans
//              The running max only moves when it grows by more than 2^8, so O is
//              rescaled rarely.  At the end the key subsets meet in shared memory and
//              the CTA writes bf16 O (one split) or a normalised partial + log-sum-exp;
//              with split-KV the last CTA of a (sequence, kv head) to finish (counter)
//              merges the splits, so no separate combine kernel runs.
// Why not tcgen05 here: its smallest tile is 64 rows, so 12 real rows would carry 5x
// padded softmax work, and softmax (not the tensor pipe) is what limits a decode CTA;
// the warp-level MMA shape matches the GQA group.  The split count is chosen so that
// two CTAs per SM cover the GPU (the ring is 96 KB), which keeps about 190 KB of KV
// in flight per SM.
// Serves the role of the FlashAttention decode path the reference takes from vLLM for
// non-MoE attention (the reference has no kernel of its own for GQA decode).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cfloat>
#include "ptx.cuh"
#include "launch.cuh"

namespace xtu {
namespace {

constexpr int AD_CWARPS = 4;
constexpr int AD_THREADS = 32 * (1 + AD_CWARPS);
constexpr int AD_KEYS = 64;   // keys per paged-cache block

template <int D>
struct AdCfg {
  static constexpr int BOXES = D / 64;                        // 64-wide (128-byte) column boxes
  static constexpr int KV_BYTES = AD_KEYS * D * 2;            // K (or V) of one page
  static constexpr int STAGE_BYTES = 2 * KV_BYTES;
  static constexpr int STAGES = D <= 64 ? 6 : 3;
  static constexpr int BYTES = 1024 + STAGES * STAGE_BYTES + 2 * STAGES * 8 + 64;
  // the end-of-CTA merge reuses the ring: O, m, l of the 4 consumer warps
  static_assert(AD_CWARPS * 16 * (D + 2) * 4 <= STAGES * STAGE_BYTES, "merge buffer");
};

struct AdParams {
  const __nv_bfloat16* q;   // [T, Hq, D], token stride q_stride
  int q_stride;
  __nv_bfloat16* o;         // [T, Hq, D], token stride o_stride
  int o_stride;
  const int* q_start;       // [B+1]
  const int* kv_len;        // [B]
  const int* block_table;   // [B, bt_stride]
  int bt_stride;
  int Hq, Hkv, G;
  float scale_log2;         // softmax scale * log2(e)
  int splits;
  float* ws_o;              // [splits, T, Hq, D] normalised partials (splits > 1)
  float* ws_lse;            // [splits, T, Hq]  m + log2(l)
  int* counters;            // [B * Hkv] zeroed; the last split CTA merges and re-zeroes
  int num_blocks;           // pages in the cache (bounds-check build)
  int T;
  int window;               // > 0: a query at position t sees keys (t - window, t] only
  const float* sinks;       // [Hq] learned sink logits (softmax scale applied), or null
  XtuStatus* status;
};

__device__ __forceinline__ void ad_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ float ad_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// shared-memory address of 16-byte chunk `ch` (8 values of d) of key row `r` in a
// K or V page laid out by TMA as BOXES boxes of [64 keys][128 bytes], 128B-swizzled
__device__ __forceinline__ uint32_t ad_chunk(uint32_t base, int r, int ch) {
  return base + (ch >> 3) * 8192 + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
}


template <int D, int MT>
__global__ void __launch_bounds__(AD_THREADS) attn_decode_kernel(const __grid_constant__ CUtensorMap tk,
                                                                 const __grid_constant__ CUtensorMap tv,
                                                                 const __grid_constant__ AdParams p) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  using C = AdCfg<D>;
  constexpr int STAGES = C::STAGES;
  constexpr int NS = AD_CWARPS / MT;   // key subsets per page
  constexpr int KW = AD_KEYS / NS;     // keys per consumer warp per page
  constexpr int NKT = KW / 8;          // 8-key n-tiles of S per warp
  constexpr int DK = D / 16;           // k-steps of Q K^T
  constexpr int DN = D / 8;            // 8-column n-tiles of O
  extern __shared__ uint8_t ad_smem_raw[];
  const uint32_t sa = smem_u32(ad_smem_raw);
  uint8_t* stages = ad_smem_raw + (((sa + 1023u) & ~1023u) - sa);
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], AD_CWARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const int sp = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int L = __ldg(p.kv_len + b);
  const int q0 = __ldg(p.q_start + b), ql = __ldg(p.q_start + b + 1) - q0;
  const int nrows = ql * p.G;
  const int nblk = (L + AD_KEYS - 1) / AD_KEYS;
  // sliding window: no query of this sequence sees a key below L - ql - window + 1
  const int jfirst = p.window > 0 ? max(0, L - ql - p.window + 1) / AD_KEYS : 0;
  const int per = (nblk - jfirst + p.splits - 1) / p.splits;
  const int j0 = min(nblk, jfirst + sp * per), j1 = min(nblk, j0 + per);
  const int nj = j1 - j0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    // ---------------- producer
    if (lane == 0) {
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
    }
    bool ok = true;
    int issued = 0;
    const int* bt = p.block_table + (size_t)b * p.bt_stride + j0;
    for (int c0 = 0; c0 < nj && ok; c0 += 32) {
      const int page = c0 + lane < nj ? __ldg(bt + c0 + lane) : 0;
      const int cnt = min(32, nj - c0);
      for (int k = 0; k < cnt; ++k) {
        const int pg = __shfl_sync(0xffffffffu, page, k);
        // a page id past the cache reads zero fill (TMA bounds); the bounds-check build reports it
        if (lane == 0) (void)XTU_IN_BOUNDS(pg >= 0 && pg < p.num_blocks, p.status, 230, pg);
        if (lane == 0) {
          const int i = c0 + k, slot = i % STAGES;
          if (i >= STAGES && !mbar_wait(&empty[slot], ((i / STAGES) - 1) & 1, p.status, 130)) {
            ok = false;
          } else {
            ++issued;
            mbar_arrive_expect_tx(&full[slot], C::STAGE_BYTES);
            uint8_t* dst = stages + slot * C::STAGE_BYTES;
            const int row = (pg * p.Hkv + kh) * AD_KEYS;
#pragma unroll
            for (int bx = 0; bx < C::BOXES; ++bx) tma_load_2d(dst + bx * 8192, &tk, &full[slot], bx * 64, row);
#pragma unroll
            for (int bx = 0; bx < C::BOXES; ++bx)
              tma_load_2d(dst + C::KV_BYTES + bx * 8192, &tv, &full[slot], bx * 64, row);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
    }
    if (!ok && lane == 0) {   // let the copies in flight land (bounded) before the CTA exits
      for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr, 0, 50000000ull);
    }
    return;
  }
  // ---------------- consumers
  const int cw = warp - 1;
  const int mt = cw % MT, ks = cw / MT;
  const int g4 = lane >> 2, tq = lane & 3;
  // this lane's two query rows (r and r + 8 of the m-tile): Q fragments and causal limit
  uint32_t qa[DK][4];
  int lim[2], low[2];
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    const int r = mt * 16 + g4 + h2 * 8;
    const bool valid = r < nrows;
    const int qi = valid ? r / p.G : 0, hh = valid ? r - (r / p.G) * p.G : 0;
    lim[h2] = valid ? L - ql + qi : L - 1;
    low[h2] = p.window > 0 ? lim[h2] - p.window + 1 : 0;
    const __nv_bfloat16* qrow = p.q + (size_t)(q0 + qi) * p.q_stride + (size_t)(kh * p.G + hh) * D;
#pragma unroll
    for (int k = 0; k < DK; ++k) {
      const uint32_t lo = valid ? __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * k + 2 * tq)) : 0u;
      const uint32_t hi = valid ? __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * k + 8 + 2 * tq)) : 0u;
      qa[k][h2] = lo;        // a0 / a1: rows g4 / g4+8, k 2tq..2tq+1
      qa[k][2 + h2] = hi;    // a2 / a3: same rows, k 8+2tq..
    }
  }
  float o[DN][4];
#pragma unroll
  for (int n = 0; n < DN; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  bool ok = true;
  for (int i = 0; i < nj; ++i) {
    const int slot = i % STAGES;
    if (!mbar_wait(&full[slot], (i / STAGES) & 1, p.status, 131)) {
      ok = false;
      break;
    }
    const uint32_t kbase_s = smem_u32(stages + slot * C::STAGE_BYTES);
    const uint32_t vbase_s = kbase_s + C::KV_BYTES;
    const int key_lo = ks * KW;                       // first key of this warp within the page
    const int kabs = (j0 + i) * AD_KEYS + key_lo;      // its absolute index
    // ---- S = Q K^T over this warp's KW keys
    float s[NKT][4];
#pragma unroll
    for (int nt = 0; nt < NKT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
      const int r = key_lo + nt * 8 + (lane & 7);
#pragma unroll
      for (int kc = 0; kc < DK / 2; ++kc) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(ad_chunk(kbase_s, r, kc * 4 + (lane >> 3)), b0, b1, b2, b3);
        ad_mma(s[nt], qa[2 * kc], b0, b1);
        ad_mma(s[nt], qa[2 * kc + 1], b2, b3);
      }
    }
    // ---- scale, mask, online softmax (rows h2 = 0: g4, 1: g4 + 8)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < NKT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kabs + nt * 8 + 2 * tq + (e & 1);
        const float v = (key <= lim[e >> 1] && key >= low[e >> 1]) ? s[nt][e] * p.scale_log2 : -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    bool need = false;
    float mnew[2];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      mx[h2] = fmaxf(mx[h2], __shfl_xor_sync(0xffffffffu, mx[h2], 1));
      mx[h2] = fmaxf(mx[h2], __shfl_xor_sync(0xffffffffu, mx[h2], 2));
      mnew[h2] = fmaxf(m[h2], mx[h2]);
      need |= mnew[h2] > m[h2] + 8.f;
    }
    if (__any_sync(0xffffffffu, need)) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const bool up = mnew[h2] > m[h2] + 8.f;
        const float f = up ? ad_ex2(m[h2] - mnew[h2]) : 1.f;
        if (up) m[h2] = mnew[h2];
        l[h2] *= f;
#pragma unroll
        for (int n = 0; n < DN; ++n) {
          o[n][2 * h2] *= f;
          o[n][2 * h2 + 1] *= f;
        }
      }
    }
    const float mb[2] = {m[0] == -INFINITY ? 0.f : m[0], m[1] == -INFINITY ? 0.f : m[1]};
    uint32_t pa[NKT / 2][4];
#pragma unroll
    for (int nt = 0; nt < NKT; ++nt) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pv[e] = ad_ex2(s[nt][e] - mb[e >> 1]);
        l[e >> 1] += pv[e];
      }
      pa[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16x2(pv[0], pv[1]);
      pa[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16x2(pv[2], pv[3]);
    }
    // ---- O += P V
#pragma unroll
    for (int kk = 0; kk < NKT / 2; ++kk) {
      const int r = key_lo + kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int dn2 = 0; dn2 < DN / 2; ++dn2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(ad_chunk(vbase_s, r, 2 * dn2 + (lane >> 4)), b0, b1, b2, b3);
        ad_mma(o[2 * dn2], pa[kk], b0, b1);
        ad_mma(o[2 * dn2 + 1], pa[kk], b2, b3);
      }
    }
    // generic-proxy reads of the slot are ordered before the TMA that refills it
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  // ---- merge the key subsets of each m-tile (the ring is idle: every load has landed)
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    l[h2] += __shfl_xor_sync(0xffffffffu, l[h2], 1);
    l[h2] += __shfl_xor_sync(0xffffffffu, l[h2], 2);
  }
  asm volatile("bar.sync 1, %0;" ::"n"(32 * AD_CWARPS) : "memory");   // all warps done with the ring
  float* co = reinterpret_cast<float*>(stages);                       // [4 warps][16 rows][D]
  float* cm = co + AD_CWARPS * 16 * D;                                 // [4][16]
  float* cl = cm + AD_CWARPS * 16;                                     // [4][16]
  {
    float* mine = co + cw * 16 * D;
#pragma unroll
    for (int n = 0; n < DN; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) mine[(g4 + (e >> 1) * 8) * D + n * 8 + 2 * tq + (e & 1)] = o[n][e];
    if (tq == 0) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        cm[cw * 16 + g4 + h2 * 8] = ok ? m[h2] : -INFINITY;
        cl[cw * 16 + g4 + h2 * 8] = ok ? l[h2] : 0.f;
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(32 * AD_CWARPS) : "memory");
  const int tid = threadIdx.x - 32;
  constexpr int C4 = D / 4;
  for (int idx = tid; idx < nrows * C4; idx += 32 * AD_CWARPS) {
    const int r = idx / C4, c = (idx - r * C4) * 4;
    const int rm = r >> 4, rr = r & 15;
    float M = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < NS; ++s2) M = fmaxf(M, cm[(s2 * MT + rm) * 16 + rr]);
    float Ls = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s2 = 0; s2 < NS; ++s2) {
      const int w = s2 * MT + rm;
      const float ms = cm[w * 16 + rr];
      const float wgt = ms == -INFINITY ? 0.f : ad_ex2(ms - M);
      Ls += wgt * cl[w * 16 + rr];
      const float4 v = *reinterpret_cast<const float4*>(co + (w * 16 + rr) * D + c);
      acc[0] += wgt * v.x;
      acc[1] += wgt * v.y;
      acc[2] += wgt * v.z;
      acc[3] += wgt * v.w;
    }
    const int qi = r / p.G, hh = r - qi * p.G;
    const int tok = q0 + qi, head = kh * p.G + hh;
    // the sink joins the softmax denominator only (once: here, or in the split merge)
    if (p.sinks != nullptr && p.splits == 1 && M != -INFINITY)
      Ls += ad_ex2(__ldg(p.sinks + head) * 1.4426950408889634f - M);
    const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
    if (p.splits == 1) {
      uint2 pk;
      pk.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
      pk.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
      *reinterpret_cast<uint2*>(p.o + (size_t)tok * p.o_stride + (size_t)head * D + c) = pk;
    } else {
      __stcg(reinterpret_cast<float4*>(p.ws_o + (((size_t)sp * p.T + tok) * p.Hq + head) * D + c),
             make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv));
      if (c == 0)
        __stcg(p.ws_lse + ((size_t)sp * p.T + tok) * p.Hq + head, Ls > 0.f ? M + __log2f(Ls) : -FLT_MAX);
    }
  }
  if (p.splits == 1) return;
  // ---- split-KV: the CTA that finishes last for this (sequence, kv head) merges every
  // split's normalised partial by its log-sum-exp (split order, so the bits do not depend
  // on which CTA came last), writes bf16 O and re-zeroes the counter
  __shared__ int s_last;
  __threadfence();
  asm volatile("bar.sync 1, %0;" ::"n"(32 * AD_CWARPS) : "memory");
  if (tid == 0) s_last = atomicAdd(p.counters + b * p.Hkv + kh, 1) == p.splits - 1;
  asm volatile("bar.sync 1, %0;" ::"n"(32 * AD_CWARPS) : "memory");
  if (!s_last) return;
  __threadfence();
  // merge weights per (row, split) once, in shared memory (the ring is free again):
  // w = exp2(lse - max lse) / sum, all loads of a pass issued together
  float* wsm = reinterpret_cast<float*>(stages);            // [32 rows][64 splits]
  for (int i = tid; i < nrows * p.splits; i += 32 * AD_CWARPS) {
    const int r = i / p.splits, s2 = i - r * p.splits;
    const int qi = r / p.G, hh = r - qi * p.G;
    wsm[r * 64 + s2] = __ldcg(p.ws_lse + ((size_t)s2 * p.T + q0 + qi) * p.Hq + kh * p.G + hh);
  }
  asm volatile("bar.sync 1, %0;" ::"n"(32 * AD_CWARPS) : "memory");
  if (tid < nrows) {
    const int hh = tid - (tid / p.G) * p.G;
    const float sk = p.sinks != nullptr ? __ldg(p.sinks + kh * p.G + hh) * 1.4426950408889634f : -FLT_MAX;
    float M = sk;
    for (int s2 = 0; s2 < p.splits; ++s2) M = fmaxf(M, wsm[tid * 64 + s2]);
    float sum = sk == -FLT_MAX ? 0.f : ad_ex2(sk - M);
    for (int s2 = 0; s2 < p.splits; ++s2) {
      const float ls = wsm[tid * 64 + s2];
      const float w = ls == -FLT_MAX ? 0.f : ad_ex2(ls - M);
      wsm[tid * 64 + s2] = w;
      sum += w;
    }
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    for (int s2 = 0; s2 < p.splits; ++s2) wsm[tid * 64 + s2] *= inv;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(32 * AD_CWARPS) : "memory");
  for (int idx = tid; idx < nrows * C4; idx += 32 * AD_CWARPS) {
    const int r = idx / C4, c = (idx - r * C4) * 4;
    const int qi = r / p.G, hh = r - qi * p.G;
    const int tok = q0 + qi, head = kh * p.G + hh;
    const float* src = p.ws_o + ((size_t)tok * p.Hq + head) * D + c;
    const size_t sstride = (size_t)p.T * p.Hq * D;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < p.splits; s0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[u] = s0 + u < p.splits ? __ldcg(reinterpret_cast<const float4*>(src + (s0 + u) * sstride))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float w = s0 + u < p.splits ? wsm[r * 64 + s0 + u] : 0.f;
        acc[0] += w * v[u].x;
        acc[1] += w * v[u].y;
        acc[2] += w * v[u].z;
        acc[3] += w * v[u].w;
      }
    }
    const float inv = 1.f;
    uint2 pk;
    pk.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
    pk.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<uint2*>(p.o + (size_t)tok * p.o_stride + (size_t)head * D + c) = pk;
  }
  if (tid == 0) p.counters[b * p.Hkv + kh] = 0;
}

}  // namespace

template <int D, int MT>
static int ad_launch(const CUtensorMap& tk, const CUtensorMap& tv, const AdParams& p, int B, cudaStream_t s) {
  using C = AdCfg<D>;
  static bool init = false;
  if (!init) {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<D, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::BYTES);
    if (e != cudaSuccess) return -(int)e;
    init = true;
  }
  launch_pdl(attn_decode_kernel<D, MT>, dim3(p.splits, p.Hkv, B), dim3(AD_THREADS), C::BYTES, s, tk, tv, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// Decode attention for GQA caches with D == DV in {64, 128} and at most 32 query rows
// (query positions x G) per (sequence, kv head).  Returns 1 on launch (the output is
// complete: split-KV partials are merged inside), 0 when the shape is not one this
// kernel serves (the caller then uses the general kernel), < 0 on error.
// counters: B * Hkv zeroed ints (needed when splits > 1), left zeroed.
// tk / tv: 2-D maps of the caches viewed as [blocks * Hkv * 64, D] with 64 x 64 boxes.
int attn_decode_gqa(const CUtensorMap& tk, const CUtensorMap& tv, const void* q, int q_stride, void* o,
                    int o_stride, const int* q_start, const int* kv_len, const int* block_table, int bt_stride,
                    int B, int max_q_len, int T, int Hq, int Hkv, int D, float scale, int splits, float* ws_o,
                    float* ws_lse, int* counters, int num_blocks, int window, const float* sinks, void* status,
                    cudaStream_t s) {
  const int G = Hq / Hkv;
  const int rows = max_q_len * G;
  if ((D != 64 && D != 128) || rows > 32 || rows <= 0) return 0;
  if (splits > 1 && counters == nullptr) return 0;
  if (splits > 64) return 0;
  AdParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.q_stride = q_stride;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.o_stride = o_stride;
  p.q_start = q_start;
  p.kv_len = kv_len;
  p.block_table = block_table;
  p.bt_stride = bt_stride;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = G;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.splits = splits < 1 ? 1 : splits;
  p.ws_o = ws_o;
  p.ws_lse = ws_lse;
  p.counters = counters;
  p.num_blocks = num_blocks;
  p.T = T;
  p.window = window;
  p.sinks = sinks;
  p.status = reinterpret_cast<XtuStatus*>(status);
  if (D == 128) return rows <= 16 ? ad_launch<128, 1>(tk, tv, p, B, s) : ad_launch<128, 2>(tk, tv, p, B, s);
  return rows <= 16 ? ad_launch<64, 1>(tk, tv, p, B, s) : ad_launch<64, 2>(tk, tv, p, B, s);
}

}  // namespace xtu
