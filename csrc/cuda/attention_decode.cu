// GQA decode attention for sm_100a: KV-bandwidth bound, so built to keep HBM busy.
//
// A decode step has 1 (or, with speculative tokens, a few) query positions per
// sequence, so the G = Hq / Hkv heads that share a KV head give 12..32 query rows per
// (sequence, kv head).  One CTA = one (kv split, kv head, sequence):
//   warp 0     producer: the split's page ids (read 32 at a time by the whole warp),
//              then one elected thread streams each 64-key page of K and V through a
//              3-deep shared-memory ring with TMA (128-byte swizzled 64 x 64 boxes).
//   warps 1-CW consumers (CW = 4; 8 when MT = 4): warp w takes m-tile (w % MT) of 16
//              query rows and key subset (w / MT) of every page (16 keys when MT = 1,
//              32 when MT = 2 or 4):
//                S = Q K^T      mma.sync m16n8k16 bf16, Q in registers, K by ldmatrix
//                online softmax in the exp2 domain (quad shuffles for the row max),
//                O += P V       P re-used from the S registers as the A fragment,
//                               V by ldmatrix.trans
//              The running max only moves when it grows by more than 2^8, so O is
//              rescaled rarely.  At the end the key subsets meet in shared memory and
//              the CTA writes bf16 O (one split) or a normalised partial + log-sum-exp;
//              with split-KV the last CTA of a (sequence, kv head) to finish (counter)
//              merges the splits, so no separate combine kernel runs.
// F8 (fp8 KV cache): K pages are e4m3 [64 keys][D] and V pages e4m3 transposed
// [D][64 keys], half the bytes of bf16 (twice the pages in the same ring).  The MMAs run
// in f16 (e4m3 converts to f16 exactly; Q is rounded to f16 once): a lane reads 4
// consecutive bytes of a K row or V^T row per k-step (one cvt.f16x2.e4m3x2 pair), and
// the contraction indices are permuted consistently on both sides -- d in Q K^T (Q is
// loaded in the same order) and the keys of each 16-key group in P V (S's n-positions
// are mapped onto the permuted keys when K rows are read and when keys are masked).
// The per-layer K scale is folded into the softmax scale and the V scale into the output.
// MT = 4 (up to 64 query rows: MTP verification steps of a GQA group of 12) runs eight
// consumer warps, one CTA per SM with a 192 KB ring: with four warps each carried one
// m-tile through all 64 keys of a page, and one warp per scheduler left every dependent
// MMA and exp exposed (measured 94 us for 4 x 15K-token sequences, 60 rows per KV head).
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
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include <cstdlib>
#include <cfloat>
#include "ptx.cuh"
#include "launch.cuh"

namespace xtu {
namespace {

constexpr int AD_KEYS = 64;   // keys per paged-cache block

// CW consumer warps: 4 (two CTAs per SM, 96 KB ring) or 8 (MT = 4: one CTA per SM, twice
// the ring, each m-tile's keys split between two warps so every scheduler runs two of them)
template <int D, bool F8 = false, int CW = 4>
struct AdCfg {
  static constexpr int BOXES = D / 64;                        // 64-wide (128-byte) column boxes (bf16)
  static constexpr int KV_BYTES = AD_KEYS * D * (F8 ? 1 : 2); // K (or V) of one page
  static constexpr int STAGE_BYTES = 2 * KV_BYTES;
  static constexpr int STAGES = (D <= 64 ? 6 : 3) * (F8 ? 2 : 1) * (CW == 8 ? 2 : 1);
  static constexpr int THREADS = 32 * (1 + CW);
  static constexpr int BYTES = 1024 + STAGES * STAGE_BYTES + 2 * STAGES * 8 + 64;
  // the end-of-CTA merge reuses the ring: O, m, l of the consumer warps
  static_assert(CW * 16 * (D + 2) * 4 <= STAGES * STAGE_BYTES, "merge buffer");
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
  float scale_log2;         // softmax scale * log2(e) (fp8: times the K scale)
  float out_scale;          // multiplies O (fp8: the V scale; else 1)
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

__device__ __forceinline__ void ad_mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// four e4m3 bytes -> two f16x2 (bytes 0,1 -> lo; bytes 2,3 -> hi), exact
__device__ __forceinline__ void e4m3x4_to_f16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// fp8 pages: byte offset of byte `b` of row `r` in a K page of D-byte rows (D = 128: 128B
// swizzle; D = 64: 64B swizzle) or a V^T page of 64-byte rows (64B swizzle)
template <int ROWB>
__device__ __forceinline__ uint32_t ad_f8_off(int r, int b) {
  if (ROWB == 128) return r * 128 + ((((b >> 4) ^ (r & 7)) << 4) | (b & 15));
  return r * 64 + ((((b >> 4) ^ ((r >> 1) & 3)) << 4) | (b & 15));
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


template <int D, int MT, bool F8, int CW>
__global__ void __launch_bounds__(32 * (1 + CW)) attn_decode_kernel(const __grid_constant__ CUtensorMap tk,
                                                                    const __grid_constant__ CUtensorMap tv,
                                                                    const __grid_constant__ AdParams p) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  using C = AdCfg<D, F8, CW>;
  constexpr int STAGES = C::STAGES;
  constexpr int AD_CWARPS = CW;
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
            if constexpr (F8) {   // K [64 keys][D bytes]; V^T [D rows][64 bytes]
              tma_load_2d(dst, &tk, &full[slot], 0, row);
              tma_load_2d(dst + C::KV_BYTES, &tv, &full[slot], 0, (pg * p.Hkv + kh) * D);
            } else {
#pragma unroll
              for (int bx = 0; bx < C::BOXES; ++bx) tma_load_2d(dst + bx * 8192, &tk, &full[slot], bx * 64, row);
#pragma unroll
              for (int bx = 0; bx < C::BOXES; ++bx)
                tma_load_2d(dst + C::KV_BYTES + bx * 8192, &tv, &full[slot], bx * 64, row);
            }
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
    if constexpr (F8) {
      // k-step s of lane tq covers d = tq * D/4 + 4 s + {0,1 | 2,3} (the order the K bytes are read in)
#pragma unroll
      for (int k = 0; k < DK; ++k) {
        const uint2 v = valid ? __ldg(reinterpret_cast<const uint2*>(qrow + tq * (D / 4) + 4 * k)) : make_uint2(0u, 0u);
        qa[k][h2] = pack_f16x2(bf16_lo(v.x), bf16_hi(v.x));
        qa[k][2 + h2] = pack_f16x2(bf16_lo(v.y), bf16_hi(v.y));
      }
    } else {
#pragma unroll
      for (int k = 0; k < DK; ++k) {
        const uint32_t lo = valid ? __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * k + 2 * tq)) : 0u;
        const uint32_t hi = valid ? __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * k + 8 + 2 * tq)) : 0u;
        qa[k][h2] = lo;        // a0 / a1: rows g4 / g4+8, k 2tq..2tq+1
        qa[k][2 + h2] = hi;    // a2 / a3: same rows, k 8+2tq..
      }
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
      if constexpr (F8) {
        // n-position g4 of tile nt is key 16 (nt/2) + 4 (g4/2) + 2 (nt%2) + g4%2 of the warp's keys
        const int r = key_lo + 16 * (nt >> 1) + 4 * (g4 >> 1) + 2 * (nt & 1) + (g4 & 1);
        uint32_t w[D / 16];
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          const uint4 v = ld_shared_v4(kbase_s + ad_f8_off<D>(r, tq * (D / 4) + 16 * c));
          w[4 * c] = v.x; w[4 * c + 1] = v.y; w[4 * c + 2] = v.z; w[4 * c + 3] = v.w;
        }
#pragma unroll
        for (int k = 0; k < DK; ++k) {
          uint32_t b0, b1;
          e4m3x4_to_f16x2(w[k], b0, b1);
          ad_mma_f16(s[nt], qa[k], b0, b1);
        }
      } else {
        const int r = key_lo + nt * 8 + (lane & 7);
#pragma unroll
        for (int kc = 0; kc < DK / 2; ++kc) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(ad_chunk(kbase_s, r, kc * 4 + (lane >> 3)), b0, b1, b2, b3);
          ad_mma(s[nt], qa[2 * kc], b0, b1);
          ad_mma(s[nt], qa[2 * kc + 1], b2, b3);
        }
      }
    }
    // ---- scale, mask, online softmax (rows h2 = 0: g4, 1: g4 + 8)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < NKT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = F8 ? kabs + 16 * (nt >> 1) + 4 * tq + 2 * (nt & 1) + (e & 1) : kabs + nt * 8 + 2 * tq + (e & 1);
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
      pa[nt >> 1][(nt & 1) * 2 + 0] = F8 ? pack_f16x2(pv[0], pv[1]) : pack_bf16x2(pv[0], pv[1]);
      pa[nt >> 1][(nt & 1) * 2 + 1] = F8 ? pack_f16x2(pv[2], pv[3]) : pack_bf16x2(pv[2], pv[3]);
    }
    // ---- O += P V
#pragma unroll
    for (int kk = 0; kk < NKT / 2; ++kk) {
      if constexpr (F8) {
        // keys 16 kk + 4 tq .. + 3 of the warp's keys, one V^T row (d) per n-tile lane
#pragma unroll
        for (int dn = 0; dn < DN; ++dn) {
          uint32_t b0, b1;
          e4m3x4_to_f16x2(ld_shared_u32(vbase_s + ad_f8_off<64>(dn * 8 + g4, key_lo + 16 * kk + 4 * tq)), b0, b1);
          ad_mma_f16(o[dn], pa[kk], b0, b1);
        }
      } else {
        const int r = key_lo + kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int dn2 = 0; dn2 < DN / 2; ++dn2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(ad_chunk(vbase_s, r, 2 * dn2 + (lane >> 4)), b0, b1, b2, b3);
          ad_mma(o[2 * dn2], pa[kk], b0, b1);
          ad_mma(o[2 * dn2 + 1], pa[kk], b2, b3);
        }
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
  float* co = reinterpret_cast<float*>(stages);                       // [CW warps][16 rows][D]
  float* cm = co + AD_CWARPS * 16 * D;                                 // [CW][16]
  float* cl = cm + AD_CWARPS * 16;                                     // [CW][16]
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
    const float inv = Ls > 0.f ? p.out_scale / Ls : 0.f;
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

template <int D, int MT, bool F8, int CW = 4>
static int ad_launch(const CUtensorMap& tk, const CUtensorMap& tv, const AdParams& p, int B, cudaStream_t s) {
  using C = AdCfg<D, F8, CW>;
  static bool init = false;
  if (!init) {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<D, MT, F8, CW>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::BYTES);
    if (e != cudaSuccess) return -(int)e;
    init = true;
  }
  launch_pdl(attn_decode_kernel<D, MT, F8, CW>, dim3(p.splits, p.Hkv, B), dim3(C::THREADS), C::BYTES, s, tk, tv, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// Decode attention for GQA caches with D == DV in {64, 128} and at most 64 query rows
// (query positions x G) per (sequence, kv head).  Returns 1 on launch (the output is
// complete: split-KV partials are merged inside), 0 when the shape is not one this
// kernel serves (the caller then uses the general kernel), < 0 on error.
// counters: B * Hkv zeroed ints (needed when splits > 1), left zeroed.
// tk / tv: 2-D maps of the caches: bf16 [blocks * Hkv * 64, D] with 64 x 64 boxes; fp8
// (kv_fp8) K [blocks * Hkv * 64, D] bytes with [64, D] boxes, V^T [blocks * Hkv * D, 64]
// bytes with [D, 64] boxes.  k_scale / v_scale: the fp8 caches' dequantisation scales.
int attn_decode_gqa(const CUtensorMap& tk, const CUtensorMap& tv, const void* q, int q_stride, void* o,
                    int o_stride, const int* q_start, const int* kv_len, const int* block_table, int bt_stride,
                    int B, int max_q_len, int T, int Hq, int Hkv, int D, float scale, int splits, float* ws_o,
                    float* ws_lse, int* counters, int num_blocks, int window, const float* sinks, void* status,
                    cudaStream_t s, int kv_fp8, float k_scale, float v_scale) {
  const int G = Hq / Hkv;
  const int rows = max_q_len * G;
  // bf16 steps of 33..64 rows (MTP verification) may be sent to the tcgen05 kernel instead
  // (XTU_ATTN_DECODE_MAX_ROWS=32); fp8 caches are read by this kernel only
  static const int max_rows_bf16 = [] {
    const char* e = getenv("XTU_ATTN_DECODE_MAX_ROWS");
    return e ? atoi(e) : 64;
  }();
  if ((D != 64 && D != 128) || rows > 64 || rows <= 0) return 0;
  if (!kv_fp8 && rows > max_rows_bf16) return 0;
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
  p.scale_log2 = scale * 1.4426950408889634f * (kv_fp8 ? k_scale : 1.f);
  p.out_scale = kv_fp8 ? v_scale : 1.f;
  p.splits = splits < 1 ? 1 : splits;
  p.ws_o = ws_o;
  p.ws_lse = ws_lse;
  p.counters = counters;
  p.num_blocks = num_blocks;
  p.T = T;
  p.window = window;
  p.sinks = sinks;
  p.status = reinterpret_cast<XtuStatus*>(status);
#define XTU_AD(DD, F)                                                                                    \
  return rows <= 16 ? ad_launch<DD, 1, F>(tk, tv, p, B, s)                                               \
                    : rows <= 32 ? ad_launch<DD, 2, F>(tk, tv, p, B, s) : ad_launch<DD, 4, F, 8>(tk, tv, p, B, s)
  if (kv_fp8) {
    if (D == 128) XTU_AD(128, true);
    XTU_AD(64, true);
  }
  if (D == 128) XTU_AD(128, false);
  XTU_AD(64, false);
#undef XTU_AD
}

}  // namespace xtu

using namespace xtu;

typedef CUresult (*PFN_encodeTiled_ad)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                       const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                       CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_ad ad_encode_fn() {
  static PFN_encodeTiled_ad fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_ad>(ptr);
  }
  return fn;
}

// byte matrix [rows, cols] (row pitch = cols) with [box_rows, cols] boxes
static int ad_tmap_u8(CUtensorMap* map, const void* base, uint64_t rows, uint32_t cols, uint32_t box_rows,
                      CUtensorMapSwizzle sw) {
  PFN_encodeTiled_ad enc = ad_encode_fn();
  if (!enc) return -100;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols % 16 != 0) return -101;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1000 - (int)r;
}

namespace xtu {
// grid (max blocks of a sequence, B, Hkv); block 256.  Page j of sequence b (j < its block
// count) -> bf16 page blk_start[b] + j of the scratch caches; V un-transposed through
// shared memory.  out_bt[b][j] = that page.
__global__ void __launch_bounds__(256) kv_dequant_gather_kernel(
    const uint8_t* __restrict__ k8, const uint8_t* __restrict__ v8, const int* __restrict__ block_table,
    int bt_stride, const int* __restrict__ blk_start, const int* __restrict__ kv_len, int Hkv, int D, int Dv,
    float k_scale, float v_scale, __nv_bfloat16* __restrict__ ko, __nv_bfloat16* __restrict__ vo,
    int* __restrict__ out_bt, int out_bt_stride, int num_blocks, XtuStatus* st) {
  __shared__ uint8_t vt[256 * (AD_KEYS + 4)];
  const int j = blockIdx.x, b = blockIdx.y, h = blockIdx.z;
  const int nb = (kv_len[b] + AD_KEYS - 1) / AD_KEYS;
  if (j >= nb) return;
  const int pg = block_table[(size_t)b * bt_stride + j];
  if (!XTU_IN_BOUNDS(pg >= 0 && pg < num_blocks, st, 232, pg) || pg < 0 || pg >= num_blocks) return;
  const int dst = blk_start[b] + j;
  if (h == 0 && threadIdx.x == 0) out_bt[(size_t)b * out_bt_stride + j] = dst;
  const uint8_t* ks = k8 + ((size_t)pg * Hkv + h) * AD_KEYS * D;
  __nv_bfloat16* kd = ko + ((size_t)dst * Hkv + h) * AD_KEYS * D;
  for (int i = threadIdx.x; i < AD_KEYS * D; i += blockDim.x) {
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(ks[i], __NV_E4M3);
    kd[i] = __float2bfloat16(__half2float(__half(hr)) * k_scale);
  }
  const uint8_t* vs = v8 + ((size_t)pg * Hkv + h) * Dv * AD_KEYS;   // [Dv][64]
  for (int i = threadIdx.x; i < Dv * AD_KEYS; i += blockDim.x) vt[(i / AD_KEYS) * (AD_KEYS + 4) + i % AD_KEYS] = vs[i];
  __syncthreads();
  __nv_bfloat16* vd = vo + ((size_t)dst * Hkv + h) * AD_KEYS * Dv;   // [64][Dv]
  for (int i = threadIdx.x; i < AD_KEYS * Dv; i += blockDim.x) {
    const int key = i / Dv, d = i % Dv;
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(vt[d * (AD_KEYS + 4) + key], __NV_E4M3);
    vd[i] = __float2bfloat16(__half2float(__half(hr)) * v_scale);
  }
}
}  // namespace xtu

extern "C" {

// Decode attention over an fp8 (e4m3) paged GQA cache: k_cache [num_blocks, Hkv, 64, D],
// v_cache [num_blocks, Hkv, D, 64] (V transposed per block), values = stored * k_scale /
// v_scale.  D in {64, 128}, at most 64 query rows (positions x G) per (sequence, kv head).
// Returns 1 when the step ran (output complete), 0 when its shape is not served here (the
// caller dequantises the step's blocks and runs the general kernel), < 0 on error.
int xtu_paged_attention_fp8(const void* q, int q_stride, const void* k_cache, const void* v_cache, void* o,
                            int o_stride, const int* q_start, const int* kv_len, const int* block_table,
                            int bt_stride, int B, int max_q_len, int T, int Hq, int Hkv, int D, int num_blocks,
                            float scale, float k_scale, float v_scale, int splits, float* ws, int* counters,
                            int window, const float* sinks, void* status, cudaStream_t s) {
  if (B <= 0 || T <= 0) return 0;
  if (Hq % Hkv != 0) return -3;
  if ((D != 64 && D != 128) || max_q_len * (Hq / Hkv) > 64) return 0;
  CUtensorMap tk, tv;
  int rc = ad_tmap_u8(&tk, k_cache, (uint64_t)num_blocks * Hkv * AD_KEYS, D, AD_KEYS,
                      D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  rc = ad_tmap_u8(&tv, v_cache, (uint64_t)num_blocks * Hkv * D, AD_KEYS, D, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  const int sp = splits < 1 ? 1 : splits;
  float* ws_o = sp > 1 ? ws : nullptr;
  float* ws_lse = sp > 1 ? ws + (size_t)sp * T * Hq * D : nullptr;
  if (sp > 1 && ws == nullptr) return -5;
  return attn_decode_gqa(tk, tv, q, q_stride, o, o_stride, q_start, kv_len, block_table, bt_stride, B, max_q_len, T,
                         Hq, Hkv, D, scale, sp, ws_o, ws_lse, counters, num_blocks, window, sinks, status, s, 1,
                         k_scale, v_scale);
}

// The step's pages of an fp8 GQA cache (k8 [num_blocks, Hkv, 64, D], v8 [num_blocks, Hkv,
// Dv, 64]) as bf16 scratch pages (ko [*, Hkv, 64, D], vo [*, Hkv, 64, Dv]): sequence b's
// pages land at blk_start[b] .. blk_start[b] + ceil(kv_len[b] / 64) - 1, and out_bt [B,
// out_bt_stride] becomes the block table that addresses them.  max_blocks: the largest
// per-sequence page count.  Dv <= 256.
int xtu_kv_dequant_gather(const void* k8, const void* v8, const int* block_table, int bt_stride,
                          const int* blk_start, const int* kv_len, int B, int max_blocks, int Hkv, int D, int Dv,
                          float k_scale, float v_scale, void* ko, void* vo, int* out_bt, int out_bt_stride,
                          int num_blocks, void* status, cudaStream_t s) {
  if (B <= 0 || max_blocks <= 0) return 0;
  if (Dv > 256) return -2;
  kv_dequant_gather_kernel<<<dim3(max_blocks, B, Hkv), 256, 0, s>>>(
      (const uint8_t*)k8, (const uint8_t*)v8, block_table, bt_stride, blk_start, kv_len, Hkv, D, Dv, k_scale,
      v_scale, (__nv_bfloat16*)ko, (__nv_bfloat16*)vo, out_bt, out_bt_stride, num_blocks,
      reinterpret_cast<XtuStatus*>(status));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

}  // extern "C"
