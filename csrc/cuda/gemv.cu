// Small-M (decode) GEMV / grouped-GEMV kernels for sm_100a, weight-streaming bound.
//
//   y[m, n] = sum_k x[m, k] * W[n, k]     (m < M <= 32 dense, <= 16 per expert grouped;
//                                          W bf16 or e4m3 + 128x128 fp32 scales)
//
// At decode the GEMMs see 1..16 rows, so the job is to stream the weights at HBM
// bandwidth.  A CTA owns one 32-row weight tile and streams it through a ring of
// shared-memory stages filled by TMA (one elected producer thread, 128-byte swizzled
// 16-row boxes, STAGES x 8 KB in flight per CTA, several CTAs per SM), so the bytes in
// flight do not depend on how many loads the compute threads can keep outstanding.
// Four consumer warps split every stage along k and do the multiply-adds on the tensor
// cores with warp-level mma.sync m16n8k16:
//   * A = 16 weight rows x 16 k, B = 16 k x 8 tokens, D = 16 rows x 8 tokens (fp32).
//   * The order of k inside each MMA is permuted (a dot product does not care) so that
//     lane t's A fragment is ONE 16-byte shared-memory load of row (t/4) and one of row
//     (t/4 + 8): lane t owns k = 16*(t%4) + [0, 16) of its warp's 64-k slice (fp8) and
//     feeds MMA g in 0..3 with k = 16*(t%4) + 4g + {0,1 | 2,3}.  Its B fragment is the
//     same k slice of token t/4, so A and B agree on the permutation.
//   * fp8: e4m3 pairs -> f16 pairs with one cvt each (exact).  The activations arrive
//     already as f16 scaled by 2^-8 (keeps x * 448 inside the f16 range; the scale and
//     2^8 are restored in fp32 with the block scale once per 64-k slice): moe_permute
//     writes the MoE rows in that form, the gate/up epilogue writes h in it, and a
//     dense call converts its few rows once in a pre-pass, so no CTA converts x per
//     stage.  bf16 weights use the bf16 MMA on bf16 activations as is.
//   * Each TMA stage carries the tile's activations of the same k range beside the
//     weights; block scales are staged in shared memory once per tile; the four warps'
//     partial sums meet in shared memory at the end.
// Grouped (MoE) forms take the routing permutation of moe_permute: expert e owns rows
// seg[e]..seg[e+1] of the permuted activations, and the grid's y index walks the list of
// experts that have rows (moe_active_kernel), so idle experts cost no CTAs.
//   * gate/up: the tile's two 16-row halves are 16 gate rows and the matching 16 up rows
//     (W13 rows interleaved in 256-row blocks), so SwiGLU is applied in registers and
//     the [T*K, 2I] intermediate never exists.  At decode (<= 16 tokens) the activations
//     are not gathered per expert at all: every expert multiplies the step's tokens (they
//     fit the MMA's 8 or 16 columns) and writes only its own tokens' rows of h, found
//     through the (expert, token) -> row map of moe_permute_decode.
//   * down: rows scaled by the pair's routing weight and written to the pair's slot row.
// Dense calls with few tiles split K across CTAs; the last CTA of a tile (completion
// counter) sums the fp32 partials.
// Replaces the reference's SIMT small-M MXFP4 kernel (xiaotu_moe/csrc/moe4_smallm.cu,
// sm_80 FP32 FMA, split-K atomics) and the FP8 pair-centric Triton decode kernels
// (vllm_xiaotu_moe/decode_moe_fp8.py:23-138).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdlib>
#include "ptx.cuh"
#include "launch.cuh"
#include "../comm/peer.cuh"

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

// four e4m3 -> two f16x2 (exact): bytes 0,1 -> lo, bytes 2,3 -> hi
__device__ __forceinline__ void e4m3x4_f16x4(uint32_t v, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(v));
}

__device__ __forceinline__ uint32_t u4w(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// MMA row i (< 8) of a 16-row half holds weight row gv_prow(i) (and i + 8 row gv_prow(i) + 8):
// the eight lanes of one shared-memory phase (MMA rows 2p, 2p + 1) then read weight rows p and
// p + 4, whose 16-byte chunks of a 64-byte k slice fall in opposite halves of the 128-byte
// swizzle atom, so the weight fragment loads are free of bank conflicts.  The epilogues map
// accumulator rows back through the same function.
__device__ __forceinline__ int gv_prow(int i) { return (i >> 1) | ((i & 1) << 2); }

constexpr int GV_CWARPS = 4;                 // consumer warps (warp 0 is the producer)
constexpr int GV_THREADS = 32 * (1 + GV_CWARPS);
constexpr int GV_ROW_BYTES = 256;            // bytes of one weight row per stage (2 x 128-B boxes)
constexpr int GV_W_BYTES = 32 * GV_ROW_BYTES;   // weight part of a stage: 32 rows
constexpr int GV_MAX_KBLK = 128;             // block scales staged per tile (K <= 16384)
constexpr int GV_MAX_ROWS = 32;              // activation rows of a dense GEMV call (NT <= 4)
#ifndef GV_STAGES_NT1
// ring depth of the one-column-tile forms: 3 stages (42 KB a CTA, five CTAs per SM) beat 4
// (four per SM) on the short MoE tiles -- a verification step's MoE layer 335.8 -> 324.4 us
// at 20 rows, decode step 20.3 -> 18.5 ms at 4 requests -- where more CTAs in flight hide
// each CTA's start-up reads better than a deeper ring; 2 and 6 measured slower
#define GV_STAGES_NT1 3
#endif
#ifndef GV_STAGES_NT2
// ring depth of the two-column-tile forms (9..16 rows): here 4 stages (three CTAs per SM)
// measured best -- qkv / o_proj at 10 rows 17.8 / 15.4 us per graph-replayed call against
// 19.0 / 15.7 (3 stages) and 21.9 / 16.9 (2 stages, five CTAs per SM)
#define GV_STAGES_NT2 4
#endif

// A stage = the tile's 32 weight rows x 256 bytes, followed by the activations of the same
// k range (bf16, 8 * NT token rows per 128-byte box), both loaded by TMA.
template <bool FP8, int NT>
struct GvCfg {
  static constexpr int KSTAGE = GV_ROW_BYTES / (FP8 ? 1 : 2);   // k per stage
  static constexpr int XROWS = 8 * NT;
  static constexpr int XBOXES = KSTAGE / 64;                     // 64 bf16 per 128-byte box
  static constexpr int X_BYTES = XBOXES * XROWS * 128;
  static constexpr int STAGE_BYTES = GV_W_BYTES + X_BYTES;       // multiple of 1024
  // 32-row tiles: two CTAs per SM still fit (NT = 4), three (NT = 2), five (NT = 1)
  static constexpr int STAGES = NT >= 4 ? 3 : NT == 1 ? GV_STAGES_NT1 : GV_STAGES_NT2;
  static constexpr int RED_FLOATS = GV_CWARPS * 32 * 2 * NT * 4;
  static constexpr int BYTES = 1024 + STAGES * STAGE_BYTES + RED_FLOATS * 4 + 2 * GV_MAX_KBLK * 4 +
                               2 * STAGES * 8 + 64;
};

// Producer: issue the TMA loads of one stage into dst (completing on bar): the 32 weight
// rows x 256 bytes of k-stage s_abs (two 128-byte column chunks; WMODE 1: two 16-row halves
// 128 rows apart; WMODE 2: rows whose byte length is not a multiple of 128, four 2-D boxes)
// and the activations of the same k range (rows x_row0 ..).  The caller has armed bar.
template <bool FP8, int NT, int WMODE>
__device__ __forceinline__ void gv_issue_stage(const CUtensorMap* tmap, const CUtensorMap* xmap, uint8_t* dst,
                                               uint64_t* bar, const int (&row0)[2], int s_abs, int x_row0) {
  using C = GvCfg<FP8, NT>;
  if (WMODE == 0) {
    tma_load_3d(dst, tmap, bar, 0, row0[0], 2 * s_abs);
  } else if (WMODE == 1) {
    tma_load_4d(dst, tmap, bar, 0, row0[0], 0, 2 * s_abs);
  } else {
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        tma_load_2d(dst + b * 4096 + h * 2048, tmap, bar, s_abs * C::KSTAGE + b * (C::KSTAGE / 2), row0[h]);
  }
  tma_load_3d(dst + GV_W_BYTES, xmap, bar, 0, x_row0, s_abs * C::XBOXES);
}

// Consumer warp cw (0..3): multiply its k slice of the landed stage at sbase into acc
// (acc[t] += sc[t] * (W x) per 16-row half t), releasing the stage (empty) as soon as its
// fragments are in registers.  Activation rows >= mcount count as zero.
template <bool FP8, int NT>
__device__ __forceinline__ void gv_mma_stage(const uint8_t* sbase, uint64_t* empty, int cw, int lane, int mcount,
                                             const float (&sc)[2], float (&acc)[2][NT][4]) {
  using C = GvCfg<FP8, NT>;
  constexpr int LK = FP8 ? 16 : 8;           // k per lane per stage
  const int g4 = lane >> 2, tq = lane & 3;
  const int c16 = (cw & 1) * 4 + tq;         // 16-byte chunk of the 128-byte row within box (cw >> 1)
  const uint8_t* box = sbase + (cw >> 1) * 4096;
  uint4 w[2][2];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = t * 16 + gv_prow(g4) + h * 8;
      w[t][h] = *reinterpret_cast<const uint4*>(box + r * 128 + ((c16 ^ (r & 7)) << 4));
    }
  // activations of token n*8+g4 for this lane's k slice (rows past mcount are zeroed)
  uint4 xr[NT][LK / 8];
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int tok = n * 8 + g4;
    const uint8_t* xrow = sbase + GV_W_BYTES + (FP8 ? cw : (cw >> 1)) * (C::XROWS * 128) + tok * 128;
#pragma unroll
    for (int q = 0; q < LK / 8; ++q) {
      const int ch = FP8 ? (2 * tq + q) : c16;
      const uint4 v = *reinterpret_cast<const uint4*>(xrow + ((ch ^ (tok & 7)) << 4));
      xr[n][q] = tok < mcount ? v : make_uint4(0, 0, 0, 0);
    }
  }
  // these generic-proxy reads must be ordered before the TMA (async proxy) that
  // refills the slot once it is released
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) mbar_arrive(empty);
  uint32_t b[NT][LK / 2];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int q = 0; q < LK / 8; ++q)
#pragma unroll
      for (int j = 0; j < 4; ++j) b[n][4 * q + j] = u4w(xr[n][q], j);   // f16 x 2^-8 (fp8) or bf16
  float d[2][NT][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) d[t][n][j] = 0.f;
#pragma unroll
  for (int g = 0; g < LK / 4; ++g) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      uint32_t a0, a1, a2, a3;
      if (FP8) {
        e4m3x4_f16x4(u4w(w[t][0], g), a0, a2);
        e4m3x4_f16x4(u4w(w[t][1], g), a1, a3);
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
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[t][n][j] = fmaf(d[t][n][j], sc[t], acc[t][n][j]);
}

// Stream one 32-row tile (rows row0[0]..+15 and row0[1]..+15 of the tensor map) over
// stages [s_begin, s_end) and multiply by activations x (rows x_row0 .. x_row0 + mcount).
// Producer: warp 0.  Consumers: warps 1..4, each with acc[tile][nt][4] for its k slices.
// Returns false (all threads) if a wait timed out.
template <bool FP8, int NT, int WMODE>
__device__ __forceinline__ bool gv_stream_tile(const CUtensorMap* tmap, const CUtensorMap* xmap, uint8_t* stages,
                                               uint64_t* full, uint64_t* empty, float* sc_sm, uint32_t& phase_base,
                                               const int (&row0)[2], int s_begin, int s_end, int K,
                                               const float* __restrict__ wscale, int sk, int scale_row_blk0,
                                               int scale_row_blk1, int x_row0, int mcount, float (&acc)[2][NT][4],
                                               XtuStatus* st) {
  using C = GvCfg<FP8, NT>;
  constexpr int CK = FP8 ? 64 : 32;          // k per warp per stage
  constexpr int KSTAGE = C::KSTAGE;
  constexpr int GV_STAGES = C::STAGES;
  constexpr int GV_STAGE_BYTES = C::STAGE_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nst = s_end - s_begin;
  bool ok = true;
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][n][i] = 0.f;
  if (warp == 0) {
    if (elect_one()) {
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const uint32_t it = phase_base + i;
        const int slot = it % GV_STAGES;
        if (it >= GV_STAGES && !mbar_wait(&empty[slot], ((it / GV_STAGES) - 1) & 1, st, 60)) { ok = false; break; }
        ++issued;
        mbar_arrive_expect_tx(&full[slot], GV_STAGE_BYTES);
        gv_issue_stage<FP8, NT, WMODE>(tmap, xmap, stages + slot * GV_STAGE_BYTES, &full[slot], row0, s_begin + i,
                                       x_row0);
      }
      if (!ok) {   // give the copies already issued (bounded) time to land before the CTA exits
        for (int j = issued > GV_STAGES ? issued - GV_STAGES : 0; j < issued; ++j) {
          const uint32_t it = phase_base + j;
          mbar_wait(&full[it % GV_STAGES], (it / GV_STAGES) & 1, nullptr, 0, 50000000ull);
        }
      }
    }
    __syncwarp();
  } else {
    const int cw = warp - 1;
    // this tile's block scales (x 2^8, the activation pre-scale) for its stage range
    const int kblk0 = (s_begin * KSTAGE) >> 7;
    const int nkblk = min(sk, ((s_end * KSTAGE + 127) >> 7)) - kblk0;
    if (FP8) {
      for (int j = threadIdx.x - 32; j < nkblk && j < GV_MAX_KBLK; j += 32 * GV_CWARPS) {
        sc_sm[j] = 256.f * __ldg(wscale + (size_t)scale_row_blk0 * sk + kblk0 + j);
        sc_sm[GV_MAX_KBLK + j] = 256.f * __ldg(wscale + (size_t)scale_row_blk1 * sk + kblk0 + j);
      }
      asm volatile("bar.sync 2, %0;" ::"n"(32 * GV_CWARPS) : "memory");
    }
    for (int i = 0; i < nst; ++i) {
      const uint32_t it = phase_base + i;
      const int slot = it % GV_STAGES;
      float sc[2] = {1.f, 1.f};
      if (FP8) {
        const int kb = min(((s_begin + i) * KSTAGE + cw * CK) >> 7, sk - 1) - kblk0;
        sc[0] = sc_sm[kb];
        sc[1] = sc_sm[GV_MAX_KBLK + kb];
      }
      if (!mbar_wait(&full[slot], (it / GV_STAGES) & 1, st, 61)) { ok = false; break; }
      gv_mma_stage<FP8, NT>(stages + slot * GV_STAGE_BYTES, &empty[slot], cw, lane, mcount, sc, acc);
    }
  }
  phase_base += nst;
  return __syncthreads_and(ok);
}

// sum the consumer warps' fragments; on return consumer warp 0 (warp 1) holds the totals
template <int NT>
__device__ __forceinline__ void gv_reduce(float (&acc)[2][NT][4], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int V = 2 * NT * 4;
  if (warp >= 1) {
    float* mine = red + ((size_t)(warp - 1) * 32 + lane) * V;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) mine[(t * NT + n) * 4 + i] = acc[t][n][i];
  }
  __syncthreads();
  if (warp == 1) {
    for (int w = 1; w < GV_CWARPS; ++w) {
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

template <bool FP8, int NT>
__device__ __forceinline__ uint8_t* gv_setup(uint64_t*& full, uint64_t*& empty, float*& red, float*& sc_sm) {
  using C = GvCfg<FP8, NT>;
  extern __shared__ uint8_t gv_smem_raw[];
  const uint32_t a = smem_u32(gv_smem_raw);
  uint8_t* base = gv_smem_raw + (((a + 1023u) & ~1023u) - a);
  red = reinterpret_cast<float*>(base + C::STAGES * C::STAGE_BYTES);
  sc_sm = red + C::RED_FLOATS;
  full = reinterpret_cast<uint64_t*>(sc_sm + 2 * GV_MAX_KBLK);
  empty = full + C::STAGES;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GV_CWARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  return base;
}

// ---------------------------------------------------------------------------
// dense: y[M, N] = x[M, K] W^T (+ bias); grid (32-row tiles, K splits)
// ---------------------------------------------------------------------------
// Tensor-parallel epilogue: instead of y, every rank's partial rows go straight into all
// ranks' receive buffers (slot [parity][rank]) by peer stores, and the tile that finishes
// last raises this rank's flag on every peer.  The rows are summed by the next kernel
// (xtu_tp_sum_rmsnorm).  Epochs: e = *ep_c + 1 (advanced by that consumer), published in
// *ep_p for it; two receive parities so use u + 1 never overwrites what use u still reads.
constexpr int GV_MAX_WORLD = 8;   // ranks a fused TP GEMV scatters to (one NVSwitch node)

struct GvPeer {
  __nv_bfloat16* const* dst;   // [world] receive buffers (symmetric), 2 * world slots each
  long long slot;              // elements per slot (>= M * N)
  int rank, world;
  int* done;                   // finished-tile counter (zeroed, left zeroed)
  int* const* flags;           // [world] peers' flag arrays
  const int* ep_c;             // epoch the consumer finished
  int* ep_p;                   // epoch this producer published
};

template <bool FP8, int NT, int WM, bool PEER = false>
__global__ void __launch_bounds__(GV_THREADS) gemv_dense_kernel(
    const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap xmap,
    const float* __restrict__ wscale, int N, int K, int M, const __nv_bfloat16* __restrict__ bias,
    void* __restrict__ y, int y_stride, int y_f32, float* __restrict__ ws, int* __restrict__ counters,
    XtuStatus* st, GvPeer pr = GvPeer{}) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  uint64_t *full, *empty;
  float *red, *sc_sm;
  uint8_t* stages = gv_setup<FP8, NT>(full, empty, red, sc_sm);
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    prefetch_tmap(&xmap);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g4 = lane >> 2, tq = lane & 3;
  const int sk = (K + 127) >> 7;
  const int kstage = GV_ROW_BYTES / (FP8 ? 1 : 2);
  const int nstages = (K + kstage - 1) / kstage;
  const int splits = gridDim.y, split = blockIdx.y;
  const int per = (nstages + splits - 1) / splits;
  const int s0 = min(nstages, split * per), s1 = min(nstages, s0 + per);
  const int r0 = blockIdx.x * 32;
  const int rows[2] = {r0, r0 + 16};
  uint32_t pb = 0;
  float acc[2][NT][4];
  if (!gv_stream_tile<FP8, NT, WM>(&tmap, &xmap, stages, full, empty, sc_sm, pb, rows, s0, s1, K, wscale, sk,
                               min(r0, N - 1) >> 7, min(r0 + 16, N - 1) >> 7, 0, M, acc, st))
    return;
  gv_reduce<NT>(acc, red);
  if (warp != 1) return;
  if (splits > 1) {
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = rows[t] + gv_prow(g4) + (i >> 1) * 8;
          const int tok = n * 8 + 2 * tq + (i & 1);
          if (row < N && tok < M) ws[((size_t)split * GV_MAX_ROWS + tok) * N + row] = acc[t][n][i];
        }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&counters[blockIdx.x], 1) == splits - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[t][n][i] = 0.f;
    // four splits per round, all their loads issued before any add (one L2 latency per
    // round, not per split); the adds keep split order, so the sum is reproducible
    constexpr int QB = NT >= 4 ? 1 : 4;      // splits per round (register budget of 32-row tiles)
    for (int q0 = 0; q0 < splits; q0 += QB) {
      float pv[QB][2][NT][4];
#pragma unroll
      for (int qq = 0; qq < QB; ++qq)
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int row = rows[t] + gv_prow(g4) + (i >> 1) * 8;
              const int tok = n * 8 + 2 * tq + (i & 1);
              const int q = q0 + qq;
              pv[qq][t][n][i] = (q < splits && row < N && tok < M) ? __ldcg(ws + ((size_t)q * GV_MAX_ROWS + tok) * N + row)
                                                                   : 0.f;
            }
#pragma unroll
      for (int qq = 0; qq < QB; ++qq)
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[t][n][i] += pv[qq][t][n][i];
    }
    if (lane == 0) counters[blockIdx.x] = 0;
  }
  // PEER: the receive-slot base of every rank, read once (the stores below could alias
  // the pointer table and the epoch as far as the compiler knows)
  __nv_bfloat16* dst[GV_MAX_WORLD];
  if (PEER) {
    const int par = (__ldcg(pr.ep_c) + 1) & 1;
    const size_t base = (size_t)(par * pr.world + pr.rank) * pr.slot;
#pragma unroll
    for (int p = 0; p < GV_MAX_WORLD; ++p) dst[p] = p < pr.world ? pr.dst[p] + base : nullptr;
  }
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = rows[t] + gv_prow(g4) + (i >> 1) * 8;
        const int tok = n * 8 + 2 * tq + (i & 1);
        if (row < N && tok < M) {
          float v = acc[t][n][i];
          if (bias) v += __bfloat162float(bias[row]);
          if (PEER) {
            const __nv_bfloat16 bv = __float2bfloat16(v);
            const size_t off = (size_t)tok * N + row;
#pragma unroll
            for (int p = 0; p < GV_MAX_WORLD; ++p)
              if (p < pr.world) dst[p][off] = bv;
          } else if (y_f32) {
            reinterpret_cast<float*>(y)[(size_t)tok * y_stride + row] = v;
          } else {
            reinterpret_cast<__nv_bfloat16*>(y)[(size_t)tok * y_stride + row] = __float2bfloat16(v);
          }
        }
      }
  if (PEER) {   // this tile's rows are out: the last tile raises the flag on every peer
    // the warp barrier orders every lane's stores before lane 0; lane 0's system-scope
    // fence (cumulative) then publishes them all before its counter increment
    __syncwarp();
    if (lane == 0) __threadfence_system();
    if (lane == 0 && atomicAdd(pr.done, 1) == (int)gridDim.x - 1) {
      *pr.done = 0;
      const int e = *pr.ep_c + 1;
      fence_acq_rel_sys();
      for (int p = 0; p < pr.world; ++p) st_release_sys(pr.flags[p] + pr.rank, e);
      *pr.ep_p = e;
    }
  }
}

// ---------------------------------------------------------------------------
// dense decode GEMM on the 5th-generation tensor cores, for 17..32 activation rows
// (speculative verification steps), where the warp-level MMAs of the kernels above bound
// the call, not HBM (four 8-token column tiles per 16 weight rows).  The weight rows are
// the MMA's M and the tokens its N:
//   CTA = one 128-row weight tile (one block-scale row) x one K split; stages of 128 k.
//   warp 0     TMA: the stage's e4m3 weights (128 rows x 128 B, 128-byte swizzle) and
//              its activations (f16 x 2^-8, 32 rows x 128 k as two 64-k swizzled chunks)
//              into a GT_RING-deep ring
//   warp 1     TMEM (32 columns) + MMA issue: D[128, 32] += Wf16 x X^T, kind::f16,
//              eight K = 16 steps per stage
//   warps 2-9  widen the stage's weights: half a row per thread (warps 2-5 the first 64 k,
//              6-9 the second), e4m3 -> f16 times the stage's block scale x 2^8 (the
//              activations carry 2^-8), into a double-buffered K-major swizzled f16 tile
//              (the widening, not HBM, paces the kernel: four warps left it at 2.2 TB/s);
//              then warps 2-5 run the epilogue (row = TMEM lane, 32 token columns): y, or
//              the split's fp32 partial, which the last split CTA of the tile sums in split
//              order.
// |W| x 2^8 must stay inside the f16 range (|W| < 255), which fp8 checkpoints meet by
// construction of their block scales.
// bf16 weights (FP8 = false: e.g. the LM head of a verification step) need no widening: the
// MMA reads each stage's weights as TMA lands them (two 64-k swizzled chunks) with the bf16
// activations, through a 5-deep ring of 40 KB stages.
// ---------------------------------------------------------------------------
#ifndef GT_RING_DEPTH
#define GT_RING_DEPTH 6
#endif
#ifndef GT_CBUF_DEPTH
#define GT_CBUF_DEPTH 2
#endif
constexpr int GT_RING = GT_RING_DEPTH;            // weight + activation stages in flight
constexpr int GT_CBUF = GT_CBUF_DEPTH;            // widened tiles in flight (widening runs ahead of the MMA)
// (qkv 14336 x 4096, 20 rows: 6 / 2 -> 25.6 us per call, 4 / 3 -> 27.9 us: the weight bytes
// in flight count for more than the widening running further ahead)
constexpr int GT_W8 = 128 * 128;                  // e4m3 weights of one stage (bytes)
constexpr int GT_X = 2 * 32 * 128;                // activations of one stage (bytes)
constexpr int GT_STAGE = GT_W8 + GT_X;            // 24 KB
constexpr int GT_WF16 = 2 * 128 * 128;            // widened weights: two 64-k chunks x 128 rows x 128 B
constexpr int GT_SMEM = 1024 + GT_RING * GT_STAGE + GT_CBUF * GT_WF16 + 256 + GV_MAX_KBLK * 4;
constexpr int GT_THREADS = 320;
// the bf16-weight form: 32 KB of weights + the activations per stage, no widened tiles
constexpr int GT_RING_BF = 5;
constexpr int GT_STAGE_BF = 2 * GT_W8 + GT_X;
constexpr int GT_SMEM_BF = 1024 + GT_RING_BF * GT_STAGE_BF + 256 + GV_MAX_KBLK * 4;

__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  // kind::f16 with A = B = f16 (format code 0), fp32 D, both operands K-major
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <bool FP8>
__global__ void __launch_bounds__(GT_THREADS, 1) gemv_tc_kernel(
    const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
    const float* __restrict__ wscale, int N, int K, int M, const __nv_bfloat16* __restrict__ bias, void* __restrict__ y,
    int y_stride, int y_f32, float* __restrict__ ws, int* __restrict__ counters, XtuStatus* st) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  extern __shared__ uint8_t gt_smem_raw[];
  const uint32_t raw = smem_u32(gt_smem_raw);
  constexpr int RING = FP8 ? GT_RING : GT_RING_BF;
  constexpr int STAGE = FP8 ? GT_STAGE : GT_STAGE_BF;
  constexpr int WB = FP8 ? GT_W8 : 2 * GT_W8;           // weight bytes of a stage
  uint8_t* ring = gt_smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* wf16 = ring + RING * STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(wf16 + (FP8 ? GT_CBUF * GT_WF16 : 0));
  uint64_t* full = bars;                    // [RING] TMA landed
  uint64_t* empty = bars + RING;            // [RING] MMA done with the stage
  uint64_t* cfull = empty + RING;           // [GT_CBUF] widened tile ready
  uint64_t* cempty = cfull + GT_CBUF;       // [GT_CBUF] MMA done with the widened tile
  uint64_t* dfull = cempty + GT_CBUF;       // accumulator complete
  uint32_t* tslot = reinterpret_cast<uint32_t*>(dfull + 1);
  float* scs = reinterpret_cast<float*>(bars + 32);   // the CTA's block scales x 2^8, [ns]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
  const int S = K / 128, sk = (K + 127) >> 7;
  const int per = (S + splits - 1) / splits;
  const int s0 = min(S, split * per), s1 = min(S, s0 + per), ns = s1 - s0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < RING; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < GT_CBUF; ++i) {
      mbar_init(&cfull[i], 8);
      mbar_init(&cempty[i], 1);
    }
    mbar_init(dfull, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tslot, 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  bool ok = true;
  if (warp == 0) {
    // ---------------- producer
    if (elect_one()) {
      prefetch_tmap(&wmap);
      prefetch_tmap(&xmap);
      int issued = 0;
      for (int i = 0; i < ns; ++i) {
        const int slot = i % RING;
        if (i >= RING && !mbar_wait(&empty[slot], ((i / RING) - 1) & 1, st, 70)) { ok = false; break; }
        ++issued;
        mbar_arrive_expect_tx(&full[slot], STAGE);
        uint8_t* dst = ring + slot * STAGE;
        // fp8: one 128-byte chunk x 128 rows; bf16: two 64-element chunks x 128 rows
        tma_load_3d(dst, &wmap, &full[slot], 0, tile * 128, (FP8 ? 1 : 2) * (s0 + i));
        tma_load_3d(dst + WB, &xmap, &full[slot], 0, 0, 2 * (s0 + i));
      }
      if (!ok) {   // give the copies already issued (bounded) time to land before the CTA exits
        for (int j = issued > RING ? issued - RING : 0; j < issued; ++j)
          mbar_wait(&full[j % RING], (j / RING) & 1, nullptr, 0, 50000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issue
    if (elect_one()) {
      constexpr uint32_t idesc = FP8 ? idesc_f16_f32(128, 32) : idesc_bf16_f32(128, 32);
      const uint32_t wf = smem_u32(wf16), rg = smem_u32(ring);
      for (int i = 0; i < ns; ++i) {
        const int slot = i % RING, c = i % GT_CBUF;
        // the activations come straight from the TMA stage: observe its barrier here too
        if (!mbar_wait(&full[slot], (i / RING) & 1, st, 75) ||
            (FP8 && !mbar_wait(&cfull[c], (i / GT_CBUF) & 1, st, 71))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = FP8 ? wf + c * GT_WF16 : rg + slot * STAGE, b0 = rg + slot * STAGE + WB;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t koff = (j >> 2) * (128 * 128) + (j & 3) * 32;
          const uint32_t xoff = (j >> 2) * (32 * 128) + (j & 3) * 32;
          mma_f16_ss(tmem, sdesc_kmajor_sw128(a0 + koff), sdesc_kmajor_sw128(b0 + xoff), idesc,
                     (i > 0 || j > 0) ? 1u : 0u);
        }
        mma_commit(&empty[slot]);
        if (FP8) mma_commit(&cempty[c]);
      }
      mma_commit(dfull);   // also on the error path: the epilogue waits on it (bounded)
    }
  } else {
    // ---------------- widen (warps 2-9): thread = half of weight row r (= TMEM lane r)
    const int q = warp & 3, r = q * 32 + lane, half = (warp - 2) >> 2;
    const int rb = min(tile * 128, N - 1) >> 7;   // the tile's block-scale row
    // the split's block scales, staged once (a global load per stage sat on every stage's path)
    if (FP8)
      for (int j = threadIdx.x - 64; j < ns; j += 256) scs[j] = 256.f * __ldg(wscale + (size_t)rb * sk + s0 + j);
    asm volatile("bar.sync 1, 256;" ::: "memory");
    for (int i = 0; i < (FP8 ? ns : 0); ++i) {
      const int slot = i % RING, c = i % GT_CBUF;
      const float sc = scs[i];
      if (!mbar_wait(&full[slot], (i / RING) & 1, st, 72)) { ok = false; break; }
      if (i >= GT_CBUF && !mbar_wait(&cempty[c], ((i / GT_CBUF) - 1) & 1, st, 73)) { ok = false; break; }
      const uint8_t* src = ring + slot * STAGE + r * 128;
      uint8_t* dstrow = wf16 + c * GT_WF16 + r * 128;
      const __half2 s2 = __floats2half2_rn(sc, sc);
#pragma unroll
      for (int ch = 4 * half; ch < 4 * half + 4; ++ch) {   // 16 e4m3 (k = 16 ch ..) -> two f16 pieces
        const uint4 v = *reinterpret_cast<const uint4*>(src + ((ch ^ (r & 7)) << 4));
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
        uint32_t h[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t lo, hi;
          e4m3x4_f16x4(wv[e], lo, hi);
          __half2 l2 = __hmul2(*reinterpret_cast<__half2*>(&lo), s2);
          __half2 h2 = __hmul2(*reinterpret_cast<__half2*>(&hi), s2);
          h[2 * e] = *reinterpret_cast<uint32_t*>(&l2);
          h[2 * e + 1] = *reinterpret_cast<uint32_t*>(&h2);
        }
        const int kc = ch >> 2, p0 = (ch & 3) * 2;   // 64-k chunk, first 16-byte piece
        uint8_t* d = dstrow + kc * (128 * 128);
        *reinterpret_cast<uint4*>(d + ((p0 ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(d + (((p0 + 1) ^ (r & 7)) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
      }
      fence_proxy_async_smem();   // generic-proxy writes -> the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&cfull[c]);
    }
    // ---------------- epilogue (warps 2-5): row r, token columns 0..31
    if (half == 0) {
      const bool have = mbar_wait(dfull, 0, st, 74) && ok;
      tc_fence_after();
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16), v);
      tmem_wait_ld();
      const int row = tile * 128 + r;
      if (have && ns > 0) {
        float acc[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) acc[t] = __uint_as_float(v[t]);
        bool emit = splits == 1;
        if (!emit) {
          // each warp settles its own 32 rows (counter per tile quarter), so no barrier
          // couples the four warps
          if (row < N) {
#pragma unroll
            for (int t = 0; t < 32; ++t)
              if (t < M) __stcg(ws + ((size_t)split * GV_MAX_ROWS + t) * N + row, acc[t]);
          }
          __threadfence();
          __syncwarp();
          int last = 0;
          if (lane == 0) last = atomicAdd(counters + tile * 4 + q, 1) == splits - 1;
          last = __shfl_sync(0xffffffffu, last, 0);
          if (last) {
            __threadfence();
            if (row < N) {
#pragma unroll
              for (int t = 0; t < 32; ++t) acc[t] = 0.f;
              for (int sp = 0; sp < splits; ++sp)   // split order: the bits do not depend on who came last
#pragma unroll
                for (int t = 0; t < 32; ++t)
                  if (t < M) acc[t] += __ldcg(ws + ((size_t)sp * GV_MAX_ROWS + t) * N + row);
            }
            if (lane == 0) counters[tile * 4 + q] = 0;
            emit = true;
          }
        }
        if (emit && row < N) {
          const float b = bias ? __bfloat162float(bias[row]) : 0.f;
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            if (t >= M) break;
            if (y_f32) reinterpret_cast<float*>(y)[(size_t)t * y_stride + row] = acc[t] + b;
            else reinterpret_cast<__nv_bfloat16*>(y)[(size_t)t * y_stride + row] = __float2bfloat16(acc[t] + b);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

// ---------------------------------------------------------------------------
// grouped gate/up + SwiGLU: grid (I / 16, experts with rows).  W13 [E, 2I, K] in 256-row
// blocks (128 gate, 128 up); a tile = 16 gate rows + the matching 16 up rows.
// ---------------------------------------------------------------------------
template <bool FP8, int NT>
__global__ void __launch_bounds__(GV_THREADS) moe_gemv_gate_up_kernel(
    const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap xmap,
    const float* __restrict__ wscale, int I, int K, const int* __restrict__ seg, const int* __restrict__ active,
    const int* __restrict__ tokrow, int ntok, __nv_bfloat16* __restrict__ h, float limit, float alpha, float beta,
    const __grid_constant__ CUtensorMap tmap_sh, const float* __restrict__ wscale_sh, int sh_row0, int has_sh,
    XtuStatus* st) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  // grid rows past the active experts: the shared expert (has_sh), as one more expert
  // over every token, its h rows at sh_row0 + token; the rest exit
  const int nact = active[0];
  const bool sh = has_sh && (int)blockIdx.y == nact;
  if (!sh && (int)blockIdx.y >= nact) return;
  const int e = sh ? 0 : active[1 + blockIdx.y];
  const int s0 = sh ? sh_row0 : seg[e], cnt = sh ? ntok : seg[e + 1] - s0;
  if (cnt <= 0) return;
  // token-direct form: x holds the step's ntok tokens (not gathered per expert); the
  // expert multiplies all of them and keeps the columns of its own tokens (tokrow)
  const int* trow = (tokrow && !sh) ? tokrow + blockIdx.y * 16 : nullptr;
  const bool direct = tokrow != nullptr;
  const int xrow0 = direct ? 0 : s0, xcnt = direct ? ntok : cnt;
  const CUtensorMap* wmap = sh ? &tmap_sh : &tmap;
  wscale = sh ? wscale_sh : wscale;
  uint64_t *full, *empty;
  float *red, *sc_sm;
  uint8_t* stages = gv_setup<FP8, NT>(full, empty, red, sc_sm);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g4 = lane >> 2, tq = lane & 3;
  const int sk = (K + 127) >> 7;
  const int kstage = GV_ROW_BYTES / (FP8 ? 1 : 2);
  const int nstages = (K + kstage - 1) / kstage;
  const int j0 = blockIdx.x * 16;
  const int grow = (j0 >> 7) * 256 + (j0 & 127);            // gate row within the expert
  const int rows[2] = {e * 2 * I + grow, e * 2 * I + grow + 128};
  const float* esc = FP8 ? wscale + (size_t)e * ((2 * I + 127) >> 7) * sk : nullptr;
  uint32_t pb = 0;
  for (int mb = 0; mb < xcnt; mb += 8 * NT) {
    const int mc = min(8 * NT, xcnt - mb);
    float acc[2][NT][4];
    if (!gv_stream_tile<FP8, NT, 1>(wmap, &xmap, stages, full, empty, sc_sm, pb, rows, 0, nstages, K, esc, sk,
                                 grow >> 7, (grow + 128) >> 7, xrow0 + mb, mc, acc, st))
      return;
    gv_reduce<NT>(acc, red);
    if (warp != 1) continue;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = j0 + gv_prow(g4) + (i >> 1) * 8;
        const int tok = n * 8 + 2 * tq + (i & 1);
        const int hr = tok >= mc ? -1 : trow ? trow[mb + tok] : s0 + mb + tok;
        if (hr >= 0) {
          float g = acc[0][n][i], u = acc[1][n][i];
          if (limit > 0.f) { g = fminf(g, limit); u = fminf(fmaxf(u, -limit), limit); }
          const float v = (g / (1.f + __expf(-alpha * g))) * (u + beta);
          if (FP8)   // the down GEMV's activation form: f16 x 2^-8
            reinterpret_cast<__half*>(h)[(size_t)hr * I + j] = __float2half_rn(v * 0.00390625f);
          else
            h[(size_t)hr * I + j] = __float2bfloat16(v);
        }
      }
  }
}

// ---------------------------------------------------------------------------
// grouped down: out[slot[row]] = w[row] * (h[row] W2[e]^T); grid (H / 32, experts with rows)
// ---------------------------------------------------------------------------
template <bool FP8, int NT>
__global__ void __launch_bounds__(GV_THREADS) moe_gemv_down_kernel(
    const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap xmap,
    const float* __restrict__ wscale, int H, int I, const int* __restrict__ seg, const int* __restrict__ active,
    const int* __restrict__ perm_slot, const float* __restrict__ perm_w, __nv_bfloat16* __restrict__ out,
    const __grid_constant__ CUtensorMap tmap_sh, const float* __restrict__ wscale_sh, int sh_row0, int sh_out0,
    int ntok, int has_sh, XtuStatus* st) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  // the grid row after the active experts is the shared expert (has_sh): h rows
  // sh_row0 + token, output rows sh_out0 + token with weight 1
  const int nact = active[0];
  const bool sh = has_sh && (int)blockIdx.y == nact;
  if (!sh && (int)blockIdx.y >= nact) return;
  const int e = sh ? 0 : active[1 + blockIdx.y];
  const int s0 = sh ? sh_row0 : seg[e], cnt = sh ? ntok : seg[e + 1] - s0;
  if (cnt <= 0) return;
  const CUtensorMap* wmap = sh ? &tmap_sh : &tmap;
  wscale = sh ? wscale_sh : wscale;
  uint64_t *full, *empty;
  float *red, *sc_sm;
  uint8_t* stages = gv_setup<FP8, NT>(full, empty, red, sc_sm);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g4 = lane >> 2, tq = lane & 3;
  const int sk = (I + 127) >> 7;
  const int kstage = GV_ROW_BYTES / (FP8 ? 1 : 2);
  const int nstages = (I + kstage - 1) / kstage;
  const int r0 = blockIdx.x * 32;
  const int rows[2] = {e * H + r0, e * H + r0 + 16};
  const float* esc = FP8 ? wscale + (size_t)e * ((H + 127) >> 7) * sk : nullptr;
  uint32_t pb = 0;
  for (int mb = 0; mb < cnt; mb += 8 * NT) {
    const int mc = min(8 * NT, cnt - mb);
    float acc[2][NT][4];
    if (!gv_stream_tile<FP8, NT, 0>(wmap, &xmap, stages, full, empty, sc_sm, pb, rows, 0, nstages, I, esc, sk,
                                 min(r0, H - 1) >> 7, min(r0 + 16, H - 1) >> 7, s0 + mb, mc, acc, st))
      return;
    gv_reduce<NT>(acc, red);
    if (warp != 1) continue;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r0 + t * 16 + gv_prow(g4) + (i >> 1) * 8;
          const int tok = n * 8 + 2 * tq + (i & 1);
          if (row < H && tok < mc) {
            const int pr = s0 + mb + tok;
            if (sh) out[(size_t)(sh_out0 + mb + tok) * H + row] = __float2bfloat16(acc[t][n][i]);
            else out[(size_t)perm_slot[pr] * H + row] = __float2bfloat16(acc[t][n][i] * perm_w[pr]);
          }
        }
  }
}

// active[0] = number of experts with rows, active[1..] = those experts in order (one warp)
__global__ void moe_active_kernel(const int* __restrict__ seg, int E, int* __restrict__ active) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  const int lane = threadIdx.x;
  int n = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const bool has = e < E && seg[e + 1] > seg[e];
    const unsigned m = __ballot_sync(0xffffffffu, has);
    if (has) active[1 + n + __popc(m & ((1u << lane) - 1u))] = e;
    n += __popc(m);
  }
  if (lane == 0) active[0] = n;
}


// ---------------------------------------------------------------------------
// MXFP4 / NVFP4 experts at decode (the reference's moe4_smallm.cu role, restated for
// tensor cores).  A stage is still 32 weight rows x 256 bytes, now 512 k of packed e2m1
// (low nibble = even k), with the activations of the same k range in bf16.  Consumer warp
// cw owns bytes [64 cw, 64 cw + 64) of each row; lane (g4, tq) decodes its 16-byte chunk
// (32 k = one MXFP4 scale group, two NVFP4 groups) of rows gv_prow(g4) and + 8 through a
// byte -> bf16-pair table in shared memory, multiplies by the row's group scale (exact in
// bf16: a power of two, or an e4m3 value times an e2m1 value), and feeds bf16 m16n8k16
// MMAs with k = 32 tq + 4 g + {0,1 | 2,3} for MMA g (the activations use the same order).
// NVFP4's per-expert fp32 global scale multiplies the fp32 result.
// ---------------------------------------------------------------------------
template <int NT>
struct Gv4Cfg {
  static constexpr int KSTAGE = 512;                            // k per stage
  static constexpr int XROWS = 8 * NT;
  static constexpr int XBOXES = KSTAGE / 64;                    // 64 bf16 per 128-byte box
  static constexpr int X_BYTES = XBOXES * XROWS * 128;
  static constexpr int STAGE_BYTES = GV_W_BYTES + X_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int RED_FLOATS = GV_CWARPS * 32 * 2 * NT * 4;
  static constexpr int BYTES = 1024 + STAGES * STAGE_BYTES + RED_FLOATS * 4 + 256 * 4 + 2 * STAGES * 8 + 64;
};

template <int NT>
__device__ __forceinline__ uint8_t* gv4_setup(uint64_t*& full, uint64_t*& empty, float*& red, uint32_t*& lut) {
  using C = Gv4Cfg<NT>;
  extern __shared__ uint8_t gv_smem_raw[];
  const uint32_t a = smem_u32(gv_smem_raw);
  uint8_t* base = gv_smem_raw + (((a + 1023u) & ~1023u) - a);
  red = reinterpret_cast<float*>(base + C::STAGES * C::STAGE_BYTES);
  lut = reinterpret_cast<uint32_t*>(red + C::RED_FLOATS);
  full = reinterpret_cast<uint64_t*>(lut + 256);
  empty = full + C::STAGES;
  // byte -> (bf16 of the low nibble, bf16 of the high nibble); e2m1 magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6
  for (int b = threadIdx.x; b < 256; b += blockDim.x) {
    const uint32_t mag[8] = {0x0000u, 0x3F00u, 0x3F80u, 0x3FC0u, 0x4000u, 0x4040u, 0x4080u, 0x40C0u};
    const int lo = b & 15, hi = b >> 4;
    const uint32_t vlo = ((lo & 8) ? 0x8000u : 0u) | mag[lo & 7];
    const uint32_t vhi = ((hi & 8) ? 0x8000u : 0u) | mag[hi & 7];
    lut[b] = vlo | (vhi << 16);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GV_CWARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  return base;
}

// bf16x2 of a group scale: e8m0 (MXFP4) or e4m3 (NVFP4)
template <bool NV>
__device__ __forceinline__ uint32_t gv4_scale2(uint8_t s) {
  uint32_t b;
  if (NV) {
    const __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)s, __NV_E4M3);
    b = __bfloat16_as_ushort(__float2bfloat16(__half2float(__half(hr))));
  } else {
    b = s == 0 ? 0x0040u : (s == 255 ? 0x7FC0u : ((uint32_t)s << 7));
  }
  return b | (b << 16);
}

__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// As gv_stream_tile for packed e2m1 weights; sc8: the weights' group-scale bytes, row-major
// [rows, K / G] (G = 32 MXFP4, 16 NVFP4) indexed by the same row numbers as the tensor map.
template <bool NV, int NT, int WMODE>
__device__ __forceinline__ bool gv4_stream_tile(const CUtensorMap* tmap, const CUtensorMap* xmap, uint8_t* stages,
                                                uint64_t* full, uint64_t* empty, const uint32_t* lut,
                                                uint32_t& phase_base, const int (&row0)[2], int nst, int K,
                                                const uint8_t* __restrict__ sc8, int x_row0, int mcount,
                                                float (&acc)[2][NT][4], XtuStatus* st) {
  using C = Gv4Cfg<NT>;
  constexpr int G = NV ? 16 : 32;
  const int ng = K / G;                       // scale groups per row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  bool ok = true;
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][n][i] = 0.f;
  if (warp == 0) {
    if (elect_one()) {
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const uint32_t it = phase_base + i;
        const int slot = it % C::STAGES;
        if (it >= C::STAGES && !mbar_wait(&empty[slot], ((it / C::STAGES) - 1) & 1, st, 62)) { ok = false; break; }
        ++issued;
        mbar_arrive_expect_tx(&full[slot], C::STAGE_BYTES);
        uint8_t* dst = stages + slot * C::STAGE_BYTES;
        if (WMODE == 0) tma_load_3d(dst, tmap, &full[slot], 0, row0[0], 2 * i);
        else tma_load_4d(dst, tmap, &full[slot], 0, row0[0], 0, 2 * i);
        tma_load_3d(dst + GV_W_BYTES, xmap, &full[slot], 0, x_row0, i * C::XBOXES);
      }
      if (!ok) {
        for (int j = issued > C::STAGES ? issued - C::STAGES : 0; j < issued; ++j) {
          const uint32_t it = phase_base + j;
          mbar_wait(&full[it % C::STAGES], (it / C::STAGES) & 1, nullptr, 0, 50000000ull);
        }
      }
    }
    __syncwarp();
  } else {
    const int cw = warp - 1;
    const int g4 = lane >> 2, tq = lane & 3;
    const int c16 = (cw & 1) * 4 + tq;        // 16-byte chunk of the 128-byte row within box (cw >> 1)
    const int xbox = cw * 2 + (tq >> 1);      // 64-element activation box of this lane's 32 k
    for (int i = 0; i < nst; ++i) {
      const uint32_t it = phase_base + i;
      const int slot = it % C::STAGES;
      // this lane's group scales for rows gv_prow(g4) / + 8 of both 16-row halves (fetched before the wait)
      const int k0 = i * C::KSTAGE + cw * 128 + tq * 32;
      uint32_t s2[2][2][2];                   // [half t][row h][group of the 32 k]
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint8_t* sr = sc8 + (size_t)(row0[t] + gv_prow(g4) + 8 * h) * ng;
          const int gi = min(k0 / G, ng - 1);
          s2[t][h][0] = gv4_scale2<NV>(__ldg(sr + gi));
          s2[t][h][1] = NV ? gv4_scale2<NV>(__ldg(sr + min(gi + 1, ng - 1))) : s2[t][h][0];
        }
      if (!mbar_wait(&full[slot], (it / C::STAGES) & 1, st, 63)) { ok = false; break; }
      const uint8_t* sbase = stages + slot * C::STAGE_BYTES;
      const uint8_t* box = sbase + (cw >> 1) * 4096;
      uint4 w[2][2];
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = t * 16 + gv_prow(g4) + h * 8;
          w[t][h] = *reinterpret_cast<const uint4*>(box + r * 128 + ((c16 ^ (r & 7)) << 4));
        }
      uint4 xr[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int tok = n * 8 + g4;
        const uint8_t* xrow = sbase + GV_W_BYTES + xbox * (C::XROWS * 128) + tok * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = *reinterpret_cast<const uint4*>(xrow + ((((tq & 1) * 4 + q) ^ (tok & 7)) << 4));
          xr[n][q] = tok < mcount ? v : make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const int grp = NV ? (g >> 2) : 0;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          // bytes 2g, 2g+1 of each row's chunk: k = 4g .. 4g + 3
          const uint32_t wa = u4w(w[t][0], g >> 1) >> (16 * (g & 1));
          const uint32_t wb = u4w(w[t][1], g >> 1) >> (16 * (g & 1));
          const uint32_t a0 = bmul2(lut[wa & 0xFF], s2[t][0][grp]);
          const uint32_t a2 = bmul2(lut[(wa >> 8) & 0xFF], s2[t][0][grp]);
          const uint32_t a1 = bmul2(lut[wb & 0xFF], s2[t][1][grp]);
          const uint32_t a3 = bmul2(lut[(wb >> 8) & 0xFF], s2[t][1][grp]);
#pragma unroll
          for (int n = 0; n < NT; ++n)
            mma_bf16_16816(acc[t][n], a0, a1, a2, a3, u4w(xr[n][g >> 1], 2 * (g & 1)),
                           u4w(xr[n][g >> 1], 2 * (g & 1) + 1));
        }
      }
    }
  }
  phase_base += nst;
  return __syncthreads_and(ok);
}

// grouped gate/up + SwiGLU for packed-4-bit experts (token-direct form as moe_gemv_gate_up_kernel)
template <bool NV, int NT>
__global__ void __launch_bounds__(GV_THREADS) moe_gemv4_gate_up_kernel(
    const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap xmap,
    const uint8_t* __restrict__ sc8, const float* __restrict__ gs, int I, int K, const int* __restrict__ seg,
    const int* __restrict__ active, const int* __restrict__ tokrow, int ntok, __nv_bfloat16* __restrict__ h,
    float limit, float alpha, float beta, XtuStatus* st) {
  griddep_wait();
  griddep_launch_dependents();
  const int nact = active[0];
  if ((int)blockIdx.y >= nact) return;
  const int e = active[1 + blockIdx.y];
  const int s0 = seg[e], cnt = seg[e + 1] - s0;
  if (cnt <= 0) return;
  const int* trow = tokrow ? tokrow + blockIdx.y * 16 : nullptr;
  const int xrow0 = trow ? 0 : s0, xcnt = trow ? ntok : cnt;
  uint64_t *full, *empty;
  float* red;
  uint32_t* lut;
  uint8_t* stages = gv4_setup<NT>(full, empty, red, lut);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g4 = lane >> 2, tq = lane & 3;
  const int nst = (K + Gv4Cfg<NT>::KSTAGE - 1) / Gv4Cfg<NT>::KSTAGE;
  const int j0 = blockIdx.x * 16;
  const int grow = (j0 >> 7) * 256 + (j0 & 127);
  const int rows[2] = {e * 2 * I + grow, e * 2 * I + grow + 128};
  const float g_s = NV ? gs[e] : 1.f;
  uint32_t pb = 0;
  for (int mb = 0; mb < xcnt; mb += 8 * NT) {
    const int mc = min(8 * NT, xcnt - mb);
    float acc[2][NT][4];
    if (!gv4_stream_tile<NV, NT, 1>(&tmap, &xmap, stages, full, empty, lut, pb, rows, nst, K, sc8, xrow0 + mb, mc,
                                    acc, st))
      return;
    gv_reduce<NT>(acc, red);
    if (warp != 1) continue;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = j0 + gv_prow(g4) + (i >> 1) * 8;
        const int tok = n * 8 + 2 * tq + (i & 1);
        const int hr = tok >= mc ? -1 : trow ? trow[mb + tok] : s0 + mb + tok;
        if (hr >= 0) {
          float g = acc[0][n][i] * g_s, u = acc[1][n][i] * g_s;
          if (limit > 0.f) { g = fminf(g, limit); u = fminf(fmaxf(u, -limit), limit); }
          h[(size_t)hr * I + j] = __float2bfloat16((g / (1.f + __expf(-alpha * g))) * (u + beta));
        }
      }
  }
}

// grouped down for packed-4-bit experts: out[slot[row]] = w[row] * (h[row] W2[e]^T)
template <bool NV, int NT>
__global__ void __launch_bounds__(GV_THREADS) moe_gemv4_down_kernel(
    const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap xmap,
    const uint8_t* __restrict__ sc8, const float* __restrict__ gs, int H, int I, const int* __restrict__ seg,
    const int* __restrict__ active, const int* __restrict__ perm_slot, const float* __restrict__ perm_w,
    __nv_bfloat16* __restrict__ out, XtuStatus* st) {
  griddep_wait();
  griddep_launch_dependents();
  const int nact = active[0];
  if ((int)blockIdx.y >= nact) return;
  const int e = active[1 + blockIdx.y];
  const int s0 = seg[e], cnt = seg[e + 1] - s0;
  if (cnt <= 0) return;
  uint64_t *full, *empty;
  float* red;
  uint32_t* lut;
  uint8_t* stages = gv4_setup<NT>(full, empty, red, lut);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g4 = lane >> 2, tq = lane & 3;
  const int nst = (I + Gv4Cfg<NT>::KSTAGE - 1) / Gv4Cfg<NT>::KSTAGE;
  const int r0 = blockIdx.x * 32;
  const int rows[2] = {e * H + r0, e * H + r0 + 16};
  const float g_s = NV ? gs[e] : 1.f;
  uint32_t pb = 0;
  for (int mb = 0; mb < cnt; mb += 8 * NT) {
    const int mc = min(8 * NT, cnt - mb);
    float acc[2][NT][4];
    if (!gv4_stream_tile<NV, NT, 0>(&tmap, &xmap, stages, full, empty, lut, pb, rows, nst, I, sc8, s0 + mb, mc, acc,
                                    st))
      return;
    gv_reduce<NT>(acc, red);
    if (warp != 1) continue;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r0 + t * 16 + gv_prow(g4) + (i >> 1) * 8;
          const int tok = n * 8 + 2 * tq + (i & 1);
          if (row < H && tok < mc) {
            const int pr = s0 + mb + tok;
            out[(size_t)perm_slot[pr] * H + row] = __float2bfloat16(acc[t][n][i] * g_s * perm_w[pr]);
          }
        }
  }
}

// Workspace of the dense GEMV: fp32 split-K partials (up to 4 splits x 16 rows x N, used
// only while the tiles do not fill the GPU) followed by the f16 activation scratch.
constexpr long long GV_WS_PART_FLOATS = 1 << 20;
constexpr long long GV_WS_X_HALVES = 1 << 19;

// x [M, K] (row stride `stride`) bf16 -> out [M, K] f16 x 2^-8, one 16-byte chunk per thread
__global__ void gv_x_f16s_kernel(const __nv_bfloat16* __restrict__ x, int M, int K, int stride,
                                 uint4* __restrict__ out) {
  griddep_wait();   // launched with PDL: nothing upstream is touched before this
  griddep_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = K >> 3;
  if (i >= M * per_row) return;
  const int r = i / per_row, c8 = i - r * per_row;
  out[i] = bf16x8_f16x8_s8(*reinterpret_cast<const uint4*>(x + (size_t)r * stride + c8 * 8));
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

typedef CUresult (*PFN_gv_encode)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Tensor maps with 128-byte swizzle whose ONE box is a whole GEMV stage operand, so a
// stage costs two TMA instructions (weights, activations) instead of eight small boxes.
static int gv_tmap_nd(CUtensorMap* map, const void* base, bool u8, int rank, const cuuint64_t* dims,
                      const cuuint64_t* strides, const cuuint32_t* box) {
  static PFN_gv_encode enc = nullptr;
  if (!enc) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      enc = reinterpret_cast<PFN_gv_encode>(p);
    if (!enc) return -100;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return -101;
  for (int i = 0; i < rank - 1; ++i)
    if (strides[i] % 16 != 0) return -101;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, u8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1000 - (int)r;
}

// weights [rows, K] viewed as (128-byte chunk element, row, chunk); one box = 32 rows x 2
// chunks, landing as [chunk][row][128 B].  halves: (element, row, half, chunk) with the
// second half 128 rows down (gate / up blocks of W13); box 16 rows x 2 halves x 2 chunks.
// rows2d: rows whose length is not a multiple of 128 bytes, as 2-D [rows, K] with 16-row boxes.
static int gv_wmap(CUtensorMap* map, const void* W, uint64_t rows, int K, bool fp8, bool halves) {
  const uint64_t eb = fp8 ? 1 : 2, rb = (uint64_t)K * eb;
  if (rb % 128 != 0) {
    if (halves) return -8;
    const cuuint64_t dims[2] = {(cuuint64_t)K, rows};
    const cuuint64_t strides[1] = {rb};
    const cuuint32_t box[2] = {(cuuint32_t)(128 / eb), 16};
    return gv_tmap_nd(map, W, fp8, 2, dims, strides, box);
  }
  const cuuint32_t c = (cuuint32_t)(128 / eb);
  if (!halves) {
    const cuuint64_t dims[3] = {c, rows, rb / 128};
    const cuuint64_t strides[2] = {rb, 128};
    const cuuint32_t box[3] = {c, 32, 2};
    return gv_tmap_nd(map, W, fp8, 3, dims, strides, box);
  }
  const cuuint64_t dims[4] = {c, rows, 2, rb / 128};
  const cuuint64_t strides[3] = {rb, 128 * rb, 128};
  const cuuint32_t box[4] = {c, 16, 2, 2};
  return gv_tmap_nd(map, W, fp8, 4, dims, strides, box);
}

// activations [rows, K] bf16 / f16 (row pitch `pitch` elements) viewed as (element, row,
// 64-element chunk); one box = xrows rows x the stage's chunks, landing as [chunk][row][128 B]
static int gv_xmap(CUtensorMap* map, const void* x, uint64_t rows, int K, int pitch, int xrows, bool fp8) {
  if (K % 64 != 0) return -8;
  if (pitch <= 0) pitch = K;
  const cuuint64_t dims[3] = {64, rows, (cuuint64_t)K / 64};
  const cuuint64_t strides[2] = {(cuuint64_t)pitch * 2, 128};
  const cuuint32_t box[3] = {64, (cuuint32_t)xrows, (cuuint32_t)(fp8 ? 4 : 2)};
  return gv_tmap_nd(map, x, false, 3, dims, strides, box);
}

template <typename Kern>
static int gv_smem_attr(Kern k, int bytes) {
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  return e == cudaSuccess ? 0 : -(int)e;
}

static inline int gv_stages_per_tile(int K, bool fp8) {
  const int kstage = GV_ROW_BYTES / (fp8 ? 1 : 2);
  return (K + kstage - 1) / kstage;
}

// K splits of a dense GEMV whose tiles do not fill the resident CTA slots: as many as
// keep every split in the first wave, at least 2 stages per split, within the workspace
static int gv_splits(int tiles, int S, int N, int slots) {
  if (tiles >= slots) return 1;
  int splits = slots / tiles;
  if (splits > 16) splits = 16;
  while (splits > 1 && (S / splits < 2 || (long long)splits * GV_MAX_ROWS * N > GV_WS_PART_FLOATS)) --splits;
  return splits;
}

// the tcgen05 form of 17..32-row calls; XTU_GEMV_TC=0 keeps them on the warp-level kernel
static bool gv_tc_enabled() {
  static const int on = [] {
    const char* e = getenv("XTU_GEMV_TC");
    return e ? atoi(e) : 1;
  }();
  return on != 0;
}

// bf16 rows -> f16 x 2^-8 rows in the workspace's activation scratch
static const void* gv_convert_x(const void* x, int rows, int K, int stride, float* ws, cudaStream_t s) {
  uint4* x16 = reinterpret_cast<uint4*>(ws + GV_WS_PART_FLOATS);
  const int chunks = rows * (K / 8);
  launch_pdl(gv_x_f16s_kernel, dim3((chunks + 255) / 256), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(x),
             rows, K, stride, x16);
  return x16;
}

extern "C" {

// y[M, N] = x[M, K] W^T (+ bias). fp8: W e4m3 [N, K] + scales [ceil(N/128), ceil(K/128)]; else W bf16.
// fp8 bit 2 (value 4): x already holds the f16 x 2^-8 rows (e.g. from xtu_rmsnorm's y16).
// ws: fp32, GV_WS_PART_FLOATS + GV_WS_X_HALVES / 2 (split-K partials, then the f16 activations
// of fp8 calls); counters: >= 512 ints, zeroed on first use, left zeroed by every launch.
int xtu_gemv(const void* W, const float* wscale, int fp8, int N, int K, const void* x, int x_stride, int M,
             const void* bias, void* y, int y_stride, int y_f32, float* ws, int* counters, void* status,
             cudaStream_t s) {
  const int x_f16s = (fp8 >> 2) & 1;
  fp8 &= 1;
  if (M <= 0 || N <= 0) return 0;
  if (M > GV_MAX_ROWS || K % 16 != 0 || ws == nullptr || counters == nullptr) return -2;
  if (K > GV_MAX_KBLK * 128) return -3;
  if (fp8 && (long long)M * K > GV_WS_X_HALVES) return -4;
  const int nt = M > 16 ? 4 : M > 8 ? 2 : 1;
  const int tiles = (N + 31) / 32;
  const int S = gv_stages_per_tile(K, fp8 != 0);
  int launches = 1;
  if (fp8 && !x_f16s) {   // activations -> f16 x 2^-8 once, not once per CTA and stage
    x = gv_convert_x(x, M, K, x_stride, ws, s);
    x_stride = K;
    ++launches;
  }
  XtuStatus* st = reinterpret_cast<XtuStatus*>(status);
  CUtensorMap tm, xm;
  int rc;
  if (M > 16 && K % 128 == 0 && gv_tc_enabled()) {
    // 17..32 rows: the tcgen05 form (see gemv_tc_kernel)
    const int tiles_tc = (N + 127) / 128, S_tc = K / 128;
    int splits = tiles_tc >= gemv_num_sms() ? 1 : gemv_num_sms() / tiles_tc;
    if (splits > S_tc) splits = S_tc;
    while (splits > 1 && ((splits - 1) * ((S_tc + splits - 1) / splits) >= S_tc ||
                          (long long)splits * GV_MAX_ROWS * N > GV_WS_PART_FLOATS || tiles_tc * 4 > 1024))
      --splits;
    if (fp8) {   // e4m3 [N, K] as (128-byte chunk, row, chunk): one chunk x 128 rows per stage
      const cuuint64_t wdims[3] = {128, (cuuint64_t)N, (cuuint64_t)K / 128};
      const cuuint64_t wstr[2] = {(cuuint64_t)K, 128};
      const cuuint32_t wbox[3] = {128, 128, 1};
      rc = gv_tmap_nd(&tm, W, true, 3, wdims, wstr, wbox);
    } else {     // bf16 [N, K] as (64-element chunk, row, chunk): two chunks x 128 rows per stage
      const cuuint64_t wdims[3] = {64, (cuuint64_t)N, (cuuint64_t)K / 64};
      const cuuint64_t wstr[2] = {(cuuint64_t)K * 2, 128};
      const cuuint32_t wbox[3] = {64, 128, 2};
      rc = gv_tmap_nd(&tm, W, false, 3, wdims, wstr, wbox);
    }
    if (rc) return rc;
    rc = gv_xmap(&xm, x, (uint64_t)M, K, x_stride, 32, false);
    if (rc) return rc;
    static bool init8 = false, init16 = false;
    if (fp8 && !init8) {
      rc = gv_smem_attr(gemv_tc_kernel<true>, GT_SMEM);
      if (rc) return rc;
      init8 = true;
    }
    if (!fp8 && !init16) {
      rc = gv_smem_attr(gemv_tc_kernel<false>, GT_SMEM_BF);
      if (rc) return rc;
      init16 = true;
    }
    if (fp8)
      launch_pdl(gemv_tc_kernel<true>, dim3(tiles_tc, splits), dim3(GT_THREADS), GT_SMEM, s, tm, xm, wscale, N, K,
                 M, (const __nv_bfloat16*)bias, y, y_stride, y_f32, ws, counters, st);
    else
      launch_pdl(gemv_tc_kernel<false>, dim3(tiles_tc, splits), dim3(GT_THREADS), GT_SMEM_BF, s, tm, xm, wscale, N,
                 K, M, (const __nv_bfloat16*)bias, y, y_stride, y_f32, ws, counters, st);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? launches : -(int)e;
  }
  rc = gv_wmap(&tm, W, (uint64_t)N, K, fp8 != 0, false);
  if (rc) return rc;
  rc = gv_xmap(&xm, x, (uint64_t)M, K, x_stride, 8 * nt, fp8 != 0);
  if (rc) return rc;
#define XTU_GEMV_LAUNCH(F, NTV, WMV)                                                                         \
  do {                                                                                                       \
    static int occ = 0;                                                                                      \
    if (!occ) {                                                                                              \
      rc = gv_smem_attr(gemv_dense_kernel<F, NTV, WMV>, GvCfg<F, NTV>::BYTES);                               \
      if (rc) return rc;                                                                                     \
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_dense_kernel<F, NTV, WMV>, GV_THREADS,     \
                                                        GvCfg<F, NTV>::BYTES) != cudaSuccess || occ < 1)      \
        occ = 1;                                                                                             \
    }                                                                                                        \
    const dim3 grid(tiles, gv_splits(tiles, S, N, occ * gemv_num_sms()));                                   \
    launch_pdl(gemv_dense_kernel<F, NTV, WMV>, grid, dim3(GV_THREADS), GvCfg<F, NTV>::BYTES, s, tm, xm, wscale, N, \
               K, M, (const __nv_bfloat16*)bias, y, y_stride, y_f32, ws, counters, st, GvPeer{});            \
  } while (0)
  const bool w2d = ((long long)K * (fp8 ? 1 : 2)) % 128 != 0;
  if (fp8) {
    if (w2d) {
      if (nt == 1) XTU_GEMV_LAUNCH(true, 1, 2); else if (nt == 2) XTU_GEMV_LAUNCH(true, 2, 2);
      else XTU_GEMV_LAUNCH(true, 4, 2);
    } else {
      if (nt == 1) XTU_GEMV_LAUNCH(true, 1, 0); else if (nt == 2) XTU_GEMV_LAUNCH(true, 2, 0);
      else XTU_GEMV_LAUNCH(true, 4, 0);
    }
  } else {
    if (w2d) {
      if (nt == 1) XTU_GEMV_LAUNCH(false, 1, 2); else if (nt == 2) XTU_GEMV_LAUNCH(false, 2, 2);
      else XTU_GEMV_LAUNCH(false, 4, 2);
    } else {
      if (nt == 1) XTU_GEMV_LAUNCH(false, 1, 0); else if (nt == 2) XTU_GEMV_LAUNCH(false, 2, 0);
      else XTU_GEMV_LAUNCH(false, 4, 0);
    }
  }
#undef XTU_GEMV_LAUNCH
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? launches : -(int)e;
}

// Tensor-parallel decode GEMV: this rank's partial y[M, N] = x W^T (W row-parallel slice)
// goes to every rank's receive buffer by peer stores and is summed there by
// xtu_tp_sum_rmsnorm; see GvPeer.  bf16 output, no bias; other arguments as xtu_gemv.
int xtu_gemv_tp(const void* W, const float* wscale, int fp8, int N, int K, const void* x, int x_stride, int M,
                float* ws, int* counters, void* const* dst, long long slot, int rank, int world, int* done,
                void* const* flags, const int* ep_c, int* ep_p, void* status, cudaStream_t s) {
  if (M <= 0 || N <= 0) return 0;
  if (M > 16 || K % 64 != 0 || ws == nullptr || counters == nullptr || (long long)M * N > slot) return -2;
  if (K > GV_MAX_KBLK * 128) return -3;
  if (fp8 && (long long)M * K > GV_WS_X_HALVES) return -4;
  if (world < 1 || world > GV_MAX_WORLD || rank < 0 || rank >= world) return -5;
  const int nt = M > 8 ? 2 : 1;
  const int tiles = (N + 31) / 32;
  const int S = gv_stages_per_tile(K, fp8 != 0);
  int launches = 1;
  if (fp8) {
    x = gv_convert_x(x, M, K, x_stride, ws, s);
    x_stride = K;
    ++launches;
  }
  CUtensorMap tm, xm;
  int rc = gv_wmap(&tm, W, (uint64_t)N, K, fp8 != 0, false);
  if (rc) return rc;
  rc = gv_xmap(&xm, x, (uint64_t)M, K, x_stride, 8 * nt, fp8 != 0);
  if (rc) return rc;
  XtuStatus* st = reinterpret_cast<XtuStatus*>(status);
  GvPeer pr;
  pr.dst = reinterpret_cast<__nv_bfloat16* const*>(dst);
  pr.slot = slot;
  pr.rank = rank;
  pr.world = world;
  pr.done = done;
  pr.flags = reinterpret_cast<int* const*>(flags);
  pr.ep_c = ep_c;
  pr.ep_p = ep_p;
  const bool w2d = ((long long)K * (fp8 ? 1 : 2)) % 128 != 0;
  if (w2d) return -8;
#define XTU_GEMV_TP_LAUNCH(F, NTV)                                                                           \
  do {                                                                                                       \
    static int occ = 0;                                                                                      \
    if (!occ) {                                                                                              \
      rc = gv_smem_attr(gemv_dense_kernel<F, NTV, 0, true>, GvCfg<F, NTV>::BYTES);                           \
      if (rc) return rc;                                                                                     \
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_dense_kernel<F, NTV, 0, true>, GV_THREADS, \
                                                        GvCfg<F, NTV>::BYTES) != cudaSuccess || occ < 1)      \
        occ = 1;                                                                                             \
    }                                                                                                        \
    const dim3 grid(tiles, gv_splits(tiles, S, N, occ * gemv_num_sms()));                                   \
    launch_pdl(gemv_dense_kernel<F, NTV, 0, true>, grid, dim3(GV_THREADS), GvCfg<F, NTV>::BYTES, s, tm, xm,    \
               wscale, N, K, M, (const __nv_bfloat16*)nullptr, (void*)nullptr, 0, 0, ws, counters, st, pr);  \
  } while (0)
  if (fp8) {
    if (nt == 1) XTU_GEMV_TP_LAUNCH(true, 1); else XTU_GEMV_TP_LAUNCH(true, 2);
  } else {
    if (nt == 1) XTU_GEMV_TP_LAUNCH(false, 1); else XTU_GEMV_TP_LAUNCH(false, 2);
  }
#undef XTU_GEMV_TP_LAUNCH
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? launches : -(int)e;
}

// grouped decode MoE: gate/up+SwiGLU then down+weight+scatter.  mmax bounds the rows of
// any one expert (<= 16); max_active bounds the experts with rows (min(E, tokens * top_k));
// n_rows: rows of the permuted activations xp [n_rows, H] and of h [n_rows, I].
// tokrow (nullable, from moe_permute_decode): xp is then the step's ntok <= 16 tokens
// [ntok, H] with row stride x_stride, not gathered per expert;
// active: E + 1 ints, filled here from seg unless active_ready says the caller already
// holds the list there; ws as for xtu_gemv (its activation scratch only).  fp8:
// xp_f16s says xp already holds f16 x 2^-8 rows (moe_permute's form); h is written in
// that form too.
int xtu_moe_gemv(const void* W13, const float* s13, const void* W2, const float* s2, int fp8, int E, int H, int I,
                 const void* xp, int xp_f16s, int x_stride, const int* tokrow, int ntok, const int* seg,
                 const int* perm_slot, const float* perm_w, void* h,
                 void* slots, int mmax, int max_active, int n_rows, int* active, int active_ready, float limit,
                 float alpha, float beta, const void* W13s, const float* s13s, const void* W2s, const float* s2s,
                 int sh_out0, float* ws, void* status, cudaStream_t s) {
  if (mmax <= 0 || n_rows <= 0) return 0;
  if (mmax > 16 || H % 32 != 0 || I % 128 != 0 || active == nullptr) return -2;
  if (H > GV_MAX_KBLK * 128 || I > GV_MAX_KBLK * 128) return -3;
  if (max_active <= 0 || max_active > E) max_active = E;
  const int nt = mmax > 8 ? 2 : 1;
  int launches = 3;
  if (tokrow && (ntok <= 0 || ntok > 16 || ntok > mmax)) return -2;
  // shared expert: one more grid row in both launches over the step's ntok tokens, its h
  // rows after the pairs' (n_rows + token), its output rows sh_out0 + token of slots.  Its
  // activations: the step's tokens (token-direct form) or xp rows n_rows .. n_rows + ntok
  // (gathered form: xtu_moe_gather_rows writes them after the permuted rows)
  const int has_sh = (W13s != nullptr && W2s != nullptr) ? 1 : 0;
  if (has_sh && ntok <= 0) return -2;
  const int x_rows = tokrow ? ntok : n_rows + (has_sh ? ntok : 0);
  if (x_stride <= 0) x_stride = H;
  if (fp8 && !xp_f16s) {
    if (ws == nullptr || (long long)x_rows * H > GV_WS_X_HALVES) return -4;
    xp = gv_convert_x(xp, x_rows, H, x_stride, ws, s);
    x_stride = H;
    ++launches;
  }
  CUtensorMap t13, t2, xm, hm;
  int rc = gv_wmap(&t13, W13, (uint64_t)E * 2 * I, H, fp8 != 0, true);
  if (rc) return rc;
  rc = gv_wmap(&t2, W2, (uint64_t)E * H, I, fp8 != 0, false);
  if (rc) return rc;
  rc = gv_xmap(&xm, xp, (uint64_t)x_rows, H, x_stride, 8 * nt, fp8 != 0);
  if (rc) return rc;
  CUtensorMap t13s = t13, t2s = t2;
  if (has_sh) {
    rc = gv_wmap(&t13s, W13s, (uint64_t)2 * I, H, fp8 != 0, true);
    if (rc) return rc;
    rc = gv_wmap(&t2s, W2s, (uint64_t)H, I, fp8 != 0, false);
    if (rc) return rc;
  }
  rc = gv_xmap(&hm, h, (uint64_t)n_rows + (has_sh ? ntok : 0), I, I, 8 * nt, fp8 != 0);
  if (rc) return rc;
  if (!active_ready) launch_pdl(moe_active_kernel, dim3(1), dim3(32), 0, s, seg, E, active);
  else --launches;
  XtuStatus* st = reinterpret_cast<XtuStatus*>(status);
  const dim3 g1(I / 16, max_active + has_sh), g2((H + 31) / 32, max_active + has_sh);
#define XTU_MOE_GEMV_LAUNCH(F, NTV)                                                                          \
  do {                                                                                                       \
    static bool init = false;                                                                                \
    if (!init) {                                                                                             \
      rc = gv_smem_attr(moe_gemv_gate_up_kernel<F, NTV>, GvCfg<F, NTV>::BYTES);                              \
      if (!rc) rc = gv_smem_attr(moe_gemv_down_kernel<F, NTV>, GvCfg<F, NTV>::BYTES);                        \
      if (rc) return rc;                                                                                     \
      init = true;                                                                                           \
    }                                                                                                        \
    launch_pdl(moe_gemv_gate_up_kernel<F, NTV>, g1, dim3(GV_THREADS), GvCfg<F, NTV>::BYTES, s, t13, xm, s13, I, \
               H, seg, active, tokrow, ntok, (__nv_bfloat16*)h, limit, alpha, beta, t13s, s13s, n_rows, has_sh, \
               st);                                                                                          \
    launch_pdl(moe_gemv_down_kernel<F, NTV>, g2, dim3(GV_THREADS), GvCfg<F, NTV>::BYTES, s, t2, hm, s2, H, I,    \
               seg, active, perm_slot, perm_w, (__nv_bfloat16*)slots, t2s, s2s, n_rows, sh_out0, ntok, has_sh,   \
               st);                                                                                          \
  } while (0)
  if (fp8) {
    if (nt == 1) XTU_MOE_GEMV_LAUNCH(true, 1); else XTU_MOE_GEMV_LAUNCH(true, 2);
  } else {
    if (nt == 1) XTU_MOE_GEMV_LAUNCH(false, 1); else XTU_MOE_GEMV_LAUNCH(false, 2);
  }
#undef XTU_MOE_GEMV_LAUNCH
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? launches : -(int)e;
}


// packed-4-bit grouped decode MoE (MXFP4: fmt 2, scales e8m0 per 32 k; NVFP4: fmt 3, scales
// e4m3 per 16 k and per-expert fp32 global scales gs13 / gs2).  W13 [E, 2I, H/2] bytes with
// gate/up rows interleaved in 128-row blocks, W2 [E, H, I/2]; scales row-major per weight row.
// xp: bf16 activations (tokrow: the step's ntok <= 16 tokens, token-direct; else permuted
// rows); h: bf16 [n_rows, I]; slots: bf16 output rows.  Other arguments as xtu_moe_gemv.
int xtu_moe_gemv4(const void* W13, const void* s13, const float* gs13, const void* W2, const void* s2,
                  const float* gs2, int fmt, int E, int H, int I, const void* xp, int x_stride, const int* tokrow,
                  int ntok, const int* seg, const int* perm_slot, const float* perm_w, void* h, void* slots, int mmax,
                  int max_active, int n_rows, int* active, int active_ready, float limit, float alpha, float beta,
                  void* status, cudaStream_t s) {
  if (mmax <= 0 || n_rows <= 0) return 0;
  if (fmt != 2 && fmt != 3) return -9;
  if (mmax > 16 || H % 256 != 0 || I % 256 != 0 || active == nullptr || s13 == nullptr || s2 == nullptr) return -2;
  if (fmt == 3 && (gs13 == nullptr || gs2 == nullptr)) return -8;
  if (tokrow && (ntok <= 0 || ntok > 16 || ntok > mmax)) return -2;
  if (max_active <= 0 || max_active > E) max_active = E;
  const int nt = mmax > 8 ? 2 : 1;
  const int x_rows = tokrow ? ntok : n_rows;
  if (x_stride <= 0) x_stride = H;
  CUtensorMap t13, t2, xm, hm;
  int rc = gv_wmap(&t13, W13, (uint64_t)E * 2 * I, H / 2, true, true);
  if (rc) return rc;
  rc = gv_wmap(&t2, W2, (uint64_t)E * H, I / 2, true, false);
  if (rc) return rc;
  {
    const cuuint64_t dims[3] = {64, (cuuint64_t)x_rows, (cuuint64_t)H / 64};
    const cuuint64_t strides[2] = {(cuuint64_t)x_stride * 2, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)(8 * nt), 8};
    rc = gv_tmap_nd(&xm, xp, false, 3, dims, strides, box);
    if (rc) return rc;
    const cuuint64_t hdims[3] = {64, (cuuint64_t)n_rows, (cuuint64_t)I / 64};
    const cuuint64_t hstrides[2] = {(cuuint64_t)I * 2, 128};
    rc = gv_tmap_nd(&hm, h, false, 3, hdims, hstrides, box);
    if (rc) return rc;
  }
  int launches = 2;
  if (!active_ready) {
    launch_pdl(moe_active_kernel, dim3(1), dim3(32), 0, s, seg, E, active);
    ++launches;
  }
  XtuStatus* st = reinterpret_cast<XtuStatus*>(status);
  const uint8_t* sc13 = reinterpret_cast<const uint8_t*>(s13);
  const uint8_t* sc2 = reinterpret_cast<const uint8_t*>(s2);
  const dim3 g1(I / 16, max_active), g2(H / 32, max_active);
#define XTU_MOE_GEMV4_LAUNCH(NVV, NTV)                                                                        \
  do {                                                                                                       \
    static bool init = false;                                                                                \
    if (!init) {                                                                                             \
      rc = gv_smem_attr(moe_gemv4_gate_up_kernel<NVV, NTV>, Gv4Cfg<NTV>::BYTES);                              \
      if (!rc) rc = gv_smem_attr(moe_gemv4_down_kernel<NVV, NTV>, Gv4Cfg<NTV>::BYTES);                        \
      if (rc) return rc;                                                                                     \
      init = true;                                                                                           \
    }                                                                                                        \
    launch_pdl(moe_gemv4_gate_up_kernel<NVV, NTV>, g1, dim3(GV_THREADS), Gv4Cfg<NTV>::BYTES, s, t13, xm, sc13, \
               gs13, I, H, seg, active, tokrow, ntok, (__nv_bfloat16*)h, limit, alpha, beta, st);             \
    launch_pdl(moe_gemv4_down_kernel<NVV, NTV>, g2, dim3(GV_THREADS), Gv4Cfg<NTV>::BYTES, s, t2, hm, sc2, gs2, \
               H, I, seg, active, perm_slot, perm_w, (__nv_bfloat16*)slots, st);                              \
  } while (0)
  if (fmt == 3) {
    if (nt == 1) XTU_MOE_GEMV4_LAUNCH(true, 1); else XTU_MOE_GEMV4_LAUNCH(true, 2);
  } else {
    if (nt == 1) XTU_MOE_GEMV4_LAUNCH(false, 1); else XTU_MOE_GEMV4_LAUNCH(false, 2);
  }
#undef XTU_MOE_GEMV4_LAUNCH
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? launches : -(int)e;
}

}  // extern "C"
