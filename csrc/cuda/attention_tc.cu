// Paged causal flash attention on the 5th-generation tensor cores (sm_100a).
//
// One CTA = one 128-row query tile of one (sequence, kv head[, kv split]).
// Rows pack the G = Hq/Hkv query heads that share a KV head: row r holds
// (position i = r / G, head g = r % G), so every K/V tile fetched from HBM is
// used by all heads of the group (GQA decode and prefill read KV once per group).
//
// Pipeline (warp specialised, 192 threads):
//   warp 0     TMA producer: K/V tiles of BN keys from the paged cache
//              ([blocks, Hkv, 64, D] bf16, one 64-key block per TMA box row range)
//   warp 1     TMEM owner + MMA issuer:
//                S_j = Q K_j^T        (kind::f16, A = Q smem K-major, B = K smem K-major) -> TMEM S[j%2]
//                O  += P_{j-1} V_{j-1} (A = P smem K-major, B = V smem MN-major)         -> TMEM O
//              so the tensor core computes S_{j} while softmax works on S_{j-1}.
//   warps 2..5 softmax (one thread per row): TMEM S -> scale, causal mask, online
//              max / sum in the exp2 domain, P (bf16) -> 128B-swizzled smem.
//              The running max is only raised when it grows by more than 2^8,
//              so O (in TMEM) is rescaled rarely; the rescale waits for the
//              previous PV MMA.  Finally O / l -> bf16 output, or (split-KV)
//              unnormalised partials + log-sum-exp for attn_combine_kernel.
//
// Replaces the reference's SM80 Triton paged / sparse-MLA kernels
// (patches/upstream/pr3-sm80-port.patch:4000-7300) and vLLM's FlashAttention
// usage for GQA (the reference calls vLLM for all non-MoE attention).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdlib>
#include <cstdint>
#include <cfloat>
#include "ptx.cuh"

namespace xtu {

constexpr int KV_BLOCK = 64;   // tokens per paged-cache block (one TMA box height)

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct AttnParams {
  const __nv_bfloat16* q;  // [T, Hq, D]
  int q_stride;            // elements between tokens
  __nv_bfloat16* o;        // [T, Hq, DV]
  int o_stride;
  const int* q_start;      // [B+1]
  const int* kv_len;       // [B]
  const int* block_table;  // [B, bt_stride]
  int bt_stride;
  int Hq, Hkv, G, rows_per_tile;  // rows_per_tile = (128 / G) * G
  int rf;                  // row replication factor (1, 2, 4): replicas split each tile's keys
  float scale_log2;        // softmax scale * log2(e)
  int splits;
  int dv_total, dv_halves;  // output width per head; CTAs that split it (MLA: 2 x 256 of 512)
  float* ws_o;             // [splits, T, Hq, dv_total] (splits > 1)
  float* ws_lse;           // [splits, T, Hq]
  int T;
  int window;              // > 0: a query at position t sees keys (t - window, t] only
  const float* sinks;      // [Hq] learned sink logits (softmax scale applied), or null
  XtuStatus* status;
};

// STAGES: K/V ring depth.  BTS: block-table entries staged in shared memory (0 = read
// the table from global memory on the fly); decode configurations prefetch the CTA's
// whole block list so the producer never waits on a dependent global load.
// VK: V is the first dims of K (MLA latent cache) and is read from the K stage itself;
// the CTA then computes DV output columns starting at its half's offset.
template <int D, int DV, int BN, int STAGES_ = 2, int BTS = 0, int VK = 0, int CS = 1>
struct AttnCfg {
  static constexpr int STAGES = STAGES_;
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int K_BYTES = BN * D * 2;
  static constexpr int V_BYTES = VK ? 0 : BN * DV * 2;
  static constexpr int P_BYTES = 128 * (BN < 64 ? 64 : BN) * 2;   // rows padded to one 128-B swizzle atom
  static constexpr int BT_BYTES = BTS * 4;
  static constexpr int SMEM = Q_BYTES + STAGES * (K_BYTES + V_BYTES) + 2 * P_BYTES + BT_BYTES + 1024 + 256;
  static constexpr int S_COL0 = 0;          // two S buffers: [0, BN), [BN, 2BN)
  static constexpr int O_COL0 = 2 * BN;     // O: [2BN, 2BN + DV)
  static constexpr int XC = 2 * BN + DV;    // CS > 1: 2 * CS exchange columns from XC
  static constexpr int TMEM_COLS = (XC + (CS > 1 ? 2 * CS : 0)) <= 256 ? 256 : 512;
  static constexpr int THREADS = 64 + 128 * CS;
  static_assert(2 * BN + DV <= 512, "TMEM budget");
  static_assert(CS == 1 || XC + 2 * CS <= TMEM_COLS, "exchange columns");
  static_assert(CS == 1 || ((BN / CS) % 16 == 0 && (DV / CS) % 32 == 0 && VK == 0), "column split");
  static_assert(D % 64 == 0 && DV % 64 == 0 && BN % 16 == 0 && (BN % 64 == 0 || 64 % BN == 0), "tile shapes");
};

// write 8 bf16 (16 B) at (row, col8) of a K-major SW128 operand tile [rows][64-col chunks]
__device__ __forceinline__ void st_sw128(uint8_t* tile, int rows, int row, int col, uint4 v) {
  const int chunk = col >> 6;          // 64-element chunk
  const int piece = (col & 63) >> 3;   // 16-byte piece in the 128-byte row
  uint8_t* base = tile + (size_t)chunk * rows * 128 + row * 128;
  *reinterpret_cast<uint4*>(base + ((piece ^ (row & 7)) << 4)) = v;
}

// EXT: the sliding window and the sinks of AttnParams are honoured (EXT = 0 compiles the
// plain causal kernel, whose softmax loop carries no extra compare).
// CS: softmax warps per TMEM lane quarter.  CS > 1 gives each row CS threads in CS warps
// (4 * CS softmax warps, CS per scheduler), each scoring 1/CS of every tile's keys; per
// tile they swap their partial row max through 2 * CS spare TMEM columns (an mbarrier
// round, bounded like every wait here), so all keep the same running max, and they swap
// their partial sums once at the end.  Each part rescales and writes 1/CS of O's columns.
template <int D, int DV, int BN, int STAGES_, int BTS, int VK, int EXT, int CS>
__global__ void __launch_bounds__(64 + 128 * CS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                    AttnParams p) {
  using C = AttnCfg<D, DV, BN, STAGES_, BTS, VK, CS>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;                       // [STAGES][K_BYTES]
  uint8_t* sV = sK + C::STAGES * C::K_BYTES;           // [STAGES][V_BYTES]
  uint8_t* sP = sV + C::STAGES * C::V_BYTES;           // [2][P_BYTES]
  int* sBT = reinterpret_cast<int*>(sP + 2 * C::P_BYTES);      // [BTS]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P_BYTES + C::BT_BYTES);
  uint64_t* kv_full = bars;                          // [STAGES]
  uint64_t* kv_empty = bars + C::STAGES;             // [STAGES]
  uint64_t* q_ready = bars + 2 * C::STAGES;
  uint64_t* s_full = q_ready + 1;                    // [2]
  uint64_t* p_full = s_full + 2;                     // [2]
  uint64_t* o_done = p_full + 2;                     // [2]
  uint64_t* xb = o_done + 2;                         // [2] CS > 1: partial-max exchange rounds
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xb + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int kvh = blockIdx.y % p.Hkv;
  const int split = (blockIdx.y / p.Hkv) % p.splits;
  const int dv_off = VK ? (blockIdx.y / (p.Hkv * p.splits)) * DV : 0;   // this CTA's output columns
  const int dv_tot = p.dv_total;
  const int q0 = p.q_start[b];
  const int q_len = p.q_start[b + 1] - q0;
  const int kv_len = p.kv_len[b];
  const int pos_per_tile = p.rows_per_tile / p.G;
  const int i0 = blockIdx.x * pos_per_tile;          // first query position (relative) of this tile
  if (i0 >= q_len) return;                           // uniform across the CTA
  const int n_pos = min(pos_per_tile, q_len - i0);
  const int ctx0 = kv_len - q_len;                   // absolute position of query 0
  const int max_pos = ctx0 + i0 + n_pos - 1;
  const int n_tiles_all = (max_pos + BN) / BN;       // keys [0, max_pos]
  // sliding window: the tile's first query sees nothing below ctx0 + i0 - window + 1
  const int t_first = (EXT && p.window > 0) ? max(0, ctx0 + i0 - p.window + 1) / BN : 0;
  const int per = (n_tiles_all - t_first + p.splits - 1) / p.splits;
  const int t_begin = t_first + split * per;
  const int t_end = min(n_tiles_all, t_begin + per);
  const int n_tiles = max(0, t_end - t_begin);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
    for (int s = 0; s < C::STAGES; ++s) { mbar_init(&kv_full[s], 1); mbar_init(&kv_empty[s], 1); }
    mbar_init(q_ready, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4 * CS);
      mbar_init(&o_done[i], 1);
      mbar_init(&xb[i], 4 * CS);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  const int n_blocks_seq = (kv_len + KV_BLOCK - 1) / KV_BLOCK;
  const int lb0 = (t_begin * BN) / KV_BLOCK;                       // first logical block of this CTA
  const int n_lb = n_tiles > 0 ? (t_end * BN + KV_BLOCK - 1) / KV_BLOCK - lb0 : 0;
  if (BTS > 0 && warp == 0) {
    const int* bt = p.block_table + (size_t)b * p.bt_stride;
    for (int i = lane; i < n_lb && i < BTS; i += 32) {
      const int lb = lb0 + i;
      sBT[i] = bt[lb < n_blocks_seq ? lb : 0];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one() && n_tiles > 0) {
      const int* bt = p.block_table + (size_t)b * p.bt_stride;
      for (int jj = 0; jj < n_tiles; ++jj) {
        const int stage = jj % C::STAGES;
        const uint32_t ph = (jj / C::STAGES) & 1;
        if (!mbar_wait(&kv_empty[stage], ph ^ 1u, p.status, 100)) break;
        mbar_arrive_expect_tx(&kv_full[stage], C::K_BYTES + C::V_BYTES);
        const int j = t_begin + jj;
        if (BN < KV_BLOCK) {
          // a tile is a slice of one 64-token block (the tensor map's box is BN rows)
          int lb = (j * BN) / KV_BLOCK;
          const int off = (j * BN) % KV_BLOCK;
          int blk;
          if (BTS > 0 && lb - lb0 < BTS) {
            blk = sBT[lb - lb0];
          } else {
            if (lb >= n_blocks_seq) lb = 0;
            blk = bt[lb];
          }
          const int row = (blk * p.Hkv + kvh) * KV_BLOCK + off;
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_2d(sK + stage * C::K_BYTES + c * (BN * 128), &tmap_k, &kv_full[stage], c * 64, row);
          if (!VK) {
#pragma unroll
            for (int c = 0; c < DV / 64; ++c)
              tma_load_2d(sV + stage * C::V_BYTES + c * (BN * 128), &tmap_v, &kv_full[stage], c * 64, row);
          }
          continue;
        }
#pragma unroll
        for (int sb = 0; sb < BN / KV_BLOCK; ++sb) {
          int lb = j * (BN / KV_BLOCK) + sb;
          int blk;
          if (BTS > 0 && lb - lb0 < BTS) {
            blk = sBT[lb - lb0];                       // staged (entries past the end hold block 0)
          } else {
            if (lb >= n_blocks_seq) lb = 0;            // past the end: any valid block, masked later
            blk = bt[lb];
          }
          const int row = (blk * p.Hkv + kvh) * KV_BLOCK;
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_2d(sK + stage * C::K_BYTES + c * (BN * 128) + sb * (KV_BLOCK * 128), &tmap_k, &kv_full[stage],
                        c * 64, row);
          if (!VK) {
#pragma unroll
            for (int c = 0; c < DV / 64; ++c)
              tma_load_2d(sV + stage * C::V_BYTES + c * (BN * 128) + sb * (KV_BLOCK * 128), &tmap_v,
                          &kv_full[stage], c * 64, row);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one() && n_tiles > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, BN, 0, 0);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, DV, 0, 1);
      bool ok = mbar_wait(q_ready, 0, p.status, 110);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      for (int jj = 0; jj <= n_tiles && ok; ++jj) {
        if (jj < n_tiles) {
          const int stage = jj % C::STAGES;
          if (!mbar_wait(&kv_full[stage], (jj / C::STAGES) & 1, p.status, 111)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + stage * C::K_BYTES);
          const uint32_t s_tmem = tmem + C::S_COL0 + (jj & 1) * BN;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = (k >> 2) * (BN * 128) + (k & 3) * 32;
            const uint32_t qoff = (k >> 2) * (128 * 128) + (k & 3) * 32;
            mma_f16_ss(s_tmem, sdesc_kmajor_sw128(q_addr + qoff), sdesc_kmajor_sw128(k_addr + off), idesc_s,
                       k > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[jj & 1]);
        }
        if (jj >= 1) {
          const int pj = jj - 1;
          if (!mbar_wait(&p_full[pj & 1], (pj >> 1) & 1, p.status, 112)) { ok = false; break; }
          tc_fence_after();
          const int stage = pj % C::STAGES;
          const uint32_t v_addr = VK ? smem_u32(sK + stage * C::K_BYTES + (dv_off / 64) * (BN * 128))
                                     : smem_u32(sV + stage * C::V_BYTES);
          const uint32_t p_addr = smem_u32(sP + (pj & 1) * C::P_BYTES);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k) {
            const uint32_t aoff = (k >> 2) * (128 * 128) + (k & 3) * 32;
            const uint64_t bd = sdesc_mnmajor_sw128(v_addr + k * 16 * 128, BN * 128, 1024);
            mma_f16_ss(tmem + C::O_COL0, sdesc_kmajor_sw128(p_addr + aoff), bd, idesc_o, (pj > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&o_done[pj & 1]);
          mma_commit(&kv_empty[stage]);
        }
      }
      if (!ok) {
        mma_commit(&o_done[0]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue (warps 2..5)
    // Row layout.  r = TMEM lane / MMA row.  With few valid query rows (decode), each
    // logical row is replicated into RF lane quarters and replica `part` only scores
    // keys [part*KP, (part+1)*KP) of every tile, so RF warps share one row's keys; the
    // replicas' (max, sum, O) are merged in the epilogue.
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const int half = CS > 1 ? (warp - 2) >> 2 : 0;   // CS > 1: which part of each tile's keys
    const int RF = CS > 1 ? 1 : p.rf;
    const int LR = 128 / RF;                 // logical rows
    constexpr int KPC = BN / CS;
    const int KP = CS > 1 ? KPC : BN / RF;   // keys per replica (or per half) per tile
    const int lr = r % LR;
    const int part = r / LR;
    const int rows_valid_all = min(p.rows_per_tile, n_pos * p.G);
    const int pi = lr / p.G, g = lr - (lr / p.G) * p.G;
    const bool row_valid = lr < rows_valid_all;
    const int tok = q0 + i0 + pi;
    const int head = kvh * p.G + g;
    const int qpos = ctx0 + i0 + pi;
    // load this row of Q into swizzled smem (the first half's warps)
    if (half == 0) {
      const __nv_bfloat16* src = p.q + (size_t)tok * p.q_stride + (size_t)head * D;
#pragma unroll 4
      for (int c8 = 0; c8 < D; c8 += 8) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row_valid) v = *reinterpret_cast<const uint4*>(src + c8);
        st_sw128(sQ, 128, r, c8, v);
      }
    }
    float m = -FLT_MAX;   // running max (log2 domain); -FLT_MAX = none yet
    float l = 0.f;
    const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
    // A warp whose 32 rows are all padding skips the softmax and only keeps the barrier
    // phases in step.  Rows whose P is written only in part (replicas) or never
    // (padding) start from zeroed P buffers.
    const bool warp_active = ((qd * 32) % LR) < rows_valid_all;
    if (RF > 1 || !warp_active) {
#pragma unroll 1
      for (int c8 = half * KPC; c8 < (half + 1) * KPC; c8 += 8) {
        st_sw128(sP, 128, r, c8, make_uint4(0, 0, 0, 0));
        st_sw128(sP + C::P_BYTES, 128, r, c8, make_uint4(0, 0, 0, 0));
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && half == 0) mbar_arrive(q_ready);
    bool ok = true;
    // CS > 1: combine one float with the other parts' threads of this row, as a max or a
    // sum (exchange round `rd`; the two column groups alternate, so a column is rewritten
    // only after every part has read it)
    auto xchg = [&](int rd, float mine, bool is_max) -> float {
      const uint32_t col = C::XC + CS * (rd & 1);
      tmem_st1(lane_base + col + half, __float_as_uint(mine));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&xb[rd & 1]);
      if (!__all_sync(0xffffffffu, mbar_wait(&xb[rd & 1], (rd >> 1) & 1, p.status, 124))) {
        ok = false;
        return mine;
      }
      tc_fence_after();
      uint32_t v[CS];
#pragma unroll
      for (int q = 0; q < CS; ++q) v[q] = tmem_ld1(lane_base + col + q);
      tmem_wait_ld();
      float acc = is_max ? -FLT_MAX : 0.f;     // every part in part order: identical in all
#pragma unroll
      for (int q = 0; q < CS; ++q) acc = is_max ? fmaxf(acc, __uint_as_float(v[q])) : acc + __uint_as_float(v[q]);
      return acc;
    };
    for (int jj = 0; jj < n_tiles && ok; ++jj) {
      const int j = t_begin + jj;
      if (!mbar_wait(&s_full[jj & 1], (jj >> 1) & 1, p.status, 120)) { ok = false; break; }
      if (!warp_active) {
        if (CS > 1) (void)xchg(jj, -FLT_MAX, true);   // keep the exchange rounds in step
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[jj & 1]);
        continue;
      }
      tc_fence_after();
      const uint32_t s_addr = lane_base + C::S_COL0 + (jj & 1) * BN;
      const int key0 = j * BN;
      const int c_lo = CS > 1 ? half * KPC : part * KP;
      // this replica's (half's) S columns -> registers, one TMEM round trip per tile.  KP is
      // a multiple of 16 (BN >= 64, RF <= 4), so 16-column chunks never pass the range.
      uint32_t sv[KPC];
#pragma unroll
      for (int ch = 0; ch < KPC / 16; ++ch)
        if (ch * 16 < KP) tmem_ld16p(s_addr + c_lo + ch * 16, sv + ch * 16);
      tmem_wait_ld();
      // keys t <= lim of the range are visible to this row (causal limit; kv_len follows from it)
      const int lim = row_valid ? qpos - (key0 + c_lo) : -1;
      // sliding window: keys t >= low are visible too (low <= 0: the whole range)
      const int low = (EXT && p.window > 0) ? qpos - p.window + 1 - (key0 + c_lo) : 0;
      const bool all_vis = __all_sync(0xffffffffu, lim >= KP - 1 && (!EXT || low <= 0));
      float mx4[4] = {-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX};
      if (CS > 1 && all_vis) {
        // whole range visible: two keys per three-input max (half the ALU instructions)
#pragma unroll
        for (int i = 0; i < KPC; i += 2)
          mx4[(i >> 1) & 3] = fmax3(mx4[(i >> 1) & 3], __uint_as_float(sv[i]), __uint_as_float(sv[i + 1]));
      } else {
#pragma unroll
        for (int ch = 0; ch < KPC / 16; ++ch) {
          if (ch * 16 < KP) {
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              const int i = ch * 16 + t;
              if (all_vis || (i <= lim && (!EXT || i >= low))) mx4[t & 3] = fmaxf(mx4[t & 3], __uint_as_float(sv[i]));
            }
          }
        }
      }
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      if (mx != -FLT_MAX) mx *= p.scale_log2;   // scale > 0: max commutes with it
      if (CS > 1) {
        mx = xchg(jj, mx, true);                   // the row's max over all parts
        if (!ok) break;
      }
      // Raise the running max only when it grows by more than 2^8.  tcgen05.ld/st are
      // warp-collective (.sync.aligned), so the O rescale is decided per warp: if any
      // row of the warp needs it, the whole warp rescales (alpha = 1 for the others).
      const bool raise = (mx > m + 8.f) || (m == -FLT_MAX && mx != -FLT_MAX);
      const float m_new = raise ? fmaxf(mx, m) : m;
      const bool lane_rescale = raise && m != -FLT_MAX && jj >= 1;
      if (__any_sync(0xffffffffu, lane_rescale)) {
        // O holds PV_{jj-1} once that MMA has completed
        if (!mbar_wait(&o_done[(jj - 1) & 1], ((jj - 1) >> 1) & 1, p.status, 121)) { ok = false; }
        __syncwarp();
        if (__any_sync(0xffffffffu, !ok)) break;
        tc_fence_after();
        const float alpha = lane_rescale ? ex2(m - m_new) : 1.f;
        l *= alpha;
#pragma unroll 1
        for (int c = half * (DV / CS); c < (half + 1) * (DV / CS); c += 16) {
          uint32_t o16[16];
          tmem_ld16(lane_base + C::O_COL0 + c, o16);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 16; ++t) o16[t] = __float_as_uint(__uint_as_float(o16[t]) * alpha);
          tmem_st16(lane_base + C::O_COL0 + c, o16);
        }
        tmem_wait_st();
      }
      m = m_new;
      const float m_use = m;
      // P buffer (jj & 1) is free once PV_{jj-2} completed
      if (jj >= 2) {
        if (!mbar_wait(&o_done[jj & 1], ((jj - 2) >> 1) & 1, p.status, 122)) { ok = false; break; }
      }
      uint8_t* pbuf = sP + (jj & 1) * C::P_BYTES;
      const float neg_m = -m_use;
      const bool live = row_valid && m_use != -FLT_MAX;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ch = 0; ch < KPC / 16; ++ch) {
        if (ch * 16 < KP) {
          uint32_t pk[8];
#pragma unroll
          for (int t = 0; t < 16; t += 2) {
            const int i = ch * 16 + t;
            float e0 = ex2(fmaf(__uint_as_float(sv[i]), p.scale_log2, neg_m));
            float e1 = ex2(fmaf(__uint_as_float(sv[i + 1]), p.scale_log2, neg_m));
            if (!all_vis) {
              e0 = (live && i <= lim && (!EXT || i >= low)) ? e0 : 0.f;
              e1 = (live && i + 1 <= lim && (!EXT || i + 1 >= low)) ? e1 : 0.f;
            }
            rs4[(t >> 1) & 3] += e0 + e1;
            pk[t >> 1] = pack_bf16x2(e0, e1);
          }
          const int c = c_lo + ch * 16;
          st_sw128(pbuf, 128, r, c, make_uint4(pk[0], pk[1], pk[2], pk[3]));
          st_sw128(pbuf, 128, r, c + 8, make_uint4(pk[4], pk[5], pk[6], pk[7]));
        }
      }
      const float rs = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      l += rs;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[jj & 1]);
    }
    // ---- epilogue
    const int last = n_tiles - 1;
    bool have_o = false;
    if (n_tiles > 0 && warp_active && ok) {
      have_o = mbar_wait(&o_done[last & 1], (last >> 1) & 1, p.status, 123);
      tc_fence_after();
    }
    if (CS > 1 && n_tiles > 0 && ok) l = xchg(n_tiles, l, false);   // the row's sum over all parts
    if (CS > 1 && !ok) have_o = false;
    // the sink joins the softmax denominator once: here when there is one split, else in
    // attn_combine_kernel
    const float sink_l2 = (EXT && p.sinks != nullptr && p.splits == 1 && row_valid)
                              ? __ldg(p.sinks + head) * 1.4426950408889634f : -FLT_MAX;
    if (RF == 1) {
      if (have_o) {
        if (sink_l2 != -FLT_MAX && m != -FLT_MAX) l += ex2(sink_l2 - m);
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
        for (int c = half * (DV / CS); c < (half + 1) * (DV / CS); c += 32) {
          uint32_t v[32];
          tmem_ld32(lane_base + C::O_COL0 + c, v);
          tmem_wait_ld();
          if (!row_valid) continue;
          if (p.splits == 1) {
            __nv_bfloat16* dst = p.o + (size_t)tok * p.o_stride + (size_t)head * dv_tot + dv_off;
            uint32_t pk[16];
#pragma unroll
            for (int t = 0; t < 16; ++t)
              pk[t] = pack_bf16x2(__uint_as_float(v[2 * t]) * inv, __uint_as_float(v[2 * t + 1]) * inv);
            uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
            for (int t = 0; t < 4; ++t) d4[t] = make_uint4(pk[4 * t], pk[4 * t + 1], pk[4 * t + 2], pk[4 * t + 3]);
          } else {
            float4* d4 = reinterpret_cast<float4*>(p.ws_o + (((size_t)split * p.T + tok) * p.Hq + head) * dv_tot + dv_off + c);
#pragma unroll
            for (int t = 0; t < 8; ++t)
              d4[t] = make_float4(__uint_as_float(v[4 * t]) * inv, __uint_as_float(v[4 * t + 1]) * inv,
                                  __uint_as_float(v[4 * t + 2]) * inv, __uint_as_float(v[4 * t + 3]) * inv);
          }
        }
        if (p.splits > 1 && row_valid && half == 0)
          p.ws_lse[((size_t)split * p.T + tok) * p.Hq + head] = l > 0.f ? m + log2f(l) : -FLT_MAX;
      } else if (n_tiles == 0 && p.splits > 1 && row_valid && half == 0) {
        float* dst = p.ws_o + (((size_t)split * p.T + tok) * p.Hq + head) * dv_tot + dv_off;
        for (int c = 0; c < DV; ++c) dst[c] = 0.f;
        p.ws_lse[((size_t)split * p.T + tok) * p.Hq + head] = -FLT_MAX;
      }
    } else if (n_tiles > 0) {
      // merge the RF replicas of each logical row through shared memory (the K/V ring
      // is idle now): ml[r] = (m, l); oacc[lr] += exp2(m - M) * O_r / L
      float* ml = reinterpret_cast<float*>(sK);                 // [128][2]
      float* oacc = ml + 256;                                   // [LR][DV]
      for (int i = r; i < LR * DV; i += 128) oacc[i] = 0.f;
      ml[2 * r] = (have_o && row_valid) ? m : -FLT_MAX;
      ml[2 * r + 1] = (have_o && row_valid) ? l : 0.f;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      float M = -FLT_MAX, L = 0.f;
      for (int q = 0; q < RF; ++q) M = fmaxf(M, ml[2 * (lr + q * LR)]);
      for (int q = 0; q < RF; ++q) {
        const float mq = ml[2 * (lr + q * LR)];
        if (mq != -FLT_MAX) L += ex2(mq - M) * ml[2 * (lr + q * LR) + 1];
      }
      if (sink_l2 != -FLT_MAX && M != -FLT_MAX) L += ex2(sink_l2 - M);
      const float f = (have_o && row_valid && m != -FLT_MAX && L > 0.f) ? ex2(m - M) / L : 0.f;
      if (warp_active) {
#pragma unroll 1
        for (int c = 0; c < DV; c += 32) {
          uint32_t v[32];
          tmem_ld32(lane_base + C::O_COL0 + c, v);
          tmem_wait_ld();
          if (f != 0.f) {
#pragma unroll
            for (int t = 0; t < 32; ++t) atomicAdd(&oacc[lr * DV + c + t], __uint_as_float(v[t]) * f);
          }
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (part == 0 && row_valid && ok) {
        const float* src = oacc + lr * DV;
        if (p.splits == 1) {
          __nv_bfloat16* dst = p.o + (size_t)tok * p.o_stride + (size_t)head * dv_tot + dv_off;
          for (int c = 0; c < DV; c += 8) {
            uint4 o;
            o.x = pack_bf16x2(src[c], src[c + 1]); o.y = pack_bf16x2(src[c + 2], src[c + 3]);
            o.z = pack_bf16x2(src[c + 4], src[c + 5]); o.w = pack_bf16x2(src[c + 6], src[c + 7]);
            *reinterpret_cast<uint4*>(dst + c) = o;
          }
        } else {
          float* dst = p.ws_o + (((size_t)split * p.T + tok) * p.Hq + head) * dv_tot + dv_off;
          for (int c = 0; c < DV; ++c) dst[c] = src[c];
          p.ws_lse[((size_t)split * p.T + tok) * p.Hq + head] = L > 0.f ? M + log2f(L) : -FLT_MAX;
        }
      }
    } else if (p.splits > 1 && row_valid && part == 0) {
      float* dst = p.ws_o + (((size_t)split * p.T + tok) * p.Hq + head) * dv_tot + dv_off;
      for (int c = 0; c < DV; ++c) dst[c] = 0.f;
      p.ws_lse[((size_t)split * p.T + tok) * p.Hq + head] = -FLT_MAX;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// merge split-KV partials: one warp per (token, head)
__global__ void attn_combine_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_lse, int splits,
                                    int T, int Hq, int DV, __nv_bfloat16* __restrict__ o, int o_stride,
                                    const float* __restrict__ sinks) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= T * Hq) return;
  const int t = gw / Hq, h = gw - (gw / Hq) * Hq;
  const float sk = sinks != nullptr ? sinks[h] * 1.4426950408889634f : -FLT_MAX;   // log2 units
  float mx = sk;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, ws_lse[((size_t)s * T + t) * Hq + h]);
  float wsum = (sk == -FLT_MAX) ? 0.f : exp2f(sk - mx);
  float w[64];
  for (int s = 0; s < splits && s < 64; ++s) {
    const float ls = ws_lse[((size_t)s * T + t) * Hq + h];
    w[s] = (mx == -FLT_MAX || ls == -FLT_MAX) ? 0.f : exp2f(ls - mx);
    wsum += w[s];
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  for (int c = lane; c < DV; c += 32) {
    float acc = 0.f;
    for (int s = 0; s < splits && s < 64; ++s) acc += w[s] * ws_o[(((size_t)s * T + t) * Hq + h) * DV + c];
    o[(size_t)t * o_stride + (size_t)h * DV + c] = __float2bfloat16(acc * inv);
  }
}

}  // namespace xtu

namespace xtu {
// warp-level GQA decode kernel (attention_decode.cu); 0 = shape not served there
int attn_decode_gqa(const CUtensorMap& tk, const CUtensorMap& tv, const void* q, int q_stride, void* o,
                    int o_stride, const int* q_start, const int* kv_len, const int* block_table, int bt_stride,
                    int B, int max_q_len, int T, int Hq, int Hkv, int D, float scale, int splits, float* ws_o,
                    float* ws_lse, int* counters, int num_blocks, int window, const float* sinks, void* status,
                    cudaStream_t s, int kv_fp8 = 0, float k_scale = 1.f, float v_scale = 1.f);
}  // namespace xtu

using namespace xtu;

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_t attn_encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(ptr);
  }
  return fn;
}

// cache viewed as [rows = blocks*Hkv*64, dim] bf16 with row pitch `pitch` elements; box {64 cols, box_rows}
static int attn_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t dim, uint64_t pitch,
                     uint32_t box_rows = 64) {
  PFN_encodeTiled_t enc = attn_encode_fn();
  if (!enc) return -100;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch * 2) % 16 != 0) return -101;
  cuuint64_t dims[2] = {dim, rows};
  cuuint64_t strides[1] = {pitch * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1000 - (int)r;
}

template <int D, int DV, int BN, int STAGES = 2, int BTS = 0, int VK = 0, int EXT = 0, int CS = 1>
static int launch_attn(const CUtensorMap& tk, const CUtensorMap& tv, const AttnParams& p, int grid_x, int B,
                       cudaStream_t s) {
  using C = AttnCfg<D, DV, BN, STAGES, BTS, VK, CS>;
  auto k = attn_fwd_kernel<D, DV, BN, STAGES, BTS, VK, EXT, CS>;
  static bool init = false;
  if (!init) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return -(int)e;
    init = true;
  }
  dim3 grid(grid_x, p.Hkv * p.splits * p.dv_halves, B);
  k<<<grid, C::THREADS, C::SMEM, s>>>(tk, tv, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// Softmax threads per row for prefill tiles of 128-wide heads: XTU_ATTN_CS = 1, 2 or 4
// in the environment (default 2; at 8K causal GQA tokens 1 / 2 / 4 measured 483 / 598 /
// 569 TFLOP/s: past two parts the exchange rounds cost more than the parallelism gains)
static int attn_softmax_parts() {
  static int v = 0;
  if (v == 0) {
    const char* e = getenv("XTU_ATTN_CS");
    v = (e && (e[0] == '1' || e[0] == '4')) ? e[0] - '0' : 2;
  }
  return v;
}

// K/V ring depth of the verification-shaped configuration: XTU_ATTN_VERIFY_STAGES = 4 or 5
static int attn_verify_stages() {
  static int v = 0;
  if (v == 0) {
    const char* e = getenv("XTU_ATTN_VERIFY_STAGES");
    v = (e && e[0] == '5') ? 5 : 4;
  }
  return v;
}

extern "C" {

// q [T, Hq, D] (token stride q_stride), caches [blocks, Hkv, 64, D|DV]; v_is_k: V = first DV dims of K (MLA).
// counters (nullable): >= B * Hkv zeroed ints that let the GQA decode kernel merge its
// split-KV partials itself (left zeroed).
int xtu_paged_attention(const void* q, int q_stride, const void* k_cache, const void* v_cache, int v_is_k, void* o,
                        int o_stride, const int* q_start, const int* kv_len, const int* block_table, int bt_stride,
                        int B, int max_q_len, int max_kv_len, int T, int Hq, int Hkv, int D, int DV, int block_size,
                        int num_blocks, float scale, int splits, float* ws, int* counters, int window,
                        const float* sinks, void* status, cudaStream_t s) {
  (void)max_kv_len;
  if (B <= 0 || T <= 0) return 0;
  if (block_size != KV_BLOCK) return -2;
  if (Hq % Hkv != 0) return -3;
  const int G = Hq / Hkv;
  if (G > 128) return -4;
  AttnParams p{};
  p.q = (const __nv_bfloat16*)q; p.q_stride = q_stride;
  p.o = (__nv_bfloat16*)o; p.o_stride = o_stride;
  p.q_start = q_start; p.kv_len = kv_len; p.block_table = block_table; p.bt_stride = bt_stride;
  p.Hq = Hq; p.Hkv = Hkv; p.G = G; p.rows_per_tile = (128 / G) * G;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.splits = splits < 1 ? 1 : splits;
  p.T = T;
  p.window = window;
  p.sinks = sinks;
  p.status = reinterpret_cast<XtuStatus*>(status);
  if (p.splits > 1) {
    if (!ws) return -5;
    p.ws_o = ws;
    p.ws_lse = ws + (size_t)p.splits * T * Hq * DV;
  }
  // MLA latent cache (576 = 512 latent + 64 rope, V = the latent): 16-key tiles read once
  // into shared memory serve both QK^T and PV; two CTAs split the 512 output columns
  const bool mla = v_is_k && D == 576 && DV == 512;
  p.dv_total = DV;
  p.dv_halves = mla ? 2 : 1;
  const uint64_t rows = (uint64_t)num_blocks * Hkv * KV_BLOCK;
  CUtensorMap tk, tv;
  int rc = attn_tmap(&tk, k_cache, rows, D, D, mla ? 16 : 64);
  if (rc) return rc;
  if (mla) tv = tk;
  else rc = v_is_k ? attn_tmap(&tv, k_cache, rows, DV, D) : attn_tmap(&tv, v_cache, rows, DV, DV);
  if (rc) return rc;
  const int pos_per_tile = p.rows_per_tile / G;
  const int grid_x = (max_q_len + pos_per_tile - 1) / pos_per_tile;
  int r = 0;
  // decode-shaped GQA steps with few query rows per KV head: the warp-level decode kernel
  if (grid_x == 1 && !v_is_k && D == DV && (D == 64 || D == 128))
    r = attn_decode_gqa(tk, tv, q, q_stride, o, o_stride, q_start, kv_len, block_table, bt_stride, B, max_q_len, T,
                        Hq, Hkv, D, scale, p.splits, p.ws_o, p.ws_lse, counters, num_blocks, window, sinks, status, s);
  if (r < 0) return r;
  if (r == 1) return 1;   // complete, split merge included
  // decode-shaped steps (all of a sequence's query rows fit one 128-row tile): 64-key
  // tiles, a 4-deep K/V ring and a staged block table keep more bytes in flight per SM
  const bool decode_shape = grid_x == 1;
  const int rows_used = max_q_len * G;
  // replica merge buffers live in the K ring: only the decode configurations (D <= 128) use it
  p.rf = (!decode_shape || D > 128) ? 1 : rows_used <= 32 ? 4 : rows_used <= 64 ? 2 : 1;
  // verification-shaped steps (33..64 rows of a 128-wide head: MTP drafts of a large GQA
  // group): 64-key tiles in a 4-deep ring, so the producer runs several pages ahead of the
  // S -> softmax -> PV chain (a 2-deep ring of 128-key tiles left one page loading at a time)
  const bool verify_shape = decode_shape && D == 128 && DV == 128 && rows_used > 32;
  // every replica scores a multiple of 16 keys per tile (the softmax reads S in 16-column chunks)
  const int bn = (decode_shape && D == 64) || verify_shape ? 64 : 128;
  while (p.rf > 1 && (bn / p.rf) % 16 != 0) p.rf >>= 1;
  // window / sinks: the EXT instantiations (GQA shapes only; MLA has neither)
  const bool ext = window > 0 || sinks != nullptr;
  if (mla && ext) return -7;
  if (mla) r = launch_attn<576, 256, 16, 2, 1024, 1>(tk, tv, p, grid_x, B, s);
  else if (verify_shape && attn_verify_stages() == 5)
    r = ext ? launch_attn<128, 128, 64, 5, 256, 0, 1>(tk, tv, p, grid_x, B, s)
            : launch_attn<128, 128, 64, 5, 256>(tk, tv, p, grid_x, B, s);
  else if (verify_shape)
    r = ext ? launch_attn<128, 128, 64, 4, 256, 0, 1>(tk, tv, p, grid_x, B, s)
            : launch_attn<128, 128, 64, 4, 256>(tk, tv, p, grid_x, B, s);
  else if (decode_shape && D == 128 && DV == 128)
    r = ext ? launch_attn<128, 128, 128, 2, 256, 0, 1>(tk, tv, p, grid_x, B, s)
            : launch_attn<128, 128, 128, 2, 256>(tk, tv, p, grid_x, B, s);
  else if (decode_shape && D == 64 && DV == 64)
    r = ext ? launch_attn<64, 64, 64, 6, 1024, 0, 1>(tk, tv, p, grid_x, B, s)
            : launch_attn<64, 64, 64, 6, 1024>(tk, tv, p, grid_x, B, s);
  else if (D == 128 && DV == 128 && attn_softmax_parts() == 4)   // four softmax threads per row
    r = ext ? launch_attn<128, 128, 128, 2, 0, 0, 1, 4>(tk, tv, p, grid_x, B, s)
            : launch_attn<128, 128, 128, 2, 0, 0, 0, 4>(tk, tv, p, grid_x, B, s);
  else if (D == 128 && DV == 128 && attn_softmax_parts() == 2)   // two softmax threads per row
    r = ext ? launch_attn<128, 128, 128, 2, 0, 0, 1, 2>(tk, tv, p, grid_x, B, s)
            : launch_attn<128, 128, 128, 2, 0, 0, 0, 2>(tk, tv, p, grid_x, B, s);
  else if (D == 128 && DV == 128)
    r = ext ? launch_attn<128, 128, 128, 2, 0, 0, 1>(tk, tv, p, grid_x, B, s)
            : launch_attn<128, 128, 128>(tk, tv, p, grid_x, B, s);
  // the other prefill shapes: two softmax threads per row unless XTU_ATTN_CS=1
  else if (D == 64 && DV == 64)
    r = attn_softmax_parts() == 1 ? (ext ? launch_attn<64, 64, 128, 2, 0, 0, 1>(tk, tv, p, grid_x, B, s)
                                         : launch_attn<64, 64, 128>(tk, tv, p, grid_x, B, s))
                                  : (ext ? launch_attn<64, 64, 128, 2, 0, 0, 1, 2>(tk, tv, p, grid_x, B, s)
                                         : launch_attn<64, 64, 128, 2, 0, 0, 0, 2>(tk, tv, p, grid_x, B, s));
  else if (D == 256 && DV == 256)
    r = attn_softmax_parts() == 1 ? (ext ? launch_attn<256, 256, 64, 2, 0, 0, 1>(tk, tv, p, grid_x, B, s)
                                         : launch_attn<256, 256, 64>(tk, tv, p, grid_x, B, s))
                                  : (ext ? launch_attn<256, 256, 64, 2, 0, 0, 1, 2>(tk, tv, p, grid_x, B, s)
                                         : launch_attn<256, 256, 64, 2, 0, 0, 0, 2>(tk, tv, p, grid_x, B, s));
  else if (D == 192 && DV == 128)
    r = attn_softmax_parts() == 1 ? (ext ? launch_attn<192, 128, 64, 2, 0, 0, 1>(tk, tv, p, grid_x, B, s)
                                         : launch_attn<192, 128, 64>(tk, tv, p, grid_x, B, s))
                                  : (ext ? launch_attn<192, 128, 64, 2, 0, 0, 1, 2>(tk, tv, p, grid_x, B, s)
                                         : launch_attn<192, 128, 64, 2, 0, 0, 0, 2>(tk, tv, p, grid_x, B, s));
  else return -6;
  if (r < 0) return r;
  if (p.splits > 1) {
    const int warps = T * Hq;
    attn_combine_kernel<<<(warps * 32 + 255) / 256, 256, 0, s>>>(p.ws_o, p.ws_lse, p.splits, T, Hq, DV,
                                                                  (__nv_bfloat16*)o, o_stride, sinks);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return -(int)e;
    return 2;
  }
  return 1;
}

}  // extern "C"
