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
  float scale_log2;        // softmax scale * log2(e)
  int splits;
  float* ws_o;             // [splits, T, Hq, DV] (splits > 1)
  float* ws_lse;           // [splits, T, Hq]
  int T;
  XtuStatus* status;
};

template <int D, int DV, int BN>
struct AttnCfg {
  static constexpr int STAGES = 2;
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int K_BYTES = BN * D * 2;
  static constexpr int V_BYTES = BN * DV * 2;
  static constexpr int P_BYTES = 128 * BN * 2;
  static constexpr int SMEM = Q_BYTES + STAGES * (K_BYTES + V_BYTES) + 2 * P_BYTES + 1024 + 256;
  static constexpr int S_COL0 = 0;          // two S buffers: [0, BN), [BN, 2BN)
  static constexpr int O_COL0 = 2 * BN;     // O: [2BN, 2BN + DV)
  static constexpr int TMEM_COLS = (2 * BN + DV) <= 256 ? 256 : 512;
  static_assert(2 * BN + DV <= 512, "TMEM budget");
  static_assert(D % 64 == 0 && DV % 64 == 0 && BN % 64 == 0, "tile shapes");
};

// write 8 bf16 (16 B) at (row, col8) of a K-major SW128 operand tile [rows][64-col chunks]
__device__ __forceinline__ void st_sw128(uint8_t* tile, int rows, int row, int col, uint4 v) {
  const int chunk = col >> 6;          // 64-element chunk
  const int piece = (col & 63) >> 3;   // 16-byte piece in the 128-byte row
  uint8_t* base = tile + (size_t)chunk * rows * 128 + row * 128;
  *reinterpret_cast<uint4*>(base + ((piece ^ (row & 7)) << 4)) = v;
}

template <int D, int DV, int BN>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                    AttnParams p) {
  using C = AttnCfg<D, DV, BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;                       // [STAGES][K_BYTES]
  uint8_t* sV = sK + C::STAGES * C::K_BYTES;           // [STAGES][V_BYTES]
  uint8_t* sP = sV + C::STAGES * C::V_BYTES;           // [2][P_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P_BYTES);
  uint64_t* kv_full = bars;                 // [STAGES]
  uint64_t* kv_empty = bars + 2;            // [STAGES]
  uint64_t* q_ready = bars + 4;
  uint64_t* s_full = bars + 5;              // [2]
  uint64_t* p_full = bars + 7;              // [2]
  uint64_t* o_done = bars + 9;              // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int kvh = blockIdx.y % p.Hkv;
  const int split = blockIdx.y / p.Hkv;
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
  const int per = (n_tiles_all + p.splits - 1) / p.splits;
  const int t_begin = split * per;
  const int t_end = min(n_tiles_all, t_begin + per);
  const int n_tiles = max(0, t_end - t_begin);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
    for (int s = 0; s < C::STAGES; ++s) { mbar_init(&kv_full[s], 1); mbar_init(&kv_empty[s], 1); }
    mbar_init(q_ready, 4);
    for (int i = 0; i < 2; ++i) { mbar_init(&s_full[i], 1); mbar_init(&p_full[i], 4); mbar_init(&o_done[i], 1); }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one() && n_tiles > 0) {
      const int* bt = p.block_table + (size_t)b * p.bt_stride;
      const int n_blocks_seq = (kv_len + KV_BLOCK - 1) / KV_BLOCK;
      for (int jj = 0; jj < n_tiles; ++jj) {
        const int stage = jj % C::STAGES;
        const uint32_t ph = (jj / C::STAGES) & 1;
        if (!mbar_wait(&kv_empty[stage], ph ^ 1u, p.status, 100)) break;
        mbar_arrive_expect_tx(&kv_full[stage], C::K_BYTES + C::V_BYTES);
        const int j = t_begin + jj;
#pragma unroll
        for (int sb = 0; sb < BN / KV_BLOCK; ++sb) {
          int lb = j * (BN / KV_BLOCK) + sb;
          if (lb >= n_blocks_seq) lb = 0;              // past the end: any valid block, masked later
          const int row = (bt[lb] * p.Hkv + kvh) * KV_BLOCK;
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_2d(sK + stage * C::K_BYTES + c * (BN * 128) + sb * (KV_BLOCK * 128), &tmap_k, &kv_full[stage],
                        c * 64, row);
#pragma unroll
          for (int c = 0; c < DV / 64; ++c)
            tma_load_2d(sV + stage * C::V_BYTES + c * (BN * 128) + sb * (KV_BLOCK * 128), &tmap_v, &kv_full[stage],
                        c * 64, row);
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
          const uint32_t v_addr = smem_u32(sV + stage * C::V_BYTES);
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
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const int pi = r / p.G, g = r - (r / p.G) * p.G;
    const bool row_valid = (r < p.rows_per_tile) && (pi < n_pos);
    const int tok = q0 + i0 + pi;
    const int head = kvh * p.G + g;
    const int qpos = ctx0 + i0 + pi;
    // load this row of Q into swizzled smem
    {
      const __nv_bfloat16* src = p.q + (size_t)tok * p.q_stride + (size_t)head * D;
#pragma unroll 4
      for (int c8 = 0; c8 < D; c8 += 8) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row_valid) v = *reinterpret_cast<const uint4*>(src + c8);
        st_sw128(sQ, 128, r, c8, v);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    float m = -FLT_MAX;   // running max (log2 domain); -FLT_MAX = none yet
    float l = 0.f;
    const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
    bool ok = true;
    for (int jj = 0; jj < n_tiles && ok; ++jj) {
      const int j = t_begin + jj;
      if (!mbar_wait(&s_full[jj & 1], (jj >> 1) & 1, p.status, 120)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_addr = lane_base + C::S_COL0 + (jj & 1) * BN;
      const int key0 = j * BN;
      // pass 1: masked row max
      float mx = -FLT_MAX;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld32(s_addr + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int key = key0 + c + t;
          const float s = __uint_as_float(v[t]) * p.scale_log2;
          if (row_valid && key <= qpos) mx = fmaxf(mx, s);
        }
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
        for (int c = 0; c < DV; c += 16) {
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
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld32(s_addr + c, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const int key = key0 + c + t;
          float e0 = 0.f, e1 = 0.f;
          if (row_valid && m_use != -FLT_MAX) {
            if (key <= qpos) e0 = ex2(__uint_as_float(v[t]) * p.scale_log2 - m_use);
            if (key + 1 <= qpos) e1 = ex2(__uint_as_float(v[t + 1]) * p.scale_log2 - m_use);
          }
          rs += e0 + e1;
          pk[t >> 1] = pack_bf16x2(e0, e1);
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          st_sw128(pbuf, 128, r, c + q4 * 8, make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]));
      }
      l += rs;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[jj & 1]);
    }
    // ---- epilogue
    if (ok && n_tiles > 0) {
      const int last = n_tiles - 1;
      if (mbar_wait(&o_done[last & 1], (last >> 1) & 1, p.status, 123)) {
        tc_fence_after();
        if (p.splits == 1) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          __nv_bfloat16* dst = p.o + (size_t)tok * p.o_stride + (size_t)head * DV;
#pragma unroll 1
          for (int c = 0; c < DV; c += 32) {
            uint32_t v[32];
            tmem_ld32(lane_base + C::O_COL0 + c, v);
            tmem_wait_ld();
            if (row_valid) {
              uint32_t pk[16];
#pragma unroll
              for (int t = 0; t < 16; ++t)
                pk[t] = pack_bf16x2(__uint_as_float(v[2 * t]) * inv, __uint_as_float(v[2 * t + 1]) * inv);
              uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
              for (int t = 0; t < 4; ++t) d4[t] = make_uint4(pk[4 * t], pk[4 * t + 1], pk[4 * t + 2], pk[4 * t + 3]);
            }
          }
        } else {
          float* dst = p.ws_o + (((size_t)split * p.T + tok) * p.Hq + head) * DV;
          const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
          for (int c = 0; c < DV; c += 32) {
            uint32_t v[32];
            tmem_ld32(lane_base + C::O_COL0 + c, v);
            tmem_wait_ld();
            if (row_valid) {
              float4* d4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
              for (int t = 0; t < 8; ++t)
                d4[t] = make_float4(__uint_as_float(v[4 * t]) * inv, __uint_as_float(v[4 * t + 1]) * inv,
                                    __uint_as_float(v[4 * t + 2]) * inv, __uint_as_float(v[4 * t + 3]) * inv);
            }
          }
          if (row_valid) p.ws_lse[((size_t)split * p.T + tok) * p.Hq + head] = l > 0.f ? m + log2f(l) : -FLT_MAX;
        }
      }
    } else if (n_tiles == 0 && p.splits > 1 && row_valid) {
      float* dst = p.ws_o + (((size_t)split * p.T + tok) * p.Hq + head) * DV;
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
                                    int T, int Hq, int DV, __nv_bfloat16* __restrict__ o, int o_stride) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= T * Hq) return;
  const int t = gw / Hq, h = gw - (gw / Hq) * Hq;
  float mx = -FLT_MAX;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, ws_lse[((size_t)s * T + t) * Hq + h]);
  float wsum = 0.f;
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

// cache viewed as [rows = blocks*Hkv*64, dim] bf16 with row pitch `pitch` elements; box {64 cols, 64 rows}
static int attn_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t dim, uint64_t pitch) {
  PFN_encodeTiled_t enc = attn_encode_fn();
  if (!enc) return -100;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch * 2) % 16 != 0) return -101;
  cuuint64_t dims[2] = {dim, rows};
  cuuint64_t strides[1] = {pitch * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1000 - (int)r;
}

template <int D, int DV, int BN>
static int launch_attn(const CUtensorMap& tk, const CUtensorMap& tv, const AttnParams& p, int grid_x, int B,
                       cudaStream_t s) {
  using C = AttnCfg<D, DV, BN>;
  auto k = attn_fwd_kernel<D, DV, BN>;
  static bool init = false;
  if (!init) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return -(int)e;
    init = true;
  }
  dim3 grid(grid_x, p.Hkv * p.splits, B);
  k<<<grid, 192, C::SMEM, s>>>(tk, tv, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

extern "C" {

// q [T, Hq, D] (token stride q_stride), caches [blocks, Hkv, 64, D|DV]; v_is_k: V = first DV dims of K (MLA)
int xtu_paged_attention(const void* q, int q_stride, const void* k_cache, const void* v_cache, int v_is_k, void* o,
                        int o_stride, const int* q_start, const int* kv_len, const int* block_table, int bt_stride,
                        int B, int max_q_len, int max_kv_len, int T, int Hq, int Hkv, int D, int DV, int block_size,
                        int num_blocks, float scale, int splits, float* ws, void* status, cudaStream_t s) {
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
  p.status = reinterpret_cast<XtuStatus*>(status);
  if (p.splits > 1) {
    if (!ws) return -5;
    p.ws_o = ws;
    p.ws_lse = ws + (size_t)p.splits * T * Hq * DV;
  }
  const uint64_t rows = (uint64_t)num_blocks * Hkv * KV_BLOCK;
  CUtensorMap tk, tv;
  int rc = attn_tmap(&tk, k_cache, rows, D, D);
  if (rc) return rc;
  rc = v_is_k ? attn_tmap(&tv, k_cache, rows, DV, D) : attn_tmap(&tv, v_cache, rows, DV, DV);
  if (rc) return rc;
  const int pos_per_tile = p.rows_per_tile / G;
  const int grid_x = (max_q_len + pos_per_tile - 1) / pos_per_tile;
  int r;
  if (D == 128 && DV == 128) r = launch_attn<128, 128, 128>(tk, tv, p, grid_x, B, s);
  else if (D == 64 && DV == 64) r = launch_attn<64, 64, 128>(tk, tv, p, grid_x, B, s);
  else if (D == 256 && DV == 256) r = launch_attn<256, 256, 64>(tk, tv, p, grid_x, B, s);
  else if (D == 192 && DV == 128) r = launch_attn<192, 128, 64>(tk, tv, p, grid_x, B, s);
  else return -6;
  if (r < 0) return r;
  if (p.splits > 1) {
    const int warps = T * Hq;
    attn_combine_kernel<<<(warps * 32 + 255) / 256, 256, 0, s>>>(p.ws_o, p.ws_lse, p.splits, T, Hq, DV,
                                                                  (__nv_bfloat16*)o, o_stride);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return -(int)e;
    return 2;
  }
  return 1;
}

}  // extern "C"
