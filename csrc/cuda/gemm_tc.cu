// tcgen05 GEMM family for sm_100a: dense and grouped (per-expert ragged) GEMMs
//   D[m, n] = sum_k A[m, k] * B[e(m), n, k]
// with A bf16 (row-major, K contiguous) and B either bf16 or fp8-e4m3 with
// 128x128 fp32 block scales (DeepSeek / GLM "weight_scale_inv" layout).
//
// Design (one persistent CTA per SM):
//   warp 0      : TMA producer (one elected lane), multi-stage smem ring
//   warp 1      : TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  : epilogue: tcgen05.ld from TMEM -> registers -> fused epilogue -> global
//   warps 6..9  : (fp8 B only) dequantize the raw e4m3 tile into a 128B-swizzled bf16
//                 tile in smem, so the MMA runs kind::f16 on exactly the values
//                 bf16(e4m3 * scale) that a dequantize-then-GEMM reference would use.
// The TMEM accumulator is double buffered (2 x BN columns) so the epilogue of
// tile i overlaps the MMAs of tile i+1.
//
// The grouped form replaces the reference's Triton `_gate_up_kernel` /
// `_down_kernel` (vllm_xiaotu_moe/gpu_prefill.py:232-395) and the FP8 twin's
// dequantize + torch.bmm + index_add_ path (vllm_xiaotu_moe/gpu_prefill_fp8.py:1172-1340).
// Its epilogues fuse the clamped SwiGLU (same semantics as
// xiaotu_moe/csrc/moe/moe_v2.hpp:174-190) and the top-k weight + scatter to the
// token's slot row (no global atomics; the per-token sum happens in moe_combine).
#include <cuda.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cstdio>
#include <cstring>
#include "ptx.cuh"

namespace xtu {

constexpr int BM = 128;        // rows per tile (one TMEM lane per row)
constexpr int BK = 64;         // bf16 K per stage = one 128-byte swizzle row
constexpr int UMMA_K = 16;     // K per tcgen05.mma kind::f16

// B formats: bf16; e4m3 + 128x128 fp32 block scales; MXFP4 (e2m1 pairs + e8m0 per 32);
// NVFP4 (e2m1 pairs + e4m3 per 16 + fp32 per expert).  All but bf16 are widened to bf16
// in shared memory by the converter warps before the tcgen05 kind::f16 MMAs.
enum BFormat : int { B_BF16 = 0, B_FP8_BLOCK128 = 1, B_MXFP4 = 2, B_NVFP4 = 3 };
enum Epilogue : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2 };

// One m-tile of the grouped problem: rows [row0, row_end) of A all belong to
// `expert`; rows past row_end that the TMA still loads are discarded.
struct MTile {
  int expert;
  int row0;
  int row_end;
  int pad;
};

struct GemmParams {
  int M, N, K;            // A is [M, K]; B is [E, N, K]; N = rows of B per expert
  int n_blocks;           // ceil(N_out_cols / BN) in B-row units
  const MTile* mtiles;    // device tile list (grouped) or nullptr (dense)
  const int* num_mtiles;  // device count (grouped) or nullptr
  int dense_mtiles;       // ceil(M / BM) for the dense form
  // epilogue
  void* D;
  int ldd;                // elements
  const float* row_scale; // multiply row m by row_scale[m] (nullable)
  const int* row_dest;    // write row m to D row row_dest[m] (nullable; <0 = drop)
  void* const* peer_D;    // (nullable) per-rank output bases: row_dest = rank * peer_rows + row,
  int peer_rows;          //   stored over NVLink into that rank's buffer (expert-parallel combine)
  float act_limit, act_alpha, act_beta;  // clamped SwiGLU
  // fp8 B
  const float* b_scale;   // [E, ceil(N/128), ceil(K/128)]
  int sb_n, sb_k;
  // fp4 B: per-row scale bytes [E, N, K/32] (e8m0) or [E, N, K/16] (e4m3); NVFP4 global [E]
  const uint8_t* b_sc8;
  int sc_k;
  const float* b_gs;
  XtuStatus* status;
};

template <int BN, int BFMT>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;           // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;           // bf16 tile fed to the MMA
  static constexpr bool CONV = BFMT != B_BF16;           // converter warps widen B to bf16
  static constexpr bool FP4 = BFMT == B_MXFP4 || BFMT == B_NVFP4;
  static constexpr int BRAW_BYTES = BFMT == B_FP8_BLOCK128 ? BN * BK : (FP4 ? BN * BK / 2 : 0);  // raw staging
  static constexpr int LUT_BYTES = FP4 ? 1024 : 0;       // byte -> two bf16 (e2m1 pair)
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + BRAW_BYTES;
  static constexpr int STAGES = CONV ? (BN == 256 ? 3 : 4) : (BN == 256 ? 4 : 6);
  static constexpr int NUM_WARPS = CONV ? 10 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + LUT_BYTES;
  static constexpr uint32_t TX_BYTES = A_BYTES + (CONV ? BRAW_BYTES : B_BYTES);
};

__device__ __forceinline__ float silu_clamped(float g, float u, float limit, float alpha, float beta) {
  if (limit > 0.f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.f + __expf(-alpha * g))) * (u + beta);
}

template <int BN, int BFMT, int EPI>
__global__ void __launch_bounds__(Cfg<BN, BFMT>::NUM_WARPS * 32, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   GemmParams p) {
  using C = Cfg<BN, BFMT>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* conv_bar = full_bar + C::STAGES;      // fp8: converted tile ready
  uint64_t* empty_bar = conv_bar + C::STAGES;
  uint64_t* tfull_bar = empty_bar + C::STAGES;    // [2]
  uint64_t* tempty_bar = tfull_bar + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&conv_bar[s], 4);  // one arrive per converter warp
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 4);  // one arrive per epilogue warp
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_mtiles = p.mtiles ? *p.num_mtiles : p.dense_mtiles;
  const int total = n_mtiles * p.n_blocks;
  const int nk = (p.K + BK - 1) / BK;

  auto tile_of = [&](int w, int& expert, int& row0, int& row_end, int& nb) {
    const int mt = w / p.n_blocks;
    nb = w - mt * p.n_blocks;
    if (p.mtiles) {
      const MTile t = p.mtiles[mt];
      expert = t.expert;
      row0 = t.row0;
      row_end = t.row_end;
    } else {
      expert = 0;
      row0 = mt * BM;
      row_end = min(p.M, row0 + BM);
    }
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        int expert, row0, row_end, nb;
        tile_of(w, expert, row0, row_end, nb);
        const int brow = expert * p.N + nb * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.status, 10)) { ok = false; break; }
          uint8_t* sA = smem + stage * C::STAGE_BYTES;
          uint8_t* sB = sA + C::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], C::TX_BYTES);
          tma_load_2d(sA, &tmap_a, &full_bar[stage], kb * BK, row0);
          if (C::FP4) {
            tma_load_2d(sB + C::B_BYTES, &tmap_b, &full_bar[stage], kb * (BK / 2), brow);
          } else if (BFMT == B_FP8_BLOCK128) {
            tma_load_2d(sB + C::B_BYTES, &tmap_b, &full_bar[stage], kb * BK, brow);
          } else {
            tma_load_2d(sB, &tmap_b, &full_bar[stage], kb * BK, brow);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // drain: wait (briefly) for every load this thread may still have in flight
        for (int s = 0; s < C::STAGES; ++s) mbar_wait(&full_bar[s], 0, nullptr, 0, 50000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, p.status, 20)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < nk; ++kb) {
          uint64_t* ready = C::CONV ? &conv_bar[stage] : &full_bar[stage];
          if (!mbar_wait(ready, phase, p.status, 21)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int j = 0; j < BK / UMMA_K; ++j) {
            const uint64_t ad = sdesc_kmajor_sw128(a_addr + j * UMMA_K * 2);
            const uint64_t bd = sdesc_kmajor_sw128(b_addr + j * UMMA_K * 2);
            mma_f16_ss(d_tmem, ad, bd, idesc, (kb | j) != 0 ? 1u : 0u);
          }
          mma_commit(&empty_bar[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit(&tfull_bar[acc]);
      }
      if (!ok) {
        // make sure no MMA is still writing TMEM before the CTA frees it
        mma_commit(&tfull_bar[0]);
        mbar_wait(&tfull_bar[0], 0, nullptr, 0, 50000000ull);
      }
    }
  } else if (warp >= 2 && warp < 6) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int r_in_tile = q * 32 + lane;    // row within the 128-row tile
    int local = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++local) {
      int expert, row0, row_end, nb;
      tile_of(w, expert, row0, row_end, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, p.status, 30)) break;
      tc_fence_after();
      const int row = row0 + r_in_tile;
      const bool row_ok = row < row_end;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      float rs = 1.f;
      int drow = row;
      if (row_ok) {
        if (p.row_scale) rs = p.row_scale[row];
        if (p.row_dest) drow = p.row_dest[row];
      }
      const bool write = row_ok && drow >= 0;
      void* dbase = p.D;
      if (p.peer_D != nullptr && write) {
        const int pr = drow / p.peer_rows;
        drow -= pr * p.peer_rows;
        dbase = p.peer_D[pr];
      }
      if (EPI == EPI_SWIGLU) {
        // B rows of this tile: [0, BN/2) gate, [BN/2, BN) up, for output cols
        // [nb*BN/2, nb*BN/2 + BN/2)
        const int out_cols = p.N / 2;
        __nv_bfloat16* D = reinterpret_cast<__nv_bfloat16*>(dbase);
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(t_row + c, g);
          tmem_ld32(t_row + BN / 2 + c, u);
          tmem_wait_ld();
          const int col0 = nb * (BN / 2) + c;
          if (write) {
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float a0 = silu_clamped(__uint_as_float(g[2 * i]), __uint_as_float(u[2 * i]), p.act_limit,
                                            p.act_alpha, p.act_beta) * rs;
              const float a1 = silu_clamped(__uint_as_float(g[2 * i + 1]), __uint_as_float(u[2 * i + 1]),
                                            p.act_limit, p.act_alpha, p.act_beta) * rs;
              packed[i] = pack_bf16x2(a0, a1);
            }
            __nv_bfloat16* dst = D + (size_t)drow * p.ldd + col0;
            if (col0 + 32 <= out_cols) {
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
            } else {
              for (int i = 0; i < 32 && col0 + i < out_cols; ++i) {
                const uint32_t v = packed[i >> 1];
                reinterpret_cast<uint16_t*>(dst)[i] = (i & 1) ? (uint16_t)(v >> 16) : (uint16_t)(v & 0xFFFF);
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld32(t_row + c, v);
          tmem_wait_ld();
          const int col0 = nb * BN + c;
          if (write && col0 < p.N) {
            if (EPI == EPI_F32) {
              float* dst = reinterpret_cast<float*>(dbase) + (size_t)drow * p.ldd + col0;
              if (col0 + 32 <= p.N) {
                float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  d4[i] = make_float4(__uint_as_float(v[4 * i]) * rs, __uint_as_float(v[4 * i + 1]) * rs,
                                      __uint_as_float(v[4 * i + 2]) * rs, __uint_as_float(v[4 * i + 3]) * rs);
              } else {
                for (int i = 0; i < 32 && col0 + i < p.N; ++i) dst[i] = __uint_as_float(v[i]) * rs;
              }
            } else {
              uint32_t packed[16];
#pragma unroll
              for (int i = 0; i < 16; ++i)
                packed[i] = pack_bf16x2(__uint_as_float(v[2 * i]) * rs, __uint_as_float(v[2 * i + 1]) * rs);
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(dbase) + (size_t)drow * p.ldd + col0;
              if (col0 + 32 <= p.N) {
                uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
              } else {
                for (int i = 0; i < 32 && col0 + i < p.N; ++i) {
                  const uint32_t x = packed[i >> 1];
                  reinterpret_cast<uint16_t*>(dst)[i] = (i & 1) ? (uint16_t)(x >> 16) : (uint16_t)(x & 0xFFFF);
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  } else if (C::FP4) {
    // ---------------- e2m1 -> bf16 dequantizer (warps 6..9) ----------------
    // 16-byte raw chunks (32 e2m1 values, low nibble = even k) go to consecutive lanes;
    // a 256-entry table maps a byte to its two bf16 values.  MXFP4 scales are powers of
    // two, so the bf16 product is exact; NVFP4 scales (e4m3 x fp32 global) are applied
    // in fp32.
    const int ct = threadIdx.x - 6 * 32;  // 0..127
    uint32_t* lut = reinterpret_cast<uint32_t*>(smem + C::STAGES * C::STAGE_BYTES + 256);
    for (int b = ct; b < 256; b += 128) {
      const uint16_t tab[8] = {0x0000, 0x3F00, 0x3F80, 0x3FC0, 0x4000, 0x4040, 0x4080, 0x40C0};
      const int lo = b & 15, hi = b >> 4;
      const uint32_t flo = (lo & 8 ? 0x8000u : 0u) | tab[lo & 7];
      const uint32_t fhi = (hi & 8 ? 0x8000u : 0u) | tab[hi & 7];
      lut[b] = flo | (fhi << 16);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    int stage = 0;
    uint32_t phase = 0;
    constexpr int CHUNKS = BN * BK / 2 / 16;        // 16-byte chunks per stage (2 per row)
    constexpr int PER_THREAD = CHUNKS / 128;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      int expert, row0, row_end, nb;
      tile_of(w, expert, row0, row_end, nb);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, p.status, 41)) { ok = false; break; }
        uint8_t* sB = smem + stage * C::STAGE_BYTES + C::A_BYTES;
        const uint8_t* raw = sB + C::B_BYTES;
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) {
          const int qi = ct + 128 * i;
          const int r = qi >> 1, hk = qi & 1;     // row, which 32 k of the 64
          const int n = min(nb * BN + r, p.N - 1);
          const uint8_t* srow = p.b_sc8 + ((size_t)expert * p.N + n) * p.sc_k;
          const uint4 q4 = reinterpret_cast<const uint4*>(raw)[qi];
          const uint32_t words[4] = {q4.x, q4.y, q4.z, q4.w};
          uint32_t out[16];
          if (BFMT == B_MXFP4) {
            const uint32_t e = srow[kb * 2 + hk];
            const uint32_t sb = e == 0 ? 0x0040u : (e == 255 ? 0x7FC0u : (e << 7));   // bf16 of 2^(e-127)
            const uint32_t s2 = sb | (sb << 16);
            const __nv_bfloat162 sc = *reinterpret_cast<const __nv_bfloat162*>(&s2);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
              for (int bi = 0; bi < 4; ++bi) {
                uint32_t v = lut[(words[wi] >> (8 * bi)) & 0xFF];
                __nv_bfloat162 x = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&v), sc);
                out[wi * 4 + bi] = *reinterpret_cast<uint32_t*>(&x);
              }
            }
          } else {
            const float gs = p.b_gs[expert];
            const int g0 = kb * 4 + hk * 2;
            const __nv_fp8_storage_t e0 = srow[g0], e1 = srow[g0 + 1];
            const float s0 = __half2float(__half(__nv_cvt_fp8_to_halfraw(e0, __NV_E4M3))) * gs;
            const float s1 = __half2float(__half(__nv_cvt_fp8_to_halfraw(e1, __NV_E4M3))) * gs;
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              const float sc = wi < 2 ? s0 : s1;     // words 0-1: k 0..15, words 2-3: k 16..31
#pragma unroll
              for (int bi = 0; bi < 4; ++bi) {
                const uint32_t v = lut[(words[wi] >> (8 * bi)) & 0xFF];
                out[wi * 4 + bi] = pack_bf16x2(bf16_lo(v) * sc, bf16_hi(v) * sc);
              }
            }
          }
          uint8_t* dst_row = sB + r * 128;
#pragma unroll
          for (int pc = 0; pc < 4; ++pc) {
            const int c = (hk * 4 + pc) ^ (r & 7);
            *reinterpret_cast<uint4*>(dst_row + c * 16) =
                make_uint4(out[4 * pc], out[4 * pc + 1], out[4 * pc + 2], out[4 * pc + 3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv_bar[stage]);
        if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
    }
  } else if (BFMT == B_FP8_BLOCK128) {
    // ---------------- fp8 -> bf16 dequantizer (warps 6..9) ----------------
    const int ct = threadIdx.x - 6 * 32;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      int expert, row0, row_end, nb;
      tile_of(w, expert, row0, row_end, nb);
      bool ok = true;
      // 16-byte chunks of the raw tile are spread over consecutive lanes (chunk q -> row
      // q / 4, k-bytes 16 * (q % 4)), so each warp-wide load reads 512 contiguous bytes
      // without bank conflicts.  The (at most two) block scales of a stage are fetched
      // before the stage's data arrives.
      constexpr int CHUNKS = BN * BK / 16;            // 16-byte chunks per stage
      constexpr int PER_THREAD = CHUNKS / 128;
      const int nblk0 = (nb * BN) >> 7;
      const int nblk_max = (p.N - 1) >> 7;
      const float* sc_e = p.b_scale + (size_t)expert * p.sb_n * p.sb_k;
      for (int kb = 0; kb < nk; ++kb) {
        const int kscale = (kb * BK) >> 7;
        const float s_lo = __ldg(sc_e + (size_t)min(nblk0, nblk_max) * p.sb_k + kscale);
        const float s_hi = BN > 128 ? __ldg(sc_e + (size_t)min(nblk0 + 1, nblk_max) * p.sb_k + kscale) : s_lo;
        if (!mbar_wait(&full_bar[stage], phase, p.status, 40)) { ok = false; break; }
        uint8_t* sB = smem + stage * C::STAGE_BYTES + C::A_BYTES;
        const uint8_t* raw = sB + C::B_BYTES;
        uint4 q[PER_THREAD];
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) q[i] = reinterpret_cast<const uint4*>(raw)[ct + 128 * i];
#pragma unroll
        for (int i = 0; i < PER_THREAD; ++i) {
          const int qi = ct + 128 * i;
          const int r = qi >> 2, c = qi & 3;
          const float sc = r < 128 ? s_lo : s_hi;
          const uint32_t words[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
          uint32_t out[8];
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            __half2_raw h01 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(words[wi] & 0xFFFF), __NV_E4M3);
            __half2_raw h23 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(words[wi] >> 16), __NV_E4M3);
            const float2 f01 = __half22float2(*reinterpret_cast<__half2*>(&h01));
            const float2 f23 = __half22float2(*reinterpret_cast<__half2*>(&h23));
            out[2 * wi] = pack_bf16x2(f01.x * sc, f01.y * sc);
            out[2 * wi + 1] = pack_bf16x2(f23.x * sc, f23.y * sc);
          }
          // 16 e4m3 -> 32 bytes of bf16 = 16-B chunks 2c and 2c+1 of the row's 128 bytes,
          // placed with the 128-byte swizzle (chunk ^ row % 8)
          uint8_t* dst_row = sB + r * 128;
          const int c0 = (2 * c) ^ (r & 7);
          const int c1 = (2 * c + 1) ^ (r & 7);
          *reinterpret_cast<uint4*>(dst_row + c0 * 16) = make_uint4(out[0], out[1], out[2], out[3]);
          *reinterpret_cast<uint4*>(dst_row + c1 * 16) = make_uint4(out[4], out[5], out[6], out[7]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv_bar[stage]);
        if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// grouped tile list: m-tiles of each expert's row segment
// ---------------------------------------------------------------------------
__global__ void build_mtiles_kernel(const int* __restrict__ seg, int E, MTile* __restrict__ tiles,
                                    int* __restrict__ count, int max_tiles) {
  // single block; blockDim.x >= 32, experts strided over threads
  __shared__ int s_tot[1024];
  const int tid = threadIdx.x;
  int local = 0;
  for (int e = tid; e < E; e += blockDim.x) {
    const int n = seg[e + 1] - seg[e];
    local += (n + BM - 1) / BM;
  }
  s_tot[tid] = local;
  __syncthreads();
  // inclusive scan (Hillis-Steele) over threads
  for (int off = 1; off < blockDim.x; off <<= 1) {
    const int v = tid >= off ? s_tot[tid - off] : 0;
    __syncthreads();
    s_tot[tid] += v;
    __syncthreads();
  }
  int pos = s_tot[tid] - local;
  for (int e = tid; e < E; e += blockDim.x) {
    const int s0 = seg[e], s1 = seg[e + 1];
    for (int r = s0; r < s1; r += BM) {
      if (pos < max_tiles) tiles[pos] = MTile{e, r, s1, 0};
      ++pos;
    }
  }
  if (tid == blockDim.x - 1) *count = min(s_tot[tid], max_tiles);
}

}  // namespace xtu

// ===========================================================================
// host side
// ===========================================================================
using namespace xtu;

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

// 2-D row-major tensor [rows, cols] of `elem_bytes` elements; box = [box_rows, box_cols]
static int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t rows,
                        uint64_t cols, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return -100;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return -101;
  if ((cols * elem_bytes) % 16 != 0) return -102;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -(int)r - 1000;
}

static int g_num_sms = 0;
static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

template <int BN, int BFMT, int EPI>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int max_work,
                       cudaStream_t stream) {
  using C = Cfg<BN, BFMT>;
  auto kern = gemm_tc_kernel<BN, BFMT, EPI>;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return -(int)e;
    attr_set = true;
  }
  int grid = max_work < num_sms() ? max_work : num_sms();
  if (grid < 1) grid = 1;
  kern<<<grid, C::NUM_WARPS * 32, C::SMEM_BYTES, stream>>>(ta, tb, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

template <int BN, int BFMT>
static int dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int max_work,
                        cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return launch_gemm<BN, BFMT, EPI_BF16>(ta, tb, p, max_work, s);
    case EPI_F32: return launch_gemm<BN, BFMT, EPI_F32>(ta, tb, p, max_work, s);
    case EPI_SWIGLU: return launch_gemm<BN, BFMT, EPI_SWIGLU>(ta, tb, p, max_work, s);
  }
  return -2;
}

extern "C" {

// status helpers -------------------------------------------------------------
int xtu_status_size() { return (int)sizeof(XtuStatus); }

// Dense GEMM: D[M,N] = A[M,K] @ B[N,K]^T.  A,B bf16; D bf16 (out_f32=0) or f32.
int xtu_gemm_bf16(const void* A, const void* B, void* D, int M, int N, int K, int ldd, int out_f32,
                  const float* row_scale, void* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, BM, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int bn = (N >= 256 && ((M + BM - 1) / BM) * ((N + 255) / 256) >= num_sms()) ? 256 : 128;
  rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, bn, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.n_blocks = (N + bn - 1) / bn;
  p.mtiles = nullptr; p.num_mtiles = nullptr;
  p.dense_mtiles = (M + BM - 1) / BM;
  p.D = D; p.ldd = ldd; p.row_scale = row_scale; p.row_dest = nullptr;
  p.status = reinterpret_cast<XtuStatus*>(status);
  const int work = p.dense_mtiles * p.n_blocks;
  const int epi = out_f32 ? EPI_F32 : EPI_BF16;
  return bn == 256 ? dispatch_epi<256, B_BF16>(epi, ta, tb, p, work, stream)
                   : dispatch_epi<128, B_BF16>(epi, ta, tb, p, work, stream);
}

// Dense GEMM with fp8-e4m3 B and [ceil(N/128), ceil(K/128)] fp32 block scales.
int xtu_gemm_fp8w(const void* A, const void* B8, const float* b_scale, void* D, int M, int N, int K, int ldd,
                  int out_f32, void* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, BM, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int bn = (N >= 256 && ((M + BM - 1) / BM) * ((N + 255) / 256) >= num_sms()) ? 256 : 128;
  rc = make_tmap_2d(&tb, B8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, bn, BK, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.n_blocks = (N + bn - 1) / bn;
  p.dense_mtiles = (M + BM - 1) / BM;
  p.D = D; p.ldd = ldd;
  p.b_scale = b_scale; p.sb_n = (N + 127) / 128; p.sb_k = (K + 127) / 128;
  p.status = reinterpret_cast<XtuStatus*>(status);
  const int work = p.dense_mtiles * p.n_blocks;
  const int epi = out_f32 ? EPI_F32 : EPI_BF16;
  return bn == 256 ? dispatch_epi<256, B_FP8_BLOCK128>(epi, ta, tb, p, work, stream)
                   : dispatch_epi<128, B_FP8_BLOCK128>(epi, ta, tb, p, work, stream);
}

// Build the m-tile list for a grouped GEMM from segment offsets seg[E+1].
int xtu_build_mtiles(const int* seg, int E, void* tiles, int* count, int max_tiles, cudaStream_t stream) {
  int threads = 32;
  while (threads < E && threads < 1024) threads <<= 1;
  build_mtiles_kernel<<<1, threads, 0, stream>>>(seg, E, reinterpret_cast<MTile*>(tiles), count, max_tiles);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

int xtu_mtile_bytes() { return (int)sizeof(MTile); }

// Grouped GEMM over experts.
//   A      : [M, K] bf16, rows permuted so each expert's rows are contiguous
//   B      : [E, N, K] bf16 (bfmt=0) or e4m3 (bfmt=1, with b_scale [E, ceil(N/128), ceil(K/128)])
//   tiles  : device MTile list + count (xtu_build_mtiles)
//   epi    : 0 = bf16 out [*, N]; 1 = f32 out; 2 = clamped SwiGLU -> bf16 out [*, N/2]
//            (B rows per 256-row block: first 128 gate, next 128 up)
//   row_scale / row_dest: per-row multiplier and destination row (nullable)
int xtu_grouped_gemm_ex(const void* A, const void* B, const void* b_scale, const float* b_gs, int bfmt, void* D,
                        int ldd, int M, int N, int K, int E, const void* tiles, const int* count, int max_mtiles,
                        int epi, const float* row_scale, const int* row_dest, float act_limit, float act_alpha,
                        float act_beta, void* const* peer_D, int peer_rows, void* status, cudaStream_t stream);

int xtu_grouped_gemm(const void* A, const void* B, const float* b_scale, int bfmt, void* D, int ldd, int M, int N,
                     int K, int E, const void* tiles, const int* count, int max_mtiles, int epi,
                     const float* row_scale, const int* row_dest, float act_limit, float act_alpha, float act_beta,
                     void* status, cudaStream_t stream) {
  return xtu_grouped_gemm_ex(A, B, b_scale, nullptr, bfmt, D, ldd, M, N, K, E, tiles, count, max_mtiles, epi,
                             row_scale, row_dest, act_limit, act_alpha, act_beta, nullptr, 0, status, stream);
}

// As xtu_grouped_gemm, plus:
//   bfmt 2 (MXFP4): B [E, N, K/2] bytes (two e2m1, low nibble = even k), b_scale [E, N, K/32] e8m0;
//   bfmt 3 (NVFP4): same B, b_scale [E, N, K/16] e4m3, b_gs [E] fp32 global scales;
//   peer_D (device array of per-rank output bases): each kept row m goes to rank
//   row_dest[m] / peer_rows, row row_dest[m] % peer_rows, by direct stores to that rank's
//   memory (the expert-parallel combine fused into the down GEMM).
int xtu_grouped_gemm_ex(const void* A, const void* B, const void* b_scale, const float* b_gs, int bfmt, void* D,
                        int ldd, int M, int N, int K, int E, const void* tiles, const int* count, int max_mtiles,
                        int epi, const float* row_scale, const int* row_dest, float act_limit, float act_alpha,
                        float act_beta, void* const* peer_D, int peer_rows, void* status, cudaStream_t stream) {
  if (peer_D != nullptr && (row_dest == nullptr || peer_rows <= 0)) return -7;
  if (M <= 0 || N <= 0 || K <= 0 || E <= 0) return 0;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, BM, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int bn = (epi == EPI_SWIGLU || N >= 256) ? 256 : 128;
  if (epi == EPI_SWIGLU && (N % 256) != 0) return -4;
  if (bfmt == B_MXFP4 || bfmt == B_NVFP4) {
    if (K % 64 != 0 || b_scale == nullptr || (bfmt == B_NVFP4 && b_gs == nullptr)) return -8;
    rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K / 2, bn, BK / 2,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
  } else if (bfmt == B_FP8_BLOCK128) {
    rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)E * N, K, bn, BK,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)E * N, K, bn, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.n_blocks = (N + bn - 1) / bn;
  p.mtiles = reinterpret_cast<const MTile*>(tiles);
  p.num_mtiles = count;
  p.D = D; p.ldd = ldd; p.row_scale = row_scale; p.row_dest = row_dest;
  p.peer_D = peer_D; p.peer_rows = peer_rows;
  p.act_limit = act_limit; p.act_alpha = act_alpha; p.act_beta = act_beta;
  p.b_scale = reinterpret_cast<const float*>(b_scale); p.sb_n = (N + 127) / 128; p.sb_k = (K + 127) / 128;
  p.b_sc8 = reinterpret_cast<const uint8_t*>(b_scale);
  p.sc_k = bfmt == B_MXFP4 ? K / 32 : K / 16;
  p.b_gs = b_gs;
  p.status = reinterpret_cast<XtuStatus*>(status);
  const int work = max_mtiles * p.n_blocks;
  if (bfmt == B_MXFP4)
    return bn == 256 ? dispatch_epi<256, B_MXFP4>(epi, ta, tb, p, work, stream)
                     : dispatch_epi<128, B_MXFP4>(epi, ta, tb, p, work, stream);
  if (bfmt == B_NVFP4)
    return bn == 256 ? dispatch_epi<256, B_NVFP4>(epi, ta, tb, p, work, stream)
                     : dispatch_epi<128, B_NVFP4>(epi, ta, tb, p, work, stream);
  if (bfmt == B_FP8_BLOCK128)
    return bn == 256 ? dispatch_epi<256, B_FP8_BLOCK128>(epi, ta, tb, p, work, stream)
                     : dispatch_epi<128, B_FP8_BLOCK128>(epi, ta, tb, p, work, stream);
  return bn == 256 ? dispatch_epi<256, B_BF16>(epi, ta, tb, p, work, stream)
                   : dispatch_epi<128, B_BF16>(epi, ta, tb, p, work, stream);
}

}  // extern "C"
