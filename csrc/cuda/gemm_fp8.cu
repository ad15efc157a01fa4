// Native fp8 tcgen05 GEMM (kind::f8f6f4) for sm_100a with DeepSeek / GLM 128x128 block scales:
//   D[m, n] = sum_kb  sa[m, kb] * sb[e(m), n / 128, kb] * sum_{k in block kb} A8[m, k] * B8[e(m), n, k]
// A8 is e4m3 with one fp32 scale per (row, 128-k block) (activations quantized on the fly,
// xtu_quant_fp8_rows or the SwiGLU epilogue below); B8 is the checkpoint's e4m3 weights with
// their fp32 128x128 block scales, used exactly as stored.
//
// Block scales cannot ride inside the MMA (they are fp32, not the power-of-two vectors of the
// block-scaled MMA kinds), so every 128-k block is a separate product: the MMA warp writes it
// into one of two TMEM partial buffers (256 columns each, the whole 512-column TMEM), and eight
// promotion warps scale it by sa * sb and add it to fp32 accumulators held in registers while
// the tensor cores fill the other buffer.  After the last block the same warps run the
// epilogue from registers.
//
//   warp 0      : TMA producer (one elected lane), 4-stage ring of 16 KB A + 32 KB B tiles
//   warp 1      : TMEM owner + MMA issuer (one elected lane), 4 x K=32 MMAs per 128-k block
//   warps 2..9  : promotion + epilogue; warp w reads TMEM lanes 32 * (w % 4) .. + 31 (rows of
//                 the tile) and one half of the tile's 256 columns
//
// Epilogues: bf16 or fp32 out (optional per-row scale, destination row, peer store and
// per-column bias), clamped SwiGLU to bf16, and clamped SwiGLU quantized to e4m3 with one
// scale per (row, 128 outputs) -- the A operand of the following down GEMM, so the MoE
// intermediate never exists in bf16.
//
// Replaces the widen-to-bf16 path of gemm_tc.cu for fp8 experts at prefill sizes and, like
// it, the reference's dequantize + torch.bmm + index_add_ FP8 prefill
// (vllm_xiaotu_moe/gpu_prefill_fp8.py:1172-1340) and its Triton FP8 kernels (:101-209).
// No TMA multicast; TMA reads only this GPU's memory (epilogue peer stores are plain stores).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "ptx.cuh"

namespace xtu {
namespace f8 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;                 // fp8 elements = 128 bytes = one scale block
constexpr int UMMA_K = 32;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;        // 16 KB
constexpr int B_BYTES = BN * BK;        // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_WARPS = 10;
constexpr int EPI_WARPS = 8;
constexpr int TMEM_COLS = 512;
constexpr int BAR_BYTES = 256;
constexpr int XCH_BYTES = 2 * 2 * BM * 4;   // [tile parity][half][row] row amax of SwiGLU_Q8
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES + XCH_BYTES;

enum Epi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2, EPI_SWIGLU_Q8 = 3 };

// one m-tile of the grouped problem (the layout xtu_build_mtiles writes)
struct Tile {
  int expert, row0, row_end, pad;
};
static_assert(sizeof(Tile) == 16, "tile layout shared with xtu_build_mtiles");

struct Params {
  int M, N, K;                 // A [M, K] e4m3, B [E, N, K] e4m3
  int n_blocks;                // ceil(N / BN)
  const Tile* tiles;           // grouped form (nullptr: dense, expert 0)
  const int* num_tiles;
  int dense_tiles;
  const float* a_scale;        // [M, K / 128]
  const float* b_scale;        // [E, ceil(N / 128), K / 128]
  int sb_n;
  void* D;                     // bf16 / fp32 [*, N]; SwiGLU: bf16 [*, N / 2]; SwiGLU_Q8: e4m3 [*, N / 2]
  int ldd;                     // elements
  float* d_scale;              // SwiGLU_Q8: [*, N / 256] fp32 (row stride lds)
  int lds;
  const float* row_scale;      // nullable
  const int* row_dest;         // nullable (< 0: drop the row)
  void* const* peer_D;         // nullable: row_dest = rank * peer_rows + row, stored into that rank's D
  int peer_rows;
  const __nv_bfloat16* bias;   // nullable, [N] (plain epilogues)
  float act_limit, act_alpha, act_beta;
  XtuStatus* status;
};

__device__ __forceinline__ float silu_clamped8(float g, float u, float limit, float alpha, float beta) {
  if (limit > 0.f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.f + __expf(-alpha * g))) * (u + beta);
}

__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

template <int EPI>
__global__ void __launch_bounds__(NUM_WARPS * 32, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* pfull = empty + STAGES;     // [2] partial product ready
  uint64_t* pempty = pfull + 2;         // [2] partial product consumed
  uint64_t* xbar = pempty + 2;          // SwiGLU_Q8 row-amax exchange, one phase per tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 1);
  float* xch = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + BAR_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], EPI_WARPS);
    }
    mbar_init(xbar, EPI_WARPS);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = p.tiles ? *p.num_tiles : p.dense_tiles;
  const int total = n_tiles * p.n_blocks;
  const int nk = p.K / BK;

  auto tile_of = [&](int w, int& expert, int& row0, int& row_end, int& nb) {
    const int mt = w / p.n_blocks;
    nb = w - mt * p.n_blocks;
    if (p.tiles) {
      const Tile t = p.tiles[mt];
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
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, 110)) { ok = false; break; }
          uint8_t* sA = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sA, &tmap_a, &full[stage], kb * BK, row0);
          tma_load_2d(sA + A_BYTES, &tmap_b, &full[stage], kb * BK, brow);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok)   // let the loads still in flight land before the CTA exits
        for (int s = 0; s < STAGES; ++s) mbar_wait(&full[s], 0, nullptr, 0, 50000000ull);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_e4m3_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0, kc = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        for (int kb = 0; kb < nk; ++kb, ++kc) {
          if (!mbar_wait(&full[stage], phase, p.status, 111)) { ok = false; break; }
          const uint32_t pb = kc & 1u;
          if (!mbar_wait(&pempty[pb], ((kc >> 1) & 1u) ^ 1u, p.status, 112)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
          const uint32_t d = tmem_base + pb * BN;
#pragma unroll
          for (int j = 0; j < BK / UMMA_K; ++j)
            mma_f8_ss(d, sdesc_kmajor_sw128(a_addr + j * UMMA_K), sdesc_kmajor_sw128(b_addr + j * UMMA_K), idesc,
                      j != 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
          mma_commit(&pfull[pb]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {   // no MMA may still write TMEM when the CTA frees it
        mma_commit(&empty[0]);
        mbar_wait(&empty[0], phase, nullptr, 0, 50000000ull);
      }
    }
  } else {
    // ---------------- promotion + epilogue (warps 2..9) ----------------
    const int ew = warp - 2;
    const int q = warp & 3;                  // TMEM lane quarter this warp may access
    const int half = ew >> 2;                // which half of the tile's columns
    const int r_in_tile = q * 32 + lane;
    constexpr bool SWI = EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_Q8;
    // two 64-column chunks: SwiGLU pairs gate column c with up column c + 128
    const int c0 = SWI ? 64 * half : 128 * half;
    const int c1 = SWI ? 128 + 64 * half : 128 * half + 64;
    uint32_t kc = 0;
    int lt = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < total && ok; w += gridDim.x, ++lt) {
      int expert, row0, row_end, nb;
      tile_of(w, expert, row0, row_end, nb);
      const int row = row0 + r_in_tile;
      const bool row_ok = row < row_end;
      const int blk0 = min((nb * BN + c0) >> 7, p.sb_n - 1);
      const int blk1 = min((nb * BN + c1) >> 7, p.sb_n - 1);
      const float* sbe = p.b_scale + (size_t)expert * p.sb_n * nk;
      const float* sar = p.a_scale + (size_t)(row_ok ? row : 0) * nk;
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;
      for (int kb = 0; kb < nk; ++kb, ++kc) {
        const float sa = row_ok ? __ldg(sar + kb) : 0.f;
        const float s0 = sa * __ldg(sbe + (size_t)blk0 * nk + kb);
        const float s1 = sa * __ldg(sbe + (size_t)blk1 * nk + kb);
        const uint32_t pb = kc & 1u;
        if (!mbar_wait(&pfull[pb], (kc >> 1) & 1u, p.status, 113)) { ok = false; break; }
        tc_fence_after();
        const uint32_t t = tmem_base + ((uint32_t)(q * 32) << 16) + pb * BN;
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          uint32_t v[32];
          tmem_ld32(t + (sub < 2 ? c0 : c1) + 32 * (sub & 1), v);
          tmem_wait_ld();
          const float sc = sub < 2 ? s0 : s1;
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[32 * sub + i] = fmaf(__uint_as_float(v[i]), sc, acc[32 * sub + i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[pb]);
      }
      if (!ok) break;
      // ---- epilogue from registers
      float rs = 1.f;
      int drow = row;
      if (row_ok) {
        if (p.row_scale) rs = p.row_scale[row];
        if (p.row_dest) drow = p.row_dest[row];
      }
      const bool write = row_ok && drow >= 0;
      if (SWI) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          acc[i] = silu_clamped8(acc[i], acc[64 + i], p.act_limit, p.act_alpha, p.act_beta) * rs;
        const int oc = nb * (BN / 2) + 64 * half;      // output column of acc[0]
        if (EPI == EPI_SWIGLU) {
          if (write) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.D) + (size_t)drow * p.ldd + oc);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_uint4(pack_bf16x2(acc[8 * i], acc[8 * i + 1]), pack_bf16x2(acc[8 * i + 2], acc[8 * i + 3]),
                                  pack_bf16x2(acc[8 * i + 4], acc[8 * i + 5]),
                                  pack_bf16x2(acc[8 * i + 6], acc[8 * i + 7]));
          }
        } else {
          // one scale per (row, 128 outputs): the tile's two halves hold 64 outputs each
          float am = 0.f;
#pragma unroll
          for (int i = 0; i < 64; ++i) am = fmaxf(am, fabsf(acc[i]));
          float* xb = xch + (lt & 1) * 2 * BM;
          xb[half * BM + r_in_tile] = am;
          __syncwarp();
          if (lane == 0) mbar_arrive(xbar);
          if (!mbar_wait(xbar, lt & 1, p.status, 114)) { ok = false; break; }
          am = fmaxf(am, xb[(half ^ 1) * BM + r_in_tile]);
          const float inv = am > 0.f ? 448.f / am : 0.f;
          if (write) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.D) + (size_t)drow * p.ldd + oc);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t wv[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int b = 16 * i + 4 * j;
                wv[j] = pack_e4m3x4(acc[b] * inv, acc[b + 1] * inv, acc[b + 2] * inv, acc[b + 3] * inv);
              }
              dst[i] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
            if (half == 0) p.d_scale[(size_t)drow * p.lds + nb] = am > 0.f ? am / 448.f : 1.f;
          }
        }
      } else {
        const int col0 = nb * BN + c0;                 // 128 contiguous columns from here
        void* dbase = p.D;
        if (p.peer_D != nullptr && write) {
          const int pr = drow / p.peer_rows;
          drow -= pr * p.peer_rows;
          dbase = p.peer_D[pr];
        }
        if (p.bias) {
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            const int c = min(col0 + i, p.N - 1);
            acc[i] += __bfloat162float(p.bias[c]);
          }
        }
        if (write) {
          if (EPI == EPI_F32) {
            float* dst = reinterpret_cast<float*>(dbase) + (size_t)drow * p.ldd + col0;
            if (col0 + 128 <= p.N) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                reinterpret_cast<float4*>(dst)[i] =
                    make_float4(acc[4 * i] * rs, acc[4 * i + 1] * rs, acc[4 * i + 2] * rs, acc[4 * i + 3] * rs);
            } else {
#pragma unroll
              for (int i = 0; i < 128; ++i)
                if (col0 + i < p.N) dst[i] = acc[i] * rs;
            }
          } else {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(dbase) + (size_t)drow * p.ldd + col0;
            if (col0 + 128 <= p.N) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                reinterpret_cast<uint4*>(dst)[i] =
                    make_uint4(pack_bf16x2(acc[8 * i] * rs, acc[8 * i + 1] * rs),
                               pack_bf16x2(acc[8 * i + 2] * rs, acc[8 * i + 3] * rs),
                               pack_bf16x2(acc[8 * i + 4] * rs, acc[8 * i + 5] * rs),
                               pack_bf16x2(acc[8 * i + 6] * rs, acc[8 * i + 7] * rs));
            } else {
#pragma unroll
              for (int i = 0; i < 128; ++i)
                if (col0 + i < p.N) dst[i] = __float2bfloat16(acc[i] * rs);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Rows of bf16 -> e4m3 with one fp32 scale per (row, 128 columns): scale = amax / 448
// (1 for an all-zero block), q = x * 448 / amax, saturating.  One warp per block, four
// consecutive elements per lane.
__global__ void quant_fp8_rows_kernel(const __nv_bfloat16* __restrict__ x, int rows, int K, int stride,
                                      uint8_t* __restrict__ q, float* __restrict__ s) {
  const int nb = K >> 7;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= rows * nb) return;
  const int r = gw / nb, b = gw - r * nb;
  const uint2 raw = *reinterpret_cast<const uint2*>(x + (size_t)r * stride + b * 128 + lane * 4);
  const float v0 = bf16_lo(raw.x), v1 = bf16_hi(raw.x), v2 = bf16_lo(raw.y), v3 = bf16_hi(raw.y);
  float am = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  const float inv = am > 0.f ? 448.f / am : 0.f;
  *reinterpret_cast<uint32_t*>(q + (size_t)r * K + b * 128 + lane * 4) = pack_e4m3x4(v0 * inv, v1 * inv, v2 * inv,
                                                                                     v3 * inv);
  if (lane == 0) s[(size_t)r * nb + b] = am > 0.f ? am / 448.f : 1.f;
}

}  // namespace f8
}  // namespace xtu

using namespace xtu;

typedef CUresult (*PFN_f8_encode)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [rows, cols] bytes, 128-byte swizzle, box [box_rows, 128 bytes]
static int f8_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  static PFN_f8_encode enc = nullptr;
  if (!enc) {
    void* fp = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fp, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      enc = reinterpret_cast<PFN_f8_encode>(fp);
    if (!enc) return -100;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols % 16 != 0) return -101;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1000 - (int)r;
}

static int f8_num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int EPI>
static int f8_launch(const CUtensorMap& ta, const CUtensorMap& tb, const f8::Params& p, int work, cudaStream_t s) {
  auto k = f8::gemm_fp8_kernel<EPI>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, f8::SMEM_BYTES);
    if (e != cudaSuccess) return -(int)e;
    attr = true;
  }
  const int grid = work < f8_num_sms() ? (work > 0 ? work : 1) : f8_num_sms();
  k<<<grid, f8::NUM_WARPS * 32, f8::SMEM_BYTES, s>>>(ta, tb, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

extern "C" {

// x bf16 [rows, K] (row stride `stride` elements) -> q e4m3 [rows, K], s fp32 [rows, K / 128].
int xtu_quant_fp8_rows(const void* x, int rows, int K, int stride, void* q, float* s, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (K % 128 != 0 || stride % 4 != 0) return -2;
  const long long warps = (long long)rows * (K / 128);
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  f8::quant_fp8_rows_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), rows, K, stride, reinterpret_cast<uint8_t*>(q), s);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : -(int)e;
}

// Grouped (tiles != nullptr: m-tiles from xtu_build_mtiles, E experts) or dense (E = 1) fp8 GEMM.
//   A  e4m3 [M, K], a_scale [M, K/128];  B e4m3 [E, N, K], b_scale [E, ceil(N/128), K/128]
//   epi 0: bf16 D [*, N] (ldd); 1: fp32 D; 2: clamped SwiGLU -> bf16 D [*, N/2] (B rows per 256-row
//   block: 128 gate, 128 up); 3: as 2, quantized: D e4m3 [*, N/2], d_scale [*, N/256] (row stride lds).
//   row_scale / row_dest / peer_D / peer_rows / bias as in xtu_grouped_gemm_ex (bias: epi 0/1 only).
int xtu_gemm_fp8_native(const void* A, const float* a_scale, const void* B, const float* b_scale, void* D, int ldd,
                        float* d_scale, int lds, int M, int N, int K, int E, const void* tiles, const int* count,
                        int max_tiles, int epi, const float* row_scale, const int* row_dest, const void* bias,
                        float act_limit, float act_alpha, float act_beta, void* const* peer_D, int peer_rows,
                        void* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  if (K <= 0 || K % f8::BK != 0 || a_scale == nullptr || b_scale == nullptr) return -2;
  const bool swi = epi == f8::EPI_SWIGLU || epi == f8::EPI_SWIGLU_Q8;
  if (swi && (N % f8::BN != 0 || bias != nullptr)) return -4;
  if (epi == f8::EPI_SWIGLU_Q8 && (d_scale == nullptr || ldd % 16 != 0)) return -5;
  if (peer_D != nullptr && (row_dest == nullptr || peer_rows <= 0)) return -7;
  if (epi < 0 || epi > 3) return -3;
  CUtensorMap ta, tb;
  int rc = f8_tmap(&ta, A, (uint64_t)M, (uint64_t)K, f8::BM);
  if (rc) return rc;
  rc = f8_tmap(&tb, B, (uint64_t)E * N, (uint64_t)K, f8::BN);
  if (rc) return rc;
  f8::Params p{};
  p.M = M; p.N = N; p.K = K;
  p.n_blocks = (N + f8::BN - 1) / f8::BN;
  p.tiles = reinterpret_cast<const f8::Tile*>(tiles);
  p.num_tiles = count;
  p.dense_tiles = (M + f8::BM - 1) / f8::BM;
  p.a_scale = a_scale; p.b_scale = b_scale; p.sb_n = (N + 127) / 128;
  p.D = D; p.ldd = ldd; p.d_scale = d_scale; p.lds = lds;
  p.row_scale = row_scale; p.row_dest = row_dest; p.peer_D = peer_D; p.peer_rows = peer_rows;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.act_limit = act_limit; p.act_alpha = act_alpha; p.act_beta = act_beta;
  p.status = reinterpret_cast<XtuStatus*>(status);
  const int work = (tiles ? max_tiles : p.dense_tiles) * p.n_blocks;
  switch (epi) {
    case f8::EPI_BF16: return f8_launch<f8::EPI_BF16>(ta, tb, p, work, stream);
    case f8::EPI_F32: return f8_launch<f8::EPI_F32>(ta, tb, p, work, stream);
    case f8::EPI_SWIGLU: return f8_launch<f8::EPI_SWIGLU>(ta, tb, p, work, stream);
    default: return f8_launch<f8::EPI_SWIGLU_Q8>(ta, tb, p, work, stream);
  }
}

}  // extern "C"
