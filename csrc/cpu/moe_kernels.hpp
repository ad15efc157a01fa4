// Row-dot micro-kernels of the CPU expert engine.
//
// dot_rows(): acc[r][t] = sum_k W_r[k] * X_t[k] for R <= 4 weight rows and T <= 6
// activation rows (fp32), with the weight row decoded from its storage format on the
// fly.  Two implementations share this interface: AVX-512 (moe_kernels_avx512.cpp,
// compiled with -mavx512f/bw/vl/bf16/vnni/vbmi and selected at run time from CPUID)
// and portable scalar code (moe_engine.cpp).
//
// Formats (per engine row):
//   BF16  : K x bf16
//   FP8   : K x e4m3, plus K/128 fp32 scales (the 128x128 block scale of the row's block)
//   MXFP4 : K/2 bytes (low nibble = even k), plus K/32 e8m0 bytes (2^(b-127))
//   NVFP4 : K/2 bytes, plus K/16 e4m3 scales, times one fp32 global scale
#pragma once
#include <cstddef>
#include <cstdint>

namespace xtu_cpu {

// FMT_INT4: GPTQ-style 4-bit integers (low nibble = even k) with, per row and 128-wide
// group, an fp32 (scale, zero point) pair: w = (q - zero) * scale
enum Fmt : int { FMT_BF16 = 0, FMT_FP8 = 1, FMT_MXFP4 = 2, FMT_NVFP4 = 3, FMT_INT4 = 4 };

struct RowRef {
  const uint8_t* w;     // row weights
  const uint8_t* s;     // row scales (format dependent; nullptr for bf16)
};

struct DotArgs {
  int fmt;
  int K;
  float gscale;         // NVFP4 global scale (1 otherwise)
};

// scalar reference decoders (exact)
float e4m3_to_f32(uint8_t b);
float e2m1_to_f32(uint8_t nib);

// acc[r * T + t] = sum_k W_r[k] * X[t][k]  (X[t]: pointer to activation row t, fp32)
void dot_rows_scalar(const DotArgs& a, const RowRef* rows, int R, const float* const* X, int T, float* acc);
void dot_rows_avx512(const DotArgs& a, const RowRef* rows, int R, const float* const* X, int T, float* acc);
// the same with bf16 activation rows and AVX512-BF16 dot products (vdpbf16ps): each weight is
// decoded to fp32 and rounded to bf16 (the value a GPU bf16 MMA of the widened weight uses),
// products summed in fp32.  K % 32 == 0.
void dot_rows_bf16_avx512(const DotArgs& a, const RowRef* rows, int R, const uint16_t* const* X, int T, float* acc);

// INT8-activation x MXFP4 (W4A8): xq[t] = per-32 s8 activations with exponents xe[t][k/32]
// (a = a8 * 2^c), weights w = (2*fp4) * 2^(b - 128).  acc[r*T+t] = sum of exact per-block
// integer dots scaled by 2^(c + b - 128), accumulated in fp32.
void dot_rows_w4a8_scalar(const RowRef* rows, int R, int K, const int8_t* const* xq, const int8_t* const* xe, int T,
                          float* acc);
void dot_rows_w4a8_avx512(const RowRef* rows, int R, int K, const int8_t* const* xq, const int8_t* const* xe, int T,
                          float* acc);

// per-32 power-of-two s8 quantisation of one activation row: c = ceil(log2(max|a| / 127))
void quant_row_s8_pow2(const float* x, int K, int8_t* q, int8_t* e);

bool cpu_has_avx512_bf16_vnni();

}  // namespace xtu_cpu
