// AVX-512 (F/BW/VL + BF16/VNNI/VBMI) micro-kernels of the CPU expert engine.
// Compiled with those ISA flags; the engine calls them only after checking CPUID.
#include <immintrin.h>

#include <cmath>
#include <cstring>

#include "moe_kernels.hpp"

namespace xtu_cpu {

namespace {

const float kE2M1[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f, -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

inline __m512 nibbles16(const uint8_t* p) {
  // 8 bytes -> 16 nibble indices in k order (low nibble = even k)
  uint64_t v8;
  std::memcpy(&v8, p, 8);
  const __m512i bytes = _mm512_cvtepu8_epi32(_mm_cvtsi64_si128((long long)v8));
  const __m512i idx = _mm512_set_epi32(7, 7, 6, 6, 5, 5, 4, 4, 3, 3, 2, 2, 1, 1, 0, 0);
  const __m512i sh = _mm512_set_epi32(4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0);
  const __m512i nib = _mm512_and_si512(_mm512_srlv_epi32(_mm512_permutexvar_epi32(idx, bytes), sh),
                                       _mm512_set1_epi32(0xF));
  return _mm512_permutexvar_ps(nib, _mm512_loadu_ps(kE2M1));
}

// 8 bytes -> 16 unsigned nibbles as fp32 in k order
inline __m512 int4x16(const uint8_t* p) {
  uint64_t v8;
  std::memcpy(&v8, p, 8);
  const __m512i bytes = _mm512_cvtepu8_epi32(_mm_cvtsi64_si128((long long)v8));
  const __m512i idx = _mm512_set_epi32(7, 7, 6, 6, 5, 5, 4, 4, 3, 3, 2, 2, 1, 1, 0, 0);
  const __m512i sh = _mm512_set_epi32(4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0);
  return _mm512_cvtepi32_ps(_mm512_and_si512(_mm512_srlv_epi32(_mm512_permutexvar_epi32(idx, bytes), sh),
                                             _mm512_set1_epi32(0xF)));
}

// 16 weights of row r starting at k (k % 16 == 0), decoded to fp32
inline __m512 decode16(const DotArgs& a, const RowRef& r, int k) {
  switch (a.fmt) {
    case FMT_BF16: {
      const __m256i v = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(r.w + 2 * (size_t)k));
      return _mm512_castsi512_ps(_mm512_slli_epi32(_mm512_cvtepu16_epi32(v), 16));
    }
    case FMT_FP8: {
      // e4m3 bits -> fp32 bits (sign | magnitude << 20) is the value * 2^-120 exactly,
      // subnormals included; the 2^120 is folded into the block scale
      const __m512i b = _mm512_cvtepu8_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(r.w + k)));
      const __m512i sign = _mm512_slli_epi32(_mm512_and_si512(b, _mm512_set1_epi32(0x80)), 24);
      const __m512i mag = _mm512_slli_epi32(_mm512_and_si512(b, _mm512_set1_epi32(0x7F)), 20);
      const float sc = reinterpret_cast<const float*>(r.s)[k >> 7] * 0x1p120f;
      return _mm512_mul_ps(_mm512_castsi512_ps(_mm512_or_si512(sign, mag)), _mm512_set1_ps(sc));
    }
    case FMT_MXFP4: {
      const float sc = std::ldexp(1.f, (int)r.s[k >> 5] - 127);
      return _mm512_mul_ps(nibbles16(r.w + (k >> 1)), _mm512_set1_ps(sc));
    }
    case FMT_INT4: {
      const float* sz = reinterpret_cast<const float*>(r.s) + 2 * (k >> 7);
      return _mm512_mul_ps(_mm512_sub_ps(int4x16(r.w + (k >> 1)), _mm512_set1_ps(sz[1])), _mm512_set1_ps(sz[0]));
    }
    default: {  // FMT_NVFP4
      const float sc = e4m3_to_f32(r.s[k >> 4]) * a.gscale;
      return _mm512_mul_ps(nibbles16(r.w + (k >> 1)), _mm512_set1_ps(sc));
    }
  }
}

template <int R, int T>
void dot_rt(const DotArgs& a, const RowRef* rows, const float* const* X, float* acc) {
  __m512 c[R][T];
#pragma GCC unroll 4
  for (int r = 0; r < R; ++r)
#pragma GCC unroll 6
    for (int t = 0; t < T; ++t) c[r][t] = _mm512_setzero_ps();
  for (int k = 0; k < a.K; k += 16) {
    __m512 w[R];
#pragma GCC unroll 4
    for (int r = 0; r < R; ++r) w[r] = decode16(a, rows[r], k);
#pragma GCC unroll 6
    for (int t = 0; t < T; ++t) {
      const __m512 xv = _mm512_loadu_ps(X[t] + k);
#pragma GCC unroll 4
      for (int r = 0; r < R; ++r) c[r][t] = _mm512_fmadd_ps(w[r], xv, c[r][t]);
    }
  }
  for (int r = 0; r < R; ++r)
    for (int t = 0; t < T; ++t) acc[r * T + t] = _mm512_reduce_add_ps(c[r][t]);
}

template <int R>
void dot_r(const DotArgs& a, const RowRef* rows, const float* const* X, int T, float* acc) {
  switch (T) {
    case 1: dot_rt<R, 1>(a, rows, X, acc); break;
    case 2: dot_rt<R, 2>(a, rows, X, acc); break;
    case 3: dot_rt<R, 3>(a, rows, X, acc); break;
    case 4: dot_rt<R, 4>(a, rows, X, acc); break;
    case 5: dot_rt<R, 5>(a, rows, X, acc); break;
    default: dot_rt<R, 6>(a, rows, X, acc); break;
  }
}

// e2m1 codes as bf16 bit patterns, twice (entries 0..15 and 16..31 of a vpermw table)
const uint16_t kE2M1Bf16[32] = {0x0000, 0x3F00, 0x3F80, 0x3FC0, 0x4000, 0x4040, 0x4080, 0x40C0,
                                0x8000, 0xBF00, 0xBF80, 0xBFC0, 0xC000, 0xC040, 0xC080, 0xC0C0,
                                0x0000, 0x3F00, 0x3F80, 0x3FC0, 0x4000, 0x4040, 0x4080, 0x40C0,
                                0x8000, 0xBF00, 0xBF80, 0xBFC0, 0xC000, 0xC040, 0xC080, 0xC0C0};

// 16 bytes of packed e2m1 -> 32 word indices in k order (low nibble = even k)
inline __m512i nibble_words32(const uint8_t* p) {
  const __m512i b = _mm512_cvtepu8_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p)));
  return _mm512_or_si512(_mm512_and_si512(b, _mm512_set1_epi32(0x0F)),
                         _mm512_slli_epi32(_mm512_and_si512(b, _mm512_set1_epi32(0xF0)), 12));
}

// 32 weights of row r from k (k % 32 == 0), decoded and rounded to bf16 pairs in k order.
// Packed 4-bit rows decode through a 32-entry bf16 table (vpermw) that already holds the
// block scale: MXFP4 adds the power-of-two scale to the exponent field of the nonzero
// codes (exact); NVFP4 scales the 16 codes of each of its two 16-element blocks in fp32
// and rounds them to bf16 once per block.
inline __m512bh decode32_bf16(const DotArgs& a, const RowRef& r, int k) {
  if (a.fmt == FMT_BF16) return (__m512bh)_mm512_loadu_si512(r.w + 2 * (size_t)k);
  if (a.fmt == FMT_MXFP4) {
    const int e = (int)r.s[k >> 5] - 127;
    if (e >= -120 && e <= 120) {
      const __m512i base = _mm512_loadu_si512(kE2M1Bf16);
      const __m512i lut = _mm512_mask_add_epi16(base, (__mmask32)0xFEFEFEFEu, base, _mm512_set1_epi16((short)(e << 7)));
      return (__m512bh)_mm512_permutexvar_epi16(nibble_words32(r.w + (k >> 1)), lut);
    }
  } else if (a.fmt == FMT_INT4) {
    // one 128-wide group covers the 32 weights: table (i - zero) * scale, i = 0..15, twice
    const float* sz = reinterpret_cast<const float*>(r.s) + 2 * (k >> 7);
    const __m512 q = _mm512_set_ps(15, 14, 13, 12, 11, 10, 9, 8, 7, 6, 5, 4, 3, 2, 1, 0);
    const __m512 v = _mm512_mul_ps(_mm512_sub_ps(q, _mm512_set1_ps(sz[1])), _mm512_set1_ps(sz[0]));
    const __m512i lut = (__m512i)_mm512_cvtne2ps_pbh(v, v);
    return (__m512bh)_mm512_permutexvar_epi16(nibble_words32(r.w + (k >> 1)), lut);
  } else if (a.fmt == FMT_NVFP4) {
    const __m512 codes = _mm512_loadu_ps(kE2M1);
    const float s0 = e4m3_to_f32(r.s[k >> 4]) * a.gscale, s1 = e4m3_to_f32(r.s[(k >> 4) + 1]) * a.gscale;
    const __m512i lut = (__m512i)_mm512_cvtne2ps_pbh(_mm512_mul_ps(codes, _mm512_set1_ps(s1)),
                                                     _mm512_mul_ps(codes, _mm512_set1_ps(s0)));
    // weights k+16 .. k+31 (words 16..31) read the second block's half of the table
    const __m512i idx = _mm512_mask_add_epi16(nibble_words32(r.w + (k >> 1)), (__mmask32)0xFFFF0000u,
                                              nibble_words32(r.w + (k >> 1)), _mm512_set1_epi16(16));
    return (__m512bh)_mm512_permutexvar_epi16(idx, lut);
  }
  return _mm512_cvtne2ps_pbh(decode16(a, r, k + 16), decode16(a, r, k));
}

template <int R, int T>
void dotbf_rt(const DotArgs& a, const RowRef* rows, const uint16_t* const* X, float* acc) {
  __m512 c[R][T];
#pragma GCC unroll 4
  for (int r = 0; r < R; ++r)
#pragma GCC unroll 6
    for (int t = 0; t < T; ++t) c[r][t] = _mm512_setzero_ps();
  for (int k = 0; k < a.K; k += 32) {
    __m512bh w[R];
#pragma GCC unroll 4
    for (int r = 0; r < R; ++r) w[r] = decode32_bf16(a, rows[r], k);
#pragma GCC unroll 6
    for (int t = 0; t < T; ++t) {
      const __m512bh xv = (__m512bh)_mm512_loadu_si512(X[t] + k);
#pragma GCC unroll 4
      for (int r = 0; r < R; ++r) c[r][t] = _mm512_dpbf16_ps(c[r][t], w[r], xv);
    }
  }
  for (int r = 0; r < R; ++r)
    for (int t = 0; t < T; ++t) acc[r * T + t] = _mm512_reduce_add_ps(c[r][t]);
}

template <int R>
void dotbf_r(const DotArgs& a, const RowRef* rows, const uint16_t* const* X, int T, float* acc) {
  switch (T) {
    case 1: dotbf_rt<R, 1>(a, rows, X, acc); break;
    case 2: dotbf_rt<R, 2>(a, rows, X, acc); break;
    case 3: dotbf_rt<R, 3>(a, rows, X, acc); break;
    case 4: dotbf_rt<R, 4>(a, rows, X, acc); break;
    case 5: dotbf_rt<R, 5>(a, rows, X, acc); break;
    default: dotbf_rt<R, 6>(a, rows, X, acc); break;
  }
}

// ---- W4A8 ----
const int8_t kW4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};   // 2 * e2m1

inline __m512i w4_64(const uint8_t* p) {
  // 32 bytes of nibbles -> 64 s8 values (2*fp4) in k order
  const __m512i v16 = _mm512_cvtepu8_epi16(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(p)));
  const __m512i lo = _mm512_and_si512(v16, _mm512_set1_epi16(0x0F));
  const __m512i hi = _mm512_slli_epi16(_mm512_and_si512(_mm512_srli_epi16(v16, 4), _mm512_set1_epi16(0x0F)), 8);
  const __m512i idx = _mm512_or_si512(lo, hi);
  const __m128i t = _mm_loadu_si128(reinterpret_cast<const __m128i*>(kW4));
  return _mm512_shuffle_epi8(_mm512_broadcast_i32x4(t), idx);
}

}  // namespace

void dot_rows_avx512(const DotArgs& a, const RowRef* rows, int R, const float* const* X, int T, float* acc) {
  switch (R) {
    case 1: dot_r<1>(a, rows, X, T, acc); break;
    case 2: dot_r<2>(a, rows, X, T, acc); break;
    case 3: dot_r<3>(a, rows, X, T, acc); break;
    default: dot_r<4>(a, rows, X, T, acc); break;
  }
}

void dot_rows_bf16_avx512(const DotArgs& a, const RowRef* rows, int R, const uint16_t* const* X, int T, float* acc) {
  switch (R) {
    case 1: dotbf_r<1>(a, rows, X, T, acc); break;
    case 2: dotbf_r<2>(a, rows, X, T, acc); break;
    case 3: dotbf_r<3>(a, rows, X, T, acc); break;
    default: dotbf_r<4>(a, rows, X, T, acc); break;
  }
}

void dot_rows_w4a8_avx512(const RowRef* rows, int R, int K, const int8_t* const* xq, const int8_t* const* xe, int T,
                          float* acc) {
  const __m512i ones = _mm512_set1_epi8(1);
  const __m512i bias = _mm512_set1_epi8((char)0x80);
  for (int r = 0; r < R; ++r) {
    __m512 c[6];
    for (int t = 0; t < T; ++t) c[t] = _mm512_setzero_ps();
    for (int k = 0; k < K; k += 64) {
      const __m512i w4 = w4_64(rows[r].w + (k >> 1));
      const __m512i sw = _mm512_dpbusd_epi32(_mm512_setzero_si512(), ones, w4);   // sum of w4 per lane
      const int b0 = rows[r].s[k >> 5], b1 = rows[r].s[(k >> 5) + 1];
      for (int t = 0; t < T; ++t) {
        const int8_t* q = xq[t] + k;
        const __m512i au8 = _mm512_xor_si512(_mm512_loadu_si512(q), bias);
        const __m512i d = _mm512_dpbusd_epi32(_mm512_setzero_si512(), au8, w4);
        const __m512i sg = _mm512_sub_epi32(d, _mm512_slli_epi32(sw, 7));      // exact sum a8 * w4 per lane
        const int e0 = xe[t][k >> 5], e1 = xe[t][(k >> 5) + 1];
        const __m512 s = _mm512_mask_mov_ps(_mm512_set1_ps(std::ldexp(1.f, e0 + b0 - 128)), (__mmask16)0xFF00,
                                            _mm512_set1_ps(std::ldexp(1.f, e1 + b1 - 128)));
        c[t] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(sg), s, c[t]);
      }
    }
    for (int t = 0; t < T; ++t) acc[r * T + t] = _mm512_reduce_add_ps(c[t]);
  }
}

}  // namespace xtu_cpu
