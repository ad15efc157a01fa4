// CPU expert engine: routed-expert MoE for the cold tier, computed on the host
// concurrently with the GPU.
//
// * Single weight copy, NUMA-sharded: at construction the engine copies every expert's
//   weights into memory it owns, split by rows across NUMA nodes -- node n holds columns
//   j in [j0_n, j1_n) of the gate/up projection (both the gate row and the up row of
//   each j) and rows [h0_n, h1_n) of the down projection -- so each node streams only
//   its own DRAM.  The caller may free its copy afterwards (reference behaviour:
//   xiaotu_moe/csrc/moe/moe_v2.hpp:537-640, mixed_experts.py:913-992).
// * forward(M, K, ids, weights, x, out): pairs whose expert lies outside [lo, hi) or whose
//   weight is 0 are skipped (EP-remote, GPU-tier and masked pairs cost nothing).  Phase A
//   computes h = SwiGLU_clamped(x W_gate^T, x W_up^T) per expert in 16-column tasks; phase B
//   computes out += w * (h W_down^T) in 16-row tasks that own their output columns, so
//   no atomics are needed and the result is deterministic.
// * Formats: BF16, FP8 e4m3 with 128x128 fp32 block scales, MXFP4 (e2m1 + e8m0/32),
//   NVFP4 (e2m1 + e4m3/16 + fp32 global).  MXFP4 can use INT8 activations (per-32
//   power-of-two s8 quantisation, exact integer block dots; the reference's W4A8 scheme,
//   moe_v2_packed4_w4a8.inc:380-435) once M reaches `int8_min_tokens`.
// * Clamped SwiGLU with the semantics of xiaotu_moe/csrc/moe/moe_v2.hpp:174-190:
//   clamp(g, max=limit) * sigmoid(alpha * g') * (clamp(u, +-limit) + beta).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

#include "moe_kernels.hpp"
#include "numa_pool.hpp"

namespace xtu_cpu {

// ---------------------------------------------------------------------------
// scalar decoders and kernels (portable; also the oracle of the AVX-512 ones)
// ---------------------------------------------------------------------------
float e4m3_to_f32(uint8_t b) {
  const int s = b >> 7, e = (b >> 3) & 0xF, m = b & 7;
  if (e == 0xF && m == 7) return 0.f;   // NaN code: treated as 0 like the reference engine
  float v = e == 0 ? std::ldexp((float)m, -9) : std::ldexp(1.f + m / 8.f, e - 7);
  return s ? -v : v;
}

float e2m1_to_f32(uint8_t nib) {
  static const float t[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float v = t[nib & 7];
  return (nib & 8) ? -v : v;
}

static float w_at(const DotArgs& a, const RowRef& r, int k) {
  switch (a.fmt) {
    case FMT_BF16: {
      uint16_t h;
      std::memcpy(&h, r.w + 2 * (size_t)k, 2);
      uint32_t u = (uint32_t)h << 16;
      float f;
      std::memcpy(&f, &u, 4);
      return f;
    }
    case FMT_FP8: return e4m3_to_f32(r.w[k]) * reinterpret_cast<const float*>(r.s)[k >> 7];
    case FMT_MXFP4: {
      const uint8_t byte = r.w[k >> 1];
      return e2m1_to_f32((k & 1) ? (byte >> 4) : (byte & 0xF)) * std::ldexp(1.f, (int)r.s[k >> 5] - 127);
    }
    case FMT_INT4: {
      const uint8_t byte = r.w[k >> 1];
      const float* sz = reinterpret_cast<const float*>(r.s) + 2 * (k >> 7);
      return ((float)((k & 1) ? (byte >> 4) : (byte & 0xF)) - sz[1]) * sz[0];
    }
    default: {
      const uint8_t byte = r.w[k >> 1];
      return e2m1_to_f32((k & 1) ? (byte >> 4) : (byte & 0xF)) * e4m3_to_f32(r.s[k >> 4]) * a.gscale;
    }
  }
}

void dot_rows_scalar(const DotArgs& a, const RowRef* rows, int R, const float* const* X, int T, float* acc) {
  for (int r = 0; r < R; ++r)
    for (int t = 0; t < T; ++t) acc[r * T + t] = 0.f;
  for (int k = 0; k < a.K; ++k)
    for (int r = 0; r < R; ++r) {
      const float w = w_at(a, rows[r], k);
      for (int t = 0; t < T; ++t) acc[r * T + t] += w * X[t][k];
    }
}

void quant_row_s8_pow2(const float* x, int K, int8_t* q, int8_t* e) {
  for (int b = 0; b < K / 32; ++b) {
    float m = 0.f;
    for (int i = 0; i < 32; ++i) m = std::fmax(m, std::fabs(x[b * 32 + i]));
    int c = -127;
    if (m > 0.f) {
      c = (int)std::ceil(std::log2(m / 127.f));
      while (m / std::ldexp(1.f, c) > 127.f) ++c;   // guard rounding of log2
    }
    e[b] = (int8_t)std::max(-127, std::min(127, c));
    const float inv = std::ldexp(1.f, -c);
    for (int i = 0; i < 32; ++i) {
      const float v = std::nearbyint(x[b * 32 + i] * inv);
      q[b * 32 + i] = (int8_t)std::max(-127.f, std::min(127.f, v));
    }
  }
}

void dot_rows_w4a8_scalar(const RowRef* rows, int R, int K, const int8_t* const* xq, const int8_t* const* xe, int T,
                          float* acc) {
  static const int w4t[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
  for (int r = 0; r < R; ++r)
    for (int t = 0; t < T; ++t) {
      float s = 0.f;
      for (int b = 0; b < K / 32; ++b) {
        int dot = 0;
        for (int i = 0; i < 32; ++i) {
          const int k = b * 32 + i;
          const uint8_t byte = rows[r].w[k >> 1];
          dot += w4t[(k & 1) ? (byte >> 4) : (byte & 0xF)] * xq[t][k];
        }
        s += std::ldexp((float)dot, (int)xe[t][b] + (int)rows[r].s[b] - 128);
      }
      acc[r * T + t] = s;
    }
}

bool cpu_has_avx512_bf16_vnni() {
  __builtin_cpu_init();
  return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
         __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("avx512vnni") &&
         __builtin_cpu_supports("avx512bf16") && __builtin_cpu_supports("avx512vbmi");
}

// ---------------------------------------------------------------------------
// engine
// ---------------------------------------------------------------------------
struct EngineCfg {
  int fmt, E, H, I;
  int threads;
  float limit, alpha, beta;
  int int8_mode;          // 0 off, 1 on (MXFP4), 2 auto (on when M >= int8_min_tokens)
  int int8_min_tokens;
  int deadline_ms;
};

static size_t row_bytes(int fmt, int K) {
  switch (fmt) {
    case FMT_BF16: return 2 * (size_t)K;
    case FMT_FP8: return (size_t)K;
    default: return (size_t)K / 2;
  }
}
static size_t scale_bytes(int fmt, int K) {
  switch (fmt) {
    case FMT_BF16: return 0;
    case FMT_FP8: return 4 * (size_t)((K + 127) / 128);
    case FMT_MXFP4: return (size_t)K / 32;
    case FMT_INT4: return 8 * (size_t)(K / 128);
    default: return (size_t)K / 16;
  }
}

struct NodeShard {
  int j0 = 0, j1 = 0;     // gate/up columns
  int h0 = 0, h1 = 0;     // down rows
  uint8_t* w13 = nullptr; size_t w13_bytes = 0;    // [E][2][j1-j0][row]
  uint8_t* s13 = nullptr; size_t s13_bytes = 0;
  uint8_t* w2 = nullptr;  size_t w2_bytes = 0;     // [E][h1-h0][row]
  uint8_t* s2 = nullptr;  size_t s2_bytes = 0;
};

class Engine {
 public:
  Engine(const EngineCfg& c, const uint8_t* w13, const uint8_t* s13, const uint8_t* w2, const uint8_t* s2,
         const float* gs13, const float* gs2)
      : cfg_(c), pool_(c.threads, c.deadline_ms) {
    avx512_ = cpu_has_avx512_bf16_vnni() && std::getenv("XTU_CPU_SCALAR") == nullptr;
    // bf16 activations with vdpbf16ps unless XIAOTU_MOE_BF16DOT=0 (then fp32 FMAs on decoded weights)
    const char* bd = std::getenv("XIAOTU_MOE_BF16DOT");
    bf16dot_ = avx512_ && !(bd && bd[0] == '0');
    const int nn = pool_.num_nodes();
    shards_.resize(nn);
    const int H = c.H, I = c.I, E = c.E;
    const size_t rb13 = row_bytes(c.fmt, H), sb13 = scale_bytes(c.fmt, H);
    const size_t rb2 = row_bytes(c.fmt, I), sb2 = scale_bytes(c.fmt, I);
    // Split over nodes: gate/up columns in whole 128-column blocks, down rows 16-aligned.
    // Each node's gate/up rows are stored in the GPU kernels' interleaved order -- per
    // 128-column block, 128 gate rows then the matching 128 up rows -- so a node's slice of
    // an expert is one contiguous range that the prefill ring can DMA as is.
    const int nb = I / 128;
    for (int n = 0; n < nn; ++n) {
      NodeShard& s = shards_[n];
      s.j0 = (int)((long)nb * n / nn) * 128;
      s.j1 = (int)((long)nb * (n + 1) / nn) * 128;
      s.h0 = (int)((long)H * n / nn) & ~15;
      s.h1 = n + 1 == nn ? H : (int)((long)H * (n + 1) / nn) & ~15;
      const int jn = s.j1 - s.j0, hn = s.h1 - s.h0;
      s.w13_bytes = (size_t)E * 2 * jn * rb13;
      s.s13_bytes = (size_t)E * 2 * jn * sb13;
      s.w2_bytes = (size_t)E * hn * rb2;
      s.s2_bytes = (size_t)E * hn * sb2;
      s.w13 = (uint8_t*)alloc_on_node(s.w13_bytes, n);
      s.s13 = (uint8_t*)alloc_on_node(s.s13_bytes, n);
      s.w2 = (uint8_t*)alloc_on_node(s.w2_bytes, n);
      s.s2 = (uint8_t*)alloc_on_node(s.s2_bytes, n);
    }
    // fill shards in parallel: (node, expert) tasks, each written by a worker of that node
    std::vector<int> counts(nn, E);
    pool_.parallel_for_nodes(counts, [&](int n, int e) {
      NodeShard& s = shards_[n];
      const int jn = s.j1 - s.j0, hn = s.h1 - s.h0;
      for (int half = 0; half < 2; ++half)
        for (int j = 0; j < jn; ++j) {
          const int src_row = half * I + s.j0 + j;      // checkpoint: gate rows then up rows
          const size_t dst = w13_row(e, jn, j, half);
          std::memcpy(s.w13 + dst * rb13, w13 + ((size_t)e * 2 * I + src_row) * rb13, rb13);
          copy_scales(s.s13 + dst * sb13, s13, e, 2 * I, H, src_row);
        }
      for (int h = 0; h < hn; ++h) {
        const size_t dst = (size_t)e * hn + h;
        std::memcpy(s.w2 + dst * rb2, w2 + ((size_t)e * H + s.h0 + h) * rb2, rb2);
        copy_scales(s.s2 + dst * sb2, s2, e, H, I, s.h0 + h);
      }
    });
    if (gs13) gs13_.assign(gs13, gs13 + E);
    if (gs2) gs2_.assign(gs2, gs2 + E);
  }

  ~Engine() {
    for (auto& s : shards_) {
      free_on_node(s.w13, s.w13_bytes);
      free_on_node(s.s13, s.s13_bytes);
      free_on_node(s.w2, s.w2_bytes);
      free_on_node(s.s2, s.s2_bytes);
    }
  }

  // row index inside a node shard: [e][j/128][half][j%128]
  static size_t w13_row(int e, int jn, int j, int half) {
    return ((size_t)e * (jn / 128) + j / 128) * 256 + half * 128 + (j % 128);
  }

  const NodeShard& shard(int n) const { return shards_[n]; }
  int fmt() const { return cfg_.fmt; }

  // scales of checkpoint row `row` (of a [E][rows][K] matrix) -> this engine's per-row layout
  void copy_scales(uint8_t* dst, const uint8_t* src, int e, int rows, int K, int row) const {
    switch (cfg_.fmt) {
      case FMT_BF16: return;
      case FMT_FP8: {   // checkpoint [E][ceil(rows/128)][ceil(K/128)] fp32 -> per row [ceil(K/128)]
        const int kb = (K + 127) / 128, rbk = (rows + 127) / 128;
        std::memcpy(dst, src + (((size_t)e * rbk + row / 128) * kb) * 4, (size_t)kb * 4);
        return;
      }
      case FMT_MXFP4:
        std::memcpy(dst, src + ((size_t)e * rows + row) * (K / 32), K / 32);
        return;
      case FMT_INT4:     // checkpoint [E][rows][K/128][2] fp32 (scale, zero)
        std::memcpy(dst, src + ((size_t)e * rows + row) * (K / 128) * 8, (size_t)(K / 128) * 8);
        return;
      default:
        std::memcpy(dst, src + ((size_t)e * rows + row) * (K / 16), K / 16);
        return;
    }
  }

  size_t bytes() const {
    size_t b = 0;
    for (auto& s : shards_) b += s.w13_bytes + s.s13_bytes + s.w2_bytes + s.s2_bytes;
    return b;
  }
  int nodes() const { return pool_.num_nodes(); }
  int threads() const { return pool_.num_threads(); }
  bool avx512() const { return avx512_; }
  bool timed_out() const { return pool_.timed_out(); }

  int forward(int M, int K, const int* ids, const float* wts, const uint16_t* x, float* out, int lo, int hi) {
    const int H = cfg_.H, I = cfg_.I, E = cfg_.E;
    std::memset(out, 0, sizeof(float) * (size_t)M * H);
    // 1) group (token, k) pairs by local expert; skip remote / masked pairs
    std::vector<int> cnt(E + 1, 0);
    for (int p = 0; p < M * K; ++p) {
      const int id = ids[p];
      if (id < lo || id >= hi || id - lo >= E || wts[p] == 0.f) continue;
      ++cnt[id - lo + 1];
    }
    for (int e = 0; e < E; ++e) cnt[e + 1] += cnt[e];
    const int P = cnt[E];
    if (P == 0) return 0;
    std::vector<int> seg(cnt.begin(), cnt.end()), cur(cnt.begin(), cnt.end() - 1);
    std::vector<int> ptok(P);
    std::vector<float> pw(P);
    for (int p = 0; p < M * K; ++p) {
      const int id = ids[p];
      if (id < lo || id >= hi || id - lo >= E || wts[p] == 0.f) continue;
      const int q = cur[id - lo]++;
      ptok[q] = p / K;
      pw[q] = wts[p];
    }
    std::vector<int> active;
    for (int e = 0; e < E; ++e)
      if (seg[e + 1] > seg[e]) active.push_back(e);
    // 2) activations once per token (not per pair), converted / quantised in parallel:
    // bf16 rows are read as they are by the BF16 dot kernels; the fp32 path and the INT8
    // path (MXFP4 x s8) convert each token row once
    const bool int8 = cfg_.fmt == FMT_MXFP4 && H % 64 == 0 &&
                      (cfg_.int8_mode == 1 || (cfg_.int8_mode == 2 && M >= cfg_.int8_min_tokens));
    const bool dp = bf16dot_ && !int8 && H % 32 == 0 && I % 32 == 0;
    if (!dp) {
      xf_.resize((size_t)M * H);
      if (int8) {
        xq_.resize((size_t)M * H);
        xe_.resize((size_t)M * H / 32);
      }
      parallel_rows(M, [&](int t) {
        const uint16_t* src = x + (size_t)t * H;
        float* dst = xf_.data() + (size_t)t * H;
        for (int k = 0; k < H; ++k) {
          const uint32_t u = (uint32_t)src[k] << 16;
          std::memcpy(dst + k, &u, 4);
        }
        if (int8) quant_row_s8_pow2(dst, H, xq_.data() + (size_t)t * H, xe_.data() + (size_t)t * H / 32);
      });
    }
    if (dp) hb16_.resize((size_t)P * I);
    else hbuf_.resize((size_t)P * I);
    const int nn = pool_.num_nodes();
    // 3) phase A: per node, tasks of 16 gate/up columns over all active experts
    std::vector<int> countsA(nn), countsB(nn);
    for (int n = 0; n < nn; ++n) {
      countsA[n] = (shards_[n].j1 - shards_[n].j0 + 15) / 16;
      countsB[n] = (shards_[n].h1 - shards_[n].h0 + 15) / 16;
    }
    pool_.parallel_for_nodes(countsA, [&](int n, int task) {
      const NodeShard& s = shards_[n];
      const int jn = s.j1 - s.j0;
      const int jt0 = task * 16, jt1 = std::min(jn, jt0 + 16);
      const size_t rb = row_bytes(cfg_.fmt, H), sb = scale_bytes(cfg_.fmt, H);
      for (int e : active) {
        const int q0 = seg[e], q1 = seg[e + 1];
        DotArgs da{cfg_.fmt, H, gs13_.empty() ? 1.f : gs13_[e]};
        for (int j = jt0; j < jt1; j += 2) {
          const int nj = std::min(2, jt1 - j);
          RowRef rows[4];
          for (int u = 0; u < nj; ++u) {
            const size_t g = w13_row(e, jn, j + u, 0), up = w13_row(e, jn, j + u, 1);
            rows[2 * u] = {s.w13 + g * rb, s.s13 + g * sb};
            rows[2 * u + 1] = {s.w13 + up * rb, s.s13 + up * sb};
          }
          for (int q = q0; q < q1; q += 6) {
            const int T = std::min(6, q1 - q);
            float acc[4 * 6];
            if (int8) {
              const int8_t* xq[6];
              const int8_t* xe[6];
              for (int t = 0; t < T; ++t) {
                xq[t] = xq_.data() + (size_t)ptok[q + t] * H;
                xe[t] = xe_.data() + (size_t)ptok[q + t] * H / 32;
              }
              (avx512_ ? dot_rows_w4a8_avx512 : dot_rows_w4a8_scalar)(rows, 2 * nj, H, xq, xe, T, acc);
            } else if (dp) {
              const uint16_t* xr[6];
              for (int t = 0; t < T; ++t) xr[t] = x + (size_t)ptok[q + t] * H;
              dot_rows_bf16_avx512(da, rows, 2 * nj, xr, T, acc);
            } else {
              const float* xr[6];
              for (int t = 0; t < T; ++t) xr[t] = xf_.data() + (size_t)ptok[q + t] * H;
              (avx512_ ? dot_rows_avx512 : dot_rows_scalar)(da, rows, 2 * nj, xr, T, acc);
            }
            for (int u = 0; u < nj; ++u)
              for (int t = 0; t < T; ++t) {
                float gv = acc[(2 * u) * T + t], uv = acc[(2 * u + 1) * T + t];
                if (cfg_.limit > 0.f) {
                  gv = std::fmin(gv, cfg_.limit);
                  uv = std::fmax(std::fmin(uv, cfg_.limit), -cfg_.limit);
                }
                const float h = (gv / (1.f + std::exp(-cfg_.alpha * gv))) * (uv + cfg_.beta);
                if (dp) hb16_[(size_t)(q + t) * I + s.j0 + j + u] = f32_to_bf16_rne(h);
                else hbuf_[(size_t)(q + t) * I + s.j0 + j + u] = h;
              }
          }
        }
      }
    });
    // 4) phase B: per node, tasks of 16 down rows; each task owns out[:, rows]
    pool_.parallel_for_nodes(countsB, [&](int n, int task) {
      const NodeShard& s = shards_[n];
      const int hn = s.h1 - s.h0;
      const int ht0 = task * 16, ht1 = std::min(hn, ht0 + 16);
      const size_t rb = row_bytes(cfg_.fmt, I), sb = scale_bytes(cfg_.fmt, I);
      for (int e : active) {
        const int q0 = seg[e], q1 = seg[e + 1];
        DotArgs da{cfg_.fmt, I, gs2_.empty() ? 1.f : gs2_[e]};
        for (int h = ht0; h < ht1; h += 4) {
          const int nr = std::min(4, ht1 - h);
          RowRef rows[4];
          for (int u = 0; u < nr; ++u) {
            const size_t r = (size_t)e * hn + h + u;
            rows[u] = {s.w2 + r * rb, s.s2 + r * sb};
          }
          for (int q = q0; q < q1; q += 6) {
            const int T = std::min(6, q1 - q);
            float acc[4 * 6];
            if (dp) {
              const uint16_t* hr[6];
              for (int t = 0; t < T; ++t) hr[t] = hb16_.data() + (size_t)(q + t) * I;
              dot_rows_bf16_avx512(da, rows, nr, hr, T, acc);
            } else {
              const float* hr[6];
              for (int t = 0; t < T; ++t) hr[t] = hbuf_.data() + (size_t)(q + t) * I;
              (avx512_ ? dot_rows_avx512 : dot_rows_scalar)(da, rows, nr, hr, T, acc);
            }
            for (int u = 0; u < nr; ++u)
              for (int t = 0; t < T; ++t)
                out[(size_t)ptok[q + t] * H + s.h0 + h + u] += pw[q + t] * acc[u * T + t];
          }
        }
      }
    });
    return P;
  }

 private:
  EngineCfg cfg_;
  WorkerPool pool_;
  bool avx512_ = false;
  std::vector<NodeShard> shards_;
  std::vector<float> gs13_, gs2_;
  std::vector<float> xf_, hbuf_;
  std::vector<uint16_t> hb16_;
  std::vector<int8_t> xq_, xe_;
  bool bf16dot_ = false;

  static uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
  }

  // fn(t) for every token row t in [0, M), chunks of 8 rows dealt over the NUMA nodes' workers
  template <typename F>
  void parallel_rows(int M, F fn) {
    const int nn = pool_.num_nodes();
    const int chunks = (M + 7) / 8;
    std::vector<int> counts(nn, 0);
    for (int c = 0; c < chunks; ++c) ++counts[c % nn];
    pool_.parallel_for_nodes(counts, [&](int n, int i) {
      const int c = i * nn + n;
      for (int t = c * 8; t < std::min(M, c * 8 + 8); ++t) fn(t);
    });
  }
};

}  // namespace xtu_cpu

using namespace xtu_cpu;

extern "C" {

// Weights in checkpoint layout: w13 [E, 2I, H] (gate rows then up rows), w2 [E, H, I];
// scales: fp8 [E, ceil(rows/128), ceil(K/128)] fp32; mxfp4 [E, rows, K/32] e8m0;
// nvfp4 [E, rows, K/16] e4m3 + per-expert global scales gs13/gs2.
void* xtu_cpu_engine_create(int fmt, int E, int H, int I, const void* w13, const void* s13, const void* w2,
                            const void* s2, const float* gs13, const float* gs2, int threads, float limit,
                            float alpha, float beta, int int8_mode, int int8_min_tokens, int deadline_ms) {
  if (H % 16 || I % 128) return nullptr;
  EngineCfg c{fmt, E, H, I, threads, limit, alpha, beta, int8_mode, int8_min_tokens, deadline_ms};
  try {
    return new Engine(c, (const uint8_t*)w13, (const uint8_t*)s13, (const uint8_t*)w2, (const uint8_t*)s2, gs13, gs2);
  } catch (...) {
    return nullptr;
  }
}

// x: [M, H] bf16 bits; ids/wts: [M, K]; out: [M, H] fp32 (overwritten).  Returns pairs computed.
int xtu_cpu_engine_forward(void* eng, int M, int K, const int* ids, const float* wts, const uint16_t* x, float* out,
                           int lo, int hi) {
  if (!eng) return -1;
  return static_cast<Engine*>(eng)->forward(M, K, ids, wts, x, out, lo, hi);
}

// info[0] = bytes held, [1] = NUMA nodes, [2] = threads, [3] = AVX-512 path, [4] = deadline exceeded
int xtu_cpu_engine_info(void* eng, long long* info) {
  if (!eng) return -1;
  Engine* e = static_cast<Engine*>(eng);
  info[0] = (long long)e->bytes();
  info[1] = e->nodes();
  info[2] = e->threads();
  info[3] = e->avx512() ? 1 : 0;
  info[4] = e->timed_out() ? 1 : 0;
  return 0;
}

void xtu_cpu_engine_destroy(void* eng) { delete static_cast<Engine*>(eng); }

// Shard n of the engine (for DMA): ptrs = {w13, s13, w2, s2}; ranges = {j0, j1, h0, h1};
// bytes = {w13, s13, w2, s2}.  w13 rows: [E][(j1-j0)/128][2][128][row]; w2 rows: [E][h1-h0][row].
int xtu_cpu_engine_shard(void* eng, int n, void** ptrs, int* ranges, long long* bytes) {
  Engine* e = static_cast<Engine*>(eng);
  if (!e || n < 0 || n >= e->nodes()) return -1;
  const NodeShard& s = e->shard(n);
  ptrs[0] = s.w13; ptrs[1] = s.s13; ptrs[2] = s.w2; ptrs[3] = s.s2;
  ranges[0] = s.j0; ranges[1] = s.j1; ranges[2] = s.h0; ranges[3] = s.h1;
  bytes[0] = (long long)s.w13_bytes; bytes[1] = (long long)s.s13_bytes;
  bytes[2] = (long long)s.w2_bytes; bytes[3] = (long long)s.s2_bytes;
  return 0;
}

// exact decoders exposed for conformance tests
float xtu_cpu_e4m3_to_f32(int b) { return e4m3_to_f32((uint8_t)b); }
int xtu_cpu_quant_s8(const float* x, int K, int8_t* q, int8_t* e) {
  quant_row_s8_pow2(x, K, q, e);
  return 0;
}

}  // extern "C"
