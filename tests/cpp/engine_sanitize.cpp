// Host-only driver for the CPU expert engine, built with -fsanitize=thread or
// -fsanitize=address,undefined by tests/test_cpu_engine.py: it creates a bf16 engine on a
// few worker threads (the NUMA work pool), runs several forward passes, checks them
// against a plain scalar MoE, and exits 0.  Any race, out-of-bounds access or undefined
// behaviour in the engine or its pool is reported by the sanitizer runtime.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

extern "C" {
void* xtu_cpu_engine_create(int fmt, int E, int H, int I, const void* w13, const void* s13, const void* w2,
                            const void* s2, const float* gs13, const float* gs2, int threads, float limit,
                            float alpha, float beta, int int8_mode, int int8_min_tokens, int deadline_ms);
int xtu_cpu_engine_forward(void* eng, int M, int K, const int* ids, const float* wts, const uint16_t* x, float* out,
                           int lo, int hi);
void xtu_cpu_engine_destroy(void* eng);
}

static uint16_t to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);   // round to nearest even
  return (uint16_t)(u >> 16);
}

static float from_bf16(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

int main() {
  const int E = 8, H = 256, I = 256, K = 2, M = 7, threads = 4;
  std::mt19937 rng(7);
  std::normal_distribution<float> nd(0.f, 1.f);
  std::vector<uint16_t> w13((size_t)E * 2 * I * H), w2((size_t)E * H * I), x((size_t)M * H);
  for (auto& v : w13) v = to_bf16(nd(rng) / 16.f);
  for (auto& v : w2) v = to_bf16(nd(rng) / 16.f);
  for (auto& v : x) v = to_bf16(nd(rng));
  std::vector<int> ids((size_t)M * K);
  std::vector<float> wts((size_t)M * K);
  for (int t = 0; t < M; ++t)
    for (int k = 0; k < K; ++k) {
      ids[t * K + k] = (t + 3 * k) % E;
      wts[t * K + k] = k == 0 ? 0.7f : 0.3f;
    }
  void* eng = xtu_cpu_engine_create(0, E, H, I, w13.data(), nullptr, w2.data(), nullptr, nullptr, nullptr, threads,
                                    0.f, 1.f, 0.f, 0, 0, 5000);
  if (!eng) {
    std::fprintf(stderr, "engine_create failed\n");
    return 2;
  }
  // scalar reference
  std::vector<float> ref((size_t)M * H, 0.f), h(I);
  for (int t = 0; t < M; ++t)
    for (int k = 0; k < K; ++k) {
      const int e = ids[t * K + k];
      for (int j = 0; j < I; ++j) {
        float g = 0.f, u = 0.f;
        for (int c = 0; c < H; ++c) {
          const float xv = from_bf16(x[(size_t)t * H + c]);
          g += xv * from_bf16(w13[((size_t)e * 2 * I + j) * H + c]);
          u += xv * from_bf16(w13[((size_t)e * 2 * I + I + j) * H + c]);
        }
        h[j] = g / (1.f + std::exp(-g)) * u;
      }
      for (int r = 0; r < H; ++r) {
        float s = 0.f;
        for (int j = 0; j < I; ++j) s += h[j] * from_bf16(w2[((size_t)e * H + r) * I + j]);
        ref[(size_t)t * H + r] += wts[t * K + k] * s;
      }
    }
  float amax = 0.f;
  for (float v : ref) amax = std::fmax(amax, std::fabs(v));
  std::vector<float> out((size_t)M * H);
  int rc = 0;
  for (int it = 0; it < 4 && rc == 0; ++it) {
    const int n = xtu_cpu_engine_forward(eng, M, K, ids.data(), wts.data(), x.data(), out.data(), 0, E);
    if (n != M * K) {
      std::fprintf(stderr, "forward computed %d pairs, expected %d\n", n, M * K);
      rc = 3;
      break;
    }
    float err = 0.f;
    for (size_t i = 0; i < out.size(); ++i) err = std::fmax(err, std::fabs(out[i] - ref[i]));
    if (err > 2e-2f * amax + 1e-3f) {
      std::fprintf(stderr, "iteration %d: max error %g (max |ref| %g)\n", it, err, amax);
      rc = 4;
    }
  }
  xtu_cpu_engine_destroy(eng);
  if (rc == 0) std::printf("engine_sanitize: ok\n");
  return rc;
}
