// rg_rng.cpp -- the reference's SplitMix64 generator and f32 draws (src/rng.rs:10-58),
// used to build the benchmark configurations bit-identically to the reference.
//
// SplitMix64 is counter based (the n-th state is seed ^ G + n * G), so large
// fills split the index range across threads and still produce the exact
// sequence a single generator would.
#include <math.h>
#include <stdint.h>

#include <thread>
#include <vector>

#include "../../include/rg_npu.h"

namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

inline uint64_t mix(uint64_t z) {  // rng.rs:23-26
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
inline float uniform_of(uint64_t u) { return (float)(u >> 40) / 16777216.0f; }  // rng.rs:30-32

// Box-Muller cosine branch (rng.rs:40-44), f32 steps without contraction.
inline float normal_of(uint64_t u1, uint64_t u2) {
  const float a = fmaxf(uniform_of(u1), 1e-7f);
  const float b = uniform_of(u2);
  const float two_pi = 2.0f * 3.14159265358979323846f;
  const float l = logf(a);
  const float s = sqrtf(-2.0f * l);
  const float c = cosf(two_pi * b);
  return s * c;
}

template <class F>
void parallel_range(int64_t n, F f) {
  const int64_t kMin = 1 << 20;
  unsigned hw = std::thread::hardware_concurrency();
  int64_t nt = hw ? (int64_t)hw : 1;
  if (nt > 64) nt = 64;
  if (n < kMin || nt <= 1) { f(0, n); return; }
  if (nt > n / kMin) nt = n / kMin;
  std::vector<std::thread> ts;
  for (int64_t t = 0; t < nt; ++t) {
    const int64_t b = n * t / nt, e = n * (t + 1) / nt;
    ts.emplace_back([=] { f(b, e); });
  }
  for (auto& t : ts) t.join();
}

}  // namespace

extern "C" {

void rg_rng_seed(rg_rng* r, uint64_t seed) { r->state = seed ^ kGolden; }

uint64_t rg_rng_next_u64(rg_rng* r) {
  r->state += kGolden;
  return mix(r->state);
}

void rg_rng_fill_uniform(rg_rng* r, float* out, int64_t n, float lo, float hi) {
  const uint64_t s0 = r->state;
  const float span = hi - lo;
  parallel_range(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) {
      const float u = uniform_of(mix(s0 + (uint64_t)(i + 1) * kGolden));
      const float t = span * u;
      out[i] = lo + t;  // lo + (hi - lo) * u (rng.rs:35-37)
    }
  });
  r->state = s0 + (uint64_t)n * kGolden;
}

void rg_rng_fill_normal(rg_rng* r, float* out, int64_t n, float std_scale) {
  const uint64_t s0 = r->state;
  parallel_range(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) {
      const uint64_t u1 = mix(s0 + (uint64_t)(2 * i + 1) * kGolden);
      const uint64_t u2 = mix(s0 + (uint64_t)(2 * i + 2) * kGolden);
      const float v = normal_of(u1, u2);
      out[i] = v * std_scale;  // detach_scaled (nn/init.rs:30-32); exact when std_scale == 1
    }
  });
  r->state = s0 + (uint64_t)(2 * n) * kGolden;
}

void rg_rng_fill_below(rg_rng* r, int64_t* out, int64_t n, uint64_t bound) {
  for (int64_t i = 0; i < n; ++i) out[i] = (int64_t)(rg_rng_next_u64(r) % bound);
}

float rg_kaiming_bound(int64_t fan_in) {  // nn/init.rs:7
  const float f = (float)(fan_in > 1 ? fan_in : 1);
  return sqrtf(6.0f / f);
}

float rg_bias_bound(int64_t fan_in) {  // nn/init.rs:24
  const float f = (float)(fan_in > 1 ? fan_in : 1);
  return 1.0f / sqrtf(f);
}

}  // extern "C"
