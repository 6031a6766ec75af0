// Bulk work of the synthetic-model generator: seeded normal weights and the
// Q4_K / Q6_K quantisers, multithreaded. Host-only (no CUDA); the container
// format is written by wcb/synth.py.
//
// Random numbers are counter based (a splitmix64 hash of seed, tensor index and
// element pair index, then Box-Muller), so the values do not depend on the
// thread count. Block layouts follow crates/wasm-chord-core/src/quant.rs:32-38
// (BlockQ4_K) and :121-126 (BlockQ6_K); the scale packing is the inverse of
// get_scale_min_k4 (quant.rs:43-53).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// IEEE binary16 from binary32, round to nearest even (matches numpy astype).
uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t mant = x & 0x7FFFFFu;
  int32_t exp = int32_t((x >> 23) & 0xFF);
  if (exp == 0xFF) return uint16_t(sign | 0x7C00u | (mant ? 0x200u : 0u));
  int32_t e = exp - 127 + 15;
  if (e >= 31) return uint16_t(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return uint16_t(sign);
    mant |= 0x800000u;
    int shift = 14 - e;
    uint32_t half = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1))) half++;
    return uint16_t(sign | half);
  }
  uint32_t half = (uint32_t(e) << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1))) half++;
  return uint16_t(sign | half);
}

float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1F, mant = h & 0x3FF;
  uint32_t out;
  if (exp == 0) {
    if (mant == 0) {
      out = sign;
    } else {
      int e = -1;
      do { e++; mant <<= 1; } while (!(mant & 0x400));
      out = sign | (uint32_t(127 - 15 - e) << 23) | ((mant & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    out = sign | 0x7F800000u | (mant << 13);
  } else {
    out = sign | ((exp + 112) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

template <class F>
void parallel_for(int64_t n, int threads, F fn) {
  if (threads <= 1 || n < 4096) { fn(int64_t(0), n); return; }
  std::vector<std::thread> pool;
  int64_t chunk = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    int64_t a = t * chunk, b = std::min(n, a + chunk);
    if (a >= b) break;
    pool.emplace_back([=] { fn(a, b); });
  }
  for (auto& th : pool) th.join();
}

inline float rintf_even(float v) { return std::nearbyint(v); }

void quant_q4k_block(const float* x, uint8_t* out) {
  float scale[8], mneg[8];
  for (int s = 0; s < 8; ++s) {
    float mn = x[32 * s], mx = x[32 * s];
    for (int j = 1; j < 32; ++j) { mn = std::min(mn, x[32 * s + j]); mx = std::max(mx, x[32 * s + j]); }
    mn = std::min(mn, 0.0f);
    scale[s] = (mx - mn) / 15.0f;
    mneg[s] = -mn;
  }
  float smax = 0, mmax = 0;
  for (int s = 0; s < 8; ++s) { smax = std::max(smax, scale[s]); mmax = std::max(mmax, mneg[s]); }
  uint16_t d16 = f32_to_f16(smax / 63.0f), dm16 = f32_to_f16(mmax / 63.0f);
  float d = f16_to_f32(d16), dm = f16_to_f32(dm16);
  uint8_t sc[8], mq[8];
  for (int s = 0; s < 8; ++s) {
    float a = d > 0 ? rintf_even(scale[s] / d) : 0.0f;
    float b = dm > 0 ? rintf_even(mneg[s] / dm) : 0.0f;
    sc[s] = uint8_t(std::min(63.0f, std::max(0.0f, a)));
    mq[s] = uint8_t(std::min(63.0f, std::max(0.0f, b)));
  }
  uint8_t q[256];
  for (int s = 0; s < 8; ++s) {
    float d1 = d * float(sc[s]), m1 = dm * float(mq[s]);
    for (int j = 0; j < 32; ++j) {
      float v = d1 > 0 ? rintf_even((x[32 * s + j] + m1) / d1) : 0.0f;
      q[32 * s + j] = uint8_t(std::min(15.0f, std::max(0.0f, v)));
    }
  }
  std::memcpy(out, &d16, 2);
  std::memcpy(out + 2, &dm16, 2);
  for (int j = 0; j < 4; ++j) {
    out[4 + j] = uint8_t((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    out[8 + j] = uint8_t((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
    out[12 + j] = uint8_t((sc[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
  }
  for (int p = 0; p < 4; ++p)
    for (int l = 0; l < 32; ++l)
      out[16 + 32 * p + l] = uint8_t(q[64 * p + l] | (q[64 * p + 32 + l] << 4));
}

void quant_q6k_block(const float* x, uint8_t* out) {
  float scale[16];
  for (int s = 0; s < 16; ++s) {
    float amax = 0;
    for (int j = 0; j < 16; ++j) amax = std::max(amax, std::fabs(x[16 * s + j]));
    scale[s] = amax / 31.0f;
  }
  float smax = 0;
  for (int s = 0; s < 16; ++s) smax = std::max(smax, scale[s]);
  uint16_t d16 = f32_to_f16(smax / 127.0f);
  float d = f16_to_f32(d16);
  int8_t sc[16];
  for (int s = 0; s < 16; ++s) {
    float a = d > 0 ? rintf_even(scale[s] / d) : 0.0f;
    sc[s] = int8_t(std::min(127.0f, std::max(-127.0f, a)));
  }
  uint8_t q[256];
  for (int s = 0; s < 16; ++s) {
    float ds = d * float(sc[s]);
    for (int j = 0; j < 16; ++j) {
      float v = ds != 0 ? rintf_even(x[16 * s + j] / ds) : 0.0f;
      v = std::min(31.0f, std::max(-32.0f, v));
      q[16 * s + j] = uint8_t(int(v) + 32);
    }
  }
  uint8_t* ql = out;
  uint8_t* qh = out + 128;
  for (int h = 0; h < 2; ++h)
    for (int l = 0; l < 32; ++l) {
      uint8_t q1 = q[128 * h + l], q2 = q[128 * h + l + 32], q3 = q[128 * h + l + 64], q4 = q[128 * h + l + 96];
      ql[64 * h + l] = uint8_t((q1 & 0xF) | ((q3 & 0xF) << 4));
      ql[64 * h + l + 32] = uint8_t((q2 & 0xF) | ((q4 & 0xF) << 4));
      qh[32 * h + l] = uint8_t((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  std::memcpy(out + 192, sc, 16);
  std::memcpy(out + 208, &d16, 2);
}

}  // namespace

extern "C" {

// out[i] = mean + std * N(0,1), counter-based on (seed, stream, i).
void wcb_synth_fill_normal(uint64_t seed, uint64_t stream, int64_t n, float mean, float stdv,
                           float* out, int threads) {
  const uint64_t key = mix64(seed ^ mix64(stream + 0x51ED2701ull));
  parallel_for((n + 1) / 2, threads, [&](int64_t a, int64_t b) {
    for (int64_t j = a; j < b; ++j) {
      uint64_t r = mix64(key + uint64_t(j));
      double u1 = (double((r >> 11) & 0x1FFFFFull) + 0.5) / 2097152.0;  // 21 bits, (0,1)
      double u2 = double(r >> 32) / 4294967296.0;                         // [0,1)
      double rad = std::sqrt(-2.0 * std::log(u1));
      double th = 6.283185307179586 * u2;
      out[2 * j] = float(mean + stdv * rad * std::cos(th));
      if (2 * j + 1 < n) out[2 * j + 1] = float(mean + stdv * rad * std::sin(th));
    }
  });
}

void wcb_synth_quantize_q4k(const float* x, int64_t n, uint8_t* out, int threads) {
  parallel_for(n / 256, threads, [&](int64_t a, int64_t b) {
    for (int64_t i = a; i < b; ++i) quant_q4k_block(x + 256 * i, out + 144 * i);
  });
}

void wcb_synth_quantize_q6k(const float* x, int64_t n, uint8_t* out, int threads) {
  parallel_for(n / 256, threads, [&](int64_t a, int64_t b) {
    for (int64_t i = a; i < b; ++i) quant_q6k_block(x + 256 * i, out + 210 * i);
  });
}

}  // extern "C"
