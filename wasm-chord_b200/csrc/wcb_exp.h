// exp(x) for x <= 0 with one fixed sequence of IEEE single-precision operations,
// so that the host sampler and the device sampler compute identical
// probabilities (and draw identical tokens for a seed). Cody-Waite reduction
// x = k ln2 + r, |r| <= ln2 / 2, with ln2 split in a short high part (k * hi is
// exact) and a low part, then the degree-7 Taylor polynomial of e^r in Horner
// form (truncation error below 2^-24 on that interval), scaled by 2^k through
// the exponent bits. Results below 2^-126 are flushed to 0, as are x < -87.
#pragma once
#include <cstdint>
#include <cstring>

#ifdef __CUDACC__
#define WCB_EXP_HD __host__ __device__
#else
#define WCB_EXP_HD
#endif

namespace wcb {

WCB_EXP_HD inline float wcb_mul(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
WCB_EXP_HD inline float wcb_add(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}

WCB_EXP_HD inline float wcb_exp_nonpos(float x) {
  if (!(x >= -87.0f)) return 0.0f;  // also NaN -> 0 (callers reject NaN before)
  if (x > 0.0f) x = 0.0f;
  const float kLog2e = 1.44269504088896341f;
  const float kLn2Hi = 0.693145751953125f;       // 12 significant bits: k * hi exact for |k| < 2^12
  const float kLn2Lo = 1.42860682030941723e-06f;  // ln2 - hi
  // k = floor(x * log2(e) + 0.5), the nearest integer to x / ln2
  const float f = wcb_add(wcb_mul(x, kLog2e), 0.5f);
  int k = int(f);                 // truncation toward zero
  if (float(k) > f) k -= 1;       // floor for negative non-integers
  const float kf = float(k);
  const float r = wcb_add(wcb_add(x, -wcb_mul(kf, kLn2Hi)), -wcb_mul(kf, kLn2Lo));
  float p = 1.0f / 5040.0f;
  p = wcb_add(wcb_mul(p, r), 1.0f / 720.0f);
  p = wcb_add(wcb_mul(p, r), 1.0f / 120.0f);
  p = wcb_add(wcb_mul(p, r), 1.0f / 24.0f);
  p = wcb_add(wcb_mul(p, r), 1.0f / 6.0f);
  p = wcb_add(wcb_mul(p, r), 0.5f);
  p = wcb_add(wcb_mul(p, r), 1.0f);
  p = wcb_add(wcb_mul(p, r), 1.0f);
  if (k < -126) return 0.0f;
  const uint32_t bits = uint32_t(k + 127) << 23;  // 2^k
  float scale;
  std::memcpy(&scale, &bits, 4);
  return wcb_mul(p, scale);
}

}  // namespace wcb
