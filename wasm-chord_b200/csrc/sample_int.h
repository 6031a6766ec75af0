// Integer weights for sampling over any number of candidates (the reference's
// compute_probabilities, top-k, top-p and weighted draw, sampling.rs:106-229,
// for configurations the top-k sampler of at most 1024 candidates does not
// cover: top_k = 0, or top_k > 1024).
//
// Each candidate's weight is E = floor(e * 2^31) with e = exp(l / T - max) in
// [0, 1] from wcb_exp_nonpos, so the probability of candidate i is E_i / sum E
// (the softmax, renormalised over the candidates). All sums, the top-p
// boundary and the draw are then exact integer arithmetic: their results do
// not depend on the order of the additions, so the device sampler
// (sample_dev.cu) and the host sampler (sampler.cpp) keep the same candidates
// and draw the same token for a seed. Weights below 2^-31 of the largest one
// (probabilities under 5e-10) become 0.
//
// top-p (sampling.rs:138-163) in exact arithmetic: with the candidates in the
// order (E desc, index asc), candidate r is kept while the sum of the weights
// before it is below top_p * sum E.
#pragma once
#include <cstdint>

#ifdef __CUDACC__
#define WCB_SI_HD __host__ __device__ __forceinline__
#else
#define WCB_SI_HD inline
#endif

namespace wcb {

// weight of a candidate: e in [0, 1]
WCB_SI_HD uint32_t int_weight(float e) {
  const float s = e * 2147483648.0f;  // a power of two: exact
  return s >= 2147483648.0f ? 2147483648u : (s > 0.0f ? uint32_t(s) : 0u);
}

// top_p (a float in (0, 1)) as mant * 2^-k
struct TopP {
  uint64_t mant;
  int k;
};
WCB_SI_HD TopP top_p_parts(float top_p) {
  uint32_t bits;
#ifdef __CUDA_ARCH__
  bits = __float_as_uint(top_p);
#else
  __builtin_memcpy(&bits, &top_p, 4);
#endif
  const uint32_t ex = (bits >> 23) & 0xFFu;
  TopP t;
  if (ex == 0) {
    t.mant = bits & 0x7FFFFFu;
    t.k = 149;
  } else {
    t.mant = (bits & 0x7FFFFFu) | 0x800000u;
    t.k = 150 - int(ex);
  }
  return t;
}

// x < top_p * total, exactly (x, total < 2^52)
WCB_SI_HD bool below_top_p(uint64_t x, const TopP& t, uint64_t total) {
  if (x == 0) return t.mant != 0 && total != 0;
  if (t.k > 75) return false;  // x * 2^k >= 2^76 > mant * total
  const unsigned __int128 lhs = static_cast<unsigned __int128>(x) << t.k;
  const unsigned __int128 rhs = static_cast<unsigned __int128>(t.mant) * total;
  return lhs < rhs;
}

// the draw: the 24 high bits of the splitmix64 output scaled to [0, total)
WCB_SI_HD uint64_t draw_target(uint64_t z, uint64_t total) {
  const unsigned __int128 p = static_cast<unsigned __int128>(z >> 40) * total;
  return uint64_t(p >> 24);
}

WCB_SI_HD uint64_t splitmix64_next(uint64_t* state) {
  uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace wcb
