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

// ---------------------------------------------------------------------------
// The random stream of the reference's LogitsProcessor: rand 0.9
// `rngs::StdRng::seed_from_u64(seed)` (sampling.rs:40, :75), a third-party crate
// restated from its published algorithms:
//  * StdRng is rand_chacha's ChaCha12Rng: the ChaCha block function
//    (D. J. Bernstein; RFC 8439 section 2.3 with 12 rounds instead of 20) keyed by
//    the 32-byte seed, a 64-bit block counter from 0 in words 12-13 and a zero
//    64-bit stream id in words 14-15. next_u32 hands out the keystream words in
//    order: output w is word w % 16 of block w / 16.
//  * SeedableRng::seed_from_u64 (rand_core 0.9) fills the seed 4 bytes at a time,
//    little endian, from PCG32 (XSH-RR output) whose 64-bit state is advanced
//    before each output: s = s * 6364136223846793005 + 11634580027462260723.
//  * A draw of WeightedIndex (sampling.rs:128-132) is one Uniform<f32>(0, total)
//    sample: the 23 high bits of next_u32 as the mantissa of a float in [1, 2),
//    minus 1, times the range's scale. Uniform::new(0, total) keeps scale = total:
//    (1 - 2^-23) * total rounds to a float below total for every positive normal
//    total, so its one-ulp reduction loop never runs.
// ---------------------------------------------------------------------------
struct StdRng {
  uint32_t key[8];
  uint64_t word;  // u32 outputs taken so far
};

WCB_SI_HD uint32_t rotl32(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }

#define WCB_CHACHA_QR(a, b, c, d)               \
  x[a] += x[b], x[d] = rotl32(x[d] ^ x[a], 16); \
  x[c] += x[d], x[b] = rotl32(x[b] ^ x[c], 12); \
  x[a] += x[b], x[d] = rotl32(x[d] ^ x[a], 8);  \
  x[c] += x[d], x[b] = rotl32(x[b] ^ x[c], 7)

// word j of the ChaCha keystream block `block` under `key` (64-bit counter, zero
// stream id) after `double_rounds` column + diagonal rounds
WCB_SI_HD uint32_t chacha_word(const uint32_t* key, uint64_t block, int j, int double_rounds) {
  uint32_t x[16];
  x[0] = 0x61707865u;  // "expand 32-byte k"
  x[1] = 0x3320646eu;
  x[2] = 0x79622d32u;
  x[3] = 0x6b206574u;
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int i = 0; i < 8; ++i) x[4 + i] = key[i];
  x[12] = uint32_t(block);
  x[13] = uint32_t(block >> 32);
  x[14] = 0u;
  x[15] = 0u;
  for (int r = 0; r < double_rounds; ++r) {
    WCB_CHACHA_QR(0, 4, 8, 12);
    WCB_CHACHA_QR(1, 5, 9, 13);
    WCB_CHACHA_QR(2, 6, 10, 14);
    WCB_CHACHA_QR(3, 7, 11, 15);
    WCB_CHACHA_QR(0, 5, 10, 15);
    WCB_CHACHA_QR(1, 6, 11, 12);
    WCB_CHACHA_QR(2, 7, 8, 13);
    WCB_CHACHA_QR(3, 4, 9, 14);
  }
  uint32_t out = 0;
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int i = 0; i < 16; ++i)  // a select, not an indexed load: x stays in registers
    if (i == j) out = x[i];
  // plus input word j (the state before the rounds)
  uint32_t in;
  if (j < 4) in = j == 0 ? 0x61707865u : j == 1 ? 0x3320646eu : j == 2 ? 0x79622d32u : 0x6b206574u;
  else if (j < 12) in = key[j - 4];
  else in = j == 12 ? uint32_t(block) : j == 13 ? uint32_t(block >> 32) : 0u;
  return out + in;
}
#undef WCB_CHACHA_QR

WCB_SI_HD uint32_t std_rng_next_u32(StdRng* r) {
  const uint64_t w = r->word++;
  return chacha_word(r->key, w >> 4, int(w & 15), 6);
}

inline StdRng std_rng_seed_from_u64(uint64_t s) {
  StdRng r;
  for (int i = 0; i < 8; ++i) {
    s = s * 6364136223846793005ull + 11634580027462260723ull;
    const uint32_t xorshifted = uint32_t(((s >> 18) ^ s) >> 27);
    const int rot = int(s >> 59);
    r.key[i] = rot ? (xorshifted >> rot) | (xorshifted << (32 - rot)) : xorshifted;  // 4 LE bytes = one key word
  }
  r.word = 0;
  return r;
}

// Uniform<f32>'s value in [0, 1 - 2^-23] from one u32 of the stream
WCB_SI_HD float unit_f32(uint32_t w) {
  const uint32_t bits = (w >> 9) | 0x3F800000u;
  float v;
#ifdef __CUDA_ARCH__
  v = __uint_as_float(bits);
  return __fsub_rn(v, 1.0f);
#else
  __builtin_memcpy(&v, &bits, 4);
  return v - 1.0f;
#endif
}

// the integer-weight draw: the same 23-bit value scaled to [0, total) exactly
// (total < 2^52), so the kept token whose cumulative range holds it is the one
// Uniform(0, total) picks in exact arithmetic
WCB_SI_HD uint64_t draw_target(uint32_t w, uint64_t total) {
  const unsigned __int128 p = static_cast<unsigned __int128>(w >> 9) * total;
  return uint64_t(p >> 23);
}

}  // namespace wcb
