// Host LogitsProcessor: crates/wasm-chord-runtime/src/sampling.rs:29-264.
// with_params chooses ArgMax when temperature < 1e-7, else top-k-then-top-p,
// top-k, top-p or all (:57-78); sample() applies the repetition penalty once per
// previously sampled occurrence (:86-103), then argmax (the LAST maximum wins,
// :118-125; a NaN logit is an error where the reference panics) or temperature
// softmax + top-k / top-p + a weighted draw (:106-229). The weighted draw takes one
// u32 of the reference's random stream, rand 0.9 StdRng::seed_from_u64(seed)
// (ChaCha12; restated in sample_int.h), per sampled token.
// Top-k configurations take a fixed evaluation order (sample_fixed) that the
// device sampler repeats operation for operation: the top-k candidates by
// (logit desc, index asc) (the reference's select_nth_unstable leaves ties at
// the boundary unspecified), softmax over them with wcb_exp_nonpos
// (mathematically the reference's softmax-then-renormalise), top-p and the draw.
// Every other sampled configuration (top_k = 0, or top_k > 1024) takes
// sample_int: integer weights (sample_int.h), exact sums, the same draw as the
// device's sample_full_kernel.
#pragma once
#include <algorithm>
#include <cstdint>
#include <vector>

#include "sample_int.h"

namespace wcb {

class Sampler {
 public:
  enum Kind { ARGMAX, ALL, TOPK, TOPP, TOPK_TOPP };
  Sampler(uint64_t seed, double temperature, double top_p, uint32_t top_k, float repetition_penalty);
  uint32_t sample(float* logits, size_t n);  // throws WcbError on NaN / invalid weights
  void penalize(float* logits, size_t n) const;
  static uint32_t argmax(const float* logits, size_t n);
  Kind kind() const { return kind_; }
  // top-k configurations (1 <= min(top_k, n) <= 1024) take the fixed-order path that
  // the device sampler (sample_dev.cu) reproduces exactly
  bool fixed_path(size_t n) const {
    return (kind_ == TOPK || kind_ == TOPK_TOPP) && top_k_ >= 1 && std::min(top_k_, n) <= 1024;
  }
  float temperature() const { return float(temperature_); }
  float top_p() const { return float(top_p_); }
  uint32_t top_k() const { return uint32_t(top_k_); }
  const StdRng& seed_state() const { return rng_; }
  bool greedy() const { return kind_ == ARGMAX; }
  float repetition_penalty() const { return rep_; }
  std::vector<uint32_t>& history() { return prev_; }
  // the probabilities the last sample_int / sample_fixed drew from (one per token)
  const std::vector<float>& last_probs() const { return last_probs_; }

 private:
  float uniform();
  uint32_t sample_fixed(const float* logits, size_t n);
  uint32_t sample_int(const float* logits, size_t n);

  StdRng rng_;
  Kind kind_;
  double temperature_, top_p_;
  size_t top_k_;
  float rep_;
  std::vector<uint32_t> prev_;
  std::vector<float> last_probs_;
};

}  // namespace wcb
