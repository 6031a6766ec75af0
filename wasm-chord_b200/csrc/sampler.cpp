#include "sampler.h"

#include <algorithm>
#include <cmath>
#include <numeric>

#include "gguf.h"
#include "sample_int.h"
#include "wcb_exp.h"

namespace wcb {

Sampler::Sampler(uint64_t seed, double temperature, double top_p, uint32_t top_k, float rep)
    : rng_(std_rng_seed_from_u64(seed)), temperature_(temperature), top_p_(top_p), top_k_(top_k), rep_(rep) {
  if (temperature < 1e-7) kind_ = ARGMAX;
  else if (top_k > 0 && top_p > 0.0 && top_p < 1.0) kind_ = TOPK_TOPP;
  else if (top_k > 0) kind_ = TOPK;
  else if (top_p > 0.0 && top_p < 1.0) kind_ = TOPP;
  else kind_ = ALL;
}

float Sampler::uniform() { return unit_f32(std_rng_next_u32(&rng_)); }

void Sampler::penalize(float* l, size_t n) const {
  if (rep_ == 1.0f) return;
  for (uint32_t t : prev_) {
    if (size_t(t) >= n) continue;
    if (l[t] > 0.0f) l[t] /= rep_;
    else l[t] *= rep_;
  }
}

uint32_t Sampler::argmax(const float* l, size_t n) {
  if (n == 0) return 0;
  size_t best = 0;
  for (size_t i = 0; i < n; ++i) {
    if (std::isnan(l[i])) throw WcbError(E_GENERIC, "Runtime error: NaN logit at index " + std::to_string(i));
    if (i && !(l[best] > l[i])) best = i;
  }
  return uint32_t(best);
}

uint32_t Sampler::sample_fixed(const float* l, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (std::isnan(l[i])) throw WcbError(E_GENERIC, "Runtime error: NaN logit at index " + std::to_string(i));
  const size_t K = std::min(top_k_, n);
  std::vector<uint32_t> idx(n);
  std::iota(idx.begin(), idx.end(), 0u);
  std::partial_sort(idx.begin(), idx.begin() + long(K), idx.end(),
                    [&](uint32_t a, uint32_t b) { return l[a] > l[b] || (l[a] == l[b] && a < b); });
  std::vector<uint32_t> cand(idx.begin(), idx.begin() + long(K));
  std::sort(cand.begin(), cand.end());
  const float tf = float(temperature_);
  std::vector<float> x(K), q(K);
  float mx = -INFINITY;
  for (size_t j = 0; j < K; ++j) {
    x[j] = l[cand[j]] / tf;
    mx = std::fmax(mx, x[j]);
  }
  float s = 0.0f;
  for (size_t j = 0; j < K; ++j) {
    q[j] = wcb_exp_nonpos(x[j] + (-mx));
    s += q[j];
  }
  for (size_t j = 0; j < K; ++j) q[j] = q[j] / s;
  const float tp = float(top_p_);
  if (!(tp <= 0.0f || tp >= 1.0f)) {
    std::vector<uint32_t> ord(K);
    std::iota(ord.begin(), ord.end(), 0u);
    std::stable_sort(ord.begin(), ord.end(), [&](uint32_t a, uint32_t b) { return q[a] > q[b]; });
    float cum = 0.0f;
    for (uint32_t j : ord) {
      if (cum >= tp) q[j] = 0.0f;
      else cum += q[j];
    }
    float s2 = 0.0f;
    for (size_t j = 0; j < K; ++j) s2 += q[j];
    if (s2 > 0.0f)
      for (size_t j = 0; j < K; ++j) q[j] = q[j] / s2;
  }
  float tot = 0.0f;
  for (size_t j = 0; j < K; ++j) tot += q[j];
  if (!(tot > 0.0f)) throw WcbError(E_GENERIC, "Failed to create weighted index: all weights zero");
  last_probs_.assign(n, 0.0f);
  for (size_t j = 0; j < K; ++j) last_probs_[cand[j]] = q[j] / tot;
  const float u = uniform() * tot;
  float c = 0.0f;
  for (size_t j = 0; j < K; ++j) {
    c += q[j];
    if (c > u) return cand[j];
  }
  return cand[K - 1];
}

uint32_t Sampler::sample_int(const float* l, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (std::isnan(l[i])) throw WcbError(E_GENERIC, "Runtime error: NaN logit at index " + std::to_string(i));
  // candidates: the top-k by (logit desc, index asc) when 0 < top_k < n, else all
  std::vector<uint8_t> cand(n, 1);
  if (top_k_ > 0 && top_k_ < n) {
    std::fill(cand.begin(), cand.end(), 0);
    std::vector<uint32_t> idx(n);
    std::iota(idx.begin(), idx.end(), 0u);
    std::nth_element(idx.begin(), idx.begin() + long(top_k_), idx.end(),
                     [&](uint32_t a, uint32_t b) { return l[a] > l[b] || (l[a] == l[b] && a < b); });
    for (size_t j = 0; j < top_k_; ++j) cand[idx[j]] = 1;
  }
  const float tf = float(temperature_);
  std::vector<float> x(n);
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) {
    x[i] = cand[i] ? l[i] / tf : -INFINITY;
    mx = std::fmax(mx, x[i]);
  }
  std::vector<uint32_t> E(n);
  uint64_t S = 0;
  for (size_t i = 0; i < n; ++i) {
    E[i] = int_weight(wcb_exp_nonpos(x[i] + (-mx)));
    S += E[i];
  }
  std::vector<uint8_t> kept(n, 1);
  const float tp = float(top_p_);
  if (!(tp <= 0.0f || tp >= 1.0f)) {  // top-p in exact arithmetic, (E desc, index asc)
    const TopP t = top_p_parts(tp);
    std::vector<uint32_t> ord(n);
    std::iota(ord.begin(), ord.end(), 0u);
    std::stable_sort(ord.begin(), ord.end(), [&](uint32_t a, uint32_t b) { return E[a] > E[b]; });
    uint64_t cum = 0;
    for (uint32_t i : ord) {
      kept[i] = below_top_p(cum, t, S) ? 1 : 0;
      cum += E[i];
    }
  }
  uint64_t S_kept = 0;
  for (size_t i = 0; i < n; ++i) S_kept += kept[i] ? E[i] : 0u;
  if (S_kept == 0) throw WcbError(E_GENERIC, "Failed to create weighted index: all weights zero");
  last_probs_.assign(n, 0.0f);
  for (size_t i = 0; i < n; ++i) last_probs_[i] = kept[i] ? float(double(E[i]) / double(S_kept)) : 0.0f;
  const uint64_t target = draw_target(std_rng_next_u32(&rng_), S_kept);
  uint64_t cum = 0;
  for (size_t i = 0; i < n; ++i) {
    if (!kept[i]) continue;
    cum += E[i];
    if (cum > target) return uint32_t(i);
  }
  return uint32_t(n - 1);  // unreachable: target < S_kept
}

uint32_t Sampler::sample(float* l, size_t n) {
  penalize(l, n);
  uint32_t tok;
  if (kind_ == ARGMAX) tok = argmax(l, n);
  else if (fixed_path(n)) tok = sample_fixed(l, n);
  else tok = sample_int(l, n);
  prev_.push_back(tok);
  return tok;
}

}  // namespace wcb
