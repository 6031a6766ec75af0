#include "sampler.h"

#include <algorithm>
#include <cmath>
#include <numeric>

#include "gguf.h"
#include "wcb_exp.h"

namespace wcb {

Sampler::Sampler(uint64_t seed, double temperature, double top_p, uint32_t top_k, float rep)
    : state_(seed), temperature_(temperature), top_p_(top_p), top_k_(top_k), rep_(rep) {
  if (temperature < 1e-7) kind_ = ARGMAX;
  else if (top_k > 0 && top_p > 0.0 && top_p < 1.0) kind_ = TOPK_TOPP;
  else if (top_k > 0) kind_ = TOPK;
  else if (top_p > 0.0 && top_p < 1.0) kind_ = TOPP;
  else kind_ = ALL;
}

float Sampler::uniform() {
  uint64_t z = (state_ += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return float(z >> 40) * (1.0f / 16777216.0f);
}

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

void Sampler::renormalize(std::vector<float>& p) {
  float s = 0.0f;
  for (float v : p) s += v;
  if (s > 0.0f)
    for (float& v : p) v /= s;
}

uint32_t Sampler::multinomial(const std::vector<float>& p) {
  std::vector<float> cum(p.size());
  float tot = 0.0f;
  for (size_t i = 0; i < p.size(); ++i) {
    if (!(p[i] >= 0.0f)) throw WcbError(E_GENERIC, "Failed to create weighted index: invalid weight");
    tot += p[i];
    cum[i] = tot;
  }
  if (!(tot > 0.0f)) throw WcbError(E_GENERIC, "Failed to create weighted index: all weights zero");
  const float u = uniform() * tot;
  const size_t i = size_t(std::upper_bound(cum.begin(), cum.end(), u) - cum.begin());
  return uint32_t(std::min(i, p.size() - 1));
}

uint32_t Sampler::top_p(std::vector<float>& p, float tp) {
  std::vector<size_t> idx(p.size());
  std::iota(idx.begin(), idx.end(), size_t(0));
  std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return p[a] > p[b]; });
  float cum = 0.0f;
  for (size_t i : idx) {
    if (cum >= tp) p[i] = 0.0f;
    else cum += p[i];
  }
  renormalize(p);
  return multinomial(p);
}

void Sampler::keep_top_k(std::vector<float>& p, size_t k) {
  std::vector<size_t> idx(p.size());
  std::iota(idx.begin(), idx.end(), size_t(0));
  std::nth_element(idx.begin(), idx.begin() + long(k), idx.end(), [&](size_t a, size_t b) { return p[a] > p[b]; });
  for (size_t i = k; i < idx.size(); ++i) p[idx[i]] = 0.0f;
  renormalize(p);
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
  const float u = uniform() * tot;
  float c = 0.0f;
  for (size_t j = 0; j < K; ++j) {
    c += q[j];
    if (c > u) return cand[j];
  }
  return cand[K - 1];
}

uint32_t Sampler::sample(float* l, size_t n) {
  penalize(l, n);
  uint32_t tok;
  if (kind_ == ARGMAX) {
    tok = argmax(l, n);
  } else if (fixed_path(n)) {
    tok = sample_fixed(l, n);
  } else {
    // compute_probabilities (sampling.rs:106-115)
    std::vector<float> p(n);
    const float tf = float(temperature_);
    float mx = -INFINITY;
    for (size_t i = 0; i < n; ++i) {
      p[i] = l[i] / tf;
      mx = std::fmax(mx, p[i]);
    }
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += std::exp(p[i] - mx);
    for (size_t i = 0; i < n; ++i) p[i] = std::exp(p[i] - mx) / sum;
    const float tp = float(top_p_);
    const bool tp_active = !(top_p_ <= 0.0 || top_p_ >= 1.0);
    switch (kind_) {
      case ALL: tok = multinomial(p); break;
      case TOPP: tok = tp_active ? top_p(p, tp) : multinomial(p); break;
      case TOPK:
        if (top_k_ < n) keep_top_k(p, top_k_);
        tok = multinomial(p);
        break;
      default:  // TOPK_TOPP (sampling.rs:195-229)
        if (top_k_ >= n) {
          tok = top_p(p, tp);
        } else {
          keep_top_k(p, top_k_);
          tok = tp_active ? top_p(p, tp) : multinomial(p);
        }
    }
  }
  prev_.push_back(tok);
  return tok;
}

}  // namespace wcb
