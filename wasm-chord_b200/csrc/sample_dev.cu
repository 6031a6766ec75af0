// Temperature / top-k / top-p sampling on the device (LogitsProcessor::sample,
// crates/wasm-chord-runtime/src/sampling.rs:106-229), so that sampled generation
// runs the same device-driven decode loop as greedy generation.
//
// One CTA of 1024 threads over the logits of one sequence: the repetition
// penalty (:86-103) into a scratch copy, a NaN check, then the top-k candidates
// by (logit desc, index asc) with a radix select on the order-preserving bits
// (4 passes of 8 bits over keys held in registers, warp-aggregated histogram
// counts; the ties at the threshold go to the lowest indices, through a block
// scan in index order), and the candidates ordered by index (rank counting).
// From there the arithmetic is the fixed sequence the host sampler uses
// (sampler.cpp, Sampler::sample_fixed): x = l / T, e = exp(x - max) with
// wcb_exp_nonpos, probabilities over the candidates in index order, top-p
// over (probability desc, index asc), renormalisation, and the weighted draw
// with one u32 of the sequence's StdRng stream (sample_int.h), so a seed gives
// the same tokens on host and device.
#include <cstdint>

#include "device_common.cuh"
#include "kernels.h"
#include "sample_int.h"
#include "wcb_exp.h"

namespace wcb {
namespace {

constexpr int SD_THREADS = 1024;

// inclusive warp scan / block-wide exclusive scan and total of a u64 per thread
__device__ __forceinline__ unsigned long long warp_incl_u64(unsigned long long v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}
__device__ unsigned long long block_excl_u64(unsigned long long v, unsigned long long* total, unsigned long long* ws) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned long long inc = warp_incl_u64(v);
  __syncthreads();  // ws may still be read by a previous call
  if (lane == 31) ws[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const unsigned long long w = warp_incl_u64(ws[lane]);
    ws[lane] = w;  // inclusive totals of the warps
  }
  __syncthreads();
  *total = ws[SD_THREADS / 32 - 1];
  return (warp ? ws[warp - 1] : 0ull) + inc - v;
}

constexpr int SD_REG = 32;  // logits per thread held on chip (vocabularies up to 32768)
// staged penalised logits: value i at i + i / 32, so thread t's contiguous run
// t * SD_REG + j (j < 32) sits at t * 33 + j, one bank per lane
constexpr int SD_STAGE_BYTES = (SD_THREADS * SD_REG + SD_THREADS) * 4;
__device__ __forceinline__ int stage_at(int i) { return i + (i >> 5); }

// One count of a radix pass into this warp's own histogram row: one shared atomic
// per wanted element (the lanes that hit one bin are combined by the hardware; no
// other warp adds to the row, so the largest logits, which crowd into a few bins,
// do not serialise the block).
__device__ __forceinline__ void hist_add_warp(unsigned int* hw, bool want, unsigned int bin) {
  if (want) atomicAdd(&hw[bin], 1u);
}

// The penalised logits (repetition penalty once per occurrence, sampling.rs:86-103)
// into the stage with coalesced loads; true when one is NaN.
__device__ __forceinline__ bool stage_penalised(const float* logits, const uint32_t* pen_cnt, float rep, int n,
                                                float* stage) {
  bool nan = false;
  for (int i = threadIdx.x; i < n; i += SD_THREADS) {
    float v = logits[i];
    if (rep != 1.0f) {
      const uint32_t c = pen_cnt[i];
      for (uint32_t r = 0; r < c; ++r) v = v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
    }
    nan |= v != v;
    stage[stage_at(i)] = v;
  }
  return nan;
}

// Radix step (warp 0): the highest bin at which the count of keys in it and above
// reaches rem, 8 bins a lane; the bin joins the prefix, rem drops by the count above.
__device__ __forceinline__ void pick_bin(const unsigned int* h, unsigned int prefix, int shift, unsigned int rem,
                                         unsigned int* s_prefix, unsigned int* s_rem) {
  const int lane = threadIdx.x & 31;
  unsigned int c[8], tot = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // bins from the top: 255 - 8 lane - k
    c[k] = h[255 - (8 * lane + k)];
    tot += c[k];
  }
  unsigned int inc = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned int t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  unsigned int cum = inc - tot, before = 0;
  int hit = -1;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (hit < 0 && cum + c[k] >= rem) {
      hit = k;
      before = cum;
    }
    cum += c[k];
  }
  const unsigned int hm = __ballot_sync(0xffffffffu, hit >= 0);
  if (hm != 0u && lane == __ffs(hm) - 1) {
    *s_prefix = prefix | (unsigned(255 - (8 * lane + hit)) << shift);
    *s_rem = rem - before;
  }
}

// REG: the penalised logits are staged in shared memory (coalesced loads) and every
// thread keeps the order keys of its contiguous run in registers; otherwise plog.
template <bool REG>
__global__ void __launch_bounds__(SD_THREADS) sample_kernel(const float* logits, float* plog, int n, StepState* st,
                                                            uint32_t* hist, uint32_t* pen_cnt, float rep, float temp,
                                                            int top_k, float top_p, StdRng* rng,
                                                            int hstride) {
  __shared__ unsigned int hcount[256];
  __shared__ unsigned int s_prefix, s_rem, s_nan, s_ncand, s_tok;
  __shared__ int sorted[SD_THREADS];
  __shared__ int ord[SD_THREADS];
  __shared__ float q[SD_THREADS];
  __shared__ int cidx[SD_THREADS];
  __shared__ unsigned long long ws[SD_THREADS / 32];
  __shared__ float s_sum, s_max;
  // dynamic: REG: the penalised logits (stage_at); then [warps][256] per-warp counts of a radix pass
  extern __shared__ __align__(16) uint8_t dyn[];
  float* stage = reinterpret_cast<float*>(dyn);
  unsigned int* hwarp = reinterpret_cast<unsigned int*>(dyn + (REG ? SD_STAGE_BYTES : 0));
  pdl_trigger();
  pdl_wait();
  {  // CTA b samples sequence b of a batch (its logits, state, history, counts and stream)
    const size_t b = blockIdx.x;
    logits += b * size_t(n);
    plog += b * size_t(n);
    st += b;
    hist += b * size_t(hstride);
    pen_cnt += b * size_t(n);
    rng += b;
  }
  if (st->done) return;
  const int tid = threadIdx.x;
  const int per = (n + SD_THREADS - 1) / SD_THREADS;  // REG: per <= SD_REG
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  const int cnt = i1 - i0;
  uint32_t kr[REG ? SD_REG : 1] = {};
  auto logit_at = [&](int i) -> float {
    if constexpr (REG) return stage[stage_at(i)];
    else return plog[i];
  };
  // the same trip count on every thread (the histogram's warp-wide match needs it)
  auto each = [&](auto&& f) {
    if constexpr (REG) {
#pragma unroll
      for (int j = 0; j < SD_REG; ++j) f(j);
    } else {
      for (int j = 0; j < per; ++j) f(j);
    }
  };
  auto key_at = [&](int j) -> uint32_t {
    if constexpr (REG) return kr[j];
    else return j < cnt ? order_key(plog[i0 + j]) : 0u;
  };
  if (tid == 0) {
    s_nan = 0;
    s_ncand = 0;
  }
  __syncthreads();
  // repetition penalty once per occurrence (sampling.rs:86-103), into the stage (REG)
  // or the scratch copy
  bool nan = false;
  if constexpr (REG) {
    nan = stage_penalised(logits, pen_cnt, rep, n, stage);
    __syncthreads();
    each([&](int j) { kr[j] = j < cnt ? order_key(stage[stage_at(i0 + j)]) : 0u; });
  } else {
    each([&](int j) {
      if (j < cnt) {
        const int i = i0 + j;
        float v = logits[i];
        if (rep != 1.0f) {
          const uint32_t c = pen_cnt[i];
          for (uint32_t r = 0; r < c; ++r) v = v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
        }
        nan |= v != v;
        plog[i] = v;
      }
    });
  }
  if (nan) atomicOr(&s_nan, 1u);
  __syncthreads();
  if (s_nan) {  // partial_cmp().unwrap() panics on NaN in the reference
    if (tid == 0) {
      st->err = 1;
      st->done = 1;
    }
    return;
  }
  const int K = min(top_k, n);
  // radix select of the K-th largest order key (8 bits at a time)
  unsigned int prefix = 0, pmask = 0, rem = unsigned(K);
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < (SD_THREADS / 32) * 256; b += SD_THREADS) hwarp[b] = 0;
    __syncthreads();
    each([&](int j) {
      const uint32_t key = key_at(j);
      hist_add_warp(hwarp + (tid >> 5) * 256, j < cnt && (key & pmask) == prefix, (key >> shift) & 255u);
    });
    __syncthreads();
    if (tid < 256) {  // the warps' counts of each bin
      unsigned int c = 0;
#pragma unroll 8
      for (int w = 0; w < SD_THREADS / 32; ++w) c += hwarp[w * 256 + tid];
      hcount[tid] = c;
    }
    __syncthreads();
    if (tid < 32) pick_bin(hcount, prefix, shift, rem, &s_prefix, &s_rem);
    __syncthreads();
    prefix = s_prefix;
    rem = s_rem;
    pmask |= 255u << shift;
  }
  // candidates: every key above the threshold, and the `rem` lowest-indexed keys equal to it
  unsigned int n_eq = 0;
  each([&](int j) { n_eq += (j < cnt && key_at(j) == prefix) ? 1u : 0u; });
  unsigned long long eq_total;
  unsigned int eq_rank = unsigned(block_excl_u64(n_eq, &eq_total, ws));  // equal keys in lower threads
  each([&](int j) {
    if (j < cnt) {
      const uint32_t key = key_at(j);
      bool take = key > prefix;
      if (key == prefix) take = eq_rank++ < rem;
      if (take) cidx[atomicAdd(&s_ncand, 1u)] = i0 + j;
    }
  });
  __syncthreads();
  const int nc = int(s_ncand);  // == K
  // candidates in index order: each one's rank among the (distinct) candidate indices
  if (tid < nc) {
    const int my = cidx[tid];
    int r = 0;
    for (int j = 0; j < nc; ++j) r += cidx[j] < my;
    sorted[r] = my;
  }
  __syncthreads();
  const int cand = tid < nc ? sorted[tid] : -1;
  // x = l / T, max, e = exp(x - max)
  float x = -INFINITY;
  if (cand >= 0) x = __fdiv_rn(logit_at(cand), temp);
  // the maximum is exact in any order
  float m = x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) q[tid >> 5] = m;
  __syncthreads();
  if (tid < 32) {
    float mm = q[tid];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
    if (tid == 0) s_max = mm;
  }
  __syncthreads();
  const float e = cand >= 0 ? wcb_exp_nonpos(__fadd_rn(x, -s_max)) : 0.0f;
  q[tid] = e;
  __syncthreads();
  if (tid == 0) {  // the sum in index order, as the host adds it
    float s = 0.0f;
    for (int j = 0; j < nc; ++j) s = __fadd_rn(s, q[j]);
    s_sum = s;
  }
  __syncthreads();
  float p = cand >= 0 ? __fdiv_rn(e, s_sum) : 0.0f;
  const bool tp_on = !(top_p <= 0.0f || top_p >= 1.0f);
  if (tp_on) {
    q[tid] = p;
    __syncthreads();
    // order by (probability desc, index asc): each candidate's rank
    if (tid < nc) {
      int r = 0;
      for (int j = 0; j < nc; ++j) {
        const float pj = q[j];
        r += (pj > p || (pj == p && j < tid)) ? 1 : 0;
      }
      ord[r] = tid;
    }
    __syncthreads();
    if (tid == 0) {  // top_p (sampling.rs:152-193): keep while the sum before the token is < top_p
      float cum = 0.0f;
      for (int r = 0; r < nc; ++r) {
        const int slot = ord[r];
        if (cum >= top_p) q[slot] = 0.0f;
        else cum = __fadd_rn(cum, q[slot]);
      }
      float s = 0.0f;  // renormalise: the sum in index order
      for (int j = 0; j < nc; ++j) s = __fadd_rn(s, q[j]);
      s_sum = s;
    }
    __syncthreads();
    p = cand >= 0 ? (s_sum > 0.0f ? __fdiv_rn(q[tid], s_sum) : q[tid]) : 0.0f;
    __syncthreads();
  }
  q[tid] = p;
  __syncthreads();
  if (tid == 0) {  // weighted draw: cumulative sums in index order, first one above u * total
    float tot = 0.0f;
    for (int j = 0; j < nc; ++j) tot = __fadd_rn(tot, q[j]);
    int pick = nc - 1;
    if (!(tot > 0.0f)) {
      st->err = 1;  // no positive weight (WeightedIndex fails in the reference)
      st->done = 1;
      s_tok = 0xFFFFFFFFu;
    } else {
      const float u = __fmul_rn(unit_f32(std_rng_next_u32(rng)), tot);
      float c = 0.0f;
      for (int j = 0; j < nc; ++j) {
        c = __fadd_rn(c, q[j]);
        if (c > u) {
          pick = j;
          break;
        }
      }
      s_tok = unsigned(pick);
    }
  }
  __syncthreads();
  if (s_tok != 0xFFFFFFFFu && tid == int(s_tok)) {
    st->best = (unsigned long long)(unsigned)cand;  // the key's low word carries the token
    st->nan = 0;
    finish_sample_state(st, hist, pen_cnt);
  }
}


// ---- any number of candidates (top_k = 0 or top_k > 1024): integer weights ----

// LogitsProcessor::sample for top_k = 0 or top_k > 1024 (sampling.rs:106-229),
// with the weights of sample_int.h: the repetition penalty into plog, the top-k
// candidates (k = 0: all) by a radix select of the order-preserving logit bits
// (ties at the threshold to the lowest indices), x = l / T, the maximum, the
// integer weights E (stored over plog), top-p by a binary search over the weight
// value with exact sums, the draw, generate()'s bookkeeping.
// probs (may be null) receives each token's final probability.
// SM: the penalised logits, then their x = l / T, then their integer weights, in
// dynamic shared memory (stage_at: each thread's contiguous run conflict-free, the
// logits loaded coalesced); otherwise in plog.
template <bool SM>
__global__ void __launch_bounds__(SD_THREADS) sample_full_kernel(const float* logits, float* plog, int n, StepState* st,
                                                                 uint32_t* hist, uint32_t* pen_cnt, float rep,
                                                                 float temp, int top_k, float top_p,
                                                                 StdRng* rng, float* probs, int hstride) {
  __shared__ unsigned int hcount[256];
  __shared__ unsigned long long ws[SD_THREADS / 32];
  __shared__ unsigned int s_prefix, s_rem, s_nan, s_keq, s_tok;
  __shared__ unsigned long long s_t;
  __shared__ float s_max;
  __shared__ float wmax[SD_THREADS / 32];
  pdl_trigger();
  pdl_wait();
  {  // CTA b samples sequence b of a batch (its logits, state, history, counts and stream)
    const size_t b = blockIdx.x;
    logits += b * size_t(n);
    plog += b * size_t(n);
    st += b;
    hist += b * size_t(hstride);
    pen_cnt += b * size_t(n);
    rng += b;
  }
  if (st->done) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + SD_THREADS - 1) / SD_THREADS;  // REG: per <= SD_REG
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  const int cnt = i1 - i0;
  // dynamic: SM: value i at stage_at(i); then [warps][256] per-warp counts of a radix pass
  extern __shared__ __align__(16) uint32_t sv[];
  unsigned int* hwarp = sv + (SM ? SD_STAGE_BYTES / 4 : 0);
  uint32_t* E = reinterpret_cast<uint32_t*>(plog);
  auto each = [&](auto&& f) {  // the same trip count on every thread
    if constexpr (SM) {
#pragma unroll 8
      for (int j = 0; j < SD_REG; ++j) f(j);
    } else {
      for (int j = 0; j < per; ++j) f(j);
    }
  };
  auto getf = [&](int j) -> float {
    if constexpr (SM) return __uint_as_float(sv[stage_at(i0 + j)]);
    else return plog[i0 + j];
  };
  auto setf = [&](int j, float v) {
    if constexpr (SM) sv[stage_at(i0 + j)] = __float_as_uint(v);
    else plog[i0 + j] = v;
  };
  auto getw = [&](int j) -> uint32_t {
    if constexpr (SM) return sv[stage_at(i0 + j)];
    else return E[i0 + j];
  };
  auto setw = [&](int j, uint32_t w) {
    if constexpr (SM) sv[stage_at(i0 + j)] = w;
    else E[i0 + j] = w;
  };
  if (tid == 0) s_nan = 0;
  __syncthreads();
  bool nan = false;
  if constexpr (SM) {
    nan = stage_penalised(logits, pen_cnt, rep, n, reinterpret_cast<float*>(sv));
  } else {
    each([&](int j) {  // repetition penalty once per occurrence (sampling.rs:86-103)
      if (j < cnt) {
        const int i = i0 + j;
        float v = logits[i];
        if (rep != 1.0f) {
          const uint32_t c = pen_cnt[i];
          for (uint32_t k = 0; k < c; ++k) v = v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
        }
        nan |= v != v;
        setf(j, v);
      }
    });
  }
  if (nan) atomicOr(&s_nan, 1u);
  __syncthreads();
  if (s_nan) {  // partial_cmp().unwrap() panics on NaN in the reference
    if (tid == 0) {
      st->err = 1;
      st->done = 1;
    }
    return;
  }
  // top-k candidates (0 < top_k < n): the threshold key and how many of its ties are taken
  const bool topk = top_k > 0 && top_k < n;
  unsigned int prefix = 0, rem = 0;
  if (topk) {
    unsigned int pmask = 0;
    rem = unsigned(top_k);
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < (SD_THREADS / 32) * 256; b += SD_THREADS) hwarp[b] = 0;
      __syncthreads();
      each([&](int j) {
        const uint32_t key = j < cnt ? order_key(getf(j)) : 0u;
        hist_add_warp(hwarp + (tid >> 5) * 256, j < cnt && (key & pmask) == prefix, (key >> shift) & 255u);
      });
      __syncthreads();
      if (tid < 256) {  // the warps' counts of each bin
        unsigned int c = 0;
#pragma unroll 8
        for (int w = 0; w < SD_THREADS / 32; ++w) c += hwarp[w * 256 + tid];
        hcount[tid] = c;
      }
      __syncthreads();
      if (tid < 32) pick_bin(hcount, prefix, shift, rem, &s_prefix, &s_rem);
      __syncthreads();
      prefix = s_prefix;
      rem = s_rem;
      pmask |= 255u << shift;
    }
  }
  // x = l / T over the candidates (-inf elsewhere), and the maximum
  {
    unsigned long long eq = 0;
    if (topk) each([&](int j) { eq += (j < cnt && order_key(getf(j)) == prefix) ? 1u : 0u; });
    unsigned long long eq_tot;
    unsigned int eq_rank = unsigned(block_excl_u64(eq, &eq_tot, ws));
    float mx = -INFINITY;
    each([&](int j) {
      if (j < cnt) {
        const float v = getf(j);
        bool take = true;
        if (topk) {
          const uint32_t key = order_key(v);
          take = key > prefix;
          if (key == prefix) take = eq_rank++ < rem;
        }
        const float x = take ? __fdiv_rn(v, temp) : -INFINITY;
        setf(j, x);
        mx = fmaxf(mx, x);
      }
    });
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) wmax[warp] = mx;
    __syncthreads();
    if (tid < 32) {
      float m = wmax[tid];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (tid == 0) s_max = m;
    }
    __syncthreads();
  }
  // integer weights and their total
  const float M = s_max;
  unsigned long long mine = 0;
  each([&](int j) {
    if (j < cnt) {
      const uint32_t w = int_weight(wcb_exp_nonpos(__fadd_rn(getf(j), -M)));
      setw(j, w);
      mine += w;
    }
  });
  unsigned long long S;
  block_excl_u64(mine, &S, ws);
  // top-p: the last kept weight v* (exact sums)
  const bool tp_on = !(top_p <= 0.0f || top_p >= 1.0f);  // TOPP / TOPK_TOPP (sampling.rs:57-78)
  unsigned int vstar = 0, keq = 0xFFFFFFFFu;
  if (tp_on) {
    // v* = the largest weight value v whose sum of weights >= v is not below top_p * S:
    // the weight at which the cumulative sum from the top first reaches the threshold
    // (what a search from the top finds). The sums of weights >= v fall as v
    // rises, so a binary search over v finds it; S itself is never below (top_p < 1).
    const TopP tpp = top_p_parts(top_p);
    auto sum_ge = [&](unsigned long long v) {
      unsigned long long part = 0, tot;
      each([&](int j) {
        if (j < cnt) {
          const uint32_t w = getw(j);
          part += w >= v ? w : 0u;
        }
      });
      block_excl_u64(part, &tot, ws);
      return tot;
    };
    unsigned long long lo = 0, hi = 0xFFFFFFFFull;
    while (lo < hi) {  // uniform over the block: every thread sees the same totals
      const unsigned long long mid = (lo + hi + 1) / 2;
      if (!below_top_p(sum_ge(mid), tpp, S)) lo = mid;
      else hi = mid - 1;
    }
    vstar = unsigned(lo);
    const unsigned long long C = sum_ge(lo + 1);  // the weights above v*
    unsigned long long ties = 0, tie_tot;
    each([&](int j) { ties += (j < cnt && getw(j) == vstar) ? 1u : 0u; });
    block_excl_u64(ties, &tie_tot, ws);
    if (tid == 0) {  // how many of v*'s ties (lowest indices first) are kept
      unsigned long long l2 = 0, h2 = tie_tot;  // largest r in [0, ties] with every r' < r kept
      while (l2 < h2) {
        const unsigned long long m2 = (l2 + h2 + 1) / 2;
        if (below_top_p(C + (m2 - 1) * (unsigned long long)vstar, tpp, S)) l2 = m2;
        else h2 = m2 - 1;
      }
      s_keq = unsigned(l2);
    }
    __syncthreads();
    keq = s_keq;
  }
  // kept weights and their running sum in index order
  unsigned long long eqn = 0;
  if (tp_on) each([&](int j) { eqn += (j < cnt && getw(j) == vstar) ? 1u : 0u; });
  unsigned long long eqt;
  unsigned long long er = block_excl_u64(eqn, &eqt, ws);
  unsigned long long kept = 0;
  {
    unsigned long long r = er;
    each([&](int j) {
      if (j < cnt) {
        const uint32_t w = getw(j);
        const bool k = !tp_on || w > vstar || (w == vstar && r++ < keq);
        kept += k ? w : 0u;
      }
    });
  }
  unsigned long long S_kept;
  const unsigned long long before = block_excl_u64(kept, &S_kept, ws);
  if (tid == 0) {
    s_tok = 0xFFFFFFFFu;
    if (S_kept == 0) {  // no positive weight (WeightedIndex fails in the reference)
      st->err = 1;
      st->done = 1;
    } else {
      s_t = draw_target(std_rng_next_u32(rng), S_kept);
    }
  }
  __syncthreads();
  if (S_kept == 0) return;
  const unsigned long long t = s_t;
  {
    unsigned long long r = er, cum = before;
    each([&](int j) {
      if (j < cnt) {
        const int i = i0 + j;
        const uint32_t w = getw(j);
        const bool k = !tp_on || w > vstar || (w == vstar && r++ < keq);
        if (probs) probs[i] = k ? float(double(w) / double(S_kept)) : 0.0f;
        if (k) {
          cum += w;
          if (cum > t && cum - w <= t) s_tok = unsigned(i);  // the token whose range holds t
        }
      }
    });
  }
  __syncthreads();
  if (tid == 0 && s_tok != 0xFFFFFFFFu) {
    st->best = (unsigned long long)s_tok;  // the key's low word carries the token
    st->nan = 0;
    finish_sample_state(st, hist, pen_cnt);
  }
}

}  // namespace

cudaError_t launch_sample(const float* logits, float* scratch, int n, StepState* st, uint32_t* hist,
                          uint32_t* pen_cnt, float rep, float temperature, int top_k, float top_p,
                          StdRng* rng, cudaStream_t s, int nseq, int hist_stride) {
  if (top_k < 1 || top_k > SD_THREADS || n < 1 || !(temperature > 0.0f) || nseq < 1) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(nseq));
  cfg.blockDim = dim3(SD_THREADS);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
  constexpr int HW_BYTES = (SD_THREADS / 32) * 256 * 4;  // per-warp radix counts
  if (n <= SD_THREADS * SD_REG) {  // the logits fit the shared-memory stage
    e = cudaFuncSetAttribute(sample_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SD_STAGE_BYTES + HW_BYTES);
    cfg.dynamicSmemBytes = size_t(SD_STAGE_BYTES + HW_BYTES);
    if (e == cudaSuccess)
      e = cudaLaunchKernelEx(&cfg, sample_kernel<true>, logits, scratch, n, st, hist, pen_cnt, rep, temperature,
                             top_k, top_p, rng, hist_stride);
  } else {  // static + per-warp counts exceed the default 48 KB
    e = cudaFuncSetAttribute(sample_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, HW_BYTES);
    cfg.dynamicSmemBytes = size_t(HW_BYTES);
    if (e == cudaSuccess)
      e = cudaLaunchKernelEx(&cfg, sample_kernel<false>, logits, scratch, n, st, hist, pen_cnt, rep, temperature,
                             top_k, top_p, rng, hist_stride);
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb

namespace wcb {

cudaError_t launch_sample_full(const float* logits, float* scratch, int n, StepState* st, uint32_t* hist,
                               uint32_t* pen_cnt, float rep, float temperature, int top_k, float top_p,
                               StdRng* rng, float* probs, cudaStream_t s, int nseq, int hist_stride) {
  // probs (a test hook) only for one sequence
  if (top_k < 0 || n < 1 || !(temperature > 0.0f) || nseq < 1 || (probs && nseq > 1)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(nseq));
  cfg.blockDim = dim3(SD_THREADS);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const bool sm = n <= SD_THREADS * SD_REG;  // every thread's logits fit shared memory
  constexpr int HW_BYTES = (SD_THREADS / 32) * 256 * 4;  // per-warp radix counts
  cudaError_t e = cudaSuccess;
  if (sm) {
    e = cudaFuncSetAttribute(sample_full_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SD_STAGE_BYTES + HW_BYTES);
    cfg.dynamicSmemBytes = size_t(SD_STAGE_BYTES + HW_BYTES);
    if (e == cudaSuccess)
      e = cudaLaunchKernelEx(&cfg, sample_full_kernel<true>, logits, scratch, n, st, hist, pen_cnt, rep, temperature,
                             top_k, top_p, rng, probs, hist_stride);
  } else {
    e = cudaFuncSetAttribute(sample_full_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, HW_BYTES);
    cfg.dynamicSmemBytes = size_t(HW_BYTES);
    if (e == cudaSuccess)
      e = cudaLaunchKernelEx(&cfg, sample_full_kernel<false>, logits, scratch, n, st, hist, pen_cnt, rep, temperature,
                             top_k, top_p, rng, probs, hist_stride);
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb
