// Temperature / top-k / top-p sampling on the device (LogitsProcessor::sample,
// crates/wasm-chord-runtime/src/sampling.rs:106-229), so that sampled generation
// runs the same device-driven decode loop as greedy generation.
//
// One CTA of 1024 threads over the logits of one sequence: the repetition
// penalty (:86-103) into a scratch copy, a NaN check, then the top-k candidates
// by (logit desc, index asc) with a radix select on the order-preserving bits
// (4 passes of 8 bits; the ties at the threshold go to the lowest indices,
// through a block scan in index order), and the candidates sorted by index.
// From there the arithmetic is the fixed sequence the host sampler uses
// (sampler.cpp, Sampler::sample_fixed): x = l / T, e = exp(x - max) with
// wcb_exp_nonpos, probabilities over the candidates in index order, top-p
// over (probability desc, index asc), renormalisation, and the weighted draw
// with the splitmix64 stream, so a seed gives the same tokens on host and device.
#include <cstdint>

#include "device_common.cuh"
#include "kernels.h"
#include "sample_int.h"
#include "wcb_exp.h"

namespace wcb {
namespace {

constexpr int SD_THREADS = 1024;

__device__ __forceinline__ float sd_uniform(unsigned long long* state) {
  unsigned long long z = (*state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return __fmul_rn(float(z >> 40), 1.0f / 16777216.0f);
}

// block-wide bitonic sort of SD_THREADS 64-bit keys, descending
__device__ void bitonic_desc(unsigned long long* k) {
  const int tid = threadIdx.x;
  for (int size = 2; size <= SD_THREADS; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      const int j = tid ^ stride;
      if (j > tid) {
        const bool desc = (tid & size) == 0;
        const unsigned long long a = k[tid], b = k[j];
        if (desc ? (a < b) : (a > b)) {
          k[tid] = b;
          k[j] = a;
        }
      }
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(SD_THREADS) sample_kernel(const float* logits, float* plog, int n, StepState* st,
                                                            uint32_t* hist, uint32_t* pen_cnt, float rep, float temp,
                                                            int top_k, float top_p, unsigned long long* rng) {
  __shared__ unsigned int hcount[256];
  __shared__ unsigned int s_prefix, s_rem, s_nan, s_ncand, s_tok;
  __shared__ unsigned int scan[SD_THREADS];
  __shared__ unsigned long long keys[SD_THREADS];
  __shared__ float q[SD_THREADS];
  __shared__ int cidx[SD_THREADS];
  __shared__ float s_sum, s_max;
  pdl_trigger();
  pdl_wait();
  if (st->done) return;
  const int tid = threadIdx.x;
  const int per = (n + SD_THREADS - 1) / SD_THREADS;
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  if (tid == 0) {
    s_nan = 0;
    s_ncand = 0;
  }
  __syncthreads();
  // repetition penalty once per occurrence (sampling.rs:86-103), into the scratch copy
  bool nan = false;
  for (int i = i0; i < i1; ++i) {
    float v = logits[i];
    if (rep != 1.0f) {
      const uint32_t c = pen_cnt[i];
      for (uint32_t k = 0; k < c; ++k) v = v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
    }
    nan |= v != v;
    plog[i] = v;
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
    for (int b = tid; b < 256; b += SD_THREADS) hcount[b] = 0;
    __syncthreads();
    for (int i = i0; i < i1; ++i) {
      const uint32_t key = order_key(plog[i]);
      if ((key & pmask) == prefix) atomicAdd(&hcount[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      unsigned int cum = 0;
      for (int b = 255; b >= 0; --b) {
        if (cum + hcount[b] >= rem) {
          s_prefix = prefix | (unsigned(b) << shift);
          s_rem = rem - cum;
          break;
        }
        cum += hcount[b];
      }
    }
    __syncthreads();
    prefix = s_prefix;
    rem = s_rem;
    pmask |= 255u << shift;
  }
  // candidates: every key above the threshold, and the `rem` lowest-indexed keys equal to it
  unsigned int n_eq = 0;
  for (int i = i0; i < i1; ++i) n_eq += order_key(plog[i]) == prefix;
  scan[tid] = n_eq;
  __syncthreads();
  for (int off = 1; off < SD_THREADS; off <<= 1) {  // inclusive scan in thread (= index) order
    const unsigned int v = tid >= off ? scan[tid - off] : 0u;
    __syncthreads();
    scan[tid] += v;
    __syncthreads();
  }
  unsigned int eq_rank = scan[tid] - n_eq;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = order_key(plog[i]);
    bool take = key > prefix;
    if (key == prefix) take = eq_rank++ < rem;
    if (take) cidx[atomicAdd(&s_ncand, 1u)] = i;
  }
  __syncthreads();
  const int nc = int(s_ncand);  // == K
  // candidates in index order: sort (index desc with INT_MAX padding first), read back reversed
  keys[tid] = tid < nc ? (unsigned long long)(unsigned)cidx[tid] : 0xFFFFFFFFFFFFFFFFull;
  bitonic_desc(keys);
  // keys sorted descending: the nc valid indices occupy slots [SD_THREADS - nc, SD_THREADS) in
  // descending order, so candidate tid (ascending) is at slot SD_THREADS - 1 - tid
  const int cand = tid < nc ? int(keys[SD_THREADS - 1 - tid]) : -1;
  __syncthreads();
  // x = l / T, max, e = exp(x - max)
  float x = -INFINITY;
  if (cand >= 0) x = __fdiv_rn(plog[cand], temp);
  if (tid == 0) s_max = -INFINITY;
  __syncthreads();
  // the maximum is exact in any order
  float m = x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) q[tid >> 5] = m;
  __syncthreads();
  if (tid == 0) {
    float mm = -INFINITY;
    for (int w = 0; w < SD_THREADS / 32; ++w) mm = fmaxf(mm, q[w]);
    s_max = mm;
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
    // order by (probability desc, index asc): key = (p bits, ~slot); p >= 0 so its bits order it
    keys[tid] = cand >= 0 ? (((unsigned long long)__float_as_uint(p) << 32) | (0xFFFFFFFFu - unsigned(tid))) : 0ull;
    q[tid] = p;
    bitonic_desc(keys);
    if (tid == 0) {  // top_p (sampling.rs:152-193): keep while the sum before the token is < top_p
      float cum = 0.0f;
      for (int r = 0; r < nc; ++r) {
        const int slot = int(0xFFFFFFFFu - unsigned(keys[r] & 0xFFFFFFFFull));
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
      const float u = __fmul_rn(sd_uniform(rng), tot);
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

// LogitsProcessor::sample for top_k = 0 or top_k > 1024 (sampling.rs:106-229),
// with the weights of sample_int.h: the repetition penalty into plog, the top-k
// candidates (k = 0: all) by a radix select of the order-preserving logit bits
// (ties at the threshold to the lowest indices), x = l / T, the maximum, the
// integer weights E (stored over plog), top-p by a radix search over E with
// per-bucket counts and exact sums, the draw, generate()'s bookkeeping.
// probs (may be null) receives each token's final probability.
__global__ void __launch_bounds__(SD_THREADS) sample_full_kernel(const float* logits, float* plog, int n, StepState* st,
                                                                 uint32_t* hist, uint32_t* pen_cnt, float rep,
                                                                 float temp, int top_k, float top_p,
                                                                 unsigned long long* rng, float* probs) {
  __shared__ unsigned int hcount[256];
  __shared__ unsigned long long hsum[256];
  __shared__ unsigned long long ws[SD_THREADS / 32];
  __shared__ unsigned int s_prefix, s_rem, s_nan, s_keq, s_tok;
  __shared__ unsigned long long s_c, s_t;
  __shared__ float s_max;
  __shared__ float wmax[SD_THREADS / 32];
  pdl_trigger();
  pdl_wait();
  if (st->done) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + SD_THREADS - 1) / SD_THREADS;
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  if (tid == 0) s_nan = 0;
  __syncthreads();
  bool nan = false;
  for (int i = i0; i < i1; ++i) {  // repetition penalty once per occurrence (sampling.rs:86-103)
    float v = logits[i];
    if (rep != 1.0f) {
      const uint32_t c = pen_cnt[i];
      for (uint32_t k = 0; k < c; ++k) v = v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
    }
    nan |= v != v;
    plog[i] = v;
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
      for (int b = tid; b < 256; b += SD_THREADS) hcount[b] = 0;
      __syncthreads();
      for (int i = i0; i < i1; ++i) {
        const uint32_t key = order_key(plog[i]);
        if ((key & pmask) == prefix) atomicAdd(&hcount[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        unsigned int cum = 0;
        for (int b = 255; b >= 0; --b) {
          if (cum + hcount[b] >= rem) {
            s_prefix = prefix | (unsigned(b) << shift);
            s_rem = rem - cum;
            break;
          }
          cum += hcount[b];
        }
      }
      __syncthreads();
      prefix = s_prefix;
      rem = s_rem;
      pmask |= 255u << shift;
    }
  }
  // x = l / T over the candidates (-inf elsewhere) into plog, and the maximum
  {
    unsigned long long eq = 0;
    if (topk)
      for (int i = i0; i < i1; ++i) eq += order_key(plog[i]) == prefix;
    unsigned long long eq_tot;
    unsigned int eq_rank = unsigned(block_excl_u64(eq, &eq_tot, ws));
    float mx = -INFINITY;
    for (int i = i0; i < i1; ++i) {
      bool take = true;
      if (topk) {
        const uint32_t key = order_key(plog[i]);
        take = key > prefix;
        if (key == prefix) take = eq_rank++ < rem;
      }
      const float x = take ? __fdiv_rn(plog[i], temp) : -INFINITY;
      plog[i] = x;
      mx = fmaxf(mx, x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) wmax[warp] = mx;
    __syncthreads();
    if (tid == 0) {
      float m = -INFINITY;
      for (int w = 0; w < SD_THREADS / 32; ++w) m = fmaxf(m, wmax[w]);
      s_max = m;
    }
    __syncthreads();
  }
  // integer weights (stored over plog) and their total
  uint32_t* E = reinterpret_cast<uint32_t*>(plog);
  const float M = s_max;
  unsigned long long mine = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t w = int_weight(wcb_exp_nonpos(__fadd_rn(plog[i], -M)));
    E[i] = w;
    mine += w;
  }
  unsigned long long S;
  block_excl_u64(mine, &S, ws);
  // top-p: the last kept weight v* (radix search over E from the top, exact sums)
  const bool tp_on = !(top_p <= 0.0f || top_p >= 1.0f);  // TOPP / TOPK_TOPP (sampling.rs:57-78)
  unsigned int vstar = 0, keq = 0xFFFFFFFFu;
  if (tp_on) {
    const TopP tpp = top_p_parts(top_p);
    unsigned int pfx = 0, pmask = 0;
    unsigned long long C = 0;  // sum of the weights above the current range
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += SD_THREADS) {
        hcount[b] = 0;
        hsum[b] = 0;
      }
      __syncthreads();
      for (int i = i0; i < i1; ++i) {
        const uint32_t w = E[i];
        if ((w & pmask) == pfx) {
          atomicAdd(&hcount[(w >> shift) & 255u], 1u);
          atomicAdd(&hsum[(w >> shift) & 255u], (unsigned long long)w);
        }
      }
      __syncthreads();
      if (tid == 0) {
        int b = 255;
        for (; b > 0; --b) {  // whole buckets whose last weight still starts below top_p * S
          if (!hcount[b]) continue;
          if (!below_top_p(C + hsum[b], tpp, S)) break;
          C += hsum[b];
        }
        s_prefix = pfx | (unsigned(b) << shift);
        s_c = C;
        if (shift == 0) {  // v* reached: how many of its ties (lowest indices first) are kept
          const unsigned int cnt = hcount[b];
          const unsigned long long v = (unsigned long long)((pfx | unsigned(b)) & 0xFFFFFFFFu);
          unsigned int lo = 0, hi = cnt;  // largest r in [0, cnt] with every r' < r kept
          while (lo < hi) {
            const unsigned int mid = (lo + hi + 1) / 2;
            if (below_top_p(C + (unsigned long long)(mid - 1) * v, tpp, S)) lo = mid;
            else hi = mid - 1;
          }
          s_keq = lo;
        }
      }
      __syncthreads();
      pfx = s_prefix;
      C = s_c;
      pmask |= 255u << shift;
    }
    vstar = pfx;
    keq = s_keq;
  }
  // kept weights and their running sum in index order
  unsigned long long eqn = 0;
  if (tp_on)
    for (int i = i0; i < i1; ++i) eqn += E[i] == vstar;
  unsigned long long eqt;
  unsigned long long er = block_excl_u64(eqn, &eqt, ws);
  unsigned long long kept = 0;
  {
    unsigned long long r = er;
    for (int i = i0; i < i1; ++i) {
      const uint32_t w = E[i];
      const bool k = !tp_on || w > vstar || (w == vstar && r++ < keq);
      kept += k ? w : 0u;
    }
  }
  unsigned long long S_kept;
  const unsigned long long before = block_excl_u64(kept, &S_kept, ws);
  if (tid == 0) {
    s_tok = 0xFFFFFFFFu;
    if (S_kept == 0) {  // no positive weight (WeightedIndex fails in the reference)
      st->err = 1;
      st->done = 1;
    } else {
      s_t = draw_target(splitmix64_next(reinterpret_cast<uint64_t*>(rng)), S_kept);
    }
  }
  __syncthreads();
  if (S_kept == 0) return;
  const unsigned long long t = s_t;
  {
    unsigned long long r = er, cum = before;
    for (int i = i0; i < i1; ++i) {
      const uint32_t w = E[i];
      const bool k = !tp_on || w > vstar || (w == vstar && r++ < keq);
      if (probs) probs[i] = k ? float(double(w) / double(S_kept)) : 0.0f;
      if (!k) continue;
      cum += w;
      if (cum > t && before <= t && s_tok == 0xFFFFFFFFu) s_tok = unsigned(i);  // first token past t
    }
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
                          unsigned long long* rng, cudaStream_t s) {
  if (top_k < 1 || top_k > SD_THREADS || n < 1 || !(temperature > 0.0f)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(SD_THREADS);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, sample_kernel, logits, scratch, n, st, hist, pen_cnt, rep,
                                           temperature, top_k, top_p, rng);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb

namespace wcb {

cudaError_t launch_sample_full(const float* logits, float* scratch, int n, StepState* st, uint32_t* hist,
                               uint32_t* pen_cnt, float rep, float temperature, int top_k, float top_p,
                               unsigned long long* rng, float* probs, cudaStream_t s) {
  if (top_k < 0 || n < 1 || !(temperature > 0.0f)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(SD_THREADS);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, sample_full_kernel, logits, scratch, n, st, hist, pen_cnt, rep,
                                           temperature, top_k, top_p, rng, probs);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb
