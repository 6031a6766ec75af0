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
