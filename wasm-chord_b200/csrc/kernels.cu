// Hot-path kernels of the token loop for sm_100a.
//
// Q4_K / Q6_K GEMV ("fused dequant-GEMV"): the weights stream from HBM as raw
// blocks with 128-bit loads and are never dequantised to memory. The activation
// vector is turned, once per CTA, into exact integer limbs: each 32-value group
// g gets a scale s_g = max|x|/(2^23-1) and integers X = rint(x/s_g) split into
// three byte planes (u8, u8, s8), X = 65536*x2 + 256*x1 + x0. A super-block's
// contribution is then, exactly in integers, sum_j q_j*X_j (dp4a), scaled once
// per sub-block: for Q4_K, y += d*sc*s*dot - dmin*m*s*sum(X) — the same value
// as dequantize_q4_k (quant.rs:58-115) followed by matmul_transposed
// (gemm.rs:83-143) up to the 2^-24 relative rounding of x and a different f32
// summation order.
#include <cuda_fp16.h>

#include <cfloat>
#include <cmath>

#include "kernels.h"

namespace wcb {

namespace {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int ROWS = 4;  // rows per warp group
constexpr float XQ_MAX = 8388607.0f;  // 2^23 - 1

__device__ __forceinline__ float half_bits(uint32_t b) { return __half2float(__ushort_as_half((unsigned short)b)); }

__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// Activation planes in shared memory for M columns of K values.
struct XPlanes {
  uint8_t* l0;
  uint8_t* l1;
  uint8_t* l2;
  float* scale;  // [M][K/32]
  float* sum16;  // [M][K/16]  s_g * sum(X) over 16 values
  float* red;    // [GEMV_WARPS][16]
};

__device__ __forceinline__ XPlanes carve(uint8_t* smem, int M, int K) {
  XPlanes p;
  p.l0 = smem;
  p.l1 = smem + size_t(M) * K;
  p.l2 = smem + 2 * size_t(M) * K;
  p.scale = reinterpret_cast<float*>(smem + 3 * size_t(M) * K);
  p.sum16 = p.scale + size_t(M) * (K / 32);
  p.red = p.sum16 + size_t(M) * (K / 16);
  return p;
}

// Quantises 8 consecutive activations held by one thread into the planes.
// Four consecutive threads cover one 32-value group (max reduced over them),
// two cover a 16-value half (sum of X).
__device__ __forceinline__ void quant8(const float (&v)[8], size_t off, int kglob, const XPlanes& p, int K, int t) {
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
  bool bad = false;
#pragma unroll
  for (int e = 0; e < 8; ++e) bad |= !(fabsf(v[e]) <= FLT_MAX);  // NaN / inf
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  bad = __shfl_xor_sync(0xffffffffu, int(bad), 1) | bad;
  bad = __shfl_xor_sync(0xffffffffu, int(bad), 2) | bad;
  int X[8];
  float s;
  if (!bad && amax > 0.0f) {
    const float inv = XQ_MAX / amax;
#pragma unroll
    for (int e = 0; e < 8; ++e) X[e] = max(-8388607, min(8388607, __float2int_rn(v[e] * inv)));
    s = amax / XQ_MAX;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) X[e] = 0;
    s = bad ? __int_as_float(0x7fc00000) : 0.0f;  // inf / NaN input -> NaN output
  }
  uint32_t w0[2], w1[2], w2[2];
  int sx = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int x = X[4 * h + e];
      b0 |= uint32_t(x & 0xFF) << (8 * e);
      b1 |= uint32_t((x >> 8) & 0xFF) << (8 * e);
      b2 |= uint32_t((x >> 16) & 0xFF) << (8 * e);
      sx += x;
    }
    w0[h] = b0;
    w1[h] = b1;
    w2[h] = b2;
  }
  *reinterpret_cast<uint2*>(p.l0 + off) = make_uint2(w0[0], w0[1]);
  *reinterpret_cast<uint2*>(p.l1 + off) = make_uint2(w1[0], w1[1]);
  *reinterpret_cast<uint2*>(p.l2 + off) = make_uint2(w2[0], w2[1]);
  sx += __shfl_xor_sync(0xffffffffu, sx, 1);
  const int lane = threadIdx.x & 31;
  if ((lane & 1) == 0) p.sum16[size_t(t) * (K / 16) + kglob / 16] = s * float(sx);
  if ((lane & 3) == 0) p.scale[size_t(t) * (K / 32) + kglob / 32] = s;
}

// Builds the activation planes. PRO_RMSNORM normalises row h first exactly as
// CandleTensorBackend::rms_norm does (candle_tensor_backend.rs:30-57):
// m = sqrt(sum(h^2)/K + eps), x = h / m * w (IEEE divide and sqrt).
// Every thread owns 8 consecutive values of each 2048-value round; the loads of
// up to four rounds are issued together so the prologue costs one or two DRAM
// round trips, not one per group.
template <int M, int PRO>
__device__ void build_planes(const GemvArgs& a, const XPlanes& p) {
  const int K = a.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  constexpr int ROUND = GEMV_THREADS * 8;
  constexpr int BATCH = 4;
  const int rounds = (K + ROUND - 1) / ROUND;
  __shared__ float s_part[GEMV_WARPS];
  __shared__ float s_m[4];
  for (int t = 0; t < M; ++t) {
    const float* x = a.x + size_t(t) * a.ldx;
    if (PRO == PRO_RMSNORM) {
      float ss = 0.0f;
      for (int r0 = 0; r0 < rounds; r0 += BATCH) {
        float4 v[BATCH][2];
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          const int k = (r0 + b) * ROUND + tid * 8;
          if (r0 + b < rounds && k < K) {
            v[b][0] = __ldg(reinterpret_cast<const float4*>(x + k));
            v[b][1] = __ldg(reinterpret_cast<const float4*>(x + k + 4));
          } else {
            v[b][0] = v[b][1] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int b = 0; b < BATCH; ++b)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            ss = __fadd_rn(ss, __fmul_rn(v[b][h].x, v[b][h].x));
            ss = __fadd_rn(ss, __fmul_rn(v[b][h].y, v[b][h].y));
            ss = __fadd_rn(ss, __fmul_rn(v[b][h].z, v[b][h].z));
            ss = __fadd_rn(ss, __fmul_rn(v[b][h].w, v[b][h].w));
          }
      }
      ss = warp_sum(ss);
      if (lane == 0) s_part[warp] = ss;
      __syncthreads();
      if (tid == 0) {
        float tot = 0.0f;
        for (int w = 0; w < GEMV_WARPS; ++w) tot = __fadd_rn(tot, s_part[w]);
        s_m[t] = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(K)), a.eps));
      }
      __syncthreads();
    }
    for (int r0 = 0; r0 < rounds; r0 += BATCH) {
      float4 v[BATCH][2], w[BATCH][2];
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        const int k = (r0 + b) * ROUND + tid * 8;
        if (r0 + b < rounds && k < K) {
          v[b][0] = __ldg(reinterpret_cast<const float4*>(x + k));
          v[b][1] = __ldg(reinterpret_cast<const float4*>(x + k + 4));
          if (PRO == PRO_RMSNORM) {
            w[b][0] = __ldg(reinterpret_cast<const float4*>(a.norm_w + k));
            w[b][1] = __ldg(reinterpret_cast<const float4*>(a.norm_w + k + 4));
          }
        }
      }
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        const int k = (r0 + b) * ROUND + tid * 8;
        // whole warps are in or out of range (K is a multiple of 256)
        if (r0 + b < rounds && k < K) {
          float e[8] = {v[b][0].x, v[b][0].y, v[b][0].z, v[b][0].w, v[b][1].x, v[b][1].y, v[b][1].z, v[b][1].w};
          if (PRO == PRO_RMSNORM) {
            const float g[8] = {w[b][0].x, w[b][0].y, w[b][0].z, w[b][0].w,
                                w[b][1].x, w[b][1].y, w[b][1].z, w[b][1].w};
#pragma unroll
            for (int i = 0; i < 8; ++i) e[i] = __fmul_rn(__fdiv_rn(e[i], s_m[t]), g[i]);
          }
          quant8(e, size_t(t) * K + k, k, p, K, t);
        }
      }
    }
  }
  __syncthreads();
}

// sc / m of sub-block s from the three scale words (get_scale_min_k4, quant.rs:43-53)
__device__ __forceinline__ void scale_min(int s, uint32_t w0, uint32_t w1, uint32_t w2, uint32_t& sc, uint32_t& m) {
  if (s < 4) {
    sc = byte_of(w0, s) & 63;
    m = byte_of(w1, s) & 63;
  } else {
    sc = (byte_of(w2, s - 4) & 0xF) | ((byte_of(w0, s - 4) >> 6) << 4);
    m = (byte_of(w2, s - 4) >> 4) | ((byte_of(w1, s - 4) >> 6) << 4);
  }
}

// One Q4_K chunk: 16 qs bytes (j-th of 8 in the block) = 16 values of
// sub-block 2p (low nibbles) and 16 of sub-block 2p+1 (high nibbles).
template <int M>
__device__ __forceinline__ void q4k_chunk(const uint4& qs, const uint4& hd, int j, int vbase, int K, const XPlanes& p,
                                          float (&acc)[M]) {
  const int pr = j >> 1, hh = j & 1;
  const float d = half_bits(hd.x & 0xFFFFu), dmin = half_bits(hd.x >> 16);
  uint32_t sc0, m0, sc1, m1;
  scale_min(2 * pr, hd.y, hd.z, hd.w, sc0, m0);
  scale_min(2 * pr + 1, hd.y, hd.z, hd.w, sc1, m1);
  const uint32_t w[4] = {qs.x, qs.y, qs.z, qs.w};
  uint32_t lo[4], hi[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    lo[i] = w[i] & 0x0F0F0F0Fu;
    hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
  }
  const int vlo = vbase + 64 * pr + 16 * hh, vhi = vlo + 32;
#pragma unroll
  for (int t = 0; t < M; ++t) {
    const size_t ct = size_t(t) * K;
    const uint4 a0 = *reinterpret_cast<const uint4*>(p.l0 + ct + vlo);
    const uint4 a1 = *reinterpret_cast<const uint4*>(p.l1 + ct + vlo);
    const uint4 a2 = *reinterpret_cast<const uint4*>(p.l2 + ct + vlo);
    const uint4 b0 = *reinterpret_cast<const uint4*>(p.l0 + ct + vhi);
    const uint4 b1 = *reinterpret_cast<const uint4*>(p.l1 + ct + vhi);
    const uint4 b2 = *reinterpret_cast<const uint4*>(p.l2 + ct + vhi);
    int u0 = 0, u1 = 0, u2 = 0, v0 = 0, v1 = 0, v2 = 0;
    u0 = dp4a_uu(lo[0], a0.x, u0); u0 = dp4a_uu(lo[1], a0.y, u0); u0 = dp4a_uu(lo[2], a0.z, u0); u0 = dp4a_uu(lo[3], a0.w, u0);
    u1 = dp4a_uu(lo[0], a1.x, u1); u1 = dp4a_uu(lo[1], a1.y, u1); u1 = dp4a_uu(lo[2], a1.z, u1); u1 = dp4a_uu(lo[3], a1.w, u1);
    u2 = dp4a_us(lo[0], a2.x, u2); u2 = dp4a_us(lo[1], a2.y, u2); u2 = dp4a_us(lo[2], a2.z, u2); u2 = dp4a_us(lo[3], a2.w, u2);
    v0 = dp4a_uu(hi[0], b0.x, v0); v0 = dp4a_uu(hi[1], b0.y, v0); v0 = dp4a_uu(hi[2], b0.z, v0); v0 = dp4a_uu(hi[3], b0.w, v0);
    v1 = dp4a_uu(hi[0], b1.x, v1); v1 = dp4a_uu(hi[1], b1.y, v1); v1 = dp4a_uu(hi[2], b1.z, v1); v1 = dp4a_uu(hi[3], b1.w, v1);
    v2 = dp4a_us(hi[0], b2.x, v2); v2 = dp4a_us(hi[1], b2.y, v2); v2 = dp4a_us(hi[2], b2.z, v2); v2 = dp4a_us(hi[3], b2.w, v2);
    // |sum q*X| <= 16*15*(2^23-1) < 2^31: exact in int32
    const int dlo = u2 * 65536 + u1 * 256 + u0;
    const int dhi = v2 * 65536 + v1 * 256 + v0;
    const float* sc = p.scale + size_t(t) * (K / 32);
    const float* sm = p.sum16 + size_t(t) * (K / 16);
    const float dot = float(sc0) * sc[vlo >> 5] * float(dlo) + float(sc1) * sc[vhi >> 5] * float(dhi);
    const float mn = float(m0) * sm[vlo >> 4] + float(m1) * sm[vhi >> 4];
    acc[t] += d * dot - dmin * mn;
  }
}

// One Q6_K chunk (padded 224-byte block): half hh, 16-column slice a of the
// 32-wide interleave (quant.rs:206-261) = 4 groups of 16 values.
template <int M>
__device__ __forceinline__ void q6k_chunk(const uint4& ql0, const uint4& ql1, const uint4& qh, const uint4& scw,
                                          uint32_t dbits, int hh, int aa, int vbase, int K, const XPlanes& p,
                                          float (&acc)[M]) {
  const float d = half_bits(dbits);
  const uint32_t L[4] = {ql0.x, ql0.y, ql0.z, ql0.w};
  const uint32_t Hq[4] = {ql1.x, ql1.y, ql1.z, ql1.w};
  const uint32_t Q[4] = {qh.x, qh.y, qh.z, qh.w};
  const uint32_t S[4] = {scw.x, scw.y, scw.z, scw.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t sq[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t nib = (k == 0) ? (L[i] & 0x0F0F0F0Fu)
                         : (k == 1) ? (Hq[i] & 0x0F0F0F0Fu)
                         : (k == 2) ? ((L[i] >> 4) & 0x0F0F0F0Fu)
                                    : ((Hq[i] >> 4) & 0x0F0F0F0Fu);
      const uint32_t hb = ((Q[i] >> (2 * k)) & 0x03030303u) << 4;
      sq[i] = __vsub4(nib | hb, 0x20202020u);  // signed bytes q - 32
    }
    const int sidx = 8 * hh + aa + 2 * k;
    const int scv = int(int8_t(byte_of(S[sidx >> 2], sidx & 3)));
    const int v = vbase + 128 * hh + 32 * k + 16 * aa;
#pragma unroll
    for (int t = 0; t < M; ++t) {
      const size_t ct = size_t(t) * K + v;
      const uint4 a0 = *reinterpret_cast<const uint4*>(p.l0 + ct);
      const uint4 a1 = *reinterpret_cast<const uint4*>(p.l1 + ct);
      const uint4 a2 = *reinterpret_cast<const uint4*>(p.l2 + ct);
      int u0 = 0, u1 = 0, u2 = 0;
      u0 = dp4a_su(sq[0], a0.x, u0); u0 = dp4a_su(sq[1], a0.y, u0); u0 = dp4a_su(sq[2], a0.z, u0); u0 = dp4a_su(sq[3], a0.w, u0);
      u1 = dp4a_su(sq[0], a1.x, u1); u1 = dp4a_su(sq[1], a1.y, u1); u1 = dp4a_su(sq[2], a1.z, u1); u1 = dp4a_su(sq[3], a1.w, u1);
      u2 = dp4a_ss(sq[0], a2.x, u2); u2 = dp4a_ss(sq[1], a2.y, u2); u2 = dp4a_ss(sq[2], a2.z, u2); u2 = dp4a_ss(sq[3], a2.w, u2);
      const float fd = float(u2) * 65536.0f + float(u1) * 256.0f + float(u0);
      acc[t] += d * float(scv) * p.scale[size_t(t) * (K / 32) + (v >> 5)] * fd;
    }
  }
}

// Programmatic dependent launch: a kernel launched with the PDL attribute may
// start while its predecessor drains; griddepcontrol.wait blocks until the
// predecessor has completed and its writes are visible (a no-op otherwise).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// order-preserving u32 image of a float (+0 and -0 compare equal, as in max_by)
__device__ __forceinline__ uint32_t order_key(float v) {
  if (v == 0.0f) v = 0.0f;
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int DT>
struct WRegs;
template <>
struct WRegs<DT_Q4K> {
  uint4 q[ROWS], h[ROWS];
};
template <>
struct WRegs<DT_Q6K> {
  uint4 l0[ROWS], l1[ROWS], qh[ROWS], sc[ROWS];
  uint32_t d[ROWS];
};

__device__ __forceinline__ void load_chunk(WRegs<DT_Q4K>& r, const uint8_t* const (&rw)[ROWS], int c) {
  const int b = c >> 3, j = c & 7;
#pragma unroll
  for (int i = 0; i < ROWS; ++i) {
    const uint8_t* blk = rw[i] + size_t(b) * Q4K_BYTES;
    r.h[i] = __ldg(reinterpret_cast<const uint4*>(blk));
    r.q[i] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * j));
  }
}

__device__ __forceinline__ void load_chunk(WRegs<DT_Q6K>& r, const uint8_t* const (&rw)[ROWS], int c) {
  const int b = c >> 2, hh = (c >> 1) & 1, aa = c & 1;
#pragma unroll
  for (int i = 0; i < ROWS; ++i) {
    const uint8_t* blk = rw[i] + size_t(b) * Q6K_DEV_BYTES;
    r.l0[i] = __ldg(reinterpret_cast<const uint4*>(blk + 64 * hh + 16 * aa));
    r.l1[i] = __ldg(reinterpret_cast<const uint4*>(blk + 64 * hh + 32 + 16 * aa));
    r.qh[i] = __ldg(reinterpret_cast<const uint4*>(blk + 128 + 32 * hh + 16 * aa));
    r.sc[i] = __ldg(reinterpret_cast<const uint4*>(blk + 192));
    r.d[i] = __ldg(reinterpret_cast<const unsigned short*>(blk + 208));
  }
}

template <int M>
__device__ __forceinline__ void compute_chunk(const WRegs<DT_Q4K>& r, int c, int K, const XPlanes& p,
                                              float (&acc)[ROWS][M]) {
  const int b = c >> 3, j = c & 7;
#pragma unroll
  for (int i = 0; i < ROWS; ++i) q4k_chunk<M>(r.q[i], r.h[i], j, b * QK_K, K, p, acc[i]);
}

template <int M>
__device__ __forceinline__ void compute_chunk(const WRegs<DT_Q6K>& r, int c, int K, const XPlanes& p,
                                              float (&acc)[ROWS][M]) {
  const int b = c >> 2, hh = (c >> 1) & 1, aa = c & 1;
#pragma unroll
  for (int i = 0; i < ROWS; ++i) q6k_chunk<M>(r.l0[i], r.l1[i], r.qh[i], r.sc[i], r.d[i], hh, aa, b * QK_K, K, p, acc[i]);
}

// Sampler bookkeeping of generate() (model.rs:1380-1409) after the LM head:
// the argmax token is pushed unless it is EOS (never for the first token), the
// KV position advances, max_tokens / KV capacity end the loop.
__device__ void finish_sample(const GemvArgs& a) {
  StepState* st = a.st;
  const unsigned long long best = atomicExch(&st->best, 0ull);
  const int nan = atomicExch(&st->nan, 0);
  st->ticket = 0;
  if (nan) {  // partial_cmp().unwrap() panics on NaN in the reference
    st->err = 1;
    st->done = 1;
    return;
  }
  const uint32_t tok = uint32_t(best & 0xFFFFFFFFull);
  const bool first = st->gen == 0;
  st->kv_len += st->n_tokens;
  st->position = st->kv_len;
  st->n_tokens = 1;
  if (!first && st->eos >= 0 && tok == uint32_t(st->eos)) {
    st->done = 1;
    return;
  }
  a.hist[st->nhist] = tok;
  st->nhist += 1;
  a.pen_cnt_w[tok] += 1;
  st->gen += 1;
  if (st->gen >= st->max_gen) st->done = 1;
  else if (st->kv_len + 1 > st->max_seq) {  // the next step's KV append would overflow (kv_cache.rs:48-53)
    st->err = 2;
    st->done = 1;
  }
}

// One warp set (KS warps) per group of 4 rows; the grid covers all groups.
// Weights are prefetched into registers before the activations are waited on,
// and the chunk loop keeps the next chunk's loads in flight while it computes.
template <int M, int PRO, int EPI, int DT>
__global__ void __launch_bounds__(GEMV_THREADS, (M == 1 && DT == DT_Q4K) ? 2 : 1) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = a.K;
  const XPlanes p = carve(smem, M, K);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KS = a.ksplit;
  const int gpc = GEMV_WARPS / KS;
  const int NB = K / QK_K;
  const int g = blockIdx.x * gpc + warp / KS;
  const int ks = warp % KS;
  const bool active = g < a.ngroups;
  constexpr int CPB = DT == DT_Q4K ? 8 : 4;
  constexpr int BB = DT == DT_Q4K ? Q4K_BYTES : Q6K_DEV_BYTES;
  const int NC = NB * CPB;
  const int c0 = ks * NC / KS, c1 = (ks + 1) * NC / KS;
  const size_t row_bytes = size_t(NB) * BB;

  const uint8_t* rw[ROWS];
#pragma unroll
  for (int i = 0; i < ROWS; ++i) rw[i] = nullptr;
  if (active) {
    if (EPI == EPI_SWIGLU) {
#pragma unroll
      for (int i = 0; i < ROWS; ++i) rw[i] = a.seg[i < 2 ? 0 : 1].w + size_t(2 * g + (i & 1)) * row_bytes;
    } else {
      int r = ROWS * g, sg = 0;
      while (sg < a.nseg - 1 && r >= a.seg[sg].rows) r -= a.seg[sg++].rows;
#pragma unroll
      for (int i = 0; i < ROWS; ++i) rw[i] = a.seg[sg].w + size_t(r + i) * row_bytes;
    }
  }
  WRegs<DT> cur;
  int c = c0 + lane;
  if (active && c < c1) load_chunk(cur, rw, c);

  pdl_trigger();
  pdl_wait();
  if (a.st && a.st->done) return;
  build_planes<M, PRO>(a, p);

  float acc[ROWS][M];
#pragma unroll
  for (int i = 0; i < ROWS; ++i)
#pragma unroll
    for (int t = 0; t < M; ++t) acc[i][t] = 0.0f;
  if (active) {
    for (; c < c1; c += 32) {
      WRegs<DT> nxt;
      const bool more = c + 32 < c1;
      if (more) load_chunk(nxt, rw, c + 32);
      compute_chunk<M>(cur, c, K, p, acc);
      if (more) cur = nxt;
    }
  }
#pragma unroll
  for (int i = 0; i < ROWS; ++i)
#pragma unroll
    for (int t = 0; t < M; ++t) acc[i][t] = warp_sum(acc[i][t]);

  // combine the KS warps of a row group, then run the epilogue on final values
  float* red = p.red;
  if (lane < ROWS * M) {
    float v = 0.0f;
#pragma unroll
    for (int i = 0; i < ROWS; ++i)
#pragma unroll
      for (int t = 0; t < M; ++t)
        if (lane == i * M + t) v = acc[i][t];
    red[warp * 16 + lane] = v;
  }
  __syncthreads();
  const bool lead = ks == 0 && active && lane < ROWS * M;
  if (lead) {
    float v = 0.0f;
    for (int k = 0; k < KS; ++k) v += red[(warp + k) * 16 + lane];
    red[warp * 16 + lane] = v;
  }
  __syncwarp();
  unsigned long long best = 0ull;
  int nan = 0;
  if (lead) {
    const int i = lane / M, t = lane % M;
    const float v = red[warp * 16 + lane];
    const int tok = t;  // column within this launch
    if (EPI == EPI_STORE) {
      a.y[size_t(tok) * a.ldy + ROWS * g + i] = v;
    } else if (EPI == EPI_RESID) {
      const size_t o = size_t(tok) * a.ldy + ROWS * g + i;
      a.y[o] = __fadd_rn(a.resid[size_t(tok) * a.ldr + ROWS * g + i], v);
    } else if (EPI == EPI_SWIGLU) {
      if (i < 2) {
        const float gv = v, uv = red[warp * 16 + (i + 2) * M + t];
        // ffn.rs:90-94: sigmoid = 1/(1+exp(-g)); silu = g*sigmoid; g = silu*u
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
        a.y[size_t(tok) * a.ldy + 2 * g + i] = __fmul_rn(__fmul_rn(gv, sig), uv);
      }
    } else if (EPI == EPI_LMHEAD) {
      const int n = ROWS * g + i;
      a.y[n] = v;
      if (a.gen_mode) {
        float pv = v;
        if (a.rep != 1.0f) {  // apply_repetition_penalty: once per occurrence (sampling.rs:86-103)
          const uint32_t cnt = a.pen_cnt[n];
          for (uint32_t k = 0; k < cnt; ++k) pv = pv > 0.0f ? __fdiv_rn(pv, a.rep) : __fmul_rn(pv, a.rep);
        }
        if (pv != pv) nan = 1;
        else best = (static_cast<unsigned long long>(order_key(pv)) << 32) | uint32_t(n);
      }
    } else {  // EPI_QKV
      const int vr = a.row_offset + ROWS * g + i;
      const int gtok = a.token_offset + tok;
      const int pos = a.st->position + gtok;
      const int slot = a.st->kv_len + gtok;
      const int hd = a.head_dim;
      if (vr < a.hidden + a.kv_dim) {
        // RoPE on (2i, 2i+1) pairs (attention.rs:230-262), cos/sin from the table
        if ((i & 1) == 0) {
          const float x0 = v, x1 = red[warp * 16 + (i + 1) * M + t];
          const int col = vr < a.hidden ? vr : vr - a.hidden;
          const int pi = (col % hd) >> 1;
          const float cs = a.rope_cos[size_t(pos) * (hd / 2) + pi];
          const float sn = a.rope_sin[size_t(pos) * (hd / 2) + pi];
          const float n0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
          const float n1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
          if (vr < a.hidden) {
            a.q[size_t(tok) * a.ldq + vr] = n0;
            a.q[size_t(tok) * a.ldq + vr + 1] = n1;
          } else {
            const int kh = col / hd, dd = col % hd;
            const size_t o = (size_t(kh) * a.max_seq + slot) * hd + dd;
            if (a.kv_half) {
              reinterpret_cast<__half*>(a.kc)[o] = __float2half_rn(n0);
              reinterpret_cast<__half*>(a.kc)[o + 1] = __float2half_rn(n1);
            } else {
              reinterpret_cast<float*>(a.kc)[o] = n0;
              reinterpret_cast<float*>(a.kc)[o + 1] = n1;
            }
          }
        }
      } else {
        const int col = vr - a.hidden - a.kv_dim;
        const int kh = col / hd, dd = col % hd;
        const size_t o = (size_t(kh) * a.max_seq + slot) * hd + dd;
        if (a.kv_half) reinterpret_cast<__half*>(a.vc)[o] = __float2half_rn(v);
        else reinterpret_cast<float*>(a.vc)[o] = v;
      }
    }
  }
  if (EPI == EPI_LMHEAD && a.gen_mode) {
    // CTA-wide max of the keys, one atomic per CTA; the last CTA to finish runs
    // the sampler bookkeeping (no CTA ever waits for another)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
      best = ob > best ? ob : best;
      nan |= __shfl_xor_sync(0xffffffffu, nan, o);
    }
    __shared__ unsigned long long s_best[GEMV_WARPS];
    __shared__ int s_nan[GEMV_WARPS];
    if (lane == 0) {
      s_best[warp] = best;
      s_nan[warp] = nan;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = 0ull;
      int n = 0;
      for (int w = 0; w < GEMV_WARPS; ++w) {
        b = s_best[w] > b ? s_best[w] : b;
        n |= s_nan[w];
      }
      if (b) atomicMax(&a.st->best, b);
      if (n) atomicOr(&a.st->nan, 1);
      __threadfence();
      const int prev = atomicAdd(&a.st->ticket, 1);
      if (prev == int(gridDim.x) - 1) {
        __threadfence();
        finish_sample(a);
      }
    }
  }
}

int g_sms = 0;
bool g_pdl = true;

template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && g_pdl) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <int M, int PRO, int EPI, int DT>
cudaError_t configure_gemv_t() {
  return cudaFuncSetAttribute(gemv_kernel<M, PRO, EPI, DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

template <int M, int PRO, int EPI, int DT>
cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t s) {
  const size_t smem = gemv_smem_bytes(M, a.K);
  const int gpc = GEMV_WARPS / a.ksplit;
  const int grid = (a.ngroups + gpc - 1) / gpc;
  const cudaError_t e =
      launch_ex(gemv_kernel<M, PRO, EPI, DT>, dim3(grid), dim3(GEMV_THREADS), smem, s, a.pdl != 0, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

#define WCB_GEMV_CASES(F)   \
  F(PRO_NONE, EPI_STORE)    \
  F(PRO_NONE, EPI_RESID)    \
  F(PRO_RMSNORM, EPI_QKV)   \
  F(PRO_RMSNORM, EPI_SWIGLU) \
  F(PRO_RMSNORM, EPI_STORE) \
  F(PRO_RMSNORM, EPI_LMHEAD)

template <int M>
cudaError_t launch_gemv_m(const GemvArgs& a, int pro, int epi, cudaStream_t s) {
  const int dt = a.seg[0].dtype;
#define WCB_GEMV_CASE(P, E)                                                  \
  if (pro == P && epi == E)                                                  \
    return dt == DT_Q4K ? launch_gemv_t<M, P, E, DT_Q4K>(a, s) : launch_gemv_t<M, P, E, DT_Q6K>(a, s);
  WCB_GEMV_CASES(WCB_GEMV_CASE)
#undef WCB_GEMV_CASE
  return cudaErrorInvalidValue;
}

template <int M>
cudaError_t configure_gemv_m() {
  cudaError_t e = cudaSuccess;
#define WCB_GEMV_CFG(P, E)                                      \
  if (e == cudaSuccess) e = configure_gemv_t<M, P, E, DT_Q4K>(); \
  if (e == cudaSuccess) e = configure_gemv_t<M, P, E, DT_Q6K>();
  WCB_GEMV_CASES(WCB_GEMV_CFG)
#undef WCB_GEMV_CFG
  return e;
}

// ------------------------------------------------------------- attention --
template <typename KT>
__device__ __forceinline__ float4 ld_kv4(const KT* p);
template <>
__device__ __forceinline__ float4 ld_kv4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 ld_kv4<__half>(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

constexpr int ATT_THREADS = 128;
constexpr int ATT_WARPS = ATT_THREADS / 32;

// One CTA = (kv head, query token, key split). The n_rep query heads sharing
// the kv head (repeat_kv, attention.rs:297-322) are processed together; keys
// are staged ATT_TILE at a time in shared memory, scores s = (q.k)*scale with
// the dot product in key order without contraction, causal limit j <= position+t,
// softmax with a running max, P.V (attention.rs:332-435). With several splits
// the last CTA of a (token, kv head) merges the partial results (ticket counter).
template <int HD, typename KT>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float asmem[];
  pdl_trigger();
  pdl_wait();
  const StepState* st = a.st;
  if (st->done) return;
  const int kh = blockIdx.x, t = blockIdx.y, split = blockIdx.z;
  const int n_rep = a.n_heads / a.n_kv;
  const int kv_total = st->kv_len + a.T;
  const int limit = st->position + t;
  const int nkeys = min(kv_total, limit + 1);
  const int nsplit = (nkeys + a.chunk - 1) / a.chunk;
  if (split >= nsplit) return;
  const int j0 = split * a.chunk, j1 = min(j0 + a.chunk, nkeys);
  constexpr int TS = ATT_TILE, KP = HD + 1;
  float* qs = asmem;               // [n_rep][HD]
  float* Ks = qs + n_rep * HD;     // [TS][HD+1]
  float* Vs = Ks + TS * KP;        // [TS][HD]
  float* S = Vs + TS * HD;         // [n_rep][TS]
  float* ml = S + n_rep * TS;      // [n_rep][2] running (max, sum)
  float* corr = ml + 2 * n_rep;    // [n_rep] rescale of the running sums for this tile
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* qsrc = a.q + (size_t(t) * a.n_heads + size_t(kh) * n_rep) * HD;
  for (int i = tid; i < n_rep * HD / 4; i += ATT_THREADS)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(qsrc)[i];
  for (int r = tid; r < n_rep; r += ATT_THREADS) {
    ml[2 * r] = -INFINITY;
    ml[2 * r + 1] = 0.0f;
  }
  const KT* Kp = reinterpret_cast<const KT*>(a.kc) + size_t(kh) * a.max_seq * HD;
  const KT* Vp = reinterpret_cast<const KT*>(a.vc) + size_t(kh) * a.max_seq * HD;
  constexpr int MAXI = 16;  // (n_rep * HD) / ATT_THREADS <= 16
  const int ni = (n_rep * HD + ATT_THREADS - 1) / ATT_THREADS;
  float acc[MAXI];
#pragma unroll
  for (int k = 0; k < MAXI; ++k) acc[k] = 0.0f;

  for (int tile0 = j0; tile0 < j1; tile0 += TS) {
    const int nt = min(TS, j1 - tile0);
    __syncthreads();
    {  // stage K and V rows [tile0, tile0 + nt): all loads issued before any store
      constexpr int PER = TS * HD / 4 / ATT_THREADS;  // float4 per thread per matrix
      float4 kv[PER], vv[PER];
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const int i = tid + e * ATT_THREADS;
        const int row = (i * 4) / HD;
        if (row < nt) {
          kv[e] = ld_kv4<KT>(Kp + size_t(tile0) * HD + size_t(i) * 4);
          vv[e] = ld_kv4<KT>(Vp + size_t(tile0) * HD + size_t(i) * 4);
        }
      }
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const int i = tid + e * ATT_THREADS;
        const int row = (i * 4) / HD, col = (i * 4) % HD;
        if (row < nt) {
          float* kr = Ks + row * KP + col;
          kr[0] = kv[e].x; kr[1] = kv[e].y; kr[2] = kv[e].z; kr[3] = kv[e].w;
          *reinterpret_cast<float4*>(Vs + row * HD + col) = vv[e];
        }
      }
    }
    __syncthreads();
    for (int r = warp; r < n_rep; r += ATT_WARPS) {
      float sc = -INFINITY;
      if (lane < nt) {
        float d = 0.0f;
        const float* qr = qs + r * HD;
        const float* kr = Ks + lane * KP;
#pragma unroll 16
        for (int dd = 0; dd < HD; ++dd) d = __fadd_rn(d, __fmul_rn(qr[dd], kr[dd]));
        sc = __fmul_rn(d, a.scale);
      }
      const float m_old = ml[2 * r];
      const float m_new = fmaxf(m_old, warp_max(sc));
      const float pr = lane < nt ? expf(sc - m_new) : 0.0f;
      const float psum = warp_sum(pr);
      S[r * TS + lane] = pr;
      if (lane == 0) {
        const float cf = expf(m_old - m_new);
        ml[2 * r] = m_new;
        ml[2 * r + 1] = ml[2 * r + 1] * cf + psum;
        corr[r] = cf;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {
      const int idx = tid + k * ATT_THREADS;
      if (k < ni && idx < n_rep * HD) {
        const int r = idx / HD, d = idx % HD;
        float s2 = acc[k] * corr[r];
        for (int jj = 0; jj < nt; ++jj) s2 += S[r * TS + jj] * Vs[jj * HD + d];
        acc[k] = s2;
      }
    }
  }
  __syncthreads();
  const size_t pstride = HD + 2;
  if (nsplit == 1) {
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {
      const int idx = tid + k * ATT_THREADS;
      if (k < ni && idx < n_rep * HD) {
        const int r = idx / HD, d = idx % HD;
        const float l = ml[2 * r + 1];
        a.out[(size_t(t) * a.n_heads + kh * n_rep + r) * HD + d] = l > 0.0f ? acc[k] / l : 0.0f;
      }
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < MAXI; ++k) {
    const int idx = tid + k * ATT_THREADS;
    if (k < ni && idx < n_rep * HD) {
      const int r = idx / HD, d = idx % HD;
      float* pp = a.part + ((size_t(t) * a.n_heads + kh * n_rep + r) * a.max_splits + split) * pstride;
      pp[2 + d] = acc[k];
      if (d == 0) {
        pp[0] = ml[2 * r];
        pp[1] = ml[2 * r + 1];
      }
    }
  }
  __syncthreads();
  __threadfence();
  __shared__ int s_last;
  if (tid == 0) {
    const int prev = atomicAdd(a.ticket + t * a.n_kv + kh, 1);
    s_last = (prev == nsplit - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) a.ticket[t * a.n_kv + kh] = 0;
  for (int i = tid; i < n_rep * HD; i += ATT_THREADS) {
    const int r = i / HD, d = i % HD;
    const float* pp = a.part + (size_t(t) * a.n_heads + kh * n_rep + r) * a.max_splits * pstride;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, __ldcg(pp + sp * pstride));
    float L = 0.0f, O = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float f = expf(__ldcg(pp + sp * pstride) - M);
      L += __ldcg(pp + sp * pstride + 1) * f;
      O += __ldcg(pp + sp * pstride + 2 + d) * f;
    }
    a.out[(size_t(t) * a.n_heads + kh * n_rep + r) * HD + d] = L > 0.0f ? O / L : 0.0f;
  }
}

// ------------------------------------------------------------ small ops ---
__global__ void embed_kernel(const float* emb, int vocab, int hidden, const uint32_t* ids, int T, float* x,
                             const StepState* st) {
  pdl_trigger();
  pdl_wait();
  if (st && st->done) return;
  const int t = blockIdx.y;
  const uint32_t id = ids[t];
  for (int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4; d < hidden; d += gridDim.x * blockDim.x * 4) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (id < uint32_t(vocab)) v = *reinterpret_cast<const float4*>(emb + size_t(id) * hidden + d);
    *reinterpret_cast<float4*>(x + size_t(t) * hidden + d) = v;
  }
}

__global__ void embed_last_kernel(const float* emb, int vocab, int hidden, const uint32_t* hist, float* x,
                                  const StepState* st) {
  pdl_trigger();
  pdl_wait();
  if (st->done) return;
  const uint32_t id = hist[st->nhist - 1];
  for (int d = (blockIdx.x * blockDim.x + threadIdx.x) * 4; d < hidden; d += gridDim.x * blockDim.x * 4) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (id < uint32_t(vocab)) v = *reinterpret_cast<const float4*>(emb + size_t(id) * hidden + d);
    *reinterpret_cast<float4*>(x + d) = v;
  }
}

__global__ void set_state_kernel(StepState* st, int position, int kv_len, int n_tokens) {
  st->position = position;
  st->kv_len = kv_len;
  st->n_tokens = n_tokens;
  st->done = 0;
  st->err = 0;
  st->best = 0ull;
  st->ticket = 0;
  st->nan = 0;
}

__global__ void init_gen_kernel(StepState* st, int max_gen, int eos, int max_seq) {
  st->best = 0ull;
  st->ticket = 0;
  st->nan = 0;
  st->gen = 0;
  st->nhist = 0;
  st->max_gen = max_gen;
  st->eos = eos;
  st->max_seq = max_seq;
  st->done = 0;
  st->err = 0;
}

__global__ void dequant_q4k_kernel(const uint8_t* blocks, size_t nblocks, float* out) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nblocks * QK_K) return;
  const size_t b = i / QK_K;
  const int j = int(i % QK_K);
  const uint8_t* blk = blocks + b * Q4K_BYTES;
  const float d = half_bits(uint32_t(blk[0]) | (uint32_t(blk[1]) << 8));
  const float dmin = half_bits(uint32_t(blk[2]) | (uint32_t(blk[3]) << 8));
  const int grp = j / 64, within = j % 64, sb = 2 * grp + (within >= 32);
  const uint8_t* sc = blk + 4;
  uint32_t s, m;
  if (sb < 4) {
    s = sc[sb] & 63;
    m = sc[sb + 4] & 63;
  } else {
    s = (sc[sb + 4] & 0xF) | ((sc[sb - 4] >> 6) << 4);
    m = (sc[sb + 4] >> 4) | ((sc[sb] >> 6) << 4);
  }
  const uint8_t qb = blk[16 + 32 * grp + (within & 31)];
  const uint32_t q = within < 32 ? (qb & 0xF) : (qb >> 4);
  // quant.rs:82-110: d1 = d*sc, m1 = min*m, y = d1*q - m1 (no contraction)
  out[i] = __fsub_rn(__fmul_rn(__fmul_rn(d, float(s)), float(q)), __fmul_rn(dmin, float(m)));
}

__global__ void dequant_q6k_kernel(const uint8_t* blocks, size_t nblocks, float* out) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nblocks * QK_K) return;
  const size_t b = i / QK_K;
  const int j = int(i % QK_K);
  const uint8_t* blk = blocks + b * Q6K_BYTES;
  const int hh = j / 128, r = j % 128, k = r / 32, l = r % 32;
  const uint8_t* ql = blk + 64 * hh;
  const uint8_t* qh = blk + 128 + 32 * hh;
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192) + 8 * hh;
  const float d = half_bits(uint32_t(blk[208]) | (uint32_t(blk[209]) << 8));
  const int lo = (k & 1) ? ql[l + 32] : ql[l];
  const int nib = (k < 2) ? (lo & 0xF) : (lo >> 4);
  const int q = (nib | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
  // quant.rs:228-258: y = d * scale * q, left to right
  out[i] = __fmul_rn(__fmul_rn(d, float(sc[l / 16 + 2 * k])), float(q));
}

__global__ void repack_q6k_kernel(const uint8_t* src, size_t nblocks, uint8_t* dst) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nblocks * Q6K_DEV_BYTES) return;
  const size_t b = i / Q6K_DEV_BYTES;
  const int o = int(i % Q6K_DEV_BYTES);
  dst[i] = o < Q6K_BYTES ? src[b * Q6K_BYTES + o] : 0;
}

}  // namespace

size_t gemv_smem_bytes(int M, int K) {
  return size_t(3) * M * K + sizeof(float) * (size_t(M) * (K / 32) + size_t(M) * (K / 16)) +
         sizeof(float) * GEMV_WARPS * 16;
}

int gemv_max_cols(int K) {
  for (int m = 4; m > 1; --m)
    if (gemv_smem_bytes(m, K) <= 96 * 1024) return m;
  return 1;
}

cudaError_t launch_gemv(const GemvArgs& a, int pro, int epi, cudaStream_t s) {
  switch (a.M) {
    case 1: return launch_gemv_m<1>(a, pro, epi, s);
    case 2: return launch_gemv_m<2>(a, pro, epi, s);
    case 3: return launch_gemv_m<3>(a, pro, epi, s);
    case 4: return launch_gemv_m<4>(a, pro, epi, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s) {
  const int n_rep = a.n_heads / a.n_kv;
  const int hd = a.head_dim;
  const size_t smem = sizeof(float) * (size_t(n_rep) * hd + size_t(ATT_TILE) * (hd + 1) + size_t(ATT_TILE) * hd +
                                       size_t(n_rep) * ATT_TILE + 3 * size_t(n_rep));
  if (n_rep * hd > ATT_THREADS * 16) return cudaErrorInvalidValue;
  const dim3 grid(a.n_kv, a.T, a.max_splits);
  cudaError_t e;
  if (hd == 64) {
    e = a.kv_half ? launch_ex(attn_kernel<64, __half>, grid, dim3(ATT_THREADS), smem, s, true, a)
                  : launch_ex(attn_kernel<64, float>, grid, dim3(ATT_THREADS), smem, s, true, a);
  } else if (hd == 128) {
    e = a.kv_half ? launch_ex(attn_kernel<128, __half>, grid, dim3(ATT_THREADS), smem, s, true, a)
                  : launch_ex(attn_kernel<128, float>, grid, dim3(ATT_THREADS), smem, s, true, a);
  } else {
    return cudaErrorInvalidValue;
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_embed(const float* emb, int vocab, int hidden, const uint32_t* ids, int T, float* x,
                         const StepState* st, cudaStream_t s) {
  const dim3 grid((hidden / 4 + 255) / 256, T);
  const cudaError_t e = launch_ex(embed_kernel, grid, dim3(256), 0, s, true, emb, vocab, hidden, ids, T, x, st);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_embed_last(const float* emb, int vocab, int hidden, const uint32_t* hist, float* x,
                              const StepState* st, cudaStream_t s) {
  const cudaError_t e =
      launch_ex(embed_last_kernel, dim3((hidden / 4 + 255) / 256), dim3(256), 0, s, true, emb, vocab, hidden, hist, x, st);
  return e != cudaSuccess ? e : cudaGetLastError();
}

void set_pdl(bool on) { g_pdl = on; }

cudaError_t launch_set_state(StepState* st, int position, int kv_len, int n_tokens, cudaStream_t s) {
  set_state_kernel<<<1, 1, 0, s>>>(st, position, kv_len, n_tokens);
  return cudaGetLastError();
}

cudaError_t launch_init_gen(StepState* st, int max_gen, int eos, int max_seq, cudaStream_t s) {
  init_gen_kernel<<<1, 1, 0, s>>>(st, max_gen, eos, max_seq);
  return cudaGetLastError();
}

cudaError_t gemv_configure_all() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = configure_gemv_m<1>();
  if (e == cudaSuccess) e = configure_gemv_m<2>();
  if (e == cudaSuccess) e = configure_gemv_m<3>();
  if (e == cudaSuccess) e = configure_gemv_m<4>();
  return e;
}

cudaError_t launch_dequant(const void* blocks, int dtype, size_t nblocks, float* out, cudaStream_t s) {
  const size_t n = nblocks * QK_K;
  if (n == 0) return cudaSuccess;
  const unsigned grid = unsigned((n + 255) / 256);
  if (dtype == DT_Q4K) dequant_q4k_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(blocks), nblocks, out);
  else if (dtype == DT_Q6K) dequant_q6k_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(blocks), nblocks, out);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_repack_q6k(const void* packed, size_t nblocks, void* padded, cudaStream_t s) {
  const size_t n = nblocks * Q6K_DEV_BYTES;
  if (n == 0) return cudaSuccess;
  repack_q6k_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(static_cast<const uint8_t*>(packed), nblocks,
                                                               static_cast<uint8_t*>(padded));
  return cudaGetLastError();
}

}  // namespace wcb
