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

// Builds the activation planes. PRO_RMSNORM normalises row h first exactly as
// CandleTensorBackend::rms_norm does (candle_tensor_backend.rs:30-57):
// m = sqrt(sum(h^2)/K + eps), x = h / m * w (IEEE divide and sqrt).
template <int M, int PRO>
__device__ void build_planes(const GemvArgs& a, const XPlanes& p) {
  const int K = a.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float s_part[GEMV_WARPS];
  __shared__ float s_m[4];
  if (PRO == PRO_RMSNORM) {
    for (int t = 0; t < M; ++t) {
      const float* h = a.x + size_t(t) * a.ldx;
      float ss = 0.0f;
      for (int k = threadIdx.x; k < K; k += GEMV_THREADS) ss = __fadd_rn(ss, __fmul_rn(h[k], h[k]));
      ss = warp_sum(ss);
      if (lane == 0) s_part[warp] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float tot = 0.0f;
        for (int w = 0; w < GEMV_WARPS; ++w) tot = __fadd_rn(tot, s_part[w]);
        s_m[t] = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(K)), a.eps));
      }
      __syncthreads();
    }
  }
  const int groups = M * (K / 32);
  for (int gi = warp; gi < groups; gi += GEMV_WARPS) {
    const int t = gi / (K / 32);
    const int k0 = (gi % (K / 32)) * 32;
    float v = a.x[size_t(t) * a.ldx + k0 + lane];
    if (PRO == PRO_RMSNORM) v = __fmul_rn(__fdiv_rn(v, s_m[t]), a.norm_w[k0 + lane]);
    const float amax = warp_max(fabsf(v));
    int X = 0;
    float s;
    if (amax > 0.0f && amax <= FLT_MAX) {
      const float inv = XQ_MAX / amax;
      X = __float2int_rn(v * inv);
      X = max(-8388607, min(8388607, X));
      s = amax / XQ_MAX;
    } else {
      s = (amax == 0.0f) ? 0.0f : __int_as_float(0x7fc00000);  // inf / NaN input -> NaN output
    }
    const size_t off = size_t(t) * K + k0 + lane;
    p.l0[off] = uint8_t(X & 0xFF);
    p.l1[off] = uint8_t((X >> 8) & 0xFF);
    p.l2[off] = uint8_t((X >> 16) & 0xFF);
    int sx = X;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);  // sums of 16-lane halves
    if (lane == 0) p.scale[size_t(t) * (K / 32) + k0 / 32] = s;
    if ((lane & 15) == 0) p.sum16[size_t(t) * (K / 16) + (k0 + lane) / 16] = s * float(sx);
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

__device__ __forceinline__ void resolve_row(const GemvArgs& a, int vrow, const uint8_t*& w, int& dtype, int& local) {
  int r = vrow;
  for (int s = 0; s < a.nseg; ++s) {
    if (r < a.seg[s].rows || s == a.nseg - 1) {
      w = a.seg[s].w;
      dtype = a.seg[s].dtype;
      local = r;
      return;
    }
    r -= a.seg[s].rows;
  }
}

template <int M, int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (a.st && a.st->done) return;
  const int K = a.K;
  const XPlanes p = carve(smem, M, K);
  build_planes<M, PRO>(a, p);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KS = a.ksplit;
  const int gpc = GEMV_WARPS / KS;  // row groups per CTA iteration
  const int NB = K / QK_K;

  for (int base = blockIdx.x * gpc; base < a.ngroups; base += gridDim.x * gpc) {
    const int g = base + warp / KS;
    const int ks = warp % KS;
    float acc[ROWS][M];
#pragma unroll
    for (int i = 0; i < ROWS; ++i)
#pragma unroll
      for (int t = 0; t < M; ++t) acc[i][t] = 0.0f;

    if (g < a.ngroups) {
      const uint8_t* rw[ROWS];
      int dtype = DT_Q4K;
#pragma unroll
      for (int i = 0; i < ROWS; ++i) {
        int local, dt;
        const uint8_t* w;
        if (EPI == EPI_SWIGLU) {
          const GemvSeg& sg = a.seg[i < 2 ? 0 : 1];
          w = sg.w;
          dt = sg.dtype;
          local = 2 * g + (i & 1);
        } else {
          resolve_row(a, ROWS * g + i, w, dt, local);
        }
        dtype = dt;
        rw[i] = w + size_t(local) * NB * dev_block_bytes(dt);
      }
      if (dtype == DT_Q4K) {
        const int NC = NB * 8;
        const int c0 = ks * NC / KS, c1 = (ks + 1) * NC / KS;
        for (int c = c0 + lane; c < c1; c += 32) {
          const int b = c >> 3, j = c & 7;
          uint4 qv[ROWS], hv[ROWS];
#pragma unroll
          for (int i = 0; i < ROWS; ++i) {
            const uint8_t* blk = rw[i] + size_t(b) * Q4K_BYTES;
            hv[i] = __ldg(reinterpret_cast<const uint4*>(blk));
            qv[i] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * j));
          }
#pragma unroll
          for (int i = 0; i < ROWS; ++i) q4k_chunk<M>(qv[i], hv[i], j, b * QK_K, K, p, acc[i]);
        }
      } else {
        const int NC = NB * 4;
        const int c0 = ks * NC / KS, c1 = (ks + 1) * NC / KS;
        for (int c = c0 + lane; c < c1; c += 32) {
          const int b = c >> 2, hh = (c >> 1) & 1, aa = c & 1;
          uint4 l0v[ROWS], l1v[ROWS], qhv[ROWS], scv[ROWS];
          uint32_t dv[ROWS];
#pragma unroll
          for (int i = 0; i < ROWS; ++i) {
            const uint8_t* blk = rw[i] + size_t(b) * Q6K_DEV_BYTES;
            l0v[i] = __ldg(reinterpret_cast<const uint4*>(blk + 64 * hh + 16 * aa));
            l1v[i] = __ldg(reinterpret_cast<const uint4*>(blk + 64 * hh + 32 + 16 * aa));
            qhv[i] = __ldg(reinterpret_cast<const uint4*>(blk + 128 + 32 * hh + 16 * aa));
            scv[i] = __ldg(reinterpret_cast<const uint4*>(blk + 192));
            dv[i] = __ldg(reinterpret_cast<const unsigned short*>(blk + 208));
          }
#pragma unroll
          for (int i = 0; i < ROWS; ++i)
            q6k_chunk<M>(l0v[i], l1v[i], qhv[i], scv[i], dv[i], hh, aa, b * QK_K, K, p, acc[i]);
        }
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
    if (ks == 0 && g < a.ngroups && lane < ROWS * M) {
      float v = 0.0f;
      for (int k = 0; k < KS; ++k) v += red[(warp + k) * 16 + lane];
      red[warp * 16 + lane] = v;
    }
    __syncwarp();
    if (ks == 0 && g < a.ngroups && lane < ROWS * M) {
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
      } else {  // EPI_QKV
        const int vr = ROWS * g + i;
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
            const float c = a.rope_cos[size_t(pos) * (hd / 2) + pi];
            const float sn = a.rope_sin[size_t(pos) * (hd / 2) + pi];
            const float n0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
            const float n1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
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
    __syncthreads();
  }
}

int g_sms = 0;

template <int M, int PRO, int EPI>
cudaError_t configure_gemv_t() {
  return cudaFuncSetAttribute(gemv_kernel<M, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

template <int M, int PRO, int EPI>
cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t s) {
  const size_t smem = gemv_smem_bytes(M, a.K);
  const int gpc = GEMV_WARPS / a.ksplit;
  int grid = (a.ngroups + gpc - 1) / gpc;
  const int per_sm = smem > 100 * 1024 ? 1 : 2;
  const int sms = g_sms > 0 ? g_sms : 148;
  grid = grid < sms * per_sm ? grid : sms * per_sm;
  gemv_kernel<M, PRO, EPI><<<grid, GEMV_THREADS, smem, s>>>(a);
  return cudaGetLastError();
}

#define WCB_GEMV_CASES(F)             \
  F(PRO_NONE, EPI_STORE)              \
  F(PRO_NONE, EPI_RESID)              \
  F(PRO_NONE, EPI_SWIGLU)             \
  F(PRO_NONE, EPI_QKV)                \
  F(PRO_RMSNORM, EPI_STORE)           \
  F(PRO_RMSNORM, EPI_RESID)           \
  F(PRO_RMSNORM, EPI_SWIGLU)          \
  F(PRO_RMSNORM, EPI_QKV)

template <int M>
cudaError_t launch_gemv_m(const GemvArgs& a, int pro, int epi, cudaStream_t s) {
#define WCB_GEMV_CASE(P, E) \
  if (pro == P && epi == E) return launch_gemv_t<M, P, E>(a, s);
  WCB_GEMV_CASES(WCB_GEMV_CASE)
#undef WCB_GEMV_CASE
  return cudaErrorInvalidValue;
}

template <int M>
cudaError_t configure_gemv_m() {
  cudaError_t e = cudaSuccess;
#define WCB_GEMV_CFG(P, E) \
  if (e == cudaSuccess) e = configure_gemv_t<M, P, E>();
  WCB_GEMV_CASES(WCB_GEMV_CFG)
#undef WCB_GEMV_CFG
  return e;
}

// ------------------------------------------------------------- attention --
template <typename KT>
__device__ __forceinline__ float ld_kv(const KT* p);
template <>
__device__ __forceinline__ float ld_kv<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_kv<__half>(const __half* p) { return __half2float(*p); }

constexpr int ATT_THREADS = 128;

// One CTA = (kv head, query token, key split). Scores for the n_rep query heads
// sharing the kv head (repeat_kv, attention.rs:297-322), masked j > position+t,
// softmax with max subtraction, P.V (attention.rs:332-435); partial results of
// the splits are merged by the last CTA of the (token, kv head) pair.
template <int HD, typename KT>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float asmem[];
  const StepState* st = a.st;
  if (st->done) return;
  const int kh = blockIdx.x, t = blockIdx.y, split = blockIdx.z;
  const int n_rep = a.n_heads / a.n_kv;
  const int kv_total = st->kv_len + a.T;
  const int limit = st->position + t;
  const int nkeys = min(kv_total, limit + 1);
  const int nsplit = (nkeys + a.chunk - 1) / a.chunk;
  if (split >= nsplit) return;
  const int j0 = split * a.chunk, j1 = min(j0 + a.chunk, nkeys), nj = j1 - j0;
  float* qs = asmem;               // [n_rep][HD]
  float* S = qs + n_rep * HD;      // [n_rep][chunk]
  float* ml = S + n_rep * a.chunk; // [n_rep][2]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qsrc = a.q + (size_t(t) * a.n_heads + size_t(kh) * n_rep) * HD;
  for (int i = threadIdx.x; i < n_rep * HD; i += ATT_THREADS) qs[i] = qsrc[i];
  __syncthreads();
  const KT* Kp = reinterpret_cast<const KT*>(a.kc) + size_t(kh) * a.max_seq * HD;
  const KT* Vp = reinterpret_cast<const KT*>(a.vc) + size_t(kh) * a.max_seq * HD;
  constexpr int PER = HD / 32;
  for (int j = j0 + warp; j < j1; j += ATT_THREADS / 32) {
    float kv[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) kv[e] = ld_kv<KT>(Kp + size_t(j) * HD + lane * PER + e);
    for (int r = 0; r < n_rep; ++r) {
      float d = 0.0f;
#pragma unroll
      for (int e = 0; e < PER; ++e) d += qs[r * HD + lane * PER + e] * kv[e];
      d = warp_sum(d);
      if (lane == 0) S[r * a.chunk + (j - j0)] = d * a.scale;
    }
  }
  __syncthreads();
  for (int r = warp; r < n_rep; r += ATT_THREADS / 32) {
    float mx = -INFINITY;
    for (int jj = lane; jj < nj; jj += 32) mx = fmaxf(mx, S[r * a.chunk + jj]);
    mx = warp_max(mx);
    float l = 0.0f;
    for (int jj = lane; jj < nj; jj += 32) {
      const float e = expf(S[r * a.chunk + jj] - mx);
      S[r * a.chunk + jj] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      ml[2 * r] = mx;
      ml[2 * r + 1] = l;
    }
  }
  __syncthreads();
  const size_t pstride = HD + 2;
  if (nsplit == 1) {
    for (int i = threadIdx.x; i < n_rep * HD; i += ATT_THREADS) {
      const int r = i / HD, d = i % HD;
      float acc = 0.0f;
      for (int jj = 0; jj < nj; ++jj) acc += S[r * a.chunk + jj] * ld_kv<KT>(Vp + size_t(j0 + jj) * HD + d);
      const float l = ml[2 * r + 1];
      a.out[(size_t(t) * a.n_heads + kh * n_rep + r) * HD + d] = l > 0.0f ? acc / l : 0.0f;
    }
    return;
  }
  for (int i = threadIdx.x; i < n_rep * HD; i += ATT_THREADS) {
    const int r = i / HD, d = i % HD;
    float acc = 0.0f;
    for (int jj = 0; jj < nj; ++jj) acc += S[r * a.chunk + jj] * ld_kv<KT>(Vp + size_t(j0 + jj) * HD + d);
    float* pp = a.part + ((size_t(t) * a.n_heads + kh * n_rep + r) * a.max_splits + split) * pstride;
    pp[2 + d] = acc;
    if (d == 0) {
      pp[0] = ml[2 * r];
      pp[1] = ml[2 * r + 1];
    }
  }
  __syncthreads();
  __threadfence();
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(a.ticket + t * a.n_kv + kh, 1);
    s_last = (prev == nsplit - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (threadIdx.x == 0) a.ticket[t * a.n_kv + kh] = 0;
  for (int i = threadIdx.x; i < n_rep * HD; i += ATT_THREADS) {
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
  if (st && st->done) return;
  const int t = blockIdx.y;
  const uint32_t id = ids[t];
  for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < hidden; d += gridDim.x * blockDim.x)
    x[size_t(t) * hidden + d] = id < uint32_t(vocab) ? emb[size_t(id) * hidden + d] : 0.0f;
}

__global__ void embed_last_kernel(const float* emb, int vocab, int hidden, const uint32_t* hist, float* x,
                                  const StepState* st) {
  if (st->done) return;
  const uint32_t id = hist[st->nhist - 1];
  for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < hidden; d += gridDim.x * blockDim.x)
    x[d] = id < uint32_t(vocab) ? emb[size_t(id) * hidden + d] : 0.0f;
}

constexpr int SAMPLE_THREADS = 1024;

__global__ void __launch_bounds__(SAMPLE_THREADS)
    sample_argmax_kernel(const float* logits, int V, float* work, uint32_t* hist, float rep, uint32_t* tok,
                         StepState* st, int mode, int first) {
  if (mode == 1 && st->done) return;
  const int n = st->nhist;
  for (int i = threadIdx.x; i < V; i += SAMPLE_THREADS) work[i] = logits[i];
  __syncthreads();
  if (rep != 1.0f) {
    // apply_repetition_penalty (sampling.rs:86-103): once per occurrence, in order;
    // the thread owning a token's first occurrence applies all of its repeats
    for (int e = threadIdx.x; e < n; e += SAMPLE_THREADS) {
      const uint32_t tk = hist[e];
      bool owner = tk < uint32_t(V);
      for (int f = 0; f < e && owner; ++f) owner = hist[f] != tk;
      if (!owner) continue;
      int cnt = 0;
      for (int f = e; f < n; ++f) cnt += hist[f] == tk;
      float v = work[tk];
      for (int c = 0; c < cnt; ++c) v = v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
      work[tk] = v;
    }
    __syncthreads();
  }
  // sample_argmax (sampling.rs:118-125): Iterator::max_by keeps the last maximum
  float best = -INFINITY;
  int bi = -1;
  int nan = 0;
  for (int i = threadIdx.x; i < V; i += SAMPLE_THREADS) {
    const float v = work[i];
    if (v != v) nan = 1;
    else if (bi < 0 || !(best > v)) {
      best = v;
      bi = i;
    }
  }
  nan = __syncthreads_or(nan);
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float s_v[SAMPLE_THREADS / 32];
  __shared__ int s_i[SAMPLE_THREADS / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_v[warp] = best;
    s_i[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 1; w < SAMPLE_THREADS / 32; ++w) {
    const float ov = s_v[w];
    const int oi = s_i[w];
    if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) {
      best = ov;
      bi = oi;
    }
  }
  if (bi < 0) bi = 0;
  if (nan) {
    st->err = 1;
    if (mode == 1) st->done = 1;
    *tok = 0;
    return;
  }
  *tok = uint32_t(bi);
  if (mode == 0) return;
  // generate() bookkeeping (model.rs:1380-1409)
  st->kv_len += st->n_tokens;
  st->position = st->kv_len;
  st->n_tokens = 1;
  if (first) {
    hist[st->nhist] = uint32_t(bi);
    st->nhist += 1;
    st->gen = 1;
  } else if (st->eos >= 0 && uint32_t(bi) == uint32_t(st->eos)) {
    st->done = 1;
    return;
  } else {
    hist[st->nhist] = uint32_t(bi);
    st->nhist += 1;
    st->gen += 1;
  }
  if (st->gen >= st->max_gen) st->done = 1;
  else if (st->kv_len + 1 > st->max_seq) {  // the next step's KV append would overflow (kv_cache.rs:48-53)
    st->err = 2;
    st->done = 1;
  }
}

__global__ void set_state_kernel(StepState* st, int position, int kv_len, int n_tokens) {
  st->position = position;
  st->kv_len = kv_len;
  st->n_tokens = n_tokens;
  st->done = 0;
  st->err = 0;
}

__global__ void init_gen_kernel(StepState* st, int max_gen, int eos, int max_seq) {
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
  const size_t smem = sizeof(float) * (size_t(n_rep) * a.head_dim + size_t(n_rep) * a.chunk + 2 * n_rep);
  dim3 grid(a.n_kv, a.T, a.max_splits);
  if (a.head_dim == 64) {
    if (a.kv_half) attn_kernel<64, __half><<<grid, ATT_THREADS, smem, s>>>(a);
    else attn_kernel<64, float><<<grid, ATT_THREADS, smem, s>>>(a);
  } else if (a.head_dim == 128) {
    if (a.kv_half) attn_kernel<128, __half><<<grid, ATT_THREADS, smem, s>>>(a);
    else attn_kernel<128, float><<<grid, ATT_THREADS, smem, s>>>(a);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_embed(const float* emb, int vocab, int hidden, const uint32_t* ids, int T, float* x,
                         const StepState* st, cudaStream_t s) {
  dim3 grid((hidden + 255) / 256, T);
  embed_kernel<<<grid, 256, 0, s>>>(emb, vocab, hidden, ids, T, x, st);
  return cudaGetLastError();
}

cudaError_t launch_embed_last(const float* emb, int vocab, int hidden, const uint32_t* hist, float* x,
                              const StepState* st, cudaStream_t s) {
  embed_last_kernel<<<(hidden + 255) / 256, 256, 0, s>>>(emb, vocab, hidden, hist, x, st);
  return cudaGetLastError();
}

cudaError_t launch_sample_argmax(const float* logits, int V, float* work, uint32_t* hist, float rep, uint32_t* tok,
                                 StepState* st, int mode, int first, cudaStream_t s) {
  sample_argmax_kernel<<<1, SAMPLE_THREADS, 0, s>>>(logits, V, work, hist, rep, tok, st, mode, first);
  return cudaGetLastError();
}

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
