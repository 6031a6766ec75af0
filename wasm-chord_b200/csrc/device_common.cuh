// Device helpers shared by the per-op kernels (kernels.cu) and the persistent
// decode-step kernel (decode_step.cu): dp4a wrappers, warp reductions, the
// activation limb planes, Q4_K / Q6_K chunk dot products over shared memory,
// mbarrier + bulk-copy (cp.async.bulk, no multicast) primitives and the
// generate() bookkeeping run after the argmax.
#pragma once
#include <cuda_fp16.h>

#include <cfloat>
#include <cmath>
#include <cstdint>

#include "kernels.h"

namespace wcb {
namespace {

__device__ __forceinline__ float half_bits(uint32_t b) { return __half2float(__ushort_as_half((unsigned short)b)); }
constexpr int ROWS = 4;  // rows per warp group
constexpr float XQ_MAX = 4194303.0f;  // 2^22 - 1: a 32-value dot of 4-bit weights stays below 2^31
constexpr int XQ_IMAX = 4194303;


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
  float* sum32;  // [M][K/32]  s_g * sum(X) over the group
  float* red;    // [GEMV_WARPS][16]
};

__device__ __forceinline__ XPlanes carve(uint8_t* smem, int M, int K) {
  XPlanes p;
  p.l0 = smem;
  p.l1 = smem + size_t(M) * K;
  p.l2 = smem + 2 * size_t(M) * K;
  p.scale = reinterpret_cast<float*>(smem + 3 * size_t(M) * K);
  p.sum32 = p.scale + size_t(M) * (K / 32);
  p.red = p.sum32 + size_t(M) * (K / 32);
  return p;
}

// Quantises 8 consecutive activations held by one thread into the planes.
// Four consecutive threads cover one 32-value group (max and sum of X reduced
// over them).
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
    for (int e = 0; e < 8; ++e) X[e] = max(-XQ_IMAX, min(XQ_IMAX, __float2int_rn(v[e] * inv)));
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
  sx += __shfl_xor_sync(0xffffffffu, sx, 2);  // |sum X| <= 32 * (2^22 - 1) < 2^31
  const int lane = threadIdx.x & 31;
  if ((lane & 3) == 0) {
    p.scale[size_t(t) * (K / 32) + kglob / 32] = s;
    p.sum32[size_t(t) * (K / 32) + kglob / 32] = s * float(sx);
  }
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

// One Q4_K chunk: the 32 qs bytes of sub-block pair pr = 32 values of
// sub-block 2pr (low nibbles) and 32 of sub-block 2pr+1 (high nibbles).
template <int M>
__device__ __forceinline__ void q4k_chunk(const uint4& qa, const uint4& qb, const uint4& hd, int pr, int vbase, int K,
                                          const XPlanes& p, float (&acc)[M]) {
  const float d = half_bits(hd.x & 0xFFFFu), dmin = half_bits(hd.x >> 16);
  uint32_t sc0, m0, sc1, m1;
  scale_min(2 * pr, hd.y, hd.z, hd.w, sc0, m0);
  scale_min(2 * pr + 1, hd.y, hd.z, hd.w, sc1, m1);
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    lo[i] = w[i] & 0x0F0F0F0Fu;
    hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
  }
  const int vlo = vbase + 64 * pr, vhi = vlo + 32;
#pragma unroll
  for (int t = 0; t < M; ++t) {
    const size_t ct = size_t(t) * K;
    int u0 = 0, u1 = 0, u2 = 0, v0 = 0, v1 = 0, v2 = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 a0 = *reinterpret_cast<const uint4*>(p.l0 + ct + vlo + 16 * h);
      const uint4 a1 = *reinterpret_cast<const uint4*>(p.l1 + ct + vlo + 16 * h);
      const uint4 a2 = *reinterpret_cast<const uint4*>(p.l2 + ct + vlo + 16 * h);
      const uint4 b0 = *reinterpret_cast<const uint4*>(p.l0 + ct + vhi + 16 * h);
      const uint4 b1 = *reinterpret_cast<const uint4*>(p.l1 + ct + vhi + 16 * h);
      const uint4 b2 = *reinterpret_cast<const uint4*>(p.l2 + ct + vhi + 16 * h);
      const uint32_t* L = lo + 4 * h;
      const uint32_t* H = hi + 4 * h;
      u0 = dp4a_uu(L[0], a0.x, u0); u0 = dp4a_uu(L[1], a0.y, u0); u0 = dp4a_uu(L[2], a0.z, u0); u0 = dp4a_uu(L[3], a0.w, u0);
      u1 = dp4a_uu(L[0], a1.x, u1); u1 = dp4a_uu(L[1], a1.y, u1); u1 = dp4a_uu(L[2], a1.z, u1); u1 = dp4a_uu(L[3], a1.w, u1);
      u2 = dp4a_us(L[0], a2.x, u2); u2 = dp4a_us(L[1], a2.y, u2); u2 = dp4a_us(L[2], a2.z, u2); u2 = dp4a_us(L[3], a2.w, u2);
      v0 = dp4a_uu(H[0], b0.x, v0); v0 = dp4a_uu(H[1], b0.y, v0); v0 = dp4a_uu(H[2], b0.z, v0); v0 = dp4a_uu(H[3], b0.w, v0);
      v1 = dp4a_uu(H[0], b1.x, v1); v1 = dp4a_uu(H[1], b1.y, v1); v1 = dp4a_uu(H[2], b1.z, v1); v1 = dp4a_uu(H[3], b1.w, v1);
      v2 = dp4a_us(H[0], b2.x, v2); v2 = dp4a_us(H[1], b2.y, v2); v2 = dp4a_us(H[2], b2.z, v2); v2 = dp4a_us(H[3], b2.w, v2);
    }
    // |sum q*X| <= 32*15*(2^22-1) < 2^31: exact in int32
    const int dlo = u2 * 65536 + u1 * 256 + u0;
    const int dhi = v2 * 65536 + v1 * 256 + v0;
    const float* sc = p.scale + size_t(t) * (K / 32);
    const float* sm = p.sum32 + size_t(t) * (K / 32);
    const float dot = float(sc0) * sc[vlo >> 5] * float(dlo) + float(sc1) * sc[vhi >> 5] * float(dhi);
    const float mn = float(m0) * sm[vlo >> 5] + float(m1) * sm[vhi >> 5];
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

// ---- TMA bulk copies (cp.async.bulk, no multicast) and mbarriers --------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Bounded wait for one phase of an mbarrier; false after ~2^22 polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// Q6_K chunk (64 values) of a row held in shared memory
template <int M>
__device__ __forceinline__ void q6k_chunk_smem(const uint8_t* row, int c, int K, const XPlanes& p, float (&acc)[M]) {
  const int b = c >> 2, hh = (c >> 1) & 1, aa = c & 1;
  const uint8_t* blk = row + size_t(b) * Q6K_DEV_BYTES;
  const uint4 l0 = *reinterpret_cast<const uint4*>(blk + 64 * hh + 16 * aa);
  const uint4 l1 = *reinterpret_cast<const uint4*>(blk + 64 * hh + 32 + 16 * aa);
  const uint4 qh = *reinterpret_cast<const uint4*>(blk + 128 + 32 * hh + 16 * aa);
  const uint4 sc = *reinterpret_cast<const uint4*>(blk + 192);
  const uint32_t d = *reinterpret_cast<const unsigned short*>(blk + 208);
  q6k_chunk<M>(l0, l1, qh, sc, d, hh, aa, b * QK_K, K, p, acc);
}

template <int M>
__device__ __forceinline__ void q4k_chunk_smem(const uint8_t* row, int c, int K, const XPlanes& p, float (&acc)[M]) {
  const int b = c >> 2, pr = c & 3;
  const uint8_t* blk = row + size_t(b) * Q4K_BYTES;
  const uint4 hd = *reinterpret_cast<const uint4*>(blk);
  const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * pr);
  const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * pr);
  q4k_chunk<M>(qa, qb, hd, pr, b * QK_K, K, p, acc);
}

__device__ __forceinline__ uint4 lds4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ float ldsf(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// shared-memory addresses of the activation planes
struct XAddr {
  uint32_t l[3], scale, sum32;
};

// One 64-value Q4_K chunk (sub-block pair pr of block b) of four rows held in
// shared memory at row addresses ra[]: the activation limbs of the chunk are
// loaded once and shared by the four rows.
template <int M>
__device__ __forceinline__ void q4k_chunk_rows(const uint32_t (&ra)[ROWS], int c, int K, const XAddr& xa,
                                               float (&acc)[ROWS][M]) {
  const int b = c >> 2, pr = c & 3;
  const int vlo = b * QK_K + 64 * pr, vhi = vlo + 32;
  const bool upper = pr >= 2;
  const int sh = 16 * (pr & 1);
#pragma unroll
  for (int t = 0; t < M; ++t) {
    const uint32_t xo = uint32_t(t * K);
    uint4 xl[3][2], xh[3][2];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      xl[l][0] = lds4(xa.l[l] + xo + vlo);
      xl[l][1] = lds4(xa.l[l] + xo + vlo + 16);
      xh[l][0] = lds4(xa.l[l] + xo + vhi);
      xh[l][1] = lds4(xa.l[l] + xo + vhi + 16);
    }
    const uint32_t so = 4u * uint32_t(t * (K / 32));
    const float s_lo = ldsf(xa.scale + so + 4 * (vlo >> 5)), s_hi = ldsf(xa.scale + so + 4 * (vhi >> 5));
    const float m_lo = ldsf(xa.sum32 + so + 4 * (vlo >> 5)), m_hi = ldsf(xa.sum32 + so + 4 * (vhi >> 5));
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const uint32_t blk = ra[i] + uint32_t(b * Q4K_BYTES);
      const uint4 hd = lds4(blk);
      const uint4 qa = lds4(blk + 16 + 32 * pr);
      const uint4 qb = lds4(blk + 32 + 32 * pr);
      // get_scale_min_k4 (quant.rs:43-53) for sub-blocks 2pr and 2pr+1, branch-free
      const uint32_t y = hd.y >> sh, z = hd.z >> sh, w = hd.w >> sh;
      const uint32_t y0 = y & 0xFF, y1 = (y >> 8) & 0xFF, z0 = z & 0xFF, z1 = (z >> 8) & 0xFF;
      const uint32_t w0 = w & 0xFF, w1 = (w >> 8) & 0xFF;
      const uint32_t sc0 = upper ? ((w0 & 0xF) | ((y0 >> 6) << 4)) : (y0 & 63);
      const uint32_t sc1 = upper ? ((w1 & 0xF) | ((y1 >> 6) << 4)) : (y1 & 63);
      const uint32_t mn0 = upper ? ((w0 >> 4) | ((z0 >> 6) << 4)) : (z0 & 63);
      const uint32_t mn1 = upper ? ((w1 >> 4) | ((z1 >> 6) << 4)) : (z1 & 63);
      const float d = half_bits(hd.x & 0xFFFFu), dmin = half_bits(hd.x >> 16);
      const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      int u0 = 0, u1 = 0, u2 = 0, v0 = 0, v1 = 0, v2 = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t* qq = q + 4 * h;
        const uint32_t L0 = qq[0] & 0x0F0F0F0Fu, L1 = qq[1] & 0x0F0F0F0Fu, L2 = qq[2] & 0x0F0F0F0Fu,
                       L3 = qq[3] & 0x0F0F0F0Fu;
        const uint32_t H0 = (qq[0] >> 4) & 0x0F0F0F0Fu, H1 = (qq[1] >> 4) & 0x0F0F0F0Fu,
                       H2 = (qq[2] >> 4) & 0x0F0F0F0Fu, H3 = (qq[3] >> 4) & 0x0F0F0F0Fu;
        u0 = dp4a_uu(L0, xl[0][h].x, u0); u0 = dp4a_uu(L1, xl[0][h].y, u0); u0 = dp4a_uu(L2, xl[0][h].z, u0); u0 = dp4a_uu(L3, xl[0][h].w, u0);
        u1 = dp4a_uu(L0, xl[1][h].x, u1); u1 = dp4a_uu(L1, xl[1][h].y, u1); u1 = dp4a_uu(L2, xl[1][h].z, u1); u1 = dp4a_uu(L3, xl[1][h].w, u1);
        u2 = dp4a_us(L0, xl[2][h].x, u2); u2 = dp4a_us(L1, xl[2][h].y, u2); u2 = dp4a_us(L2, xl[2][h].z, u2); u2 = dp4a_us(L3, xl[2][h].w, u2);
        v0 = dp4a_uu(H0, xh[0][h].x, v0); v0 = dp4a_uu(H1, xh[0][h].y, v0); v0 = dp4a_uu(H2, xh[0][h].z, v0); v0 = dp4a_uu(H3, xh[0][h].w, v0);
        v1 = dp4a_uu(H0, xh[1][h].x, v1); v1 = dp4a_uu(H1, xh[1][h].y, v1); v1 = dp4a_uu(H2, xh[1][h].z, v1); v1 = dp4a_uu(H3, xh[1][h].w, v1);
        v2 = dp4a_us(H0, xh[2][h].x, v2); v2 = dp4a_us(H1, xh[2][h].y, v2); v2 = dp4a_us(H2, xh[2][h].z, v2); v2 = dp4a_us(H3, xh[2][h].w, v2);
      }
      // |sum q*X| <= 32*15*(2^22-1) < 2^31: exact in int32
      const int dlo = u2 * 65536 + u1 * 256 + u0;
      const int dhi = v2 * 65536 + v1 * 256 + v0;
      const float dot = float(sc0) * s_lo * float(dlo) + float(sc1) * s_hi * float(dhi);
      const float mn = float(mn0) * m_lo + float(mn1) * m_hi;
      acc[i][t] += d * dot - dmin * mn;
    }
  }
}

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

// ---- mma.sync m16n8k16 (fp16 in, fp32 accumulate) for the attention kernels ----
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two 8 x 8 fp16 matrices, transposed: lanes 0-7 give the row addresses of
// matrix 0, lanes 8-15 those of matrix 1
__device__ __forceinline__ void ldsm_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// v = hi + lo with hi = fp16(v), lo = fp16(v - hi), for a pair of values
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = pack_half2(x - hf.x, y - hf.y);
}

// Sampler bookkeeping of generate() (model.rs:1380-1409) after the LM head:
// the argmax token is pushed unless it is EOS (never for the first token), the
// KV position advances, max_tokens / KV capacity end the loop.
__device__ __noinline__ void finish_sample_state(StepState* st, uint32_t* hist, uint32_t* pen_cnt_w) {
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
  hist[st->nhist] = tok;
  st->nhist += 1;
  pen_cnt_w[tok] += 1;
  st->gen += 1;
  if (st->gen >= st->max_gen) st->done = 1;
  else if (st->kv_len + 1 > st->max_seq) {  // the next step's KV append would overflow (kv_cache.rs:48-53)
    st->err = 2;
    st->done = 1;
  }
}

}  // namespace
}  // namespace wcb
