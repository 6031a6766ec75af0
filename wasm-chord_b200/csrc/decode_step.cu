// Persistent decode step: one cooperative launch per generated token.
//
// Every CTA (one per SM) owns a fixed share of the rows of every weight matrix
// of the step; the host lists each CTA's tiles (whole-K row groups) in
// consumption order: layer by layer [q;k;v], o, gate/up, down, then the LM
// head. The tiles stream into a ring of shared-memory slots with cp.async.bulk
// copies completing on mbarriers. A producer warp refills a slot with the tile
// nslots further on as soon as every consumer warp has left it (an "empty"
// mbarrier), so the copies run ahead across phase boundaries: weights never
// depend on the activations.
//
// Activations that cross CTAs travel as (float bits, tag) pairs written with
// one 64-bit store; the tag names the producing phase of this launch
// (epoch * 1024 + phase + 1). A consumer thread spins (bounded) on the
// elements it reads until they carry the expected tag, so a phase starts as
// soon as its own inputs exist: there are no counters, fences or grid-wide
// barriers between phases. Per phase a CTA quantises its input into integer
// limbs (with candle's RMSNorm fused in), then its warps run the dp4a dot
// products of the tiles and the fused epilogues (RoPE + KV append, residual
// add, SwiGLU, LM-head penalty + argmax) independently of one another.
//
// Attention runs on the first n_heads * S CTAs, one per (query head, key
// split): each reads its keys' K / V rows straight from the cache into
// registers (issued before this step's q is polled), keeps a running softmax
// per warp, merges the warps in shared memory and writes its normalised
// partial output with the split's (max, sum). The O-projection phase merges
// the S splits of a head while it builds its input, so no CTA waits for a
// ticket or re-reads partials.
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <vector>

#include "device_common.cuh"
#include "kernels.h"

namespace wcb {

namespace {

constexpr int MK_W = 15;            // consumer warps per CTA
constexpr int MK_T = MK_W * 32;     // consumer threads per CTA
constexpr int MK_THREADS = MK_T + 32;  // + the producer warp (16 warps: 128 registers a thread)
constexpr int MK_MAX_K = MK_MAX_INPUT;  // longest GEMV input (limb planes in shared memory)
constexpr int MK_GPT = 32;          // most groups in one tile
constexpr int MK_ANB = 8;          // attention: cache rows per lane in flight (K and V each)
constexpr int MK_ASMAX = 4;        // most key splits of one query head

// Key splits of one query head: as few as hold every row in flight at once
// (MK_W warps x MK_ANB loads of 512 bytes), at most smax; never an empty split.
__host__ __device__ __forceinline__ int att_splits(int nkeys, int head_dim, int kv_half, int smax) {
  const int cap = MK_W * MK_ANB * (512 / (head_dim * (kv_half ? 2 : 4)));
  const int sp = (nkeys + cap - 1) / cap;
  return sp < 1 ? 1 : (sp > smax ? smax : sp);
}
constexpr uint32_t MK_MBAR_POLLS = 1u << 21;  // ~1 us suspends: about 2 s in all

// barrier of the consumer warps (the producer warp never joins it)
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(MK_T) : "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// (value, tag) pairs: one single-copy-atomic 64-bit access each
__device__ __forceinline__ void st_tag(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void ld_tag2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint32_t tag_of(unsigned long long w) { return uint32_t(w >> 32); }
__device__ __forceinline__ float val_of(unsigned long long w) { return __uint_as_float(uint32_t(w)); }

// Tensor parallelism: words written by other GPUs (peer stores over NVLink) are
// read and written at system scope.
__device__ __forceinline__ unsigned long long ld_sys(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ void st_sys(unsigned long long* p, unsigned long long w) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// first word of rank r's partial sums of the o (kd 0) or down (kd 1) projection of
// `layer` in an exchange buffer; consecutive layers alternate between two copies
__device__ __forceinline__ size_t xslot(const MkArgs& a, int kd, int layer, int r) {
  return a.xofs + ((size_t(kd) * 2 + size_t(layer & 1)) * size_t(a.tp_size) + size_t(r)) * size_t(a.hidden);
}

// Reads N (even; 16-byte aligned start) tagged values, spinning until every
// one carries `tag`; false when the bound expires. skip: read once, no wait.
template <int N>
__device__ __forceinline__ bool poll_tagged(const unsigned long long* p, uint32_t tag, float (&out)[N], bool skip,
                                            unsigned long long limit_ns) {
  unsigned long long w[N];
#pragma unroll
  for (int i = 0; i < N; i += 2) ld_tag2(p + i, w[i], w[i + 1]);
  bool ok = true;
#pragma unroll
  for (int i = 0; i < N; ++i) ok &= tag_of(w[i]) == tag;
  if (!ok && !skip) {
    const unsigned long long t0 = gtime();
    while (true) {
#pragma unroll
      for (int i = 0; i < N; i += 2)
        if (tag_of(w[i]) != tag || tag_of(w[i + 1]) != tag) ld_tag2(p + i, w[i], w[i + 1]);
      ok = true;
#pragma unroll
      for (int i = 0; i < N; ++i) ok &= tag_of(w[i]) == tag;
      if (ok || gtime() - t0 > limit_ns) break;
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = val_of(w[i]);
  return ok || skip;
}

// Bounded wait for one phase of an mbarrier. Each try_wait suspends the
// thread until the phase completes or about a microsecond passes (time hint),
// so waiting warps (the producer most of all) do not take issue slots from
// the computing ones.
__device__ __forceinline__ bool mbar_wait_n(uint64_t* bar, uint32_t parity, uint32_t polls) {
  const uint32_t addr = smem_u32(bar);
  {  // the phase is usually complete already: a non-blocking test first
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  for (uint32_t it = 0; it < polls; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity), "n"(1000)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// Limb planes of one GEMV input (K = 256 * NB values), laid out so that the
// eight lanes of a quarter warp, which read the same 16-value piece of eight
// consecutive blocks, hit consecutive 16-byte words:
//   x[plane 0..2][piece s 0..3][pair pr 0..3] rows of RS bytes, 16 bytes per block
//   (value o of block b: pr = o / 64, s = (o % 64) / 16)
//   scale / sum32[sub-block j 0..7] rows of NBS floats, one per block
// RS = 16 (mod 128) and NBS = 4 (mod 16) spread the writers over the banks.
struct Planes {
  uint32_t x;      // shared address of the limb rows
  uint32_t scale;  // shared address of the scales
  uint32_t sum32;
  int RS, NBS;
};

__host__ __device__ __forceinline__ int planes_rs(int NB) { return ((NB * 16 + 111) / 128) * 128 + 16; }
__host__ __device__ __forceinline__ int planes_nbs(int NB) { return ((NB + 11) / 16) * 16 + 4; }
__host__ __device__ __forceinline__ size_t planes_bytes(int K) {
  const int NB = K / QK_K;
  return size_t(48) * planes_rs(NB) + 2 * sizeof(float) * 8 * size_t(planes_nbs(NB));
}

__device__ __forceinline__ Planes planes_at(uint32_t base, int K) {
  Planes p;
  const int NB = K / QK_K;
  p.RS = planes_rs(NB);
  p.NBS = planes_nbs(NB);
  p.x = base;
  p.scale = base + 48u * uint32_t(p.RS);
  p.sum32 = p.scale + 4u * 8u * uint32_t(p.NBS);
  return p;
}

__device__ __forceinline__ void sts2(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void stsf(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Quantises the 8 values v[] at input index k (k % 8 == 0) into the planes.
// Four consecutive lanes hold one 32-value group: X = rint(x / s) with
// s = max|x| / (2^22 - 1), split into bytes X = 65536 x2 + 256 x1 + x0.
__device__ __forceinline__ void quant8_planes(const float (&v)[8], int k, const Planes& p) {
  float amax = 0.0f;
  bool bad = false;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    amax = fmaxf(amax, fabsf(v[e]));
    bad |= !(fabsf(v[e]) <= FLT_MAX);  // NaN / inf
  }
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
  uint32_t w[3][2];
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
    w[0][h] = b0;
    w[1][h] = b1;
    w[2][h] = b2;
  }
  const int b = k >> 8, o = k & 255, pr = o >> 6, sp = (o >> 4) & 3, half = (o >> 3) & 1;
#pragma unroll
  for (int pl = 0; pl < 3; ++pl)
    sts2(p.x + uint32_t(((pl * 4 + sp) * 4 + pr) * p.RS + b * 16 + half * 8), w[pl][0], w[pl][1]);
  sx += __shfl_xor_sync(0xffffffffu, sx, 1);
  sx += __shfl_xor_sync(0xffffffffu, sx, 2);  // |sum X| <= 32 * (2^22 - 1) < 2^31
  if ((threadIdx.x & 3) == 0) {
    const uint32_t j = uint32_t(o >> 5);
    stsf(p.scale + 4u * (j * uint32_t(p.NBS) + uint32_t(b)), s);
    stsf(p.sum32 + 4u * (j * uint32_t(p.NBS) + uint32_t(b)), s * float(sx));
  }
}

// Dot products of one (4-row group, 64-value chunk) unit of a Q4_K tile for
// the lane's chunk: pair pr = lane / 8 of block b. The same arithmetic as the
// per-op GEMV: exact integer dp4a over the limbs, one scale per sub-block
// (dequantize_q4_k, quant.rs:58-115, folded into the sum). Values 0-15 and
// 16-31 of the two sub-blocks are taken in two passes to keep few limbs live.
__device__ __forceinline__ void q4k_unit(const uint32_t (&ra)[ROWS], int b, int pr, const Planes& P,
                                         float (&acc)[ROWS]) {
  int du[ROWS][6];
#pragma unroll
  for (int i = 0; i < ROWS; ++i)
#pragma unroll
    for (int j = 0; j < 6; ++j) du[i][j] = 0;
  const uint32_t step = uint32_t(4 * P.RS);  // next piece s
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint4 xl[3], xh[3];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      const uint32_t r0 = P.x + uint32_t(((l * 4) * 4 + pr) * P.RS + b * 16);
      xl[l] = lds4(r0 + uint32_t(h) * step);        // sub-block 2pr, values 16h..16h+15
      xh[l] = lds4(r0 + uint32_t(2 + h) * step);    // sub-block 2pr+1, same values
    }
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const uint4 qv = lds4(ra[i] + uint32_t(b * Q4K_BYTES + 16 + 32 * pr + 16 * h));
      const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
      const uint32_t xs[3][4] = {{xl[0].x, xl[0].y, xl[0].z, xl[0].w},
                                 {xl[1].x, xl[1].y, xl[1].z, xl[1].w},
                                 {xl[2].x, xl[2].y, xl[2].z, xl[2].w}};
      const uint32_t ys[3][4] = {{xh[0].x, xh[0].y, xh[0].z, xh[0].w},
                                 {xh[1].x, xh[1].y, xh[1].z, xh[1].w},
                                 {xh[2].x, xh[2].y, xh[2].z, xh[2].w}};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t lo = q[e] & 0x0F0F0F0Fu, hi = (q[e] >> 4) & 0x0F0F0F0Fu;
        du[i][0] = dp4a_uu(lo, xs[0][e], du[i][0]);
        du[i][1] = dp4a_uu(lo, xs[1][e], du[i][1]);
        du[i][2] = dp4a_us(lo, xs[2][e], du[i][2]);
        du[i][3] = dp4a_uu(hi, ys[0][e], du[i][3]);
        du[i][4] = dp4a_uu(hi, ys[1][e], du[i][4]);
        du[i][5] = dp4a_us(hi, ys[2][e], du[i][5]);
      }
    }
  }
  const uint32_t jl = uint32_t(2 * pr), jh = jl + 1;
  const float s_lo = ldsf(P.scale + 4u * (jl * uint32_t(P.NBS) + uint32_t(b)));
  const float s_hi = ldsf(P.scale + 4u * (jh * uint32_t(P.NBS) + uint32_t(b)));
  const float m_lo = ldsf(P.sum32 + 4u * (jl * uint32_t(P.NBS) + uint32_t(b)));
  const float m_hi = ldsf(P.sum32 + 4u * (jh * uint32_t(P.NBS) + uint32_t(b)));
  const bool upper = pr >= 2;
  const int sh = 16 * (pr & 1);
#pragma unroll
  for (int i = 0; i < ROWS; ++i) {
    const uint4 hd = lds4(ra[i] + uint32_t(b * Q4K_BYTES));
    // get_scale_min_k4 (quant.rs:43-53) for sub-blocks 2pr and 2pr+1, branch-free
    const uint32_t y = hd.y >> sh, z = hd.z >> sh, w = hd.w >> sh;
    const uint32_t y0 = y & 0xFF, y1 = (y >> 8) & 0xFF, z0 = z & 0xFF, z1 = (z >> 8) & 0xFF;
    const uint32_t w0 = w & 0xFF, w1 = (w >> 8) & 0xFF;
    const uint32_t sc0 = upper ? ((w0 & 0xF) | ((y0 >> 6) << 4)) : (y0 & 63);
    const uint32_t sc1 = upper ? ((w1 & 0xF) | ((y1 >> 6) << 4)) : (y1 & 63);
    const uint32_t mn0 = upper ? ((w0 >> 4) | ((z0 >> 6) << 4)) : (z0 & 63);
    const uint32_t mn1 = upper ? ((w1 >> 4) | ((z1 >> 6) << 4)) : (z1 & 63);
    const float d = half_bits(hd.x & 0xFFFFu), dmin = half_bits(hd.x >> 16);
    // |sum q*X| <= 32*15*(2^22-1) < 2^31: exact in int32
    const int dlo = du[i][2] * 65536 + du[i][1] * 256 + du[i][0];
    const int dhi = du[i][5] * 65536 + du[i][4] * 256 + du[i][3];
    const float dot = float(sc0) * s_lo * float(dlo) + float(sc1) * s_hi * float(dhi);
    const float mn = float(mn0) * m_lo + float(mn1) * m_hi;
    acc[i] += d * dot - dmin * mn;
  }
}

// Q6_K (224-byte padded blocks): chunk q = lane / 8 of block b = half hh = q/2,
// 16-column slice aa = q%2 of the 32-wide interleave (quant.rs:206-261): four
// 16-value pieces k = 0..3 at values 128 hh + 32 k + 16 aa; pieces k and k+2
// share the low / high nibbles of one ql word set and are taken together.
__device__ __forceinline__ void q6k_unit(const uint32_t (&ra)[ROWS], int b, int q, const Planes& P,
                                         float (&acc)[ROWS]) {
  const int hh = q >> 1, aa = q & 1;
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    uint4 xa[3], xb[3];
    float sa, sb;
    {
      const int ka = kk, kb = kk + 2;  // pieces: pr = 2hh + (k >> 1), s = 2(k & 1) + aa
      const int pra = 2 * hh + (ka >> 1), spa = 2 * (ka & 1) + aa;
      const int prb = 2 * hh + (kb >> 1), spb = 2 * (kb & 1) + aa;
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        xa[l] = lds4(P.x + uint32_t(((l * 4 + spa) * 4 + pra) * P.RS + b * 16));
        xb[l] = lds4(P.x + uint32_t(((l * 4 + spb) * 4 + prb) * P.RS + b * 16));
      }
      sa = ldsf(P.scale + 4u * (uint32_t(4 * hh + ka) * uint32_t(P.NBS) + uint32_t(b)));
      sb = ldsf(P.scale + 4u * (uint32_t(4 * hh + kb) * uint32_t(P.NBS) + uint32_t(b)));
    }
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const uint32_t blk = ra[i] + uint32_t(b * Q6K_DEV_BYTES);
      const uint4 ql = lds4(blk + 64 * hh + 32 * kk + 16 * aa);
      const uint4 qh = lds4(blk + 128 + 32 * hh + 16 * aa);
      const uint4 scw = lds4(blk + 192);
      const float d = half_bits(lds4(blk + 208).x & 0xFFFFu);
      const uint32_t L[4] = {ql.x, ql.y, ql.z, ql.w};
      const uint32_t Q[4] = {qh.x, qh.y, qh.z, qh.w};
      const uint32_t S[4] = {scw.x, scw.y, scw.z, scw.w};
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int k = kk + 2 * t;
        const uint4* xx = t == 0 ? xa : xb;
        uint32_t sq[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t nib = t == 0 ? (L[e] & 0x0F0F0F0Fu) : ((L[e] >> 4) & 0x0F0F0F0Fu);
          const uint32_t hb = ((Q[e] >> (2 * k)) & 0x03030303u) << 4;
          sq[e] = __vsub4(nib | hb, 0x20202020u);  // signed bytes q - 32
        }
        const int sidx = 8 * hh + aa + 2 * k;
        const int scv = int(int8_t(byte_of(S[sidx >> 2], sidx & 3)));
        int u0 = 0, u1 = 0, u2 = 0;
        u0 = dp4a_su(sq[0], xx[0].x, u0); u0 = dp4a_su(sq[1], xx[0].y, u0); u0 = dp4a_su(sq[2], xx[0].z, u0); u0 = dp4a_su(sq[3], xx[0].w, u0);
        u1 = dp4a_su(sq[0], xx[1].x, u1); u1 = dp4a_su(sq[1], xx[1].y, u1); u1 = dp4a_su(sq[2], xx[1].z, u1); u1 = dp4a_su(sq[3], xx[1].w, u1);
        u2 = dp4a_ss(sq[0], xx[2].x, u2); u2 = dp4a_ss(sq[1], xx[2].y, u2); u2 = dp4a_ss(sq[2], xx[2].z, u2); u2 = dp4a_ss(sq[3], xx[2].w, u2);
        const float fd = float(u2) * 65536.0f + float(u1) * 256.0f + float(u0);
        acc[i] += d * float(scv) * (t == 0 ? sa : sb) * fd;
      }
    }
  }
}

// Shared-memory carve-up of one CTA (sizes in MkArgs, set on the host):
//   [slots]  nslots x slot_bytes weight tiles
//   [region] limb planes (GEMV phases) or attention staging
//   [parts]  the part list; [share] this CTA's groups [g0, g1) of each part (g0 | g1 << 16)
//   [rsd]    residual rows of this CTA's o / down share
//   [rope]   cos, sin of the step's position (head_dim / 2 each)
//   [pen]    penalty counts of this CTA's LM-head rows
//   [misc]   red[64] floats, part[part_floats] floats, flags[8]
//   [bars]   full[nslots]
struct MkSmem {
  uint8_t* slots;
  uint8_t* region;
  MkPart* parts;
  uint32_t* share;
  float* rsd;
  float* rcos;
  float* rsin;
  uint32_t* pen;
  float* red;
  float* part;  // [groups of the CTA's share][chunks][ROWS] partial sums of a split part's 8-block chunks
  int* flags;  // [0] abort, [1] attention ticket result, [2] NaN seen
  uint64_t* full;
  uint64_t* empty;
};

// Byte offsets of the carve-up (host and device agree on them).
struct MkOffsets {
  size_t region, parts, share, rsd, rcos, rsin, pen, red, part, flags, full, empty, total;
};

__host__ __device__ __forceinline__ MkOffsets mk_offsets(const MkArgs& a) {
  MkOffsets o;
  size_t x = size_t(a.nslots) * a.slot_bytes;
  o.region = x;
  x += a.region_bytes;
  o.parts = x;
  x += sizeof(MkPart) * size_t(a.nparts);
  o.share = x;
  x += sizeof(uint32_t) * size_t(a.nparts);
  x = (x + 15) / 16 * 16;  // red is read as 64-bit words: keep what follows 16-byte aligned
  o.rsd = x;
  x += sizeof(float) * size_t(a.res_rows);
  o.rcos = x;
  x += sizeof(float) * size_t(a.head_dim / 2);
  o.rsin = x;
  x += sizeof(float) * size_t(a.head_dim / 2);
  o.pen = x;
  x += sizeof(uint32_t) * size_t(a.lm_rows);
  o.red = x;
  x += sizeof(float) * 64;
  o.part = x;
  x += sizeof(float) * size_t(a.part_floats);
  o.flags = x;
  x += sizeof(int) * 8;
  x = (x + 7) / 8 * 8;
  o.full = x;
  x += sizeof(uint64_t) * size_t(a.nslots);
  o.empty = x;
  x += sizeof(uint64_t) * size_t(a.nslots);
  o.total = x;
  return o;
}

__device__ __forceinline__ MkSmem mk_carve(const MkArgs& a, uint8_t* b) {
  const MkOffsets o = mk_offsets(a);
  MkSmem s;
  s.slots = b;
  s.region = b + o.region;
  s.parts = reinterpret_cast<MkPart*>(b + o.parts);
  s.share = reinterpret_cast<uint32_t*>(b + o.share);
  s.rsd = reinterpret_cast<float*>(b + o.rsd);
  s.rcos = reinterpret_cast<float*>(b + o.rcos);
  s.rsin = reinterpret_cast<float*>(b + o.rsin);
  s.pen = reinterpret_cast<uint32_t*>(b + o.pen);
  s.red = reinterpret_cast<float*>(b + o.red);
  s.part = reinterpret_cast<float*>(b + o.part);
  s.flags = reinterpret_cast<int*>(b + o.flags);
  s.full = reinterpret_cast<uint64_t*>(b + o.full);
  s.empty = reinterpret_cast<uint64_t*>(b + o.empty);
  return s;
}

// Groups [g0, g1) of a part owned by CTA c of n.
__host__ __device__ __forceinline__ void cta_share(int ngroups, int c, int n, int& g0, int& g1) {
  if (ngroups < 65536 && c < 65536) {  // the products fit 32 bits: no 64-bit division
    g0 = int(unsigned(c) * unsigned(ngroups) / unsigned(n));
    g1 = int(unsigned(c + 1) * unsigned(ngroups) / unsigned(n));
    return;
  }
  g0 = int((long long)c * ngroups / n);
  g1 = int((long long)(c + 1) * ngroups / n);
}

// Bulk copies of one tile (ng whole-K groups from group g) into dst.
__device__ void issue_tile(const MkPart* Pp, const MkTile& T, uint8_t* dst, uint64_t* bar) {
  const int kind = Pp->kind, nseg = Pp->nseg;
  const size_t row_bytes = size_t(Pp->K / QK_K) * dev_block_bytes(Pp->dtype);
  const uint32_t bytes = uint32_t(4u * T.ng * row_bytes);
  mbar_expect_tx(bar, bytes);
  if (kind == MK_GU) {
    const uint32_t half = bytes / 2;
    bulk_g2s(dst, Pp->w[0] + size_t(2 * T.g) * row_bytes, half, bar);
    bulk_g2s(dst + half, Pp->w[1] + size_t(2 * T.g) * row_bytes, half, bar);
    return;
  }
  int r0 = 4 * T.g;
  const int r1 = 4 * (T.g + T.ng);
  if (Pp->row_stride) {  // a K-chain part: each row's slice of the input is its own copy
    for (int r = r0; r < r1; ++r)
      bulk_g2s(dst + size_t(r - r0) * row_bytes, Pp->w[0] + size_t(r) * size_t(Pp->row_stride), uint32_t(row_bytes),
               bar);
    return;
  }
  int base = 0;
  for (int sg = 0; sg < 3 && r0 < r1; ++sg) {
    const int s1 = sg == 0 ? Pp->rows0 : sg == 1 && nseg > 1 ? base + Pp->rows1 : r1;
    if (r0 < s1) {
      const int e = min(r1, s1);
      const uint32_t nb = uint32_t(size_t(e - r0) * row_bytes);
      bulk_g2s(dst, Pp->w[sg] + size_t(r0 - base) * row_bytes, nb, bar);
      dst += nb;
      r0 = e;
    }
    base = s1;
  }
}

// Cursor over one CTA's tiles in consumption order: part by part, gpt groups of
// the CTA's share of each part at a time (attention parts have no weights).
struct TileCursor {
  int pi, g, g1;  // part, next group, end of the CTA's share of the part
};

// share: this CTA's group ranges of the parts (null: computed)
__device__ __forceinline__ bool next_tile(const MkPart* parts, int nparts, TileCursor& t, MkTile& T,
                                          const uint32_t* share) {
  while (t.g >= t.g1) {
    if (++t.pi >= nparts) return false;
    if (parts[t.pi].kind == MK_ATT) {
      t.g = t.g1 = 0;
      continue;
    }
    if (share) {
      const uint32_t r = share[t.pi];
      t.g = int(r & 0xFFFFu);
      t.g1 = int(r >> 16);
    } else {
      cta_share(parts[t.pi].ngroups, blockIdx.x, gridDim.x, t.g, t.g1);
    }
  }
  const int gpt = parts[t.pi].gpt;
  T.g = uint16_t(t.g);
  T.part = uint16_t(t.pi);
  T.ng = uint8_t(min(gpt, t.g1 - t.g));
  t.g += gpt;
  return true;
}

// Per-launch values every thread keeps.
struct Ctx {
  uint32_t tag0;  // epoch * 1024 + 1: tag of phase p is tag0 + p
  int position, kv_len;
  const float* x0;  // layer-0 input: the embedding row of the step's token
  int R0;           // first row of this CTA's o / down share (residual stash)
  int g0;           // first group of this CTA in the current part
  float rm;  // 1 / RMSNorm divisor of the current phase's input (1 without norm)
  unsigned long long best;
  int nan;
  int S;                         // key splits of each query head's attention (att_splits)
  unsigned long long wait_ns;    // bound of every spin wait on another CTA's data
};

__device__ __forceinline__ float pick4(const float (&v)[ROWS], int i) {
  return i == 0 ? v[0] : i == 1 ? v[1] : i == 2 ? v[2] : v[3];
}

// Fused epilogue of group g (all lanes hold the four row sums v[]; lane i < 4
// handles row i). gi: stash index of the group's first row.
__device__ __forceinline__ void group_epilogue(const MkArgs& a, const MkPart& P, int g, const float (&v)[ROWS],
                                               Ctx& c, const MkSmem& sm) {
  const int lane = threadIdx.x & 31;
  if (lane >= ROWS || P.phase == a.drop_phase) return;  // drop_phase: a test withholds this phase's outputs
  const int i = lane;
  const int gi = ROWS * (g - c.g0);
  const float vi = pick4(v, i);
  const uint32_t tag = c.tag0 + uint32_t(P.phase);
  if (P.kind == MK_QKV) {
    const int hid = a.qdim, hd = a.head_dim, kvd = a.n_kv * a.head_dim;
    const int vr = P.row_offset + ROWS * g + i;
    const size_t esz = a.kv_half ? 2 : 4;
    if (vr < hid + kvd) {
      if ((i & 1) == 0) {  // RoPE on (2j, 2j+1) pairs (attention.rs:230-262), table values
        const float x0 = vi, x1 = pick4(v, i + 1);
        const int pi2 = ((vr < hid ? vr : vr - hid) % hd) >> 1;  // rotation pair of the row
        const float cs = sm.rcos[pi2], sn = sm.rsin[pi2];
        const float n0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        const float n1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        if (vr < hid) {
          st_tag(a.q + vr, n0, tag);
          st_tag(a.q + vr + 1, n1, tag);
        } else {
          const int col = vr - hid;
          const size_t off = size_t(P.phase / 5) * a.kv_layer_elems + (size_t(col / hd) * a.max_seq + c.kv_len) * hd +
                             col % hd;
          if (a.kv_half) {
            reinterpret_cast<__half*>(a.kcache)[off] = __float2half_rn(n0);
            reinterpret_cast<__half*>(a.kcache)[off + 1] = __float2half_rn(n1);
          } else {
            reinterpret_cast<float*>(a.kcache)[off] = n0;
            reinterpret_cast<float*>(a.kcache)[off + 1] = n1;
          }
          // attention reads this step's row through the tagged copy, rounded like the cache
          const float k0 = a.kv_half ? __half2float(__float2half_rn(n0)) : n0;
          const float k1 = a.kv_half ? __half2float(__float2half_rn(n1)) : n1;
          st_tag(a.knew + col, k0, tag);
          st_tag(a.knew + col + 1, k1, tag);
        }
      }
    } else {
      const int col = vr - hid - kvd;
      const size_t off = size_t(P.phase / 5) * a.kv_layer_elems + (size_t(col / hd) * a.max_seq + c.kv_len) * hd +
                         col % hd;
      float vv = vi;
      if (a.kv_half) {
        reinterpret_cast<__half*>(a.vcache)[off] = __float2half_rn(vv);
        vv = __half2float(__float2half_rn(vv));
      } else {
        reinterpret_cast<float*>(a.vcache)[off] = vv;
      }
      st_tag(a.vnew + col, vv, tag);
    }
    (void)esz;
  } else if (P.kind == MK_O || P.kind == MK_D) {  // attention / FFN out + residual (layer.rs:68, :86)
    const int r = ROWS * g + i;
    if (a.tp_size > 1) {
      // this rank's partial sum (its heads / FFN rows) to slot tp_rank of every rank;
      // the owner of row r adds the residual when the next phase builds its input
      const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(vi);
      const size_t off = xslot(a, P.kind == MK_D, P.phase / 5, a.tp_rank) + size_t(r);
      for (int rr = 0; rr < a.tp_size; ++rr) st_sys(a.peers[rr] + off, w);
    } else {
      st_tag((P.kind == MK_O ? a.xb : a.xa) + r, __fadd_rn(sm.rsd[r - c.R0], vi), tag);
    }
  } else if (P.kind == MK_GU) {  // ffn.rs:90-94: silu(g) * u
    if (i < 2) {
      const float gv = vi, uv = pick4(v, i + 2);
      const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
      st_tag(a.act + 2 * g + i, __fmul_rn(__fmul_rn(gv, sig), uv), tag);
    }
  } else {  // MK_LM (rows of this rank's vocabulary slice)
    const int n = ROWS * g + i;
    a.logits[n] = vi;
    if (a.gen_mode == 1) {
      float pv = vi;
      if (a.rep != 1.0f) {  // apply_repetition_penalty: once per occurrence (sampling.rs:86-103)
        const uint32_t cnt = sm.pen[gi + i];
        for (uint32_t k = 0; k < cnt; ++k) pv = pv > 0.0f ? __fdiv_rn(pv, a.rep) : __fmul_rn(pv, a.rep);
      }
      if (pv != pv) c.nan = 1;
      else {
        const unsigned long long key =
            (static_cast<unsigned long long>(order_key(pv)) << 32) | uint32_t(a.vocab_off + n);
        c.best = key > c.best ? key : c.best;
      }
    }
  }
}

// The O phase's inputs k .. k + 7 (one head h = k / head_dim) from S > 1 key
// splits: sum_s e^(m_s - M) l_s o_s / sum_s e^(m_s - M) l_s with M = max m_s,
// o_s the split's normalised output.
__device__ __forceinline__ bool poll_att_merged(const MkArgs& a, int k, int S, uint32_t tag, float (&v)[8], bool skip,
                                                unsigned long long limit_ns) {
  const int h = k / a.head_dim;
  bool ok = true;
  float M = -INFINITY, L = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = 0.0f;
  for (int s = 0; s < S; ++s) {
    float o[8], ml[2];
    ok &= poll_tagged<2>(a.attml + (size_t(s) * a.n_heads + h) * 2, tag, ml, skip, limit_ns);
    ok &= poll_tagged<8>(a.att + size_t(s) * a.hidden + k, tag, o, skip, limit_ns);
    const float mn = fmaxf(M, ml[0]);
    const float c0 = M == -INFINITY ? 0.0f : expf(M - mn), c1 = expf(ml[0] - mn) * ml[1];
    L = L * c0 + c1;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = v[e] * c0 + o[e] * c1;
    M = mn;
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] *= inv;
  return ok;
}

// Tensor parallelism: this CTA's rows of the residual stream are the previous
// residual (stashed in rsd) plus every rank's partial sum of the o (kd 0) or down
// (kd 1) projection of phase `dep`, added in rank order as the per-op exchange does
// (the same sum on every rank); they are published for all CTAs under the
// producing phase's tag. Kept out of line (arguments by value): it runs once per
// phase and would add to the register pressure of the input build. xr: rank 0's
// partial sums in this rank's exchange buffer. False when a wait expired.
__device__ __noinline__ bool tp_residual_rows(const unsigned long long* xr, unsigned long long* dst, int hidden,
                                              int tp, uint32_t tag, int R0, const float* rsd, bool skip,
                                              unsigned long long wait_ns, StepState* st) {
  int h0, h1;
  cta_share(hidden / ROWS, blockIdx.x, gridDim.x, h0, h1);
  bool ok = true;
  for (int j = ROWS * h0 + int(threadIdx.x); j < ROWS * h1; j += MK_T) {
    float sum = 0.0f;
    for (int r = 0; r < tp; ++r) {
      const unsigned long long* p = xr + size_t(r) * hidden + j;
      unsigned long long wv = ld_sys(p);
      if (tag_of(wv) != tag && !skip) {  // bounded: a rank that stopped ends the step with an error
        const unsigned long long t0 = gtime();
        while (tag_of(wv) != tag) {
          if (gtime() - t0 > wait_ns) {
            atomicOr(&st->err, 16);
            ok = false;
            break;
          }
          wv = ld_sys(p);
        }
      }
      sum = __fadd_rn(sum, val_of(wv));
    }
    st_tag(dst + j, __fadd_rn(rsd[j - R0], sum), tag);
  }
  return ok;
}

// Input planes of the phase starting at part pi (R rounds of MK_T * 8 values).
// With P.norm the planes hold x * w and each warp leaves its share of sum(x^2)
// in red[]: candle's rms_norm (candle_tensor_backend.rs:30-57), x / m * w with
// m = sqrt(sum(x^2)/K + eps), is applied as W(x * w) / m after the dot
// products, so quantisation does not wait for the reduction.
// Also stages what the phase's epilogues read: the residual rows of this
// CTA's o / down share, the RoPE cos / sin of its q / k rows and the penalty
// counts of its LM-head rows. Ends with every thread's planes written (the
// caller's barrier publishes them). Returns false when a wait expired.
template <int R>
__device__ bool build_input(const MkArgs& a, int pi, const MkPart& P, const Ctx& c, const MkSmem& sm, bool skip) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = P.K;
  const Planes pl = planes_at(smem_u32(sm.region), K);
  // staged epilogue inputs that do not depend on this phase's input (the RoPE
  // table of the step's position is staged once per launch)
  if (P.kind == MK_LM) {
    int g0, g1;
    cta_share(P.ngroups, blockIdx.x, gridDim.x, g0, g1);
    for (int r = tid; r < ROWS * (g1 - g0); r += MK_T) sm.pen[r] = __ldg(a.pen_cnt + a.vocab_off + ROWS * g0 + r);
  }
  const unsigned long long* src = nullptr;
  const float* plain = nullptr;
  switch (P.kind) {
    case MK_QKV:
      if (P.dep < 0) plain = c.x0;
      else src = a.xa;
      break;
    case MK_O: src = a.att; break;
    case MK_GU: src = a.xb; break;
    case MK_D: src = a.act + P.kofs; break;
    default: src = a.xa; break;  // MK_LM
  }
  const bool stash = P.kind == MK_QKV || P.kind == MK_GU;  // residual of the o / down share
  const int R1 = c.R0 + a.res_rows;
  const uint32_t tag = c.tag0 + uint32_t(P.dep);
  bool ok = true;
  if (a.tp_size > 1 && (P.kind == MK_GU || P.kind == MK_LM || (P.kind == MK_QKV && P.dep >= 0)))
    ok = tp_residual_rows(a.peers[a.tp_rank] + xslot(a, P.kind == MK_GU ? 0 : 1, P.dep / 5, 0),
                          P.kind == MK_GU ? a.xb : a.xa, a.hidden, a.tp_size, tag, c.R0, sm.rsd, skip, c.wait_ns,
                          a.st);
  float v[R][8], w[R][8];
  uint32_t pending = 0;  // bit 4 r + q: value pair q of round r still carries an older tag
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int k = r * MK_T * 8 + tid * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[r][e] = w[r][e] = 0.0f;
    if (k < K) {
      if (P.norm) {
        const float4 w0 = __ldg(reinterpret_cast<const float4*>(P.norm + k));
        const float4 w1 = __ldg(reinterpret_cast<const float4*>(P.norm + k + 4));
        w[r][0] = w0.x; w[r][1] = w0.y; w[r][2] = w0.z; w[r][3] = w0.w;
        w[r][4] = w1.x; w[r][5] = w1.y; w[r][6] = w1.z; w[r][7] = w1.w;
      }
      if (plain) {
        const float4 x0 = __ldg(reinterpret_cast<const float4*>(plain + k));
        const float4 x1 = __ldg(reinterpret_cast<const float4*>(plain + k + 4));
        v[r][0] = x0.x; v[r][1] = x0.y; v[r][2] = x0.z; v[r][3] = x0.w;
        v[r][4] = x1.x; v[r][5] = x1.y; v[r][6] = x1.z; v[r][7] = x1.w;
      } else if (P.kind == MK_O && c.S > 1) {
        ok &= poll_att_merged(a, k, c.S, tag, v[r], skip, c.wait_ns);
      } else {  // first reads of every round issued together; the pairs not there yet are re-read below
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          unsigned long long w0, w1;
          ld_tag2(src + k + 2 * q2, w0, w1);
          v[r][2 * q2] = val_of(w0);
          v[r][2 * q2 + 1] = val_of(w1);
          if (tag_of(w0) != tag || tag_of(w1) != tag) pending |= 1u << (4 * r + q2);
        }
      }
    }
  }
  if (pending && !skip) {  // bounded wait for the values of later producers
    const unsigned long long t0 = gtime();
    while (true) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          if (!(pending & (1u << (4 * r + q2)))) continue;
          unsigned long long w0, w1;
          ld_tag2(src + r * MK_T * 8 + tid * 8 + 2 * q2, w0, w1);
          if (tag_of(w0) == tag && tag_of(w1) == tag) {
            v[r][2 * q2] = val_of(w0);
            v[r][2 * q2 + 1] = val_of(w1);
            pending &= ~(1u << (4 * r + q2));
          }
        }
      if (!pending) break;
      if (gtime() - t0 > c.wait_ns) {
        ok = false;
        break;
      }
    }
  }
  if (stash)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int k = r * MK_T * 8 + tid * 8;
      if (k < K)
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (k + e >= c.R0 && k + e < R1) sm.rsd[k + e - c.R0] = v[r][e];
    }
  if (P.norm) {  // this warp's share of sum(x^2), summed over the warps after the caller's barrier
    float ss = 0.0f;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(v[r][e], v[r][e]));
    ss = warp_sum(ss);
    if (lane == 0) sm.red[warp] = ss;
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int k = r * MK_T * 8 + tid * 8;
    if (k < K) {  // whole warps are in or out (K is a multiple of 256)
      float e8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) e8[e] = P.norm ? __fmul_rn(v[r][e], w[r][e]) : v[r][e];
      quant8_planes(e8, k, pl);
    }
  }
  return ok;
}

// 16 bytes of a cache row as floats: 4 f32 or 8 f16 values
__device__ __forceinline__ void kv_unpack(const uint4& u, float (&f)[4]) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}
__device__ __forceinline__ void kv_unpack(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Attention of one (query head h, key split s of S) item of a decode step over
// layer `layer`'s cache: keys [j0, j1) of the keys the query at `position`
// sees (attention.rs:332-435: scores (q.k) * scale, causal limit j <= position,
// softmax, weighted sum of V; repeat_kv, attention.rs:297-322, reads KV head
// h / n_rep). Keys written by earlier steps come from the cache, this step's
// key (slot kv_len) from the tagged copy of the QKV phase. Each lane holds 16
// bytes of a row, LPK lanes one row; a warp takes every (MK_W * KPL)-th row
// from row j0 + warp * KPL, MK_ANB rows per lane in flight (the first ones
// requested before q is polled, the rest prefetched into L2 meanwhile), and
// keeps a running softmax; the warps are merged in shared memory. The output
// is this split's normalised partial (S == 1: the attention output) and, with
// S > 1, the split's maximum and sum for the merge in the O phase.
template <int HD, typename KT>
__device__ __forceinline__ void mk_attention(const MkArgs& a, const MkSmem& sm, int layer, int h, int s, int S,
                                             int j0, int j1, const Ctx& c, uint32_t qtag, uint32_t otag) {
  constexpr int EPL = 16 / int(sizeof(KT));  // values per lane of a row
  constexpr int LPK = HD / EPL;               // lanes per row
  constexpr int KPL = 32 / LPK;               // rows per warp-wide load
  constexpr int NB = MK_ANB;                  // rows per lane in flight
  constexpr int STRIDE = MK_W * KPL;          // rows between a lane's consecutive rows
  constexpr int RW = HD * int(sizeof(KT)) / 16;  // 16-byte words per row
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = lane / LPK, li = lane - sub * LPK;
  const int kh = h / (a.n_heads / a.n_kv);
  const size_t lofs = size_t(layer) * a.kv_layer_elems + size_t(kh) * a.max_seq * HD + size_t(li) * EPL;
  const uint4* Kp = reinterpret_cast<const uint4*>(reinterpret_cast<const KT*>(a.kcache) + lofs);
  const uint4* Vp = reinterpret_cast<const uint4*>(reinterpret_cast<const KT*>(a.vcache) + lofs);
  const int old_end = min(j1, c.kv_len);            // rows written by earlier steps
  const bool has_new = c.kv_len >= j0 && c.kv_len < j1;  // this step's row
  const bool new_here = has_new && warp == MK_W - 1;     // the warp that takes it
  const int wb = j0 + warp * KPL;                   // this warp's first row (warp-uniform)
  float* wm = reinterpret_cast<float*>(sm.region);  // [MK_W] maxima, [MK_W] sums
  float* wl = wm + MK_W;
  float* wa = wl + MK_W;                            // [MK_W][HD] outputs
  float* knew = wa + MK_W * HD;                     // [HD] this step's K row
  float* vnew = knew + HD;                          // [HD] this step's V row
  // the first rows of this lane go to registers, the rest into L2, before q is
  // polled: the rows do not depend on this step. Rows past the end re-read the
  // last row and are masked out.
  uint4 kr[NB], vr[NB];
  const int last = max(old_end - 1, 0);
#pragma unroll
  for (int e = 0; e < NB; ++e) {
    const size_t jj = size_t(min(wb + sub + e * STRIDE, last));
    kr[e] = __ldcg(Kp + jj * RW);
    vr[e] = __ldcg(Vp + jj * RW);
  }
  for (int jj = wb + sub + NB * STRIDE; jj < old_end; jj += STRIDE) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(Kp + size_t(jj) * RW));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(Vp + size_t(jj) * RW));
  }
  float q[EPL];
  if (!poll_tagged<EPL>(a.q + size_t(h) * HD + size_t(li) * EPL, qtag, q, false, c.wait_ns)) {
    sm.flags[0] = 1;
    atomicOr(&a.st->err, 8);
  }
  if (new_here && sub == 0) {  // this step's K and V rows, from the tagged copies of the QKV phase
    bool ok;
    {
      float f[EPL];
      ok = poll_tagged<EPL>(a.knew + size_t(kh) * HD + size_t(li) * EPL, qtag, f, false, c.wait_ns);
#pragma unroll
      for (int i = 0; i < EPL; ++i) knew[li * EPL + i] = f[i];
    }
    {
      float f[EPL];
      ok &= poll_tagged<EPL>(a.vnew + size_t(kh) * HD + size_t(li) * EPL, qtag, f, false, c.wait_ns);
#pragma unroll
      for (int i = 0; i < EPL; ++i) vnew[li * EPL + i] = f[i];
    }
    if (!ok) {
      sm.flags[0] = 1;
      atomicOr(&a.st->err, 8);
    }
  }
  __syncwarp();
  // running softmax of this warp's rows (max m, sum l, weighted V sum acc)
  float m = -INFINITY, l = 0.0f, acc[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) acc[i] = 0.0f;
  for (int b0 = wb; b0 < old_end; b0 += NB * STRIDE) {
    if (b0 != wb) {
#pragma unroll
      for (int e = 0; e < NB; ++e) {
        const size_t jj = size_t(min(b0 + sub + e * STRIDE, last));
        kr[e] = __ldcg(Kp + jj * RW);
        vr[e] = __ldcg(Vp + jj * RW);
      }
    }
    float sc[NB];
    float mx = m;
#pragma unroll
    for (int e = 0; e < NB; ++e) {
      float kf[EPL];
      kv_unpack(kr[e], kf);
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < EPL; ++i) d = fmaf(q[i], kf[i], d);
#pragma unroll
      for (int o = 1; o < LPK; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      sc[e] = b0 + sub + e * STRIDE < old_end ? d * a.attn_scale : -INFINITY;
      mx = fmaxf(mx, sc[e]);
    }
    if (mx != -INFINITY) {  // rescale to the new maximum, then add this batch's rows
      const float cf = expf(m - mx);
      l *= cf;
#pragma unroll
      for (int i = 0; i < EPL; ++i) acc[i] *= cf;
#pragma unroll
      for (int e = 0; e < NB; ++e) {
        const float p = sc[e] == -INFINITY ? 0.0f : expf(sc[e] - mx);
        float vf[EPL];
        kv_unpack(vr[e], vf);
        l += p;
#pragma unroll
        for (int i = 0; i < EPL; ++i) acc[i] = fmaf(p, vf[i], acc[i]);
      }
      m = mx;
    }
  }
  if (new_here) {  // this step's row (first lane group)
    float d = 0.0f;
    if (sub == 0) {
#pragma unroll
      for (int i = 0; i < EPL; ++i) d = fmaf(q[i], knew[li * EPL + i], d);
    }
#pragma unroll
    for (int o = 1; o < LPK; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (sub == 0) {
      const float sc = d * a.attn_scale, mx = fmaxf(m, sc);
      const float cf = expf(m - mx), p = expf(sc - mx);
      l = l * cf + p;
#pragma unroll
      for (int i = 0; i < EPL; ++i) acc[i] = fmaf(p, vnew[li * EPL + i], acc[i] * cf);
      m = mx;
    }
  }
  // merge the lane groups of the warp, then the warps
#pragma unroll
  for (int o = LPK; o < 32; o <<= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, o), lo = __shfl_xor_sync(0xffffffffu, l, o);
    const float mn = fmaxf(m, mo);
    const float c0 = mn == -INFINITY ? 0.0f : expf(m - mn), c1 = mn == -INFINITY ? 0.0f : expf(mo - mn);
    l = l * c0 + lo * c1;
#pragma unroll
    for (int i = 0; i < EPL; ++i) acc[i] = acc[i] * c0 + __shfl_xor_sync(0xffffffffu, acc[i], o) * c1;
    m = mn;
  }
  if (lane < LPK) {
#pragma unroll
    for (int i = 0; i < EPL; ++i) wa[warp * HD + li * EPL + i] = acc[i];
    if (lane == 0) {
      wm[warp] = m;
      wl[warp] = l;
    }
  }
  cbar();
  for (int d = tid; d < HD; d += MK_T) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < MK_W; ++w) M = fmaxf(M, wm[w]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < MK_W; ++w) {
      const float f = wm[w] == -INFINITY ? 0.0f : expf(wm[w] - M);  // a warp without rows adds nothing
      L += wl[w] * f;
      O += wa[w * HD + d] * f;
    }
    const float out = L > 0.0f ? O / L : 0.0f;
    if (S == 1) {
      st_tag(a.att + size_t(h) * HD + d, out, otag);
    } else {
      st_tag(a.att + size_t(s) * a.hidden + size_t(h) * HD + d, out, otag);
      if (d == 0) {
        st_tag(a.attml + (size_t(s) * a.n_heads + h) * 2, M, otag);
        st_tag(a.attml + (size_t(s) * a.n_heads + h) * 2 + 1, L, otag);
      }
    }
  }
}

template <int HD, typename KT>
__device__ __forceinline__ void attention_phase(const MkArgs& a, const MkSmem& sm, const MkPart& P, const Ctx& c) {
  const int S = c.S;
  if (int(blockIdx.x) >= a.n_heads * S) return;
  const int h = int(blockIdx.x) / S, s = int(blockIdx.x) - h * S;
  const int nkeys = min(c.kv_len + 1, c.position + 1);
  const int chunk = (nkeys + S - 1) / S;
  const int j0 = s * chunk, j1 = min(nkeys, j0 + chunk);
  const uint32_t qtag = c.tag0 + uint32_t(P.dep), otag = c.tag0 + uint32_t(P.phase);
  mk_attention<HD, KT>(a, sm, P.phase / 5, h, s, S, j0, j1, c, qtag, otag);
}

// Tensor parallelism, end of a generate step (the last CTA of each rank): the
// rank's argmax key (order-preserving logit bits | token id, NaN flag in bit 31 of
// the low word) goes to slot tp_rank of every rank's key words, then the ranks'
// keys are max-reduced (the same result on every rank). Bounded: a rank that
// stopped ends the generate loop with error 16. keys: offset (words) of the key
// words in each exchange buffer.
__device__ __noinline__ bool exchange_keys(StepState* st, unsigned long long* const* peers, size_t keys, int rank,
                                           int tp, uint32_t tag0, unsigned long long wait_ns) {
  const unsigned long long tag = static_cast<unsigned long long>(tag0 + 1023u) << 32;  // no phase has this tag
  const unsigned long long best = atomicExch(&st->best, 0ull);
  const int nan = atomicExch(&st->nan, 0);
  const uint32_t hi = uint32_t(best >> 32), lo = (uint32_t(best) & 0x7FFFFFFFu) | (nan ? 0x80000000u : 0u);
  for (int r = 0; r < tp; ++r) {  // one 64-bit store per word: value and tag arrive together
    st_sys(peers[r] + keys + 2 * size_t(rank), tag | hi);
    st_sys(peers[r] + keys + 2 * size_t(rank) + 1, tag | lo);
  }
  const unsigned long long* own = peers[rank] + keys;
  unsigned long long kmax = 0ull;
  int n = 0;
  const unsigned long long t0 = gtime();
  for (int r = 0; r < tp; ++r) {
    unsigned long long x, y;
    while (true) {
      x = ld_sys(own + 2 * r);
      y = ld_sys(own + 2 * r + 1);
      if ((x >> 32) == (tag >> 32) && (y >> 32) == (tag >> 32)) break;
      if (gtime() - t0 > wait_ns) {
        atomicOr(&st->err, 16);
        st->ticket = 0;
        st->done = 1;
        return false;
      }
    }
    const unsigned long long k = ((x & 0xFFFFFFFFull) << 32) | (y & 0x7FFFFFFFull);
    kmax = k > kmax ? k : kmax;
    n |= int((y >> 31) & 1u);
  }
  st->best = kmax;
  st->nan = n;
  return true;
}

// One instantiation per (head_dim, KV cache type, Q6_K weights present), so a
// kernel carries only the code its model runs.
template <int HD, typename KT, bool Q6>
__global__ void __launch_bounds__(MK_THREADS, 1) decode_step_kernel(const MkArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const MkSmem sm = mk_carve(a, smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  StepState* st = a.st;
  if (st->done) return;  // the generate loop has ended: every CTA returns at once
  TileCursor cur{-1, 0, 0};  // the producer lane's next tile
  int kp = 0;                // tiles the producer lane has issued
  if (tid == MK_T) {  // producer lane: barriers, then the first tiles straight from the global part list
    for (int s = 0; s < a.nslots; ++s) {
      mbar_init(sm.full + s, 1);
      mbar_init(sm.empty + s, MK_W);
    }
    mbar_fence_init();
    MkTile T;
    for (; kp < a.nslots && next_tile(a.parts, a.nparts, cur, T, nullptr); ++kp)
      issue_tile(a.parts + T.part, T, sm.slots + size_t(kp) * a.slot_bytes, sm.full + kp);
  }
  {
    const int4* src = reinterpret_cast<const int4*>(a.parts);
    int4* dst = reinterpret_cast<int4*>(sm.parts);
    for (int i = tid; i < a.nparts * int(sizeof(MkPart) / 16); i += MK_THREADS) dst[i] = src[i];
    for (int i = tid; i < a.nparts; i += MK_THREADS) {  // this CTA's groups of every part
      int g0 = 0, g1 = 0;
      if (a.parts[i].kind != MK_ATT) cta_share(a.parts[i].ngroups, cta, gridDim.x, g0, g1);
      sm.share[i] = uint32_t(g0) | (uint32_t(g1) << 16);
    }
  }
  if (tid < 8) sm.flags[tid] = 0;
  for (int i = tid; i < a.head_dim / 2; i += MK_THREADS) {  // cos / sin of this step's position (attention.rs:230-248)
    sm.rcos[i] = __ldg(a.rope_cos + size_t(st->position) * (a.head_dim / 2) + i);
    sm.rsin[i] = __ldg(a.rope_sin + size_t(st->position) * (a.head_dim / 2) + i);
  }
  Ctx c;
  c.tag0 = uint32_t(st->epoch) * 1024u + 1u;
  c.position = st->position;
  c.kv_len = st->kv_len;
  {
    const uint32_t tok = a.gen_mode ? a.hist[st->nhist - 1] : a.ids[0];
    c.x0 = tok < uint32_t(a.vocab) ? a.emb + size_t(tok) * a.hidden : a.zero;  // model.rs:847-864
    int g0, g1;
    cta_share(a.hidden / ROWS, cta, gridDim.x, g0, g1);
    c.R0 = ROWS * g0;
  }
  c.g0 = 0;
  c.rm = 1.0f;
  c.best = 0ull;
  c.nan = 0;
  c.S = att_splits(min(c.kv_len + 1, c.position + 1), a.head_dim, a.kv_half, a.att_smax);
  c.wait_ns = 1000000ull * unsigned(st->wait_ms > 0 ? st->wait_ms : 2000);
  __syncthreads();
  if (warp == MK_W) {  // ---- producer: refill each slot once the consumer warps have left it
    if (lane != 0) return;
    MkTile T;
    for (; next_tile(sm.parts, a.nparts, cur, T, sm.share); ++kp) {
      const int s = kp % a.nslots, use = kp / a.nslots;
      if (!mbar_wait_n(sm.empty + s, uint32_t((use - 1) & 1), MK_MBAR_POLLS)) {
        atomicOr(&st->err, 4);  // the consumers stopped taking tiles
        return;
      }
      fence_proxy_async();
      issue_tile(sm.parts + T.part, T, sm.slots + size_t(s) * a.slot_bytes, sm.full + s);
    }
    return;
  }

  bool abort_ = false;
  int k = 0, U = 0;
  for (int pi = 0; pi < a.nparts; ++pi) {
    const MkPart& P = sm.parts[pi];
    if (P.kind == MK_ATT) {
      // the QKV phase is done with the region; a warp whose weight wait expired has
      // raised the abort flag before this barrier, so every warp takes the same branch
      // (the attention has barriers of its own)
      cbar();
      abort_ = *reinterpret_cast<volatile int*>(sm.flags) != 0;
      if (!abort_) {
        attention_phase<HD, KT>(a, sm, P, c);
      }
      continue;
    }
    const int g0 = int(sm.share[pi] & 0xFFFFu), g1 = int(sm.share[pi] >> 16);
    c.g0 = g0;
    if (P.first) {
      cbar();  // the previous phase is done with the region and the stashes
          bool ok;
      const int rounds = (P.K + MK_T * 8 - 1) / (MK_T * 8);
      if (rounds <= 1) ok = build_input<1>(a, pi, P, c, sm, abort_);
      else if (rounds == 2) ok = build_input<2>(a, pi, P, c, sm, abort_);
      else if (rounds == 3) ok = build_input<3>(a, pi, P, c, sm, abort_);
      else ok = build_input<4>(a, pi, P, c, sm, abort_);
      if (!ok) {
        sm.flags[0] = 1;
        atomicOr(&st->err, 8);
      }
      cbar();
      abort_ = *reinterpret_cast<volatile int*>(sm.flags) != 0;
      U = 0;
      if (P.norm) {
        float tot = 0.0f;
        for (int i = 0; i < MK_W; ++i) tot = __fadd_rn(tot, sm.red[i]);
        c.rm = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(P.K)), P.eps)));
      } else {
        c.rm = 1.0f;
      }
    }
    const int NB = P.K / QK_K;
    const uint32_t row_bytes = uint32_t(NB * dev_block_bytes(P.dtype));
    const Planes pl = planes_at(smem_u32(sm.region), P.K);
    const int gpt = P.gpt;
    if (NB > 8) {
      // Rows longer than 2048 values: a tile holds few whole-K groups (one for K >= 7168),
      // so whole-K units would leave most warps idle while the ring's few tiles are in
      // flight. The units are (group, 8-block chunk) pairs dealt round-robin to the warps
      // across tiles; the chunks' partial sums meet in part and are added in chunk order
      // once the part's last tile is done, then the epilogues run.
      const int CH = (NB + 7) / 8;                  // this part's 8-block chunks
      const int CHS = P.kchain ? int(P.kchs) : CH;  // chunks of the whole row (a K chain: all its parts)
      const int CB = P.kchain ? int(P.kch0) : 0;    // this part's first chunk in the row
      int gb = 0;  // CTA-local index of the tile's first group
      for (int tg = g0; tg < g1; tg += gpt, ++k) {
        const int tng = min(gpt, g1 - tg);
        const int s = k % a.nslots, use = k / a.nslots;
        if (!mbar_wait_n(sm.full + s, uint32_t(use & 1), abort_ ? 4096u : MK_MBAR_POLLS)) {
          if (!abort_ && lane == 0) {
            atomicOr(&st->err, 4);
            sm.flags[0] = 1;
          }
          abort_ = true;
        }
        const uint32_t sbase = smem_u32(sm.slots + size_t(s) * a.slot_bytes);
        for (int ul = (warp - (gb * CH) % MK_W + MK_W) % MK_W; ul < tng * CH; ul += MK_W) {
          const int gl = ul / CH, b = (ul - gl * CH) * 8 + (lane & 7);
          float acc[ROWS] = {0.0f, 0.0f, 0.0f, 0.0f};
          if (!abort_ && b < NB) {
            uint32_t ra[ROWS];
#pragma unroll
            for (int i = 0; i < ROWS; ++i) {
              const int ro = P.kind == MK_GU ? (i < 2 ? 2 * gl + i : 2 * tng + 2 * gl + (i - 2)) : ROWS * gl + i;
              ra[i] = sbase + uint32_t(ro) * row_bytes;
            }
            if (!Q6 || P.dtype == DT_Q4K) q4k_unit(ra, b, lane >> 3, pl, acc);
            else q6k_unit(ra, b, lane >> 3, pl, acc);
          }
#pragma unroll
          for (int i = 0; i < ROWS; ++i) acc[i] = warp_sum(acc[i]);
          if (lane == 0)
#pragma unroll
            for (int i = 0; i < ROWS; ++i) sm.part[((gb + gl) * CHS + CB + (ul - gl * CH)) * ROWS + i] = acc[i];
        }
        gb += tng;
        __syncwarp();
        if (lane == 0) mbar_arrive(sm.empty + s);  // this warp is done with the slot
      }
      cbar();  // every chunk's partial sums are in part
      if (P.kchain == 1) continue;  // the chain's next part adds its chunks first
      for (int gl = warp; gl < g1 - g0; gl += MK_W) {
        float v[ROWS] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int ch = 0; ch < CHS; ++ch)
#pragma unroll
          for (int i = 0; i < ROWS; ++i) v[i] += sm.part[(gl * CHS + ch) * ROWS + i];
        if (P.norm)
#pragma unroll
          for (int i = 0; i < ROWS; ++i) v[i] = __fmul_rn(v[i], c.rm);
        if (!abort_) group_epilogue(a, P, g0 + gl, v, c, sm);
      }
      cbar();  // part is free for the next split part
    } else {
      for (int tg = g0; tg < g1; tg += gpt, ++k) {
        const int tng = min(gpt, g1 - tg);
        const int s = k % a.nslots, use = k / a.nslots;
        // every consumer warp waits for every tile and arrives on its slot
        if (!mbar_wait_n(sm.full + s, uint32_t(use & 1), abort_ ? 4096u : MK_MBAR_POLLS)) {
          if (!abort_ && lane == 0) {
            atomicOr(&st->err, 4);
            sm.flags[0] = 1;
          }
          abort_ = true;
        }
        const uint32_t sbase = smem_u32(sm.slots + size_t(s) * a.slot_bytes);
        // one group (4 rows, whole K) per warp; lane = (pair lane / 8, block lane % 8 + 8 j)
        for (int u = (warp - U % MK_W + MK_W) % MK_W; u < tng; u += MK_W) {
          float acc[ROWS] = {0.0f, 0.0f, 0.0f, 0.0f};
          if (!abort_) {
            uint32_t ra[ROWS];
#pragma unroll
            for (int i = 0; i < ROWS; ++i) {
              const int ro = P.kind == MK_GU ? (i < 2 ? 2 * u + i : 2 * tng + 2 * u + (i - 2)) : ROWS * u + i;
              ra[i] = sbase + uint32_t(ro) * row_bytes;
            }
            if (!Q6 || P.dtype == DT_Q4K)
              for (int b = lane & 7; b < NB; b += 8) q4k_unit(ra, b, lane >> 3, pl, acc);
            else
              for (int b = lane & 7; b < NB; b += 8) q6k_unit(ra, b, lane >> 3, pl, acc);
          }
          float v[ROWS];
#pragma unroll
          for (int i = 0; i < ROWS; ++i) v[i] = warp_sum(acc[i]);
          if (P.norm)
#pragma unroll
            for (int i = 0; i < ROWS; ++i) v[i] = __fmul_rn(v[i], c.rm);
          if (!abort_) group_epilogue(a, P, tg + u, v, c, sm);
        }
        U += tng;
        // leave the slot: the producer refills it with the tile nslots further on
        __syncwarp();
        if (lane == 0) mbar_arrive(sm.empty + s);
      }
    }
    if (P.kind != MK_LM) continue;
    // LM head: CTA max of the argmax keys, one atomic per CTA; the last CTA to
    // finish runs the sampler bookkeeping and advances the epoch
    cbar();
    unsigned long long* rb = reinterpret_cast<unsigned long long*>(sm.red);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ob = __shfl_xor_sync(0xffffffffu, c.best, o);
      c.best = ob > c.best ? ob : c.best;
      c.nan |= __shfl_xor_sync(0xffffffffu, c.nan, o);
    }
    if (lane == 0) {
      rb[warp] = c.best;
      if (c.nan) atomicOr(sm.flags + 2, 1);
    }
    cbar();
    if (tid == 0) {
      unsigned long long bmax = 0ull;
      for (int i = 0; i < MK_W; ++i) bmax = rb[i] > bmax ? rb[i] : bmax;
      if (a.gen_mode == 1) {
        if (bmax) atomicMax(&st->best, bmax);
        if (sm.flags[2]) atomicOr(&st->nan, 1);
      }
      __threadfence();
      const int prev = atomicAdd(&st->ticket, 1);
      if (prev == int(gridDim.x) - 1) {
        __threadfence();
        const bool ok = !(a.gen_mode == 1 && a.tp_size > 1) ||
                        exchange_keys(st, a.peers, a.xofs + 4 * size_t(a.tp_size) * size_t(a.hidden), a.tp_rank,
                                      a.tp_size, c.tag0, c.wait_ns);
        st->epoch += 1;
        if (a.gen_mode == 1) {
          if (ok) finish_sample_state(st, a.hist, a.pen_cnt);
        } else {
          st->ticket = 0;
        }
      }
    }
  }
}

int g_mk_sms = 0;
size_t g_mk_smem_max = 0;

using StepKernel = void (*)(MkArgs);
StepKernel step_kernel(int head_dim, int kv_half, int has_q6) {
  const int i = (head_dim == 128 ? 4 : 0) + (kv_half ? 2 : 0) + (has_q6 ? 1 : 0);
  static const StepKernel k[8] = {
      decode_step_kernel<64, float, false>,  decode_step_kernel<64, float, true>,
      decode_step_kernel<64, __half, false>, decode_step_kernel<64, __half, true>,
      decode_step_kernel<128, float, false>, decode_step_kernel<128, float, true>,
      decode_step_kernel<128, __half, false>, decode_step_kernel<128, __half, true>};
  return k[i];
}

}  // namespace

int decode_step_grid() {
  if (g_mk_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_mk_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_mk_sms <= 0) g_mk_sms = 148;
  }
  return g_mk_sms;
}

cudaError_t decode_step_configure() {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  g_mk_smem_max = size_t(optin) - 1024;
  decode_step_grid();
  for (int i = 0; i < 8; ++i) {
    e = cudaFuncSetAttribute(step_kernel(i & 4 ? 128 : 64, i & 2, i & 1), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(g_mk_smem_max));
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

bool decode_step_plan(MkPart* parts, int nparts, MkArgs& a, int n_rep, size_t* smem) {
  if (g_mk_smem_max == 0) return false;
  if (n_rep > 16 || (a.head_dim != 64 && a.head_dim != 128)) return false;
  const int grid = decode_step_grid();
  int kmax = 0;
  size_t gmax = 0;
  for (int i = 0; i < nparts; ++i) {
    if (parts[i].kind == MK_ATT) continue;
    if (parts[i].K % QK_K || parts[i].K > MK_MAX_K || parts[i].ngroups < 1) return false;
    // a K chain takes the split path (more than 8 blocks a part, whole 8-block chunks but the last)
    if (parts[i].kchain && (parts[i].K <= 8 * QK_K || parts[i].kind != MK_D)) return false;
    kmax = std::max(kmax, parts[i].K);
    gmax = std::max(gmax, 4 * size_t(parts[i].K / QK_K) * dev_block_bytes(parts[i].dtype));
  }
  // attention: one CTA per (query head, key split), at most MK_ASMAX splits
  a.att_smax = std::min(MK_ASMAX, grid / std::max(1, a.n_heads));
  if (a.att_smax < 1) return false;
  // attention's shared memory: the warps' maxima, sums and outputs, this step's K and V rows
  const size_t att_bytes = sizeof(float) * (size_t(MK_W) * (a.head_dim + 2) + 2 * a.head_dim);
  size_t region = std::max(planes_bytes(kmax), att_bytes);
  region = (region + 127) / 128 * 128;
  const size_t slot = std::max<size_t>(32 * 1024, (gmax + 1023) / 1024 * 1024);
  // groups of one tile (whole-K rows that fit a slot); the kernel walks each CTA's
  // share of every part in tiles of gpt groups
  int res_rows = 0, lm_rows = 0, part_floats = ROWS;
  for (int i = 0; i < nparts; ++i) {
    if (parts[i].kind == MK_ATT) continue;
    const size_t group = 4 * size_t(parts[i].K / QK_K) * dev_block_bytes(parts[i].dtype);
    parts[i].gpt = uint16_t(std::min<size_t>(MK_GPT, slot / group));
    for (int c = 0; c < grid; ++c) {
      int g0, g1;
      cta_share(parts[i].ngroups, c, grid, g0, g1);
      const int rows = ROWS * (g1 - g0);
      if (parts[i].kind == MK_O || parts[i].kind == MK_D) res_rows = std::max(res_rows, rows);
      if (parts[i].kind == MK_LM) lm_rows = std::max(lm_rows, rows);
      const int NB = parts[i].K / QK_K;
      if (NB > 8)  // split part: a float per (group, 8-block chunk of the row, row)
        part_floats = std::max(part_floats, (g1 - g0) * (parts[i].kchain ? int(parts[i].kchs) : (NB + 7) / 8) * ROWS);
    }
  }
  a.nparts = nparts;
  a.part_floats = part_floats;
  a.slot_bytes = int(slot);
  a.region_bytes = int(region);
  a.kmax = kmax;
  a.res_rows = std::max(res_rows, 4);
  a.lm_rows = std::max(lm_rows, 4);
  a.nslots = 1;
  const size_t fixed = mk_offsets(a).total - slot;
  if (fixed + 3 * slot > g_mk_smem_max) return false;
  a.nslots = int(std::min<size_t>(8, (g_mk_smem_max - fixed) / (slot + 16)));
  while (a.nslots > 2 && mk_offsets(a).total > g_mk_smem_max) --a.nslots;
  *smem = mk_offsets(a).total;
  if (*smem > g_mk_smem_max) return false;
  {  // the 64-bit words of the carve-up (argmax keys in red, the mbarriers) must be 8-byte aligned
    const MkOffsets o = mk_offsets(a);
    if (o.red % 8 || o.full % 8 || o.empty % 8 || o.parts % 16) return false;
  }
  int per_sm = 0;
  a.has_q6 = 0;
  for (int i = 0; i < nparts; ++i)
    if (parts[i].kind != MK_ATT && parts[i].dtype == DT_Q6K) a.has_q6 = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel(a.head_dim, a.kv_half, a.has_q6), MK_THREADS,
                                                    *smem) != cudaSuccess ||
      per_sm < 1)
    return false;
  return true;
}

cudaError_t launch_decode_step(const MkArgs& a, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(decode_step_grid());
  cfg.blockDim = dim3(MK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, step_kernel(a.head_dim, a.kv_half, a.has_q6), a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb
