// Persistent decode step: one cooperative launch per generated token.
//
// Every CTA (one per SM) owns a fixed share of the rows of every weight matrix
// of the step. Its producer warp walks that share phase after phase (layer by
// layer: [q;k;v], o, gate/up, down, then the LM head) and streams it into a
// ring of shared-memory slots with cp.async.bulk copies completing on
// mbarriers. Weights never depend on the activations, so the copies run ahead
// across phase boundaries and HBM stays busy while the consumer warps wait for
// the inputs of the next phase.
//
// Consumer warps, per phase: wait until the phase's input vector is complete
// (a per-phase counter that each CTA increments after writing its share, read
// with acquire semantics; waits are bounded and flag an error word on expiry),
// quantise the input into integer limbs (the same planes as the per-op GEMV,
// with the RMSNorm of candle's rms_norm fused in), run the dp4a dot products of
// each weight tile, reduce the K slices in a fixed order and apply the fused
// epilogue (RoPE + KV append, residual add, SwiGLU, LM-head penalty + argmax).
// The attention phase runs on the first n_kv * splits CTAs: split-K over the
// keys with the previous steps' K/V staged before the wait, merged by the last
// CTA of each KV head.
//
// Data written by one CTA and read by another inside the launch is read with
// ld.global.cg (L2), never through the non-coherent L1.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cmath>

#include "device_common.cuh"
#include "kernels.h"

namespace wcb {

namespace {

constexpr int MK_CW = 15;               // consumer warps (16 warps per CTA: 128 registers a thread)
constexpr int MK_CT = MK_CW * 32;       // consumer threads
constexpr int MK_THREADS = MK_CT + 32;  // + the producer warp
constexpr int MK_MAX_K = 16384;         // longest GEMV input kept in registers by the plane builder
constexpr int MK_RND = (MK_MAX_K + MK_CT * 8 - 1) / (MK_CT * 8);
constexpr int MK_TS = 32;               // keys per attention tile
constexpr long long MK_WAIT_CYCLES = 4000000000ll;  // ~2 s at 2 GHz: bound of every spin wait

// named barrier of the consumer warps (the producer warp never joins it)
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(MK_CT) : "memory"); }

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <typename KT>
__device__ __forceinline__ float4 ldcg_kv4(const KT* p);
template <>
__device__ __forceinline__ float4 ldcg_kv4<float>(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}
template <>
__device__ __forceinline__ float4 ldcg_kv4<__half>(const __half* p) {
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(p));
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

// Shared-memory carve-up of one CTA (sizes in MkArgs, set on the host):
//   [slots]   nslots x slot_bytes weight tiles
//   [region]  activation planes (GEMV phases) or attention staging
//   [part]    2 x part_units x 16 floats: per-unit partial sums, ping-pong per tile
//   [misc]    gacc[16], red[64], flags[8]
//   [bars]    full[nslots], empty[nslots]
struct MkSmem {
  uint8_t* slots;
  uint8_t* region;
  float* part;
  float* gacc;
  float* red;
  int* flags;  // [0] abort
  uint64_t* full;
  uint64_t* empty;
};

__device__ __forceinline__ MkSmem mk_carve(uint8_t* smem, const MkArgs& a) {
  MkSmem s;
  s.slots = smem;
  uint8_t* p = smem + size_t(a.nslots) * a.slot_bytes;
  s.region = p;
  p += a.region_bytes;
  s.part = reinterpret_cast<float*>(p);
  p += sizeof(float) * 2 * 16 * size_t(a.part_units);
  s.gacc = reinterpret_cast<float*>(p);
  s.red = s.gacc + 16;
  s.flags = reinterpret_cast<int*>(s.red + 64);
  s.full = reinterpret_cast<uint64_t*>(s.flags + 8);
  s.empty = s.full + a.nslots;
  return s;
}

// Groups [g0, g1) of a part owned by CTA c of n.
__device__ __forceinline__ void cta_share(int ngroups, int c, int n, int& g0, int& g1) {
  g0 = int((long long)c * ngroups / n);
  g1 = int((long long)(c + 1) * ngroups / n);
}

// Tile t of this CTA's share: groups [g, g + ng), k-blocks [kb0, kb0 + nkb).
struct Tile {
  int g, ng, kb0, nkb;
};

__device__ __forceinline__ int tiles_of(const MkPart& P, int g0, int g1) {
  const int nb = P.K / QK_K;
  if (g1 <= g0) return 0;
  if (P.kbt >= nb) return (g1 - g0 + P.gpt - 1) / P.gpt;
  return (g1 - g0) * ((nb + P.kbt - 1) / P.kbt);
}

__device__ __forceinline__ Tile tile_at(const MkPart& P, int g0, int g1, int t) {
  const int nb = P.K / QK_K;
  Tile r;
  if (P.kbt >= nb) {
    r.g = g0 + t * P.gpt;
    r.ng = min(P.gpt, g1 - r.g);
    r.kb0 = 0;
    r.nkb = nb;
  } else {
    const int kt = (nb + P.kbt - 1) / P.kbt;
    r.g = g0 + t / kt;
    r.ng = 1;
    r.kb0 = (t % kt) * P.kbt;
    r.nkb = min(P.kbt, nb - r.kb0);
  }
  return r;
}

// Global address of row r (0-based within the part) of a non-SwiGLU part.
__device__ __forceinline__ const uint8_t* part_row(const MkPart& P, int r, size_t row_bytes) {
  if (r < P.rows[0]) return P.w[0] + size_t(r) * row_bytes;
  r -= P.rows[0];
  if (P.nseg > 1 && r < P.rows[1]) return P.w[1] + size_t(r) * row_bytes;
  r -= P.rows[1];
  return P.w[2] + size_t(r) * row_bytes;
}

// Producer: the bulk copies of one tile into slot memory dst (completing on bar).
__device__ void issue_tile(const MkPart& P, const Tile& T, uint8_t* dst, uint64_t* bar) {
  const size_t bb = dev_block_bytes(P.dtype);
  const size_t row_bytes = size_t(P.K / QK_K) * bb;
  const uint32_t rb = uint32_t(size_t(T.nkb) * bb);
  mbar_expect_tx(bar, 4u * uint32_t(T.ng) * rb);
  const bool whole = T.nkb * bb == row_bytes;
  if (P.kind == MK_GU) {
    if (whole) {
      const uint32_t bytes = 2u * uint32_t(T.ng) * rb;
      bulk_g2s(dst, P.w[0] + size_t(2 * T.g) * row_bytes, bytes, bar);
      bulk_g2s(dst + bytes, P.w[1] + size_t(2 * T.g) * row_bytes, bytes, bar);
    } else {
      for (int i = 0; i < 4; ++i)
        bulk_g2s(dst + i * rb, P.w[i >> 1] + size_t(2 * T.g + (i & 1)) * row_bytes + size_t(T.kb0) * bb, rb, bar);
    }
    return;
  }
  if (whole) {
    int r0 = 4 * T.g;
    const int r1 = 4 * (T.g + T.ng);
    int base = 0;
    for (int sg = 0; sg < 3 && r0 < r1; ++sg) {
      const int s1 = base + (sg < P.nseg ? P.rows[sg] : 0);
      if (r0 < s1) {
        const int e = min(r1, s1);
        const uint32_t bytes = uint32_t(size_t(e - r0) * row_bytes);
        bulk_g2s(dst, P.w[sg] + size_t(r0 - base) * row_bytes, bytes, bar);
        dst += bytes;
        r0 = e;
      }
      base = s1;
    }
    return;
  }
  for (int i = 0; i < 4; ++i)
    bulk_g2s(dst + i * rb, part_row(P, 4 * T.g + i, row_bytes) + size_t(T.kb0) * bb, rb, bar);
}

// Bounded wait of consumer thread 0 for counter >= target; 0 on expiry.
__device__ __forceinline__ int wait_counter(const int* c, int target) {
  if (ld_acquire(c) >= target) return 1;
  const long long t0 = clock64();
  while (ld_acquire(c) < target) {
    if (clock64() - t0 > MK_WAIT_CYCLES) return 0;
  }
  return 1;
}

// Consumer thread 0 publishes this CTA's share of a phase (after a consumer
// barrier, so every consumer thread's writes are ordered before it).
__device__ __forceinline__ void signal_counter(int* c) {
  __threadfence();
  atomicAdd(c, 1);
}

// Limb planes (M = 1) of the input vector x[K] of a GEMV phase, K <= MK_MAX_K
// and a multiple of 256. With norm: RMSNorm first, as candle's rms_norm
// (candle_tensor_backend.rs:30-57): m = sqrt(sum(x^2)/K + eps), x / m * w, IEEE
// divide and square root. All loads are issued before any use (one L2 round
// trip); cg selects ld.global.cg for vectors written inside this launch.
__device__ void mk_planes(const float* x, bool cg, const float* norm, float eps, int K, const XPlanes& p,
                          float* red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float4 v[MK_RND][2], g[MK_RND][2];
#pragma unroll
  for (int r = 0; r < MK_RND; ++r) {
    const int k = r * MK_CT * 8 + tid * 8;
    v[r][0] = v[r][1] = g[r][0] = g[r][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (k < K) {
      const float4* src = reinterpret_cast<const float4*>(x + k);
      if (cg) {
        v[r][0] = __ldcg(src);
        v[r][1] = __ldcg(src + 1);
      } else {
        v[r][0] = __ldg(src);
        v[r][1] = __ldg(src + 1);
      }
      if (norm) {
        g[r][0] = __ldg(reinterpret_cast<const float4*>(norm + k));
        g[r][1] = __ldg(reinterpret_cast<const float4*>(norm + k + 4));
      }
    }
  }
  float m = 1.0f;
  if (norm) {
    float ss = 0.0f;
#pragma unroll
    for (int r = 0; r < MK_RND; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        ss = __fadd_rn(ss, __fmul_rn(v[r][h].x, v[r][h].x));
        ss = __fadd_rn(ss, __fmul_rn(v[r][h].y, v[r][h].y));
        ss = __fadd_rn(ss, __fmul_rn(v[r][h].z, v[r][h].z));
        ss = __fadd_rn(ss, __fmul_rn(v[r][h].w, v[r][h].w));
      }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    cbar();
    float tot = 0.0f;
    for (int w = 0; w < MK_CW; ++w) tot = __fadd_rn(tot, red[w]);
    m = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(K)), eps));
  }
#pragma unroll
  for (int r = 0; r < MK_RND; ++r) {
    const int k = r * MK_CT * 8 + tid * 8;
    if (k < K) {  // whole warps are in or out (K is a multiple of 256)
      float e[8] = {v[r][0].x, v[r][0].y, v[r][0].z, v[r][0].w, v[r][1].x, v[r][1].y, v[r][1].z, v[r][1].w};
      if (norm) {
        const float w8[8] = {g[r][0].x, g[r][0].y, g[r][0].z, g[r][0].w, g[r][1].x, g[r][1].y, g[r][1].z, g[r][1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = __fmul_rn(__fdiv_rn(e[i], m), w8[i]);
      }
      quant8(e, size_t(k), k, p, K, 0);
    }
  }
  cbar();
}

// K slices per group of a tile: enough units to occupy the consumer warps, at
// least 32 chunks (one per lane) per slice.
__device__ __forceinline__ int mk_ksplit(int ng, int nch) {
  return max(1, min((MK_CW + ng - 1) / ng, nch / 32));
}

// Dot products of one tile: unit u = (group gl, K slice ks) per warp; lanes
// stride over the 64-value chunks; warp sums land in part[u][row].
template <int DT>
__device__ void mk_tile_dots(const MkPart& P, const Tile& T, const uint8_t* sbase, const uint8_t* region,
                             float* part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int BB = DT == DT_Q4K ? Q4K_BYTES : Q6K_DEV_BYTES;
  const int rb = T.nkb * BB;
  const int nch = T.nkb * 4;
  const int KS = mk_ksplit(T.ng, nch);
  const int units = T.ng * KS;
  XPlanes p = carve(const_cast<uint8_t*>(region), 1, P.K);
  const int ko = T.kb0 * QK_K;  // first input element of the tile
  p.l0 += ko;
  p.l1 += ko;
  p.l2 += ko;
  p.scale += ko / 32;
  p.sum32 += ko / 32;
  XAddr xad;
  xad.l[0] = smem_u32(p.l0);
  xad.l[1] = smem_u32(p.l1);
  xad.l[2] = smem_u32(p.l2);
  xad.scale = smem_u32(p.scale);
  xad.sum32 = smem_u32(p.sum32);
  const uint32_t sb = smem_u32(sbase);
  for (int u = warp; u < units; u += MK_CW) {
    const int gl = u / KS, ks = u - gl * KS;
    int ro[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i)
      ro[i] = P.kind == MK_GU ? (i < 2 ? 2 * gl + i : 2 * T.ng + 2 * gl + (i - 2)) : ROWS * gl + i;
    float acc[ROWS][1];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) acc[i][0] = 0.0f;
    const int c0 = ks * nch / KS, c1 = (ks + 1) * nch / KS;
    if (DT == DT_Q4K) {
      uint32_t ra[ROWS];
#pragma unroll
      for (int i = 0; i < ROWS; ++i) ra[i] = sb + uint32_t(ro[i] * rb);
      for (int c = c0 + lane; c < c1; c += 32) q4k_chunk_rows<1>(ra, c, P.K, xad, acc);
    } else {
      for (int c = c0 + lane; c < c1; c += 32) {
#pragma unroll
        for (int i = 0; i < ROWS; ++i) q6k_chunk_smem<1>(sbase + size_t(ro[i]) * rb, c, P.K, p, acc[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const float v = warp_sum(acc[i][0]);
      if (lane == i) part[u * 16 + i] = v;
    }
  }
}

// Per-launch values every consumer thread keeps.
struct MkCtx {
  int position, kv_len;
  const float* x0;  // layer-0 input: the embedding row of the step's token
  unsigned long long best;
  int nan;
};

// Fixed-order sum of a tile's K slices and the fused epilogue; warp gl handles
// group gl of the tile, lane i < 4 its row i.
__device__ void mk_epilogue(const MkArgs& a, const MkPart& P, const Tile& T, const float* part, float* gacc,
                            MkCtx& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = P.K / QK_K;
  const int KS = mk_ksplit(T.ng, T.nkb * 4);
  for (int gl = warp; gl < T.ng; gl += MK_CW) {
    float v = 0.0f;
    if (lane < ROWS)
      for (int ks = 0; ks < KS; ++ks) v += part[(gl * KS + ks) * 16 + lane];
    if (T.nkb < nb) {  // one group's K range over several tiles (then T.ng == 1, warp 0)
      if (T.kb0 > 0 && lane < ROWS) v = gacc[lane] + v;
      if (T.kb0 + T.nkb < nb) {
        if (lane < ROWS) gacc[lane] = v;
        continue;
      }
    }
    const float v1 = __shfl_down_sync(0xffffffffu, v, 1);
    const float v2 = __shfl_down_sync(0xffffffffu, v, 2);
    if (lane >= ROWS) continue;
    const int i = lane, g = T.g + gl;
    if (P.kind == MK_QKV) {
      const int hid = a.hidden, hd = a.head_dim, kvd = a.n_kv * a.head_dim;
      const int vr = P.row_offset + ROWS * g + i;
      const size_t esz = a.kv_half ? 2 : 4;
      uint8_t* kc = static_cast<uint8_t*>(a.kcache) + size_t(P.layer) * a.kv_layer_elems * esz;
      uint8_t* vc = static_cast<uint8_t*>(a.vcache) + size_t(P.layer) * a.kv_layer_elems * esz;
      if (vr < hid + kvd) {
        if ((i & 1) == 0) {  // RoPE on (2j, 2j+1) pairs (attention.rs:230-262), table values
          const int col = vr < hid ? vr : vr - hid;
          const int pi = (col % hd) >> 1;
          const float cs = __ldg(a.rope_cos + size_t(c.position) * (hd / 2) + pi);
          const float sn = __ldg(a.rope_sin + size_t(c.position) * (hd / 2) + pi);
          const float n0 = __fsub_rn(__fmul_rn(v, cs), __fmul_rn(v1, sn));
          const float n1 = __fadd_rn(__fmul_rn(v, sn), __fmul_rn(v1, cs));
          if (vr < hid) {
            a.q[vr] = n0;
            a.q[vr + 1] = n1;
          } else {
            const size_t off = (size_t(col / hd) * a.max_seq + c.kv_len) * hd + col % hd;
            if (a.kv_half) {
              reinterpret_cast<__half*>(kc)[off] = __float2half_rn(n0);
              reinterpret_cast<__half*>(kc)[off + 1] = __float2half_rn(n1);
            } else {
              reinterpret_cast<float*>(kc)[off] = n0;
              reinterpret_cast<float*>(kc)[off + 1] = n1;
            }
          }
        }
      } else {
        const int col = vr - hid - kvd;
        const size_t off = (size_t(col / hd) * a.max_seq + c.kv_len) * hd + col % hd;
        if (a.kv_half) reinterpret_cast<__half*>(vc)[off] = __float2half_rn(v);
        else reinterpret_cast<float*>(vc)[off] = v;
      }
    } else if (P.kind == MK_O) {  // attention out + residual (layer.rs:68)
      const int r = ROWS * g + i;
      const float res = P.layer == 0 ? __ldg(c.x0 + r) : __ldcg(a.xa + r);
      a.xb[r] = __fadd_rn(res, v);
    } else if (P.kind == MK_D) {  // FFN out + residual (layer.rs:86)
      const int r = ROWS * g + i;
      a.xa[r] = __fadd_rn(__ldcg(a.xb + r), v);
    } else if (P.kind == MK_GU) {  // ffn.rs:90-94: silu(g) * u
      if (i < 2) {
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
        a.act[2 * g + i] = __fmul_rn(__fmul_rn(v, sig), v2);
      }
    } else {  // MK_LM
      const int n = ROWS * g + i;
      a.logits[n] = v;
      if (a.gen_mode) {
        float pv = v;
        if (a.rep != 1.0f) {  // apply_repetition_penalty: once per occurrence (sampling.rs:86-103)
          const uint32_t cnt = a.pen_cnt[n];
          for (uint32_t k = 0; k < cnt; ++k) pv = pv > 0.0f ? __fdiv_rn(pv, a.rep) : __fmul_rn(pv, a.rep);
        }
        if (pv != pv) c.nan = 1;
        else {
          const unsigned long long key = (static_cast<unsigned long long>(order_key(pv)) << 32) | uint32_t(n);
          c.best = key > c.best ? key : c.best;
        }
      }
    }
  }
}

// Attention of one (KV head kh, key split) item of a decode step (T = 1) over
// the layer's cache, the n_rep query heads of kh together (repeat_kv,
// attention.rs:297-322): scores (q.k) * scale with the dot in key order and no
// contraction, causal limit j <= position, softmax with a running max, P.V
// (attention.rs:332-435). Keys of earlier steps are staged before the wait on
// the QKV phase; this step's key (slot kv_len), q and v after it. With several
// splits the last CTA of kh (ticket) merges the partials. Returns after the
// item's output is published on the attention counter (or on abort).
template <int HD, typename KT>
__device__ void mk_attention(const MkArgs& a, const MkSmem& sm, const MkPart& P, int kh, int split, int nsplit,
                             int chunk, int nkeys, const MkCtx& c, int& abort_) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_rep = a.n_heads / a.n_kv;
  constexpr int TS = MK_TS, KP = HD + 1;
  float* qs = reinterpret_cast<float*>(sm.region);  // [n_rep][HD]
  float* Ks = qs + n_rep * HD;                      // [TS][HD+1]
  float* Vs = Ks + TS * KP;                         // [TS][HD]
  float* S = Vs + TS * HD;                          // [n_rep][TS]
  float* ml = S + n_rep * TS;                       // [n_rep][2] running (max, sum)
  float* corr = ml + 2 * n_rep;                     // [n_rep]
  float* mm = corr + n_rep;                         // [n_rep][nsplit]
  const size_t esz = a.kv_half ? 2 : 4;
  const KT* Kp = reinterpret_cast<const KT*>(static_cast<const uint8_t*>(a.kcache) +
                                             size_t(P.layer) * a.kv_layer_elems * esz) +
                 size_t(kh) * a.max_seq * HD;
  const KT* Vp = reinterpret_cast<const KT*>(static_cast<const uint8_t*>(a.vcache) +
                                             size_t(P.layer) * a.kv_layer_elems * esz) +
                 size_t(kh) * a.max_seq * HD;
  const int j0 = split * chunk, j1 = min(j0 + chunk, nkeys);
  constexpr int PER = (TS * HD / 4 + MK_CT - 1) / MK_CT;  // float4 per thread per matrix and tile
  // stages the rows of keys [max(t0, lo), min(t0 + nt, hi)) of the tile at t0
  auto stage = [&](int t0, int nt, int lo, int hi) {
    float4 kv[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int i = tid + e * MK_CT;
      const int row = (i * 4) / HD, key = t0 + row;
      if (i < TS * HD / 4 && row < nt && key >= lo && key < hi) kv[e] = ldcg_kv4<KT>(Kp + size_t(t0) * HD + size_t(i) * 4);
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int i = tid + e * MK_CT;
      const int row = (i * 4) / HD, col = (i * 4) % HD, key = t0 + row;
      if (i < TS * HD / 4 && row < nt && key >= lo && key < hi) {
        float* kr = Ks + row * KP + col;
        kr[0] = kv[e].x;
        kr[1] = kv[e].y;
        kr[2] = kv[e].z;
        kr[3] = kv[e].w;
      }
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int i = tid + e * MK_CT;
      const int row = (i * 4) / HD, key = t0 + row;
      if (i < TS * HD / 4 && row < nt && key >= lo && key < hi) kv[e] = ldcg_kv4<KT>(Vp + size_t(t0) * HD + size_t(i) * 4);
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int i = tid + e * MK_CT;
      const int row = (i * 4) / HD, col = (i * 4) % HD, key = t0 + row;
      if (i < TS * HD / 4 && row < nt && key >= lo && key < hi) *reinterpret_cast<float4*>(Vs + row * HD + col) = kv[e];
    }
  };
  const int nt0 = min(TS, j1 - j0);
  stage(j0, nt0, 0, c.kv_len);  // keys of earlier steps: independent of this step
  if (tid == 0) {
    if (!abort_ && !wait_counter(a.cnt + P.dep * 32, P.dep_target)) {
      atomicOr(&a.st->err, 8);
      sm.flags[0] = 1;
    }
  }
  cbar();
  abort_ = *reinterpret_cast<volatile int*>(sm.flags);
  if (abort_) return;
  for (int i = tid; i < n_rep * HD / 4; i += MK_CT)
    reinterpret_cast<float4*>(qs)[i] = __ldcg(reinterpret_cast<const float4*>(a.q + size_t(kh) * n_rep * HD) + i);
  for (int r = tid; r < n_rep; r += MK_CT) {
    ml[2 * r] = -INFINITY;
    ml[2 * r + 1] = 0.0f;
  }
  stage(j0, nt0, c.kv_len, nkeys);  // this step's key
  constexpr int MAXI = (16 * HD + MK_CT - 1) / MK_CT;  // outputs per thread, n_rep <= 16
  float acc[MAXI];
#pragma unroll
  for (int k = 0; k < MAXI; ++k) acc[k] = 0.0f;
  for (int t0 = j0; t0 < j1; t0 += TS) {
    const int nt = min(TS, j1 - t0);
    if (t0 != j0) {
      cbar();
      stage(t0, nt, 0, nkeys);
    }
    cbar();
    for (int r = warp; r < n_rep; r += MK_CW) {
      float sc = -INFINITY;
      if (lane < nt) {
        float d = 0.0f;
        const float* qr = qs + r * HD;
        const float* kr = Ks + lane * KP;
#pragma unroll 4
        for (int dd = 0; dd < HD; ++dd) d = __fadd_rn(d, __fmul_rn(qr[dd], kr[dd]));
        sc = __fmul_rn(d, a.attn_scale);
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
    cbar();
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {
      const int idx = tid + k * MK_CT;
      if (idx < n_rep * HD) {
        const int r = idx / HD, d = idx % HD;
        float s2 = acc[k] * corr[r];
        for (int jj = 0; jj < nt; ++jj) s2 += S[r * TS + jj] * Vs[jj * HD + d];
        acc[k] = s2;
      }
    }
  }
  cbar();
  int* cnt = a.cnt + P.phase * 32;
  if (nsplit == 1) {
#pragma unroll
    for (int k = 0; k < MAXI; ++k) {
      const int idx = tid + k * MK_CT;
      if (idx < n_rep * HD) {
        const int r = idx / HD, d = idx % HD;
        const float l = ml[2 * r + 1];
        a.att[size_t(kh * n_rep + r) * HD + d] = l > 0.0f ? acc[k] / l : 0.0f;
      }
    }
    cbar();
    if (tid == 0) signal_counter(cnt);
    return;
  }
  const size_t pstride = HD + 2;
  const size_t hstride = size_t(a.max_splits) * pstride;
#pragma unroll
  for (int k = 0; k < MAXI; ++k) {
    const int idx = tid + k * MK_CT;
    if (idx < n_rep * HD) {
      const int r = idx / HD, d = idx % HD;
      float* pp = a.part + size_t(kh * n_rep + r) * hstride + size_t(split) * pstride;
      pp[2 + d] = acc[k];
      if (d == 0) {
        pp[0] = ml[2 * r];
        pp[1] = ml[2 * r + 1];
      }
    }
  }
  cbar();
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(a.ticket + kh, 1);
    sm.flags[1] = prev == nsplit - 1;
  }
  cbar();
  if (!*reinterpret_cast<volatile int*>(sm.flags + 1)) return;
  __threadfence();
  if (tid == 0) a.ticket[kh] = 0;
  const float* pbase = a.part + size_t(kh) * n_rep * hstride;
  for (int i = tid; i < n_rep * nsplit; i += MK_CT) {
    const int r = i / nsplit, sp = i % nsplit;
    mm[r * nsplit + sp] = __ldcg(pbase + r * hstride + sp * pstride);
  }
  cbar();
  for (int r = warp; r < n_rep; r += MK_CW) {
    float M = -INFINITY;
    for (int sp = lane; sp < nsplit; sp += 32) M = fmaxf(M, mm[r * nsplit + sp]);
    M = warp_max(M);
    float L = 0.0f;
    for (int sp = lane; sp < nsplit; sp += 32) {
      const float f = expf(mm[r * nsplit + sp] - M);
      L += __ldcg(pbase + r * hstride + sp * pstride + 1) * f;
      mm[r * nsplit + sp] = f;
    }
    L = warp_sum(L);
    if (lane == 0) ml[2 * r + 1] = L;
  }
  cbar();
  for (int i = tid; i < n_rep * HD; i += MK_CT) {
    const int r = i / HD, d = i % HD;
    const float* pp = pbase + r * hstride + 2 + d;
    float O = 0.0f;
    int sp = 0;
    for (; sp + 4 <= nsplit; sp += 4) {
      const float o0 = __ldcg(pp + (sp + 0) * pstride), o1 = __ldcg(pp + (sp + 1) * pstride);
      const float o2 = __ldcg(pp + (sp + 2) * pstride), o3 = __ldcg(pp + (sp + 3) * pstride);
      O += o0 * mm[r * nsplit + sp] + o1 * mm[r * nsplit + sp + 1] + o2 * mm[r * nsplit + sp + 2] +
           o3 * mm[r * nsplit + sp + 3];
    }
    for (; sp < nsplit; ++sp) O += __ldcg(pp + sp * pstride) * mm[r * nsplit + sp];
    const float L = ml[2 * r + 1];
    a.att[size_t(kh * n_rep + r) * HD + d] = L > 0.0f ? O / L : 0.0f;
  }
  cbar();
  if (tid == 0) signal_counter(cnt);
}

template <int HD>
__device__ void mk_attention_phase(const MkArgs& a, const MkSmem& sm, const MkPart& P, const MkCtx& c,
                                   int& abort_) {
  // split rule: at most max_splits pieces of a multiple of 32 keys, so that
  // n_kv * splits <= grid and every item has a CTA of its own
  const int nkeys = min(c.kv_len + 1, c.position + 1);
  int chunk = (nkeys + a.max_splits - 1) / a.max_splits;
  chunk = max(MK_TS, (chunk + MK_TS - 1) / MK_TS * MK_TS);
  const int nsplit = (nkeys + chunk - 1) / chunk;
  const int item = blockIdx.x;
  if (item >= a.n_kv * nsplit || abort_) return;
  const int kh = item / nsplit, split = item - kh * nsplit;
  if (a.kv_half) mk_attention<HD, __half>(a, sm, P, kh, split, nsplit, chunk, nkeys, c, abort_);
  else mk_attention<HD, float>(a, sm, P, kh, split, nsplit, chunk, nkeys, c, abort_);
}

__global__ void __launch_bounds__(MK_THREADS, 1) decode_step_kernel(const MkArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const MkSmem sm = mk_carve(smem, a);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  StepState* st = a.st;
  if (st->done) return;  // the generate loop has ended: every CTA returns at once
  if (tid == 0) {
    for (int s = 0; s < a.nslots; ++s) {
      mbar_init(sm.full + s, 1);
      mbar_init(sm.empty + s, MK_CW);
    }
    mbar_fence_init();
    sm.flags[0] = 0;
    sm.flags[1] = 0;
  }
  __syncthreads();

  if (warp == MK_CW) {  // ---- producer: this CTA's weight tiles, in consumption order
    if (lane != 0) return;
    int i = 0;
    for (int pi = 0; pi < a.nparts; ++pi) {
      const MkPart P = a.parts[pi];
      if (P.kind == MK_ATT) continue;
      int g0, g1;
      cta_share(P.ngroups, blockIdx.x, gridDim.x, g0, g1);
      const int nt = tiles_of(P, g0, g1);
      for (int t = 0; t < nt; ++t, ++i) {
        const int s = i % a.nslots, use = i / a.nslots;
        if (use > 0 && !mbar_wait(sm.empty + s, uint32_t((use - 1) & 1))) {
          atomicOr(&st->err, 8);  // the consumers stopped taking tiles: stop issuing
          return;
        }
        fence_proxy_async();
        issue_tile(P, tile_at(P, g0, g1, t), sm.slots + size_t(s) * a.slot_bytes, sm.full + s);
      }
    }
    return;
  }

  // ---- consumers
  MkCtx c;
  c.position = st->position;
  c.kv_len = st->kv_len;
  {
    const uint32_t tok = a.gen_mode ? a.hist[st->nhist - 1] : a.ids[0];
    c.x0 = tok < uint32_t(a.vocab) ? a.emb + size_t(tok) * a.hidden : a.zero;  // model.rs:847-864
  }
  c.best = 0ull;
  c.nan = 0;
  int abort_ = 0;
  int i = 0, pp = 0;
  for (int pi = 0; pi < a.nparts; ++pi) {
    const MkPart P = a.parts[pi];
    if (P.kind == MK_ATT) {
      if (a.head_dim == 64) mk_attention_phase<64>(a, sm, P, c, abort_);
      else mk_attention_phase<128>(a, sm, P, c, abort_);
      continue;
    }
    if (P.first) {
      if (P.dep >= 0) {
        if (tid == 0 && !abort_ && !wait_counter(a.cnt + P.dep * 32, P.dep_target)) {
          atomicOr(&st->err, 8);
          sm.flags[0] = 1;
        }
        cbar();
        abort_ = *reinterpret_cast<volatile int*>(sm.flags);
      }
      if (!abort_) {
        const float* in;
        bool cg = true;
        switch (P.kind) {
          case MK_QKV: in = P.layer == 0 ? c.x0 : a.xa; cg = P.layer != 0; break;
          case MK_O: in = a.att; break;
          case MK_GU: in = a.xb; break;
          case MK_D: in = a.act; break;
          default: in = a.xa; break;  // MK_LM
        }
        mk_planes(in, cg, P.norm, P.eps, P.K, carve(sm.region, 1, P.K), sm.red);
      }
    }
    int g0, g1;
    cta_share(P.ngroups, blockIdx.x, gridDim.x, g0, g1);
    const int nt = tiles_of(P, g0, g1);
    for (int t = 0; t < nt; ++t, ++i) {
      const int s = i % a.nslots, use = i / a.nslots;
      const Tile T = tile_at(P, g0, g1, t);
      float* part = sm.part + size_t(pp) * a.part_units * 16;
      if (!mbar_wait(sm.full + s, uint32_t(use & 1))) {
        atomicOr(&st->err, 4);
        sm.flags[0] = 1;
      }
      if (!abort_) {
        if (P.dtype == DT_Q4K) mk_tile_dots<DT_Q4K>(P, T, sm.slots + size_t(s) * a.slot_bytes, sm.region, part);
        else mk_tile_dots<DT_Q6K>(P, T, sm.slots + size_t(s) * a.slot_bytes, sm.region, part);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(sm.empty + s);
      cbar();
      abort_ = *reinterpret_cast<volatile int*>(sm.flags);
      if (!abort_) mk_epilogue(a, P, T, part, sm.gacc, c);
      pp ^= 1;
    }
    if (!P.last) continue;
    if (P.kind != MK_LM) {
      cbar();
      if (tid == 0) signal_counter(a.cnt + P.phase * 32);
      continue;
    }
    // LM head: CTA max of the argmax keys, one atomic per CTA; the last CTA
    // to finish runs the sampler bookkeeping and clears the phase counters
    unsigned long long* rb = reinterpret_cast<unsigned long long*>(sm.red);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ob = __shfl_xor_sync(0xffffffffu, c.best, o);
      c.best = ob > c.best ? ob : c.best;
      c.nan |= __shfl_xor_sync(0xffffffffu, c.nan, o);
    }
    if (lane == 0) {
      rb[warp] = c.best;
      sm.flags[2 + (warp & 3)] = 0;
    }
    cbar();
    if (lane == 0 && c.nan) atomicOr(sm.flags + 2, 1);
    cbar();
    if (tid == 0) {
      unsigned long long b = 0ull;
      for (int w = 0; w < MK_CW; ++w) b = rb[w] > b ? rb[w] : b;
      if (a.gen_mode) {
        if (b) atomicMax(&st->best, b);
        if (sm.flags[2]) atomicOr(&st->nan, 1);
      }
      __threadfence();
      const int prev = atomicAdd(&st->ticket, 1);
      if (prev == int(gridDim.x) - 1) {
        __threadfence();
        for (int ph = 0; ph < a.nphases; ++ph) a.cnt[ph * 32] = 0;
        if (a.gen_mode) finish_sample_state(st, a.hist, a.pen_cnt);
        else st->ticket = 0;
      }
    }
  }
}

int g_mk_sms = 0;
size_t g_mk_smem_max = 0;

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
  return cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(g_mk_smem_max));
}

bool decode_step_plan(MkPart* parts, int nparts, MkArgs& a, int n_rep, size_t* smem) {
  if (g_mk_smem_max == 0) return false;
  if (n_rep > 16 || (a.head_dim != 64 && a.head_dim != 128)) return false;
  int kmax = 0;
  for (int i = 0; i < nparts; ++i)
    if (parts[i].kind != MK_ATT) kmax = std::max(kmax, parts[i].K);
  if (kmax > MK_MAX_K || kmax % QK_K) return false;
  const int grid = decode_step_grid();
  a.max_splits = std::max(1, grid / a.n_kv);
  const size_t att_floats = size_t(n_rep) * a.head_dim + size_t(MK_TS) * (a.head_dim + 1) +
                            size_t(MK_TS) * a.head_dim + size_t(n_rep) * MK_TS + 3 * size_t(n_rep) +
                            size_t(n_rep) * a.max_splits;
  size_t region = std::max(gemv_planes_bytes(1, kmax), att_floats * sizeof(float));
  region = (region + 127) / 128 * 128;
  const int slot = 32 * 1024;
  // tile shapes and the widest tile's unit count
  int units = 1;
  for (int i = 0; i < nparts; ++i) {
    MkPart& P = parts[i];
    if (P.kind == MK_ATT) continue;
    const int nb = P.K / QK_K;
    const size_t bb = dev_block_bytes(P.dtype);
    const size_t group = 4 * size_t(nb) * bb;
    if (group <= size_t(slot)) {
      P.gpt = int(slot / group);
      P.kbt = nb;
    } else {
      P.gpt = 1;
      P.kbt = int(slot / (4 * bb));
    }
    const int nch = P.kbt * 4;
    for (int ng = 1; ng <= P.gpt; ++ng) {
      const int ks = std::max(1, std::min((MK_CW + ng - 1) / ng, nch / 32));
      units = std::max(units, ng * ks);
    }
  }
  const size_t fixed = region + sizeof(float) * 2 * 16 * size_t(units) + sizeof(float) * (16 + 64) + 8 * sizeof(int);
  if (fixed + 2 * (size_t(slot) + 16) > g_mk_smem_max) return false;
  const int nslots = int(std::min<size_t>(8, (g_mk_smem_max - fixed) / (size_t(slot) + 16)));
  a.slot_bytes = slot;
  a.nslots = nslots;
  a.region_bytes = int(region);
  a.part_units = units;
  *smem = size_t(nslots) * slot + fixed + 16 * size_t(nslots);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, MK_THREADS, *smem) != cudaSuccess ||
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_step_kernel, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb
