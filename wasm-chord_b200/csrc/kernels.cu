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

#include <algorithm>
#include <cfloat>
#include <cmath>

#include "device_common.cuh"
#include "kernels.h"

namespace wcb {

namespace {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
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

__device__ void finish_sample(const GemvArgs& a) { finish_sample_state(a.st, a.hist, a.pen_cnt_w); }


// Fused epilogue of output j (= row i * M + token t) of row group g: v is the
// output, fin the group's 16 values (SwiGLU pairs a gate row with its up row,
// RoPE a row with the next). Shared by the quantised and the dense GEMV.
template <int M, int EPI>
__device__ __forceinline__ void gemv_out(const GemvArgs& a, int g, int j, float v, const float* fin,
                                         unsigned long long& best, int& nan) {
  const int i = j / M, t = j % M;
  const int tok = t;  // column within this launch
  if (EPI == EPI_PEER) {
    const int n = ROWS * g + i;
    const unsigned long long w =
        (static_cast<unsigned long long>(uint32_t(a.st->epoch) * 512u + uint32_t(a.peer_phase) + 1u) << 32) |
        __float_as_uint(v);
    for (int r = 0; r < a.tp_size; ++r)  // one 64-bit store per rank: value and tag arrive together
      asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(a.peers[r] + size_t(a.tp_rank) * a.ldy + n),
                   "l"(w)
                   : "memory");
  } else if (EPI == EPI_STORE) {
    a.y[size_t(tok) * a.ldy + ROWS * g + i] = v;
  } else if (EPI == EPI_RESID) {
    const size_t off = size_t(tok) * a.ldy + ROWS * g + i;
    a.y[off] = __fadd_rn(a.resid[size_t(tok) * a.ldr + ROWS * g + i], v);
  } else if (EPI == EPI_SWIGLU) {
    if (i < 2) {
      const float gv = v, uv = fin[(i + 2) * M + t];
      // ffn.rs:90-94: sigmoid = 1/(1+exp(-g)); silu = g*sigmoid; g = silu*u
      const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
      a.y[size_t(tok) * a.ldy + 2 * g + i] = __fmul_rn(__fmul_rn(gv, sig), uv);
    }
  } else if (EPI == EPI_LMHEAD) {
    const int n = ROWS * g + i;
    const int tok_id = a.vocab_off + n;  // rows of this launch start at token vocab_off
    a.y[n] = v;
    if (a.gen_mode) {
      float pv = v;
      if (a.rep != 1.0f) {  // apply_repetition_penalty: once per occurrence (sampling.rs:86-103)
        const uint32_t cnt = a.pen_cnt[tok_id];
        for (uint32_t k = 0; k < cnt; ++k) pv = pv > 0.0f ? __fdiv_rn(pv, a.rep) : __fmul_rn(pv, a.rep);
      }
      if (pv != pv) nan = 1;
      else {
        const unsigned long long key = (static_cast<unsigned long long>(order_key(pv)) << 32) | uint32_t(tok_id);
        best = key > best ? key : best;
      }
    }
  } else {  // EPI_QKV
    const int vr = a.row_offset + ROWS * g + i;
    const int gtok = a.token_offset + tok;
    const int pos = a.st->position + gtok;
    const int slot_kv = a.st->kv_len + gtok;
    const int hd = a.head_dim;
    if (vr < a.hidden + a.kv_dim) {
      // RoPE on (2i, 2i+1) pairs (attention.rs:230-262), cos/sin from the table
      if ((i & 1) == 0) {
        const float x0 = v, x1 = fin[(i + 1) * M + t];
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
          const size_t off = (size_t(kh) * a.max_seq + slot_kv) * hd + dd;
          if (a.kv_half) {
            reinterpret_cast<__half*>(a.kc)[off] = __float2half_rn(n0);
            reinterpret_cast<__half*>(a.kc)[off + 1] = __float2half_rn(n1);
          } else {
            reinterpret_cast<float*>(a.kc)[off] = n0;
            reinterpret_cast<float*>(a.kc)[off + 1] = n1;
          }
        }
      }
    } else {
      const int col = vr - a.hidden - a.kv_dim;
      const int kh = col / hd, dd = col % hd;
      const size_t off = (size_t(kh) * a.max_seq + slot_kv) * hd + dd;
      if (a.kv_half) reinterpret_cast<__half*>(a.vc)[off] = __float2half_rn(v);
      else reinterpret_cast<float*>(a.vc)[off] = v;
    }
  }
}

// End of an LM-head launch in generate mode: CTA-wide max of the argmax keys,
// one atomic per CTA; the last CTA to finish runs the sampler bookkeeping (no
// CTA ever waits for another). GEMV_THREADS threads.
__device__ __forceinline__ void lmhead_reduce(const GemvArgs& a, unsigned long long best, int nan) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
  if (tid == 0) {
    unsigned long long b = 0ull;
    int n = 0;
    for (int w = 0; w < GEMV_WARPS; ++w) {
      b = s_best[w] > b ? s_best[w] : b;
      n |= s_nan[w];
    }
    if (b) atomicMax(&a.st->best, b);
    if (n) atomicOr(&a.st->nan, 1);
    if (a.gen_mode == 1) {  // mode 2: the key is reduced over ranks before the bookkeeping
      __threadfence();
      const int prev = atomicAdd(&a.st->ticket, 1);
      if (prev == int(gridDim.x) - 1) {
        __threadfence();
        finish_sample(a);
      }
    }
  }
}

// Dense weights (GGUF F32 / F16, gguf.rs:446-467, stored as read): y = x W^T for
// M <= 4 activation rows with the fused epilogues of the quantised GEMV. A CTA
// takes two row groups (8 rows) at a time, one warp per weight row; the lanes
// stride over 16-byte pieces of the row (coalesced) and read the activations
// through L1, normalised on the fly as candle's rms_norm does (x / m * w, m =
// sqrt(sum(x^2)/K + eps)). The dot products are fp32 like the reference's
// matmul_transposed (gemm.rs:83-143), in a different order.
template <int M, int PRO, int EPI, int DT>
__global__ void __launch_bounds__(GEMV_THREADS) dense_gemv_kernel(const GemvArgs a) {
  __shared__ float s_fin[2][16];
  __shared__ float s_part[GEMV_WARPS];
  __shared__ float s_m[4];
  pdl_trigger();
  pdl_wait();
  if (a.st && a.st->done) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K;
  if (PRO == PRO_RMSNORM) {
    for (int t = 0; t < M; ++t) {
      const float* x = a.x + size_t(t) * a.ldx;
      float ss = 0.0f;
      for (int k = tid; k < K; k += GEMV_THREADS) ss = __fadd_rn(ss, __fmul_rn(x[k], x[k]));
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
  }
  constexpr int EPL = DT == DT_F32 ? 4 : 8;  // values in one 16-byte piece
  const size_t row_bytes = size_t(K) * (DT == DT_F32 ? 4 : 2);
  unsigned long long best = 0ull;
  int nan = 0;
  for (int gb = 2 * int(blockIdx.x); gb < a.ngroups; gb += 2 * int(gridDim.x)) {
    const int gl = warp >> 2, i = warp & 3, g = gb + gl;
    if (g < a.ngroups) {
      const uint8_t* row;
      if (EPI == EPI_SWIGLU) {
        row = a.seg[i < 2 ? 0 : 1].w + size_t(2 * g + (i & 1)) * row_bytes;  // gate rows, then up rows
      } else {
        int vr = ROWS * g + i, sg = 0;
        while (sg + 1 < a.nseg && vr >= a.seg[sg].rows) vr -= a.seg[sg++].rows;
        row = a.seg[sg].w + size_t(vr) * row_bytes;
      }
      float acc[M];
#pragma unroll
      for (int t = 0; t < M; ++t) acc[t] = 0.0f;
      for (int c = lane; c < K / EPL; c += 32) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row) + c);
        float w[EPL];
        if (DT == DT_F32) {
          w[0] = __uint_as_float(u.x);
          w[1] = __uint_as_float(u.y);
          w[2] = __uint_as_float(u.z);
          w[3] = __uint_as_float(u.w);
        } else {
          const uint32_t h[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[e]));
            w[(2 * e) % EPL] = f.x;
            w[(2 * e + 1) % EPL] = f.y;
          }
        }
        const int k = c * EPL;
#pragma unroll
        for (int t = 0; t < M; ++t) {
          const float* x = a.x + size_t(t) * a.ldx + k;
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            float xv = __ldg(x + e);
            if (PRO == PRO_RMSNORM) xv = __fmul_rn(__fdiv_rn(xv, s_m[t]), __ldg(a.norm_w + k + e));
            acc[t] = fmaf(w[e], xv, acc[t]);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < M; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0) s_fin[gl][i * M + t] = v;
      }
    }
    __syncthreads();
    if (tid < 32) {
      const int gl2 = tid >> 4, j = tid & 15, g2 = gb + gl2;
      if (g2 < a.ngroups && j < ROWS * M) gemv_out<M, EPI>(a, g2, j, s_fin[gl2][j], s_fin[gl2], best, nan);
    }
    __syncthreads();
  }
  if (EPI == EPI_LMHEAD && a.gen_mode) lmhead_reduce(a, best, nan);
}

// Shared-memory layout of one GEMV CTA (sizes from the host, GemvArgs):
//   [slot 0][slot 1]   weight stages: stage_groups groups of 4 rows, raw blocks
//   [planes]           activation limbs (XPlanes)
//   [part]             per-unit partial sums  (stage_groups * ksplit * 16 floats)
//   [fin]              per-group final sums   (stage_groups * 16 floats)
//   [bar]              two mbarriers
struct GemvSmem {
  uint8_t* slot[2];
  XPlanes p;
  float* part;
  float* fin;
  uint64_t* bar;
};

__device__ __forceinline__ GemvSmem gemv_carve(uint8_t* smem, const GemvArgs& a, int M) {
  GemvSmem g;
  g.slot[0] = smem;
  g.slot[1] = smem + a.slot_bytes;
  uint8_t* q = smem + 2 * size_t(a.slot_bytes);
  g.p = carve(q, M, a.K);
  q += gemv_planes_bytes(M, a.K);
  g.part = reinterpret_cast<float*>(q);
  q += sizeof(float) * size_t(a.stage_groups) * a.ksplit * 16;
  g.fin = reinterpret_cast<float*>(q);
  q += sizeof(float) * size_t(a.stage_groups) * 16;
  g.bar = reinterpret_cast<uint64_t*>(q);
  return g;
}

// Issues the bulk copies of stage `stage` (groups [gs, ge) of this CTA) into
// slot `slot`: one copy per contiguous row range (per segment, or the gate and
// the up rows of SwiGLU pairs).
template <int EPI>
__device__ void issue_stage(const GemvArgs& a, const GemvSmem& sm, int slot, int gs, int ge, size_t row_bytes) {
  uint64_t* bar = sm.bar + slot;
  const int ng = ge - gs;
  uint8_t* dst = sm.slot[slot];
  if (EPI == EPI_SWIGLU) {
    const uint32_t bytes = uint32_t(2 * ng * row_bytes);
    mbar_expect_tx(bar, 2 * bytes);
    bulk_g2s(dst, a.seg[0].w + size_t(2 * gs) * row_bytes, bytes, bar);
    bulk_g2s(dst + bytes, a.seg[1].w + size_t(2 * gs) * row_bytes, bytes, bar);
    return;
  }
  mbar_expect_tx(bar, uint32_t(4 * ng * row_bytes));
  int r0 = ROWS * gs;
  const int r1 = ROWS * ge;
  int base = 0;
  for (int sg = 0; sg < a.nseg && r0 < r1; ++sg) {
    const int s0 = base, s1 = base + a.seg[sg].rows;
    base = s1;
    if (r0 >= s1) continue;
    const int e = min(r1, s1);
    const uint32_t bytes = uint32_t(size_t(e - r0) * row_bytes);
    bulk_g2s(dst, a.seg[sg].w + size_t(r0 - s0) * row_bytes, bytes, bar);
    dst += bytes;
    r0 = e;
  }
}

// Fused dequant-GEMV. The grid is at most one wave; CTA c owns row groups
// [c*G/grid, (c+1)*G/grid). Its weights stream through two shared-memory
// stages with TMA bulk copies; the first two stages are issued before the
// kernel waits on its predecessor (programmatic dependent launch), so weight
// traffic overlaps the previous kernel. Warps take (row group, K slice) units.
template <int M, int PRO, int EPI, int DT>
__global__ void __launch_bounds__(GEMV_THREADS, M == 1 ? 2 : 1) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K;
  const GemvSmem sm = gemv_carve(smem, a, M);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KS = a.ksplit;
  const int NB = K / QK_K;
  constexpr int BB = DT == DT_Q4K ? Q4K_BYTES : Q6K_DEV_BYTES;
  const size_t row_bytes = size_t(NB) * BB;
  const int NC = NB * 4;  // 64-value chunks per row
  const int g_begin = int((long long)blockIdx.x * a.ngroups / gridDim.x);
  const int g_end = int((long long)(blockIdx.x + 1) * a.ngroups / gridDim.x);
  const int SG = a.stage_groups;
  const int nstages = (g_end - g_begin + SG - 1) / SG;

  if (tid == 0) {
    mbar_init(sm.bar + 0, 1);
    mbar_init(sm.bar + 1, 1);
    mbar_fence_init();
    for (int st = 0; st < 2 && st < nstages; ++st)
      issue_stage<EPI>(a, sm, st, g_begin + st * SG, min(g_end, g_begin + (st + 1) * SG), row_bytes);
  }
  pdl_trigger();
  pdl_wait();
  if (a.st && a.st->done) {
    // wait (bounded) for the copies issued above before the CTA retires
    if (tid == 0)
      for (int st = 0; st < 2 && st < nstages; ++st) mbar_wait(sm.bar + st, 0);
    return;
  }
  build_planes<M, PRO>(a, sm.p);  // ends with __syncthreads (the barrier init is visible too)

  unsigned long long best = 0ull;
  int nan = 0;
  for (int st = 0; st < nstages; ++st) {
    const int slot = st & 1;
    const int gs = g_begin + st * SG, ge = min(g_end, gs + SG), ng = ge - gs;
    const bool ok = mbar_wait(sm.bar + slot, uint32_t((st >> 1) & 1));
    if (__syncthreads_or(!ok)) {  // a copy never landed: report, give the other slot a bounded wait, stop
      if (tid == 0) {
        if (a.st) atomicOr(&a.st->err, 4);
        mbar_wait(sm.bar + (slot ^ 1), uint32_t((st >> 1) & 1));
      }
      return;
    }
    const uint8_t* sbase = sm.slot[slot];
    const uint32_t sbase_a = smem_u32(sbase);
    XAddr xad;
    xad.l[0] = smem_u32(sm.p.l0);
    xad.l[1] = smem_u32(sm.p.l1);
    xad.l[2] = smem_u32(sm.p.l2);
    xad.scale = smem_u32(sm.p.scale);
    xad.sum32 = smem_u32(sm.p.sum32);
    const int units = ng * KS;
    for (int u = warp; u < units; u += GEMV_WARPS) {
      const int gl = u / KS, ks = u % KS;
      const uint8_t* rw[ROWS];
#pragma unroll
      for (int i = 0; i < ROWS; ++i) {
        if (EPI == EPI_SWIGLU)
          rw[i] = sbase + size_t((i < 2 ? 0 : 2 * ng) + 2 * gl + (i & 1)) * row_bytes;
        else
          rw[i] = sbase + size_t(ROWS * gl + i) * row_bytes;
      }
      float acc[ROWS][M];
#pragma unroll
      for (int i = 0; i < ROWS; ++i)
#pragma unroll
        for (int t = 0; t < M; ++t) acc[i][t] = 0.0f;
      const int c1 = (ks + 1) * NC / KS;
      if (DT == DT_Q4K) {
        uint32_t ra[ROWS];
#pragma unroll
        for (int i = 0; i < ROWS; ++i) ra[i] = sbase_a + uint32_t(rw[i] - sbase);
        for (int c = ks * NC / KS + lane; c < c1; c += 32) q4k_chunk_rows<M>(ra, c, K, xad, acc);
      } else {
        for (int c = ks * NC / KS + lane; c < c1; c += 32) {
#pragma unroll
          for (int i = 0; i < ROWS; ++i) q6k_chunk_smem<M>(rw[i], c, K, sm.p, acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < ROWS; ++i)
#pragma unroll
        for (int t = 0; t < M; ++t) {
          const float v = warp_sum(acc[i][t]);
          if (lane == i * M + t) sm.part[u * 16 + lane] = v;
        }
    }
    __syncthreads();
    // fixed-order sum of the K slices of every (group, output)
    for (int o = tid; o < ng * 16; o += GEMV_THREADS) {
      const int gl = o >> 4, j = o & 15;
      float v = 0.0f;
      if (j < ROWS * M)
        for (int k = 0; k < KS; ++k) v += sm.part[(gl * KS + k) * 16 + j];
      sm.fin[o] = v;
    }
    __syncthreads();
    for (int o = tid; o < ng * 16; o += GEMV_THREADS) {
      const int gl = o >> 4, j = o & 15;
      if (j >= ROWS * M) continue;
      gemv_out<M, EPI>(a, gs + gl, j, sm.fin[o], sm.fin + gl * 16, best, nan);
    }
    __syncthreads();  // the slot, part and fin are free again
    if (tid == 0 && st + 2 < nstages) {
      fence_proxy_async();
      issue_stage<EPI>(a, sm, slot, g_begin + (st + 2) * SG, min(g_end, g_begin + (st + 3) * SG), row_bytes);
    }
  }
  if (EPI == EPI_LMHEAD && a.gen_mode) lmhead_reduce(a, best, nan);
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

// dynamic shared memory a GEMV CTA may use: the device's per-block opt-in
// limit less 2 KB for the kernel's static shared memory
size_t g_smem_max = 200 * 1024;

template <int M, int PRO, int EPI, int DT>
cudaError_t configure_gemv_t() {
  return cudaFuncSetAttribute(gemv_kernel<M, PRO, EPI, DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(g_smem_max));
}

// Grid, stage size and K split of one launch: a single wave of CTAs (two per
// SM when two double-buffered stages fit in half of the shared memory).
template <int DT>
size_t plan_gemv(GemvArgs& a, int M, int* grid) {
  const int NB = a.K / QK_K;
  const size_t row_bytes = size_t(NB) * (DT == DT_Q4K ? Q4K_BYTES : Q6K_DEV_BYTES);
  const size_t group_bytes = ROWS * row_bytes;
  const size_t planes = gemv_planes_bytes(M, a.K);
  const int sms = g_sms > 0 ? g_sms : 148;
  const int NC = NB * 4;
  for (int per_sm = 2; per_sm >= 1; --per_sm) {
    const size_t budget = per_sm == 2 ? 108 * 1024 : g_smem_max;
    const int G = std::min(a.ngroups, sms * per_sm);
    const int gpc = (a.ngroups + G - 1) / G;
    const size_t extra = sizeof(float) * 9 * 16 + 64;  // part + fin per group (KS <= 8) + barriers
    if (planes + 2 * (group_bytes + extra) > budget && per_sm == 2) continue;
    int SG = int((budget - planes) / (2 * group_bytes + extra));
    SG = std::max(1, std::min(SG, gpc));
    int ks = 1;
    while (ks < 8 && SG * ks * 2 <= 8 && NC / (ks * 2) >= 16) ks *= 2;
    a.ksplit = ks;
    a.stage_groups = SG;
    a.slot_bytes = int((SG * group_bytes + 127) / 128 * 128);
    *grid = G;
    return 2 * size_t(a.slot_bytes) + planes + sizeof(float) * size_t(SG) * ks * 16 + sizeof(float) * SG * 16 + 16;
  }
  return 0;
}

template <int M, int PRO, int EPI, int DT>
cudaError_t launch_gemv_t(const GemvArgs& a0, cudaStream_t s) {
  GemvArgs a = a0;
  int grid = 0;
  const size_t smem = plan_gemv<DT>(a, M, &grid);
  if (smem == 0 || smem > g_smem_max) return cudaErrorInvalidValue;
  const cudaError_t e =
      launch_ex(gemv_kernel<M, PRO, EPI, DT>, dim3(grid), dim3(GEMV_THREADS), smem, s, a.pdl != 0, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

#define WCB_GEMV_CASES(F)   \
  F(PRO_NONE, EPI_STORE)    \
  F(PRO_NONE, EPI_PEER)     \
  F(PRO_NONE, EPI_RESID)    \
  F(PRO_RMSNORM, EPI_QKV)   \
  F(PRO_RMSNORM, EPI_SWIGLU) \
  F(PRO_RMSNORM, EPI_STORE) \
  F(PRO_RMSNORM, EPI_LMHEAD)

template <int M, int P, int E, int DT>
cudaError_t launch_dense_t(const GemvArgs& a, cudaStream_t s) {
  const int grid = std::max(1, std::min((a.ngroups + 1) / 2, 4 * (g_sms > 0 ? g_sms : 148)));
  const cudaError_t e = launch_ex(dense_gemv_kernel<M, P, E, DT>, dim3(grid), dim3(GEMV_THREADS), 0, s, a.pdl != 0, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int M>
cudaError_t launch_gemv_m(const GemvArgs& a, int pro, int epi, cudaStream_t s) {
  const int dt = a.seg[0].dtype;
  if (dt == DT_F32 || dt == DT_F16) {  // dense weights
#define WCB_DENSE_CASE(P, E)                                                  \
  if (pro == P && epi == E)                                                   \
    return dt == DT_F32 ? launch_dense_t<M, P, E, DT_F32>(a, s) : launch_dense_t<M, P, E, DT_F16>(a, s);
    WCB_GEMV_CASES(WCB_DENSE_CASE)
#undef WCB_DENSE_CASE
    return cudaErrorInvalidValue;
  }
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
  float* mm = corr + n_rep;        // [n_rep][max_splits] split maxima, then merge weights
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
  // merge: running max / sum of every (head, split) staged in shared memory first,
  // then each (head, dim) output reads its nsplit partial sums with independent loads
  const size_t hstride = size_t(a.max_splits) * pstride;
  const float* pbase = a.part + (size_t(t) * a.n_heads + size_t(kh) * n_rep) * hstride;
  for (int i = tid; i < n_rep * nsplit; i += ATT_THREADS) {
    const int r = i / nsplit, sp = i % nsplit;
    mm[r * nsplit + sp] = __ldcg(pbase + r * hstride + sp * pstride);
  }
  __syncthreads();
  for (int r = warp; r < n_rep; r += ATT_WARPS) {
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
  __syncthreads();
  for (int i = tid; i < n_rep * HD; i += ATT_THREADS) {
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
  st->epoch += 1;  // tags of this forward's partial sums (tensor parallelism)
}

__global__ void add_kernel(float* dst, const float* a, const float* b, size_t n, const StepState* st) {
  if (st && st->done) return;
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    dst[i] = __fadd_rn(a[i], b[i]);
}

__global__ void tp_reduce_add_kernel(float* dst, const float* resid, const unsigned long long* recv, int tp, size_t n,
                                     int phase, StepState* st) {
  if (st->done) return;
  const uint32_t tag = uint32_t(st->epoch) * 512u + uint32_t(phase) + 1u;
  const unsigned long long limit_ns = 1000000ull * unsigned(st->wait_ms > 0 ? st->wait_ms : 2000);
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    float sum = 0.0f;
    for (int r = 0; r < tp; ++r) {
      const unsigned long long* p = recv + size_t(r) * n + i;
      unsigned long long w;
      asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
      if (uint32_t(w >> 32) != tag) {
        unsigned long long t0;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        while (true) {
          asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
          if (uint32_t(w >> 32) == tag) break;
          unsigned long long t1;
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
          // a rank stopped: report it, end this step (later kernels see done and
          // return at once) and let every other waiting thread give up too
          if (t1 - t0 > limit_ns) {
            atomicOr(&st->err, 16);
            st->done = 1;
            break;
          }
          if (*reinterpret_cast<volatile int*>(&st->err) & 16) break;
        }
      }
      sum = __fadd_rn(sum, __uint_as_float(uint32_t(w)));
    }
    dst[i] = __fadd_rn(resid[i], sum);
  }
}

__global__ void tp_pack_key_kernel(StepState* st, unsigned long long* key) {
  key[0] = st->best;
  key[1] = st->nan ? 1ull : 0ull;
}

__global__ void tp_finish_kernel(StepState* st, const unsigned long long* key, uint32_t* hist, uint32_t* pen_cnt) {
  if (st->done) return;
  st->best = key[0];
  st->nan = key[1] ? 1 : 0;
  finish_sample_state(st, hist, pen_cnt);
  st->epoch += 1;  // tags of the next step's partial sums
}

__global__ void tp_key_exchange_kernel(StepState* st, unsigned long long* const* peers, const unsigned long long* own,
                                       int rank, int tp, size_t key_off, uint32_t* hist, uint32_t* pen_cnt) {
  if (st->done) return;
  const unsigned long long tag = (unsigned long long)(uint32_t(st->epoch) * 512u + 512u) << 32;
  const unsigned long long best = st->best;
  const uint32_t hi = uint32_t(best >> 32), lo = (uint32_t(best) & 0x7FFFFFFFu) | (st->nan ? 0x80000000u : 0u);
  for (int r = 0; r < tp; ++r) {  // one 64-bit store per word: value and tag arrive together
    unsigned long long* p = peers[r] + key_off + 2 * size_t(rank);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(tag | hi) : "memory");
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p + 1), "l"(tag | lo) : "memory");
  }
  const unsigned long long limit_ns = 1000000ull * unsigned(st->wait_ms > 0 ? st->wait_ms : 2000);
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  unsigned long long kmax = 0;
  int nan = 0;
  for (int r = 0; r < tp; ++r) {
    const unsigned long long* p = own + key_off + 2 * size_t(r);
    unsigned long long a, b;
    while (true) {
      asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
      asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(b) : "l"(p + 1) : "memory");
      if ((a >> 32) == (tag >> 32) && (b >> 32) == (tag >> 32)) break;
      unsigned long long t1;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
      if (t1 - t0 > limit_ns) {  // a rank stopped: report it and end the step
        atomicOr(&st->err, 16);
        st->done = 1;
        return;
      }
    }
    const unsigned long long k = ((a & 0xFFFFFFFFull) << 32) | (b & 0x7FFFFFFFull);
    kmax = k > kmax ? k : kmax;
    nan |= int((b >> 31) & 1u);
  }
  st->best = kmax;
  st->nan = nan;
  finish_sample_state(st, hist, pen_cnt);
  st->epoch += 1;  // tags of the next step's partial sums
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


int gemv_max_cols(int K) {
  for (int m = 4; m > 1; --m)
    if (gemv_planes_bytes(m, K) <= 64 * 1024) return m;
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
                                       size_t(n_rep) * ATT_TILE + 3 * size_t(n_rep) +
                                       (a.max_splits > 1 ? size_t(n_rep) * a.max_splits : 0));
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
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

cudaError_t launch_add(float* dst, const float* a, const float* b, size_t n, const StepState* st, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const unsigned grid = unsigned(std::min<size_t>((n + 255) / 256, 1184));
  add_kernel<<<grid, 256, 0, s>>>(dst, a, b, n, st);
  return cudaGetLastError();
}

cudaError_t launch_tp_reduce_add(float* dst, const float* resid, const unsigned long long* recv, int tp_size,
                                 size_t n, int phase, StepState* st, cudaStream_t s) {
  const unsigned grid = unsigned(std::min<size_t>((n + 255) / 256, 148));
  tp_reduce_add_kernel<<<grid, 256, 0, s>>>(dst, resid, recv, tp_size, n, phase, st);
  return cudaGetLastError();
}

cudaError_t launch_tp_pack_key(StepState* st, unsigned long long* key, cudaStream_t s) {
  tp_pack_key_kernel<<<1, 1, 0, s>>>(st, key);
  return cudaGetLastError();
}

cudaError_t launch_tp_finish(StepState* st, const unsigned long long* key, uint32_t* hist, uint32_t* pen_cnt,
                             cudaStream_t s) {
  tp_finish_kernel<<<1, 1, 0, s>>>(st, key, hist, pen_cnt);
  return cudaGetLastError();
}

cudaError_t launch_tp_key_exchange(StepState* st, unsigned long long* const* peers, const unsigned long long* own,
                                   int tp_rank, int tp_size, size_t key_off, uint32_t* hist, uint32_t* pen_cnt,
                                   cudaStream_t s) {
  tp_key_exchange_kernel<<<1, 1, 0, s>>>(st, peers, own, tp_rank, tp_size, key_off, hist, pen_cnt);
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
  int optin = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e == cudaSuccess) g_smem_max = size_t(optin) - 2048;
  if (e == cudaSuccess) e = configure_gemv_m<1>();
  if (e == cudaSuccess) e = configure_gemv_m<2>();
  if (e == cudaSuccess) e = configure_gemv_m<3>();
  if (e == cudaSuccess) e = configure_gemv_m<4>();
  const int att_max = int(std::min<size_t>(g_smem_max, 200 * 1024));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_kernel<64, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, att_max);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_kernel<64, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize, att_max);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_kernel<128, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, att_max);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_kernel<128, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize, att_max);
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
