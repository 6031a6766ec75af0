// Batched greedy decode of independent sequences (the serving path behind
// wcb_generate_batch): the weight contractions of one decode step for B <= 32
// sequences on the 5th-generation tensor cores, plus the small per-sequence
// kernels around them (embedding, sampler).
//
// Contraction (matmul_transposed, gemm.rs:83-143, over the dequantised weights
// of quant.rs:43-261): y[b][n] = sum_k W[n][k] x[b][k]. A Q4_K weight is
// d*sc_s*q - dmin*m_s on sub-block s, so
//     y[b][n] = sum_s ( d*sc_s * sum_{k in s} q[n][k] x[b][k]  -  dmin*m_s * sum_{k in s} x[b][k] )
// and a Q6_K weight is d*sc_s*(q - 32) on 16-value sub-blocks. The quants q are
// small integers, exact in fp16, so the MMA A operand (M = 128 weight rows) is
// the raw quant, unpacked in shared memory with integer ops only; the B operand
// (N = 16 or 32 sequences) is the activation split into fp16 hi + lo halves, so
// q*hi + q*lo carries ~22 significant bits of x. Each sub-block accumulates
// into its own TMEM columns (fp32); the CUDA cores read them back with
// tcgen05.ld and apply the per-row, per-sub-block scales in fp32.
//
// Work split: a CTA owns one 128-row tile and a slice of the K super-blocks.
// Raw blocks stream into a 2-deep shared-memory ring with cp.async (16-byte,
// coalesced along each row); weights are static, so the first two super-blocks
// are requested before the PDL wait on the previous kernel. The last CTA of a
// tile (atomic ticket) sums the slices in slice order and runs the fused
// epilogue: residual add (+ per-tile sums of squares for the next RMSNorm),
// SwiGLU (ffn.rs:90-94), or RoPE + KV append per sequence (attention.rs:140-162).
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cmath>

#include "device_common.cuh"
#include "kernels.h"

namespace wcb {
namespace {

constexpr int BD_THREADS = 128;
constexpr int BD_STEP = 128;                    // K values per MMA round (half a super-block)
constexpr int BD_A_BYTES = BATCH_TILE * BD_STEP * 2;  // fp16 A tile of one round (32 KB)
constexpr int BD_LBO_A = (BATCH_TILE / 8) * 128;       // next 8-column K chunk of A (2048 B)

// shared-memory carve-up of one CTA (NB = MMA N)
template <int NB>
struct BdLayout {
  static constexpr int X_BYTES = NB * BD_STEP * 2;      // one fp16 half of the activations
  static constexpr int A_OFF = 0;
  static constexpr int XH_OFF = A_OFF + BD_A_BYTES;
  static constexpr int XL_OFF = XH_OFF + X_BYTES;
  static constexpr int XS_OFF = XL_OFF + X_BYTES;           // float [4][NB] Q4_K sub-block sums of x
  static constexpr int CS_OFF = XS_OFF + 4 * NB * 4;        // float [NB][16] sums of 8-value chunks
  static constexpr int RM_OFF = CS_OFF + NB * 16 * 4;       // float [NB] RMSNorm divisors
  static constexpr int SI_OFF = RM_OFF + NB * 4;            // int [3][NB] position, KV slot, done
  static constexpr int EX_OFF = SI_OFF + 3 * NB * 4;        // float [64][NB] epilogue exchange
  static constexpr int BAR_OFF = EX_OFF + 64 * NB * 4;      // mbarrier of the MMAs
  static constexpr int TS_OFF = BAR_OFF + 8;                // TMEM base address
  static constexpr int RAW_OFF = (TS_OFF + 4 + 127) / 128 * 128;  // [2][128][block bytes] ring
  static constexpr int TMEM_COLS = 8 * NB;                  // 8 sub-block accumulators of NB columns
};

template <int NB>
constexpr size_t bd_smem(int block_bytes) {
  return size_t(BdLayout<NB>::RAW_OFF) + size_t(2) * BATCH_TILE * block_bytes;
}

// byte offset of element (row, k) in a K-major, no-swizzle operand tile whose
// 8-column K chunks are lbo bytes apart (core matrices of 8 rows x 16 bytes)
__device__ __forceinline__ int op_off(int row, int k, int lbo) {
  return (k >> 3) * lbo + (row >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2;
}

// SM100 shared-memory matrix descriptor: K-major, no swizzle
__device__ __forceinline__ uint64_t bd_desc(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFF);
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((128u >> 4) & 0x3FFF) << 32;  // next 8-row group
  d |= uint64_t(1) << 46;                     // descriptor version for sm_100
  return d;
}

// instruction descriptor: f16 x f16 -> f32, both K-major, M = 128, N = NB
template <int NB>
__host__ __device__ constexpr uint32_t bd_idesc() {
  return (1u << 4) | (uint32_t(NB >> 3) << 17) | (uint32_t(BATCH_TILE >> 4) << 24);
}

template <int NB>
__device__ __forceinline__ void bd_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(bd_idesc<NB>()), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void bd_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// NB consecutive fp32 TMEM columns of this thread's lane
template <int NB>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[NB]);

template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// four quants (bytes 0..3 of w, each < 2048 - bias) as two fp16 pairs q - bias:
// 0x6400 | q is the fp16 value 1024 + q, so one subtraction gives q - bias exactly
__device__ __forceinline__ void quads_to_half(uint32_t w, __half2 bias, uint32_t& lo, uint32_t& hi) {
  uint32_t a = __byte_perm(w, 0x64u, 0x4140);
  uint32_t b = __byte_perm(w, 0x64u, 0x4342);
  __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias);
  __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
  lo = *reinterpret_cast<uint32_t*>(&ha);
  hi = *reinterpret_cast<uint32_t*>(&hb);
}


// weight row r (0..127) of tile `tile` in the virtual matrix (rows past the end
// are clamped to the last row: loaded, never stored)
__device__ __forceinline__ const uint8_t* bd_row(const BatchGemmArgs& a, int epi, int tile, int r, size_t row_bytes) {
  if (epi == BEPI_SWIGLU) {
    const int g = min(tile * (BATCH_TILE / 2) + (r & 63), a.rows - 1);
    return a.seg[r >> 6].w + size_t(g) * row_bytes;
  }
  int v = min(tile * BATCH_TILE + r, a.rows - 1), sg = 0;
  while (sg < a.nseg - 1 && v >= a.seg[sg].rows) v -= a.seg[sg++].rows;
  return a.seg[sg].w + size_t(v) * row_bytes;
}

__device__ __forceinline__ int bd_tile_dtype(const BatchGemmArgs& a, int epi, int tile) {
  if (epi == BEPI_SWIGLU) return a.seg[0].dtype;
  int v = tile * BATCH_TILE, sg = 0;
  while (sg < a.nseg - 1 && v >= a.seg[sg].rows) v -= a.seg[sg++].rows;
  return a.seg[sg].dtype;
}

template <int NB>
__global__ void __launch_bounds__(BD_THREADS) bgemm_kernel(const BatchGemmArgs a, const int epi) {
  using L = BdLayout<NB>;
  constexpr uint32_t LBO_X = (NB / 8) * 128;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* At = sm + L::A_OFF;
  uint8_t* Xh = sm + L::XH_OFF;
  uint8_t* Xl = sm + L::XL_OFF;
  float* xs = reinterpret_cast<float*>(sm + L::XS_OFF);
  float* cs = reinterpret_cast<float*>(sm + L::CS_OFF);
  float* rm = reinterpret_cast<float*>(sm + L::RM_OFF);
  int* si = reinterpret_cast<int*>(sm + L::SI_OFF);
  float* ex = reinterpret_cast<float*>(sm + L::EX_OFF);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L::TS_OFF);
  uint8_t* raw = sm + L::RAW_OFF;
  __shared__ const uint8_t* rp[BATCH_TILE];  // this tile's weight rows
  __shared__ int s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int nsb = a.K / QK_K;
  const int sb0 = split * a.sb_per_split;
  const int nloc = min(nsb, sb0 + a.sb_per_split) - sb0;
  const int tdt = bd_tile_dtype(a, epi, tile);
  const bool q4 = tdt == DT_Q4K;
  const int bb = q4 ? Q4K_BYTES : Q6K_DEV_BYTES;
  const size_t row_bytes = size_t(nsb) * bb;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(L::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  rp[tid] = bd_row(a, epi, tile, tid, row_bytes);
  // the padding sequences (b >= B) stay zero in both activation halves
  for (int i = tid; i < 2 * L::X_BYTES / 16; i += BD_THREADS)
    reinterpret_cast<uint4*>(Xh)[i] = make_uint4(0u, 0u, 0u, 0u);
  pdl_trigger();
  __syncthreads();
  const int chunks = bb / 16;
  auto load_sb = [&](int j) {  // super-block j of the slice into ring slot j & 1
    uint8_t* dst = raw + (j & 1) * BATCH_TILE * bb;
    const size_t src_off = size_t(sb0 + j) * bb;
    for (int c = tid; c < BATCH_TILE * chunks; c += BD_THREADS) {
      const int r = c / chunks, pc = c - r * chunks;
      cp_async16(dst + r * bb + pc * 16, rp[r] + src_off + pc * 16);
    }
  };
  load_sb(0);
  cp_async_commit();
  if (nloc > 1) load_sb(1);
  cp_async_commit();
  pdl_wait();  // activations, norms and sequence states come from earlier kernels
  if (tid < a.B) {
    const StepState* st = a.st + tid;
    si[tid] = st->position;
    si[NB + tid] = st->kv_len;
    si[2 * NB + tid] = st->done;
    if (a.norm_w) {  // x / sqrt(mean(x^2) + eps) * w (candle_tensor_backend.rs:30-57)
      float tot = 0.0f;
      for (int t = 0; t < a.sq_tiles; ++t) tot = __fadd_rn(tot, a.sq_in[t * a.B + tid]);
      rm[tid] = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(a.K)), a.eps));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane_tmem = tmem + (uint32_t(warp * 32) << 16);

  float acc[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
  bool ok = true;
  uint32_t phase = 0;
  for (int j = 0; j < nloc; ++j) {
    cp_async_wait<1>();
    __syncthreads();  // every thread's copies of super-block j have landed
    const uint8_t* blk = raw + (j & 1) * BATCH_TILE * bb + tid * bb;  // this thread's row
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      const int kg = (sb0 + j) * QK_K + h * BD_STEP;
      // (1) the row's 128 quants of this round as fp16 integers, and its sub-block scales
      float d1[8], m1[4];
      if (q4) {
        const uint4 hd = *reinterpret_cast<const uint4*>(blk);
        const float d = half_bits(hd.x & 0xFFFFu), dmin = half_bits(hd.x >> 16);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t sc, mn;
          scale_min(4 * h + u, hd.y, hd.z, hd.w, sc, mn);
          d1[u] = __fmul_rn(d, float(sc));
          m1[u] = __fmul_rn(dmin, float(mn));
        }
        const __half2 bias = __float2half2_rn(1024.0f);
#pragma unroll
        for (int p = 0; p < 2; ++p) {  // sub-block pair 2h+p: low nibbles = sub-block 2p, high = 2p+1
          const uint8_t* qs = blk + 16 + 32 * (2 * h + p);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint2 q8 = *reinterpret_cast<const uint2*>(qs + 8 * w);
            uint4 lo, hi;
            quads_to_half(q8.x & 0x0F0F0F0Fu, bias, lo.x, lo.y);
            quads_to_half(q8.y & 0x0F0F0F0Fu, bias, lo.z, lo.w);
            quads_to_half((q8.x >> 4) & 0x0F0F0F0Fu, bias, hi.x, hi.y);
            quads_to_half((q8.y >> 4) & 0x0F0F0F0Fu, bias, hi.z, hi.w);
            *reinterpret_cast<uint4*>(At + op_off(tid, 64 * p + 8 * w, BD_LBO_A)) = lo;
            *reinterpret_cast<uint4*>(At + op_off(tid, 64 * p + 32 + 8 * w, BD_LBO_A)) = hi;
          }
        }
      } else {  // Q6_K half h: value 32g + l = ql nibble | 2 bits of qh (quant.rs:206-261)
        const float d = half_bits(uint32_t(blk[208]) | (uint32_t(blk[209]) << 8));
        const int8_t* scv = reinterpret_cast<const int8_t*>(blk + 192 + 8 * h);
#pragma unroll
        for (int u = 0; u < 8; ++u) d1[u] = __fmul_rn(d, float(scv[u]));
        const uint8_t* ql = blk + 64 * h;
        const uint8_t* qh = blk + 128 + 32 * h;
        const __half2 bias = __float2half2_rn(1056.0f);  // 1024 + the Q6_K offset 32
#pragma unroll
        for (int l8 = 0; l8 < 4; ++l8) {
          const uint2 a0 = *reinterpret_cast<const uint2*>(ql + 8 * l8);
          const uint2 a1 = *reinterpret_cast<const uint2*>(ql + 32 + 8 * l8);
          const uint2 hb = *reinterpret_cast<const uint2*>(qh + 8 * l8);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint2 src = (g & 1) ? a1 : a0;
            const int sh = g < 2 ? 0 : 4;
            const uint32_t q0 = ((src.x >> sh) & 0x0F0F0F0Fu) | (((hb.x >> (2 * g)) & 0x03030303u) << 4);
            const uint32_t q1 = ((src.y >> sh) & 0x0F0F0F0Fu) | (((hb.y >> (2 * g)) & 0x03030303u) << 4);
            uint4 o;
            quads_to_half(q0, bias, o.x, o.y);
            quads_to_half(q1, bias, o.z, o.w);
            *reinterpret_cast<uint4*>(At + op_off(tid, 32 * g + 8 * l8, BD_LBO_A)) = o;
          }
        }
      }
      // (2) the activations of this round (RMSNorm applied), split into fp16 hi + lo
      for (int i = tid; i < NB * 16; i += BD_THREADS) {
        const int b = i % NB, kc = i / NB;
        if (b >= a.B) continue;
        const float* xr = a.x + size_t(b) * a.ldx + kg + 8 * kc;
        const float4 f0 = *reinterpret_cast<const float4*>(xr);
        const float4 f1 = *reinterpret_cast<const float4*>(xr + 4);
        float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
        if (a.norm_w) {
          const float* nw = a.norm_w + kg + 8 * kc;
          const float m = rm[b];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fdiv_rn(v[e], m), nw[e]);
        }
        __half hv[8], lv[8];
        float sum = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          hv[e] = __float2half_rn(v[e]);
          lv[e] = __float2half_rn(__fsub_rn(v[e], __half2float(hv[e])));
          sum = __fadd_rn(sum, v[e]);
        }
        const int off = op_off(b, 8 * kc, LBO_X);
        *reinterpret_cast<uint4*>(Xh + off) = *reinterpret_cast<const uint4*>(hv);
        *reinterpret_cast<uint4*>(Xl + off) = *reinterpret_cast<const uint4*>(lv);
        cs[b * 16 + kc] = sum;
      }
      fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
      tc_fence_before();
      __syncthreads();
      // (3) one thread issues the MMAs: sub-block u accumulates into columns u*NB..
      if (tid == 0) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(At), xh0 = smem_u32(Xh), xl0 = smem_u32(Xl);
        const int nsub = q4 ? 4 : 8, kper = q4 ? 2 : 1;  // 16-value MMA steps per sub-block
        for (int u = 0; u < nsub; ++u) {
          for (int kk = 0; kk < kper; ++kk) {
            const uint32_t c16 = uint32_t(u * kper + kk);
            const uint64_t ad = bd_desc(a0 + c16 * 2 * BD_LBO_A, BD_LBO_A);
            bd_mma<NB>(tmem + uint32_t(u * NB), ad, bd_desc(xh0 + c16 * 2 * LBO_X, LBO_X), kk > 0 ? 1u : 0u);
            bd_mma<NB>(tmem + uint32_t(u * NB), ad, bd_desc(xl0 + c16 * 2 * LBO_X, LBO_X), 1u);
          }
        }
        bd_commit(bar);
      }
      if (q4 && tid < 4 * NB) {  // sums of x over each 32-value sub-block (the dmin*m term)
        const int u = tid / NB, b = tid % NB;
        const float* c = cs + b * 16 + 4 * u;
        xs[u * NB + b] = __fadd_rn(__fadd_rn(__fadd_rn(c[0], c[1]), c[2]), c[3]);
      }
      __syncthreads();
      // (4) accumulators -> scaled into this row's running sums
      ok &= mbar_wait(bar, phase);
      phase ^= 1u;
      tc_fence_after();
      if (q4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float v[NB];
          tmem_ld<NB>(lane_tmem + uint32_t(u * NB), v);
#pragma unroll
          for (int b = 0; b < NB; ++b) acc[b] += d1[u] * v[b] - m1[u] * xs[u * NB + b];
        }
      } else {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float v[NB];
          tmem_ld<NB>(lane_tmem + uint32_t(u * NB), v);
#pragma unroll
          for (int b = 0; b < NB; ++b) acc[b] += d1[u] * v[b];
        }
      }
      tc_fence_before();
    }
    if (j + 2 < nloc) load_sb(j + 2);  // every thread is past its reads of slot j & 1
    cp_async_commit();
  }
  cp_async_wait<0>();
  const bool all_ok = __syncthreads_and(ok);
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS));
  }
  if (!all_ok) {  // a bounded wait expired: report it, store nothing
    if (tid == 0) atomicOr(&a.st[0].err, 4);
    return;
  }

  // K slices: the last CTA of the tile sums them in slice order
  if (a.splits > 1) {
    const size_t P = size_t(gridDim.x) * BATCH_TILE;  // slice row stride
    float* pp = a.part + size_t(split) * a.B * P + size_t(tile) * BATCH_TILE + tid;
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if (b < a.B) pp[size_t(b) * P] = acc[b];
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.ticket + tile, 1) == a.splits - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid == 0) a.ticket[tile] = 0;
    const float* p0 = a.part + size_t(tile) * BATCH_TILE + tid;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b >= a.B) continue;
      float s2 = 0.0f;
      for (int sp = 0; sp < a.splits; ++sp) s2 = __fadd_rn(s2, __ldcg(p0 + (size_t(sp) * a.B + b) * P));
      acc[b] = s2;
    }
  }

  if (epi == BEPI_SWIGLU) {  // ffn.rs:90-94: g * (1 / (1 + exp(-g))) * u
    if (tid >= 64) {
#pragma unroll
      for (int b = 0; b < NB; ++b) ex[(tid - 64) * NB + b] = acc[b];
    }
    __syncthreads();
    const int r = tile * (BATCH_TILE / 2) + tid;
    if (tid < 64 && r < a.rows) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b >= a.B) continue;
        const float gv = acc[b], uv = ex[tid * NB + b];
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
        a.y[size_t(b) * a.ldy + r] = __fmul_rn(__fmul_rn(gv, sig), uv);
      }
    }
    return;
  }
  const int n = tile * BATCH_TILE + tid;
  const bool valid = n < a.rows;
  if (epi == BEPI_STORE) {
    if (valid) {
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (b < a.B) a.y[size_t(b) * a.ldy + n] = acc[b];
    }
    return;
  }
  if (epi == BEPI_RESID) {  // layer.rs:68 / :86, and the sums of squares of the new stream
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float v = 0.0f;
      if (valid && b < a.B) {
        v = __fadd_rn(a.resid[size_t(b) * a.ldr + n], acc[b]);
        a.y[size_t(b) * a.ldy + n] = v;
      }
      const float s2 = warp_sum(__fmul_rn(v, v));
      if (lane == 0) ex[warp * NB + b] = s2;
    }
    __syncthreads();
    if (tid < a.B)
      a.sq_out[tile * a.B + tid] =
          __fadd_rn(__fadd_rn(__fadd_rn(ex[tid], ex[NB + tid]), ex[2 * NB + tid]), ex[3 * NB + tid]);
    return;
  }
  // BEPI_QKV: RoPE on (2i, 2i+1) pairs of q and k (attention.rs:230-262), the
  // pair's other value from the neighbouring lane; K / V appended at each
  // sequence's KV slot (kv_cache.rs:44-67)
  float other[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) other[b] = __shfl_xor_sync(0xffffffffu, acc[b], 1);
  if (!valid) return;
  const int hd = a.head_dim;
  const int* pos = si;
  const int* slot = si + NB;
  const int* done = si + 2 * NB;
  if (n < a.hidden + a.kv_dim) {
    const int col = n < a.hidden ? n : n - a.hidden;
    const int pi = (col % hd) >> 1;
    const bool odd = n & 1;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b >= a.B) continue;
      const float cs_ = a.rope_cos[size_t(pos[b]) * (hd / 2) + pi];
      const float sn_ = a.rope_sin[size_t(pos[b]) * (hd / 2) + pi];
      const float x0 = odd ? other[b] : acc[b], x1 = odd ? acc[b] : other[b];
      const float r = odd ? __fadd_rn(__fmul_rn(x0, sn_), __fmul_rn(x1, cs_))
                          : __fsub_rn(__fmul_rn(x0, cs_), __fmul_rn(x1, sn_));
      if (n < a.hidden) {
        a.q[size_t(b) * a.ldq + n] = r;
      } else if (!done[b]) {
        const size_t off = size_t(b) * a.seq_stride + (size_t(col / hd) * a.max_seq + slot[b]) * hd + col % hd;
        if (a.kv_half) reinterpret_cast<__half*>(a.kc)[off] = __float2half_rn(r);
        else reinterpret_cast<float*>(a.kc)[off] = r;
      }
    }
  } else {
    const int col = n - a.hidden - a.kv_dim;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b >= a.B || done[b]) continue;
      const size_t off = size_t(b) * a.seq_stride + (size_t(col / hd) * a.max_seq + slot[b]) * hd + col % hd;
      if (a.kv_half) reinterpret_cast<__half*>(a.vc)[off] = __float2half_rn(acc[b]);
      else reinterpret_cast<float*>(a.vc)[off] = acc[b];
    }
  }
}

__global__ void bembed_kernel(const float* emb, int vocab, int hidden, const StepState* st, const uint32_t* hist,
                              int hist_cap, float* x, float* sq) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  const int nh = st[b].nhist;
  const uint32_t id = hist[size_t(b) * hist_cap + (nh > 0 ? nh - 1 : 0)];
  const float* row = id < uint32_t(vocab) ? emb + size_t(id) * hidden : nullptr;  // unknown id: zeros
  float s2 = 0.0f;
  for (int d = tid * 4; d < hidden; d += blockDim.x * 4) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row) v = *reinterpret_cast<const float4*>(row + d);
    *reinterpret_cast<float4*>(x + size_t(b) * hidden + d) = v;
    s2 = __fadd_rn(s2, __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                                 __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w))));
  }
  __shared__ float red[32];
  s2 = warp_sum(s2);
  if ((tid & 31) == 0) red[tid >> 5] = s2;
  __syncthreads();
  if (tid == 0) {
    float t = 0.0f;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) t = __fadd_rn(t, red[w]);
    sq[b] = t;
  }
}

// LogitsProcessor::sample for temperature 0 (sampling.rs:57-125) on sequence b:
// repetition penalty once per occurrence, argmax with the last maximum winning,
// then generate()'s bookkeeping (model.rs:1380-1409)
__global__ void bsample_kernel(const float* logits, int vocab, StepState* st, uint32_t* hist, int hist_cap,
                               uint32_t* pen_cnt, float rep) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  StepState* s = st + b;
  if (s->done) return;
  const float* lg = logits + size_t(b) * vocab;
  uint32_t* pc = pen_cnt + size_t(b) * vocab;
  unsigned long long best = 0ull;
  int nan = 0;
  for (int n = tid; n < vocab; n += blockDim.x) {
    float pv = lg[n];
    if (rep != 1.0f) {
      const uint32_t cnt = pc[n];
      for (uint32_t k = 0; k < cnt; ++k) pv = pv > 0.0f ? __fdiv_rn(pv, rep) : __fmul_rn(pv, rep);
    }
    if (pv != pv) nan = 1;
    else {
      const unsigned long long key = (static_cast<unsigned long long>(order_key(pv)) << 32) | uint32_t(n);
      best = key > best ? key : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
    nan |= __shfl_xor_sync(0xffffffffu, nan, o);
  }
  __shared__ unsigned long long s_best[32];
  __shared__ int s_nan[32];
  if ((tid & 31) == 0) {
    s_best[tid >> 5] = best;
    s_nan[tid >> 5] = nan;
  }
  __syncthreads();
  if (tid == 0) {
    unsigned long long bb = 0ull;
    int nn = 0;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) {
      bb = s_best[w] > bb ? s_best[w] : bb;
      nn |= s_nan[w];
    }
    s->best = bb;
    s->nan = nn;
    finish_sample_state(s, hist + size_t(b) * hist_cap, pc);
  }
}

int g_bd_sms = 0;

template <typename Kern, typename... Args>
cudaError_t bd_launch(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace

int batch_gemm_tiles(const BatchGemmArgs& a, int epi) {
  const int per = epi == BEPI_SWIGLU ? BATCH_TILE / 2 : BATCH_TILE;
  return (a.rows + per - 1) / per;
}

void batch_gemm_plan(BatchGemmArgs& a, int epi) {
  if (g_bd_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&g_bd_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_bd_sms <= 0)
      g_bd_sms = 148;
  }
  const int tiles = batch_gemm_tiles(a, epi), nsb = a.K / QK_K;
  bool q6 = false;
  for (int i = 0; i < a.nseg; ++i) q6 |= a.seg[i].dtype == DT_Q6K;
  const int target = (q6 ? 1 : 2) * g_bd_sms;  // resident CTAs of one wave
  int splits = std::min(nsb, std::max(1, (target + tiles - 1) / tiles));
  const int per = (nsb + splits - 1) / splits;
  a.sb_per_split = per;
  a.splits = (nsb + per - 1) / per;
}

cudaError_t batch_configure() {
  cudaError_t e = cudaFuncSetAttribute(bgemm_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(bd_smem<16>(Q6K_DEV_BYTES)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(bgemm_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(bd_smem<32>(Q6K_DEV_BYTES)));
  return e;
}

cudaError_t launch_batch_gemm(BatchGemmArgs a, int epi, cudaStream_t s) {
  if (a.B < 1 || a.B > BATCH_MAX || a.K % QK_K != 0 || a.rows < 1) return cudaErrorInvalidValue;
  batch_gemm_plan(a, epi);
  int bb = Q4K_BYTES;
  for (int i = 0; i < a.nseg; ++i)
    if (a.seg[i].dtype == DT_Q6K) bb = Q6K_DEV_BYTES;
  const dim3 grid(batch_gemm_tiles(a, epi), a.splits);
  cudaError_t e;
  if (a.B <= 16) e = bd_launch(bgemm_kernel<16>, grid, dim3(BD_THREADS), bd_smem<16>(bb), s, a, epi);
  else e = bd_launch(bgemm_kernel<32>, grid, dim3(BD_THREADS), bd_smem<32>(bb), s, a, epi);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_batch_embed(const float* emb, int vocab, int hidden, const StepState* st, const uint32_t* hist,
                               int hist_cap, float* x, float* sq, int B, cudaStream_t s) {
  if (hidden % 4 != 0) return cudaErrorInvalidValue;
  const cudaError_t e = bd_launch(bembed_kernel, dim3(B), dim3(256), 0, s, emb, vocab, hidden, st, hist, hist_cap, x, sq);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_batch_sample(const float* logits, int vocab, StepState* st, uint32_t* hist, int hist_cap,
                                uint32_t* pen_cnt, float rep, int B, cudaStream_t s) {
  const cudaError_t e =
      bd_launch(bsample_kernel, dim3(B), dim3(512), 0, s, logits, vocab, st, hist, hist_cap, pen_cnt, rep);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb
