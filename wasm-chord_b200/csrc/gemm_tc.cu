// Q4_K / Q6_K prefill GEMM on the 5th-generation tensor cores (tcgen05).
//
// y[t][n] = sum_k x[t][k] * W[n][k] for T >= 16 tokens: the dense contraction
// of the prefill (matmul_transposed, gemm.rs:83-143, over the dequantised
// weights of quant.rs:58-261). One CTA computes a 128-token x 128-row tile.
// Per 64-value K block, 128 threads dequantise 128 weight rows with the
// reference formula (d*sc*q - dmin*m in f32, no contraction) and 128 threads
// load 128 activation rows (RMSNorm applied on the fly when requested); both
// are split into fp16 hi + lo halves and written to shared memory in the
// canonical K-major core-matrix layout. One elected thread issues
// tcgen05.mma (kind::f16, M=128, N=128, K=16) for hi*hi + hi*lo + lo*hi into a
// TMEM accumulator (fp32), so the products carry ~22 significant bits, and
// commits to an mbarrier that frees the double-buffered stage. The epilogue
// reads TMEM with tcgen05.ld and applies the same fused epilogues as the GEMV
// (residual add, SwiGLU pairs, RoPE + KV-cache write).
#include <cuda_fp16.h>

#include <cfloat>
#include <cmath>

#include "kernels.h"

namespace wcb {
namespace {

constexpr int TC_THREADS = 256;
constexpr int TILE_T = 128;  // tokens (MMA M)
constexpr int TILE_N = 128;  // weight rows (MMA N)
constexpr int KB = 64;       // K per stage
constexpr int CORE_BYTES = 128;                 // 8 rows x 16 bytes
constexpr int SBO = CORE_BYTES;                 // next 8-row group
constexpr int LBO = (TILE_T / 8) * CORE_BYTES;  // next 8-column K chunk (2048 B)
constexpr int TILE_BYTES = TILE_T * KB * 2;     // one 128 x 64 fp16 operand (16 KB)

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ float halfbits(uint32_t b) { return __half2float(__ushort_as_half((unsigned short)b)); }

// byte offset of element (row, k) of a 128 x 64 K-major tile
__device__ __forceinline__ int tile_off(int row, int k) {
  return (k >> 3) * LBO + (row >> 3) * SBO + (row & 7) * 16 + (k & 7) * 2;
}

// SM100 shared-memory matrix descriptor: K-major, no swizzle
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFF);
  d |= uint64_t((LBO >> 4) & 0x3FFF) << 16;
  d |= uint64_t((SBO >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;  // descriptor version for sm_100
  return d;                // base offset 0, legacy LBO mode, layout type 0 (no swizzle)
}

// instruction descriptor: f16 x f16 -> f32, both K-major, M = 128, N = 128
constexpr uint32_t IDESC = (1u << 4) | (uint32_t(TILE_N >> 3) << 17) | (uint32_t(TILE_T >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void bar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_addr(bar);
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

__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
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

__device__ __forceinline__ void split_store(uint8_t* hi_tile, uint8_t* lo_tile, int row, int k0, const float (&v)[8]) {
  __half h[8], l[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    h[e] = __float2half_rn(v[e]);
    l[e] = __float2half_rn(v[e] - __half2float(h[e]));
  }
  const int off = tile_off(row, k0);
  *reinterpret_cast<uint4*>(hi_tile + off) = *reinterpret_cast<const uint4*>(h);
  *reinterpret_cast<uint4*>(lo_tile + off) = *reinterpret_cast<const uint4*>(l);
}

// the three 16-byte words of a Q4_K block that 64 values [64*kq, 64*kq+64) need
struct Q4Raw {
  uint4 hd, qa, qb;
};
__device__ __forceinline__ Q4Raw q4k_raw(const uint8_t* blk, int kq) {
  Q4Raw r;
  r.hd = *reinterpret_cast<const uint4*>(blk);
  r.qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * kq);
  r.qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * kq);
  return r;
}

// 64 dequantised values [64*kq, 64*kq+64) of a Q4_K block (quant.rs:58-115)
__device__ __forceinline__ void deq_q4k_64(const Q4Raw& raw, int kq, float (&w)[64]) {
  const uint4 hd = raw.hd, qa = raw.qa, qb = raw.qb;
  const float d = halfbits(hd.x & 0xFFFFu), dmin = halfbits(hd.x >> 16);
  const uint8_t* sc = reinterpret_cast<const uint8_t*>(&hd) + 4;
  uint32_t s0, m0, s1, m1;
  const int j0 = 2 * kq, j1 = 2 * kq + 1;
  if (j0 < 4) {
    s0 = sc[j0] & 63; m0 = sc[j0 + 4] & 63;
    s1 = sc[j1] & 63; m1 = sc[j1 + 4] & 63;
  } else {
    s0 = (sc[j0 + 4] & 0xF) | ((sc[j0 - 4] >> 6) << 4); m0 = (sc[j0 + 4] >> 4) | ((sc[j0] >> 6) << 4);
    s1 = (sc[j1 + 4] & 0xF) | ((sc[j1 - 4] >> 6) << 4); m1 = (sc[j1 + 4] >> 4) | ((sc[j1] >> 6) << 4);
  }
  const float d1 = __fmul_rn(d, float(s0)), mm1 = __fmul_rn(dmin, float(m0));
  const float d2 = __fmul_rn(d, float(s1)), mm2 = __fmul_rn(dmin, float(m1));
  const uint8_t* q = reinterpret_cast<const uint8_t*>(&qa);
  const uint8_t* q2 = reinterpret_cast<const uint8_t*>(&qb);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const uint32_t b = j < 16 ? q[j] : q2[j - 16];
    w[j] = __fsub_rn(__fmul_rn(d1, float(b & 0xF)), mm1);
    w[32 + j] = __fsub_rn(__fmul_rn(d2, float(b >> 4)), mm2);
  }
}

// the 32 values of sub-block 2*kq + half of a Q4_K block: the low (half 0) or high
// (half 1) nibbles of the pair's 32 quant bytes, exactly as deq_q4k_64 computes them
__device__ __forceinline__ void deq_q4k_32(const Q4Raw& raw, int kq, int half, float (&w)[32]) {
  const uint4 hd = raw.hd, qa = raw.qa, qb = raw.qb;
  const float d = halfbits(hd.x & 0xFFFFu), dmin = halfbits(hd.x >> 16);
  const uint8_t* sc = reinterpret_cast<const uint8_t*>(&hd) + 4;
  const int j = 2 * kq + half;
  uint32_t s0, m0;
  if (j < 4) {
    s0 = sc[j] & 63; m0 = sc[j + 4] & 63;
  } else {
    s0 = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4); m0 = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
  const float d1 = __fmul_rn(d, float(s0)), mm1 = __fmul_rn(dmin, float(m0));
  const uint8_t* q = reinterpret_cast<const uint8_t*>(&qa);
  const uint8_t* q2 = reinterpret_cast<const uint8_t*>(&qb);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint32_t b = i < 16 ? q[i] : q2[i - 16];
    w[i] = __fsub_rn(__fmul_rn(d1, float(half ? (b >> 4) : (b & 0xF))), mm1);
  }
}

// 64 dequantised values [64*kq, 64*kq+64) of a padded Q6_K block (quant.rs:206-261)
__device__ __forceinline__ void deq_q6k_64(const uint8_t* blk, int kq, float (&w)[64]) {
  const float d = halfbits(uint32_t(blk[208]) | (uint32_t(blk[209]) << 8));
#pragma unroll 8
  for (int j = 0; j < 64; ++j) {
    const int v = 64 * kq + j;
    const int hh = v / 128, r = v % 128, k = r / 32, l = r % 32;
    const uint8_t* ql = blk + 64 * hh;
    const uint8_t* qh = blk + 128 + 32 * hh;
    const int8_t* s = reinterpret_cast<const int8_t*>(blk + 192) + 8 * hh;
    const int lo = (k & 1) ? ql[l + 32] : ql[l];
    const int nib = (k < 2) ? (lo & 0xF) : (lo >> 4);
    const int qv = (nib | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
    w[j] = __fmul_rn(__fmul_rn(d, float(s[l / 16 + 2 * k])), float(qv));
  }
}

// 32 dequantised values [64*kq + 32*half, +32) of a padded Q6_K block
__device__ __forceinline__ void deq_q6k_32(const uint8_t* blk, int kq, int half, float (&w)[32]) {
  const float d = halfbits(uint32_t(blk[208]) | (uint32_t(blk[209]) << 8));
#pragma unroll 8
  for (int j = 0; j < 32; ++j) {
    const int v = 64 * kq + 32 * half + j;
    const int hh = v / 128, r = v % 128, k = r / 32, l = r % 32;
    const uint8_t* ql = blk + 64 * hh;
    const uint8_t* qh = blk + 128 + 32 * hh;
    const int8_t* s = reinterpret_cast<const int8_t*>(blk + 192) + 8 * hh;
    const int lo = (k & 1) ? ql[l + 32] : ql[l];
    const int nib = (k < 2) ? (lo & 0xF) : (lo >> 4);
    const int qv = (nib | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
    w[j] = __fmul_rn(__fmul_rn(d, float(s[l / 16 + 2 * k])), float(qv));
  }
}

__device__ __forceinline__ void expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

template <int DT>
__device__ __forceinline__ const uint8_t* weight_row(const GemvArgs& a, int r, int epi, size_t row_bytes) {
  // r: row within the virtual (concatenated or gate/up interleaved) weight
  if (epi == EPI_SWIGLU) return a.seg[r & 1].w + size_t(r >> 1) * row_bytes;
  int sg = 0;
  while (sg < a.nseg - 1 && r >= a.seg[sg].rows) r -= a.seg[sg++].rows;
  return a.seg[sg].w + size_t(r) * row_bytes;
}

// XP: the activation tiles come prepared (fp16 hi / lo, core-matrix layout, the
// RMSNorm weight applied) from stage_x_kernel and are fetched with two bulk copies
// per K block, and all 256 threads dequantise weights (two per row, 32 values
// each); otherwise threads 128..255 stage the activations themselves.
template <int PRO, int EPI, int DT, bool XP>
__global__ void __launch_bounds__(TC_THREADS, 1) gemm_tc_kernel(const GemvArgs a, const float* row_m) {
  extern __shared__ __align__(1024) uint8_t tsm[];
  // [buf][A_hi, A_lo, B_hi, B_lo] tiles, then the MMA and activation-load mbarriers and the TMEM address
  uint8_t* tiles = tsm;
  uint64_t* bar = reinterpret_cast<uint64_t*>(tsm + 2 * 4 * TILE_BYTES);
  uint64_t* bar_a = bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K, NB = K / QK_K;
  const size_t row_bytes = size_t(NB) * (DT == DT_Q4K ? Q4K_BYTES : Q6K_DEV_BYTES);
  const int t0 = blockIdx.y * TILE_T;
  const int r0 = blockIdx.x * TILE_N;  // first virtual weight row of the tile
  const int total_rows = a.ngroups * 4;
  const int nkb = K / KB;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(TILE_N));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    bar_init(bar);
    bar_init(bar + 1);
    bar_init(bar_a);
    bar_init(bar_a + 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  // the weight thread's first block, then each next one requested before the current is used
  const int wr = XP ? (tid & (TILE_N - 1)) : tid;  // weight row of this thread
  const int wh = XP ? (tid >> 7) : 0;               // XP: which 32 of the block's 64 values
  Q4Raw wraw{};
  const uint8_t* wrow = nullptr;
  if (DT == DT_Q4K && (XP || tid < TILE_N) && r0 + wr < total_rows) {
    wrow = weight_row<DT>(a, r0 + wr, EPI, row_bytes);
    wraw = q4k_raw(wrow, 0);
  }
  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb >= 2) ok &= bar_wait(bar + buf, uint32_t(((kb - 2) >> 1) & 1));
    uint8_t* Ahi = tiles + (buf * 4 + 0) * TILE_BYTES;
    uint8_t* Alo = tiles + (buf * 4 + 1) * TILE_BYTES;
    uint8_t* Bhi = tiles + (buf * 4 + 2) * TILE_BYTES;
    uint8_t* Blo = tiles + (buf * 4 + 3) * TILE_BYTES;
    if (XP) {
      if (tid == 0) {  // the buffer's previous MMAs are done: fetch this block's activation tiles
        const uint8_t* src = a.xprep + (size_t(blockIdx.y) * nkb + kb) * 2 * TILE_BYTES;
        expect_tx(bar_a + buf, 2 * TILE_BYTES);
        bulk_load(Ahi, src, TILE_BYTES, bar_a + buf);
        bulk_load(Alo, src + TILE_BYTES, TILE_BYTES, bar_a + buf);
      }
      const int r = r0 + wr;
      float w[32];
      if (r < total_rows) {
        const uint8_t* row = weight_row<DT>(a, r, EPI, row_bytes);
        const int b = (kb * KB) / QK_K, kq = (kb * KB / 64) & 3;
        if (DT == DT_Q4K) {
          deq_q4k_32(wraw, kq, wh, w);
          if (kb + 1 < nkb) {
            const int b1 = ((kb + 1) * KB) / QK_K, kq1 = ((kb + 1) * KB / 64) & 3;
            wraw = q4k_raw(wrow + size_t(b1) * Q4K_BYTES, kq1);
          }
        } else {
          deq_q6k_32(row + size_t(b) * Q6K_DEV_BYTES, kq, wh, w);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = 0.0f;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = w[8 * c + e];
        split_store(Bhi, Blo, wr, 32 * wh + 8 * c, v);
      }
    } else if (tid < TILE_N) {  // weight row tid of the tile
      const int r = r0 + tid;
      float w[64];
      if (r < total_rows) {
        const uint8_t* row = weight_row<DT>(a, r, EPI, row_bytes);
        const int b = (kb * KB) / QK_K, kq = (kb * KB / 64) & 3;
        if (DT == DT_Q4K) {
          deq_q4k_64(wraw, kq, w);
          if (kb + 1 < nkb) {
            const int b1 = ((kb + 1) * KB) / QK_K, kq1 = ((kb + 1) * KB / 64) & 3;
            wraw = q4k_raw(wrow + size_t(b1) * Q4K_BYTES, kq1);
          }
        } else {
          deq_q6k_64(row + size_t(b) * Q6K_DEV_BYTES, kq, w);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) w[j] = 0.0f;
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = w[8 * c + e];
        split_store(Bhi, Blo, tid, 8 * c, v);
      }
    } else {  // activation row (token) tid - 128
      const int rl = tid - TILE_N, t = t0 + rl;
      float xv[64];
      if (t < a.M) {
        const float* xr = a.x + size_t(t) * a.ldx + kb * KB;
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
          const float4 f = *reinterpret_cast<const float4*>(xr + j);
          xv[j] = f.x; xv[j + 1] = f.y; xv[j + 2] = f.z; xv[j + 3] = f.w;
        }
        if (PRO == PRO_RMSNORM) {  // x = h / m * w (candle_tensor_backend.rs:30-57): h * w staged
          // here, the per-token 1/m applied to the sums (sum W (h w / m) = (1/m) sum W (h w))
          const float* nw = a.norm_w + kb * KB;
#pragma unroll
          for (int j = 0; j < 64; ++j) xv[j] = __fmul_rn(xv[j], nw[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) xv[j] = 0.0f;
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = xv[8 * c + e];
        split_store(Ahi, Alo, rl, 8 * c, v);
      }
    }
    fence_async_smem();
    fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      if (XP) ok &= bar_wait(bar_a + buf, uint32_t((kb >> 1) & 1));  // the activation tiles landed
      fence_after_sync();
      const uint32_t ah = smem_addr(Ahi), al = smem_addr(Alo), bh = smem_addr(Bhi), bl = smem_addr(Blo);
#pragma unroll
      for (int ks = 0; ks < KB / 16; ++ks) {
        const uint32_t koff = uint32_t(2 * ks * LBO);
        const uint32_t acc0 = (kb > 0 || ks > 0) ? 1u : 0u;
        mma_f16(tmem, make_desc(ah + koff), make_desc(bh + koff), acc0);
        mma_f16(tmem, make_desc(ah + koff), make_desc(bl + koff), 1u);
        mma_f16(tmem, make_desc(al + koff), make_desc(bh + koff), 1u);
      }
      mma_commit(bar + buf);
    }
  }
  ok &= bar_wait(bar + ((nkb - 1) & 1), uint32_t(((nkb - 1) >> 1) & 1));
  fence_after_sync();
  if (!ok && tid == 0 && a.st) atomicOr(&a.st->err, 4);

  // epilogue: warp w reads TMEM lanes 32*(w%4) .. +32 (tokens), columns 64*(w/4) .. +64 (rows)
  const int rl = 32 * (warp & 3) + lane;
  const int t = t0 + rl;
  const int cbase = 64 * (warp >> 2);
#pragma unroll 1
  for (int c16 = 0; c16 < 64; c16 += 16) {
    float v[16];
    tmem_ld16(tmem + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(cbase + c16), v);
    if (!ok || t >= a.M) continue;
    if (PRO == PRO_RMSNORM) {
      const float m = row_m[t];
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = __fdiv_rn(v[e], m);
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int r = r0 + cbase + c16 + e;  // virtual weight row
      if (r >= total_rows) continue;
      const float val = v[e];
      const int tok = t;
      if (EPI == EPI_STORE) {
        a.y[size_t(tok) * a.ldy + r] = val;
      } else if (EPI == EPI_RESID) {
        a.y[size_t(tok) * a.ldy + r] = __fadd_rn(a.resid[size_t(tok) * a.ldr + r], val);
      } else if (EPI == EPI_SWIGLU) {
        if ((e & 1) == 0) {  // columns (2i, 2i+1) = (gate, up) of output r/2
          const float gv = val, uv = v[e + 1];
          const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
          a.y[size_t(tok) * a.ldy + (r >> 1)] = __fmul_rn(__fmul_rn(gv, sig), uv);
        }
      } else if (EPI == EPI_QKV) {
        const int vr = a.row_offset + r;
        const int gtok = a.token_offset + tok;
        const int pos = a.st->position + gtok;
        const int slot_kv = a.st->kv_len + gtok;
        const int hd = a.head_dim;
        if (vr < a.hidden + a.kv_dim) {
          if ((e & 1) == 0) {  // RoPE pair (vr, vr+1) (attention.rs:230-262)
            const float x0 = val, x1 = v[e + 1];
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
          if (a.kv_half) reinterpret_cast<__half*>(a.vc)[off] = __float2half_rn(val);
          else reinterpret_cast<float*>(a.vc)[off] = val;
        }
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TILE_N));
  }
}

// m_t = sqrt(sum(h_t^2)/K + eps) per token (the divisor of candle's rms_norm)
__global__ void row_rms_kernel(const float* x, int ldx, int K, float eps, float* m) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float* r = x + size_t(blockIdx.x) * ldx;
  float ss = 0.0f;
  for (int k = threadIdx.x * 4; k < K; k += blockDim.x * 4) {
    const float4 f = *reinterpret_cast<const float4*>(r + k);
    ss = __fadd_rn(ss, __fmul_rn(f.x, f.x));
    ss = __fadd_rn(ss, __fmul_rn(f.y, f.y));
    ss = __fadd_rn(ss, __fmul_rn(f.z, f.z));
    ss = __fadd_rn(ss, __fmul_rn(f.w, f.w));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.0f;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) tot = __fadd_rn(tot, part[w]);
    m[blockIdx.x] = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(K)), eps));
  }
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

constexpr size_t TC_SMEM = size_t(2) * 4 * TILE_BYTES + 64;

template <int PRO, int EPI, int DT>
cudaError_t launch_tc_t(const GemvArgs& a, const float* row_m, cudaStream_t s) {
  const int rows = a.ngroups * 4;
  const dim3 grid((rows + TILE_N - 1) / TILE_N, (a.M + TILE_T - 1) / TILE_T);
  const cudaError_t e =
      a.xprep ? launch_pdl(gemm_tc_kernel<PRO, EPI, DT, true>, grid, dim3(TC_THREADS), TC_SMEM, s, a.pdl != 0, a, row_m)
              : launch_pdl(gemm_tc_kernel<PRO, EPI, DT, false>, grid, dim3(TC_THREADS), TC_SMEM, s, a.pdl != 0, a,
                           row_m);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int PRO, int EPI>
cudaError_t configure_tc_pe() {
  cudaError_t e = cudaSuccess;
  auto set = [&](auto kern) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(TC_SMEM));
  };
  set(gemm_tc_kernel<PRO, EPI, DT_Q4K, false>);
  set(gemm_tc_kernel<PRO, EPI, DT_Q6K, false>);
  set(gemm_tc_kernel<PRO, EPI, DT_Q4K, true>);
  set(gemm_tc_kernel<PRO, EPI, DT_Q6K, true>);
  return e;
}

// the activations of a GEMM as the kernel's A tiles: [token tile][K block] pairs of
// 16 KB fp16 tiles (hi, lo) in the core-matrix layout, times the RMSNorm weight when
// given (its per-token divisor is applied in the GEMM epilogue); rows past T are zero
__global__ void stage_x_kernel(const float* x, int ldx, int T, int K, const float* norm_w, uint8_t* out) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int kb = blockIdx.x, tt = blockIdx.y, nkb = K / KB;
  const int r = threadIdx.x >> 1, h = threadIdx.x & 1;  // token row of the tile, which 32 values
  const int t = tt * TILE_T + r;
  float v[32];
  if (t < T) {
    const float* xr = x + size_t(t) * ldx + kb * KB + 32 * h;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 f = *reinterpret_cast<const float4*>(xr + j);
      v[j] = f.x; v[j + 1] = f.y; v[j + 2] = f.z; v[j + 3] = f.w;
    }
    if (norm_w) {
      const float* nw = norm_w + kb * KB + 32 * h;
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(v[j], nw[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.0f;
  }
  uint8_t* hi = out + (size_t(tt) * nkb + kb) * 2 * TILE_BYTES;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float w8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) w8[e] = v[8 * c + e];
    split_store(hi, hi + TILE_BYTES, r, 32 * h + 8 * c, w8);
  }
}

}  // namespace

cudaError_t gemm_tc_configure() {
  cudaError_t e = configure_tc_pe<PRO_NONE, EPI_STORE>();
  if (e == cudaSuccess) e = configure_tc_pe<PRO_NONE, EPI_RESID>();
  if (e == cudaSuccess) e = configure_tc_pe<PRO_RMSNORM, EPI_QKV>();
  if (e == cudaSuccess) e = configure_tc_pe<PRO_RMSNORM, EPI_SWIGLU>();
  return e;
}

cudaError_t launch_stage_x(const float* x, int ldx, int T, int K, const float* norm_w, uint8_t* out, cudaStream_t s) {
  if (K % KB != 0 || T < 1) return cudaErrorInvalidValue;
  const cudaError_t e = launch_pdl(stage_x_kernel, dim3(K / KB, (T + TILE_T - 1) / TILE_T), dim3(TC_THREADS), 0, s,
                                   true, x, ldx, T, K, norm_w, out);
  return e != cudaSuccess ? e : cudaGetLastError();
}

size_t stage_x_bytes(int T, int K) { return size_t((T + TILE_T - 1) / TILE_T) * (K / KB) * 2 * TILE_BYTES; }

cudaError_t launch_row_rms(const float* x, int ldx, int T, int K, float eps, float* m, bool pdl, cudaStream_t s) {
  const cudaError_t e = launch_pdl(row_rms_kernel, dim3(T), dim3(256), 0, s, pdl, x, ldx, K, eps, m);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_gemm_tc(const GemvArgs& a, int pro, int epi, const float* row_m, cudaStream_t s) {
  const bool q4 = a.seg[0].dtype == DT_Q4K;
#define WCB_TC_CASE(P, E)                                                                             \
  if (pro == P && epi == E)                                                                           \
    return q4 ? launch_tc_t<P, E, DT_Q4K>(a, row_m, s) : launch_tc_t<P, E, DT_Q6K>(a, row_m, s);
  WCB_TC_CASE(PRO_NONE, EPI_STORE)
  WCB_TC_CASE(PRO_NONE, EPI_RESID)
  WCB_TC_CASE(PRO_RMSNORM, EPI_QKV)
  WCB_TC_CASE(PRO_RMSNORM, EPI_SWIGLU)
#undef WCB_TC_CASE
  return cudaErrorInvalidValue;
}

}  // namespace wcb
