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

constexpr int BD_THREADS = 256;                        // 8 warps: two threads per weight row
constexpr int BD_A_BYTES = BATCH_TILE * QK_K * 2;      // fp16 quants of one super-block (64 KB)
constexpr int BD_LBO_A = (BATCH_TILE / 8) * 128;       // next 8-column K chunk of A (2048 B)
constexpr int BD_MAX_SPLITS = 8;                       // K slices of a tile = CTAs of one cluster

// shared-memory carve-up of one CTA (NB = MMA N)
template <int NB>
struct BdLayout {
  static constexpr int X_BYTES = NB * QK_K * 2;             // one fp16 half of a super-block's activations
  static constexpr int CP = NB + 1;                         // padded row of the result slice
  static constexpr int A_OFF = 0;                           // A tile; then the K-slice result
  static constexpr int XH_OFF = A_OFF + BD_A_BYTES;
  static constexpr int XL_OFF = XH_OFF + X_BYTES;
  static constexpr int XS_OFF = XL_OFF + X_BYTES;           // float [8][NB] Q4_K sub-block sums of x w
  static constexpr int C_OFF = A_OFF;                       // float [128][CP] this CTA's K-slice result (after the MMAs)
  static constexpr int RM_OFF = XS_OFF + 8 * NB * 4;        // float [NB] RMSNorm divisors
  static constexpr int SI_OFF = RM_OFF + NB * 4;            // int [3][NB] position, KV slot, done
  static constexpr int RED_OFF = SI_OFF + 3 * NB * 4;       // float [16][NB] partial sums of squares
  static constexpr int NW_OFF = RED_OFF + 16 * NB * 4;      // float [2][256] RMSNorm weights of the ring's blocks
  static constexpr int BAR_OFF = NW_OFF + 2 * QK_K * 4;     // mbarrier of the MMAs
  static constexpr int TS_OFF = BAR_OFF + 8;                // TMEM base address
  static constexpr int RAW_OFF = (TS_OFF + 4 + 127) / 128 * 128;  // [2][128][block bytes] ring
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

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory location in cluster CTA `rank`
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// (not volatile: the slices only change before the cluster barrier that precedes
// these loads, so the compiler may issue them together)
__device__ __forceinline__ float ld_cluster(uint32_t addr) {
  float v;
  asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
// bounded spin on an mbarrier phase (no suspension: the waiters have nothing else to do)
__device__ __forceinline__ bool mbar_spin(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t it = 0; it < (1u << 24); ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// One CTA: a 128-row tile x a slice of the K super-blocks. 256 threads: thread
// t owns weight row t % 128 and K half t / 128 of every super-block (its 128
// quants and its 4 Q4_K / 8 Q6_K sub-block scales). Per super-block the CTA
// unpacks the quants and stages the activations, one thread issues the MMAs
// (one TMEM accumulator of NB columns per sub-block), then every thread reads
// back the accumulators of its half and scales them into its running sums.
// The slices of a tile form one thread-block cluster: each CTA leaves its
// 128 x B result in shared memory, and after a cluster barrier CTA c adds the
// slices (in slice order, over distributed shared memory) for rows
// [c*128/S, (c+1)*128/S) and runs the epilogue on them.
template <int NB>
__global__ void __launch_bounds__(BD_THREADS, 1) bgemm_kernel(const BatchGemmArgs a, const int epi) {
  using L = BdLayout<NB>;
  constexpr int CP = L::CP;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t* At = sm + L::A_OFF;
  uint8_t* Xh = sm + L::XH_OFF;
  uint8_t* Xl = sm + L::XL_OFF;
  float* xs = reinterpret_cast<float*>(sm + L::XS_OFF);
  float* C = reinterpret_cast<float*>(sm + L::C_OFF);
  float* rm = reinterpret_cast<float*>(sm + L::RM_OFF);
  int* si = reinterpret_cast<int*>(sm + L::SI_OFF);
  float* red = reinterpret_cast<float*>(sm + L::RED_OFF);
  float* nw = reinterpret_cast<float*>(sm + L::NW_OFF);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L::TS_OFF);
  uint8_t* raw = sm + L::RAW_OFF;
  __shared__ const uint8_t* rp[BATCH_TILE];  // this tile's weight rows

  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (BATCH_TILE - 1), hk = tid >> 7;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int nsb = a.K / QK_K;
  const int sb0 = split * a.sb_per_split;
  const int nloc = min(nsb, sb0 + a.sb_per_split) - sb0;
  const int tdt = bd_tile_dtype(a, epi, tile);
  const bool q4 = tdt == DT_Q4K;
  const int bb = q4 ? Q4K_BYTES : Q6K_DEV_BYTES;
  const size_t row_bytes = size_t(nsb) * bb;
  // TMEM: Q4_K one accumulator of 2NB columns (hi | lo halves of the activations);
  // Q6_K one per sub-block of a K half (8 x 2NB)
  const uint32_t tcols = uint32_t(q4 ? 2 * NB : 16 * NB);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(tcols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  if (tid < BATCH_TILE) rp[tid] = bd_row(a, epi, tile, tid, row_bytes);
  // the padding sequences (b >= B) stay zero in both activation halves
  for (int i = tid; i < 2 * L::X_BYTES / 16; i += BD_THREADS)
    reinterpret_cast<uint4*>(Xh)[i] = make_uint4(0u, 0u, 0u, 0u);
  pdl_trigger();
  __syncthreads();
  const int chunks = bb / 16;
  auto load_sb = [&](int j) {  // super-block j of the slice (+ its norm weights) into ring slot j & 1
    uint8_t* dst = raw + (j & 1) * BATCH_TILE * bb;
    const size_t src_off = size_t(sb0 + j) * bb;
    for (int c = tid; c < BATCH_TILE * chunks; c += BD_THREADS) {
      const int r = c / chunks, pc = c - r * chunks;
      cp_async16(dst + r * bb + pc * 16, rp[r] + src_off + pc * 16);
    }
    if (a.norm_w && tid < QK_K / 4)
      cp_async16(nw + (j & 1) * QK_K + 4 * tid, a.norm_w + size_t(sb0 + j) * QK_K + 4 * tid);
  };
  load_sb(0);
  cp_async_commit();
  if (nloc > 1) load_sb(1);
  cp_async_commit();
  pdl_wait();  // activations, norm statistics and sequence states come from earlier kernels

  // sequence states; RMSNorm divisors from the producer's partial sums of squares,
  // added in a fixed order (BD_THREADS / NB parts of consecutive entries, then the parts)
  constexpr int PARTS = BD_THREADS / NB;
  {
    const int b = tid % NB, part = tid / NB;
    if (part == 0 && b < a.B) {
      const StepState* st = a.st + b;
      si[b] = st->position;
      si[NB + b] = st->kv_len;
      si[2 * NB + b] = st->done;
    }
    if (a.norm_w) {
      const int per = (a.sq_tiles + PARTS - 1) / PARTS;
      const int t0 = part * per, t1 = min(a.sq_tiles, t0 + per);
      float tot = 0.0f;
      if (b < a.B) {
#pragma unroll 8
        for (int t = t0; t < t1; ++t) tot = __fadd_rn(tot, a.sq_in[t * a.B + b]);
      }
      red[part * NB + b] = tot;
    }
  }
  __syncthreads();
  if (a.norm_w && tid < a.B) {  // x / sqrt(mean(x^2) + eps) * w (candle_tensor_backend.rs:30-57)
    float tot = 0.0f;
    for (int p = 0; p < PARTS; ++p) tot = __fadd_rn(tot, red[p * NB + tid]);
    rm[tid] = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(a.K)), a.eps));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane_tmem = tmem + (uint32_t((warp & 3) * 32) << 16);

  float acc[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
  bool ok = true;
  uint32_t phase = 0;
  // activation staging: thread (b = tid % NB, g = tid / NB) owns values [g*NB, g*NB + NB)
  // of sequence b in each super-block (a whole Q4_K sub-block when NB = 32, half of
  // one when NB = 16: the other half is lane tid ^ 16). The B operand holds the fp16
  // hi halves in rows 0..NB-1 and the lo halves in rows NB..2NB-1, so one MMA (N = 2NB)
  // takes both.
  constexpr uint32_t LBO_X2 = (2 * NB / 8) * 128;
  const int xb = tid % NB, xg = tid / NB;
  const float* xrow = a.x + size_t(xb) * a.ldx;
  const bool xon = xb < a.B;
  // descriptors: the address field (bits 0-13, 16-byte units) advances by 2 * LBO per 16-value step
  const uint64_t adesc0 = bd_desc(smem_u32(At), BD_LBO_A);
  const uint64_t xdesc0 = bd_desc(smem_u32(Xh), LBO_X2);
  for (int j = 0; j < nloc; ++j) {
    const int kg = (sb0 + j) * QK_K;
    // this thread's activations of the super-block, loaded first so their latency
    // hides behind the unpacking
    float4 xq[NB / 4];
    if (xon) {
      const float4* src = reinterpret_cast<const float4*>(xrow + kg + xg * NB);
#pragma unroll
      for (int e = 0; e < NB / 4; ++e) xq[e] = src[e];
    }
    cp_async_wait<1>();
    __syncthreads();  // super-block j (and its norm weights) have landed
    const uint8_t* blk = raw + (j & 1) * BATCH_TILE * bb + row * bb;
    // (1) this thread's 128 quants (K half hk) as fp16 integers. Q4_K: sc_s * q (at most
    // 63 * 15 = 945, exact), so the whole super-block shares the scale d and one
    // accumulator; the dmin * m_s * sum(x) terms are added on the CUDA cores.
    // Q6_K: q - 32 with d * sc_s per 16-value sub-block applied after the MMA.
    float d1[8], m1[4], dq = 0.0f, dmq = 0.0f;
    if (q4) {
      const uint4 hd = *reinterpret_cast<const uint4*>(blk);
      dq = half_bits(hd.x & 0xFFFFu);
      dmq = half_bits(hd.x >> 16);
      const __half2 bias = __float2half2_rn(1024.0f);
#pragma unroll
      for (int p = 0; p < 2; ++p) {  // sub-block pair 2hk+p: low nibbles = sub-block 2p, high = 2p+1
        uint32_t sc0, mn0, sc1, mn1;
        scale_min(4 * hk + 2 * p, hd.y, hd.z, hd.w, sc0, mn0);
        scale_min(4 * hk + 2 * p + 1, hd.y, hd.z, hd.w, sc1, mn1);
        m1[2 * p] = float(mn0);
        m1[2 * p + 1] = float(mn1);
        const __half2 s0 = __float2half2_rn(float(sc0)), s1 = __float2half2_rn(float(sc1));
#pragma unroll
        for (int w = 0; w < 2; ++w) {  // 16 bytes = values 16w..16w+15 of both sub-blocks
          const uint4 q16 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * (2 * hk + p) + 16 * w);
          const uint32_t qw[4] = {q16.x, q16.y, q16.z, q16.w};
          uint32_t lo[8], hi[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            quads_to_half(qw[e] & 0x0F0F0F0Fu, bias, lo[2 * e], lo[2 * e + 1]);
            quads_to_half((qw[e] >> 4) & 0x0F0F0F0Fu, bias, hi[2 * e], hi[2 * e + 1]);
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            __half2 l2 = __hmul2(*reinterpret_cast<__half2*>(&lo[e]), s0);
            __half2 h2 = __hmul2(*reinterpret_cast<__half2*>(&hi[e]), s1);
            lo[e] = *reinterpret_cast<uint32_t*>(&l2);
            hi[e] = *reinterpret_cast<uint32_t*>(&h2);
          }
          const int k = 128 * hk + 64 * p + 16 * w;
          *reinterpret_cast<uint4*>(At + op_off(row, k, BD_LBO_A)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *reinterpret_cast<uint4*>(At + op_off(row, k + 8, BD_LBO_A)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
          *reinterpret_cast<uint4*>(At + op_off(row, k + 32, BD_LBO_A)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(At + op_off(row, k + 40, BD_LBO_A)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
        }
      }
    } else {  // Q6_K half hk: value 32g + l = ql nibble | 2 bits of qh (quant.rs:206-261)
      const float d = half_bits(uint32_t(blk[208]) | (uint32_t(blk[209]) << 8));
      const int8_t* scv = reinterpret_cast<const int8_t*>(blk + 192 + 8 * hk);
#pragma unroll
      for (int u = 0; u < 8; ++u) d1[u] = __fmul_rn(d, float(scv[u]));
      const uint8_t* ql = blk + 64 * hk;
      const uint8_t* qh = blk + 128 + 32 * hk;
      const __half2 bias = __float2half2_rn(1056.0f);  // 1024 + the Q6_K offset 32
#pragma unroll
      for (int l16 = 0; l16 < 2; ++l16) {
        const uint4 a0 = *reinterpret_cast<const uint4*>(ql + 16 * l16);
        const uint4 a1 = *reinterpret_cast<const uint4*>(ql + 32 + 16 * l16);
        const uint4 hb = *reinterpret_cast<const uint4*>(qh + 16 * l16);
        const uint32_t w0[4] = {a0.x, a0.y, a0.z, a0.w}, w1[4] = {a1.x, a1.y, a1.z, a1.w};
        const uint32_t wh[4] = {hb.x, hb.y, hb.z, hb.w};
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int sh = g < 2 ? 0 : 4;
          uint32_t o[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t src = (g & 1) ? w1[e] : w0[e];
            const uint32_t q = ((src >> sh) & 0x0F0F0F0Fu) | (((wh[e] >> (2 * g)) & 0x03030303u) << 4);
            quads_to_half(q, bias, o[2 * e], o[2 * e + 1]);
          }
          const int k = 128 * hk + 32 * g + 16 * l16;
          *reinterpret_cast<uint4*>(At + op_off(row, k, BD_LBO_A)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(At + op_off(row, k + 8, BD_LBO_A)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
      }
    }
    // (2) the activations x * w (the RMSNorm divisor is applied to the sums at the
    // end: sum W (x w / m) = (1/m) sum W (x w)), split into fp16 hi + lo
    float sum = 0.0f;
    if (xon) {
#pragma unroll
      for (int c = 0; c < NB / 8; ++c) {
        float v[8] = {xq[2 * c].x, xq[2 * c].y, xq[2 * c].z, xq[2 * c].w,
                      xq[2 * c + 1].x, xq[2 * c + 1].y, xq[2 * c + 1].z, xq[2 * c + 1].w};
        if (a.norm_w) {
          const float4* w4 = reinterpret_cast<const float4*>(nw + (j & 1) * QK_K + xg * NB + 8 * c);
          const float4 w0 = w4[0], w1 = w4[1];
          const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(v[e], wv[e]);
        }
        __half hv[8], lv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          hv[e] = __float2half_rn(v[e]);
          lv[e] = __float2half_rn(__fsub_rn(v[e], __half2float(hv[e])));
          sum = __fadd_rn(sum, v[e]);
        }
        const int k = xg * NB + 8 * c;
        *reinterpret_cast<uint4*>(Xh + op_off(xb, k, LBO_X2)) = *reinterpret_cast<const uint4*>(hv);
        *reinterpret_cast<uint4*>(Xh + op_off(NB + xb, k, LBO_X2)) = *reinterpret_cast<const uint4*>(lv);
      }
    }
    if (NB == 16) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 16));  // lanes g, g^1 of a sub-block
    if (xon && (NB == 32 || (xg & 1) == 0)) xs[(xg * NB / 32) * NB + xb] = sum;  // sum of x w over the sub-block
    fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
    tc_fence_before();
    __syncthreads();
    if (q4) {
      // (3) one thread issues the 16 MMAs of the super-block into the one accumulator
      if (tid == 0) {
        tc_fence_after();
#pragma unroll 1
        for (int c16 = 0; c16 < QK_K / 16; ++c16)
          bd_mma<2 * NB>(tmem, adesc0 + uint64_t(c16) * (2 * BD_LBO_A / 16),
                         xdesc0 + uint64_t(c16) * (2 * LBO_X2 / 16), c16 > 0 ? 1u : 0u);
        bd_commit(bar);
      }
      // (4) thread (row, hk) reads the hi (hk = 0) or lo (hk = 1) half of its row's
      // accumulator: acc += d * dot - dmin * sum_s m_s * sum(x w) over its 4 sub-blocks
#pragma unroll
      for (int uu = 0; uu < 4; ++uu) {  // the min terms while the MMAs run
        const float mm = dmq * m1[uu];
        const float4* x4 = reinterpret_cast<const float4*>(xs + (4 * hk + uu) * NB);
#pragma unroll
        for (int b4 = 0; b4 < NB / 4; ++b4) {
          const float4 s4 = x4[b4];
          acc[4 * b4 + 0] -= mm * s4.x;
          acc[4 * b4 + 1] -= mm * s4.y;
          acc[4 * b4 + 2] -= mm * s4.z;
          acc[4 * b4 + 3] -= mm * s4.w;
        }
      }
      ok &= mbar_spin(bar, phase);
      phase ^= 1u;
      tc_fence_after();
      float v[NB];
      tmem_ld<NB>(lane_tmem + uint32_t(hk * NB), v);
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[b] += dq * v[b];
    } else {
      // Q6_K: sub-blocks 0-7 (K half 0), then 8-15 (K half 1), 8 accumulators of 2NB
      // columns each pass; the threads of that half read them back
#pragma unroll 1
      for (int pass = 0; pass < 2; ++pass) {
        if (tid == 0) {
          tc_fence_after();
#pragma unroll 1
          for (int u = 0; u < 8; ++u) {
            const uint64_t c16 = uint64_t(8 * pass + u);
            bd_mma<2 * NB>(tmem + uint32_t(u * 2 * NB), adesc0 + c16 * (2 * BD_LBO_A / 16),
                           xdesc0 + c16 * (2 * LBO_X2 / 16), 0u);
          }
          bd_commit(bar);
        }
        ok &= mbar_spin(bar, phase);
        phase ^= 1u;
        tc_fence_after();
        if (hk == pass) {
#pragma unroll
          for (int u = 0; u < 8; ++u) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              float v[NB];
              tmem_ld<NB>(lane_tmem + uint32_t(u * 2 * NB + half * NB), v);
#pragma unroll
              for (int b = 0; b < NB; ++b) acc[b] += d1[u] * v[b];
            }
          }
        }
        tc_fence_before();
        __syncthreads();  // the accumulators are free for the next pass
      }
    }
    tc_fence_before();
    if (j + 2 < nloc) load_sb(j + 2);  // every thread is past its unpacking of ring slot j & 1
    cp_async_commit();
  }
  if (a.norm_w) {  // the RMSNorm divisor of each sequence (candle_tensor_backend.rs:30-57)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = __fdiv_rn(acc[b], rm[b < a.B ? b : 0]);
  }
  cp_async_wait<0>();
  const bool all_ok = __syncthreads_and(ok);
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
  }
  // the two K halves of each row, added in a fixed order
  if (hk == 1) {
#pragma unroll
    for (int b = 0; b < NB; ++b) C[row * CP + b] = acc[b];
  }
  __syncthreads();
  if (hk == 0) {
#pragma unroll
    for (int b = 0; b < NB; ++b) C[row * CP + b] = __fadd_rn(acc[b], C[row * CP + b]);
  }
  const int S = a.splits;
  if (S > 1) cluster_sync_all();  // every slice's C is complete and visible to the cluster
  else __syncthreads();
  const int crank = S > 1 ? int(cluster_rank()) : 0;
  uint32_t cbase[BD_MAX_SPLITS];
#pragma unroll
  for (int q = 0; q < BD_MAX_SPLITS; ++q) cbase[q] = q < S ? cluster_map(smem_u32(C), uint32_t(q)) : 0u;
  auto reduced = [&](int r, int b) {  // row r of the tile, sequence b, over the slices in order
    float v = 0.0f;
    const uint32_t off = uint32_t(r * CP + b) * 4u;
#pragma unroll
    for (int q = 0; q < BD_MAX_SPLITS; ++q)
      if (q < S) v = __fadd_rn(v, ld_cluster(cbase[q] + off));
    return v;
  };
  if (!all_ok && tid == 0) atomicOr(&a.st[0].err, 4);  // a bounded wait expired: store nothing

  if (all_ok) {
    float* sq = reinterpret_cast<float*>(Xh);  // the activation tile is free: [pairs][NB] sums of squares
    const int* pos = si;
    const int* slot = si + NB;
    const int* done = si + 2 * NB;
    if (epi == BEPI_SWIGLU) {  // ffn.rs:90-94: g * (1 / (1 + exp(-g))) * u
      const int O = ((BATCH_TILE / 2 + S - 1) / S + 1) & ~1;  // outputs of this CTA (even)
      const int o0 = crank * O, o1 = min(BATCH_TILE / 2, o0 + O);
      const int P2 = (o1 - o0 + 1) / 2;
      for (int u = tid; u < P2 * a.B; u += BD_THREADS) {
        const int pr = u % P2, b = u / P2, o = o0 + 2 * pr;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int r = tile * (BATCH_TILE / 2) + o + e;
          if (o + e >= o1 || r >= a.rows) continue;
          const float gv = reduced(o + e, b), uv = reduced(BATCH_TILE / 2 + o + e, b);
          const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
          a.y[size_t(b) * a.ldy + r] = __fmul_rn(__fmul_rn(gv, sig), uv);
        }
      }
    } else {
      const int RPC = ((BATCH_TILE + S - 1) / S + 1) & ~1;  // rows of this CTA (even)
      const int r0 = crank * RPC, r1 = min(BATCH_TILE, r0 + RPC);
      const int P2 = (r1 - r0 + 1) / 2;
      for (int u = tid; u < P2 * a.B; u += BD_THREADS) {
        const int pr = u % P2, b = u / P2, r = r0 + 2 * pr;
        const int n = tile * BATCH_TILE + r;
        const bool ok0 = r < r1 && n < a.rows, ok1 = r + 1 < r1 && n + 1 < a.rows;
        const float v0 = ok0 ? reduced(r, b) : 0.0f, v1 = ok1 ? reduced(r + 1, b) : 0.0f;
        if (epi == BEPI_STORE) {
          if (ok0) a.y[size_t(b) * a.ldy + n] = v0;
          if (ok1) a.y[size_t(b) * a.ldy + n + 1] = v1;
        } else if (epi == BEPI_RESID) {  // layer.rs:68 / :86
          const float* rr = a.resid + size_t(b) * a.ldr + n;
          const float y0 = ok0 ? __fadd_rn(rr[0], v0) : 0.0f;
          const float y1 = ok1 ? __fadd_rn(rr[1], v1) : 0.0f;
          if (ok0) a.y[size_t(b) * a.ldy + n] = y0;
          if (ok1) a.y[size_t(b) * a.ldy + n + 1] = y1;
          sq[pr * NB + b] = __fadd_rn(__fmul_rn(y0, y0), __fmul_rn(y1, y1));
        } else if (ok0) {  // BEPI_QKV: RoPE on (2i, 2i+1) pairs of q and k (attention.rs:230-262),
          // K / V appended at each sequence's KV slot (kv_cache.rs:44-67)
          const int hd = a.head_dim;
          if (n < a.hidden + a.kv_dim) {
            const int col = n < a.hidden ? n : n - a.hidden;
            const int pi = (col % hd) >> 1;
            const float cs_ = a.rope_cos[size_t(pos[b]) * (hd / 2) + pi];
            const float sn_ = a.rope_sin[size_t(pos[b]) * (hd / 2) + pi];
            const float n0 = __fsub_rn(__fmul_rn(v0, cs_), __fmul_rn(v1, sn_));
            const float n1 = __fadd_rn(__fmul_rn(v0, sn_), __fmul_rn(v1, cs_));
            if (n < a.hidden) {
              a.q[size_t(b) * a.ldq + n] = n0;
              a.q[size_t(b) * a.ldq + n + 1] = n1;
            } else if (!done[b]) {
              const size_t off = size_t(b) * a.seq_stride + (size_t(col / hd) * a.max_seq + slot[b]) * hd + col % hd;
              if (a.kv_half) {
                reinterpret_cast<__half*>(a.kc)[off] = __float2half_rn(n0);
                reinterpret_cast<__half*>(a.kc)[off + 1] = __float2half_rn(n1);
              } else {
                reinterpret_cast<float*>(a.kc)[off] = n0;
                reinterpret_cast<float*>(a.kc)[off + 1] = n1;
              }
            }
          } else if (!done[b]) {
            const int col = n - a.hidden - a.kv_dim;
            const size_t off = size_t(b) * a.seq_stride + (size_t(col / hd) * a.max_seq + slot[b]) * hd + col % hd;
            if (a.kv_half) {
              reinterpret_cast<__half*>(a.vc)[off] = __float2half_rn(v0);
              reinterpret_cast<__half*>(a.vc)[off + 1] = __float2half_rn(v1);
            } else {
              reinterpret_cast<float*>(a.vc)[off] = v0;
              reinterpret_cast<float*>(a.vc)[off + 1] = v1;
            }
          }
        }
      }
      if (epi == BEPI_RESID) {  // this slice's sums of squares per sequence, pairs added in order
        __syncthreads();
        if (tid < a.B) {
          float t = 0.0f;
          for (int pr = 0; pr < P2; ++pr) t = __fadd_rn(t, sq[pr * NB + tid]);
          a.sq_out[(size_t(tile) * S + crank) * a.B + tid] = t;
        }
      }
    }
  }
  if (S > 1) cluster_sync_all();  // no CTA leaves while others still read its slice
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
// then generate()'s bookkeeping (model.rs:1380-1409). BS_SPLIT CTAs per sequence
// each scan a slice of the vocabulary; the last to finish runs the bookkeeping.
constexpr int BS_SPLIT = 8;

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
  const int per = (vocab + BS_SPLIT - 1) / BS_SPLIT;
  const int v0 = blockIdx.y * per, v1 = min(vocab, v0 + per);
  constexpr int U = 8;  // independent loads in flight per thread
  for (int n0 = v0 + tid; n0 < v1; n0 += U * blockDim.x) {
    float v[U];
    uint32_t cnt[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int n = n0 + u * blockDim.x;
      v[u] = n < v1 ? lg[n] : 0.0f;
      cnt[u] = (n < v1 && rep != 1.0f) ? pc[n] : 0u;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int n = n0 + u * blockDim.x;
      if (n >= v1) continue;
      float pv = v[u];
      for (uint32_t k = 0; k < cnt[u]; ++k) pv = pv > 0.0f ? __fdiv_rn(pv, rep) : __fmul_rn(pv, rep);
      if (pv != pv) nan = 1;
      else {
        const unsigned long long key = (static_cast<unsigned long long>(order_key(pv)) << 32) | uint32_t(n);
        best = key > best ? key : best;
      }
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
    if (bb) atomicMax(&s->best, bb);
    if (nn) atomicOr(&s->nan, 1);
    __threadfence();
    if (atomicAdd(&s->ticket, 1) == BS_SPLIT - 1) {  // the last slice runs the bookkeeping
      __threadfence();
      finish_sample_state(s, hist + size_t(b) * hist_cap, pc);
    }
  }
}

// Decode attention of one (kv head, sequence, split) for the batched step
// (attention.rs:332-435 for one query token at position kv_len): the n_rep <= 8
// query heads of the kv head are processed together. Each warp takes 32 keys at
// a time, one per lane: the lane reads its key's K row straight from the cache
// and scores it against all query heads (queries broadcast from shared memory);
// the warp keeps a running max / sum per head, writes its probabilities to
// shared memory and accumulates P.V with each lane owning HD/32 dimensions of
// every head (V rows read coalesced). The 4 warps merge in shared memory, the
// splits through a partial buffer and a ticket (the last CTA merges).
template <typename KT>
__device__ __forceinline__ void load8(const KT* p, float (&f)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <int N, typename KT>
__device__ __forceinline__ void loadn(const KT* p, float (&f)[N]) {
  if constexpr (N == 2) {
    if constexpr (sizeof(KT) == 2) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(p));
      f[0] = t.x; f[1] = t.y;
    } else {
      const float2 t = *reinterpret_cast<const float2*>(p);
      f[0] = t.x; f[1] = t.y;
    }
  } else {
    if constexpr (sizeof(KT) == 2) {
      const uint2 u = *reinterpret_cast<const uint2*>(p);
      const float2 t0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 t1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      f[0] = t0.x; f[1] = t0.y; f[2] = t1.x; f[3] = t1.y;
    } else {
      const float4 t = *reinterpret_cast<const float4*>(p);
      f[0] = t.x; f[1] = t.y; f[2] = t.z; f[3] = t.w;
    }
  }
}

constexpr int BA_THREADS = 128;
constexpr int BA_NR = 8;  // query heads per kv head (at most)

template <int HD, typename KT>
__global__ void __launch_bounds__(BA_THREADS) battn_kernel(const AttnArgs a) {
  constexpr int DPL = HD / 32;  // output dimensions per lane
  __shared__ __align__(16) float qs[BA_NR * HD];
  __shared__ __align__(16) float ps[4][32][BA_NR];
  __shared__ float wm[4][BA_NR], wl[4][BA_NR];
  __shared__ __align__(16) float wo[4][BA_NR][HD];
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  const int kh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;
  const StepState* st = a.st + b;
  if (st->done) return;
  const int nkeys = st->kv_len + 1;  // keys 0..position, this step's included
  const int nsplit = (nkeys + a.chunk - 1) / a.chunk;
  if (split >= nsplit) return;
  const int j0 = split * a.chunk, j1 = min(j0 + a.chunk, nkeys);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_rep = a.n_heads / a.n_kv;
  const float* qsrc = a.q + (size_t(b) * a.n_heads + size_t(kh) * n_rep) * HD;
  for (int i = tid; i < BA_NR * HD; i += BA_THREADS) qs[i] = i < n_rep * HD ? qsrc[i] : 0.0f;
  __syncthreads();
  const size_t base = size_t(b) * a.seq_stride + size_t(kh) * a.max_seq * HD;
  const KT* Kp = reinterpret_cast<const KT*>(a.kc) + base;
  const KT* Vp = reinterpret_cast<const KT*>(a.vc) + base;

  float m[BA_NR], l[BA_NR], o[BA_NR][DPL];
#pragma unroll
  for (int r = 0; r < BA_NR; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) o[r][d] = 0.0f;
  }
  // V rows of the warp's 32 keys are requested before the scores are computed
  // (raw 32-bit words, when they fit in registers), so their latency overlaps it
  constexpr int RW = DPL * int(sizeof(KT)) / 4;  // 32-bit words of V per lane per key
  constexpr bool PRE = RW <= 2;
  for (int k0 = j0 + warp * 32; k0 < j1; k0 += 4 * 32) {
    const int j = k0 + lane;
    const bool valid = j < j1;
    const int nk = min(32, j1 - k0);
    const KT* vb = Vp + size_t(k0) * HD + lane * DPL;
    uint32_t vr[PRE ? 32 : 1][PRE ? RW : 1];
    if constexpr (PRE) {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        if (jj < nk) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(vb + size_t(jj) * HD);
#pragma unroll
          for (int w = 0; w < RW; ++w) vr[jj][w] = src[w];
        } else {
#pragma unroll
          for (int w = 0; w < RW; ++w) vr[jj][w] = 0u;
        }
      }
    }
    float s[BA_NR];
#pragma unroll
    for (int r = 0; r < BA_NR; ++r) s[r] = 0.0f;
    if (valid) {
      const KT* kr = Kp + size_t(j) * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 8) {
        float kf[8];
        load8<KT>(kr + c, kf);
#pragma unroll
        for (int r = 0; r < BA_NR; ++r) {
          const float4 q0 = *reinterpret_cast<const float4*>(qs + r * HD + c);
          const float4 q1 = *reinterpret_cast<const float4*>(qs + r * HD + c + 4);
          s[r] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] + q1.y * kf[5] +
                  q1.z * kf[6] + q1.w * kf[7];
        }
      }
    }
    // running softmax per head (attention.rs:380-410)
#pragma unroll
    for (int r = 0; r < BA_NR; ++r) {
      const float sc = valid ? s[r] * a.scale : -INFINITY;
      const float mn = fmaxf(m[r], warp_max(sc));
      const float p = valid ? expf(sc - mn) : 0.0f;
      const float cf = expf(m[r] - mn);
      l[r] = l[r] * cf + warp_sum(p);
      m[r] = mn;
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[r][d] *= cf;
      ps[warp][lane][r] = p;
    }
    __syncwarp();
    if constexpr (PRE) {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        if (jj >= nk) break;
        float v[DPL];
        if constexpr (sizeof(KT) == 2) {
#pragma unroll
          for (int w = 0; w < RW; ++w) {
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&vr[jj][w]));
            v[2 * w] = t.x;
            v[2 * w + 1] = t.y;
          }
        } else {
#pragma unroll
          for (int w = 0; w < RW; ++w) v[w] = __uint_as_float(vr[jj][w]);
        }
        const float4 p0 = *reinterpret_cast<const float4*>(&ps[warp][jj][0]);
        const float4 p1 = *reinterpret_cast<const float4*>(&ps[warp][jj][4]);
        const float pr[BA_NR] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int r = 0; r < BA_NR; ++r)
#pragma unroll
          for (int d = 0; d < DPL; ++d) o[r][d] += pr[r] * v[d];
      }
    } else {
      for (int j8 = 0; j8 < nk; j8 += 8) {  // 8 rows in flight at a time
        float v[8][DPL];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (j8 + e < nk) loadn<DPL, KT>(vb + size_t(j8 + e) * HD, v[e]);
          else {
#pragma unroll
            for (int d = 0; d < DPL; ++d) v[e][d] = 0.0f;
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float4 p0 = *reinterpret_cast<const float4*>(&ps[warp][min(j8 + e, 31)][0]);
          const float4 p1 = *reinterpret_cast<const float4*>(&ps[warp][min(j8 + e, 31)][4]);
          const float pr[BA_NR] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
          for (int r = 0; r < BA_NR; ++r)
#pragma unroll
            for (int d = 0; d < DPL; ++d) o[r][d] += pr[r] * v[e][d];
        }
      }
    }
    __syncwarp();
  }
  // merge the 4 warps (a warp without keys has m = -inf, l = 0)
#pragma unroll
  for (int r = 0; r < BA_NR; ++r) {
    if (lane == 0) {
      wm[warp][r] = m[r];
      wl[warp][r] = l[r];
    }
#pragma unroll
    for (int d = 0; d < DPL; ++d) wo[warp][r][lane * DPL + d] = o[r][d];
  }
  __syncthreads();
  const size_t pstride = HD + 2;
  for (int i = tid; i < n_rep * HD; i += BA_THREADS) {
    const int r = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][r]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = expf(wm[w][r] - M);
      L += wl[w][r] * f;
      O += wo[w][r][d] * f;
    }
    const size_t head = size_t(b) * a.n_heads + size_t(kh) * n_rep + r;
    if (nsplit == 1) {
      a.out[head * HD + d] = L > 0.0f ? O / L : 0.0f;
    } else {
      float* pp = a.part + (head * a.max_splits + split) * pstride;
      pp[2 + d] = O;
      if (d == 0) {
        pp[0] = M;
        pp[1] = L;
      }
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(a.ticket + b * a.n_kv + kh, 1) == nsplit - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) a.ticket[b * a.n_kv + kh] = 0;
  for (int i = tid; i < n_rep * HD; i += BA_THREADS) {
    const int r = i / HD, d = i % HD;
    const size_t head = size_t(b) * a.n_heads + size_t(kh) * n_rep + r;
    const float* pb = a.part + head * a.max_splits * pstride;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, __ldcg(pb + sp * pstride));
    float L = 0.0f, O = 0.0f;
#pragma unroll 4
    for (int sp = 0; sp < nsplit; ++sp) {
      const float f = expf(__ldcg(pb + sp * pstride) - M);
      L += __ldcg(pb + sp * pstride + 1) * f;
      O += __ldcg(pb + sp * pstride + 2 + d) * f;
    }
    a.out[head * HD + d] = L > 0.0f ? O / L : 0.0f;
  }
}

// Tensor parallelism: y = resid + (the all-reduced partial sums), and the
// per-128-row-tile sums of squares of y for the next RMSNorm (grid: tiles x B)
__global__ void bresid_kernel(float* y, const float* resid, const float* add, int B, int H, float* sq) {
  pdl_trigger();
  pdl_wait();
  const int tile = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, n = tile * BATCH_TILE + tid;
  float v = 0.0f;
  if (n < H) {
    v = __fadd_rn(resid[size_t(b) * H + n], add[size_t(b) * H + n]);
    y[size_t(b) * H + n] = v;
  }
  __shared__ float red[BATCH_TILE / 32];
  const float s2 = warp_sum(__fmul_rn(v, v));
  if ((tid & 31) == 0) red[tid >> 5] = s2;
  __syncthreads();
  if (tid == 0) {
    float t = 0.0f;
    for (int w = 0; w < BATCH_TILE / 32; ++w) t = __fadd_rn(t, red[w]);
    sq[size_t(tile) * B + b] = t;
  }
}

// Tensor parallelism, LM head split by vocabulary: each sequence's best
// (order-preserving logit bits << 32 | token id) over this rank's rows after
// the repetition penalty, and a NaN flag, max-reduced into keys[2b], keys[2b+1]
// (zeroed before); the ranks then max all-reduce the keys
__global__ void bkey_kernel(const float* logits, int vl, int vocab_off, int vocab, const StepState* st,
                            const uint32_t* pen_cnt, float rep, unsigned long long* keys) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  if (st[b].done) return;
  const float* lg = logits + size_t(b) * vl;
  const uint32_t* pc = pen_cnt + size_t(b) * vocab + vocab_off;
  const int per = (vl + gridDim.y - 1) / gridDim.y;
  const int v0 = blockIdx.y * per, v1 = min(vl, v0 + per);
  unsigned long long best = 0ull;
  int nan = 0;
  for (int n = v0 + tid; n < v1; n += blockDim.x) {
    float pv = lg[n];
    if (rep != 1.0f) {
      const uint32_t cnt = pc[n];
      for (uint32_t k = 0; k < cnt; ++k) pv = pv > 0.0f ? __fdiv_rn(pv, rep) : __fmul_rn(pv, rep);
    }
    if (pv != pv) nan = 1;
    else {
      const unsigned long long key =
          (static_cast<unsigned long long>(order_key(pv)) << 32) | uint32_t(vocab_off + n);
      best = key > best ? key : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
    nan |= __shfl_xor_sync(0xffffffffu, nan, o);
  }
  if ((tid & 31) == 0) {
    if (best) atomicMax(keys + 2 * b, best);
    if (nan) atomicMax(keys + 2 * b + 1, 1ull);
  }
}

// generate()'s bookkeeping of every unfinished sequence from the reduced keys
__global__ void bfinish_kernel(StepState* st, const unsigned long long* keys, uint32_t* hist, int hist_cap,
                               uint32_t* pen_cnt, int vocab) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  StepState* s = st + b;
  if (threadIdx.x != 0 || s->done) return;
  s->best = keys[2 * b];
  s->nan = keys[2 * b + 1] ? 1 : 0;
  finish_sample_state(s, hist + size_t(b) * hist_cap, pen_cnt + size_t(b) * vocab);
}

// The same decode attention on the tensor cores, for an fp16 cache: per warp,
// 32-key tiles of its 64 keys are staged in shared memory (cp.async), the n_rep
// query heads are the rows of a 16-row mma.sync.m16n8k16 operand (rows n_rep..15
// are zero), S = Q K^T and O += P V run as fp16 products with q and p split
// into hi + lo halves, and the running softmax works on the accumulator
// fragments. Warps and splits merge as in battn_kernel.
constexpr int BF_TS = 32;  // keys per staged tile

template <int HD>
__global__ void __launch_bounds__(BA_THREADS) bfa_kernel(const AttnArgs a) {
  constexpr int P = HD + 8;  // halves per staged row (conflict-free fragment loads)
  extern __shared__ __align__(16) uint8_t fsm[];
  __half* Kw = reinterpret_cast<__half*>(fsm) + (threadIdx.x >> 5) * (2 * BF_TS * P);
  __half* Vw = Kw + BF_TS * P;
  __shared__ float wm[4][BA_NR], wl[4][BA_NR];
  __shared__ __align__(16) float wo[4][BA_NR][HD];
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  const int kh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;
  const StepState* st = a.st + b;
  if (st->done) return;
  const int nkeys = st->kv_len + 1;
  const int nsplit = (nkeys + a.chunk - 1) / a.chunk;
  if (split >= nsplit) return;
  const int j0 = split * a.chunk, j1 = min(j0 + a.chunk, nkeys);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int n_rep = a.n_heads / a.n_kv;
  const size_t base = size_t(b) * a.seq_stride + size_t(kh) * a.max_seq * HD;
  const __half* Kg = reinterpret_cast<const __half*>(a.kc) + base;
  const __half* Vg = reinterpret_cast<const __half*>(a.vc) + base;
  // Q rows: head g of the kv head (zero for g >= n_rep); rows 8..15 are zero
  uint32_t qh[HD / 16][4], ql[HD / 16][4];
  {
    const float* qr = a.q + (size_t(b) * a.n_heads + size_t(kh) * n_rep + min(g, n_rep - 1)) * HD;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const int c = ks * 16 + 2 * tq;
      float2 x0 = *reinterpret_cast<const float2*>(qr + c), x2 = *reinterpret_cast<const float2*>(qr + c + 8);
      if (g >= n_rep) x0 = x2 = make_float2(0.f, 0.f);
      split2(x0.x, x0.y, qh[ks][0], ql[ks][0]);
      split2(x2.x, x2.y, qh[ks][2], ql[ks][2]);
      qh[ks][1] = ql[ks][1] = qh[ks][3] = ql[ks][3] = 0u;
    }
  }
  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m = -INFINITY, l = 0.0f;  // row g
  const int wk0 = j0 + warp * (a.chunk / 4), wk1 = min(j1, wk0 + a.chunk / 4);
  for (int t0 = wk0; t0 < wk1; t0 += BF_TS) {
    const int nt = min(BF_TS, wk1 - t0);
    __syncwarp();
    constexpr int CH = HD / 8;  // 16-byte chunks per row
    for (int i = lane; i < BF_TS * CH; i += 32) {
      const int row = i / CH, c = (i % CH) * 8;
      if (row < nt) {
        cp_async16(Kw + row * P + c, Kg + size_t(t0 + row) * HD + c);
        cp_async16(Vw + row * P + c, Vg + size_t(t0 + row) * HD + c);
      } else {
        *reinterpret_cast<uint4*>(Kw + row * P + c) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(Vw + row * P + c) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    float sc[BF_TS / 8][4];
#pragma unroll
    for (int nb = 0; nb < BF_TS / 8; ++nb) {
      sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.0f;
      const __half* kr = Kw + (nb * 8 + g) * P + 2 * tq;
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr + ks * 16);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + ks * 16 + 8);
        mma16816(sc[nb], qh[ks], b0, b1);
        mma16816(sc[nb], ql[ks], b0, b1);
      }
    }
    float mx = m;
#pragma unroll
    for (int nb = 0; nb < BF_TS / 8; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = nb * 8 + 2 * tq + e;
        const float v = key < nt ? sc[nb][e] * a.scale : -INFINITY;
        sc[nb][e] = v;
        mx = fmaxf(mx, v);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float cf = expf(m - mx);  // m = -inf on the first tile: 0
    float ps = 0.0f;
#pragma unroll
    for (int nb = 0; nb < BF_TS / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float p = sc[nb][e] == -INFINITY ? 0.0f : expf(sc[nb][e] - mx);
        sc[nb][e] = p;
        ps += p;
      }
      sc[nb][2] = sc[nb][3] = 0.0f;  // rows 8..15 carry nothing
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l = l * cf + ps;
    m = mx;
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      o[n][0] *= cf;
      o[n][1] *= cf;
    }
#pragma unroll
    for (int ks = 0; ks < BF_TS / 16; ++ks) {
      uint32_t ph[4], pl[4];
      split2(sc[2 * ks][0], sc[2 * ks][1], ph[0], pl[0]);
      split2(sc[2 * ks + 1][0], sc[2 * ks + 1][1], ph[2], pl[2]);
      ph[1] = pl[1] = ph[3] = pl[3] = 0u;
      const int vrow = ks * 16 + (lane & 15);
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        uint32_t b0, b1;
        ldsm_x2_trans(smem_u32(Vw + vrow * P + n * 8), b0, b1);
        mma16816(o[n], ph, b0, b1);
        mma16816(o[n], pl, b0, b1);
      }
    }
  }
  // merge the 4 warps (a warp without keys has m = -inf, l = 0)
  if (g < n_rep) {
    if (tq == 0) {
      wm[warp][g] = m;
      wl[warp][g] = l;
    }
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      wo[warp][g][n * 8 + 2 * tq] = o[n][0];
      wo[warp][g][n * 8 + 2 * tq + 1] = o[n][1];
    }
  }
  __syncthreads();
  const size_t pstride = HD + 2;
  for (int i = tid; i < n_rep * HD; i += BA_THREADS) {
    const int r = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][r]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = expf(wm[w][r] - M);
      L += wl[w][r] * f;
      O += wo[w][r][d] * f;
    }
    const size_t head = size_t(b) * a.n_heads + size_t(kh) * n_rep + r;
    if (nsplit == 1) {
      a.out[head * HD + d] = L > 0.0f ? O / L : 0.0f;
    } else {
      float* pp = a.part + (head * a.max_splits + split) * pstride;
      pp[2 + d] = O;
      if (d == 0) {
        pp[0] = M;
        pp[1] = L;
      }
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(a.ticket + b * a.n_kv + kh, 1) == nsplit - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) a.ticket[b * a.n_kv + kh] = 0;
  for (int i = tid; i < n_rep * HD; i += BA_THREADS) {
    const int r = i / HD, d = i % HD;
    const size_t head = size_t(b) * a.n_heads + size_t(kh) * n_rep + r;
    const float* pb = a.part + head * a.max_splits * pstride;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, __ldcg(pb + sp * pstride));
    float L = 0.0f, O = 0.0f;
#pragma unroll 4
    for (int sp = 0; sp < nsplit; ++sp) {
      const float f = expf(__ldcg(pb + sp * pstride) - M);
      L += __ldcg(pb + sp * pstride + 1) * f;
      O += __ldcg(pb + sp * pstride + 2 + d) * f;
    }
    a.out[head * HD + d] = L > 0.0f ? O / L : 0.0f;
  }
}

int g_bd_sms = 0;
// thread-block clusters of 1, 2, 4, 8 CTAs that fit on the GPU at once, per
// [NB = 16, 32][Q4_K-only, with Q6_K] shared-memory footprint (0: not queried)
int g_bd_cap[2][2][4] = {};

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
  // K slices (one cluster per tile): the most that still run as a single wave,
  // i.e. every tile's cluster resident at once (more slices = less K per CTA)
  const int tiles = batch_gemm_tiles(a, epi), nsb = a.K / QK_K;
  bool q6 = false;
  for (int i = 0; i < a.nseg; ++i) q6 |= a.seg[i].dtype == DT_Q6K;
  const int* cap = g_bd_cap[a.B > 16 ? 1 : 0][q6 ? 1 : 0];
  int splits = 1;
  for (int si = 3; si >= 1; --si) {
    const int sz = 1 << si;
    const int c = cap[si] > 0 ? cap[si] : g_bd_sms / sz;
    if (sz <= nsb && tiles <= c) {
      splits = sz;
      break;
    }
  }
  const int per = (nsb + splits - 1) / splits;
  a.sb_per_split = per;
  a.splits = (nsb + per - 1) / per;
}

template <int NB>
void bd_query_capacity(int (&cap)[2][4]) {
  for (int q6 = 0; q6 < 2; ++q6)
    for (int si = 0; si < 4; ++si) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 1u << si);
      cfg.blockDim = dim3(BD_THREADS);
      cfg.dynamicSmemBytes = bd_smem<NB>(q6 ? Q6K_DEV_BYTES : Q4K_BYTES);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = 1u << si;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, bgemm_kernel<NB>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      cap[q6][si] = n;
    }
}

cudaError_t batch_configure() {
  cudaError_t e = cudaFuncSetAttribute(bgemm_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(bd_smem<16>(Q6K_DEV_BYTES)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(bgemm_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(bd_smem<32>(Q6K_DEV_BYTES)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(bfa_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             4 * 2 * BF_TS * (128 + 8) * 2);
  if (e == cudaSuccess) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&g_bd_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || g_bd_sms <= 0)
      g_bd_sms = 148;
    bd_query_capacity<16>(g_bd_cap[0]);
    bd_query_capacity<32>(g_bd_cap[1]);
  }
  return e;
}

cudaError_t launch_batch_gemm(BatchGemmArgs a, int epi, cudaStream_t s) {
  if (a.B < 1 || a.B > BATCH_MAX || a.K % QK_K != 0 || a.rows < 1) return cudaErrorInvalidValue;
  batch_gemm_plan(a, epi);
  int bb = Q4K_BYTES;
  for (int i = 0; i < a.nseg; ++i)
    if (a.seg[i].dtype == DT_Q6K) bb = Q6K_DEV_BYTES;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(batch_gemm_tiles(a, epi), a.splits);
  cfg.blockDim = dim3(BD_THREADS);
  cfg.dynamicSmemBytes = a.B <= 16 ? bd_smem<16>(bb) : bd_smem<32>(bb);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // the K slices of a tile: one cluster
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = unsigned(a.splits);
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = a.B <= 16 ? cudaLaunchKernelEx(&cfg, bgemm_kernel<16>, a, epi)
                                  : cudaLaunchKernelEx(&cfg, bgemm_kernel<32>, a, epi);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_batch_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.n_heads % a.n_kv != 0 || a.n_heads / a.n_kv > BA_NR || a.chunk < 1) return cudaErrorInvalidValue;
  const dim3 grid(a.n_kv, a.T, a.max_splits);
  cudaError_t e;
  if (a.kv_half && a.chunk % (4 * BF_TS) == 0) {  // fp16 cache: the tensor-core kernel
    const size_t smem = size_t(4) * 2 * BF_TS * (a.head_dim + 8) * 2;
    if (a.head_dim == 64) e = bd_launch(bfa_kernel<64>, grid, dim3(BA_THREADS), smem, s, a);
    else if (a.head_dim == 128) e = bd_launch(bfa_kernel<128>, grid, dim3(BA_THREADS), smem, s, a);
    else return cudaErrorInvalidValue;
    return e != cudaSuccess ? e : cudaGetLastError();
  }
  if (a.head_dim == 64)
    e = a.kv_half ? bd_launch(battn_kernel<64, __half>, grid, dim3(BA_THREADS), 0, s, a)
                  : bd_launch(battn_kernel<64, float>, grid, dim3(BA_THREADS), 0, s, a);
  else if (a.head_dim == 128)
    e = a.kv_half ? bd_launch(battn_kernel<128, __half>, grid, dim3(BA_THREADS), 0, s, a)
                  : bd_launch(battn_kernel<128, float>, grid, dim3(BA_THREADS), 0, s, a);
  else
    return cudaErrorInvalidValue;
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_batch_resid(float* y, const float* resid, const float* add, int B, int H, float* sq,
                               cudaStream_t s) {
  if (H % BATCH_TILE != 0) return cudaErrorInvalidValue;
  const cudaError_t e = bd_launch(bresid_kernel, dim3(H / BATCH_TILE, B), dim3(BATCH_TILE), 0, s, y, resid, add, B, H, sq);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_batch_keys(const float* logits, int vl, int vocab_off, int vocab, const StepState* st,
                              const uint32_t* pen_cnt, float rep, unsigned long long* keys, int B, cudaStream_t s) {
  const cudaError_t e = bd_launch(bkey_kernel, dim3(B, 8), dim3(512), 0, s, logits, vl, vocab_off, vocab, st, pen_cnt,
                                  rep, keys);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_batch_finish(StepState* st, const unsigned long long* keys, uint32_t* hist, int hist_cap,
                                uint32_t* pen_cnt, int vocab, int B, cudaStream_t s) {
  const cudaError_t e = bd_launch(bfinish_kernel, dim3(B), dim3(32), 0, s, st, keys, hist, hist_cap, pen_cnt, vocab);
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
      bd_launch(bsample_kernel, dim3(B, BS_SPLIT), dim3(512), 0, s, logits, vocab, st, hist, hist_cap, pen_cnt, rep);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb
