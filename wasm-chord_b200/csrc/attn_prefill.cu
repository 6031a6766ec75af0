// Causal attention of a prefill chunk on the tensor cores (attention.rs:332-435 for
// T query tokens at positions position .. position+T-1 over keys 0 .. position+t).
//
// One CTA = one KV head x TQ = 128 / n_rep query tokens: its 8 warps are the
// n_rep query heads sharing the KV head (repeat_kv, attention.rs:297-322) times
// 16-token row blocks, so every K / V tile staged in shared memory serves all
// of them. Per 64-key tile a warp computes S = Q K^T (16 x 64) with
// mma.sync.m16n8k16 (fp16 operands, fp32 accumulate), applies the scale, the
// causal mask and a running softmax on the accumulator fragments, and adds
// P V into its 16 x HD output fragments (the S accumulator layout is the A
// operand layout of the second product). Precision: q and p are split into
// fp16 hi + lo halves (two products each); an f32 KV cache is split the same
// way in shared memory (three products), an f16 cache is used as is.
#include <cuda_fp16.h>

#include <cfloat>
#include <cmath>

#include "device_common.cuh"
#include "kernels.h"

namespace wcb {
namespace {

constexpr int FA_THREADS = 256;  // 8 warps
constexpr int FA_BK = 64;        // keys per tile

template <int HD, bool F32KV>
struct FaSmem {
  static constexpr int PITCH = HD + 8;  // halves per staged row (conflict-free fragment loads)
  static constexpr int TILE = FA_BK * PITCH * 2;  // bytes of one fp16 K or V tile
  // [K hi, V hi, (K lo, V lo)] for one tile
  static constexpr int BYTES = TILE * (F32KV ? 4 : 2);
};

template <int HD, typename KT>
__global__ void __launch_bounds__(FA_THREADS) fa_prefill_kernel(const AttnArgs a) {
  constexpr bool F32KV = sizeof(KT) == 4;
  using L = FaSmem<HD, F32KV>;
  constexpr int P = L::PITCH;
  extern __shared__ __align__(16) uint8_t fsm[];
  __half* Kh = reinterpret_cast<__half*>(fsm);
  __half* Vh = Kh + FA_BK * P;
  __half* Kl = Vh + FA_BK * P;  // f32 cache only
  __half* Vl = Kl + FA_BK * P;
  pdl_trigger();
  pdl_wait();
  const StepState* st = a.st;
  if (st->done) return;
  const int n_rep = a.n_heads / a.n_kv;
  const int TQ = 128 / n_rep;  // query tokens per CTA
  const int kh = blockIdx.x, t0 = blockIdx.y * TQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int r = warp % n_rep;             // query head within the KV head
  const int tb = t0 + (warp / n_rep) * 16;  // first query token of this warp
  const int head = kh * n_rep + r;
  const int pos0 = st->position;
  // keys this CTA needs: up to the last position of its tokens
  const int t_last = min(t0 + TQ, a.T) - 1;
  const int nkeys = min(st->kv_len + a.T, pos0 + t_last + 1);

  // Q fragments (A operand, 16 tokens x HD), split into hi / lo halves
  uint32_t qh[HD / 16][4], ql[HD / 16][4];
  {
    const int ta = tb + g, tb8 = tb + g + 8;
    const float* qa = a.q + (size_t(min(ta, a.T - 1)) * a.n_heads + head) * HD;
    const float* qb = a.q + (size_t(min(tb8, a.T - 1)) * a.n_heads + head) * HD;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const int c = ks * 16 + 2 * tq;
      const float2 a0 = *reinterpret_cast<const float2*>(qa + c);
      const float2 a1 = *reinterpret_cast<const float2*>(qb + c);
      const float2 a2 = *reinterpret_cast<const float2*>(qa + c + 8);
      const float2 a3 = *reinterpret_cast<const float2*>(qb + c + 8);
      split2(a0.x, a0.y, qh[ks][0], ql[ks][0]);
      split2(a1.x, a1.y, qh[ks][1], ql[ks][1]);
      split2(a2.x, a2.y, qh[ks][2], ql[ks][2]);
      split2(a3.x, a3.y, qh[ks][3], ql[ks][3]);
    }
  }
  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};  // rows g and g + 8
  const int posa = pos0 + tb + g, posb = pos0 + tb + g + 8;  // causal limits of the two rows

  const KT* Kg = reinterpret_cast<const KT*>(a.kc) + size_t(kh) * a.max_seq * HD;
  const KT* Vg = reinterpret_cast<const KT*>(a.vc) + size_t(kh) * a.max_seq * HD;
  for (int j0 = 0; j0 < nkeys; j0 += FA_BK) {
    const int nk = min(FA_BK, nkeys - j0);
    __syncthreads();  // the previous tile is no longer read
    // stage K and V rows [j0, j0 + nk) as fp16 (hi, and lo for an f32 cache); rows
    // past nk are zero
    constexpr int CH = HD / 8;  // 8-value chunks per row
    for (int i = tid; i < FA_BK * CH; i += FA_THREADS) {
      const int row = i / CH, c = (i % CH) * 8;
      uint4 kh4 = make_uint4(0, 0, 0, 0), vh4 = kh4, kl4 = kh4, vl4 = kh4;
      if (row < nk) {
        if constexpr (F32KV) {
          const float* kr = reinterpret_cast<const float*>(Kg) + size_t(j0 + row) * HD + c;
          const float* vr = reinterpret_cast<const float*>(Vg) + size_t(j0 + row) * HD + c;
          const float4 k0 = *reinterpret_cast<const float4*>(kr), k1 = *reinterpret_cast<const float4*>(kr + 4);
          const float4 v0 = *reinterpret_cast<const float4*>(vr), v1 = *reinterpret_cast<const float4*>(vr + 4);
          split2(k0.x, k0.y, kh4.x, kl4.x);
          split2(k0.z, k0.w, kh4.y, kl4.y);
          split2(k1.x, k1.y, kh4.z, kl4.z);
          split2(k1.z, k1.w, kh4.w, kl4.w);
          split2(v0.x, v0.y, vh4.x, vl4.x);
          split2(v0.z, v0.w, vh4.y, vl4.y);
          split2(v1.x, v1.y, vh4.z, vl4.z);
          split2(v1.z, v1.w, vh4.w, vl4.w);
        } else {
          kh4 = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(Kg) + size_t(j0 + row) * HD + c);
          vh4 = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(Vg) + size_t(j0 + row) * HD + c);
        }
      }
      *reinterpret_cast<uint4*>(Kh + row * P + c) = kh4;
      *reinterpret_cast<uint4*>(Vh + row * P + c) = vh4;
      if constexpr (F32KV) {
        *reinterpret_cast<uint4*>(Kl + row * P + c) = kl4;
        *reinterpret_cast<uint4*>(Vl + row * P + c) = vl4;
      }
    }
    __syncthreads();
    // warp-uniform skips: rows past the chunk, or a tile masked for all 16 rows
    if (tb >= a.T || j0 > pos0 + min(tb + 15, a.T - 1)) continue;
    // S = Q K^T: 8 blocks of 8 keys
    float s[FA_BK / 8][4];
#pragma unroll
    for (int nb = 0; nb < FA_BK / 8; ++nb) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.0f;
      const __half* kr = Kh + (nb * 8 + g) * P + 2 * tq;
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr + ks * 16);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + ks * 16 + 8);
        mma16816(s[nb], qh[ks], b0, b1);
        mma16816(s[nb], ql[ks], b0, b1);
        if constexpr (F32KV) {
          const __half* klr = Kl + (nb * 8 + g) * P + 2 * tq;
          const uint32_t c0 = *reinterpret_cast<const uint32_t*>(klr + ks * 16);
          const uint32_t c1 = *reinterpret_cast<const uint32_t*>(klr + ks * 16 + 8);
          mma16816(s[nb], qh[ks], c0, c1);
        }
      }
    }
    // scale, causal mask, running softmax (rows g and g + 8 of the warp's block)
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int nb = 0; nb < FA_BK / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j0 + nb * 8 + 2 * tq + (e & 1);
        const int lim = e < 2 ? posa : posb;
        const float v = (key <= lim && key < nkeys) ? s[nb][e] * a.scale : -INFINITY;
        s[nb][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float cf[2], ps[2] = {0.0f, 0.0f};
#pragma unroll
    for (int h = 0; h < 2; ++h) cf[h] = mx[h] == -INFINITY ? 1.0f : expf(mrow[h] - mx[h]);
#pragma unroll
    for (int nb = 0; nb < FA_BK / 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = mx[e >> 1];
        const float p = s[nb][e] == -INFINITY ? 0.0f : expf(s[nb][e] - m);
        s[nb][e] = p;
        ps[e >> 1] += p;
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ps[h] += __shfl_xor_sync(0xffffffffu, ps[h], 1);
      ps[h] += __shfl_xor_sync(0xffffffffu, ps[h], 2);
      lrow[h] = lrow[h] * cf[h] + ps[h];
      mrow[h] = mx[h];
    }
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      o[n][0] *= cf[0];
      o[n][1] *= cf[0];
      o[n][2] *= cf[1];
      o[n][3] *= cf[1];
    }
    // O += P V: 16-key steps; P (hi, lo) from the S fragments, V via ldmatrix.trans
#pragma unroll
    for (int ks = 0; ks < FA_BK / 16; ++ks) {
      uint32_t ph[4], pl[4];
      split2(s[2 * ks][0], s[2 * ks][1], ph[0], pl[0]);
      split2(s[2 * ks][2], s[2 * ks][3], ph[1], pl[1]);
      split2(s[2 * ks + 1][0], s[2 * ks + 1][1], ph[2], pl[2]);
      split2(s[2 * ks + 1][2], s[2 * ks + 1][3], ph[3], pl[3]);
      const int vrow = ks * 16 + (lane & 15);  // lanes 0-7: keys 0-7, lanes 8-15: keys 8-15
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        uint32_t b0, b1;
        ldsm_x2_trans(smem_u32(Vh + vrow * P + n * 8), b0, b1);
        mma16816(o[n], ph, b0, b1);
        mma16816(o[n], pl, b0, b1);
        if constexpr (F32KV) {
          uint32_t c0, c1;
          ldsm_x2_trans(smem_u32(Vl + vrow * P + n * 8), c0, c1);
          mma16816(o[n], ph, c0, c1);
        }
      }
    }
  }
  if (tb >= a.T) return;
  // O / l, rows g and g + 8 (tokens tb + g, tb + g + 8)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int t = tb + g + 8 * h;
    if (t >= a.T) continue;
    const float inv = lrow[h] > 0.0f ? 1.0f / lrow[h] : 0.0f;
    float* out = a.out + (size_t(t) * a.n_heads + head) * HD;
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      const float2 v = make_float2(lrow[h] > 0.0f ? o[n][2 * h] * inv : 0.0f,
                                   lrow[h] > 0.0f ? o[n][2 * h + 1] * inv : 0.0f);
      *reinterpret_cast<float2*>(out + n * 8 + 2 * tq) = v;
    }
  }
}

template <typename Kern>
cudaError_t fa_launch(Kern kern, dim3 grid, size_t smem, cudaStream_t s, const AttnArgs& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(FA_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

cudaError_t attention_prefill_configure() {
  cudaError_t e = cudaFuncSetAttribute(fa_prefill_kernel<128, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       FaSmem<128, true>::BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(fa_prefill_kernel<64, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             FaSmem<64, true>::BYTES);
  return e;
}

bool attention_prefill_supported(int n_heads, int n_kv, int head_dim) {
  const int n_rep = n_kv > 0 ? n_heads / n_kv : 0;
  return (head_dim == 64 || head_dim == 128) && n_kv > 0 && n_heads % n_kv == 0 &&
         (n_rep == 1 || n_rep == 2 || n_rep == 4 || n_rep == 8);
}

cudaError_t launch_attention_prefill(const AttnArgs& a, cudaStream_t s) {
  if (!attention_prefill_supported(a.n_heads, a.n_kv, a.head_dim) || a.T < 1) return cudaErrorInvalidValue;
  const int tq = 128 / (a.n_heads / a.n_kv);
  const dim3 grid(a.n_kv, (a.T + tq - 1) / tq);
  cudaError_t e;
  if (a.head_dim == 64)
    e = a.kv_half ? fa_launch(fa_prefill_kernel<64, __half>, grid, FaSmem<64, false>::BYTES, s, a)
                  : fa_launch(fa_prefill_kernel<64, float>, grid, FaSmem<64, true>::BYTES, s, a);
  else
    e = a.kv_half ? fa_launch(fa_prefill_kernel<128, __half>, grid, FaSmem<128, false>::BYTES, s, a)
                  : fa_launch(fa_prefill_kernel<128, float>, grid, FaSmem<128, true>::BYTES, s, a);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace wcb
