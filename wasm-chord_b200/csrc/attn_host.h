// Host side of the kernel-level attention entry points (wcb_attention_dev and
// wcb_attention_dev_noalloc): one definition of the argument checks, the key
// split rule, the scratch layout and the launch sequence, so that the entry
// point with library-owned scratch and the one with a fixed scratch array
// cannot drift apart. Implemented in api.cpp.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "kernels.h"

namespace wcb {
namespace attn_host {

// WCB_OK, or the error code after recording the message for wcb_last_error:
// null or unaligned (16-byte) pointers, unsupported shapes.
uint32_t check_args(const float* q, const float* k, const float* v, const float* out, uint32_t n_tokens,
                    uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t max_seq, uint32_t kv_len);

// Kernel arguments, with the key split of a single-token call (at most 64
// splits of a multiple of 32 keys).
AttnArgs make_args(const float* q, const float* k, const float* v, float* out, uint32_t n_tokens, uint32_t n_heads,
                   uint32_t n_kv_heads, uint32_t head_dim, uint32_t max_seq, uint32_t kv_len);

// Scratch layout: StepState (256 bytes) | tickets [T][n_kv] (256-byte rounded)
// | split partials [n_heads][splits][head_dim + 2] floats (single-token calls).
size_t ticket_bytes(const AttnArgs& a);
size_t scratch_bytes(const AttnArgs& a);

// Points a at the scratch, writes the step state and launches the kernel on s.
// The tickets must be zero (the kernel leaves them zero after a completed call).
cudaError_t run(AttnArgs a, uint8_t* scratch, uint32_t kv_len, uint32_t position, cudaStream_t s);

}  // namespace attn_host
}  // namespace wcb
