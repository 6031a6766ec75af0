// wcb_attention_dev_noalloc: the GQA attention kernel for callers that cannot
// allocate GPU memory.
//
// wcb_attention_dev obtains its scratch (step state, split tickets and the
// partial results of the key splits) with cudaMalloc the first time a device
// needs it, and again whenever a larger problem needs more. Some hosts cannot
// allow that after they have started: a runtime that has already handed all
// device memory to its own pool, or a serving loop that must never pause every
// stream for the device-wide synchronisation cudaMalloc and cudaFree imply.
// This variant takes its scratch from a fixed array compiled into the library
// instead, so it never allocates; the caller still provides q, the K/V caches
// and the output.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>

#include "../../include/wcb.h"
#include "kernels.h"

namespace {

// Largest scratch a call may use: the 256-byte step state, one ticket per
// (query token, kv head) and, for a single query token, the partial results of
// up to 64 key splits (n_heads * splits * (head_dim + 2) floats). 4 MiB covers
// 64 query heads of 128 dimensions at 64 splits with room to spare. Every GPU
// that loads the library holds this array until the process exits.
constexpr size_t kScratchBytes = size_t(4) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
std::map<int, uint8_t*> g_addr;  // device ordinal -> device address of g_noalloc_scratch

uint32_t fail(uint32_t code, const std::string& msg);

// Set-up, once per device with that device current: the host-side name of the
// array is only a stand-in, so its device address is looked up here and passed
// to the kernel explicitly.
uint32_t scratch_for_current_device(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(WCB_ERR_BACKEND_UNSUPPORTED, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_addr.find(dev);
  if (it == g_addr.end()) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(WCB_ERR_BACKEND_UNSUPPORTED,
                  std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    e = wcb::gemv_configure_all();  // kernel attributes; sets no memory aside
    if (e != cudaSuccess) return fail(WCB_ERR_BACKEND_UNSUPPORTED, std::string("configure: ") + cudaGetErrorString(e));
    it = g_addr.emplace(dev, static_cast<uint8_t*>(p)).first;
  }
  *out = it->second;
  return WCB_OK;
}

}  // namespace

// Error strings of this entry point go through wcb_last_error like every other call.
extern "C" __attribute__((visibility("hidden"))) void wcb_internal_set_last_error(const char* msg);

namespace {
uint32_t fail(uint32_t code, const std::string& msg) {
  wcb_internal_set_last_error(msg.c_str());
  return code;
}
}  // namespace

extern "C" uint32_t wcb_attention_dev_noalloc(const float* q, const float* k_cache, const float* v_cache, float* out,
                                              uint32_t n_tokens, uint32_t n_heads, uint32_t n_kv_heads,
                                              uint32_t head_dim, uint32_t max_seq, uint32_t kv_len, uint32_t position,
                                              void* stream) {
  if (!q || !k_cache || !v_cache || !out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
  if ((head_dim != 64 && head_dim != 128) || n_kv_heads == 0 || n_heads % n_kv_heads ||
      n_heads / n_kv_heads > 16 || n_tokens == 0 || n_tokens > 4096 || kv_len < n_tokens || kv_len > max_seq)
    return fail(WCB_ERR_INVALID_ARGUMENT,
                "Invalid tensor shape: need head_dim 64|128, n_heads % n_kv_heads == 0 (<= 16 per kv head), "
                "1 <= n_tokens <= kv_len <= max_seq");
  wcb::AttnArgs a{};
  a.q = q;
  a.kc = k_cache;
  a.vc = v_cache;
  a.kv_half = 0;
  a.out = out;
  a.n_heads = int(n_heads);
  a.n_kv = int(n_kv_heads);
  a.head_dim = int(head_dim);
  a.max_seq = int(max_seq);
  a.T = int(n_tokens);
  a.scale = 1.0f / std::sqrt(float(head_dim));
  if (n_tokens == 1) {  // the split rule of wcb_attention_dev: <= 64 splits of a multiple of 32 keys
    int sp = int((kv_len + 31) / 32);
    sp = sp < 1 ? 1 : (sp > 64 ? 64 : sp);
    int ch = int((kv_len + uint32_t(sp) - 1) / uint32_t(sp));
    ch = (ch + 31) / 32 * 32;
    a.chunk = ch;
    a.max_splits = int((kv_len + uint32_t(ch) - 1) / uint32_t(ch));
  } else {
    a.chunk = int(max_seq);
    a.max_splits = 1;
  }
  // layout: step state | tickets | partials (same as wcb_attention_dev)
  const size_t tickets = (sizeof(int) * size_t(a.T) * a.n_kv + 255) / 256 * 256;
  const size_t part = a.T == 1 ? sizeof(float) * size_t(a.n_heads) * a.max_splits * (a.head_dim + 2) : 0;
  const size_t need = 256 + tickets + part;
  if (need > kScratchBytes)
    return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid tensor shape: this call needs " + std::to_string(need) +
                                              " bytes of scratch, more than the fixed " +
                                              std::to_string(kScratchBytes) + " bytes of wcb_attention_dev_noalloc");
  uint8_t* scratch = nullptr;
  const uint32_t rc = scratch_for_current_device(&scratch);
  if (rc != WCB_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  wcb::StepState* st = reinterpret_cast<wcb::StepState*>(scratch);
  a.ticket = reinterpret_cast<int*>(scratch + 256);
  a.part = reinterpret_cast<float*>(scratch + 256 + tickets);
  a.st = st;
  // the array keeps whatever the previous call left: the split tickets must start at zero
  cudaError_t e = cudaMemsetAsync(a.ticket, 0, tickets, s);
  if (e == cudaSuccess) e = wcb::launch_set_state(st, int(position), int(kv_len - n_tokens), a.T, s);
  if (e == cudaSuccess) e = wcb::launch_attention(a, s);
  if (e != cudaSuccess) return fail(WCB_ERR_BACKEND_UNSUPPORTED, std::string("Backend error: attention: ") +
                                                                 cudaGetErrorString(e));
  return WCB_OK;
}
