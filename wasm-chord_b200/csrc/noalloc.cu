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

#include <cstdint>
#include <map>
#include <mutex>
#include <string>

#include "../../include/wcb.h"
#include "attn_host.h"
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
  namespace ah = wcb::attn_host;
  // the same checks, split rule and scratch layout as wcb_attention_dev (attn_host.h)
  const uint32_t rc0 = ah::check_args(q, k_cache, v_cache, out, n_tokens, n_heads, n_kv_heads, head_dim, max_seq,
                                      kv_len);
  if (rc0 != WCB_OK) return rc0;
  const wcb::AttnArgs a = ah::make_args(q, k_cache, v_cache, out, n_tokens, n_heads, n_kv_heads, head_dim, max_seq,
                                        kv_len);
  const size_t need = ah::scratch_bytes(a);
  if (need > kScratchBytes)
    return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid tensor shape: this call needs " + std::to_string(need) +
                                              " bytes of scratch, more than the fixed " +
                                              std::to_string(kScratchBytes) + " bytes of wcb_attention_dev_noalloc");
  uint8_t* scratch = nullptr;
  const uint32_t rc = scratch_for_current_device(&scratch);
  if (rc != WCB_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the array keeps whatever the previous call left: the split tickets must start at zero
  cudaError_t e = cudaMemsetAsync(scratch + 256, 0, ah::ticket_bytes(a), s);
  if (e == cudaSuccess) e = ah::run(a, scratch, kv_len, position, s);
  if (e != cudaSuccess) return fail(WCB_ERR_BACKEND_UNSUPPORTED, std::string("Backend error: attention: ") +
                                                                 cudaGetErrorString(e));
  return WCB_OK;
}
