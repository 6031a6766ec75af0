// C ABI (include/wcb.h). Error handling follows the reference C ABI
// (crates/wasm-chord-runtime/src/abi.rs, lib.rs:80-118): every entry point
// returns a uint32 ErrorCode and records the message in a thread-local slot
// read by wcb_last_error; no C++ exception crosses the boundary.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <string>

#include "../../include/wcb.h"
#include "attn_host.h"
#include "gguf.h"
#include "kernels.h"
#include "model.h"
#include "nccl_rt.h"
#include "sampler.h"
#include "tokenizer.h"

namespace {

thread_local std::string g_last_error;

std::mutex g_mu;
std::map<uint32_t, std::shared_ptr<wcb::Model>> g_models;
std::map<uint32_t, std::shared_ptr<wcb::Sampler>> g_samplers;
struct Stream {
  std::shared_ptr<wcb::Model> model;
  uint64_t session;
};
std::map<uint32_t, Stream> g_streams;
uint32_t g_next_model = 1;
uint32_t g_next_sampler = 1;
uint32_t g_next_stream = 1;
std::map<uint32_t, std::shared_ptr<wcb::Tokenizer>> g_tokenizers;
uint32_t g_next_tokenizer = 1;

std::shared_ptr<wcb::Tokenizer> get_tokenizer(uint32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_tokenizers.find(h);
  if (it == g_tokenizers.end()) throw wcb::WcbError(WCB_ERR_INVALID_ARGUMENT, "Invalid tokenizer handle");
  return it->second;
}

// the reference takes &str: the text must be well-formed UTF-8
bool valid_utf8(const char* s, size_t n) {
  size_t i = 0;
  while (i < n) {
    const unsigned char c = static_cast<unsigned char>(s[i]);
    size_t need;
    unsigned char lo = 0x80, hi = 0xBF;
    if (c < 0x80) need = 0;
    else if (c >= 0xC2 && c <= 0xDF) need = 1;
    else if (c == 0xE0) need = 2, lo = 0xA0;
    else if ((c >= 0xE1 && c <= 0xEC) || c == 0xEE || c == 0xEF) need = 2;
    else if (c == 0xED) need = 2, hi = 0x9F;
    else if (c == 0xF0) need = 3, lo = 0x90;
    else if (c >= 0xF1 && c <= 0xF3) need = 3;
    else if (c == 0xF4) need = 3, hi = 0x8F;
    else return false;
    if (need && i + need >= n) return false;  // truncated sequence
    for (size_t k = 1; k <= need; ++k) {
      const unsigned char d = static_cast<unsigned char>(s[i + k]);
      if (d < (k == 1 ? lo : 0x80) || d > (k == 1 ? hi : 0xBF)) return false;
    }
    i += need + 1;
  }
  return true;
}

// copies a string into a caller buffer (NUL-terminated, truncated to cap - 1 bytes)
void copy_out(const std::string& s, char* out, size_t cap, size_t* n_out) {
  *n_out = s.size();
  if (out && cap) {
    const size_t k = std::min(cap - 1, s.size());
    std::memcpy(out, s.data(), k);
    out[k] = '\0';
  }
}

uint32_t fail(uint32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

template <class F>
uint32_t guarded(F&& fn) {
  try {
    return fn();
  } catch (const wcb::WcbError& e) {
    return fail(e.code, e.what());
  } catch (const std::bad_alloc&) {
    return fail(WCB_ERR_OOM, "Memory allocation failed");
  } catch (const std::exception& e) {
    return fail(WCB_ERR_GENERIC, std::string("Runtime error: ") + e.what());
  } catch (...) {
    return fail(WCB_ERR_GENERIC, "Unknown error");
  }
}

std::shared_ptr<wcb::Model> get_model(uint32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_models.find(h);
  if (it == g_models.end()) throw wcb::WcbError(WCB_ERR_INVALID_ARGUMENT, "Invalid model handle");
  return it->second;
}

wcb::GenParams params_of(const wcb_gen_config* c) {
  wcb::GenParams g;
  g.max_tokens = c->max_tokens;
  g.temperature = c->temperature;
  g.top_p = c->top_p;
  g.top_k = c->top_k;
  g.repetition_penalty = c->repetition_penalty;
  g.seed = c->seed;
  g.eos = c->eos_id;
  return g;
}

uint32_t cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? WCB_ERR_OOM : WCB_ERR_BACKEND_UNSUPPORTED,
              std::string("Backend error: ") + what + ": " + cudaGetErrorString(e));
}

// Per device, for wcb_gemv_dev: kernel attributes set once, and BATCH_MAX zeroed
// sequence states for the batched tensor-core GEMM (it reads position / kv_len /
// done of each activation row and records an expired bounded wait in state 0).
struct GemvDevice {
  bool configured = false;
  wcb::StepState* states = nullptr;
};
std::mutex g_gemv_mu;
std::map<int, GemvDevice> g_gemv_dev;

cudaError_t gemv_device(GemvDevice** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_gemv_mu);
  GemvDevice& g = g_gemv_dev[dev];
  if (!g.configured) {
    e = wcb::gemv_configure_all();
    if (e == cudaSuccess) e = wcb::gemm_tc_configure();
    if (e == cudaSuccess) e = wcb::batch_configure();
    if (e == cudaSuccess && !g.states) {
      void* p = nullptr;
      e = cudaMalloc(&p, sizeof(wcb::StepState) * wcb::BATCH_MAX);
      if (e == cudaSuccess) e = cudaMemset(p, 0, sizeof(wcb::StepState) * wcb::BATCH_MAX);
      if (e == cudaSuccess) g.states = static_cast<wcb::StepState*>(p);
      else if (p) cudaFree(p);
    }
    if (e != cudaSuccess) return e;
    g.configured = true;
  }
  *out = &g;
  return cudaSuccess;
}

}  // namespace

// lets the other translation units of the library report through wcb_last_error
extern "C" __attribute__((visibility("hidden"))) void wcb_internal_set_last_error(const char* msg) {
  g_last_error = msg ? msg : "";
}

extern "C" {

void wcb_gen_config_default(wcb_gen_config* c) {
  if (!c) return;
  c->max_tokens = 100;
  c->temperature = 0.7f;
  c->top_p = 0.9f;
  c->top_k = 40;
  c->repetition_penalty = 1.1f;
  c->seed = 42;
  c->eos_id = 2;
}

static_assert(offsetof(wcb_load_opts, wait_ms) == WCB_LOAD_OPTS_V1_SIZE, "v1 fields end where wait_ms starts");
static_assert(sizeof(wcb_load_opts) == WCB_LOAD_OPTS_V1_SIZE + 4, "wcb_load_opts has no padding");

void wcb_load_opts_init(wcb_load_opts* o) {
  if (!o) return;
  std::memset(o, 0, sizeof(*o));
  o->struct_size = uint32_t(sizeof(wcb_load_opts));
  o->kv_dtype = WCB_KV_F32;
  o->max_batch = 1;
  o->tp_size = 1;
  o->wait_ms = 2000;
}

size_t wcb_struct_layout(const char* s, const char* f) {
  if (!s) return SIZE_MAX;
  const std::string st(s), fl(f ? f : "");
#define WCB_FIELD(T, F) \
  if (fl == #F) return offsetof(T, F);
  if (st == "wcb_load_opts") {
    if (!f) return sizeof(wcb_load_opts);
    WCB_FIELD(wcb_load_opts, struct_size) WCB_FIELD(wcb_load_opts, device) WCB_FIELD(wcb_load_opts, max_seq)
    WCB_FIELD(wcb_load_opts, kv_dtype) WCB_FIELD(wcb_load_opts, max_batch) WCB_FIELD(wcb_load_opts, flags)
    WCB_FIELD(wcb_load_opts, tp_rank) WCB_FIELD(wcb_load_opts, tp_size) WCB_FIELD(wcb_load_opts, tp_id)
    WCB_FIELD(wcb_load_opts, wait_ms)
  } else if (st == "wcb_gen_config") {
    if (!f) return sizeof(wcb_gen_config);
    WCB_FIELD(wcb_gen_config, max_tokens) WCB_FIELD(wcb_gen_config, temperature) WCB_FIELD(wcb_gen_config, top_p)
    WCB_FIELD(wcb_gen_config, top_k) WCB_FIELD(wcb_gen_config, repetition_penalty) WCB_FIELD(wcb_gen_config, seed)
    WCB_FIELD(wcb_gen_config, eos_id)
  } else if (st == "wcb_model_config") {
    if (!f) return sizeof(wcb_model_config);
    WCB_FIELD(wcb_model_config, vocab_size) WCB_FIELD(wcb_model_config, hidden_size)
    WCB_FIELD(wcb_model_config, num_layers) WCB_FIELD(wcb_model_config, num_heads)
    WCB_FIELD(wcb_model_config, num_kv_heads) WCB_FIELD(wcb_model_config, intermediate_size)
    WCB_FIELD(wcb_model_config, max_seq_len) WCB_FIELD(wcb_model_config, head_dim)
    WCB_FIELD(wcb_model_config, rms_norm_eps) WCB_FIELD(wcb_model_config, rope_theta)
  }
#undef WCB_FIELD
  return SIZE_MAX;
}

uint32_t wcb_model_load(const char* path, const wcb_load_opts* opts, uint32_t* out_handle) {
  return guarded([&]() -> uint32_t {
    if (!path || !out_handle) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *out_handle = 0;
    wcb::LoadOptions o;
    if (opts) {
      // read only the bytes the caller initialised; later fields keep their defaults
      if (opts->struct_size < WCB_LOAD_OPTS_V1_SIZE)
        return fail(WCB_ERR_INVALID_ARGUMENT,
                    "Invalid argument: wcb_load_opts.struct_size is " + std::to_string(opts->struct_size) +
                        " (initialise the options with wcb_load_opts_init)");
      wcb_load_opts v;
      wcb_load_opts_init(&v);
      std::memcpy(&v, opts, std::min<size_t>(opts->struct_size, sizeof(v)));
      o.device = v.device;
      o.max_seq = v.max_seq;
      if (v.kv_dtype > WCB_KV_F16) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: kv_dtype");
      o.kv_half = v.kv_dtype == WCB_KV_F16;
      o.max_batch = v.max_batch ? v.max_batch : 1;
      o.flags = v.flags;
      o.tp_rank = v.tp_rank;
      o.tp_size = v.tp_size ? v.tp_size : 1;
      if (o.tp_size > 8 || o.tp_rank >= o.tp_size)
        return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: tp_rank / tp_size");
      std::memcpy(o.tp_id, v.tp_id, sizeof(o.tp_id));
      if (v.wait_ms > 60000) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: wait_ms > 60000");
      o.wait_ms = v.wait_ms ? v.wait_ms : 2000;
    }
    auto m = std::make_shared<wcb::Model>(path, o);
    std::lock_guard<std::mutex> lk(g_mu);
    const uint32_t h = g_next_model++;
    g_models[h] = std::move(m);
    *out_handle = h;
    return WCB_OK;
  });
}

uint32_t wcb_model_free(uint32_t h) {
  return guarded([&]() -> uint32_t {
    std::shared_ptr<wcb::Model> m;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_models.find(h);
      if (it == g_models.end()) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid model handle");
      m = std::move(it->second);
      g_models.erase(it);
      for (auto s = g_streams.begin(); s != g_streams.end();)
        s = s->second.model == m ? g_streams.erase(s) : std::next(s);
    }
    return WCB_OK;
  });
}

uint32_t wcb_model_config_get(uint32_t h, wcb_model_config* out) {
  return guarded([&]() -> uint32_t {
    if (!out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    auto m = get_model(h);
    const wcb::ModelConfig& c = m->config();
    out->vocab_size = c.vocab;
    out->hidden_size = c.hidden;
    out->num_layers = c.layers;
    out->num_heads = c.heads;
    out->num_kv_heads = c.kv_heads;
    out->intermediate_size = c.ffn;
    out->max_seq_len = c.max_seq;
    out->head_dim = c.head_dim();
    out->rms_norm_eps = c.eps;
    out->rope_theta = c.theta;
    return WCB_OK;
  });
}

uint32_t wcb_forward(uint32_t h, const uint32_t* ids, size_t n, size_t position, float* logits_out) {
  return guarded([&]() -> uint32_t {
    if ((!ids && n) || !logits_out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    get_model(h)->forward(ids, n, position, logits_out);
    return WCB_OK;
  });
}

uint32_t wcb_clear_kv(uint32_t h) {
  return guarded([&]() -> uint32_t {
    get_model(h)->clear_kv();
    return WCB_OK;
  });
}

uint32_t wcb_kv_len(uint32_t h, size_t* out) {
  return guarded([&]() -> uint32_t {
    if (!out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *out = get_model(h)->kv_len();
    return WCB_OK;
  });
}

uint32_t wcb_generate_tokens(uint32_t h, const uint32_t* prompt, size_t n, const wcb_gen_config* cfg, uint32_t* out,
                             size_t cap, size_t* n_out) {
  return guarded([&]() -> uint32_t {
    if (!cfg || !n_out || (!out && cap) || (!prompt && n))
      return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *n_out = 0;
    auto m = get_model(h);
    std::vector<uint32_t> toks = m->generate(prompt, n, params_of(cfg));
    *n_out = toks.size();
    std::memcpy(out, toks.data(), sizeof(uint32_t) * std::min(cap, toks.size()));
    return WCB_OK;
  });
}

uint32_t wcb_generate_batch(uint32_t h, const uint32_t* prompts, const size_t* lens, size_t n_seq,
                            const wcb_gen_config* cfg, uint32_t* out, size_t cap, size_t* n_out) {
  return guarded([&]() -> uint32_t {
    if (!cfg || !n_out || !lens || (!out && cap) || !prompts)
      return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    auto m = get_model(h);
    for (size_t s = 0; s < n_seq; ++s) n_out[s] = 0;
    const std::vector<std::vector<uint32_t>> toks = m->generate_batch(prompts, lens, n_seq, params_of(cfg));
    for (size_t s = 0; s < n_seq; ++s) {
      n_out[s] = toks[s].size();
      std::memcpy(out + s * cap, toks[s].data(), sizeof(uint32_t) * std::min(cap, toks[s].size()));
    }
    return WCB_OK;
  });
}

uint32_t wcb_infer(uint32_t h, const uint32_t* prompt, size_t n, const wcb_gen_config* cfg, uint32_t* out_stream) {
  return guarded([&]() -> uint32_t {
    if (!cfg || !out_stream || (!prompt && n)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *out_stream = 0;
    auto m = get_model(h);
    m->start(prompt, n, params_of(cfg));
    std::lock_guard<std::mutex> lk(g_mu);
    const uint32_t id = g_next_stream++;
    g_streams[id] = Stream{m, m->session_id()};
    *out_stream = id;
    return WCB_OK;
  });
}

static std::shared_ptr<wcb::Model> stream_model(uint32_t sid) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_streams.find(sid);
  if (it == g_streams.end()) throw wcb::WcbError(WCB_ERR_INVALID_ARGUMENT, "Invalid stream handle");
  if (it->second.model->session_id() != it->second.session)
    throw wcb::WcbError(WCB_ERR_INVALID_ARGUMENT, "Invalid stream handle: a newer generation replaced it");
  return it->second.model;
}

uint32_t wcb_next_tokens(uint32_t sid, size_t max_tokens, uint32_t* out, size_t* n_out, uint32_t* finished) {
  return guarded([&]() -> uint32_t {
    if (!n_out || (!out && max_tokens)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *n_out = 0;
    if (finished) *finished = 0;
    auto m = stream_model(sid);
    bool fin = false;
    std::vector<uint32_t> t = m->next(max_tokens, &fin);
    std::memcpy(out, t.data(), sizeof(uint32_t) * t.size());
    *n_out = t.size();
    if (finished) *finished = fin ? 1u : 0u;
    return WCB_OK;
  });
}

int32_t wcb_next_token(uint32_t sid, uint32_t* out_token) {
  if (!out_token) {
    fail(WCB_ERR_INVALID_ARGUMENT, "Invalid buffer pointer");
    return -2;
  }
  size_t n = 0;
  uint32_t fin = 0;
  if (wcb_next_tokens(sid, 1, out_token, &n, &fin) != WCB_OK) return -2;
  return n ? 1 : -1;
}

uint32_t wcb_close_stream(uint32_t sid) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_streams.erase(sid)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid stream handle");
  return WCB_OK;
}

uint32_t wcb_batch_info(uint32_t h, uint32_t* slots, uint32_t* launches_per_step) {
  return guarded([&]() -> uint32_t {
    if (!slots || !launches_per_step) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    auto m = get_model(h);
    *slots = m->batch_slots();
    *launches_per_step = uint32_t(m->launches_per_batch_step());
    return WCB_OK;
  });
}

uint32_t wcb_model_launches_per_step(uint32_t h, uint32_t* out) {
  return guarded([&]() -> uint32_t {
    if (!out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *out = uint32_t(get_model(h)->launches_per_decode_step());
    return WCB_OK;
  });
}

uint32_t wcb_sampler_new(const wcb_gen_config* cfg, uint32_t* out) {
  return guarded([&]() -> uint32_t {
    if (!cfg || !out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    auto s = std::make_shared<wcb::Sampler>(cfg->seed, cfg->temperature, cfg->top_p, cfg->top_k,
                                            cfg->repetition_penalty);
    std::lock_guard<std::mutex> lk(g_mu);
    const uint32_t id = g_next_sampler++;
    g_samplers[id] = std::move(s);
    *out = id;
    return WCB_OK;
  });
}

uint32_t wcb_sampler_sample(uint32_t sid, float* logits, size_t n, uint32_t* tok) {
  return guarded([&]() -> uint32_t {
    if (!logits || !tok) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    std::shared_ptr<wcb::Sampler> s;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_samplers.find(sid);
      if (it == g_samplers.end()) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid sampler handle");
      s = it->second;
    }
    *tok = s->sample(logits, n);
    return WCB_OK;
  });
}

uint32_t wcb_sampler_probs(uint32_t sid, float* out, size_t n) {
  return guarded([&]() -> uint32_t {
    if (!out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    std::shared_ptr<wcb::Sampler> s;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_samplers.find(sid);
      if (it == g_samplers.end()) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid sampler handle");
      s = it->second;
    }
    const std::vector<float>& p = s->last_probs();
    if (p.size() != n)
      return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: the last sampled draw had " + std::to_string(p.size()) +
                                                " probabilities (none after an argmax), not " + std::to_string(n));
    std::copy(p.begin(), p.end(), out);
    return WCB_OK;
  });
}

uint32_t wcb_sampler_free(uint32_t sid) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_samplers.erase(sid)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid sampler handle");
  return WCB_OK;
}

size_t wcb_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return 0;
  const std::string msg = g_last_error.empty() ? std::string("No error") : g_last_error;
  g_last_error.clear();
  const size_t n = std::min(len - 1, msg.size());
  std::memcpy(buf, msg.data(), n);
  buf[n] = 0;
  return n;
}

const char* wcb_version(void) { return "wcb-0.1.0 (sm_100a)"; }

uint32_t wcb_tp_id(uint8_t out[128]) {
  if (!out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
  return guarded([&]() -> uint32_t {
    ncclUniqueId id;
    const ncclResult_t r = wcb::nccl().GetUniqueId(&id);
    if (r != ncclSuccess)
      throw wcb::WcbError(wcb::E_BACKEND, std::string("Backend error: ncclGetUniqueId: ") + wcb::nccl().GetErrorString(r));
    static_assert(sizeof(id) == 128, "NCCL unique id size");
    std::memcpy(out, &id, sizeof(id));
    return WCB_OK;
  });
}

uint32_t wcb_dequant_dev(const void* blocks, uint32_t dtype, size_t nblocks, float* out, void* stream) {
  if (dtype != WCB_DTYPE_Q4_K && dtype != WCB_DTYPE_Q6_K)
    return fail(WCB_ERR_INVALID_ARGUMENT, "Unsupported data type: dequant supports Q4_K and Q6_K");
  if (nblocks && (!blocks || !out)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
  const cudaError_t e = wcb::launch_dequant(blocks, int(dtype), nblocks, out, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? WCB_OK : cuda_fail(e, "dequant");
}

uint32_t wcb_repack_q6k_dev(const void* packed, size_t nblocks, void* padded, void* stream) {
  if (nblocks && (!packed || !padded)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
  const cudaError_t e = wcb::launch_repack_q6k(packed, nblocks, padded, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? WCB_OK : cuda_fail(e, "repack");
}

uint32_t wcb_gemv_dev(const void* w, uint32_t dtype, size_t n, size_t k, const float* x, size_t m, float* y,
                      void* stream) {
  if (dtype != WCB_DTYPE_Q4_K && dtype != WCB_DTYPE_Q6_K)
    return fail(WCB_ERR_INVALID_ARGUMENT, "Unsupported data type: gemv supports Q4_K and Q6_K");
  if (!w || !x || !y) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
  if (k == 0 || k % 256 || n == 0 || n % 4 || m == 0 || m > 4096 || k > (1u << 20) || n > (1u << 28))
    return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid tensor shape: need k % 256 == 0, n % 4 == 0, 1 <= m <= 4096");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15)
    return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: x and w must be 16-byte aligned");
  GemvDevice* gd = nullptr;
  {
    const cudaError_t e = gemv_device(&gd);
    if (e != cudaSuccess) return cuda_fail(e, "configure");
  }
  if (m > 4 && m <= size_t(wcb::BATCH_MAX)) {
    // 5..32 rows: the batched decode GEMM (tcgen05, M = 128 weight rows, N = 2 x rows),
    // one launch that reads every weight byte once
    wcb::BatchGemmArgs b{};
    b.seg[0].w = static_cast<const uint8_t*>(w);
    b.seg[0].dtype = int(dtype);
    b.seg[0].rows = int(n);
    b.nseg = 1;
    b.rows = int(n);
    b.K = int(k);
    b.B = int(m);
    b.x = x;
    b.ldx = int(k);
    b.y = y;
    b.ldy = int(n);
    b.st = gd->states;
    const cudaError_t e = wcb::launch_batch_gemm(b, wcb::BEPI_STORE, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WCB_OK : cuda_fail(e, "batched gemm");
  }
  wcb::GemvArgs a{};
  a.seg[0].w = static_cast<const uint8_t*>(w);
  a.seg[0].dtype = int(dtype);
  a.seg[0].rows = int(n);
  a.nseg = 1;
  a.K = int(k);
  a.ngroups = int(n / 4);
  a.ldx = int(k);
  a.ldy = int(n);
  if (m >= size_t(wcb::TC_MIN_TOKENS)) {  // tensor-core GEMM (tcgen05)
    a.M = int(m);
    a.x = x;
    a.y = y;
    const cudaError_t e = wcb::launch_gemm_tc(a, wcb::PRO_NONE, wcb::EPI_STORE, nullptr, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? WCB_OK : cuda_fail(e, "gemm");
  }
  const int mmax = wcb::gemv_max_cols(int(k));
  for (size_t c0 = 0; c0 < m; c0 += size_t(mmax)) {
    wcb::GemvArgs b = a;
    b.M = int(std::min(size_t(mmax), m - c0));
    b.x = x + c0 * k;
    b.y = y + c0 * n;
    const cudaError_t e = wcb::launch_gemv(b, wcb::PRO_NONE, wcb::EPI_STORE, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "gemv");
  }
  return WCB_OK;
}

}  // extern "C"

namespace wcb {
namespace attn_host {

uint32_t check_args(const float* q, const float* k, const float* v, const float* out, uint32_t T, uint32_t nh,
                    uint32_t nkv, uint32_t hd, uint32_t max_seq, uint32_t kv_len) {
  if (!q || !k || !v || !out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
  // the kernel reads q and the K / V rows and writes out with 16-byte accesses
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: q, k_cache, v_cache and out must be 16-byte aligned");
  if ((hd != 64 && hd != 128) || nkv == 0 || nh % nkv || nh / nkv > 16 || T == 0 || T > 4096 || kv_len < T ||
      kv_len > max_seq)
    return fail(WCB_ERR_INVALID_ARGUMENT,
                "Invalid tensor shape: need head_dim 64|128, n_heads % n_kv_heads == 0 (<= 16 per kv head), "
                "1 <= n_tokens <= kv_len <= max_seq");
  return WCB_OK;
}

AttnArgs make_args(const float* q, const float* k, const float* v, float* out, uint32_t T, uint32_t nh,
                   uint32_t nkv, uint32_t hd, uint32_t max_seq, uint32_t kv_len) {
  AttnArgs a{};
  a.q = q;
  a.kc = k;
  a.vc = v;
  a.kv_half = 0;
  a.out = out;
  a.n_heads = int(nh);
  a.n_kv = int(nkv);
  a.head_dim = int(hd);
  a.max_seq = int(max_seq);
  a.T = int(T);
  a.scale = 1.0f / std::sqrt(float(hd));
  if (T == 1) {  // at most 64 splits of a multiple of 32 keys
    int sp = int((kv_len + 31) / 32);
    sp = sp < 1 ? 1 : (sp > 64 ? 64 : sp);
    int c = int((kv_len + uint32_t(sp) - 1) / uint32_t(sp));
    c = (c + 31) / 32 * 32;
    a.chunk = c;
    a.max_splits = int((kv_len + uint32_t(c) - 1) / uint32_t(c));
  } else {
    a.chunk = int(max_seq);
    a.max_splits = 1;
  }
  return a;
}

size_t ticket_bytes(const AttnArgs& a) { return (sizeof(int) * size_t(a.T) * a.n_kv + 255) / 256 * 256; }

size_t scratch_bytes(const AttnArgs& a) {
  const size_t part = a.T == 1 ? sizeof(float) * size_t(a.n_heads) * a.max_splits * (a.head_dim + 2) : 0;
  return 256 + ticket_bytes(a) + part;
}

cudaError_t run(AttnArgs a, uint8_t* scratch, uint32_t kv_len, uint32_t position, cudaStream_t s) {
  StepState* st = reinterpret_cast<StepState*>(scratch);
  a.ticket = reinterpret_cast<int*>(scratch + 256);
  a.part = reinterpret_cast<float*>(scratch + 256 + ticket_bytes(a));
  a.st = st;
  cudaError_t e = launch_set_state(st, int(position), int(kv_len - uint32_t(a.T)), a.T, s);
  if (e == cudaSuccess) e = launch_attention(a, s);
  return e;
}

}  // namespace attn_host
}  // namespace wcb

namespace {
// Scratch of wcb_attention_dev (StepState, split tickets, split partials),
// allocated once per device with cudaMalloc and grown on demand, and the
// devices whose kernel attributes (shared-memory limits) are set.
std::mutex g_attn_mu;
std::map<int, std::pair<void*, size_t>> g_attn_scratch;
std::map<int, bool> g_attn_configured;
}  // namespace

extern "C" {

uint32_t wcb_attention_dev(const float* q, const float* k_cache, const float* v_cache, float* out, uint32_t n_tokens,
                           uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t max_seq,
                           uint32_t kv_len, uint32_t position, void* stream) {
  namespace ah = wcb::attn_host;
  const uint32_t rc = ah::check_args(q, k_cache, v_cache, out, n_tokens, n_heads, n_kv_heads, head_dim, max_seq,
                                     kv_len);
  if (rc != WCB_OK) return rc;
  const wcb::AttnArgs a = ah::make_args(q, k_cache, v_cache, out, n_tokens, n_heads, n_kv_heads, head_dim, max_seq,
                                        kv_len);
  const size_t need = ah::scratch_bytes(a);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  uint8_t* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_attn_mu);
    if (!g_attn_configured[dev]) {  // kernel attributes are per device
      e = wcb::gemv_configure_all();
      if (e != cudaSuccess) return cuda_fail(e, "configure");
      g_attn_configured[dev] = true;
    }
    auto& slot = g_attn_scratch[dev];
    if (slot.second < need) {
      if (slot.first) {
        cudaDeviceSynchronize();
        cudaFree(slot.first);
        slot.first = nullptr;
        slot.second = 0;
      }
      e = cudaMalloc(&slot.first, need);
      if (e == cudaSuccess) e = cudaMemset(slot.first, 0, need);
      if (e != cudaSuccess) return cuda_fail(e, "attention scratch");
      slot.second = need;
    }
    scratch = static_cast<uint8_t*>(slot.first);
  }
  e = ah::run(a, scratch, kv_len, position, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? WCB_OK : cuda_fail(e, "attention");
}

uint32_t wcb_model_tp_handle(uint32_t h, uint8_t out[64]) {
  return guarded([&]() -> uint32_t {
    if (!out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    get_model(h)->tp_ipc_handle(out);
    return WCB_OK;
  });
}

uint32_t wcb_model_tp_connect(uint32_t h, const uint8_t* handles, uint32_t n_ranks) {
  return guarded([&]() -> uint32_t {
    if (!handles) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    get_model(h)->tp_connect(handles, n_ranks);
    return WCB_OK;
  });
}

uint32_t wcb_model_tp_abort(uint32_t h) {
  return guarded([&]() -> uint32_t {
    get_model(h)->tp_abort();
    return WCB_OK;
  });
}

uint32_t wcb_model_stream(uint32_t h, void** out) {
  return guarded([&]() -> uint32_t {
    if (!out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *out = get_model(h)->stream();
    return WCB_OK;
  });
}

}  // extern "C"

extern "C" {

uint32_t wcb_tokenizer_load(const char* gguf_path, uint32_t* out_handle) {
  return guarded([&]() -> uint32_t {
    if (!gguf_path || !out_handle) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *out_handle = 0;
    const wcb::GgufFile f(gguf_path);
    auto t = std::make_shared<wcb::Tokenizer>(wcb::Tokenizer::from_gguf(f));
    std::lock_guard<std::mutex> lk(g_mu);
    const uint32_t h = g_next_tokenizer++;
    g_tokenizers[h] = std::move(t);
    *out_handle = h;
    return WCB_OK;
  });
}

uint32_t wcb_tokenizer_free(uint32_t h) {
  return guarded([&]() -> uint32_t {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_tokenizers.erase(h)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid tokenizer handle");
    return WCB_OK;
  });
}

uint32_t wcb_tokenizer_info(uint32_t h, uint32_t* vocab_size, uint32_t* bos, uint32_t* eos, uint32_t* unk) {
  return guarded([&]() -> uint32_t {
    if (!vocab_size || !bos || !eos || !unk) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    auto t = get_tokenizer(h);
    *vocab_size = uint32_t(t->vocab_size());
    *bos = t->special().bos;
    *eos = t->special().eos;
    *unk = t->special().unk;
    return WCB_OK;
  });
}

uint32_t wcb_tokenizer_set_special(uint32_t h, uint32_t add_bos, uint32_t add_eos) {
  return guarded([&]() -> uint32_t {
    auto t = get_tokenizer(h);
    t->set_add_bos(add_bos != 0);
    t->set_add_eos(add_eos != 0);
    return WCB_OK;
  });
}

uint32_t wcb_tokenize(uint32_t h, const char* text, uint32_t add_special, uint32_t* out, size_t cap, size_t* n_out) {
  return guarded([&]() -> uint32_t {
    if (!text || !n_out || (!out && cap)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    const size_t n = std::strlen(text);
    if (!valid_utf8(text, n)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: text is not valid UTF-8");
    const std::vector<uint32_t> ids = get_tokenizer(h)->encode(std::string(text, n), add_special != 0);
    *n_out = ids.size();
    if (cap) std::memcpy(out, ids.data(), sizeof(uint32_t) * std::min(cap, ids.size()));
    return WCB_OK;
  });
}

uint32_t wcb_detokenize(uint32_t h, const uint32_t* ids, size_t n, uint32_t skip_special, char* out, size_t cap,
                        size_t* n_out) {
  return guarded([&]() -> uint32_t {
    if (!n_out || (!ids && n)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    copy_out(get_tokenizer(h)->decode(ids, n, skip_special != 0), out, cap, n_out);
    return WCB_OK;
  });
}

uint32_t wcb_generate_text(uint32_t model, uint32_t tokenizer, const char* prompt, const wcb_gen_config* cfg,
                           char* out, size_t cap, size_t* n_out) {
  return guarded([&]() -> uint32_t {
    if (!prompt || !cfg || !n_out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    const size_t n = std::strlen(prompt);
    if (!valid_utf8(prompt, n)) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: text is not valid UTF-8");
    auto t = get_tokenizer(tokenizer);
    auto m = get_model(model);
    // Model::generate (model.rs:1322-1415): encode with BOS, the tokenizer's EOS ends
    // the loop, and the whole sequence (prompt + generated) is decoded without specials
    std::vector<uint32_t> ids = t->encode(std::string(prompt, n), true);
    wcb::GenParams g = params_of(cfg);
    g.eos = t->special().eos;
    const std::vector<uint32_t> gen = m->generate(ids.data(), ids.size(), g);
    ids.insert(ids.end(), gen.begin(), gen.end());
    copy_out(t->decode(ids.data(), ids.size(), true), out, cap, n_out);
    return WCB_OK;
  });
}

}  // extern "C"
