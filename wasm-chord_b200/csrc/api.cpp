// C ABI (include/wcb.h). Error handling follows the reference C ABI
// (crates/wasm-chord-runtime/src/abi.rs, lib.rs:80-118): every entry point
// returns a uint32 ErrorCode and records the message in a thread-local slot
// read by wcb_last_error; no C++ exception crosses the boundary.
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <string>

#include "../../include/wcb.h"
#include "gguf.h"
#include "kernels.h"
#include "model.h"
#include "sampler.h"

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

}  // namespace

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

uint32_t wcb_model_load(const char* path, const wcb_load_opts* opts, uint32_t* out_handle) {
  return guarded([&]() -> uint32_t {
    if (!path || !out_handle) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *out_handle = 0;
    wcb::LoadOptions o;
    if (opts) {
      o.device = opts->device;
      o.max_seq = opts->max_seq;
      if (opts->kv_dtype > WCB_KV_F16) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: kv_dtype");
      o.kv_half = opts->kv_dtype == WCB_KV_F16;
      o.max_batch = opts->max_batch ? opts->max_batch : 1;
      o.flags = opts->flags;
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
    size_t off = 0;
    for (size_t s = 0; s < n_seq; ++s) {
      n_out[s] = 0;
      std::vector<uint32_t> toks = m->generate(prompts + off, lens[s], params_of(cfg));
      n_out[s] = toks.size();
      std::memcpy(out + s * cap, toks.data(), sizeof(uint32_t) * std::min(cap, toks.size()));
      off += lens[s];
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
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = wcb::gemv_configure_all();
    if (e != cudaSuccess) return cuda_fail(e, "configure");
    configured = true;
  }
  wcb::GemvArgs a{};
  a.seg[0].w = static_cast<const uint8_t*>(w);
  a.seg[0].dtype = int(dtype);
  a.seg[0].rows = int(n);
  a.nseg = 1;
  a.K = int(k);
  a.ngroups = int(n / 4);
  const int chunks = int(k / 256) * (dtype == WCB_DTYPE_Q4_K ? 8 : 4);
  int ks = 1;
  while (ks < 8 && a.ngroups * ks < 148 * 16 && chunks / (ks * 2) >= 16) ks *= 2;
  a.ksplit = ks;
  a.ldx = int(k);
  a.ldy = int(n);
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

uint32_t wcb_model_stream(uint32_t h, void** out) {
  return guarded([&]() -> uint32_t {
    if (!out) return fail(WCB_ERR_INVALID_ARGUMENT, "Invalid argument: null pointer");
    *out = get_model(h)->stream();
    return WCB_OK;
  });
}

}  // extern "C"
