// ORACLE — test infrastructure only. Nothing in the product links or calls
// this file; tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
// it as the checker and as the timed CPU baseline.
//
// A CPU restatement, in C++17, of the wasm-chord reference's transformer token
// loop (default features: no memory64, no GPU backends). Every function cites
// the reference function it restates (paths relative to the wasm-chord tree).
// Build: g++ -O2 -ffp-contract=off (no fast-math, no FMA contraction), so f32
// expressions round exactly as the Rust source does (Rust never contracts).
//
// Pinning: Q4_K/Q6_K dequantisation is checked bit-exactly against gguf-py
// 0.19.0 (an independent implementation of the same ggml formats) and the
// reference's known-answer tests are restated in tests/test_oracle.py.
// Summation order of the two third-party candle ops (rms_norm, the LM-head
// matmul) is not pinned: candle's rms_norm is restated as a sequential f32 sum
// and the LM head as matmul_transposed's sequential dot product. The
// stochastic-sampling random stream (rand 0.9 StdRng = ChaCha12, seeded by
// rand_core's seed_from_u64, and the Uniform<f32> draw of WeightedIndex) is
// restated from those crates' published algorithms (they are not under the
// reference tree); its ChaCha block function is pinned by the RFC 8439 ChaCha20
// known-answer vectors (tests/test_oracle.py), the seeding and the draw are not.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <numeric>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace oracle {

// Error kinds mirror wasm-chord-core/src/error.rs:5-32 and their C-ABI codes
// (wasm-chord-runtime/src/lib.rs:80-103).
enum Code : uint32_t { OK = 0, GENERIC = 1, OOM = 2, INVALID_ARG = 3, PARSE = 4, BACKEND = 5, IO = 7 };
struct Error : std::runtime_error {
  uint32_t code;
  Error(uint32_t c, const std::string& m) : std::runtime_error(m), code(c) {}
};

static thread_local std::string g_last_error;

// half::f16::to_f32 (half 2.7): exact widening, subnormals included.
float f16_to_f32(uint16_t h) {
  uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1F, mant = h & 0x3FF, out;
  if (exp == 0) {
    if (mant == 0) {
      out = sign;
    } else {
      int e = -1;
      do { e++; mant <<= 1; } while (!(mant & 0x400));
      out = sign | (uint32_t(127 - 15 - e) << 23) | ((mant & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    out = sign | 0x7F800000u | (mant << 13);
  } else {
    out = sign | ((exp + 112) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

// ---------------------------------------------------------------------------
// quant.rs
// ---------------------------------------------------------------------------
// get_scale_min_k4 — wasm-chord-core/src/quant.rs:43-53
static inline void get_scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
  if (j < 4) {
    *d = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *d = uint8_t((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *m = uint8_t((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

// dequantize_q4_k — quant.rs:58-115. Block = {d f16, dmin f16, scales[12], qs[128]}.
void dequantize_q4_k(const uint8_t* blk, float* out) {
  uint16_t dbits, mbits;
  std::memcpy(&dbits, blk, 2);
  std::memcpy(&mbits, blk + 2, 2);
  const float d = f16_to_f32(dbits);
  const float min = f16_to_f32(mbits);
  const uint8_t* scales = blk + 4;
  const uint8_t* qs = blk + 16;
  for (int i = 0; i < 4; ++i) {
    uint8_t sc, m;
    get_scale_min_k4(2 * i, scales, &sc, &m);
    const float d1 = d * float(sc);
    const float m1 = min * float(m);
    get_scale_min_k4(2 * i + 1, scales, &sc, &m);
    const float d2 = d * float(sc);
    const float m2 = min * float(m);
    for (int j = 0; j < 32; ++j) out[64 * i + j] = d1 * float(qs[32 * i + j] & 0xF) - m1;
    for (int j = 0; j < 32; ++j) out[64 * i + 32 + j] = d2 * float(qs[32 * i + j] >> 4) - m2;
  }
}

// dequantize_q6_k — quant.rs:206-261. Block = {ql[128], qh[64], scales i8[16], d f16}.
void dequantize_q6_k(const uint8_t* blk, float* out) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
  uint16_t dbits;
  std::memcpy(&dbits, blk + 208, 2);
  const float d = f16_to_f32(dbits);
  for (int half = 0; half < 2; ++half) {
    const uint8_t* l8 = ql + 64 * half;
    const uint8_t* h8 = qh + 32 * half;
    const int8_t* s = sc + 8 * half;
    float* y = out + 128 * half;
    for (int l = 0; l < 32; ++l) {
      const int is = l / 16;
      const int8_t q1 = int8_t((l8[l] & 0x0F) | ((h8[l] & 3) << 4)) - 32;
      const int8_t q2 = int8_t((l8[l + 32] & 0x0F) | (((h8[l] >> 2) & 3) << 4)) - 32;
      const int8_t q3 = int8_t((l8[l] >> 4) | (((h8[l] >> 4) & 3) << 4)) - 32;
      const int8_t q4 = int8_t((l8[l + 32] >> 4) | (((h8[l] >> 6) & 3) << 4)) - 32;
      y[l] = d * float(s[is]) * float(q1);
      y[l + 32] = d * float(s[is + 2]) * float(q2);
      y[l + 64] = d * float(s[is + 4]) * float(q3);
      y[l + 96] = d * float(s[is + 6]) * float(q4);
    }
  }
}

// ---------------------------------------------------------------------------
// GGUF — wasm-chord-core/src/formats/gguf.rs
// ---------------------------------------------------------------------------
enum DType { F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9,
             Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, UNSUPPORTED = 255 };

struct MetaValue {
  int type = -1;  // GGUF value type
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  std::vector<MetaValue> arr;
  bool as_u32(uint32_t* out) const {  // MetadataValue::as_u32, gguf.rs:50-62
    switch (type) {
      case 0: case 2: case 4: case 10: *out = uint32_t(u); return true;
      case 1: case 3: case 5: case 11: *out = uint32_t(i); return true;
      default: return false;
    }
  }
  bool as_f32(float* out) const {  // gguf.rs:64-70
    if (type == 6) { *out = float(f); return true; }
    if (type == 12) { *out = float(f); return true; }
    return false;
  }
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;
  DType dtype;
  uint64_t offset;
  uint64_t numel;
  uint64_t size_bytes;
};

// TensorDesc::new byte sizes — wasm-chord-core/src/tensor.rs:133-189
static uint64_t tensor_bytes(DType t, uint64_t n) {
  switch (t) {
    case Q4_0: case Q4_1: return n / 32 * 16;
    case Q8_0: case Q8_1: return n / 32 * 33;
    case Q4_K: return n / 256 * 144;
    case Q6_K: return n / 256 * 210;
    case Q5_K: return n / 256 * 176;
    case Q2_K: case Q3_K: case Q5_0: case Q5_1: case UNSUPPORTED: return n / 2;
    case F32: return n * 4;
    case F16: return n * 2;
  }
  return n / 2;
}

struct Gguf {
  std::ifstream f;
  uint32_t version = 0;
  std::map<std::string, MetaValue> meta;
  std::vector<TensorInfo> tensors;
  std::map<std::string, size_t> by_name;
  uint64_t data_offset = 0;
  std::string arch;

  template <class T> T rd() {
    T v;
    f.read(reinterpret_cast<char*>(&v), sizeof(T));
    if (!f) throw Error(IO, "unexpected end of file");
    return v;
  }
  std::string rd_str() {
    uint64_t n = rd<uint64_t>();
    if (n > (1ull << 32)) throw Error(PARSE, "string too long");
    std::string s(n, '\0');
    if (n) f.read(&s[0], std::streamsize(n));
    if (!f) throw Error(IO, "unexpected end of file");
    return s;
  }
  // read_typed_value — gguf.rs:389-405 (arrays of arrays are rejected there too)
  MetaValue rd_value(uint32_t t, bool allow_array) {
    MetaValue v;
    v.type = int(t);
    switch (t) {
      case 0: v.u = rd<uint8_t>(); break;
      case 1: v.i = rd<int8_t>(); break;
      case 2: v.u = rd<uint16_t>(); break;
      case 3: v.i = rd<int16_t>(); break;
      case 4: v.u = rd<uint32_t>(); break;
      case 5: v.i = rd<int32_t>(); break;
      case 6: v.f = rd<float>(); break;
      case 7: v.u = rd<uint8_t>() != 0; break;
      case 8: v.s = rd_str(); break;
      case 9: {
        if (!allow_array) throw Error(PARSE, "Unknown typed value: 9");
        uint32_t et = rd<uint32_t>();
        uint64_t n = rd<uint64_t>();
        for (uint64_t k = 0; k < n; ++k) v.arr.push_back(rd_value(et, false));
        break;
      }
      case 10: v.u = rd<uint64_t>(); break;
      case 11: v.i = rd<int64_t>(); break;
      case 12: v.f = rd<double>(); break;
      default: throw Error(PARSE, "Unknown metadata value type: " + std::to_string(t));
    }
    return v;
  }
  // parse_header — gguf.rs:111-159, tensor_data_offset — :162-172
  void open(const std::string& path) {
    f.open(path, std::ios::binary);
    if (!f) throw Error(IO, "cannot open " + path);
    if (rd<uint32_t>() != 0x46554747u) throw Error(PARSE, "Invalid GGUF magic");
    version = rd<uint32_t>();
    if (version < 2 || version > 3) throw Error(PARSE, "Unsupported GGUF version: " + std::to_string(version));
    uint64_t n_tensors = rd<uint64_t>();
    uint64_t n_kv = rd<uint64_t>();
    for (uint64_t k = 0; k < n_kv; ++k) {
      std::string key = rd_str();
      uint32_t t = rd<uint32_t>();
      meta[key] = rd_value(t, true);
    }
    for (uint64_t k = 0; k < n_tensors; ++k) {  // parse_tensor_info — gguf.rs:414-444
      TensorInfo ti;
      ti.name = rd_str();
      uint32_t nd = rd<uint32_t>();
      if (nd > 8) throw Error(PARSE, "too many dims");
      ti.numel = 1;
      for (uint32_t d = 0; d < nd; ++d) { ti.dims.push_back(rd<uint64_t>()); ti.numel *= ti.dims.back(); }
      uint32_t dt = rd<uint32_t>();
      switch (dt) {  // parse_dtype — gguf.rs:446-467
        case 0: case 1: case 2: case 3: case 6: case 7: case 8: case 9: case 10: case 11:
        case 12: case 13: case 14: ti.dtype = DType(dt); break;
        default: ti.dtype = UNSUPPORTED;
      }
      ti.offset = rd<uint64_t>();
      ti.size_bytes = tensor_bytes(ti.dtype, ti.numel);
      by_name[ti.name] = tensors.size();
      tensors.push_back(ti);
    }
    uint64_t pos = uint64_t(f.tellg());
    data_offset = (pos + 31) & ~uint64_t(31);
    auto it = meta.find("general.architecture");
    arch = (it != meta.end() && it->second.type == 8) ? it->second.s : "unknown";
  }
  const MetaValue* get(const std::string& k) const {
    auto it = meta.find(k);
    return it == meta.end() ? nullptr : &it->second;
  }
  uint32_t cfg_u32(const std::string& a, const std::string& b, uint32_t dflt) const {
    uint32_t v;
    const MetaValue* m = get(a);
    if (!m) m = get(b);
    if (m && m->as_u32(&v)) return v;
    return dflt;
  }
  float cfg_f32(const std::string& a, const std::string& b, float dflt) const {
    float v;
    const MetaValue* m = get(a);
    if (!m) m = get(b);
    if (m && m->as_f32(&v)) return v;
    return dflt;
  }
  std::vector<uint8_t> raw(const TensorInfo& t) {
    std::vector<uint8_t> buf(t.size_bytes);
    f.clear();
    f.seekg(std::streamoff(data_offset + t.offset));
    if (t.size_bytes) f.read(reinterpret_cast<char*>(buf.data()), std::streamsize(t.size_bytes));
    if (!f) throw Error(IO, "failed to fill whole buffer: " + t.name);
    return buf;
  }
};

// TransformerConfig — transformer/config.rs:6-41; extract_config — gguf.rs:208-276
struct Config {
  uint32_t vocab = 32000, hidden = 2048, layers = 22, heads = 32, kv_heads = 4, ffn = 5632, max_seq = 2048;
  float eps = 1e-5f, theta = 10000.0f;
  uint32_t head_dim() const { return hidden / heads; }
};

static Config extract_config(const Gguf& g) {
  const std::string& a = g.arch;
  Config c;
  c.vocab = g.cfg_u32(a + ".vocab_size", "vocab_size", 32000);
  c.hidden = g.cfg_u32(a + ".embedding_length", a + ".hidden_size", 2048);
  c.layers = g.cfg_u32(a + ".block_count", a + ".num_layers", 22);
  c.heads = g.cfg_u32(a + ".attention.head_count", a + ".num_heads", 32);
  c.kv_heads = g.cfg_u32(a + ".attention.head_count_kv", a + ".num_kv_heads", 4);
  c.ffn = g.cfg_u32(a + ".feed_forward_length", a + ".intermediate_size", 5632);
  c.max_seq = g.cfg_u32(a + ".context_length", a + ".max_seq_len", 2048);
  c.eps = g.cfg_f32(a + ".attention.layer_norm_rms_epsilon", "rms_norm_eps", 1e-5f);
  c.theta = g.cfg_f32(a + ".rope.freq_base", "rope_theta", 10000.0f);
  return c;
}

static int g_load_threads = 8;  // load-time dequantisation (independent blocks, identical values)

template <class F>
static void par_blocks(size_t n, F fn) {
  const int th = std::max(1, g_load_threads);
  if (th == 1 || n < 4096) {
    for (size_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::vector<std::thread> pool;
  const size_t chunk = (n + size_t(th) - 1) / size_t(th);
  for (int t = 0; t < th; ++t) {
    const size_t a = size_t(t) * chunk, b = std::min(n, a + chunk);
    if (a >= b) break;
    pool.emplace_back([=, &fn] { for (size_t i = a; i < b; ++i) fn(i); });
  }
  for (auto& p : pool) p.join();
}

// TensorLoader::load_tensor — wasm-chord-core/src/tensor_loader.rs:50-149 (f32 result)
static std::vector<float> load_tensor(Gguf& g, const TensorInfo& t) {
  std::vector<uint8_t> raw = g.raw(t);
  std::vector<float> out(t.numel, 0.0f);
  switch (t.dtype) {
    case F32:
      for (uint64_t i = 0; i + 4 <= raw.size() && i / 4 < t.numel; i += 4) std::memcpy(&out[i / 4], &raw[i], 4);
      break;
    case F16:
      for (uint64_t i = 0; i + 2 <= raw.size() && i / 2 < t.numel; i += 2) {
        uint16_t h;
        std::memcpy(&h, &raw[i], 2);
        out[i / 2] = f16_to_f32(h);
      }
      break;
    case Q4_K:
      if (t.numel % 256) throw Error(INVALID_ARG, "Output buffer must be 256 elements");
      par_blocks(raw.size() / 144, [&](size_t b) { dequantize_q4_k(&raw[144 * b], &out[256 * b]); });
      break;
    case Q6_K:
      if (t.numel % 256) throw Error(INVALID_ARG, "Output buffer must be 256 elements");
      par_blocks(raw.size() / 210, [&](size_t b) { dequantize_q6_k(&raw[210 * b], &out[256 * b]); });
      break;
    default:
      throw Error(INVALID_ARG, "Unsupported dtype for loading: " + t.name);
  }
  return out;
}

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
static int g_threads = 1;  // threads for the LM head (candle runs it multithreaded)
static int g_proj_threads = 1;  // threads for the projections (the reference runs them on one)
// 1: one output row at a time, exactly the reference's loop (timed CPU baseline);
// 0: four independent rows interleaved per pass (same per-row arithmetic, faster)
static int g_faithful = 0;

template <class F>
static void par_rows(size_t n, int threads, F fn) {
  if (threads <= 1 || n < 64) { fn(size_t(0), n); return; }
  std::vector<std::thread> pool;
  size_t chunk = (n + size_t(threads) - 1) / size_t(threads);
  for (int t = 0; t < threads; ++t) {
    size_t a = size_t(t) * chunk, b = std::min(n, a + chunk);
    if (a >= b) break;
    pool.emplace_back([=] { fn(a, b); });
  }
  for (auto& th : pool) th.join();
}

// matmul_transposed — wasm-chord-cpu/src/gemm.rs:83-143: C[i,j] = sum_l A[i,l]*B[j,l],
// l ascending into one f32 accumulator (the 4-way unroll adds in the same order).
// Rows j are independent, so splitting them over threads leaves every result unchanged.
void matmul_transposed(const float* a, const float* b, float* c, size_t m, size_t k, size_t n, int threads) {
  for (size_t i = 0; i < m; ++i) {
    const float* ar = a + i * k;
    par_rows(n, threads, [&](size_t j0, size_t j1) {
      size_t j = j0;
      // four independent rows at a time: each row still sums in its own order
      for (; !g_faithful && j + 4 <= j1; j += 4) {
        const float* b0 = b + j * k;
        const float *b1 = b0 + k, *b2 = b1 + k, *b3 = b2 + k;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        for (size_t l = 0; l < k; ++l) {
          const float x = ar[l];
          s0 += x * b0[l];
          s1 += x * b1[l];
          s2 += x * b2[l];
          s3 += x * b3[l];
        }
        c[i * n + j] = s0; c[i * n + j + 1] = s1; c[i * n + j + 2] = s2; c[i * n + j + 3] = s3;
      }
      for (; j < j1; ++j) {
        const float* br = b + j * k;
        float s = 0.0f;
        for (size_t l = 0; l < k; ++l) s += ar[l] * br[l];
        c[i * n + j] = s;
      }
    });
  }
}

// CandleTensorBackend::rms_norm — wasm-chord-cpu/src/candle_tensor_backend.rs:30-57,
// which calls candle_nn::ops::rms_norm: per row m = sqrt(sum(x^2)/dim + eps),
// y = x / m * alpha. Summation order restated as sequential (unpinned, see header).
void rms_norm(const float* x, const float* w, float eps, size_t seq, size_t hidden, float* out) {
  for (size_t s = 0; s < seq; ++s) {
    const float* r = x + s * hidden;
    float sum2 = 0.0f;
    for (size_t i = 0; i < hidden; ++i) sum2 += r[i] * r[i];
    const float m = std::sqrt(sum2 / float(hidden) + eps);
    for (size_t i = 0; i < hidden; ++i) out[s * hidden + i] = r[i] / m * w[i];
  }
}

// MultiHeadAttention::apply_rope — transformer/attention.rs:203-265 (interleaved pairs)
void apply_rope(float* t, size_t start_pos, size_t seq, size_t heads, size_t hd, float theta) {
  for (size_t s = 0; s < seq; ++s) {
    const size_t pos = start_pos + s;
    for (size_t h = 0; h < heads; ++h) {
      float* base = t + (s * heads + h) * hd;
      for (size_t i = 0; i < hd; i += 2) {
        const float freq = 1.0f / std::pow(theta, float(i) / float(hd));
        const float angle = float(pos) * freq;
        const float c = std::cos(angle), sn = std::sin(angle);
        const float x0 = base[i], x1 = base[i + 1];
        base[i] = x0 * c - x1 * sn;
        base[i + 1] = x0 * sn + x1 * c;
      }
    }
  }
}

// compute_attention (+ repeat_kv) — transformer/attention.rs:297-435
void compute_attention(const float* q, const float* k, const float* v, size_t seq, size_t kv_seq,
                       size_t position, size_t heads, size_t kv_heads, size_t hd, float* out) {
  const size_t n_rep = heads / kv_heads;
  const float scale = 1.0f / std::sqrt(float(hd));
  std::fill(out, out + seq * heads * hd, 0.0f);
  std::vector<float> scores(kv_seq);
  for (size_t h = 0; h < heads; ++h) {
    const size_t kh = h / n_rep;
    for (size_t i = 0; i < seq; ++i) {
      const float* qv = q + (i * heads + h) * hd;
      for (size_t j = 0; j < kv_seq; ++j) {
        const float* kv = k + (j * kv_heads + kh) * hd;
        float sc = 0.0f;
        for (size_t d = 0; d < hd; ++d) sc += qv[d] * kv[d];
        scores[j] = sc * scale;
        if (j > position + i) scores[j] = -INFINITY;
      }
      float mx = -INFINITY;
      for (size_t j = 0; j < kv_seq; ++j) mx = std::fmax(mx, scores[j]);  // fold(f32::max)
      float sum = 0.0f;
      for (size_t j = 0; j < kv_seq; ++j) {
        if (std::isfinite(scores[j])) {
          scores[j] = std::exp(scores[j] - mx);
          sum += scores[j];
        } else {
          scores[j] = 0.0f;
        }
      }
      if (sum > 0.0f)
        for (size_t j = 0; j < kv_seq; ++j) scores[j] /= sum;
      float* o = out + (i * heads + h) * hd;
      for (size_t j = 0; j < kv_seq; ++j) {
        const float* vv = v + (j * kv_heads + kh) * hd;
        const float wgt = scores[j];
        for (size_t d = 0; d < hd; ++d) o[d] += wgt * vv[d];
      }
    }
  }
}

// KVCache — transformer/kv_cache.rs:6-73. [max_seq][n_kv][hd] f32.
struct KVCache {
  std::vector<float> keys, values;
  size_t cur = 0, max_seq, n_kv, hd;
  KVCache(size_t m, size_t nk, size_t h) : keys(m * nk * h, 0.0f), values(m * nk * h, 0.0f), max_seq(m), n_kv(nk), hd(h) {}
  void clear() {
    std::fill(keys.begin(), keys.end(), 0.0f);
    std::fill(values.begin(), values.end(), 0.0f);
    cur = 0;
  }
  // append — kv_cache.rs:44-67 (returns the new length; the caller reads [0, len))
  size_t append(const float* k, const float* v, size_t seq) {
    if (cur + seq > max_seq)
      throw Error(PARSE, "KV cache overflow: " + std::to_string(cur) + " + " + std::to_string(seq) + " > " + std::to_string(max_seq));
    const size_t row = n_kv * hd;
    std::copy(k, k + seq * row, keys.begin() + cur * row);
    std::copy(v, v + seq * row, values.begin() + cur * row);
    cur += seq;
    return cur;
  }
};

// ---------------------------------------------------------------------------
// sampling.rs — LogitsProcessor
// ---------------------------------------------------------------------------
// rand 0.9 rngs::StdRng (sampling.rs:40, :75): rand_chacha's ChaCha12Rng, a block
// RNG over the ChaCha keystream (RFC 8439 section 2.3, here with `rounds` rounds,
// 12 for StdRng): state = 4 constant words, the 32-byte seed as 8 little-endian
// key words, a 64-bit block counter (words 12-13, from 0) and a 64-bit stream id
// (words 14-15, 0). Words are handed out in keystream order, one block at a time.
struct Rng {
  uint32_t st[16];
  uint32_t buf[16];
  int pos = 16;
  int rounds;
  Rng(const uint8_t seed[32], int rounds_) : rounds(rounds_) {
    static const char sigma[] = "expand 32-byte k";
    for (int i = 0; i < 4; ++i) st[i] = le32(reinterpret_cast<const uint8_t*>(sigma) + 4 * i);
    for (int i = 0; i < 8; ++i) st[4 + i] = le32(seed + 4 * i);
    st[12] = st[13] = st[14] = st[15] = 0;
  }
  // SeedableRng::seed_from_u64 (rand_core 0.9): 32 seed bytes, 4 at a time, from a
  // PCG32 whose state is first advanced by an LCG step, output = XSH-RR permutation
  explicit Rng(uint64_t seed) : Rng(pcg_fill(seed).data(), 12) {}
  static std::vector<uint8_t> pcg_fill(uint64_t state) {
    std::vector<uint8_t> out(32);
    for (size_t off = 0; off < out.size(); off += 4) {
      state = state * 6364136223846793005ull + 11634580027462260723ull;
      const uint32_t xs = uint32_t(((state >> 18) ^ state) >> 27);
      const unsigned rot = unsigned(state >> 59);
      const uint32_t x = (xs >> rot) | (xs << ((32u - rot) & 31u));
      for (int b = 0; b < 4; ++b) out[off + b] = uint8_t(x >> (8 * b));
    }
    return out;
  }
  static uint32_t le32(const uint8_t* p) {
    return uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24;
  }
  static uint32_t rotl(uint32_t v, unsigned c) { return (v << c) | (v >> (32u - c)); }
  static void quarter(uint32_t* w, int a, int b, int c, int d) {
    w[a] += w[b]; w[d] ^= w[a]; w[d] = rotl(w[d], 16);
    w[c] += w[d]; w[b] ^= w[c]; w[b] = rotl(w[b], 12);
    w[a] += w[b]; w[d] ^= w[a]; w[d] = rotl(w[d], 8);
    w[c] += w[d]; w[b] ^= w[c]; w[b] = rotl(w[b], 7);
  }
  // one keystream block at the current counter into buf, then counter + 1
  void refill() {
    uint32_t w[16];
    std::memcpy(w, st, sizeof(w));
    for (int r = 0; r < rounds; r += 2) {
      quarter(w, 0, 4, 8, 12); quarter(w, 1, 5, 9, 13); quarter(w, 2, 6, 10, 14); quarter(w, 3, 7, 11, 15);
      quarter(w, 0, 5, 10, 15); quarter(w, 1, 6, 11, 12); quarter(w, 2, 7, 8, 13); quarter(w, 3, 4, 9, 14);
    }
    for (int i = 0; i < 16; ++i) buf[i] = w[i] + st[i];
    if (++st[12] == 0) ++st[13];
    pos = 0;
  }
  uint32_t next_u32() {
    if (pos >= 16) refill();
    return buf[pos++];
  }
};

// rand 0.9 distr::uniform::UniformFloat<f32>: new(low, high) and sample()
struct UniformF32 {
  float low, scale;
  UniformF32(float lo, float hi) : low(lo), scale(hi - lo) {
    const float max_rand = 1.0f - FLT_EPSILON;
    while (scale * max_rand + low >= hi) {  // shrink the scale by one ulp until the top value stays below hi
      uint32_t b;
      std::memcpy(&b, &scale, 4);
      --b;
      std::memcpy(&scale, &b, 4);
    }
  }
  float sample(Rng& r) const {
    const uint32_t bits = (r.next_u32() >> 9) | (127u << 23);  // [1, 2)
    float v;
    std::memcpy(&v, &bits, 4);
    return (v - 1.0f) * scale + low;
  }
};

enum SamplingKind { ARGMAX, ALL, TOPK, TOPP, TOPK_TOPP };

struct LogitsProcessor {
  Rng rng;
  SamplingKind kind;
  double temperature = 0, p = 0;
  size_t k = 0;
  float rep;
  std::vector<uint32_t> prev;

  // with_params — sampling.rs:57-78
  LogitsProcessor(uint64_t seed, double t, double top_p, size_t top_k, float rep_pen) : rng(seed), rep(rep_pen) {
    temperature = t; p = top_p; k = top_k;
    if (t < 1e-7) kind = ARGMAX;
    else if (top_k > 0 && top_p > 0.0 && top_p < 1.0) kind = TOPK_TOPP;
    else if (top_k > 0) kind = TOPK;
    else if (top_p > 0.0 && top_p < 1.0) kind = TOPP;
    else kind = ALL;
  }
  // apply_repetition_penalty — sampling.rs:86-103 (once per occurrence)
  void penalize(float* logits, size_t n) const {
    if (rep == 1.0f) return;
    for (uint32_t t : prev) {
      if (size_t(t) < n) {
        if (logits[t] > 0.0f) logits[t] /= rep;
        else logits[t] *= rep;
      }
    }
  }
  // compute_probabilities — sampling.rs:106-115
  std::vector<float> probs(const float* logits, size_t n) const {
    std::vector<float> s(n);
    const float tf = float(temperature);
    for (size_t i = 0; i < n; ++i) s[i] = logits[i] / tf;
    float mx = -INFINITY;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, s[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += std::exp(s[i] - mx);
    for (size_t i = 0; i < n; ++i) s[i] = std::exp(s[i] - mx) / sum;
    return s;
  }
  // sample_argmax — sampling.rs:118-125: Iterator::max_by keeps the LAST maximum;
  // partial_cmp().unwrap() panics on NaN (reported here as an error).
  static uint32_t argmax(const float* l, size_t n) {
    if (n == 0) return 0;
    size_t best = 0;
    if (std::isnan(l[0])) throw Error(GENERIC, "NaN logit");
    for (size_t i = 1; i < n; ++i) {
      if (std::isnan(l[i])) throw Error(GENERIC, "NaN logit");
      if (!(l[best] > l[i])) best = i;
    }
    return uint32_t(best);
  }
  // sample_multinomial — sampling.rs:128-132: rand 0.9 WeightedIndex::new (running f32
  // totals, the last one the total) and sample (Uniform(0, total), then the first
  // index whose running total exceeds the drawn value)
  uint32_t multinomial(const std::vector<float>& pr) {
    std::vector<float> cum(pr.size());
    float tot = 0.0f;
    for (size_t i = 0; i < pr.size(); ++i) {
      if (!(pr[i] >= 0.0f)) throw Error(GENERIC, "Failed to create weighted index: invalid weight");
      tot += pr[i];
      cum[i] = tot;
    }
    if (!(tot > 0.0f)) throw Error(GENERIC, "Failed to create weighted index: all weights zero");
    const float u = UniformF32(0.0f, tot).sample(rng);
    size_t i = size_t(std::upper_bound(cum.begin(), cum.end(), u) - cum.begin());
    return uint32_t(std::min(i, pr.size() - 1));
  }
  static void renorm(std::vector<float>& pr) {
    float sum = 0.0f;
    for (float v : pr) sum += v;
    if (sum > 0.0f)
      for (float& v : pr) v /= sum;
  }
  // sample_topp — sampling.rs:138-163
  uint32_t topp(std::vector<float>& pr, float top_p) {
    std::vector<size_t> idx(pr.size());
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return pr[a] > pr[b]; });
    float cum = 0.0f;
    for (size_t i : idx) {
      if (cum >= top_p) pr[i] = 0.0f;
      else cum += pr[i];
    }
    renorm(pr);
    return multinomial(pr);
  }
  // top-k selection — sampling.rs:168-192 (select_nth_unstable_by: ties at the cut unpinned)
  static void keep_topk(std::vector<float>& pr, size_t top_k) {
    std::vector<size_t> idx(pr.size());
    std::iota(idx.begin(), idx.end(), 0);
    std::nth_element(idx.begin(), idx.begin() + long(top_k), idx.end(), [&](size_t a, size_t b) { return pr[a] > pr[b]; });
    for (size_t i = top_k; i < idx.size(); ++i) pr[idx[i]] = 0.0f;
    renorm(pr);
  }
  // the distribution sample() draws from, without the draw: penalty on a copy,
  // compute_probabilities, top-k, top-p, renormalisation (sampling.rs:106-229)
  std::vector<float> distribution(const float* logits, size_t n) const {
    std::vector<float> l(logits, logits + n);
    penalize(l.data(), n);
    std::vector<float> pr = probs(l.data(), n);
    auto nucleus = [&](std::vector<float>& q, float top_p) {  // sample_topp's mask (sampling.rs:138-163)
      std::vector<size_t> idx(q.size());
      std::iota(idx.begin(), idx.end(), 0);
      std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return q[a] > q[b]; });
      float cum = 0.0f;
      for (size_t i : idx) {
        if (cum >= top_p) q[i] = 0.0f;
        else cum += q[i];
      }
      renorm(q);
    };
    const bool tp = !(p <= 0.0 || p >= 1.0);
    if (kind == TOPP) {
      if (tp) nucleus(pr, float(p));
    } else if (kind == TOPK) {
      if (k < n) keep_topk(pr, k);
    } else if (kind == TOPK_TOPP) {
      if (k >= n) nucleus(pr, float(p));
      else {
        keep_topk(pr, k);
        if (tp) nucleus(pr, float(p));
      }
    }
    return pr;
  }
  // sample — sampling.rs:232-264
  uint32_t sample(float* logits, size_t n) {
    penalize(logits, n);
    uint32_t tok;
    if (kind == ARGMAX) {
      tok = argmax(logits, n);
    } else {
      std::vector<float> pr = probs(logits, n);
      if (kind == ALL) {
        tok = multinomial(pr);
      } else if (kind == TOPP) {
        tok = (p <= 0.0 || p >= 1.0) ? multinomial(pr) : topp(pr, float(p));
      } else if (kind == TOPK) {
        if (k >= n) tok = multinomial(pr);
        else { keep_topk(pr, k); tok = multinomial(pr); }
      } else {  // sample_topk_topp — sampling.rs:195-229
        if (k >= n) tok = topp(pr, float(p));
        else {
          keep_topk(pr, k);
          tok = (p <= 0.0 || p >= 1.0) ? multinomial(pr) : topp(pr, float(p));
        }
      }
    }
    prev.push_back(tok);
    return tok;
  }
};

// ---------------------------------------------------------------------------
// Model — transformer/model.rs
// ---------------------------------------------------------------------------
struct Layer {
  std::vector<float> wq, wk, wv, wo, wg, wu, wd, attn_norm, ffn_norm;
};

struct Model {
  Config cfg;
  std::vector<float> emb, out_norm, lm_head;
  std::vector<Layer> layers;
  std::vector<KVCache> kv;

  // Model::new — model.rs:188-213 (zero weights, unit norms). Tensors are
  // allocated when loaded; finish() gives the ones the file lacks their
  // Model::new value (zeros, or ones for norms).
  explicit Model(const Config& c) : cfg(c) {
    layers.resize(c.layers);
    for (uint32_t i = 0; i < c.layers; ++i) kv.emplace_back(c.max_seq, c.kv_heads, c.head_dim());
  }
  void finish() {
    const size_t H = cfg.hidden, kvd = size_t(cfg.kv_heads) * cfg.head_dim();
    auto fill = [](std::vector<float>& v, size_t n, float x) { if (v.empty()) v.assign(n, x); };
    fill(emb, size_t(cfg.vocab) * H, 0.0f);
    fill(out_norm, H, 1.0f);
    fill(lm_head, size_t(cfg.vocab) * H, 0.0f);
    for (auto& L : layers) {
      fill(L.wq, H * H, 0.0f); fill(L.wk, H * kvd, 0.0f); fill(L.wv, H * kvd, 0.0f); fill(L.wo, H * H, 0.0f);
      fill(L.wg, H * cfg.ffn, 0.0f); fill(L.wu, H * cfg.ffn, 0.0f); fill(L.wd, H * cfg.ffn, 0.0f);
      fill(L.attn_norm, H, 1.0f); fill(L.ffn_norm, H, 1.0f);
    }
  }

  static void copy_into(std::vector<float>& dst, std::vector<float>&& src, size_t expected, const std::string& name) {
    if (expected != src.size())
      throw Error(GENERIC, "tensor " + name + " has " + std::to_string(src.size()) + " elements, expected " + std::to_string(expected));
    dst = std::move(src);
  }

  // load_from_gguf — model.rs:364-763 (default-feature path)
  void load(Gguf& g) {
    auto find = [&](const std::string& n) -> const TensorInfo* {
      auto it = g.by_name.find(n);
      return it == g.by_name.end() ? nullptr : &g.tensors[it->second];
    };
    // each name is tried in turn; a name that is absent or fails to load falls through
    const size_t H = cfg.hidden, kvd = size_t(cfg.kv_heads) * cfg.head_dim();
    auto first_loadable = [&](std::initializer_list<const char*> names, std::vector<float>& dst, size_t n) -> bool {
      for (const char* nm : names) {
        const TensorInfo* ti = find(nm);
        if (!ti) continue;
        std::vector<float> v;
        try { v = load_tensor(g, *ti); } catch (const Error&) { continue; }
        copy_into(dst, std::move(v), n, ti->name);
        return true;
      }
      return false;
    };
    if (!first_loadable({"token_embd.weight", "model.embed_tokens.weight", "embed_tokens.weight"}, emb,
                        size_t(cfg.vocab) * H))
      throw Error(PARSE, "Missing token embeddings");
    first_loadable({"output_norm.weight"}, out_norm, H);
    if (!first_loadable({"output.weight", "lm_head.weight", "model.lm_head.weight"}, lm_head, size_t(cfg.vocab) * H)) {
      lm_head.assign(size_t(cfg.vocab) * H, 0.0f);
      // weight tying through transpose_matrix(emb, rows=hidden, cols=vocab) — model.rs:47-55, :596-606
      const size_t rows = cfg.hidden, cols = cfg.vocab;
      for (size_t i = 0; i < rows; ++i)
        for (size_t j = 0; j < cols; ++j) lm_head[j * rows + i] = emb[i * cols + j];
    }
    for (uint32_t li = 0; li < cfg.layers; ++li) {
      Layer& L = layers[li];
      const std::string p = "blk." + std::to_string(li) + ".";
      auto ld = [&](const char* base, std::vector<float>& dst, size_t n, bool try_bare) {
        const TensorInfo* ti = find(p + base + ".weight");
        if (!ti && try_bare) ti = find(p + base);
        if (ti) {
          std::vector<float> v;
          try { v = load_tensor(g, *ti); } catch (const Error&) { return; }  // `if let Ok(..)`: failures leave zeros
          copy_into(dst, std::move(v), n, ti->name);
        }
      };
      ld("attn_q", L.wq, H * H, true); ld("attn_k", L.wk, H * kvd, true); ld("attn_v", L.wv, H * kvd, true);
      ld("attn_output", L.wo, H * H, true);
      ld("attn_norm", L.attn_norm, H, false);
      ld("ffn_gate", L.wg, H * cfg.ffn, false); ld("ffn_up", L.wu, H * cfg.ffn, false);
      ld("ffn_down", L.wd, H * cfg.ffn, false);
      ld("ffn_norm", L.ffn_norm, H, false);
    }
    finish();
  }

  // MultiHeadAttention::forward — attention.rs:67-194
  std::vector<float> attention(const Layer& L, KVCache& c, const std::vector<float>& x, size_t seq, size_t position) {
    const size_t H = cfg.hidden, hd = cfg.head_dim(), kvd = size_t(cfg.kv_heads) * hd;
    std::vector<float> q(seq * H), k(seq * kvd), v(seq * kvd);
    matmul_transposed(x.data(), L.wq.data(), q.data(), seq, H, H, g_proj_threads);
    matmul_transposed(x.data(), L.wk.data(), k.data(), seq, H, kvd, g_proj_threads);
    matmul_transposed(x.data(), L.wv.data(), v.data(), seq, H, kvd, g_proj_threads);
    apply_rope(q.data(), position, seq, cfg.heads, hd, cfg.theta);
    apply_rope(k.data(), position, seq, cfg.kv_heads, hd, cfg.theta);
    const size_t kv_len = c.append(k.data(), v.data(), seq);
    std::vector<float> att(seq * H);
    compute_attention(q.data(), c.keys.data(), c.values.data(), seq, kv_len, position, cfg.heads, cfg.kv_heads, hd, att.data());
    std::vector<float> out(seq * H);
    matmul_transposed(att.data(), L.wo.data(), out.data(), seq, H, H, g_proj_threads);
    return out;
  }

  // FeedForward::forward — ffn.rs:54-109
  std::vector<float> ffn(const Layer& L, const std::vector<float>& x, size_t seq) {
    const size_t H = cfg.hidden, F = cfg.ffn;
    std::vector<float> gate(seq * F), up(seq * F), out(seq * H);
    matmul_transposed(x.data(), L.wg.data(), gate.data(), seq, H, F, g_proj_threads);
    matmul_transposed(x.data(), L.wu.data(), up.data(), seq, H, F, g_proj_threads);
    for (size_t i = 0; i < gate.size(); ++i) {
      const float sig = 1.0f / (1.0f + std::exp(-gate[i]));
      const float silu = gate[i] * sig;
      gate[i] = silu * up[i];
    }
    matmul_transposed(gate.data(), L.wd.data(), out.data(), seq, F, H, g_proj_threads);
    return out;
  }

  // TransformerLayer::forward — layer.rs:37-89 (per-layer RMSNorm eps is 1e-6)
  std::vector<float> layer(uint32_t li, const std::vector<float>& x, size_t seq, size_t position) {
    const Layer& L = layers[li];
    const size_t H = cfg.hidden;
    std::vector<float> normed(seq * H);
    rms_norm(x.data(), L.attn_norm.data(), 1e-6f, seq, H, normed.data());
    std::vector<float> a = attention(L, kv[li], normed, seq, position);
    std::vector<float> h(seq * H);
    for (size_t i = 0; i < h.size(); ++i) h[i] = x[i] + a[i];
    rms_norm(h.data(), L.ffn_norm.data(), 1e-6f, seq, H, normed.data());
    std::vector<float> f = ffn(L, normed, seq);
    for (size_t i = 0; i < h.size(); ++i) h[i] = h[i] + f[i];
    return h;
  }

  // Model::forward — model.rs:832-1192: returns logits of the last token only
  std::vector<float> forward(const uint32_t* ids, size_t seq, size_t position) {
    const size_t H = cfg.hidden;
    if (seq == 0) throw Error(INVALID_ARG, "empty token sequence");
    std::vector<float> x(seq * H, 0.0f);
    for (size_t s = 0; s < seq; ++s)
      for (size_t d = 0; d < H; ++d) {
        const size_t e = size_t(ids[s]) * H + d;
        if (e < emb.size()) x[s * H + d] = emb[e];
        else break;
      }
    for (uint32_t li = 0; li < cfg.layers; ++li) x = layer(li, x, seq, position);
    std::vector<float> normed(seq * H);
    rms_norm(x.data(), out_norm.data(), cfg.eps, seq, H, normed.data());
    std::vector<float> logits(cfg.vocab);
    matmul_transposed(normed.data() + (seq - 1) * H, lm_head.data(), logits.data(), 1, H, cfg.vocab, g_threads);
    return logits;
  }

  void clear_kv() { for (auto& c : kv) c.clear(); }  // model.rs:1547

  // Model::generate — model.rs:1322-1415, on token ids (no tokenizer): prefill in
  // 8-token chunks at position = chunk_start, first token sampled without an EOS
  // check, then decode until max_tokens tokens or EOS (checked before the push).
  std::vector<uint32_t> generate(const uint32_t* prompt, size_t n, size_t max_tokens, double temperature, double top_p,
                                 size_t top_k, float rep, uint64_t seed, uint32_t eos,
                                 std::vector<float>* first_logits, std::vector<float>* step_logits) {
    LogitsProcessor lp(seed, temperature, top_p, top_k, rep);
    clear_kv();
    if (n == 0) throw Error(PARSE, "Empty token sequence");
    std::vector<uint32_t> tokens(prompt, prompt + n);
    std::vector<float> logits;
    for (size_t cs = 0; cs < n; cs += 8) {
      const size_t ce = std::min(cs + 8, n);
      logits = forward(tokens.data() + cs, ce - cs, cs);
    }
    if (first_logits) *first_logits = logits;
    if (step_logits) step_logits->insert(step_logits->end(), logits.begin(), logits.end());
    std::vector<uint32_t> gen;
    uint32_t next = lp.sample(logits.data(), logits.size());
    tokens.push_back(next);
    gen.push_back(next);
    size_t generated = 1;
    while (generated < max_tokens) {
      const uint32_t last = tokens.back();
      const size_t pos = kv.empty() ? tokens.size() - 1 : kv[0].cur;
      logits = forward(&last, 1, pos);
      if (step_logits) step_logits->insert(step_logits->end(), logits.begin(), logits.end());
      next = lp.sample(logits.data(), logits.size());
      if (next == eos) break;
      tokens.push_back(next);
      gen.push_back(next);
      ++generated;
    }
    return gen;
  }
};

struct Handle {
  Gguf g;
  std::unique_ptr<Model> m;
};

}  // namespace oracle

using namespace oracle;

#define ORACLE_TRY(body)                  \
  try {                                   \
    body;                                 \
    return OK;                            \
  } catch (const Error& e) {              \
    g_last_error = e.what();              \
    return e.code;                        \
  } catch (const std::bad_alloc&) {       \
    g_last_error = "out of memory";       \
    return OOM;                           \
  } catch (const std::exception& e) {     \
    g_last_error = e.what();              \
    return GENERIC;                       \
  }

extern "C" {

size_t oracle_last_error(char* buf, size_t len) {
  if (!buf || !len) return 0;
  size_t n = std::min(len - 1, g_last_error.size());
  std::memcpy(buf, g_last_error.data(), n);
  buf[n] = 0;
  return n;
}

// lm_threads: threads for the LM head; proj_threads: threads for all projections
void oracle_set_threads(int lm_threads, int proj_threads) {
  g_threads = std::max(1, lm_threads);
  g_proj_threads = std::max(1, proj_threads);
  g_load_threads = std::max(g_threads, g_proj_threads);
}

// faithful = 1: matmul_transposed walks one output row at a time, the
// reference's exact loop (used when timing the CPU baseline)
void oracle_set_faithful(int faithful) { g_faithful = faithful ? 1 : 0; }

uint32_t oracle_open(const char* path, void** out) {
  ORACLE_TRY({
    auto h = std::make_unique<Handle>();
    h->g.open(path);
    Config c = extract_config(h->g);
    h->m = std::make_unique<Model>(c);
    h->m->load(h->g);
    *out = h.release();
  });
}

void oracle_free(void* h) { delete static_cast<Handle*>(h); }

// vocab, hidden, layers, heads, kv_heads, ffn, max_seq, head_dim
void oracle_config(void* h, uint32_t* out8, float* eps_theta) {
  const Config& c = static_cast<Handle*>(h)->m->cfg;
  uint32_t v[8] = {c.vocab, c.hidden, c.layers, c.heads, c.kv_heads, c.ffn, c.max_seq, c.head_dim()};
  std::memcpy(out8, v, sizeof(v));
  eps_theta[0] = c.eps;
  eps_theta[1] = c.theta;
}

uint32_t oracle_forward(void* h, const uint32_t* ids, size_t n, size_t position, float* logits) {
  ORACLE_TRY({
    Model& m = *static_cast<Handle*>(h)->m;
    std::vector<float> l = m.forward(ids, n, position);
    std::memcpy(logits, l.data(), l.size() * sizeof(float));
  });
}

void oracle_clear_kv(void* h) { static_cast<Handle*>(h)->m->clear_kv(); }

size_t oracle_kv_len(void* h) {
  Model& m = *static_cast<Handle*>(h)->m;
  return m.kv.empty() ? 0 : m.kv[0].cur;
}

// step_logits (optional): receives vocab floats for the prefill and each decode step
uint32_t oracle_generate(void* h, const uint32_t* prompt, size_t n, size_t max_tokens, float temperature, float top_p,
                         size_t top_k, float rep, uint64_t seed, uint32_t eos, uint32_t* out, size_t cap, size_t* n_out,
                         float* step_logits, size_t step_cap) {
  ORACLE_TRY({
    Model& m = *static_cast<Handle*>(h)->m;
    std::vector<float> steps;
    std::vector<uint32_t> g = m.generate(prompt, n, max_tokens, temperature, top_p, top_k, rep, seed, eos, nullptr,
                                         step_logits ? &steps : nullptr);
    *n_out = g.size();
    std::memcpy(out, g.data(), std::min(cap, g.size()) * sizeof(uint32_t));
    if (step_logits) std::memcpy(step_logits, steps.data(), std::min(step_cap, steps.size()) * sizeof(float));
  });
}

// dequantised copy of one named tensor (TensorLoader::load_tensor)
uint32_t oracle_tensor_f32(void* h, const char* name, float* out, size_t cap, size_t* numel) {
  ORACLE_TRY({
    Handle& hd = *static_cast<Handle*>(h);
    auto it = hd.g.by_name.find(name);
    if (it == hd.g.by_name.end()) throw Error(GENERIC, std::string("Tensor not found: ") + name);
    std::vector<float> v = load_tensor(hd.g, hd.g.tensors[it->second]);
    *numel = v.size();
    std::memcpy(out, v.data(), std::min(cap, v.size()) * sizeof(float));
  });
}

void oracle_dequant_q4k(const uint8_t* blocks, size_t nblocks, float* out) {
  for (size_t b = 0; b < nblocks; ++b) dequantize_q4_k(blocks + 144 * b, out + 256 * b);
}

void oracle_dequant_q6k(const uint8_t* blocks, size_t nblocks, float* out) {
  for (size_t b = 0; b < nblocks; ++b) dequantize_q6_k(blocks + 210 * b, out + 256 * b);
}

void oracle_matmul_transposed(const float* a, const float* b, float* c, size_t m, size_t k, size_t n) {
  matmul_transposed(a, b, c, m, k, n, g_proj_threads);
}

void oracle_rms_norm(const float* x, const float* w, float eps, size_t seq, size_t hidden, float* out) {
  rms_norm(x, w, eps, seq, hidden, out);
}

void oracle_rope(float* t, size_t start_pos, size_t seq, size_t heads, size_t hd, float theta) {
  apply_rope(t, start_pos, seq, heads, hd, theta);
}

void oracle_attention(const float* q, const float* k, const float* v, size_t seq, size_t kv_seq, size_t position,
                      size_t heads, size_t kv_heads, size_t hd, float* out) {
  compute_attention(q, k, v, seq, kv_seq, position, heads, kv_heads, hd, out);
}

// KV cache append semantics (kv_cache.rs:44-67) on a caller-visible cache
void* oracle_kv_new(size_t max_seq, size_t n_kv, size_t hd) { return new KVCache(max_seq, n_kv, hd); }
void oracle_kv_free(void* c) { delete static_cast<KVCache*>(c); }
uint32_t oracle_kv_append(void* c, const float* k, const float* v, size_t seq, size_t* len) {
  ORACLE_TRY({ *len = static_cast<KVCache*>(c)->append(k, v, seq); });
}
const float* oracle_kv_keys(void* c) { return static_cast<KVCache*>(c)->keys.data(); }
const float* oracle_kv_values(void* c) { return static_cast<KVCache*>(c)->values.data(); }

// LogitsProcessor (sampling.rs:29-264)
void* oracle_sampler_new(uint64_t seed, double temperature, double top_p, size_t top_k, float rep) {
  return new LogitsProcessor(seed, temperature, top_p, top_k, rep);
}
void oracle_sampler_free(void* s) { delete static_cast<LogitsProcessor*>(s); }
// the keystream block `counter` of ChaCha with `rounds` rounds under a 32-byte key
// (zero stream id): the known-answer check of the random stream's block function
void oracle_chacha_block(const uint8_t* key, uint64_t counter, int rounds, uint32_t* out16) {
  Rng r(key, rounds);
  r.st[12] = uint32_t(counter);
  r.st[13] = uint32_t(counter >> 32);
  for (int i = 0; i < 16; ++i) out16[i] = r.next_u32();
}
// the first n u32 outputs of StdRng::seed_from_u64(seed)
void oracle_std_rng_u32(uint64_t seed, size_t n, uint32_t* out) {
  Rng r(seed);
  for (size_t i = 0; i < n; ++i) out[i] = r.next_u32();
}
uint32_t oracle_sampler_sample(void* s, float* logits, size_t n, uint32_t* tok) {
  ORACLE_TRY({ *tok = static_cast<LogitsProcessor*>(s)->sample(logits, n); });
}
void oracle_sampler_penalize(void* s, float* logits, size_t n) { static_cast<LogitsProcessor*>(s)->penalize(logits, n); }
int oracle_sampler_kind(void* s) { return static_cast<LogitsProcessor*>(s)->kind; }
void oracle_sampler_distribution(void* s, const float* logits, size_t n, float* out) {
  const std::vector<float> d = static_cast<LogitsProcessor*>(s)->distribution(logits, n);
  std::copy(d.begin(), d.end(), out);
}

}  // extern "C"
