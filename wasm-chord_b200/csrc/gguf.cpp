#include "gguf.h"

#include <cstring>

namespace wcb {

bool GgufValue::as_u32(uint32_t* out) const {  // MetadataValue::as_u32 (gguf.rs:50-62)
  switch (type) {
    case 0: case 2: case 4: case 10: *out = uint32_t(u); return true;
    case 1: case 3: case 5: case 11: *out = uint32_t(i); return true;
    default: return false;
  }
}

bool GgufValue::as_f32(float* out) const {  // MetadataValue::as_f32 (gguf.rs:64-70)
  if (type == 6 || type == 12) {
    *out = float(f);
    return true;
  }
  return false;
}

static uint64_t desc_bytes(uint32_t t, uint64_t n) {  // tensor.rs:133-189
  switch (t) {
    case 0: return n * 4;
    case 1: return n * 2;
    case 2: case 3: return n / 32 * 16;
    case 8: case 9: return n / 32 * 33;
    case 12: return n / 256 * 144;
    case 13: return n / 256 * 176;
    case 14: return n / 256 * 210;
    default: return n / 2;
  }
}

template <class T>
T GgufFile::rd() {
  T v;
  if (std::fread(&v, sizeof(T), 1, f_) != 1) throw WcbError(E_IO, "failed to fill whole buffer");
  return v;
}

std::string GgufFile::rd_str() {
  const uint64_t n = rd<uint64_t>();
  if (n > (uint64_t(1) << 32)) throw WcbError(E_PARSE, "Parse error: string length out of range");
  std::string s(n, '\0');
  if (n && std::fread(&s[0], 1, n, f_) != n) throw WcbError(E_IO, "failed to fill whole buffer");
  return s;
}

GgufValue GgufFile::rd_value(uint32_t t, bool allow_array) {
  GgufValue v;
  v.type = t;
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
      if (!allow_array) throw WcbError(E_PARSE, "Parse error: Unknown typed value: 9");
      const uint32_t et = rd<uint32_t>();
      const uint64_t n = rd<uint64_t>();
      if (et == 8) {  // strings are kept (the tokenizer's vocabulary and merges)
        if (n > (uint64_t(1) << 26)) throw WcbError(E_PARSE, "Parse error: array length out of range");
        v.strs.reserve(size_t(n));
        for (uint64_t k = 0; k < n; ++k) v.strs.push_back(rd_str());
      } else {
        for (uint64_t k = 0; k < n; ++k) rd_value(et, false);  // numeric arrays: no key needs one
      }
      break;
    }
    case 10: v.u = rd<uint64_t>(); break;
    case 11: v.i = rd<int64_t>(); break;
    case 12: v.f = rd<double>(); break;
    default: throw WcbError(E_PARSE, "Parse error: Unknown metadata value type: " + std::to_string(t));
  }
  return v;
}

GgufFile::GgufFile(const std::string& path) {
  f_ = std::fopen(path.c_str(), "rb");
  if (!f_) throw WcbError(E_IO, "IO error: cannot open " + path);
  try {
    if (rd<uint32_t>() != 0x46554747u) throw WcbError(E_PARSE, "Invalid model format: Invalid GGUF magic");
    version_ = rd<uint32_t>();
    if (version_ < 2 || version_ > 3)
      throw WcbError(E_PARSE, "Invalid model format: Unsupported GGUF version: " + std::to_string(version_));
    const uint64_t n_tensors = rd<uint64_t>();
    const uint64_t n_kv = rd<uint64_t>();
    for (uint64_t k = 0; k < n_kv; ++k) {
      std::string key = rd_str();
      const uint32_t t = rd<uint32_t>();
      meta_[key] = rd_value(t, true);
    }
    for (uint64_t k = 0; k < n_tensors; ++k) {
      GgufTensor t;
      t.name = rd_str();
      const uint32_t nd = rd<uint32_t>();
      if (nd > 8) throw WcbError(E_PARSE, "Parse error: tensor " + t.name + " has too many dimensions");
      t.numel = 1;
      for (uint32_t d = 0; d < nd; ++d) {
        t.dims.push_back(rd<uint64_t>());
        t.numel *= t.dims.back();
      }
      const uint32_t dt = rd<uint32_t>();
      const bool known = dt <= 3 || (dt >= 6 && dt <= 14);
      t.dtype = known ? dt : 255u;
      t.offset = rd<uint64_t>();
      t.nbytes = desc_bytes(t.dtype, t.numel);
      index_[t.name] = tensors_.size();
      tensors_.push_back(t);
    }
    const uint64_t pos = uint64_t(std::ftell(f_));
    data_offset_ = (pos + 31) & ~uint64_t(31);
    // a truncated file is reported here, before any device work, rather than by
    // the read of its first missing tensor (tensor_loader.rs:50-149 fails there
    // with "failed to fill whole buffer")
    if (std::fseek(f_, 0, SEEK_END) != 0) throw WcbError(E_IO, "IO error: seek failed");
    const uint64_t size = uint64_t(std::ftell(f_));
    for (const GgufTensor& t : tensors_)
      if (t.dtype != 255u && data_offset_ + t.offset + t.nbytes > size)
        throw WcbError(E_IO, "IO error: failed to fill whole buffer: tensor " + t.name + " ends at byte " +
                                 std::to_string(data_offset_ + t.offset + t.nbytes) + " of a " +
                                 std::to_string(size) + "-byte file (truncated)");
    auto it = meta_.find("general.architecture");
    arch_ = (it != meta_.end() && it->second.type == 8) ? it->second.s : "unknown";
  } catch (...) {
    std::fclose(f_);
    f_ = nullptr;
    throw;
  }
}

GgufFile::~GgufFile() {
  if (f_) std::fclose(f_);
}

const GgufTensor* GgufFile::find(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

const GgufValue* GgufFile::get(const std::string& k) const {
  auto it = meta_.find(k);
  return it == meta_.end() ? nullptr : &it->second;
}

uint32_t GgufFile::cfg_u32(const std::string& a, const std::string& b, uint32_t dflt) const {
  const GgufValue* v = get(a);
  if (!v) v = get(b);
  uint32_t out;
  return (v && v->as_u32(&out)) ? out : dflt;
}

float GgufFile::cfg_f32(const std::string& a, const std::string& b, float dflt) const {
  const GgufValue* v = get(a);
  if (!v) v = get(b);
  float out;
  return (v && v->as_f32(&out)) ? out : dflt;
}

ModelConfig GgufFile::config() const {  // extract_config (gguf.rs:208-276)
  const std::string& a = arch_;
  ModelConfig c;
  c.vocab = cfg_u32(a + ".vocab_size", "vocab_size", 32000);
  c.hidden = cfg_u32(a + ".embedding_length", a + ".hidden_size", 2048);
  c.layers = cfg_u32(a + ".block_count", a + ".num_layers", 22);
  c.heads = cfg_u32(a + ".attention.head_count", a + ".num_heads", 32);
  c.kv_heads = cfg_u32(a + ".attention.head_count_kv", a + ".num_kv_heads", 4);
  c.ffn = cfg_u32(a + ".feed_forward_length", a + ".intermediate_size", 5632);
  c.max_seq = cfg_u32(a + ".context_length", a + ".max_seq_len", 2048);
  c.eps = cfg_f32(a + ".attention.layer_norm_rms_epsilon", "rms_norm_eps", 1e-5f);
  c.theta = cfg_f32(a + ".rope.freq_base", "rope_theta", 10000.0f);
  return c;
}

void GgufFile::read_range(const GgufTensor& t, uint64_t offset, uint64_t bytes, void* dst) const {
  if (offset + bytes > t.nbytes) throw WcbError(E_IO, "IO error: range outside tensor " + t.name);
  if (std::fseek(f_, long(data_offset_ + t.offset + offset), SEEK_SET) != 0)
    throw WcbError(E_IO, "IO error: seek failed for " + t.name);
  if (bytes && std::fread(dst, 1, bytes, f_) != bytes)
    throw WcbError(E_IO, "IO error: failed to fill whole buffer (" + t.name + ")");
}

void GgufFile::read(const GgufTensor& t, void* dst) const {
  if (std::fseek(f_, long(data_offset_ + t.offset), SEEK_SET) != 0)
    throw WcbError(E_IO, "IO error: seek failed for " + t.name);
  if (t.nbytes && std::fread(dst, 1, t.nbytes, f_) != t.nbytes)
    throw WcbError(E_IO, "IO error: failed to fill whole buffer (" + t.name + ")");
}

}  // namespace wcb
