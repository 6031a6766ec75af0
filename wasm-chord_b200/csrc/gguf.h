// GGUF v2/v3 reader: header, metadata key/values, tensor directory, data offset.
// Follows crates/wasm-chord-core/src/formats/gguf.rs: magic and version check
// (:111-124), metadata value types (:347-405), tensor infos (:414-444), dtype
// ids (:446-467), 32-byte alignment of the data section (:162-172) and the
// config keys, fallbacks and defaults of extract_config (:208-276).
#pragma once
#include <cstdint>
#include <cstdio>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace wcb {

// ErrorCode values (wasm-chord-runtime/src/lib.rs:80-89)
enum : uint32_t { E_OK = 0, E_GENERIC = 1, E_OOM = 2, E_INVALID = 3, E_PARSE = 4, E_BACKEND = 5, E_IO = 7 };

struct WcbError : std::runtime_error {
  uint32_t code;
  WcbError(uint32_t c, const std::string& m) : std::runtime_error(m), code(c) {}
};

struct GgufValue {
  uint32_t type = 0xFFFFFFFFu;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  std::vector<std::string> strs;  // an array of strings (tokenizer.ggml.tokens / merges); other arrays are skipped
  bool as_u32(uint32_t* out) const;
  bool as_f32(float* out) const;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;  // ne, innermost first
  uint32_t dtype = 0;          // GGUF type id (unknown ids map to 255)
  uint64_t offset = 0;         // relative to the data section
  uint64_t numel = 0;
  uint64_t nbytes = 0;         // TensorDesc::new size (tensor.rs:133-189)
};

struct ModelConfig {
  uint32_t vocab = 32000, hidden = 2048, layers = 22, heads = 32, kv_heads = 4, ffn = 5632, max_seq = 2048;
  float eps = 1e-5f, theta = 10000.0f;
  uint32_t head_dim() const { return heads ? hidden / heads : 0; }
};

class GgufFile {
 public:
  explicit GgufFile(const std::string& path);
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;

  const GgufTensor* find(const std::string& name) const;
  const GgufValue* value(const std::string& key) const { return get(key); }
  ModelConfig config() const;
  // reads the raw bytes of a tensor into dst (nbytes bytes)
  void read(const GgufTensor& t, void* dst) const;
  // reads bytes [offset, offset + bytes) of a tensor's data into dst
  void read_range(const GgufTensor& t, uint64_t offset, uint64_t bytes, void* dst) const;
  uint32_t version() const { return version_; }
  uint64_t data_offset() const { return data_offset_; }
  const std::vector<GgufTensor>& tensors() const { return tensors_; }

 private:
  template <class T> T rd();
  std::string rd_str();
  GgufValue rd_value(uint32_t type, bool allow_array);
  const GgufValue* get(const std::string& k) const;
  uint32_t cfg_u32(const std::string& a, const std::string& b, uint32_t dflt) const;
  float cfg_f32(const std::string& a, const std::string& b, float dflt) const;

  FILE* f_ = nullptr;
  uint32_t version_ = 0;
  uint64_t data_offset_ = 0;
  std::string arch_;
  std::map<std::string, GgufValue> meta_;
  std::vector<GgufTensor> tensors_;
  std::map<std::string, size_t> index_;
};

}  // namespace wcb
