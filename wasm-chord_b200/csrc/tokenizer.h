// Text <-> token ids for generate(&str): the reference's BPE tokenizer with its
// SentencePiece space marker, greedy-longest-match fallback and byte fallback
// (crates/wasm-chord-core/src/tokenizer.rs).
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "gguf.h"

namespace wcb {

struct SpecialIds {
  uint32_t bos = 1, eos = 2, unk = 0;  // SpecialTokens::default (tokenizer.rs:28-40)
};

class Tokenizer {
 public:
  // Tokenizer::new (tokenizer.rs:63-80): add_bos true, add_eos false
  Tokenizer(std::vector<std::string> id_to_token, std::vector<std::pair<std::string, std::string>> merges,
            SpecialIds special);
  // Tokenizer::from_gguf (tokenizer.rs:82-147): tokenizer.ggml.tokens / .merges / *_token_id
  static Tokenizer from_gguf(const GgufFile& f);

  std::vector<uint32_t> encode(const std::string& text, bool add_special) const;   // tokenizer.rs:207-231
  std::string decode(const uint32_t* ids, size_t n, bool skip_special) const;      // tokenizer.rs:353-395
  size_t vocab_size() const { return vocab_.size(); }                              // distinct token strings
  const SpecialIds& special() const { return special_; }
  void set_add_bos(bool v) { add_bos_ = v; }
  void set_add_eos(bool v) { add_eos_ = v; }

 private:
  std::vector<uint32_t> encode_bpe(const std::string& text) const;       // tokenizer.rs:233-311
  std::vector<uint32_t> fallback_encode(const std::string& text) const;  // tokenizer.rs:313-351
  void byte_fallback(const std::string& piece, std::vector<uint32_t>& out) const;

  std::unordered_map<std::string, uint32_t> vocab_;       // token -> id (a later duplicate wins, like HashMap::insert)
  std::unordered_map<uint32_t, std::string> reverse_;     // id -> token, built from vocab_ (tokenizer.rs:68-69)
  std::unordered_map<std::string, size_t> merge_rank_;    // "a\x01b" -> rank (a later duplicate wins)
  size_t n_merges_ = 0;
  SpecialIds special_;
  bool add_bos_ = true, add_eos_ = false;
};

}  // namespace wcb
