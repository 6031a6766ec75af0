#include "tokenizer.h"

#include <algorithm>
#include <cstdio>
#include <functional>
#include <queue>

namespace wcb {
namespace {

const std::string kSpaceMarker = "\xE2\x96\x81";  // U+2581, SentencePiece's word boundary

// the byte length of the UTF-8 sequence starting with lead byte c (1 for an
// invalid lead: the reference splits a Rust &str, which is always valid UTF-8)
size_t utf8_len(unsigned char c) {
  if (c < 0x80) return 1;
  if ((c & 0xE0) == 0xC0) return 2;
  if ((c & 0xF0) == 0xE0) return 3;
  if ((c & 0xF8) == 0xF0) return 4;
  return 1;
}

std::vector<std::string> split_chars(const std::string& s) {  // text.chars()
  std::vector<std::string> out;
  for (size_t i = 0; i < s.size();) {
    const size_t n = std::min(utf8_len(static_cast<unsigned char>(s[i])), s.size() - i);
    out.emplace_back(s, i, n);
    i += n;
  }
  return out;
}

std::string replace_all(const std::string& s, const std::string& from, const std::string& to) {
  std::string out;
  out.reserve(s.size());
  for (size_t i = 0; i < s.size();) {
    if (s.compare(i, from.size(), from) == 0) {
      out += to;
      i += from.size();
    } else {
      out += s[i++];
    }
  }
  return out;
}

// String::from_utf8_lossy: each maximal ill-formed subpart becomes U+FFFD
std::string utf8_lossy(const std::string& b) {
  static const std::string kRepl = "\xEF\xBF\xBD";
  std::string out;
  out.reserve(b.size());
  const size_t n = b.size();
  size_t i = 0;
  while (i < n) {
    const unsigned char c = static_cast<unsigned char>(b[i]);
    if (c < 0x80) {
      out += char(c);
      ++i;
      continue;
    }
    size_t need;
    unsigned char lo = 0x80, hi = 0xBF;  // allowed range of the second byte
    if (c >= 0xC2 && c <= 0xDF) need = 1;
    else if (c == 0xE0) need = 2, lo = 0xA0;
    else if ((c >= 0xE1 && c <= 0xEC) || c == 0xEE || c == 0xEF) need = 2;
    else if (c == 0xED) need = 2, hi = 0x9F;
    else if (c == 0xF0) need = 3, lo = 0x90;
    else if (c >= 0xF1 && c <= 0xF3) need = 3;
    else if (c == 0xF4) need = 3, hi = 0x8F;
    else {
      out += kRepl;
      ++i;
      continue;
    }
    size_t k = 1;
    bool bad = false;
    for (; k <= need; ++k) {
      if (i + k >= n) break;  // truncated at the end
      const unsigned char d = static_cast<unsigned char>(b[i + k]);
      const unsigned char l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
      if (d < l || d > h) {
        bad = true;
        break;
      }
    }
    if (!bad && k > need) {
      out.append(b, i, need + 1);
      i += need + 1;
    } else {
      out += kRepl;  // the bytes [i, i + k) are one maximal subpart
      i += k;
    }
  }
  return out;
}

bool is_ws(uint32_t cp) {  // char::is_whitespace (Unicode White_Space)
  return (cp >= 0x09 && cp <= 0x0D) || cp == 0x20 || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
         (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
         cp == 0x3000;
}

uint32_t decode_cp(const std::string& s, size_t i, size_t* len) {  // s is valid UTF-8
  const unsigned char c = static_cast<unsigned char>(s[i]);
  const size_t n = utf8_len(c);
  *len = n;
  if (n == 1) return c;
  uint32_t cp = c & (n == 2 ? 0x1F : n == 3 ? 0x0F : 0x07);
  for (size_t k = 1; k < n; ++k) cp = (cp << 6) | (static_cast<unsigned char>(s[i + k]) & 0x3F);
  return cp;
}

std::string trim(const std::string& s) {  // str::trim
  size_t b = 0;
  while (b < s.size()) {
    size_t len;
    if (!is_ws(decode_cp(s, b, &len))) break;
    b += len;
  }
  size_t e = s.size();
  while (e > b) {
    size_t p = e - 1;  // start of the last code point
    while (p > b && (static_cast<unsigned char>(s[p]) & 0xC0) == 0x80) --p;
    size_t len;
    if (!is_ws(decode_cp(s, p, &len))) break;
    e = p;
  }
  return s.substr(b, e - b);
}

// u8::from_str_radix(hex, 16): an optional '+', then at least one hex digit, value < 256
bool parse_hex_u8(const std::string& h, uint8_t* out) {
  size_t i = 0;
  if (i < h.size() && h[i] == '+') ++i;
  if (i == h.size()) return false;
  uint32_t v = 0;
  for (; i < h.size(); ++i) {
    const char c = h[i];
    uint32_t d;
    if (c >= '0' && c <= '9') d = uint32_t(c - '0');
    else if (c >= 'a' && c <= 'f') d = uint32_t(c - 'a' + 10);
    else if (c >= 'A' && c <= 'F') d = uint32_t(c - 'A' + 10);
    else return false;
    v = v * 16 + d;
    if (v > 255) return false;
  }
  *out = uint8_t(v);
  return true;
}

std::string byte_token(unsigned char b) {  // format!("<0x{:02X}>", byte)
  char buf[8];
  std::snprintf(buf, sizeof(buf), "<0x%02X>", unsigned(b));
  return buf;
}

}  // namespace

Tokenizer::Tokenizer(std::vector<std::string> id_to_token, std::vector<std::pair<std::string, std::string>> merges,
                     SpecialIds special)
    : special_(special) {
  for (size_t id = 0; id < id_to_token.size(); ++id) vocab_[id_to_token[id]] = uint32_t(id);
  for (const auto& kv : vocab_) reverse_[kv.second] = kv.first;
  // merge ranks as encode_bpe builds them (tokenizer.rs:250-254): a repeated pair keeps its last rank
  n_merges_ = merges.size();
  for (size_t r = 0; r < merges.size(); ++r) merge_rank_[merges[r].first + '\x01' + merges[r].second] = r;
}

Tokenizer Tokenizer::from_gguf(const GgufFile& f) {
  const GgufValue* toks = f.value("tokenizer.ggml.tokens");
  if (!toks || toks->type != 9 || toks->strs.empty())
    throw WcbError(E_PARSE, "Parse error: No tokenizer.ggml.tokens in metadata");
  std::vector<std::pair<std::string, std::string>> merges;
  if (const GgufValue* m = f.value("tokenizer.ggml.merges")) {
    for (const std::string& s : m->strs) {  // "a b": exactly two parts split on ' ' (tokenizer.rs:102-117)
      const size_t sp = s.find(' ');
      if (sp == std::string::npos || s.find(' ', sp + 1) != std::string::npos) continue;
      merges.emplace_back(s.substr(0, sp), s.substr(sp + 1));
    }
  }
  SpecialIds sp;
  auto id_of = [&](const char* key, uint32_t dflt) {
    const GgufValue* v = f.value(key);
    uint32_t out;
    return (v && v->as_u32(&out)) ? out : dflt;
  };
  sp.bos = id_of("tokenizer.ggml.bos_token_id", 1);
  sp.eos = id_of("tokenizer.ggml.eos_token_id", 2);
  sp.unk = id_of("tokenizer.ggml.unknown_token_id", 0);
  return Tokenizer(toks->strs, std::move(merges), sp);
}

std::vector<uint32_t> Tokenizer::encode(const std::string& text, bool add_special) const {
  std::vector<uint32_t> out;
  if (text.empty()) return out;
  if (add_special && add_bos_) out.push_back(special_.bos);
  const std::vector<uint32_t> body = encode_bpe(kSpaceMarker + replace_all(text, " ", kSpaceMarker));
  out.insert(out.end(), body.begin(), body.end());
  if (add_special && add_eos_) out.push_back(special_.eos);
  return out;
}

void Tokenizer::byte_fallback(const std::string& piece, std::vector<uint32_t>& out) const {
  for (unsigned char b : piece) {
    auto it = vocab_.find(byte_token(b));
    out.push_back(it != vocab_.end() ? it->second : special_.unk);
  }
}

std::vector<uint32_t> Tokenizer::encode_bpe(const std::string& text) const {
  std::vector<uint32_t> out;
  if (text.empty()) return out;
  std::vector<std::string> tok = split_chars(text);
  if (n_merges_ == 0) return fallback_encode(text);
  // The reference rescans every adjacent pair after each merge and merges the
  // lowest-ranked one, the leftmost on ties (only equal pairs share a rank). The
  // same order comes from a heap of (rank, left position) over a linked list of
  // pieces: a piece keeps its first character's position, so positions stay in
  // left-to-right order, and an entry whose pieces changed since it was pushed is
  // stale and skipped.
  const size_t n = tok.size();
  std::vector<size_t> prev(n), next(n);
  std::vector<uint32_t> ver(n, 0);
  std::vector<bool> alive(n, true);
  for (size_t i = 0; i < n; ++i) {
    prev[i] = i == 0 ? SIZE_MAX : i - 1;
    next[i] = i + 1 == n ? SIZE_MAX : i + 1;
  }
  struct Cand {
    size_t rank, left, right;
    uint32_t vl, vr;
    bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : left > o.left; }
  };
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
  auto push = [&](size_t l) {
    if (l == SIZE_MAX || next[l] == SIZE_MAX) return;
    const size_t r = next[l];
    auto it = merge_rank_.find(tok[l] + '\x01' + tok[r]);
    if (it != merge_rank_.end()) heap.push(Cand{it->second, l, r, ver[l], ver[r]});
  };
  for (size_t i = 0; i + 1 < n; ++i) push(i);
  while (!heap.empty()) {
    const Cand c = heap.top();
    heap.pop();
    if (!alive[c.left] || !alive[c.right] || ver[c.left] != c.vl || ver[c.right] != c.vr || next[c.left] != c.right)
      continue;
    tok[c.left] += tok[c.right];
    ++ver[c.left];
    alive[c.right] = false;
    next[c.left] = next[c.right];
    if (next[c.right] != SIZE_MAX) prev[next[c.right]] = c.left;
    push(prev[c.left]);
    push(c.left);
  }
  for (size_t i = 0; i != SIZE_MAX && i < n; i = next[i]) {
    const std::string& t = tok[i];
    auto it = vocab_.find(t);
    if (it != vocab_.end()) out.push_back(it->second);
    else byte_fallback(t, out);
  }
  return out;
}

std::vector<uint32_t> Tokenizer::fallback_encode(const std::string& text) const {
  std::vector<uint32_t> out;
  const std::vector<std::string> ch = split_chars(text);
  size_t i = 0;
  while (i < ch.size()) {
    bool found = false;
    for (size_t len = std::min<size_t>(ch.size() - i, 20); len >= 1; --len) {  // longest first
      std::string sub;
      for (size_t k = 0; k < len; ++k) sub += ch[i + k];
      auto it = vocab_.find(sub);
      if (it != vocab_.end()) {
        out.push_back(it->second);
        i += len;
        found = true;
        break;
      }
    }
    if (!found) {
      byte_fallback(ch[i], out);
      ++i;
    }
  }
  return out;
}

std::string Tokenizer::decode(const uint32_t* ids, size_t n, bool skip_special) const {
  std::string bytes;
  for (size_t k = 0; k < n; ++k) {
    const uint32_t id = ids[k];
    if (skip_special && (id == special_.bos || id == special_.eos || id == special_.unk)) continue;
    auto it = reverse_.find(id);
    if (it == reverse_.end()) continue;
    const std::string& t = it->second;
    if (t.size() >= 4 && t.compare(0, 3, "<0x") == 0 && t.back() == '>') {
      uint8_t b;
      if (parse_hex_u8(t.substr(3, t.size() - 4), &b)) bytes += char(b);
    } else {
      bytes += t;
    }
  }
  return trim(replace_all(utf8_lossy(bytes), kSpaceMarker, " "));
}

}  // namespace wcb
