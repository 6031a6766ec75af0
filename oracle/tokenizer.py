"""Test infrastructure: a plain-Python restatement of the reference tokenizer
(crates/wasm-chord-core/src/tokenizer.rs), the oracle the C++ tokenizer behind
wcb_tokenize / wcb_detokenize is checked against. Only the tests import it.

Pinned by the reference's own unit tests (tokenizer.rs:428-500), reproduced as
known-answer tests in tests/test_tokenizer.py.
"""
from typing import Dict, List, Optional, Sequence, Tuple

SPACE_MARKER = "▁"

# char::is_whitespace: the Unicode White_Space property (str::trim)
_WS = set(range(0x09, 0x0E)) | {0x20, 0x85, 0xA0, 0x1680, 0x2028, 0x2029, 0x202F, 0x205F, 0x3000} | set(
    range(0x2000, 0x200B))


def rust_trim(s: str) -> str:
    b, e = 0, len(s)
    while b < e and ord(s[b]) in _WS:
        b += 1
    while e > b and ord(s[e - 1]) in _WS:
        e -= 1
    return s[b:e]


def parse_hex_u8(h: str) -> Optional[int]:
    """u8::from_str_radix(h, 16)."""
    if h.startswith("+"):
        h = h[1:]
    if not h or any(c not in "0123456789abcdefABCDEF" for c in h):
        return None
    v = int(h, 16)
    return v if v < 256 else None


class Tokenizer:
    def __init__(self, tokens: Sequence[str], merges: Sequence[Tuple[str, str]], bos: int = 1, eos: int = 2,
                 unk: int = 0):
        # Tokenizer::new (tokenizer.rs:63-80); the vocab HashMap keeps a duplicate's last id
        self.vocab: Dict[str, int] = {}
        for i, t in enumerate(tokens):
            self.vocab[t] = i
        self.reverse: Dict[int, str] = {v: k for k, v in self.vocab.items()}
        self.merges = list(merges)
        self.bos, self.eos, self.unk = bos, eos, unk
        self.add_bos, self.add_eos = True, False

    @staticmethod
    def merges_from_strings(strs: Sequence[str]) -> List[Tuple[str, str]]:
        """tokenizer.rs:102-117: 'a b' split on ' ' into exactly two parts."""
        out = []
        for s in strs:
            parts = s.split(" ")
            if len(parts) == 2:
                out.append((parts[0], parts[1]))
        return out

    def encode(self, text: str, add_special: bool = True) -> List[int]:
        """tokenizer.rs:207-231"""
        if not text:
            return []
        out = []
        if add_special and self.add_bos:
            out.append(self.bos)
        out += self._encode_bpe(SPACE_MARKER + text.replace(" ", SPACE_MARKER))
        if add_special and self.add_eos:
            out.append(self.eos)
        return out

    def _byte_fallback(self, piece: str) -> List[int]:
        return [self.vocab.get("<0x%02X>" % b, self.unk) for b in piece.encode("utf-8")]

    def _encode_bpe(self, text: str) -> List[int]:
        """tokenizer.rs:233-311"""
        if not text:
            return []
        tokens = list(text)
        if not self.merges:
            return self._fallback_encode(text)
        ranks: Dict[Tuple[str, str], int] = {}
        for r, pair in enumerate(self.merges):  # a repeated pair keeps its last rank
            ranks[pair] = r
        while len(tokens) > 1:
            best, best_rank = None, None
            for i in range(len(tokens) - 1):
                r = ranks.get((tokens[i], tokens[i + 1]))
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = i, r
            if best is None:
                break
            tokens[best] = tokens[best] + tokens[best + 1]
            del tokens[best + 1]
        out = []
        for t in tokens:
            if t in self.vocab:
                out.append(self.vocab[t])
            else:
                out += self._byte_fallback(t)
        return out

    def _fallback_encode(self, text: str) -> List[int]:
        """tokenizer.rs:313-351: longest match of at most 20 chars, else the char's bytes"""
        chars = list(text)
        out, i = [], 0
        while i < len(chars):
            for n in range(min(len(chars) - i, 20), 0, -1):
                sub = "".join(chars[i:i + n])
                if sub in self.vocab:
                    out.append(self.vocab[sub])
                    i += n
                    break
            else:
                out += self._byte_fallback(chars[i])
                i += 1
        return out

    def decode(self, ids: Sequence[int], skip_special: bool = True) -> str:
        """tokenizer.rs:353-395"""
        special = {self.bos, self.eos, self.unk} if skip_special else set()
        data = bytearray()
        for i in ids:
            if i in special:
                continue
            t = self.reverse.get(i)
            if t is None:
                continue
            if t.startswith("<0x") and t.endswith(">"):
                b = parse_hex_u8(t[3:-1])
                if b is not None:
                    data.append(b)
            else:
                data += t.encode("utf-8")
        # String::from_utf8_lossy replaces each maximal ill-formed subpart by U+FFFD,
        # as Python's 'replace' error handler does
        text = bytes(data).decode("utf-8", errors="replace")
        return rust_trim(text.replace(SPACE_MARKER, " "))
