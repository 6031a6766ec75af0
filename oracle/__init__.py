"""ctypes binding of the oracle (oracle.cpp): TEST INFRASTRUCTURE ONLY.

The oracle is the CPU restatement of the wasm-chord reference path used as the
parity checker by tests/, __graft_entry__.smoke() and as the timed CPU baseline
by bench.py. The product (wasm-chord_b200/) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "liboracle.so")
_LIB = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    src = os.path.join(HERE, "oracle.cpp")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(src) > os.path.getmtime(LIB_PATH):
        build()
    L = C.CDLL(LIB_PATH)
    sz, vp, u32, f32 = C.c_size_t, C.c_void_p, C.c_uint32, C.c_float
    L.oracle_last_error.argtypes = [C.c_char_p, sz]
    L.oracle_last_error.restype = sz
    L.oracle_set_threads.argtypes = [C.c_int, C.c_int]
    L.oracle_set_threads.restype = None
    L.oracle_set_faithful.argtypes = [C.c_int]
    L.oracle_set_faithful.restype = None
    L.oracle_open.argtypes = [C.c_char_p, C.POINTER(vp)]
    L.oracle_open.restype = u32
    L.oracle_free.argtypes = [vp]
    L.oracle_free.restype = None
    L.oracle_config.argtypes = [vp, vp, vp]
    L.oracle_config.restype = None
    L.oracle_forward.argtypes = [vp, vp, sz, sz, vp]
    L.oracle_forward.restype = u32
    L.oracle_clear_kv.argtypes = [vp]
    L.oracle_clear_kv.restype = None
    L.oracle_kv_len.argtypes = [vp]
    L.oracle_kv_len.restype = sz
    L.oracle_generate.argtypes = [vp, vp, sz, sz, f32, f32, sz, f32, C.c_uint64, u32, vp, sz, C.POINTER(sz), vp, sz]
    L.oracle_generate.restype = u32
    L.oracle_tensor_f32.argtypes = [vp, C.c_char_p, vp, sz, C.POINTER(sz)]
    L.oracle_tensor_f32.restype = u32
    for n in ("oracle_dequant_q4k", "oracle_dequant_q6k"):
        getattr(L, n).argtypes = [vp, sz, vp]
        getattr(L, n).restype = None
    L.oracle_matmul_transposed.argtypes = [vp, vp, vp, sz, sz, sz]
    L.oracle_matmul_transposed.restype = None
    L.oracle_rms_norm.argtypes = [vp, vp, f32, sz, sz, vp]
    L.oracle_rms_norm.restype = None
    L.oracle_rope.argtypes = [vp, sz, sz, sz, sz, f32]
    L.oracle_rope.restype = None
    L.oracle_attention.argtypes = [vp, vp, vp, sz, sz, sz, sz, sz, sz, vp]
    L.oracle_attention.restype = None
    L.oracle_kv_new.argtypes = [sz, sz, sz]
    L.oracle_kv_new.restype = vp
    L.oracle_kv_free.argtypes = [vp]
    L.oracle_kv_free.restype = None
    L.oracle_kv_append.argtypes = [vp, vp, vp, sz, C.POINTER(sz)]
    L.oracle_kv_append.restype = u32
    L.oracle_kv_keys.argtypes = [vp]
    L.oracle_kv_keys.restype = C.POINTER(f32)
    L.oracle_kv_values.argtypes = [vp]
    L.oracle_kv_values.restype = C.POINTER(f32)
    L.oracle_sampler_new.argtypes = [C.c_uint64, C.c_double, C.c_double, sz, f32]
    L.oracle_sampler_new.restype = vp
    L.oracle_sampler_free.argtypes = [vp]
    L.oracle_chacha_block.restype = None
    L.oracle_chacha_block.argtypes = [vp, C.c_uint64, C.c_int, vp]
    L.oracle_std_rng_u32.restype = None
    L.oracle_std_rng_u32.argtypes = [C.c_uint64, sz, vp]
    L.oracle_sampler_free.restype = None
    L.oracle_sampler_sample.argtypes = [vp, vp, sz, C.POINTER(u32)]
    L.oracle_sampler_sample.restype = u32
    L.oracle_sampler_penalize.argtypes = [vp, vp, sz]
    L.oracle_sampler_penalize.restype = None
    L.oracle_sampler_kind.argtypes = [vp]
    L.oracle_sampler_kind.restype = C.c_int
    L.oracle_sampler_distribution.argtypes = [vp, vp, sz, vp]
    L.oracle_sampler_distribution.restype = None
    _LIB = L
    return L


class OracleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"oracle error {code}: {msg}")
        self.code = code


def _err(code: int) -> None:
    if code:
        buf = C.create_string_buffer(2048)
        lib().oracle_last_error(buf, len(buf))
        raise OracleError(code, buf.value.decode(errors="replace"))


def set_threads(lm_head: int, projections: int) -> None:
    lib().oracle_set_threads(lm_head, projections)


def set_faithful(faithful: bool) -> None:
    """True: matmul_transposed walks one output row at a time, the reference's
    exact loop (for timing); False: four rows per pass, same per-row arithmetic."""
    lib().oracle_set_faithful(1 if faithful else 0)


def f32p(a: np.ndarray) -> int:
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data


def dequant_q4k(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    n = b.size // 144
    out = np.empty(n * 256, dtype=np.float32)
    lib().oracle_dequant_q4k(b.ctypes.data, n, out.ctypes.data)
    return out


def dequant_q6k(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    n = b.size // 210
    out = np.empty(n * 256, dtype=np.float32)
    lib().oracle_dequant_q6k(b.ctypes.data, n, out.ctypes.data)
    return out


def matmul_transposed(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    n = b.shape[0]
    c = np.empty((m, n), dtype=np.float32)
    lib().oracle_matmul_transposed(a.ctypes.data, b.ctypes.data, c.ctypes.data, m, k, n)
    return c


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    seq, hidden = x.shape
    out = np.empty_like(x)
    lib().oracle_rms_norm(x.ctypes.data, w.ctypes.data, eps, seq, hidden, out.ctypes.data)
    return out


def rope(t: np.ndarray, start_pos: int, heads: int, head_dim: int, theta: float) -> np.ndarray:
    t = np.array(t, dtype=np.float32, copy=True, order="C")
    seq = t.size // (heads * head_dim)
    lib().oracle_rope(t.ctypes.data, start_pos, seq, heads, head_dim, theta)
    return t


def attention(q, k, v, seq, kv_seq, position, heads, kv_heads, head_dim) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty(seq * heads * head_dim, dtype=np.float32)
    lib().oracle_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, seq, kv_seq, position, heads, kv_heads,
                           head_dim, out.ctypes.data)
    return out


class KVCache:
    def __init__(self, max_seq: int, n_kv: int, head_dim: int):
        self._h = lib().oracle_kv_new(max_seq, n_kv, head_dim)
        self.size = max_seq * n_kv * head_dim

    def append(self, k: np.ndarray, v: np.ndarray, seq: int) -> int:
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        n = C.c_size_t(0)
        _err(lib().oracle_kv_append(self._h, k.ctypes.data, v.ctypes.data, seq, C.byref(n)))
        return n.value

    def keys(self) -> np.ndarray:
        return np.ctypeslib.as_array(lib().oracle_kv_keys(self._h), shape=(self.size,)).copy()

    def values(self) -> np.ndarray:
        return np.ctypeslib.as_array(lib().oracle_kv_values(self._h), shape=(self.size,)).copy()

    def __del__(self):
        try:
            lib().oracle_kv_free(self._h)
        except Exception:
            pass


class Sampler:
    KINDS = ["ArgMax", "All", "TopK", "TopP", "TopKThenTopP"]

    def __init__(self, seed: int, temperature: float, top_p: float, top_k: int, rep: float):
        self._h = lib().oracle_sampler_new(seed, temperature, top_p, top_k, rep)

    @property
    def kind(self) -> str:
        return self.KINDS[lib().oracle_sampler_kind(self._h)]

    def sample(self, logits: np.ndarray) -> int:
        t = C.c_uint32(0)
        _err(lib().oracle_sampler_sample(self._h, f32p(logits), logits.size, C.byref(t)))
        return t.value

    def penalize(self, logits: np.ndarray) -> None:
        lib().oracle_sampler_penalize(self._h, f32p(logits), logits.size)

    def distribution(self, logits: np.ndarray) -> np.ndarray:
        """The probabilities sample() would draw from (penalty, compute_probabilities,
        top-k, top-p, renormalisation; sampling.rs:106-229), without drawing."""
        out = np.empty(logits.size, dtype=np.float32)
        lib().oracle_sampler_distribution(self._h, f32p(logits), logits.size, out.ctypes.data)
        return out

    def __del__(self):
        try:
            lib().oracle_sampler_free(self._h)
        except Exception:
            pass


def chacha_block(key: bytes, counter: int, rounds: int) -> list:
    """The 16 words of keystream block `counter` of ChaCha with `rounds` rounds
    (64-bit counter, zero stream id)."""
    assert len(key) == 32
    out = (C.c_uint32 * 16)()
    kb = C.create_string_buffer(bytes(key), 32)
    lib().oracle_chacha_block(C.addressof(kb), counter, rounds, C.addressof(out))
    return list(out)


def std_rng_u32(seed: int, n: int) -> list:
    """The first n u32 outputs of rand 0.9 StdRng::seed_from_u64(seed)."""
    out = (C.c_uint32 * n)()
    lib().oracle_std_rng_u32(seed, n, C.addressof(out))
    return list(out)


class OracleModel:
    """The reference Model (default features) on the CPU."""

    def __init__(self, path: str):
        h = C.c_void_p(0)
        _err(lib().oracle_open(os.fsencode(path), C.byref(h)))
        self._h = h.value
        cfg = np.zeros(8, dtype=np.uint32)
        et = np.zeros(2, dtype=np.float32)
        lib().oracle_config(self._h, cfg.ctypes.data, et.ctypes.data)
        (self.vocab, self.hidden, self.layers, self.heads, self.kv_heads, self.ffn, self.max_seq,
         self.head_dim) = (int(v) for v in cfg)
        self.eps, self.theta = float(et[0]), float(et[1])

    def close(self):
        if self._h:
            lib().oracle_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, ids: Sequence[int], position: int) -> np.ndarray:
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
        out = np.empty(self.vocab, dtype=np.float32)
        _err(lib().oracle_forward(self._h, a.ctypes.data, a.size, position, out.ctypes.data))
        return out

    def clear_kv_cache(self):
        lib().oracle_clear_kv(self._h)

    def kv_len(self) -> int:
        return lib().oracle_kv_len(self._h)

    def tensor(self, name: str) -> np.ndarray:
        n = C.c_size_t(0)
        _err(lib().oracle_tensor_f32(self._h, name.encode(), None, 0, C.byref(n)))
        out = np.empty(n.value, dtype=np.float32)
        _err(lib().oracle_tensor_f32(self._h, name.encode(), out.ctypes.data, out.size, C.byref(n)))
        return out

    def generate(self, prompt: Sequence[int], max_tokens: int, temperature: float = 0.0, top_p: float = 1.0,
                 top_k: int = 0, repetition_penalty: float = 1.0, seed: int = 42, eos_id: Optional[int] = 2,
                 return_logits: bool = False):
        a = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        cap = max(1, max_tokens)
        out = np.zeros(cap, dtype=np.uint32)
        n = C.c_size_t(0)
        steps = np.zeros((cap, self.vocab), dtype=np.float32) if return_logits else None
        eos = 0xFFFFFFFF if eos_id is None else eos_id
        _err(lib().oracle_generate(self._h, a.ctypes.data, a.size, max_tokens, temperature, top_p, top_k,
                                   repetition_penalty, seed, eos, out.ctypes.data, cap, C.byref(n),
                                   steps.ctypes.data if steps is not None else None,
                                   steps.size if steps is not None else 0))
        toks: List[int] = out[: min(n.value, cap)].tolist()
        if return_logits:
            return toks, steps
        return toks
