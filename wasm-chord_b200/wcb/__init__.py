"""Python binding of the wcb C ABI (include/wcb.h), shaped like wasm-chord's
``wasm-chord-runtime`` API: ``Model.load_from_gguf`` / ``forward`` /
``generate`` / ``clear_kv_cache`` and ``GenerationConfig`` with the reference
defaults (crates/wasm-chord-runtime/src/transformer/config.rs:60-78).

The binding only marshals arguments; all compute runs in ``libwcb.so`` on the
GPU. There is no CPU fallback: loading a model without a CUDA device raises.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os
from typing import List, Optional, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwcb.so")

WCB_OK = 0
ERROR_NAMES = {
    0: "Ok", 1: "GenericFailure", 2: "OutOfMemory", 3: "InvalidArgument", 4: "ModelParseError",
    5: "BackendUnsupported", 6: "ShaderCompileError", 7: "IoError",
}
DTYPE_Q4_K = 12
DTYPE_Q6_K = 14
KV_F32 = 0
KV_F16 = 1

EXPORTED = [
    "wcb_gen_config_default", "wcb_model_load", "wcb_model_free", "wcb_model_config_get", "wcb_forward",
    "wcb_clear_kv", "wcb_kv_len", "wcb_generate_tokens", "wcb_generate_batch", "wcb_sampler_new",
    "wcb_sampler_sample", "wcb_sampler_free", "wcb_sampler_probs", "wcb_last_error", "wcb_version", "wcb_dequant_dev",
    "wcb_repack_q6k_dev", "wcb_gemv_dev", "wcb_model_stream", "wcb_infer", "wcb_next_tokens",
    "wcb_next_token", "wcb_close_stream", "wcb_model_launches_per_step", "wcb_batch_info", "wcb_tokenizer_load", "wcb_tokenizer_free",
    "wcb_tokenizer_info", "wcb_tokenizer_set_special", "wcb_tokenize", "wcb_detokenize", "wcb_generate_text",
    "wcb_attention_dev",
    "wcb_attention_dev_noalloc", "wcb_tp_id", "wcb_model_tp_handle", "wcb_model_tp_connect", "wcb_model_tp_abort",
    "wcb_load_opts_init", "wcb_struct_layout",
]

# the ctypes mirrors of include/wcb.h's structs, checked against the library's
# own sizes and offsets by check_layouts()
STRUCTS = {}


class WcbError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class _LoadOpts(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("device", C.c_int32), ("max_seq", C.c_uint32),
                ("kv_dtype", C.c_uint32), ("max_batch", C.c_uint32), ("flags", C.c_uint32),
                ("tp_rank", C.c_uint32), ("tp_size", C.c_uint32), ("tp_id", C.c_uint8 * 128),
                ("wait_ms", C.c_uint32)]


class _ModelConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_uint32), ("hidden_size", C.c_uint32), ("num_layers", C.c_uint32),
                ("num_heads", C.c_uint32), ("num_kv_heads", C.c_uint32), ("intermediate_size", C.c_uint32),
                ("max_seq_len", C.c_uint32), ("head_dim", C.c_uint32), ("rms_norm_eps", C.c_float),
                ("rope_theta", C.c_float)]


class _GenConfig(C.Structure):
    _fields_ = [("max_tokens", C.c_uint32), ("temperature", C.c_float), ("top_p", C.c_float),
                ("top_k", C.c_uint32), ("repetition_penalty", C.c_float), ("seed", C.c_uint64),
                ("eos_id", C.c_uint32)]


STRUCTS.update({"wcb_load_opts": _LoadOpts, "wcb_model_config": _ModelConfig, "wcb_gen_config": _GenConfig})

_LIB = None


def _point_at_shared_nccl() -> None:
    """The library loads NCCL at run time; point it at the copy PyTorch ships
    so a process that uses both loads one NCCL, whichever is imported first."""
    if os.environ.get("WCB_NCCL_LIB"):
        return
    import importlib.util
    spec = importlib.util.find_spec("nvidia")
    for base in (spec.submodule_search_locations or []) if spec else []:
        cand = os.path.join(base, "nccl", "lib", "libnccl.so.2")
        if os.path.exists(cand):
            os.environ["WCB_NCCL_LIB"] = cand
            return


def lib() -> C.CDLL:
    """Loads libwcb.so (building it first if it is missing)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        from . import build
        build.build_lib()
    _point_at_shared_nccl()
    L = C.CDLL(LIB_PATH)
    u32, sz, vp = C.c_uint32, C.c_size_t, C.c_void_p
    L.wcb_gen_config_default.argtypes = [C.POINTER(_GenConfig)]
    L.wcb_gen_config_default.restype = None
    L.wcb_model_load.argtypes = [C.c_char_p, C.POINTER(_LoadOpts), C.POINTER(u32)]
    L.wcb_model_free.argtypes = [u32]
    L.wcb_model_config_get.argtypes = [u32, C.POINTER(_ModelConfig)]
    L.wcb_forward.argtypes = [u32, vp, sz, sz, vp]
    L.wcb_clear_kv.argtypes = [u32]
    L.wcb_kv_len.argtypes = [u32, C.POINTER(sz)]
    L.wcb_generate_tokens.argtypes = [u32, vp, sz, C.POINTER(_GenConfig), vp, sz, C.POINTER(sz)]
    L.wcb_generate_batch.argtypes = [u32, vp, vp, sz, C.POINTER(_GenConfig), vp, sz, vp]
    L.wcb_sampler_new.argtypes = [C.POINTER(_GenConfig), C.POINTER(u32)]
    L.wcb_sampler_sample.argtypes = [u32, vp, sz, C.POINTER(u32)]
    L.wcb_sampler_free.argtypes = [u32]
    L.wcb_sampler_probs.argtypes = [u32, vp, sz]
    L.wcb_last_error.argtypes = [C.c_char_p, sz]
    L.wcb_last_error.restype = sz
    L.wcb_version.restype = C.c_char_p
    L.wcb_dequant_dev.argtypes = [vp, u32, sz, vp, vp]
    L.wcb_repack_q6k_dev.argtypes = [vp, sz, vp, vp]
    L.wcb_gemv_dev.argtypes = [vp, u32, sz, sz, vp, sz, vp, vp]
    L.wcb_model_stream.argtypes = [u32, C.POINTER(vp)]
    L.wcb_infer.argtypes = [u32, vp, sz, C.POINTER(_GenConfig), C.POINTER(u32)]
    L.wcb_next_tokens.argtypes = [u32, sz, vp, C.POINTER(sz), C.POINTER(u32)]
    L.wcb_next_token.argtypes = [u32, C.POINTER(u32)]
    L.wcb_next_token.restype = C.c_int32
    L.wcb_close_stream.argtypes = [u32]
    L.wcb_model_launches_per_step.argtypes = [u32, C.POINTER(u32)]
    L.wcb_batch_info.argtypes = [u32, C.POINTER(u32), C.POINTER(u32)]
    L.wcb_tokenizer_load.argtypes = [C.c_char_p, C.POINTER(u32)]
    L.wcb_tokenizer_free.argtypes = [u32]
    L.wcb_tokenizer_info.argtypes = [u32, C.POINTER(u32), C.POINTER(u32), C.POINTER(u32), C.POINTER(u32)]
    L.wcb_tokenizer_set_special.argtypes = [u32, u32, u32]
    L.wcb_tokenize.argtypes = [u32, C.c_char_p, u32, vp, sz, C.POINTER(sz)]
    L.wcb_detokenize.argtypes = [u32, vp, sz, u32, C.c_char_p, sz, C.POINTER(sz)]
    L.wcb_generate_text.argtypes = [u32, u32, C.c_char_p, C.POINTER(_GenConfig), C.c_char_p, sz, C.POINTER(sz)]
    L.wcb_attention_dev.argtypes = [vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, vp]
    L.wcb_attention_dev_noalloc.argtypes = [vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, vp]
    L.wcb_tp_id.argtypes = [vp]
    L.wcb_model_tp_handle.argtypes = [u32, vp]
    L.wcb_model_tp_connect.argtypes = [u32, vp, u32]
    L.wcb_model_tp_abort.argtypes = [u32]
    L.wcb_load_opts_init.argtypes = [C.POINTER(_LoadOpts)]
    L.wcb_load_opts_init.restype = None
    L.wcb_struct_layout.argtypes = [C.c_char_p, C.c_char_p]
    L.wcb_struct_layout.restype = sz
    for name in EXPORTED:
        f = getattr(L, name)
        if f.restype is C.c_int and name != "wcb_next_token":  # ctypes default
            f.restype = u32
    _LIB = L
    return L


def check_layouts() -> None:
    """Raises if a ctypes struct of this binding differs in size or field
    offsets from the library's (wcb_struct_layout)."""
    L = lib()
    for name, cls in STRUCTS.items():
        want = L.wcb_struct_layout(name.encode(), None)
        if want != C.sizeof(cls):
            raise RuntimeError(f"{name}: library size {want}, binding size {C.sizeof(cls)}")
        for fname, _ in cls._fields_:
            off = L.wcb_struct_layout(name.encode(), fname.encode())
            if off != getattr(cls, fname).offset:
                raise RuntimeError(f"{name}.{fname}: library offset {off}, binding offset "
                                   f"{getattr(cls, fname).offset}")


def last_error() -> str:
    buf = C.create_string_buffer(4096)
    lib().wcb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def _check(code: int) -> None:
    if code != WCB_OK:
        raise WcbError(code, last_error())


def version() -> str:
    return lib().wcb_version().decode()


@dataclasses.dataclass
class TransformerConfig:
    """transformer/config.rs:6-41"""
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    intermediate_size: int
    max_seq_len: int
    rms_norm_eps: float
    rope_theta: float
    head_dim: int


@dataclasses.dataclass
class GenerationConfig:
    """GenerationConfig (config.rs:60-78) with its defaults, plus the sampler
    seed generate() fixes at 42 (model.rs:1336) and the tokenizer's EOS id."""
    max_tokens: int = 100
    temperature: float = 0.7
    top_p: float = 0.9
    top_k: int = 40
    repetition_penalty: float = 1.1
    seed: int = 42
    eos_id: Optional[int] = 2

    def _c(self) -> _GenConfig:
        c = _GenConfig()
        c.max_tokens = int(self.max_tokens)
        c.temperature = float(self.temperature)
        c.top_p = float(self.top_p)
        c.top_k = int(self.top_k)
        c.repetition_penalty = float(self.repetition_penalty)
        c.seed = int(self.seed)
        c.eos_id = 0xFFFFFFFF if self.eos_id is None else int(self.eos_id)
        return c


def _u32(ids: Sequence[int]) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))


class Model:
    """One model replica on one GPU (the reference's ``Model``)."""

    def __init__(self, handle: int):
        self._h = handle
        cfg = _ModelConfig()
        _check(lib().wcb_model_config_get(handle, C.byref(cfg)))
        self.config = TransformerConfig(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                                        cfg.num_kv_heads, cfg.intermediate_size, cfg.max_seq_len,
                                        cfg.rms_norm_eps, cfg.rope_theta, cfg.head_dim)

    @classmethod
    def load_from_gguf(cls, path: str, device: int = 0, max_seq: int = 0, kv_dtype: int = KV_F32,
                       max_batch: int = 1, use_graphs: bool = True, use_pdl: bool = True,
                       use_tensor_cores: bool = True, use_persistent: bool = True, tp_rank: int = 0,
                       tp_size: int = 1, tp_id: bytes = b"", stream_weights: bool = False,
                       host_sampling: bool = False, wait_ms: int = 0) -> "Model":
        """Loads a GGUF file. tp_size > 1: this process holds tensor-parallel rank
        tp_rank's shard and joins the group named by tp_id (tp_unique_id() on one
        rank, the same bytes on every rank); forward() then fills only this rank's
        vocabulary slice of the logits. stream_weights: the layer weights stay in pinned
        host memory and stream to the GPU layer by layer (models larger than its memory).
        wait_ms: bound of the device-side waits on other ranks (0: the library's 2000 ms)."""
        flags = ((0 if use_graphs else 1) | (0 if use_pdl else 2) | (0 if use_tensor_cores else 4)
                 | (0 if use_persistent else 8) | (16 if stream_weights else 0) | (32 if host_sampling else 0))
        o = _LoadOpts()
        lib().wcb_load_opts_init(C.byref(o))
        o.device, o.max_seq, o.kv_dtype, o.max_batch = device, max_seq, kv_dtype, max_batch
        o.flags, o.tp_rank, o.tp_size = flags, tp_rank, tp_size
        if wait_ms:
            o.wait_ms = wait_ms
        if tp_size > 1:
            if len(tp_id) != 128:
                raise ValueError("tp_id must be the 128 bytes of tp_unique_id()")
            C.memmove(o.tp_id, tp_id, 128)
        h = C.c_uint32(0)
        _check(lib().wcb_model_load(os.fsencode(path), C.byref(o), C.byref(h)))
        return cls(h.value)

    def close(self) -> None:
        if self._h:
            lib().wcb_model_free(self._h)
            self._h = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> int:
        return self._h

    def forward(self, token_ids: Sequence[int], position: int) -> np.ndarray:
        """Model::forward (model.rs:832): logits of the last token, float32[vocab]."""
        ids = _u32(token_ids)
        out = np.empty(self.config.vocab_size, dtype=np.float32)
        _check(lib().wcb_forward(self._h, ids.ctypes.data, ids.size, int(position), out.ctypes.data))
        return out

    def clear_kv_cache(self) -> None:
        _check(lib().wcb_clear_kv(self._h))

    def kv_len(self) -> int:
        n = C.c_size_t(0)
        _check(lib().wcb_kv_len(self._h, C.byref(n)))
        return n.value

    def generate_tokens(self, prompt_ids: Sequence[int], config: GenerationConfig) -> List[int]:
        """Model::generate (model.rs:1322-1415) on token ids; returns the generated ids."""
        ids = _u32(prompt_ids)
        cap = max(1, int(config.max_tokens))
        out = np.zeros(cap, dtype=np.uint32)
        n = C.c_size_t(0)
        c = config._c()
        _check(lib().wcb_generate_tokens(self._h, ids.ctypes.data, ids.size, C.byref(c), out.ctypes.data, cap,
                                         C.byref(n)))
        return out[: min(n.value, cap)].tolist()

    def generate_text(self, prompt: str, tokenizer: "Tokenizer", config: GenerationConfig) -> str:
        """Model::generate(prompt, tokenizer, config) (model.rs:1322-1415): the prompt and
        the generated text, decoded together; the tokenizer's EOS ends the loop."""
        c = config._c()
        n = C.c_size_t(0)
        p = prompt.encode("utf-8")
        # room for the prompt and 256 bytes per generated token
        buf = C.create_string_buffer(len(p) + 256 * (max(1, int(config.max_tokens)) + 8))
        _check(lib().wcb_generate_text(self._h, tokenizer._h, p, C.byref(c), buf, len(buf), C.byref(n)))
        if n.value + 1 > len(buf):
            raise WcbError(1, f"generated text of {n.value} bytes exceeds the {len(buf)}-byte buffer")
        return buf.raw[: n.value].decode("utf-8")

    def generate_batch(self, prompts: Sequence[Sequence[int]], config: GenerationConfig) -> List[List[int]]:
        flat = _u32([t for p in prompts for t in p])
        lens = np.asarray([len(p) for p in prompts], dtype=np.uintp)
        cap = max(1, int(config.max_tokens))
        out = np.zeros((len(prompts), cap), dtype=np.uint32)
        n_out = np.zeros(len(prompts), dtype=np.uintp)
        c = config._c()
        _check(lib().wcb_generate_batch(self._h, flat.ctypes.data, lens.ctypes.data, len(prompts), C.byref(c),
                                        out.ctypes.data, cap, n_out.ctypes.data))
        return [out[i, : min(int(n_out[i]), cap)].tolist() for i in range(len(prompts))]

    def infer(self, prompt_ids: Sequence[int], config: GenerationConfig) -> "TokenStream":
        """Starts generate()'s loop as a stream (wasmchord_infer, abi.rs:119-150)."""
        ids = _u32(prompt_ids)
        c = config._c()
        s = C.c_uint32(0)
        _check(lib().wcb_infer(self._h, ids.ctypes.data, ids.size, C.byref(c), C.byref(s)))
        return TokenStream(s.value)

    def tp_ipc_handle(self) -> bytes:
        """This rank's receive-buffer IPC handle (64 bytes) for tp_connect."""
        buf = (C.c_uint8 * 64)()
        _check(lib().wcb_model_tp_handle(self._h, buf))
        return bytes(buf)

    def tp_connect(self, handles) -> None:
        """Every rank's tp_ipc_handle() in rank order: decode steps then exchange
        partial sums by peer stores instead of NCCL."""
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _check(lib().wcb_model_tp_connect(self._h, buf, len(handles)))

    def tp_abort(self) -> None:
        """Abandons this rank's tensor-parallel group after another rank failed
        (ncclCommAbort); every later call on the model fails, close() does not wait
        for the other ranks. Safe to call from a watchdog thread."""
        _check(lib().wcb_model_tp_abort(self._h))

    def batch_info(self) -> Tuple[int, int]:
        """(KV slots of one batched decode step, kernels one batched step launches)."""
        slots, launches = C.c_uint32(0), C.c_uint32(0)
        _check(lib().wcb_batch_info(self._h, C.byref(slots), C.byref(launches)))
        return int(slots.value), int(launches.value)

    def launches_per_step(self) -> int:
        n = C.c_uint32(0)
        _check(lib().wcb_model_launches_per_step(self._h, C.byref(n)))
        return n.value

    def stream(self) -> int:
        s = C.c_void_p(0)
        _check(lib().wcb_model_stream(self._h, C.byref(s)))
        return s.value or 0


class Tokenizer:
    """Tokenizer (crates/wasm-chord-core/src/tokenizer.rs) loaded from a GGUF file's
    tokenizer.ggml.* metadata."""

    def __init__(self, path: str):
        h = C.c_uint32(0)
        _check(lib().wcb_tokenizer_load(path.encode(), C.byref(h)))
        self._h = h.value

    def close(self) -> None:
        if self._h:
            lib().wcb_tokenizer_free(self._h)
            self._h = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> Tuple[int, int, int, int]:
        """(vocab size, bos id, eos id, unk id)"""
        v = [C.c_uint32(0) for _ in range(4)]
        _check(lib().wcb_tokenizer_info(self._h, *[C.byref(x) for x in v]))
        return tuple(int(x.value) for x in v)

    def set_special(self, add_bos: bool, add_eos: bool) -> None:
        _check(lib().wcb_tokenizer_set_special(self._h, int(add_bos), int(add_eos)))

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        b = text.encode("utf-8")
        n = C.c_size_t(0)
        _check(lib().wcb_tokenize(self._h, b, int(add_special_tokens), None, 0, C.byref(n)))
        out = np.zeros(max(1, n.value), dtype=np.uint32)
        _check(lib().wcb_tokenize(self._h, b, int(add_special_tokens), out.ctypes.data, out.size, C.byref(n)))
        return out[: n.value].tolist()

    def encode_bytes(self, text: bytes, add_special_tokens: bool = True) -> List[int]:
        """encode() of raw bytes (the library rejects bytes that are not UTF-8)."""
        n = C.c_size_t(0)
        out = np.zeros(4 * len(text) + 8, dtype=np.uint32)
        _check(lib().wcb_tokenize(self._h, text, int(add_special_tokens), out.ctypes.data, out.size, C.byref(n)))
        return out[: n.value].tolist()

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        a = _u32(ids)
        n = C.c_size_t(0)
        _check(lib().wcb_detokenize(self._h, a.ctypes.data, a.size, int(skip_special_tokens), None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value + 1)
        _check(lib().wcb_detokenize(self._h, a.ctypes.data, a.size, int(skip_special_tokens), buf, len(buf),
                                    C.byref(n)))
        return buf.raw[: n.value].decode("utf-8")


class TokenStream:
    """A generation stream (wasmchord_next_token / close_stream, abi.rs:155-200)."""

    def __init__(self, handle: int):
        self._h = handle
        self.finished = False

    def next_tokens(self, max_tokens: int) -> List[int]:
        out = np.zeros(max(1, max_tokens), dtype=np.uint32)
        n = C.c_size_t(0)
        fin = C.c_uint32(0)
        _check(lib().wcb_next_tokens(self._h, max_tokens, out.ctypes.data, C.byref(n), C.byref(fin)))
        self.finished = bool(fin.value)
        return out[: n.value].tolist()

    def next_token(self) -> Optional[int]:
        t = C.c_uint32(0)
        r = lib().wcb_next_token(self._h, C.byref(t))
        if r == -2:
            raise WcbError(1, last_error())
        return None if r == -1 else t.value

    def close(self) -> None:
        if self._h:
            lib().wcb_close_stream(self._h)
            self._h = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class LogitsProcessor:
    """sampling.rs:29-264 through the C ABI (host sampler); sampled draws take the
    reference's rand 0.9 StdRng::seed_from_u64(seed) stream."""

    def __init__(self, seed: int, temperature: float, top_p: float, top_k: int, repetition_penalty: float):
        c = GenerationConfig(temperature=temperature, top_p=top_p, top_k=top_k,
                             repetition_penalty=repetition_penalty, seed=seed)._c()
        h = C.c_uint32(0)
        _check(lib().wcb_sampler_new(C.byref(c), C.byref(h)))
        self._h = h.value

    def sample(self, logits: np.ndarray) -> int:
        if logits.dtype != np.float32 or not logits.flags.c_contiguous:
            raise TypeError("logits must be a contiguous float32 array (it is modified in place)")
        t = C.c_uint32(0)
        _check(lib().wcb_sampler_sample(self._h, logits.ctypes.data, logits.size, C.byref(t)))
        return t.value

    def last_probs(self, n: int) -> np.ndarray:
        """The n probabilities the last sampled draw used (zero outside the kept candidates)."""
        out = np.empty(n, dtype=np.float32)
        _check(lib().wcb_sampler_probs(self._h, out.ctypes.data, n))
        return out

    def __del__(self):
        try:
            lib().wcb_sampler_free(self._h)
        except Exception:
            pass


# ---- kernel-level entry points on device pointers ---------------------------
def dequant_dev(blocks_ptr: int, dtype: int, nblocks: int, out_ptr: int, stream: int = 0) -> None:
    _check(lib().wcb_dequant_dev(blocks_ptr, dtype, nblocks, out_ptr, stream or None))


def repack_q6k_dev(packed_ptr: int, nblocks: int, padded_ptr: int, stream: int = 0) -> None:
    _check(lib().wcb_repack_q6k_dev(packed_ptr, nblocks, padded_ptr, stream or None))


def gemv_dev(w_ptr: int, dtype: int, n: int, k: int, x_ptr: int, m: int, y_ptr: int, stream: int = 0) -> None:
    """wcb_gemv_dev: y[m][n] = x[m][k] . W[n][k] on device pointers (matmul_transposed,
    gemm.rs:83-143). W and x 16-byte aligned, k % 256 == 0, n % 4 == 0, 1 <= m <= 4096;
    m <= 4 runs the dp4a GEMV, 5..32 the batched tensor-core GEMM, larger m the prefill GEMM."""
    _check(lib().wcb_gemv_dev(w_ptr, dtype, n, k, x_ptr, m, y_ptr, stream or None))


def attention_dev(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, n_tokens: int, n_heads: int, n_kv_heads: int,
                  head_dim: int, max_seq: int, kv_len: int, position: int, stream: int = 0) -> None:
    _check(lib().wcb_attention_dev(q_ptr, k_ptr, v_ptr, out_ptr, n_tokens, n_heads, n_kv_heads, head_dim, max_seq,
                                   kv_len, position, stream or None))


def attention_dev_noalloc(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, n_tokens: int, n_heads: int,
                          n_kv_heads: int, head_dim: int, max_seq: int, kv_len: int, position: int,
                          stream: int = 0) -> None:
    """wcb_attention_dev with the library's fixed scratch array (no GPU allocation)."""
    _check(lib().wcb_attention_dev_noalloc(q_ptr, k_ptr, v_ptr, out_ptr, n_tokens, n_heads, n_kv_heads, head_dim,
                                           max_seq, kv_len, position, stream or None))


def tp_unique_id() -> bytes:
    """A fresh tensor-parallel group id (128 bytes) for Model.load_from_gguf(tp_id=...)."""
    buf = (C.c_uint8 * 128)()
    _check(lib().wcb_tp_id(buf))
    return bytes(buf)
