"""Seeded synthetic Llama-architecture GGUF models (Q4_K / Q6_K weights).

The workloads have no downloadable checkpoint, so every model used by the tests
and the benchmark is written here: 2-D weights quantised to GGUF Q4_K (144-byte super-blocks of 256 values) or Q6_K (210-byte super-blocks),
embeddings and norm vectors stored as f32. Weights are N(0, 0.02) (norm
vectors 1 + N(0, 0.02)) from a counter-based generator (csrc/synth.cpp) keyed
on (seed, tensor index, element index), so a model is reproducible on any host.

Container format: GGUF v3 as read by the reference parser
(crates/wasm-chord-core/src/formats/gguf.rs:111-159 header, :347-412 metadata,
:414-444 tensor infos, :162-172 32-byte data alignment). Metadata keys are the
ones ``extract_config`` reads (gguf.rs:208-276). Tensor names are the ones
``Model::load_from_gguf`` looks up (transformer/model.rs:432-760).

Block layouts follow crates/wasm-chord-core/src/quant.rs:32-38 (BlockQ4_K) and
:121-126 (BlockQ6_K); the scale packing is the inverse of ``get_scale_min_k4``
(quant.rs:43-53). Any valid quantiser is acceptable because parity is defined
on the dequantised values; this one is a plain min/max rounding quantiser.
"""
from __future__ import annotations

import dataclasses
import os
import struct

import numpy as np

QK_K = 256
Q4_K_BYTES = 144
Q6_K_BYTES = 210

GGML_F32 = 0
GGML_F16 = 1
GGML_Q4_K = 12
GGML_Q6_K = 14


# --------------------------------------------------------------------------
# quantisers
# --------------------------------------------------------------------------
def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    """Quantise a float32 vector (len % 256 == 0) to Q4_K blocks, uint8 [nb,144]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.size % QK_K == 0
    xb = x.reshape(-1, 8, 32)
    nb = xb.shape[0]
    mn = np.minimum(xb.min(axis=-1), np.float32(0))
    mx = xb.max(axis=-1)
    scale = (mx - mn) / np.float32(15)
    mneg = -mn
    d16 = (scale.max(axis=-1) / np.float32(63)).astype(np.float16)
    dm16 = (mneg.max(axis=-1) / np.float32(63)).astype(np.float16)
    d32 = d16.astype(np.float32)[:, None]
    dm32 = dm16.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32 > 0, np.rint(scale / d32), 0).clip(0, 63).astype(np.uint8)
        mq = np.where(dm32 > 0, np.rint(mneg / dm32), 0).clip(0, 63).astype(np.uint8)
        d1 = (d32 * sc.astype(np.float32))[..., None]
        m1 = (dm32 * mq.astype(np.float32))[..., None]
        q = np.where(d1 > 0, np.rint((xb + m1) / d1), 0).clip(0, 15).astype(np.uint8)
    out = np.empty((nb, Q4_K_BYTES), dtype=np.uint8)
    out[:, 0:2] = d16.reshape(nb, 1).view(np.uint8)
    out[:, 2:4] = dm16.reshape(nb, 1).view(np.uint8)
    # 12 scale bytes: the inverse of get_scale_min_k4 (quant.rs:43-53)
    lo_sc, hi_sc = sc[:, :4], sc[:, 4:]
    lo_m, hi_m = mq[:, :4], mq[:, 4:]
    out[:, 4:8] = (lo_sc & 63) | ((hi_sc >> 4) << 6)
    out[:, 8:12] = (lo_m & 63) | ((hi_m >> 4) << 6)
    out[:, 12:16] = (hi_sc & 0xF) | ((hi_m & 0xF) << 4)
    # qs: pair p holds sub-block 2p in the low nibbles and 2p+1 in the high ones
    qp = q.reshape(nb, 4, 2, 32)
    out[:, 16:] = (qp[:, :, 0, :] | (qp[:, :, 1, :] << 4)).reshape(nb, 128)
    return out


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    """Quantise a float32 vector (len % 256 == 0) to Q6_K blocks, uint8 [nb,210]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.size % QK_K == 0
    xb = x.reshape(-1, 16, 16)
    nb = xb.shape[0]
    amax = np.abs(xb).max(axis=-1)
    scale = amax / np.float32(31)
    d16 = (scale.max(axis=-1) / np.float32(127)).astype(np.float16)
    d32 = d16.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32 > 0, np.rint(scale / d32), 0).clip(-127, 127).astype(np.int8)
        ds = (d32 * sc.astype(np.float32))[..., None]
        q = np.where(ds != 0, np.rint(xb / ds), 0).clip(-32, 31).astype(np.int16) + 32
    q = q.astype(np.uint8).reshape(nb, 2, 4, 32)  # [half, quarter k, l]
    out = np.empty((nb, Q6_K_BYTES), dtype=np.uint8)
    q1, q2, q3, q4 = q[:, :, 0], q[:, :, 1], q[:, :, 2], q[:, :, 3]
    ql = np.empty((nb, 2, 64), dtype=np.uint8)
    ql[:, :, :32] = (q1 & 0xF) | ((q3 & 0xF) << 4)
    ql[:, :, 32:] = (q2 & 0xF) | ((q4 & 0xF) << 4)
    qh = (q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d16.reshape(nb, 1).view(np.uint8)
    return out


def dequantize_q4_k_np(blocks: np.ndarray) -> np.ndarray:
    """numpy restatement of quant.rs:58-115 (used only for generator self-checks)."""
    b = blocks.reshape(-1, Q4_K_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    dm = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    s = b[:, 4:16].astype(np.uint8)
    sc = np.empty((b.shape[0], 8), np.uint8)
    mn = np.empty((b.shape[0], 8), np.uint8)
    sc[:, :4] = s[:, 0:4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    d1 = d * sc.astype(np.float32)
    m1 = dm * mn.astype(np.float32)
    qs = b[:, 16:].reshape(-1, 4, 32)
    q = np.stack([qs & 0xF, qs >> 4], axis=2).reshape(-1, 8, 32).astype(np.float32)
    return (d1[..., None] * q - m1[..., None]).reshape(-1)


# --------------------------------------------------------------------------
# model presets
# --------------------------------------------------------------------------
@dataclasses.dataclass
class SynthConfig:
    vocab_size: int = 32000
    hidden_size: int = 2048
    num_layers: int = 22
    num_heads: int = 32
    num_kv_heads: int = 4
    intermediate_size: int = 5632
    context_length: int = 4096
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    # "q4_k" = Q4_K everywhere; "q4_k_m" = Q6_K for output.weight and for
    # attn_v / ffn_down in even layers, Q4_K elsewhere
    quant_mix: str = "q4_k"
    seed: int = 0
    weight_std: float = 0.02
    # > 0: layer i repeats the tensors of layer i % layer_period (deep models for
    # timing runs without generating every layer's values)
    layer_period: int = 0

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads


PRESETS = {
    # TinyLlama-1.1B architecture
    "tinyllama": SynthConfig(),
    # Llama-2-7B architecture with the Q4_K_M mix
    "llama7b": SynthConfig(hidden_size=4096, num_layers=32, num_heads=32, num_kv_heads=32,
                           intermediate_size=11008, quant_mix="q4_k_m"),
    # Llama-2-70B architecture, Q4_K
    "llama70b": SynthConfig(hidden_size=8192, num_layers=80, num_heads=64, num_kv_heads=8,
                            intermediate_size=28672),
    # small configurations for parity tests (K must be a multiple of 256)
    "tiny": SynthConfig(vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                        num_kv_heads=2, intermediate_size=512, context_length=256),
    "tiny_mix": SynthConfig(vocab_size=768, hidden_size=512, num_layers=2, num_heads=8,
                            num_kv_heads=8, intermediate_size=768, context_length=160,
                            quant_mix="q4_k_m"),
    # splits over 2 tensor-parallel ranks (hidden / 2 and intermediate / 2 multiples of 256)
    "tiny_tp": SynthConfig(vocab_size=1024, hidden_size=512, num_layers=2, num_heads=8,
                           num_kv_heads=4, intermediate_size=1024, context_length=256),
}


def tensor_plan(cfg: SynthConfig):
    """Ordered (name, shape_ne, ggml_type) list. ne = GGUF dims, innermost first."""
    H, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    kv = cfg.num_kv_heads * cfg.head_dim
    plan = [("token_embd.weight", (H, V), GGML_F32)]
    for i in range(cfg.num_layers):
        mix6 = cfg.quant_mix == "q4_k_m" and i % 2 == 0
        plan += [
            (f"blk.{i}.attn_norm.weight", (H,), GGML_F32),
            (f"blk.{i}.attn_q.weight", (H, H), GGML_Q4_K),
            (f"blk.{i}.attn_k.weight", (H, kv), GGML_Q4_K),
            (f"blk.{i}.attn_v.weight", (H, kv), GGML_Q6_K if mix6 else GGML_Q4_K),
            (f"blk.{i}.attn_output.weight", (H, H), GGML_Q4_K),
            (f"blk.{i}.ffn_norm.weight", (H,), GGML_F32),
            (f"blk.{i}.ffn_gate.weight", (H, F), GGML_Q4_K),
            (f"blk.{i}.ffn_up.weight", (H, F), GGML_Q4_K),
            (f"blk.{i}.ffn_down.weight", (F, H), GGML_Q6_K if mix6 else GGML_Q4_K),
        ]
    plan += [
        ("output_norm.weight", (H,), GGML_F32),
        ("output.weight", (H, V), GGML_Q6_K if cfg.quant_mix == "q4_k_m" else GGML_Q4_K),
    ]
    return plan


def _tensor_nbytes(ne, ggml_type) -> int:
    n = int(np.prod(ne))
    if ggml_type == GGML_F32:
        return 4 * n
    if ggml_type == GGML_F16:
        return 2 * n
    if ggml_type == GGML_Q4_K:
        return n // QK_K * Q4_K_BYTES
    if ggml_type == GGML_Q6_K:
        return n // QK_K * Q6_K_BYTES
    raise ValueError(ggml_type)


_CLIB = None


def _clib():
    """The compiled bulk generator (csrc/synth.cpp -> wcb/libwcb_synth.so)."""
    global _CLIB
    if _CLIB is None:
        import ctypes
        path = os.path.join(os.path.dirname(__file__), "libwcb_synth.so")
        if not os.path.exists(path):
            from . import build as _build
            _build.build_synth()
        lib = ctypes.CDLL(path)
        c = ctypes
        lib.wcb_synth_fill_normal.argtypes = [c.c_uint64, c.c_uint64, c.c_int64, c.c_float,
                                              c.c_float, c.c_void_p, c.c_int]
        lib.wcb_synth_quantize_q4k.argtypes = [c.c_void_p, c.c_int64, c.c_void_p, c.c_int]
        lib.wcb_synth_quantize_q6k.argtypes = [c.c_void_p, c.c_int64, c.c_void_p, c.c_int]
        _CLIB = lib
    return _CLIB


def _threads() -> int:
    return max(1, min(32, os.cpu_count() or 1))


def normal(seed: int, stream: int, n: int, mean: float, std: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    _clib().wcb_synth_fill_normal(seed, stream, n, mean, std, out.ctypes.data, _threads())
    return out


def quantize_q4_k_fast(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((x.size // QK_K, Q4_K_BYTES), dtype=np.uint8)
    _clib().wcb_synth_quantize_q4k(x.ctypes.data, x.size, out.ctypes.data, _threads())
    return out


def quantize_q6_k_fast(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((x.size // QK_K, Q6_K_BYTES), dtype=np.uint8)
    _clib().wcb_synth_quantize_q6k(x.ctypes.data, x.size, out.ctypes.data, _threads())
    return out


def _gen_tensor(index, name, ne, ggml_type, cfg: SynthConfig) -> bytes:
    n = int(np.prod(ne))
    mean = 1.0 if name.endswith("norm.weight") else 0.0
    vals = normal(cfg.seed, index, n, mean, cfg.weight_std)
    if ggml_type == GGML_F32:
        return vals.tobytes()
    if ggml_type == GGML_F16:
        return vals.astype(np.float16).tobytes()
    if ggml_type == GGML_Q4_K:
        return quantize_q4_k_fast(vals).tobytes()
    if ggml_type == GGML_Q6_K:
        return quantize_q6_k_fast(vals).tobytes()
    raise ValueError(ggml_type)


# --------------------------------------------------------------------------
# GGUF writer
# --------------------------------------------------------------------------
def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _kv_u32(key, v):
    return _s(key) + struct.pack("<II", 4, v)


def _kv_f32(key, v):
    return _s(key) + struct.pack("<If", 6, v)


def _kv_str(key, v):
    return _s(key) + struct.pack("<I", 8) + _s(v)


ALIGN = 32


def write_gguf(path: str, cfg: SynthConfig, plan=None, extra_kv=None) -> str:
    """Write a GGUF v3 file for ``cfg``; returns ``path``."""
    plan = plan if plan is not None else tensor_plan(cfg)
    arch = "llama"
    kvs = [
        _kv_str("general.architecture", arch),
        _kv_str("general.name", "wcb-synthetic"),
        _kv_u32(f"{arch}.vocab_size", cfg.vocab_size),
        _kv_u32(f"{arch}.embedding_length", cfg.hidden_size),
        _kv_u32(f"{arch}.block_count", cfg.num_layers),
        _kv_u32(f"{arch}.attention.head_count", cfg.num_heads),
        _kv_u32(f"{arch}.attention.head_count_kv", cfg.num_kv_heads),
        _kv_u32(f"{arch}.feed_forward_length", cfg.intermediate_size),
        _kv_u32(f"{arch}.context_length", cfg.context_length),
        _kv_f32(f"{arch}.attention.layer_norm_rms_epsilon", cfg.rms_norm_eps),
        _kv_f32(f"{arch}.rope.freq_base", cfg.rope_theta),
        _kv_u32("general.alignment", ALIGN),
    ]
    for k, v in (extra_kv or {}).items():
        kvs.append(_kv_u32(k, v) if isinstance(v, int) else _kv_f32(k, v))
    infos = []
    offset = 0
    offsets = []
    for name, ne, t in plan:
        offsets.append(offset)
        info = _s(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
        info += struct.pack("<IQ", t, offset)
        infos.append(info)
        nbytes = _tensor_nbytes(ne, t)
        offset += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    header = b"GGUF" + struct.pack("<IQQ", 3, len(plan), len(kvs)) + b"".join(kvs) + b"".join(infos)
    pad = (-len(header)) % ALIGN
    tmp = path + ".tmp"
    cache = {}  # layer_period: (layer % period, tensor) -> bytes of its first occurrence
    with open(tmp, "wb") as f:
        f.write(header + b"\0" * pad)
        for index, ((name, ne, t), off) in enumerate(zip(plan, offsets)):
            key = None
            if cfg.layer_period > 0 and name.startswith("blk."):
                layer, rest = name[4:].split(".", 1)
                key = (int(layer) % cfg.layer_period, rest)
            if key is None:
                data = _gen_tensor(index, name, ne, t, cfg)
            else:
                if key not in cache:
                    cache[key] = _gen_tensor(index, name, ne, t, cfg)
                data = cache[key]
            f.write(data)
            f.write(b"\0" * ((-len(data)) % ALIGN))
    os.replace(tmp, path)
    return path


def make_model(preset_or_cfg, path: str, **overrides) -> str:
    """Write the named preset (optionally with field overrides) to ``path``."""
    cfg = preset_or_cfg
    if isinstance(cfg, str):
        cfg = PRESETS[cfg]
    cfg = dataclasses.replace(cfg, **overrides)
    return write_gguf(path, cfg)


def cached_model(preset: str, directory: str, **overrides) -> str:
    """Return a GGUF path for ``preset`` under ``directory``, writing it once."""
    cfg = dataclasses.replace(PRESETS[preset], **overrides)
    tag = "_".join(f"{k}{v}" for k, v in sorted(overrides.items()))
    path = os.path.join(directory, f"wcb_{preset}{'_' + tag if tag else ''}.gguf")
    if not os.path.exists(path):
        os.makedirs(directory, exist_ok=True)
        write_gguf(path, cfg)
    return path


def random_prompt(n: int, vocab: int, seed: int = 1) -> np.ndarray:
    """Uniform random prompt ids in [3, vocab) (ids 0-2 are BOS/EOS/UNK by convention)."""
    rng = np.random.default_rng(seed)
    return rng.integers(3, vocab, size=n, dtype=np.int64).astype(np.uint32)
