"""CPU checks of the synthetic-model generator and of the C ABI library that
need no GPU: symbol exports, error codes and the host sampler."""
import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

import wcb
from wcb import synth

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_fast_quantizers_match_numpy():
    x = synth.normal(7, 3, 256 * 200, 0.0, 0.02)
    assert np.array_equal(synth.quantize_q4_k_fast(x), synth.quantize_q4_k(x))
    assert np.array_equal(synth.quantize_q6_k_fast(x), synth.quantize_q6_k(x))


def test_normal_generator_is_deterministic_and_normal():
    a = synth.normal(0, 5, 100001, 0.0, 1.0)
    b = synth.normal(0, 5, 100001, 0.0, 1.0)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1.0) < 0.02
    assert not np.array_equal(a[:1000], synth.normal(0, 6, 1000, 0.0, 1.0))


def test_gguf_file_reads_back_with_gguf_py(tiny_mix_gguf):
    from gguf import GGUFReader
    r = GGUFReader(tiny_mix_gguf)
    names = {t.name: t for t in r.tensors}
    cfg = synth.PRESETS["tiny_mix"]
    plan = synth.tensor_plan(cfg)
    assert [p[0] for p in plan] == [t.name for t in r.tensors]
    for name, ne, ty in plan:
        t = names[name]
        assert int(t.tensor_type) == ty
        assert tuple(int(d) for d in t.shape) == tuple(ne)
    assert int(names["blk.0.attn_v.weight"].tensor_type) == synth.GGML_Q6_K
    assert int(names["blk.1.attn_v.weight"].tensor_type) == synth.GGML_Q4_K
    f = r.fields["llama.context_length"]
    assert int(f.parts[f.data[0]][0]) == cfg.context_length


def test_layer_period_repeats_layer_bytes(tmp_path):
    """Deep timing models (the 80-layer 70B shape) repeat a period of layers: every
    tensor of layer i holds the bytes of layer i % period, the rest stay distinct, and
    the file reads back like any other."""
    from gguf import GGUFReader
    path = synth.make_model("tiny", str(tmp_path / "p.gguf"), num_layers=5, layer_period=2)
    t = {x.name: np.array(x.data).tobytes() for x in GGUFReader(path).tensors}
    for name in ("attn_q.weight", "attn_norm.weight", "ffn_down.weight"):
        assert t[f"blk.4.{name}"] == t[f"blk.2.{name}"] == t[f"blk.0.{name}"]
        assert t[f"blk.3.{name}"] == t[f"blk.1.{name}"]
        assert t[f"blk.1.{name}"] != t[f"blk.0.{name}"]
    plain = synth.make_model("tiny", str(tmp_path / "q.gguf"), num_layers=5)
    t2 = {x.name: np.array(x.data).tobytes() for x in GGUFReader(plain).tensors}
    assert t2["blk.0.attn_q.weight"] == t["blk.0.attn_q.weight"]  # the period keeps layer 0's stream
    assert t2["blk.2.attn_q.weight"] != t2["blk.0.attn_q.weight"]


def _declared_symbols():
    hdr = open(os.path.join(REPO, "include", "wcb.h")).read()
    return sorted(set(re.findall(r"\b(wcb_[a-z0-9_]+)\s*\(", hdr)))


def test_library_exports_every_declared_symbol():
    L = wcb.lib()
    declared = _declared_symbols()
    assert len(declared) >= 18
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) == set(wcb.EXPORTED)


def test_version_and_defaults():
    assert wcb.version().startswith("wcb-")
    c = wcb._GenConfig()
    wcb.lib().wcb_gen_config_default(C.byref(c))
    assert (c.max_tokens, c.top_k, c.seed, c.eos_id) == (100, 40, 42, 2)
    assert abs(c.temperature - 0.7) < 1e-7 and abs(c.top_p - 0.9) < 1e-7
    assert abs(c.repetition_penalty - 1.1) < 1e-7


def test_load_errors_without_touching_the_gpu(tmp_path):
    with pytest.raises(wcb.WcbError) as e:
        wcb.Model.load_from_gguf(str(tmp_path / "missing.gguf"))
    assert e.value.code == 7  # IoError
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + b"\0" * 64)
    with pytest.raises(wcb.WcbError) as e:
        wcb.Model.load_from_gguf(str(bad))
    assert e.value.code == 4 and "magic" in e.value.message
    v9 = tmp_path / "v9.gguf"
    v9.write_bytes(b"GGUF" + struct.pack("<IQQ", 9, 0, 0))
    with pytest.raises(wcb.WcbError) as e:
        wcb.Model.load_from_gguf(str(v9))
    assert e.value.code == 4 and "version" in e.value.message


@pytest.mark.parametrize("overrides,code,words", [
    (dict(hidden_size=768, num_heads=8, num_kv_heads=2), 5, "head_dim must be 64 or 128"),
    (dict(vocab_size=510), 5, "multiple of 4"),
    (dict(hidden_size=2048, num_heads=32, num_kv_heads=1), 5, "more than 16 query heads"),
    (dict(hidden_size=384, num_heads=6, num_kv_heads=4), 3, "inconsistent"),
    (dict(intermediate_size=300), 5, "multiples of 256"),
    (dict(hidden_size=320, num_heads=5, num_kv_heads=5), 5, "multiples of 256"),
])
def test_unsupported_shapes_are_refused_before_any_device_work(tmp_path, overrides, code, words):
    """Shapes the kernels do not cover (head_dim other than 64 / 128, hidden or FFN
    sizes off the 256-value Q4_K block, a vocabulary not a multiple of 4, more than 16
    query heads per KV head) and inconsistent head counts are refused from the GGUF
    header alone, with the reference's error codes, before any GPU call."""
    import dataclasses
    cfg = dataclasses.replace(synth.PRESETS["tiny"], **overrides)
    path = synth.write_gguf(str(tmp_path / "m.gguf"), cfg,
                            plan=[("token_embd.weight", (cfg.hidden_size, cfg.vocab_size), synth.GGML_F32)])
    with pytest.raises(wcb.WcbError) as e:
        wcb.Model.load_from_gguf(path)
    assert e.value.code == code and words in e.value.message


def test_last_error_is_taken_once():
    L = wcb.lib()
    h = C.c_uint32(0)
    assert L.wcb_model_load(b"/nonexistent/x.gguf", None, C.byref(h)) == 7
    assert h.value == 0
    assert "cannot open" in wcb.last_error()
    assert wcb.last_error() == "No error"


def test_gemv_argument_errors_without_touching_the_gpu():
    # wcb_gemv_dev validates dtype, pointers, shape and 16-byte alignment on the host,
    # before any CUDA call; the addresses below are never dereferenced
    cases = [
        (4096, 99, 4, 256, 4096, 1),        # unsupported dtype
        (0, wcb.DTYPE_Q4_K, 4, 256, 4096, 1),  # null weights
        (4096, wcb.DTYPE_Q4_K, 4, 100, 4096, 1),  # k % 256 != 0
        (4096, wcb.DTYPE_Q4_K, 6, 256, 4096, 1),  # n % 4 != 0
        (4096, wcb.DTYPE_Q4_K, 4, 256, 4096, 4097),  # m > 4096
        (4096, wcb.DTYPE_Q4_K, 4, 256, 4096 + 4, 8),  # x off a 16-byte boundary
        (4096 + 8, wcb.DTYPE_Q4_K, 4, 256, 4096, 1),  # W off a 16-byte boundary
    ]
    for w, dt, n, k, x, m in cases:
        with pytest.raises(wcb.WcbError) as e:
            wcb.gemv_dev(w, dt, n, k, x, m, 8192)
        assert e.value.code == 3, (w, dt, n, k, x, m)


def test_invalid_handles():
    L = wcb.lib()
    assert L.wcb_model_free(12345) == 3
    n = C.c_size_t(0)
    assert L.wcb_kv_len(12345, C.byref(n)) == 3


def test_host_sampler_matches_oracle_argmax_and_penalty():
    import oracle
    rng = np.random.default_rng(11)
    s_w = wcb.LogitsProcessor(42, 0.0, 0.9, 40, 1.3)
    s_o = oracle.Sampler(42, 0.0, 0.9, 40, 1.3)
    for _ in range(30):
        l = rng.standard_normal(300).astype(np.float32)
        l[rng.integers(0, 300)] = l.max()  # a tie
        a, b = l.copy(), l.copy()
        assert s_w.sample(a) == s_o.sample(b)
        assert np.array_equal(a, b)


def test_host_sampler_nan_is_generic_failure():
    s = wcb.LogitsProcessor(42, 0.0, 0.9, 40, 1.0)
    with pytest.raises(wcb.WcbError) as e:
        s.sample(np.array([0.0, np.nan], np.float32))
    assert e.value.code == 1


def test_struct_layouts_match_the_library():
    # every ctypes mirror has the library's size and field offsets
    wcb.check_layouts()
    L = wcb.lib()
    assert L.wcb_struct_layout(b"wcb_load_opts", b"tp_id") + 128 == 160  # WCB_LOAD_OPTS_V1_SIZE
    assert L.wcb_struct_layout(b"wcb_load_opts", b"wait_ms") == 160
    assert L.wcb_struct_layout(b"wcb_load_opts", b"no_such_field") == C.c_size_t(-1).value
    assert L.wcb_struct_layout(b"no_such_struct", None) == C.c_size_t(-1).value


def test_load_opts_init_and_struct_size_checks():
    L = wcb.lib()
    o = wcb._LoadOpts()
    L.wcb_load_opts_init(C.byref(o))
    assert (o.struct_size, o.max_batch, o.tp_size, o.wait_ms, o.device) == (C.sizeof(wcb._LoadOpts), 1, 1, 2000, 0)
    h = C.c_uint32(0)
    # a zero struct_size (options never initialised) is refused before any file or GPU access
    z = wcb._LoadOpts()
    assert L.wcb_model_load(b"/nonexistent/x.gguf", C.byref(z), C.byref(h)) == 3
    assert "struct_size" in wcb.last_error()
    # an older caller's shorter struct (no wait_ms) is accepted: the next failure is the missing file
    o.struct_size = 160
    o.wait_ms = 0xDEAD  # past struct_size: never read
    assert L.wcb_model_load(b"/nonexistent/x.gguf", C.byref(o), C.byref(h)) == 7
    o.struct_size = C.sizeof(wcb._LoadOpts)
    o.wait_ms = 60001
    assert L.wcb_model_load(b"/nonexistent/x.gguf", C.byref(o), C.byref(h)) == 3
    assert "wait_ms" in wcb.last_error()


@pytest.mark.parametrize("entry", ["wcb_attention_dev", "wcb_attention_dev_noalloc"])
def test_attention_argument_errors_without_touching_the_gpu(entry):
    # both attention entry points validate pointers, alignment and shapes on the host
    # before any CUDA call; the addresses below are never dereferenced
    f = getattr(wcb.lib(), entry)
    base = 1 << 20
    ok = dict(q=base, k=base + 4096, v=base + 8192, out=base + 12288)
    cases = [
        dict(ok, q=0),
        dict(ok, q=base + 4),          # q off a 16-byte boundary
        dict(ok, k=base + 4096 + 8),   # K cache
        dict(ok, v=base + 8192 + 12),  # V cache
        dict(ok, out=base + 12288 + 4),
    ]
    for c in cases:
        assert f(c["q"], c["k"], c["v"], c["out"], 1, 8, 2, 64, 128, 16, 15, None) == 3, c
    assert "aligned" in wcb.last_error() or "null" in wcb.last_error()
    # shape errors: head_dim 96, kv_len > max_seq, n_heads not a multiple of n_kv_heads
    for args in [(1, 8, 2, 96, 128, 16, 15), (1, 8, 2, 64, 128, 129, 128), (1, 6, 4, 64, 128, 16, 15)]:
        assert f(ok["q"], ok["k"], ok["v"], ok["out"], *args, None) == 3, args
