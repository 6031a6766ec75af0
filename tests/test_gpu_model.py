"""Model-level parity through the C ABI: forward logits within max-abs 1e-2 and
relative 1e-3 of the oracle, greedy generate() sequences identical, and the
reference's edge semantics (first token without EOS check, KV overflow error,
forward at a position different from the KV length)."""
import os

import numpy as np
import pytest

import oracle
import wcb
from wcb import synth

pytestmark = pytest.mark.gpu

ABS_TOL = 1e-2
REL_TOL = 1e-3


def assert_logits_close(got, ref):
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64)).max()
    scale = np.abs(ref).max()
    assert err <= ABS_TOL, f"max abs err {err}"
    assert err <= REL_TOL * scale, f"rel err {err / scale}"


@pytest.fixture(scope="module")
def tiny_pair(tiny_gguf, gpu):
    oracle.set_threads(os.cpu_count() or 1, os.cpu_count() or 1)
    return wcb.Model.load_from_gguf(tiny_gguf), oracle.OracleModel(tiny_gguf)


def test_config_matches_gguf(tiny_pair):
    m, o = tiny_pair
    c = m.config
    assert (c.vocab_size, c.hidden_size, c.num_layers, c.num_heads, c.num_kv_heads, c.intermediate_size) == \
        (o.vocab, o.hidden, o.layers, o.heads, o.kv_heads, o.ffn)
    assert c.max_seq_len == 256 and c.head_dim == 64


def test_forward_prefill_and_decode_logits(tiny_pair):
    m, o = tiny_pair
    m.clear_kv_cache()
    o.clear_kv_cache()
    prompt = synth.random_prompt(20, 512, seed=2).tolist()
    assert_logits_close(m.forward(prompt, 0), o.forward(prompt, 0))
    for i, t in enumerate([7, 300, 5, 511, 42]):
        assert_logits_close(m.forward([t], 20 + i), o.forward([t], 20 + i))
    assert m.kv_len() == o.kv_len() == 25


def test_forward_chunked_prefill_matches(tiny_pair):
    m, o = tiny_pair
    m.clear_kv_cache()
    o.clear_kv_cache()
    prompt = synth.random_prompt(40, 512, seed=4).tolist()
    for c in range(0, 40, 8):  # generate()'s 8-token chunks (model.rs:1363-1371)
        got = m.forward(prompt[c:c + 8], c)
        ref = o.forward(prompt[c:c + 8], c)
    assert_logits_close(got, ref)


def test_forward_position_differs_from_kv_len(tiny_pair):
    # the KV append uses the cache length, RoPE and the mask use `position`
    m, o = tiny_pair
    m.clear_kv_cache()
    o.clear_kv_cache()
    m.forward([10, 11, 12], 0)
    o.forward([10, 11, 12], 0)
    assert_logits_close(m.forward([13, 14], 7), o.forward([13, 14], 7))
    assert_logits_close(m.forward([15], 1), o.forward([15], 1))


def test_out_of_vocab_token_embeds_zero(tiny_pair):
    m, o = tiny_pair
    m.clear_kv_cache()
    o.clear_kv_cache()
    assert_logits_close(m.forward([3, 600, 9], 0), o.forward([3, 600, 9], 0))


def test_kv_overflow_is_model_parse_error(tiny_pair):
    m, _ = tiny_pair
    m.clear_kv_cache()
    m.forward(list(range(3, 253)), 0)
    with pytest.raises(wcb.WcbError) as e:
        m.forward(list(range(3, 13)), 250)
    assert e.value.code == 4 and "overflow" in e.value.message
    assert m.kv_len() == 250
    with pytest.raises(wcb.WcbError) as e:
        m.forward([], 0)
    assert e.value.code == 3


@pytest.mark.parametrize("rep", [1.0, 1.1])
def test_greedy_generate_identical(tiny_pair, rep):
    m, o = tiny_pair
    prompt = synth.random_prompt(24, 512, seed=8).tolist()
    cfg = wcb.GenerationConfig(max_tokens=64, temperature=0.0, repetition_penalty=rep, eos_id=None)
    got = m.generate_tokens(prompt, cfg)
    ref = o.generate(prompt, 64, repetition_penalty=rep, eos_id=None)
    assert got == ref
    assert len(got) == 64 and m.kv_len() == 24 + 63


def test_greedy_generate_edge_semantics(tiny_pair):
    m, o = tiny_pair
    prompt = synth.random_prompt(9, 512, seed=12).tolist()
    base = o.generate(prompt, 12, eos_id=None)
    for mt in (0, 1, 2):
        assert m.generate_tokens(prompt, wcb.GenerationConfig(max_tokens=mt, temperature=0.0,
                                                              repetition_penalty=1.0, eos_id=None)) == base[:max(mt, 1)]
    for eos in (base[0], base[4]):
        cfg = wcb.GenerationConfig(max_tokens=12, temperature=0.0, repetition_penalty=1.0, eos_id=eos)
        assert m.generate_tokens(prompt, cfg) == o.generate(prompt, 12, eos_id=eos)
    with pytest.raises(wcb.WcbError) as e:
        m.generate_tokens([], wcb.GenerationConfig(max_tokens=4, temperature=0.0))
    assert e.value.code == 4


def test_generate_runs_into_kv_overflow(tiny_pair):
    m, o = tiny_pair
    prompt = synth.random_prompt(250, 512, seed=13).tolist()
    with pytest.raises(wcb.WcbError) as e:
        m.generate_tokens(prompt, wcb.GenerationConfig(max_tokens=20, temperature=0.0, repetition_penalty=1.0,
                                                       eos_id=None))
    assert e.value.code == 4
    with pytest.raises(oracle.OracleError) as e2:
        o.generate(prompt, 20, eos_id=None)
    assert e2.value.code == 4


def test_generate_without_graphs_matches(tiny_gguf, tiny_pair):
    _, o = tiny_pair
    m2 = wcb.Model.load_from_gguf(tiny_gguf, use_graphs=False)
    prompt = synth.random_prompt(16, 512, seed=14).tolist()
    cfg = wcb.GenerationConfig(max_tokens=20, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    assert m2.generate_tokens(prompt, cfg) == o.generate(prompt, 20, repetition_penalty=1.1, eos_id=None)
    m2.close()


def test_sampled_generate_is_seeded(tiny_pair):
    m, _ = tiny_pair
    prompt = synth.random_prompt(10, 512, seed=15).tolist()
    cfg = wcb.GenerationConfig(max_tokens=16, temperature=0.8, top_p=0.9, top_k=40, repetition_penalty=1.1,
                               seed=7, eos_id=None)
    a = m.generate_tokens(prompt, cfg)
    b = m.generate_tokens(prompt, cfg)
    assert a == b and len(a) == 16 and all(0 <= t < 512 for t in a)


def test_generate_batch_matches_single(tiny_pair):
    m, _ = tiny_pair
    prompts = [synth.random_prompt(n, 512, seed=20 + n).tolist() for n in (5, 17, 33)]
    cfg = wcb.GenerationConfig(max_tokens=10, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    assert m.generate_batch(prompts, cfg) == [m.generate_tokens(p, cfg) for p in prompts]


def test_q6k_mix_mha_model(tiny_mix_gguf, gpu):
    m = wcb.Model.load_from_gguf(tiny_mix_gguf)
    o = oracle.OracleModel(tiny_mix_gguf)
    prompt = synth.random_prompt(30, 768, seed=3).tolist()
    assert_logits_close(m.forward(prompt, 0), o.forward(prompt, 0))
    assert_logits_close(m.forward([77], 30), o.forward([77], 30))
    cfg = wcb.GenerationConfig(max_tokens=32, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    assert m.generate_tokens(prompt, cfg) == o.generate(prompt, 32, repetition_penalty=1.1, eos_id=None)
    m.close()


def test_f16_kv_cache_close(tiny_gguf, gpu):
    m = wcb.Model.load_from_gguf(tiny_gguf, kv_dtype=wcb.KV_F16)
    o = oracle.OracleModel(tiny_gguf)
    prompt = synth.random_prompt(40, 512, seed=6).tolist()
    got, ref = m.forward(prompt, 0), o.forward(prompt, 0)
    assert np.abs(got - ref).max() <= 5e-2 * np.abs(ref).max()
    m.close()


@pytest.mark.slow
def test_tinyllama_64_greedy_tokens_identical(model_dir, gpu):
    """TinyLlama-1.1B architecture, 128-token random prompt: first 64 greedy tokens
    identical to the oracle, logits of the prefill within tolerance."""
    path = synth.cached_model("tinyllama", model_dir)
    oracle.set_threads(os.cpu_count() or 1, os.cpu_count() or 1)
    m = wcb.Model.load_from_gguf(path)
    o = oracle.OracleModel(path)
    prompt = synth.random_prompt(128, 32000, seed=1).tolist()
    assert_logits_close(m.forward(prompt, 0), o.forward(prompt, 0))
    cfg = wcb.GenerationConfig(max_tokens=64, temperature=0.0, repetition_penalty=1.0, eos_id=2)
    ref, steps = o.generate(prompt, 64, repetition_penalty=1.0, eos_id=2, return_logits=True)
    got = m.generate_tokens(prompt, cfg)
    gaps = []
    for row in steps[: len(ref)]:
        top2 = np.partition(row, -2)[-2:]
        gaps.append(float(top2[1] - top2[0]))
    assert got == ref, f"first mismatch at {next(i for i, (a, b) in enumerate(zip(got, ref)) if a != b)}; " \
                       f"smallest top-1/top-2 gap {min(gaps):.3g}"
    m.close()


def test_stream_api_matches_generate(tiny_pair):
    m, o = tiny_pair
    prompt = synth.random_prompt(18, 512, seed=30).tolist()
    cfg = wcb.GenerationConfig(max_tokens=25, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    ref = o.generate(prompt, 25, repetition_penalty=1.1, eos_id=None)
    s = m.infer(prompt, cfg)
    got = []
    for chunk in (1, 3, 7, 100):
        got += s.next_tokens(chunk)
    assert got == ref and s.finished
    assert s.next_tokens(4) == []
    s2 = m.infer(prompt, cfg)
    one = []
    while True:
        t = s2.next_token()
        if t is None:
            break
        one.append(t)
    assert one == ref
    with pytest.raises(wcb.WcbError):  # a newer generation on the model invalidates the old stream
        s.next_tokens(1)
    s.close()
    s2.close()


def test_stream_api_stops_at_eos(tiny_pair):
    m, o = tiny_pair
    prompt = synth.random_prompt(11, 512, seed=31).tolist()
    base = o.generate(prompt, 20, eos_id=None)
    cfg = wcb.GenerationConfig(max_tokens=20, temperature=0.0, repetition_penalty=1.0, eos_id=base[5])
    s = m.infer(prompt, cfg)
    got = s.next_tokens(50)
    assert got == o.generate(prompt, 20, eos_id=base[5]) and s.finished


def test_prefill_gemv_and_tensor_core_paths(tiny_gguf, tiny_pair):
    """Prompts of >= 16 tokens run the tcgen05 GEMM; the GEMV-only model (and the
    model without programmatic dependent launch) must agree with the oracle too."""
    _, o = tiny_pair
    prompt = synth.random_prompt(70, 512, seed=40).tolist()
    o.clear_kv_cache()
    ref = o.forward(prompt, 0)
    for kw in ({}, {"use_tensor_cores": False}, {"use_pdl": False}):
        m = wcb.Model.load_from_gguf(tiny_gguf, **kw)
        assert_logits_close(m.forward(prompt, 0), ref)
        cfg = wcb.GenerationConfig(max_tokens=12, temperature=0.0, repetition_penalty=1.1, eos_id=None)
        assert m.generate_tokens(prompt, cfg) == o.generate(prompt, 12, repetition_penalty=1.1, eos_id=None)
        m.close()
