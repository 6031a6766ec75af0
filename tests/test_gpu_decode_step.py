"""The persistent decode step (one cooperative launch per token) against the
per-op kernels (one launch per projection / attention / LM head) and the
oracle: greedy tokens identical, one-token forward logits within fp32
summation-order noise, long contexts whose attention splits span several key
tiles, Q4_K_M mixes and an f16 KV cache."""
import numpy as np
import pytest

import oracle
import wcb
from wcb import synth

pytestmark = pytest.mark.gpu


def _pair(path, **kw):
    return (wcb.Model.load_from_gguf(path, **kw),
            wcb.Model.load_from_gguf(path, use_persistent=False, **kw))


def _close(a, b, rel=1e-4):
    err = np.abs(a.astype(np.float64) - b.astype(np.float64)).max()
    assert err <= rel * np.abs(b).max(), f"max abs err {err}"


def test_one_launch_per_decode_step(tiny_gguf, gpu):
    p, q = _pair(tiny_gguf)
    prompt = synth.random_prompt(12, 512, seed=30).tolist()
    cfg = wcb.GenerationConfig(max_tokens=8, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    p.generate_tokens(prompt, cfg)
    q.generate_tokens(prompt, cfg)
    assert p.launches_per_step() == 1
    assert q.launches_per_step() > 1
    p.close()
    q.close()


@pytest.mark.parametrize("rep", [1.0, 1.1])
def test_tokens_match_oracle_and_per_op(tiny_gguf, gpu, rep):
    p, q = _pair(tiny_gguf)
    o = oracle.OracleModel(tiny_gguf)
    prompt = synth.random_prompt(33, 512, seed=31).tolist()
    cfg = wcb.GenerationConfig(max_tokens=48, temperature=0.0, repetition_penalty=rep, eos_id=None)
    got = p.generate_tokens(prompt, cfg)
    assert got == q.generate_tokens(prompt, cfg)
    assert got == o.generate(prompt, 48, repetition_penalty=rep, eos_id=None)
    p.close()
    q.close()


def test_forward_one_token_logits(tiny_gguf, gpu):
    p, q = _pair(tiny_gguf)
    o = oracle.OracleModel(tiny_gguf)
    prompt = synth.random_prompt(50, 512, seed=32).tolist()
    for m in (p, q, o):
        m.forward(prompt, 0)
    for i, t in enumerate([3, 511, 600, 42]):  # 600 is out of vocabulary: zero embedding
        a, b, r = p.forward([t], 50 + i), q.forward([t], 50 + i), o.forward([t], 50 + i)
        _close(a, b)
        assert np.abs(a - r).max() <= 1e-3 * np.abs(r).max()
    # a forward at a position below the KV length (the reference allows it)
    _close(p.forward([9], 20), q.forward([9], 20))
    p.close()
    q.close()


def test_q4_k_m_mix(tiny_mix_gguf, gpu):
    p, q = _pair(tiny_mix_gguf)
    o = oracle.OracleModel(tiny_mix_gguf)
    prompt = synth.random_prompt(40, 768, seed=33).tolist()
    cfg = wcb.GenerationConfig(max_tokens=40, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    got = p.generate_tokens(prompt, cfg)
    assert got == q.generate_tokens(prompt, cfg)
    assert got == o.generate(prompt, 40, repetition_penalty=1.1, eos_id=None)
    p.close()
    q.close()


def test_f16_kv_cache(tiny_gguf, gpu):
    p, q = _pair(tiny_gguf, kv_dtype=wcb.KV_F16)
    prompt = synth.random_prompt(60, 512, seed=34).tolist()
    for m in (p, q):
        m.forward(prompt, 0)
    for i, t in enumerate([5, 77, 200]):
        _close(p.forward([t], 60 + i), q.forward([t], 60 + i))
    p.close()
    q.close()


@pytest.mark.slow
def test_tinyllama_long_context(model_dir, gpu):
    """1500-token prompt: each attention item covers several 32-key tiles."""
    path = synth.cached_model("tinyllama", model_dir)
    p, q = _pair(path)
    prompt = synth.random_prompt(1500, 32000, seed=35).tolist()
    cfg = wcb.GenerationConfig(max_tokens=24, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    assert p.generate_tokens(prompt, cfg) == q.generate_tokens(prompt, cfg)
    for m in (p, q):
        m.clear_kv_cache()
        m.forward(prompt, 0)
    _close(p.forward([123], 1500), q.forward([123], 1500))
    p.close()
    q.close()


@pytest.mark.parametrize("kv", [wcb.KV_F32, wcb.KV_F16])
def test_split_attention_matches_oracle(model_dir, gpu, kv):
    """A 700-token context: each query head's attention runs as several key
    splits (2 with an f16 cache, 3 with f32), merged by the O-projection phase;
    greedy tokens equal the oracle's (f32 cache) and the per-op kernels', and
    one-token logits agree, also at a position below the KV length."""
    path = synth.cached_model("tiny", model_dir, context_length=2048)
    p, q = _pair(path, kv_dtype=kv)
    prompt = synth.random_prompt(700, 512, seed=36).tolist()
    cfg = wcb.GenerationConfig(max_tokens=20, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    got = p.generate_tokens(prompt, cfg)
    assert got == q.generate_tokens(prompt, cfg)
    assert p.launches_per_step() == 1
    if kv == wcb.KV_F32:
        o = oracle.OracleModel(path)
        assert got == o.generate(prompt, 20, repetition_penalty=1.1, eos_id=None)
    for m in (p, q):
        m.clear_kv_cache()
        m.forward(prompt, 0)
    for i, t in enumerate([17, 300]):
        _close(p.forward([t], 700 + i), q.forward([t], 700 + i))
    _close(p.forward([9], 250), q.forward([9], 250))
    p.close()
    q.close()


def test_bounded_tag_wait_expires_into_an_error(tiny_gguf, gpu, monkeypatch):
    """The persistent step's waits for other CTAs' data are bounded: with the outputs
    of one phase withheld (a test hook: phase 3, layer 0's gate/up) and wait_ms = 200,
    their consumers' waits run out and generate fails with BackendUnsupported naming
    the expired wait within seconds, instead of hanging or returning tokens; with the
    hook removed the same model generates the oracle's tokens again."""
    import time
    m = wcb.Model.load_from_gguf(tiny_gguf, wait_ms=200)
    o = oracle.OracleModel(tiny_gguf)
    prompt = synth.random_prompt(20, 512, seed=37).tolist()
    cfg = wcb.GenerationConfig(max_tokens=8, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    monkeypatch.setenv("WCB_TEST_DROP_PHASE", "3")
    t0 = time.time()
    with pytest.raises(wcb.WcbError) as e:
        m.generate_tokens(prompt, cfg)
    assert e.value.code == 5 and "bounded wait expired" in e.value.message, e.value.message
    assert time.time() - t0 < 10.0
    monkeypatch.delenv("WCB_TEST_DROP_PHASE")
    assert m.generate_tokens(prompt, cfg) == o.generate(prompt, 8, repetition_penalty=1.0, eos_id=None)
    assert m.launches_per_step() == 1
    m.close()
