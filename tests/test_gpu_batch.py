"""Batched serving through wcb_generate_batch: sequences prefilled into their
own KV slots, then decoded together with the tensor-core step (weights read once
per step for all sequences). Each sequence's greedy tokens must equal the
oracle's generate() on that prompt (model.rs:1322-1415): ragged prompts,
repetition penalty, EOS inside the batch, more sequences than slots, KV
overflow, a Q4_K_M (Q6_K) model, and the fp16 KV cache."""
import os

import pytest

import oracle
import wcb
from wcb import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_batch(tiny_gguf, gpu):
    oracle.set_threads(os.cpu_count() or 1, os.cpu_count() or 1)
    m = wcb.Model.load_from_gguf(tiny_gguf, max_batch=8)
    yield m, oracle.OracleModel(tiny_gguf)
    m.close()


def prompts_of(lengths, vocab, seed):
    return [synth.random_prompt(n, vocab, seed=seed + i).tolist() for i, n in enumerate(lengths)]


def test_batch_slots(tiny_batch):
    m, _ = tiny_batch
    assert m.batch_info()[0] == 8


@pytest.mark.parametrize("rep", [1.0, 1.1])
def test_batch_matches_oracle(tiny_batch, rep):
    m, o = tiny_batch
    prompts = prompts_of([5, 17, 33, 64, 9, 120, 2, 48], 512, seed=40)
    cfg = wcb.GenerationConfig(max_tokens=64, temperature=0.0, repetition_penalty=rep, eos_id=None)
    got = m.generate_batch(prompts, cfg)
    slots, launches = m.batch_info()
    assert slots == 8 and launches == 1 + 5 * 2 + 1 + 1  # embed, 5 per layer, LM head, sampler
    for p, g in zip(prompts, got):
        assert g == o.generate(p, 64, repetition_penalty=rep, eos_id=None)


def test_batch_groups_eos_and_single_equivalence(tiny_batch):
    m, _ = tiny_batch
    prompts = prompts_of([7, 30, 12, 3, 25, 40, 18, 9, 60, 11, 4], 512, seed=70)  # 11 > 8 slots: two groups
    free = wcb.GenerationConfig(max_tokens=24, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    singles = [m.generate_tokens(p, free) for p in prompts]
    eos = singles[2][6]  # ends sequence 2 early, and any other that emits it after its first token
    cfg = wcb.GenerationConfig(max_tokens=24, temperature=0.0, repetition_penalty=1.1, eos_id=eos)
    want = [m.generate_tokens(p, cfg) for p in prompts]
    got = m.generate_batch(prompts, cfg)
    assert got == want
    assert len(got[2]) < 24
    for n in (1, 2):  # max_tokens 1: the prefill token only
        c = wcb.GenerationConfig(max_tokens=n, temperature=0.0, repetition_penalty=1.0, eos_id=None)
        assert m.generate_batch(prompts[:3], c) == [m.generate_tokens(p, c) for p in prompts[:3]]


def test_batch_kv_overflow(tiny_batch):
    m, _ = tiny_batch
    prompts = prompts_of([10, 250], 512, seed=90)  # context 256: the second overflows
    cfg = wcb.GenerationConfig(max_tokens=20, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    with pytest.raises(wcb.WcbError):
        m.generate_tokens(prompts[1], cfg)
    with pytest.raises(wcb.WcbError):
        m.generate_batch(prompts, cfg)
    # the model stays usable
    ok = prompts_of([6, 8], 512, seed=95)
    assert m.generate_batch(ok, cfg) == [m.generate_tokens(p, cfg) for p in ok]


def test_batch_q6k_mix(tiny_mix_gguf, gpu):
    m = wcb.Model.load_from_gguf(tiny_mix_gguf, max_batch=4)
    o = oracle.OracleModel(tiny_mix_gguf)
    prompts = prompts_of([30, 7, 50, 19], 768, seed=11)
    cfg = wcb.GenerationConfig(max_tokens=32, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    got = m.generate_batch(prompts, cfg)
    for p, g in zip(prompts, got):
        assert g == o.generate(p, 32, repetition_penalty=1.1, eos_id=None)
    m.close()


def test_batch_f16_kv(tiny_gguf, gpu):
    m = wcb.Model.load_from_gguf(tiny_gguf, kv_dtype=wcb.KV_F16, max_batch=4)
    o = oracle.OracleModel(tiny_gguf)
    prompts = prompts_of([40, 13, 26, 8], 512, seed=120)
    cfg = wcb.GenerationConfig(max_tokens=16, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    got = m.generate_batch(prompts, cfg)
    for p, g in zip(prompts, got):
        assert g == o.generate(p, 16, repetition_penalty=1.0, eos_id=None)
    m.close()


def test_batch_sampled_on_the_device(tiny_batch):
    """Sampled configs run the batched step too, with one device sampler per slot (its
    own history, penalty counts and random stream, started from the config's seed as a
    sequence's own generate() starts). Keeping only the most probable token (top_k 1, or
    a vanishing top_p through the full-vocabulary sampler) reproduces the greedy batch,
    which is checked against the oracle above; real sampling is deterministic for a seed,
    and identical prompts in different slots draw identical tokens."""
    m, _ = tiny_batch
    prompts = prompts_of([9, 31, 4, 17, 50, 12], 512, seed=90)
    greedy = m.generate_batch(prompts, wcb.GenerationConfig(max_tokens=32, temperature=0.0, repetition_penalty=1.1,
                                                           eos_id=None))
    for k, p in ((1, 1.0), (0, 1e-6)):
        c = wcb.GenerationConfig(max_tokens=32, temperature=0.8, top_k=k, top_p=p, repetition_penalty=1.1, seed=3,
                                 eos_id=None)
        assert m.generate_batch(prompts, c) == greedy, (k, p)
        assert m.batch_info()[1] == 1 + 5 * 2 + 1 + 1  # the batched step ran, its sampler in place
    batch = prompts + [prompts[0], prompts[0]]  # 8 sequences: one batched group
    for k, p in ((40, 0.9), (0, 0.9)):
        c = wcb.GenerationConfig(max_tokens=32, temperature=0.8, top_k=k, top_p=p, repetition_penalty=1.1, seed=5,
                                 eos_id=None)
        a = m.generate_batch(batch, c)
        assert a == m.generate_batch(batch, c)
        assert a[0] == a[-1] == a[-2]
        assert all(len(x) == 32 and all(0 <= t < 512 for t in x) for x in a)
        assert any(x != g for x, g in zip(a, greedy))
