"""Sampled decoding (LogitsProcessor::sample, sampling.rs:106-229). The
reference's rand StdRng stream is not reproduced, so sampled token sequences
are checked by distribution: the host sampler's top-k / top-k + top-p path (the
fixed evaluation order the device sampler repeats) must only draw tokens of
the top-k set / nucleus, and its draw frequencies must match the exact
probabilities computed here in float64 from the reference's definitions. The
device sampler must then draw exactly the host sampler's tokens (gpu)."""
import numpy as np
import pytest

import wcb
from wcb import synth


def exact_probs(logits, temperature, top_k, top_p):
    """compute_probabilities + sample_topk(_topp) (sampling.rs:106-229) in float64,
    top-k ties broken by lower index."""
    n = logits.size
    x = logits.astype(np.float64) / temperature
    p = np.exp(x - x.max())
    p /= p.sum()
    order = sorted(range(n), key=lambda i: (-logits[i], i))
    keep = np.zeros(n, bool)
    keep[order[:min(top_k, n)]] = True
    p = np.where(keep, p, 0.0)
    p /= p.sum()
    if 0.0 < top_p < 1.0:
        cum = 0.0
        for i in sorted(range(n), key=lambda i: (-p[i], i)):
            if cum >= top_p:
                p[i] = 0.0
            else:
                cum += p[i]
        p /= p.sum()
    return p


@pytest.mark.parametrize("top_k,top_p", [(8, 1.0), (20, 0.8), (5, 0.5)])
def test_host_topk_topp_draws_match_the_distribution(top_k, top_p):
    rng = np.random.default_rng(4)
    logits = rng.normal(0.0, 1.5, 300).astype(np.float32)
    logits[7] = logits[9] = logits.max()  # a tie at the top
    want = exact_probs(logits, 0.8, top_k, top_p)
    s = wcb.LogitsProcessor(123, 0.8, top_p, top_k, 1.0)
    draws = 20000
    counts = np.zeros(300)
    for _ in range(draws):
        counts[s.sample(logits.copy())] += 1
    assert counts[want == 0].sum() == 0  # nothing outside the top-k set / nucleus
    live = want > 0
    chi2 = (((counts[live] - draws * want[live]) ** 2) / (draws * want[live])).sum()
    dof = live.sum() - 1
    assert chi2 < dof + 6 * np.sqrt(2 * dof) + 10, (chi2, dof)


def test_host_sampler_is_seeded():
    rng = np.random.default_rng(5)
    logits = rng.normal(0.0, 2.0, 1000).astype(np.float32)
    a = wcb.LogitsProcessor(7, 0.7, 0.9, 40, 1.1)
    b = wcb.LogitsProcessor(7, 0.7, 0.9, 40, 1.1)
    assert [a.sample(logits.copy()) for _ in range(50)] == [b.sample(logits.copy()) for _ in range(50)]


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [dict(top_k=40, top_p=1.0, rep=1.0), dict(top_k=40, top_p=0.9, rep=1.1),
                                 dict(top_k=200, top_p=0.95, rep=1.3), dict(top_k=1, top_p=0.5, rep=1.0)])
def test_device_sampler_draws_the_host_samplers_tokens(tiny_gguf, gpu, cfg):
    dev = wcb.Model.load_from_gguf(tiny_gguf, use_persistent=False)
    host = wcb.Model.load_from_gguf(tiny_gguf, use_persistent=False, host_sampling=True)
    prompt = synth.random_prompt(24, 512, seed=9).tolist()
    for seed in (1, 2, 3):
        g = wcb.GenerationConfig(max_tokens=48, temperature=0.8, top_p=cfg["top_p"], top_k=cfg["top_k"],
                                 repetition_penalty=cfg["rep"], seed=seed, eos_id=None)
        assert dev.generate_tokens(prompt, g) == host.generate_tokens(prompt, g)
    dev.close()
    host.close()


@pytest.mark.gpu
def test_device_sampling_on_the_default_model(tiny_gguf, gpu):
    """A model with the persistent greedy kernel samples through the per-op decode graph."""
    m = wcb.Model.load_from_gguf(tiny_gguf)
    prompt = synth.random_prompt(24, 512, seed=9).tolist()
    g = wcb.GenerationConfig(max_tokens=32, temperature=0.9, top_p=0.9, top_k=40, repetition_penalty=1.1,
                             seed=5, eos_id=None)
    a, b = m.generate_tokens(prompt, g), m.generate_tokens(prompt, g)
    assert a == b and len(a) == 32 and all(0 <= t < 512 for t in a)
    greedy = wcb.GenerationConfig(max_tokens=16, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    g1 = m.generate_tokens(prompt, greedy)  # the persistent greedy path still follows
    assert g1 == m.generate_tokens(prompt, greedy)
    m.close()
