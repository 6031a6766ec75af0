"""Sampled decoding (LogitsProcessor::sample, sampling.rs:106-229). Every draw
takes one u32 of the reference's random stream (rand 0.9 StdRng::seed_from_u64,
restated; the oracle's copy is pinned by the ChaCha known answers), checked here
by reading it back through draws over equal weights, and on the same logits the
host sampler draws the oracle's tokens. Its probabilities are computed in another
order than the reference's (softmax over the kept candidates), so they are also
checked by distribution: for every sampling kind (top-k, top-k + top-p, top-p
alone, all tokens, top-k above 1024) the host sampler's probabilities must equal
the oracle's (compute_probabilities, top-k, top-p, renormalisation as the
reference computes them), it must draw only kept tokens, and its draw frequencies
must match the exact probabilities (chi-squared). The device sampler must then
draw exactly the host sampler's tokens, and sampled generate() on the device the
oracle's tokens (gpu)."""
import oracle
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


ORACLE_CASES = [  # (vocab, top_k, top_p): every sampling kind of sampling.rs:57-78
    (300, 20, 0.8),     # top-k then top-p, 20 <= 1024 candidates (fixed-order path)
    (300, 0, 0.9),      # top-p alone over all tokens
    (300, 0, 1.0),      # all tokens
    (3000, 1500, 0.8),  # top-k above 1024 then top-p
    (3000, 2000, 1.0),  # top-k above 1024
    (3000, 5000, 0.7),  # top_k >= vocab: top-p over all tokens
]


@pytest.mark.parametrize("n,top_k,top_p", ORACLE_CASES)
def test_host_probabilities_match_the_oracle(n, top_k, top_p):
    """The distribution each draw uses equals the oracle's within f32 rounding: the
    same kept tokens, probabilities within 2e-6 absolute and 1e-4 relative."""
    rng = np.random.default_rng(n + top_k)
    for trial in range(4):
        logits = rng.normal(0.0, 1.2, n).astype(np.float32)
        s = wcb.LogitsProcessor(17 + trial, 0.9, top_p, top_k, 1.0)
        o = oracle.Sampler(17 + trial, 0.9, top_p, top_k, 1.0)
        want = o.distribution(logits)
        s.sample(logits.copy())
        got = s.last_probs(n)
        assert np.array_equal(got > 0, want > 0), (trial, int((got > 0).sum()), int((want > 0).sum()))
        err = np.abs(got.astype(np.float64) - want)
        assert np.all(err <= 2e-6 + 1e-4 * want), (trial, float(err.max()))


@pytest.mark.parametrize("top_k,top_p", [(0, 0.9), (0, 1.0), (1500, 0.85)])
def test_host_full_path_draws_match_the_oracle_distribution(top_k, top_p):
    """chi-squared of the draws of the configurations without a 1024-candidate bound
    against the oracle's probabilities (the logits are drawn so that no token
    has a vanishing probability)."""
    n = 2000 if top_k else 400
    rng = np.random.default_rng(11)
    logits = rng.normal(0.0, 0.5, n).astype(np.float32)
    s = wcb.LogitsProcessor(99, 1.0, top_p, top_k, 1.0)
    want = oracle.Sampler(99, 1.0, top_p, top_k, 1.0).distribution(logits).astype(np.float64)
    draws = 60000
    counts = np.zeros(n)
    for _ in range(draws):
        counts[s.sample(logits.copy())] += 1
    assert counts[want == 0].sum() == 0
    live = want > 0
    chi2 = (((counts[live] - draws * want[live]) ** 2) / (draws * want[live])).sum()
    dof = live.sum() - 1
    assert chi2 < dof + 6 * np.sqrt(2 * dof) + 10, (chi2, dof)


@pytest.mark.parametrize("n,top_k,top_p,temp", [(300, 40, 0.9, 0.7), (3000, 40, 0.9, 0.7), (300, 0, 0.9, 0.8),
                                                (3000, 0, 1.0, 1.0), (3000, 1500, 0.8, 0.9)])
def test_host_sampler_draws_the_oracles_tokens(n, top_k, top_p, temp):
    """On the same logits the host sampler draws exactly the oracle's token at every
    step (the same stream position and penalty history): its probabilities differ
    from the oracle's only by f32 rounding, far below the stream's 2^-23 resolution."""
    for seed in (42, 7):
        rng = np.random.default_rng(seed + n)
        a = wcb.LogitsProcessor(seed, temp, top_p, top_k, 1.1)
        b = oracle.Sampler(seed, temp, top_p, top_k, 1.1)
        for step in range(150):
            logits = rng.normal(0.0, 2.0, n).astype(np.float32)
            assert a.sample(logits.copy()) == b.sample(logits.copy()), (seed, step)


@pytest.mark.parametrize("temp,top_p,top_k", [(1e-7, 0.9, 40), (0.5e-7, 0.9, 40), (0.7, 0.0, 40), (0.7, 1.0, 40),
                                              (0.7, 0.0, 0), (0.7, 1.0, 0), (0.7, 0.5, 1), (0.7, 0.9, 300),
                                              (0.7, 0.9, 301), (0.7, 0.9, 5000), (2.0, 0.999, 0), (0.05, 0.9, 40)])
def test_host_sampler_edges_of_with_params(temp, top_p, top_k):
    """The boundaries of with_params (sampling.rs:57-78: temperature at 1e-7, top_p at
    0 and 1, top_k 0, 1, = n, = n + 1 and above n) and of sample_topk /
    sample_topk_topp (top_k >= n): token for token the oracle's draws over 300 logits."""
    rng = np.random.default_rng(3)
    a = wcb.LogitsProcessor(11, temp, top_p, top_k, 1.2)
    b = oracle.Sampler(11, temp, top_p, top_k, 1.2)
    for step in range(60):
        logits = rng.normal(0.0, 2.0, 300).astype(np.float32)
        assert a.sample(logits.copy()) == b.sample(logits.copy()), (b.kind, step)


@pytest.mark.parametrize("seed", [0, 42, 7919])
def test_host_draws_read_the_reference_stream(seed):
    """Equal logits make every probability a power of two, so the token drawn is the
    top bits of the stream's next u32: 10 bits over 1024 tokens on the top-k path
    (float weights, as the reference's WeightedIndex), 12 bits over 4096 tokens on the
    integer-weight path (top_k = 0). Both equal the oracle's StdRng words."""
    words = oracle.std_rng_u32(seed, 300)
    s = wcb.LogitsProcessor(seed, 0.8, 1.0, 1024, 1.0)
    assert [s.sample(np.zeros(1024, np.float32)) for _ in range(300)] == [w >> 22 for w in words]
    s = wcb.LogitsProcessor(seed, 0.8, 1.0, 0, 1.0)
    assert [s.sample(np.zeros(4096, np.float32)) for _ in range(300)] == [w >> 20 for w in words]


def test_host_sampler_is_seeded():
    rng = np.random.default_rng(5)
    logits = rng.normal(0.0, 2.0, 1000).astype(np.float32)
    a = wcb.LogitsProcessor(7, 0.7, 0.9, 40, 1.1)
    b = wcb.LogitsProcessor(7, 0.7, 0.9, 40, 1.1)
    assert [a.sample(logits.copy()) for _ in range(50)] == [b.sample(logits.copy()) for _ in range(50)]


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [dict(top_k=40, top_p=1.0, rep=1.0), dict(top_k=40, top_p=0.9, rep=1.1),
                                 dict(top_k=200, top_p=0.95, rep=1.3), dict(top_k=1, top_p=0.5, rep=1.0),
                                 dict(top_k=0, top_p=0.9, rep=1.1), dict(top_k=0, top_p=1.0, rep=1.0),
                                 dict(top_k=600, top_p=0.8, rep=1.2)])
@pytest.mark.parametrize("persistent", [False, True])
def test_device_sampler_draws_the_host_samplers_tokens(tiny_gguf, gpu, cfg, persistent):
    """Per-op decode graph + sampler kernel, or the single-launch decode step + sampler
    kernel (2 launches per step): the host sampler's tokens for every seed."""
    dev = wcb.Model.load_from_gguf(tiny_gguf, use_persistent=persistent)
    host = wcb.Model.load_from_gguf(tiny_gguf, use_persistent=persistent, host_sampling=True)
    prompt = synth.random_prompt(24, 512, seed=9).tolist()
    for seed in (1, 2, 3):
        g = wcb.GenerationConfig(max_tokens=48, temperature=0.8, top_p=cfg["top_p"], top_k=cfg["top_k"],
                                 repetition_penalty=cfg["rep"], seed=seed, eos_id=None)
        assert dev.generate_tokens(prompt, g) == host.generate_tokens(prompt, g)
    assert (dev.launches_per_step() == 2) == persistent
    dev.close()
    host.close()


@pytest.mark.gpu
@pytest.mark.parametrize("persistent", [False, True])
def test_device_sampled_generate_matches_the_oracle(tiny_gguf, gpu, persistent):
    """Sampled generate() on the device against the oracle's generate() with the same
    seed: the reference's default configuration (top-k 40 then top-p 0.9, T 0.7, penalty
    1.1) and top-p alone over the whole vocabulary. The draws take the same StdRng words;
    the device's logits differ from the oracle's by about 1e-6, so a draw could only
    differ where it falls that close to a cumulative boundary."""
    m = wcb.Model.load_from_gguf(tiny_gguf, use_persistent=persistent)
    o = oracle.OracleModel(tiny_gguf)
    prompt = synth.random_prompt(24, 512, seed=9).tolist()
    for top_k, top_p, seed in ((40, 0.9, 42), (40, 0.9, 1234), (0, 0.9, 42)):
        g = wcb.GenerationConfig(max_tokens=32, temperature=0.7, top_p=top_p, top_k=top_k,
                                 repetition_penalty=1.1, seed=seed, eos_id=None)
        want = o.generate(prompt, 32, temperature=0.7, top_p=top_p, top_k=top_k, repetition_penalty=1.1,
                          seed=seed, eos_id=None)
        assert m.generate_tokens(prompt, g) == want, (top_k, top_p, seed)
    m.close()


@pytest.mark.gpu
def test_device_sampling_on_the_default_model(tiny_gguf, gpu):
    """The reference's default configuration (T 0.7-0.9, top-p 0.9, top-k 40, penalty
    1.1) samples through the single-launch decode step and the sampler kernel; greedy
    decoding on the same model follows with one launch per step."""
    m = wcb.Model.load_from_gguf(tiny_gguf)
    prompt = synth.random_prompt(24, 512, seed=9).tolist()
    g = wcb.GenerationConfig(max_tokens=32, temperature=0.9, top_p=0.9, top_k=40, repetition_penalty=1.1,
                             seed=5, eos_id=None)
    a, b = m.generate_tokens(prompt, g), m.generate_tokens(prompt, g)
    assert a == b and len(a) == 32 and all(0 <= t < 512 for t in a)
    assert m.launches_per_step() == 2
    greedy = wcb.GenerationConfig(max_tokens=16, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    g1 = m.generate_tokens(prompt, greedy)  # the persistent greedy path still follows
    assert g1 == m.generate_tokens(prompt, greedy)
    assert m.launches_per_step() == 1
    m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("top_k,top_p", [(1500, 0.9), (2500, 1.0), (0, 0.95)])
@pytest.mark.parametrize("persistent", [False, True])
def test_device_full_sampler_on_a_large_vocabulary(model_dir, gpu, top_k, top_p, persistent):
    """top_k above 1024 (and no top_k) over a 3072-token vocabulary: the device's
    sample_full_kernel draws exactly the host sampler's tokens, with no host round trip
    per token (per step one launch of the decode graph, or the single-launch decode
    step and the sampler kernel)."""
    path = synth.cached_model("tiny", model_dir, vocab_size=3072)
    dev = wcb.Model.load_from_gguf(path, use_persistent=persistent)
    host = wcb.Model.load_from_gguf(path, use_persistent=persistent, host_sampling=True)
    prompt = synth.random_prompt(20, 3072, seed=12).tolist()
    for seed in (4, 5):
        g = wcb.GenerationConfig(max_tokens=40, temperature=1.1, top_p=top_p, top_k=top_k,
                                 repetition_penalty=1.1, seed=seed, eos_id=None)
        assert dev.generate_tokens(prompt, g) == host.generate_tokens(prompt, g)
    assert dev.launches_per_step() == 2 if persistent else dev.launches_per_step() > 2
    dev.close()
    host.close()


@pytest.mark.gpu
@pytest.mark.parametrize("top_k,top_p", [(40, 0.9), (0, 0.9), (2000, 1.0)])
def test_device_samplers_above_the_staged_vocabulary(model_dir, gpu, top_k, top_p):
    """A 40000-token vocabulary (more logits than the samplers stage in shared memory):
    both device samplers read the penalised logits from global memory and still draw
    exactly the host sampler's tokens."""
    path = synth.cached_model("tiny", model_dir, vocab_size=40000)
    dev = wcb.Model.load_from_gguf(path)
    host = wcb.Model.load_from_gguf(path, host_sampling=True)
    prompt = synth.random_prompt(20, 40000, seed=13).tolist()
    for seed in (6, 7):
        g = wcb.GenerationConfig(max_tokens=24, temperature=0.9, top_p=top_p, top_k=top_k,
                                 repetition_penalty=1.1, seed=seed, eos_id=None)
        assert dev.generate_tokens(prompt, g) == host.generate_tokens(prompt, g)
    dev.close()
    host.close()
