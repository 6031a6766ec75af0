"""Weight streaming (load flag bit 4): the layer weights stay in pinned host
memory and are copied into a two-slot device ring one layer ahead of the
compute. It runs the per-op kernels, so logits and token sequences must be
bit-identical to a resident model on the per-op kernels (no persistent decode
kernel), for greedy and seeded sampled generation, prefill and decode, Q4_K and
Q4_K_M (Q6_K) models."""
import numpy as np
import pytest

import wcb
from wcb import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which", ["tiny", "tiny_mix"])
def test_streamed_weights_match_resident(which, tiny_gguf, tiny_mix_gguf, gpu):
    path = tiny_gguf if which == "tiny" else tiny_mix_gguf
    vocab = 512 if which == "tiny" else 768
    res = wcb.Model.load_from_gguf(path, use_persistent=False)
    stm = wcb.Model.load_from_gguf(path, stream_weights=True)
    prompt = synth.random_prompt(40, vocab, seed=7).tolist()
    assert np.array_equal(res.forward(prompt, 0), stm.forward(prompt, 0))
    for i, t in enumerate([3, 100, 5]):
        assert np.array_equal(res.forward([t], 40 + i), stm.forward([t], 40 + i))
    greedy = wcb.GenerationConfig(max_tokens=24, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    assert res.generate_tokens(prompt, greedy) == stm.generate_tokens(prompt, greedy)
    sampled = wcb.GenerationConfig(max_tokens=12, temperature=0.8, top_p=0.9, top_k=40, repetition_penalty=1.1,
                                   seed=3, eos_id=None)
    assert res.generate_tokens(prompt, sampled) == stm.generate_tokens(prompt, sampled)
    # a long prompt: several prefill chunks' worth of layer passes through the ring
    long_prompt = synth.random_prompt(min(200, stm.config.max_seq_len - 30), vocab, seed=8).tolist()
    assert res.generate_tokens(long_prompt, greedy) == stm.generate_tokens(long_prompt, greedy)
    res.close()
    stm.close()
