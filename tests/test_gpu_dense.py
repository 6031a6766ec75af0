"""F32 / F16 2-D weights and the tied-embedding LM head (model.rs:482-606,
gguf.rs:446-467, tensor_loader.rs:50-149), which the reference loads as well as
Q4_K / Q6_K: a model whose output.weight is absent uses transpose_matrix(token
embeddings) as its LM head (model.rs:596-606, reproduced as the reference does
it); projections stored as F16 or F32 run the dense-weight GEMV with the same
fused epilogues. Logits within max-abs 1e-2 and 1e-3 of max |logit| of the
oracle, greedy tokens identical."""
import numpy as np
import pytest

import oracle
import wcb
from wcb import synth

pytestmark = pytest.mark.gpu


def _close(got, ref):
    err = float(np.abs(got.astype(np.float64) - ref.astype(np.float64)).max())
    assert err <= 1e-2 and err <= 1e-3 * float(np.abs(ref).max()), err


def _plan(cfg, tied=False, dense=False):
    plan = []
    for name, ne, t in synth.tensor_plan(cfg):
        if tied and name == "output.weight":
            continue
        if dense and t != synth.GGML_F32:
            if name == "output.weight" or name.startswith("blk.0.attn_q") or name.startswith("blk.0.attn_output") \
                    or name.startswith("blk.0.ffn_gate") or name.startswith("blk.0.ffn_up"):
                t = synth.GGML_F16
            elif name.startswith("blk.0.attn_k") or name.startswith("blk.0.ffn_down"):
                t = synth.GGML_F32
        plan.append((name, ne, t))
    return plan


@pytest.fixture(scope="module", params=["tied", "dense", "tied_dense"])
def variant(request, model_dir, gpu, tmp_path_factory):
    cfg = synth.PRESETS["tiny"]
    kind = request.param
    path = str(tmp_path_factory.mktemp("dense") / f"{kind}.gguf")
    synth.write_gguf(path, cfg, plan=_plan(cfg, tied="tied" in kind, dense="dense" in kind))
    return kind, path


def test_logits_and_greedy_tokens_match_the_oracle(variant):
    kind, path = variant
    m = wcb.Model.load_from_gguf(path)
    o = oracle.OracleModel(path)
    prompt = synth.random_prompt(40, 512, seed=21).tolist()  # >= 16 tokens: quantised layers take the GEMM
    _close(m.forward(prompt, 0), o.forward(prompt, 0))
    for i, t in enumerate([3, 500, 77]):
        _close(m.forward([t], 40 + i), o.forward([t], 40 + i))
    cfg = wcb.GenerationConfig(max_tokens=32, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    o.clear_kv_cache()
    assert m.generate_tokens(prompt, cfg) == o.generate(prompt, 32, repetition_penalty=1.1, eos_id=None)
    assert m.launches_per_step() > 1  # dense weights run the per-op kernels
    m.close()


def test_batch_and_streaming_with_dense_weights(variant):
    kind, path = variant
    o = oracle.OracleModel(path)
    prompts = [synth.random_prompt(n, 512, seed=30 + n).tolist() for n in (9, 25, 14)]
    cfg = wcb.GenerationConfig(max_tokens=12, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    want = []
    for p in prompts:
        o.clear_kv_cache()
        want.append(o.generate(p, 12, repetition_penalty=1.0, eos_id=None))
    m = wcb.Model.load_from_gguf(path, max_batch=4)
    assert m.generate_batch(prompts, cfg) == want  # one sequence after the other
    m.close()
    s = wcb.Model.load_from_gguf(path, stream_weights=True)
    assert [s.generate_tokens(p, cfg) for p in prompts] == want
    s.close()
