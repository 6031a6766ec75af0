"""Parity at the widths of the 7B and 70B configurations, where head_dim is 128.

Two truncated models keep every real width and only drop layers:
  * Llama-2-7B shape: hidden 4096, 32 MHA heads, FFN 11008, the Q4_K_M mix
    (Q6_K attn_v / ffn_down in even layers and Q6_K output), 2 layers;
  * Llama-2-70B shape: hidden 8192, 64 query / 8 KV heads, FFN 28672, Q4_K,
    1 layer;
both with vocab 32000. Every path the full-size configurations run is compared
with the oracle (the reference CPU path, crates/wasm-chord-runtime/src/
transformer/attention.rs:332-435 at head_dim 128, quant.rs:206-261 for Q6_K):
tensor-core prefill (gemm_tc_kernel, fa_prefill_kernel<128>), the persistent
single-launch decode step, the per-op decode kernels, weight streaming and the
batched tensor-core step. Bars: logits max-abs 1e-2 and 1e-3 of max |logit|;
64 greedy tokens identical (32 per sequence for the batched step)."""
import dataclasses
import os
from typing import Dict, List

import numpy as np
import pytest

import oracle
import wcb
from wcb import synth

pytestmark = pytest.mark.gpu

ABS_TOL = 1e-2
REL_TOL = 1e-3
PROMPT = 40                # >= 16 tokens: the tensor-core prefill path
DECODE_IDS = [7, 31999, 1234, 5]
GEN = 64
MAX_SEQ = 320
WIDE = {"7b": ("llama7b", dict(num_layers=2, context_length=1024)),
        "70b": ("llama70b", dict(num_layers=1, context_length=1024))}
BATCH_LENS = [5, 40, 17, 64, 9]  # 5 sequences through 4 slots: two groups


@dataclasses.dataclass
class Ref:
    path: str
    prompt: List[int]
    prefill: np.ndarray
    decode: List[np.ndarray]
    gen: Dict[float, List[int]]
    batch_prompts: List[List[int]]
    batch: List[List[int]]


def assert_logits_close(got, ref, what=""):
    err = float(np.abs(got.astype(np.float64) - ref.astype(np.float64)).max())
    scale = float(np.abs(ref).max())
    assert err <= ABS_TOL and err <= REL_TOL * scale, f"{what}: max abs err {err}, max |logit| {scale}"


@pytest.fixture(scope="module", params=sorted(WIDE))
def wide(request, model_dir, gpu):
    preset, ov = WIDE[request.param]
    path = synth.cached_model(preset, model_dir, **ov)
    cores = os.cpu_count() or 1
    oracle.set_threads(cores, cores)  # rows are independent: results do not depend on the thread count
    o = oracle.OracleModel(path)
    prompt = synth.random_prompt(PROMPT, o.vocab, seed=5).tolist()
    prefill = o.forward(prompt, 0)
    decode = [o.forward([t], PROMPT + i) for i, t in enumerate(DECODE_IDS)]
    gen = {}
    for rep in (1.0, 1.1):
        o.clear_kv_cache()
        gen[rep] = o.generate(prompt, GEN, repetition_penalty=rep, eos_id=None)
    bp = [synth.random_prompt(n, o.vocab, seed=200 + i).tolist() for i, n in enumerate(BATCH_LENS)]
    batch = []
    for p in bp:
        o.clear_kv_cache()
        batch.append(o.generate(p, 32, repetition_penalty=1.1, eos_id=None))
    o.close()
    return Ref(path, prompt, prefill, decode, gen, bp, batch)


# load options of each single-sequence path
PATHS = {"persistent": {}, "per_op": {"use_persistent": False}, "streamed": {"stream_weights": True}}


@pytest.mark.parametrize("kind", sorted(PATHS))
def test_wide_forward_logits(wide, kind):
    m = wcb.Model.load_from_gguf(wide.path, max_seq=MAX_SEQ, **PATHS[kind])
    assert m.config.head_dim == 128
    assert_logits_close(m.forward(wide.prompt, 0), wide.prefill, f"{kind} prefill")
    for i, t in enumerate(DECODE_IDS):  # one token per forward: the decode kernels
        assert_logits_close(m.forward([t], PROMPT + i), wide.decode[i], f"{kind} decode step {i}")
    m.close()


@pytest.mark.parametrize("rep", [1.0, 1.1])
@pytest.mark.parametrize("kind", sorted(PATHS))
def test_wide_greedy_generate(wide, kind, rep):
    m = wcb.Model.load_from_gguf(wide.path, max_seq=MAX_SEQ, **PATHS[kind])
    n = GEN if kind != "streamed" else 32
    cfg = wcb.GenerationConfig(max_tokens=n, temperature=0.0, repetition_penalty=rep, eos_id=None)
    got = m.generate_tokens(wide.prompt, cfg)
    want = wide.gen[rep][:n]
    assert got == want, f"{kind}: first mismatch at " \
                        f"{next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), len(got))}"
    steps = m.launches_per_step()
    if kind == "persistent":
        assert steps == 1  # the single-launch decode step ran (the 70B width: its down projection as a K chain)
    if kind == "per_op":
        assert steps > 1
    m.close()


def test_wide_batched_decode(wide):
    m = wcb.Model.load_from_gguf(wide.path, max_seq=MAX_SEQ, max_batch=4)
    assert m.batch_info()[0] == 4
    cfg = wcb.GenerationConfig(max_tokens=32, temperature=0.0, repetition_penalty=1.1, eos_id=None)
    got = m.generate_batch(wide.batch_prompts, cfg)
    for i, (g, w) in enumerate(zip(got, wide.batch)):
        assert g == w, f"sequence {i} (prompt of {len(wide.batch_prompts[i])} tokens)"
    m.close()
