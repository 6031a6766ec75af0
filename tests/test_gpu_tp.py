"""Tensor parallelism over 2 GPUs (one process per GPU, NCCL all-reduce after the
attention-out and down projections, LM head split by vocabulary): greedy tokens
identical to the oracle and to one GPU, each rank's logits slice within the
parity tolerance. Skipped when fewer than 2 GPUs are visible."""
import numpy as np
import pytest

import oracle
import wcb
from wcb import synth

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count()


def _rank_main(rank, world, path, tp_id, prompt, q):
    try:
        import torch
        torch.cuda.set_device(rank)
        m = wcb.Model.load_from_gguf(path, device=rank, tp_rank=rank, tp_size=world, tp_id=tp_id)
        logits = m.forward(prompt, 0)
        vocab = m.config.vocab_size
        part = vocab // world
        cfg = wcb.GenerationConfig(max_tokens=40, temperature=0.0, repetition_penalty=1.1, eos_id=None)
        toks = m.generate_tokens(prompt, cfg)
        m.close()
        q.put((rank, logits[rank * part:(rank + 1) * part].copy(), toks, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))


def test_tp2_matches_oracle(model_dir, gpu):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    path = synth.cached_model("tiny_tp", model_dir)
    prompt = synth.random_prompt(21, 1024, seed=40).tolist()
    tp_id = wcb.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, path, tp_id, prompt, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, lg, toks, err = q.get(timeout=600)
        res[r] = (lg, toks, err)
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert res[r][2] is None, res[r][2]
    o = oracle.OracleModel(path)
    ref = o.forward(prompt, 0)
    got = np.concatenate([res[0][0], res[1][0]])
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= 1e-2 and err <= 1e-3 * np.abs(ref).max(), err
    o.clear_kv_cache()
    ref_toks = o.generate(prompt, 40, repetition_penalty=1.1, eos_id=None)
    assert res[0][1] == ref_toks and res[1][1] == ref_toks
