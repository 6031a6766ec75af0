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


def _rank_main(rank, world, path, tp_id, prompt, q, port, persistent=True):
    try:
        import torch
        torch.cuda.set_device(rank)
        m = wcb.Model.load_from_gguf(path, device=rank, tp_rank=rank, tp_size=world, tp_id=tp_id,
                                     use_persistent=persistent)
        if port:  # decode steps exchange partial sums by peer stores (IPC handles over gloo)
            import torch.distributed as dist
            dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
            handles = [None] * world
            dist.all_gather_object(handles, m.tp_ipc_handle())
            dist.destroy_process_group()
            m.tp_connect(handles)
        logits = m.forward(prompt, 0)
        vocab = m.config.vocab_size
        part = vocab // world
        cfg = wcb.GenerationConfig(max_tokens=40, temperature=0.0, repetition_penalty=1.1, eos_id=None)
        toks = m.generate_tokens(prompt, cfg)
        steps = m.launches_per_step()
        m.close()
        q.put((rank, logits[rank * part:(rank + 1) * part].copy(), (toks, steps), None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _check_launches(res, world, exchange):
    """Decode steps of a connected group run the persistent single-launch step;
    NCCL-only groups and use_persistent=False run the per-op kernels."""
    for r in range(world):
        steps = res[r][1][1]
        if exchange == "peer":
            assert steps == 1, (r, steps)
        else:
            assert steps > 1, (r, steps)


@pytest.mark.parametrize("exchange", ["nccl", "peer", "peer_per_op"])
def test_tp2_matches_oracle(model_dir, gpu, exchange):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    path = synth.cached_model("tiny_tp", model_dir)
    prompt = synth.random_prompt(21, 1024, seed=40).tolist()
    res = _run_ranks(2, path, prompt, exchange)
    _check_launches(res, 2, exchange)
    res = {r: (lg, toks[0], err) for r, (lg, toks, err) in res.items()}
    o = oracle.OracleModel(path)
    ref = o.forward(prompt, 0)
    got = np.concatenate([res[0][0], res[1][0]])
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= 1e-2 and err <= 1e-3 * np.abs(ref).max(), err
    o.clear_kv_cache()
    ref_toks = o.generate(prompt, 40, repetition_penalty=1.1, eos_id=None)
    assert res[0][1] == ref_toks and res[1][1] == ref_toks


def _batch_rank_main(rank, world, path, tp_id, prompts, q):
    try:
        import torch
        torch.cuda.set_device(rank)
        m = wcb.Model.load_from_gguf(path, device=rank, tp_rank=rank, tp_size=world, tp_id=tp_id, max_batch=4)
        cfg = wcb.GenerationConfig(max_tokens=24, temperature=0.0, repetition_penalty=1.1, eos_id=None)
        out = m.generate_batch(prompts, cfg)
        slots, launches = m.batch_info()
        m.close()
        q.put((rank, out, slots, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))


def test_tp2_batched_decode_matches_oracle(model_dir, gpu):
    """generate_batch on a tensor-parallel model: the batched tensor-core step with
    row-parallel partial sums all-reduced and a vocabulary-split LM head."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    path = synth.cached_model("tiny_tp", model_dir)
    prompts = [synth.random_prompt(n, 1024, seed=60 + n).tolist() for n in (9, 21, 4, 33, 16)]  # 5 > 4 slots
    tp_id = wcb.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_batch_rank_main, args=(r, 2, path, tp_id, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, out, slots, err = q.get(timeout=600)
        res[r] = (out, slots, err)
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert res[r][2] is None, res[r][2]
        assert res[r][1] == 4
    o = oracle.OracleModel(path)
    for i, p in enumerate(prompts):
        o.clear_kv_cache()
        want = o.generate(p, 24, repetition_penalty=1.1, eos_id=None)
        assert res[0][0][i] == want and res[1][0][i] == want, i


def _run_ranks(world, path, prompt, exchange):
    import torch.multiprocessing as mp
    tp_id = wcb.tp_unique_id()
    port = _free_port() if exchange.startswith("peer") else 0
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, path, tp_id, prompt, q, port, exchange != "peer_per_op"))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, lg, toks, err = q.get(timeout=900)
        res[r] = (lg, toks, err)
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert res[r][2] is None, res[r][2]
    return res


@pytest.mark.parametrize("world,exchange", [(2, "nccl"), (2, "peer"), (2, "peer_per_op"), (4, "peer"),
                                            (8, "peer")])
def test_tp_70b_width_matches_oracle(model_dir, gpu, world, exchange):
    """The Llama-2-70B widths (hidden 8192, 64 / 8 heads, head_dim 128, FFN 28672),
    two layers, split over 2 / 4 / 8 ranks: every rank's logits slice within the
    tolerance and 40 greedy tokens identical to the oracle, through the persistent
    single-launch decode step (peer exchange) and the per-op kernels."""
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    path = synth.cached_model("llama70b", model_dir, num_layers=2, context_length=1024)
    prompt = synth.random_prompt(33, 32000, seed=41).tolist()
    res = _run_ranks(world, path, prompt, exchange)
    _check_launches(res, world, exchange)
    res = {r: (lg, toks[0], err) for r, (lg, toks, err) in res.items()}
    import os
    oracle.set_threads(os.cpu_count() or 1, os.cpu_count() or 1)
    o = oracle.OracleModel(path)
    ref = o.forward(prompt, 0)
    got = np.concatenate([res[r][0] for r in range(world)])
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= 1e-2 and err <= 1e-3 * np.abs(ref).max(), err
    o.clear_kv_cache()
    ref_toks = o.generate(prompt, 40, repetition_penalty=1.1, eos_id=None)
    for r in range(world):
        assert res[r][1] == ref_toks, r


def _expiry_rank(rank, path, tp_id, port, q, ev_stop, ev_done):
    """Rank 1 stops taking steps; rank 0's next step must fail within its wait bound."""
    try:
        import os
        import time
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import torch
        torch.cuda.set_device(rank)
        import torch.distributed as dist
        m = wcb.Model.load_from_gguf(path, device=rank, tp_rank=rank, tp_size=2, tp_id=tp_id, wait_ms=300)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
        handles = [None] * 2
        dist.all_gather_object(handles, m.tp_ipc_handle())
        dist.destroy_process_group()
        m.tp_connect(handles)
        prompt = synth.random_prompt(12, 1024, seed=3).tolist()
        cfg = wcb.GenerationConfig(max_tokens=64, temperature=0.0, repetition_penalty=1.0, eos_id=None)
        # prefill (NCCL, both ranks), then decode steps: partial sums and the argmax keys
        # through peer stores only, so every wait on the other rank in a step is bounded
        s = m.infer(prompt, cfg)
        toks = s.next_tokens(5)
        if rank == 1:
            ev_stop.set()  # from here on rank 1 takes no step
            ev_done.wait(120)
            m.tp_abort()  # the group is torn down
            m.close()
            q.put((rank, toks, None, None, None))
            return
        ev_stop.wait(120)
        t0 = time.time()
        err1 = err2 = None
        try:
            s.next_tokens(4)  # decode steps whose partial sums rank 1 never sends
        except wcb.WcbError as e:
            err1 = (e.code, e.message, time.time() - t0)
        try:
            s.next_tokens(1)
        except wcb.WcbError as e:
            err2 = (e.code, e.message)
        t1 = time.time()
        m.close()
        ev_done.set()
        q.put((rank, toks, err1, err2, time.time() - t1))
    except Exception as e:  # reported to the parent
        ev_stop.set()
        ev_done.set()
        q.put((rank, None, None, None, repr(e)))


def test_tp2_peer_wait_expiry_is_an_error(model_dir, gpu):
    """A bounded wait that runs out surfaces as an error code, not a hang or a
    wrong answer: with wait_ms = 300 and rank 1 idle between steps, rank 0's next
    decode steps (peer-store exchange only, no NCCL call) fail with
    BackendUnsupported naming the tensor-parallel exchange within a few seconds, the
    next call fails at once, and the model is freed cleanly."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    path = synth.cached_model("tiny_tp", model_dir)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ev_stop, ev_done = ctx.Event(), ctx.Event()
    port = _free_port()
    tp_id = wcb.tp_unique_id()
    procs = [ctx.Process(target=_expiry_rank, args=(r, path, tp_id, port, q, ev_stop, ev_done)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, toks, e1, e2, extra = q.get(timeout=300)
        res[r] = (toks, e1, e2, extra)
    for p in procs:
        p.join(timeout=60)
    assert res[1][3] is None and not isinstance(res[0][3], str), (res[0][3], res[1][3])
    assert res[0][0] == res[1][0] and len(res[0][0]) == 5
    code, msg, dt = res[0][1]
    assert code == 5 and "tensor-parallel exchange" in msg, msg
    assert dt < 5.0, dt
    assert res[0][2] is not None and res[0][2][0] == 5 and "has failed" in res[0][2][1]
    assert res[0][3] < 30.0  # close() did not wait for the idle rank


def _watchdog_gpu_rank(rank, path, tp_id, port, q):
    """Rank 1 exits between steps; rank 0 learns it from the heartbeat before its next launch."""
    try:
        import os
        import time
        from datetime import timedelta
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import torch
        torch.cuda.set_device(rank)
        from torch.distributed import TCPStore

        from wcb.tp import Watchdog
        m = wcb.Model.load_from_gguf(path, device=rank, tp_rank=rank, tp_size=2, tp_id=tp_id)
        store = TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=60))
        wd = Watchdog(store, rank, 2, lambda r: m.tp_abort(), interval=0.1, timeout=1.5).start()
        prompt = synth.random_prompt(10, 1024, seed=4).tolist()
        cfg = wcb.GenerationConfig(max_tokens=6, temperature=0.0, repetition_penalty=1.0, eos_id=None)
        toks = m.generate_tokens(prompt, cfg)  # NCCL all-reduces on both ranks
        torch.cuda.synchronize()
        if rank == 1:
            q.put((rank, toks, None, None))
            q.close()
            q.join_thread()
            os._exit(0)  # between steps, with nothing in flight: the process is simply gone
        failed = wd.wait_failure(30.0)
        t0 = time.time()
        err = None
        try:
            m.generate_tokens(prompt, cfg)
        except wcb.WcbError as e:
            err = (e.code, e.message, time.time() - t0)
        t1 = time.time()
        m.close()
        wd.stop()
        q.put((rank, toks, (failed, err), time.time() - t1))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))


def test_tp2_watchdog_aborts_the_group_when_a_rank_exits(model_dir, gpu):
    """Rank 1's process exits between steps. Rank 0's host watchdog (a TCPStore
    heartbeat) reports it and calls tp_abort (ncclCommAbort) before rank 0 launches
    anything else; rank 0's next generate then fails at once and the model is freed
    without waiting for the lost rank."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    path = synth.cached_model("tiny_tp", model_dir)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    tp_id = wcb.tp_unique_id()
    procs = [ctx.Process(target=_watchdog_gpu_rank, args=(r, path, tp_id, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, toks, info, extra = q.get(timeout=300)
        res[r] = (toks, info, extra)
    for p in procs:
        p.join(timeout=60)
    assert not isinstance(res[0][2], str) and res[1][2] is None, (res[0][2], res[1][2])
    assert res[0][0] == res[1][0]
    failed, err = res[0][1]
    assert failed == 1
    assert err is not None and err[0] == 5 and "has failed" in err[1] and err[2] < 1.0
    assert res[0][2] < 30.0
