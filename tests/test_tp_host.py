"""Host side of tensor parallelism, no GPU: group ids, shard shapes of the
synthetic model, and the 2-rank id exchange over gloo."""
import os

import pytest

import wcb
from wcb import synth


def test_tp_unique_id_is_128_fresh_bytes():
    a, b = wcb.tp_unique_id(), wcb.tp_unique_id()
    assert len(a) == 128 and len(b) == 128 and a != b


def test_tiny_tp_preset_splits_over_two_ranks():
    c = synth.PRESETS["tiny_tp"]
    kvd = c.num_kv_heads * c.head_dim
    for tp in (2,):
        assert c.num_heads % tp == 0 and c.num_kv_heads % tp == 0
        assert (c.hidden_size // tp) % 256 == 0 and (c.intermediate_size // tp) % 256 == 0
        assert c.vocab_size % (4 * tp) == 0 and (kvd // tp) % 4 == 0


def test_llama70b_splits_over_eight_ranks():
    c = synth.PRESETS["llama70b"]
    for tp in (2, 4, 8):
        assert c.num_heads % tp == 0 and c.num_kv_heads % tp == 0
        assert (c.hidden_size // tp) % 256 == 0 and (c.intermediate_size // tp) % 256 == 0
        assert c.vocab_size % (4 * tp) == 0


def _exchange(rank, world, port, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    obj = [wcb.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    q.put((rank, obj[0]))
    dist.destroy_process_group()


def test_group_id_broadcast_over_gloo():
    """The bench and the tests hand rank 0's id to every rank this way."""
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_exchange, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert got[0] == got[1] and len(got[0]) == 128


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _watchdog_rank(rank, port, q, exit_after):
    import time
    from datetime import timedelta

    from torch.distributed import TCPStore

    from wcb.tp import Watchdog
    store = TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=30))
    fired = []
    wd = Watchdog(store, rank, 2, lambda r: fired.append(r), interval=0.1, timeout=1.0).start()
    if rank == 1:
        time.sleep(exit_after)
        q.put(("exit", 1, time.time()))
        q.close()
        q.join_thread()  # the message is out before the process ends
        os._exit(0)  # no clean-up: the heartbeat simply stops, as when a rank dies
    quiet = wd.wait_failure(exit_after - 0.3)  # nothing may be reported while rank 1 is alive
    q.put(("quiet", quiet, time.time()))
    r = wd.wait_failure(15.0)
    q.put(("fired", r, time.time()))
    wd.stop()


def test_watchdog_reports_a_rank_that_exits():
    """Two ranks (processes) share a TCPStore heartbeat; rank 1 exits without any
    clean-up between steps. Rank 0's watchdog stays quiet while rank 1 is alive,
    then reports rank 1 within its timeout (the callback is where a model calls
    tp_abort). No GPU: the failure is made and detected on the host."""
    import torch.multiprocessing as mp
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_watchdog_rank, args=(r, port, q, 2.0)) for r in range(2)]
    for p in ps:
        p.start()
    ev = {}
    for _ in range(3):
        kind, r, t = q.get(timeout=60)
        ev[kind] = (r, t)
    for p in ps:
        p.join(timeout=30)
    assert ev["quiet"][0] is None
    assert ev["fired"][0] == 1
    delay = ev["fired"][1] - ev["exit"][1]
    assert 0.5 < delay < 6.0, delay


def test_watchdog_rejects_a_timeout_below_the_interval():
    from wcb.tp import Watchdog
    with pytest.raises(ValueError):
        Watchdog(None, 0, 2, lambda r: None, interval=1.0, timeout=0.5)


def test_truncated_and_incomplete_files_fail_before_any_device_work(tmp_path):
    """A GGUF cut short fails with IoError naming the tensor, and one without the
    token embeddings (the reference's one required tensor, model.rs:432-446) with
    ModelParseError, both before the library touches a GPU (none here)."""
    cfg = synth.PRESETS["tiny"]
    full = synth.make_model("tiny", str(tmp_path / "full.gguf"))
    cut = tmp_path / "cut.gguf"
    data = open(full, "rb").read()
    cut.write_bytes(data[: len(data) - 5000])
    with pytest.raises(wcb.WcbError) as e:
        wcb.Model.load_from_gguf(str(cut))
    assert e.value.code == 7 and "truncated" in e.value.message
    plan = [p for p in synth.tensor_plan(cfg) if p[0] != "token_embd.weight"]
    noemb = synth.write_gguf(str(tmp_path / "noemb.gguf"), cfg, plan=plan)
    with pytest.raises(wcb.WcbError) as e:
        wcb.Model.load_from_gguf(noemb)
    assert e.value.code == 4 and "Missing token embeddings" in e.value.message
