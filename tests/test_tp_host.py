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
