"""wcb_attention_dev_noalloc: the attention entry point for callers that cannot
allocate GPU memory while running (their device memory already belongs to their
own pool, or they cannot afford the device-wide pause of cudaMalloc / cudaFree).
It must give the same results as wcb_attention_dev, whose scratch the library
allocates, on consecutive calls that reuse the fixed scratch array. This file
is collected last so that a failure here stops a -x run only after every other
test has run."""
import numpy as np
import pytest

import wcb
from wcb import synth

pytestmark = pytest.mark.gpu


def _inputs(T, nh, nkv, hd, kv_len, max_seq, seed):
    import torch
    q = synth.normal(seed, 1, T * nh * hd, 0.0, 1.0)
    kc = np.zeros((nkv, max_seq, hd), np.float32)
    vc = np.zeros((nkv, max_seq, hd), np.float32)
    kc[:, :kv_len] = synth.normal(seed, 2, nkv * kv_len * hd, 0.0, 1.0).reshape(nkv, kv_len, hd)
    vc[:, :kv_len] = synth.normal(seed, 3, nkv * kv_len * hd, 0.0, 1.0).reshape(nkv, kv_len, hd)
    return tuple(torch.from_numpy(a).cuda() for a in (q, kc, vc))


def _both(T, nh, nkv, hd, kv_len, position, max_seq, seed):
    import torch
    q, k, v = _inputs(T, nh, nkv, hd, kv_len, max_seq, seed)
    ref = torch.full((T * nh * hd,), float("nan"), device="cuda")
    got = torch.full((T * nh * hd,), float("nan"), device="cuda")
    args = (T, nh, nkv, hd, max_seq, kv_len, position)
    wcb.attention_dev(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), *args)
    wcb.attention_dev_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), got.data_ptr(), *args)
    torch.cuda.synchronize()
    return got.cpu().numpy(), ref.cpu().numpy()


def test_noalloc_matches_allocating_entry_on_consecutive_calls(gpu):
    calls = [
        (1, 32, 4, 64, 333, 332, 4096, 1),    # TinyLlama heads, split decode
        (1, 64, 8, 128, 2048, 2047, 4096, 2),  # 70B heads, 64 splits
        (1, 32, 4, 64, 40, 39, 4096, 3),     # fewer splits than the call before
        (6, 8, 2, 64, 50, 44, 128, 4),        # several query tokens
    ]
    for T, nh, nkv, hd, kv_len, pos, max_seq, seed in calls:
        got, ref = _both(T, nh, nkv, hd, kv_len, pos, max_seq, seed)
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_noalloc_rejects_more_than_its_scratch(gpu):
    # 128 query heads of 128 dims at 64 splits need 4.26 MB > 4 MiB; the size is checked
    # on the host before any device access, so these 16-byte aligned addresses are never read
    a = 1 << 20
    with pytest.raises(wcb.WcbError) as e:
        wcb.attention_dev_noalloc(a, a + 256, a + 512, a + 768, 1, 128, 8, 128, 4096, 4096, 4095)
    assert e.value.code == 3 and "scratch" in e.value.message
