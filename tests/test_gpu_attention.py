"""GQA attention over a device KV cache through the C ABI (wcb_attention_dev)
against the oracle's compute_attention (attention.rs:332-435), including the
split-K decode path whose partial results are merged by the last CTA."""
import numpy as np
import pytest

import oracle
import wcb
from wcb import synth

pytestmark = pytest.mark.gpu


def run_case(T, nh, nkv, hd, kv_len, position, max_seq, seed=0):
    import torch
    q = synth.normal(seed, 1, T * nh * hd, 0.0, 1.0)
    k = synth.normal(seed, 2, kv_len * nkv * hd, 0.0, 1.0)  # reference layout [kv_len][n_kv][hd]
    v = synth.normal(seed, 3, kv_len * nkv * hd, 0.0, 1.0)
    ref = oracle.attention(q, k, v, T, kv_len, position, nh, nkv, hd)
    kc = np.zeros((nkv, max_seq, hd), np.float32)
    vc = np.zeros((nkv, max_seq, hd), np.float32)
    kc[:, :kv_len] = k.reshape(kv_len, nkv, hd).transpose(1, 0, 2)
    vc[:, :kv_len] = v.reshape(kv_len, nkv, hd).transpose(1, 0, 2)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, kc, vc))
    out = torch.empty(T * nh * hd, dtype=torch.float32, device="cuda")
    wcb.attention_dev(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), T, nh, nkv, hd, max_seq,
                      kv_len, position)
    torch.cuda.synchronize()
    return out.cpu().numpy(), ref


@pytest.mark.parametrize("kv_len", [1, 31, 33, 200, 2048, 2304])
def test_decode_gqa_tinyllama_heads(gpu, kv_len):
    got, ref = run_case(1, 32, 4, 64, kv_len, kv_len - 1, 4096)
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("kv_len", [7, 640])
def test_decode_mha_hd128(gpu, kv_len):
    got, ref = run_case(1, 32, 32, 128, kv_len, kv_len - 1, 1024, seed=3)
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_decode_70b_heads(gpu):
    got, ref = run_case(1, 64, 8, 128, 1100, 1099, 2048, seed=4)
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("T,kv_len,position", [(5, 5, 0), (8, 40, 32), (64, 64, 0), (3, 10, 2)])
def test_prefill_causal(gpu, T, kv_len, position):
    # position below kv_len - T is the reference quirk of a forward at an earlier position
    got, ref = run_case(T, 8, 2, 64, kv_len, position, 128, seed=5)
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_rejects_bad_shapes(gpu):
    with pytest.raises(wcb.WcbError) as e:
        wcb.attention_dev(1, 1, 1, 1, 1, 32, 4, 96, 64, 10, 9)
    assert e.value.code == 3
    with pytest.raises(wcb.WcbError):
        wcb.attention_dev(1, 1, 1, 1, 4, 32, 4, 64, 64, 3, 0)
