"""Kernel-level parity through the C ABI on device buffers: dequantisation is
bit-exact against the oracle, the fused dequant-GEMV matches the oracle's
dequantised weights times x (float64 reference) to fp32 rounding."""
import numpy as np
import pytest

import oracle
import wcb
from wcb import synth

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _sync():
    import torch
    torch.cuda.synchronize()


def _rand_q4k(n, k, seed):
    x = synth.normal(seed, 1, n * k, 0.0, 0.02)
    return synth.quantize_q4_k_fast(x)


def _rand_q6k(n, k, seed):
    x = synth.normal(seed, 2, n * k, 0.0, 0.02)
    return synth.quantize_q6_k_fast(x)


@pytest.mark.parametrize("dtype", [wcb.DTYPE_Q4_K, wcb.DTYPE_Q6_K])
def test_dequant_bit_exact(gpu, dtype):
    import torch
    rng = np.random.default_rng(1)
    nb = 4096
    if dtype == wcb.DTYPE_Q4_K:
        blocks = _rand_q4k(nb, 256, 3)
        blocks[:256, 4:16] = rng.integers(0, 256, size=(256, 12), dtype=np.uint8)
        blocks[256:300, 0:4] = rng.integers(0, 256, size=(44, 4), dtype=np.uint8)  # any f16 d/dmin incl. subnormals
        ref = oracle.dequant_q4k(blocks)
    else:
        blocks = _rand_q6k(nb, 256, 3)
        blocks[:256, :210] = rng.integers(0, 256, size=(256, 210), dtype=np.uint8)
        ref = oracle.dequant_q6k(blocks)
    d = _dev(blocks.reshape(-1))
    out = torch.empty(nb * 256, dtype=torch.float32, device="cuda")
    wcb.dequant_dev(d.data_ptr(), dtype, nb, out.data_ptr())
    _sync()
    got = out.cpu().numpy()
    same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
    assert same.all(), f"{(~same).sum()} values differ"


def _gemv_case(n, k, m, dtype, seed=0):
    import torch
    if dtype == wcb.DTYPE_Q4_K:
        blocks = _rand_q4k(n, k, seed)
        w = oracle.dequant_q4k(blocks).reshape(n, k)
        dev_blocks = _dev(blocks.reshape(-1))
    else:
        blocks = _rand_q6k(n, k, seed)
        w = oracle.dequant_q6k(blocks).reshape(n, k)
        packed = _dev(blocks.reshape(-1))
        dev_blocks = torch.empty(blocks.shape[0] * 224, dtype=torch.uint8, device="cuda")
        wcb.repack_q6k_dev(packed.data_ptr(), blocks.shape[0], dev_blocks.data_ptr())
    x = synth.normal(seed + 100, 7, m * k, 0.0, 1.0).reshape(m, k)
    xd = _dev(x)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    wcb.gemv_dev(dev_blocks.data_ptr(), dtype, n, k, xd.data_ptr(), m, y.data_ptr())
    _sync()
    got = y.cpu().numpy()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    return got, ref


# the Q4_K decode shapes of the GEMV microbenchmark ([N, K], M = 1 and 16)
@pytest.mark.parametrize("n,k", [(2048, 2048), (5632, 2048), (4096, 4096), (11008, 4096), (32000, 4096)])
@pytest.mark.parametrize("m", [1, 16])
def test_gemv_q4k_microbench_shapes(gpu, n, k, m):
    got, ref = _gemv_case(n, k, m, wcb.DTYPE_Q4_K)
    err = np.abs(got - ref).max()
    assert err <= 1e-5 * np.abs(ref).max() * np.sqrt(k / 256), err


@pytest.mark.parametrize("n,k,m", [(4, 256, 1), (8, 512, 3), (260, 768, 5), (1024, 11008, 2), (64, 28672, 1)])
def test_gemv_q4k_ragged(gpu, n, k, m):
    got, ref = _gemv_case(n, k, m, wcb.DTYPE_Q4_K, seed=3)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max() * np.sqrt(k / 256)


@pytest.mark.parametrize("n,k,m", [(4096, 4096, 1), (4096, 11008, 1), (32000, 4096, 1), (12, 256, 4), (256, 1024, 9), (512, 4096, 40)])
def test_gemv_q6k(gpu, n, k, m):
    got, ref = _gemv_case(n, k, m, wcb.DTYPE_Q6_K, seed=5)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max() * np.sqrt(k / 256)


# 5..32 activation rows run the batched decode GEMM (tcgen05, one launch): ragged
# row counts, one-super-block K, Q6_K, and the largest microbenchmark shape
@pytest.mark.parametrize("n,k,m,dtype", [
    (2048, 2048, 32, wcb.DTYPE_Q4_K), (11008, 4096, 24, wcb.DTYPE_Q4_K), (260, 768, 7, wcb.DTYPE_Q4_K),
    (4, 256, 5, wcb.DTYPE_Q4_K), (32000, 4096, 16, wcb.DTYPE_Q4_K), (4096, 4096, 17, wcb.DTYPE_Q6_K),
    (388, 1280, 32, wcb.DTYPE_Q6_K)])
def test_gemv_batched_rows(gpu, n, k, m, dtype):
    got, ref = _gemv_case(n, k, m, dtype, seed=13)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max() * np.sqrt(k / 256)


def test_gemv_m512_prefill_shape(gpu):
    got, ref = _gemv_case(2048, 2048, 512, wcb.DTYPE_Q4_K, seed=9)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max() * np.sqrt(2048 / 256)


def test_gemv_linearity_at_full_size(gpu):
    # size-independent property at the largest microbenchmark shape: W(a x) = a W(x) for a power of two
    import torch
    n, k = 32000, 4096
    blocks = _rand_q4k(n, k, 21)
    d = _dev(blocks.reshape(-1))
    x = synth.normal(22, 7, k, 0.0, 1.0)
    xs = torch.stack([_dev(x), _dev(x * np.float32(8.0))])
    y = torch.empty((2, n), dtype=torch.float32, device="cuda")
    wcb.gemv_dev(d.data_ptr(), wcb.DTYPE_Q4_K, n, k, xs.data_ptr(), 2, y.data_ptr())
    _sync()
    yy = y.cpu().numpy()
    assert np.array_equal(yy[0] * np.float32(8.0), yy[1])


def test_gemv_rejects_bad_shapes(gpu):
    with pytest.raises(wcb.WcbError) as e:
        wcb.gemv_dev(1, wcb.DTYPE_Q4_K, 4, 100, 1, 1, 1)
    assert e.value.code == 3
    # x or W off a 16-byte boundary is refused on the host (the kernels read 16-byte vectors)
    with pytest.raises(wcb.WcbError) as e:
        wcb.gemv_dev(4096, wcb.DTYPE_Q4_K, 4, 256, 4096 + 4, 8, 8192)
    assert e.value.code == 3
    with pytest.raises(wcb.WcbError) as e:
        wcb.gemv_dev(4096 + 8, wcb.DTYPE_Q4_K, 4, 256, 4096, 1, 8192)
    assert e.value.code == 3
