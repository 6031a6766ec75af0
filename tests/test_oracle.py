"""The oracle against the reference's own known-answer tests (restated from the
wasm-chord tree) and against gguf-py 0.19.0's independent Q4_K/Q6_K
dequantisers. These pin the oracle before it is used as the parity checker."""
import math

import numpy as np
import pytest

import oracle
from wcb import synth


# ---- gemm.rs:181-226 -------------------------------------------------------
def test_matmul_transposed_kat():
    a = np.array([[1, 2], [3, 4]], np.float32)
    b_t = np.array([[1, 3], [2, 4]], np.float32)
    assert oracle.matmul_transposed(a, b_t).tolist() == [[7, 10], [15, 22]]


def test_matmul_transposed_sequential_order():
    # one f32 accumulator, l ascending: 1e8 + 1 - 1e8 == 0 in f32
    a = np.array([[1e8, 1.0, -1e8]], np.float32)
    b = np.array([[1.0, 1.0, 1.0]], np.float32)
    assert oracle.matmul_transposed(a, b)[0, 0] == 0.0


# ---- sampling.rs:281-329 ---------------------------------------------------
def test_argmax_kat():
    s = oracle.Sampler(42, 0.0, 1.0, 0, 1.0)
    assert s.kind == "ArgMax"
    assert s.sample(np.array([1.0, 3.0, 2.0, 5.0, 1.5], np.float32)) == 3


def test_argmax_last_maximum_wins():
    s = oracle.Sampler(42, 0.0, 1.0, 0, 1.0)
    assert s.sample(np.array([2.0, 7.0, 7.0, 1.0], np.float32)) == 2


def test_argmax_nan_is_error():
    s = oracle.Sampler(42, 0.0, 1.0, 0, 1.0)
    with pytest.raises(oracle.OracleError):
        s.sample(np.array([1.0, np.nan, 2.0], np.float32))


def test_repetition_penalty_kat():
    s = oracle.Sampler(42, 0.0, 1.0, 0, 1.5)
    assert s.sample(np.array([5.0, 3.0, 2.0], np.float32)) == 0
    l = np.array([5.0, 3.0, 2.0], np.float32)
    s.penalize(l)
    assert l[0] < 5.0 and l[0] == np.float32(5.0) / np.float32(1.5)


def test_repetition_penalty_per_occurrence_and_sign():
    s = oracle.Sampler(42, 0.0, 1.0, 0, 2.0)
    assert s.sample(np.array([1.0, 4.0, -3.0], np.float32)) == 1
    assert s.sample(np.array([3.0, 4.0, -3.0], np.float32)) == 0  # 4/2 = 2 < 3
    assert s.sample(np.array([0.0, 9.0, -3.0], np.float32)) == 1  # 9/2 = 4.5
    l = np.array([1.0, 4.0, -3.0], np.float32)
    s.penalize(l)  # history [1, 0, 1]: token 1 twice, token 0 once
    assert l.tolist() == [0.5, 1.0, -3.0]
    s2 = oracle.Sampler(42, 0.0, 1.0, 0, 2.0)
    s2.sample(np.array([0.0, 0.0, 5.0], np.float32))
    neg = np.array([0.0, 0.0, -3.0], np.float32)
    s2.penalize(neg)
    assert neg[2] == -6.0  # negative logits are multiplied


def test_sampling_kinds_follow_with_params():
    assert oracle.Sampler(1, 0.0, 0.9, 40, 1.1).kind == "ArgMax"
    assert oracle.Sampler(1, 0.7, 0.9, 40, 1.1).kind == "TopKThenTopP"
    assert oracle.Sampler(1, 0.7, 1.0, 40, 1.1).kind == "TopK"
    assert oracle.Sampler(1, 0.7, 0.9, 0, 1.1).kind == "TopP"
    assert oracle.Sampler(1, 0.7, 1.0, 0, 1.1).kind == "All"


def test_topk_membership():
    for seed in range(20):
        s = oracle.Sampler(seed, 1.0, 1.0, 2, 1.0)
        assert s.sample(np.array([1.0, 5.0, 3.0, 2.0, 4.0], np.float32)) in (1, 4)


def test_topp_membership():
    for seed in range(20):
        s = oracle.Sampler(seed, 1.0, 0.9, 0, 1.0)
        assert s.sample(np.array([10.0, 5.0, 2.0, 1.0] + [0.0] * 6, np.float32)) <= 3


# ---- the random stream: rand 0.9 StdRng::seed_from_u64 (sampling.rs:40, :75) ----
# RFC 8439 appendix A.1, ChaCha20 block function test vectors 1 and 2 (all-zero key
# and nonce, block counters 0 and 1), as keystream bytes
RFC8439_A1 = [
    "76b8e0ada0f13d90405d6ae55386bd28bdd219b8a08ded1aa836efcc8b770dc7"
    "da41597c5157488d7724e03fb8d84a376a43b8f41518a11cc387b669b2ee6586",
    "9f07e7be5551387a98ba977c732d080dcb0f29a048e3656912c6533e32ee7aed"
    "29b721769ce64e43d57133b074d839d531ed1f28510afb45ace10a1f4b794d6f",
]


def test_chacha_block_known_answers():
    """The block function under the oracle's StdRng (ChaCha12) is ChaCha: with 20
    rounds it reproduces the RFC's keystream, and a block counter of 1 is the next block."""
    for counter, hexbytes in enumerate(RFC8439_A1):
        words = oracle.chacha_block(bytes(32), counter, 20)
        assert b"".join(w.to_bytes(4, "little") for w in words).hex() == hexbytes


def _py_std_rng(seed: int, n: int) -> list:
    """A second restatement: rand_core 0.9 seed_from_u64 (PCG32 fill) + rand_chacha
    0.9 ChaCha12Rng, one word at a time."""
    M = (1 << 64) - 1
    key = []
    for _ in range(8):
        seed = (seed * 6364136223846793005 + 11634580027462260723) & M
        xs = (((seed >> 18) ^ seed) >> 27) & 0xFFFFFFFF
        rot = seed >> 59
        key.append(((xs >> rot) | (xs << (32 - rot))) & 0xFFFFFFFF)

    def rotl(v, c):
        return ((v << c) | (v >> (32 - c))) & 0xFFFFFFFF

    def block(ctr):
        s = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574] + key + [ctr & 0xFFFFFFFF, ctr >> 32, 0, 0]
        x = list(s)
        for _ in range(6):
            for a, b, c, d in ((0, 4, 8, 12), (1, 5, 9, 13), (2, 6, 10, 14), (3, 7, 11, 15),
                               (0, 5, 10, 15), (1, 6, 11, 12), (2, 7, 8, 13), (3, 4, 9, 14)):
                x[a] = (x[a] + x[b]) & 0xFFFFFFFF
                x[d] = rotl(x[d] ^ x[a], 16)
                x[c] = (x[c] + x[d]) & 0xFFFFFFFF
                x[b] = rotl(x[b] ^ x[c], 12)
                x[a] = (x[a] + x[b]) & 0xFFFFFFFF
                x[d] = rotl(x[d] ^ x[a], 8)
                x[c] = (x[c] + x[d]) & 0xFFFFFFFF
                x[b] = rotl(x[b] ^ x[c], 7)
        return [(x[i] + s[i]) & 0xFFFFFFFF for i in range(16)]

    return [block(w // 16)[w % 16] for w in range(n)]


@pytest.mark.parametrize("seed", [0, 1, 42, (1 << 64) - 1])
def test_std_rng_stream_restatements_agree(seed):
    assert oracle.std_rng_u32(seed, 40) == _py_std_rng(seed, 40)


def test_sampled_draw_reads_the_stream():
    """WeightedIndex over 1024 equal weights (every probability exactly 2^-10) picks
    floor(u * 1024) for u = Uniform<f32>(0, 1): the top 10 bits of each u32 of the stream."""
    words = oracle.std_rng_u32(42, 200)
    s = oracle.Sampler(42, 0.8, 1.0, 0, 1.0)
    assert [s.sample(np.zeros(1024, np.float32)) for _ in range(200)] == [w >> 22 for w in words]


# ---- tests/test_attention.rs:256-278, test_rope.rs, test_kv_cache_fix.rs ----
def test_attention_single_token_is_v():
    heads, kv_heads, hd = 4, 2, 8
    q = np.full(heads * hd, 2.0, np.float32)
    k = np.full(kv_heads * hd, 2.0, np.float32)
    v = np.full(kv_heads * hd, 5.0, np.float32)
    out = oracle.attention(q, k, v, 1, 1, 0, heads, kv_heads, hd)
    assert np.all(out == 5.0)


def test_attention_causal_mask():
    heads, kv_heads, hd = 2, 1, 4
    rng = np.random.default_rng(0)
    q = rng.standard_normal(2 * heads * hd).astype(np.float32)
    k = rng.standard_normal(3 * kv_heads * hd).astype(np.float32)
    v = rng.standard_normal(3 * kv_heads * hd).astype(np.float32)
    # position 0, two queries: query 0 sees key 0 only, query 1 keys 0..1; key 2 is masked for both
    out = oracle.attention(q, k, v, 2, 3, 0, heads, kv_heads, hd).reshape(2, heads, hd)
    assert np.allclose(out[0, 0], v[:hd])
    v2 = v.copy()
    v2[2 * hd:] = 100.0
    out2 = oracle.attention(q, k, v2, 2, 3, 0, heads, kv_heads, hd).reshape(2, heads, hd)
    assert np.array_equal(out, out2)


def test_rope_identity_at_zero_and_norm():
    rng = np.random.default_rng(3)
    t = rng.standard_normal(4 * 64).astype(np.float32)
    assert np.array_equal(oracle.rope(t, 0, 4, 64, 10000.0), t)
    r = oracle.rope(t, 37, 4, 64, 10000.0)
    assert not np.array_equal(r, t)
    for h in range(4):
        a, b = t[h * 64:(h + 1) * 64], r[h * 64:(h + 1) * 64]
        assert math.isclose(np.linalg.norm(a), np.linalg.norm(b), rel_tol=1e-5)


def test_rope_interleaved_pairs():
    t = np.zeros(8, np.float32)
    t[0] = 1.0  # pair (0, 1) rotates by pos * 1
    r = oracle.rope(t, 1, 1, 8, 10000.0)
    assert r[0] == np.float32(math.cos(1.0)) and r[1] == np.float32(math.sin(1.0))
    assert np.all(r[2:] == 0.0)


def test_kv_cache_append_tracking():
    c = oracle.KVCache(4, 2, 4)
    assert c.append(np.full(16, 1.0), np.full(16, 2.0), 2) == 2
    keys, vals = c.keys(), c.values()
    assert keys[0] == 1.0 and keys[15] == 1.0 and vals[0] == 2.0
    assert c.append(np.full(8, 3.0), np.full(8, 4.0), 1) == 3
    keys, vals = c.keys(), c.values()
    assert keys[0] == 1.0 and keys[15] == 1.0 and keys[16] == 3.0 and keys[23] == 3.0 and vals[16] == 4.0
    assert c.append(np.full(8, 5.0), np.full(8, 6.0), 1) == 4
    with pytest.raises(oracle.OracleError) as e:
        c.append(np.full(8, 5.0), np.full(8, 6.0), 1)
    assert e.value.code == 4 and "overflow" in str(e.value)


# ---- quant.rs vs gguf-py ----------------------------------------------------
def _gguf_dequant(blocks, qtype):
    import gguf.quants as gq
    from gguf import GGMLQuantizationType as T
    return gq.dequantize(blocks.reshape(-1), getattr(T, qtype)).reshape(-1).astype(np.float32)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q4k_dequant_bit_exact_vs_gguf_py(seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(256 * 64) * 0.02).astype(np.float32)
    blocks = synth.quantize_q4_k(x)
    # random scale bytes too, so every get_scale_min_k4 branch and bit is exercised
    blocks[:32, 4:16] = rng.integers(0, 256, size=(32, 12), dtype=np.uint8)
    ref = _gguf_dequant(blocks, "Q4_K")
    got = oracle.dequant_q4k(blocks)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("seed", [0, 1])
def test_q6k_dequant_bit_exact_vs_gguf_py(seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(256 * 64) * 0.02).astype(np.float32)
    blocks = synth.quantize_q6_k(x)
    blocks[:16, :208] = rng.integers(0, 256, size=(16, 208), dtype=np.uint8)
    ref = _gguf_dequant(blocks, "Q6_K")
    got = oracle.dequant_q6k(blocks)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q4k_subnormal_and_special_halves():
    blocks = np.zeros((4, 144), np.uint8)
    for i, (d, dm) in enumerate([(0x0001, 0x0002), (0x03FF, 0x8001), (0x7BFF, 0x0400), (0x3C00, 0x3C00)]):
        blocks[i, 0:2] = np.frombuffer(np.uint16(d).tobytes(), np.uint8)
        blocks[i, 2:4] = np.frombuffer(np.uint16(dm).tobytes(), np.uint8)
        blocks[i, 4:16] = 0xFF
        blocks[i, 16:] = np.arange(128, dtype=np.uint8) * 7
    ref = _gguf_dequant(blocks, "Q4_K")
    got = oracle.dequant_q4k(blocks)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


# ---- model level ------------------------------------------------------------
def test_tiny_forward_shape_and_kv(tiny_gguf):
    m = oracle.OracleModel(tiny_gguf)
    assert (m.vocab, m.hidden, m.layers, m.heads, m.kv_heads, m.ffn) == (512, 256, 2, 4, 2, 512)
    logits = m.forward([1, 2, 3], 0)
    assert logits.shape == (512,) and np.all(np.isfinite(logits))
    assert m.kv_len() == 3
    m.forward([4], 3)
    assert m.kv_len() == 4
    m.clear_kv_cache()
    assert m.kv_len() == 0


def test_tiny_forward_chunking_is_exact(tiny_gguf):
    # prefill in one call == prefill in chunks (per-token arithmetic is identical)
    m = oracle.OracleModel(tiny_gguf)
    ids = list(range(5, 25))
    a = m.forward(ids, 0)
    m.clear_kv_cache()
    for c in range(0, 20, 8):
        b = m.forward(ids[c:c + 8], c)
    assert np.array_equal(a, b)


def test_tiny_generate_semantics(tiny_gguf):
    m = oracle.OracleModel(tiny_gguf)
    prompt = synth.random_prompt(12, 512, seed=5).tolist()
    g = m.generate(prompt, 10, eos_id=None)
    assert len(g) == 10
    assert m.generate(prompt, 0, eos_id=None) == g[:1]  # the first token is always produced
    assert m.generate(prompt, 1, eos_id=None) == g[:1]
    # EOS is checked before the push, and never for the first token
    j = next(i for i in range(1, 10) if g[i] == g[3])
    assert m.generate(prompt, 10, eos_id=g[3]) == g[:j]
    assert m.generate(prompt, 10, eos_id=g[0]) == g[: next((i for i in range(1, 10) if g[i] == g[0]), 10)]
    with pytest.raises(oracle.OracleError):
        m.generate([], 4)


def test_kv_overflow_is_parse_error(tiny_gguf):
    m = oracle.OracleModel(tiny_gguf)
    m.forward(list(range(3, 3 + 250)), 0)
    with pytest.raises(oracle.OracleError) as e:
        m.forward(list(range(3, 13)), 250)
    assert e.value.code == 4
