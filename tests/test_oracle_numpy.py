"""A second, independent restatement of the reference forward pass, in float64 numpy,
checked against the C++ oracle on whole models.

The oracle (oracle/oracle.cpp) is the checker of every GPU path; its parts are pinned
one by one (dequantisation against gguf-py, the reference's unit tests), but no output
of the reference's whole forward exists here (no Rust toolchain). This test restates
that forward from the reference source directly, independently of the oracle's code:

* weights: gguf-py's dequantisers (Q4_K / Q6_K) over the file's raw blocks;
* per layer (layer.rs:37-89): RMSNorm with eps 1e-6 (candle rms_norm: x / sqrt(mean(x^2)
  + eps) * w), Q / K / V = x W^T (matmul_transposed, gemm.rs:83-143), RoPE on interleaved
  pairs with freq = 1 / theta^(i / head_dim) for i = 0, 2, 4, ... and angle = position *
  freq (attention.rs:203-262), the KV cache append, causal softmax attention with repeat_kv
  for grouped heads and scale 1 / sqrt(head_dim) (attention.rs:297-435), the output
  projection and residual, then SwiGLU silu(g) * u (ffn.rs:54-109) and its residual;
* the final RMSNorm with the file's epsilon and the LM head on the last position
  (model.rs:936-1037); out-of-vocabulary ids embed as zeros (model.rs:847-864).

Computed in float64, it differs from the f32 oracle only by rounding; a logic slip in
either (a transposed weight, a wrong RoPE pair or frequency, a mask off by one, the wrong
epsilon) moves the logits by orders of magnitude more than the bar below."""
import numpy as np
import pytest

import oracle
from wcb import synth

# of max |logit|: the f32 oracle agrees to 1.2e-6 - 1.6e-6 on these models; a wrong RoPE
# frequency moves the logits by 4.8e-2, the final-norm epsilon used in the layers by 4.5e-3
REL = 2e-5


def _load(path):
    from gguf import GGUFReader
    import gguf.quants as gq
    r = GGUFReader(path)
    f = r.fields

    def field(name):
        x = f[name]
        return x.parts[x.data[0]][0]

    cfg = dict(vocab=int(field("llama.vocab_size")), hidden=int(field("llama.embedding_length")),
               layers=int(field("llama.block_count")), heads=int(field("llama.attention.head_count")),
               kv_heads=int(field("llama.attention.head_count_kv")),
               eps=float(field("llama.attention.layer_norm_rms_epsilon")),
               theta=float(field("llama.rope.freq_base")))
    w = {}
    for t in r.tensors:
        shape = tuple(int(d) for d in reversed(t.shape))  # GGUF ne is innermost first
        data = np.array(t.data)
        if int(t.tensor_type) in (0, 1):  # F32 / F16
            w[t.name] = data.astype(np.float64).reshape(shape)
        else:
            w[t.name] = gq.dequantize(data.reshape(-1), t.tensor_type).astype(np.float64).reshape(shape)
    return cfg, w


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def _rope(x, pos, theta):
    # x: [T, heads, hd]; pairs (2i, 2i+1) rotated by angle = pos * theta^-(2i / hd)
    hd = x.shape[-1]
    i = np.arange(0, hd, 2)
    freq = 1.0 / theta ** (i / hd)
    ang = pos[:, None] * freq[None, :]  # [T, hd/2]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


class NumpyModel:
    def __init__(self, path):
        self.cfg, self.w = _load(path)
        c = self.cfg
        self.hd = c["hidden"] // c["heads"]
        self.k = [np.zeros((0, c["kv_heads"], self.hd)) for _ in range(c["layers"])]
        self.v = [np.zeros((0, c["kv_heads"], self.hd)) for _ in range(c["layers"])]

    def forward(self, ids, position):
        c, w, hd = self.cfg, self.w, self.hd
        emb = w["token_embd.weight"]
        x = np.stack([emb[t] if t < c["vocab"] else np.zeros(c["hidden"]) for t in ids])
        T = len(ids)
        pos = np.arange(position, position + T, dtype=np.float64)
        n_rep = c["heads"] // c["kv_heads"]
        for l in range(c["layers"]):
            p = f"blk.{l}."
            h = _rms(x, w[p + "attn_norm.weight"], 1e-6)
            q = (h @ w[p + "attn_q.weight"].T).reshape(T, c["heads"], hd)
            k = (h @ w[p + "attn_k.weight"].T).reshape(T, c["kv_heads"], hd)
            v = (h @ w[p + "attn_v.weight"].T).reshape(T, c["kv_heads"], hd)
            q, k = _rope(q, pos, c["theta"]), _rope(k, pos, c["theta"])
            self.k[l] = np.concatenate([self.k[l], k])
            self.v[l] = np.concatenate([self.v[l], v])
            K = np.repeat(self.k[l], n_rep, axis=1)  # repeat_kv: query head h reads KV head h // n_rep
            V = np.repeat(self.v[l], n_rep, axis=1)
            s = np.einsum("thd,jhd->thj", q, K) / np.sqrt(hd)
            j = np.arange(K.shape[0])
            s = np.where(j[None, None, :] > (position + np.arange(T))[:, None, None], -np.inf, s)
            s = np.exp(s - s.max(axis=-1, keepdims=True))
            s /= s.sum(axis=-1, keepdims=True)
            att = np.einsum("thj,jhd->thd", s, V).reshape(T, c["hidden"])
            x = x + att @ w[p + "attn_output.weight"].T
            h = _rms(x, w[p + "ffn_norm.weight"], 1e-6)
            g = h @ w[p + "ffn_gate.weight"].T
            u = h @ w[p + "ffn_up.weight"].T
            x = x + ((g / (1.0 + np.exp(-g))) * u) @ w[p + "ffn_down.weight"].T
        last = _rms(x[-1], w["output_norm.weight"], c["eps"])
        head = w["output.weight"] if "output.weight" in w else emb
        return head @ last


@pytest.mark.parametrize("preset", ["tiny", "tiny_mix", "tiny_tp"])
def test_numpy_restatement_matches_the_oracle(model_dir, preset):
    path = synth.cached_model(preset, model_dir)
    o = oracle.OracleModel(path)
    n = NumpyModel(path)
    vocab = n.cfg["vocab"]
    prompt = synth.random_prompt(13, vocab, seed=21).tolist()
    steps = [(prompt, 0), ([5], 13), ([vocab + 7], 14), ([vocab - 1], 15)]  # incl. an out-of-vocabulary id
    for ids, pos in steps:
        got = np.asarray(o.forward(ids, pos), dtype=np.float64)
        want = n.forward(ids, pos)
        err = np.abs(got - want).max()
        assert err <= REL * np.abs(want).max(), (preset, pos, err, np.abs(want).max())
    o.close()


def _penalised_argmax(logits, history, rep):
    """sampling.rs:86-103 then :118-125: the penalty once per previous occurrence, then the
    argmax with the last maximum winning (Iterator::max_by)."""
    l = logits.copy()
    if rep != 1.0:
        for t in history:
            l[t] = l[t] / rep if l[t] > 0.0 else l[t] * rep
    m = l.max()
    return int(len(l) - 1 - np.argmax(l[::-1])), l, m


@pytest.mark.parametrize("preset,rep", [("tiny", 1.1), ("tiny_mix", 1.3)])
def test_oracle_generate_bookkeeping_against_numpy(model_dir, preset, rep):
    """generate() (model.rs:1322-1415) with the oracle's tokens fed back into the numpy
    restatement: every token is the numpy model's penalised argmax (or within f32 rounding
    of it), the history holds the sampled tokens only, and an EOS id ends the sequence
    before it is pushed, except as the first token."""
    path = synth.cached_model(preset, model_dir)
    o = oracle.OracleModel(path)
    n = NumpyModel(path)
    vocab = n.cfg["vocab"]
    prompt = synth.random_prompt(11, vocab, seed=22).tolist()
    toks = o.generate(prompt, 24, repetition_penalty=rep, eos_id=None)
    assert len(toks) == 24
    logits = n.forward(prompt, 0)
    history = []
    for i, t in enumerate(toks):
        if i > 0:
            logits = n.forward([toks[i - 1]], len(prompt) + i - 1)
        best, pen, m = _penalised_argmax(logits, history, rep)
        assert t == best or m - pen[t] <= REL * np.abs(pen).max(), (i, t, best, m - pen[t])
        history.append(t)
    # EOS: a token the sequence produces again later ends it at that later occurrence
    eos = next(t for i, t in enumerate(toks) if i >= 2)
    o.clear_kv_cache()
    cut = o.generate(prompt, 24, repetition_penalty=rep, eos_id=eos)
    first_eos = toks.index(eos, 1)  # the first token is never checked
    assert cut == toks[:first_eos]
    o.clear_kv_cache()
    first = o.generate(prompt, 24, repetition_penalty=rep, eos_id=toks[0])
    assert first[0] == toks[0] and len(first) >= 1  # an EOS as the first token is kept
    o.close()


# the 7B and 70B widths accumulate over longer rows (K up to 28672): 5e-6 - 8e-6 measured
REL_WIDE = 4e-5


@pytest.mark.parametrize("preset,layers", [("llama7b", 2), ("llama70b", 1)])
def test_numpy_restatement_matches_the_oracle_at_head_dim_128(model_dir, preset, layers):
    """The widths of the 7B (32 heads of 128, FFN 11008, the Q4_K_M mix with Q6_K attn_v /
    ffn_down in even layers) and 70B configurations (64 query / 8 KV heads of 128, FFN 28672),
    truncated to one or two layers and a 2048-token vocabulary so the check stays a CPU test:
    the oracle that checks the GPU paths at these widths against the numpy restatement."""
    path = synth.cached_model(preset, model_dir, num_layers=layers, vocab_size=2048, context_length=256)
    o = oracle.OracleModel(path)
    n = NumpyModel(path)
    assert n.hd == 128
    prompt = synth.random_prompt(13, 2048, seed=21).tolist()
    for ids, pos in [(prompt, 0), ([5], 13), ([2048 + 3], 14)]:
        got = np.asarray(o.forward(ids, pos), dtype=np.float64)
        want = n.forward(ids, pos)
        err = np.abs(got - want).max()
        assert err <= REL_WIDE * np.abs(want).max(), (preset, pos, err, np.abs(want).max())
    o.close()
