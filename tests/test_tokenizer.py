"""The C++ tokenizer behind wcb_tokenize / wcb_detokenize against the Python
restatement of crates/wasm-chord-core/src/tokenizer.rs (oracle/tokenizer.py):
the reference's own unit tests (tokenizer.rs:428-500) as known answers for
both, then identical ids and text on seeded random inputs with and without BPE
merges, duplicate vocabulary entries and merges, byte fallback, unknown ids,
ill-formed byte sequences in decode, Unicode whitespace trimming, and the
GGUF metadata path (tokenizer.ggml.tokens / merges / *_token_id); these run on
the CPU. The last test (gpu) runs generate(&str) through the device loop."""
import random

import gguf
import pytest

import wcb
from oracle.tokenizer import Tokenizer as Ref


def write_vocab(path, tokens, merges=None, bos=1, eos=2, unk=0):
    w = gguf.GGUFWriter(path, "llama")
    w.add_token_list(tokens)
    if merges is not None:
        w.add_token_merges(merges)
    w.add_bos_token_id(bos)
    w.add_eos_token_id(eos)
    w.add_unk_token_id(unk)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def reference_test_vocab():
    """create_test_tokenizer (tokenizer.rs:431-447): ids as list positions."""
    toks = [""] * 262
    toks[0], toks[1], toks[2] = "<unk>", "<s>", "</s>"
    for b in range(256):
        toks[b + 3] = "<0x%02X>" % b
    toks[259], toks[260], toks[261] = "▁hello", "▁world", "▁test"
    return toks


@pytest.fixture(scope="module")
def ref_pair(tmp_path_factory):
    toks = reference_test_vocab()
    p = write_vocab(str(tmp_path_factory.mktemp("tok") / "kat.gguf"), toks)
    return wcb.Tokenizer(p), Ref(toks, [])


def test_reference_unit_tests(ref_pair):
    t, r = ref_pair
    for tok in (t, r):
        enc = tok.encode("hello world", True)
        assert len(enc) >= 2 and enc[0] == 1            # test_encode_simple
        assert tok.encode("hello", True)[0] == 1         # test_special_tokens
        assert len(tok.encode("unknown", True)) > 1      # test_unknown_token (byte fallback)
    assert t.decode([259, 260], False) == r.decode([259, 260], False) == "hello world"  # test_decode_simple
    assert t.info() == (262, 1, 2, 0)                   # test_vocab_size
    assert t.encode("hello world") == r.encode("hello world") == [1, 259, 260]
    # the byte fallback of "unknown": ▁ is E2 96 81, then one byte per ASCII letter
    assert t.encode("unknown") == r.encode("unknown") == [1] + [b + 3 for b in "▁unknown".encode()]
    assert t.encode("") == r.encode("") == []


ALPHABET = list("abcdefgh ") + ["é", "ß", "中", "😀", "▁"]


def random_text(rng, n):
    return "".join(rng.choice(ALPHABET) for _ in range(n))


def bpe_vocab(rng):
    """A small BPE vocabulary: specials, byte tokens, single chars and merged pieces."""
    toks = ["<unk>", "<s>", "</s>"] + ["<0x%02X>" % b for b in range(256)]
    chars = ["▁"] + [c for c in ALPHABET if c not in (" ", "▁")]
    toks += chars
    merges = []
    pieces = list(chars)
    for _ in range(60):
        a, b = rng.choice(pieces), rng.choice(pieces)
        if len(a) + len(b) > 6:
            continue
        merges.append(f"{a} {b}")
        if a + b not in toks:
            toks.append(a + b)
            pieces.append(a + b)
    merges.append(merges[0])          # a repeated merge: its last rank counts
    merges.append("a b c")            # three parts: ignored
    toks.append(toks[300])            # a repeated token: the later id wins
    return toks, merges


@pytest.mark.parametrize("with_merges", [True, False])
def test_random_texts_match_oracle(tmp_path, with_merges):
    rng = random.Random(11 + with_merges)
    toks, merges = bpe_vocab(rng)
    p = write_vocab(str(tmp_path / "v.gguf"), toks, merges if with_merges else None)
    t = wcb.Tokenizer(p)
    r = Ref(toks, Ref.merges_from_strings(merges) if with_merges else [])
    for i in range(200):
        text = random_text(rng, rng.randint(1, 40))
        ids = t.encode(text, True)
        assert ids == r.encode(text, True), text
        assert t.decode(ids, True) == r.decode(ids, True)
        assert t.decode(ids, False) == r.decode(ids, False)
    t.set_special(False, True)
    r.add_bos, r.add_eos = False, True
    assert t.encode("abc ab", True) == r.encode("abc ab", True)
    assert t.encode("abc ab", True)[-1] == 2


def test_decode_edge_cases(tmp_path):
    toks = reference_test_vocab() + ["<0x>", "<0x+4A>", "<0x1FF>", " 　", "x ", "\x1c"]
    p = write_vocab(str(tmp_path / "e.gguf"), toks)
    t, r = wcb.Tokenizer(p), Ref(toks, [])
    rng = random.Random(5)
    cases = [
        [0xC3 + 3, 0xA9 + 3],              # é from two byte tokens
        [0xE2 + 3, 0x28 + 3, 0xA1 + 3],    # ill-formed: E2 then '(' then a stray continuation
        [0xF0 + 3, 0x9F + 3, 0x98 + 3],    # truncated 4-byte sequence at the end
        [0xED + 3, 0xA0 + 3, 0x80 + 3],    # a surrogate encoding
        [0xC0 + 3, 0x80 + 3, 0xFF + 3],    # never-valid bytes
        [262, 263, 264, 265, 266, 267],    # odd byte-looking tokens, Unicode whitespace, U+001C
        [1, 2, 0, 259, 99999],             # specials and an unknown id
    ]
    cases += [[rng.randrange(0, 268) for _ in range(rng.randint(1, 12))] for _ in range(300)]
    for ids in cases:
        for skip in (True, False):
            assert t.decode(ids, skip) == r.decode(ids, skip), (ids, skip)


def test_invalid_utf8_is_rejected(ref_pair):
    t, _ = ref_pair
    with pytest.raises(wcb.WcbError):
        t.encode_bytes(b"ab\xff")


def test_missing_vocabulary_is_a_parse_error(tmp_path):
    w = gguf.GGUFWriter(str(tmp_path / "n.gguf"), "llama")
    w.add_uint32("llama.block_count", 1)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(wcb.WcbError, match="tokenizer.ggml.tokens"):
        wcb.Tokenizer(str(tmp_path / "n.gguf"))


@pytest.mark.gpu
def test_generate_text_matches_oracle(tiny_gguf, gpu, tmp_path):
    """Model::generate(&str) (model.rs:1322-1415) through wcb_generate_text: the
    tokenizer's ids into the device generate loop, the whole sequence decoded."""
    import oracle
    rng = random.Random(3)
    toks, merges = bpe_vocab(rng)
    toks = (toks + ["▁p%d" % i for i in range(512)])[:512]  # the tiny model's vocabulary size
    p = write_vocab(str(tmp_path / "t.gguf"), toks, merges)
    tok, ref = wcb.Tokenizer(p), Ref(toks, Ref.merges_from_strings(merges))
    m = wcb.Model.load_from_gguf(tiny_gguf)
    o = oracle.OracleModel(tiny_gguf)
    for prompt in ("abc déf 中", "h g f e d c b a", "😀 ab"):
        cfg = wcb.GenerationConfig(max_tokens=20, temperature=0.0, repetition_penalty=1.1)
        ids = ref.encode(prompt, True)
        want = ref.decode(ids + o.generate(ids, 20, repetition_penalty=1.1, eos_id=ref.eos), True)
        assert m.generate_text(prompt, tok, cfg) == want
    m.close()
