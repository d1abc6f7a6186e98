"""Host-side decode logic on CPU: the tokenizer and argmax tests of src/tokenizer.rs,
and generate_tokens semantics (src/generate.rs:43-91) for both the Python loop and
the C++ loop of libammon_b200.so, driven by the CPU oracle model."""
import numpy as np
import pytest

import ammon_b200 as ab
from ammon_b200.tokenizer import BpeTokenizer  # the C++ tokenizer (ab_bpe_*)


@pytest.fixture(scope="module")
def toy(known):
    k = known["tokenizer"]
    return BpeTokenizer.from_parts(k["toy_vocab"], k["toy_scores"], k["max_token_length"])


def test_encodes_with_bos_dummy_prefix_and_merge(toy, known):
    k = known["tokenizer"]["encode_ab_bos"]
    ids = toy.encode(k["text"], k["bos"], k["eos"])
    assert ids[:3] == k["expect_prefix"]


def test_decode_strips_space_after_bos(toy, known):
    for prev, tok, want in known["tokenizer"]["decode_strip"]:
        assert toy.decode(prev, tok) == want


def test_argmax_picks_first_on_ties(known):
    k = known["tokenizer"]["argmax_ties"]
    assert ab.sample_argmax(k["logits"]) == k["expect"]
    assert ab.native_sample_argmax(k["logits"]) == k["expect"]


def test_byte_token_decode(known):
    k = known["tokenizer"]
    tok = BpeTokenizer.from_parts(k["byte_vocab"], [0.0] * len(k["byte_vocab"]), 8)
    prev, t, want = k["byte_decode"]
    assert tok.decode(prev, t) == want


def test_byte_fallback_and_eos():
    # llama2.c layout: ids 3..258 are the byte pieces <0x00>..<0xFF>
    vocab = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)] + [" ", "a"]
    tok = BpeTokenizer.from_parts(vocab, [0.0] * len(vocab), 8)
    ids = tok.encode("az", True, True)
    assert ids[0] == 1 and ids[-1] == 2
    assert ord("z") + 3 in ids  # unknown byte falls back to byte + 3
    assert tok.decode(0, ord("z") + 3) == "z"


def test_tokenizer_file_roundtrip(tmp_path, known):
    import struct

    k = known["tokenizer"]
    p = tmp_path / "tok.bin"
    with open(p, "wb") as f:
        f.write(struct.pack("<I", k["max_token_length"]))
        for s, sc in zip(k["toy_vocab"], k["toy_scores"]):
            b = s.encode()
            f.write(struct.pack("<fi", sc, len(b)) + b)
    tok = BpeTokenizer.from_path(str(p), len(k["toy_vocab"]))
    assert tok.encode("ab", True, False) == BpeTokenizer.from_parts(
        k["toy_vocab"], k["toy_scores"], 8).encode("ab", True, False)


def test_argmax_native_matches_python_random():
    rng = np.random.default_rng(0)
    for _ in range(20):
        x = rng.integers(-3, 3, size=257).astype(np.float32)
        assert ab.native_sample_argmax(x) == ab.sample_argmax(x.tolist())


class OracleModel:
    def __init__(self, orc, **cfg):
        self.m = orc.Model(**cfg)
        self.cfg = cfg

    def vocab_size(self):
        return self.cfg["vocab"]

    def max_seq_len(self):
        return self.cfg["seq"]

    def step(self, token, pos):
        return self.m.step(token, pos)


CFG = dict(dim=32, layers=2, heads=4, kv_heads=2, head_dim=8, hidden=48, vocab=97, seq=20,
           seed=4)


@pytest.mark.parametrize("loop", ["python", "native"])
def test_generate_tokens_matches_oracle_loop(orc, loop):
    prompt = [5, 9, 11]
    ref = orc.Model(**CFG)
    want, _ = ref.generate_tokens(prompt, 15)
    model = OracleModel(orc, **CFG)
    run = ab.generate_tokens if loop == "python" else ab.native_generate_tokens
    out = run(model, prompt, 15)
    assert out.tokens == want
    assert out.prompt_tokens == 3
    assert len(out.tokens) == 14 and out.tokens[:2] == [9, 11]
    # clamp to max_seq_len and stop_on
    model2 = OracleModel(orc, **CFG)
    out2 = run(model2, prompt, 1000)
    assert len(out2.tokens) == CFG["seq"] - 1
    model3 = OracleModel(orc, **CFG)
    stop = want[5]
    out3 = run(model3, prompt, 15, stop_on=stop)
    assert out3.tokens == want[:want.index(stop)]


@pytest.mark.parametrize("loop", ["python", "native"])
def test_generate_tokens_rejects_empty_prompt(orc, loop):
    model = OracleModel(orc, **CFG)
    run = ab.generate_tokens if loop == "python" else ab.native_generate_tokens
    with pytest.raises((ValueError, ab.AmmonError)):
        run(model, [], 10)


def test_generate_with_tokenizer(orc, toy):
    class Tiny:
        def vocab_size(self):
            return 7

        def max_seq_len(self):
            return 6

        def step(self, token, pos):
            l = np.zeros(7, np.float32)
            l[5] = 1.0  # always "ab"
            return l

    out = ab.generate(Tiny(), toy, "ab", ab.GenerateOptions(max_new_tokens=5))
    assert out.tokens[:2] == [6, 5]
    assert out.text.startswith("ab")
