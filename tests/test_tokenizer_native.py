"""The C++ BPE tokenizer (ab_bpe_*, src/tokenizer.rs:18-178) on CPU: the reference's own
tokenizer tests (known answers), and identical ids / strings to the Python restatement of
the reference loop on seeded random vocabularies and texts (multi-byte characters, byte
fallback, ties between equal scores, ill-formed pieces read from a tokenizer.bin)."""
import struct

import numpy as np
import pytest

from ammon_b200.tokenizer import BpeTokenizer as NativeBpeTokenizer
from oracle.tokenizer_ref import BpeTokenizer


@pytest.fixture(scope="module")
def toy(known):
    k = known["tokenizer"]
    return NativeBpeTokenizer.from_parts(k["toy_vocab"], k["toy_scores"], k["max_token_length"])


def test_known_answers(toy, known):
    k = known["tokenizer"]
    e = k["encode_ab_bos"]
    assert toy.encode(e["text"], e["bos"], e["eos"])[:3] == e["expect_prefix"]
    for prev, tok, want in k["decode_strip"]:
        assert toy.decode(prev, tok) == want
    byte = NativeBpeTokenizer.from_parts(k["byte_vocab"], [0.0] * len(k["byte_vocab"]), 8)
    prev, t, want = k["byte_decode"]
    assert byte.decode(prev, t) == want
    assert toy.vocab_size() == len(k["toy_vocab"]) and toy.max_token_length() == 8


def _random_vocab(rng, n_merges):
    alphabet = list("abcdefgh ") + ["é", "ß", "€", "😀", "中"]
    vocab = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    vocab += alphabet
    pieces = set(vocab)
    while len(vocab) < 259 + len(alphabet) + n_merges:
        a = vocab[rng.integers(259, len(vocab))]
        b = vocab[rng.integers(259, len(vocab))]
        if len(a + b) <= 8 and a + b not in pieces:
            vocab.append(a + b)
            pieces.add(a + b)
    # scores from a small set: many exact ties between candidate pairs
    scores = [0.0] * 259 + [float(rng.integers(-3, 4)) for _ in range(len(vocab) - 259)]
    return vocab, scores


def _random_text(rng, n):
    chars = list("abcdefgh  ") + ["é", "ß", "€", "😀", "中", "z", "Q", "ü", "\n"]
    return "".join(chars[rng.integers(0, len(chars))] for _ in range(n))


@pytest.mark.parametrize("seed", range(6))
def test_matches_the_reference_loop_on_random_vocabularies(seed):
    rng = np.random.default_rng(seed)
    vocab, scores = _random_vocab(rng, 60)
    py = BpeTokenizer.from_parts(vocab, scores, 8)
    nat = NativeBpeTokenizer.from_parts(vocab, scores, 8)
    for _ in range(25):
        text = _random_text(rng, int(rng.integers(0, 40)))
        for bos, eos in ((True, False), (False, True), (True, True), (False, False)):
            assert nat.encode(text, bos, eos) == py.encode(text, bos, eos), text
    for prev in (0, 1, 7):
        for tok in list(range(len(vocab))) + [-1, len(vocab), 10 ** 6]:
            assert nat.decode(prev, tok) == py.decode(prev, tok), (prev, tok)


def test_byte_pieces_follow_from_str_radix():
    vocab = ["<unk>", "<s>", "</s>", "<0x41>", "<0x+41>", "<0x0041>", "<0x>", "<0x141>",
             "<0xG1>", "<0x 41>", "<0x4_1>", "<0xe9>", " <0x42>"]
    py = BpeTokenizer.from_parts(vocab, [0.0] * len(vocab), 8)
    nat = NativeBpeTokenizer.from_parts(vocab, [0.0] * len(vocab), 8)
    want = ["A", "A", "A", "<0x>", "<0x141>", "<0xG1>", "<0x 41>", "<0x4_1>", "é"]
    for i, w in enumerate(want):
        assert nat.decode(0, 3 + i) == w == py.decode(0, 3 + i), vocab[3 + i]
    assert nat.decode(1, 12) == "B" == py.decode(1, 12)  # space stripped after BOS, then a byte


def test_tokenizer_bin_with_ill_formed_pieces(tmp_path):
    """Pieces are read with String::from_utf8_lossy: each maximal ill-formed subpart becomes
    one U+FFFD, and encode finds the replaced piece by its bytes."""
    raw = [b"<unk>", b"<s>", b"</s>", b"a", b"\xff", b"\xe2\x82", b"x\xc3", b"\xe2\x82a",
           b"\xf0\x9f\x98", b" "]
    p = tmp_path / "tok.bin"
    with open(p, "wb") as f:
        f.write(struct.pack("<I", 7))
        for i, b in enumerate(raw):
            f.write(struct.pack("<fi", float(i % 3), len(b)) + b)
        f.write(b"trailing bytes are not read")
    nat = NativeBpeTokenizer.from_path(str(p), len(raw))
    want = [b.decode("utf-8", errors="replace") for b in raw]
    assert [nat.decode(0, i) for i in range(len(raw))] == want
    assert want[5] == "�" and want[7] == "�a" and want[8] == "�"
    py = BpeTokenizer.from_path(str(p), len(raw))
    for text in ["a", "�a", "a�", "a� a", "��a", ""]:
        assert nat.encode(text, True, True) == py.encode(text, True, True), text
    assert nat.max_token_length() == 7


def test_tokenizer_bin_errors(tmp_path):
    p = tmp_path / "short.bin"
    p.write_bytes(struct.pack("<I", 8) + struct.pack("<fi", 0.0, 3) + b"ab")
    with pytest.raises(Exception, match="read tokenizer piece 0"):
        NativeBpeTokenizer.from_path(str(p), 1)
    p.write_bytes(struct.pack("<I", 8) + struct.pack("<fi", 0.0, -1))
    with pytest.raises(Exception, match="negative length"):
        NativeBpeTokenizer.from_path(str(p), 1)
    with pytest.raises(Exception, match="open tokenizer"):
        NativeBpeTokenizer.from_path(str(tmp_path / "missing.bin"), 1)


def test_byte_fallback_outside_a_small_vocabulary_is_an_error():
    """The reference indexes vocab[id] for byte-fallback ids while merging (a panic when the
    vocabulary is smaller); the library returns an error instead."""
    vocab = ["<unk>", "<s>", "</s>", "a", " "]
    nat = NativeBpeTokenizer.from_parts(vocab, [0.0] * 5, 8)
    with pytest.raises(Exception, match="has no piece"):
        nat.encode("az", True, False)
    with pytest.raises(IndexError):
        BpeTokenizer.from_parts(vocab, [0.0] * 5, 8).encode("az", True, False)
    assert nat.encode("a", False, False) == [4, 3]


def test_long_text_encodes_fast():
    """O(n log n) merges: 200k characters in well under the reference loop's quadratic time."""
    import time

    rng = np.random.default_rng(9)
    vocab, scores = _random_vocab(rng, 200)
    nat = NativeBpeTokenizer.from_parts(vocab, scores, 8)
    text = _random_text(rng, 200_000)
    t0 = time.perf_counter()
    ids = nat.encode(text, True, True)
    assert time.perf_counter() - t0 < 5.0
    assert ids[0] == 1 and ids[-1] == 2
    # the head of the same text against the reference loop (quadratic, so a short slice)
    py = BpeTokenizer.from_parts(vocab, scores, 8)
    assert nat.encode(text[:300], True, True) == py.encode(text[:300], True, True)
