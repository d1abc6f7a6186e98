"""Batched prefill: a prompt's positions of one cache stream run as the rows of a few passes
(rows sharing one [seq, kv_heads, head] cache, each attending over positions 0 .. its own),
against the oracle stepping the same prompt one token at a time (src/generate.rs:60-66).

Bars: fp32 within rel 1e-5 (logits and the cache rows), greedy ids bit-exact; bf16 within
2e-2 against the oracle with the same bf16 rounding points. Pass sizes cover the GEMV (<= 4
rows) and the tensor-core GEMM (5..256 rows) and a last pass shorter than the others."""
import numpy as np
import pytest

import ammon_b200 as ab

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
BF16_TOL = 2e-2


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def rt():
    r = ab.create_runtime(0)
    yield r
    r.synchronize()


def model(rt, orc, cfg, bf16=False, batch=1, seed=7):
    o = orc.Model(**cfg, bf16=bf16, seed=seed)
    g = ab.LlamaModel(rt, ab.LlamaConfig(cfg["dim"], cfg["layers"], cfg["heads"],
                                         cfg["kv_heads"], cfg["head_dim"], cfg["hidden"],
                                         cfg["vocab"], cfg["seq"], batch=batch,
                                         rope_theta=cfg.get("theta", 10000.0),
                                         dtype=ab.BF16 if bf16 else ab.F32))
    g.init_synthetic(seed, 0.02)
    return o, g


SMALL = dict(dim=128, layers=2, heads=4, kv_heads=2, head_dim=32, hidden=256, vocab=96, seq=64)


@pytest.mark.parametrize("rows", [256, 8, 4, 1])
def test_prefill_fp32_matches_the_token_loop(rt, orc, rows):
    """21 prompt tokens in passes of `rows` (21; 8+8+5; 4 x 5 + 1; 21 x 1): the last
    token's logits and greedy id, every cache row the prompt wrote, and the decode that
    follows all match the oracle's token-at-a-time run."""
    o, g = model(rt, orc, SMALL)
    prompt = np.random.default_rng(rows).integers(0, SMALL["vocab"], 21).tolist()
    g.set_prefill_rows(rows)
    logits, am = g.prefill(prompt)
    for pos, tok in enumerate(prompt):
        want = o.step(tok, pos)
    assert rel(logits, want) < FP32_TOL, rel(logits, want)
    assert am == orc.sample_argmax(want) == int(np.argmax(logits))
    # the cache the prompt left, against the same model stepped one token at a time
    o2, g2 = model(rt, orc, SMALL)
    for pos, tok in enumerate(prompt):
        g2.step(tok, pos)
    for layer in range(SMALL["layers"]):
        for got, ref in ((g.cache().layer(layer).key, g2.cache().layer(layer).key),
                         (g.cache().layer(layer).value, g2.cache().layer(layer).value)):
            a, b = got.read(), ref.read()
            assert rel(a[:21], b[:21]) < FP32_TOL
            assert not a[21:].any() and not b[21:].any()
    # decoding continues from the prefilled cache
    tok = am
    for pos in range(21, 25):
        got = g.step(tok, pos)
        want = o.step(tok, pos)
        assert rel(got, want) < FP32_TOL, (pos, rel(got, want))
        tok = orc.sample_argmax(want)
    g.close()
    g2.close()


@pytest.mark.parametrize("head,n", [(64, 40), (128, 40), (128, 150)])
def test_prefill_bf16_one_stream_of_a_batch(rt, orc, head, n):
    """bf16 weights and cache (tensor-core GEMM, tensor-core attention over the shared
    cache): stream 1 of 3 prefilled with n tokens in one pass (150: a 160-column GEMM)
    matches its oracle; the other streams' caches stay untouched, and a batched step
    afterwards serves stream 1 at position n next to fresh streams 0 and 2."""
    cfg = dict(dim=8 * head, layers=2, heads=8, kv_heads=2, head_dim=head, hidden=1024,
               vocab=640, seq=n + 56, theta=500000.0)
    o, g = model(rt, orc, cfg, bf16=True, batch=3, seed=13)
    prompt = np.random.default_rng(head).integers(0, cfg["vocab"], n).tolist()
    logits, am = g.prefill(prompt, stream=1)
    for pos, tok in enumerate(prompt):
        want = o.step(tok, pos)
    assert rel(logits, want) < BF16_TOL, rel(logits, want)
    assert am == int(np.argmax(logits))
    key = g.cache().layer(0).key.read()  # bf16 bits [3, seq, kv, head]
    assert not key[0].any() and not key[2].any() and key[1, :n].any() and not key[1, n:].any()
    fresh = [orc.Model(**cfg, bf16=True, seed=13) for _ in range(2)]
    toks = [5, am, 77]
    got, _ = g.step_batch(toks, [0, n, 0])
    assert rel(got[1], o.step(am, n)) < BF16_TOL
    assert rel(got[0], fresh[0].step(5, 0)) < BF16_TOL
    assert rel(got[2], fresh[1].step(77, 0)) < BF16_TOL
    g.close()


def test_prefill_at_an_offset_continues_a_sequence(rt, orc):
    """A second prompt chunk prefilled at pos0 = 9 after 9 decode steps: the same as the
    oracle stepping all 30 tokens."""
    o, g = model(rt, orc, SMALL)
    toks = np.random.default_rng(3).integers(0, SMALL["vocab"], 30).tolist()
    for pos in range(9):
        g.step(toks[pos], pos)
    g.set_prefill_rows(16)
    logits, am = g.prefill(toks[9:], pos0=9)
    for pos, tok in enumerate(toks):
        want = o.step(tok, pos)
    assert rel(logits, want) < FP32_TOL
    assert am == orc.sample_argmax(want)
    g.close()


@pytest.mark.parametrize("prompt,max_new,stop", [
    ([3, 9, 27, 81, 50], 40, None),     # prompt, then greedy picks to the step limit
    ([3, 9, 27, 81, 50], 4, None),      # the step limit ends inside the prompt
    ([3, 9, 27, 81, 50], 40, 27),       # a forced prompt id is the stop id
    ([3, 9, 27, 81, 50], 40, "gen"),    # a generated id is the stop id
    ([42], 12, None),                   # one prompt token
])
def test_generate_with_prefill_matches_the_reference_loop(rt, orc, prompt, max_new, stop):
    o, g = model(rt, orc, SMALL)
    if stop == "gen":
        full, _ = o.generate_tokens(prompt, max_new)
        stop = full[len(prompt) + 3]
        o.reset()
    want, _ = o.generate_tokens(prompt, max_new, stop_on=stop)
    got = g.generate(prompt, max_new, stop_on=stop)
    assert got.tokens == list(want), (got.tokens, list(want))
    g.close()


def test_prefill_argument_checks(rt, orc):
    o, g = model(rt, orc, SMALL, batch=2)
    with pytest.raises(ab.AmmonError, match="stream 2 out of range"):
        g.prefill([1, 2], stream=2)
    with pytest.raises(ab.AmmonError, match="pass max_seq_len"):
        g.prefill([1] * 10, pos0=60)
    with pytest.raises(ab.AmmonError, match="out of range for vocab"):
        g.prefill([1, 96])
    with pytest.raises(ab.AmmonError, match="at most 256 rows"):
        g.set_prefill_rows(257)
    with pytest.raises(ab.AmmonError, match="batch-1 model"):
        g.generate([1, 2], 5)
    g.close()


def test_text_generate_uses_the_prefill_loop(rt, orc, known):
    """generate() (src/generate.rs:93-118) with the C++ tokenizer: the library model runs its
    prefill loop and returns the same ids and text as the reference loop over the oracle."""
    from ammon_b200.tokenizer import BpeTokenizer as NativeBpeTokenizer

    k = known["tokenizer"]
    tok = NativeBpeTokenizer.from_parts(k["toy_vocab"], k["toy_scores"], k["max_token_length"])
    o, g = model(rt, orc, SMALL)

    class Oracle:
        def vocab_size(self):
            return SMALL["vocab"]

        def max_seq_len(self):
            return SMALL["seq"]

        def step(self, token, pos):
            return o.step(token, pos)

    opts = ab.GenerateOptions(max_new_tokens=20)
    want = ab.generate(Oracle(), tok, "abab ba", opts)
    got = ab.generate(g, tok, "abab ba", opts)
    assert got.tokens == want.tokens and got.text == want.text
    g.close()
