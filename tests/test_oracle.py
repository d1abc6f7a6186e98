"""Pins the CPU oracle against the reference's own known answers and fp64 attention
oracle (Ammon tests/kernels.rs), before any GPU result is compared with it."""
import math

import numpy as np
import pytest


def test_embed_known_answer(orc, known):
    k = known["embed_gathers_selected_row"]
    assert orc.embed(np.array(k["table"], np.float32), k["token"]).tolist() == k["expect"]


def test_rope_identity_at_pos_zero(orc, known):
    k = known["rope_at_pos_zero_is_identity"]
    q = np.array(k["q"], np.float32)
    kc = np.array(k["k"], np.float32)
    orc.rope(q, kc, k["position"], k["theta"])
    assert q.ravel().tolist() == k["expect_q"]


@pytest.mark.parametrize("name", ["gemv_identity", "gemv_writes_cache_row_at_position"])
def test_gemv_known_answers(orc, known, name):
    k = known[name]
    out = np.zeros(k["out_shape"], np.float32)
    orc.gemv(np.array(k["x"], np.float32), np.array(k["w"], np.float32), out, k["position"])
    assert out.ravel().tolist() == k["expect"]


def test_swiglu_of_zero(orc, known):
    k = known["swiglu_of_zero_is_zero"]
    assert orc.swiglu(k["hb"], k["hb2"]).tolist() == k["expect"]


def test_rmsnorm_of_ones(orc, known):
    k = known["rmsnorm_matches_llama3_cuda_formula"]
    got = orc.rmsnorm(k["x"], k["w"])
    scale = 1.0 / np.sqrt(np.float32(1.0) + np.float32(1e-5))
    assert np.all(np.abs(got - scale) < k["tol"])
    x = np.array(k["x"], np.float32)
    orc.rmsnorm_inplace(x, k["w"])
    assert np.array_equal(x, got)


def test_add_known_answer(orc, known):
    k = known["tensor_add_into_is_elementwise"]
    assert orc.add(k["a"], k["b"]).tolist() == k["expect"]


def test_rope_store_known_answer(orc, known):
    k = known["rope_store_writes_rotated_k_from_scratch"]
    q = np.array(k["q"], np.float32)
    cache = np.zeros(k["cache_shape"], np.float32)
    orc.rope_store(q, np.array(k["k_proj"], np.float32), cache, k["position"], k["theta"])
    c, s = math.cos(k["angle"]), math.sin(k["angle"])
    rot = lambda a, b: (a * c - b * s, a * s + b * c)
    assert np.allclose(q.ravel(), rot(1.0, 2.0), atol=k["tol"], rtol=0)
    assert cache.ravel()[:2].tolist() == k["expect_k_row0"]
    assert np.allclose(cache.ravel()[2:], rot(3.0, 4.0), atol=k["tol"], rtol=0)


def test_cache_store_known_answer(orc, known):
    k = known["cache_store_writes_row_at_position"]
    cache = np.zeros(k["cache_shape"], np.float32)
    orc.cache_store(np.array(k["src"], np.float32), cache, k["position"])
    assert cache.ravel().tolist() == k["expect"]


def test_identity_matmul_then_cache_store(orc, known):
    k = known["semantic_gemv_then_cache_store_matches_serial_identity"]
    proj = orc.matmul(np.array(k["w"], np.float32), np.array(k["x"], np.float32))
    cache = np.zeros(k["cache_shape"], np.float32)
    orc.cache_store(proj, cache, k["position"])
    assert cache.ravel().tolist() == k["expect"]
    k2 = known["tensor_matmul_into_is_gemv"]
    assert orc.matmul(np.array(k2["w"], np.float32), np.array(k2["x"], np.float32)).tolist() == \
        k2["expect"]


def test_pseudo_random_matches_numpy_restatement(orc):
    from tests.golden.make_golden import pseudo_random

    for seed in (11, 12, 13):
        assert np.array_equal(orc.pseudo_random(500, seed), pseudo_random(500, seed))


def _case_inputs(orc, spec, c):
    qh, kvh, hd, seq = c["q_heads"], c["kv_heads"], c["head"], c["seq"]
    q = orc.pseudo_random(qh * hd, spec["q_seed"]).reshape(qh, hd)
    key = orc.pseudo_random(seq * kvh * hd, spec["key_seed"]).reshape(seq, kvh, hd)
    value = orc.pseudo_random(seq * kvh * hd, spec["value_seed"]).reshape(seq, kvh, hd)
    return q, key, value


def test_attention_oracles_match_reference_fp64(orc, known, attention_golden):
    """The reference's split/serial attention test (tests/kernels.rs:429-491), run on the
    oracle's restatements: both stay within 1e-4 of the fp64 oracle, whose committed
    fixture comes from an independent numpy restatement. Dead splits keep NaN poison."""
    spec = known["attention_cases"]
    for ci, c in enumerate(spec["cases"]):
        q, key, value = _case_inputs(orc, spec, c)
        assert np.array_equal(q.ravel(), attention_golden[f"case{ci}_q"])
        splits = -(-c["seq"] // 8)
        for pos in c["positions"]:
            want = attention_golden[f"case{ci}_pos{pos}"]
            f64 = orc.cpu_attention_f64(c["q_heads"], c["kv_heads"], c["head"], q, key, value, pos)
            assert np.allclose(f64, want, rtol=0, atol=1e-12)
            partial = np.full((c["q_heads"], splits, c["head"] + 2), np.nan, np.float32)
            orc.attention_partial(q, key, value, partial, pos)
            split = orc.attention_combine(partial, c["head"], pos).ravel()
            serial = orc.attention(q, key, value, c["seq"], pos).ravel()
            for name, got in (("split", split), ("serial", serial)):
                err = np.abs(got.astype(np.float64) - want).max()
                assert err < spec["tol"], (name, ci, pos, err)


def test_sample_argmax_first_on_ties(orc, known):
    k = known["tokenizer"]["argmax_ties"]
    assert orc.sample_argmax(k["logits"]) == k["expect"]


def test_bf16_rounding_is_nearest_even(orc):
    vals = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40, np.inf], np.float32)
    bits = orc.to_bf16_bits(vals)
    import torch

    ref = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, ref)


def test_normal_generator_moments(orc):
    w = orc.normal(1 << 20, 3, 7, 0.0, 0.02)
    assert abs(float(w.mean())) < 1e-4
    assert abs(float(w.std()) - 0.02) < 2e-4
    # deterministic and stream-separated
    assert np.array_equal(w[:100], orc.normal(100, 3, 7, 0.0, 0.02))
    assert not np.array_equal(w[:100], orc.normal(100, 3, 8, 0.0, 0.02))
    bits = orc.normal_bf16_bits(1000, 3, 7, 0.0, 0.02)
    assert np.array_equal(bits, orc.to_bf16_bits(w[:1000]))


def test_generate_tokens_semantics(orc):
    """src/generate.rs:43-91: prompt tokens after the first are forced and emitted; the loop
    runs max_new_tokens - 1 positions; stop_on ends it without emitting."""
    m = orc.Model(16, 1, 2, 1, 8, 32, 50, 12, seed=5)
    prompt = [3, 7, 9]
    toks, margins = m.generate_tokens(prompt, 10)
    assert len(toks) == 9 and toks[:2] == [7, 9]
    assert all(margins[:2] == -1.0) and all(margins[2:] >= 0)
    m.reset()
    toks2, _ = m.generate_tokens(prompt, 100)  # clamped to max_seq_len 12
    assert len(toks2) == 11 and toks2[:9] == toks
    m.reset()
    toks3, _ = m.generate_tokens(prompt, 10, stop_on=toks[4])
    assert toks3 == toks[:toks.index(toks[4])]
    with pytest.raises(ValueError):
        m.generate_tokens([], 10)


def test_model_step_matches_module_composition(orc):
    """or_model_step equals the explicit block sequence; bf16 mode stays near fp32."""
    cfg = dict(dim=64, layers=2, heads=4, kv_heads=2, head_dim=16, hidden=96, vocab=100, seq=16)
    a = orc.Model(**cfg, seed=9)
    b = orc.Model(**cfg, seed=9)
    for pos, tok in enumerate([5, 17, 3]):
        la = a.step(tok, pos)
        b.embed_token(tok)
        for layer in range(2):
            b.attention_block(layer, pos)
            b.ffn_block(layer)
        lb = b.classify()
        assert np.array_equal(la, lb)
    c = orc.Model(**cfg, seed=9, bf16=True)
    for pos, tok in enumerate([5, 17, 3]):
        lc = c.step(tok, pos)
    assert np.abs(lc - la).max() < 2e-2 * max(1.0, np.abs(la).max())
