"""GPU ports of the reference's kernel tests (tests/kernels.rs), through the C ABI,
plus bit-exact parity of the serial-order kernels with the CPU oracle."""
import math

import numpy as np
import pytest

import ammon_b200 as ab
from ammon_b200 import kernels as K

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    r = ab.create_runtime(0)
    yield r
    r.synchronize()


def step_buf(rt, token, position):
    p = ab.DecodeStep.parcel(rt)
    rt.deposit(p, [ab.DecodeStep(token, position)])
    return p


def run(scheme, t):
    scheme.submit()
    return t.read()


def test_embed_gathers_selected_row(rt, known):
    k = known["embed_gathers_selected_row"]
    table = ab.Tensor.from_f32(rt, (2, 2), k["table"])
    x = ab.Tensor.from_f32(rt, (2,), [0.0, 0.0])
    s = rt.scheme()
    K.EmbedKernel.prepare(rt).record(s, "embed", table, step_buf(rt, k["token"], 0), x).over_1d(2)
    assert run(s, x).tolist() == k["expect"]


def test_rope_at_pos_zero_is_identity(rt, known):
    k = known["rope_at_pos_zero_is_identity"]
    q = ab.Tensor.from_f32(rt, (2, 2), k["q"])
    kc = ab.Tensor.from_f32(rt, (1, 2, 2), k["k"])
    s = rt.scheme()
    K.RopeKernel.prepare(rt).record(s, "rope", q, kc, step_buf(rt, 0, 0), k["theta"])
    assert run(s, q).ravel().tolist() == k["expect_q"]


@pytest.mark.parametrize("name", ["gemv_identity", "gemv_writes_cache_row_at_position"])
def test_gemv_known_answers(rt, known, name):
    k = known[name]
    x = ab.Tensor.from_f32(rt, (2,), k["x"])
    w = ab.Tensor.from_f32(rt, (2, 2), k["w"])
    out = ab.Tensor.zeros(rt, k["out_shape"])
    s = rt.scheme()
    K.GemvKernel.prepare(rt).record(s, "gemv", x, w, out, step_buf(rt, 0, k["position"]))
    assert run(s, out).ravel().tolist() == k["expect"]


def test_swiglu_of_zero_is_zero(rt, known):
    k = known["swiglu_of_zero_is_zero"]
    hb = ab.Tensor.from_f32(rt, (2,), k["hb"])
    hb2 = ab.Tensor.from_f32(rt, (2,), k["hb2"])
    s = rt.scheme()
    K.SwigluKernel.prepare(rt).record(s, "swiglu", hb, hb2)
    assert run(s, hb).tolist() == k["expect"]


def test_rmsnorm_matches_llama3_cuda_formula(rt, known):
    k = known["rmsnorm_matches_llama3_cuda_formula"]
    x = ab.Tensor.from_f32(rt, (4,), k["x"])
    w = ab.Tensor.from_f32(rt, (4,), k["w"])
    o = ab.Tensor.zeros(rt, (4,))
    s = rt.scheme()
    K.RmsnormKernel.prepare(rt).record(s, "rms", x, w, o)
    scale = 1.0 / math.sqrt(1.0 + 1e-5)
    assert np.all(np.abs(run(s, o) - scale) < k["tol"])


def test_deposit_feeds_embed_without_rerecord(rt, known):
    k = known["deposit_feeds_embed_without_rerecord"]
    table = ab.Tensor.from_f32(rt, (2, 2), k["table"])
    step = step_buf(rt, 0, 0)
    x = ab.Tensor.from_f32(rt, (2,), [0.0, 0.0])
    worker = rt.scheme()
    K.EmbedKernel.prepare(rt).record(worker, "embed", table, step, x)
    for token, want in zip(k["tokens"], k["expect"]):
        rt.deposit(step, [ab.DecodeStep(token, 0)])
        worker.submit()
        assert x.read().tolist() == want
    stats = worker.replay_stats()
    assert stats.records - stats.specialization_promotions == k["records_minus_promotions"]
    assert stats.replays == 2


def test_tensor_add_into_is_elementwise(rt, known):
    k = known["tensor_add_into_is_elementwise"]
    a = ab.Tensor.from_f32(rt, (2,), k["a"])
    b = ab.Tensor.from_f32(rt, (2,), k["b"])
    out = ab.Tensor.zeros(rt, (2,))
    s = rt.scheme()
    K.TensorKernels.prepare(rt).add_into(s, "add", a, b, out)
    assert run(s, out).tolist() == k["expect"]


def test_rope_store_writes_rotated_k_from_scratch(rt, known):
    k = known["rope_store_writes_rotated_k_from_scratch"]
    q = ab.Tensor.from_f32(rt, (1, 2), k["q"])
    kp = ab.Tensor.from_f32(rt, (2,), k["k_proj"])
    kc = ab.Tensor.zeros(rt, k["cache_shape"])
    s = rt.scheme()
    K.RopeStoreKernel.prepare(rt).record(s, "rope_store", q, kp, kc, step_buf(rt, 0, 1),
                                         k["theta"])
    s.submit()
    q_out, k_out = q.read().ravel(), kc.read().ravel()
    c, sn = math.cos(k["angle"]), math.sin(k["angle"])
    rot = lambda a, b: (a * c - b * sn, a * sn + b * c)
    assert np.allclose(q_out, rot(1.0, 2.0), atol=k["tol"], rtol=0)
    assert k_out[:2].tolist() == k["expect_k_row0"]
    assert np.allclose(k_out[2:], rot(3.0, 4.0), atol=k["tol"], rtol=0)


def test_cache_store_writes_row_at_position(rt, known):
    k = known["cache_store_writes_row_at_position"]
    src = ab.Tensor.from_f32(rt, (2,), k["src"])
    dst = ab.Tensor.zeros(rt, k["cache_shape"])
    s = rt.scheme()
    K.CacheStoreKernel.prepare(rt).record(s, "store", src, dst, step_buf(rt, 0, k["position"]))
    assert run(s, dst).ravel().tolist() == k["expect"]


def test_semantic_gemv_then_cache_store_matches_serial_identity(rt, known):
    k = known["semantic_gemv_then_cache_store_matches_serial_identity"]
    x = ab.Tensor.from_f32(rt, (2,), k["x"])
    w = ab.Tensor.from_f32(rt, (2, 2), k["w"])
    scratch = ab.Tensor.zeros(rt, (k["scratch_len"],))
    cache = ab.Tensor.zeros(rt, k["cache_shape"])
    s = rt.scheme()
    proj = scratch.narrow(0, 0, 2)
    K.TensorKernels.prepare(rt).matmul_into(s, "wv", w, x, proj)
    K.CacheStoreKernel.prepare(rt).record(s, "wv_store", proj, cache,
                                          step_buf(rt, 0, k["position"]))
    assert run(s, cache).ravel().tolist() == k["expect"]


def test_tensor_matmul_into_is_gemv(rt, known):
    k = known["tensor_matmul_into_is_gemv"]
    w = ab.Tensor.from_f32(rt, (2, 2), k["w"])
    x = ab.Tensor.from_f32(rt, (2,), k["x"])
    out = ab.Tensor.zeros(rt, (2,))
    s = rt.scheme()
    K.TensorKernels.prepare(rt).matmul_into(s, "gemv", w, x, out)
    assert run(s, out).tolist() == k["expect"]


def _attention_case(rt, orc, spec, c, golden, ci):
    qh, kvh, hd, seq = c["q_heads"], c["kv_heads"], c["head"], c["seq"]
    splits = -(-seq // ab.ATTENTION_SPLIT)
    q_host = orc.pseudo_random(qh * hd, spec["q_seed"])
    key_host = orc.pseudo_random(seq * kvh * hd, spec["key_seed"])
    value_host = orc.pseudo_random(seq * kvh * hd, spec["value_seed"])
    q = ab.Tensor.from_f32(rt, (qh, hd), q_host)
    key = ab.Tensor.from_f32(rt, (seq, kvh, hd), key_host)
    value = ab.Tensor.from_f32(rt, (seq, kvh, hd), value_host)
    pk = K.AttentionPartialKernel.prepare(rt)
    ck = K.AttentionCombineKernel.prepare(rt)
    sk = K.AttentionKernel.prepare(rt)
    for pos in c["positions"]:
        step = step_buf(rt, 0, pos)
        # dead splits keep NaN; the combine must never read them
        partial = ab.Tensor.from_array(rt, np.full((qh, splits, hd + 2), np.nan, np.float32))
        split_out = ab.Tensor.zeros(rt, (qh, hd))
        serial_out = ab.Tensor.zeros(rt, (qh, hd))
        att = ab.Tensor.zeros(rt, (qh, seq))
        s = rt.scheme()
        pk.record(s, "attn_partial", q, key, value, partial, step)
        ck.record(s, "attn_combine", partial, split_out, step)
        sk.record(s, "attn_serial", q, att, serial_out, key, value, step)
        s.submit()
        want = golden[f"case{ci}_pos{pos}"]
        for name, got in (("split", split_out.read().ravel()), ("serial", serial_out.read().ravel())):
            err = np.abs(got.astype(np.float64) - want).max()
            assert err < spec["tol"], (name, c, pos, err)


def test_split_attention_matches_reference_across_split_boundaries(rt, orc, known,
                                                                   attention_golden):
    spec = known["attention_cases"]
    _attention_case(rt, orc, spec, spec["cases"][0], attention_golden, 0)


def test_split_attention_matches_reference_for_gqa_and_head_widths(rt, orc, known,
                                                                   attention_golden):
    spec = known["attention_cases"]
    for ci in range(1, len(spec["cases"])):
        _attention_case(rt, orc, spec, spec["cases"][ci], attention_golden, ci)


# ---- bit-exact parity of the serial-order kernels with the oracle --------------------------
def test_rmsnorm_bit_exact_vs_oracle(rt, orc):
    for dim in (288, 4096, 777):
        x_host = orc.normal(dim, 1, 100 + dim, 0.0, 1.0)
        w_host = orc.normal(dim, 1, 200 + dim, 1.0, 0.01)
        x = ab.Tensor.from_array(rt, x_host)
        w = ab.Tensor.from_array(rt, w_host)
        o = ab.Tensor.zeros(rt, (dim,))
        s = rt.scheme()
        K.RmsnormKernel.prepare(rt).record(s, "rms", x, w, o)
        K.RmsnormInplaceKernel.prepare(rt).record(s, "rms_inplace", x, w)
        s.submit()
        want = orc.rmsnorm(x_host, w_host)
        assert np.array_equal(o.read(), want)
        assert np.array_equal(x.read(), want)


def test_gemv_serial_bit_exact_vs_oracle(rt, orc):
    n, d, seq, pos = 300, 70, 5, 3
    x_host = orc.normal(n, 2, 1, 0.0, 1.0)
    w_host = orc.normal(d * n, 2, 2, 0.0, 0.05).reshape(d, n)
    out = ab.Tensor.zeros(rt, (seq, d))
    s = rt.scheme()
    K.GemvKernel.prepare(rt).record(s, "gemv", ab.Tensor.from_array(rt, x_host),
                                    ab.Tensor.from_array(rt, w_host), out, step_buf(rt, 0, pos))
    s.submit()
    want = np.zeros((seq, d), np.float32)
    orc.gemv(x_host, w_host, want, pos)
    assert np.array_equal(out.read(), want)


def test_embed_bf16_table_and_batch(rt, orc):
    vocab, dim = 50, 72
    bits = orc.normal_bf16_bits(vocab * dim, 3, 1, 0.0, 0.02).reshape(vocab, dim)
    table = ab.Tensor.from_array(rt, bits, ab.BF16)
    steps = ab.DecodeStep.parcel(rt, 3)
    toks = [7, 0, 49]
    rt.deposit(steps, [ab.DecodeStep(t, 0) for t in toks])
    x = ab.Tensor.zeros(rt, (3, dim))
    s = rt.scheme()
    ab.Embedding(rt).record(s, table, steps, x)
    s.submit()
    assert np.array_equal(x.read(), orc.from_bf16_bits(bits[toks].ravel()).reshape(3, dim))


def test_embed_flags_out_of_range_token(rt):
    table = ab.Tensor.from_f32(rt, (2, 4), np.arange(8, dtype=np.float32))
    x = ab.Tensor.zeros(rt, (4,))
    s = rt.scheme()
    ab.Embedding(rt).record(s, table, step_buf(rt, 5, 0), x)
    s.submit()
    with pytest.raises(ab.DeviceError):
        rt.synchronize()
    rt.synchronize()  # flag cleared
