"""Parity of the standalone op entry points the per-op and split-attention workloads time:
RmsNorm rows in f32 and bf16 (bit-exact against the oracle's reduction order), RoPE in its
batched form (one DecodeStep per q row; identical to one launch per row), and the fused
flash-decoding entry ab_kernel_attention_decode against a float64 reference on the same
bf16/f32 cache values, with a different position per batch row."""
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


def steps(rt, pairs):
    p = ab.DecodeStep.parcel(rt, len(pairs))
    rt.deposit(p, [ab.DecodeStep(t, pos) for t, pos in pairs])
    return p


@pytest.mark.parametrize("xbf16,wbf16,obf16", [(False, False, False), (True, True, True),
                                               (False, True, True), (True, False, False)])
def test_rmsnorm_rows_bit_exact_vs_oracle(rt, orc, xbf16, wbf16, obf16):
    rows, dim = 5, 1000
    x_f = orc.normal(rows * dim, 4, 1, 0.0, 1.0).reshape(rows, dim)
    w_f = orc.normal(dim, 4, 2, 1.0, 0.01)
    if xbf16:
        x_f = orc.round_bf16(x_f)
    if wbf16:
        w_f = orc.round_bf16(w_f)
    want = np.stack([orc.rmsnorm(x_f[r], w_f) for r in range(rows)])
    xt = (ab.Tensor.from_array(rt, orc.to_bf16_bits(x_f).reshape(rows, dim), ab.BF16) if xbf16
          else ab.Tensor.from_array(rt, x_f))
    wt = (ab.Tensor.from_array(rt, orc.to_bf16_bits(w_f), ab.BF16) if wbf16
          else ab.Tensor.from_array(rt, w_f))
    o = ab.Tensor.zeros(rt, (rows, dim), ab.BF16 if obf16 else ab.F32)
    s = rt.scheme()
    K.RmsnormKernel.prepare(rt).record(s, "rms", xt, wt, o)
    if xbf16 == obf16:
        K.RmsnormInplaceKernel.prepare(rt).record(s, "rms_inplace", xt, wt)
    s.submit()
    got = o.read_f32() if obf16 else o.read()
    exp = orc.round_bf16(want) if obf16 else want
    assert np.array_equal(got, exp)
    if xbf16 == obf16:
        assert np.array_equal(xt.read_f32() if xbf16 else xt.read(), exp)


def test_rope_batched_rows_equal_single_row_launches(rt, orc):
    B, H, KV, hd, seq, theta = 6, 4, 2, 16, 12, 500000.0
    q_host = orc.normal(B * H * hd, 5, 1, 0.0, 1.0).reshape(B, H, hd)
    k_host = orc.normal(seq * KV * hd, 5, 2, 0.0, 1.0).reshape(seq, KV, hd)
    positions = [0, 3, 11, 2, 7, 5]
    # batched: one launch, shared k
    q = ab.Tensor.from_array(rt, q_host)
    k = ab.Tensor.from_array(rt, k_host)
    s = rt.scheme()
    K.RopeKernel.prepare(rt).record(s, "rope", q, k, steps(rt, [(0, p) for p in positions]),
                                    theta)
    s.submit()
    qb, kb = q.read(), k.read()
    # one launch per row
    k1 = ab.Tensor.from_array(rt, k_host)
    q_rows = []
    for b, p in enumerate(positions):
        qr = ab.Tensor.from_array(rt, q_host[b])
        s1 = rt.scheme()
        K.RopeKernel.prepare(rt).record(s1, "rope", qr, k1, steps(rt, [(0, p)]), theta)
        s1.submit()
        q_rows.append(qr.read())
    assert np.array_equal(qb, np.stack(q_rows))
    assert np.array_equal(kb, k1.read())
    # and the oracle's rotation at these small positions
    qo, ko = q_host.copy(), k_host.copy()
    for b, p in enumerate(positions):
        orc.rope(qo[b], ko, p, theta)
    assert np.abs(qb - qo).max() < 1e-5 and np.abs(kb - ko).max() < 1e-5
    # untouched k rows stay untouched
    untouched = [r for r in range(seq) if r not in positions]
    assert np.array_equal(kb[untouched], k_host[untouched])


def test_rope_batched_per_row_caches(rt, orc):
    B, H, KV, hd, seq, theta = 3, 2, 1, 8, 4, 10000.0
    q_host = orc.normal(B * H * hd, 6, 1, 0.0, 1.0).reshape(B, H, hd)
    k_host = orc.normal(B * seq * KV * hd, 6, 2, 0.0, 1.0).reshape(B, seq, KV, hd)
    positions = [1, 1, 3]
    q = ab.Tensor.from_array(rt, q_host)
    k = ab.Tensor.from_array(rt, k_host)
    s = rt.scheme()
    K.RopeKernel.prepare(rt).record(s, "rope", q, k, steps(rt, [(0, p) for p in positions]),
                                    theta)
    s.submit()
    qo, ko = q_host.copy(), k_host.copy()
    for b, p in enumerate(positions):
        orc.rope(qo[b], ko[b], p, theta)
    assert np.abs(q.read() - qo).max() < 1e-5 and np.abs(k.read() - ko).max() < 1e-5


def _attention_ref(q, kc, vc, pos, kv_heads):
    """float64 softmax(q.K / sqrt(hd)) V over positions 0..pos, GQA heads h -> h // group."""
    heads, hd = q.shape
    g = heads // kv_heads
    out = np.zeros((heads, hd))
    for h in range(heads):
        kk = kc[:pos + 1, h // g].astype(np.float64)
        vv = vc[:pos + 1, h // g].astype(np.float64)
        sc = kk @ q[h].astype(np.float64) / np.sqrt(hd)
        p = np.exp(sc - sc.max())
        out[h] = (p / p.sum()) @ vv
    return out


@pytest.mark.parametrize("kv_bf16,hd,heads,kv_heads", [(True, 128, 32, 8), (True, 64, 8, 8),
                                                       (False, 64, 12, 12), (False, 128, 4, 1)])
def test_fused_attention_entry_matches_float64(rt, orc, kv_bf16, hd, heads, kv_heads):
    B, seq = 3, 700
    positions = [699, 0, 333]
    q_host = orc.normal(B * heads * hd, 2, 1, 0.0, 1.0).reshape(B, heads, hd)
    k_f = orc.normal(B * seq * kv_heads * hd, 2, 2, 0.0, 1.0).reshape(B, seq, kv_heads, hd)
    v_f = orc.normal(B * seq * kv_heads * hd, 2, 3, 0.0, 1.0).reshape(B, seq, kv_heads, hd)
    if kv_bf16:
        k_f, v_f = orc.round_bf16(k_f), orc.round_bf16(v_f)
        kc = ab.Tensor.from_array(rt, orc.to_bf16_bits(k_f).reshape(k_f.shape), ab.BF16)
        vc = ab.Tensor.from_array(rt, orc.to_bf16_bits(v_f).reshape(v_f.shape), ab.BF16)
    else:
        kc, vc = ab.Tensor.from_array(rt, k_f), ab.Tensor.from_array(rt, v_f)
    q = ab.Tensor.from_array(rt, q_host)
    out = ab.Tensor.zeros(rt, (B, heads * hd))
    s = rt.scheme()
    K.AttentionDecodeKernel.prepare(rt).record(s, "attn", q, kc, vc, out,
                                               steps(rt, [(0, p) for p in positions]))
    for _ in range(2):  # the second replay reuses the reset tickets
        s.submit()
        got = out.read().reshape(B, heads, hd)
        for b, p in enumerate(positions):
            want = _attention_ref(q_host[b], k_f[b], v_f[b], p, kv_heads)
            err = np.abs(got[b] - want).max() / np.abs(want).max()
            # bf16 K/V run on the mma path (Q and P as bf16 hi + lo pairs); f32 K/V in fp32
            assert err < (1e-4 if kv_bf16 else 1e-5), (b, p, err)
    s.close()


@pytest.mark.parametrize("kv_bf16,hd,heads,kv_heads,rows,p0", [
    (True, 128, 32, 8, 100, 317),   # the prompt kernel (64 queries per K/V tile), G = 4
    (True, 64, 8, 8, 70, 0),        # G = 1, positions from 0
    (True, 128, 16, 2, 16, 50),     # G = 8, the smallest batch the prompt kernel takes
    (True, 64, 8, 4, 9, 200),       # fewer rows: the split decode kernel over one cache
    (False, 64, 8, 2, 40, 90),      # f32 K/V: the warp kernel over one cache
])
def test_fused_attention_shared_cache_matches_float64(rt, orc, kv_bf16, hd, heads, kv_heads,
                                                      rows, p0):
    """Rows that are consecutive positions of one sequence, over one [seq, kv, head] cache:
    row b attends over positions 0 .. p0 + b (causal), against float64."""
    seq = p0 + rows + 37
    q_host = orc.normal(rows * heads * hd, 8, 1, 0.0, 1.0).reshape(rows, heads, hd)
    k_f = orc.normal(seq * kv_heads * hd, 8, 2, 0.0, 1.0).reshape(seq, kv_heads, hd)
    v_f = orc.normal(seq * kv_heads * hd, 8, 3, 0.0, 1.0).reshape(seq, kv_heads, hd)
    if kv_bf16:
        k_f, v_f = orc.round_bf16(k_f), orc.round_bf16(v_f)
        kc = ab.Tensor.from_array(rt, orc.to_bf16_bits(k_f).reshape(k_f.shape), ab.BF16)
        vc = ab.Tensor.from_array(rt, orc.to_bf16_bits(v_f).reshape(v_f.shape), ab.BF16)
    else:
        kc, vc = ab.Tensor.from_array(rt, k_f), ab.Tensor.from_array(rt, v_f)
    q = ab.Tensor.from_array(rt, q_host)
    for out_dt in (ab.F32, ab.BF16):
        out = ab.Tensor.zeros(rt, (rows, heads * hd), out_dt)
        s = rt.scheme()
        K.AttentionDecodeKernel.prepare(rt).record(s, "attn", q, kc, vc, out,
                                                   steps(rt, [(0, p0 + b) for b in range(rows)]))
        s.submit()
        got = (out.read_f32() if out_dt == ab.BF16 else out.read()).reshape(rows, heads, hd)
        worst = 0.0
        for b in range(rows):
            want = _attention_ref(q_host[b], k_f, v_f, p0 + b, kv_heads)
            worst = max(worst, float(np.abs(got[b] - want).max() / np.abs(want).max()))
        tol = 1e-2 if out_dt == ab.BF16 else (1e-4 if kv_bf16 else 1e-5)
        assert worst < tol, (out_dt, worst)
        s.close()


def test_fused_attention_entry_validation(rt):
    q = ab.Tensor.zeros(rt, (2, 3, 64))
    kc = ab.Tensor.zeros(rt, (2, 16, 1, 64))
    out = ab.Tensor.zeros(rt, (2, 3 * 64))
    s = rt.scheme()
    with pytest.raises(ab.ValidationError, match="query_heads / kv_heads"):
        K.AttentionDecodeKernel.prepare(rt).record(s, "attn", q, kc, kc, out,
                                                   steps(rt, [(0, 0), (0, 0)]))
    assert s.ir_node_count() == 0
