"""Parity of the fused decode path (modules and model) with the CPU oracle.

Tolerances (stated by the north star): fp32 activations within rel 1e-5, measured as
max |gpu - oracle| / max |oracle| over the tensor; bf16 configs within 2e-2 against the
oracle run with the same bf16 rounding points; integer results (gathered rows, cache
positions, greedy ids of fp32 configs) bit-exact."""
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


def make_pair(rt, orc, bf16=False, batch=1, seed=7, **cfg):
    base = dict(dim=128, layers=2, heads=4, kv_heads=2, head_dim=32, hidden=256, vocab=96,
                seq=48, theta=10000.0)
    base.update(cfg)
    o = orc.Model(base["dim"], base["layers"], base["heads"], base["kv_heads"],
                  base["head_dim"], base["hidden"], base["vocab"], base["seq"],
                  theta=base["theta"], bf16=bf16, seed=seed)
    c = ab.LlamaConfig(base["dim"], base["layers"], base["heads"], base["kv_heads"],
                       base["head_dim"], base["hidden"], base["vocab"], base["seq"],
                       batch=batch, rope_theta=base["theta"],
                       dtype=ab.BF16 if bf16 else ab.F32)
    g = ab.LlamaModel(rt, c)
    g.init_synthetic(seed, 0.02)
    return o, g


@pytest.mark.parametrize("bf16", [False, True])
def test_synthetic_weights_bit_identical_to_oracle(rt, orc, bf16):
    o, g = make_pair(rt, orc, bf16=bf16)
    for name in ab.WEIGHT_IDS:
        for layer in (0, 1) if name not in ("embed", "wcls", "rms_final") else (0,):
            got = g.weight(name, layer).read()
            want = o.weight(name, layer)
            if bf16 and name.startswith("rms"):
                want = orc.to_bf16_bits(want).reshape(want.shape)
            assert np.array_equal(got, want), (name, layer)


def _block_setup(rt, g, layer=0):
    w = ab.CausalAttentionBlockWeights(g.weight("rms_att", layer), g.weight("wq", layer),
                                       g.weight("wk", layer), g.weight("wv", layer),
                                       g.weight("wo", layer))
    f = ab.SwiGluBlockWeights(g.weight("rms_ffn", layer), g.weight("w1", layer),
                              g.weight("w3", layer), g.weight("w2", layer))
    return w, f


@pytest.mark.parametrize("bf16", [False, True])
def test_attention_and_swiglu_blocks_match_oracle(rt, orc, bf16):
    """Each block, recorded once and replayed at positions 0..n, against the oracle's
    or_attention_block / or_ffn_block (src/blocks.rs:178-278 order)."""
    o, g = make_pair(rt, orc, bf16=bf16, layers=1, seq=80)
    cfg = g.cfg
    w, f = _block_setup(rt, g)
    cache = ab.KvCache(rt, 1, cfg.seq, cfg.kv_heads, cfg.head_dim, cfg.dtype)
    layer = cache.layer(0)
    attn = ab.CausalAttentionBlock(rt, cfg.dim, cfg.heads, cfg.seq)
    ffn = ab.SwiGluBlock(rt, cfg.dim, cfg.hidden)
    x = ab.Tensor.zeros(rt, (cfg.dim,))
    step = ab.DecodeStep.parcel(rt)
    s_att, s_ffn = rt.scheme(), rt.scheme()
    attn.record(s_att, x, w, layer, step)
    ffn.record(s_ffn, x, f)
    assert s_att.ir_node_count() == 3 and s_ffn.ir_node_count() == 2
    tol = BF16_TOL if bf16 else FP32_TOL
    for pos, tok in enumerate([3, 17, 17, 60, 1, 95, 40, 2, 9, 33, 70, 71]):
        o.embed_token(tok)
        x.write(o.tensor("x"))
        rt.deposit(step, [ab.DecodeStep(tok, pos)])
        s_att.submit()
        o.attention_block(0, pos)
        assert rel(x.read(), o.tensor("x")) < tol, ("attn", pos)
        kc = cache.layer(0)
        got_k = layer.key.read_f32()[: pos + 1]
        got_v = layer.value.read_f32()[: pos + 1]
        assert rel(got_k, o.cache(False)[0, : pos + 1]) < tol
        assert rel(got_v, o.cache(True)[0, : pos + 1]) < tol
        s_ffn.submit()
        o.ffn_block(0)
        assert rel(x.read(), o.tensor("x")) < tol, ("ffn", pos)
    assert s_att.replay_stats().records == 1


def test_block_validation_adds_no_node(rt, orc):
    o, g = make_pair(rt, orc, layers=1)
    cfg = g.cfg
    w, f = _block_setup(rt, g)
    attn = ab.CausalAttentionBlock(rt, cfg.dim, cfg.heads, cfg.seq)
    cache = ab.KvCache(rt, 1, cfg.seq, cfg.kv_heads, cfg.head_dim)
    s = rt.scheme()
    x = ab.Tensor.zeros(rt, (cfg.dim,))
    step = ab.DecodeStep.parcel(rt)
    bad = ab.CausalAttentionBlockWeights(w.norm, w.query, w.key, w.query, w.output)
    with pytest.raises(ab.ValidationError, match="wk and wv row counts differ"):
        attn.record(s, x, bad, cache.layer(0), step)
    small = ab.KvCache(rt, 1, cfg.seq // 2, cfg.kv_heads, cfg.head_dim)
    with pytest.raises(ab.ValidationError, match="`seq`"):
        attn.record(s, x, w, small.layer(0), step)
    assert s.ir_node_count() == 0
    with pytest.raises(ab.ValidationError, match="not divisible"):
        ab.CausalAttentionBlock(rt, 130, 4, 16)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 6])
def test_linear_matches_oracle(rt, orc, dtype, batch):
    d_out, d_in = 301, 512
    x_host = orc.normal(batch * d_in, 5, 1, 0.0, 1.0).reshape(batch, d_in)
    if dtype == "f32":
        w_host = orc.normal(d_out * d_in, 5, 2, 0.0, 0.05).reshape(d_out, d_in)
        w = ab.Tensor.from_array(rt, w_host)
        want = np.stack([orc.matmul(w_host, x_host[b]) for b in range(batch)])
        x = ab.Tensor.from_array(rt, x_host)
        tol = FP32_TOL
    else:
        bits = orc.normal_bf16_bits(d_out * d_in, 5, 2, 0.0, 0.05).reshape(d_out, d_in)
        w = ab.Tensor.from_array(rt, bits, ab.BF16)
        xb = orc.to_bf16_bits(x_host).reshape(batch, d_in)
        x = ab.Tensor.from_array(rt, xb, ab.BF16)
        xr = orc.from_bf16_bits(xb).reshape(batch, d_in)
        want = np.stack([orc.matmul_bf16(bits, xr[b]) for b in range(batch)])
        tol = 1e-5  # same bf16 inputs, fp32 accumulation: only the order differs
    out = ab.Tensor.zeros(rt, (batch, d_out))
    s = rt.scheme()
    ab.Linear(rt).record(s, w, x, out)
    s.submit()
    assert rel(out.read(), want) < tol


def test_model_logits_match_oracle_fp32_gqa(rt, orc):
    o, g = make_pair(rt, orc, layers=2, theta=500000.0)
    for pos, tok in enumerate([5, 90, 12, 12, 44, 3, 71, 8]):
        assert rel(g.step(tok, pos), o.step(tok, pos)) < FP32_TOL, pos


def test_model_logits_match_oracle_bf16(rt, orc):
    o, g = make_pair(rt, orc, bf16=True, layers=2, heads=8, kv_heads=2, head_dim=16,
                     theta=500000.0)
    for pos, tok in enumerate([5, 90, 12, 12, 44, 3]):
        assert rel(g.step(tok, pos), o.step(tok, pos)) < BF16_TOL, pos


def test_batched_model_matches_independent_streams(rt, orc):
    B = 3
    o, g = make_pair(rt, orc, batch=B)
    refs = [orc.Model(128, 2, 4, 2, 32, 256, 96, 48, seed=7) for _ in range(B)]
    seqs = [[4, 8, 15, 16, 23], [42, 42, 1, 2, 3], [95, 0, 50, 60, 70]]
    for pos in range(5):
        toks = [seqs[b][pos] for b in range(B)]
        logits, am = g.step_batch(toks, [pos] * B, logits=True, argmax=True)
        for b in range(B):
            want = refs[b].step(toks[b], pos)
            assert rel(logits[b], want) < FP32_TOL, (pos, b)
            assert am[b] == orc.sample_argmax(logits[b])


def test_tiny_llama_greedy_tokens_bit_identical(rt, orc):
    """dim 288, 6 layers, 6/6 heads, hidden 768, vocab 32000, seq 256,
    seed 0; 8 uniform prompt ids in [3, 32000) then 128 greedy tokens at batch 1."""
    cfg = dict(dim=288, layers=6, heads=6, kv_heads=6, head_dim=48, hidden=768, vocab=32000,
               seq=256)
    o = orc.Model(**cfg, seed=0)
    prompt = orc.uniform_tokens(8, 0, 1000, 3, 32000).tolist()
    want, margins = o.generate_tokens(prompt, 8 + 128)
    g = ab.LlamaModel(rt, ab.LlamaConfig(**cfg))
    g.init_synthetic(0, 0.02)
    out = g.generate_tokens_native(prompt, 8 + 128)
    assert len(out.tokens) == 135
    assert out.tokens == want, (np.nonzero(np.array(out.tokens) != np.array(want))[0][:5],
                                float(margins[7:].min()))
    g.reset()
    out_py = ab.generate_tokens(g, prompt, 8 + 128)
    assert out_py.tokens == want


@pytest.mark.parametrize("batch", [5, 8, 20, 64, 128, 200])
def test_batched_bf16_model_on_tensor_cores(rt, orc, batch):
    """Batches above 4 with bf16 weights run every projection on the tcgen05 GEMM (row tiles
    of 128, split-K where K allows; 128 and 200 columns run two CTAs per SM with two or
    three stages): each stream matches its own oracle decode."""
    cfg = dict(dim=512, layers=2, heads=8, kv_heads=2, head_dim=64, hidden=1024, vocab=640,
               seq=24, theta=500000.0)
    o, g = make_pair(rt, orc, bf16=True, batch=batch, seed=13, **cfg)
    streams = [0, 1, batch // 2, batch - 1]
    refs = {b: orc.Model(cfg["dim"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                         cfg["head_dim"], cfg["hidden"], cfg["vocab"], cfg["seq"],
                         theta=cfg["theta"], bf16=True, seed=13) for b in streams}
    rng = np.random.default_rng(batch)
    toks = rng.integers(0, cfg["vocab"], size=(5, batch))
    for pos in range(5):
        logits, am = g.step_batch(toks[pos].tolist(), [pos] * batch, logits=True, argmax=True)
        for b in streams:
            want = refs[b].step(int(toks[pos, b]), pos)
            assert rel(logits[b], want) < BF16_TOL, (batch, pos, b, rel(logits[b], want))
        assert all(am[b] == int(np.argmax(logits[b])) for b in range(batch))
    labels = g.scheme().node_labels()
    # the operand norms: standalone after the embedding, else inside the residual fold before
    assert "attn_qkv_rope_norm" in labels
    assert any(l.endswith("ffn_gate_up_swiglu_norm") for l in labels), labels


@pytest.mark.parametrize("batch", [5, 32, 256])
def test_batched_fp32_model_on_tensor_cores(rt, orc, batch):
    """Batches above 4 with fp32 weights run every projection as 3xTF32 on the tcgen05
    tf32 pipe (exact hi/lo splits of weights and activations): each stream stays within
    the fp32 bar of its own oracle decode and picks the oracle's greedy id. The vocab
    ends in a partial 128-row tile and the K widths exercise split-K."""
    cfg = dict(dim=256, layers=2, heads=4, kv_heads=4, head_dim=64, hidden=512, vocab=1000,
               seq=16, theta=10000.0)
    o, g = make_pair(rt, orc, batch=batch, seed=11, **cfg)
    streams = sorted({0, 1, batch // 2, batch - 1})
    refs = {b: orc.Model(cfg["dim"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                         cfg["head_dim"], cfg["hidden"], cfg["vocab"], cfg["seq"],
                         theta=cfg["theta"], seed=11) for b in streams}
    rng = np.random.default_rng(batch + 1)
    toks = rng.integers(0, cfg["vocab"], size=(4, batch))
    for pos in range(4):
        logits, am = g.step_batch(toks[pos].tolist(), [pos] * batch, logits=True, argmax=True)
        for b in streams:
            want = refs[b].step(int(toks[pos, b]), pos)
            assert rel(logits[b], want) < FP32_TOL, (batch, pos, b, rel(logits[b], want))
            assert int(am[b]) == orc.sample_argmax(want), (batch, pos, b)
        assert all(am[b] == int(np.argmax(logits[b])) for b in range(batch))
    labels = g.scheme().node_labels()
    assert "attn_qkv_rope_split" in labels and "attn_wo_residual_split" in labels
    assert any(l.endswith("final_norm_classifier_split") for l in labels), labels


def test_device_greedy_loop_matches_host_loop(rt, orc):
    """decode_device (argmax and the next DecodeStep on the device) emits the ids the
    reference loop (generate.rs:43-91 with host sample_argmax) emits."""
    B = 2
    o, g = make_pair(rt, orc, batch=B, seq=64)
    refs = [orc.Model(128, 2, 4, 2, 32, 256, 96, 64, seed=7) for _ in range(B)]
    prompts = [[3, 9, 27], [81, 50, 2]]
    want = [r.generate_tokens(p, 40)[0] for r, p in zip(refs, prompts)]
    for pos in range(2):
        g.step_batch([prompts[b][pos] for b in range(B)], [pos] * B, logits=False)
    got = g.decode_device([prompts[b][2] for b in range(B)], [2] * B, 37)
    for b in range(B):
        assert got[:, b].tolist() == want[b][2:], b
    with pytest.raises(ab.AmmonError, match="passes max_seq_len"):
        g.decode_device([1] * B, [60] * B, 10)


def test_step_scheme_labels_and_node_timing(rt, orc):
    o, g = make_pair(rt, orc)
    s = g.scheme()
    labels = s.node_labels()
    assert labels[0] == "embed" and labels[-1] == "argmax"
    assert labels.count("attn_qkv_rope") == g.cfg.layers
    ms = s.time_nodes(iters=2)
    assert len(ms) == len(labels) and all(t > 0 for t in ms)


def test_position_beyond_seq_is_rejected(rt, orc):
    o, g = make_pair(rt, orc)
    with pytest.raises(ab.AmmonError, match="beyond max_seq_len"):
        g.step(1, g.cfg.seq)
    with pytest.raises(ab.AmmonError, match="out of range"):
        g.step(g.cfg.vocab, 0)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_swiglu_result_independent_of_kernel_and_ksplit(rt, orc, dtype, monkeypatch):
    """The gate/up SwiGLU runs in the GEMV epilogue (batch <= 4), the single-split GEMM
    epilogue or, split over k, the fold kernel. All three use one expression
    (src/kernels.rs:462-476 order), so with sums that are exact in fp32 whatever their order
    (x = +-4096 normalises to exactly +-1, gate/up weights are small integers, w2 copies hb[r]
    into row r) the block's result is bit-identical for every path and split count."""
    dim, hidden = 512, 256
    rng = np.random.default_rng(11)
    x_host = np.where(rng.random((8, dim)) < 0.5, -4096.0, 4096.0).astype(np.float32)
    w1 = (rng.integers(-1, 2, (hidden, dim)) * (rng.random((hidden, dim)) < 0.08)).astype(
        np.float32)
    w3 = (rng.integers(-2, 3, (hidden, dim)) * (rng.random((hidden, dim)) < 0.08)).astype(
        np.float32)
    w2 = np.zeros((dim, hidden), np.float32)
    w2[np.arange(hidden), np.arange(hidden)] = 1.0
    gain = np.ones(dim, np.float32)
    dt = ab.BF16 if dtype == "bf16" else ab.F32

    def dev(a):
        return ab.Tensor.from_array(rt, orc.to_bf16_bits(a).reshape(a.shape) if dt == ab.BF16
                                    else a, dt)

    w = ab.SwiGluBlockWeights(dev(gain), dev(w1), dev(w3), dev(w2))

    def run(batch, max_ksplit=None):
        if max_ksplit:
            monkeypatch.setenv("AMMON_B200_GEMM_MAX_KSPLIT", str(max_ksplit))
        else:
            monkeypatch.delenv("AMMON_B200_GEMM_MAX_KSPLIT", raising=False)
        ffn = ab.SwiGluBlock(rt, dim, hidden, max_batch=batch)
        x = ab.Tensor.from_array(rt, x_host[:batch])
        s = rt.scheme()
        ffn.record(s, x, w)
        s.submit()
        out = x.read()
        monkeypatch.delenv("AMMON_B200_GEMM_MAX_KSPLIT", raising=False)
        return out, s.node_labels()

    split, labels_split = run(8)
    single, labels_single = run(8, max_ksplit=1)
    gemv, labels_gemv = run(4)
    assert "ffn_gate_up_swiglu_splitk" in labels_split, labels_split
    assert "ffn_gate_up_swiglu_splitk" not in labels_single, labels_single
    assert np.array_equal(split, single)
    if dt == ab.BF16:
        assert np.array_equal(split[:4], gemv)
    else:
        # 3xTF32 carries the f32 w2 operand as tf32 hi + lo halves, and lo keeps 11 of its up
        # to 13 significant bits: the identity projection of hb is exact to ~2^-22 relative,
        # far below one ulp of the +-4096 residual it lands on
        assert np.abs(split[:4] - gemv).max() <= 2.0 ** -10
    # and the value itself: silu(g) * u of the exact integer sums, against float64
    g = x_host[:8] / 4096.0 @ w1.T.astype(np.float64)
    u = x_host[:8] / 4096.0 @ w3.T.astype(np.float64)
    h = g / (1.0 + np.exp(-g)) * u
    if dt == ab.BF16:
        h = orc.round_bf16(h.astype(np.float32)).reshape(h.shape)
    want = x_host[:8].astype(np.float64)
    want[:, :hidden] += h
    assert rel(split, want) < 1e-6
