"""Parity at the shapes the benchmark reports, against the CPU oracle and float64.

* Llama-3-8B-shaped bf16 (dim 4096, 32/8 heads, head 128, SwiGLU 14336, the full 128256-row
  vocabulary and classifier, RoPE theta 500000; two layers of it): batch 1 on the GEMV path
  at positions 128 and 600, batch 64 on the tcgen05 GEMM with split-K at positions 600..663
  (one per stream). The K/V rows before the decoded position are seeded values written into
  both caches, so a step at position 600 reads 600 cached rows without decoding 600 tokens.
  Bar: logits within 2e-2 (max |gpu - oracle| / max |oracle|), K/V rows written at the
  position within 2e-2, greedy ids equal to the oracle's first maximum wherever its top two
  logits are further apart than twice the observed logit error.
* Llama-shaped 110M fp32 at 256 streams (dim 768, 12 layers, 12/12 heads, SwiGLU 2048, vocab
  32000, seed 1, 16-token uniform prompts as the benchmark draws them): 17 greedy tokens of
  every stream from the device loop; four streams against the oracle's generate_tokens
  (src/generate.rs:43-91) bit-identical, and the next step's logits within 1e-5.
* RoPE at positions 0, 1, 4095 and 8191 with theta 500000 (32 x 128 q, 8 x 128 k rows).
* The fused split attention at contexts 4096 and 32768 for batch 1 and 8 (32/8 heads, head
  128, bf16 K/V) against float64, 1e-4.
"""
import os

import numpy as np
import pytest

import ammon_b200 as ab
from ammon_b200 import kernels as K

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
FP32_TOL = 1e-5
L8B = dict(dim=4096, layers=2, heads=32, kv_heads=8, head_dim=128, hidden=14336, vocab=128256,
           seq=1024, theta=500000.0)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def bf16_to_f32(bits):
    return (np.asarray(bits).astype(np.uint32) << 16).view(np.float32)


@pytest.fixture(scope="module")
def rt():
    r = ab.create_runtime(0)
    yield r
    r.synchronize()


@pytest.fixture(scope="module")
def oracle_8b(orc):
    orc.set_threads(os.cpu_count() or 1)
    c = L8B
    m = orc.Model(c["dim"], c["layers"], c["heads"], c["kv_heads"], c["head_dim"], c["hidden"],
                  c["vocab"], c["seq"], theta=c["theta"], bf16=True, seed=3)
    yield m
    m.close()


def _model_8b(rt, batch, fused=True):
    c = L8B
    old = os.environ.get("AMMON_B200_FUSED_STEP")
    os.environ["AMMON_B200_FUSED_STEP"] = "1" if fused else "0"
    try:
        g = ab.LlamaModel(rt, ab.LlamaConfig(c["dim"], c["layers"], c["heads"], c["kv_heads"],
                                             c["head_dim"], c["hidden"], c["vocab"], c["seq"],
                                             batch=batch, rope_theta=c["theta"],
                                             dtype=ab.BF16))
    finally:
        if old is None:
            os.environ.pop("AMMON_B200_FUSED_STEP")
        else:
            os.environ["AMMON_B200_FUSED_STEP"] = old
    g.init_synthetic(3, 0.02)
    return g


def _seed_caches(g, o, batch, streams, seed):
    """Seeded N(0, 1) bf16 K/V in every row of the model's cache; the compared streams' rows
    are copied into the oracle's per-stream caches (state k holds stream streams[k])."""
    cache = g.cache()
    for layer in range(g.cfg.layers):
        lay = cache.layer(layer)
        lay.key.fill_normal(seed, 2 * layer)
        lay.value.fill_normal(seed, 2 * layer + 1)
        kb, vb = lay.key.read(), lay.value.read()
        for k, b in enumerate(streams):
            o.select_stream(k)
            o.set_cache(layer, kb[b] if batch > 1 else kb, vb[b] if batch > 1 else vb)


def _check_step(g, o, batch, streams, tokens, positions, tag):
    logits, am = g.step_batch(tokens, positions, logits=True, argmax=True)
    assert all(int(am[b]) == int(np.argmax(logits[b])) for b in range(batch)), tag
    # the K/V rows this step appended, last layer
    lay = g.cache().layer(g.cfg.layers - 1)
    kall, vall = lay.key.read(), lay.value.read()
    for k, b in enumerate(streams):
        o.select_stream(k)
        want = o.step(tokens[b], positions[b])
        err = rel(logits[b], want)
        assert err < BF16_TOL, (tag, b, err)
        kd = bf16_to_f32(kall[b] if batch > 1 else kall)
        vd = bf16_to_f32(vall[b] if batch > 1 else vall)
        p = positions[b]
        assert rel(kd[p], o.cache(False)[-1, p]) < BF16_TOL, (tag, b, "k")
        assert rel(vd[p], o.cache(True)[-1, p]) < BF16_TOL, (tag, b, "v")
    return logits, am


@pytest.mark.parametrize("path", ["fused", "graph"])
def test_llama3_8b_shape_batch1(rt, orc, oracle_8b, path):
    """Batch 1, both ways the library runs it: the persistent single-launch step (the default)
    and the per-kernel step graph (GEMV projections at K = 4096 and 14336, the 128256-row
    classifier); attention over 129 and 601 positions (the second step reads the first
    step's row)."""
    g = _model_8b(rt, 1, fused=path == "fused")
    o = oracle_8b
    o.select_stream(0)
    _seed_caches(g, o, 1, [0], seed=31)
    labels = g.scheme().node_labels()
    if path == "fused":
        assert labels == ["decode_step"]
    else:
        assert "final_norm_classifier" in labels
        assert not any(l.endswith("_splitk") for l in labels)
    for pos, tok in ((128, 91234), (600, 17)):
        logits, am = _check_step(g, o, 1, [0], [tok], [pos], f"b1 pos {pos}")
        want = o.tensor("logits")
        abs_err = float(np.abs(logits[0].astype(np.float64) - want).max())
        top2 = np.sort(want)[-2:]
        if top2[1] - top2[0] > 2 * abs_err:
            assert int(am[0]) == orc.sample_argmax(want), pos
    g.close()


def test_llama3_8b_shape_batch64_tensor_cores(rt, orc, oracle_8b):
    """Batch 64: the tcgen05 GEMM with split-K folds (K = 4096 and 14336), the classifier over
    128256 rows in 128-row tiles, attention on the tensor-core flash-decoding kernel with one
    position per stream (600..663). Four streams against the oracle."""
    B = 64
    g = _model_8b(rt, B)
    o = oracle_8b
    streams = [0, 1, 31, 63]
    _seed_caches(g, o, B, streams, seed=32)
    labels = g.scheme().node_labels()
    # the w2 folds carry the next operand norm (the next layer's, then the classifier's)
    assert any(l.startswith("ffn_down_residual_splitk") for l in labels), labels
    assert "attn_qkv_rope_splitk" in labels, labels
    rng = np.random.default_rng(64)
    tokens = [int(t) for t in rng.integers(0, L8B["vocab"], B)]
    positions = [600 + b for b in range(B)]
    logits, am = _check_step(g, o, B, streams, tokens, positions, "b64")
    for k, b in enumerate(streams):
        o.select_stream(k)
        want = o.tensor("logits")
        abs_err = float(np.abs(logits[b].astype(np.float64) - want).max())
        top2 = np.sort(want)[-2:]
        if top2[1] - top2[0] > 2 * abs_err:
            assert int(am[b]) == orc.sample_argmax(want), b
    o.select_stream(0)
    g.close()


def test_llama_110m_fp32_256_streams_greedy_ids(rt, orc):
    """BASELINE config 2's shape at its full batch: 256 streams, 16-token prompts, greedy ids
    from the device loop (3xTF32 tcgen05 GEMM, f32 K/V attention) bit-identical to the
    oracle's generate_tokens for four streams, then the next step's logits within 1e-5."""
    orc.set_threads(os.cpu_count() or 1)
    cfg = dict(dim=768, layers=12, heads=12, kv_heads=12, head_dim=64, hidden=2048,
               vocab=32000, seq=1024)
    B, P, N = 256, 16, 17
    g = ab.LlamaModel(rt, ab.LlamaConfig(**cfg, batch=B, rope_theta=10000.0))
    g.init_synthetic(1, 0.02)
    prompts = np.stack([orc.uniform_tokens(P, 1, 1000 + b, 3, cfg["vocab"]) for b in range(B)])
    for pos in range(P - 1):
        g.step_batch(prompts[:, pos].tolist(), [pos] * B, logits=False)
    ids = g.decode_device(prompts[:, P - 1].tolist(), [P - 1] * B, N)  # positions P .. P+N-1
    assert ids.shape == (N, B)
    o = orc.Model(**cfg, theta=10000.0, seed=1)
    streams = [0, 1, 127, 255]
    for k, b in enumerate(streams):
        o.select_stream(k)
        toks, margins = o.generate_tokens(prompts[b].tolist(), P + N)
        greedy = toks[P - 1:]
        assert ids[:, b].tolist() == greedy, (b, float(np.min(margins[P - 1:])))
    last = ids[-1].tolist()
    logits, _ = g.step_batch(last, [P + N - 1] * B, logits=True)
    for k, b in enumerate(streams):
        o.select_stream(k)
        want = o.step(last[b], P + N - 1)
        assert rel(logits[b], want) < FP32_TOL, (b, rel(logits[b], want))
    o.close()
    g.close()


def test_rope_long_positions_theta_5e5(rt, orc):
    """The batched RoPE at positions 0, 1, 4095 and 8191, theta 500000, 32 x 128 q heads and
    the k rows of an [8192, 8, 128] cache. Position 0 is the identity, bit for bit. Every
    rotated pair keeps its length (rel 1e-6). Against the exact float64 rotation each element
    stays within the fp32 envelope |pair| * (pos * freq * 4 ulp + 4 ulp): the angle pos * freq
    is formed in fp32 from a powf whose last-bit differences between libraries grow with the
    position. The oracle (glibc powf / cosf / sinf) is held to the same envelope."""
    H, KV, hd, seq, theta = 32, 8, 128, 8192, 500000.0
    positions = [0, 1, 4095, 8191]
    B = len(positions)
    q_host = orc.normal(B * H * hd, 9, 1, 0.0, 1.0).reshape(B, H, hd)
    k_host = orc.normal(seq * KV * hd, 9, 2, 0.0, 1.0).reshape(seq, KV, hd)
    q = ab.Tensor.from_array(rt, q_host)
    k = ab.Tensor.from_array(rt, k_host)
    st = ab.DecodeStep.parcel(rt, B)
    rt.deposit(st, [ab.DecodeStep(0, p) for p in positions])
    s = rt.scheme()
    K.RopeKernel.prepare(rt).record(s, "rope", q, k, st, theta)
    s.submit()
    qg, kg = q.read(), k.read()
    assert np.array_equal(qg[0], q_host[0]) and np.array_equal(kg[0], k_host[0])
    ulp = 2.0 ** -23
    j = np.arange(0, hd, 2)
    freq = theta ** (-(j.astype(np.float64)) / hd)

    def exact(v, pos):  # v [..., hd]
        a = pos * freq
        c, sn = np.cos(a), np.sin(a)
        v = v.astype(np.float64)
        out = np.empty_like(v)
        out[..., 0::2] = v[..., 0::2] * c - v[..., 1::2] * sn
        out[..., 1::2] = v[..., 0::2] * sn + v[..., 1::2] * c
        norm = np.hypot(v[..., 0::2], v[..., 1::2])
        bound = norm * (pos * freq * 4 * ulp + 4 * ulp) + 1e-30
        return out, np.repeat(bound, 2, axis=-1)

    for i, pos in enumerate(positions):
        for got, src in ((qg[i], q_host[i]), (kg[pos], k_host[pos])):
            want, bound = exact(src, pos)
            assert np.all(np.abs(got - want) <= bound), (pos, float(
                (np.abs(got - want) / bound).max()))
            n0 = np.hypot(src[..., 0::2].astype(np.float64), src[..., 1::2])
            n1 = np.hypot(got[..., 0::2].astype(np.float64), got[..., 1::2])
            assert np.abs(n1 - n0).max() <= 1e-6 * n0.max(), pos
        qo, ko = q_host[i].copy(), k_host.copy()
        orc.rope(qo, ko, pos, theta)
        want, bound = exact(q_host[i], pos)
        assert np.all(np.abs(qo - want) <= bound), ("oracle", pos)
    s.close()


@pytest.mark.parametrize("ctx", [4096, 32768])
@pytest.mark.parametrize("batch", [1, 8])
def test_split_attention_long_context_matches_float64(rt, ctx, batch):
    """BASELINE config 3's kernel at contexts 4096 and 32768 (32 query / 8 kv heads, head 128,
    bf16 K/V, fp32 q and output): the device-chosen split ranges over the whole context, rows
    at different positions (the last at ctx - 1), two replays, against float64 at 1e-4."""
    H, KV, hd = 32, 8, 128
    kc = ab.Tensor.zeros(rt, (batch, ctx, KV, hd), ab.BF16).fill_normal(2, 2)
    vc = ab.Tensor.zeros(rt, (batch, ctx, KV, hd), ab.BF16).fill_normal(2, 3)
    q = ab.Tensor.zeros(rt, (batch, H, hd)).fill_normal(2, 1)
    out = ab.Tensor.zeros(rt, (batch, H * hd))
    positions = [ctx - 1 - (ctx // (batch + 1)) * b - 37 * (b % 2) for b in range(batch)]
    positions[-1] = ctx - 1
    assert all(0 <= p < ctx for p in positions)
    st = ab.DecodeStep.parcel(rt, batch)
    rt.deposit(st, [ab.DecodeStep(0, p) for p in positions])
    s = rt.scheme()
    K.AttentionDecodeKernel.prepare(rt).record(s, "attn", q, kc, vc, out, st)
    kh = bf16_to_f32(kc.read())
    vh = bf16_to_f32(vc.read())
    qh = q.read()
    for _ in range(2):
        s.submit()
        got = out.read().reshape(batch, H, hd)
        for b, p in enumerate(positions):
            for kv in range(KV):
                kk = kh[b, : p + 1, kv].astype(np.float64)
                vv = vh[b, : p + 1, kv].astype(np.float64)
                g = H // KV
                sc = qh[b, kv * g:(kv + 1) * g].astype(np.float64) @ kk.T / np.sqrt(hd)
                w = np.exp(sc - sc.max(axis=1, keepdims=True))
                want = (w / w.sum(axis=1, keepdims=True)) @ vv
                err = rel(got[b, kv * g:(kv + 1) * g], want)
                assert err < 1e-4, (ctx, batch, b, kv, err)
    s.close()
