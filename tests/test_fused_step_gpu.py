"""The persistent single-launch decode step (batch 1, bf16 weights, one GPU): one cooperative
kernel runs the embedding, every layer (src/blocks.rs:178-278 order), the final norm, the
classifier and the greedy pick. Checked against the CPU oracle at the bf16 bar (2e-2), against
the per-kernel step graph of the same model (AMMON_B200_FUSED_STEP=0), through the device
greedy loop (its sample feedback), with positions whose attention spans many CTAs (the
blocks' partials folded by the last CTA of each kv head), and on its error path: a grid
barrier that one CTA never reaches ends every CTA's bounded wait, the step reports
AB_ERR_DEVICE, and the device keeps working."""
import os

import numpy as np
import pytest

import ammon_b200 as ab

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
CFG = dict(dim=256, layers=2, heads=4, kv_heads=2, head_dim=64, hidden=512, vocab=1000,
           seq=300, theta=500000.0)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def rt():
    r = ab.create_runtime(0)
    yield r
    r.synchronize()


def _model(rt, cfg=CFG, seed=5, **env):
    old = {k: os.environ.get(k) for k in env}
    os.environ.update({k: str(v) for k, v in env.items()})
    try:
        c = cfg
        g = ab.LlamaModel(rt, ab.LlamaConfig(c["dim"], c["layers"], c["heads"], c["kv_heads"],
                                             c["head_dim"], c["hidden"], c["vocab"], c["seq"],
                                             batch=1, rope_theta=c["theta"], dtype=ab.BF16))
        g.init_synthetic(seed, 0.02)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return g


def _oracle(orc, cfg=CFG, seed=5):
    c = cfg
    return orc.Model(c["dim"], c["layers"], c["heads"], c["kv_heads"], c["head_dim"],
                     c["hidden"], c["vocab"], c["seq"], theta=c["theta"], bf16=True, seed=seed)


def test_fused_step_is_one_launch_and_matches_oracle(rt, orc):
    g = _model(rt)
    assert g.scheme().node_labels() == ["decode_step"]
    o = _oracle(orc)
    toks = [3, 999, 17, 17, 512, 0, 44, 1, 250, 6]
    for pos, tok in enumerate(toks):
        logits, am = g.step_batch([tok], [pos], logits=True, argmax=True)
        want = o.step(tok, pos)
        assert rel(logits[0], want) < BF16_TOL, (pos, rel(logits[0], want))
        assert int(am[0]) == int(np.argmax(logits[0]))
    # the K/V rows the step appended, both layers
    for layer in range(CFG["layers"]):
        lay = g.cache().layer(layer)
        kd = (lay.key.read().astype(np.uint32) << 16).view(np.float32)[: len(toks)]
        vd = (lay.value.read().astype(np.uint32) << 16).view(np.float32)[: len(toks)]
        assert rel(kd, o.cache(False)[layer, : len(toks)]) < BF16_TOL
        assert rel(vd, o.cache(True)[layer, : len(toks)]) < BF16_TOL
    g.close()
    o.close()


@pytest.mark.parametrize("pos", [31, 32, 95, 211, 299])
def test_fused_step_long_positions_fold_partials(rt, orc, pos):
    """Seeded K/V rows before `pos` in both caches; one step at pos: the attention splits the
    positions over up to 74 CTAs per kv head (32-position blocks) and folds their partials."""
    g = _model(rt)
    o = _oracle(orc)
    cache = g.cache()
    for layer in range(CFG["layers"]):
        lay = cache.layer(layer)
        lay.key.fill_normal(41, 2 * layer)
        lay.value.fill_normal(41, 2 * layer + 1)
        o.set_cache(layer, lay.key.read(), lay.value.read())
    logits, am = g.step_batch([123], [pos], logits=True, argmax=True)
    want = o.step(123, pos)
    assert rel(logits[0], want) < BF16_TOL, rel(logits[0], want)
    g.close()
    o.close()


def test_fused_step_agrees_with_the_step_graph(rt):
    """The same synthetic model through the persistent step and through the per-kernel step
    graph: logits within the bf16 bar of each other at every position, equal greedy ids
    wherever the top two logits are further apart than the observed difference."""
    fused = _model(rt)
    graph = _model(rt, AMMON_B200_FUSED_STEP=0)
    assert graph.scheme().node_labels() != ["decode_step"]
    tok = 7
    for pos in range(40):
        a, am_a = fused.step_batch([tok], [pos], logits=True, argmax=True)
        a = a[0].copy()
        am_a = int(am_a[0])
        b, am_b = graph.step_batch([tok], [pos], logits=True, argmax=True)
        b = b[0].copy()
        am_b = int(am_b[0])
        assert rel(a, b) < BF16_TOL, (pos, rel(a, b))
        top2 = np.sort(b)[-2:]
        if top2[1] - top2[0] > 2 * float(np.abs(a - b).max()):
            assert am_a == am_b, pos
        tok = am_b
    fused.close()
    graph.close()


def test_fused_device_loop_matches_its_host_loop(rt):
    """decode_device (argmax and the next DecodeStep written by the kernel's last CTA) emits
    the ids that the host loop through step() emits on the same kernel."""
    a = _model(rt)
    b = _model(rt)
    prompt = [11, 22, 33]
    for pos in range(2):
        a.step_batch([prompt[pos]], [pos], logits=False)
        b.step_batch([prompt[pos]], [pos], logits=False)
    got = a.decode_device([prompt[2]], [2], 60)[:, 0].tolist()
    want, tok = [], prompt[2]
    for pos in range(2, 62):
        _, am = b.step_batch([tok], [pos], logits=False, argmax=True)
        tok = int(am[0])
        want.append(tok)
    assert got == want
    with pytest.raises(ab.AmmonError, match="passes max_seq_len"):
        a.decode_device([1], [290], 20)
    a.close()
    b.close()


def test_fused_step_trace_records_every_barrier(rt):
    g = _model(rt, AMMON_B200_STEP_TRACE=1)
    g.step_batch([5], [0], logits=False)
    tr = g.step_trace()
    assert tr is not None and tr.shape[:2] == (1 + 5 * CFG["layers"], 4)
    assert np.all(tr[:, 3] == 0)  # one GPU: no all-reduce barriers
    arrive, release = tr[:, 0].astype(np.int64), tr[:, 1].astype(np.int64)
    assert np.all(arrive > 0) and np.all(release >= arrive)
    # every CTA leaves a barrier after the last CTA arrived at it
    assert np.all(release.min(axis=1) >= arrive.max(axis=1))
    assert np.all(np.diff(arrive.max(axis=1)) >= 0)
    g.close()


def test_fused_step_wait_limit_ends_a_stalled_barrier(rt, orc):
    """CTA 0 never arrives at the third grid barrier (test hook): every other CTA's wait there
    runs out after the runtime's wait limit (20 ms here), the launch ends, the step raises
    DeviceError (bounded wait timed out) and the next launches on the same device work."""
    g = _model(rt, AMMON_B200_TEST_STALL_BARRIER=3)
    old = rt.wait_limit_ms
    rt.wait_limit_ms = 20
    try:
        with pytest.raises(ab.DeviceError, match="bounded wait timed out"):
            g.step_batch([9], [0], logits=False)
    finally:
        rt.wait_limit_ms = old
    g.close()
    h = _model(rt)
    o = _oracle(orc)
    logits, _ = h.step_batch([9], [0], logits=True)
    assert rel(logits[0], o.step(9, 0)) < BF16_TOL
    h.close()
    o.close()


def test_step_logits_into_registered_and_plain_host_buffers(rt):
    """step() copies the logits straight into the model's page-locked buffer
    (ab_host_register) and through the staging buffer into any other host memory, including
    memory registered over less than the copy: all give the same values."""
    import ctypes as C

    from ammon_b200 import _abi

    g = _model(rt)
    assert g._registered
    a, _ = g.step_batch([3], [0], logits=True)
    a = a.copy()
    plain = np.zeros((1, CFG["vocab"]), np.float32)
    steps = (_abi.DecodeStep_t * 1)((3, 0))
    ab._check(_abi.lib().ab_llama_step(g._h, steps, 1,
                                       plain.ctypes.data_as(C.POINTER(C.c_float)), None))
    assert np.array_equal(plain, a)
    # a buffer page-locked over its first half only: the copy does not fit the registered
    # range, so it takes the staging buffer and still fills every logit
    half = np.zeros((1, CFG["vocab"]), np.float32)
    ab._check(_abi.lib().ab_host_register(half.ctypes.data, half.nbytes // 2))
    try:
        ab._check(_abi.lib().ab_llama_step(g._h, steps, 1,
                                           half.ctypes.data_as(C.POINTER(C.c_float)), None))
    finally:
        ab._check(_abi.lib().ab_host_unregister(half.ctypes.data))
    assert np.array_equal(half, a)
    g.close()
