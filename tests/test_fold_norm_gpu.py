"""The residual k-split fold with the next RMSNorm in one kernel (splitk_residual_norm_kernel)
computes exactly what the fold kernel followed by the norm kernel computes: the same model
recorded both ways gives bit-identical logits and greedy ids, on the bf16 tensor-core path
(batch 64) and the fp32 3xTF32 path (batch 8, tf32 halves of the normalised rows)."""
import os

import numpy as np
import pytest

import ammon_b200 as ab
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

CFG = dict(dim=512, layers=2, heads=8, kv_heads=4, head_dim=64, hidden=1024, vocab=256, seq=64)


def _decode(rt, dtype, batch, fused):
    old = os.environ.get("AMMON_B200_FOLD_NORM")
    os.environ["AMMON_B200_FOLD_NORM"] = "1" if fused else "0"
    try:
        m = ab.LlamaModel(rt, ab.LlamaConfig(**CFG, batch=batch, rope_theta=500000.0,
                                             dtype=dtype))
        m.init_synthetic(23, 0.02)
        toks = orc.uniform_tokens(batch, 23, 1, 3, CFG["vocab"]).tolist()
        out = []
        for pos in range(5):  # the first step records the scheme under this setting
            logits, am = m.step_batch(toks, [pos] * batch, logits=True, argmax=True)
            out.append((logits.copy(), am.copy()))
            toks = [int(t) for t in am]
        labels = m.scheme().node_labels()
        m.close()
        return out, labels
    finally:
        if old is None:
            del os.environ["AMMON_B200_FOLD_NORM"]
        else:
            os.environ["AMMON_B200_FOLD_NORM"] = old


@pytest.mark.parametrize("dtype,batch", [(ab.BF16, 64), (ab.F32, 8)])
def test_fold_norm_fusion_is_bit_exact(dtype, batch):
    rt = ab.create_runtime(0)
    try:
        fused, lf = _decode(rt, dtype, batch, True)
        plain, lp = _decode(rt, dtype, batch, False)
    finally:
        rt.close()
    # the fused graph has fewer nodes: each residual fold took the norm after it
    assert any("+" in l for l in lf) and not any("+" in l for l in lp)
    assert len(lf) < len(lp)
    for (a, ia), (b, ib) in zip(fused, plain):
        assert np.array_equal(a, b)
        assert np.array_equal(ia, ib)
