"""ab_attention_decode_noalloc: the allocation-free variant of the fused flash-decoding
attention, for callers that must not allocate device memory themselves (hosts whose
device memory belongs to their own pooling allocator, or loops that cannot take
cudaFree's device-wide synchronisation). Its split scratch is a static device array
inside the library.

Checked through the C ABI against the existing attention entry points
(ab_kernel_attention_partial + ab_kernel_attention_combine, which take caller-allocated
scratch) on the same inputs, on two calls in a row. Runs last, and also alone in a fresh
process (the first call on the device performs the array's address lookup)."""
import numpy as np
import pytest

import ammon_b200 as ab
from ammon_b200 import _abi

pytestmark = pytest.mark.gpu

TOL = 1e-5  # fp32 outputs: max |noalloc - existing| / max |existing|


def rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def rt():
    r = ab.create_runtime(0)
    yield r
    r.synchronize()


def _existing(rt, q_host, k, v, positions, kvd_shape):
    """Attention of each batch row through ab_kernel_attention_partial/combine."""
    B, H, hd = q_host.shape
    S = kvd_shape[0]
    splits = -(-S // ab.ATTENTION_SPLIT)
    outs = []
    for b in range(B):
        q = ab.Tensor.from_array(rt, q_host[b])
        kb = k.narrow(0, b, 1).reshape(kvd_shape)
        vb = v.narrow(0, b, 1).reshape(kvd_shape)
        step = ab.DecodeStep.parcel(rt)
        rt.deposit(step, [ab.DecodeStep(0, positions[b])])
        partial = ab.Tensor.zeros(rt, (H, splits, hd + 2))
        xb = ab.Tensor.zeros(rt, (H, hd))
        s = rt.scheme()
        ab.kernels.AttentionPartialKernel.prepare(rt).record(s, "p", q, kb, vb, partial, step)
        ab.kernels.AttentionCombineKernel.prepare(rt).record(s, "c", partial, xb, step)
        s.submit()
        outs.append(xb.read().reshape(-1))
    return np.stack(outs)


@pytest.mark.parametrize("kv_dtype", [ab.BF16, ab.F32])
def test_noalloc_attention_matches_existing_entry_point(rt, orc, kv_dtype):
    B, H, KV, hd, S = 2, 8, 2, 128, 512
    lib = _abi.lib()
    k_host = orc.normal(B * S * KV * hd, 21, 1, 0.0, 1.0).reshape(B, S, KV, hd)
    v_host = orc.normal(B * S * KV * hd, 21, 2, 0.0, 1.0).reshape(B, S, KV, hd)
    if kv_dtype == ab.BF16:
        k = ab.Tensor.from_array(rt, orc.to_bf16_bits(k_host).reshape(k_host.shape), ab.BF16)
        v = ab.Tensor.from_array(rt, orc.to_bf16_bits(v_host).reshape(v_host.shape), ab.BF16)
    else:
        k = ab.Tensor.from_array(rt, k_host)
        v = ab.Tensor.from_array(rt, v_host)
    out = ab.Tensor.zeros(rt, (B, H * hd))
    step = ab.DecodeStep.parcel(rt, B)
    for call, positions in enumerate(([100, 300], [511, 7])):
        q_host = orc.normal(B * H * hd, 22, 10 + call, 0.0, 1.0).reshape(B, H, hd)
        q = ab.Tensor.from_array(rt, q_host)
        rt.deposit(step, [ab.DecodeStep(0, p) for p in positions])
        status = lib.ab_attention_decode_noalloc(rt.stream, q.t, k.t, v.t, out.t, step.t)
        ab._check(status)
        got = out.read()
        want = _existing(rt, q_host, k, v, positions, (S, KV, hd))
        assert rel(got, want) < TOL, (call, rel(got, want))


def test_noalloc_rejects_shapes_beyond_the_static_scratch(rt):
    """batch 64 x 128 heads x (128 + 2) floats exceeds the 4 MiB of partials for any split
    count, so the call is refused on the host. The tensors are real device allocations all
    the same, so nothing could read foreign memory even if it were not."""
    lib = _abi.lib()
    B, H, KV, hd, S = 64, 128, 16, 128, 64
    q = ab.Tensor.zeros(rt, (B, H, hd))
    kc = ab.Tensor.zeros(rt, (B, S, KV, hd), ab.BF16)
    out = ab.Tensor.zeros(rt, (B, H * hd))
    step = ab.DecodeStep.parcel(rt, B)
    status = lib.ab_attention_decode_noalloc(rt.stream, q.t, kc.t, kc.t, out.t, step.t)
    assert status == _abi.AB_ERR_ARGUMENT
    msg = lib.ab_last_error().decode()
    assert "static scratch holds" in msg, msg


def test_noalloc_rejects_host_pointers(rt):
    """A pointer that is not device memory is refused before any launch."""
    lib = _abi.lib()
    host = np.zeros(8 * 128, np.float32)
    q = ab.Tensor(ab.Tensor._desc(host.ctypes.data, ab.F32, (8, 128)))
    kc = ab.Tensor.zeros(rt, (64, 2, 128), ab.BF16)
    out = ab.Tensor.zeros(rt, (8 * 128,))
    step = ab.DecodeStep.parcel(rt)
    status = lib.ab_attention_decode_noalloc(rt.stream, q.t, kc.t, kc.t, out.t, step.t)
    assert status == _abi.AB_ERR_ARGUMENT
    assert "device memory" in lib.ab_last_error().decode()
