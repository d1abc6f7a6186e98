"""ab_attention_decode_noalloc: the allocation-free variant of the fused flash-decoding
attention, for callers that must not allocate device memory themselves (hosts whose
device memory belongs to their own pooling allocator, or loops that cannot take
cudaFree's device-wide synchronisation). Its split scratch is a static device array
inside the library.

Checked through the C ABI against the existing attention entry points
(ab_kernel_attention_partial + ab_kernel_attention_combine, which take caller-allocated
scratch) and against float64 on the same inputs, on several calls in a row; a position
beyond the cache is reported through the companion status call. Runs last, and also alone
in a fresh process (the first call on the device performs the array's address lookup)."""
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


def _float64(q_host, k_host, v_host, positions):
    """Softmax attention over positions 0..pos of each row in float64 (src/kernels.rs:412-460
    semantics, GQA: query head h reads kv head h // (H / KV))."""
    B, H, hd = q_host.shape
    KV = k_host.shape[2]
    out = np.zeros((B, H * hd))
    for b in range(B):
        p = positions[b]
        for h in range(H):
            kv = h // (H // KV)
            sc = k_host[b, : p + 1, kv].astype(np.float64) @ q_host[b, h] / np.sqrt(hd)
            w = np.exp(sc - sc.max())
            out[b, h * hd:(h + 1) * hd] = (w / w.sum()) @ v_host[b, : p + 1, kv]
    return out


def _status(lib, rt):
    flags = _abi.C.c_uint32(0)
    status = lib.ab_attention_decode_noalloc_status(rt.stream, _abi.C.byref(flags))
    return status, flags.value


@pytest.mark.parametrize("kv_dtype", [ab.BF16, ab.F32])
def test_noalloc_attention_matches_existing_entry_point(rt, orc, kv_dtype):
    """Four calls in a row (positions that end inside a tile, on a 64-position tile boundary
    and on the 256-position minimum split boundary) against the existing entry points and
    against float64 on the same (bf16-rounded) K/V."""
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
    if kv_dtype == ab.BF16:
        k_host = orc.round_bf16(k_host).reshape(k_host.shape)
        v_host = orc.round_bf16(v_host).reshape(v_host.shape)
    out = ab.Tensor.zeros(rt, (B, H * hd))
    step = ab.DecodeStep.parcel(rt, B)
    for call, positions in enumerate(([100, 300], [511, 7], [255, 256], [63, 64])):
        q_host = orc.normal(B * H * hd, 22, 10 + call, 0.0, 1.0).reshape(B, H, hd)
        q = ab.Tensor.from_array(rt, q_host)
        rt.deposit(step, [ab.DecodeStep(0, p) for p in positions])
        status = lib.ab_attention_decode_noalloc(rt.stream, q.t, k.t, v.t, out.t, step.t)
        ab._check(status)
        got = out.read()
        want = _existing(rt, q_host, k, v, positions, (S, KV, hd))
        assert rel(got, want) < TOL, (call, rel(got, want))
        # the fused bf16 kernel multiplies through bf16 hi + lo halves of q and p
        f64 = _float64(q_host, k_host, v_host, positions)
        assert rel(got, f64) < (1e-4 if kv_dtype == ab.BF16 else TOL), (call, rel(got, f64))
    assert _status(lib, rt) == (_abi.AB_OK, 0)


def test_noalloc_reports_a_position_beyond_seq(rt):
    """A row whose position is >= seq gets a zero row and raises the sticky flag word, which
    the status call reports as AB_ERR_DEVICE once and then clears; the other row is computed
    as usual. Nothing reads outside the cache: the row has no positions to attend over."""
    lib = _abi.lib()
    B, H, KV, hd, S = 2, 4, 2, 64, 128
    k = ab.Tensor.zeros(rt, (B, S, KV, hd), ab.BF16).fill_normal(3, 1)
    v = ab.Tensor.zeros(rt, (B, S, KV, hd), ab.BF16).fill_normal(3, 2)
    q = ab.Tensor.zeros(rt, (B, H, hd)).fill_normal(3, 3)
    out = ab.Tensor.zeros(rt, (B, H * hd)).fill_normal(3, 4)
    step = ab.DecodeStep.parcel(rt, B)
    rt.deposit(step, [ab.DecodeStep(0, 40), ab.DecodeStep(0, S)])
    ab._check(lib.ab_attention_decode_noalloc(rt.stream, q.t, k.t, v.t, out.t, step.t))
    status, flags = _status(lib, rt)
    assert status == _abi.AB_ERR_DEVICE and flags == 2, (status, flags)
    assert "seq_len" in lib.ab_last_error().decode()
    got = out.read()
    assert np.all(got[1] == 0.0) and np.abs(got[0]).max() > 0
    assert _status(lib, rt) == (_abi.AB_OK, 0)


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
