"""C-ABI boundary on CPU: the library loads, exports exactly what the header declares,
and record-time validation follows the reference's contract (errors name the
parameter / rank / symbolic dim, and a rejected record adds no node:
tests/kernels.rs:125-146,357-378,540-556). No kernel runs here."""
import ctypes as C
import subprocess

import numpy as np
import pytest

import ammon_b200 as ab
from ammon_b200 import _abi

FAKE = 0x10000  # device pointers are never dereferenced at record time


def fake(shape, dtype=ab.F32, ptr=FAKE):
    return ab.Tensor(ab.Tensor._desc(ptr, dtype, shape))


def step1():
    return fake((1, 2), ab.U32, ptr=FAKE * 2)


@pytest.fixture()
def scheme():
    s = ab.Scheme(None)
    yield s
    s.close()


def test_library_exports_every_header_symbol():
    _abi.lib()
    declared = set(_abi.header_symbols())
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert declared, "header parse found no declarations"
    assert declared <= exported, sorted(declared - exported)
    assert {s for s in exported if s.startswith("ab_")} == declared
    assert set(_abi.SIGNATURES) == declared


def expect_error(fn, *needles, cls=ab.ValidationError):
    with pytest.raises(cls) as e:
        fn()
    for n in needles:
        assert n in str(e.value), str(e.value)
    return e.value


def test_gemv_rejects_rank1_output(scheme):
    g = ab.kernels.GemvKernel.prepare(None)
    before = scheme.ir_node_count()
    expect_error(lambda: g.record(scheme, "gemv_rank1", fake((2,)), fake((2, 2)), fake((2,)),
                                  step1()), "expected rank 2")
    assert scheme.ir_node_count() == before


def test_rope_rejects_rank2_kv_cache(scheme):
    k = ab.kernels.RopeKernel.prepare(None)
    before = scheme.ir_node_count()
    expect_error(lambda: k.record(scheme, "rope_rank", fake((2, 2)), fake((1, 4)), step1(),
                                  ab.DEFAULT_ROPE_THETA), "parameter `k`", "expected rank 3")
    assert scheme.ir_node_count() == before


def test_embed_rejects_dim_mismatch(scheme):
    k = ab.kernels.EmbedKernel.prepare(None)
    before = scheme.ir_node_count()
    expect_error(lambda: k.record(scheme, "embed_dim", fake((2, 2)), step1(), fake((3,))),
                 "parameter `x`", "`dim`")
    assert scheme.ir_node_count() == before


def test_valid_records_add_nodes(scheme):
    ab.kernels.EmbedKernel.prepare(None).record(scheme, "embed", fake((2, 2)), step1(),
                                                fake((2,)))
    ab.kernels.TensorKernels.prepare(None).matmul_into(scheme, "mm", fake((2, 2)), fake((2,)),
                                                       fake((2,)))
    assert scheme.ir_node_count() == 2


def test_attention_partial_contract(scheme):
    k = ab.kernels.AttentionPartialKernel.prepare(None)
    q, kc = fake((4, 200)), fake((16, 2, 200))
    expect_error(lambda: k.record(scheme, "p", q, kc, kc, fake((4, 2, 202)), step1()),
                 "exceeds 128")
    q, kc = fake((4, 64)), fake((16, 2, 64))
    expect_error(lambda: k.record(scheme, "p", q, kc, kc, fake((4, 1, 66)), step1()),
                 "parameter `partial`", "`splits`")
    expect_error(lambda: k.record(scheme, "p", q, kc, kc, fake((4, 2, 64)), step1()),
                 "parameter `partial`", "`slot`")
    assert scheme.ir_node_count() == 0
    k.record(scheme, "p", q, kc, kc, fake((4, 2, 66)), step1())
    assert scheme.ir_node_count() == 1


def test_step_parcel_contract(scheme):
    k = ab.kernels.EmbedKernel.prepare(None)
    expect_error(lambda: k.record(scheme, "e", fake((4, 8)), fake((1, 3), ab.U32), fake((8,))),
                 "parameter `step`")
    expect_error(lambda: k.record(scheme, "e", fake((4, 8)), step1(), fake((2, 8))),
                 "parameter `step`", "batch needs 2")


def test_linear_contract(scheme):
    lin = ab.Linear(None)
    expect_error(lambda: lin.record(scheme, fake((4, 8)), fake((7,)), fake((4,))),
                 "parameter `x`", "`d_in`")
    expect_error(lambda: lin.record(scheme, fake((4, 8)), fake((8,)), fake((5,))),
                 "parameter `out`", "`d_out`")
    expect_error(lambda: lin.record(scheme, fake((4, 8), ab.F32), fake((8,), ab.BF16),
                                    fake((4,))), "f32 weights")
    assert scheme.ir_node_count() == 0


def test_submit_without_runtime_is_an_argument_error(scheme):
    with pytest.raises(ab.AmmonError) as e:
        scheme.submit()
    assert e.value.code == _abi.AB_ERR_ARGUMENT


def test_view_arithmetic():
    t = fake((4, 6))
    n = t.narrow(0, 1, 2)
    assert n.shape == (2, 6) and n.data_ptr == FAKE + 6 * 4
    r = t.reshape((24,))
    assert r.shape == (24,)
    with pytest.raises(ab.ValidationError):
        t.reshape((5, 5))
    with pytest.raises(ab.ValidationError):
        t.narrow(0, 3, 2)
