"""Failure paths of the device waits and of the communicator, made on the host (no GPU fault,
trap or hang): the limit of every bounded wait is a runtime parameter; the tensor-parallel
all-reduce kernel, run on one GPU over ranks whose arrival words sit in this GPU's memory,
sums the ranks in rank order when all arrive and gives up after the limit when one never
does (DeviceError, device still usable); a communicator whose second rank never joins ends
the first rank's create call after its timeout with the rendezvous communicator aborted.
The reference has no device-side waits or collectives; its contract that a failure surfaces
as an error before anything else runs (src/blocks.rs:183-216) is the model."""
import os
import subprocess
import sys
import time

import numpy as np
import pytest

import ammon_b200 as ab

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def rt():
    r = ab.create_runtime(0)
    yield r
    r.synchronize()


def _partials(world, n):
    i = np.arange(n)
    return [np.float32(r + 1) + np.float32(0.25) * (i % 7).astype(np.float32)
            for r in range(world)]


def test_wait_limit_is_a_runtime_parameter(rt):
    old = rt.wait_limit_ms
    assert old > 0
    rt.wait_limit_ms = 37
    assert rt.wait_limit_ms == 37
    with pytest.raises(ab.AmmonError, match="at least 1 ms"):
        rt.wait_limit_ms = 0
    rt.wait_limit_ms = old
    assert rt.wait_limit_ms == old


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("n", [1, 1000, 4096, 70001])
def test_loopback_reduce_sums_every_rank_in_order(rt, world, n):
    got = ab.Comm.loopback_reduce(rt, world, (1 << world) - 1, n)
    want = np.zeros(n, np.float32)
    for part in _partials(world, n):
        want = want + part
    assert np.array_equal(got, want)


@pytest.mark.parametrize("world,ready", [(2, 0b01), (4, 0b1011), (8, 0b01111111)])
def test_loopback_reduce_with_a_rank_that_never_arrives_times_out(rt, world, ready):
    old = rt.wait_limit_ms
    rt.wait_limit_ms = 20
    try:
        t0 = time.time()
        with pytest.raises(ab.DeviceError, match="bounded wait timed out"):
            ab.Comm.loopback_reduce(rt, world, ready, 4096)
        assert time.time() - t0 < 10
    finally:
        rt.wait_limit_ms = old
    # the device still answers: the same reduce with every rank arriving
    got = ab.Comm.loopback_reduce(rt, world, (1 << world) - 1, 4096)
    want = np.zeros(4096, np.float32)
    for part in _partials(world, 4096):
        want = want + part
    assert np.array_equal(got, want)


_NEVER_JOINS = r"""
import sys, time
import torch  # loads the NCCL library the communicator binds to
import numpy as np
import ammon_b200 as ab
rt = ab.create_runtime(0)
uid = ab.Comm.unique_id()
t0 = time.time()
try:
    ab.Comm(rt, uid, 0, 2, timeout_ms=3000)
    print("JOINED")
    sys.exit(1)
except ab.AmmonError as e:
    dt = time.time() - t0
    print("ERROR", dt, str(e))
got = ab.Comm.loopback_reduce(rt, 2, 3, 1024)
print("AFTER", float(got[0]))
rt.close()
"""


def test_communicator_with_a_rank_that_never_joins_times_out():
    """Rank 0 of a world of 2 whose rank 1 never starts: the create call returns after its
    3 s timeout with the rendezvous aborted, and the process keeps using its GPU. Run in a
    child process so that NCCL's state of the failed rendezvous dies with it."""
    r = subprocess.run([sys.executable, "-c", _NEVER_JOINS], cwd=ROOT, capture_output=True,
                       text=True, timeout=240)
    out = r.stdout
    assert r.returncode == 0, (out, r.stderr[-3000:])
    err = [l for l in out.splitlines() if l.startswith("ERROR")]
    assert err, out
    _, dt, msg = err[0].split(" ", 2)
    assert "did not" in msg or "joined" in msg, msg
    assert "aborted" in msg, msg
    assert 2.5 < float(dt) < 60, dt
    assert "AFTER 3.0" in out, out
