"""The data-parallel split of the 110M workload's 256 independent streams (no collective on
the data path), on CPU with gloo ranks: every rank takes bench.stream_assignment's contiguous
block, decodes its streams with the CPU oracle (one step each), and the ranks' results
gathered afterwards equal one process decoding all the streams. The timing reduction
(max over ranks) and the whole-job value (all ranks' streams / that time) are checked the
same way. A shrunken model of the 110M layout keeps the oracle fast; the split only depends
on the stream count."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

W110 = bench.WORKLOADS["llama-110m-f32"]
SMALL = dict(dim=32, layers=1, heads=4, kv_heads=4, head_dim=8, hidden=48, vocab=64, seq=8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_stream_blocks_partition_the_batch(world):
    seen = []
    for rank in range(world):
        B, first, split = bench.stream_assignment(W110, 0, "auto", world, rank)
        assert B == 256 // world and first == rank * B and split == (world > 1)
        seen.extend(range(first, first + B))
    assert seen == list(range(256))
    # tensor parallel ranks (the 8B default) all decode the same streams
    W8B = bench.WORKLOADS["llama3-8b-bf16"]
    assert {bench.stream_assignment(W8B, 0, "auto", world, r)[:2] for r in range(world)} == {
        (1, 0)}
    # an explicit --batch is per rank, replicas decode distinct streams
    assert [bench.stream_assignment(W110, 3, "replicas", world, r)[1]
            for r in range(world)] == [3 * r for r in range(world)]


def _worker(rank, world, port, out):
    import torch
    import torch.distributed as dist

    from oracle import oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, first, split = bench.stream_assignment(W110, 0, "auto", world, rank)
        m = orc.Model(**SMALL, seed=1)
        ids = np.zeros(B, np.int64)
        for k in range(B):
            m.reset()
            tok = orc.uniform_tokens(1, 1, 1000 + first + k, 3, SMALL["vocab"])[0]
            ids[k] = orc.sample_argmax(m.step(int(tok), 0))
        m.close()
        # the bench's timing reduction: every rank's device time, max over ranks
        t = torch.tensor([0.5 + 0.25 * rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gathered = [torch.zeros(B, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(ids))
        if rank == 0:
            out.put((float(t.item()), torch.cat(gathered).numpy().tolist(), B, split))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_decode_the_split_like_one_process(orc):
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    t_max, ids, B, split = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert split and B == 128 and t_max == 0.75
    m = orc.Model(**SMALL, seed=1)
    want = []
    for s in range(256):
        m.reset()
        tok = orc.uniform_tokens(1, 1, 1000 + s, 3, SMALL["vocab"])[0]
        want.append(orc.sample_argmax(m.step(int(tok), 0)))
    m.close()
    assert ids == want
    # whole-job value as bench.py reports it for the split: all ranks' streams / max time
    assert world * B * 1 / t_max == 256 / 0.75


def test_reference_arm_config_matches_the_gpu_arm(tmp_path):
    """The reference arm's config is built by the GPU arm's function from the same positions,
    so the two lines name one workload (same keys, same values)."""
    import json
    import subprocess

    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload",
                        "tiny-llama-f32", "--steps", "2", "--warmup", "3"], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])

    class A:
        warmup, steps = 3, 2

    w = bench.WORKLOADS["tiny-llama-f32"]
    first, last = bench.timed_positions(w, A)
    assert d["config"] == bench.decode_config(w, 1, first, last, 1, "single")
    assert d["config"]["positions"] == f"{w['prompt'] - 1 + 3}..{w['prompt'] - 1 + 3 + 1}"
    assert "full tokens" in d["cpu_baseline"]["sample"]
