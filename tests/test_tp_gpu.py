"""Tensor parallelism on real GPUs: two ranks (one process per GPU) decode through the
NVLink peer all-reduce (steps of up to 64 rows) or NCCL's (forced, or wider steps) captured
in the step graph, and every rank's logits and greedy ids match the
CPU oracle's single-device model. Needs two visible GPUs (skipped otherwise)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(dim=128, layers=2, heads=4, kv_heads=2, head_dim=32, hidden=256, vocab=96, seq=32)
# divisible over 4 and 8 ranks (heads, kv heads, FFN columns, vocab rows)
CFG8 = dict(dim=512, layers=2, heads=16, kv_heads=8, head_dim=32, hidden=1024, vocab=256, seq=32)
TOKENS = [5, 90, 12, 12, 44, 3]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, bf16, batch, out, cfg=None, ckpt=None, prefill=False,
            fused=None, first_batch=None, env=None):
    import datetime

    import torch
    import torch.distributed as dist

    import ammon_b200 as ab
    from oracle import oracle as orc

    cfg_d = cfg or CFG
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    os.environ.update(env or {})
    if fused is not None:
        os.environ["AMMON_B200_FUSED_STEP"] = "1" if fused else "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    comm = model = None
    try:
        rt = ab.create_runtime(rank)
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(ab.Comm.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = ab.Comm(rt, bytes(uid.cpu().numpy().tobytes()), rank, world)
        if first_batch is not None:
            # an earlier model of another batch on the same communicator (as bench.py's
            # batch-1 line before its batch-64 record): it sets up the peer slots first
            first = ab.LlamaModel(rt, ab.LlamaConfig(**cfg_d, batch=first_batch,
                                                     rope_theta=500000.0,
                                                     dtype=ab.BF16 if bf16 else ab.F32), comm)
            first.init_synthetic(17, 0.02)
            first.step_batch([TOKENS[0]] * first_batch, [0] * first_batch, logits=False)
            first.close()
        cfg = ab.LlamaConfig(**cfg_d, batch=batch, rope_theta=500000.0,
                             dtype=ab.BF16 if bf16 else ab.F32)
        if ckpt:  # every rank loads its own shard of one llama2.c file
            model = ab.LlamaModel.from_llama2c(rt, ckpt, cfg.dtype, batch, 500000.0, comm)
        else:
            model = ab.LlamaModel(rt, cfg, comm)
            model.init_synthetic(17, 0.02)
        ref = orc.Model(**cfg_d, theta=500000.0, bf16=bf16, seed=17)
        worst, same = 0.0, True
        if fused is not None:
            same &= ("decode_step" in model.scheme().node_labels()) == fused
        if prefill:
            # the prompt in one pass of 6 rows, then in passes of 2 over the same positions
            # (row all-reduces over the NVLink peer slots); then decode continues from the cache
            for want_pos, tok in enumerate(TOKENS):
                want = ref.step(tok, want_pos)
            for rows in (0, 2):
                model.set_prefill_rows(rows)
                logits, am = model.prefill(TOKENS)
                worst = max(worst, float(np.abs(logits - want).max() / np.abs(want).max()))
                same &= am == int(np.argmax(logits)) == orc.sample_argmax(want)
            tok, start = am, len(TOKENS)
            for pos in range(start, start + 3):
                logits, am = model.step_batch([tok] * batch, [pos] * batch, logits=True,
                                              argmax=True)
                want = ref.step(tok, pos)
                worst = max(worst, float(np.abs(logits[0] - want).max() / np.abs(want).max()))
                same &= int(am[0]) == orc.sample_argmax(want)
                tok = int(am[0])
            out.put((rank, worst, same, True))
            return
        for pos, tok in enumerate(TOKENS):
            logits, am = model.step_batch([tok] * batch, [pos] * batch, logits=True, argmax=True)
            want = ref.step(tok, pos)
            for b in range(batch):
                worst = max(worst, float(np.abs(logits[b] - want).max() / np.abs(want).max()))
                same &= int(am[b]) == int(np.argmax(logits[b]))
        # device greedy loop agrees across ranks
        toks = model.decode_device([TOKENS[-1]] * batch, [len(TOKENS) - 1] * batch, 8)
        gathered = [None] * world
        dist.all_gather_object(gathered, toks.tolist())
        out.put((rank, worst, same, all(g == gathered[0] for g in gathered)))
    finally:
        if model is not None:
            model.close()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def _run(bf16, batch, world=2, cfg=None, ckpt=None, prefill=False, fused=None,
         first_batch=None, env=None):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, bf16, batch, q, cfg, ckpt,
                                                    prefill, fused, first_batch, env))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [q.get(timeout=5) for _ in range(world)]


def test_tensor_parallel_fp32_matches_oracle():
    for rank, worst, same, agree in _run(False, 1):
        assert worst < 1e-5, (rank, worst)
        assert same and agree


@pytest.mark.parametrize("nccl", [False, True])
def test_tensor_parallel_bf16_batched_matches_oracle(nccl):
    # batch 6: the NVLink peer all-reduce (up to 64 rows), or NCCL's when forced
    env = {"AMMON_B200_TP_NCCL": "1"} if nccl else None
    for rank, worst, same, agree in _run(True, 6, env=env):
        assert worst < 2e-2, (rank, worst)
        assert same and agree


@pytest.mark.parametrize("world", [4, 8])
def test_tensor_parallel_wide_matches_oracle(world):
    """Four or eight ranks (one kv head per rank at eight): the peer all-reduce with more
    sources, at batch 1 and batch 6 (NVLink peer slots)."""
    for rank, worst, same, agree in _run(False, 1, world, CFG8):
        assert worst < 1e-5, (world, rank, worst)
        assert same and agree
    for rank, worst, same, agree in _run(True, 6, world, CFG8):
        assert worst < 2e-2, (world, rank, worst)
        assert same and agree


def test_tensor_parallel_llama2c_shards_match_oracle(tmp_path):
    """Each rank slices its rows / columns out of one llama2.c checkpoint written with the
    oracle's fp32 weights; the sharded decode matches the oracle's single-device model."""
    from oracle import oracle as orc
    from test_checkpoint import write_llama2c

    path = str(tmp_path / "tp.bin")
    write_llama2c(path, orc.Model(**CFG, theta=500000.0, seed=17).weight, CFG)
    for rank, worst, same, agree in _run(False, 1, ckpt=path):
        assert worst < 1e-5, (rank, worst)
        assert same and agree


def test_tensor_parallel_prefill_matches_oracle():
    """Sharded prefill passes (row all-reduces over the NVLink peer slots at 6 and at 2
    rows) leave every rank with the oracle's last-token logits and a cache the decode
    continues from."""
    for rank, worst, same, _ in _run(False, 1, prefill=True):
        assert worst < 1e-5, (rank, worst)
        assert same


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_persistent_step_matches_oracle(world):
    """bf16 at batch 1 runs the persistent single-launch step on every rank: partial wo / w2
    rows go straight into every rank's exchange block over NVLink, a system-scope arrival
    counter per rank closes each all-reduce site, the ranks' argmax candidates merge inside
    the kernel. Logits match the single-device oracle at the bf16 bar, every rank picks the
    same ids, and the per-kernel TP step graph (AMMON_B200_FUSED_STEP=0) agrees."""
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cfg = CFG if world == 2 else CFG8
    fused = _run(True, 1, world, cfg, fused=True)
    for rank, worst, same, agree in fused:
        assert worst < 2e-2, (world, rank, worst)
        assert same and agree
    graph = _run(True, 1, world, cfg, fused=False)
    for rank, worst, same, agree in graph:
        assert worst < 2e-2, (world, rank, worst)
        assert same and agree


def test_tensor_parallel_models_of_two_batches_share_a_communicator():
    # a batch-1 model then a batch-6 model on one communicator (the peer slots the first one
    # set up serve both): the second one is created and matches the oracle
    for rank, worst, same, agree in _run(True, 6, first_batch=1):
        assert worst < 2e-2, (rank, worst)
        assert same and agree
