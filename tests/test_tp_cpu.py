"""The tensor-parallel decomposition, on CPU with two gloo ranks: each rank computes one
decoder layer from its shards (ammon_b200.tp.shard_plan, the plan model.cu follows),
rank 0's partial projections carry the residual, and an all-reduce sums the partials into
the replicated residual stream. The result must equal the CPU oracle's single-device
layer (src/blocks.rs:178-278 order) within the fp32 bar."""
import os
import socket

import numpy as np
import pytest

CFG = dict(dim=64, layers=1, heads=4, kv_heads=2, head_dim=16, hidden=96, vocab=40, seq=8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rmsnorm(x, w, eps=1e-5):
    return w * (x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + eps))


def _worker(rank, world, port, out):
    import torch
    import torch.distributed as dist

    from ammon_b200.tp import shard_plan, take
    from oracle import oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = orc.Model(**CFG, seed=21)
        plan = shard_plan(CFG["dim"], CFG["heads"], CFG["kv_heads"], CFG["head_dim"],
                          CFG["hidden"], CFG["vocab"], rank, world)
        hd = CFG["head_dim"]
        tok, pos = 7, 0
        x = m.weight("embed")[tok].astype(np.float64)
        # attention block: local heads, local kv heads (position 0: attention returns v)
        xb = _rmsnorm(x, m.weight("rms_att"))
        q = take(m.weight("wq"), plan["wq"]) @ xb
        v = take(m.weight("wv"), plan["wv"]) @ xb
        g = CFG["heads"] // CFG["kv_heads"]
        o = np.concatenate([v[(h // g) * hd:(h // g + 1) * hd] for h in range(q.size // hd)])
        y = take(m.weight("wo"), plan["wo"]) @ o
        if rank == 0:
            y = y + x
        t = torch.from_numpy(y.copy())
        dist.all_reduce(t)
        x1 = t.numpy()
        # SwiGLU block
        xb = _rmsnorm(x1, m.weight("rms_ffn"))
        h1 = take(m.weight("w1"), plan["w1"]) @ xb
        h3 = take(m.weight("w3"), plan["w3"]) @ xb
        hb = h1 / (1 + np.exp(-h1)) * h3
        y = take(m.weight("w2"), plan["w2"]) @ hb
        if rank == 0:
            y = y + x1
        t = torch.from_numpy(y.copy())
        dist.all_reduce(t)
        x2 = t.numpy()
        if rank == 0:
            m.embed_token(tok)
            m.attention_block(0, pos)
            m.ffn_block(0)
            want = m.tensor("x")
            out.put(float(np.abs(x2 - want).max() / np.abs(want).max()))
        # shards tile the global tensors exactly
        spans = [None] * world
        dist.all_gather_object(spans, plan)
        if rank == 0:
            ok = True
            for name in ("wq", "wk", "wv", "wo", "w1", "w3", "w2", "wcls"):
                cut = sorted((s[name][1], s[name][2]) for s in spans)
                ok &= cut[0][0] == 0 and all(a[1] == b[0] for a, b in zip(cut, cut[1:]))
            out.put(ok)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_layer_matches_oracle_on_two_gloo_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = q.get(timeout=5)
    tiles = q.get(timeout=5)
    assert err < 1e-5, err
    assert tiles


def test_shard_plan_rejects_uneven_splits():
    from ammon_b200.tp import shard_plan

    with pytest.raises(ValueError, match="kv_heads"):
        shard_plan(4096, 32, 8, 128, 14336, 128256, 0, 16)
    p = shard_plan(4096, 32, 8, 128, 14336, 128256, 7, 8)
    assert p["wk"] == (0, 7 * 128, 8 * 128) and p["w2"] == (1, 7 * 1792, 8 * 1792)
    assert p["wcls"] == (0, 7 * 16032, 8 * 16032)
