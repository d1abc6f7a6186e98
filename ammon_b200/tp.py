"""Tensor-parallel shard plan of the Llama-shaped model (mirrors model.cu's
create_model / ab_llama_init_synthetic).

Rank r of `world` holds, for each weight, a contiguous range along one axis of the
global tensor: row shards for wq, wk, wv, w1, w3 and the classifier, column shards for
wo and w2; the embedding table and the norm gains are replicated. The residual stream is
replicated: after wo and after w2 the ranks' partial projections are summed into it by an
all-reduce, rank 0's partial carrying the residual itself.
"""
from __future__ import annotations

from typing import Dict, Tuple


def shard_plan(dim: int, heads: int, kv_heads: int, head_dim: int, hidden: int, vocab: int,
               rank: int, world: int) -> Dict[str, Tuple[int, int, int]]:
    """name -> (axis, start, stop) of this rank's slice of the global weight."""
    for name, n in (("heads", heads), ("kv_heads", kv_heads), ("hidden", hidden),
                    ("vocab", vocab)):
        if n % world:
            raise ValueError(f"{name} {n} is not divisible by {world} ranks")
    qd = heads // world * head_dim
    kvd = kv_heads // world * head_dim
    f = hidden // world
    v = vocab // world
    r = rank
    return {
        "wq": (0, r * qd, (r + 1) * qd),
        "wk": (0, r * kvd, (r + 1) * kvd),
        "wv": (0, r * kvd, (r + 1) * kvd),
        "wo": (1, r * qd, (r + 1) * qd),
        "w1": (0, r * f, (r + 1) * f),
        "w3": (0, r * f, (r + 1) * f),
        "w2": (1, r * f, (r + 1) * f),
        "wcls": (0, r * v, (r + 1) * v),
        "embed": (0, 0, vocab),
    }


def take(weight, spec):
    axis, lo, hi = spec
    return weight[lo:hi] if axis == 0 else weight[:, lo:hi]
