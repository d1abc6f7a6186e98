"""Generate tests/golden/attention_f64.npz: the reference test suite's fp64 attention
oracle (Ammon tests/kernels.rs:400-427) evaluated on its own five cases
(tests/kernels.rs:493-538) with its own xorshift inputs (tests/kernels.rs:380-390).

This is a pure-numpy restatement, written independently of oracle/oracle.c, so the
committed fixture cross-checks the C oracle. When the reference checkout is present
(`AMMON_REFERENCE` or the default path below), the script also confirms that the case
table in known_answers.json matches the reference test file's literals.

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def pseudo_random(length: int, seed: int) -> np.ndarray:
    """xorshift32 of tests/kernels.rs:380-390 (u32 wrapping arithmetic)."""
    state = (seed * 2654435761 + 1) & 0xFFFFFFFF
    out = np.empty(length, np.float32)
    for i in range(length):
        state ^= (state << 13) & 0xFFFFFFFF
        state ^= state >> 17
        state ^= (state << 5) & 0xFFFFFFFF
        out[i] = np.float32(state % 2001) / np.float32(1000.0) - np.float32(1.0)
    return out


def cpu_attention(q_heads, kv_heads, head, q, key, value, pos) -> np.ndarray:
    """tests/kernels.rs:400-427 in float64."""
    kv_dim = kv_heads * head
    kv_mul = q_heads // kv_heads
    q = q.astype(np.float64).reshape(q_heads, head)
    key = key.astype(np.float64).reshape(-1, kv_dim)
    value = value.astype(np.float64).reshape(-1, kv_dim)
    out = np.zeros((q_heads, head), np.float64)
    for h in range(q_heads):
        base = (h // kv_mul) * head
        k = key[: pos + 1, base:base + head]
        v = value[: pos + 1, base:base + head]
        scores = (k @ q[h]) / np.sqrt(head)
        w = np.exp(scores - scores.max())
        out[h] = (w[:, None] * v).sum(0) / w.sum()
    return out.reshape(-1)


def check_reference_table(cases) -> None:
    ref = os.environ.get("AMMON_REFERENCE")
    if not ref:
        print("AMMON_REFERENCE (a checkout of the reference crate) not set; case table not "
              "re-checked")
        return
    path = os.path.join(ref, "tests", "kernels.rs")
    if not os.path.exists(path):
        print(f"{path} absent; case table not re-checked")
        return
    text = open(path).read()
    pat = re.compile(r"AttentionCase\s*\{\s*q_heads:\s*(\d+),\s*kv_heads:\s*(\d+),\s*head:\s*(\d+),"
                     r"\s*seq:\s*(\d+),\s*positions:\s*&\[([\d,\s]+)\]")
    found = [(int(a), int(b), int(c), int(d), [int(p) for p in e.split(",") if p.strip()])
             for a, b, c, d, e in pat.findall(text)]
    mine = [(c["q_heads"], c["kv_heads"], c["head"], c["seq"], c["positions"]) for c in cases]
    assert found == mine, f"case table differs from the reference: {found} vs {mine}"
    print("case table matches tests/kernels.rs")


def main() -> None:
    spec = json.load(open(os.path.join(HERE, "known_answers.json")))["attention_cases"]
    check_reference_table(spec["cases"])
    arrays = {}
    for ci, c in enumerate(spec["cases"]):
        qh, kvh, hd, seq = c["q_heads"], c["kv_heads"], c["head"], c["seq"]
        q = pseudo_random(qh * hd, spec["q_seed"])
        key = pseudo_random(seq * kvh * hd, spec["key_seed"])
        value = pseudo_random(seq * kvh * hd, spec["value_seed"])
        arrays[f"case{ci}_q"] = q
        arrays[f"case{ci}_key_head"] = key[:64]
        for pos in c["positions"]:
            arrays[f"case{ci}_pos{pos}"] = cpu_attention(qh, kvh, hd, q, key, value, pos)
    np.savez_compressed(os.path.join(HERE, "attention_f64.npz"), **arrays)
    print("wrote attention_f64.npz with", len(arrays), "arrays")


if __name__ == "__main__":
    main()
