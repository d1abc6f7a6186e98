"""bench.py's bookkeeping on CPU: the algorithmic byte and FLOP counts its roofline figures
divide by (restated here by hand on the 8B shapes), the prompt id generator, and the
reference arm's JSON line on the tiny workload."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

W8B = bench.WORKLOADS["llama3-8b-bf16"]


def test_step_bytes_8b_batch1():
    # weights once: per layer (4096 x 6144 + 4096 x 4096 + 3 x 4096 x 14336) bf16, the
    # classifier 128256 x 4096; plus K/V rows 0..pos for 32 layers of 8 x 128 bf16 each
    d, F, V, L = 4096, 14336, 128256, 32
    weights = L * (d * 6144 + d * d + 3 * d * F) * 2 + V * d * 2
    sb = bench.step_bytes(W8B, 1, 199.0)
    kv = L * 2 * 1024 * 2 * 200
    assert abs(sb - weights - kv) / sb < 2e-3  # activations and gains are the remainder
    assert 15.0e9 < weights < 15.1e9  # the 15.01 GB the metric is quoted with


def test_step_bytes_grow_with_position_and_batch():
    assert bench.step_bytes(W8B, 64, 300) > bench.step_bytes(W8B, 64, 100)
    kv64 = bench.step_bytes(W8B, 64, 100) - bench.step_bytes(W8B, 64, 99)
    assert kv64 == 64 * 32 * 2 * 1024 * 2
    # tensor parallel over 8 ranks: one rank's share of the weights and K/V
    assert bench.step_bytes(W8B, 1, 0, shards=8) < bench.step_bytes(W8B, 1, 0) / 7


def test_prefill_flops_by_hand():
    P = 2048
    per_token = 2 * 32 * (4096 * (4096 + 2 * 1024) + 4096 * 4096 + 3 * 4096 * 14336)
    attn = 32 * 4 * 4096 * P * (P + 1) // 2
    assert bench.prefill_flops(W8B, P) == P * per_token + attn + 2 * 128256 * 4096


def test_prompt_tokens_are_seeded_and_in_range():
    a = bench.prompt_tokens(3, 1000, 128, 3, 128256)
    assert a == bench.prompt_tokens(3, 1000, 128, 3, 128256)
    assert a != bench.prompt_tokens(3, 1001, 128, 3, 128256)
    assert all(3 <= t < 128256 for t in a)


@pytest.mark.slow
def test_reference_arm_prints_one_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload",
                        "tiny-llama-f32", "--steps", "2", "--warmup", "1"], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "tokens/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["e2e"]["value"] == d["value"]


def test_sub_decodes_fit_their_contexts():
    # the `configs` decodes of the default line: prompt, 8 warm-up steps, the timed steps and
    # the e2e steps (min(steps, 64)) all stay inside each workload's KV cache
    for name, steps in bench.SUB_DECODES:
        w = bench.WORKLOADS[name]
        need = w["prompt"] - 1 + 8 + steps + min(steps, 64) + 1
        assert need <= w["seq"], (name, need)
    # the 110M streams split over every rank count of the scaling run
    w = bench.WORKLOADS["llama-110m-f32"]
    for world in (1, 2, 4, 8):
        per, first, split = bench.stream_assignment(w, 0, "replicas", world, world - 1)
        assert per * world == 256 and first == 256 - per and split == (world > 1)


def test_cpu_decode_baseline_on_the_tiny_workload():
    w = bench.WORKLOADS["tiny-llama-f32"]
    base = bench.cpu_decode_baseline(w, 1, [10, 20])
    assert base["value"] > 0 and base["unit"] == "tokens/s" and base["kind"] == "port"
    assert base["cores"] >= 1 and "[10, 20]" in base["sample"]


def test_reference_positions_sample_the_timed_range():
    # the default 8B run: positions 135..390, twelve tokens timed, both ends included
    p = bench.reference_positions(135, 390, 256)
    assert len(p) == bench.REF_SAMPLES and p[0] == 135 and p[-1] == 390
    assert p == sorted(set(p)) and all(135 <= x <= 390 for x in p)
    assert bench.reference_positions(10, 11, 2) == [10, 11]
    assert bench.reference_positions(7, 7, 1) == [7]


def test_other_configs_selection_and_errors(monkeypatch):
    # stand-ins for the GPU runners: which sub-records run at N = 1 and N > 1, and a failing
    # one reported in place instead of failing the line
    import argparse

    calls = []

    def fake_decode(args, name, steps, env):
        calls.append((name, steps, env["world"]))
        if name == "tiny-llama-f32":
            raise RuntimeError("boom")
        return {"value": 1.0}

    monkeypatch.setattr(bench, "run_sub_decode", fake_decode)
    for fn in ("run_attention_micro", "run_ops_micro", "run_prefill_micro"):
        monkeypatch.setattr(bench, fn, lambda a, fn=fn: {"value": 2.0, "n_gpus": 1,
                                                          "steps": a.steps, "fn": fn})
    args = argparse.Namespace(steps=256, warmup=8, layers=0, seq=0, no_parity=False,
                              no_cpu_baseline=True, prompt_len=2048)
    out = bench.run_other_configs(args, {"world": 1})
    assert out["tiny-llama-f32"]["error"].startswith("RuntimeError: boom")
    assert out["llama-110m-f32"] == {"value": 1.0}
    assert out["prefill"]["steps"] == 5 and "n_gpus" not in out["prefill"]
    assert set(out) == {"tiny-llama-f32", "llama-110m-f32", "split-attention", "ops", "prefill"}
    calls.clear()
    out = bench.run_other_configs(args, {"world": 4})
    assert set(out) == {"llama-110m-f32"} and calls == [("llama-110m-f32", 256, 4)]
