#!/usr/bin/env python
"""Decode throughput of the B200-native Ammon decode layer path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--batch B]
                    [--impl ammon|reference]

Workload (default): the Llama-3-8B-shaped bf16 decode (dim 4096, 32 layers, 32/8 heads,
head_dim 128, SwiGLU 14336, vocab 128256, RoPE theta 500000, max context 8192,
N(0, 0.02) synthetic weights from seed 3, a 128-token uniform prompt) at batch 1.
One step = one greedy decode token for every stream of the batch.

value:  tokens/s of the device-resident greedy loop (graph replays, device argmax feeds
        the next DecodeStep), CUDA events on the decode stream, max over ranks.
e2e:    tokens/s through the reference-facing step() (AutoregressiveModel::step): every
        step uploads the DecodeSteps and reads [batch, vocab] fp32 logits back to the
        host (into a page-locked buffer) together with the library's greedy pick of them
        (sample_argmax's first-maximum rule, on the device), which feeds the next step.
With N > 1 (one process per GPU under torch.distributed.run):
  --parallel tp (default for the bf16 8B workload): the model is tensor parallel over the
        ranks (heads, kv heads, FFN columns and vocab split; one all-reduce after wo and one
        after w2 per layer over NVLink: inside the persistent step at batch 1, the peer
        all-reduce kernel up to 64 rows, NCCL beyond); all ranks decode the same
        batch, so value is that batch's tokens/s ("scaling": "strong").
  --parallel replicas (default for the fp32 workloads): every rank decodes its own batch
        of independent streams with no collective; value is the sum over ranks
        ("scaling": "weak").
The default line also carries `batch64` (the same 8B decode at batch 64) and `configs`, the
other BASELINE.json configurations, each with its own metric, unit, roofline and CPU
baseline: the tiny fp32 decode, the 110M fp32 decode of 256 streams (split data-parallel
over the ranks at N > 1, the only sub-record run there), and at N = 1 the split-attention,
per-op and prefill microbenchmarks (`--workload attention|ops|prefill` run them alone).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/sec (batch 1 and 64) at 1/2/4/8 B200; per-kernel HBM GB/s vs peak"

WORKLOADS = {
    "llama3-8b-bf16": dict(dim=4096, layers=32, heads=32, kv_heads=8, head_dim=128,
                           hidden=14336, vocab=128256, seq=8192, theta=500000.0, bf16=True,
                           seed=3, prompt=128, batch=1,
                           title="Llama-3-8B-shaped bf16 decode"),
    "llama-110m-f32": dict(dim=768, layers=12, heads=12, kv_heads=12, head_dim=64, hidden=2048,
                           vocab=32000, seq=1024, theta=10000.0, bf16=False, seed=1, prompt=16,
                           batch=256, split_streams=True,
                           title="Llama-shaped 110M fp32 multi-stream decode"),
    "tiny-llama-f32": dict(dim=288, layers=6, heads=6, kv_heads=6, head_dim=48, hidden=768,
                           vocab=32000, seq=256, theta=10000.0, bf16=False, seed=0, prompt=8,
                           batch=1, title="Tiny llama2.c fp32 decode"),
}

# Kernel microbenchmarks (one JSON line each, GB/s against the measured HBM peak)
MICRO = {
    "ops": "Per-op microbench: RmsNorm rows {1,64,4096} x dim {4096,8192}, RoPE 32x128 at "
           "positions 0-8191 (theta 500000), SwiGLU rows {1,64} x 14336, embedding gather "
           "from 128256 x 4096; N(0,1) activations in f32 and bf16",
    "prefill": "Batched prefill of one stream on the Llama-3-8B-shaped bf16 model: a uniform "
               "prompt (seed 3) in passes of up to 256 rows, last token's logits read back",
    "attention": "Split attention decode: 32 query / 8 kv heads, head_dim 128, bf16 K/V, fp32 "
                 "accumulation; context {4096,32768,131072} x batch {1,8,64}; N(0,1) seed 2",
}

SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


# ----------------------------------------------------------------------------- helpers
class StdoutToStderr:
    """Sends file descriptor 1 to stderr while NCCL initialises (NCCL may print its
    version banner on stdout, which must carry only the JSON line)."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        import ctypes

        ctypes.CDLL(None).fflush(None)
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)
        return False


def _mix64(z):
    M = (1 << 64) - 1
    z = (z + 0x9E3779B97F4A7C15) & M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    return z ^ (z >> 31)


def prompt_tokens(seed, stream, n, lo, hi):
    """Uniform ids in [lo, hi): the generator the oracle uses (splitmix64 of seed/stream)."""
    M = (1 << 64) - 1
    key = _mix64(((seed * 0xD1B54A32D192ED03) & M) ^ _mix64(stream))
    return [lo + _mix64((key + i) & M) % (hi - lo) for i in range(n)]


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(kernel, workload, algorithmic=None):
    """Per-launch DRAM bytes of `kernel` from a committed ncu summary of this workload
    (profiles/<kernel>*<workload>*.md, a `traffic_bytes_per_launch:` entry). When the summary
    also states the capture's `algorithmic_bytes_per_launch:` (position-dependent launches,
    e.g. attention), the traffic is scaled to this launch's algorithmic bytes."""
    import glob
    import re

    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", f"{kernel}*{workload}*.md"))):
        text = open(path).read()
        m = re.search(r"traffic_bytes_per_launch:\s*\|?\s*([0-9.]+)", text)
        if not m:
            continue
        traffic = float(m.group(1))
        a = re.search(r"algorithmic_bytes_per_launch:\s*\|?\s*([0-9.]+)", text)
        if a and algorithmic:
            traffic *= algorithmic / float(a.group(1))
        return traffic
    return None


class ClockSampler:
    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def layer_bytes(w, batch, shards=1, attn_pos=None):
    """Algorithmic bytes per launch of each fused kernel (weights once, activations and
    KV rows read/written), for the kernel labels the step graph records. With tensor
    parallelism over `shards` ranks, one rank's share (the weights and K/V are split).
    attn_pos: the position the attention launch decodes at (K/V rows 0..pos per stream)."""
    e = 2 if w["bf16"] else 4
    d, F, V = w["dim"], w["hidden"] // shards, w["vocab"] // shards
    qd = w["heads"] // shards * w["head_dim"]
    kvd = w["kv_heads"] // shards * w["head_dim"]
    out = {
        "ffn_gate_up_swiglu": 2 * F * d * e + batch * (d * 4 + F * e) + d * e,
        "ffn_down_residual": d * F * e + batch * (F * e + 2 * d * 4),
        "attn_qkv_rope": (qd + 2 * kvd) * d * e + batch * (d * 4 + qd * 4 + 2 * kvd * e) + d * e,
        "attn_wo_residual": d * qd * e + batch * (qd * e + 2 * d * 4),
        "final_norm_classifier": V * d * e + batch * (d * 4 + V * 4) + d * e,
    }
    if attn_pos is not None:
        out["attn_decode"] = batch * (2 * kvd * e * (attn_pos + 1) + qd * 4 + qd * e)
    out["attn_wo_partial"] = out["attn_wo_residual"]
    out["ffn_down_partial"] = out["ffn_down_residual"]
    return out


def step_bytes(w, batch, mean_pos, shards=1):
    """Algorithmic bytes of one decode step (per rank): all weights once, the K/V rows
    read by attention for every stream (positions 0..pos), the new K/V row written."""
    e = 2 if w["bf16"] else 4
    L = w["layers"]
    kvd = w["kv_heads"] // shards * w["head_dim"]
    lb = layer_bytes(w, batch, shards)
    per_layer = (lb["attn_qkv_rope"] + lb["attn_wo_residual"] + lb["ffn_gate_up_swiglu"] +
                 lb["ffn_down_residual"])
    kv = L * batch * 2 * kvd * e * (mean_pos + 1)
    return L * per_layer + lb["final_norm_classifier"] + kv


# ----------------------------------------------------------------------------- CPU
def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_port_model(w, seq):
    """The oracle port of the reference's kernels (oracle/oracle.c, the serial per-row order
    of src/kernels.rs) holding the workload's whole model: every layer and the full
    classifier, its seeded weights drawn on the host by the generator the GPU uses. Returns
    (model, threads)."""
    from oracle import oracle as orc

    threads = host_threads()
    orc.set_threads(threads)
    t0 = time.perf_counter()
    m = orc.Model(w["dim"], w["layers"], w["heads"], w["kv_heads"], w["head_dim"], w["hidden"],
                  w["vocab"], seq, theta=w["theta"], bf16=w["bf16"], seed=w["seed"])
    print(f"cpu port: {w['title']} built in {time.perf_counter() - t0:.1f} s on {threads} "
          "threads", file=sys.stderr, flush=True)
    return m, threads


def cpu_token_times(m, positions, token=7):
    """Seconds of one full decode token (embedding, every layer, final norm, classifier) of
    one stream at each position. The cache rows before a position are whatever the state
    holds (zeros unless decoded): the work of a step depends on the position only."""
    out = []
    for pos in positions:
        t0 = time.perf_counter()
        m.step(token, pos)
        out.append(time.perf_counter() - t0)
    return out


def cpu_streams_sampled(w, batch):
    """Streams of a batch timed per step by the CPU arms: the port decodes streams one after
    another at the same cost each, so a step of B streams is B x one stream's token. Large
    models time one stream per step; small ones up to 8."""
    big = w["layers"] * (4 * w["dim"] ** 2 + 3 * w["dim"] * w["hidden"]) > 10 ** 9
    return 1 if big else min(batch, 8)


# ----------------------------------------------------------------------------- microbenchmarks
class LaunchTimer:
    """Median device time of a recorded scheme: each timed replay follows a write of a
    buffer larger than L2 (so every launch reads from HBM), CUDA events on the runtime's
    stream around the replay alone."""

    def __init__(self, rt, flush_bytes=512 << 20):
        import torch

        self.rt = rt
        self.torch = torch
        self.ext = torch.cuda.ExternalStream(rt.stream)
        self.flush = torch.empty(flush_bytes // 4, dtype=torch.float32, device="cuda")

    def __call__(self, sch, iters, warmup=3):
        torch = self.torch
        for _ in range(warmup):
            sch.submit()
        pairs = []
        for _ in range(iters):
            with torch.cuda.stream(self.ext):
                self.flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(self.ext)
            sch.submit()
            e1.record(self.ext)
            pairs.append((e0, e1))
        self.rt.synchronize()
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in pairs)


def _micro_line(kind, cases, peak, peak_kind, clocks, cpu, extra=None):
    # the HBM-scale cases (above 64 MB moved) summarise the line; small ones are latency
    big = [c for c in cases if c["bytes"] >= (64 << 20)] or cases
    agg = sum(c["bytes"] for c in big) / sum(c["us"] for c in big) / 1e3
    top = max(cases, key=lambda c: c["bytes"])
    line = {
        "metric": f"per-kernel HBM GB/s vs peak ({kind} microbench)", "value": agg,
        "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32+bf16" if kind == "ops" else "bf16",
        "data": "synthetic", "config": {"workload": MICRO[kind],
                                        "l2": "L2 flushed (512 MB write) before every launch"},
        "roofline": {"kernel": top["op"], "bound": "hbm", "achieved": top["gbs"], "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": top["gbs"] / peak,
                     "bytes_per_launch": top["bytes"], "launch_ms": top["us"] / 1e3,
                     "traffic": None},
        "cases": cases, "clocks": clocks, "gpu_launches": len(cases),
    }
    if cpu:
        line["cpu_baseline"] = cpu
    if extra:
        line.update(extra)
    return line


def run_ops_micro(args):
    import numpy as np
    import torch

    import ammon_b200 as ab
    from ammon_b200 import kernels as K

    torch.cuda.set_device(0)
    rt = ab.create_runtime(0)
    timer = LaunchTimer(rt)
    peak, peak_kind = load_peaks()
    cases = []

    def add(op, dtype, shape, nbytes, sch, iters=20):
        us = timer(sch, iters) * 1e3
        cases.append({"op": op, "dtype": dtype, "shape": shape, "bytes": nbytes,
                      "us": round(us, 3), "gbs": round(nbytes / us / 1e3, 1),
                      "frac": round(nbytes / us / 1e3 / peak, 4)})

    with ClockSampler(0) as clocks:
        for dt, esz in ((ab.F32, 4), (ab.BF16, 2)):
            name = "f32" if dt == ab.F32 else "bf16"
            for dim in (4096, 8192):
                w = ab.Tensor.zeros(rt, (dim,), dt).fill_normal(7, 1, 1.0, 0.01)
                for rows in (1, 64, 4096):
                    x = ab.Tensor.zeros(rt, (rows, dim), dt).fill_normal(7, 2)
                    o = ab.Tensor.zeros(rt, (rows, dim), dt)
                    s = rt.scheme()
                    K.RmsnormKernel.prepare(rt).record(s, "rmsnorm", x, w, o)
                    add("rmsnorm", name, [rows, dim], rows * dim * 2 * esz + dim * esz, s)
                    s.close()
            for rows in (1, 64):
                hb = ab.Tensor.zeros(rt, (rows, 14336), dt).fill_normal(7, 3)
                hb2 = ab.Tensor.zeros(rt, (rows, 14336), dt).fill_normal(7, 4)
                s = rt.scheme()
                K.SwigluKernel.prepare(rt).record(s, "swiglu", hb, hb2)
                add("swiglu", name, [rows, 14336], rows * 14336 * 3 * esz, s)
                s.close()
            table = ab.Tensor.zeros(rt, (128256, 4096), dt).fill_normal(7, 5)
            for n in (1, 64, 4096):
                from oracle import oracle as orc

                ids = orc.uniform_tokens(n, 7, 6, 0, 128256).tolist()
                st = ab.DecodeStep.parcel(rt, n)
                rt.deposit(st, [ab.DecodeStep(int(t), 0) for t in ids])
                x = ab.Tensor.zeros(rt, (n, 4096), dt)
                s = rt.scheme()
                ab.Embedding(rt).record(s, table, st, x)
                add("embed", name, [n, 4096], n * 4096 * 2 * esz, s)
                s.close()
                if n == 4096:
                    got = x.read_f32() if dt == ab.BF16 else x.read()
                    row = table.narrow(0, ids[-1], 1)
                    want = row.read_f32() if dt == ab.BF16 else row.read()
                    assert np.array_equal(got[-1], want.ravel()), "embed spot check"
            table.free()
        # RoPE: 8192 rows (one per position 0..8191) of q [32, 128] and the shared k cache
        q = ab.Tensor.zeros(rt, (8192, 32, 128)).fill_normal(7, 7)
        k = ab.Tensor.zeros(rt, (8192, 8, 128)).fill_normal(7, 8)
        st = ab.DecodeStep.parcel(rt, 8192)
        rt.deposit(st, [ab.DecodeStep(0, p) for p in range(8192)])
        s = rt.scheme()
        K.RopeKernel.prepare(rt).record(s, "rope", q, k, st, 500000.0)
        add("rope", "f32", [8192, 32, 128], 8192 * (4096 + 1024) * 4 * 2, s)
        s.close()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as orc

        rows, dim = 64, 4096
        xh = orc.normal(rows * dim, 7, 2, 0.0, 1.0).reshape(rows, dim)
        wh = orc.normal(dim, 7, 1, 1.0, 0.01)
        t0 = time.perf_counter()
        reps = 50
        for _ in range(reps):
            for r in range(rows):
                orc.rmsnorm(xh[r], wh)
        dt_s = (time.perf_counter() - t0) / reps
        cpu = {"value": (rows * dim * 8 + dim * 4) / dt_s / 1e9, "unit": "GB/s", "cores": 1,
               "kind": "port", "sample": "oracle rmsnorm, 64 rows x 4096 f32, 50 repetitions"}
    line = _micro_line("ops", cases, peak, peak_kind, clocks.summary(), cpu)
    rt.close()
    return line


def run_attention_micro(args):
    import numpy as np
    import torch

    import ammon_b200 as ab
    from ammon_b200 import kernels as K

    torch.cuda.set_device(0)
    rt = ab.create_runtime(0)
    timer = LaunchTimer(rt)
    peak, peak_kind = load_peaks()
    H, KV, hd = 32, 8, 128
    ctxs = [int(c) for c in args.contexts.split(",")]
    batches = [int(b) for b in args.batches.split(",")]
    rows_max = max(batches) * max(ctxs) * KV
    # one K and one V buffer of [rows, 128] bf16 rows serve every case as [B, ctx, 8, 128]
    kbuf = ab.Tensor.zeros(rt, (rows_max, hd), ab.BF16).fill_normal(2, 2)
    vbuf = ab.Tensor.zeros(rt, (rows_max, hd), ab.BF16).fill_normal(2, 3)
    cases = []
    worst = 0.0
    with ClockSampler(0) as clocks:
        for ctx in ctxs:
            for B in batches:
                kc = kbuf.narrow(0, 0, B * ctx * KV).reshape((B, ctx, KV, hd))
                vc = vbuf.narrow(0, 0, B * ctx * KV).reshape((B, ctx, KV, hd))
                q = ab.Tensor.zeros(rt, (B, H, hd)).fill_normal(2, 1)
                out = ab.Tensor.zeros(rt, (B, H * hd))
                st = ab.DecodeStep.parcel(rt, B)
                rt.deposit(st, [ab.DecodeStep(0, ctx - 1)] * B)
                s = rt.scheme()
                K.AttentionDecodeKernel.prepare(rt).record(s, "attn_decode", q, kc, vc, out, st)
                nbytes = B * KV * ctx * hd * 2 * 2 + B * H * hd * 4 * 2
                iters = 5 if nbytes > (8 << 30) else 20
                us = timer(s, iters) * 1e3
                # spot check: the last row's first kv group against float64
                b = B - 1
                kr = kbuf.narrow(0, b * ctx * KV, ctx * KV).read_f32().reshape(ctx, KV, hd)
                vr = vbuf.narrow(0, b * ctx * KV, ctx * KV).read_f32().reshape(ctx, KV, hd)
                qh = q.read()[b]
                got = out.read()[b].reshape(H, hd)
                g = H // KV
                for h in range(g):
                    sc = kr[:, 0].astype(np.float64) @ qh[h].astype(np.float64) / np.sqrt(hd)
                    p = np.exp(sc - sc.max())
                    want = (p / p.sum()) @ vr[:, 0].astype(np.float64)
                    worst = max(worst, float(np.abs(got[h] - want).max() /
                                             max(np.abs(want).max(), 1e-30)))
                cases.append({"op": "attn_decode", "dtype": "bf16", "shape": [B, ctx],
                              "bytes": nbytes, "us": round(us, 3),
                              "gbs": round(nbytes / us / 1e3, 1),
                              "frac": round(nbytes / us / 1e3 / peak, 4)})
                s.close()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as orc

        ctx = 4096
        qh = orc.normal(H * hd, 2, 1, 0.0, 1.0).reshape(H, hd)
        kh = orc.round_bf16(orc.normal(ctx * KV * hd, 2, 2, 0.0, 1.0)).reshape(ctx, KV, hd)
        vh = orc.round_bf16(orc.normal(ctx * KV * hd, 2, 3, 0.0, 1.0)).reshape(ctx, KV, hd)
        t0 = time.perf_counter()
        reps = 5
        for _ in range(reps):
            orc.attention(qh, kh, vh, ctx, ctx - 1)
        dt_s = (time.perf_counter() - t0) / reps
        cpu = {"value": KV * ctx * hd * 2 * 2 / dt_s / 1e9, "unit": "GB/s", "cores": 1,
               "kind": "port", "sample": "oracle serial attention (the reference's "
                                         "attention kernel), batch 1 x ctx 4096, bf16-rounded K/V "
                                         "counted at 2 bytes per element"}
    line = _micro_line("attention", cases, peak, peak_kind, clocks.summary(), cpu,
                       {"parity": {"max_rel_err_vs_float64": worst, "tolerance": 1e-4}})
    kbuf.free()
    vbuf.free()
    rt.close()
    return line


def prefill_flops(w, P):
    """Algorithmic FLOPs of prefilling P positions from 0: every projection once per
    position (2 x weights), attention over positions 0..p for each p (QK and PV: 4 x heads x
    head_dim per position attended), and the classifier for the last position only."""
    d, F, V = w["dim"], w["hidden"], w["vocab"]
    qd, kvd = w["heads"] * w["head_dim"], w["kv_heads"] * w["head_dim"]
    per_layer = d * (qd + 2 * kvd) + qd * d + 3 * d * F
    attn = 4 * qd * P * (P + 1) // 2
    return w["layers"] * (2 * P * per_layer + attn) + 2 * V * d


def run_prefill_micro(args):
    import numpy as np
    import torch

    import ammon_b200 as ab

    w = dict(WORKLOADS["llama3-8b-bf16"])
    if args.layers:  # profiling aid, as for the decode workloads
        w["layers"] = args.layers
    if args.seq:
        w["seq"] = args.seq
    P = args.prompt_len
    torch.cuda.set_device(0)
    rt = ab.create_runtime(0)
    cfg = ab.LlamaConfig(w["dim"], w["layers"], w["heads"], w["kv_heads"], w["head_dim"],
                         w["hidden"], w["vocab"], w["seq"], batch=1, rope_theta=w["theta"],
                         dtype=ab.BF16)
    g = ab.LlamaModel(rt, cfg)
    g.init_synthetic(w["seed"], 0.02)
    prompt = prompt_tokens(w["seed"], 0, P, 0, w["vocab"])
    ext = torch.cuda.ExternalStream(rt.stream)
    for _ in range(args.warmup):
        g.prefill(prompt)
    dev_ms, e2e_s = [], []
    with ClockSampler(0) as clocks:
        for _ in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(ext)
            t0 = time.perf_counter()
            logits, am = g.prefill(prompt)
            t1 = time.perf_counter()
            e1.record(ext)
            torch.cuda.synchronize()
            dev_ms.append(e0.elapsed_time(e1))
            e2e_s.append(t1 - t0)
    ms = statistics.median(dev_ms)
    launches = g.prefill_launches()
    passes = (P + 255) // 256
    # the dominant kernel live: the gate/up projection of the timed prefill's last pass, each
    # node of that pass replayed alone between CUDA events
    last_rows = P - (passes - 1) * 256
    sch = g.prefill_scheme(last_rows)
    node_ms = dict()
    for label, t in zip(sch.node_labels(), sch.time_nodes(3)):
        node_ms.setdefault(label, []).append(t)
    gu_ms = statistics.mean(node_ms["ffn_gate_up_swiglu"])
    gu_flops = 2 * (2 * w["hidden"]) * w["dim"] * last_rows
    if args.no_parity:
        print(json.dumps({"workload": "prefill", "tokens_per_s": P / ms * 1e3,
                          "launches": launches}), flush=True)
        g.close()
        rt.close()
        return None
    # the reference's way on the same kernels: one decode step per prompt token
    loop_n = 32
    rt.synchronize()
    t0 = time.perf_counter()
    for pos in range(loop_n):
        g.step_batch([prompt[pos]], [pos], logits=False)
    loop_tps = loop_n / (time.perf_counter() - t0)
    # parity on a 256-token prompt: prefill against that token loop (bf16 rounding points
    # differ between the GEMM and GEMV paths: the bf16 bar applies)
    n_chk = 256
    want = None
    for pos in range(n_chk):
        want, _ = g.step_batch([prompt[pos]], [pos], logits=True)
    want = want[0].copy()
    got, _ = g.prefill(prompt[:n_chk])
    err = float(np.abs(got - want).max() / np.abs(want).max())
    l2err = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    flops = prefill_flops(w, P)
    peak = 1341.5
    peak_kind = "fallback"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops_sustained"])
            peak_kind = "measured (sustained)"
    except Exception:
        pass
    achieved = flops / (ms / 1e3) / 1e12
    burst, burst_kind = 1590.0, "fallback"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            burst = float(json.load(f)["bf16_tflops"])
            burst_kind = "measured (burst: the node is timed alone)"
    except Exception:
        pass
    gu_tf = gu_flops / (gu_ms / 1e3) / 1e12
    line = {
        "metric": "prefill prompt tokens/s (one stream, batched passes)", "value": P / ms * 1e3,
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": MICRO["prefill"] + (f" ({w['layers']} layers: profiling case)"
                                                   if args.layers else ""),
                   "prompt": P, "rows_per_pass": 256,
                   "passes": passes, "l2": "weights (15 GB) exceed L2 every pass"},
        "roofline": {"bound": "tensor", "kernel": "ffn_gate_up_swiglu", "achieved": gu_tf,
                     "peak": burst, "peak_kind": burst_kind, "unit": "TFLOP/s",
                     "frac": gu_tf / burst, "flops_per_launch": gu_flops, "launch_ms": gu_ms,
                     "rows": last_rows,
                     "traffic": profile_traffic("gemm_tc_prefill", "llama3-8b-bf16")},
        "prefill_roofline": {"achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                             "unit": "TFLOP/s", "frac": achieved / peak,
                             "flops_per_prefill": flops},
        "kernels_last_pass_ms": {k: round(sum(v), 4) for k, v in node_ms.items()},
        "e2e": {"value": P / statistics.median(e2e_s), "unit": "tokens/s",
                "h2d_bytes_per_step": P * 8, "d2h_bytes_per_step": w["vocab"] * 4 + 4},
        "token_loop": {"value": loop_tps, "unit": "tokens/s",
                       "what": "the same model fed one DecodeStep per prompt token "
                               "(src/generate.rs:60-66), logits not read back"},
        "parity": {"max_rel_err_vs_token_loop": err, "rel_l2_err_vs_token_loop": l2err,
                   "greedy_id_equal": bool(int(np.argmax(got)) == int(np.argmax(want))),
                   "tolerance": 4e-2, "prompt": n_chk,
                   "note": "two bf16 paths (GEMM passes vs GEMV steps), each held to 2e-2 "
                           "against the oracle by the tests: their difference is bounded by "
                           "twice that"},
        "clocks": clocks.summary(),
        "gpu_launches": launches * args.steps,
    }
    g.close()
    rt.close()
    if not args.no_cpu_baseline:
        pos = [0, P // 4, P // 2, 3 * P // 4, P - 1]
        m, threads = cpu_port_model(w, P)
        per_token = cpu_token_times(m, pos)
        m.close()
        line["cpu_baseline"] = {
            "value": 1.0 / statistics.mean(per_token), "unit": "tokens/s", "cores": threads,
            "kind": "port", "sample": "the reference feeds a prompt one decode step per token: "
                                      "full tokens (every layer, the full classifier) of the "
                                      f"oracle port at positions {pos}"}
    return line


def decode_config(w, B, first, last, world, mode):
    """The `config` object of a decode line; the GPU arm and the reference arm build it with
    this one function, so the two lines describe the same workload."""
    return {"workload": w["title"], "batch": B, "seq_len": w["seq"],
            "positions": f"{first}..{last}",
            "parallelism": mode if world > 1 else "single",
            "l2": "inputs larger than L2 (weights stream every step)"}


def timed_positions(w, args):
    """Positions the timed steps decode: the prompt's forced ids fill positions
    0 .. prompt - 2, the warm-up steps start at prompt - 1, the timed ones follow."""
    first = w["prompt"] - 1 + args.warmup
    return first, first + args.steps - 1


def parallel_mode(w, args, world):
    mode = args.parallel
    if mode == "auto":
        mode = "tp" if w["bf16"] else "replicas"
    if world == 1:
        return "single"
    if mode == "tp":
        return f"tp{world}"
    return f"dp{world}" if w.get("split_streams") else f"replicas{world}"


def stream_assignment(w, batch, parallel, world, rank):
    """(streams this rank decodes, global id of its first stream, whether the workload's
    streams are split over the ranks). The 110M workload's 256 independent streams split
    data-parallel into contiguous blocks of 256 / world per rank with no collective; tensor
    parallel ranks all decode the same streams (0 ..); replicas each decode their own batch
    (rank * batch ..). An explicit batch is per rank and never split."""
    mode = parallel
    if mode == "auto":
        mode = "tp" if w["bf16"] else "replicas"
    tp = world > 1 and mode == "tp"
    if batch:
        return batch, 0 if tp else rank * batch, False
    batch = w["batch"]
    if w.get("split_streams") and world > 1 and not tp:
        if batch % world:
            raise SystemExit(f"{batch} streams do not split over {world} ranks")
        per = batch // world
        return per, rank * per, True
    return batch, 0 if tp else rank * batch, False


def cpu_decode_baseline(w, B, positions):
    """cpu_baseline of a decode sub-record: full tokens of the oracle port (every layer, the
    full classifier) at `positions`, the streams of a batch decoded one after another, so
    the port's tokens/s is one over its mean token time whatever the batch."""
    m, threads = cpu_port_model(w, max(positions) + 1)
    S = cpu_streams_sampled(w, B)
    times = []
    for pos in positions:
        times += cpu_token_times(m, [pos] * S)
    m.close()
    return {"value": 1.0 / statistics.mean(times), "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": f"full tokens (every layer, the full classifier) of the oracle port at "
                      f"positions {positions}, {S} stream(s) each; the port decodes the "
                      f"{B} streams of a step one after another"}


# The other BASELINE.json configurations ride in the default line's `configs` object, each
# with its own metric and unit: the tiny fp32 decode (128 tokens) and the 110M fp32 decode
# of 256 streams (256 tokens; split data-parallel over the ranks at N > 1, no collective),
# and at N = 1 the split-attention, per-op and prefill microbenchmarks.
SUB_DECODES = (("tiny-llama-f32", 128), ("llama-110m-f32", 256))
SUB_KEEP = ("value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling", "dtype",
            "config", "step_bytes", "step_gbs", "step_frac", "roofline", "kernels", "e2e",
            "gpu_launches", "clocks")


def configs_wanted(args, w):
    return batch64_wanted(args, w) and not args.no_configs


def run_sub_decode(args, name, steps, env):
    w = dict(WORKLOADS[name])
    rank, world = env["rank"], env["world"]
    per, sbase, split = stream_assignment(w, 0, "replicas", world, rank)
    sub_args = argparse.Namespace(**vars(args))
    sub_args.steps, sub_args.warmup, sub_args.e2e_steps = steps, 8, 0
    env2 = dict(env, tp=False, split_streams=split, sbase=sbase, batch=per, comm=None)
    line = run_decode(sub_args, w, per, env2, name=name)
    sub = {"metric": "decode tokens/sec", **{k: line[k] for k in SUB_KEEP}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        first, last = timed_positions(w, sub_args)
        sub["cpu_baseline"] = cpu_decode_baseline(w, per, [first, (first + last) // 2, last])
    return sub


def run_other_configs(args, env):
    """The `configs` object of the default line. A sub-record that fails carries its error
    instead of failing the headline line."""
    out = {}
    world = env["world"]
    for name, steps in SUB_DECODES:
        if world > 1 and not WORKLOADS[name].get("split_streams"):
            continue  # one stream: nothing to partition over the ranks
        try:
            out[name] = run_sub_decode(args, name, steps, env)
        except Exception as e:  # noqa: BLE001 - reported in the line
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if world > 1:
        return out
    for key, fn, steps in (("split-attention", run_attention_micro, 0),
                           ("ops", run_ops_micro, 0), ("prefill", run_prefill_micro, 5)):
        a = argparse.Namespace(**vars(args))
        a.steps, a.warmup, a.layers, a.seq, a.no_parity = steps, 3, 0, 0, False
        try:
            sub = fn(a)
            for k in ("n_gpus", "higher_is_better", "scaling", "vs_baseline", "data"):
                sub.pop(k, None)
            out[key] = sub
        except Exception as e:  # noqa: BLE001
            out[key] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return out


def batch64_wanted(args, w):
    """The default 8B line carries batch 64 as a sub-record (BASELINE metric: batch 1 and
    64); other workloads and explicit --batch runs report one batch."""
    return (args.workload == "llama3-8b-bf16" and not args.batch_given and not args.layers
            and not args.no_batch64)


# Tokens the reference arm times per batch: the work of a token depends on its position only,
# so an evenly spaced sample of the timed positions stands for all of them and the arm ends in
# well under a minute (an 8B token takes ~0.4 s on 16 host threads) while the GPUs wait.
REF_SAMPLES = 12


def reference_positions(first, last, steps):
    """Evenly spaced sample (at most REF_SAMPLES, both ends included) of first..last."""
    n = max(1, min(steps, REF_SAMPLES))
    return sorted({first + (last - first) * i // max(n - 1, 1) for i in range(n)})


def run_reference(args, w, rank, world):
    """The reference arm: the oracle port of the reference's per-token kernels on the host
    cores, full tokens (every layer and the full classifier) at a sample of the positions the
    GPU arm times, streams decoded one after another."""
    if rank != 0:
        return
    first, last = timed_positions(w, args)
    positions = reference_positions(first, last, args.steps)
    m, threads = cpu_port_model(w, last + 1)
    mode = parallel_mode(w, args, world)
    cpu_token_times(m, [first - 1])  # untimed warm-up token

    def arm(B):
        S = cpu_streams_sampled(w, B)
        steps = []
        for pos in positions:
            steps.append(sum(cpu_token_times(m, [pos] * S)) * B / S)
        step_s = statistics.mean(steps)
        value = B / step_s
        sample = (f"full tokens of the oracle port at {len(positions)} positions evenly "
                  f"spaced over {first}..{last}, "
                  + ("one stream per step" if S == 1 else f"{S} streams per step")
                  + (f", scaled to the batch's {B} streams (decoded one after another)"
                     if S < B else ""))
        return {"value": value, "ms_per_step": step_s * 1e3,
                "config": decode_config(w, B, first, last, world, mode),
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                                 "kind": "port", "sample": sample},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}

    top = arm(args.batch)
    line = {"impl": "reference", "metric": METRIC, "value": top["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": top["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if w["bf16"] else "f32", "data": "synthetic",
            "config": top["config"], "cpu_baseline": top["cpu_baseline"], "e2e": top["e2e"]}
    if batch64_wanted(args, w):
        sub = arm(64)
        line["batch64"] = {"value": sub["value"], "unit": "tokens/s",
                           "ms_per_step": sub["ms_per_step"], "config": sub["config"],
                           "cpu_baseline": sub["cpu_baseline"], "e2e": sub["e2e"]}
    m.close()
    print(json.dumps(line), flush=True)


def run_decode(args, w, B, env, name=None):
    """One decode line of the GPU arm at batch B (per rank): the device greedy loop timed
    between CUDA events (max over ranks), e2e through step(), per-kernel times and the
    roofline of the dominant kernel. `name`: the workload's key (default: --workload)."""
    import numpy as np
    import torch

    import ammon_b200 as ab

    rank, world, local, dist = env["rank"], env["world"], env["local"], env["dist"]
    tp, split_streams = env["tp"], env["split_streams"]
    rt = env["rt"]
    cfg = ab.LlamaConfig(w["dim"], w["layers"], w["heads"], w["kv_heads"], w["head_dim"],
                         w["hidden"], w["vocab"], w["seq"], batch=B, rope_theta=w["theta"],
                         dtype=ab.BF16 if w["bf16"] else ab.F32)
    with StdoutToStderr():
        model = ab.LlamaModel(rt, cfg, env["comm"])
        model.init_synthetic(w["seed"], 0.02)
    P = w["prompt"]
    # tensor parallel ranks decode the same streams; replicas and data-parallel ranks each
    # decode their own (batch 64 of the default line: streams 0..63 on every arm)
    sbase = env["sbase"] if B == env["batch"] else (0 if tp else rank * B)
    prompts = [prompt_tokens(w["seed"], 1000 + sbase + b, P, 3, w["vocab"]) for b in range(B)]
    # prompt: forced tokens at positions 0..P-2
    for pos in range(P - 1):
        model.step_batch([prompts[b][pos] for b in range(B)], [pos] * B, logits=False)
    start_tok = [prompts[b][P - 1] for b in range(B)]
    pos0 = P - 1
    e2e_steps = args.e2e_steps or min(args.steps, 64)
    need = pos0 + args.warmup + args.steps + e2e_steps + 1
    if need > w["seq"]:
        raise SystemExit(f"steps exceed the workload's max context ({need} > {w['seq']})")

    # warm-up (device greedy loop)
    toks = model.decode_device(start_tok, [pos0] * B, args.warmup)
    start_tok = toks[-1].tolist()
    pos0 += args.warmup

    ext = torch.cuda.ExternalStream(rt.stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    rt.synchronize()
    with ClockSampler(local) as clocks:
        ev0.record(ext)
        toks = model.decode_device(start_tok, [pos0] * B, args.steps)
        ev1.record(ext)
        ev1.synchronize()
    rt.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t = ev0.elapsed_time(ev1) / 1e3
    if dist:
        tt = torch.tensor([t], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    start_tok = toks[-1].tolist()
    first, last = pos0, pos0 + args.steps - 1
    pos0 += args.steps
    streams = B if tp else world * B
    value = streams * args.steps / t
    # our kernels per device-loop step: the step graph's kernel nodes (not the NCCL
    # collectives, not the logits gather of step()) plus the sample feedback
    step_labels = model.scheme().node_labels()
    if step_labels == ["decode_step"]:
        nodes_loop = 1  # the persistent step: its last CTA also writes the next DecodeStep
    else:
        nodes_loop = len([l for l in step_labels
                          if "allreduce" not in l and "allgather" not in l]) + (2 if tp else 1)

    # e2e through the reference-facing step(): DecodeSteps up, [B, vocab] logits down
    tok = start_tok
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        # logits come back to the host every step; the next token is the library's greedy
        # pick of them (sample_argmax's first-maximum rule, computed on the device)
        logits, am = model.step_batch(tok, [pos0 + i] * B, logits=True, argmax=True)
        tok = [int(t) for t in am]
    t_e2e = time.perf_counter() - t0
    if dist:
        tt = torch.tensor([t_e2e], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_e2e = float(tt.item())
    e2e = streams * e2e_steps / t_e2e

    # per-kernel times (each node launched alone between CUDA events on the decode stream)
    sch = model.scheme()
    labels = sch.node_labels()
    times = sch.time_nodes(iters=3)
    per_label = {}
    for l, ms in zip(labels, times):
        c = per_label.setdefault(l, [0, 0.0])
        c[0] += 1
        c[1] += ms
    total_ms = sum(times)
    shards = world if tp else 1
    # the timed nodes replay the last deposited steps: the e2e loop's final position
    lb = layer_bytes(w, B, shards, attn_pos=pos0 + e2e_steps - 1)
    # the persistent single-launch step moves one whole step's algorithmic bytes
    lb["decode_step"] = step_bytes(w, B, pos0 + e2e_steps - 1, shards)
    dom = max(per_label, key=lambda l: per_label[l][1])
    n_dom, ms_dom = per_label[dom]
    t_launch = ms_dom / n_dom / 1e3
    peak, peak_kind = load_peaks()
    achieved = lb[dom] / t_launch / 1e9 if dom in lb else None
    mean_pos = (first + last) / 2
    sb = step_bytes(w, B, mean_pos, shards)
    suffix = "" if B == 1 else f"_b{B}"
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong" if tp or split_streams else "weak",
        "vs_baseline": None,
        "dtype": "bf16" if w["bf16"] else "f32", "data": "synthetic",
        "config": decode_config(w, B, first, last, world, parallel_mode(w, args, world)),
        "step_bytes": sb, "step_gbs": sb / (t / args.steps) / 1e9,
        "step_frac": sb / (t / args.steps) / 1e9 / peak,
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": achieved / peak if achieved else None,
                     "bytes_per_launch": lb.get(dom), "launch_ms": t_launch * 1e3,
                     "traffic": profile_traffic(dom, (name or args.workload) + suffix,
                                                lb.get(dom))},
        "kernels": {l: {"launches": c[0], "ms": round(c[1], 4),
                        "share": round(c[1] / total_ms, 4),
                        "gbs": round(lb[l] * c[0] / (c[1] / 1e3) / 1e9, 1) if l in lb else None}
                    for l, c in sorted(per_label.items(), key=lambda kv: -kv[1][1])},
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 8 * B,
                "d2h_bytes_per_step": 4 * B * w["vocab"] + 4 * B},
        "gpu_launches": nodes_loop * args.steps,
        "clocks": clocks.summary(),
    }
    model.close()
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--workload", default="llama3-8b-bf16", choices=sorted(WORKLOADS) +
                    sorted(MICRO))
    ap.add_argument("--contexts", default="4096,32768,131072", help="attention microbench")
    ap.add_argument("--batches", default="1,8,64", help="attention microbench")
    ap.add_argument("--prompt-len", type=int, default=2048, help="prefill microbench")
    ap.add_argument("--no-parity", action="store_true",
                    help="profiling aid: prefill microbench without the token-loop comparison "
                         "(prints a short line, not a bench line)")
    ap.add_argument("--batch", type=int, default=0,
                    help="streams per rank (default: the workload's; the 110M workload's 256 "
                         "streams are split over the ranks)")
    ap.add_argument("--no-batch64", action="store_true",
                    help="the default 8B line without its batch-64 sub-record")
    ap.add_argument("--no-configs", action="store_true",
                    help="the default 8B line without its `configs` object (the other "
                         "workloads and the kernel microbenchmarks)")
    ap.add_argument("--impl", default="ammon", choices=["ammon", "reference"])
    ap.add_argument("--parallel", default="auto", choices=["auto", "tp", "replicas"],
                    help="N > 1: tensor parallel (8B default) or independent replicas")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=0, help="default: min(steps, 64)")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling aid: fewer layers of the same shapes (not a bench line)")
    ap.add_argument("--prompt", type=int, default=0,
                    help="profiling aid: shorter prompt (fewer launches before the timed loop)")
    ap.add_argument("--seq", type=int, default=0,
                    help="profiling aid: smaller KV cache (max context)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.batch_given = args.batch > 0
    if args.workload in MICRO:
        if int(os.environ.get("RANK", "0")) != 0:
            return  # single-GPU kernel microbenchmarks: other ranks have nothing to do
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "kernel microbenchmarks "
                              "report the oracle's CPU rate as cpu_baseline in the main arm"}))
            return
        line = {"ops": run_ops_micro, "attention": run_attention_micro,
                "prefill": run_prefill_micro}[args.workload](args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    w = dict(WORKLOADS[args.workload])
    if args.layers:
        w["layers"] = args.layers
        w["title"] += f" ({args.layers} layers: profiling case)"
    if args.prompt:
        w["prompt"] = args.prompt
    if args.seq:
        w["seq"] = args.seq

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    args.batch, sbase, split_streams = stream_assignment(w, args.batch, args.parallel, world,
                                                         rank)
    if args.impl == "reference":
        run_reference(args, w, rank, world)
        return

    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        with StdoutToStderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)

    import ammon_b200 as ab

    rt = ab.create_runtime(local)
    mode = args.parallel
    if mode == "auto":
        mode = "tp" if w["bf16"] else "replicas"
    tp = world > 1 and mode == "tp"
    comm = None
    if tp:
        # rank 0 makes the NCCL id of the model's communicator; torch.distributed carries it
        with StdoutToStderr():
            uid = torch.zeros(ab._abi.COMM_ID_BYTES, dtype=torch.uint8, device="cuda")
            if rank == 0:
                uid.copy_(torch.frombuffer(bytearray(ab.Comm.unique_id()), dtype=torch.uint8))
            dist.broadcast(uid, 0)
            comm = ab.Comm(rt, bytes(uid.cpu().numpy().tobytes()), rank, world)
    env = dict(rank=rank, world=world, local=local, dist=dist, tp=tp, sbase=sbase,
               batch=args.batch,
               split_streams=split_streams, rt=rt, comm=comm)
    line = run_decode(args, w, args.batch, env)
    if batch64_wanted(args, w):
        # a sub-record that fails carries its error instead of failing the headline line
        try:
            sub = run_decode(args, w, 64, env)
            line["batch64"] = {k: sub[k] for k in (
                "value", "unit", "ms_per_step", "config", "step_bytes", "step_gbs",
                "step_frac", "roofline", "kernels", "e2e", "gpu_launches", "clocks")}
        except Exception as e:  # noqa: BLE001 - reported in the line
            line["batch64"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if configs_wanted(args, w):
        line["configs"] = run_other_configs(args, env)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        first, last = timed_positions(w, args)
        cpos = [first, (first + last) // 2, last]
        m, threads = cpu_port_model(w, last + 1)
        per_token = cpu_token_times(m, cpos)
        m.close()
        v = 1.0 / statistics.mean(per_token)
        base = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": "full tokens (every layer, the full classifier) of the oracle port "
                          f"at positions {cpos}, one stream"}
        line["cpu_baseline"] = base
        if "value" in line.get("batch64", {}):
            line["batch64"]["cpu_baseline"] = dict(
                base, sample=base["sample"] + "; the port decodes the 64 streams one after "
                                              "another, 64 such tokens per step")
    if rank == 0:
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    rt.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
