#!/usr/bin/env python
"""Benchmark of the SpAtten progressive sparse-attention hot path on B200.

Workload (one "step"): the standalone progressive-quantised attention op on
batch 8 x 12 heads x seq 4096 x head_dim 64, Q/K/V fp16 drawn i.i.d. N(0,1)
from seed 1 (synthetic, Q then K then V): Q quantised to int8, K to 4-bit
MSB/LSB planes, exact int8 scores, LSB refetch for rows whose max softmax
probability is below 0.1, V pruned at p < 1e-3, P.V, token importance [B, S]
and per-head |O| sums. Inputs (151 MB) exceed the 126 MB L2, so no flush is
needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU; each rank processes its own
batch of 8 (weak scaling, no collective on the data path). Rank 0 prints one
JSON line. ``--impl reference`` times the CPU restatement of the op (the
reference has no GPU path for it) on rank 0 over a bounded sample.
"""
import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, H, S, D = 8, 12, 4096, 64
SEED = 1
REFETCH_THR = 0.1
V_THR = 1e-3
SM_SCALE = 1.0 / math.sqrt(D)
METRIC = "sparse_attn_tokens_per_s"
UNIT = "tokens/s"
LAUNCHES_PER_STEP = 5  # quant Q, quant K planes, attention, token reduce, head reduce


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seq", type=int, default=S)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def config(seq):
    return {"workload": f"progressive_attention B{B} H{H} S{seq} D{D} fp16 seed{SEED}",
            "batch": B, "heads": H, "seq_len": seq, "head_dim": D,
            "refetch_threshold": REFETCH_THR, "v_prune_threshold": V_THR,
            "l2": "inputs 151 MB > 126 MB L2 (no flush)"}


def make_inputs(seed, seq, torch):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, seq, D, generator=g).half() for _ in range(3)]


def algorithmic_bytes(seq, refetch_frac):
    """Bytes one attention launch must move: int8 Q + scale, MSB plane + K
    scale, V and O (fp16), plus the LSB plane for the refetched share."""
    rows = B * H * seq
    return rows * (D + 4 + D // 2 + 4 + 2 * D + 2 * D) + refetch_frac * rows * (D // 2) + B * seq * 4


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during a region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def visible_gpu_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


def cpu_sample(torch, q, k, v, heads):
    """Time the CPU restatement on one batch element and `heads` heads."""
    from oracle.prog_attn_torch import run_sample
    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.perf_counter()
    run_sample(q[0, :heads].float(), k[0, :heads].float(), v[0, :heads], SM_SCALE, REFETCH_THR, V_THR)
    return time.perf_counter() - t0


def reference_arm(args, torch, rank, world):
    if rank != 0:
        return
    seq = args.seq
    q, k, v = make_inputs(SEED, seq, torch)
    from oracle.prog_attn_torch import run_sample
    nthreads = os.cpu_count() or 1
    torch.set_num_threads(nthreads)
    heads = H

    def step(i):
        b = i % B
        run_sample(q[b].float(), k[b].float(), v[b], SM_SCALE, REFETCH_THR, V_THR)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    dt = (time.perf_counter() - t0) / args.steps
    tokens = seq * heads / H
    val = tokens / dt
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config(seq),
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": nthreads, "kind": "port",
                             "sample": f"one batch element (all {H} heads, S={seq}) per step, "
                                       "torch fp32 restatement of the op on the host cores"},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def ours_arm(args, torch, rank, world, local_rank):
    import torch.distributed as dist
    import spatten_b200 as sp
    from spatten_b200._native import MODE_QUANT
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    seq = args.seq
    qh, kh, vh = make_inputs(SEED + rank, seq, torch)
    qh, kh, vh = (t.pin_memory() for t in (qh, kh, vh))
    q, k, v = (t.to(dev) for t in (qh, kh, vh))
    st = torch.cuda.current_stream(dev)

    def step(q, k, v):
        q8, qs = sp.quant_q_int8(q)
        kp = sp.quant_k_planes(k)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        r = sp.prog_attn(q8, kp.msb, v, k1=kp.lsb, mode=MODE_QUANT, q_scale=qs, k_scale=kp.scale,
                         sm_scale=SM_SCALE, refetch_thr=REFETCH_THR, v_thr=V_THR, want_tok=True,
                         want_head=True)
        e1.record(st)
        return r, (e0, e1)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(max(3, args.warmup)):
        step(q, k, v)
    torch.cuda.synchronize(dev)
    # refetched share of rows, for the algorithmic LSB bytes
    q8, qs = sp.quant_q_int8(q)
    kp = sp.quant_k_planes(k)
    r = sp.prog_attn(q8, kp.msb, v, k1=kp.lsb, mode=MODE_QUANT, q_scale=qs, k_scale=kp.scale,
                     sm_scale=SM_SCALE, refetch_thr=REFETCH_THR, v_thr=V_THR, want_refetch=True)
    refetch_frac = float(r.refetch.float().mean())
    del q8, qs, kp, r

    sampler = ClockSampler(visible_gpu_index(local_rank))
    sampler.start()
    time.sleep(0.5)
    barrier()
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    ev = []
    t0.record(st)
    for _ in range(args.steps):
        _, e = step(q, k, v)
        ev.append(e)
    t1.record(st)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / args.steps
    attn_ms = sum(a.elapsed_time(b) for a, b in ev) / len(ev)

    # end to end through the public API: pinned host in, host out
    out_h = torch.empty((B, H, seq, D), dtype=torch.float16).pin_memory()
    tok_h = torch.empty((B, seq), dtype=torch.float32).pin_memory()
    head_h = torch.empty((H,), dtype=torch.float32).pin_memory()

    def e2e_step():
        qd, kd, vd = (t.to(dev, non_blocking=True) for t in (qh, kh, vh))
        res = sp.progressive_attention(qd, kd, vd, refetch_threshold=REFETCH_THR,
                                       v_prune_threshold=V_THR, sm_scale=SM_SCALE,
                                       return_importance=True)
        out_h.copy_(res.out, non_blocking=True)
        tok_h.copy_(res.token_importance, non_blocking=True)
        head_h.copy_(res.head_abs_sum, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(st)
    for _ in range(args.steps):
        e2e_step()
    a1.record(st)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = a0.elapsed_time(a1) / args.steps

    if world > 1:
        t = torch.tensor([ms, attn_ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, attn_ms, e2e_ms = (float(x) for x in t.tolist())
    if rank != 0:
        return
    tokens = B * seq * world
    alg = algorithmic_bytes(seq, refetch_frac)
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, peak_src = 6650.0, "fallback"
    if os.path.exists(peaks_path):
        with open(peaks_path) as f:
            peak = float(json.load(f).get("hbm_gbs", peak))
        peak_src = "measured"
    achieved = alg / (attn_ms * 1e-3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "prog_attn_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    line = {
        "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "s8 scores / f32 softmax / f16 P.V", "data": "synthetic", "config": config(seq),
        "hbm_gbs": achieved, "attn_ms": attn_ms, "refetch_fraction": refetch_frac,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": peak_src, "algorithmic_bytes": alg,
                     "note": "attention launch incl. importance reduce; kernel is exp/ALU bound"},
        "clocks": clocks,
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": 3 * B * H * seq * D * 2,
                "d2h_bytes_per_step": B * H * seq * D * 2 + B * seq * 4 + H * 4},
    }
    if world == 1 and not args.no_cpu_baseline:
        qc, kc, vc = (t.cpu() for t in (qh, kh, vh))
        hs = H
        dt = cpu_sample(torch, qc, kc, vc, hs)
        line["cpu_baseline"] = {"value": seq * hs / H / dt, "unit": UNIT,
                                "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"one batch element, {hs} heads, S={seq}: torch fp32 "
                                          "restatement of the op on all host cores"}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, torch, rank, world)
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        ours_arm(args, torch, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
