#!/usr/bin/env python
"""W8A8 decode tokens/s (TinyLlama-1.1B shape) + GEMV HBM GB/s vs peak.

One step = one decode token through every W8A8 Linear of a TinyLlama-1.1B
shaped decoder (22 layers x [q|k|v, o, gate|up, down] + lm_head, batch 1,
1.04 GB of INT8 weights, inputs larger than L2), replayed as a CUDA graph
holding one persistent leafq decode launch (leafq_decode_plan_run).  With
--gpus N each rank runs its own replica (an independent request stream);
value is the sum over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  --impl reference times the reference's own
CPU kernels (oracle/_ref, compiled from the reference sources) on the host
cores for the same metric and workload.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "W8A8 decode tokens/s (TinyLlama-1.1B shape) + GEMV HBM GB/s vs peak"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="bounded CPU-baseline sample (rank 0, N=1)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--case", choices=sorted(CASES),
                   help="run one small single-kernel case three times and exit (for ncu captures)")
    return p.parse_args()


def _case_weight(rows, cols, bits, group, device):
    import torch

    import leaf_b200 as lq
    from leaf_b200.stack import random_w8_weight

    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    if bits == 8:
        return random_w8_weight(rows, cols, gen, device)
    rng = np.random.default_rng(0)
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = (rng.random((rows, cols // group), dtype=np.float32) * 1e-3 + 1e-4).astype(np.float32)
    return lq.QuantWeight.from_host(packed, scales, rows, cols, 4, group, device=device)


# name: (tokens, rows, cols, weight bits, group, activation bits)
CASES = {
    "gemv": (1, 11264, 2048, 8, 2048, 8),       # gate|up decode GEMV, 23 MB
    "lmhead": (1, 32000, 2048, 8, 2048, 8),     # lm_head decode GEMV, 65.5 MB
    "gemm": (512, 5632, 2048, 8, 2048, 8),      # config 2 prefill GEMM
    "gemm_down": (512, 2048, 5632, 8, 5632, 8),  # config 2 down_proj shape
    "gemm_big": (4096, 5632, 2048, 8, 2048, 8),  # large-M prefill
    "w4": (1, 11008, 4096, 4, 32, 32),          # config 1 INT4 weight-only GEMV
    "decode_small": None,                        # persistent decode kernel, 3-layer stack
}


def run_case(name):
    import torch

    import leaf_b200 as lq

    if name == "decode_small":
        # The persistent decode kernel on a 3-layer TinyLlama-width stack
        # (132 MB of weights: larger than L2, small enough for ncu replays).
        from leaf_b200.stack import LinearStack, StackShape

        torch.cuda.set_device(0)
        stack = LinearStack(StackShape(layers=3))
        for _ in range(3):
            stack.run_persistent()
        torch.cuda.synchronize()
        if lq.load().leafq_device_status() != 0:
            raise RuntimeError("device status not ok")
        print(json.dumps({"case": name, "layers": 3, "step_bytes": stack.shape.step_bytes(1),
                          "status": "ok"}))
        return
    tokens, rows, cols, bits, group, abits = CASES[name]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    w = _case_weight(rows, cols, bits, group, device)
    x = torch.randn(tokens, cols, device=device)
    y = torch.empty(tokens, rows, device=device)
    ws = lq.Workspace(device)
    for _ in range(3):
        lq.linear(x, w, activation_bits=abits, out=y, workspace=ws)
    torch.cuda.synchronize()
    if lq.load().leafq_device_status() != 0:
        raise RuntimeError("device status not ok")
    print(json.dumps({"case": name, "tokens": tokens, "rows": rows, "cols": cols, "bits": bits,
                      "group": group, "activation_bits": abits, "status": "ok"}))


def measured_peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def workload_config(n_gpus):
    return {
        "workload": "tinyllama-1.1b w8a8 decode linear stack: 22 x [qkv 2560x2048, o 2048x2048, "
                    "gate_up 11264x2048, down 2048x5632] + lm_head 32000x2048, batch 1 per GPU",
        "model": "TinyLlama-1.1B shape (random-init INT8 per-row weights)",
        "global_batch": n_gpus,
        "seq_len": 1,
        "parallelism": f"replicas x{n_gpus}",
        "l2": "inputs larger than L2 (1.04 GB of weights streamed per step)",
    }


# ----------------------------------------------------------------- CPU side
def cpu_reference_stack(threads: int, seconds: float, steps: int = 0, warmup: int = 0):
    """Times the reference's own CPU kernels (oracle/_ref) on one decode
    token of the same stack (separate q, k, v, gate, up projections as the
    reference calls them).  Returns (tokens_per_s, kind, sample text,
    per-step seconds list)."""
    import oracle
    from leaf_b200.stack import StackShape

    shape = StackShape()
    kind = "reference" if oracle.ref_available() else "port"
    rng = np.random.default_rng(7)
    h, f, kv = shape.hidden, shape.intermediate, shape.kv_heads * shape.head_dim
    names = [("q", h, h), ("k", kv, h), ("v", kv, h), ("o", h, h), ("gate", f, h), ("up", f, h),
             ("down", h, f)]
    # Two distinct layer copies (2 x 44 MB) cycle through the 22 layers so
    # the weights are not cache-resident; lm_head is its own 65.5 MB.
    layers = []
    for _ in range(2):
        layers.append({n: (rng.integers(-127, 128, (r, c), dtype=np.int8),
                           (rng.random((r, 1), dtype=np.float32) * 1e-3 + 1e-4).astype(np.float32))
                       for n, r, c in names})
    head = (rng.integers(-127, 128, (shape.vocab, h), dtype=np.int8),
            (rng.random((shape.vocab, 1), dtype=np.float32) * 1e-3 + 1e-4).astype(np.float32))
    x0 = rng.standard_normal((1, h)).astype(np.float32)

    def run(w, x, n):
        if kind == "reference":
            return oracle.ref_linear_int(x, w[0], w[1], 8, w[0].shape[1], None, threads=threads, mode=0)
        return oracle.linear_int(x, w[0], w[1], 8, w[0].shape[1], None)

    def token():
        x = x0
        for i in range(shape.layers):
            L = layers[i % 2]
            q = run(L["q"], x, "q")
            run(L["k"], x, "k")
            run(L["v"], x, "v")
            o = run(L["o"], q, "o")
            run(L["gate"], o, "gate")
            up = run(L["up"], o, "up")
            x = run(L["down"], up, "down")
        return run(head, x, "lm_head")

    for _ in range(max(warmup, 1)):
        token()
    times = []
    start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        token()
        times.append(time.perf_counter() - t0)
        if steps and len(times) >= steps:
            break
        if not steps and time.perf_counter() - start >= seconds:
            break
    per = float(np.mean(times))
    sample = (f"{len(times)} decode tokens of the full 22-layer stack + lm_head (2 distinct layer "
              f"weight copies cycled), {threads} threads, reference Workers grain 32")
    return 1.0 / per, kind, sample, times


# ----------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, index: int, path: Path):
        self.path = path
        self.proc = None
        query = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.file = open(path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", f"--query-gpu={query}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.close()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for name, col in (("hw_slowdown", 5), ("hw_thermal_slowdown", 6),
                              ("sw_thermal_slowdown", 7), ("sw_power_cap", 8)):
                if r[col].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ----------------------------------------------------------------- arms
def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = max(1, min(os.cpu_count() or 1, 64))
    try:
        import oracle
        if not oracle.ref_available():
            oracle.build()
    except Exception as exc:  # noqa: BLE001
        print(json.dumps({"impl": "reference", "unavailable": f"CPU reference kernels missing: {exc}"}))
        return
    value, kind, sample, times = cpu_reference_stack(threads, 0.0, steps=args.steps, warmup=args.warmup)
    ms = 1000.0 * float(np.mean(times))
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
        "config": workload_config(1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import leaf_b200 as lq
    from leaf_b200.stack import LinearStack

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    stack = LinearStack(tokens=1, seed=1234 + rank, device=device)
    # Reference point: the same step as one leafq_linear launch per linear
    # (89 launches, programmatic dependent launch), CUDA events, 20 replays.
    stack.capture(pdl=True)
    for _ in range(3):
        stack.graph.replay()
    p_start, p_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p_start.record()
    for _ in range(20):
        stack.graph.replay()
    p_end.record()
    torch.cuda.synchronize(device)
    per_linear_ms = p_start.elapsed_time(p_end) / 20
    # The measured path: the whole step as one persistent launch.
    stack.capture_persistent()
    launches = stack.launches_per_step(persistent=True)
    step_bytes = stack.shape.step_bytes(1)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream(device)
    for _ in range(max(args.warmup, 3)):
        stack.replay()
    torch.cuda.synchronize(device)

    out_dir = REPO / "gpurun_out"
    out_dir.mkdir(exist_ok=True)
    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    smi_id = visible[local_rank] if local_rank < len(visible) else str(device.index)
    sampler = ClockSampler(smi_id, out_dir / f"clocks_rank{rank}.csv")
    time.sleep(0.3)
    # ------------------------------------------------ device-timed value
    barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        stack.graph.replay()
    end.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    ms_total = max_over_ranks(start.elapsed_time(end))
    # ------------------------------------------------ end to end (host buffers)
    x_host = torch.randn(stack.x.shape, dtype=torch.float32).pin_memory()
    logits_host = torch.empty(stack.logits.shape, dtype=torch.float32).pin_memory()
    barrier()
    torch.cuda.synchronize(device)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.steps):
        stack.x.copy_(x_host, non_blocking=True)
        stack.graph.replay()
        logits_host.copy_(stack.logits, non_blocking=True)
    e_end.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms_total = max_over_ranks(e_start.elapsed_time(e_end))
    time.sleep(0.2)
    clocks = sampler.stop()
    status = lq.load().leafq_device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}: {lq.load().leafq_last_error().decode()}")

    ms_step = ms_total / args.steps
    value = world * 1000.0 / ms_step
    e2e_ms_step = e2e_ms_total / args.steps
    peak, peak_kind = measured_peaks()
    achieved = step_bytes / (ms_step * 1e-3) / 1e9
    traffic = read_traffic()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = max(1, min(os.cpu_count() or 1, 64))
        try:
            cpu_value, kind, sample, _ = cpu_reference_stack(threads, args.cpu_seconds)
            cpu = {"value": cpu_value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample}
        except Exception as exc:  # noqa: BLE001
            cpu = {"value": None, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": f"failed: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": workload_config(world),
            "roofline": {
                "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic,
                "kernel": "decode_persistent_kernel (the step's only kernel; one launch per step)",
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6650 GB/s",
                "algorithmic_bytes_per_step": step_bytes,
            },
            "e2e": {"value": world * 1000.0 / e2e_ms_step, "unit": UNIT,
                    "h2d_bytes_per_step": int(stack.x.numel() * 4),
                    "d2h_bytes_per_step": int(stack.logits.numel() * 4),
                    "ms_per_step": e2e_ms_step},
            "gpu_launches": launches * args.steps,
            "per_linear_launch_ms_per_step": per_linear_ms,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "when": datetime.datetime.now(datetime.timezone.utc).isoformat(timespec="seconds"),
        }
        print(json.dumps(line), flush=True)


def read_traffic():
    """DRAM bytes per decode step from the committed ncu summary, if any."""
    path = REPO / "profiles" / "decode_persistent_tinyllama_step.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_step:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def main():
    args = parse()
    if args.case:
        run_case(args.case)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # The CPU arm runs on rank 0 only; other ranks exit without work.
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
