#!/usr/bin/env python
"""W8A8 decode tokens/s (TinyLlama-1.1B shape) + GEMV HBM GB/s vs peak.

One step = one greedy decode token of a whole TinyLlama-1.1B-shaped W8A8
decoder (config 3: 22 layers, hidden 2048, 32 query / 4 KV heads, SwiGLU
5632, RMSNorm, RoPE, vocab 32000; random-init per-row INT8 weights, batch 1)
after a 128-token random prompt: embedding, every layer's norms, q|k|v,
RoPE, KV append, attention over the cache, o, gate|up, SiLU, down,
residuals, final norm, lm_head and the argmax -- one launch of the
whole-model kernel (leafq_model_plan_run), bit-identical to the reference
decoder.  Decode positions 128..255 (the 128 generated tokens of config 3),
repeated for K steps; 1.04 GB of weights streamed per step (larger than L2).
With --gpus N each rank decodes its own request stream (data-parallel
replicas); value is the sum over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  --impl reference times the reference's own
CPU decoder (oracle/_ref/leaf_decoder, compiled from the reference sources)
on the host cores for the same metric and workload shape.
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
    p.add_argument("--steps", type=int, default=254)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--cpu-tokens", type=int, default=32,
                   help="tokens the bounded CPU-baseline sample generates (rank 0, N=1)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", choices=("decode", "batch"), default="decode",
                   help="decode: config 3 (batch 1, the headline); batch: config 4 (64 sequences x "
                        "512-token prompts, 256 greedy tokens each, split over the ranks)")
    p.add_argument("--batch-split", choices=("dp", "tp"), default="dp",
                   help="batch workload on N GPUs: dp = the sequences split over the ranks (full "
                        "weights each); tp = every linear's rows split over the ranks with an NCCL "
                        "all-gather of each output (all sequences on every rank)")
    p.add_argument("--tp-gather", choices=("peer", "nccl"), default="peer",
                   help="tp decode-step gathers: the library's peer-memory all-gather over NVLink "
                        "(captured in the step's CUDA graph) or NCCL (eager)")
    p.add_argument("--case", choices=sorted(CASES),
                   help="run one small single-kernel case three times and exit (for ncu captures)")
    return p.parse_args()


def _case_weight(rows, cols, bits, group, device):
    import torch

    import leaf_b200 as lq
    from leaf_b200.stack import random_w8_weight

    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    if bits == 8 and group == cols:
        return random_w8_weight(rows, cols, gen, device)
    if bits == 8:
        data = torch.randint(-127, 128, (rows, cols), generator=gen, device=device, dtype=torch.int8)
        scales = torch.rand(rows, cols // group, generator=gen, device=device) * 1e-3 + 1e-4
        return lq.QuantWeight(data, scales, rows, cols, 8, group)
    rng = np.random.default_rng(0)
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = (rng.random((rows, cols // group), dtype=np.float32) * 1e-3 + 1e-4).astype(np.float32)
    return lq.QuantWeight.from_host(packed, scales, rows, cols, 4, group, device=device)


# name: (tokens, rows, cols, weight bits, group, activation bits)
CASES = {
    "gemv0": (1, 5632, 2048, 8, 2048, 8),       # config 0 decode GEMV, 11.5 MB
    "gemv": (1, 11264, 2048, 8, 2048, 8),       # gate|up decode GEMV, 23 MB
    "lmhead": (1, 32000, 2048, 8, 2048, 8),     # lm_head decode GEMV, 65.5 MB
    "gemm": (512, 5632, 2048, 8, 2048, 8),      # config 2 prefill GEMM
    "gemm_down": (512, 2048, 5632, 8, 5632, 8),  # config 2 down_proj shape
    "gemm_big": (4096, 5632, 2048, 8, 2048, 8),  # large-M prefill
    "gemm_grouped": (512, 5632, 2048, 8, 128, 8),  # config 2 shape, grouped INT8 (int8_group_size 128)
    "w4": (1, 11008, 4096, 4, 32, 32),          # config 1 INT4 weight-only GEMV
    "graph_gemm": None,                          # graph INT8 GEMM, [k, n] weight, m=512 k=2048 n=5632
    "decode_small": None,                        # persistent decode kernel, 3-layer stack
    "model_small": None,                         # whole-model decode kernel, 3-layer model
    "batch_step": None,                          # config 4: 64 x 512 prefill + 2 decode steps, 22 layers
    "batch_step_small": None,                    # the same with 2 layers (for --set full captures)
}


def run_case(name):
    import torch

    import leaf_b200 as lq

    if name == "model_small":
        # The whole-model decode kernel on a 3-layer TinyLlama-width model
        # (198 MB of weights: larger than L2, small enough for ncu replays).
        from leaf_b200.decoder import Decoder
        from leaf_b200.stack import RandomDecoderModel, StackShape

        torch.cuda.set_device(0)
        model = RandomDecoderModel(StackShape(layers=3), seed=5)
        dec = Decoder(model)
        model.release()
        dec.build_fused()
        dec.forward(list(range(1, 129)))
        for _ in range(3):
            dec.step_fused()
        torch.cuda.synchronize()
        if dec.device_status() != 0:
            raise RuntimeError("device status not ok")
        print(json.dumps({"case": name, "layers": 3, "status": "ok"}))
        dec.close()
        return
    if name in ("batch_step", "batch_step_small"):
        # Config 4's operators: a 64 x 512-token batched prefill, then two
        # decode steps of all 64 sequences (per-operator launches, no graph,
        # so every kernel appears in a launch list).
        from leaf_b200.decoder import Decoder
        from leaf_b200.stack import RandomDecoderModel, StackShape

        torch.cuda.set_device(0)
        layers = 22 if name == "batch_step" else 2
        model = RandomDecoderModel(StackShape(layers=layers), seed=1)
        dec = Decoder(model, sequences=BATCH_SEQUENCES, capacity=BATCH_PROMPT + 8)
        model.release()
        prompts = np.random.default_rng(0).integers(0, 32000, size=(BATCH_SEQUENCES, BATCH_PROMPT)).tolist()
        dec.forward_batch(prompts)
        b = dec._bufs(1)
        for _ in range(2):
            dec._forward_device(b, 1)
        torch.cuda.synchronize()
        if dec.device_status() != 0:
            raise RuntimeError("device status not ok")
        print(json.dumps({"case": name, "layers": layers, "sequences": BATCH_SEQUENCES, "status": "ok"}))
        return
    if name == "graph_gemm":
        # The graph executor's gemm_i8_per_channel on the tensor cores, its
        # weight [k, n] as the graph stores it (read MN-major).
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        gen = torch.Generator(device=dev)
        gen.manual_seed(0)
        m, k, n = 512, 2048, 5632
        a = torch.randint(-127, 128, (m, k), generator=gen, device=dev, dtype=torch.int8)
        b = torch.randint(-127, 128, (k, n), generator=gen, device=dev, dtype=torch.int8)
        sc = torch.rand(n, generator=gen, device=dev) * 0.01
        for _ in range(3):
            lq.gemm_i8_per_channel(a, b, None, 0.01, sc)
        torch.cuda.synchronize()
        if lq.load().leafq_device_status() != 0:
            raise RuntimeError("device status not ok")
        print(json.dumps({"case": name, "m": m, "k": k, "n": n, "status": "ok"}))
        return
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


def measured_bf16_tflops():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["bf16_tflops"])
    return 1590.0  # fallback burst figure


PROMPT = 128   # config 3: 128 random prompt ids, then 128 greedy tokens
GENERATED = 128


def workload_config(n_gpus):
    return {
        "workload": "tinyllama-1.1b w8a8 greedy decode, whole decoder per step (22 layers: RMSNorm, "
                    "q|k|v, RoPE, KV cache, GQA attention, o, gate|up, SiLU, down, residuals; final "
                    "norm, lm_head 32000x2048, argmax), 128-token prompt, positions 128..255, batch 1 "
                    "per GPU",
        "model": "TinyLlama-1.1B shape (random-init INT8 per-row weights)",
        "global_batch": n_gpus,
        "seq_len": PROMPT + GENERATED,
        "parallelism": f"replicas x{n_gpus}",
        "l2": "inputs larger than L2 (1.04 GB of weights streamed per step)",
    }


# ----------------------------------------------------------------- CPU side
def cpu_reference_decoder(threads: int, new_tokens: int, warmup: int = 0, prompt: int = PROMPT):
    """The reference's own CPU decoder (oracle/_ref/leaf_decoder built from
    engine/src/decoder.cpp with leaf/cli.py's flags) on a TinyLlama-shaped
    W8A8 artifact (seeded random weights written by oracle/fixture.py in the
    reference's export format), 128-token prompt, activation bits 8.
    Returns (decode tokens/s, sample text)."""
    import tempfile

    import oracle
    from oracle import fixture as fx

    if not oracle.REF_DECODER.exists():
        raise RuntimeError("oracle/_ref/leaf_decoder is not built")
    with tempfile.TemporaryDirectory() as tmp:
        work = Path(tmp)
        art = work / "tinyllama_w8.leaf"
        fx.write_artifact(art, fx.TINYLLAMA, fx.llama_tensors(fx.TINYLLAMA, 7, 0.0), 8, 64)
        ids = fx.prompt_ids(fx.TINYLLAMA, 3, prompt)
        with (work / "tokens.bin").open("wb") as f:
            f.write(np.asarray([1, len(ids)], dtype="<u4").tobytes())
            f.write(np.asarray(ids, dtype="<u4").tobytes())
        cmd = [str(oracle.REF_DECODER), str(art), str(work / "tokens.bin"), str(work / "logits.bin"),
               str(work / "metrics.json"), "bench-generate", str(threads), "1", str(warmup),
               str(new_tokens), "0", "1", "8"]
        subprocess.run(cmd, check=True, capture_output=True, text=True)
        metrics = json.loads((work / "metrics.json").read_text())
    steps = metrics.get("decode_samples_ms") or []
    if not steps:
        raise RuntimeError("reference decoder reported no decode steps")
    per_ms = float(np.mean(steps))
    sample = (f"{len(steps)} greedy decode steps (positions {prompt}..{prompt + len(steps) - 1}) of the "
              f"reference decoder bench-generate on a TinyLlama-shape W8A8 artifact, {threads} threads")
    return 1000.0 / per_ms, sample


# ----------------------------------------------------------------- clocks
def smi_index(local_rank, device):
    """nvidia-smi's index of this rank's GPU (CUDA_VISIBLE_DEVICES maps it)."""
    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    return visible[local_rank] if local_rank < len(visible) else str(device.index)


class ClockSampler:
    """nvidia-smi clock / throttle samples every 100 ms while the timed region
    runs, written to a file in a private temporary directory."""

    def __init__(self, index, name: str):
        import tempfile

        self.dir = tempfile.TemporaryDirectory(prefix="leafq_clocks_")
        self.path = Path(self.dir.name) / name
        self.proc = None
        query = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.file = open(self.path, "w")
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
        self.dir.cleanup()
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
    batch = args.workload == "batch"
    # Config 4: the reference serves the requests one after another, so one
    # request's decode rate (after a 512-token prompt) is its throughput.
    new_tokens = max(2, min(args.steps + 1, 9 if batch else GENERATED))
    try:
        value, sample = cpu_reference_decoder(threads, new_tokens, warmup=min(args.warmup, 1),
                                              prompt=BATCH_PROMPT if batch else PROMPT)
    except Exception as exc:  # noqa: BLE001
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU decoder failed: {exc}"}))
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": new_tokens - 1,
        "warmup": args.warmup, "ms_per_step": 1000.0 / value, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
        "config": workload_config(1) if not batch else {
            "workload": f"config 4 on the reference: {BATCH_SEQUENCES} requests served one after another; "
                        f"one {BATCH_PROMPT}-token request timed", "global_batch": BATCH_SEQUENCES},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import leaf_b200 as lq
    from leaf_b200._lib import check
    from leaf_b200.decoder import Decoder
    from leaf_b200.stack import RandomDecoderModel, StackShape, decoder_step_bytes

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    shape = StackShape()
    model = RandomDecoderModel(shape, seed=1234 + rank, device=device)
    dec = Decoder(model, device=device)
    model.release()
    del model
    dec.build_fused()
    lib = lq.load()
    stream = torch.cuda.current_stream(device)
    gen = torch.Generator().manual_seed(99 + rank)
    prompt = torch.randint(0, shape.vocab, (PROMPT,), generator=gen).tolist()

    # Prefill the prompt (per-operator path), first token by argmax.
    logits = dec.forward(prompt)
    check(lib.leafq_argmax(stream.cuda_stream, logits.data_ptr(), 1, shape.vocab, dec.token.data_ptr()))
    first = dec.token.clone()

    def rewind():
        """Back to the state right after the prompt: the next step decodes
        position 128 again (cache rows >= 128 are rewritten)."""
        dec.position.fill_(PROMPT)
        dec.token.copy_(first)

    def steps_device(k):
        done = 0
        while done < k:
            rewind()
            r = min(GENERATED - 1, k - done)
            for _ in range(r):
                dec.step_fused()
            done += r

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Reference point: the same decode step as per-operator kernels replayed
    # from one CUDA graph (about 200 launches per token).
    dec.capture_decode()
    rewind()
    for _ in range(3):
        dec.graph.replay()
    rewind()
    g_start, g_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g_start.record(stream)
    for _ in range(GENERATED - 1):
        dec.graph.replay()
    g_end.record(stream)
    torch.cuda.synchronize(device)
    per_op_us = g_start.elapsed_time(g_end) * 1000.0 / (GENERATED - 1)

    steps_device(max(args.warmup, 3))
    torch.cuda.synchronize(device)
    if lib.leafq_device_status() != 0:
        raise RuntimeError(f"device status: {lib.leafq_last_error().decode()}")

    rates = linear_rates(device, measured_peaks()[0])

    sampler = ClockSampler(smi_index(local_rank, device), f"clocks_rank{rank}.csv")
    time.sleep(0.3)
    # ------------------------------------------------ device-timed value
    barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    steps_device(args.steps)
    end.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    ms_total = max_over_ranks(start.elapsed_time(end))
    # ------------------------------------------------ end to end (host tokens)
    # A streaming loop: every step copies its input token from pinned host
    # memory, runs, and copies the produced token back to the host (and
    # waits for it, as a server streaming tokens does).
    # Each step is one replay of Decoder.capture_stream_step's graph (token
    # in from pinned memory, the fused step, token out to pinned memory).  One
    # pinned word serves as both: the step's result lands where the next step
    # copies its input from, and the host reads it there after every step.
    tok_in = torch.empty(1, dtype=torch.int32).pin_memory()
    tok_out = tok_in
    tok_host = tok_out.numpy()
    step_graph = dec.capture_stream_step(tok_in, tok_out)
    first_host = first.cpu()
    for _ in range(3):
        dec.position.fill_(PROMPT)
        tok_in.copy_(first_host)
        step_graph.replay()
        stream.synchronize()
    barrier()
    torch.cuda.synchronize(device)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    done = 0
    while done < args.steps:
        dec.position.fill_(PROMPT)
        tok_in.copy_(first_host)
        r = min(GENERATED - 1, args.steps - done)
        for _ in range(r):
            step_graph.replay()
            stream.synchronize()
            streamed = int(tok_host[0])  # the token a server would send now
        done += r
    e_end.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms_total = max_over_ranks(e_start.elapsed_time(e_end))
    time.sleep(0.2)
    clocks = sampler.stop()
    status = lib.leafq_device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}: {lib.leafq_last_error().decode()}")
    del step_graph
    # Rank 0's greedy tokens after its prompt (model seed 1234, prompt seed
    # 99): the unsharded answer the row-sharded runs at N > 1 must give.
    rewind()
    for _ in range(TP_TOKENS - 1):
        dec.step_fused()
    replica_tokens = [int(first.item())] + [int(t) for t in dec.history[PROMPT + 1:PROMPT + TP_TOKENS].tolist()]
    dec.close()
    del dec
    torch.cuda.empty_cache()

    extra = {}
    if world == 1:
        # Config 4 (64 x 512-token prompts) on this GPU beside the headline.
        c4 = batch_run("dp", "nccl", 1, rank, device, BATCH_LINE_STEPS, args.warmup)
        c4.pop("_tokens")
        extra["config4"] = dict(c4, workload=f"config 4: {BATCH_SEQUENCES} sequences x {BATCH_PROMPT}-token "
                                             f"random prompts decoded together on one GPU, "
                                             f"{BATCH_LINE_STEPS} greedy decode steps timed")
    else:
        extra.update(multi_gpu_paths(args, rank, world, device, replica_tokens))

    ms_step = ms_total / args.steps
    value = world * 1000.0 / ms_step
    e2e_ms_step = e2e_ms_total / args.steps
    peak, peak_kind = measured_peaks()
    positions = [PROMPT + (i % (GENERATED - 1)) for i in range(args.steps)]
    step_bytes = float(np.mean([decoder_step_bytes(shape, p) for p in positions]))
    achieved = step_bytes / (ms_step * 1e-3) / 1e9
    traffic = DECODE_TRAFFIC_RATIO * step_bytes

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = max(1, min(os.cpu_count() or 1, 64))
        try:
            cpu_value, sample = cpu_reference_decoder(threads, args.cpu_tokens)
            cpu = {"value": cpu_value, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample}
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
                "kernel": "decode_model_kernel (the step's only kernel; one launch per token)",
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6650 GB/s",
                "algorithmic_bytes_per_step": step_bytes,
            },
            "e2e": {"value": world * 1000.0 / e2e_ms_step, "unit": UNIT,
                    "h2d_bytes_per_step": int(tok_in.numel() * 4),
                    "d2h_bytes_per_step": int(tok_out.numel() * 4),
                    "ms_per_step": e2e_ms_step},
            "gpu_launches": args.steps,
            "per_operator_graph_us_per_token": per_op_us,
            "linear_rates": rates,
            "clocks": clocks,
            "cpu_baseline": cpu,
            **extra,
            "when": datetime.datetime.now(datetime.timezone.utc).isoformat(timespec="seconds"),
        }
        print(json.dumps(line), flush=True)


TP_TOKENS = 17  # greedy tokens compared between the sharded and unsharded config-3 decoders
TP_STEPS = 64   # config-3 tp decode steps timed


def config3_tp_run(world, rank, device, warmup):
    """Config 3 (batch 1, 128-token prompt) with every linear's rows split
    over the ranks and each decode-step output gathered by the library's
    peer-memory all-gather inside the step's CUDA graph (per-operator
    kernels).  Model seed 1234 and prompt seed 99 on every rank: rank 0's
    replica decoded the same request unsharded.  Returns (tokens/s, tokens)."""
    import torch
    import torch.distributed as dist

    import leaf_b200 as lq
    from leaf_b200._lib import check
    from leaf_b200.decoder import Decoder
    from leaf_b200.stack import RandomDecoderModel, StackShape

    shape = StackShape()
    model = RandomDecoderModel(shape, seed=1234, device=device)
    dec = Decoder(model, device=device, group=dist.group.WORLD, gather="peer")
    model.release()
    del model
    gen = torch.Generator().manual_seed(99)
    prompt = torch.randint(0, shape.vocab, (PROMPT,), generator=gen).tolist()
    dec.capture_decode()
    tokens = dec.generate(prompt, TP_TOKENS)
    stream = torch.cuda.current_stream(device)
    dec.reset()
    logits = dec.forward(prompt)
    check(lq.load().leafq_argmax(stream.cuda_stream, logits.data_ptr(), 1, shape.vocab,
                                 dec._bufs(1)["ids"].data_ptr()))
    for _ in range(max(warmup, 3)):
        dec._decode_step()
    torch.cuda.synchronize(device)
    _barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(TP_STEPS):
        dec._decode_step()
    b.record(stream)
    torch.cuda.synchronize(device)
    _barrier(world)
    ms = _max_over_ranks(a.elapsed_time(b), world, device)
    status = lq.load().leafq_device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}: {lq.load().leafq_last_error().decode()}")
    dec.close()
    del dec
    torch.cuda.empty_cache()
    return TP_STEPS / (ms * 1e-3), tokens


def gather_timing(world, device):
    """Microseconds per all-gather of one decode-step output ([tokens, rows]
    fp32, rows split evenly over the ranks): the library's peer-memory
    gather (send + collect kernels, 20 per CUDA graph, replayed) and NCCL's
    all_gather_into_tensor (eager); max over ranks."""
    import torch
    import torch.distributed as dist

    from leaf_b200.parallel import PeerAllGather

    rank = dist.get_rank()
    stream = torch.cuda.current_stream(device)
    out = {}
    shapes = ((1, 2048), (1, 11264), (64, 2048), (64, 11264))
    peer = PeerAllGather(max(t * r for t, r in shapes))
    try:
        for tokens, rows in shapes:
            n = rows // world
            local = torch.randn(tokens, n, device=device)
            full = torch.empty(tokens, rows, device=device)
            for _ in range(3):
                peer.run(local, rank * n, rows, full)
            torch.cuda.synchronize(device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(20):
                    peer.run(local, rank * n, rows, full)
            graph.replay()
            torch.cuda.synchronize(device)
            _barrier(world)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(10):
                graph.replay()
            b.record(stream)
            torch.cuda.synchronize(device)
            peer_us = _max_over_ranks(a.elapsed_time(b) * 1e3 / 200, world, device)
            del graph
            flat = torch.empty(tokens * rows, device=device)
            for _ in range(3):
                dist.all_gather_into_tensor(flat, local.reshape(-1))
            torch.cuda.synchronize(device)
            _barrier(world)
            a.record(stream)
            for _ in range(50):
                dist.all_gather_into_tensor(flat, local.reshape(-1))
            b.record(stream)
            torch.cuda.synchronize(device)
            nccl_us = _max_over_ranks(a.elapsed_time(b) * 1e3 / 50, world, device)
            out[f"{tokens}x{rows}"] = {"peer_us": peer_us, "nccl_us": nccl_us, "bytes": tokens * rows * 4}
    finally:
        peer.close()
    return out


def multi_gpu_paths(args, rank, world, device, replica_tokens):
    """The row-sharded (tp) and sequence-split (dp) paths of configs 3 and 4
    on this job's N GPUs, beside the replica value, with a parity check:
    every sharded run's greedy tokens against unsharded runs of the same
    requests (config 4: the dp run, whose ranks hold full weights; config 3:
    rank 0's replica)."""
    import torch
    import torch.distributed as dist

    steps, warmup = BATCH_LINE_STEPS, args.warmup
    runs = {}
    for name, split, gather in (("dp", "dp", "nccl"), ("tp_peer", "tp", "peer"), ("tp_nccl", "tp", "nccl")):
        runs[name] = batch_run(split, gather, world, rank, device, steps, warmup)
    tp3_value, tp3_tokens = config3_tp_run(world, rank, device, warmup)
    gathers = gather_timing(world, device)
    # dp tokens of every rank's sequences, in sequence order, onto every rank.
    mine = torch.tensor(runs["dp"]["_tokens"], dtype=torch.int32, device=device)
    every = torch.empty((world,) + tuple(mine.shape), dtype=torch.int32, device=device)
    dist.all_gather_into_tensor(every, mine)
    unsharded = every.reshape(-1, mine.shape[1]).cpu().tolist()
    parity = {
        "config4_tp_peer": runs["tp_peer"]["_tokens"] == unsharded,
        "config4_tp_nccl": runs["tp_nccl"]["_tokens"] == unsharded,
        "config3_tp_peer": tp3_tokens == replica_tokens if rank == 0 else None,
    }
    for r in runs.values():
        r.pop("_tokens")
    return {
        "tp": {
            "config4_peer": runs["tp_peer"], "config4_nccl": runs["tp_nccl"],
            "config3_peer": {"decode_tokens_per_s": tp3_value, "steps": TP_STEPS,
                             "note": "batch 1, per-operator kernels in one CUDA graph per step"},
            "split": f"every linear's rows split over {world} GPUs, outputs all-gathered",
        },
        "dp": {"config4": runs["dp"], "split": f"{BATCH_SEQUENCES // world} sequences per GPU, full weights"},
        "gather_us": gathers,
        "tp_parity": all(v for v in parity.values() if v is not None),
        "tp_parity_detail": parity,
        "tp_parity_tokens": f"{BATCH_SEQUENCES} sequences x {steps + 1} tokens (config 4), {TP_TOKENS} tokens (config 3)",
    }


GEMV_COPIES = 32  # distinct config-0 weights per replay: 32 x 11.5 MB > L2


def linear_rates(device, peak_gbs):
    """Configs 0, 1 and 2 as figures beside the headline step.

    Config 0 (W8A8 GEMV, M=1, K=2048, N=5632, bias): GEMV_COPIES distinct
    seeded weights, one leafq_linear each with programmatic dependent launch
    (each launch streams its weights while the previous one finishes),
    captured in a CUDA graph and replayed; per-GEMV time = graph time /
    GEMV_COPIES.  The lm_head shape (N=32000) the same way with 4 copies.
    Config 1 (INT4 weight-only GEMV, K=4096, N=11008, groups of 32): 8
    distinct weights the same way.
    Config 2 (W8A8 prefill GEMM, M=512 tokens with 1% outliers x20,
    K=2048, N=5632 and K=5632, N=2048): 8 launches per graph on distinct
    weights, activation quantisation included."""
    import torch

    import leaf_b200 as lq
    from leaf_b200._lib import LEAFQ_FLAG_PDL
    from leaf_b200.stack import random_w8_weight

    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    stream = torch.cuda.current_stream(device)

    def timed(calls, reps=10):
        for fn in calls:
            fn()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for fn in calls:
                fn()
        for _ in range(3):
            graph.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize(device)
        del graph
        return a.elapsed_time(b) * 1e3 / (reps * len(calls))  # us per call

    out = {}
    ws = lq.Workspace(device)
    for name, rows, cols, copies in (("gemv_config0", 5632, 2048, GEMV_COPIES), ("gemv_lm_head", 32000, 2048, 4)):
        weights = []
        for _ in range(copies):
            w = random_w8_weight(rows, cols, gen, device)
            w.bias = torch.randn(rows, generator=gen, device=device) * 0.01
            weights.append(w)
        x = torch.randn(1, cols, generator=gen, device=device)
        ys = [torch.empty(1, rows, device=device) for _ in weights]
        us = timed([lambda w=w, y=y: lq.linear(x, w, out=y, workspace=ws, flags=LEAFQ_FLAG_PDL)
                    for w, y in zip(weights, ys)])
        nbytes = rows * cols + 4 * rows + 4 * rows + 4 * cols + 4 * rows  # W, scales, bias, x, y
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"rows": rows, "cols": cols, "us_per_call": us, "achieved": gbs, "unit": "GB/s",
                     "peak": peak_gbs, "frac": gbs / peak_gbs, "bytes_per_call": nbytes,
                     "method": f"{copies} distinct weights (> L2) back to back with PDL in one CUDA graph, "
                               "CUDA events"}
        del weights, ys
        torch.cuda.empty_cache()
    # Config 1: INT4 weight-only GEMV (M=1, K=4096, N=11008, groups of 32,
    # fp32 activations), 8 distinct weights of 28.2 MB (> L2).
    rows, cols, group = 11008, 4096, 32
    weights = []
    for _ in range(8):
        packed = torch.randint(0, 256, (rows, cols // 2), generator=gen, device=device, dtype=torch.uint8)
        scales = torch.rand(rows, cols // group, generator=gen, device=device) * 1e-3 + 1e-4
        weights.append(lq.QuantWeight(packed, scales, rows, cols, 4, group))
    x = torch.randn(1, cols, generator=gen, device=device)
    ys = [torch.empty(1, rows, device=device) for _ in weights]
    us = timed([lambda w=w, y=y: lq.linear(x, w, activation_bits=32, out=y, flags=LEAFQ_FLAG_PDL)
                for w, y in zip(weights, ys)])
    nbytes = rows * cols // 2 + 4 * rows * (cols // group) + 4 * cols + 4 * rows  # W, scales, x, y
    gbs = nbytes / (us * 1e-6) / 1e9
    out["gemv_w4a32_config1"] = {"rows": rows, "cols": cols, "group": group, "us_per_call": us, "achieved": gbs,
                                 "unit": "GB/s", "peak": peak_gbs, "frac": gbs / peak_gbs, "bytes_per_call": nbytes,
                                 "method": "8 distinct weights (> L2) back to back with PDL in one CUDA graph, "
                                           "CUDA events"}
    del weights, ys
    torch.cuda.empty_cache()
    peak_top = 2.0 * measured_bf16_tflops()
    tokens = 512
    xg = torch.randn(tokens, 5632, generator=gen, device=device)
    mask = torch.rand(tokens, 5632, generator=gen, device=device) < 0.01
    xg = torch.where(mask, xg * 20.0, xg)
    for n, k in ((5632, 2048), (2048, 5632)):
        wl = [random_w8_weight(n, k, gen, device) for _ in range(8)]
        xk = xg[:, :k].contiguous()
        yl = [torch.empty(tokens, n, device=device) for _ in wl]
        us = timed([lambda w=w, y=y: lq.linear(xk, w, out=y, workspace=ws, flags=LEAFQ_FLAG_PDL)
                    for w, y in zip(wl, yl)])
        tops = 2.0 * tokens * n * k / (us * 1e-6) / 1e12
        out[f"gemm_config2_n{n}_k{k}"] = {"us_per_call": us, "achieved": tops, "unit": "TOP/s", "peak": peak_top,
                                          "frac": tops / peak_top,
                                          "peak_source": "2 x measured bf16 burst (no INT8 figure measured)",
                                          "method": "8 distinct weights back to back in one CUDA graph "
                                                    "(activation quantisation included)"}
        del wl, yl
    # The same prefill GEMM at 4096 tokens (CTA-pair tiles), quantisation included.
    big = 4096
    xb = torch.randn(big, 2048, generator=gen, device=device)
    wl = [random_w8_weight(5632, 2048, gen, device) for _ in range(4)]
    yl = [torch.empty(big, 5632, device=device) for _ in wl]
    us = timed([lambda w=w, y=y: lq.linear(xb, w, out=y, workspace=ws, flags=LEAFQ_FLAG_PDL) for w, y in zip(wl, yl)],
               reps=5)
    tops = 2.0 * big * 5632 * 2048 / (us * 1e-6) / 1e12
    out["gemm_m4096_n5632_k2048"] = {"us_per_call": us, "achieved": tops, "unit": "TOP/s", "peak": peak_top,
                                     "frac": tops / peak_top,
                                     "peak_source": "2 x measured bf16 burst (no INT8 figure measured)",
                                     "method": "4 distinct weights back to back in one CUDA graph "
                                               "(activation quantisation included)"}
    del wl, yl, xb
    # The graph executor's INT8 GEMM (gemm_i8_per_channel) at the config-2
    # shape with its weight as the graph stores it, [k, n] (read MN-major by
    # the tensor cores): 8 distinct weights, codes given.
    m, k, n = 512, 2048, 5632
    codes = torch.randint(-127, 128, (m, k), generator=gen, device=device, dtype=torch.int8)
    bl = [torch.randint(-127, 128, (k, n), generator=gen, device=device, dtype=torch.int8) for _ in range(8)]
    sc = torch.rand(n, generator=gen, device=device) * 0.01
    us = timed([lambda b=b: lq.gemm_i8_per_channel(codes, b, None, 0.01, sc) for b in bl])
    tops = 2.0 * m * n * k / (us * 1e-6) / 1e12
    out["graph_gemm_i8_per_channel_m512_k2048_n5632"] = {
        "us_per_call": us, "achieved": tops, "unit": "TOP/s", "peak": peak_top, "frac": tops / peak_top,
        "peak_source": "2 x measured bf16 burst (no INT8 figure measured)",
        "method": "8 distinct [k, n] weights back to back in one CUDA graph (codes given, output allocated per call)"}
    del bl
    torch.cuda.empty_cache()
    # Grouped INT8 (int8_group_size 128) at the config-2 shape on the tensor
    # cores (gemm_w8a8_grouped_tc_kernel), activation quantisation included.
    group = 128
    wl = [_case_weight(5632, 2048, 8, group, device) for _ in range(8)]
    xk = xg[:, :2048].contiguous()
    yl = [torch.empty(tokens, 5632, device=device) for _ in wl]
    us = timed([lambda w=w, y=y: lq.linear(xk, w, out=y, workspace=ws, flags=LEAFQ_FLAG_PDL)
                for w, y in zip(wl, yl)])
    tops = 2.0 * tokens * 5632 * 2048 / (us * 1e-6) / 1e12
    out["gemm_grouped_g128_m512_n5632_k2048"] = {
        "us_per_call": us, "achieved": tops, "unit": "TOP/s", "peak": peak_top, "frac": tops / peak_top,
        "peak_source": "2 x measured bf16 burst (no INT8 figure measured)",
        "method": "8 distinct weights back to back in one CUDA graph (activation quantisation included)"}
    del wl, yl
    torch.cuda.empty_cache()
    return out


BATCH_SEQUENCES, BATCH_PROMPT, BATCH_GENERATED = 64, 512, 256  # config 4
BATCH_LINE_STEPS = 32  # config-4 decode steps timed beside the headline (N=1 line, and each split at N>1)


def _max_over_ranks(v, world, device):
    import torch
    import torch.distributed as dist

    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def batch_prompts():
    """Config 4's 64 seeded random 512-id prompts (identical on every rank)."""
    import torch

    from leaf_b200.stack import StackShape

    gen = torch.Generator().manual_seed(7)
    return torch.randint(0, StackShape().vocab, (BATCH_SEQUENCES, BATCH_PROMPT), generator=gen)


def batch_run(split, gather, world, rank, device, steps, warmup, sampler_name=None):
    """Config 4 on this rank's GPU: 64 requests of 512 random prompt ids,
    greedy decode (``Decoder(sequences=...)``: one KV cache and position per
    sequence, every linear over all sequences' rows).

    split "dp": the sequences split over the ranks, full weights on each;
    split "tp": every linear's rows split over the ranks (``Decoder(group=)``),
    all sequences on every rank, each linear's output all-gathered (decode
    steps by ``gather``: the library's peer-memory all-gather in the step's
    CUDA graph, or NCCL; the prompt by NCCL).

    Times the prefill and ``steps`` decode steps with CUDA events (max over
    ranks), then runs ``generate_batch`` from host prompts to host tokens
    (the end-to-end figure) and returns this rank's tokens [seqs][steps + 1]
    for the parity check."""
    import torch
    import torch.distributed as dist

    import leaf_b200 as lq
    from leaf_b200.decoder import Decoder
    from leaf_b200.stack import RandomDecoderModel, StackShape

    tp = split == "tp" and world > 1
    if BATCH_SEQUENCES % world:
        raise SystemExit(f"{BATCH_SEQUENCES} sequences do not split over {world} ranks")
    seqs = BATCH_SEQUENCES if tp else BATCH_SEQUENCES // world
    steps = min(steps, BATCH_GENERATED - 1)
    shape = StackShape()
    model = RandomDecoderModel(shape, seed=1234, device=device)
    dec = Decoder(model, device=device, sequences=seqs, capacity=BATCH_PROMPT + BATCH_GENERATED,
                  group=dist.group.WORLD if tp else None, gather=gather)
    model.release()
    del model
    lib = lq.load()
    stream = torch.cuda.current_stream(device)
    every = batch_prompts()
    prompts = every.tolist() if tp else every[rank * seqs:(rank + 1) * seqs].tolist()
    dec.capture_decode()

    def prefill():
        dec.reset()
        logits = dec.forward_batch(prompts)
        lq._lib.check(lib.leafq_argmax(stream.cuda_stream, logits.data_ptr(), seqs, shape.vocab,
                                       dec._bufs(1)["ids"].data_ptr()))

    prefill()
    for _ in range(max(warmup, 3)):
        dec._decode_step()
    torch.cuda.synchronize(device)
    sampler = None
    if sampler_name:
        sampler = ClockSampler(smi_index(device.index, device), sampler_name)
        time.sleep(0.3)
    _barrier(world)
    torch.cuda.synchronize(device)
    p0, p1, d1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    p0.record(stream)
    prefill()
    p1.record(stream)
    for _ in range(steps):
        dec._decode_step()
    d1.record(stream)
    torch.cuda.synchronize(device)
    _barrier(world)
    prefill_ms = _max_over_ranks(p0.elapsed_time(p1), world, device)
    decode_ms = _max_over_ranks(p1.elapsed_time(d1), world, device)
    # End to end through the public API: generate_batch from host prompts to
    # host tokens (prompt upload, prefill, every decode step, tokens back).
    _barrier(world)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    dec.reset()
    tokens = dec.generate_batch(prompts, steps + 1)
    torch.cuda.synchronize(device)
    e2e_s = _max_over_ranks(time.perf_counter() - t0, world, device)
    _barrier(world)
    clocks = None
    if sampler is not None:
        time.sleep(0.2)
        clocks = sampler.stop()
    status = lib.leafq_device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}: {lib.leafq_last_error().decode()}")
    assert all(len(t) == steps + 1 for t in tokens)
    dec.close()
    del dec
    torch.cuda.empty_cache()
    h, kv, d, layers = shape.hidden, shape.kv_heads, shape.hidden // shape.heads, shape.layers
    weight_bytes = (shape.weight_bytes() + shape.scale_bytes()) / (world if tp else 1)
    mean_keys = BATCH_PROMPT + (steps + 1) / 2
    step_bytes = weight_bytes + layers * seqs * 2 * kv * d * 4 * mean_keys
    ms_step = decode_ms / steps
    return {
        "decode_tokens_per_s": BATCH_SEQUENCES * steps / (decode_ms * 1e-3),
        "ms_per_step": ms_step, "steps": steps,
        "prefill": {"ms": prefill_ms, "tokens_per_s": BATCH_SEQUENCES * BATCH_PROMPT / (prefill_ms * 1e-3)},
        "e2e_tokens_per_s": BATCH_SEQUENCES * (steps + 1) / e2e_s,
        "hbm_gbs_per_gpu": step_bytes / (ms_step * 1e-3) / 1e9,
        "algorithmic_bytes_per_step_per_gpu": step_bytes,
        "sequences_per_gpu": seqs,
        "clocks": clocks,
        "_tokens": tokens,
    }


def run_batch(args, rank, world, local_rank):
    """Config 4 as the bench line (--workload batch): 64 requests of 512
    random prompt ids, greedy decode; one step = one decode token for every
    sequence; value = generated tokens/s over the whole job (prefill beside
    it).  With N ranks the sequences are split over the GPUs (dp) or every
    linear's rows are (tp).  Every sequence's tokens equal the
    single-sequence decoder's and the reference's
    (tests/test_gpu_decoder_batch.py)."""
    import torch

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    tp = args.batch_split == "tp" and world > 1
    r = batch_run(args.batch_split, args.tp_gather, world, rank, device, args.steps, args.warmup,
                  sampler_name=f"clocks_batch_rank{rank}.csv")
    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        threads = max(1, min(os.cpu_count() or 1, 64))
        try:
            cpu_value, sample = cpu_reference_decoder(threads, 9, prompt=BATCH_PROMPT)
            cpu = {"value": cpu_value, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": sample + "; the reference serves the 64 requests one after another, so "
                                      "this is its config-4 throughput"}
        except Exception as exc:  # noqa: BLE001
            cpu = {"value": None, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": f"failed: {exc}"}
    seqs = r["sequences_per_gpu"]
    steps = r["steps"]
    line = {
        "metric": METRIC, "value": r["decode_tokens_per_s"], "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {
            "workload": f"config 4: tinyllama-1.1b w8a8, {BATCH_SEQUENCES} sequences x {BATCH_PROMPT}-token "
                        f"random prompts, greedy decode (one step = one token for every sequence), "
                        f"positions {BATCH_PROMPT}..{BATCH_PROMPT + steps - 1}",
            "model": "TinyLlama-1.1B shape (random-init INT8 per-row weights)",
            "global_batch": BATCH_SEQUENCES, "seq_len": BATCH_PROMPT + BATCH_GENERATED,
            "parallelism": (f"tp{world} (every linear's rows split over the GPUs, each output "
                            f"all-gathered: decode steps by {args.tp_gather}, the prompt by NCCL; all "
                            f"{seqs} sequences on every GPU)") if tp else
                           f"dp{world} ({seqs} sequences per GPU, full weights each)",
            "l2": "inputs larger than L2 (1.04 GB of weights and the KV caches streamed per step)",
        },
        "prefill": r["prefill"],
        "roofline": {
            "bound": "hbm", "achieved": r["hbm_gbs_per_gpu"], "peak": peak, "unit": "GB/s",
            "frac": r["hbm_gbs_per_gpu"] / peak, "traffic": None,
            "kernel": "whole decode step (per-operator kernels in one CUDA graph)",
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
            "algorithmic_bytes_per_step": r["algorithmic_bytes_per_step_per_gpu"],
        },
        "e2e": {"value": r["e2e_tokens_per_s"], "unit": UNIT,
                "h2d_bytes_per_step": int(seqs * BATCH_PROMPT * 4 / (steps + 1)),
                "d2h_bytes_per_step": int(seqs * 4),
                "note": "generate_batch wall time including the prompt prefill"},
        "clocks": r["clocks"],
        "cpu_baseline": cpu,
        "when": datetime.datetime.now(datetime.timezone.utc).isoformat(timespec="seconds"),
    }
    print(json.dumps(line), flush=True)


# DRAM traffic of decode_model_kernel per algorithmic byte: dram__bytes_read.sum +
# dram__bytes_write.sum over decoder_step_bytes, from the ncu capture of
# `bench.py --case model_small` (3 layers at full width; traffic grows with the
# weights streamed, each read once, so the ratio carries to the 22-layer step).
DECODE_TRAFFIC_RATIO = 1.024


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
        if args.workload == "batch":
            run_batch(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
