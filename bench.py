#!/usr/bin/env python
"""Throughput benchmark of the ratchet train step on B200 (one process per GPU).

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--workload 25m]

Prints ONE JSON line (rank 0).  Workloads:
  25m  ratchet decoder d512 L8 H8 MLP2048 vocab 8192 block 512 batch 32 (16,384 tokens/step),
       quinary codes, matmul_mode=int8, int8_backward; embeddings/RMSNorm fp32 with AdamW.
Synthetic data: uint16 token ids uniform in [0, 8192) from a fixed seed, random-init weights.

value  tokens/s with the token batch resident on the device, timed with CUDA events between a
       barrier + synchronize on both sides, max over ranks.
e2e    the same step through the public API with the batch copied every step from pinned host
       memory and the loss copied back to pinned host memory.
roofline  the library kernel family with the largest share of device time in the timed region:
       algorithmic bytes (or flops) per launch / mean launch time (CUDA events on its stream).
cpu_baseline  the CPU restatement of the reference's fp32 eager step (oracle/model_fp32.py) on
       this host's cores over a bounded token sample (rank 0, N = 1).
--impl reference  times that same CPU step as the reference arm.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    "25m": dict(name="ratchet-decoder-25m", n_embd=512, n_layer=8, n_head=8, vocab=8192, block=512,
                batch=32, max_code=2, seed=1337, ref_batch=2),
}
METRIC = "ratchet train-step tokens/s"


# DRAM bytes (read + write) that ncu measured for one launch of a family's kernel, and that
# launch's algorithmic bytes (profiles/gemm_i8_fwd_16384x512x2048.md,
# profiles/quant_rows_sr_bf16_16384x2048.md).  The roofline's `traffic` for the dominant family is
# this ratio times the family's mean algorithmic bytes per launch (traffic grows in proportion
# with the rows processed).  Below 1: outputs still resident in L2 when the kernel ends.
NCU_TRAFFIC = {
    "gemm_i8": ((9.59e6 + 9.11e6), 76.6e6, "profiles/gemm_i8_fwd_16384x512x2048.md"),
    "quant_rows_sr": ((67.15e6 + 7.62e6), 100.7e6, "profiles/quant_rows_sr_bf16_16384x2048.md"),
}


def _traffic(family: str, bytes_per_launch: float) -> tuple[float | None, str | None]:
    if family not in NCU_TRAFFIC:
        return None, None
    measured, algorithmic, source = NCU_TRAFFIC[family]
    return round(measured / algorithmic * bytes_per_launch), source


def _load_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            pass
    return {}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices: list[int]):
        self.gpus = set(gpu_indices)
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx not in self.gpus:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_reference_steps(wl: dict, batch: int, steps: int, warmup: int) -> dict:
    """Times the CPU fp32 restatement of the reference step (oracle/model_fp32.py)."""
    import torch

    from oracle.model_fp32 import Config, build_seeded, train_step

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = Config(vocab_size=wl["vocab"], block_size=wl["block"], n_layer=wl["n_layer"],
                 n_head=wl["n_head"], n_embd=wl["n_embd"], max_code=wl["max_code"])
    model = build_seeded(cfg, wl["seed"]).train()
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.0)
    gen = torch.Generator().manual_seed(wl["seed"])
    tokens = torch.randint(0, wl["vocab"], (batch, wl["block"] + 1), generator=gen)
    for _ in range(warmup):
        train_step(model, opt, tokens)
    t0 = time.perf_counter()
    for _ in range(steps):
        train_step(model, opt, tokens)
    dt = time.perf_counter() - t0
    tokens_per_step = batch * wl["block"]
    return {"value": tokens_per_step * steps / dt, "unit": "tokens/s", "cores": threads,
            "seconds_per_step": dt / steps, "tokens_per_step": tokens_per_step}


def run_reference(args, wl: dict, rank: int) -> None:
    if rank != 0:
        return
    res = cpu_reference_steps(wl, wl["ref_batch"], args.steps, args.warmup)
    sample = (f"{wl['ref_batch']} x {wl['block']} tokens per step of the {wl['name']} config "
              f"(fp32 eager, fused ratchet update, AdamW), {args.steps} timed steps")
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["seconds_per_step"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl["name"], "tokens_per_step": res["tokens_per_step"],
                   "sample_of": f"batch {wl['batch']} x {wl['block']}"},
        "cpu_baseline": {"value": res["value"], "unit": "tokens/s", "cores": res["cores"],
                         "kind": "port", "sample": sample},
        "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def int8_peak_probe(torch, device) -> dict:
    """Large-K int8 GEMM throughput: this library's tcgen05 kernel and torch._int_mm (cuBLAS)."""
    from local_ai_training_b200.int8_matmul import _scaled_int8_mm_into

    n = 8192
    a = torch.randint(-127, 128, (n, n), device=device, dtype=torch.int8)
    b = torch.randint(-3, 4, (n, n), device=device, dtype=torch.int8)
    sa = torch.ones(n, device=device)
    out = torch.empty((n, n), device=device, dtype=torch.bfloat16)
    res = {}

    def timeit(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps / 1e3

    t = timeit(lambda: _scaled_int8_mm_into(a, b.t(), sa, None, out))
    res["ours_tops"] = 2 * n**3 / t / 1e12
    try:
        t2 = timeit(lambda: torch._int_mm(a, b.t()))
        res["cublas_int_mm_tops"] = 2 * n**3 / t2 / 1e12
    except Exception as exc:  # noqa: BLE001
        res["cublas_int_mm_tops"] = None
        res["cublas_error"] = str(exc)[:120]
    return res


def summarize_profile(profile: dict, steps: int) -> dict:
    """profile: family -> [(seconds, flops, bytes)] over `steps` steps."""
    fams = {}
    for name, entries in profile.items():
        total = sum(t for t, _, _ in entries)
        fams[name] = {
            "launches": len(entries), "launches_per_step": len(entries) / steps,
            "total_s": total, "mean_us": total / len(entries) * 1e6,
            "flops_per_launch": sum(f for _, f, _ in entries) / len(entries),
            "bytes_per_launch": sum(b for _, _, b in entries) / len(entries),
        }
    return fams


def run_ours(args, wl: dict, rank: int, local_rank: int, world: int) -> None:
    import torch
    import torch.distributed as dist

    from local_ai_training_b200 import ModelConfig, _lib, build_seeded_model

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    config = ModelConfig(vocab_size=wl["vocab"], block_size=wl["block"], n_layer=wl["n_layer"],
                         n_head=wl["n_head"], n_embd=wl["n_embd"], dropout=0.0,
                         matmul_mode="int8", int8_backward=True)
    model = build_seeded_model(config, max_code=wl["max_code"], seed=wl["seed"]).to(device).train()
    for layer in model.ratchet_layers():
        layer.sr_seed = wl["seed"] + 7 * (rank + 1)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.0, fused=True,
                            capturable=True)
    gen = torch.Generator().manual_seed(wl["seed"] + rank)
    batch, block = wl["batch"], wl["block"]
    host_tokens = torch.randint(0, wl["vocab"], (batch, block + 1), generator=gen,
                                dtype=torch.int64).to(torch.int16).pin_memory()
    dev_tokens16 = torch.empty(host_tokens.shape, device=device, dtype=torch.int16)
    dev_tokens16.copy_(host_tokens)
    tokens_resident = dev_tokens16.long()
    loss_host = torch.zeros(1, dtype=torch.float32).pin_memory()

    ddp = None
    if world > 1:
        # data parallel: reduce-scatter of bf16 grad_W by owned rows during backward, rank-local
        # update, all-gather of the owned packed rows, averaged support gradients
        from local_ai_training_b200.dist import RatchetDataParallel

        ddp = RatchetDataParallel(model, bucket_layers=args.dp_bucket_layers)

    def step(tokens):
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            _, loss = model(tokens[:, :-1], tokens[:, 1:])
        loss.backward()
        if ddp is None:
            model.ratchet_update(validate=False)
            opt.step()
        else:
            ddp.step(opt)  # support all-reduce, owned-row updates, AdamW, re-replication
        return loss

    def eager_step(tokens):
        opt.zero_grad(set_to_none=True)
        return step(tokens)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    # warm-up (eager, on a side stream as graph capture requires), then capture one whole step:
    # token widening, forward, backward with the fused ratchet updates, AdamW.
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(args.warmup):
            eager_step(tokens_resident)
    torch.cuda.current_stream(device).wait_stream(side)
    barrier()
    graph, graph_error = None, None
    if not args.no_graph:
        try:
            opt.zero_grad(set_to_none=True)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                static_loss = step(dev_tokens16.long())
            for _ in range(2):
                graph.replay()
            barrier()
        except Exception as exc:  # noqa: BLE001 - report and time eagerly instead
            graph = None
            graph_error = f"{type(exc).__name__}: {str(exc)[:200]}"
            torch.cuda.synchronize()
    status = _lib.device_status(device, clear=True)

    def run_step():
        if graph is not None:
            graph.replay()
            return static_loss
        return eager_step(dev_tokens16.long())

    def timed(fn) -> float:
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            fn()
        end.record()
        barrier()
        el = torch.tensor([start.elapsed_time(end) / 1e3], device=device)
        if world > 1:
            dist.all_reduce(el, op=dist.ReduceOp.MAX)
        return float(el.item())

    # ---- A: batch resident in HBM
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
    elapsed = timed(run_step)
    clocks = sampler.stop() if sampler else None

    # ---- B: end to end, batch copied from pinned host memory, loss copied back every step
    def e2e_step():
        dev_tokens16.copy_(host_tokens, non_blocking=True)
        loss = run_step()
        loss_host.copy_(loss.detach().float().reshape(1), non_blocking=True)

    e_elapsed = timed(e2e_step)

    # ---- C: CUDA events around every library call.  Preferred: a second captured graph whose
    # event-record nodes re-time each call on every replay (no launch gaps); otherwise eager steps.
    profile_mode = "graph"
    fams_acc: dict = {}
    try:
        if graph is None:
            raise RuntimeError("no graph")
        _lib.PROFILE, _lib.PROFILE_EXTERNAL = {}, True
        pgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(pgraph, pool=graph.pool()):
            step(dev_tokens16.long())
        template, _lib.PROFILE = _lib.PROFILE, None
        barrier()
        pstart, pend = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p_elapsed = 0.0
        for _ in range(args.steps):
            pstart.record()
            pgraph.replay()
            pend.record()
            pend.synchronize()
            p_elapsed += pstart.elapsed_time(pend) / 1e3
            for name, entries in template.items():
                acc = fams_acc.setdefault(name, [])
                acc.extend((st.elapsed_time(en) / 1e3, fl, nb) for st, en, fl, nb in entries)
        del pgraph
    except Exception as exc:  # noqa: BLE001 - fall back to timing eager steps
        profile_mode = f"eager ({type(exc).__name__})"
        fams_acc = {}
        _lib.PROFILE, _lib.PROFILE_EXTERNAL = {}, False
        p_elapsed = timed(lambda: eager_step(tokens_resident))
        for name, entries in _lib.PROFILE.items():
            fams_acc[name] = [(st.elapsed_time(en) / 1e3, fl, nb) for st, en, fl, nb in entries]
        _lib.PROFILE = None
    _lib.PROFILE_EXTERNAL = False
    status |= _lib.device_status(device, clear=True)

    tokens_per_step = batch * block * world
    fams = summarize_profile(fams_acc, args.steps)
    gpu_launches = sum(f["launches"] for f in fams.values())  # library kernels per K steps

    peak_info = int8_peak_probe(torch, device) if rank == 0 and not args.no_peak_probe else {}
    used_graph = graph is not None
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        graph = None  # a graph holding NCCL work is released before the group goes
        torch.cuda.synchronize()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = _load_peaks()
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    bf16_peak = peaks.get("bf16_tflops", 1590.0)
    int8_peak = max(v for v in (peak_info.get("ours_tops"), peak_info.get("cublas_int_mm_tops"), 0.0)
                    if v is not None)
    int8_peak_source = "measured in this run (int8 GEMM probe)"
    if not int8_peak:  # probe skipped: nominal dense int8 of the part
        int8_peak, int8_peak_source = 4500.0, "nominal dense int8 (probe skipped)"
    dominant = max(fams, key=lambda k: fams[k]["total_s"])
    kernels = {}
    for name, f in sorted(fams.items(), key=lambda kv: -kv[1]["total_s"]):
        mean_s = f["mean_us"] / 1e6
        gbs = f["bytes_per_launch"] / mean_s / 1e9
        entry = {"launches_per_step": f["launches_per_step"], "mean_us": round(f["mean_us"], 2),
                 "share_of_step": round(f["total_s"] / p_elapsed, 4),
                 "GB_per_s": round(gbs, 1), "hbm_frac": round(gbs / hbm_peak, 3)}
        if f["flops_per_launch"] > 0:
            tf = f["flops_per_launch"] / mean_s / 1e12
            entry["TFLOP_per_s"] = round(tf, 1)
            if name == "gemm_i8":
                entry["int8_frac_datasheet_4500"] = round(tf / 4500.0, 3)
                entry["int8_frac_measured"] = round(tf / int8_peak, 3) if int8_peak else None
            else:
                entry["bf16_frac_measured"] = round(tf / bf16_peak, 3)
        kernels[name] = entry
    d = fams[dominant]
    mean_s = d["mean_us"] / 1e6
    # The bound of the dominant family: its arithmetic intensity against the ridge point.
    if d["flops_per_launch"] > 0:
        tensor_peak = int8_peak if dominant == "gemm_i8" else bf16_peak
        t_compute = d["flops_per_launch"] / (tensor_peak * 1e12)
        t_memory = d["bytes_per_launch"] / (hbm_peak * 1e9)
        if t_compute >= t_memory:
            achieved = d["flops_per_launch"] / mean_s / 1e12
            roofline = {"kernel": dominant, "bound": "tensor", "achieved": round(achieved, 1),
                        "peak": round(tensor_peak, 1), "unit": "TFLOP/s",
                        "frac": round(achieved / tensor_peak, 3),
                        "traffic": _traffic(dominant, d["bytes_per_launch"])[0],
                        "traffic_source": _traffic(dominant, d["bytes_per_launch"])[1],
                        "peak_source": int8_peak_source if dominant == "gemm_i8"
                        else "MEASURED_PEAKS.json bf16_tflops"}
        else:
            achieved = d["bytes_per_launch"] / mean_s / 1e9
            roofline = {"kernel": dominant, "bound": "hbm", "achieved": round(achieved, 1),
                        "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 3),
                        "traffic": _traffic(dominant, d["bytes_per_launch"])[0],
                        "traffic_source": _traffic(dominant, d["bytes_per_launch"])[1],
                        "peak_source": "MEASURED_PEAKS.json hbm_gbs"}
    else:
        achieved = d["bytes_per_launch"] / mean_s / 1e9
        roofline = {"kernel": dominant, "bound": "hbm", "achieved": round(achieved, 1),
                    "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 3),
                    "traffic": _traffic(dominant, d["bytes_per_launch"])[0],
                    "traffic_source": _traffic(dominant, d["bytes_per_launch"])[1],
                    "peak_source": "MEASURED_PEAKS.json hbm_gbs"}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        res = cpu_reference_steps(wl, wl["ref_batch"], steps=2, warmup=1)
        cpu = {"value": res["value"], "unit": "tokens/s", "cores": res["cores"], "kind": "port",
               "sample": (f"{wl['ref_batch']} x {wl['block']} tokens per step, 2 timed steps of the "
                          f"same config, fp32 eager CPU restatement of the reference step")}
    value = tokens_per_step * args.steps / elapsed
    h2d = host_tokens.numel() * host_tokens.element_size()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": wl["name"], "n_embd": wl["n_embd"], "n_layer": wl["n_layer"],
                   "n_head": wl["n_head"], "vocab": wl["vocab"], "seq_len": block,
                   "global_batch": batch * world, "codes": 2 * wl["max_code"] + 1,
                   "matmul_mode": "int8", "int8_backward": True,
                   "parallelism": f"dp{world}" if world > 1 else "single",
                   "l2": "working set (activations, logits) far above the 126 MB L2"},
        "e2e": {"value": tokens_per_step * args.steps / e_elapsed, "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "gpu_launches": gpu_launches,
        "cuda_graph": used_graph,
        "cuda_graph_error": graph_error,
        "profile_pass": profile_mode,
        "profile_ms_per_step": p_elapsed / args.steps * 1e3,
        "clocks": clocks,
        "int8_peak_probe_tops": {k: (round(v, 1) if isinstance(v, float) else v) for k, v in peak_info.items()},
        "kernels": kernels,
        "device_status": status,
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default="25m")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-graph", action="store_true", help="time eager steps (no CUDA graph)")
    parser.add_argument("--dp-bucket-layers", type=int, default=4,
                        help="N>1: layers whose grad_W reduce-scatters are batched into one group")
    parser.add_argument("--no-peak-probe", action="store_true",
                        help="skip the 8192^3 int8 GEMM probe (ours vs torch._int_mm)")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl, rank)
        return
    run_ours(args, wl, rank, local_rank, world)


if __name__ == "__main__":
    main()
