#!/usr/bin/env python
"""Throughput benchmark of the ratchet train step on B200 (one process per GPU).

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--workload 1b|25m]

Prints ONE JSON line (rank 0).  Workloads (synthetic uint16 token ids, uniform in [0, 8192),
from a fixed seed; random-init weights of the architecture):
  1b   (default) ratchet decoder d2048 L20 H16 MLP8192 vocab 8192 block 1024, septenary codes,
       GLOBAL batch 256 sequences (262,144 tokens) at every N: each of the N ranks takes 256/N
       sequences as micro-batches of 16 whose grad_W accumulate, then one update per step --
       bf16 grad_W reduce-scattered by output-row ownership, rank-local update, all-gather of
       the int8 code|pressure bytes.  Fixed global batch: strong scaling.
  25m  ratchet decoder d512 L8 H8 MLP2048 vocab 8192 block 512, batch 32 sequences per rank
       (16,384 tokens), quinary codes (weak scaling).  At N = 1 the 1b line also carries this
       workload's measurement under "workloads".
Both: matmul_mode=int8, int8_backward; embeddings/RMSNorm fp32 with AdamW.

value  tokens/s with the token batch resident on the device, timed with CUDA events between a
       barrier + synchronize on both sides, max over ranks.
e2e    the same step through the public API with the batch copied every step from pinned host
       memory and the loss copied back to pinned host memory.
roofline  the library kernel family with the largest share of device time in the timed region:
       algorithmic bytes (or flops) per launch / mean launch time (CUDA events on its stream).
collectives  (N > 1) time the compute stream waited per step for each collective group.
cpu_baseline  the CPU restatement of the reference's fp32 eager step (oracle/model_fp32.py) on
       this host's cores over a bounded token sample (rank 0, N = 1).
--impl reference  times that same CPU step as the reference arm.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    "1b": dict(name="ratchet-decoder-1b", n_embd=2048, n_layer=20, n_head=16, vocab=8192,
               block=1024, global_batch=256, micro_batch=16, max_code=3, seed=1338,
               ref_batch=1, ref_seq=256),
    "25m": dict(name="ratchet-decoder-25m", n_embd=512, n_layer=8, n_head=8, vocab=8192, block=512,
                batch_per_rank=32, micro_batch=32, max_code=2, seed=1337, ref_batch=2,
                ref_seq=512),
}
METRIC = "ratchet train-step tokens/s"


def sequences_per_rank(wl: dict, world: int) -> int:
    if "global_batch" in wl:
        if wl["global_batch"] % world:
            raise SystemExit(f"global batch {wl['global_batch']} is not divisible by {world} ranks")
        return wl["global_batch"] // world
    return wl["batch_per_rank"]


# DRAM bytes (read + write) that ncu measured for one launch of a family's kernel at a shape of the
# workload, and that launch's algorithmic bytes (the profiles named below).  The roofline's
# `traffic` for the dominant family is this ratio times the family's mean algorithmic bytes per
# launch (traffic grows in proportion with the tiles processed).  Below 1: outputs still resident
# in L2 when the kernel ends; above 1: operand tiles read again by later waves of tiles.
NCU_TRAFFIC = {
    ("gemm_i8", "ratchet-decoder-25m"): ((9.6e6 + 7.8e6), 76.6e6,
                                         "profiles/gemm_i8_fwd_16384x512x2048.md"),
    ("quant_rows_sr", "ratchet-decoder-25m"): ((67.2e6 + 4.5e6), 100.7e6,
                                               "profiles/quant_sr_staged_bf16_16384x2048.md"),
    ("gemm_i8", "ratchet-decoder-1b"): ((46.3e6 + 145.8e6), 247.6e6,
                                        "profiles/gemm_i8_fwd_16384x2048x6144.md"),
    ("gemm_gradw_bf16", "ratchet-decoder-1b"): ((418.6e6 + 42.4e6), 318.8e6,
                                                "profiles/gemm_gradw_bf16_16384x6144x2048.md"),
}


def _traffic(family: str, workload: str, bytes_per_launch: float) -> tuple[float | None, str | None]:
    key = (family, workload)
    if key not in NCU_TRAFFIC:
        return None, None
    measured, algorithmic, source = NCU_TRAFFIC[key]
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
def cpu_model_name() -> str:
    """The host CPU's model name (lscpu / /proc/cpuinfo)."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def cpu_reference_steps(wl: dict, steps: int, warmup: int) -> dict:
    """Times the CPU fp32 restatement of the reference step (oracle/model_fp32.py) on a sample
    of ref_batch x ref_seq tokens of the workload's model."""
    import torch

    from oracle.model_fp32 import Config, build_seeded, train_step

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = Config(vocab_size=wl["vocab"], block_size=wl["block"], n_layer=wl["n_layer"],
                 n_head=wl["n_head"], n_embd=wl["n_embd"], max_code=wl["max_code"])
    model = build_seeded(cfg, wl["seed"]).train()
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.0)
    gen = torch.Generator().manual_seed(wl["seed"])
    batch, seq = wl["ref_batch"], wl["ref_seq"]
    tokens = torch.randint(0, wl["vocab"], (batch, seq + 1), generator=gen)
    for _ in range(warmup):
        train_step(model, opt, tokens)
    t0 = time.perf_counter()
    for _ in range(steps):
        train_step(model, opt, tokens)
    dt = time.perf_counter() - t0
    tokens_per_step = batch * seq
    return {"value": tokens_per_step * steps / dt, "unit": "tokens/s", "cores": threads,
            "seconds_per_step": dt / steps, "tokens_per_step": tokens_per_step,
            "cpu_model": cpu_model_name()}


def _sample_text(wl: dict, steps: int) -> str:
    return (f"{wl['ref_batch']} x {wl['ref_seq']} tokens per step of the {wl['name']} model "
            f"(fp32 eager restatement of the reference step: fused ratchet update of every "
            f"layer, AdamW), {steps} timed steps")


def run_reference(args, wl: dict, rank: int, world: int) -> None:
    if rank != 0:
        return
    res = cpu_reference_steps(wl, args.steps, args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["seconds_per_step"] * 1e3, "higher_is_better": True,
        "scaling": "strong" if "global_batch" in wl else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl["name"], "tokens_per_step": res["tokens_per_step"],
                   "sample_of": f"{sequences_per_rank(wl, world) * world} x {wl['block']} tokens"},
        "cpu_baseline": {"value": res["value"], "unit": "tokens/s", "cores": res["cores"],
                         "cpu_model": res["cpu_model"], "kind": "port",
                         "sample": _sample_text(wl, args.steps)},
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


def measure(args, wl: dict, rank: int, local_rank: int, world: int, *, steps: int,
            profile_steps: int, sample_clocks: bool) -> dict:
    """Builds the workload's model on this rank's GPU and times its train step: resident
    tokens (`value`), end to end from pinned host memory (`e2e`), and per library call (profile
    pass).  Returns the raw measurements; rank 0 formats them."""
    import torch
    import torch.distributed as dist

    from local_ai_training_b200 import ModelConfig, _lib, build_seeded_model
    from local_ai_training_b200.dist import RatchetDataParallel

    device = torch.device("cuda", local_rank)
    config = ModelConfig(vocab_size=wl["vocab"], block_size=wl["block"], n_layer=wl["n_layer"],
                         n_head=wl["n_head"], n_embd=wl["n_embd"], dropout=0.0,
                         matmul_mode="int8", int8_backward=True,
                         fused_grad_quant=args.fused_grad_quant,
                         logits_chunk_rows=args.logits_chunk_rows)
    model = build_seeded_model(config, max_code=wl["max_code"], seed=wl["seed"]).to(device).train()
    for layer in model.ratchet_layers():
        layer.sr_seed = wl["seed"] + 7
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.0, fused=True,
                            capturable=True)
    seqs = sequences_per_rank(wl, world)
    mb = min(wl["micro_batch"], seqs)
    if seqs % mb:
        raise SystemExit(f"{seqs} sequences per rank are not a multiple of micro-batch {mb}")
    micro = seqs // mb
    # deferred grouped updates after backward, grad_W accumulated over the micro-batches, and
    # (N > 1) reduce-scatter by owned rows, owner update, all-gather of the packed bytes
    ddp = RatchetDataParallel(model, bucket_layers=args.dp_bucket_layers, accumulation_steps=micro)
    gen = torch.Generator().manual_seed(wl["seed"] + rank)
    block = wl["block"]
    host_tokens = torch.randint(0, wl["vocab"], (seqs, block + 1), generator=gen,
                                dtype=torch.int64).to(torch.int16).pin_memory()
    dev_tokens16 = torch.empty(host_tokens.shape, device=device, dtype=torch.int16)
    dev_tokens16.copy_(host_tokens)
    loss_host = torch.zeros(1, dtype=torch.float32).pin_memory()

    def step():
        tokens = dev_tokens16.long()  # uint16 ids widened on the device
        losses = []
        for i in range(micro):
            chunk = tokens[i * mb:(i + 1) * mb]
            with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                _, loss = model(chunk[:, :-1], chunk[:, 1:])
            loss.backward()
            losses.append(loss.detach())
        ddp.step(opt)  # support sync, owned-row updates, AdamW, re-replication
        return losses[0] if micro == 1 else torch.stack(losses).mean()

    def eager_step():
        opt.zero_grad(set_to_none=True)
        return step()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    # warm-up (eager, on a side stream as graph capture requires), then capture one whole step:
    # token widening, every micro-batch's forward and backward, the updates, AdamW, collectives
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(args.warmup):
            eager_step()
    torch.cuda.current_stream(device).wait_stream(side)
    barrier()
    graph, graph_error, static_loss = None, None, None
    if not args.no_graph:
        try:
            opt.zero_grad(set_to_none=True)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                static_loss = step()
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
        return eager_step()

    def timed(fn, n) -> float:
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(n):
            fn()
        end.record()
        barrier()
        el = torch.tensor([start.elapsed_time(end) / 1e3], device=device)
        if world > 1:
            dist.all_reduce(el, op=dist.ReduceOp.MAX)
        return float(el.item())

    # ---- A: batch resident in HBM
    sampler = ClockSampler(list(range(world))) if (rank == 0 and sample_clocks) else None
    if sampler:
        sampler.start()
    elapsed = timed(run_step, steps)
    clocks = sampler.stop() if sampler else None

    # ---- B: end to end, batch copied from pinned host memory, loss copied back every step
    def e2e_step():
        dev_tokens16.copy_(host_tokens, non_blocking=True)
        loss = run_step()
        loss_host.copy_(loss.detach().float().reshape(1), non_blocking=True)

    e_elapsed = timed(e2e_step, steps)

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
            step()
        template, _lib.PROFILE = _lib.PROFILE, None
        barrier()
        pstart, pend = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p_elapsed = 0.0
        for _ in range(profile_steps):
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
        p_elapsed = timed(eager_step, profile_steps)
        for name, entries in _lib.PROFILE.items():
            fams_acc[name] = [(st.elapsed_time(en) / 1e3, fl, nb) for st, en, fl, nb in entries]
        _lib.PROFILE = None
    _lib.PROFILE_EXTERNAL = False
    status |= _lib.device_status(device, clear=True)

    replicas = None
    if world > 1:  # the replicated state must agree on every rank after the timed steps
        ck = ddp.state_checksum()
        lo, hi = ck.clone(), ck.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        replicas = bool(torch.equal(lo, hi))
    peak_mem = torch.cuda.max_memory_allocated(device)
    used_graph = graph is not None
    graph = None  # a graph holding NCCL work is released before the process group goes
    del model, opt, ddp
    torch.cuda.synchronize()
    return {
        "elapsed": elapsed, "e_elapsed": e_elapsed, "p_elapsed": p_elapsed, "steps": steps,
        "profile_steps": profile_steps, "profile_mode": profile_mode,
        "fams": summarize_profile(fams_acc, profile_steps), "clocks": clocks,
        "status": status, "graph": used_graph, "graph_error": graph_error,
        "tokens_per_step": seqs * block * world, "sequences_per_rank": seqs,
        "micro_batch": mb, "micro_batches": micro,
        "h2d": host_tokens.numel() * host_tokens.element_size(), "replicas_agree": replicas,
        "peak_mem_gb": round(peak_mem / 1e9, 2),
    }


def kernel_report(res: dict, workload: str, peaks: dict, int8_peak: float,
                  int8_peak_source: str) -> dict:
    """Per-family table, the dominant family's roofline and the collectives' waits."""
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    # the kernels are timed inside a step of seconds under the power cap: the sustained GEMM rate
    bf16_peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1408.0))
    bf16_source = ("MEASURED_PEAKS.json bf16_tflops_sustained (of measured; kernels timed inside "
                   "a long step)" if "bf16_tflops_sustained" in peaks else
                   "MEASURED_PEAKS.json bf16_tflops (of measured)" if "bf16_tflops" in peaks else
                   "fallback 1.4 PFLOP/s sustained")
    steps = res["profile_steps"]
    fams = {k: v for k, v in res["fams"].items() if not k.startswith("comm_")}
    comm = {k[len("comm_"):]: v for k, v in res["fams"].items() if k.startswith("comm_")}
    kernels = {}
    for name, f in sorted(fams.items(), key=lambda kv: -kv[1]["total_s"]):
        mean_s = f["mean_us"] / 1e6
        gbs = f["bytes_per_launch"] / mean_s / 1e9
        t_mem = f["bytes_per_launch"] / (hbm_peak * 1e9)
        entry = {"launches_per_step": f["launches_per_step"], "mean_us": round(f["mean_us"], 2),
                 "share_of_step": round(f["total_s"] / res["p_elapsed"], 4),
                 "GB_per_s": round(gbs, 1), "hbm_frac": round(gbs / hbm_peak, 3)}
        t_bound = t_mem
        if f["flops_per_launch"] > 0:
            tf = f["flops_per_launch"] / mean_s / 1e12
            peak = int8_peak if name == "gemm_i8" else bf16_peak
            t_bound = max(t_mem, f["flops_per_launch"] / (peak * 1e12))
            entry["TFLOP_per_s"] = round(tf, 1)
            if name == "gemm_i8":
                entry["int8_frac_datasheet_4500"] = round(tf / 4500.0, 3)
                entry["int8_frac_measured"] = round(tf / int8_peak, 3) if int8_peak else None
            else:
                entry["bf16_frac_measured"] = round(tf / bf16_peak, 3)
        # the fraction of the binding roofline: max(flops / tensor peak, bytes / HBM) over time
        entry["binding_frac"] = round(t_bound / mean_s, 3)
        kernels[name] = entry
    dominant = max(fams, key=lambda k: fams[k]["total_s"])
    d = fams[dominant]
    mean_s = d["mean_us"] / 1e6
    traffic, source = _traffic(dominant, workload, d["bytes_per_launch"])
    tensor = False
    if d["flops_per_launch"] > 0:
        tensor_peak = int8_peak if dominant == "gemm_i8" else bf16_peak
        tensor = d["flops_per_launch"] / (tensor_peak * 1e12) >= d["bytes_per_launch"] / (hbm_peak * 1e9)
    if tensor:
        achieved = d["flops_per_launch"] / mean_s / 1e12
        roofline = {"kernel": dominant, "bound": "tensor", "achieved": round(achieved, 1),
                    "peak": round(tensor_peak, 1), "unit": "TFLOP/s",
                    "frac": round(achieved / tensor_peak, 3),
                    "peak_source": int8_peak_source if dominant == "gemm_i8" else bf16_source}
    else:
        achieved = d["bytes_per_launch"] / mean_s / 1e9
        roofline = {"kernel": dominant, "bound": "hbm", "achieved": round(achieved, 1),
                    "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 3),
                    "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"}
    roofline.update({"traffic": traffic, "traffic_source": source,
                     "algorithmic_bytes_per_launch": round(d["bytes_per_launch"]),
                     "algorithmic_flops_per_launch": d["flops_per_launch"],
                     "mean_launch_us": round(d["mean_us"], 2)})
    collectives = {name: {"waits_per_step": c["launches_per_step"],
                          "exposed_ms_per_step": round(c["total_s"] / steps * 1e3, 3)}
                   for name, c in comm.items()}
    launches = sum(f["launches"] for f in fams.values()) / steps
    return {"kernels": kernels, "roofline": roofline, "collectives": collectives,
            "launches_per_step": launches}


def run_ours(args, wl: dict, rank: int, local_rank: int, world: int) -> None:
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    big = wl["name"] == WORKLOADS["1b"]["name"]
    res = measure(args, wl, rank, local_rank, world, steps=args.steps,
                  profile_steps=min(args.steps, 3) if big else args.steps, sample_clocks=True)
    secondary = None
    if world == 1 and big and not args.no_secondary:
        torch.cuda.empty_cache()
        secondary = measure(args, WORKLOADS["25m"], rank, local_rank, world, steps=args.steps,
                            profile_steps=args.steps, sample_clocks=False)
    peak_info = int8_peak_probe(torch, device) if rank == 0 and not args.no_peak_probe else {}
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = _load_peaks()
    int8_peak = max([v for v in (peak_info.get("ours_tops"), peak_info.get("cublas_int_mm_tops"))
                     if v is not None] or [0.0])
    int8_peak_source = "measured in this run (best 8192^3 int8 GEMM: ours or torch._int_mm)"
    if not int8_peak:  # probe skipped: nominal dense int8 of the part
        int8_peak, int8_peak_source = 4500.0, "nominal dense int8 (probe skipped)"
    rep = kernel_report(res, wl["name"], peaks, int8_peak, int8_peak_source)

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        c = cpu_reference_steps(wl, steps=2, warmup=1)
        cpu = {"value": c["value"], "unit": "tokens/s", "cores": c["cores"],
               "cpu_model": c["cpu_model"], "kind": "port", "sample": _sample_text(wl, 2)}
    tokens = res["tokens_per_step"]
    line = {
        "metric": METRIC, "value": tokens * args.steps / res["elapsed"], "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["elapsed"] / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if "global_batch" in wl else "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic (uniform uint16 token ids, random-init weights)",
        "config": {"workload": wl["name"], "n_embd": wl["n_embd"], "n_layer": wl["n_layer"],
                   "n_head": wl["n_head"], "vocab": wl["vocab"], "seq_len": wl["block"],
                   "global_batch": res["sequences_per_rank"] * world,
                   "micro_batch": res["micro_batch"], "micro_batches_per_rank": res["micro_batches"],
                   "codes": 2 * wl["max_code"] + 1, "matmul_mode": "int8", "int8_backward": True,
                   "parallelism": f"dp{world}" if world > 1 else "single",
                   "logits_chunk_rows": args.logits_chunk_rows,
                   "l2": "inputs larger than L2: working set (activations, weights) of many GB"},
        "e2e": {"value": tokens * args.steps / res["e_elapsed"], "unit": "tokens/s",
                "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": 4},
        "roofline": rep["roofline"],
        "cpu_baseline": cpu,
        "gpu_launches": int(round(rep["launches_per_step"] * args.steps)),
        "cuda_graph": res["graph"],
        "cuda_graph_error": res["graph_error"],
        "profile_pass": res["profile_mode"],
        "profile_ms_per_step": res["p_elapsed"] / res["profile_steps"] * 1e3,
        "clocks": res["clocks"],
        "int8_peak_probe_tops": {k: (round(v, 1) if isinstance(v, float) else v)
                                 for k, v in peak_info.items()},
        "kernels": rep["kernels"],
        "collectives": rep["collectives"],
        "replicas_agree": res["replicas_agree"],
        "peak_mem_gb": res["peak_mem_gb"],
        "device_status": res["status"],
    }
    if secondary is not None:
        srep = kernel_report(secondary, WORKLOADS["25m"]["name"], peaks, int8_peak,
                             int8_peak_source)
        sw = WORKLOADS["25m"]
        line["workloads"] = {sw["name"]: {
            "value": secondary["tokens_per_step"] * args.steps / secondary["elapsed"],
            "unit": "tokens/s", "ms_per_step": secondary["elapsed"] / args.steps * 1e3,
            "e2e": {"value": secondary["tokens_per_step"] * args.steps / secondary["e_elapsed"],
                    "unit": "tokens/s", "h2d_bytes_per_step": secondary["h2d"],
                    "d2h_bytes_per_step": 4},
            "global_batch": secondary["sequences_per_rank"], "seq_len": sw["block"],
            "codes": 2 * sw["max_code"] + 1, "cuda_graph": secondary["graph"],
            "roofline": srep["roofline"], "kernels": srep["kernels"],
            "gpu_launches_per_step": srep["launches_per_step"],
            "device_status": secondary["status"]}}
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default="1b")
    parser.add_argument("--no-secondary", action="store_true",
                        help="N = 1, workload 1b: skip the 25m measurement carried in the line")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--fused-grad-quant", action="store_true",
                        help="ModelConfig(fused_grad_quant=True): the producer backwards also "
                             "stochastic-round the layer gradients (same results)")
    parser.add_argument("--logits-chunk-rows", type=int, default=8192,
                        help="ModelConfig(logits_chunk_rows): the lm_head + loss over blocks of this "
                             "many tokens, no [tokens, vocab] tensor stored (0: materialised)")
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
        run_reference(args, wl, rank, world)
        return
    run_ours(args, wl, rank, local_rank, world)


if __name__ == "__main__":
    main()
