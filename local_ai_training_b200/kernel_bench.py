"""Kernel microbenchmarks of the ratchet-linear hot path (the 25M model's layer shapes).

    python -m local_ai_training_b200.kernel_bench all              # every kernel, three shapes
    python -m local_ai_training_b200.kernel_bench gradw --m 16384 --n 1536 --k 512 --reps 3

Each case times R launches with CUDA events after warm-up (L2 flushed between launches unless
--no-flush) and prints one JSON line: mean launch time, algorithmic bytes and flops per launch,
and the fractions of the measured HBM / tensor peaks.  Used as the small, single-kernel command
for ncu captures.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import _lib
from .int8_matmul import (
    _quantize_rows_fused,
    _scaled_int8_mm_into,
    dequant_rows_bf16,
    grad_weight_bf16,
)

SHAPES = [(512, 512), (512, 2048), (2048, 512)]  # (K in, N out) of the 25M model's ratchet layers
SHAPES_1B = [(2048, 6144), (2048, 2048), (2048, 8192), (8192, 2048)]  # the ~1B model's layers


def _peaks() -> dict:
    path = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    peaks = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
    if path.exists():
        data = json.loads(path.read_text())
        peaks.update({k: data[k] for k in ("hbm_gbs", "bf16_tflops") if k in data})
        peaks["source"] = "MEASURED_PEAKS.json"
    return peaks


class _Flusher:
    """Replaces the L2 contents by reading a 256 MB buffer that is never written after set-up:
    the timed kernel then starts with a cold and clean L2 (a write flush would leave ~126 MB of
    dirty lines whose write-back lands inside the timed region)."""

    def __init__(self, device):
        self.buf = torch.zeros(32 * 1024 * 1024, dtype=torch.float64, device=device)
        self.out = torch.empty((), dtype=torch.float64, device=device)

    def __call__(self):
        torch.sum(self.buf, dim=0, out=self.out)


def _time(fn, reps: int, flush: _Flusher | None) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        if flush is not None:
            flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e) / 1e3
    return total / reps


def _report(name, shape, t, nbytes, flops, peak_tensor, peaks):
    out = {"kernel": name, "shape": shape, "us": round(t * 1e6, 2),
           "GB_per_s": round(nbytes / t / 1e9, 1), "hbm_frac": round(nbytes / t / 1e9 / peaks["hbm_gbs"], 3)}
    if flops:
        tf = flops / t / 1e12
        out["TFLOP_per_s"] = round(tf, 1)
        out["tensor_peak"] = peak_tensor
        out["tensor_frac"] = round(tf / peak_tensor, 3)
        out["roofline_time_frac"] = round(max(flops / (peak_tensor * 1e12), nbytes / (peaks["hbm_gbs"] * 1e9)) / t, 3)
    print(json.dumps(out), flush=True)
    return out


def bench_gemm_fwd(m, k, n, reps, flush, peaks, int8_peak, out_dtype=torch.bfloat16):
    dev = torch.device("cuda")
    q = torch.randint(-127, 128, (m, k), device=dev, dtype=torch.int8)
    s = torch.rand(m, device=dev) + 0.01
    code = torch.randint(-3, 4, (n, k), device=dev, dtype=torch.int8)
    scale = torch.rand(n, device=dev) * 0.045 + 0.005
    out = torch.empty((m, n), device=dev, dtype=out_dtype)
    t = _time(lambda: _scaled_int8_mm_into(q, code.t(), s, scale, out, rhs_abs_max=7), reps, flush)
    nbytes = m * k + n * k + 4 * (m + n) + m * n * out.element_size()
    return _report("gemm_i8_fwd", [m, k, n], t, nbytes, 2.0 * m * n * k, int8_peak, peaks)


def bench_gemm_grad_input(m, k, n, reps, flush, peaks, int8_peak):
    dev = torch.device("cuda")
    gq = torch.randint(-127, 128, (m, n), device=dev, dtype=torch.int8)
    gs = torch.rand(m, device=dev) + 0.01
    code = torch.randint(-2, 3, (n, k), device=dev, dtype=torch.int8)
    out = torch.empty((m, k), device=dev, dtype=torch.bfloat16)
    t = _time(lambda: _scaled_int8_mm_into(gq, code, gs, None, out, rhs_abs_max=7), reps, flush)
    nbytes = m * n + n * k + 4 * m + 2 * m * k
    return _report("gemm_i8_grad_input", [m, n, k], t, nbytes, 2.0 * m * n * k, int8_peak, peaks)


def bench_gradw(m, k, n, reps, flush, peaks):
    dev = torch.device("cuda")
    g = (torch.randn(m, n, device=dev) * 1e-3).to(torch.bfloat16)
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    out = torch.empty((n, k), device=dev, dtype=torch.float32)
    t = _time(lambda: grad_weight_bf16(g, x, out=out), reps, flush)
    nbytes = 2 * m * (n + k) + 4 * n * k
    return _report("gemm_gradw_bf16", [m, n, k], t, nbytes, 2.0 * m * n * k, peaks["bf16_tflops"], peaks)


def bench_quant_sr(m, n, reps, flush, peaks, dtype=torch.float32):
    """The grad_output quantiser as the layer calls it: column-scaled, stochastic, Philox step on
    the device; an fp32 gradient also gets its bf16 copy written (a bf16 one is used in place)."""
    dev = torch.device("cuda")
    g = (torch.randn(m, n, device=dev) * 1e-3).to(dtype)
    cs = torch.rand(n, device=dev) * 0.04 + 0.01
    gbf = torch.empty((m, n), device=dev, dtype=torch.bfloat16) if dtype != torch.bfloat16 else None
    step_dev = torch.zeros(2, device=dev, dtype=torch.int32)
    t = _time(lambda: _quantize_rows_fused(g, cs, stochastic=True, seed=7, step=0, layer=0,
                                           bf16_copy=gbf, step_dev=step_dev), reps, flush)
    nbytes = m * n * (g.element_size() + 1 + (2 if gbf is not None else 0)) + 4 * m + 4 * n
    return _report(f"quant_rows_sr_{str(dtype).split('.')[-1]}", [m, n], t, nbytes, 0, 0, peaks)


def bench_quant_rn(m, k, reps, flush, peaks, dtype=torch.bfloat16):
    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).to(dtype)
    t = _time(lambda: _quantize_rows_fused(x), reps, flush)
    return _report(f"quant_rows_rn_{str(dtype).split('.')[-1]}", [m, k], t,
                   m * k * (x.element_size() + 1) + 4 * m, 0, 0, peaks)


def bench_dequant(m, k, reps, flush, peaks):
    dev = torch.device("cuda")
    q = torch.randint(-127, 128, (m, k), device=dev, dtype=torch.int8)
    s = torch.rand(m, device=dev)
    t = _time(lambda: dequant_rows_bf16(q, s), reps, flush)
    return _report("dequant", [m, k], t, 3 * m * k + 4 * m, 0, 0, peaks)


def bench_update_grouped(shapes, reps, flush, peaks, name):
    """One grouped update launch per row length over the layers `shapes` ((rows, cols) each,
    bf16 gradients), as the train step runs it after backward."""
    dev = torch.device("cuda")
    groups: dict = {}
    keep = []
    for rows, cols in shapes:
        grad = (torch.randn(rows, cols, device=dev) * 1e-3).to(torch.bfloat16)
        packed = (torch.randint(0, 7, (rows, cols), device=dev, dtype=torch.uint8)
                  | (torch.randint(0, 15, (rows, cols), device=dev, dtype=torch.uint8) << 4))
        code = torch.empty((rows, cols), device=dev, dtype=torch.int8)
        counts = torch.zeros(4, device=dev, dtype=torch.int64)
        rms = torch.zeros(1, device=dev)
        keep.append((grad, packed, code, counts, rms))
        groups.setdefault(cols, []).append(len(keep) - 1)
    descs = {}
    for cols, idx in groups.items():
        arr = (_lib.UpdateLayer * len(idx))()
        for d, i in zip(arr, idx):
            grad, packed, code, counts, rms = keep[i]
            d.grad, d.ldg, d.rows = grad.data_ptr(), cols, grad.shape[0]
            d.packed, d.ldp, d.code_out, d.ldc = packed.data_ptr(), cols, code.data_ptr(), cols
            d.rms_ema, d.counts, d.rms_sum, d.grad_mul = None, counts.data_ptr(), rms.data_ptr(), 1.0
        descs[cols] = arr
    stream = _lib.stream_of(keep[0][0])

    def run():
        for cols, arr in descs.items():
            _lib.check(_lib.lib().rt_ratchet_update_grouped(
                arr, len(arr), _lib.BF16, 0, cols, 1, 0.0, 3, 8, 0.5, 1.5, 1e-8, stream))

    t = _time(run, reps, flush)
    weights = sum(r * c for r, c in shapes)
    rows = sum(r for r, _ in shapes)
    return _report(name, [len(shapes), weights], t, weights * 5 + 4 * rows, 0, 0, peaks)


def model_layer_shapes(d: int, layers: int, vocab: int) -> list[tuple[int, int]]:
    """(rows, cols) of every ratchet matrix of the decoder: qkv, projection, expand, contract per
    block and the lm_head."""
    block = [(3 * d, d), (d, d), (4 * d, d), (d, 4 * d)]
    return block * layers + [(vocab, d)]


def bench_update(rows, cols, reps, flush, peaks, grad_dtype=torch.float32):
    dev = torch.device("cuda")
    grad = (torch.randn(rows, cols, device=dev) * 1e-3).to(grad_dtype)
    packed = torch.randint(0, 256, (rows, cols), device=dev, dtype=torch.uint8)
    packed = (packed & 0x0F).clamp(max=4) | (torch.randint(0, 15, (rows, cols), device=dev, dtype=torch.uint8) << 4)
    code = torch.empty((rows, cols), device=dev, dtype=torch.int8)
    counts = torch.zeros(4, device=dev, dtype=torch.int64)
    rr = torch.empty(rows, device=dev)

    def run():
        _lib.check(_lib.lib().rt_ratchet_update(
            grad.data_ptr(), _lib.dtype_code(grad), 1, cols, rows, cols, packed.data_ptr(), cols,
            code.data_ptr(), cols, 1, None, 0.0, 2, 8, 0.5, 1.5, 1e-8, counts.data_ptr(),
            rr.data_ptr(), None, None, _lib.stream_of(grad)))

    t = _time(run, reps, flush)
    nbytes = rows * cols * (grad.element_size() + 3) + 4 * rows
    return _report(f"ratchet_update_{str(grad_dtype).split('.')[-1]}", [rows, cols], t, nbytes, 0, 0, peaks)


def bench_rmsnorm_bwd(m, k, reps, flush, peaks, dtype=torch.float32):
    from .int8_backward import rmsnorm_backward

    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).to(dtype)
    gy = (torch.randn(m, k, device=dev) * 1e-2).to(dtype)
    w = torch.rand(k, device=dev) + 0.5
    t = _time(lambda: rmsnorm_backward(gy, x, w), reps, flush)
    return _report(f"rmsnorm_bwd_{str(dtype).split('.')[-1]}", [m, k], t, 3 * m * k * x.element_size(),
                   0, 0, peaks)


def bench_producers(m, k, reps, flush, peaks, dtype=torch.float32):
    from .int8_fused import fused_gelu_quantize, fused_rmsnorm_quantize, fused_transpose_quantize

    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).to(dtype)
    w = torch.rand(k, device=dev) + 0.5
    es = x.element_size()
    # as the train step calls them: int8 rows, scales and the bf16 dequantised copy
    t = _time(lambda: fused_rmsnorm_quantize(x, w, dequant_out=True), reps, flush)
    _report(f"rmsnorm_quant_{str(dtype).split('.')[-1]}", [m, k], t, m * k * (es + 3), 0, 0, peaks)
    xg = torch.randn(m, 4 * k, device=dev).to(torch.bfloat16)
    t = _time(lambda: fused_gelu_quantize(xg, dequant_out=True), reps, flush)
    _report("gelu_quant_bfloat16", [m, 4 * k], t, m * 4 * k * (2 + 3), 0, 0, peaks)
    heads = k // 64
    xt = torch.randn(m // 512, heads, 512, 64, device=dev, dtype=torch.bfloat16)
    t = _time(lambda: fused_transpose_quantize(xt, dequant_out=True), reps, flush)
    _report("transpose_quant_bfloat16", list(xt.shape), t, xt.numel() * 5, 0, 0, peaks)


def bench_gelu_bwd(m, k, reps, flush, peaks):
    from .int8_backward import gelu_backward

    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    gy = (torch.randn(m, k, device=dev) * 1e-2).to(torch.bfloat16)
    t = _time(lambda: gelu_backward(gy, x), reps, flush)
    return _report("gelu_bwd_bfloat16", [m, k], t, 3 * m * k * 2, 0, 0, peaks)


def bench_cross_entropy(m, vocab, reps, flush, peaks):
    """The lm_head loss kernels: per-row max / log-sum-exp / loss of fp32 logits, then the bf16
    logit gradient."""
    from .cross_entropy import cross_entropy_grad_bf16, cross_entropy_rows

    dev = torch.device("cuda")
    logits = torch.randn(m, vocab, device=dev) * 2.0
    targets = torch.randint(0, vocab, (m,), device=dev)
    t = _time(lambda: cross_entropy_rows(logits, targets), reps, flush)
    _report("ce_fwd_float32", [m, vocab], t, 4 * m * vocab, 0, 0, peaks)
    row_max, row_logsum, _ = cross_entropy_rows(logits, targets)
    count = torch.tensor([float(m)], device=dev)
    gl = torch.ones((), device=dev)
    t = _time(lambda: cross_entropy_grad_bf16(logits, targets, row_max, row_logsum, gl, count),
              reps, flush)
    return _report("ce_bwd_float32", [m, vocab], t, 6 * m * vocab, 0, 0, peaks)


def bench_matmul_bf16(m, k, n, reps, flush, peaks):
    """The lm_head's bf16 grad_input GEMM: [m, k] x [k, n] (k = vocab)."""
    from .int8_matmul import matmul_bf16

    dev = torch.device("cuda")
    a = (torch.randn(m, k, device=dev) * 1e-3).to(torch.bfloat16)
    b = torch.randn(k, n, device=dev).to(torch.bfloat16)
    t = _time(lambda: matmul_bf16(a, b), reps, flush)
    return _report("gemm_bf16", [m, k, n], t, 2 * (m * k + k * n + m * n), 2.0 * m * n * k,
                   peaks["bf16_tflops"], peaks)


def bench_unpack(rows, cols, reps, flush, peaks):
    """The code-mirror refresh after the data-parallel all-gather of `packed`."""
    dev = torch.device("cuda")
    packed = (torch.randint(0, 7, (rows, cols), device=dev, dtype=torch.uint8)
              | (torch.randint(0, 15, (rows, cols), device=dev, dtype=torch.uint8) << 4))
    code = torch.empty((rows, cols), device=dev, dtype=torch.int8)

    def run():
        _lib.check(_lib.lib().rt_unpack_code_pressure(
            packed.data_ptr(), cols, rows, cols, 3, code.data_ptr(), cols, None, 0,
            _lib.stream_of(packed)))

    t = _time(run, reps, flush)
    return _report("unpack_codes", [rows, cols], t, 2 * rows * cols, 0, 0, peaks)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("kernel", choices=["all", "all1b", "fwd", "grad_input", "gradw", "quant_sr",
                                           "quant_rn", "dequant", "update", "update_grouped",
                                           "rmsnorm_bwd", "producers", "gelu_bwd", "ce",
                                           "matmul_bf16", "unpack"])
    parser.add_argument("--m", type=int, default=16384)
    parser.add_argument("--k", type=int, default=512)
    parser.add_argument("--n", type=int, default=2048)
    parser.add_argument("--reps", type=int, default=20)
    parser.add_argument("--layers", type=int, default=20, help="update_grouped: decoder blocks")
    parser.add_argument("--no-flush", action="store_true")
    parser.add_argument("--dtype", choices=["f32", "bf16"], default="f32",
                        help="input dtype of quant_sr / quant_rn")
    parser.add_argument("--int8-peak", type=float, default=4500.0,
                        help="INT8 dense peak (TOPS) for the fractions; datasheet by default")
    args = parser.parse_args()
    peaks = _peaks()
    flush = None if args.no_flush else _Flusher(torch.device("cuda"))
    m = args.m
    if args.kernel == "all":
        for k, n in SHAPES:
            bench_gemm_fwd(m, k, n, args.reps, flush, peaks, args.int8_peak)
            bench_gemm_grad_input(m, k, n, args.reps, flush, peaks, args.int8_peak)
            bench_gradw(m, k, n, args.reps, flush, peaks)
            bench_quant_sr(m, n, args.reps, flush, peaks, torch.float32)
            bench_quant_sr(m, n, args.reps, flush, peaks, torch.bfloat16)
            bench_quant_rn(m, k, args.reps, flush, peaks)
            bench_dequant(m, k, args.reps, flush, peaks)
            bench_update(n, k, args.reps, flush, peaks)
        bench_update(8192, 2048, args.reps, flush, peaks)
        bench_update(8192, 2048, args.reps, flush, peaks, torch.bfloat16)
        bench_update_grouped(model_layer_shapes(512, 8, 8192), args.reps, flush, peaks,
                             "ratchet_update_grouped_25m")
        bench_update_grouped(model_layer_shapes(2048, 20, 8192), args.reps, flush, peaks,
                             "ratchet_update_grouped_1b")
        bench_rmsnorm_bwd(m, 512, args.reps, flush, peaks)
        bench_producers(m, 512, args.reps, flush, peaks)
        bench_gelu_bwd(m, 2048, args.reps, flush, peaks)
        bench_cross_entropy(m, 8192, args.reps, flush, peaks)
        bench_matmul_bf16(m, 8192, 512, args.reps, flush, peaks)
        return
    if args.kernel == "all1b":  # the ~1B decoder's layer shapes, M = 16384 tokens
        for k, n in SHAPES_1B:
            bench_gemm_fwd(m, k, n, args.reps, flush, peaks, args.int8_peak)
            bench_gemm_grad_input(m, k, n, args.reps, flush, peaks, args.int8_peak)
            bench_gradw(m, k, n, args.reps, flush, peaks)
            bench_quant_sr(m, n, args.reps, flush, peaks, torch.bfloat16)
        bench_update(8192, 2048, args.reps, flush, peaks, torch.bfloat16)
        bench_update_grouped(model_layer_shapes(2048, 20, 8192), args.reps, flush, peaks,
                             "ratchet_update_grouped_1b")
        bench_rmsnorm_bwd(m, 2048, args.reps, flush, peaks)
        return
    if args.kernel == "fwd":
        bench_gemm_fwd(m, args.k, args.n, args.reps, flush, peaks, args.int8_peak)
    elif args.kernel == "grad_input":
        bench_gemm_grad_input(m, args.k, args.n, args.reps, flush, peaks, args.int8_peak)
    elif args.kernel == "gradw":
        bench_gradw(m, args.k, args.n, args.reps, flush, peaks)
    elif args.kernel == "quant_sr":
        bench_quant_sr(m, args.n, args.reps, flush, peaks,
                       torch.bfloat16 if args.dtype == "bf16" else torch.float32)
    elif args.kernel == "quant_rn":
        bench_quant_rn(m, args.k, args.reps, flush, peaks,
                       torch.bfloat16 if args.dtype == "bf16" else torch.float32)
    elif args.kernel == "dequant":
        bench_dequant(m, args.k, args.reps, flush, peaks)
    elif args.kernel == "update":
        bench_update(args.n, args.k, args.reps, flush, peaks,
                     torch.bfloat16 if args.dtype == "bf16" else torch.float32)
    elif args.kernel == "update_grouped":
        bench_update_grouped(model_layer_shapes(args.k, args.layers, 8192), args.reps, flush,
                             peaks, f"ratchet_update_grouped_d{args.k}")
    elif args.kernel == "rmsnorm_bwd":
        bench_rmsnorm_bwd(m, args.k, args.reps, flush, peaks)
    elif args.kernel == "producers":
        bench_producers(m, args.k, args.reps, flush, peaks)
    elif args.kernel == "gelu_bwd":
        bench_gelu_bwd(m, args.k, args.reps, flush, peaks)
    elif args.kernel == "ce":
        bench_cross_entropy(m, args.n, args.reps, flush, peaks)
    elif args.kernel == "matmul_bf16":
        bench_matmul_bf16(m, args.k, args.n, args.reps, flush, peaks)
    elif args.kernel == "unpack":
        bench_unpack(args.n, args.k, args.reps, flush, peaks)


if __name__ == "__main__":
    main()
