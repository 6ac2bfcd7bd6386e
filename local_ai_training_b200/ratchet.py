"""Master-weight-free discrete linear layers (the ratchet) on sm_100a.

API-compatible with the reference module ratchet.py: the same classes, constructor arguments,
buffers (`packed` uint8 code|pressure nibbles, `_scale` fp32 or `log_scale`), properties,
update/validation methods, statistics and audits.  The compute runs in the CUDA library:

* int8 mode: tcgen05 int8 GEMMs (forward, grad_input with fused stochastic-rounding quant), the
  tcgen05 bf16 grad_weight GEMM and the one-pass ratchet update kernel;
* bf16 / fp32 modes: the matmuls of the reference are torch (cuBLAS) ops, grad_weight in bf16 mode
  is the tcgen05 GEMM, and the update is always the CUDA kernel.

CPU tensors are rejected for every compute op ("requires CUDA"); the CPU fp32 restatement of the
reference lives in oracle/ and is used only as the test checker and the reported CPU baseline.

Layout: besides `packed`, each layer keeps a non-persistent int8 code mirror (the GEMM operand,
[out, in] row-major).  The update kernel rewrites it together with `packed`; if `packed` is
modified from outside (its version counter moves), the mirror is rebuilt by the unpack kernel.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from . import _lib
from .int8_matmul import (
    _quantize_rows_fused,
    _scaled_int8_mm_into,
    dequant_rows_bf16,
    grad_weight_bf16,
    matmul_bf16,
    quantize_rows,
)


def _require_cuda(t: Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} requires CUDA; this build runs the ratchet on sm_100a only")


class _RatchetMatmul(torch.autograd.Function):
    """BF16/int8 matmul whose backward exposes the effective-weight gradient (ratchet.py:18-182).

    Same argument list as the reference.  `code` is the layer's int8 code tensor [out, in];
    `gradient_sink(grad_weight_fp32, tile_start, tile_end, round_bf16=..., want_grad_scale=...)`
    receives the whole [out, in] gradient at once (rows are independent, so one launch covers
    every tile of the reference's tile loop) and returns the trainable-scale gradient when asked.
    """

    @staticmethod
    def forward(ctx, inputs, inputs_int8, inputs_scale, code, scale, mode, fuse_backward_update,
                int8_backward, tile_size, gradient_sink, residual=None, inputs_dequant=None):
        input_shape = inputs.shape
        flat_inputs = inputs.flatten(0, -2)
        out_features = code.shape[0]
        ctx.input_shape = input_shape
        ctx.input_dtype = inputs.dtype
        # the reference returns `.to(inputs.dtype)`; a layer may ask for another output dtype
        layer = getattr(gradient_sink, "__self__", None)
        result_dtype = getattr(layer, "output_dtype", None) or inputs.dtype
        # residual (fp32): the output is residual + the layer output, the block's residual add;
        # the layer output's own dtype still decides how its gradient is rounded in backward
        ctx.has_residual = residual is not None
        ctx.output_dtype = result_dtype
        ctx.mode = mode
        ctx.fuse_backward_update = fuse_backward_update
        ctx.int8_backward = int8_backward
        ctx.tile_size = tile_size
        ctx.gradient_sink = gradient_sink
        _require_cuda(code, "the ratchet matmul")

        if mode == "int8":
            ctx.has_dequant = False
            if inputs_int8 is not None and inputs_scale is not None:
                q = inputs_int8.flatten(0, -2)
                s = inputs_scale.flatten(0, -1)
                if inputs_dequant is not None:
                    # the producer also wrote bf16(bf16(q)·bf16(s)): keep it as the grad_weight
                    # operand instead of the int8 rows (no dequant pass in backward)
                    ctx.save_for_backward(inputs_dequant.flatten(0, -2), s, code, scale)
                    ctx.has_dequant = True
                else:
                    ctx.save_for_backward(q, s, code, scale)
                ctx.used_fused_int8 = True
            else:
                if not inputs.is_cuda:
                    raise RuntimeError("quantize_rows requires CUDA; the int8 path is GPU-only")
                q, s = quantize_rows(flat_inputs)
                ctx.save_for_backward(flat_inputs, code, scale)
                ctx.used_fused_int8 = False
            out_dtype = result_dtype if result_dtype in (torch.float32, torch.bfloat16) else torch.bfloat16
            res_flat = None
            if residual is not None and residual.dtype == torch.float32:
                out_dtype = torch.float32
                res_flat = residual.reshape(q.shape[0], out_features)
                if res_flat.stride(1) != 1:
                    res_flat = res_flat.contiguous()
            output = torch.empty((q.shape[0], out_features), device=q.device, dtype=out_dtype)
            # rhs = codeᵀ: (in, out) view of the [out, in] code tensor, K-major for the GEMM
            _scaled_int8_mm_into(q, code.t(), s, scale.float().contiguous(), output,
                                 rhs_abs_max=_code_bound(gradient_sink), residual=res_flat)
            output = output.reshape(*input_shape[:-1], out_features)
            if residual is None:
                return output.to(result_dtype)
            if res_flat is None:  # a residual in another dtype: the add the reference performs
                return residual + output.to(result_dtype)
            return output

        _require_cuda(inputs, "the ratchet matmul")
        ctx.save_for_backward(flat_inputs, code, scale)
        ctx.used_fused_int8 = False
        if mode == "fp32":
            effective = code.to(torch.float32) * scale.to(torch.float32)[:, None]
            output = flat_inputs.to(torch.float32) @ effective.t()
        elif mode == "bf16":
            effective = code.to(torch.bfloat16) * scale.to(torch.bfloat16)[:, None]
            output = flat_inputs.to(torch.bfloat16) @ effective.t()
        else:
            raise ValueError("matmul_mode must be fp32, bf16, or int8")
        output = output.reshape(*input_shape[:-1], out_features).to(result_dtype)
        return output if residual is None else residual + output

    @staticmethod
    def backward(ctx, grad_output):
        grad_residual = grad_output if ctx.has_residual else None
        # the layer output's own gradient: the residual sum's gradient in the output's dtype (the
        # cast autograd applies at the add); an fp32 gradient meeting a bf16 output is rounded by
        # the quantiser on the int8 path, cast here otherwise
        round_grad_bf16 = (ctx.has_residual and ctx.output_dtype == torch.bfloat16
                           and grad_output.dtype == torch.float32)
        if ctx.used_fused_int8:
            q, s, code, scale = ctx.saved_tensors
            flat_inputs = None
            # ratchet.py:73-76 (already done by the producer when it saved the bf16 rows)
            inputs_bf16 = q if ctx.has_dequant else dequant_rows_bf16(q, s)
        else:
            flat_inputs, code, scale = ctx.saved_tensors
            inputs_bf16 = None if ctx.mode == "fp32" else flat_inputs.to(torch.bfloat16)
        flat_gradient = grad_output.flatten(0, -2)
        out_features, in_features = code.shape
        grad_bf16 = None
        if round_grad_bf16 and not (ctx.int8_backward and ctx.used_fused_int8
                                    and ctx.fuse_backward_update):
            flat_gradient = flat_gradient.to(torch.bfloat16)

        # ---- grad_input (ratchet.py:84-141)
        if ctx.mode == "fp32":
            gradient_fp32 = flat_gradient.to(torch.float32)
            effective = code.to(torch.float32) * scale.to(torch.float32)[:, None]
            grad_input = gradient_fp32 @ effective
        elif ctx.int8_backward and ctx.used_fused_int8 and ctx.fuse_backward_update:
            # fold the per-out scale into the gradient, stochastic-round to int8 (one pass that
            # also writes bf16(gradient) for grad_weight), int8 GEMM against the codes
            # a bf16 gradient with unit column stride is already the grad_weight operand; any
            # other gets its bf16 copy written by the same pass
            if flat_gradient.dtype == torch.bfloat16 and flat_gradient.stride(1) == 1:
                grad_bf16, bf16_copy = flat_gradient, None
            else:
                grad_bf16 = torch.empty(flat_gradient.shape, device=flat_gradient.device,
                                        dtype=torch.bfloat16)
                bf16_copy = grad_bf16
            pre = _take_prequantized(ctx.gradient_sink, flat_gradient, round_grad_bf16)
            if pre is not None:  # quantised by the op that produced the gradient
                gq, gs, grad_bf16 = pre
            else:
                seed, step, layer, step_dev = _sr_key(ctx.gradient_sink)
                gq, gs = _quantize_rows_fused(flat_gradient, scale.float(), stochastic=True,
                                              seed=seed, step=step, layer=layer,
                                              bf16_copy=bf16_copy,
                                              step_dev=step_dev,  # the call advances step_dev
                                              round_input_bf16=round_grad_bf16)
            gi_dtype = ctx.input_dtype if ctx.input_dtype in (torch.float32, torch.bfloat16) else torch.bfloat16
            grad_input = torch.empty((gq.shape[0], in_features), device=gq.device, dtype=gi_dtype)
            _scaled_int8_mm_into(gq, code, gs, None, grad_input,
                                 rhs_abs_max=_code_bound(ctx.gradient_sink))
        else:
            # ratchet.py:135-141: bf16 gradient against bf16(code)·bf16(scale), on the tcgen05 GEMM
            grad_bf16 = flat_gradient.to(torch.bfloat16)
            effective = dequant_rows_bf16(code, scale.float().contiguous())
            grad_input = matmul_bf16(grad_bf16, effective)

        # ---- grad_weight (ratchet.py:148-163)
        if ctx.mode != "fp32" and grad_bf16 is None:
            grad_bf16 = flat_gradient.to(torch.bfloat16)
        grad_scale = _deliver_weight_gradient(
            ctx.gradient_sink, ctx.mode, ctx.fuse_backward_update, grad_bf16, inputs_bf16,
            flat_gradient, flat_inputs, code, bool(ctx.needs_input_grad[4]))
        return (grad_input.reshape(ctx.input_shape).to(ctx.input_dtype), None, None, None,
                grad_scale, None, None, None, None, None, grad_residual, None)


def _deliver_weight_gradient(gradient_sink, mode: str, fuse_backward_update: bool,
                             grad_bf16: Tensor | None, inputs_bf16: Tensor | None,
                             flat_gradient: Tensor | None, flat_inputs: Tensor | None,
                             code: Tensor, want_scale: bool) -> Tensor | None:
    """grad_W of one ratchet layer (ratchet.py:148-169) handed to where it is consumed: the
    data-parallel reduce-scatter buffer, the fused update (sink), or the pending gradient.
    Returns the trainable-scale gradient when asked for."""
    out_features = code.shape[0]
    dp = getattr(getattr(gradient_sink, "__self__", None), "_dp", None)
    if dp is not None and mode != "fp32":
        # data-parallel: the bf16-rounded grad_W goes to the layer's reduce-scatter buffer and
        # the update runs later on the owned rows of the summed gradient
        layer = gradient_sink.__self__
        target = dp.grad_target(layer)
        grad_weight_bf16(grad_bf16, inputs_bf16, out=target.out, accumulate=target.accumulate,
                         addend=target.addend)
        grad_scale = None
        if want_scale:
            # the trainable-scale gradient is linear in grad_W: the micro-batch that completes
            # the step's total returns it for the whole step, the earlier ones zero
            grad_scale = ((target.out.float() * code.float()).sum(dim=1) if target.last else
                          torch.zeros(out_features, device=code.device, dtype=torch.float32))
        dp.grad_ready(layer)
        return grad_scale
    if mode == "fp32":
        grad_weight = flat_gradient.to(torch.float32).t() @ flat_inputs.to(torch.float32)
        round_bf16 = False
    else:
        layer = getattr(gradient_sink, "__self__", None)
        if (fuse_backward_update and isinstance(layer, DiscreteRatchetLinear)
                and layer.fused_gradw_update):
            done, grad_scale = layer._grad_weight_update(grad_bf16, inputs_bf16, want_scale)
            if done:
                return grad_scale
        grad_weight = grad_weight_bf16(grad_bf16, inputs_bf16)
        round_bf16 = True
    return _sink_weight_gradient(gradient_sink, fuse_backward_update, grad_weight, round_bf16,
                                 code, want_scale)


def _sink_weight_gradient(gradient_sink, fuse_backward_update: bool, grad_weight: Tensor,
                          round_bf16: bool, code: Tensor, want_scale: bool) -> Tensor | None:
    """A whole [out, in] grad_W (fp32; rounded to bf16 first when round_bf16, as the reference's
    bf16 GEMM output is) to the fused update or the pending gradient."""
    if fuse_backward_update:
        return gradient_sink(grad_weight, 0, code.shape[0], round_bf16=round_bf16,
                             want_grad_scale=want_scale)
    if round_bf16:
        grad_weight = grad_weight.to(torch.bfloat16).float()
    gradient_sink(grad_weight, None, None)
    return (grad_weight * code.float()).sum(dim=1) if want_scale else None


def ratchet_update_grouped(entries: list[tuple["DiscreteRatchetLinear", Tensor, int, int, float]],
                           *, stats_weights: dict | None = None) -> None:
    """The fused update (normalise, bucket, pressure/code step; ratchet.py:487-556, 265-301) of
    many layers after backward, in as few launches as possible (rt_ratchet_update_grouped).

    entries: (layer, gradient rows, row_start, row_end, grad_mul) -- `gradient` holds rows
    [row_start, row_end) of the layer's effective-weight gradient (fp32 or bf16, unit column
    stride), multiplied by grad_mul inside the kernel.  Per layer the result is that of
    `_capture_weight_gradient` on gradient * grad_mul; the layer's move counters and rms sum
    accumulate in its pending statistics.  stats_weights (optional): layer -> the weight count
    to record for the layer's statistics instead of its updated rows (data-parallel owners
    report the whole matrix)."""
    groups: dict[tuple, list] = {}
    for layer, grad, row_start, row_end, grad_mul in entries:
        pk = layer.packed
        _require_cuda(pk, "the ratchet update")
        if grad.dtype not in (torch.float32, torch.bfloat16):
            grad = grad.float()
        if grad.stride(-1) != 1:
            grad = grad.contiguous()
        if grad.shape != (row_end - row_start, layer.in_features):
            raise ValueError("grouped update: gradient rows do not match the row range")
        key = (pk.device, grad.dtype, layer.in_features, layer.max_code,
               layer.pressure_threshold, float(layer.bucket_low), float(layer.bucket_high),
               float(layer.eps), float(layer.rms_ema_beta))
        groups.setdefault(key, []).append((layer, grad, row_start, row_end, grad_mul))
    for key, items in groups.items():
        device, dtype, cols, max_code, threshold, low, high, eps, beta = key
        descs = (_lib.UpdateLayer * len(items))()
        for d, (layer, grad, row_start, row_end, grad_mul) in zip(descs, items):
            layer._pending_stat_slots(device)
            mirror = layer.code_int8()
            pk = layer.packed
            d.grad = grad.data_ptr()
            d.ldg = grad.stride(0)
            d.rows = row_end - row_start
            d.packed = pk[row_start:row_end].data_ptr()
            d.ldp = pk.stride(0)
            d.code_out = mirror[row_start:row_end].data_ptr()
            d.ldc = mirror.stride(0)
            d.rms_ema = (layer.rms_ema[row_start:row_end].data_ptr()
                         if beta > 0.0 else None)
            d.counts = layer._pending_counts.data_ptr()
            d.rms_sum = layer._pending_rms.data_ptr()
            d.grad_mul = float(grad_mul)
        first = items[0][1]
        ev = _lib.prof_start(first)
        _lib.check(_lib.lib().rt_ratchet_update_grouped(
            descs, len(items), _lib.dtype_code(first), 0, cols, 1, beta, max_code, threshold,
            low, high, eps, _lib.stream_of(first)))
        if ev is not None:
            rows = sum(r1 - r0 for _, _, r0, r1, _ in items)
            _lib.prof_stop(ev, "ratchet_update", first, 0.0,
                           rows * cols * (first.element_size() + 3) + 4 * rows)
        for layer, grad, row_start, row_end, grad_mul in items:
            weights = (stats_weights or {}).get(layer)
            layer._pending_stats_total_weights += (
                weights if weights is not None else (row_end - row_start) * layer.in_features)
            layer._pending_stats_rms_sum = layer._pending_rms[0]


def _code_bound(sink) -> int:
    """|code| bound of the layer behind a gradient sink (its max_code; the layer keeps every code
    within it), or 0 when the codes come from elsewhere."""
    layer = getattr(sink, "__self__", None)
    return int(layer.max_code) if isinstance(layer, DiscreteRatchetLinear) else 0


def _sr_key(sink) -> tuple[int | None, int, int, Tensor | None]:
    layer = getattr(sink, "__self__", None)
    if isinstance(layer, DiscreteRatchetLinear):
        return layer._next_sr_key()
    return None, 0, 0, None


class GradientQuantPlan:
    """The int8-backward quantisation a ratchet layer will apply to its output gradient
    (ratchet.py:117-134: fold the layer's row scales into the gradient, stochastic-round each
    token row to int8), attached by the layer's forward to its output tensor as
    `_ratchet_grad_plan`.  The op that consumes that output produces the gradient in its own
    backward; it may quantise the gradient in the same pass (the same values, Philox stream and
    step advance as the layer's own quantisation) and `deliver` the result, which the layer's
    backward then uses instead of reading the gradient again.

    round_if_fp32: an fp32 gradient is rounded to bf16 first (a bf16 layer output whose residual
    sum is fp32)."""

    __slots__ = ("layer", "round_if_fp32")

    def __init__(self, layer: "DiscreteRatchetLinear", round_if_fp32: bool) -> None:
        self.layer = layer
        self.round_if_fp32 = round_if_fp32

    def col_scale(self) -> Tensor:
        return self.layer.scale.detach().float().contiguous()

    def sr_key(self) -> tuple[int, int, int, Tensor | None]:
        """(seed, step, layer id, step_dev) of the layer's next quantisation; a host-drawn seed
        when the layer has none (int8_matmul.py:200)."""
        seed, step, layer_id, step_dev = self.layer._next_sr_key()
        if seed is None:
            seed = int(torch.randint(0, 2**31 - 1, (1,)).item())
        return seed, step, layer_id, step_dev

    def deliver(self, gradient: Tensor, q: Tensor, row_scale: Tensor, grad_bf16: Tensor,
                round_bf16: bool) -> None:
        self.layer._prequant_grad = (gradient, q, row_scale, grad_bf16, round_bf16)


def grad_plan_of(tensor: Tensor) -> GradientQuantPlan | None:
    """The GradientQuantPlan a ratchet layer attached to its output tensor, if any."""
    return getattr(tensor, "_ratchet_grad_plan", None)


def _take_prequantized(sink, flat_gradient: Tensor, round_bf16: bool):
    """(q, row_scale, grad_bf16) delivered for exactly this gradient tensor, else None."""
    layer = getattr(sink, "__self__", None)
    pre = getattr(layer, "_prequant_grad", None)
    if pre is None:
        return None
    layer._prequant_grad = None
    gradient, q, row_scale, grad_bf16, rounded = pre
    if (gradient.data_ptr() != flat_gradient.data_ptr() or gradient.dtype != flat_gradient.dtype
            or gradient.numel() != flat_gradient.numel() or not flat_gradient.is_contiguous()
            or rounded != round_bf16 or q.shape != flat_gradient.shape):
        return None
    return q, row_scale, grad_bf16


def pack_code_pressure(code: Tensor, pressure: Tensor, max_code: int) -> Tensor:
    """Pack signed code (low nibble) and pressure (high nibble) into one uint8 (ratchet.py:185-192).

    Lossless for code in [-max_code, max_code] (max_code <= 7) and pressure in [-7, 7].
    """
    low = (code.to(torch.int16) + max_code) & 0x0F
    high = (pressure.to(torch.int16) + 7) & 0x0F
    return (low | (high << 4)).to(torch.uint8)


def unpack_code_pressure(packed: Tensor, max_code: int) -> tuple[Tensor, Tensor]:
    """ratchet.py:195-199; CUDA tensors go through the unpack kernel."""
    if packed.is_cuda and packed.dim() == 2 and packed.dtype == torch.uint8:
        code = torch.empty(packed.shape, device=packed.device, dtype=torch.int8)
        pressure = torch.empty(packed.shape, device=packed.device, dtype=torch.int8)
        rows, cols = packed.shape
        _lib.check(_lib.lib().rt_unpack_code_pressure(
            packed.data_ptr(), packed.stride(0), rows, cols, max_code, code.data_ptr(),
            code.stride(0), pressure.data_ptr(), pressure.stride(0), _lib.stream_of(packed)))
        return code, pressure
    value = packed.to(torch.int16)
    code = ((value & 0x0F) - max_code).to(torch.int8)
    pressure = ((value >> 4) - 7).to(torch.int8)
    return code, pressure


@dataclass(frozen=True)
class RatchetUpdateStats:
    total_weights: int
    positive_moves: int
    negative_moves: int
    blocked_positive_moves: int
    blocked_negative_moves: int
    gradient_rms_mean: float

    @property
    def code_moves(self) -> int:
        return self.positive_moves + self.negative_moves

    @property
    def blocked_moves(self) -> int:
        return self.blocked_positive_moves + self.blocked_negative_moves

    def materialize(self) -> RatchetUpdateStats:
        """Return a copy with all fields as python scalars (forces the GPU->CPU sync)."""

        def scalar(v: object) -> object:
            return v.item() if isinstance(v, torch.Tensor) else v

        return RatchetUpdateStats(
            total_weights=int(scalar(self.total_weights)),
            positive_moves=int(scalar(self.positive_moves)),
            negative_moves=int(scalar(self.negative_moves)),
            blocked_positive_moves=int(scalar(self.blocked_positive_moves)),
            blocked_negative_moves=int(scalar(self.blocked_negative_moves)),
            gradient_rms_mean=float(scalar(self.gradient_rms_mean)),
        )


@dataclass(frozen=True)
class RatchetAuditReport:
    ratchet_layers: int
    ratchet_weights: int
    ratchet_state_bytes: int
    support_parameter_bytes: int
    violations: tuple[str, ...]


def bucket_pressure(z: Tensor, *, low: float = 0.5, high: float = 1.5) -> Tensor:
    """Convert normalized gradients to integer pressure in descent direction (ratchet.py:248-262).

    Format helper with the reference's semantics; the update kernel applies the same rule fused.
    """
    if not 0 <= low < high:
        raise ValueError("pressure bucket thresholds must satisfy 0 <= low < high")
    magnitude = z.abs()
    bucket = torch.where(
        magnitude >= high,
        torch.full_like(z, 2, dtype=torch.int16),
        torch.where(magnitude >= low, torch.ones_like(z, dtype=torch.int16),
                    torch.zeros_like(z, dtype=torch.int16)),
    )
    return -torch.sign(z).to(torch.int16) * bucket


class DiscreteRatchetLinear(nn.Module):
    """Linear layer with integer codes and pressure, but no master weight parameter."""

    # fused update: grad_W goes from the GEMM's split-K partial tiles straight into the update
    # kernel (never stored; identical results).  Off by default: summing up to ~18 partials per
    # element inside the row-wise update ran slower on B200 than the all-SM split-K reduce it
    # replaces followed by the update
    fused_gradw_update: bool = False

    def __init__(
        self,
        in_features: int,
        out_features: int,
        *,
        max_code: int,
        pressure_threshold: int = 8,
        bucket_low: float = 0.5,
        bucket_high: float = 1.5,
        eps: float = 1e-8,
        rms_ema_beta: float = 0.0,
        pressure_leak_period: int = 0,
        trainable_scale: bool = False,
        compile_update: bool = False,
        matmul_mode: str = "fp32",
        initial_weight: Tensor | None = None,
        fuse_backward_update: bool = False,
        int8_backward: bool = False,
        tile_size: int = 256,
    ) -> None:
        super().__init__()
        # compile_update is accepted for API compatibility: the update is always the fused kernel.
        self.compile_update = compile_update
        if in_features <= 0 or out_features <= 0:
            raise ValueError("in_features and out_features must be positive")
        if max_code not in (1, 2, 3, 4, 5, 6, 7):
            raise ValueError("max_code must be in 1..7 (3..15 states); 7 is the 4-bit packing cap")
        if pressure_threshold <= 0 or pressure_threshold > 127:
            raise ValueError("pressure_threshold must be in [1, 127]")
        if not 0 <= bucket_low < bucket_high:
            raise ValueError("bucket thresholds must satisfy 0 <= low < high")
        if eps <= 0:
            raise ValueError("eps must be positive")
        if matmul_mode not in ("fp32", "bf16", "int8"):
            raise ValueError("matmul_mode must be fp32, bf16, or int8")

        self.in_features = in_features
        self.out_features = out_features
        self.max_code = max_code
        self.pressure_threshold = pressure_threshold
        self.bucket_low = bucket_low
        self.bucket_high = bucket_high
        self.eps = eps
        if not 0.0 <= rms_ema_beta < 1.0:
            raise ValueError("rms_ema_beta must be in [0, 1)")
        self.rms_ema_beta = rms_ema_beta
        if pressure_leak_period < 0:
            raise ValueError("pressure_leak_period must be a non-negative integer")
        self.pressure_leak_period = pressure_leak_period
        self._update_count = 0
        if rms_ema_beta > 0.0:
            self.register_buffer("rms_ema", torch.zeros(out_features))
        self.trainable_scale = trainable_scale
        self.matmul_mode = matmul_mode
        self.fuse_backward_update = fuse_backward_update
        self.int8_backward = int8_backward
        self.tile_size = tile_size

        # Initialisation is the reference's, op for op, so seeded models match (ratchet.py:369-392).
        if initial_weight is None:
            reference = torch.empty(out_features, in_features, dtype=torch.float32)
            nn.init.kaiming_uniform_(reference, a=5**0.5)
        else:
            if initial_weight.shape != (out_features, in_features):
                raise ValueError(
                    f"initial_weight must have shape {(out_features, in_features)}, "
                    f"got {tuple(initial_weight.shape)}"
                )
            reference = initial_weight.detach().to(dtype=torch.float32)
        row_max = reference.abs().amax(dim=1)
        scale = (row_max / max_code).clamp_min(torch.finfo(torch.float32).eps)
        code = torch.round(reference / scale[:, None]).clamp(-max_code, max_code)
        zero_pressure = torch.zeros_like(code, dtype=torch.int8)
        self.register_buffer("packed", pack_code_pressure(code.to(torch.int8), zero_pressure, max_code))
        if trainable_scale:
            self.log_scale = nn.Parameter(scale.log())
        else:
            self.register_buffer("_scale", scale)

        self._effective_weight: Tensor | None = None
        self._pending_weight_gradient: Tensor | None = None
        self._reset_pending_stats()
        # int8 code mirror of `packed` (not a buffer: derived, rebuilt on demand)
        self._code_mirror: Tensor | None = None
        self._code_mirror_key: tuple | None = None
        # None: the output follows the input dtype (the reference's `.to(inputs.dtype)`)
        self.output_dtype: torch.dtype | None = None
        # Stochastic-rounding key of the int8 grad_input quant: (seed, step, layer).  With
        # sr_seed None the seed is drawn from the host RNG per call, as the reference does; a fixed
        # sr_seed keeps the step counter in device memory (graph-capturable, advanced per call).
        self.sr_seed: int | None = None
        self.sr_layer: int = 0
        self._sr_step = 0
        self._sr_step_dev: Tensor | None = None
        # output gradient already quantised by the op that produced it (GradientQuantPlan)
        self._prequant_grad = None
        # data-parallel runtime this layer's gradient goes to (local_ai_training_b200.dist)
        self._dp = None

    # ------------------------------------------------------------------ construction helpers
    @classmethod
    def from_reference(cls, reference: Tensor, *, max_code: int, pressure_threshold: int = 8,
                       bucket_low: float = 0.5, bucket_high: float = 1.5,
                       eps: float = 1e-8) -> DiscreteRatchetLinear:
        if reference.ndim != 2:
            raise ValueError("reference weight must be a matrix")
        return cls(reference.shape[1], reference.shape[0], max_code=max_code,
                   pressure_threshold=pressure_threshold, bucket_low=bucket_low,
                   bucket_high=bucket_high, eps=eps, initial_weight=reference)

    def _reset_pending_stats(self) -> None:
        self._pending_stats_total_weights = 0
        self._pending_counts: Tensor | None = None
        self._pending_stats_rms_sum = 0.0
        # optional int64[5] row of a caller-owned per-step buffer (RatchetGPT hands one to every
        # layer so that one reduction aggregates the whole model); cleared with the stats
        self._stats_slot: Tensor | None = None

    def _next_sr_key(self) -> tuple[int | None, int, int, Tensor | None]:
        if self.sr_seed is None:
            step = self._sr_step
            self._sr_step += 1
            return None, step, self.sr_layer, None
        if self._sr_step_dev is None or self._sr_step_dev.device != self.packed.device:
            self._sr_step_dev = torch.zeros(2, device=self.packed.device, dtype=torch.int32)
        return self.sr_seed, 0, self.sr_layer, self._sr_step_dev

    # ------------------------------------------------------------------ state views
    @property
    def has_pending_gradient(self) -> bool:
        eager_pending = self._effective_weight is not None and self._effective_weight.grad is not None
        return eager_pending or self._pending_weight_gradient is not None

    @property
    def persistent_state_bytes(self) -> int:
        return (self.packed.numel() * self.packed.element_size()
                + self.scale.numel() * self.scale.element_size())

    @property
    def code(self) -> Tensor:
        return unpack_code_pressure(self.packed, self.max_code)[0]

    @property
    def pressure(self) -> Tensor:
        return unpack_code_pressure(self.packed, self.max_code)[1]

    @property
    def scale(self) -> Tensor:
        return self.log_scale.exp() if self.trainable_scale else self._scale

    def effective_weight(self) -> Tensor:
        return self.code.to(dtype=self.scale.dtype) * self.scale[:, None]

    def _refresh_code_mirror(self) -> None:
        """Re-derives the int8 code mirror from `packed` in place, for writers of `packed` that do
        not move its version counter (collectives writing into it)."""
        pk = self.packed
        key = (pk.device, pk.data_ptr(), pk._version)
        if self._code_mirror is None or self._code_mirror.shape != pk.shape or not pk.is_cuda:
            self._code_mirror = None
            self.code_int8()
            return
        rows, cols = pk.shape
        ev = _lib.prof_start(pk)
        _lib.check(_lib.lib().rt_unpack_code_pressure(
            pk.data_ptr(), pk.stride(0), rows, cols, self.max_code, self._code_mirror.data_ptr(),
            self._code_mirror.stride(0), None, 0, _lib.stream_of(pk)))
        if ev is not None:
            _lib.prof_stop(ev, "unpack_codes", pk, 0.0, 2 * rows * cols)
        self._code_mirror_key = key

    def code_int8(self) -> Tensor:
        """The int8 code tensor the GEMMs read, kept in step with `packed`."""
        pk = self.packed
        key = (pk.device, pk.data_ptr(), pk._version)
        if self._code_mirror is None or self._code_mirror_key != key:
            if pk.is_cuda:
                mirror = torch.empty(pk.shape, device=pk.device, dtype=torch.int8)
                rows, cols = pk.shape
                _lib.check(_lib.lib().rt_unpack_code_pressure(
                    pk.data_ptr(), pk.stride(0), rows, cols, self.max_code, mirror.data_ptr(),
                    mirror.stride(0), None, 0, _lib.stream_of(pk)))
            else:
                mirror = unpack_code_pressure(pk, self.max_code)[0]
            self._code_mirror = mirror
            self._code_mirror_key = key
        return self._code_mirror

    # ------------------------------------------------------------------ forward
    def forward(self, inputs: Tensor, *, inputs_int8: Tensor | None = None,
                inputs_scale: Tensor | None = None, residual: Tensor | None = None,
                inputs_dequant: Tensor | None = None) -> Tensor:
        """residual (optional): returns residual + layer(inputs), the add fused into the int8
        GEMM epilogue when residual is fp32.  inputs_dequant (with inputs_int8/inputs_scale):
        bf16(bf16(inputs_int8)·bf16(inputs_scale)) written by the producer, saved for the
        grad_weight GEMM instead of the int8 rows."""
        if self.matmul_mode != "fp32" or self.fuse_backward_update:
            output = _RatchetMatmul.apply(
                inputs, inputs_int8, inputs_scale, self.code_int8(), self.scale, self.matmul_mode,
                self.fuse_backward_update, self.int8_backward, self.tile_size,
                self._capture_weight_gradient, residual,
                inputs_dequant if self.matmul_mode == "int8" else None,
            )
            if (self.matmul_mode == "int8" and self.int8_backward and self.fuse_backward_update
                    and inputs_int8 is not None and inputs_scale is not None
                    and output.requires_grad):
                # backward will stochastic-round this output's gradient: let the op that
                # consumes the output quantise the gradient where it produces it
                result_dtype = getattr(self, "output_dtype", None) or inputs.dtype
                output._ratchet_grad_plan = GradientQuantPlan(
                    self, residual is not None and result_dtype == torch.bfloat16)
            return output
        _require_cuda(inputs, "the ratchet layer")
        effective = self.effective_weight().to(dtype=inputs.dtype)
        if self.training and torch.is_grad_enabled():
            if self.trainable_scale:
                effective.retain_grad()
            else:
                effective = effective.detach().requires_grad_(True)
            self._effective_weight = effective
        output = F.linear(inputs, effective)
        return output if residual is None else residual + output

    # ------------------------------------------------------------------ update
    def _run_update(self, gradient: Tensor, row_start: int, row_end: int, *, normalize: bool,
                    round_bf16: bool, counts: Tensor, want_grad_scale: bool = False,
                    row_rms: Tensor | None = None, rms_sum: Tensor | None = None) -> Tensor | None:
        """One launch of the update kernel over rows [row_start, row_end)."""
        pk = self.packed
        _require_cuda(pk, "the ratchet update")
        mirror = self.code_int8()
        rows = row_end - row_start
        if gradient.dtype not in (torch.float32, torch.bfloat16):
            gradient = gradient.float()
        if gradient.device != pk.device:
            gradient = gradient.to(pk.device)
        if gradient.stride(-1) != 1:
            gradient = gradient.contiguous()
        ema = None
        if self.rms_ema_beta > 0.0:
            ema = self.rms_ema
            if not ema.is_cuda:
                raise RuntimeError("rms_ema must live on the layer's CUDA device")
        grad_scale = torch.empty(rows, device=pk.device, dtype=torch.float32) if want_grad_scale else None
        pk_rows = pk[row_start:row_end]
        mirror_rows = mirror[row_start:row_end]
        ev = _lib.prof_start(pk)
        _lib.check(_lib.lib().rt_ratchet_update(
            gradient.data_ptr(), _lib.dtype_code(gradient), int(round_bf16), gradient.stride(0),
            rows, self.in_features, pk_rows.data_ptr(), pk.stride(0), mirror_rows.data_ptr(),
            mirror.stride(0), int(normalize),
            None if ema is None else ema[row_start:row_end].data_ptr(), float(self.rms_ema_beta),
            self.max_code, self.pressure_threshold, float(self.bucket_low),
            float(self.bucket_high), float(self.eps), counts.data_ptr(),
            _lib.ptr(row_rms), _lib.ptr(rms_sum), _lib.ptr(grad_scale), _lib.stream_of(pk)))
        if ev is not None:
            _lib.prof_stop(ev, "ratchet_update", pk, 0.0,
                           rows * self.in_features * (gradient.element_size() + 3) + 4 * rows)
        return grad_scale

    def _pending_stat_slots(self, device) -> None:
        if self._pending_counts is None:
            # one buffer for the four move counters and the rms sum (bit pattern of a float)
            self._pending_buf = (self._stats_slot if self._stats_slot is not None else
                                 torch.zeros(5, device=device, dtype=torch.int64))
            self._pending_counts = self._pending_buf[:4]
            self._pending_rms = self._pending_buf[4:].view(torch.float32)[:1]

    def _grad_weight_update(self, grad_bf16: Tensor, inputs_bf16: Tensor,
                            want_grad_scale: bool) -> tuple[bool, Tensor | None]:
        """The fused update of grad_W = grad_bf16ᵀ·inputs_bf16 (ratchet.py:148-163 then
        _capture_weight_gradient) without storing grad_W: one GEMM writing split-K partial tiles
        and the update reading them (rt_grad_weight_ratchet_update).  Returns (False, None) when
        the operands' layout does not allow it (the caller then takes the two-step path)."""
        pk = self.packed
        mt, out_features = grad_bf16.shape
        if (not pk.is_cuda or grad_bf16.dtype != torch.bfloat16
                or inputs_bf16.dtype != torch.bfloat16 or inputs_bf16.shape[0] != mt
                or out_features != self.out_features or inputs_bf16.shape[1] != self.in_features
                or self.in_features % 8 != 0 or mt == 0):
            return False, None
        for t in (grad_bf16, inputs_bf16):
            if t.stride(1) != 1 or (t.stride(0) * 2) % 16 != 0 or t.data_ptr() % 16 != 0:
                return False, None
        self._pending_stat_slots(pk.device)
        mirror = self.code_int8()
        ema = self.rms_ema if self.rms_ema_beta > 0.0 else None
        grad_scale = (torch.empty(out_features, device=pk.device, dtype=torch.float32)
                      if want_grad_scale else None)
        need = _lib.lib().rt_grad_weight_update_workspace_bytes(mt, out_features, self.in_features)
        ws = _lib.workspace(pk.device, need)
        ev = _lib.prof_start(pk)
        _lib.check(_lib.lib().rt_grad_weight_ratchet_update(
            grad_bf16.data_ptr(), grad_bf16.stride(0), inputs_bf16.data_ptr(),
            inputs_bf16.stride(0), mt, out_features, self.in_features, _lib.ptr(ws), need,
            pk.data_ptr(), pk.stride(0), mirror.data_ptr(), mirror.stride(0), _lib.ptr(ema),
            float(self.rms_ema_beta), self.max_code, self.pressure_threshold,
            float(self.bucket_low), float(self.bucket_high), float(self.eps),
            self._pending_counts.data_ptr(), None, self._pending_rms.data_ptr(),
            _lib.ptr(grad_scale), _lib.stream_of(pk)))
        if ev is not None:
            n, k = out_features, self.in_features
            _lib.prof_stop(ev, "gemm_gradw_update", pk, 2.0 * mt * n * k,
                           2 * mt * (n + k) + 3 * n * k + 4 * n)
        self._pending_stats_total_weights += out_features * self.in_features
        self._pending_stats_rms_sum = self._pending_rms[0]
        return True, grad_scale

    def _capture_weight_gradient(self, gradient: Tensor, tile_start: int | None,
                                 tile_end: int | None, *, round_bf16: bool = False,
                                 want_grad_scale: bool = False) -> Tensor | None:
        if not self.fuse_backward_update:
            if self._pending_weight_gradient is not None:
                raise RuntimeError(
                    "ratchet layer has multiple pending effective-weight gradients "
                    "(missing ratchet_update or unsupported weight sharing)"
                )
            self._pending_weight_gradient = gradient
            return None
        assert tile_start is not None and tile_end is not None
        if gradient.shape != (tile_end - tile_start, self.in_features):
            raise ValueError("fused tile gradient shape mismatch")
        self._pending_stat_slots(gradient.device)
        grad_scale = self._run_update(gradient, tile_start, tile_end, normalize=True,
                                      round_bf16=round_bf16, counts=self._pending_counts,
                                      want_grad_scale=want_grad_scale, rms_sum=self._pending_rms)
        self._pending_stats_total_weights += (tile_end - tile_start) * self.in_features
        self._pending_stats_rms_sum = self._pending_rms[0]
        return grad_scale

    @torch.no_grad()
    def _normalize(self, gradient: Tensor, row_start: int, row_end: int) -> Tensor:
        """Row-RMS normalisation (ratchet.py:539-556) as torch ops, for inspection.

        The update kernel normalises internally with the same formula; this helper also advances
        rms_ema like the reference does.
        """
        grad = gradient.float()
        ms = grad.square().mean(dim=1, keepdim=True)
        if self.rms_ema_beta > 0.0:
            ema = self.rms_ema[row_start:row_end].unsqueeze(1)
            fired = ms > 0
            updated_ema = torch.where(ema == 0, ms, self.rms_ema_beta * ema + (1.0 - self.rms_ema_beta) * ms)
            ema = torch.where(fired, updated_ema, ema)
            self.rms_ema[row_start:row_end] = ema.squeeze(1)
            rms = ema.sqrt()
        else:
            rms = ms.sqrt()
        return grad / (rms + self.eps)

    @torch.no_grad()
    def apply_weight_gradient(self, gradient: Tensor, *, validate: bool = True) -> RatchetUpdateStats:
        if tuple(gradient.shape) != (self.out_features, self.in_features):
            raise ValueError(
                f"gradient must have shape {(self.out_features, self.in_features)}, "
                f"got {tuple(gradient.shape)}"
            )
        _require_cuda(self.packed, "the ratchet update")
        if validate and not torch.isfinite(gradient).all():
            raise FloatingPointError("ratchet gradient contains NaN or Inf")
        row_rms = torch.empty(self.out_features, device=self.packed.device, dtype=torch.float32)
        counts = torch.zeros(4, device=self.packed.device, dtype=torch.int64)
        self._run_update(gradient, 0, self.out_features, normalize=True, round_bf16=False,
                         counts=counts, row_rms=row_rms)
        if validate:
            self._validate_state()
        return RatchetUpdateStats(
            total_weights=self.out_features * self.in_features,
            positive_moves=counts[0], negative_moves=counts[1],
            blocked_positive_moves=counts[2], blocked_negative_moves=counts[3],
            gradient_rms_mean=row_rms.mean(),
        )

    @torch.no_grad()
    def apply_normalized_gradient(self, normalized: Tensor, *, validate: bool = True) -> RatchetUpdateStats:
        if tuple(normalized.shape) != (self.out_features, self.in_features):
            raise ValueError(
                f"normalized gradient must have shape {(self.out_features, self.in_features)}, "
                f"got {tuple(normalized.shape)}"
            )
        _require_cuda(self.packed, "the ratchet update")
        counts = torch.zeros(4, device=self.packed.device, dtype=torch.int64)
        self._run_update(normalized, 0, self.out_features, normalize=False, round_bf16=False,
                         counts=counts)
        if validate:
            self._validate_state()
        return RatchetUpdateStats(
            total_weights=self.out_features * self.in_features,
            positive_moves=counts[0], negative_moves=counts[1],
            blocked_positive_moves=counts[2], blocked_negative_moves=counts[3],
            gradient_rms_mean=0.0,
        )

    @torch.no_grad()
    def _maybe_leak_pressure(self) -> None:
        if self.pressure_leak_period <= 0:
            return
        self._update_count += 1
        if self._update_count % self.pressure_leak_period != 0:
            return
        pk = self.packed
        _require_cuda(pk, "the pressure leak")
        rows, cols = pk.shape
        _lib.check(_lib.lib().rt_ratchet_leak(pk.data_ptr(), pk.stride(0), rows, cols,
                                              self.max_code, _lib.stream_of(pk)))

    def ratchet_update(self, *, validate: bool = True) -> RatchetUpdateStats:
        if self.fuse_backward_update:
            if validate:
                self._validate_state()
            counts = self._pending_counts
            zero = 0
            stats = RatchetUpdateStats(
                total_weights=self._pending_stats_total_weights,
                positive_moves=counts[0] if counts is not None else zero,
                negative_moves=counts[1] if counts is not None else zero,
                blocked_positive_moves=counts[2] if counts is not None else zero,
                blocked_negative_moves=counts[3] if counts is not None else zero,
                gradient_rms_mean=self._pending_stats_rms_sum / max(1, self.out_features),
            )
            self._reset_pending_stats()
            self._maybe_leak_pressure()
            return stats.materialize() if validate else stats
        elif self.matmul_mode != "fp32":
            if self._pending_weight_gradient is None:
                raise RuntimeError("ratchet layer has no pending effective-weight gradient")
            try:
                stats = self.apply_weight_gradient(self._pending_weight_gradient, validate=validate)
            finally:
                self._pending_weight_gradient = None
        else:
            if self._effective_weight is None or self._effective_weight.grad is None:
                raise RuntimeError("ratchet layer has no pending effective-weight gradient")
            try:
                stats = self.apply_weight_gradient(self._effective_weight.grad, validate=validate)
            finally:
                self._effective_weight = None
        self._maybe_leak_pressure()
        return stats.materialize() if validate else stats

    def discard_pending_gradient(self) -> None:
        if self._pending_weight_gradient is not None:
            self._pending_weight_gradient = None
        self._effective_weight = None

    def _validate_state(self) -> None:
        """ratchet.py:672-679 through the validation kernel and the device status word; also
        raises FloatingPointError for non-finite gradients met by earlier fused updates."""
        pk = self.packed
        if not pk.is_cuda:
            code, pressure = unpack_code_pressure(pk, self.max_code)
            if code.min().item() < -self.max_code or code.max().item() > self.max_code:
                raise RuntimeError("ratchet code escaped its allowed range")
            if pressure.abs().max().item() > 7:
                raise RuntimeError("ratchet pressure escaped the packed nibble range")
            if not torch.isfinite(self.scale).all() or torch.any(self.scale <= 0):
                raise RuntimeError("ratchet row scales must remain positive and finite")
            return
        rows, cols = pk.shape
        scale = self.scale.detach().float().contiguous()
        _lib.check(_lib.lib().rt_ratchet_validate(pk.data_ptr(), pk.stride(0), rows, cols,
                                                  self.max_code, scale.data_ptr(),
                                                  _lib.stream_of(pk)))
        status = _lib.device_status(pk.device, clear=True)
        if status & _lib.STATUS_NONFINITE_GRADIENT:
            raise FloatingPointError("ratchet gradient contains NaN or Inf")
        if status & _lib.STATUS_CODE_RANGE:
            raise RuntimeError("ratchet code escaped its allowed range")
        if status & _lib.STATUS_PRESSURE_RANGE:
            raise RuntimeError("ratchet pressure escaped the packed nibble range")
        if status & _lib.STATUS_SCALE_INVALID:
            raise RuntimeError("ratchet row scales must remain positive and finite")
        if status & _lib.STATUS_WAIT_TIMEOUT:
            raise RuntimeError("a CUDA pipeline wait timed out (device status word)")

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"states={2 * self.max_code + 1}, threshold={self.pressure_threshold}, bias=False")


class _EmbeddingLookup(torch.autograd.Function):
    """Forward: rows of fp32 `code * scale` gathered straight from `packed` (the
    reference's F.embedding over the materialised effective weight, ratchet.py:740-747).
    Backward: the output gradient and the token ids become the layer's pending row-sparse
    weight gradient (no [rows, dim] gradient tensor)."""

    @staticmethod
    def forward(ctx, token_ids, anchor, layer):
        flat = token_ids.reshape(-1).to(torch.int64).contiguous()
        pk = layer.packed
        scale = layer.scale.detach().float().contiguous()
        out = torch.empty((flat.numel(), layer.embedding_dim), device=pk.device,
                          dtype=torch.float32)
        ev = _lib.prof_start(pk)
        _lib.check(_lib.lib().rt_embedding_forward(
            pk.data_ptr(), pk.stride(0), scale.data_ptr(), layer.max_code, flat.data_ptr(),
            flat.numel(), layer.num_embeddings, layer.embedding_dim, out.data_ptr(),
            out.stride(0), _lib.stream_of(pk)))
        if ev is not None:
            _lib.prof_stop(ev, "embedding", pk, 0.0, flat.numel() * layer.embedding_dim * 5)
        ctx.layer = layer
        ctx.save_for_backward(flat)
        return out.reshape(*token_ids.shape, layer.embedding_dim)

    @staticmethod
    def backward(ctx, grad):
        (flat,) = ctx.saved_tensors
        layer = ctx.layer
        g = grad.reshape(-1, layer.embedding_dim)
        if g.dtype != torch.float32:
            g = g.float()
        layer._sparse_gradient = (flat, g.contiguous())
        return None, None, None


class RatchetEmbedding(DiscreteRatchetLinear):
    """Master-weight-free token embedding (ratchet.py:688-749): rows are tokens.

    On CUDA the forward gathers `code * scale` rows straight from `packed` (no [rows, dim]
    effective weight), backward keeps the output gradient and the token ids, and
    `ratchet_update` updates only the rows of the tokens seen (rt_embedding_ratchet_update): the
    other rows have a zero gradient in the reference, which leaves them unchanged.  A trainable
    scale keeps the reference's dense effective-weight path (its gradient reaches log_scale
    through autograd)."""

    def __init__(self, num_embeddings: int, embedding_dim: int, *, max_code: int,
                 pressure_threshold: int = 8, bucket_low: float = 0.5, bucket_high: float = 1.5,
                 eps: float = 1e-8, rms_ema_beta: float = 0.0, pressure_leak_period: int = 0,
                 trainable_scale: bool = False, compile_update: bool = False,
                 initial_weight: Tensor | None = None) -> None:
        if initial_weight is None:
            initial_weight = torch.randn(num_embeddings, embedding_dim)
        super().__init__(embedding_dim, num_embeddings, max_code=max_code,
                         pressure_threshold=pressure_threshold, bucket_low=bucket_low,
                         bucket_high=bucket_high, eps=eps, rms_ema_beta=rms_ema_beta,
                         pressure_leak_period=pressure_leak_period,
                         trainable_scale=trainable_scale, compile_update=compile_update,
                         matmul_mode="fp32", initial_weight=initial_weight)
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim

    def forward(self, token_ids: Tensor) -> Tensor:  # type: ignore[override]
        _require_cuda(self.packed, "the ratchet embedding")
        training = self.training and torch.is_grad_enabled()
        if not self.trainable_scale:
            if training:
                # the gradient of this forward replaces any earlier one (the reference's fresh
                # effective-weight leaf per forward)
                self._sparse_gradient = None
                anchor = torch.empty(0, device=self.packed.device, requires_grad=True)
                return _EmbeddingLookup.apply(token_ids.to(self.packed.device), anchor, self)
            with torch.no_grad():
                return _EmbeddingLookup.apply(token_ids.to(self.packed.device), None, self)
        effective = self.effective_weight()
        if training:
            effective = effective.detach().requires_grad_(True)
            self._effective_weight = effective
        return F.embedding(token_ids, effective)

    @property
    def has_pending_gradient(self) -> bool:
        return getattr(self, "_sparse_gradient", None) is not None or super().has_pending_gradient

    def discard_pending_gradient(self) -> None:
        self._sparse_gradient = None
        super().discard_pending_gradient()

    @torch.no_grad()
    def ratchet_update(self, *, validate: bool = True) -> RatchetUpdateStats:
        pending = getattr(self, "_sparse_gradient", None)
        if pending is None:
            return super().ratchet_update(validate=validate)
        self._sparse_gradient = None
        tokens, grad = pending
        if validate and not torch.isfinite(grad).all():
            raise FloatingPointError("ratchet gradient contains NaN or Inf")
        pk = self.packed
        sorted_tokens, order = torch.sort(tokens, stable=True)
        mirror = self.code_int8()
        counts = torch.zeros(4, device=pk.device, dtype=torch.int64)
        rms_sum = torch.zeros(1, device=pk.device, dtype=torch.float32)
        n, dim = grad.shape
        need = _lib.lib().rt_embedding_update_workspace_bytes(n, dim)
        work = _lib.workspace(pk.device, need)
        ema = self.rms_ema if self.rms_ema_beta > 0.0 else None
        ev = _lib.prof_start(pk)
        _lib.check(_lib.lib().rt_embedding_ratchet_update(
            grad.data_ptr(), grad.stride(0), sorted_tokens.data_ptr(), order.data_ptr(), n,
            self.num_embeddings, dim, _lib.ptr(work), need, pk.data_ptr(), pk.stride(0),
            mirror.data_ptr(), mirror.stride(0), _lib.ptr(ema), float(self.rms_ema_beta),
            self.max_code, self.pressure_threshold, float(self.bucket_low),
            float(self.bucket_high), float(self.eps), counts.data_ptr(), rms_sum.data_ptr(),
            _lib.stream_of(pk)))
        if ev is not None:
            _lib.prof_stop(ev, "embedding_update", pk, 0.0, n * dim * 4 * 2 + n * dim * 2)
        if validate:
            self._validate_state()
        stats = RatchetUpdateStats(
            total_weights=self.out_features * self.in_features,
            positive_moves=counts[0], negative_moves=counts[1],
            blocked_positive_moves=counts[2], blocked_negative_moves=counts[3],
            gradient_rms_mean=rms_sum[0] / max(1, self.out_features))
        self._maybe_leak_pressure()
        return stats.materialize() if validate else stats

    def extra_repr(self) -> str:
        return (f"num_embeddings={self.num_embeddings}, embedding_dim={self.embedding_dim}, "
                f"states={2 * self.max_code + 1}, threshold={self.pressure_threshold}")


@dataclass(frozen=True)
class PersistentFootprint:
    """Static byte accounting for the trainable matrices, ratchet vs FP32+AdamW."""

    ratchet_weights: int
    ratchet_matrix_bytes: int
    fp32_master_bytes: int
    fp32_optimizer_bytes: int

    @property
    def fp32_matrix_bytes(self) -> int:
        return self.fp32_master_bytes + self.fp32_optimizer_bytes

    @property
    def reduction_ratio(self) -> float:
        return self.fp32_matrix_bytes / max(self.ratchet_matrix_bytes, 1)


def compare_persistent_footprint(model: nn.Module) -> PersistentFootprint:
    weights = 0
    ratchet_bytes = 0
    for module in model.modules():
        if isinstance(module, DiscreteRatchetLinear):
            weights += module.packed.numel()
            ratchet_bytes += module.persistent_state_bytes
    return PersistentFootprint(ratchet_weights=weights, ratchet_matrix_bytes=ratchet_bytes,
                               fp32_master_bytes=weights * 4, fp32_optimizer_bytes=weights * 8)


def audit_no_master_weights(model: nn.Module, *, raise_on_violation: bool = False) -> RatchetAuditReport:
    violations: list[str] = []
    ratchet_layers = 0
    ratchet_weights = 0
    ratchet_state_bytes = 0
    for module_name, module in model.named_modules():
        if not isinstance(module, DiscreteRatchetLinear):
            continue
        ratchet_layers += 1
        ratchet_weights += module.packed.numel()
        ratchet_state_bytes += module.persistent_state_bytes
        prefix = module_name or "<root>"
        for parameter_name, parameter in module.named_parameters(recurse=False):
            if parameter.is_floating_point() and parameter.ndim >= 2:
                violations.append(f"{prefix}.{parameter_name}: floating matrix parameter")
        if module.packed.dtype != torch.uint8:
            violations.append(f"{prefix}.packed: expected uint8, got {module.packed.dtype}")
        if module.scale.ndim != 1 or module.scale.shape[0] != module.out_features:
            violations.append(f"{prefix}.scale: expected one scale per output row")
    support_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    report = RatchetAuditReport(ratchet_layers=ratchet_layers, ratchet_weights=ratchet_weights,
                                ratchet_state_bytes=ratchet_state_bytes,
                                support_parameter_bytes=support_bytes, violations=tuple(violations))
    if raise_on_violation and violations:
        raise RuntimeError("ratchet master-weight audit failed: " + "; ".join(violations))
    return report
