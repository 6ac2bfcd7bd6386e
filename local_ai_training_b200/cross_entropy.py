"""lm_head + token cross-entropy as one autograd step (model.py:244-249 of the reference:
`logits = lm_head(final_norm(h)); loss = F.cross_entropy(logits.flatten(0, 1), targets.flatten())`).

Forward: the lm_head's self-quantising int8 matmul (ratchet.py:46-65) writes the logits, then one
kernel pass per row gives max, log-sum-exp and the row loss (the logits are read once instead of
log_softmax's read + write and nll's read).  Backward: one kernel pass writes the bf16 logit
gradient the lm_head grad GEMMs consume (the reference materialises an fp32 gradient, then casts
it to bf16, ratchet.py:139-141, 161); grad_input and grad_W then follow the layer's own backward
(bf16 grad_input against bf16(code·scale), grad_W delivered to the fused update or the
data-parallel reduce-scatter).  Values: the loss is the mean over targets != ignore_index, the
gradient is exp(log p)·w − [j = t]·w with w = grad_loss / count, as torch computes them; the sum
of exponentials runs in a different order than torch's, so results agree to fp32 rounding.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from .int8_matmul import _scaled_int8_mm_into, dequant_rows_bf16, matmul_bf16, quantize_rows
from .int8_matmul import grad_weight_bf16
from .ratchet import (DiscreteRatchetLinear, _code_bound, _deliver_weight_gradient,
                      _require_cuda, _sink_weight_gradient)

IGNORE_INDEX = -100


def cross_entropy_rows(logits: Tensor, targets: Tensor, ignore_index: int = IGNORE_INDEX, *,
                       out: tuple[Tensor, Tensor, Tensor] | None = None):
    """Per-row (max, logsum, loss) of 2-D logits [rows, classes] (fp32 or bf16), written into
    `out` (three contiguous fp32 [rows] tensors) when given."""
    _require_cuda(logits, "cross_entropy_rows")
    rows, cols = logits.shape
    targets = targets.reshape(-1).to(torch.int64).contiguous()
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    if out is None:
        row_max = torch.empty(rows, device=logits.device, dtype=torch.float32)
        row_logsum = torch.empty_like(row_max)
        row_loss = torch.empty_like(row_max)
    else:
        row_max, row_logsum, row_loss = out
        for t in out:
            if t.shape != (rows,) or t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError("cross_entropy_rows out must be three contiguous float32 [rows]")
    ev = _lib.prof_start(logits)
    _lib.check(_lib.lib().rt_cross_entropy_fwd(
        logits.data_ptr(), _lib.dtype_code(logits), logits.stride(0), rows, cols,
        targets.data_ptr(), int(ignore_index), row_max.data_ptr(), row_logsum.data_ptr(),
        row_loss.data_ptr(), _lib.stream_of(logits)))
    if ev is not None:
        _lib.prof_stop(ev, "cross_entropy", logits, 0.0, rows * cols * logits.element_size())
    return row_max, row_logsum, row_loss


def cross_entropy_grad_bf16(logits: Tensor, targets: Tensor, row_max: Tensor, row_logsum: Tensor,
                            grad_loss: Tensor, count: Tensor, extra: Tensor | None = None,
                            ignore_index: int = IGNORE_INDEX) -> Tensor:
    """bf16 gradient of mean cross-entropy w.r.t. the logits (plus an optional fp32 gradient)."""
    rows, cols = logits.shape
    out = torch.empty((rows, cols), device=logits.device, dtype=torch.bfloat16)
    if extra is not None:
        extra = extra.reshape(rows, cols).float()
        if extra.stride(1) != 1:
            extra = extra.contiguous()
    grad_loss = grad_loss.reshape(1).float().contiguous()
    ev = _lib.prof_start(logits)
    _lib.check(_lib.lib().rt_cross_entropy_bwd(
        logits.data_ptr(), _lib.dtype_code(logits), logits.stride(0), rows, cols,
        targets.data_ptr(), int(ignore_index), row_max.data_ptr(), row_logsum.data_ptr(),
        grad_loss.data_ptr(), count.data_ptr(), _lib.ptr(extra),
        0 if extra is None else extra.stride(0), out.data_ptr(), out.stride(0),
        _lib.stream_of(logits)))
    if ev is not None:
        _lib.prof_stop(ev, "cross_entropy", logits, 0.0,
                       rows * cols * (logits.element_size() + 2 + (4 if extra is not None else 0)))
    return out


class _LMHeadCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, inputs, targets, code, scale, gradient_sink, ignore_index):
        ctx.set_materialize_grads(False)
        input_shape = inputs.shape
        flat_inputs = inputs.flatten(0, -2)
        out_features = code.shape[0]
        q, s = quantize_rows(flat_inputs)
        logits = torch.empty((q.shape[0], out_features), device=q.device,
                             dtype=inputs.dtype if inputs.dtype in (torch.float32, torch.bfloat16)
                             else torch.float32)
        _scaled_int8_mm_into(q, code.t(), s, scale.float().contiguous(), logits,
                             rhs_abs_max=_code_bound(gradient_sink))
        flat_targets = targets.reshape(-1).to(torch.int64).contiguous()
        row_max, row_logsum, row_loss = cross_entropy_rows(logits, flat_targets, ignore_index)
        count = (flat_targets != ignore_index).sum().float().reshape(1)
        loss = row_loss.sum() / count[0]
        ctx.save_for_backward(flat_inputs, code, scale, logits, flat_targets, row_max, row_logsum,
                              count)
        ctx.input_shape = input_shape
        ctx.input_dtype = inputs.dtype
        ctx.gradient_sink = gradient_sink
        ctx.ignore_index = ignore_index
        ctx.fuse_backward_update = getattr(gradient_sink.__self__, "fuse_backward_update", True)
        return logits.reshape(*input_shape[:-1], out_features), loss

    @staticmethod
    def backward(ctx, grad_logits, grad_loss):
        (flat_inputs, code, scale, logits, flat_targets, row_max, row_logsum,
         count) = ctx.saved_tensors
        if grad_loss is None:
            grad_loss = torch.zeros((), device=logits.device)
        extra = None if grad_logits is None else grad_logits.reshape(logits.shape)
        grad_bf16 = cross_entropy_grad_bf16(logits, flat_targets, row_max, row_logsum, grad_loss,
                                            count, extra, ctx.ignore_index)
        # bf16 grad_input against bf16(code)·bf16(scale) (ratchet.py:135-141) on the tcgen05 GEMM
        effective = dequant_rows_bf16(code, scale.float().contiguous())
        grad_input = matmul_bf16(grad_bf16, effective)
        grad_scale = _deliver_weight_gradient(
            ctx.gradient_sink, "int8", ctx.fuse_backward_update, grad_bf16,
            flat_inputs.to(torch.bfloat16), None, flat_inputs, code, bool(ctx.needs_input_grad[3]))
        return (grad_input.reshape(ctx.input_shape).to(ctx.input_dtype), None, None, grad_scale,
                None, None)


class _GradWeightChunks:
    """grad_W = sum over row chunks c of dl_c^T x_c, delivered as the one GEMM over all rows would
    deliver it: to a data-parallel GradTarget (fp32 accumulator, bf16 total, or bf16 after an fp32
    addend), or, with no target, returned in fp32.  The chunks' products add in fp32; only the
    total is rounded (the reference rounds the whole GEMM's output once)."""

    def __init__(self, target):
        self.target = target
        self.acc: Tensor | None = None
        self.first = True

    def add(self, dl: Tensor, x: Tensor, last: bool) -> None:
        t = self.target
        if t is None or (t.addend is None and t.out.dtype != torch.float32 and not last):
            # no target, or a bf16 single-micro-batch target before the last chunk: own fp32 sum
            if self.acc is None:
                self.acc = grad_weight_bf16(dl, x)
            else:
                grad_weight_bf16(dl, x, out=self.acc, accumulate=True)
        elif t.out.dtype == torch.float32:  # an earlier micro-batch's fp32 accumulator
            grad_weight_bf16(dl, x, out=t.out, accumulate=t.accumulate or not self.first)
        elif not last:  # the last micro-batch: chunks add into its addend, the last one rounds
            grad_weight_bf16(dl, x, out=t.addend, accumulate=True)
        else:
            grad_weight_bf16(dl, x, out=t.out, addend=t.addend if t.addend is not None else self.acc)
        self.first = False


class _LMHeadCrossEntropyChunked(torch.autograd.Function):
    """The same loss and gradients as _LMHeadCrossEntropy without a [tokens, vocab] tensor: the
    forward runs the lm_head GEMM and the row statistics over blocks of `chunk_rows` tokens into
    one reused logits block, and backward recomputes each block's logits (the int8 GEMM again),
    forms its bf16 logit gradient and runs that block's grad_input rows and its share of grad_W
    before the next.  Per row the loss, the logit gradient and grad_input are those of the
    unchunked path; grad_W sums the blocks' products in fp32 before its one rounding.  The block
    is bf16: the GEMM rounds every logit to bf16 in either output dtype (the reference's bf16
    GEMM output), so half the bytes hold the same values."""

    @staticmethod
    def forward(ctx, inputs, targets, code, scale, gradient_sink, ignore_index, chunk_rows):
        input_shape = inputs.shape
        flat_inputs = inputs.flatten(0, -2)
        rows = flat_inputs.shape[0]
        vocab = code.shape[0]
        q, s = quantize_rows(flat_inputs)
        scale_f = scale.float().contiguous()
        block = torch.empty((min(chunk_rows, rows), vocab), device=q.device, dtype=torch.bfloat16)
        stats = torch.empty((3, rows), device=q.device, dtype=torch.float32)
        row_max, row_logsum, row_loss = stats[0], stats[1], stats[2]
        flat_targets = targets.reshape(-1).to(torch.int64).contiguous()
        bound = _code_bound(gradient_sink)
        for r0 in range(0, rows, chunk_rows):
            r1 = min(rows, r0 + chunk_rows)
            logits = block[: r1 - r0]
            _scaled_int8_mm_into(q[r0:r1], code.t(), s[r0:r1], scale_f, logits,
                                 rhs_abs_max=bound)
            cross_entropy_rows(logits, flat_targets[r0:r1], ignore_index,
                               out=(row_max[r0:r1], row_logsum[r0:r1], row_loss[r0:r1]))
        count = (flat_targets != ignore_index).sum().float().reshape(1)
        loss = row_loss.sum() / count[0]
        ctx.save_for_backward(flat_inputs, q, s, code, scale, flat_targets, row_max, row_logsum,
                              count)
        ctx.input_shape = input_shape
        ctx.input_dtype = inputs.dtype
        ctx.gradient_sink = gradient_sink
        ctx.ignore_index = ignore_index
        ctx.chunk_rows = chunk_rows
        ctx.fuse_backward_update = getattr(gradient_sink.__self__, "fuse_backward_update", True)
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        flat_inputs, q, s, code, scale, flat_targets, row_max, row_logsum, count = ctx.saved_tensors
        if grad_loss is None:
            grad_loss = torch.zeros((), device=q.device)
        rows, width = flat_inputs.shape
        vocab = code.shape[0]
        chunk_rows = ctx.chunk_rows
        scale_f = scale.float().contiguous()
        effective = dequant_rows_bf16(code, scale_f)
        inputs_bf16 = flat_inputs.to(torch.bfloat16)
        grad_input = torch.empty((rows, width), device=q.device, dtype=torch.bfloat16)
        block = torch.empty((min(chunk_rows, rows), vocab), device=q.device, dtype=torch.bfloat16)
        sink = ctx.gradient_sink
        layer = getattr(sink, "__self__", None)
        dp = getattr(layer, "_dp", None)
        target = dp.grad_target(layer) if dp is not None else None
        chunks = _GradWeightChunks(target)
        bound = _code_bound(sink)
        for r0 in range(0, rows, chunk_rows):
            r1 = min(rows, r0 + chunk_rows)
            logits = block[: r1 - r0]
            _scaled_int8_mm_into(q[r0:r1], code.t(), s[r0:r1], scale_f, logits,
                                 rhs_abs_max=bound)
            dl = cross_entropy_grad_bf16(logits, flat_targets[r0:r1], row_max[r0:r1],
                                         row_logsum[r0:r1], grad_loss, count, None,
                                         ctx.ignore_index)
            matmul_bf16(dl, effective, out=grad_input[r0:r1])
            chunks.add(dl, inputs_bf16[r0:r1], last=r1 == rows)
        want_scale = bool(ctx.needs_input_grad[3])
        if dp is not None:
            grad_scale = None
            if want_scale:
                grad_scale = ((target.out.float() * code.float()).sum(dim=1) if target.last else
                              torch.zeros(vocab, device=code.device, dtype=torch.float32))
            dp.grad_ready(layer)
        else:
            grad_scale = _sink_weight_gradient(sink, ctx.fuse_backward_update, chunks.acc, True,
                                               code, want_scale)
        return (grad_input.reshape(ctx.input_shape).to(ctx.input_dtype), None, None, grad_scale,
                None, None, None)


def fused_lm_head_applies(layer, inputs: Tensor) -> bool:
    """The fused path covers a self-quantising int8 ratchet lm_head on CUDA inputs."""
    return (isinstance(layer, DiscreteRatchetLinear) and layer.matmul_mode == "int8"
            and inputs.is_cuda and layer.packed.is_cuda)


def lm_head_cross_entropy(layer: DiscreteRatchetLinear, inputs: Tensor, targets: Tensor,
                          ignore_index: int = IGNORE_INDEX,
                          chunk_rows: int = 0) -> tuple[Tensor | None, Tensor]:
    """(logits, mean cross-entropy) of `layer(inputs)` against `targets` in one autograd step.

    chunk_rows > 0: the tokens are processed in blocks of that many rows and no logits are
    returned (None): neither the [tokens, vocab] logits nor their gradient is ever stored."""
    if chunk_rows and chunk_rows > 0:
        loss = _LMHeadCrossEntropyChunked.apply(inputs, targets, layer.code_int8(), layer.scale,
                                                layer._capture_weight_gradient, ignore_index,
                                                int(chunk_rows))
        return None, loss
    return _LMHeadCrossEntropy.apply(inputs, targets, layer.code_int8(), layer.scale,
                                     layer._capture_weight_gradient, ignore_index)
