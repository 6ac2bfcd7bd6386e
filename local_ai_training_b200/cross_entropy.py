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
from .ratchet import DiscreteRatchetLinear, _code_bound, _deliver_weight_gradient, _require_cuda

IGNORE_INDEX = -100


def cross_entropy_rows(logits: Tensor, targets: Tensor, ignore_index: int = IGNORE_INDEX):
    """Per-row (max, logsum, loss) of 2-D logits [rows, classes] (fp32 or bf16)."""
    _require_cuda(logits, "cross_entropy_rows")
    rows, cols = logits.shape
    targets = targets.reshape(-1).to(torch.int64).contiguous()
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    row_max = torch.empty(rows, device=logits.device, dtype=torch.float32)
    row_logsum = torch.empty_like(row_max)
    row_loss = torch.empty_like(row_max)
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


def fused_lm_head_applies(layer, inputs: Tensor) -> bool:
    """The fused path covers a self-quantising int8 ratchet lm_head on CUDA inputs."""
    return (isinstance(layer, DiscreteRatchetLinear) and layer.matmul_mode == "int8"
            and inputs.is_cuda and layer.packed.is_cuda)


def lm_head_cross_entropy(layer: DiscreteRatchetLinear, inputs: Tensor, targets: Tensor,
                          ignore_index: int = IGNORE_INDEX) -> tuple[Tensor, Tensor]:
    """(logits, mean cross-entropy) of `layer(inputs)` against `targets` in one autograd step."""
    return _LMHeadCrossEntropy.apply(inputs, targets, layer.code_int8(), layer.scale,
                                     layer._capture_weight_gradient, ignore_index)
