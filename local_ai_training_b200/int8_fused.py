"""Fused producers of pre-quantised ratchet inputs (reference int8_fused.py) on sm_100a.

Each producer reads its input once per row and writes the int8 row plus its fp32 scale; the
autograd wrappers return (int8, scale, dummy) exactly like the reference so that the ratchet
layer receives pre-quantised inputs and the gradient flows back through the dummy.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from .int8_backward import gelu_backward, rmsnorm_backward


def _rows(x: Tensor) -> Tensor:
    flat = x.flatten(0, -2)
    if flat.stride(-1) != 1:
        flat = flat.contiguous()
    if flat.dtype not in (torch.float32, torch.bfloat16):
        flat = flat.float()
    return flat


def _dequant_buffer(m: int, k: int, device, want: bool) -> Tensor | None:
    return torch.empty((m, k), device=device, dtype=torch.bfloat16) if want else None


def fused_rmsnorm_quantize(x: Tensor, weight: Tensor, eps: float = 1e-5, *,
                           dequant_out: bool = False):
    """RMSNorm -> per-token int8 (int8_fused.py:14-56).  dequant_out: also returns
    bf16(bf16(q)·bf16(s)) [tokens, features], the layer's grad_weight operand (ratchet.py:73-76),
    written by the same kernel."""
    if not x.is_cuda:
        raise RuntimeError("CUDA required")
    flat = _rows(x)
    m, k = flat.shape
    out = torch.empty((m, k), device=x.device, dtype=torch.int8)
    scale = torch.empty((m,), device=x.device, dtype=torch.float32)
    dq = _dequant_buffer(m, k, x.device, dequant_out)
    w = weight.detach().float().contiguous()
    ev = _lib.prof_start(flat)
    _lib.check(_lib.lib().rt_rmsnorm_quantize(
        flat.data_ptr(), _lib.dtype_code(flat), flat.stride(0), w.data_ptr(), float(eps), m, k,
        out.data_ptr(), out.stride(0), scale.data_ptr(), _lib.ptr(dq),
        0 if dq is None else dq.stride(0), _lib.stream_of(flat)))
    _lib.prof_stop(ev, "rmsnorm_quant", flat, 0.0,
                   m * k * (flat.element_size() + 1 + (2 if dequant_out else 0)) + 4 * m)
    if dequant_out:
        return out.reshape(x.shape), scale.reshape(x.shape[:-1]), dq
    return out.reshape(x.shape), scale.reshape(x.shape[:-1])


def fused_gelu_quantize(x: Tensor, *, dequant_out: bool = False):
    """tanh-GELU -> per-token int8 (int8_fused.py:58-101); dequant_out as in
    fused_rmsnorm_quantize."""
    if not x.is_cuda:
        raise RuntimeError("CUDA required")
    flat = _rows(x)
    m, k = flat.shape
    out = torch.empty((m, k), device=x.device, dtype=torch.int8)
    scale = torch.empty((m,), device=x.device, dtype=torch.float32)
    dq = _dequant_buffer(m, k, x.device, dequant_out)
    ev = _lib.prof_start(flat)
    _lib.check(_lib.lib().rt_gelu_quantize(
        flat.data_ptr(), _lib.dtype_code(flat), flat.stride(0), m, k, out.data_ptr(),
        out.stride(0), scale.data_ptr(), _lib.ptr(dq), 0 if dq is None else dq.stride(0),
        _lib.stream_of(flat)))
    _lib.prof_stop(ev, "gelu_quant", flat, 0.0,
                   m * k * (flat.element_size() + 1 + (2 if dequant_out else 0)) + 4 * m)
    if dequant_out:
        return out.reshape(x.shape), scale.reshape(x.shape[:-1]), dq
    return out.reshape(x.shape), scale.reshape(x.shape[:-1])


def fused_transpose_quantize(x: Tensor, *, dequant_out: bool = False):
    """[B, H, T, D] heads -> (B*T, H*D) per-token int8 (int8_fused.py:103-151); dequant_out as
    in fused_rmsnorm_quantize."""
    if not x.is_cuda:
        raise RuntimeError("CUDA required")
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    b, h, t, d = x.shape
    out = torch.empty((b * t, h * d), device=x.device, dtype=torch.int8)
    scale = torch.empty((b * t,), device=x.device, dtype=torch.float32)
    dq = _dequant_buffer(b * t, h * d, x.device, dequant_out)
    ev = _lib.prof_start(x)
    _lib.check(_lib.lib().rt_transpose_quantize(
        x.data_ptr(), _lib.dtype_code(x), b, h, t, d, x.stride(0), x.stride(1), x.stride(2),
        x.stride(3), out.data_ptr(), out.stride(0), scale.data_ptr(), _lib.ptr(dq),
        0 if dq is None else dq.stride(0), _lib.stream_of(x)))
    _lib.prof_stop(ev, "transpose_quant", x, 0.0,
                   b * h * t * d * (x.element_size() + 1 + (2 if dequant_out else 0)) + 4 * b * t)
    if dequant_out:
        return out, scale, dq
    return out, scale


def _no_zero_grads(ctx, *outputs: Tensor) -> None:
    """The int8 codes, row scales (and dequantised copies) carry no gradient: mark them so, and
    let backward see None for gradients nobody produced instead of zero tensors autograd would
    fill (one fill kernel per output per call)."""
    ctx.mark_non_differentiable(*outputs)
    ctx.set_materialize_grads(False)


class FusedRMSNormQuantizeFn(torch.autograd.Function):
    """(int8, scale, dummy) like the reference.  `dummy_dtype` (default: x's dtype, the
    reference) sets the dtype of the dummy, i.e. of the consuming layer's input gradient.

    residual_out=True also returns x itself as a fourth output, to be consumed as the residual
    of the block (`x + sublayer(norm(x))`): its gradient then arrives here and is added to the
    RMSNorm input gradient by the same kernel, instead of autograd summing the two branches.

    grad_plan: the GradientQuantPlan x carries when a ratchet layer produced it; the input
    gradient computed here is then also quantised for that layer by the same kernel.

    dequant_out=True appends a last output: the bf16 dequantised rows for the consuming layer's
    grad_weight (`inputs_dequant` of DiscreteRatchetLinear.forward)."""

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, eps: float = 1e-5, dummy_dtype=None,
                residual_out: bool = False, grad_plan=None, dequant_out: bool = False):
        produced = fused_rmsnorm_quantize(x, weight, eps, dequant_out=dequant_out)
        int8_out, scale_out = produced[0], produced[1]
        ctx.save_for_backward(x, weight)
        ctx.eps = eps
        ctx.grad_plan = grad_plan
        ctx.residual_out = residual_out
        dummy = torch.empty(x.shape, device=x.device, dtype=dummy_dtype or x.dtype)
        _no_zero_grads(ctx, int8_out, scale_out, *produced[2:])
        outputs = (int8_out, scale_out, dummy) + ((x,) if residual_out else ()) + produced[2:]
        return outputs

    @staticmethod
    def backward(ctx, grad_int8, grad_scale, grad_dummy, *grad_rest):
        # grad_rest: the residual output's gradient (residual_out), then the dequant copy's (None)
        grad_residual = grad_rest[0] if ctx.residual_out else None
        if grad_dummy is None:
            return grad_residual, None, None, None, None, None, None
        x, weight = ctx.saved_tensors
        fuse = grad_residual is not None and x.dtype == torch.float32
        plan = ctx.grad_plan if (fuse or grad_residual is None) else None
        grad_x, grad_w = rmsnorm_backward(grad_dummy, x, weight, ctx.eps,
                                          residual_grad=grad_residual if fuse else None,
                                          quant_plan=plan)
        if grad_residual is not None and not fuse:
            grad_x = grad_x + grad_residual
        return grad_x, grad_w, None, None, None, None, None


class FusedGELUQuantizeFn(torch.autograd.Function):
    """(int8, scale, dummy) like the reference; `dummy_dtype` and `grad_plan` as in
    FusedRMSNormQuantizeFn."""

    @staticmethod
    def forward(ctx, x: Tensor, dummy_dtype=None, grad_plan=None, dequant_out: bool = False):
        produced = fused_gelu_quantize(x, dequant_out=dequant_out)
        ctx.save_for_backward(x)
        ctx.grad_plan = grad_plan
        dummy = torch.empty(x.shape, device=x.device, dtype=dummy_dtype or x.dtype)
        _no_zero_grads(ctx, *produced)
        return (produced[0], produced[1], dummy) + produced[2:]

    @staticmethod
    def backward(ctx, grad_int8, grad_scale, grad_dummy, grad_dq=None):
        if grad_dummy is None:
            return None, None, None, None
        (x,) = ctx.saved_tensors
        return gelu_backward(grad_dummy, x, quant_plan=ctx.grad_plan), None, None, None


class FusedTransposeQuantizeFn(torch.autograd.Function):
    """(int8, scale, dummy) like the reference; dequant_out as in FusedRMSNormQuantizeFn."""

    @staticmethod
    def forward(ctx, attended: Tensor, dequant_out: bool = False):
        produced = fused_transpose_quantize(attended, dequant_out=dequant_out)
        ctx.save_for_backward(attended)
        batch_size, n_head, seq_len, head_dim = attended.shape
        dummy = torch.empty((batch_size, seq_len, n_head * head_dim), device=attended.device,
                            dtype=attended.dtype)
        _no_zero_grads(ctx, *produced)
        return (produced[0], produced[1], dummy) + produced[2:]

    @staticmethod
    def backward(ctx, grad_int8, grad_scale, grad_dummy, grad_dq=None):
        if grad_dummy is None:
            return None, None
        (attended,) = ctx.saved_tensors
        batch_size, n_head, seq_len, head_dim = attended.shape
        return grad_dummy.view(batch_size, seq_len, n_head, head_dim).transpose(1, 2), None


def heads_gather_quantize(grads: tuple[Tensor, Tensor, Tensor], plan) -> Tensor | None:
    """[B, T, 3·H·D] gradient of a q|k|v projection output from the gradients of its three
    [B, H, T, D] head views, quantised in the same kernel for the projection (GradientQuantPlan);
    None when the layout does not allow 16-byte chunks (the caller concatenates instead)."""
    from .int8_backward import _SrOutputs

    g0 = grads[0]
    b, h, t, d = g0.shape
    if (d % 8 != 0 or g0.dtype not in (torch.float32, torch.bfloat16)
            or any(g.dtype != g0.dtype or g.shape != g0.shape or g.stride(3) != 1
                   or g.data_ptr() % 16 != 0 for g in grads)):
        return None
    es = g0.element_size()
    if any((st * es) % 16 != 0 for g in grads for st in g.stride()[:3]):
        return None
    rows, cols = b * t, 3 * h * d
    out = torch.empty((rows, cols), device=g0.device, dtype=g0.dtype)
    sr = _SrOutputs(plan, rows, cols, out)
    if not sr.usable():
        return None
    import ctypes

    src = (ctypes.c_void_p * 3)(*[g.data_ptr() for g in grads])
    strides = (ctypes.c_int64 * 12)(*[s for g in grads for s in g.stride()])
    args = sr.args()
    ev = _lib.prof_start(out)
    _lib.check(_lib.lib().rt_heads_gather_sr(
        ctypes.addressof(src), ctypes.addressof(strides), _lib.dtype_code(g0), b, h, t, d,
        out.data_ptr(), out.stride(0), args[0], *args[2:], _lib.stream_of(out)))
    _lib.prof_stop(ev, "heads_gather_sr", out, 0.0,
                   rows * cols * (2 * es + 1 + (0 if sr.bf16_copy is None else 2)))
    sr.deliver(out)
    return out.view(b, t, cols)


class QKVHeadsFn(torch.autograd.Function):
    """(query, key, value) [B, H, T, D] head views of a q|k|v projection output [B, T, 3C]
    (model.py:61-70: `.chunk(3, dim=-1)`, then view and transpose of each part).  Backward forms
    the [B, T, 3C] gradient of the projection output from the three head gradients in one
    kernel that also quantises it for the projection (`plan`, a GradientQuantPlan), instead of
    autograd's concatenation followed by the projection's own quantisation pass."""

    @staticmethod
    def forward(ctx, qkv: Tensor, n_head: int, plan):
        b, t, c3 = qkv.shape
        c = c3 // 3
        ctx.plan = plan
        ctx.shape = qkv.shape
        parts = qkv.chunk(3, dim=-1)
        return tuple(p.view(b, t, n_head, c // n_head).transpose(1, 2) for p in parts)

    @staticmethod
    def backward(ctx, gq, gk, gv):
        b, t, c3 = ctx.shape
        grads = [g for g in (gq, gk, gv)]
        if all(g is None for g in grads):
            return None, None, None
        if any(g is None for g in grads):
            ref = next(g for g in grads if g is not None)
            grads = [torch.zeros_like(ref) if g is None else g for g in grads]
        out = heads_gather_quantize(tuple(grads), ctx.plan) if ctx.plan is not None else None
        if out is None:
            out = torch.cat([g.transpose(1, 2).reshape(b, t, c3 // 3) for g in grads], dim=-1)
        return out, None, None
