"""Backward kernels of the fused producers (reference int8_backward.py) on sm_100a."""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib


def _contig(t: Tensor) -> Tensor:
    t = t.contiguous()
    return t if t.dtype in (torch.float32, torch.bfloat16) else t.float()


def rmsnorm_backward(grad_y: Tensor, x: Tensor, w: Tensor, eps: float = 1e-5, *,
                     residual_grad: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """RMSNorm backward in one kernel (int8_backward.py:7-51): dx (stored through bf16 into x's
    dtype, as the reference's Triton kernel stores it) and dw = sum over tokens of
    grad_y * x * rsqrt(mean(x^2) + eps), accumulated per column with fp32 reductions.
    residual_grad (fp32 x only): the gradient of the residual branch that leaves x untouched;
    it is added to dx by the same kernel (the sum autograd would form for the two branches)."""
    if not x.is_cuda:
        raise RuntimeError("CUDA required")
    x_flat = _contig(x.flatten(0, -2))
    gy_flat = _contig(grad_y.flatten(0, -2))
    m, k = x_flat.shape
    grad_x = torch.empty(x_flat.shape, device=x.device,
                         dtype=x.dtype if x.dtype in (torch.float32, torch.bfloat16) else torch.float32)
    add = None
    if residual_grad is not None:
        if grad_x.dtype != torch.float32:
            raise TypeError("an added residual gradient needs a float32 input")
        add = residual_grad.reshape(m, k).float()
        if not add.is_contiguous():
            add = add.contiguous()
    wf = w.detach().float().contiguous()
    grad_w = torch.zeros(k, device=x.device, dtype=torch.float32)
    ev = _lib.prof_start(x_flat)
    _lib.check(_lib.lib().rt_rmsnorm_backward(
        gy_flat.data_ptr(), _lib.dtype_code(gy_flat), x_flat.data_ptr(), _lib.dtype_code(x_flat),
        wf.data_ptr(), float(eps), m, k, grad_x.data_ptr(), _lib.dtype_code(grad_x),
        grad_w.data_ptr(), _lib.ptr(add), _lib.stream_of(x_flat)))
    _lib.prof_stop(ev, "rmsnorm_bwd", x_flat, 0.0,
                   m * k * (gy_flat.element_size() + x_flat.element_size() + grad_x.element_size()))
    return grad_x.reshape(x.shape).to(x.dtype), grad_w.to(w.dtype)


def gelu_backward(grad_y: Tensor, x: Tensor) -> Tensor:
    """tanh-GELU backward (int8_backward.py:53-89), stored through bf16 into x's dtype."""
    if not x.is_cuda:
        raise RuntimeError("CUDA required")
    x_flat = _contig(x.flatten(0, -2))
    gy_flat = _contig(grad_y.flatten(0, -2))
    m, k = x_flat.shape
    if gy_flat.dtype != x_flat.dtype:  # the vector kernel takes one dtype for both operands
        gy_flat = gy_flat.to(x_flat.dtype)
    grad_x = torch.empty(x_flat.shape, device=x.device,
                         dtype=x.dtype if x.dtype in (torch.float32, torch.bfloat16) else torch.float32)
    ev = _lib.prof_start(x_flat)
    _lib.check(_lib.lib().rt_gelu_backward(
        gy_flat.data_ptr(), _lib.dtype_code(gy_flat), x_flat.data_ptr(), _lib.dtype_code(x_flat),
        m, k, grad_x.data_ptr(), _lib.dtype_code(grad_x), _lib.stream_of(x_flat)))
    _lib.prof_stop(ev, "gelu_bwd", x_flat, 0.0,
                   m * k * (gy_flat.element_size() + x_flat.element_size() + grad_x.element_size()))
    return grad_x.reshape(x.shape).to(x.dtype)
