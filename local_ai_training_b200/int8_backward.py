"""Backward kernels of the fused producers (reference int8_backward.py) on sm_100a."""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib


def _contig(t: Tensor) -> Tensor:
    t = t.contiguous()
    return t if t.dtype in (torch.float32, torch.bfloat16) else t.float()


def _aligned(*tensors: Tensor | None) -> bool:
    return all(t is None or t.data_ptr() % 16 == 0 for t in tensors)


class _SrOutputs:
    """Buffers and key of one fused stochastic-rounding quantisation (GradientQuantPlan)."""

    def __init__(self, plan, rows: int, cols: int, grad: Tensor) -> None:
        self.plan = plan
        self.round_bf16 = bool(plan.round_if_fp32 and grad.dtype == torch.float32)
        self.col_scale = plan.col_scale()
        self.q = torch.empty((rows, cols), device=grad.device, dtype=torch.int8)
        self.row_scale = torch.empty((rows,), device=grad.device, dtype=torch.float32)
        # a bf16 gradient is itself the grad_weight operand; any other gets a bf16 copy
        self.bf16_copy = (None if grad.dtype == torch.bfloat16 else
                          torch.empty((rows, cols), device=grad.device, dtype=torch.bfloat16))
        self.seed, self.step, self.layer, self.step_dev = plan.sr_key()

    def usable(self) -> bool:
        return self.col_scale.numel() == self.q.shape[1] and _aligned(self.col_scale)

    def args(self) -> tuple:
        return (_lib.ptr(self.col_scale), int(self.round_bf16), self.seed & (2**64 - 1),
                self.step & 0xFFFFFFFF, self.layer & 0xFFFFFFFF, _lib.ptr(self.step_dev),
                self.q.data_ptr(), self.q.stride(0), self.row_scale.data_ptr(),
                _lib.ptr(self.bf16_copy), 0 if self.bf16_copy is None else self.bf16_copy.stride(0))

    def deliver(self, grad: Tensor) -> None:
        self.plan.deliver(grad, self.q, self.row_scale,
                          grad if self.bf16_copy is None else self.bf16_copy, self.round_bf16)


def rmsnorm_backward(grad_y: Tensor, x: Tensor, w: Tensor, eps: float = 1e-5, *,
                     residual_grad: Tensor | None = None,
                     quant_plan=None) -> tuple[Tensor, Tensor]:
    """RMSNorm backward in one kernel (int8_backward.py:7-51): dx (stored through bf16 into x's
    dtype, as the reference's Triton kernel stores it) and dw = sum over tokens of
    grad_y * x * rsqrt(mean(x^2) + eps), accumulated per column with fp32 reductions.
    residual_grad (fp32 x only): the gradient of the residual branch that leaves x untouched;
    it is added to dx by the same kernel (the sum autograd would form for the two branches).
    quant_plan (GradientQuantPlan of the ratchet layer whose output is x): dx is that layer's
    output gradient; the same kernel also quantises it for the layer's int8 grad_input GEMM."""
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
    sr = None
    if (quant_plan is not None and m > 0 and k % 8 == 0 and k <= 4096 and grad_x.dtype == x.dtype
            and _aligned(gy_flat, x_flat, wf, grad_w, add)):
        sr = _SrOutputs(quant_plan, m, k, grad_x)
        if not sr.usable():
            sr = None
    # the weight gradient's per-CTA partial rows, summed in a fixed order by the library
    need = _lib.lib().rt_rmsnorm_backward_workspace_bytes(m, k)
    work = _lib.workspace(x.device, need)
    ev = _lib.prof_start(x_flat)
    if sr is not None:
        _lib.check(_lib.lib().rt_rmsnorm_backward_sr(
            gy_flat.data_ptr(), _lib.dtype_code(gy_flat), x_flat.data_ptr(),
            _lib.dtype_code(x_flat), wf.data_ptr(), float(eps), m, k, grad_x.data_ptr(),
            _lib.dtype_code(grad_x), grad_w.data_ptr(), _lib.ptr(add), *sr.args(),
            _lib.ptr(work), need, _lib.stream_of(x_flat)))
        sr.deliver(grad_x)
    else:
        _lib.check(_lib.lib().rt_rmsnorm_backward(
            gy_flat.data_ptr(), _lib.dtype_code(gy_flat), x_flat.data_ptr(),
            _lib.dtype_code(x_flat), wf.data_ptr(), float(eps), m, k, grad_x.data_ptr(),
            _lib.dtype_code(grad_x), grad_w.data_ptr(), _lib.ptr(add), _lib.ptr(work), need,
            _lib.stream_of(x_flat)))
    _lib.prof_stop(ev, "rmsnorm_bwd" if sr is None else "rmsnorm_bwd_sr", x_flat, 0.0,
                   m * k * (gy_flat.element_size() + x_flat.element_size() + grad_x.element_size()
                            + (0 if add is None else 4)
                            + (0 if sr is None else 1 + (0 if sr.bf16_copy is None else 2))))
    return grad_x.reshape(x.shape).to(x.dtype), grad_w.to(w.dtype)


def gelu_backward(grad_y: Tensor, x: Tensor, *, quant_plan=None) -> Tensor:
    """tanh-GELU backward (int8_backward.py:53-89), stored through bf16 into x's dtype.
    quant_plan (GradientQuantPlan of the ratchet layer whose output is x): the result is that
    layer's output gradient; the same kernel also quantises it for the layer's int8 grad_input
    GEMM."""
    if not x.is_cuda:
        raise RuntimeError("CUDA required")
    x_flat = _contig(x.flatten(0, -2))
    gy_flat = _contig(grad_y.flatten(0, -2))
    m, k = x_flat.shape
    if gy_flat.dtype != x_flat.dtype:  # the vector kernel takes one dtype for both operands
        gy_flat = gy_flat.to(x_flat.dtype)
    grad_x = torch.empty(x_flat.shape, device=x.device,
                         dtype=x.dtype if x.dtype in (torch.float32, torch.bfloat16) else torch.float32)
    if (quant_plan is not None and m > 0 and k % 8 == 0 and k <= 16384 and grad_x.dtype == x.dtype
            and _aligned(gy_flat, x_flat, grad_x)):
        sr = _SrOutputs(quant_plan, m, k, grad_x)
        if sr.usable():
            ev = _lib.prof_start(x_flat)
            _lib.check(_lib.lib().rt_gelu_backward_sr(
                gy_flat.data_ptr(), x_flat.data_ptr(), _lib.dtype_code(x_flat), m, k,
                grad_x.data_ptr(), *(sr.args()[:1] + sr.args()[2:]), _lib.stream_of(x_flat)))
            _lib.prof_stop(ev, "gelu_bwd_sr", x_flat, 0.0,
                           m * k * (3 * x_flat.element_size() + 1
                                    + (0 if sr.bf16_copy is None else 2)))
            sr.deliver(grad_x)
            return grad_x.reshape(x.shape)
    ev = _lib.prof_start(x_flat)
    _lib.check(_lib.lib().rt_gelu_backward(
        gy_flat.data_ptr(), _lib.dtype_code(gy_flat), x_flat.data_ptr(), _lib.dtype_code(x_flat),
        m, k, grad_x.data_ptr(), _lib.dtype_code(grad_x), _lib.stream_of(x_flat)))
    _lib.prof_stop(ev, "gelu_bwd", x_flat, 0.0,
                   m * k * (gy_flat.element_size() + x_flat.element_size() + grad_x.element_size()))
    return grad_x.reshape(x.shape).to(x.dtype)
