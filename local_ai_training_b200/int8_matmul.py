"""int8 GEMM with row/column dequantisation and per-token int8 quantisation on sm_100a.

API-compatible with the reference module int8_matmul.py (quantize_rows, quantize_rows_colscaled,
quantize_columns, scaled_int8_mm); every op runs the CUDA library through the C ABI and raises
on CPU tensors with the reference's messages.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib

_TINY = torch.finfo(torch.float32).tiny


def _as_quantizable(values: Tensor) -> Tensor:
    if values.dtype in (torch.float32, torch.bfloat16):
        return values
    if values.is_floating_point():
        return values.float()
    raise TypeError("row quantization requires a floating-point tensor")


def _quantize_rows_fused(
    values: Tensor,
    col_scale: Tensor | None = None,
    *,
    stochastic: bool = False,
    seed: int | None = None,
    step: int = 0,
    layer: int = 0,
    bf16_copy: Tensor | None = None,
    step_dev: Tensor | None = None,
    round_input_bf16: bool = False,
) -> tuple[Tensor, Tensor]:
    """Row quantisation kernel (int8_matmul.py:106-150, 181-207).

    stochastic=True draws the seed from the host RNG when none is given (the reference's
    `torch.randint(0, 2**31 - 1, (1,))`, int8_matmul.py:200); (seed, step, layer) key the Philox
    stream.  bf16_copy, when given (rows × cols bf16, unit column stride), receives bf16(values).
    step_dev (int32 [2] on the device, zeros to start), when given: element 0 is read by the
    kernel instead of `step` and advanced by one by the call; element 1 is the kernel's arrival
    count (zero between calls).  round_input_bf16 (fp32 values): each value is rounded to bf16 first.
    """
    if values.ndim != 2:
        raise ValueError("row quantization requires a 2D tensor")
    values = _as_quantizable(values)
    m, k = values.shape
    out = torch.empty((m, k), device=values.device, dtype=torch.int8)
    scale = torch.empty((m,), device=values.device, dtype=torch.float32)
    if m == 0:
        return out, scale
    if col_scale is not None:
        col_scale = col_scale.contiguous()
    if stochastic and seed is None:
        seed = int(torch.randint(0, 2**31 - 1, (1,)).item())
    ev = _lib.prof_start(values)
    _lib.check(
        _lib.lib().rt_quantize_rows(
            values.data_ptr(), _lib.dtype_code(values), m, k, values.stride(0), values.stride(1),
            _lib.ptr(col_scale), int(stochastic), int(round_input_bf16),
            int(seed or 0) & (2**64 - 1), int(step) & 0xFFFFFFFF,
            int(layer) & 0xFFFFFFFF, _lib.ptr(step_dev), out.data_ptr(), out.stride(0),
            scale.data_ptr(),
            _lib.ptr(bf16_copy), 0 if bf16_copy is None else bf16_copy.stride(0),
            _lib.stream_of(values),
        )
    )
    if ev is not None:
        nbytes = m * k * (values.element_size() + 1 + (2 if bf16_copy is not None else 0)) + 4 * m
        _lib.prof_stop(ev, "quant_rows_sr" if stochastic else "quant_rows", values, 0.0, nbytes)
    return out, scale


def quantize_rows(values: Tensor) -> tuple[Tensor, Tensor]:
    """Symmetrically quantize each row and return int8 values plus FP32 scales (CUDA-only)."""
    if not values.is_cuda:
        raise RuntimeError("quantize_rows requires CUDA; the int8 path is GPU-only")
    return _quantize_rows_fused(values)


def quantize_rows_colscaled(
    values: Tensor, col_scale: Tensor, *, stochastic: bool = False, seed: int | None = None,
    step: int = 0, layer: int = 0,
) -> tuple[Tensor, Tensor]:
    """Row-quantize values after per-column scaling, fused in one pass (CUDA-only)."""
    if not values.is_cuda:
        raise RuntimeError("quantize_rows_colscaled requires CUDA; the int8 path is GPU-only")
    if col_scale.ndim != 1 or values.ndim != 2 or col_scale.shape[0] != values.shape[1]:
        raise ValueError("col_scale must be 1-D with length values.shape[1]")
    if col_scale.dtype != torch.float32:
        raise TypeError("col_scale must be float32")
    return _quantize_rows_fused(values, col_scale, stochastic=stochastic, seed=seed, step=step,
                                layer=layer)


def quantize_columns(values: Tensor) -> tuple[Tensor, Tensor]:
    """Per-column symmetric quantisation (int8_matmul.py:153-178 semantics, fp32 arithmetic)."""
    if not values.is_cuda:
        raise RuntimeError("quantize_columns requires CUDA; the int8 path is GPU-only")
    if values.ndim != 2:
        raise ValueError("column quantization requires a 2D tensor")
    q_t, scale = _quantize_rows_fused(values.t())
    return q_t.t().contiguous(), scale


def _scaled_int8_mm_into(
    lhs: Tensor, rhs: Tensor, lhs_scale: Tensor, rhs_scale: Tensor | None, out: Tensor,
    rhs_abs_max: int = 0, residual: Tensor | None = None,
) -> Tensor:
    """No-sync core: out = bf16((float(lhs @ rhs) * lhs_scale[m]) * rhs_scale[n]).

    `out` is (M, N) bf16, or fp32 receiving the bf16-rounded values (the widening cast of
    ratchet.py:67 fused into the epilogue).  Operands are passed with their strides.
    rhs_abs_max: a guaranteed bound on |rhs| (ratchet codes: 7) or 0; it only lets the epilogue
    use a cheaper exact accumulator conversion.  residual (fp32 `out` only): out = residual + value.
    """
    m, k = lhs.shape
    _, n = rhs.shape
    ev = _lib.prof_start(lhs)
    _lib.check(
        _lib.lib().rt_scaled_int8_mm(
            lhs.data_ptr(), lhs.stride(0), lhs.stride(1), rhs.data_ptr(), rhs.stride(0),
            rhs.stride(1), lhs_scale.data_ptr(), _lib.ptr(rhs_scale), out.data_ptr(),
            _lib.dtype_code(out), out.stride(0), m, n, k, int(rhs_abs_max), _lib.ptr(residual),
            0 if residual is None else residual.stride(0), _lib.stream_of(lhs),
        )
    )
    if ev is not None:
        # operands, scales, the output and (fused residual add) the fp32 residual tile reads
        _lib.prof_stop(ev, "gemm_i8", lhs, 2.0 * m * n * k,
                       m * k + n * k + 4 * (m + n) + m * n * out.element_size()
                       + (4 * m * n if residual is not None else 0))
    return out


def scaled_int8_mm(lhs: Tensor, rhs: Tensor, lhs_scale: Tensor, rhs_scale: Tensor) -> Tensor:
    """Multiply int8 matrices and fuse row/column scale dequantization into BF16 output."""
    if not lhs.is_cuda or not rhs.is_cuda:
        raise RuntimeError("scaled_int8_mm requires CUDA operands")
    if lhs.ndim != 2 or rhs.ndim != 2:
        raise ValueError("scaled_int8_mm operands must be 2D")
    if lhs.dtype != torch.int8 or rhs.dtype != torch.int8:
        raise TypeError("scaled_int8_mm operands must be int8")
    if lhs.shape[1] != rhs.shape[0]:
        raise ValueError("scaled_int8_mm inner dimensions must match")
    if lhs.device != rhs.device:
        raise ValueError("scaled_int8_mm operands must share a device")
    m, k = lhs.shape
    _, n = rhs.shape
    if lhs_scale.shape != (m,) or rhs_scale.shape != (n,):
        raise ValueError("scaled_int8_mm scales must match output rows and columns")
    for name, scale in (("lhs", lhs_scale), ("rhs", rhs_scale)):
        if scale.device != lhs.device or scale.dtype != torch.float32:
            raise TypeError(f"{name} scale must be FP32 on the operand device")
        if not torch.isfinite(scale).all() or torch.any(scale <= 0):
            raise ValueError(f"{name} scale must be finite and positive")
    if 1 not in lhs.stride():
        lhs = lhs.contiguous()
    if 1 not in rhs.stride():
        rhs = rhs.contiguous()
    out = torch.empty((m, n), device=lhs.device, dtype=torch.bfloat16)
    return _scaled_int8_mm_into(lhs, rhs, lhs_scale.contiguous(), rhs_scale.contiguous(), out)


def grad_weight_bf16(grad: Tensor, inputs: Tensor, out: Tensor | None = None, *,
                     accumulate: bool = False, addend: Tensor | None = None) -> Tensor:
    """gw[n, k] (+)= sum_m grad[m, n] * inputs[m, k]: bf16 operands, fp32 accumulation/output
    (the per-tile grad_weight GEMM of ratchet.py:148-163 as one tcgen05 launch).

    addend (fp32 [n, k], optional): out = round(addend + gw) in out's dtype -- the last
    micro-batch of an accumulated step writing the bf16 total."""
    if grad.dtype != torch.bfloat16 or inputs.dtype != torch.bfloat16:
        raise TypeError("grad_weight_bf16 operands must be bfloat16")
    if grad.stride(1) != 1:
        grad = grad.contiguous()
    if inputs.stride(1) != 1:
        inputs = inputs.contiguous()
    mt, n = grad.shape
    mt2, k = inputs.shape
    if mt != mt2:
        raise ValueError("grad_weight_bf16 token dimensions must match")
    if out is None:
        out = torch.empty((n, k), device=grad.device, dtype=torch.float32)
        accumulate = False
    need = _lib.lib().rt_grad_weight_workspace_bytes(mt, n, k)
    ws = _lib.workspace(grad.device, need)
    ev = _lib.prof_start(grad)
    if addend is not None:
        if addend.dtype != torch.float32 or addend.shape != (n, k) or addend.stride(1) != 1:
            raise TypeError("grad_weight_bf16 addend must be a float32 [out, in] row-major matrix")
        _lib.check(
            _lib.lib().rt_grad_weight_bf16_add(
                grad.data_ptr(), grad.stride(0), inputs.data_ptr(), inputs.stride(0),
                addend.data_ptr(), addend.stride(0), out.data_ptr(), _lib.dtype_code(out),
                out.stride(0), mt, n, k, _lib.ptr(ws), 0 if ws is None else ws.numel(),
                _lib.stream_of(grad),
            )
        )
    else:
        _lib.check(
            _lib.lib().rt_grad_weight_bf16(
                grad.data_ptr(), grad.stride(0), inputs.data_ptr(), inputs.stride(0),
                out.data_ptr(), _lib.dtype_code(out), out.stride(0), mt, n, k, int(accumulate),
                _lib.ptr(ws), 0 if ws is None else ws.numel(), _lib.stream_of(grad),
            )
        )
    if ev is not None:
        extra = 4 * n * k if (accumulate or addend is not None) else 0  # the fp32 read
        _lib.prof_stop(ev, "gemm_gradw_bf16", grad, 2.0 * mt * n * k,
                       2 * mt * (n + k) + out.element_size() * n * k + extra)
    return out


def matmul_bf16(a: Tensor, b: Tensor, out_dtype: torch.dtype = torch.bfloat16, *,
                out: Tensor | None = None) -> Tensor:
    """a[M, K] @ b[K, N] with bf16 operands and fp32 accumulation on the tcgen05 GEMM (the bf16
    grad_input matmul of ratchet.py:135-141); output bf16 (RN) or float32, into `out` (a row-major
    [M, N] view, e.g. a row slice of a larger matrix) when given."""
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("matmul_bf16 operands must be bfloat16")
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("matmul_bf16 needs a[M, K] and b[K, N]")
    _require = [t for t in (a, b) if not t.is_cuda]
    if _require:
        raise RuntimeError("matmul_bf16 requires CUDA operands")
    if a.stride(1) != 1:
        a = a.contiguous()
    if b.stride(1) != 1:
        b = b.contiguous()
    m, k = a.shape
    n = b.shape[1]
    if out is None:
        out = torch.empty((m, n), device=a.device, dtype=out_dtype)
    elif (out.shape != (m, n) or out.dtype not in (torch.bfloat16, torch.float32)
          or out.stride(1) != 1 or out.device != a.device):
        raise ValueError("matmul_bf16 out must be a [M, N] bf16 or float32 view with unit column "
                         "stride on the operands' device")
    if out.numel() == 0:
        return out
    ev = _lib.prof_start(a)
    _lib.check(_lib.lib().rt_matmul_bf16(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), out.data_ptr(),
        _lib.dtype_code(out), out.stride(0), m, n, k, _lib.stream_of(a)))
    if ev is not None:
        _lib.prof_stop(ev, "gemm_bf16", a, 2.0 * m * n * k,
                       2 * (m * k + k * n) + out.element_size() * m * n)
    return out


def dequant_rows_bf16(q: Tensor, scale: Tensor) -> Tensor:
    """bf16(bf16(q) * bf16(scale[:, None])) (ratchet.py:73-76)."""
    if q.stride(1) != 1:
        q = q.contiguous()
    rows, cols = q.shape
    out = torch.empty((rows, cols), device=q.device, dtype=torch.bfloat16)
    ev = _lib.prof_start(q)
    _lib.check(
        _lib.lib().rt_dequant_rows_bf16(
            q.data_ptr(), q.stride(0), scale.contiguous().data_ptr(), out.data_ptr(), out.stride(0),
            rows, cols, _lib.stream_of(q),
        )
    )
    if ev is not None:
        _lib.prof_stop(ev, "dequant", q, 0.0, 3 * rows * cols + 4 * rows)
    return out
