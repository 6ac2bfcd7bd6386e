"""numpy front end of the CPU oracle (oracle/ratchet_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the checker and by
bench.py's CPU-baseline legs.  The product package never imports it.

Each function restates the reference arithmetic cited in ratchet_oracle.c and takes/returns numpy
arrays (C-contiguous copies are made here).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import build as _build

_LIB: ctypes.CDLL | None = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path: Path = _build.build()
        handle = ctypes.CDLL(str(path))
        handle.or_bf16_round.argtypes = [ctypes.c_float]
        handle.or_bf16_round.restype = ctypes.c_float
        handle.or_philox4x32_10.argtypes = [_u32p, _u32p, _u32p]
        handle.or_sr_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64]
        handle.or_sr_uniform.restype = ctypes.c_float
        handle.or_quantize_rows.argtypes = [_f32p, _i64, _i64, _vp, ctypes.c_int, ctypes.c_uint64,
                                            ctypes.c_uint32, ctypes.c_uint32, _i8p, _f32p]
        handle.or_scaled_int8_mm.argtypes = [_i8p, _i8p, _f32p, _vp, _i64, _i64, _i64, _f32p, _vp]
        handle.or_dequant_rows.argtypes = [_i8p, _f32p, _i64, _i64, _f32p]
        handle.or_grad_weight.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p]
        handle.or_ratchet_update.argtypes = [_f32p, ctypes.c_int, _i64, _i64, _u8p, _vp, ctypes.c_int,
                                             _vp, ctypes.c_double, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_double, ctypes.c_double, ctypes.c_double, _i64p,
                                             _vp, _vp, _f32p]
        handle.or_ratchet_update.restype = ctypes.c_int64
        handle.or_ratchet_leak.argtypes = [_u8p, _i64]
        handle.or_rmsnorm_quantize.argtypes = [_f32p, _f32p, ctypes.c_double, _i64, _i64, _i8p, _f32p, _f32p]
        handle.or_gelu_quantize.argtypes = [_f32p, _i64, _i64, _i8p, _f32p, _f32p]
        handle.or_rmsnorm_backward.argtypes = [_f32p, _f32p, _f32p, ctypes.c_double, _i64, _i64, _f32p, _f32p]
        handle.or_gelu_backward.argtypes = [_f32p, _f32p, _i64, _f32p]
        _LIB = handle
    return _LIB


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16, returned as float32 (vectorised bit arithmetic)."""
    a = _f32(x).copy()
    u = a.view(np.uint32)
    nan = np.isnan(a)
    rounded = (u + (np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))) & np.uint32(0xFFFF0000)
    u[...] = np.where(nan, u | np.uint32(0x00400000), rounded)
    return a


def philox4x32_10(counter, key) -> np.ndarray:
    out = np.zeros(4, np.uint32)
    lib().or_philox4x32_10(np.asarray(counter, np.uint32), np.asarray(key, np.uint32), out)
    return out


def sr_uniform(seed: int, step: int, layer: int, index: int) -> float:
    return float(lib().or_sr_uniform(seed, step, layer, index))


def quantize_rows(x, col_scale=None, *, stochastic=False, seed=0, step=0, layer=0):
    """int8_matmul.py:225-239 (RN) and :139-146 (SR): returns (q int8, scale fp32)."""
    x = _f32(x)
    rows, cols = x.shape
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(rows, np.float32)
    cs = None if col_scale is None else _f32(col_scale)
    lib().or_quantize_rows(x, rows, cols, _ptr(cs), int(stochastic), seed, step, layer, q, s)
    return q, s


def scaled_int8_mm(lhs, rhs, lhs_scale, rhs_scale=None, *, return_acc=False):
    """int8_matmul.py:64-79: bf16((float(lhs @ rhs) * ls) * rs) as float32 (and the int32 acc)."""
    lhs = np.ascontiguousarray(lhs, np.int8)
    rhs = np.ascontiguousarray(rhs, np.int8)
    m, k = lhs.shape
    k2, n = rhs.shape
    assert k == k2
    out = np.zeros((m, n), np.float32)
    acc = np.zeros((m, n), np.int32) if return_acc else None
    rs = None if rhs_scale is None else _f32(rhs_scale)
    lib().or_scaled_int8_mm(lhs, rhs, _f32(lhs_scale), _ptr(rs), m, n, k, out, _ptr(acc))
    return (out, acc) if return_acc else out


def dequant_rows(q, s) -> np.ndarray:
    """ratchet.py:73-76: bf16(bf16(q) * bf16(s)) as float32."""
    q = np.ascontiguousarray(q, np.int8)
    out = np.zeros(q.shape, np.float32)
    lib().or_dequant_rows(q, _f32(s), q.shape[0], q.shape[1], out)
    return out


def grad_weight(g, x) -> np.ndarray:
    """ratchet.py:148-163 without the bf16 output rounding: sum over tokens in double."""
    g, x = _f32(g), _f32(x)
    mt, n = g.shape
    _, k = x.shape
    out = np.zeros((n, k), np.float32)
    lib().or_grad_weight(g, x, mt, n, k, out)
    return out


def ratchet_update(grad, packed, *, max_code, threshold=8, bucket_low=0.5, bucket_high=1.5,
                   eps=1e-8, normalize=True, round_bf16=False, rms_ema=None, beta=0.0,
                   want_grad_scale=False):
    """ratchet.py:248-301 + 539-556 on a copy of `packed`.

    Returns dict(packed, code, counts[4], row_rms, rms_ema, grad_scale, skipped_rows).
    """
    g = _f32(grad)
    rows, cols = g.shape
    pk = np.ascontiguousarray(packed, np.uint8).copy()
    code = np.zeros((rows, cols), np.int8)
    counts = np.zeros(4, np.int64)
    row_rms = np.zeros(rows, np.float32)
    ema = None if rms_ema is None else _f32(rms_ema).copy()
    gs = np.zeros(rows, np.float32) if want_grad_scale else None
    scratch = np.zeros(2 * cols, np.float32)
    skipped = lib().or_ratchet_update(g, int(round_bf16), rows, cols, pk, _ptr(code), int(normalize),
                                      _ptr(ema), float(beta), int(max_code), int(threshold),
                                      float(bucket_low), float(bucket_high), float(eps), counts,
                                      _ptr(row_rms), _ptr(gs), scratch)
    return dict(packed=pk, code=code, counts=counts, row_rms=row_rms, rms_ema=ema, grad_scale=gs,
                skipped_rows=int(skipped))


def ratchet_leak(packed) -> np.ndarray:
    pk = np.ascontiguousarray(packed, np.uint8).copy()
    lib().or_ratchet_leak(pk, pk.size)
    return pk


def pack_code_pressure(code, pressure, max_code) -> np.ndarray:
    """ratchet.py:185-192."""
    low = (np.asarray(code, np.int16) + max_code) & 0x0F
    high = (np.asarray(pressure, np.int16) + 7) & 0x0F
    return (low | (high << 4)).astype(np.uint8)


def unpack_code_pressure(packed, max_code):
    """ratchet.py:195-199."""
    v = np.asarray(packed, np.int16)
    return ((v & 0x0F) - max_code).astype(np.int8), ((v >> 4) - 7).astype(np.int8)


def rmsnorm_quantize(x, w, eps=1e-5):
    x = _f32(x)
    rows, cols = x.shape
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(rows, np.float32)
    lib().or_rmsnorm_quantize(x, _f32(w), eps, rows, cols, q, s, np.zeros(cols, np.float32))
    return q, s


def gelu_quantize(x):
    x = _f32(x)
    rows, cols = x.shape
    q = np.zeros((rows, cols), np.int8)
    s = np.zeros(rows, np.float32)
    lib().or_gelu_quantize(x, rows, cols, q, s, np.zeros(cols, np.float32))
    return q, s


def transpose_quantize(x):
    """[B,H,T,D] -> (B*T, H*D) rows, RN quant (int8_fused.py:103-131)."""
    x = _f32(x)
    b, h, t, d = x.shape
    joined = np.ascontiguousarray(x.transpose(0, 2, 1, 3).reshape(b * t, h * d))
    return quantize_rows(joined)


def rmsnorm_backward(gy, x, w, eps=1e-5) -> np.ndarray:
    gy, x = _f32(gy), _f32(x)
    rows, cols = x.shape
    dx = np.zeros((rows, cols), np.float32)
    lib().or_rmsnorm_backward(gy, x, _f32(w), eps, rows, cols, dx, np.zeros(cols, np.float32))
    return dx


def gelu_backward(gy, x) -> np.ndarray:
    gy, x = _f32(gy), _f32(x)
    dx = np.zeros(x.shape, np.float32)
    lib().or_gelu_backward(gy.reshape(-1), x.reshape(-1), x.size, dx.reshape(-1))
    return dx
