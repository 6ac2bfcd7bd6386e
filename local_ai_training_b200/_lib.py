"""ctypes binding of libratchet_b200.so (the C ABI declared in include/ratchet_b200.h).

The library is loaded once per process.  Status codes map to the exception types the reference
raises for the same conditions: invalid shapes/alignment -> ValueError, dtypes -> TypeError,
everything else -> RuntimeError.  There is no fallback: if the library cannot be loaded, every op
raises.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _build

F32, BF16, I8, U8 = 0, 1, 2, 3

STATUS_NONFINITE_GRADIENT = 0x1
STATUS_WAIT_TIMEOUT = 0x2
STATUS_CODE_RANGE = 0x4
STATUS_PRESSURE_RANGE = 0x8
STATUS_SCALE_INVALID = 0x10
STATUS_INDEX_RANGE = 0x20

_ERR_INVALID, _ERR_DTYPE, _ERR_ALIGN = 1, 2, 3
ABI_VERSION = 2

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_d = ctypes.c_double

_SIGNATURES = {
    "rt_abi_version": ([], _i),
    "rt_last_error": ([], ctypes.c_char_p),
    "rt_device_status": ([_p, _i, _p], _i),
    "rt_sm_count": ([_p], _i),
    "rt_quantize_rows": ([_p, _i, _i64, _i64, _i64, _i64, _p, _i, _i, _u64, _u32, _u32, _p, _p, _i64,
                          _p, _p, _i64, _p], _i),
    "rt_scaled_int8_mm": ([_p, _i64, _i64, _p, _i64, _i64, _p, _p, _p, _i, _i64, _i64, _i64, _i64,
                           _i, _p, _i64, _p], _i),
    "rt_grad_weight_bf16": ([_p, _i64, _p, _i64, _p, _i, _i64, _i64, _i64, _i64, _i, _p, _i64, _p],
                            _i),
    "rt_grad_weight_workspace_bytes": ([_i64, _i64, _i64], _i64),
    "rt_grad_weight_ratchet_update": ([_p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64,
                                       _p, _i64, _p, _d, _i, _i, _d, _d, _d, _p, _p, _p, _p, _p],
                                      _i),
    "rt_grad_weight_update_workspace_bytes": ([_i64, _i64, _i64], _i64),
    "rt_grad_weight_bf16_add": ([_p, _i64, _p, _i64, _p, _i64, _p, _i, _i64, _i64, _i64, _i64, _p,
                                 _i64, _p], _i),
    "rt_matmul_bf16": ([_p, _i64, _p, _i64, _p, _i, _i64, _i64, _i64, _i64, _p], _i),
    "rt_ratchet_update_grouped": ([_p, _i, _i, _i, _i64, _i, _d, _i, _i, _d, _d, _d, _p], _i),
    "rt_grad_weight_bf16_noalloc": ([_p, _i64, _p, _i64, _p, _i, _i64, _i64, _i64, _i64, _i, _p],
                                    _i),
    "rt_dequant_rows_bf16": ([_p, _i64, _p, _p, _i64, _i64, _i64, _p], _i),
    "rt_ratchet_update": ([_p, _i, _i, _i64, _i64, _i64, _p, _i64, _p, _i64, _i, _p, _d, _i, _i,
                           _d, _d, _d, _p, _p, _p, _p, _p], _i),
    "rt_ratchet_leak": ([_p, _i64, _i64, _i64, _i, _p], _i),
    "rt_unpack_code_pressure": ([_p, _i64, _i64, _i64, _i, _p, _i64, _p, _i64, _p], _i),
    "rt_ratchet_validate": ([_p, _i64, _i64, _i64, _i, _p, _p], _i),
    "rt_rmsnorm_quantize": ([_p, _i, _i64, _p, _d, _i64, _i64, _p, _i64, _p, _p, _i64, _p], _i),
    "rt_gelu_quantize": ([_p, _i, _i64, _i64, _i64, _p, _i64, _p, _p, _i64, _p], _i),
    "rt_transpose_quantize": ([_p, _i, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64,
                               _p, _p, _i64, _p], _i),
    "rt_rmsnorm_backward": ([_p, _i, _p, _i, _p, _d, _i64, _i64, _p, _i, _p, _p, _p, _i64, _p],
                            _i),
    "rt_rmsnorm_backward_workspace_bytes": ([_i64, _i64], _i64),
    "rt_gelu_backward": ([_p, _i, _p, _i, _i64, _i64, _p, _i, _p], _i),
    "rt_rmsnorm_backward_sr": ([_p, _i, _p, _i, _p, _d, _i64, _i64, _p, _i, _p, _p, _p, _i, _u64,
                                _u32, _u32, _p, _p, _i64, _p, _p, _i64, _p, _i64, _p], _i),
    "rt_gelu_backward_sr": ([_p, _p, _i, _i64, _i64, _p, _p, _u64, _u32, _u32, _p, _p, _i64, _p,
                             _p, _i64, _p], _i),
    "rt_heads_gather_sr": ([_p, _p, _i, _i64, _i64, _i64, _i64, _p, _i64, _p, _u64, _u32, _u32,
                            _p, _p, _i64, _p, _p, _i64, _p], _i),
    "rt_embedding_forward": ([_p, _i64, _p, _i, _p, _i64, _i64, _i64, _p, _i64, _p], _i),
    "rt_embedding_update_workspace_bytes": ([_i64, _i64], _i64),
    "rt_embedding_ratchet_update": ([_p, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _i64, _p,
                                     _i64, _p, _d, _i, _i, _d, _d, _d, _p, _p, _p], _i),
    "rt_token_windows": ([_p, _i64, _p, _i64, _i64, _p, _p, _p], _i),
    "rt_cross_entropy_fwd": ([_p, _i, _i64, _i64, _i64, _p, _i64, _p, _p, _p, _p], _i),
    "rt_cross_entropy_bwd": ([_p, _i, _i64, _i64, _i64, _p, _i64, _p, _p, _p, _p, _p, _i64, _p,
                              _i64, _p], _i),
}


class UpdateLayer(ctypes.Structure):
    """struct rt_update_layer of include/ratchet_b200.h (one layer of a grouped update)."""

    _fields_ = [("grad", _p), ("ldg", _i64), ("rows", _i64), ("packed", _p), ("ldp", _i64),
                ("code_out", _p), ("ldc", _i64), ("rms_ema", _p), ("counts", _p),
                ("rms_sum", _p), ("grad_mul", ctypes.c_float)]


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Loads the library (building it first only if the file is missing)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            path = _build.LIB_PATH
            if not path.exists():
                _build.build()
            handle = ctypes.CDLL(str(path))
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = res
            version = handle.rt_abi_version()
            if version != ABI_VERSION:
                raise RuntimeError(f"libratchet_b200 ABI {version}, expected {ABI_VERSION}")
            _LIB = handle
    return _LIB


def check(rc: int) -> None:
    if rc == 0:
        return
    message = (lib().rt_last_error() or b"").decode(errors="replace")
    if rc in (_ERR_INVALID, _ERR_ALIGN):
        raise ValueError(message)
    if rc == _ERR_DTYPE:
        raise TypeError(message)
    raise RuntimeError(message)


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.int8:
        return I8
    if t.dtype == torch.uint8:
        return U8
    raise TypeError(f"unsupported dtype {t.dtype}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def device_status(device: torch.device, *, clear: bool = True) -> int:
    """Reads (and clears) the sticky device status word; synchronises the current stream."""
    out = ctypes.c_uint32(0)
    with torch.cuda.device(device):
        check(lib().rt_device_status(ctypes.byref(out), int(clear),
                                     torch.cuda.current_stream(device).cuda_stream))
    return int(out.value)


_WORKSPACES: dict[torch.device, torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """Per-device scratch for split-K partial tiles (zero-initialised once; the kernels leave
    its ticket words zero).  Reused by every call on the device's streams in order."""
    if nbytes <= 0:
        return None
    ws = _WORKSPACES.get(device)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, device=device, dtype=torch.uint8)
        _WORKSPACES[device] = ws
    return ws


# Opt-in timing of library calls: when PROFILE is a dict, each wrapped call records a pair of CUDA
# events on its stream plus its algorithmic flops and bytes under a kernel-family name.
PROFILE: dict | None = None
# When True the events are created as external events, so that a CUDA graph captured while
# profiling holds event-record nodes and each replay re-times every library call.
PROFILE_EXTERNAL = False


def prof_start(t: torch.Tensor):
    if PROFILE is None:
        return None
    ev = torch.cuda.Event(enable_timing=True, external=PROFILE_EXTERNAL)
    ev.record(torch.cuda.current_stream(t.device))
    return ev


def prof_stop(start, name: str, t: torch.Tensor, flops: float, nbytes: float) -> None:
    if start is None or PROFILE is None:
        return
    end = torch.cuda.Event(enable_timing=True, external=PROFILE_EXTERNAL)
    end.record(torch.cuda.current_stream(t.device))
    PROFILE.setdefault(name, []).append((start, end, float(flops), float(nbytes)))


def sm_count() -> int:
    out = ctypes.c_int(0)
    check(lib().rt_sm_count(ctypes.byref(out)))
    return int(out.value)
