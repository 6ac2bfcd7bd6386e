"""GPU: rt_grad_weight_bf16_noalloc (static device scratch) against rt_grad_weight_bf16 with a
caller workspace, called through the C ABI.

Both entry points pick the same split count for a shape, so the tolerance is exact equality
(bitwise), on two calls in a row.  Collected last so it also runs after every other GPU test.
"""

from __future__ import annotations

import pytest
import torch

from local_ai_training_b200 import _lib
from local_ai_training_b200.int8_matmul import grad_weight_bf16

pytestmark = pytest.mark.gpu

SHAPES = [
    (16384, 512, 512),    # split-K over the token dimension
    (16384, 2048, 512),
    (16384, 512, 2048),
    (4096, 8192, 512),    # enough tiles: no split
    (1000, 300, 72),      # ragged tiles
]


def _noalloc(g: torch.Tensor, x: torch.Tensor, out: torch.Tensor, accumulate: bool) -> None:
    mt, n = g.shape
    k = x.shape[1]
    _lib.check(
        _lib.lib().rt_grad_weight_bf16_noalloc(
            g.data_ptr(), g.stride(0), x.data_ptr(), x.stride(0), out.data_ptr(),
            _lib.dtype_code(out), out.stride(0), mt, n, k, int(accumulate), _lib.stream_of(g),
        )
    )


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry(cuda_device, shape, out_dtype):
    mt, n, k = shape
    gen = torch.Generator(device=cuda_device).manual_seed(mt + n + k)
    g = torch.randn((mt, n), device=cuda_device, generator=gen).to(torch.bfloat16)
    x = torch.randn((mt, k), device=cuda_device, generator=gen).to(torch.bfloat16)
    want = torch.empty((n, k), device=cuda_device, dtype=out_dtype)
    grad_weight_bf16(g, x, want)
    for _ in range(2):  # two calls in a row: scratch left by the first must not change the second
        got = torch.full((n, k), float("nan"), device=cuda_device, dtype=out_dtype)
        _noalloc(g, x, got, False)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    assert _lib.device_status(cuda_device, clear=True) == 0


def test_noalloc_accumulate_matches(cuda_device):
    mt, n, k = 16384, 512, 512
    gen = torch.Generator(device=cuda_device).manual_seed(7)
    g = torch.randn((mt, n), device=cuda_device, generator=gen).to(torch.bfloat16)
    x = torch.randn((mt, k), device=cuda_device, generator=gen).to(torch.bfloat16)
    base = torch.randn((n, k), device=cuda_device, generator=gen)
    want = base.clone()
    grad_weight_bf16(g, x, want, accumulate=True)
    grad_weight_bf16(g, x, want, accumulate=True)
    got = base.clone()
    _noalloc(g, x, got, True)
    _noalloc(g, x, got, True)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_noalloc_takes_no_device_memory(cuda_device):
    mt, n, k = 16384, 512, 512
    g = torch.randn((mt, n), device=cuda_device).to(torch.bfloat16)
    x = torch.randn((mt, k), device=cuda_device).to(torch.bfloat16)
    out = torch.empty((n, k), device=cuda_device)
    _noalloc(g, x, out, False)  # first call in this context: scratch address set-up
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    reserved_before = torch.cuda.memory_reserved()
    for _ in range(3):
        _noalloc(g, x, out, False)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_reserved() == reserved_before
    assert free_after == free_before
