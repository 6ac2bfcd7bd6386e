"""GPU: the boundary cases of the staged row kernels against the CPU oracle, bit for bit.

The stochastic-rounding quantiser decides most elements in fixed point and re-does those within
a few 2^-16 units of an integer (and whole rows with a tiny or zero maximum) by the IEEE
division; the update compares each |g| with per-row thresholds found by a ballot over adjacent
floats.  These tests put many elements exactly on, or one unit either side of, those decision
points, and run the rows whose thresholds or scales leave the ranges the fast paths cover.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SEED, STEP, LAYER = 12345, 9, 4


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def _edge_rows(cols: int, rng: np.random.Generator, *, probes: bool) -> np.ndarray:
    """Rows of a quantiser input: zero, tiny-maximum, subnormal, single-element, scale-multiple
    rows, then (probes) rows whose every element lands on a stochastic-rounding decision point."""
    rows = [np.zeros(cols, np.float32),
            (rng.standard_normal(cols) * 1e-31).astype(np.float32),
            (rng.standard_normal(cols) * 1e-39).astype(np.float32)]
    single = np.zeros(cols, np.float32)
    single[cols // 3] = -3.5
    rows.append(single)
    mult = (rng.integers(-127, 128, cols) * 2.0**-7).astype(np.float32)
    mult[0] = 127 * 2.0**-7
    rows.append(mult)
    huge = (rng.standard_normal(cols) * 1e30).astype(np.float32)
    rows.append(huge)
    if probes:
        # scale 2^-7 (amax 127/128 at column 0); element c of row r holds (k - u + j·2^-17)·2^-7
        # with u its own draw, so RN(v/scale) + u = k + j·2^-17 exactly: an integer (j = 0) or
        # 1-3 units of 2^-17 either side of one
        for _ in range(6):
            r = len(rows)
            u = np.array([O.sr_uniform(SEED, STEP, LAYER, r * cols + c) for c in range(cols)])
            k = rng.integers(-126, 127, cols).astype(np.float64)
            j = rng.integers(-3, 4, cols).astype(np.float64)
            v = ((k - u + j * 2.0**-17) * 2.0**-7).astype(np.float32)
            assert np.array_equal(v.astype(np.float64), (k - u + j * 2.0**-17) * 2.0**-7)
            v[0] = 127 * 2.0**-7
            rows.append(v)
    return np.stack(rows)


@pytest.mark.parametrize("cols", [512, 1032, 2048, 6144, 8192])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("colscale", [False, True])
def test_stochastic_rounding_edge_rows(cuda_device, cols, dtype, colscale):
    from local_ai_training_b200.int8_matmul import _quantize_rows_fused

    rng = np.random.default_rng(cols)
    probes = dtype == torch.float32 and not colscale
    edge = _edge_rows(cols, rng, probes=probes)
    rand = (rng.standard_normal((300, cols)) * 1e-3).astype(np.float32)
    x = np.concatenate([edge, rand])
    xt = torch.from_numpy(x).to(cuda_device, dtype)
    xv = _np(xt)  # the values the kernel sees (bf16-rounded for bf16)
    cs = (rng.random(cols) * 0.04 + 0.01).astype(np.float32) if colscale else None
    cst = None if cs is None else torch.from_numpy(cs).to(cuda_device)
    copy = torch.empty(x.shape, device=cuda_device, dtype=torch.bfloat16)
    q, s = _quantize_rows_fused(xt, cst, stochastic=True, seed=SEED, step=STEP, layer=LAYER,
                                bf16_copy=copy)
    qo, so = O.quantize_rows(xv, cs, stochastic=True, seed=SEED, step=STEP, layer=LAYER)
    np.testing.assert_array_equal(_np(s), so)
    np.testing.assert_array_equal(_np(q), qo)
    np.testing.assert_array_equal(_np(copy), O.bf16_round(xv))


@pytest.mark.parametrize("cols", [512, 2048])
def test_stochastic_rounding_fp32_rounded_to_bf16_first(cuda_device, cols):
    """The residual-stream gradients: fp32 in, rounded to bf16, the bf16 copy written."""
    from local_ai_training_b200.int8_matmul import _quantize_rows_fused

    rng = np.random.default_rng(7 + cols)
    x = np.concatenate([_edge_rows(cols, rng, probes=False),
                        (rng.standard_normal((500, cols)) * 1e-2).astype(np.float32)])
    cs = (rng.random(cols) * 0.04 + 0.01).astype(np.float32)
    xt = torch.from_numpy(x).to(cuda_device)
    copy = torch.empty(x.shape, device=cuda_device, dtype=torch.bfloat16)
    q, s = _quantize_rows_fused(xt, torch.from_numpy(cs).to(cuda_device), stochastic=True,
                                seed=SEED, step=STEP, layer=LAYER, bf16_copy=copy,
                                round_input_bf16=True)
    xr = O.bf16_round(x)
    qo, so = O.quantize_rows(xr, cs, stochastic=True, seed=SEED, step=STEP, layer=LAYER)
    np.testing.assert_array_equal(_np(s), so)
    np.testing.assert_array_equal(_np(q), qo)
    np.testing.assert_array_equal(_np(copy), xr)


@pytest.mark.parametrize("shape,dtype", [((16384, 2048), torch.bfloat16),
                                         ((16384, 512), torch.float32),
                                         ((2048, 8192), torch.bfloat16),
                                         ((4096, 6144), torch.bfloat16)])
def test_stochastic_rounding_full_size_matches_oracle(cuda_device, shape, dtype):
    """Every row of a step-sized gradient (the grid-stride loop and its staging ring)."""
    from local_ai_training_b200.int8_matmul import _quantize_rows_fused

    torch.manual_seed(shape[1])
    x = (torch.randn(shape, device=cuda_device) * 1e-3).to(dtype)
    cs = torch.rand(shape[1], device=cuda_device) * 0.04 + 0.01
    q, s = _quantize_rows_fused(x, cs, stochastic=True, seed=SEED, step=STEP, layer=LAYER)
    qo, so = O.quantize_rows(_np(x), _np(cs), stochastic=True, seed=SEED, step=STEP, layer=LAYER)
    np.testing.assert_array_equal(_np(s), so)
    np.testing.assert_array_equal(_np(q), qo)


# ------------------------------------------------------------------------------------ update
def _update_case(rows: int, cols: int, rng: np.random.Generator) -> np.ndarray:
    """Gradient rows for the threshold search: every row's magnitudes lie within a few ulps of
    one value m, so |g| / rms sits on the bucket bounds 1 and 1 + 2^-22 for most elements;
    plus zero, subnormal, overflowing (sum of squares inf) and ordinary rows."""
    g = np.empty((rows, cols), np.float32)
    for r in range(rows):
        kind = r % 8
        if kind == 0:
            g[r] = 0.0
        elif kind == 1:
            g[r] = (rng.standard_normal(cols) * 1e-40).astype(np.float32)
        elif kind == 2:
            g[r] = (rng.standard_normal(cols) * 1e25).astype(np.float32)
        elif kind == 3:
            g[r] = (rng.standard_normal(cols) * 1e-3).astype(np.float32)
        else:
            m = np.float32(2.0 ** rng.integers(-20, 4)) * np.float32(1 + rng.random())
            k = rng.integers(-6, 7, cols)
            mag = (m.astype(np.float64) * (1 + k * 2.0**-23)).astype(np.float32)
            g[r] = np.where(rng.random(cols) < 0.5, -mag, mag)
    return g


@pytest.mark.parametrize("cols", [136, 512, 2048, 8192])
@pytest.mark.parametrize("grad_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("low,high,beta", [(1.0, 1.0 + 2.0**-22, 0.0), (0.0, 1.0, 0.0),
                                           (0.5, 1.5, 0.9)])
def test_update_threshold_edges_match_oracle(cuda_device, cols, grad_dtype, low, high, beta):
    from tests.test_gpu_kernels import _update_gpu

    rng = np.random.default_rng(cols + int(low * 10))
    rows = 96
    max_code = 3
    g = _update_case(rows, cols, rng)
    gt = torch.from_numpy(g).to(cuda_device, grad_dtype)
    code = rng.integers(-max_code, max_code + 1, (rows, cols))
    pressure = rng.integers(-7, 8, (rows, cols))
    packed = O.pack_code_pressure(code, pressure, max_code)
    ema0 = (rng.random(rows) * 1e-4).astype(np.float32) if beta > 0 else None
    out = _update_gpu(gt, torch.from_numpy(packed).to(cuda_device), max_code=max_code,
                      threshold=2, low=low, high=high,
                      ema=None if ema0 is None else torch.from_numpy(ema0).to(cuda_device),
                      beta=beta, want_gs=True)
    ref = O.ratchet_update(_np(gt), packed, max_code=max_code, threshold=2, bucket_low=low,
                           bucket_high=high, rms_ema=ema0, beta=beta, want_grad_scale=True)
    np.testing.assert_array_equal(_np(out["packed"]), ref["packed"])
    np.testing.assert_array_equal(_np(out["code"]), ref["code"])
    np.testing.assert_array_equal(_np(out["counts"]), ref["counts"])
    np.testing.assert_array_equal(_np(out["row_rms"]), ref["row_rms"])
    np.testing.assert_array_equal(_np(out["grad_scale"]), ref["grad_scale"])
    if beta > 0:
        np.testing.assert_array_equal(_np(out["rms_ema"]), ref["rms_ema"])


def test_grouped_update_edges_with_gradient_multiplier(cuda_device):
    """The grouped launch over layers of two row counts, each gradient scaled by its grad_mul
    (a power of two: exact), against the oracle on the scaled gradients."""
    import ctypes

    from local_ai_training_b200 import _lib

    rng = np.random.default_rng(3)
    cols, max_code = 2048, 3
    layers, keep = [], []
    for rows, mul in ((96, 0.25), (40, 1.0), (200, 0.5)):
        g = _update_case(rows, cols, rng)
        gt = torch.from_numpy(g).to(cuda_device, torch.bfloat16)
        code = rng.integers(-max_code, max_code + 1, (rows, cols))
        pressure = rng.integers(-7, 8, (rows, cols))
        packed = O.pack_code_pressure(code, pressure, max_code)
        pk = torch.from_numpy(packed).to(cuda_device)
        cd = torch.empty_like(pk, dtype=torch.int8)
        counts = torch.zeros(4, device=cuda_device, dtype=torch.int64)
        rsum = torch.zeros(1, device=cuda_device)
        keep.append((gt, packed, pk, cd, counts, rsum, mul))
        layers.append(_lib.UpdateLayer(gt.data_ptr(), gt.stride(0), rows, pk.data_ptr(),
                                       pk.stride(0), cd.data_ptr(), cd.stride(0), None,
                                       counts.data_ptr(), rsum.data_ptr(), mul))
    arr = (_lib.UpdateLayer * len(layers))(*layers)
    _lib.check(_lib.lib().rt_ratchet_update_grouped(
        ctypes.cast(arr, ctypes.c_void_p), len(layers), _lib.dtype_code(keep[0][0]), 0, cols, 1,
        0.0, max_code, 2, 1.0, 1.0 + 2.0**-22, 1e-8, _lib.stream_of(keep[0][0])))
    for gt, packed, pk, cd, counts, rsum, mul in keep:
        ref = O.ratchet_update(_np(gt) * np.float32(mul), packed, max_code=max_code, threshold=2,
                               bucket_low=1.0, bucket_high=1.0 + 2.0**-22)
        np.testing.assert_array_equal(_np(pk), ref["packed"])
        np.testing.assert_array_equal(_np(cd), ref["code"])
        np.testing.assert_array_equal(_np(counts), ref["counts"])
        np.testing.assert_allclose(_np(rsum)[0], ref["row_rms"].astype(np.float64).sum(),
                                   rtol=1e-5)


@pytest.mark.parametrize("rows,cols,dtype", [(4096, 8192, torch.bfloat16), (1000, 6144, torch.bfloat16),
                                             (333, 512, torch.bfloat16), (300, 136, torch.float32)])
def test_gelu_quantize_staged_equals_generic_kernel(cuda_device, rows, cols, dtype):
    """The GELU -> int8 producer on 16-byte rows (staged for wide rows, one row group per CTA
    otherwise) against the one-CTA-per-row kernel that a row stride off the 16-byte grid selects,
    on the same values: int8 rows, scales and the bf16 dequantised copy bit for bit."""
    from local_ai_training_b200.int8_fused import fused_gelu_quantize

    torch.manual_seed(cols)
    base = (torch.randn(rows, cols + 1, device=cuda_device) * 2).to(dtype)
    ragged = base[:, :cols]  # row stride cols + 1
    packed = ragged.contiguous()
    q1, s1, d1 = fused_gelu_quantize(packed, dequant_out=True)
    q2, s2, d2 = fused_gelu_quantize(ragged, dequant_out=True)
    assert torch.equal(s1, s2)
    assert torch.equal(q1, q2)
    assert torch.equal(d1, d2)
