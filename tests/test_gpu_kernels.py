"""GPU parity: every CUDA kernel of the C ABI against the CPU oracle on the same seeded inputs.

Bars: bit-exact for integer/byte outputs, quantised values, row scales and bf16-rounded GEMM
outputs; grad_weight (fp32 accumulation in tensor-core order) within 1e-5 relative Frobenius of a
double-precision sum (the north-star gate is 1e-2).  Full benchmark sizes are checked through exact
integer arithmetic on the device (int32 sums of int8 products are exact in fp32 below 2^24).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


# ------------------------------------------------------------------------------ quantisation
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("shape", ["67x35", "128x256", "1x513", "255x1", "300x1", "1x255"])
def test_quantize_rows_matches_reference_golden(cuda_device, dtype, shape):
    from local_ai_training_b200.int8_matmul import quantize_rows, quantize_rows_colscaled

    g = load_golden("quant_rows.npz")
    key = f"{dtype}_{shape}"
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    x = torch.from_numpy(g[f"{key}_x"]).to(cuda_device, tdt)
    q, s = quantize_rows(x)
    np.testing.assert_array_equal(_np(q), g[f"{key}_q"])
    np.testing.assert_array_equal(_np(s), g[f"{key}_s"])
    qc, sc = quantize_rows_colscaled(x, torch.from_numpy(g[f"{key}_cs"]).to(cuda_device))
    np.testing.assert_array_equal(_np(qc), g[f"{key}_qc"])
    np.testing.assert_array_equal(_np(sc), g[f"{key}_sc"])


@pytest.mark.parametrize("shape", [(16384, 512), (16384, 2048), (64, 8192), (7, 40000), (33, 1032)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quantize_rows_vector_paths_match_oracle(cuda_device, shape, dtype):
    from local_ai_training_b200.int8_matmul import quantize_rows

    torch.manual_seed(1)
    x = torch.randn(shape, device=cuda_device).to(dtype)
    q, s = quantize_rows(x)
    rows = slice(0, min(shape[0], 512))
    qo, so = O.quantize_rows(_np(x[rows]))
    np.testing.assert_array_equal(_np(q[rows]), qo)
    np.testing.assert_array_equal(_np(s[rows]), so)


def test_quantize_rows_noncontiguous(cuda_device):
    from local_ai_training_b200.int8_matmul import quantize_rows

    torch.manual_seed(11)
    base = torch.randn(70, 48, device=cuda_device, dtype=torch.bfloat16) * 2.0
    view = base.t()
    q, s = quantize_rows(view)
    qo, so = O.quantize_rows(_np(view))
    np.testing.assert_array_equal(_np(q), qo)
    np.testing.assert_array_equal(_np(s), so)


@pytest.mark.parametrize("shape", [(67, 35), (256, 512), (64, 2048), (5, 13)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stochastic_rounding_matches_philox_replica(cuda_device, shape, dtype):
    from local_ai_training_b200.int8_matmul import _quantize_rows_fused

    torch.manual_seed(5)
    g = (torch.randn(shape, device=cuda_device) * 1e-3).to(dtype)
    cs = torch.rand(shape[1], device=cuda_device) * 0.04 + 0.01
    gbf = torch.empty(shape, device=cuda_device, dtype=torch.bfloat16)
    q, s = _quantize_rows_fused(g, cs, stochastic=True, seed=7, step=3, layer=2, bf16_copy=gbf)
    qo, so = O.quantize_rows(_np(g), _np(cs), stochastic=True, seed=7, step=3, layer=2)
    np.testing.assert_array_equal(_np(q), qo)
    np.testing.assert_array_equal(_np(s), so)
    np.testing.assert_array_equal(_np(gbf), O.bf16_round(_np(g)))


@pytest.mark.parametrize("shape", [(16384, 1536), (67, 35), (3, 8)])
def test_device_step_is_read_then_advanced_by_each_call(cuda_device, shape):
    """step_dev[0] replaces `step` and each call advances it once all CTAs have read it."""
    from local_ai_training_b200.int8_matmul import _quantize_rows_fused

    torch.manual_seed(8)
    g = torch.randn(shape, device=cuda_device)
    step_dev = torch.tensor([5, 0], device=cuda_device, dtype=torch.int32)
    rows = slice(0, min(shape[0], 64))
    for step in (5, 6, 7):
        q, _ = _quantize_rows_fused(g, None, stochastic=True, seed=3, step=0, layer=1,
                                    step_dev=step_dev)
        qo, _ = O.quantize_rows(_np(g[rows]), stochastic=True, seed=3, step=step, layer=1)
        np.testing.assert_array_equal(_np(q[rows]), qo)
    assert step_dev.tolist() == [8, 0]


def test_stochastic_rounding_unbiased_over_a_million_draws(cuda_device):
    from local_ai_training_b200.int8_matmul import _quantize_rows_fused

    for value in (0.3, -1.7, 2.5):
        x = torch.full((1, 1_000_001), value, device=cuda_device)
        x[0, 0] = 4.0
        q, s = _quantize_rows_fused(x, None, stochastic=True, seed=99, step=1, layer=0)
        mean = (q[0, 1:].double() * s[0].double()).mean().item()
        assert abs(mean - value) < 0.0025 * s[0].item(), (value, mean)


# ------------------------------------------------------------------------------ int8 GEMM
@pytest.mark.parametrize("case", ["ragged", "aligned", "wide"])
def test_scaled_int8_mm_matches_reference_golden(cuda_device, case):
    from local_ai_training_b200.int8_matmul import scaled_int8_mm

    g = load_golden("scaled_mm.npz")
    dev = lambda a: torch.from_numpy(a).to(cuda_device)  # noqa: E731
    out = scaled_int8_mm(dev(g[f"{case}_lhs"]), dev(g[f"{case}_rhs"]), dev(g[f"{case}_ls"]),
                         dev(g[f"{case}_rs"]))
    assert out.dtype == torch.bfloat16
    np.testing.assert_array_equal(_np(out), g[f"{case}_out"])


@pytest.mark.parametrize("m,k,n", [(128, 128, 128), (67, 48, 53), (300, 512, 384), (129, 1024, 256),
                                   (1, 16, 1), (513, 2048, 96), (256, 4096, 520)])
@pytest.mark.parametrize("layout", ["kk", "kn", "mk", "mn"])
def test_scaled_int8_mm_tcgen05_layouts_match_oracle(cuda_device, m, k, n, layout):
    """All four operand majornesses of the tcgen05 kernel (strides decide, as in the reference)."""
    from local_ai_training_b200.int8_matmul import _scaled_int8_mm_into

    torch.manual_seed(m * 7 + k + n)
    lhs = torch.randint(-127, 128, (m, k), dtype=torch.int8)
    rhs = torch.randint(-4, 5, (k, n), dtype=torch.int8)
    ls = torch.rand(m) * 0.05 + 1e-3
    rs = torch.rand(n) * 0.05 + 5e-3
    expected, acc = O.scaled_int8_mm(lhs.numpy(), rhs.numpy(), ls.numpy(), rs.numpy(), return_acc=True)
    dl = lhs.to(cuda_device) if layout[0] == "k" else lhs.t().contiguous().to(cuda_device).t()
    dr = rhs.t().contiguous().to(cuda_device).t() if layout[1] == "k" else rhs.to(cuda_device)
    if layout[0] == "m":
        dl = lhs.t().contiguous().to(cuda_device).t()
    for out_dtype in (torch.bfloat16, torch.float32):
        out = torch.empty((m, n), device=cuda_device, dtype=out_dtype)
        _scaled_int8_mm_into(dl, dr, ls.to(cuda_device), rs.to(cuda_device), out)
        np.testing.assert_array_equal(_np(out), expected)
    # rhs_scale = None means 1.0 (the grad_input call)
    out = torch.empty((m, n), device=cuda_device, dtype=torch.bfloat16)
    _scaled_int8_mm_into(dl, dr, ls.to(cuda_device), None, out)
    np.testing.assert_array_equal(_np(out), O.scaled_int8_mm(lhs.numpy(), rhs.numpy(), ls.numpy(), None))


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_scaled_int8_mm_full_range_accumulators_round_like_oracle(cuda_device, out_dtype):
    """|acc| up to 127·127·8192 > 2^24: the int32 -> fp32 conversion of the epilogue rounds."""
    from local_ai_training_b200.int8_matmul import _scaled_int8_mm_into

    torch.manual_seed(21)
    m, k, n = 256, 8192, 384
    lhs = torch.randint(-127, 128, (m, k), dtype=torch.int8)
    lhs[:8] = 127  # rows of maximal sums against the all-127 columns below
    rhs = torch.randint(-127, 128, (k, n), dtype=torch.int8)
    rhs[:, :8] = 127
    rhs[:, 8:16] = -127
    ls = torch.rand(m) * 0.05 + 1e-3
    rs = torch.rand(n) * 0.05 + 5e-3
    expected, acc = O.scaled_int8_mm(lhs.numpy(), rhs.numpy(), ls.numpy(), rs.numpy(), return_acc=True)
    assert np.abs(acc).max() > 2**24
    out = torch.empty((m, n), device=cuda_device, dtype=out_dtype)
    _scaled_int8_mm_into(lhs.to(cuda_device), rhs.t().contiguous().to(cuda_device).t(),
                         ls.to(cuda_device), rs.to(cuda_device), out)
    np.testing.assert_array_equal(_np(out), expected)


@pytest.mark.parametrize("m,k,n,pad", [(16384, 512, 512, 0), (300, 512, 96, 0), (129, 256, 520, 0),
                                       (200, 128, 64, 3)])
@pytest.mark.parametrize("inplace", [False, True])
def test_scaled_int8_mm_residual_epilogue(cuda_device, m, k, n, pad, inplace):
    """out = residual + fp32(bf16(...)), the block's residual add in the epilogue: TMA-loaded
    residual tiles (16-byte rows) and the lane-per-row path (pad breaks the row alignment)."""
    from local_ai_training_b200.int8_matmul import _scaled_int8_mm_into

    torch.manual_seed(m + n + pad)
    lhs = torch.randint(-127, 128, (m, k), device=cuda_device, dtype=torch.int8)
    code = torch.randint(-3, 4, (n, k), device=cuda_device, dtype=torch.int8)
    ls = torch.rand(m, device=cuda_device) * 0.01 + 1e-3
    rs = torch.rand(n, device=cuda_device) * 0.05 + 5e-3
    base = torch.randn(m, n + pad, device=cuda_device)
    residual = base[:, :n]
    expected = residual + ((lhs.float() @ code.float().t()) * ls[:, None] * rs[None, :]).to(
        torch.bfloat16).float()
    if inplace:
        out = residual
        _scaled_int8_mm_into(lhs, code.t(), ls, rs, out, rhs_abs_max=7, residual=residual)
    else:
        out = torch.empty(m, n, device=cuda_device)
        _scaled_int8_mm_into(lhs, code.t(), ls, rs, out, rhs_abs_max=7, residual=residual)
    assert torch.equal(out, expected)


@pytest.mark.parametrize("bound", [0, 7])
@pytest.mark.parametrize("k,n", [(512, 512), (512, 2048), (2048, 512), (4096, 256)])
def test_scaled_int8_mm_full_size_exact(cuda_device, k, n, bound):
    """The 25M model's layer shapes, M = 16384: exact integer sums on the device as the checker;
    bound = 7 (the codes' bound) takes the 2-op accumulator conversion up to K·128·7 < 2^22."""
    from local_ai_training_b200.int8_matmul import _scaled_int8_mm_into, quantize_rows

    torch.manual_seed(1337)
    a = torch.randn(16384, k, device=cuda_device, dtype=torch.bfloat16)
    q, s = quantize_rows(a)
    code = torch.randint(-3, 4, (n, k), device=cuda_device, dtype=torch.int8)
    scale = torch.rand(n, device=cuda_device) * 0.045 + 0.005
    out = torch.empty((16384, n), device=cuda_device, dtype=torch.bfloat16)
    q[:4] = -128 if k == 4096 else q[:4]  # extreme sums near the conversion bound
    code[:4] = 7 if k == 4096 else code[:4]
    _scaled_int8_mm_into(q, code.t(), s, scale, out, rhs_abs_max=bound)
    acc = q.float() @ code.float().t()  # exact: |acc| <= 128*7*4096 < 2^24
    expected = ((acc * s[:, None]) * scale[None, :]).to(torch.bfloat16)
    assert torch.equal(out, expected)
    # grad_input form: B = code (MN-major), no column scale
    gi = torch.empty((16384, k), device=cuda_device, dtype=torch.bfloat16)
    gq = torch.randint(-127, 128, (16384, n), device=cuda_device, dtype=torch.int8)
    _scaled_int8_mm_into(gq, code, s, None, gi, rhs_abs_max=bound)
    acc2 = gq.float() @ code.float()
    assert torch.equal(gi, (acc2 * s[:, None]).to(torch.bfloat16))


# ------------------------------------------------------------------------------ grad_weight
@pytest.mark.parametrize("mt,n,k", [(64, 128, 256), (1000, 200, 72), (16384, 512, 512),
                                    (4096, 2048, 512), (300, 16, 16), (33, 11, 16)])
def test_grad_weight_matches_double_sum(cuda_device, mt, n, k):
    from local_ai_training_b200.int8_matmul import grad_weight_bf16

    torch.manual_seed(mt + n + k)
    g = (torch.randn(mt, n, device=cuda_device) * 1e-2).to(torch.bfloat16)
    x = torch.randn(mt, k, device=cuda_device).to(torch.bfloat16)
    gw = grad_weight_bf16(g, x)
    ref = (g.double().t() @ x.double()).float()
    rel = ((gw - ref).norm() / ref.norm()).item()
    assert rel < 1e-5, rel
    # accumulate = True adds a second pass on top
    gw2 = grad_weight_bf16(g, x, out=gw.clone(), accumulate=True)
    rel2 = ((gw2 - 2 * ref).norm() / (2 * ref).norm()).item()
    assert rel2 < 1e-5, rel2


def test_grad_weight_small_matches_oracle(cuda_device):
    from local_ai_training_b200.int8_matmul import grad_weight_bf16

    torch.manual_seed(3)
    g = torch.randn(40, 48, device=cuda_device).to(torch.bfloat16)
    x = torch.randn(40, 32, device=cuda_device).to(torch.bfloat16)
    gw = grad_weight_bf16(g, x)
    ref = O.grad_weight(_np(g), _np(x))
    np.testing.assert_allclose(_np(gw), ref, rtol=1e-5, atol=1e-5)


def test_dequant_matches_oracle(cuda_device):
    from local_ai_training_b200.int8_matmul import dequant_rows_bf16

    torch.manual_seed(2)
    for shape in ((16384, 512), (37, 29)):
        q = torch.randint(-127, 128, shape, device=cuda_device, dtype=torch.int8)
        s = torch.rand(shape[0], device=cuda_device) * 0.1 + 1e-3
        out = dequant_rows_bf16(q, s)
        np.testing.assert_array_equal(_np(out[:300]), O.dequant_rows(_np(q[:300]), _np(s[:300])))


# ------------------------------------------------------------------------------ ratchet update
def _update_gpu(grad, packed, *, max_code, threshold=8, low=0.5, high=1.5, eps=1e-8,
                normalize=True, round_bf16=False, ema=None, beta=0.0, want_gs=False):
    from local_ai_training_b200 import _lib

    rows, cols = packed.shape
    dev = grad.device
    pk = packed.clone()
    code = torch.empty_like(pk, dtype=torch.int8)
    counts = torch.zeros(4, device=dev, dtype=torch.int64)
    row_rms = torch.empty(rows, device=dev)
    rms_sum = torch.zeros(1, device=dev)
    gs = torch.empty(rows, device=dev) if want_gs else None
    ema_t = None if ema is None else ema.clone()
    _lib.check(_lib.lib().rt_ratchet_update(
        grad.data_ptr(), _lib.dtype_code(grad), int(round_bf16), grad.stride(0), rows, cols,
        pk.data_ptr(), pk.stride(0), code.data_ptr(), code.stride(0), int(normalize),
        None if ema_t is None else ema_t.data_ptr(), beta, max_code, threshold, low, high, eps,
        counts.data_ptr(), row_rms.data_ptr(), rms_sum.data_ptr(),
        None if gs is None else gs.data_ptr(), _lib.stream_of(grad)))
    return dict(packed=pk, code=code, counts=counts, row_rms=row_rms, rms_ema=ema_t, grad_scale=gs,
                rms_sum=rms_sum)


@pytest.mark.parametrize("m,rows,cols", [(16384, 512, 512), (16384, 1536, 512), (4096, 8192, 512),
                                          (300, 200, 136), (16384, 512, 2048)])
@pytest.mark.parametrize("ema", [False, True])
def test_grad_weight_update_equals_gemm_then_update(cuda_device, m, rows, cols, ema):
    """rt_grad_weight_ratchet_update (grad_W from split-K partial tiles, never stored) gives the
    update that rt_grad_weight_bf16 followed by rt_ratchet_update(round_bf16=1) gives."""
    from local_ai_training_b200 import _lib
    from local_ai_training_b200.int8_matmul import grad_weight_bf16

    torch.manual_seed(m + rows + cols)
    max_code = 2
    g = (torch.randn(m, rows, device=cuda_device) * 1e-3).to(torch.bfloat16)
    x = torch.randn(m, cols, device=cuda_device).to(torch.bfloat16)
    code = torch.randint(-max_code, max_code + 1, (rows, cols))
    pressure = torch.randint(-7, 8, (rows, cols))
    packed = torch.from_numpy(O.pack_code_pressure(code.numpy(), pressure.numpy(), max_code))
    packed = packed.to(cuda_device)
    ema0 = torch.rand(rows, device=cuda_device) * 1e-6 if ema else None
    beta = 0.9 if ema else 0.0
    gw = grad_weight_bf16(g, x)
    ref = _update_gpu(gw, packed, max_code=max_code, round_bf16=True, ema=ema0, beta=beta,
                      want_gs=True)
    pk = packed.clone()
    mirror = torch.empty_like(pk, dtype=torch.int8)
    counts = torch.zeros(4, device=cuda_device, dtype=torch.int64)
    rms_sum = torch.zeros(1, device=cuda_device)
    row_rms = torch.empty(rows, device=cuda_device)
    gs = torch.empty(rows, device=cuda_device)
    ema_t = None if ema0 is None else ema0.clone()
    need = _lib.lib().rt_grad_weight_update_workspace_bytes(m, rows, cols)
    ws = torch.empty(need, device=cuda_device, dtype=torch.uint8)
    _lib.check(_lib.lib().rt_grad_weight_ratchet_update(
        g.data_ptr(), g.stride(0), x.data_ptr(), x.stride(0), m, rows, cols, ws.data_ptr(), need,
        pk.data_ptr(), pk.stride(0), mirror.data_ptr(), mirror.stride(0),
        None if ema_t is None else ema_t.data_ptr(), beta, max_code, 8, 0.5, 1.5, 1e-8,
        counts.data_ptr(), row_rms.data_ptr(), rms_sum.data_ptr(), gs.data_ptr(),
        _lib.stream_of(g)))
    assert torch.equal(pk, ref["packed"])
    assert torch.equal(mirror, ref["code"])
    assert torch.equal(counts, ref["counts"])
    assert torch.equal(row_rms, ref["row_rms"])
    assert torch.equal(gs, ref["grad_scale"])
    if ema:
        assert torch.equal(ema_t, ref["rms_ema"])
    torch.testing.assert_close(rms_sum, ref["rms_sum"], rtol=1e-5, atol=0)


@pytest.mark.parametrize("idx", range(7))
def test_update_matches_oracle_bit_exact(cuda_device, idx):
    g = load_golden("update_random.npz")
    rows, cols, max_code, thr = (int(v) for v in g[f"c{idx}_meta"])
    low, high, beta = (float(v) for v in g[f"c{idx}_fmeta"])
    ema0 = g.get(f"c{idx}_ema0")
    grad = torch.from_numpy(g[f"c{idx}_grad"]).to(cuda_device)
    packed = torch.from_numpy(g[f"c{idx}_packed0"]).to(cuda_device)
    out = _update_gpu(grad, packed, max_code=max_code, threshold=thr, low=low, high=high,
                      ema=None if ema0 is None else torch.from_numpy(ema0).to(cuda_device),
                      beta=beta, want_gs=True)
    ref = O.ratchet_update(g[f"c{idx}_grad"], g[f"c{idx}_packed0"], max_code=max_code,
                           threshold=thr, bucket_low=low, bucket_high=high, rms_ema=ema0, beta=beta,
                           want_grad_scale=True)
    np.testing.assert_array_equal(_np(out["packed"]), ref["packed"])
    np.testing.assert_array_equal(_np(out["code"]), ref["code"])
    np.testing.assert_array_equal(_np(out["counts"]), ref["counts"])
    np.testing.assert_array_equal(_np(out["row_rms"]), ref["row_rms"])
    np.testing.assert_array_equal(_np(out["grad_scale"]), ref["grad_scale"])
    np.testing.assert_allclose(_np(out["rms_sum"])[0], ref["row_rms"].astype(np.float64).sum(),
                               rtol=1e-5)
    if beta > 0:
        np.testing.assert_array_equal(_np(out["rms_ema"]), ref["rms_ema"])
    # and against the reference's own result (reduction order may flip a boundary weight)
    assert int((_np(out["packed"]) != g[f"c{idx}_packed1"]).sum()) <= max(1, rows * cols // 100_000)


@pytest.mark.parametrize("rows,cols", [(512, 512), (2048, 512), (512, 2048), (64, 8192), (8, 12000),
                                       (3, 5)])
@pytest.mark.parametrize("grad_dtype", [torch.float32, torch.bfloat16])
def test_update_shapes_match_oracle(cuda_device, rows, cols, grad_dtype):
    torch.manual_seed(rows + cols)
    max_code = 2
    grad = (torch.randn(rows, cols, device=cuda_device) * 1e-3).to(grad_dtype)
    code = torch.randint(-max_code, max_code + 1, (rows, cols))
    pressure = torch.randint(-7, 8, (rows, cols))
    packed = torch.from_numpy(O.pack_code_pressure(code.numpy(), pressure.numpy(), max_code))
    for round_bf16 in (False, True):
        out = _update_gpu(grad, packed.to(cuda_device), max_code=max_code, round_bf16=round_bf16)
        ref = O.ratchet_update(_np(grad), packed.numpy(), max_code=max_code, round_bf16=round_bf16)
        np.testing.assert_array_equal(_np(out["packed"]), ref["packed"])
        np.testing.assert_array_equal(_np(out["counts"]), ref["counts"])


def test_update_golden_trajectory_on_gpu(cuda_device):
    g = load_golden("update_golden.npz")
    for max_code in (2, 3, 4):
        packed = torch.from_numpy(g[f"mc{max_code}_packed0"]).to(cuda_device)
        for step in range(60):
            grad = torch.from_numpy(g[f"mc{max_code}_grads"][step]).to(cuda_device)
            out = _update_gpu(grad, packed, max_code=max_code, normalize=False)
            packed = out["packed"]
            np.testing.assert_array_equal(_np(packed), g[f"mc{max_code}_packs"][step])
            np.testing.assert_array_equal(_np(out["counts"]), g[f"mc{max_code}_moves"][step])


def test_update_skips_nonfinite_rows_and_flags(cuda_device):
    from local_ai_training_b200 import _lib

    _lib.device_status(cuda_device, clear=True)
    grad = torch.ones(4, 64, device=cuda_device)
    grad[2, 5] = float("nan")
    packed = torch.full((4, 64), 0x72, device=cuda_device, dtype=torch.uint8)
    out = _update_gpu(grad, packed, max_code=2)
    assert torch.equal(out["packed"][2], packed[2])
    status = _lib.device_status(cuda_device, clear=True)
    assert status & _lib.STATUS_NONFINITE_GRADIENT


def test_leak_unpack_validate(cuda_device):
    from local_ai_training_b200 import _lib
    from local_ai_training_b200.ratchet import unpack_code_pressure

    rng = np.random.default_rng(4)
    code = rng.integers(-3, 4, (33, 70))
    pressure = rng.integers(-7, 8, (33, 70))
    packed_np = O.pack_code_pressure(code, pressure, 3)
    pk = torch.from_numpy(packed_np).to(cuda_device)
    c, p = unpack_code_pressure(pk, 3)
    np.testing.assert_array_equal(_np(c), code)
    np.testing.assert_array_equal(_np(p), pressure)
    _lib.check(_lib.lib().rt_ratchet_leak(pk.data_ptr(), pk.stride(0), 33, 70, 3, _lib.stream_of(pk)))
    np.testing.assert_array_equal(_np(pk), O.ratchet_leak(packed_np))
    _lib.device_status(cuda_device, clear=True)
    scale = torch.ones(33, device=cuda_device)
    _lib.check(_lib.lib().rt_ratchet_validate(pk.data_ptr(), pk.stride(0), 33, 70, 3,
                                              scale.data_ptr(), _lib.stream_of(pk)))
    assert _lib.device_status(cuda_device, clear=True) == 0
    pk[0, 0] = 0xFF  # pressure +8, code 12 > 3
    scale[3] = -1.0
    _lib.check(_lib.lib().rt_ratchet_validate(pk.data_ptr(), pk.stride(0), 33, 70, 3,
                                              scale.data_ptr(), _lib.stream_of(pk)))
    status = _lib.device_status(cuda_device, clear=True)
    assert status & _lib.STATUS_CODE_RANGE and status & _lib.STATUS_PRESSURE_RANGE
    assert status & _lib.STATUS_SCALE_INVALID


# ------------------------------------------------------------------------------ producers
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rmsnorm_quantize_matches_oracle(cuda_device, dtype):
    from local_ai_training_b200.int8_fused import fused_rmsnorm_quantize

    torch.manual_seed(8)
    x = torch.randn(300, 512, device=cuda_device).to(dtype)
    w = torch.rand(512, device=cuda_device) + 0.5
    q, s = fused_rmsnorm_quantize(x, w, 1e-5)
    qo, so = O.rmsnorm_quantize(_np(x), _np(w), 1e-5)
    np.testing.assert_array_equal(_np(q), qo)
    np.testing.assert_array_equal(_np(s), so)


def test_gelu_quantize_matches_oracle(cuda_device):
    from local_ai_training_b200.int8_fused import fused_gelu_quantize

    torch.manual_seed(9)
    x = torch.randn(256, 2048, device=cuda_device) * 2
    q, s = fused_gelu_quantize(x)
    qo, so = O.gelu_quantize(_np(x))
    # tanhf of CUDA and of the C library may differ by an ulp: allow rare one-step differences
    np.testing.assert_allclose(_np(s), so, rtol=1e-6)
    diff = np.abs(_np(q).astype(np.int32) - qo.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-3


def test_transpose_quantize_matches_oracle(cuda_device):
    from local_ai_training_b200.int8_fused import fused_transpose_quantize

    torch.manual_seed(10)
    x = torch.randn(4, 8, 128, 64, device=cuda_device, dtype=torch.bfloat16)
    q, s = fused_transpose_quantize(x)
    qo, so = O.transpose_quantize(_np(x))
    np.testing.assert_array_equal(_np(q), qo)
    np.testing.assert_array_equal(_np(s), so)


@pytest.mark.parametrize("kind", ["rmsnorm", "gelu", "transpose"])
@pytest.mark.parametrize("width", [512, 2048, 100])  # 100: the generic one-CTA-per-row kernels
def test_producer_dequant_copy_equals_dequant_pass(cuda_device, kind, width):
    """The bf16 rows a producer writes beside its int8 output are exactly what the backward's
    dequant pass makes of them: bf16(bf16(q) * bf16(s))."""
    from local_ai_training_b200.int8_fused import (fused_gelu_quantize, fused_rmsnorm_quantize,
                                                   fused_transpose_quantize)
    from local_ai_training_b200.int8_matmul import dequant_rows_bf16

    torch.manual_seed(width)
    if kind == "rmsnorm":
        x = torch.randn(333, width, device=cuda_device)
        w = torch.rand(width, device=cuda_device) + 0.5
        q, s, dq = fused_rmsnorm_quantize(x, w, 1e-5, dequant_out=True)
        q2, s2 = fused_rmsnorm_quantize(x, w, 1e-5)
    elif kind == "gelu":
        x = (torch.randn(333, width, device=cuda_device) * 2).to(torch.bfloat16)
        q, s, dq = fused_gelu_quantize(x, dequant_out=True)
        q2, s2 = fused_gelu_quantize(x)
    else:
        heads = 4 if width % 4 == 0 else 2
        x = torch.randn(3, heads, 111, width // heads, device=cuda_device, dtype=torch.bfloat16)
        q, s, dq = fused_transpose_quantize(x, dequant_out=True)
        q2, s2 = fused_transpose_quantize(x)
    assert torch.equal(q, q2) and torch.equal(s, s2)
    q = q.reshape(-1, q.shape[-1])
    assert dq.dtype == torch.bfloat16 and dq.shape == q.shape
    assert torch.equal(dq, dequant_rows_bf16(q, s.reshape(-1)))


def test_producer_backwards_match_oracle(cuda_device):
    from local_ai_training_b200.int8_backward import gelu_backward, rmsnorm_backward

    torch.manual_seed(12)
    x = torch.randn(64, 512, device=cuda_device)
    gy = torch.randn(64, 512, device=cuda_device) * 1e-2
    w = torch.rand(512, device=cuda_device) + 0.5
    dx, dw = rmsnorm_backward(gy, x, w, 1e-5)
    np.testing.assert_allclose(_np(dx), O.rmsnorm_backward(_np(gy), _np(x), _np(w), 1e-5),
                               rtol=1e-2, atol=1e-6)
    ref_dw = (gy.double() * x.double() * torch.rsqrt((x.double() ** 2).mean(1, keepdim=True) + 1e-5)).sum(0)
    torch.testing.assert_close(dw.double(), ref_dw, rtol=1e-4, atol=1e-6)
    dg = gelu_backward(gy, x)
    np.testing.assert_allclose(_np(dg), O.gelu_backward(_np(gy), _np(x)), rtol=1e-2, atol=1e-6)


@pytest.mark.parametrize("rows,cols,dtype", [(16384, 512, torch.float32), (16384, 2048, torch.float32),
                                             (16384, 512, torch.bfloat16), (300, 100, torch.float32)])
def test_rmsnorm_weight_gradient_is_deterministic(cuda_device, rows, cols, dtype):
    """dw sums per-CTA partial rows in a fixed order (the 100-wide rows take the generic kernel's
    per-column sum over rows): repeated calls give the same bits, close to a double sum."""
    from local_ai_training_b200.int8_backward import rmsnorm_backward

    torch.manual_seed(rows + cols)
    x = torch.randn(rows, cols, device=cuda_device).to(dtype)
    gy = (torch.randn(rows, cols, device=cuda_device) * 1e-2).to(dtype)
    w = torch.rand(cols, device=cuda_device) + 0.5
    dws = [rmsnorm_backward(gy, x, w, 1e-5)[1] for _ in range(3)]
    for other in dws[1:]:
        assert torch.equal(dws[0], other)
    xd, gd = x.double(), gy.double()
    ref = (gd * xd * torch.rsqrt((xd ** 2).mean(1, keepdim=True) + 1e-5)).sum(0)
    torch.testing.assert_close(dws[0].double(), ref, rtol=1e-4, atol=1e-5)
