"""GPU parity at the ~1B decoder's layer shapes (d 2048, MLP 8192, vocab 8192, M = 16384 tokens
per micro-batch, septenary codes), the grouped update, the grad_W addend epilogue and the
deferred / accumulated update runtime.

Bars: bit-exact for int8 GEMM outputs (exact integer sums on the device as the checker), packed
states, code mirrors and move counters; grad_weight within 1e-5 relative Frobenius of a double
sum (5e-5 for the 16384-term sums of the 1B shapes); the accumulated step bit-identical to one
step on the same gradient total.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

M = 16384
MAX_CODE = 3  # septenary
GEMM_SHAPES = [(2048, 6144), (2048, 2048), (2048, 8192), (8192, 2048)]  # (in K, out N)


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def _packed(rows: int, cols: int, seed: int, max_code: int = MAX_CODE) -> torch.Tensor:
    rng = np.random.default_rng(seed)
    code = rng.integers(-max_code, max_code + 1, (rows, cols))
    pressure = rng.integers(-7, 8, (rows, cols))
    return torch.from_numpy(O.pack_code_pressure(code, pressure, max_code))


# ------------------------------------------------------------------------------ int8 GEMMs
@pytest.mark.parametrize("k,n", GEMM_SHAPES, ids=[f"{k}to{n}" for k, n in GEMM_SHAPES])
@pytest.mark.parametrize("bound", [0, MAX_CODE])
def test_gemm_1b_shapes_exact(cuda_device, k, n, bound):
    """Forward (q · codeᵀ, row x column scales) and grad_input (g_q · code, row scale) at the 1B
    layer shapes: |acc| <= 127·3·8192 < 2^24, so the fp32 device matmul of the int8 values is
    the exact integer sum."""
    from local_ai_training_b200.int8_matmul import _scaled_int8_mm_into, quantize_rows

    torch.manual_seed(1338 + k + n)
    a = torch.randn(M, k, device=cuda_device, dtype=torch.bfloat16)
    q, s = quantize_rows(a)
    code = torch.randint(-MAX_CODE, MAX_CODE + 1, (n, k), device=cuda_device, dtype=torch.int8)
    scale = torch.rand(n, device=cuda_device) * 0.045 + 0.005
    out = torch.empty((M, n), device=cuda_device, dtype=torch.bfloat16)
    _scaled_int8_mm_into(q, code.t(), s, scale, out, rhs_abs_max=bound)
    acc = q.float() @ code.float().t()
    assert torch.equal(out, ((acc * s[:, None]) * scale[None, :]).to(torch.bfloat16))
    del acc, out
    gq = torch.randint(-127, 128, (M, n), device=cuda_device, dtype=torch.int8)
    gs = torch.rand(M, device=cuda_device) * 1e-4 + 1e-6
    gi = torch.empty((M, k), device=cuda_device, dtype=torch.bfloat16)
    _scaled_int8_mm_into(gq, code, gs, None, gi, rhs_abs_max=bound)
    acc2 = gq.float() @ code.float()
    assert torch.equal(gi, (acc2 * gs[:, None]).to(torch.bfloat16))


# ------------------------------------------------------------------------------ grad_weight
@pytest.mark.parametrize("n,k", [(8192, 2048), (2048, 8192), (6144, 2048), (2048, 2048)])
def test_grad_weight_1b_shapes_match_double_sum(cuda_device, n, k):
    from local_ai_training_b200.int8_matmul import grad_weight_bf16

    torch.manual_seed(n + k)
    g = (torch.randn(M, n, device=cuda_device) * 1e-3).to(torch.bfloat16)
    x = torch.randn(M, k, device=cuda_device).to(torch.bfloat16)
    for out_dtype in (torch.float32, torch.bfloat16):
        gw = grad_weight_bf16(g, x, out=torch.empty(n, k, device=cuda_device, dtype=out_dtype))
        ref = g.double().t() @ x.double()
        rel = ((gw.double() - ref).norm() / ref.norm()).item()
        # 16384-term fp32 sums in tensor-core order: ~2e-5 relative (north-star gate 1e-2)
        assert rel < (5e-5 if out_dtype == torch.float32 else 4e-3), (out_dtype, rel)


@pytest.mark.parametrize("mt,n,k", [(16384, 2048, 2048), (16384, 512, 512), (1000, 300, 72),
                                    (0, 64, 32)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_grad_weight_addend_equals_add_then_round(cuda_device, mt, n, k, out_dtype):
    """out = round(addend + gᵀx): the micro-batch accumulation's last GEMM, on the split-K path
    (512 x 512), the one-pass path (2048 x 2048), ragged tiles and an empty token dimension."""
    from local_ai_training_b200.int8_matmul import grad_weight_bf16

    torch.manual_seed(mt + n + k)
    g = (torch.randn(mt, n, device=cuda_device) * 1e-3).to(torch.bfloat16)
    x = torch.randn(mt, k, device=cuda_device).to(torch.bfloat16)
    addend = torch.randn(n, k, device=cuda_device) * 1e-2
    gw = grad_weight_bf16(g, x)  # fp32, the same GEMM
    want = (addend + gw).to(out_dtype)
    got = torch.full((n, k), float("nan"), device=cuda_device, dtype=out_dtype)
    grad_weight_bf16(g, x, out=got, addend=addend)
    assert torch.equal(got, want)
    if out_dtype == torch.float32:  # the addend may be the output itself
        inplace = addend.clone()
        grad_weight_bf16(g, x, out=inplace, addend=inplace)
        assert torch.equal(inplace, addend + gw)


# ------------------------------------------------------------------------------ updates
def _update_one(grad, packed, *, max_code, ema=None, beta=0.0):
    from local_ai_training_b200 import _lib

    rows, cols = packed.shape
    pk = packed.clone()
    code = torch.empty_like(pk, dtype=torch.int8)
    counts = torch.zeros(4, device=grad.device, dtype=torch.int64)
    rms_sum = torch.zeros(1, device=grad.device)
    ema_t = None if ema is None else ema.clone()
    _lib.check(_lib.lib().rt_ratchet_update(
        grad.data_ptr(), _lib.dtype_code(grad), 0, grad.stride(0), rows, cols, pk.data_ptr(),
        pk.stride(0), code.data_ptr(), code.stride(0), 1,
        None if ema_t is None else ema_t.data_ptr(), beta, max_code, 8, 0.5, 1.5, 1e-8,
        counts.data_ptr(), None, rms_sum.data_ptr(), None, _lib.stream_of(grad)))
    return pk, code, counts, rms_sum, ema_t


def _grouped(layers, *, max_code, beta=0.0):
    """layers: list of (grad, packed, ema or None, grad_mul); returns per-layer results."""
    from local_ai_training_b200 import _lib

    descs = (_lib.UpdateLayer * len(layers))()
    outs = []
    for d, (grad, packed, ema, mul) in zip(descs, layers):
        pk = packed.clone()
        code = torch.empty_like(pk, dtype=torch.int8)
        counts = torch.zeros(4, device=grad.device, dtype=torch.int64)
        rms_sum = torch.zeros(1, device=grad.device)
        ema_t = None if ema is None else ema.clone()
        d.grad, d.ldg, d.rows = grad.data_ptr(), grad.stride(0), packed.shape[0]
        d.packed, d.ldp = pk.data_ptr(), pk.stride(0)
        d.code_out, d.ldc = code.data_ptr(), code.stride(0)
        d.rms_ema = None if ema_t is None else ema_t.data_ptr()
        d.counts, d.rms_sum, d.grad_mul = counts.data_ptr(), rms_sum.data_ptr(), mul
        outs.append((pk, code, counts, rms_sum, ema_t))
    g0 = layers[0][0]
    _lib.check(_lib.lib().rt_ratchet_update_grouped(
        descs, len(layers), _lib.dtype_code(g0), 0, g0.shape[1], 1, beta, max_code, 8, 0.5, 1.5,
        1e-8, _lib.stream_of(g0)))
    return outs


@pytest.mark.parametrize("rows,cols", [(8192, 2048), (2048, 8192)])
def test_update_1b_shapes_match_oracle(cuda_device, rows, cols):
    """The update at the 1B matrices (lm_head / expand 8192 x 2048, contract 2048 x 8192), per
    layer and grouped, bit-exact against the CPU oracle."""
    torch.manual_seed(rows * 3 + cols)
    grad = (torch.randn(rows, cols, device=cuda_device) * 1e-3).to(torch.bfloat16)
    packed = _packed(rows, cols, rows + cols)
    ref = O.ratchet_update(_np(grad), packed.numpy(), max_code=MAX_CODE)
    pk, code, counts, _, _ = _update_one(grad, packed.to(cuda_device), max_code=MAX_CODE)
    np.testing.assert_array_equal(_np(pk), ref["packed"])
    np.testing.assert_array_equal(_np(code), ref["code"])
    np.testing.assert_array_equal(_np(counts), ref["counts"])
    (gpk, gcode, gcounts, _, _), = _grouped([(grad, packed.to(cuda_device), None, 1.0)],
                                            max_code=MAX_CODE)
    assert torch.equal(gpk, pk) and torch.equal(gcode, code) and torch.equal(gcounts, counts)


@pytest.mark.parametrize("cols", [512, 2048, 8192, 136])
@pytest.mark.parametrize("grad_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("ema", [False, True])
def test_grouped_update_equals_per_layer_updates(cuda_device, cols, grad_dtype, ema):
    """Layers of different row counts (ragged blocks, one empty) in one grouped launch, each with
    its gradient multiplier, equal one rt_ratchet_update per layer on grad · grad_mul."""
    torch.manual_seed(cols + (7 if ema else 0))
    beta = 0.9 if ema else 0.0
    rows_list = [1536, 512, 3, 0, 2048, 257]
    muls = [1.0, 0.5, 0.125, 1.0, 0.25, 1.0]
    layers, expected = [], []
    for i, (rows, mul) in enumerate(zip(rows_list, muls)):
        grad = (torch.randn(rows, cols, device=cuda_device) * 1e-3).to(grad_dtype)
        packed = _packed(rows, cols, 100 + i).to(cuda_device)
        ema0 = torch.rand(rows, device=cuda_device) * 1e-6 if ema else None
        layers.append((grad, packed, ema0, mul))
        scaled = (grad.float() * mul).to(grad_dtype)  # exact: powers of two
        expected.append(_update_one(scaled, packed, max_code=MAX_CODE, ema=ema0, beta=beta)
                        if rows else None)
    outs = _grouped(layers, max_code=MAX_CODE, beta=beta)
    for got, want, rows in zip(outs, expected, rows_list):
        if rows == 0:
            assert torch.equal(got[2], torch.zeros_like(got[2]))
            continue
        for a, b in zip(got[:3], want[:3]):
            assert torch.equal(a, b)
        # the rms sum adds per-CTA partials atomically: the grouping of rows may differ
        torch.testing.assert_close(got[3], want[3], rtol=1e-5, atol=0)
        if ema:
            assert torch.equal(got[4], want[4])


# ------------------------------------------------------------------------------ runtime
def _tiny_model(device, *, int8_backward: bool):
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    cfg = ModelConfig(vocab_size=512, block_size=64, n_layer=2, n_head=4, n_embd=128,
                      matmul_mode="int8", int8_backward=int8_backward)
    model = build_seeded_model(cfg, max_code=MAX_CODE, seed=11).to(device).train()
    for layer in model.ratchet_layers():
        layer.sr_seed = 5
    return model


def _state(model):
    return [t.clone() for t in model.state_dict().values()]


def test_deferred_grouped_update_equals_update_inside_backward(cuda_device):
    """One process without torch.distributed: the runtime's deferred, grouped update after
    backward leaves the same state as the update inside each layer's backward (3 steps, int8
    backward with its stochastic rounding)."""
    from local_ai_training_b200.dist import RatchetDataParallel

    tokens = torch.randint(0, 512, (8, 65), generator=torch.Generator().manual_seed(3))
    tokens = tokens.to(cuda_device)
    fused, deferred = (_tiny_model(cuda_device, int8_backward=True) for _ in range(2))
    ddp = RatchetDataParallel(deferred)
    assert ddp.world == 1
    opt_a = torch.optim.AdamW(fused.parameters(), lr=1e-3)
    opt_b = torch.optim.AdamW(deferred.parameters(), lr=1e-3)
    for _ in range(3):
        for model, opt in ((fused, opt_a), (deferred, opt_b)):
            opt.zero_grad(set_to_none=True)
            with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                _, loss = model(tokens[:, :-1], tokens[:, 1:])
            loss.backward()
            if model is fused:
                stats_a = model.ratchet_update(validate=True)
                opt.step()
            else:
                stats_b = ddp.step(opt, validate=True)
    for a, b in zip(_state(fused), _state(deferred)):
        assert torch.equal(a, b)
    assert stats_a.code_moves == stats_b.code_moves
    assert stats_a.total_weights == stats_b.total_weights


def test_accumulated_micro_batches_equal_one_batch_step(cuda_device):
    """accumulation_steps = 2 over the same micro-batch twice equals one step on that batch bit
    for bit: the bf16 total round(G + G) halved is bf16(G), and the support gradients g + g
    halved are g (int8_backward off, so every backward pass is deterministic)."""
    from local_ai_training_b200.dist import RatchetDataParallel

    tokens = torch.randint(0, 512, (8, 65), generator=torch.Generator().manual_seed(4))
    tokens = tokens.to(cuda_device)
    one, two = (_tiny_model(cuda_device, int8_backward=False) for _ in range(2))
    d1 = RatchetDataParallel(one)
    d2 = RatchetDataParallel(two, accumulation_steps=2)
    o1 = torch.optim.AdamW(one.parameters(), lr=1e-3)
    o2 = torch.optim.AdamW(two.parameters(), lr=1e-3)
    for _ in range(2):
        o1.zero_grad(set_to_none=True)
        o2.zero_grad(set_to_none=True)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            _, loss1 = one(tokens[:, :-1], tokens[:, 1:])
        loss1.backward()
        s1 = d1.step(o1, validate=True)
        for _ in range(2):
            with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                _, loss2 = two(tokens[:, :-1], tokens[:, 1:])
            loss2.backward()
        s2 = d2.step(o2, validate=True)
        assert torch.equal(loss1, loss2)
    for a, b in zip(_state(one), _state(two)):
        assert torch.equal(a, b)
    assert s1.code_moves == s2.code_moves
    with pytest.raises(RuntimeError, match="accumulation_steps"):
        for _ in range(3):
            with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                _, loss2 = two(tokens[:, :-1], tokens[:, 1:])
            loss2.backward()
