"""GPU: gradient producers fused with the consuming ratchet layer's stochastic-rounding quant.

Each fused kernel (RMSNorm backward, GELU backward, q|k|v head gather) must give exactly what the
two-pass path gives: its own output, then `quantize_rows(G, col_scale, stochastic, key)` of that
output — int8 rows, row scales and the bf16 copy bit-identical, the step counter advanced once.
The model-level test checks a whole train step with the fusion on and off.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


class _Plan:
    """GradientQuantPlan stand-in with a fixed key."""

    def __init__(self, col_scale, seed, layer_id, round_if_fp32, device):
        self._cs = col_scale
        self.seed, self.layer_id = seed, layer_id
        self.round_if_fp32 = round_if_fp32
        self.step_dev = torch.zeros(2, device=device, dtype=torch.int32)
        self.delivered = None

    def col_scale(self):
        return self._cs

    def sr_key(self):
        return self.seed, 0, self.layer_id, self.step_dev

    def deliver(self, gradient, q, row_scale, grad_bf16, round_bf16):
        self.delivered = (gradient, q, row_scale, grad_bf16, round_bf16)


def _two_pass_quant(grad, col_scale, seed, layer_id, round_bf16):
    from local_ai_training_b200.int8_matmul import _quantize_rows_fused

    flat = grad.reshape(-1, grad.shape[-1])
    step_dev = torch.zeros(2, device=grad.device, dtype=torch.int32)
    copy = None
    if flat.dtype != torch.bfloat16:
        copy = torch.empty(flat.shape, device=grad.device, dtype=torch.bfloat16)
    q, s = _quantize_rows_fused(flat, col_scale, stochastic=True, seed=seed, step=0, layer=layer_id,
                                bf16_copy=copy, step_dev=step_dev, round_input_bf16=round_bf16)
    return q, s, (flat if copy is None else copy), step_dev


def _check_delivery(plan, grad, col_scale, round_bf16):
    gradient, q, s, gb, rounded = plan.delivered
    assert gradient.data_ptr() == grad.data_ptr()
    assert rounded == round_bf16
    q2, s2, gb2, sd2 = _two_pass_quant(grad, col_scale, plan.seed, plan.layer_id, round_bf16)
    assert torch.equal(s, s2)
    assert torch.equal(q, q2)
    assert torch.equal(gb.reshape(gb2.shape), gb2)
    assert torch.equal(plan.step_dev, sd2)
    assert plan.step_dev.tolist() == [1, 0]


@pytest.mark.parametrize("rows,cols,x_dtype,gy_dtype,residual,round_if_fp32", [
    (4096, 512, torch.float32, torch.bfloat16, True, True),
    (4096, 512, torch.float32, torch.bfloat16, True, False),
    (1000, 256, torch.float32, torch.float32, False, False),
    (77, 1024, torch.bfloat16, torch.bfloat16, False, False),
    (33, 2048, torch.float32, torch.bfloat16, True, True),
])
def test_rmsnorm_backward_sr_matches_two_passes(cuda_device, rows, cols, x_dtype, gy_dtype,
                                                residual, round_if_fp32):
    from local_ai_training_b200.int8_backward import rmsnorm_backward

    torch.manual_seed(rows + cols)
    x = torch.randn(rows, cols, device=cuda_device).to(x_dtype)
    gy = (torch.randn(rows, cols, device=cuda_device) * 1e-2).to(gy_dtype)
    w = torch.rand(cols, device=cuda_device) + 0.5
    add = torch.randn(rows, cols, device=cuda_device) * 1e-2 if residual else None
    cs = torch.rand(cols, device=cuda_device) * 0.1 + 0.01
    plan = _Plan(cs, 1234, 17, round_if_fp32, cuda_device)
    gx, gw = rmsnorm_backward(gy, x, w, residual_grad=add, quant_plan=plan)
    gx2, gw2 = rmsnorm_backward(gy, x, w, residual_grad=add)
    assert torch.equal(gx, gx2)
    # dw: per-CTA partials summed with atomics, in arrival order (fp32 rounding of ~rows terms)
    assert torch.allclose(gw, gw2, rtol=1e-5, atol=1e-5)
    assert plan.delivered is not None
    _check_delivery(plan, gx, cs, round_if_fp32 and gx.dtype == torch.float32)


@pytest.mark.parametrize("rows,cols,dtype", [(4096, 2048, torch.bfloat16), (300, 1024, torch.float32),
                                             (5, 64, torch.bfloat16), (129, 4096, torch.bfloat16)])
def test_gelu_backward_sr_matches_two_passes(cuda_device, rows, cols, dtype):
    from local_ai_training_b200.int8_backward import gelu_backward

    torch.manual_seed(rows * 3 + cols)
    x = (torch.randn(rows, cols, device=cuda_device) * 2).to(dtype)
    gy = (torch.randn(rows, cols, device=cuda_device) * 1e-2).to(dtype)
    cs = torch.rand(cols, device=cuda_device) * 0.1 + 0.01
    plan = _Plan(cs, 99, 3, False, cuda_device)
    g = gelu_backward(gy, x, quant_plan=plan)
    assert torch.equal(g, gelu_backward(gy, x))
    assert plan.delivered is not None
    _check_delivery(plan, g, cs, False)


@pytest.mark.parametrize("layout", ["bhtd", "bthd", "mixed"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_heads_gather_sr_matches_cat_and_quant(cuda_device, layout, dtype):
    from local_ai_training_b200.int8_fused import heads_gather_quantize

    torch.manual_seed(5)
    b, h, t, d = 4, 8, 96, 64

    def make(kind):
        if kind == "bhtd":
            return torch.randn(b, h, t, d, device=cuda_device).to(dtype)
        return torch.randn(b, t, h, d, device=cuda_device).to(dtype).transpose(1, 2)

    kinds = {"bhtd": ["bhtd"] * 3, "bthd": ["bthd"] * 3, "mixed": ["bhtd", "bthd", "bhtd"]}[layout]
    grads = tuple(make(k) * 1e-2 for k in kinds)
    cs = torch.rand(3 * h * d, device=cuda_device) * 0.1 + 0.01
    plan = _Plan(cs, 7, 1 << 16, False, cuda_device)
    out = heads_gather_quantize(grads, plan)
    assert out is not None
    ref = torch.cat([g.transpose(1, 2).reshape(b, t, h * d) for g in grads], dim=-1)
    assert torch.equal(out, ref)
    _check_delivery(plan, out, cs, False)


@pytest.mark.parametrize("bf16_activations", [True, False])
def test_fused_grad_quant_model_steps_bit_exact(cuda_device, bf16_activations):
    """Two train steps with the producers quantising the ratchet layers' output gradients and
    with the layers quantising them: loss, logits, gradients and every ratchet state identical
    (RMSNorm weight gradients to fp32 rounding: their atomics sum in arrival order)."""
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    def run(fused):
        cfg = ModelConfig(vocab_size=256, block_size=32, n_layer=2, n_head=2, n_embd=64,
                          dropout=0.0, pressure_threshold=2, matmul_mode="int8",
                          int8_backward=True, bf16_activations=bf16_activations,
                          fused_grad_quant=fused)
        model = build_seeded_model(cfg, max_code=2, seed=4).to(cuda_device).train()
        for n, layer in enumerate(model.ratchet_layers()):
            layer.sr_seed = 9
            layer.sr_layer = n
        gen = torch.Generator().manual_seed(2)
        out = []
        for _ in range(2):
            tokens = torch.randint(0, 256, (4, 33), generator=gen).to(cuda_device)
            logits, loss = model(tokens[:, :-1], tokens[:, 1:])
            loss.backward()
            grads = [(n, p.grad.clone()) for n, p in model.named_parameters() if p.grad is not None]
            model.ratchet_update(validate=False)
            model.zero_grad(set_to_none=True)
            out.append((logits.detach().clone(), float(loss), grads))
        prequant_left = [l._prequant_grad is not None for l in model.ratchet_layers()]
        return out, [l.packed.clone() for l in model.ratchet_layers()], prequant_left

    fused, pf, left = run(True)
    plain, pp, _ = run(False)
    assert not any(left)  # every delivered quantisation was consumed
    for (lf, xf, gf), (lp, xp, gp) in zip(fused, plain):
        assert torch.equal(lf, lp)
        assert xf == xp
        assert [n for n, _ in gf] == [n for n, _ in gp]
        for (name, a), (_, b) in zip(gf, gp):
            if name.endswith("norm.weight"):
                assert torch.allclose(a, b, rtol=1e-5, atol=1e-9), name
            else:
                assert torch.equal(a, b), name
    assert all(torch.equal(a, b) for a, b in zip(pf, pp))


def test_fused_grad_quant_covers_the_block_layers(cuda_device, monkeypatch):
    """In the int8 model every ratchet layer but the last block's contraction and the lm_head
    receives its quantised output gradient from the producing kernel."""
    from local_ai_training_b200 import ModelConfig, build_seeded_model
    from local_ai_training_b200 import ratchet as R

    cfg = ModelConfig(vocab_size=256, block_size=32, n_layer=2, n_head=2, n_embd=64, dropout=0.0,
                      pressure_threshold=2, matmul_mode="int8", int8_backward=True,
                      fused_grad_quant=True)
    model = build_seeded_model(cfg, max_code=2, seed=4).to(cuda_device).train()
    used = []
    orig = R._take_prequantized

    def spy(sink, flat_gradient, round_bf16):
        r = orig(sink, flat_gradient, round_bf16)
        used.append((sink.__self__, r is not None))
        return r

    monkeypatch.setattr(R, "_take_prequantized", spy)
    tokens = torch.randint(0, 256, (4, 33), generator=torch.Generator().manual_seed(1)).to(cuda_device)
    _, loss = model(tokens[:, :-1], tokens[:, 1:])
    loss.backward()
    names = {id(m): n for n, m in model.named_modules()}
    hit = sorted(names[id(layer)] for layer, ok in used if ok)
    miss = sorted(names[id(layer)] for layer, ok in used if not ok)
    assert miss == ["blocks.1.feed_forward.contract"], miss
    assert len(hit) == 4 * 2 - 1, hit
