"""GPU: the reference's hot-path layer tests (tests/test_ratchet.py of the reference) against this
build's DiscreteRatchetLinear, plus layer-level parity with the CPU oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def test_int8_mode_forward_matches_integer_reference(cuda_device):
    # reference tests/test_ratchet.py:325-339
    from local_ai_training_b200 import DiscreteRatchetLinear
    from local_ai_training_b200.int8_matmul import quantize_rows

    torch.manual_seed(6)
    layer = DiscreteRatchetLinear(35, 53, max_code=4, matmul_mode="int8").cuda().eval()
    inputs = torch.randn(2, 3, 35, device="cuda")
    quantized, input_scale = quantize_rows(inputs.flatten(0, -2))
    expected = ((quantized.float() @ layer.code.t().float()) * input_scale[:, None]
                * layer.scale[None, :]).to(torch.bfloat16)
    actual = layer(inputs)
    assert torch.equal(actual, expected.reshape(2, 3, 53).float())


@pytest.mark.parametrize("k,n", [(512, 512), (512, 2048), (2048, 512)])
def test_int8_forward_full_size_matches_oracle_rows(cuda_device, k, n):
    from local_ai_training_b200 import DiscreteRatchetLinear

    torch.manual_seed(1337)
    layer = DiscreteRatchetLinear(k, n, max_code=3, matmul_mode="int8").cuda().eval()
    x = torch.randn(16384, k, device="cuda", dtype=torch.bfloat16)
    out = layer(x)
    q, s = O.quantize_rows(_np(x[:256]))
    ref = O.scaled_int8_mm(q, _np(layer.code).T.copy(), s, _np(layer.scale))
    np.testing.assert_array_equal(_np(out[:256]), ref)


def test_int8_effective_weight_gradient_stays_close_to_eager_autograd(cuda_device):
    # reference tests/test_ratchet.py:342-357
    from local_ai_training_b200 import DiscreteRatchetLinear

    torch.manual_seed(7)
    layer = DiscreteRatchetLinear(35, 53, max_code=3, matmul_mode="int8").cuda().train()
    inputs = torch.randn(67, 35, device="cuda", requires_grad=True)
    reference_inputs = inputs.detach().clone().requires_grad_(True)
    reference_weight = layer.effective_weight().detach().requires_grad_(True)
    reference = torch.nn.functional.linear(reference_inputs, reference_weight)
    reference.float().square().mean().backward()
    layer(inputs).float().square().mean().backward()
    relative_error = ((layer._pending_weight_gradient - reference_weight.grad).norm()
                      / reference_weight.grad.norm())
    assert relative_error < 0.03


@pytest.mark.parametrize("mode", ["bf16", "int8"])
def test_matmul_modes_capture_effective_gradient_and_clear(cuda_device, mode):
    # reference tests/test_ratchet.py:260-288
    from local_ai_training_b200 import DiscreteRatchetLinear

    torch.manual_seed(2)
    layer = DiscreteRatchetLinear(35, 53, max_code=3, matmul_mode=mode).cuda().train()
    inputs = torch.randn(2, 3, 35, device="cuda", requires_grad=True)
    output = layer(inputs)
    assert output.shape == (2, 3, 53)
    output.sum().backward()
    assert layer.has_pending_gradient
    assert layer._pending_weight_gradient.shape == (53, 35)
    assert torch.isfinite(layer._pending_weight_gradient).all()
    output2 = layer(inputs)
    with pytest.raises(RuntimeError, match="missing ratchet_update"):
        output2.sum().backward()
    layer.ratchet_update()
    layer(inputs).sum().backward()
    layer.discard_pending_gradient()
    assert not layer.has_pending_gradient


def test_int8_backward_grad_input_matches_bf16_within_tolerance(cuda_device):
    # reference tests/test_ratchet.py:359-387
    from local_ai_training_b200 import DiscreteRatchetLinear
    from local_ai_training_b200.int8_matmul import quantize_rows

    torch.manual_seed(11)
    weight = torch.randn(48, 32, device="cuda")
    common = dict(max_code=2, matmul_mode="int8", fuse_backward_update=True, initial_weight=weight)
    bf16_bwd = DiscreteRatchetLinear(32, 48, **common).cuda().train()
    int8_bwd = DiscreteRatchetLinear(32, 48, int8_backward=True, **common).cuda().train()
    inputs = torch.randn(40, 32, device="cuda")
    quantized, input_scale = quantize_rows(inputs)
    in_a = inputs.detach().clone().requires_grad_(True)
    in_b = inputs.detach().clone().requires_grad_(True)
    out_a = bf16_bwd(in_a, inputs_int8=quantized, inputs_scale=input_scale)
    out_b = int8_bwd(in_b, inputs_int8=quantized, inputs_scale=input_scale)
    assert torch.equal(out_a, out_b)
    grad_out = torch.randn_like(out_a)
    out_a.backward(grad_out)
    out_b.backward(grad_out)
    rel = (in_b.grad - in_a.grad).norm() / in_a.grad.norm()
    assert rel < 0.03, f"int8 grad_input relerr {rel:.4f} exceeds 0.03"
    assert torch.equal(int8_bwd.packed, bf16_bwd.packed)


@pytest.mark.parametrize("max_code", [2, 3, 4])
@pytest.mark.parametrize("trainable_scale", [False, True])
@pytest.mark.parametrize("matmul_mode", ["fp32", "bf16", "int8"])
def test_fused_backward_equivalence(cuda_device, max_code, trainable_scale, matmul_mode):
    # reference tests/test_ratchet.py:390-445
    from local_ai_training_b200 import DiscreteRatchetLinear

    torch.manual_seed(42)
    inputs = torch.randn(5, 7, 16, device="cuda", requires_grad=True)
    weight = torch.randn(32, 16, device="cuda")
    eager = DiscreteRatchetLinear(16, 32, max_code=max_code, trainable_scale=trainable_scale,
                                  matmul_mode=matmul_mode, fuse_backward_update=False,
                                  initial_weight=weight).cuda()
    fused = DiscreteRatchetLinear(16, 32, max_code=max_code, trainable_scale=trainable_scale,
                                  matmul_mode=matmul_mode, fuse_backward_update=True, tile_size=11,
                                  initial_weight=weight).cuda()
    eager.train()
    fused.train()
    inputs_eager = inputs.detach().clone().requires_grad_()
    inputs_fused = inputs.detach().clone().requires_grad_()
    out_eager = eager(inputs_eager)
    out_fused = fused(inputs_fused)
    grad_out = torch.randn_like(out_eager)
    out_eager.backward(grad_out)
    out_fused.backward(grad_out)
    stats_eager = eager.ratchet_update()
    stats_fused = fused.ratchet_update()
    assert stats_fused.total_weights == stats_eager.total_weights
    assert stats_fused.positive_moves == stats_eager.positive_moves
    assert stats_fused.negative_moves == stats_eager.negative_moves
    assert stats_fused.blocked_positive_moves == stats_eager.blocked_positive_moves
    assert stats_fused.blocked_negative_moves == stats_eager.blocked_negative_moves
    assert abs(stats_fused.gradient_rms_mean - stats_eager.gradient_rms_mean) <= 1e-4 * (
        1 + abs(stats_eager.gradient_rms_mean))
    assert torch.equal(fused.packed, eager.packed)
    if trainable_scale:
        torch.testing.assert_close(fused.log_scale.grad, eager.log_scale.grad, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("max_code, code_sum, pressure_sum, total_moves",
                         [(2, 15, -32, 59), (3, 14, -32, 62), (4, 9, -32, 65)])
def test_update_matches_golden_reference(cuda_device, max_code, code_sum, pressure_sum, total_moves):
    # reference tests/test_ratchet.py:196-208 on the GPU layer (same seeded init)
    from local_ai_training_b200 import DiscreteRatchetLinear

    torch.manual_seed(1234)
    layer = DiscreteRatchetLinear(8, 6, max_code=max_code, pressure_threshold=8).cuda()
    total = 0
    for _ in range(60):
        total += layer.apply_normalized_gradient((torch.randn(6, 8) * 2.0).cuda()).code_moves
    assert int(layer.code.sum()) == code_sum
    assert int(layer.pressure.sum()) == pressure_sum
    assert total == total_moves


def test_saturation_and_nibble_bounds_under_adversarial_updates(cuda_device):
    # reference tests/test_ratchet.py:224-233
    from local_ai_training_b200 import DiscreteRatchetLinear

    torch.manual_seed(0)
    for max_code in (2, 3, 4):
        for threshold in (1, 2, 4, 8):
            layer = DiscreteRatchetLinear(8, 6, max_code=max_code, pressure_threshold=threshold).cuda()
            for step in range(200):
                sign = 1.0 if step % 7 < 5 else -1.0
                layer.apply_normalized_gradient((sign * (3.0 + torch.rand(6, 8))).cuda(), validate=False)
            layer._validate_state()
            assert int(layer.pressure.abs().max()) <= 7
            assert int(layer.code.abs().max()) <= max_code


def test_zero_gradient_stays_finite_and_nonfinite_raises(cuda_device):
    from local_ai_training_b200 import DiscreteRatchetLinear

    layer = DiscreteRatchetLinear(4, 2, max_code=3).cuda()
    stats = layer.apply_weight_gradient(torch.zeros(2, 4, device="cuda"))
    assert int(stats.code_moves) == 0 and np.isfinite(float(stats.gradient_rms_mean))
    assert torch.count_nonzero(layer.pressure).item() == 0
    bad = torch.ones(2, 4, device="cuda")
    bad[0, 0] = float("inf")
    with pytest.raises(FloatingPointError):
        layer.apply_weight_gradient(bad)


def test_config1_layer_step_matches_reference_trajectory(cuda_device):
    """The single-layer case on the GPU layer (fp32 mode, fused backward, 10 steps): the packed state
    after every step equals the reference's up to reduction-order boundary flips."""
    from local_ai_training_b200 import DiscreteRatchetLinear, pack_code_pressure

    g = load_golden("config1.npz")
    layer = DiscreteRatchetLinear(256, 256, max_code=2, fuse_backward_update=True).cuda().train()
    code0 = torch.from_numpy(g["code0"])
    layer.packed.copy_(pack_code_pressure(code0, torch.zeros_like(code0), 2).cuda())
    layer._scale.copy_(torch.from_numpy(g["scale"]).cuda())
    x = torch.from_numpy(g["x"]).cuda()
    grad_out = torch.from_numpy(g["grad_out"]).cuda()
    mismatched = 0
    for step in range(10):
        inp = x.clone().requires_grad_(True)
        out = layer(inp)
        if step == 0:
            torch.testing.assert_close(out, torch.from_numpy(g["out0"]).cuda(), rtol=1e-5, atol=1e-5)
        out.backward(grad_out)
        if step == 0:
            torch.testing.assert_close(inp.grad, torch.from_numpy(g["gin0"]).cuda(), rtol=1e-5, atol=1e-6)
        layer.ratchet_update(validate=False)
        mismatched += int((_np(layer.packed) != g["packs"][step]).sum())
        layer.packed.copy_(torch.from_numpy(g["packs"][step]).cuda())  # continue from reference state
    assert mismatched <= 10, mismatched


def test_pressure_leak_on_gpu(cuda_device):
    from local_ai_training_b200 import DiscreteRatchetLinear, pack_code_pressure, unpack_code_pressure

    layer = DiscreteRatchetLinear(8, 4, max_code=2, pressure_leak_period=3).cuda()
    code, _ = unpack_code_pressure(layer.packed.cpu(), 2)
    layer.packed.copy_(pack_code_pressure(code, torch.full_like(code, 5), 2).cuda())
    for _ in range(3):
        layer._maybe_leak_pressure()
    assert int(layer.pressure.max()) == 4 and int(layer.pressure.min()) == 4


def test_code_mirror_follows_external_packed_writes(cuda_device):
    from local_ai_training_b200 import DiscreteRatchetLinear

    torch.manual_seed(3)
    layer = DiscreteRatchetLinear(64, 32, max_code=3, matmul_mode="int8").cuda().eval()
    x = torch.randn(16, 64, device="cuda")
    before = layer(x)
    layer.packed.copy_(torch.flip(layer.packed, dims=[1]))  # external write bumps the version
    after = layer(x)
    assert not torch.equal(before, after)
    assert torch.equal(layer.code_int8(), layer.code)
