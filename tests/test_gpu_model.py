"""GPU: model-level int8 train steps through the package (the call sites of the hot path)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


def _tiny(mode: str, int8_backward: bool = False):
    from local_ai_training_b200 import ModelConfig

    return ModelConfig(vocab_size=11, block_size=8, n_layer=2, n_head=2, n_embd=16, dropout=0.0,
                       matmul_mode=mode, int8_backward=int8_backward)


def test_fp32_mode_model_step_matches_reference_fixture(cuda_device):
    """fp32 mode on the GPU (cuBLAS matmuls, CUDA update kernel) reproduces the reference's
    tiny-model step: logits, loss, and the packed state of every layer (reduction-order flips
    of a boundary weight allowed up to 2 weights in total)."""
    from local_ai_training_b200 import build_seeded_model

    g = load_golden("model_tiny.npz")
    model = build_seeded_model(_tiny("fp32"), max_code=3, seed=5).to(cuda_device).train()
    tokens = torch.from_numpy(g["tokens"]).to(cuda_device)
    logits, loss = model(tokens[:, :8], tokens[:, 1:])
    np.testing.assert_allclose(logits.detach().cpu().numpy(), g["logits"], rtol=1e-4, atol=1e-5)
    assert abs(float(loss) - float(g["loss"])) < 1e-4
    loss.backward()
    stats = model.ratchet_update()
    mism = 0
    for key, value in model.state_dict().items():
        if key.endswith("packed"):
            mism += int((value.cpu().numpy() != g[f"state1::{key}"]).sum())
    assert mism <= 2, mism
    assert abs(stats.code_moves - int(g["moves"][:2].sum())) <= 2


@pytest.mark.parametrize("int8_backward", [False, True])
def test_int8_model_trains_and_clears_temporaries(cuda_device, int8_backward):
    from local_ai_training_b200 import DiscreteRatchetLinear, build_seeded_model

    model = build_seeded_model(_tiny("int8", int8_backward), max_code=3, seed=5).to(cuda_device).train()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-2)
    gen = torch.Generator().manual_seed(0)
    tokens = torch.randint(0, 11, (4, 9), generator=gen).to(cuda_device)
    losses = []
    for _ in range(30):
        opt.zero_grad(set_to_none=True)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            logits, loss = model(tokens[:, :8], tokens[:, 1:])
        loss.backward()
        stats = model.ratchet_update()
        opt.step()
        losses.append(float(loss))
    assert all(math.isfinite(v) for v in losses)
    assert losses[-1] < losses[0]
    layers = [m for m in model.modules() if isinstance(m, DiscreteRatchetLinear)]
    assert stats.total_weights == sum(layer.packed.numel() for layer in layers)
    assert all(not layer.has_pending_gradient for layer in layers)


def test_int8_25m_shape_step_runs_and_matches_fp32_loss(cuda_device):
    """One 25M-config step (batch reduced to 4 x 512): finite, and the int8 forward loss agrees
    with the fp32 forward of the same seeded model within the quantisation error."""
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    kw = dict(vocab_size=8192, block_size=512, n_layer=8, n_head=8, n_embd=512, dropout=0.0)
    gen = torch.Generator().manual_seed(1337)
    tokens = torch.randint(0, 8192, (4, 513), generator=gen).to(cuda_device)
    m8 = build_seeded_model(ModelConfig(**kw, matmul_mode="int8", int8_backward=True), max_code=2,
                            seed=1337).to(cuda_device).train()
    m32 = build_seeded_model(ModelConfig(**kw, matmul_mode="fp32"), max_code=2,
                             seed=1337).to(cuda_device).eval()
    with torch.no_grad():
        _, l32 = m32(tokens[:, :-1], tokens[:, 1:])
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        _, l8 = m8(tokens[:, :-1], tokens[:, 1:])
    assert abs(float(l8) - float(l32)) < 0.02 * float(l32)
    l8.backward()
    stats = m8.ratchet_update()
    assert stats.total_weights == 25_165_824 + 4_194_304
    assert stats.code_moves >= 0 and math.isfinite(stats.gradient_rms_mean)


def test_bf16_activation_plumbing_matches_reference_plumbing(cuda_device):
    """bf16 producer dummies (the default) against the reference's fp32 dummies: logits, loss,
    every packed state and the embedding gradient are bit-identical over three steps (the
    RMSNorm weight gradients use fp32 reductions and are compared to 1e-5)."""
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    kw = dict(vocab_size=512, block_size=64, n_layer=2, n_head=4, n_embd=128, dropout=0.0,
              matmul_mode="int8", int8_backward=True)
    models = []
    for bf16 in (False, True):
        m = build_seeded_model(ModelConfig(**kw, bf16_activations=bf16), max_code=2,
                               seed=3).to(cuda_device).train()
        for layer in m.ratchet_layers():
            layer.sr_seed = 11
        models.append(m)
    gen = torch.Generator().manual_seed(4)
    for step in range(3):
        tokens = torch.randint(0, 512, (4, 65), generator=gen).to(cuda_device)
        outs = []
        for m in models:
            for p in m.parameters():
                p.grad = None
            with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                logits, loss = m(tokens[:, :-1], tokens[:, 1:])
            loss.backward()
            m.ratchet_update(validate=False)
            outs.append((logits.float(), loss.detach()))
        assert torch.equal(outs[0][0], outs[1][0]), step
        assert torch.equal(outs[0][1], outs[1][1]), step
        for la, lb in zip(models[0].ratchet_layers(), models[1].ratchet_layers(), strict=True):
            assert torch.equal(la.packed, lb.packed), step
        ga = models[0].token_embedding.weight.grad
        gb = models[1].token_embedding.weight.grad
        assert torch.equal(ga, gb), step
        for (na, pa), (_, pb) in zip(models[0].named_parameters(), models[1].named_parameters()):
            torch.testing.assert_close(pa.grad, pb.grad, rtol=1e-5, atol=1e-7, msg=na)


@pytest.mark.parametrize("flag", ["fused_residual", "producer_dequant", "fused_gradw_update"])
@pytest.mark.parametrize("int8_backward", [False, True])
def test_fusions_match_unfused_bit_exact(cuda_device, int8_backward, flag):
    """fused_residual: the residual adds in the GEMM epilogues and in the RMSNorm backward kernel
    compute the same fp32 values as `x + f(x)` with autograd's gradient sum.  producer_dequant:
    the producers' bf16 rows equal the backward's dequant of the saved int8 rows.  Loss, logits,
    every ratchet state and the embedding gradient are bit-identical over two steps."""
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    def run(fused):
        kw = {} if flag == "fused_gradw_update" else {flag: fused}
        cfg = ModelConfig(vocab_size=256, block_size=32, n_layer=2, n_head=2, n_embd=64,
                          dropout=0.0, pressure_threshold=2, matmul_mode="int8",
                          int8_backward=int8_backward, **kw)
        model = build_seeded_model(cfg, max_code=2, seed=4).to(cuda_device).train()
        for layer in model.ratchet_layers():
            layer.sr_seed = 9
            if flag == "fused_gradw_update":
                layer.fused_gradw_update = fused
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
        return out, [l.packed.clone() for l in model.ratchet_layers()]

    fused, pf = run(True)
    plain, pp = run(False)
    for (lf, xf, gf), (lp, xp, gp) in zip(fused, plain):
        assert torch.equal(lf, lp)
        assert xf == xp
        assert [n for n, _ in gf] == [n for n, _ in gp]
        for (name, a), (_, b) in zip(gf, gp):
            if name.endswith("norm.weight"):
                # the RMSNorm weight gradient sums per-CTA partials with atomics: its fp32
                # rounding depends on arrival order, run to run, fused or not
                assert torch.allclose(a, b, rtol=1e-5, atol=1e-9), name
            else:
                assert torch.equal(a, b), name
    assert all(torch.equal(a, b) for a, b in zip(pf, pp))
