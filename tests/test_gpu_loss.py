"""GPU: the token cross-entropy kernels and the fused lm_head + cross-entropy step.

Reference: torch's F.cross_entropy (mean, ignore_index -100) on the same fp32 logits, on the GPU.
Bars: loss within 1e-6 relative; per-row loss within 2e-6 absolute; the bf16 logit gradient equal
to torch's fp32 gradient rounded to bf16 except where the two sums of exponentials round apart
(at most one bf16 ulp, on under 0.1 % of elements).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _torch_reference(logits, targets, extra=None):
    x = logits.detach().float().clone().requires_grad_(True)
    loss = F.cross_entropy(x, targets)
    total = loss if extra is None else loss + (x * extra).sum()
    total.backward()
    return loss.detach(), x.grad


def _ulp_diff(a_bf16, b_bf16):
    """|a - b| in units of one bf16 step at b's magnitude (0 where equal); differences below
    1e-10 count as equal (fp32 rounding residue where a gradient cancels to almost zero)."""
    a, b = a_bf16.float(), b_bf16.float()
    step = torch.ldexp(torch.ones_like(b), torch.frexp(b.abs().clamp_min(1e-30))[1] - 8)
    d = ((a - b).abs() / step).round().int()
    return torch.where((a - b).abs() < 1e-10, torch.zeros_like(d), d)


@pytest.mark.parametrize("rows,cols,dtype", [(512, 8192, torch.float32), (300, 1000, torch.float32),
                                             (64, 8192, torch.bfloat16), (7, 13, torch.float32)])
def test_cross_entropy_matches_torch(cuda_device, rows, cols, dtype):
    from local_ai_training_b200.cross_entropy import cross_entropy_grad_bf16, cross_entropy_rows

    torch.manual_seed(rows + cols)
    logits = (torch.randn(rows, cols, device=cuda_device) * 3).to(dtype)
    targets = torch.randint(0, cols, (rows,), device=cuda_device)
    targets[::5] = -100  # ignored rows
    row_max, row_logsum, row_loss = cross_entropy_rows(logits, targets)
    count = (targets != -100).sum().float().reshape(1)
    loss = row_loss.sum() / count[0]
    ref_loss, ref_grad = _torch_reference(logits, targets)
    assert torch.allclose(loss, ref_loss, rtol=1e-6, atol=0)
    ref_rows = F.cross_entropy(logits.float(), targets, reduction="none")
    assert (row_loss - ref_rows).abs().max().item() < 2e-6
    grad = cross_entropy_grad_bf16(logits, targets, row_max, row_logsum,
                                   torch.ones((), device=cuda_device), count)
    d = _ulp_diff(grad, ref_grad.to(torch.bfloat16))
    assert d.max().item() <= 1
    assert (d > 0).float().mean().item() < 1e-3
    assert torch.equal(grad[::5], torch.zeros_like(grad[::5]))  # ignored rows


def test_cross_entropy_extra_gradient_and_scale(cuda_device):
    from local_ai_training_b200.cross_entropy import cross_entropy_grad_bf16, cross_entropy_rows

    torch.manual_seed(3)
    logits = torch.randn(128, 4096, device=cuda_device)
    targets = torch.randint(0, 4096, (128,), device=cuda_device)
    extra = torch.randn(128, 4096, device=cuda_device) * 1e-4
    row_max, row_logsum, _ = cross_entropy_rows(logits, targets)
    count = torch.tensor([128.0], device=cuda_device)
    grad = cross_entropy_grad_bf16(logits, targets, row_max, row_logsum,
                                   torch.full((), 2.0, device=cuda_device), count, extra)
    x = logits.clone().requires_grad_(True)
    (2.0 * F.cross_entropy(x, targets) + (x * extra).sum()).backward()
    d = _ulp_diff(grad, x.grad.to(torch.bfloat16))
    assert d.max().item() <= 1 and (d > 0).float().mean().item() < 1e-3


def test_out_of_range_target_flags_and_is_ignored(cuda_device):
    from local_ai_training_b200 import _lib
    from local_ai_training_b200.cross_entropy import cross_entropy_rows

    logits = torch.randn(4, 10, device=cuda_device)
    targets = torch.tensor([1, 2, 10, 3], device=cuda_device)
    _lib.device_status(cuda_device, clear=True)
    _, _, row_loss = cross_entropy_rows(logits, targets)
    assert row_loss[2].item() == 0.0
    assert _lib.device_status(cuda_device, clear=True) & 0x4


@pytest.mark.parametrize("int8_backward", [False, True])
def test_fused_lm_head_cross_entropy_step_matches_unfused(cuda_device, int8_backward):
    """One model step with the fused lm_head + cross-entropy and with F.cross_entropy from the
    same state: identical logits, loss to fp32 rounding, embedding gradients to bf16 rounding,
    and ratchet states that differ only where a one-ulp bf16 gradient difference crosses a
    bucket threshold (a small fraction of pressures, fewer codes)."""
    from local_ai_training_b200 import ModelConfig, build_seeded_model
    from local_ai_training_b200.ratchet import unpack_code_pressure

    def run(fused):
        cfg = ModelConfig(vocab_size=512, block_size=64, n_layer=2, n_head=2, n_embd=64,
                          dropout=0.0, pressure_threshold=2, matmul_mode="int8",
                          int8_backward=int8_backward, fused_cross_entropy=fused)
        model = build_seeded_model(cfg, max_code=2, seed=3).to(cuda_device).train()
        for layer in model.ratchet_layers():
            layer.sr_seed = 5
        tokens = torch.randint(0, 512, (8, 65), generator=torch.Generator().manual_seed(8))
        tokens = tokens.to(cuda_device)
        logits, loss = model(tokens[:, :-1], tokens[:, 1:])
        loss.backward()
        emb_grad = model.token_embedding.weight.grad.clone()
        moves = int(model.ratchet_update(validate=False).code_moves)
        return logits.detach(), float(loss), emb_grad, moves, [l.packed.clone() for l in
                                                              model.ratchet_layers()]

    lf, xf, gf, mf, pf = run(True)
    lp, xp, gp, mp, pp = run(False)
    assert torch.equal(lf, lp)
    assert xf == pytest.approx(xp, rel=1e-6)
    assert torch.allclose(gf, gp, rtol=1e-2, atol=1e-6)
    assert mf > 0
    total = sum(a.numel() for a in pf)
    mism = sum(int((a != b).sum()) for a, b in zip(pf, pp))
    code_mism = sum(int((unpack_code_pressure(a, 2)[0] != unpack_code_pressure(b, 2)[0]).sum())
                    for a, b in zip(pf, pp))
    assert mism <= total // 200, (mism, total)
    assert code_mism <= total // 2000, (code_mism, total)


def _chunk_model(cuda_device, chunk_rows, vocab=512, block=64, n_embd=64, n_layer=2):
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    cfg = ModelConfig(vocab_size=vocab, block_size=block, n_layer=n_layer, n_head=2,
                      n_embd=n_embd, dropout=0.0, pressure_threshold=2, matmul_mode="int8",
                      int8_backward=True, logits_chunk_rows=chunk_rows)
    model = build_seeded_model(cfg, max_code=2, seed=3).to(cuda_device).train()
    for layer in model.ratchet_layers():
        layer.sr_seed = 5
    return model


@pytest.mark.parametrize("accumulation", [0, 1, 2])
def test_chunked_lm_head_matches_materialised_step(cuda_device, accumulation):
    """logits_chunk_rows (ragged last block) against the materialised fused path from the same
    state: the same loss bit for bit, embedding gradients to bf16 rounding, ratchet states equal
    up to the fp32 order of the lm_head grad_W sum (boundary weights only); with the deferred
    data-parallel update at one rank, with and without gradient accumulation."""
    from local_ai_training_b200.dist import RatchetDataParallel
    from local_ai_training_b200.ratchet import unpack_code_pressure

    tokens = torch.randint(0, 512, (8, 65), generator=torch.Generator().manual_seed(8))
    tokens = tokens.to(cuda_device)

    def run(chunk):
        model = _chunk_model(cuda_device, chunk)
        ddp = RatchetDataParallel(model, accumulation_steps=accumulation) if accumulation else None
        parts = tokens.chunk(accumulation) if accumulation else [tokens]
        losses = []
        for part in parts:
            logits, loss = model(part[:, :-1], part[:, 1:])
            assert (logits is None) == (chunk > 0)
            loss.backward()
            losses.append(float(loss))
        if ddp is not None:
            ddp.synchronize_gradients()
        emb_grad = model.token_embedding.weight.grad.clone()
        if ddp is not None:
            ddp.ratchet_update()
        else:
            model.ratchet_update(validate=False)
        return losses, emb_grad, [l.packed.clone() for l in model.ratchet_layers()]

    xc, gc, pc = run(96)
    xm, gm, pm = run(0)
    assert xc == xm
    assert torch.allclose(gc, gm, rtol=1e-2, atol=1e-6)
    total = sum(a.numel() for a in pc)
    mism = sum(int((a != b).sum()) for a, b in zip(pc, pm))
    code_mism = sum(int((unpack_code_pressure(a, 2)[0] != unpack_code_pressure(b, 2)[0]).sum())
                    for a, b in zip(pc, pm))
    assert mism <= total // 500, (mism, total)
    assert code_mism <= total // 5000, (code_mism, total)


def test_chunked_lm_head_stores_no_token_by_vocab_tensor(cuda_device):
    """16384 tokens x 8192 classes: with logits_chunk_rows = 2048 the step's peak allocation stays
    below one bf16 [16384, 8192] tensor (268 MB); materialised, it exceeds the fp32 logits."""
    tokens = torch.randint(0, 8192, (16, 1025), generator=torch.Generator().manual_seed(2))
    tokens = tokens.to(cuda_device)
    full_bf16 = 16384 * 8192 * 2
    peaks = {}
    for chunk in (2048, 0):
        model = _chunk_model(cuda_device, chunk, vocab=8192, block=1024, n_layer=1)
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        logits, loss = model(tokens[:, :-1], tokens[:, 1:])
        loss.backward()
        torch.cuda.synchronize()
        peaks[chunk] = torch.cuda.max_memory_allocated() - base
        del model, logits, loss
    assert peaks[2048] < full_bf16, peaks
    assert peaks[0] > 2 * full_bf16, peaks


def test_chunked_lm_head_ignored_targets_match_materialised(cuda_device):
    """lm_head_cross_entropy over row blocks (ragged last block, ignore_index rows in several
    blocks) against the materialised call: the same loss bit for bit, the same grad_input."""
    from local_ai_training_b200 import DiscreteRatchetLinear
    from local_ai_training_b200.cross_entropy import IGNORE_INDEX, lm_head_cross_entropy

    torch.manual_seed(21)
    layer = DiscreteRatchetLinear(256, 1000, matmul_mode="int8", int8_backward=True,
                                  max_code=2).to(cuda_device)
    x = torch.randn(700, 256, device=cuda_device)
    targets = torch.randint(0, 1000, (700,), device=cuda_device)
    targets[::7] = IGNORE_INDEX
    out = {}
    for chunk in (0, 192):
        xi = x.clone().requires_grad_(True)
        logits, loss = lm_head_cross_entropy(layer, xi, targets, chunk_rows=chunk)
        assert (logits is None) == (chunk > 0)
        loss.backward()
        layer.discard_pending_gradient()
        out[chunk] = (loss.detach(), xi.grad.clone())
    assert torch.equal(out[0][0], out[192][0])
    torch.testing.assert_close(out[192][1], out[0][1], rtol=0, atol=0)
