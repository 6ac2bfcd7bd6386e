"""GPU: the row-sparse ratchet embedding (reference ratchet.py:688-749), the device-resident
uint16 token shard (data.py:238-287) and checkpoint resume (checkpoint.py:23-106).

Bars: the embedding forward bit-exact against code·scale rows; the sparse update bit-exact
against the CPU oracle's dense update on the reference's dense embedding gradient (rows summed in
position order, as the reference's CPU embedding backward adds them); token windows equal to
slicing; a resumed run equal, bit for bit, to an uninterrupted one.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("rows,dim,n_tok,beta", [(8192, 512, 4096, 0.0), (97, 64, 300, 0.5),
                                                 (64, 2048, 1000, 0.0)])
def test_sparse_embedding_update_matches_dense_oracle(cuda_device, rows, dim, n_tok, beta):
    from local_ai_training_b200 import RatchetEmbedding

    torch.manual_seed(rows + dim)
    layer = RatchetEmbedding(rows, dim, max_code=2, pressure_threshold=2,
                             rms_ema_beta=beta).to(cuda_device).train()
    if beta > 0:
        layer.rms_ema.copy_(torch.rand(rows, device=cuda_device) * 1e-4)
    tokens = torch.randint(0, rows, (n_tok,), device=cuda_device)
    tokens[:8] = tokens[0]  # a token repeated at several positions
    out = layer(tokens)
    effective = layer.code.float() * layer.scale[:, None]
    assert torch.equal(out, effective[tokens])
    grad = torch.randn(n_tok, dim, device=cuda_device) * 1e-2
    packed0 = _np(layer.packed)
    ema0 = _np(layer.rms_ema).copy() if beta > 0 else None
    out.backward(grad)
    stats = layer.ratchet_update(validate=True)
    # the reference's dense gradient: position-order sums (CPU index_add), zeros elsewhere
    dense = torch.zeros(rows, dim).index_add_(0, tokens.cpu(), grad.cpu()).numpy()
    ref = O.ratchet_update(dense, packed0, max_code=2, threshold=2, rms_ema=ema0, beta=beta)
    np.testing.assert_array_equal(_np(layer.packed), ref["packed"])
    np.testing.assert_array_equal(_np(layer.code_int8()), ref["code"])
    if beta > 0:
        np.testing.assert_array_equal(_np(layer.rms_ema), ref["rms_ema"])
    assert stats.positive_moves == int(ref["counts"][0])
    assert stats.negative_moves == int(ref["counts"][1])
    assert stats.total_weights == rows * dim
    assert stats.gradient_rms_mean == pytest.approx(float(ref["row_rms"].mean()), rel=1e-5)
    assert not layer.has_pending_gradient


def test_ratchet_embedding_model_trains(cuda_device):
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    cfg = ModelConfig(vocab_size=256, block_size=32, n_layer=1, n_head=2, n_embd=64,
                      matmul_mode="int8", int8_backward=True, ratchet_embedding=True,
                      pressure_threshold=2)
    model = build_seeded_model(cfg, max_code=2, seed=5).to(cuda_device).train()
    emb = model.token_embedding
    before = emb.packed.clone()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    tokens = torch.randint(0, 256, (8, 33), device=cuda_device)
    for _ in range(3):
        opt.zero_grad(set_to_none=True)
        _, loss = model(tokens[:, :-1], tokens[:, 1:])
        loss.backward()
        model.ratchet_update(validate=True)
        opt.step()
        assert torch.isfinite(loss)
    assert not torch.equal(before, emb.packed)
    untouched = torch.ones(256, dtype=torch.bool, device=cuda_device)
    untouched[tokens[:, :-1].reshape(-1)] = False
    assert torch.equal(before[untouched], emb.packed[untouched])


def test_token_windows_equal_slicing(cuda_device, tmp_path):
    import hashlib
    import json

    from local_ai_training_b200.data import batch_from_starts, load_token_shard, make_batch_schedule

    ids = torch.randint(0, 65535, (10_000,), dtype=torch.int64)
    (tmp_path / "t.uint16").write_bytes(ids.to(torch.uint16).numpy().tobytes())
    tj = "{}"
    (tmp_path / "m.json").write_text(json.dumps({
        "token_dtype": "uint16", "tokens_file": "t.uint16", "actual_tokens": ids.numel(),
        "tokenizer_json": tj, "tokenizer_sha256": hashlib.sha256(tj.encode()).hexdigest()}))
    shard = load_token_shard(tmp_path / "m.json", validation_fraction=0.1, device=cuda_device)
    train = ids[:-1000]
    assert shard.train_ids.dtype == torch.uint16 and shard.train_ids.is_cuda
    assert torch.equal(shard.train_ids.cpu().to(torch.int64), train)
    starts = make_batch_schedule(data_length=train.numel(), steps=2, batch_size=16, block_size=128,
                                 seed=3)[0]
    x, y = batch_from_starts(shard.train_ids, starts, block_size=128)
    idx = starts[:, None] + torch.arange(128)[None, :]
    assert torch.equal(x.cpu(), train[idx]) and torch.equal(y.cpu(), train[idx + 1])
    with pytest.raises(ValueError, match="exceeds"):
        batch_from_starts(shard.train_ids, torch.tensor([train.numel() - 128]), block_size=128)


def _step(model, ddp, opt, tokens, micro):
    for chunk in tokens.chunk(micro):
        _, loss = model(chunk[:, :-1], chunk[:, 1:])
        loss.backward()
    stats = ddp.step(opt)
    opt.zero_grad(set_to_none=True)
    return loss.detach(), stats


def test_resume_from_checkpoint_equals_uninterrupted_run(cuda_device, tmp_path):
    """Deferred grouped updates, two accumulated micro-batches, stochastic rounding on: two
    steps, save, two more steps, against load + the same two steps."""
    pytest.importorskip("safetensors")
    from local_ai_training_b200 import ModelConfig, build_seeded_model
    from local_ai_training_b200.checkpoint import load_checkpoint, save_checkpoint
    from local_ai_training_b200.dist import RatchetDataParallel

    cfg = ModelConfig(vocab_size=128, block_size=32, n_layer=2, n_head=2, n_embd=64,
                      matmul_mode="int8", int8_backward=True, pressure_threshold=2,
                      rms_ema_beta=0.5)

    def build(seed):
        model = build_seeded_model(cfg, max_code=3, seed=seed).to(cuda_device).train()
        for layer in model.ratchet_layers():
            layer.sr_seed = 17
        opt = torch.optim.AdamW(model.parameters(), lr=1e-3, fused=True, capturable=True)
        return model, opt, RatchetDataParallel(model, accumulation_steps=2)

    gen = torch.Generator().manual_seed(8)
    batches = [torch.randint(0, 128, (8, 33), generator=gen).to(cuda_device) for _ in range(4)]
    model, opt, ddp = build(1)
    for b in batches[:2]:
        _step(model, ddp, opt, b, 2)
    save_checkpoint(tmp_path / "ck", model=model, optimizer=opt, step=2, max_code=3,
                    vocabulary=(), experiment_config={"matmul_mode": "int8"})
    losses = [_step(model, ddp, opt, b, 2)[0] for b in batches[2:]]
    resumed, ropt, rddp = build(99)
    load_checkpoint(tmp_path / "ck", model=resumed, optimizer=ropt, expected_max_code=3,
                    expected_vocabulary=(), expected_matmul_mode="int8")
    rlosses = [_step(resumed, rddp, ropt, b, 2)[0] for b in batches[2:]]
    for a, b in zip(losses, rlosses):
        assert torch.equal(a, b)
    for (k, a), b in zip(model.state_dict().items(), resumed.state_dict().values()):
        assert torch.equal(a, b), k
