"""Host logic of checkpoints and token shards (no GPU): the reference's checkpoint format and
validation messages (checkpoint.py:23-106), the token-shard metadata checks and the seeded batch
schedule (data.py:238-276)."""

from __future__ import annotations

import hashlib
import json

import pytest
import torch

pytest.importorskip("safetensors")


def _tiny(seed: int):
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    cfg = ModelConfig(vocab_size=32, block_size=8, n_layer=1, n_head=2, n_embd=16,
                      matmul_mode="int8", int8_backward=True)
    return build_seeded_model(cfg, max_code=2, seed=seed)


def test_checkpoint_round_trip_uses_the_reference_keys(tmp_path):
    from safetensors.torch import load_file

    from local_ai_training_b200.checkpoint import load_checkpoint, save_checkpoint

    model = _tiny(1)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    for p in model.parameters():  # some optimizer state to carry
        p.grad = torch.full_like(p, 0.01)
    opt.step()
    layer = model.ratchet_layers()[0]
    layer._sr_step_dev = torch.tensor([5, 0], dtype=torch.int32)
    base = save_checkpoint(tmp_path / "ckpt", model=model, optimizer=opt, step=7, max_code=2,
                           vocabulary=("a", "b"), experiment_config={"matmul_mode": "int8"})
    tensors = load_file(base.with_suffix(".safetensors"))
    assert {k.removeprefix("model::") for k in tensors if k.startswith("model::")} == set(
        model.state_dict())
    assert any(k.startswith("optimizer::") for k in tensors) and "rng::cpu" in tensors
    meta = json.loads(base.with_suffix(".json").read_text())
    assert meta["format_version"] == 1 and meta["step"] == 7 and meta["max_code"] == 2

    fresh = _tiny(2)
    fresh_opt = torch.optim.AdamW(fresh.parameters(), lr=1e-3)
    got = load_checkpoint(base, model=fresh, optimizer=fresh_opt, expected_max_code=2,
                          expected_vocabulary=("a", "b"), expected_matmul_mode="int8")
    assert got["step"] == 7
    for (k, a), b in zip(model.state_dict().items(), fresh.state_dict().values()):
        assert torch.equal(a, b), k
    for p, q in zip(model.parameters(), fresh.parameters()):
        for name, value in opt.state[p].items():
            assert torch.equal(torch.as_tensor(value), torch.as_tensor(fresh_opt.state[q][name]))
    assert torch.equal(fresh.ratchet_layers()[0]._sr_step_dev, torch.tensor([5, 0],
                                                                            dtype=torch.int32))


@pytest.mark.parametrize("kwargs,message", [
    (dict(expected_max_code=3), "code range"),
    (dict(expected_vocabulary=("x",)), "vocabulary"),
    (dict(expected_matmul_mode="fp32"), "matmul_mode"),
])
def test_checkpoint_validation_messages(tmp_path, kwargs, message):
    from local_ai_training_b200.checkpoint import load_checkpoint, save_checkpoint

    model = _tiny(1)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    base = save_checkpoint(tmp_path / "c", model=model, optimizer=opt, step=1, max_code=2,
                           vocabulary=("a",), experiment_config={"matmul_mode": "int8"})
    args = dict(expected_max_code=2, expected_vocabulary=("a",), expected_matmul_mode="int8")
    args.update(kwargs)
    with pytest.raises(ValueError, match=message):
        load_checkpoint(base, model=_tiny(1), optimizer=opt, **args)


def _shard(tmp_path, tokens: list[int], *, dtype="uint16", corrupt_hash=False):
    tok_json = json.dumps({"model": "bpe", "vocab": 64})
    data = torch.tensor(tokens, dtype=torch.int64).to(torch.uint16)
    (tmp_path / "tokens.uint16").write_bytes(data.numpy().tobytes())
    meta = {"token_dtype": dtype, "tokens_file": "tokens.uint16", "actual_tokens": len(tokens),
            "tokenizer_json": tok_json,
            "tokenizer_sha256": hashlib.sha256(tok_json.encode()).hexdigest()}
    if corrupt_hash:
        meta["tokenizer_sha256"] = "0" * 64
    path = tmp_path / "shard.json"
    path.write_text(json.dumps(meta))
    return path


@pytest.mark.parametrize("case,message", [
    ("dtype", "unsupported token shard dtype"),
    ("hash", "tokenizer hash mismatch"),
    ("short", "too short"),
    ("fraction", "validation_fraction"),
])
def test_token_shard_metadata_checks(tmp_path, case, message):
    from local_ai_training_b200.data import load_token_shard

    path = _shard(tmp_path, list(range(5 if case == "short" else 100)),
                  dtype="uint32" if case == "dtype" else "uint16", corrupt_hash=case == "hash")
    with pytest.raises(ValueError, match=message):
        load_token_shard(path, validation_fraction=1.5 if case == "fraction" else 0.1)


def test_batch_schedule_is_the_seeded_reference_schedule():
    from local_ai_training_b200.data import make_batch_schedule

    got = make_batch_schedule(data_length=1000, steps=3, batch_size=4, block_size=16, seed=9)
    want = torch.randint(0, 1000 - 16, (3, 4), generator=torch.Generator().manual_seed(9))
    assert torch.equal(got, want)
    with pytest.raises(ValueError, match="exceed block_size"):
        make_batch_schedule(data_length=16, steps=1, batch_size=1, block_size=16, seed=0)
