"""GPU: the data-parallel runtime end to end.

* One rank (any box): the DP path — bf16 grad_W into the reduce-scatter buffer, owned-row
  update, mirror refresh — leaves exactly the state of the single-process fused step.
* Two ranks (boxes with two or more GPUs, NCCL): replicated state stays identical on both ranks
  and the global statistics count every row once.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _cfg(int8_backward: bool):
    from local_ai_training_b200 import ModelConfig

    # threshold 2 with rms_ema so that codes move within a few steps and the EMA path runs
    return ModelConfig(vocab_size=64, block_size=32, n_layer=2, n_head=2, n_embd=64, dropout=0.0,
                       pressure_threshold=2, rms_ema_beta=0.5, matmul_mode="int8",
                       int8_backward=int8_backward)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _step(model, tokens, ddp=None):
    _, loss = model(tokens[:, :-1], tokens[:, 1:])
    loss.backward()
    if ddp is None:
        stats = model.ratchet_update(validate=False)
    else:
        ddp.synchronize_gradients()
        stats = ddp.ratchet_update(validate=False)
    model.zero_grad(set_to_none=True)
    return float(loss), stats


@pytest.mark.parametrize("int8_backward", [False, True])
def test_single_rank_dp_equals_fused_single_process(cuda_device, int8_backward):
    from local_ai_training_b200 import build_seeded_model
    from local_ai_training_b200.dist import RatchetDataParallel

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0,
                            world_size=1)
    try:
        plain = build_seeded_model(_cfg(int8_backward), max_code=2, seed=9).to(cuda_device).train()
        dp_model = build_seeded_model(_cfg(int8_backward), max_code=2, seed=9).to(cuda_device).train()
        for a, b in zip(plain.ratchet_layers(), dp_model.ratchet_layers()):
            a.sr_seed = b.sr_seed = 21
        ddp = RatchetDataParallel(dp_model)
        gen = torch.Generator().manual_seed(4)
        before = [l.packed.clone() for l in plain.ratchet_layers()]
        moves = 0
        for _ in range(3):
            tokens = torch.randint(0, 64, (4, 33), generator=gen).to(cuda_device)
            la, sa = _step(plain, tokens)
            lb, sb = _step(dp_model, tokens, ddp)
            assert la == lb
            assert int(sa.code_moves) == int(sb.code_moves)
            assert int(sa.total_weights) == int(sb.total_weights)
            moves += int(sa.code_moves)
        assert moves > 0
        for a, b, c in zip(plain.ratchet_layers(), dp_model.ratchet_layers(), before):
            assert torch.equal(a.packed, b.packed)
            assert torch.equal(a.code_int8(), b.code_int8())
            assert torch.equal(a.rms_ema, b.rms_ema)
        assert any(not torch.equal(a.packed, c) for a, c in zip(plain.ratchet_layers(), before))
        ddp.detach()
    finally:
        dist.destroy_process_group()


def _two_rank_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from datetime import timedelta

    from local_ai_training_b200 import build_seeded_model
    from local_ai_training_b200.dist import RatchetDataParallel

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    device = torch.device("cuda", rank)
    model = build_seeded_model(_cfg(True), max_code=2, seed=9).to(device).train()
    for layer in model.ratchet_layers():
        layer.sr_seed = 21
    before = [l.packed.clone() for l in model.ratchet_layers()]
    ddp = RatchetDataParallel(model)
    gen = torch.Generator().manual_seed(100 + rank)
    moves = 0
    for _ in range(3):
        tokens = torch.randint(0, 64, (4, 33), generator=gen).to(device)
        _, stats = _step(model, tokens, ddp)
        moves += int(stats.code_moves)
    changed = sum(int((b != l.packed).sum()) for b, l in zip(before, model.ratchet_layers()))
    torch.save({"packed": [l.packed.cpu() for l in model.ratchet_layers()],
                "mirror": [l.code_int8().cpu() for l in model.ratchet_layers()],
                "ema": [l.rms_ema.cpu() for l in model.ratchet_layers()],
                "moves": moves, "changed": changed},
               os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_state_stays_replicated(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_two_rank_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn")
    r0, r1 = (torch.load(tmp_path / f"rank{r}.pt") for r in range(2))
    for a, b in zip(r0["packed"], r1["packed"]):
        assert torch.equal(a, b)
    for a, b in zip(r0["mirror"], r1["mirror"]):
        assert torch.equal(a, b)
    for a, b in zip(r0["ema"], r1["ema"]):
        assert torch.equal(a, b)
    assert r0["moves"] == r1["moves"] and r0["moves"] > 0
    assert r0["changed"] == r1["changed"] and r0["changed"] > 0


def _accum_resume_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    """Two ranks, two accumulated micro-batches per step: the replicated state agrees across
    ranks, and a run resumed from rank 0's checkpoint equals the uninterrupted one."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from datetime import timedelta

    from local_ai_training_b200 import build_seeded_model
    from local_ai_training_b200.checkpoint import load_checkpoint, save_checkpoint
    from local_ai_training_b200.dist import RatchetDataParallel

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    device = torch.device("cuda", rank)

    def build(seed):
        model = build_seeded_model(_cfg(True), max_code=2, seed=seed).to(device).train()
        for layer in model.ratchet_layers():
            layer.sr_seed = 21
        opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
        return model, opt, RatchetDataParallel(model, accumulation_steps=2)

    def step(model, ddp, opt, tokens):
        for chunk in tokens.chunk(2):
            _, loss = model(chunk[:, :-1], chunk[:, 1:])
            loss.backward()
        stats = ddp.step(opt)
        opt.zero_grad(set_to_none=True)
        return int(stats.code_moves)

    gen = torch.Generator().manual_seed(200 + rank)
    batches = [torch.randint(0, 64, (8, 33), generator=gen).to(device) for _ in range(4)]
    model, opt, ddp = build(9)
    moves = sum(step(model, ddp, opt, b) for b in batches[:2])
    save_checkpoint(os.path.join(out_dir, "ck"), model=model, optimizer=opt, step=2, max_code=2,
                    vocabulary=(), experiment_config={"matmul_mode": "int8"})
    moves += sum(step(model, ddp, opt, b) for b in batches[2:])
    resumed, ropt, rddp = build(123)
    load_checkpoint(os.path.join(out_dir, "ck"), model=resumed, optimizer=ropt, expected_max_code=2,
                    expected_vocabulary=(), expected_matmul_mode="int8")
    for b in batches[2:]:
        step(resumed, rddp, ropt, b)
    same = all(torch.equal(a, b) for a, b in zip(model.state_dict().values(),
                                                 resumed.state_dict().values()))
    torch.save({"packed": [l.packed.cpu() for l in model.ratchet_layers()], "moves": moves,
                "resume_equal": same}, os.path.join(out_dir, f"acc{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_accumulation_and_resume(tmp_path):
    pytest.importorskip("safetensors")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_accum_resume_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn")
    r0, r1 = (torch.load(tmp_path / f"acc{r}.pt") for r in range(2))
    for a, b in zip(r0["packed"], r1["packed"]):
        assert torch.equal(a, b)
    assert r0["moves"] == r1["moves"] and r0["moves"] > 0
    assert r0["resume_equal"] and r1["resume_equal"]
