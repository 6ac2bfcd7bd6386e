"""Host logic of the data-parallel runtime on CPU: two gloo ranks.

The ratchet arithmetic itself is the CPU oracle here (stub layers apply `oracle.ratchet_update`
to the rows they own); what is under test is the runtime around it: row ownership, the
reduce-scatter of bf16 gradients and the 1/P scaling, the all-gather of `packed` and `rms_ema`,
the global step statistics and the support-parameter averaging.  The result must equal one
process applying the update to the whole matrix with the averaged gradient.
"""

from __future__ import annotations

import os
import warnings

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

SHAPES = [(8, 16, 0.0), (16, 8, 0.5), (4, 12, 0.0)]  # (out, in, rms_ema_beta)
MAX_CODE, THRESHOLD = 2, 3


class _StubLayer(torch.nn.Module):
    """The attributes and methods RatchetDataParallel uses, with oracle arithmetic on CPU."""

    fuse_backward_update = True
    matmul_mode = "int8"

    def __init__(self, out_features: int, in_features: int, beta: float, seed: int) -> None:
        super().__init__()
        rng = np.random.default_rng(seed)
        code = rng.integers(-MAX_CODE, MAX_CODE + 1, (out_features, in_features), dtype=np.int8)
        pressure = rng.integers(-2, 3, (out_features, in_features), dtype=np.int8)
        self.packed = torch.from_numpy(O.pack_code_pressure(code, pressure, MAX_CODE))
        self.out_features, self.in_features = out_features, in_features
        self.rms_ema_beta = beta
        self.rms_ema = torch.zeros(out_features)
        self.sr_layer = 0
        self._dp = None
        self.reset()

    def reset(self) -> None:
        self._pending_buf = torch.zeros(5, dtype=torch.int64)
        self._pending_rms = self._pending_buf[4:].view(torch.float32)[:1]
        self._pending_stats_total_weights = 0
        self._pending_stats_rms_sum = 0.0

    def _capture_weight_gradient(self, gradient, row_start, row_end, *, round_bf16=False):
        ema = self.rms_ema[row_start:row_end].numpy() if self.rms_ema_beta > 0 else None
        out = O.ratchet_update(gradient.float().numpy(), self.packed[row_start:row_end].numpy(),
                               max_code=MAX_CODE, threshold=THRESHOLD, rms_ema=ema,
                               beta=self.rms_ema_beta)
        self.packed[row_start:row_end] = torch.from_numpy(out["packed"])
        if ema is not None:
            self.rms_ema[row_start:row_end] = torch.from_numpy(out["rms_ema"])
        self._pending_buf[:4] += torch.from_numpy(out["counts"])
        self._pending_rms += float(out["row_rms"].sum())
        return None

    def _refresh_code_mirror(self) -> None:
        return None


class _StubModel(torch.nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.layers = torch.nn.ModuleList(_StubLayer(o, i, b, 100 + n)
                                          for n, (o, i, b) in enumerate(SHAPES))
        self.norm = torch.nn.Parameter(torch.ones(6))

    def ratchet_layers(self):
        return list(self.layers)

    def ratchet_update(self, *, validate=False):
        from local_ai_training_b200.ratchet import RatchetUpdateStats

        counts = sum(l._pending_buf[:4] for l in self.layers)
        stats = RatchetUpdateStats(
            total_weights=sum(l._pending_stats_total_weights for l in self.layers),
            positive_moves=counts[0], negative_moves=counts[1],
            blocked_positive_moves=counts[2], blocked_negative_moves=counts[3],
            gradient_rms_mean=float(sum(l._pending_rms[0] / l.out_features for l in self.layers))
            / len(self.layers))
        for l in self.layers:
            l.reset()
        return stats


def _local_grad(rank: int, n: int, shape) -> torch.Tensor:
    g = torch.Generator().manual_seed(1000 * rank + n)
    return (torch.randn(shape[0], shape[1], generator=g) * 1e-2).to(torch.bfloat16)


def _init(rank: int, world: int, out_dir: str) -> None:
    # file rendezvous in the test's own directory: no TCP port to race for
    dist.init_process_group("gloo", init_method=f"file://{os.path.join(out_dir, 'store')}",
                            rank=rank, world_size=world)


def _worker(rank: int, world: int, out_dir: str) -> None:
    _init(rank, world, out_dir)
    from local_ai_training_b200.dist import RatchetDataParallel

    model = _StubModel()
    ddp = RatchetDataParallel(model)
    # "backward": last layer first, as autograd produces them
    for n in reversed(range(len(SHAPES))):
        layer = model.layers[n]
        ddp.grad_buffer(layer).copy_(_local_grad(rank, n, SHAPES[n][:2]))
        ddp.grad_ready(layer)
    model.norm.grad = torch.full((6,), float(rank + 1))
    # step(): support all-reduce, owned-row updates, the optimizer, re-replication
    stats = ddp.step(torch.optim.SGD([model.norm], lr=1.0))
    torch.save({"packed": [l.packed.clone() for l in model.layers],
                "ema": [l.rms_ema.clone() for l in model.layers],
                "norm_grad": model.norm.grad.clone(), "norm": model.norm.detach().clone(),
                "sr_layer": [l.sr_layer for l in model.layers],
                "stats": [int(stats.positive_moves), int(stats.negative_moves),
                          int(stats.blocked_positive_moves), int(stats.blocked_negative_moves),
                          int(stats.total_weights), float(stats.gradient_rms_mean)]},
               os.path.join(out_dir, f"rank{rank}.pt"))
    dist.destroy_process_group()


def _run_ranks(fn, world: int, tmp_path):
    """Spawns the ranks; returns the directory holding their outputs.  The ranks only compute and
    save (every check runs here), so an exception from the spawn / rendezvous is infrastructure:
    it is retried once in a fresh directory, with a warning that carries the first error (a first
    run on a cold machine has failed this way once)."""
    for attempt in range(2):
        out = tmp_path / f"run{attempt}"
        out.mkdir()
        try:
            mp.start_processes(fn, args=(world, str(out)), nprocs=world, start_method="spawn")
            return out
        except Exception as exc:  # ProcessRaisedException / ProcessExitedException
            if attempt == 1:
                raise
            warnings.warn(f"gloo ranks failed once, retrying: {exc!r}")
    raise AssertionError("unreachable")


def test_row_owner_update_equals_single_process_update(tmp_path):
    world = 2
    tmp_path = _run_ranks(_worker, world, tmp_path)
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    # replicated state: identical on both ranks
    for a, b in zip(res[0]["packed"], res[1]["packed"]):
        assert torch.equal(a, b)
    for a, b in zip(res[0]["ema"], res[1]["ema"]):
        assert torch.equal(a, b)
    assert res[0]["stats"] == res[1]["stats"]
    # support gradient averaged
    assert torch.equal(res[0]["norm_grad"], torch.full((6,), 1.5))
    assert torch.equal(res[0]["norm"], torch.full((6,), -0.5))
    assert torch.equal(res[1]["norm"], torch.full((6,), -0.5))
    # per-rank stochastic-rounding streams
    assert res[0]["sr_layer"] == [0, 0, 0] and res[1]["sr_layer"] == [1 << 16] * 3
    # single process: the whole matrix, gradient = bf16 sum of the ranks' bf16 grads, halved
    counts = np.zeros(4, np.int64)
    rms_means = []
    fresh = _StubModel()
    for n, (o, i, beta) in enumerate(SHAPES):
        g = (_local_grad(0, n, (o, i)).float() + _local_grad(1, n, (o, i)).float())
        g = g.to(torch.bfloat16).float() * 0.5
        layer = fresh.layers[n]
        ema = np.zeros(o, np.float32) if beta > 0 else None
        out = O.ratchet_update(g.numpy(), layer.packed.numpy(), max_code=MAX_CODE,
                               threshold=THRESHOLD, rms_ema=ema, beta=beta)
        np.testing.assert_array_equal(res[0]["packed"][n].numpy(), out["packed"])
        if beta > 0:
            np.testing.assert_array_equal(res[0]["ema"][n].numpy(), out["rms_ema"])
        counts += out["counts"]
        rms_means.append(out["row_rms"].sum() / o)
    assert res[0]["stats"][:4] == counts.tolist()
    assert res[0]["stats"][4] == sum(o * i for o, i, _ in SHAPES)
    assert res[0]["stats"][5] == pytest.approx(float(np.mean(rms_means)), rel=1e-6)


def test_rejects_rows_not_divisible_by_ranks(tmp_path):
    world = 2
    tmp_path = _run_ranks(_reject_worker, world, tmp_path)
    for r in range(world):
        assert (tmp_path / f"ok{r}").read_text() == "ValueError"


def _reject_worker(rank: int, world: int, out_dir: str) -> None:
    _init(rank, world, out_dir)
    from local_ai_training_b200.dist import RatchetDataParallel

    model = _StubModel()
    model.layers[0].out_features = 7
    try:
        RatchetDataParallel(model)
        result = "accepted"
    except ValueError:
        result = "ValueError"
    with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
        f.write(result)
    dist.destroy_process_group()


MICRO = 2


def _apply_target(target, g: torch.Tensor) -> None:
    """What the grad_weight GEMM does with a GradTarget (fp32 arithmetic, one rounding)."""
    if target.addend is not None:
        target.out.copy_((target.addend + g.float()).to(target.out.dtype))
    elif target.accumulate:
        target.out.add_(g.float())
    else:
        target.out.copy_(g.to(target.out.dtype))


def _micro_grad(rank: int, micro: int, n: int, shape) -> torch.Tensor:
    g = torch.Generator().manual_seed(5000 + 100 * rank + 10 * micro + n)
    return torch.randn(shape[0], shape[1], generator=g) * 1e-2


def _accum_worker(rank: int, world: int, out_dir: str) -> None:
    _init(rank, world, out_dir)
    from local_ai_training_b200.dist import RatchetDataParallel

    model = _StubModel()
    ddp = RatchetDataParallel(model, accumulation_steps=MICRO)
    for micro in range(MICRO):
        for n in reversed(range(len(SHAPES))):
            layer = model.layers[n]
            target = ddp.grad_target(layer)
            assert target.last == (micro == MICRO - 1)
            _apply_target(target, _micro_grad(rank, micro, n, SHAPES[n][:2]))
            ddp.grad_ready(layer)
        # the support gradient accumulates over micro-batches as autograd does
        g = torch.full((6,), float(rank + 1 + micro))
        model.norm.grad = g if model.norm.grad is None else model.norm.grad + g
    extra = "none"
    try:  # a third micro-batch before the update is refused
        ddp.grad_target(model.layers[0])
    except RuntimeError:
        extra = "RuntimeError"
    stats = ddp.step(torch.optim.SGD([model.norm], lr=1.0))
    torch.save({"packed": [l.packed.clone() for l in model.layers],
                "norm_grad": model.norm.grad.clone(), "extra": extra,
                "stats": [int(stats.positive_moves), int(stats.negative_moves),
                          int(stats.total_weights)]},
               os.path.join(out_dir, f"rank{rank}.pt"))
    dist.destroy_process_group()


def test_accumulated_micro_batches_equal_one_update_of_the_mean(tmp_path):
    """Two ranks x two micro-batches: each rank's bf16 total round(g0 + g1), summed across ranks
    (bf16), divided by 4, then one update -- identical on both ranks."""
    world = 2
    tmp_path = _run_ranks(_accum_worker, world, tmp_path)
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    assert res[0]["extra"] == res[1]["extra"] == "RuntimeError"
    for a, b in zip(res[0]["packed"], res[1]["packed"]):
        assert torch.equal(a, b)
    # support: mean over ranks and micro-batches of (rank + 1 + micro)
    assert torch.equal(res[0]["norm_grad"], torch.full((6,), 2.0))
    fresh = _StubModel()
    counts = np.zeros(4, np.int64)
    for n, (o, i, beta) in enumerate(SHAPES):
        totals = [(_micro_grad(r, 0, n, (o, i)) + _micro_grad(r, 1, n, (o, i))).to(torch.bfloat16)
                  for r in range(world)]
        g = (totals[0].float() + totals[1].float()).to(torch.bfloat16).float() * 0.25
        ema = np.zeros(o, np.float32) if beta > 0 else None
        out = O.ratchet_update(g.numpy(), fresh.layers[n].packed.numpy(), max_code=MAX_CODE,
                               threshold=THRESHOLD, rms_ema=ema, beta=beta)
        np.testing.assert_array_equal(res[0]["packed"][n].numpy(), out["packed"])
        counts += out["counts"]
    assert res[0]["stats"][:2] == counts[:2].tolist()
    assert res[0]["stats"][2] == sum(o * i for o, i, _ in SHAPES)


def test_single_process_accumulation_without_distributed():
    """No process group: world 1, the micro-batch gradients accumulate and one update runs."""
    from local_ai_training_b200.dist import RatchetDataParallel

    assert not dist.is_initialized()
    model = _StubModel()
    ddp = RatchetDataParallel(model, accumulation_steps=MICRO)
    assert ddp.world == 1 and ddp.rank == 0
    for micro in range(MICRO):
        for n in reversed(range(len(SHAPES))):
            layer = model.layers[n]
            _apply_target(ddp.grad_target(layer), _micro_grad(0, micro, n, SHAPES[n][:2]))
            ddp.grad_ready(layer)
    model.norm.grad = torch.full((6,), 3.0)
    ddp.step(torch.optim.SGD([model.norm], lr=1.0))
    assert torch.equal(model.norm.grad, torch.full((6,), 1.5))
    fresh = _StubModel()
    for n, (o, i, beta) in enumerate(SHAPES):
        g = (_micro_grad(0, 0, n, (o, i)) + _micro_grad(0, 1, n, (o, i))).to(torch.bfloat16)
        g = g.float() * 0.5
        ema = np.zeros(o, np.float32) if beta > 0 else None
        out = O.ratchet_update(g.numpy(), fresh.layers[n].packed.numpy(), max_code=MAX_CODE,
                               threshold=THRESHOLD, rms_ema=ema, beta=beta)
        np.testing.assert_array_equal(model.layers[n].packed.numpy(), out["packed"])
