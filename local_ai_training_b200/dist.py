"""Deferred ratchet updates, gradient accumulation and data parallelism over torch.distributed.

The reference trains on one device with one batch per update; its step is forward, backward with
the fused per-layer update (ratchet.py:18-182, 487-537), then `RatchetGPT.ratchet_update`
(model.py) and the optimizer for the support parameters.  `RatchetDataParallel` keeps the result
of that step exact while it

* defers the update of every layer to after backward and runs all of them in one or two
  grouped launches (rows are independent, and each layer's grad_input has read its codes
  before the update, so the state equals updating each layer inside its own backward);
* accumulates grad_W over `accumulation_steps` micro-batches: the first micro-batch writes the
  layer's fp32 accumulator, the next ones add to it, and the last one writes the bf16-rounded
  total (`round(acc + its own grad_W)`) -- the reference's bf16 rounding of the GEMM output
  (ratchet.py:162-163) happens once, on the accumulated sum;
* splits the tokens of a step across P ranks (one process per GPU):
  - codes, row scales and `packed` stay replicated (every rank runs every GEMM locally);
  - rank r owns rows [r·N/P, (r+1)·N/P) of every ratchet matrix [N, K] (N % P == 0);
  - the bf16 grad_W total is reduce-scattered (sum) as soon as backward produces it, so rank r
    receives the summed rows it owns while backward continues;
  - the update runs on the owned rows only, on the gradient of the global mean loss
    (sum / (P·micro-batches), applied inside the update kernel; rows are independent, so the
    row RMS over the full K is exact), then an all-gather of the owned `packed` rows (1 byte per
    weight: code and pressure) and of `rms_ema` re-replicates the state, and the int8 code
    mirror is re-derived from `packed`;
  - support parameters (embeddings, RMSNorm weights, trainable scales) have their gradients
    averaged with one all-reduce before the optimizer step; the move counters and gradient-RMS
    sums of the step are summed across ranks, so `ratchet_update` reports global statistics.

With one process (torch.distributed not initialised, or a one-rank group) there are no
collectives.  No data-path collective other than these; no remote memory is read by any kernel.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor

from . import _lib
from .ratchet import DiscreteRatchetLinear, RatchetUpdateStats, ratchet_update_grouped


@dataclass
class GradTarget:
    """Where one micro-batch's grad_W of a layer goes: `out` (+)= grad_W when `accumulate`, or
    out = round(addend + grad_W) when `addend` is given, else out = round(grad_W)."""

    out: Tensor
    accumulate: bool = False
    addend: Tensor | None = None
    last: bool = True  # the micro-batch that completes the layer's gradient of the step


@dataclass
class _LayerState:
    layer: DiscreteRatchetLinear
    row_start: int
    row_end: int
    grad: Tensor | None = None      # bf16 [N, K]: this rank's grad_W total of the step
    shard: Tensor | None = None     # bf16 [N/P, K]: the summed owned rows (grad itself at P=1)
    acc: Tensor | None = None       # fp32 [N, K]: accumulator over the earlier micro-batches
    micro: int = 0                  # micro-batch gradients delivered this step
    work: object | None = None      # pending reduce-scatter


class RatchetDataParallel:
    """Deferred, accumulated and (across ranks) row-sharded ratchet updates for the layers of
    `model` (see the module docstring).

    Usage per step::

        for tokens in micro_batches:           # accumulation_steps of them
            loss = model(tokens); loss.backward()
        stats = ddp.step(optimizer)            # support sync, owned-row update, AdamW, gather
    """

    def __init__(self, model: torch.nn.Module, group: dist.ProcessGroup | None = None, *,
                 bucket_layers: int = 4, accumulation_steps: int = 1) -> None:
        """bucket_layers: gradients of this many consecutive layers (in backward order) are
        reduce-scattered as one batched group of collectives (one NCCL launch), the last group
        when the first layer's gradient arrives.  accumulation_steps: micro-batches (backward
        passes) per update."""
        if group is not None or (dist.is_available() and dist.is_initialized()):
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
            self._nccl = dist.get_backend(group) == "nccl"
        else:
            self.world, self.rank, self._nccl = 1, 0, False
        if accumulation_steps < 1:
            raise ValueError("accumulation_steps must be at least 1")
        self.model = model
        self.group = group
        self.accumulation_steps = int(accumulation_steps)
        self.bucket_layers = max(1, int(bucket_layers))
        self._pending: list[_LayerState] = []
        layers = (model.ratchet_layers() if hasattr(model, "ratchet_layers") else
                  [m for m in model.modules() if isinstance(m, DiscreteRatchetLinear)])
        self.states: list[_LayerState] = []
        for layer in layers:
            if not layer.fuse_backward_update or layer.matmul_mode == "fp32":
                raise ValueError("data-parallel ratchet layers need fuse_backward_update=True and "
                                 "matmul_mode 'bf16' or 'int8'")
            if layer.out_features % self.world != 0:
                raise ValueError(f"out_features {layer.out_features} is not divisible by the "
                                 f"{self.world} ranks")
            rows = layer.out_features // self.world
            self.states.append(_LayerState(layer, self.rank * rows, (self.rank + 1) * rows))
            layer._dp = self
            # each rank rounds its own tokens' gradient: give it its own stochastic-rounding
            # stream (the rank enters the Philox key next to the layer id)
            layer.sr_layer = (layer.sr_layer & 0xFFFF) | (self.rank << 16)
        self._by_layer = {id(s.layer): s for s in self.states}
        # support parameters: everything trainable, trainable ratchet scales included (their
        # gradient is linear in grad_W, so averaging local contributions is exact)
        self.support = [p for p in model.parameters() if p.requires_grad]

    # ------------------------------------------------------------------ called from backward
    def grad_target(self, layer: DiscreteRatchetLinear) -> GradTarget:
        """The buffer this micro-batch's grad_W of `layer` is written to (see GradTarget)."""
        state = self._by_layer[id(layer)]
        pk = layer.packed
        n, k = layer.out_features, layer.in_features
        if state.grad is None or state.grad.device != pk.device:
            state.grad = torch.empty(n, k, device=pk.device, dtype=torch.bfloat16)
            state.shard = (state.grad if self.world == 1 else
                           torch.empty(n // self.world, k, device=pk.device,
                                       dtype=torch.bfloat16))
            state.acc = None
        if state.micro >= self.accumulation_steps:
            raise RuntimeError(
                "ratchet layer produced more gradients than accumulation_steps "
                f"({self.accumulation_steps}) before ratchet_update")
        m, last = state.micro, state.micro == self.accumulation_steps - 1
        if self.accumulation_steps == 1:
            return GradTarget(state.grad)
        if state.acc is None or state.acc.device != pk.device:
            state.acc = torch.empty(n, k, device=pk.device, dtype=torch.float32)
        if last:
            return GradTarget(state.grad, addend=state.acc)
        return GradTarget(state.acc, accumulate=m > 0, last=False)

    def grad_buffer(self, layer: DiscreteRatchetLinear) -> Tensor:
        """The bf16 buffer of a single-micro-batch step (accumulation_steps == 1)."""
        target = self.grad_target(layer)
        if target.accumulate or target.addend is not None:
            raise RuntimeError("grad_buffer is the single-micro-batch form; use grad_target")
        return target.out

    def grad_ready(self, layer: DiscreteRatchetLinear) -> None:
        state = self._by_layer[id(layer)]
        state.micro += 1
        if state.micro < self.accumulation_steps:
            return
        if self.world == 1:
            state.work = _Done()
            return
        state.work = _Pending()
        self._pending.append(state)
        if len(self._pending) >= self.bucket_layers or state is self.states[0]:
            self._flush()

    def _flush(self) -> None:
        """Starts the reduce-scatters of the pending layers (one batched group under NCCL)."""
        pending, self._pending = self._pending, []
        if not pending:
            return
        op = dist.ReduceOp.SUM
        if self._nccl and len(pending) > 1:
            device = pending[0].grad.device
            with dist._coalescing_manager(group=self.group, device=device, async_ops=True) as cm:
                for st in pending:
                    dist.reduce_scatter_tensor(st.shard, st.grad, op=op, group=self.group)
            for st in pending:
                st.work = cm
        else:
            for st in pending:
                st.work = dist.reduce_scatter_tensor(st.shard, st.grad, op=op, group=self.group,
                                                     async_op=True)

    # ------------------------------------------------------------------ after backward
    @torch.no_grad()
    def synchronize_gradients(self) -> None:
        """Averages the support-parameter gradients over ranks and micro-batches (one all-reduce
        of a flat fp32 buffer across ranks)."""
        self._finish_support(self._start_support())

    @torch.no_grad()
    def ratchet_update(self, *, validate: bool = False) -> RatchetUpdateStats:
        """Updates the owned rows of every layer from the summed gradient, re-replicates `packed`
        (and `rms_ema`), sums the step statistics across ranks and returns the model's
        aggregated update statistics (ratchet.py:627-668 / model.py ratchet_update)."""
        self._update_owned_rows()
        self._finish_gathers(self._start_gathers())
        return self._finish_stats(validate)

    @torch.no_grad()
    def step(self, optimizer: torch.optim.Optimizer, *,
             validate: bool = False) -> RatchetUpdateStats:
        """synchronize_gradients + optimizer.step + ratchet_update with the communication
        overlapped: the support all-reduce runs during the owned-row updates, the re-replication
        all-gather during the optimizer step."""
        support = self._start_support()
        self._update_owned_rows()
        gathers = self._start_gathers()
        self._finish_support(support)
        optimizer.step()
        self._finish_gathers(gathers)
        return self._finish_stats(validate)

    def _start_support(self):
        grads = [p.grad for p in self.support if p.grad is not None]
        if not grads:
            return None
        if self.world == 1:
            if self.accumulation_steps > 1:  # mean over the micro-batches' mean losses
                torch._foreach_mul_(grads, 1.0 / self.accumulation_steps)
            return None
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        return work, flat, grads

    def _finish_support(self, handle) -> None:
        if handle is None:
            return
        work, flat, grads = handle
        ev = _lib.prof_start(flat)
        work.wait()
        if ev is not None:
            _lib.prof_stop(ev, "comm_support_all_reduce_wait", flat, 0.0, 0.0)
        flat.mul_(1.0 / (self.world * self.accumulation_steps))
        offset = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[offset:offset + n].view_as(g))
            offset += n

    def _update_owned_rows(self) -> None:
        for state in self.states:
            if state.work is None:
                raise RuntimeError("ratchet layer has no pending effective-weight gradient "
                                   f"(or fewer than accumulation_steps={self.accumulation_steps} "
                                   "micro-batches)")
        self._flush()  # layers whose gradient arrived after the last full group
        waited = set()
        ev = _lib.prof_start(self.states[0].layer.packed) if self.world > 1 else None
        for state in self.states:
            if id(state.work) not in waited:  # a batched group is waited for once
                state.work.wait()
                waited.add(id(state.work))
            state.work = None
            state.micro = 0
        if ev is not None:  # how long the compute stream waited for the reduce-scatters
            _lib.prof_stop(ev, "comm_reduce_scatter_wait", self.states[0].layer.packed, 0.0, 0.0)
        # the gradient of the global mean loss: the sum over ranks and micro-batches, divided
        mul = 1.0 / (self.world * self.accumulation_steps)
        whole = {s.layer: s.layer.out_features * s.layer.in_features for s in self.states}
        grouped = [s for s in self.states if _is_device_layer(s.layer)]
        if grouped:
            ratchet_update_grouped([(s.layer, s.shard, s.row_start, s.row_end, mul)
                                    for s in grouped], stats_weights=whole)
        for state in self.states:
            if _is_device_layer(state.layer):
                continue
            # any other object with the layer interface: its own update on the scaled rows
            shard = state.shard
            if mul != 1.0:
                shard.mul_(mul)
            state.layer._capture_weight_gradient(shard, state.row_start, state.row_end,
                                                 round_bf16=False)
            state.layer._pending_stats_total_weights = whole[state.layer]

    def _start_gathers(self):
        """Re-replication: every layer's owned packed rows (and rms_ema rows), as one group of
        collectives where the backend can batch them."""
        if self.world == 1:
            return None
        pairs = []
        for state in self.states:
            layer = state.layer
            pk = layer.packed
            pairs.append((pk, pk[state.row_start:state.row_end]))
            if layer.rms_ema_beta > 0.0:
                pairs.append((layer.rms_ema, layer.rms_ema[state.row_start:state.row_end]))
        return self._all_gather_many(pairs)

    def _finish_gathers(self, handle) -> None:
        if handle is None:
            return
        ev = _lib.prof_start(self.states[0].layer.packed)
        for work in handle:
            work.wait()
        if ev is not None:
            _lib.prof_stop(ev, "comm_all_gather_wait", self.states[0].layer.packed, 0.0, 0.0)
        for state in self.states:
            state.layer._refresh_code_mirror()

    def _finish_stats(self, validate: bool) -> RatchetUpdateStats:
        if self.world > 1:
            self._reduce_step_stats()
        if hasattr(self.model, "ratchet_update"):
            return self.model.ratchet_update(validate=validate)
        updates = [s.layer.ratchet_update(validate=validate) for s in self.states]
        return _aggregate(updates, validate)

    def _all_gather_many(self, pairs: list[tuple[Tensor, Tensor]]) -> list:
        """Starts in-place all-gathers (each input is this rank's block of its output); returns
        the handles to wait for."""
        if self._nccl:
            device = pairs[0][0].device
            with dist._coalescing_manager(group=self.group, device=device, async_ops=True) as cm:
                for out, inp in pairs:
                    dist.all_gather_into_tensor(out, inp, group=self.group)
            return [cm]
        return [dist.all_gather_into_tensor(out, inp.contiguous(), group=self.group,
                                            async_op=True) for out, inp in pairs]

    def _reduce_step_stats(self) -> None:
        """Sums each layer's [4 counters, rms sum] across ranks in one all-reduce (float64 holds
        the integer counters exactly)."""
        bufs = [s.layer._pending_buf for s in self.states]
        counts = torch.stack([b[:4] for b in bufs]).to(torch.float64)
        rms = torch.stack([b[4:].view(torch.float32)[:1] for b in bufs]).to(torch.float64)
        both = torch.cat([counts, rms], dim=1)
        dist.all_reduce(both, op=dist.ReduceOp.SUM, group=self.group)
        for i, b in enumerate(bufs):
            b[:4].copy_(both[i, :4].round().to(torch.int64))
            b[4:].view(torch.float32)[:1].copy_(both[i, 4:5].to(torch.float32))
        for s in self.states:
            s.layer._pending_stats_rms_sum = s.layer._pending_rms[0]

    def state_checksum(self) -> Tensor:
        """int64 [2] device tensor: the sum and the position-weighted sum of every byte of every
        layer's `packed` (replicated state: equal on every rank after a step)."""
        total = None
        for i, state in enumerate(self.states):
            pk = state.layer.packed.reshape(-1).to(torch.int64)
            weights = torch.arange(pk.numel(), device=pk.device, dtype=torch.int64) % 65521 + 1
            part = torch.stack([pk.sum(), (pk * weights).sum() * (i + 1)])
            total = part if total is None else total + part
        return total

    def detach(self) -> None:
        """Returns the layers to single-process training with updates inside backward."""
        for state in self.states:
            state.layer._dp = None
            state.layer.sr_layer &= 0xFFFF


def _is_device_layer(layer) -> bool:
    return isinstance(layer, DiscreteRatchetLinear) and layer.packed.is_cuda


class _Done:
    def wait(self) -> None:
        return None


class _Pending:
    """Placeholder until the layer's reduce-scatter group is started."""

    def wait(self) -> None:
        raise RuntimeError("reduce-scatter was never started")


def _aggregate(updates: list[RatchetUpdateStats], validate: bool) -> RatchetUpdateStats:
    stats = RatchetUpdateStats(
        total_weights=sum(u.total_weights for u in updates),
        positive_moves=sum(u.positive_moves for u in updates),
        negative_moves=sum(u.negative_moves for u in updates),
        blocked_positive_moves=sum(u.blocked_positive_moves for u in updates),
        blocked_negative_moves=sum(u.blocked_negative_moves for u in updates),
        gradient_rms_mean=(sum(u.gradient_rms_mean for u in updates) / len(updates)
                           if updates else 0.0),
    )
    return stats.materialize() if validate else stats
