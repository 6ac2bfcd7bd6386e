"""Data-parallel ratchet training: one process per GPU over torch.distributed.

The reference trains on one device; its step is forward, backward with the fused per-layer update
(ratchet.py:18-182, 487-537), then `RatchetGPT.ratchet_update` (model.py) and the optimizer for the
support parameters.  Data parallelism splits the tokens of a step across ranks and keeps the
update exact for the global batch:

* codes, row scales and `packed` stay replicated (every rank runs every GEMM locally);
* rank r owns rows [r·N/P, (r+1)·N/P) of every ratchet matrix [N, K] (P ranks, N % P == 0);
* backward writes each layer's bf16-rounded grad_W (the value the reference hands its update,
  ratchet.py:162-163) into a per-layer buffer and immediately starts an asynchronous
  reduce-scatter (sum), so rank r receives the summed rows it owns while backward continues;
* the update runs on the owned rows only, on the gradient of the global mean loss (sum / P;
  rows are independent, so the row RMS over the full K is exact), then an all-gather of the
  owned `packed` rows (1 byte per weight: code and pressure) and of `rms_ema` re-replicates the
  state, and the int8 code mirror is re-derived from `packed`;
* support parameters (embeddings, RMSNorm weights, trainable scales) have their gradients
  averaged with one all-reduce before the optimizer step; the move counters and gradient-RMS
  sums of the step are summed across ranks, so `ratchet_update` reports global statistics.

No data-path collective other than these; no remote memory is read by any kernel.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor

from .ratchet import DiscreteRatchetLinear, RatchetUpdateStats


@dataclass
class _LayerState:
    layer: DiscreteRatchetLinear
    row_start: int
    row_end: int
    grad: Tensor | None = None      # bf16 [N, K]: this rank's grad_W of the step
    shard: Tensor | None = None     # bf16 [N/P, K]: the summed owned rows
    work: object | None = None      # pending reduce-scatter


class RatchetDataParallel:
    """Row-owner data parallelism for the ratchet layers of `model` (see the module docstring).

    Usage per step::

        loss = model(x, y); loss.backward()
        ddp.synchronize_gradients()       # support-parameter gradients averaged
        optimizer.step()
        stats = ddp.ratchet_update()      # owned-row update, state re-replicated, global stats
    """

    def __init__(self, model: torch.nn.Module, group: dist.ProcessGroup | None = None, *,
                 bucket_layers: int = 4) -> None:
        """bucket_layers: gradients of this many consecutive layers (in backward order) are
        reduce-scattered as one batched group of collectives (one NCCL launch), the last group
        when the first layer's gradient arrives."""
        if not dist.is_initialized():
            raise RuntimeError("RatchetDataParallel needs an initialised torch.distributed group")
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.bucket_layers = max(1, int(bucket_layers))
        self._pending: list[_LayerState] = []
        self._nccl = dist.get_backend(group) == "nccl"
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
    def grad_buffer(self, layer: DiscreteRatchetLinear) -> Tensor:
        state = self._by_layer[id(layer)]
        pk = layer.packed
        if state.grad is None or state.grad.device != pk.device:
            state.grad = torch.empty(layer.out_features, layer.in_features, device=pk.device,
                                     dtype=torch.bfloat16)
            state.shard = (state.grad if self.world == 1 else
                           torch.empty(layer.out_features // self.world, layer.in_features,
                                       device=pk.device, dtype=torch.bfloat16))
        if state.work is not None:
            raise RuntimeError("ratchet layer produced a second gradient before ratchet_update "
                               "(gradient accumulation is not supported by the data-parallel "
                               "runtime)")
        return state.grad

    def grad_ready(self, layer: DiscreteRatchetLinear) -> None:
        state = self._by_layer[id(layer)]
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
        """Averages the support-parameter gradients (one all-reduce of a flat fp32 buffer)."""
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
        if self.world == 1:
            return None
        grads = [p.grad for p in self.support if p.grad is not None]
        if not grads:
            return None
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        return work, flat, grads

    def _finish_support(self, handle) -> None:
        if handle is None:
            return
        work, flat, grads = handle
        work.wait()
        flat.mul_(1.0 / self.world)
        offset = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[offset:offset + n].view_as(g))
            offset += n

    def _update_owned_rows(self) -> None:
        for state in self.states:
            if state.work is None:
                raise RuntimeError("ratchet layer has no pending effective-weight gradient")
        self._flush()  # layers whose gradient arrived after the last full group
        waited = set()
        for state in self.states:
            layer = state.layer
            if id(state.work) not in waited:  # a batched group is waited for once
                state.work.wait()
                waited.add(id(state.work))
            state.work = None
            shard = state.shard
            if self.world > 1:
                shard.mul_(1.0 / self.world)  # the gradient of the global mean loss
            layer._capture_weight_gradient(shard, state.row_start, state.row_end,
                                           round_bf16=False)
            layer._pending_stats_total_weights = layer.out_features * layer.in_features

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
        for work in handle:
            work.wait()
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
        if dist.get_backend(self.group) == "nccl":
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

    def detach(self) -> None:
        """Returns the layers to single-process training."""
        for state in self.states:
            state.layer._dp = None
            state.layer.sr_layer &= 0xFFFF


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
