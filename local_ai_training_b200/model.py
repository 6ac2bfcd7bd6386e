"""GPT decoder whose dense matrices are ratchet layers (reference model.py) on sm_100a.

Same configuration fields, module tree, parameter names and initialisation order as the reference
(so seeded models and state_dicts match); the int8 path routes through the fused producers and
the ratchet layers of this package.  The lm_head and the token cross-entropy run as fused CUDA
kernels of this library (cross_entropy.py); attention (SDPA), the embedding lookup and the
optimizer stay PyTorch ops.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal

import torch
import torch.utils.checkpoint
from torch import Tensor, nn
from torch.nn import functional as F

from .int8_fused import (FusedGELUQuantizeFn, FusedRMSNormQuantizeFn, FusedTransposeQuantizeFn,
                         QKVHeadsFn)
from .ratchet import DiscreteRatchetLinear, RatchetEmbedding, RatchetUpdateStats, grad_plan_of


@dataclass(frozen=True)
class ModelConfig:
    vocab_size: int
    block_size: int = 128
    n_layer: int = 2
    n_head: int = 4
    n_embd: int = 128
    dropout: float = 0.0
    pressure_threshold: int = 8
    bucket_low: float = 0.5
    bucket_high: float = 1.5
    trainable_scale: bool = False
    rms_ema_beta: float = 0.0
    pressure_leak_period: int = 0
    compile_update: bool = False
    gradient_checkpointing: bool = False
    matmul_mode: Literal["fp32", "bf16", "int8"] = "fp32"
    int8_backward: bool = False
    qat: bool = False
    ratchet_embedding: bool = False
    # int8 mode: carry the producer dummies (and so the qkv/expand outputs and every ratchet
    # grad_input) in bf16.  Those tensors hold bf16-rounded values in the reference too (GEMM
    # epilogue, SDPA, GELU backward), so results are identical while HBM traffic halves; the
    # contract layer keeps an fp32 output so the residual-stream gradient stays fp32.
    bf16_activations: bool = True
    # int8 mode with targets: the self-quantising lm_head GEMM and the token cross-entropy run as
    # one autograd step (local_ai_training_b200.cross_entropy); False keeps F.cross_entropy
    fused_cross_entropy: bool = True
    # with the fused cross-entropy: > 0 runs the lm_head and the loss over blocks of this many
    # tokens, recomputing each block's logits in backward, and forward returns (None, loss) -- no
    # [tokens, vocab] logits or logit gradient is stored; 0 returns the logits as the reference does
    logits_chunk_rows: int = 0
    # int8 mode: the residual adds of each block run in the epilogue of the sublayer's last GEMM
    # and in the RMSNorm backward kernel (TransformerBlock.forward); False keeps `x + f(x)`
    fused_residual: bool = True
    # int8 backward: the backward kernel that produces a ratchet layer's output gradient (RMSNorm
    # backward, GELU backward, the q|k|v head gather) also stochastic-rounds it for the layer's
    # int8 grad_input GEMM (GradientQuantPlan).  Results are identical either way; off by default
    # because on B200 the fused row passes (instruction-bound Philox rounding behind the
    # producer's own row reduction) ran slower than the two separate passes
    fused_grad_quant: bool = False
    # int8 mode: each fused producer (RMSNorm / GELU / head-transpose quantisers) also writes the
    # bf16 dequantised rows its consuming layer's grad_weight GEMM uses, saved instead of the int8
    # rows, so backward has no dequant pass (identical values; 2 instead of 1 byte per saved
    # activation)
    producer_dequant: bool = True

    def __post_init__(self) -> None:
        if min(self.vocab_size, self.block_size, self.n_layer, self.n_head, self.n_embd) <= 0:
            raise ValueError("model dimensions must be positive")
        if self.n_embd % self.n_head != 0:
            raise ValueError("n_embd must be divisible by n_head")
        if not 0 <= self.dropout < 1:
            raise ValueError("dropout must be in [0, 1)")
        if self.matmul_mode not in {"fp32", "bf16", "int8"}:
            raise ValueError("matmul_mode must be fp32, bf16, or int8")


def _sinusoidal_positions(block_size: int, n_embd: int) -> Tensor:
    positions = torch.arange(block_size, dtype=torch.float32)[:, None]
    even_dimensions = torch.arange(0, n_embd, 2, dtype=torch.float32)
    frequencies = torch.exp(-math.log(10_000.0) * even_dimensions / n_embd)
    encoding = torch.zeros(block_size, n_embd, dtype=torch.float32)
    encoding[:, 0::2] = torch.sin(positions * frequencies)
    if n_embd > 1:
        encoding[:, 1::2] = torch.cos(positions * frequencies[: encoding[:, 1::2].shape[1]])
    return encoding


def _linear(config: ModelConfig, in_features: int, out_features: int, max_code: int | None):
    if max_code is None:
        return nn.Linear(in_features, out_features, bias=False)
    if config.qat:
        raise ValueError("the QAT control arm (master weights) is not part of this build")
    return DiscreteRatchetLinear(
        in_features,
        out_features,
        max_code=max_code,
        pressure_threshold=config.pressure_threshold,
        bucket_low=config.bucket_low,
        bucket_high=config.bucket_high,
        trainable_scale=config.trainable_scale,
        rms_ema_beta=config.rms_ema_beta,
        pressure_leak_period=config.pressure_leak_period,
        compile_update=config.compile_update,
        matmul_mode=config.matmul_mode,
        fuse_backward_update=True,
        int8_backward=config.int8_backward,
    )


class CausalSelfAttention(nn.Module):
    def __init__(self, config: ModelConfig, *, max_code: int | None) -> None:
        super().__init__()
        self.qkv = _linear(config, config.n_embd, 3 * config.n_embd, max_code)
        self.projection = _linear(config, config.n_embd, config.n_embd, max_code)
        self.n_head = config.n_head
        self.head_size = config.n_embd // config.n_head
        self.dropout = config.dropout
        self.fused_grad_quant = config.fused_grad_quant
        self.producer_dequant = config.producer_dequant

    def forward(self, inputs: Tensor, *, inputs_int8: Tensor | None = None,
                inputs_scale: Tensor | None = None, residual: Tensor | None = None,
                inputs_dequant: Tensor | None = None) -> Tensor:
        """residual (int8 path): returns residual + attention(...), the add in the projection's
        GEMM epilogue.  inputs_dequant: the producer's bf16 dequantised rows (qkv grad_weight)."""
        batch_size, sequence_length, channels = inputs.shape
        if inputs_int8 is not None:
            qkv = self.qkv(inputs, inputs_int8=inputs_int8, inputs_scale=inputs_scale,
                           inputs_dequant=inputs_dequant)
        else:
            qkv = self.qkv(inputs)
        plan = grad_plan_of(qkv) if self.fused_grad_quant else None
        if plan is not None:
            # the gradients of the three head views come back as the projection's quantised
            # output gradient in one kernel
            query, key, value = QKVHeadsFn.apply(qkv, self.n_head, plan)
        else:
            def heads(tensor: Tensor) -> Tensor:
                return tensor.view(batch_size, sequence_length, self.n_head,
                                   self.head_size).transpose(1, 2)

            query, key, value = (heads(t) for t in qkv.chunk(3, dim=-1))

        attended = F.scaled_dot_product_attention(
            query, key, value,
            dropout_p=self.dropout if self.training else 0.0, is_causal=True,
        )
        if getattr(self.projection, "matmul_mode", "fp32") == "int8":
            attn_int8, attn_scale, dummy_joined, *dq = FusedTransposeQuantizeFn.apply(
                attended, self.producer_dequant)
            return self.projection(dummy_joined, inputs_int8=attn_int8, inputs_scale=attn_scale,
                                   residual=residual, inputs_dequant=dq[0] if dq else None)
        joined = attended.transpose(1, 2).contiguous().view(batch_size, sequence_length, channels)
        out = self.projection(joined)
        return out if residual is None else residual + out


class FeedForward(nn.Module):
    def __init__(self, config: ModelConfig, *, max_code: int | None) -> None:
        super().__init__()
        hidden_size = 4 * config.n_embd
        self.expand = _linear(config, config.n_embd, hidden_size, max_code)
        self.contract = _linear(config, hidden_size, config.n_embd, max_code)
        self.dropout = config.dropout
        self.fused_grad_quant = config.fused_grad_quant
        self.producer_dequant = config.producer_dequant
        self.dummy_dtype = None
        if config.matmul_mode == "int8" and config.bf16_activations and max_code is not None:
            self.dummy_dtype = torch.bfloat16
            self.contract.output_dtype = torch.float32

    def forward(self, inputs: Tensor, *, inputs_int8: Tensor | None = None,
                inputs_scale: Tensor | None = None, residual: Tensor | None = None,
                inputs_dequant: Tensor | None = None) -> Tensor:
        """residual (int8 path, no active dropout): returns residual + feed_forward(...), the add
        in the contraction's GEMM epilogue.  inputs_dequant: the producer's bf16 dequantised rows
        (expand grad_weight)."""
        if inputs_int8 is not None:
            expanded = self.expand(inputs, inputs_int8=inputs_int8, inputs_scale=inputs_scale,
                                   inputs_dequant=inputs_dequant)
        else:
            expanded = self.expand(inputs)
        fuse_residual = residual is not None and (self.dropout == 0.0 or not self.training)
        if getattr(self.contract, "matmul_mode", "fp32") == "int8":
            plan = grad_plan_of(expanded) if self.fused_grad_quant else None
            gelu_int8, gelu_scale, dummy_gelu, *dq = FusedGELUQuantizeFn.apply(
                expanded, self.dummy_dtype, plan, self.producer_dequant)
            contracted = self.contract(dummy_gelu, inputs_int8=gelu_int8, inputs_scale=gelu_scale,
                                       residual=residual if fuse_residual else None,
                                       inputs_dequant=dq[0] if dq else None)
        else:
            contracted = self.contract(F.gelu(expanded))
            fuse_residual = False
        if fuse_residual:
            return contracted
        out = F.dropout(contracted, p=self.dropout, training=self.training)
        return out if residual is None else residual + out


class TransformerBlock(nn.Module):
    def __init__(self, config: ModelConfig, *, max_code: int | None) -> None:
        super().__init__()
        self.attention_norm = nn.RMSNorm(config.n_embd)
        self.attention = CausalSelfAttention(config, max_code=max_code)
        self.feed_forward_norm = nn.RMSNorm(config.n_embd)
        self.feed_forward = FeedForward(config, max_code=max_code)
        self.dummy_dtype = (torch.bfloat16 if config.matmul_mode == "int8" and config.bf16_activations
                            and max_code is not None else None)
        self.fused_residual = config.fused_residual and max_code is not None
        self.fused_grad_quant = config.fused_grad_quant
        self.producer_dequant = config.producer_dequant

    def forward(self, inputs: Tensor) -> Tensor:
        # int8 path with fused residuals: the RMSNorm producer hands x on as the residual, the
        # sublayer's last GEMM adds it in its epilogue, and in backward the residual gradient is
        # added to the RMSNorm input gradient by the same kernel (same values as `x + f(x)`)
        fused = self.fused_residual and inputs.dtype == torch.float32
        if getattr(self.attention.qkv, "matmul_mode", "fp32") == "int8":
            if fused:
                # with the residual fused, this norm's input gradient is the whole gradient of
                # `inputs`: quantise it for the ratchet layer that produced `inputs`, if any
                plan = grad_plan_of(inputs) if self.fused_grad_quant else None
                attn_int8, attn_scale, dummy_in, res, *dq = FusedRMSNormQuantizeFn.apply(
                    inputs, self.attention_norm.weight, 1e-5, self.dummy_dtype, True, plan,
                    self.producer_dequant)
                inputs = self.attention(dummy_in, inputs_int8=attn_int8, inputs_scale=attn_scale,
                                        residual=res, inputs_dequant=dq[0] if dq else None)
            else:
                attn_int8, attn_scale, dummy_in, *dq = FusedRMSNormQuantizeFn.apply(
                    inputs, self.attention_norm.weight, 1e-5, self.dummy_dtype, False, None,
                    self.producer_dequant)
                inputs = inputs + self.attention(dummy_in, inputs_int8=attn_int8,
                                                 inputs_scale=attn_scale,
                                                 inputs_dequant=dq[0] if dq else None)
        else:
            inputs = inputs + self.attention(self.attention_norm(inputs))
        if getattr(self.feed_forward.expand, "matmul_mode", "fp32") == "int8":
            if fused:
                plan = grad_plan_of(inputs) if self.fused_grad_quant else None
                ffn_int8, ffn_scale, dummy_in, res, *dq = FusedRMSNormQuantizeFn.apply(
                    inputs, self.feed_forward_norm.weight, 1e-5, self.dummy_dtype, True, plan,
                    self.producer_dequant)
                inputs = self.feed_forward(dummy_in, inputs_int8=ffn_int8, inputs_scale=ffn_scale,
                                           residual=res, inputs_dequant=dq[0] if dq else None)
            else:
                ffn_int8, ffn_scale, dummy_in, *dq = FusedRMSNormQuantizeFn.apply(
                    inputs, self.feed_forward_norm.weight, 1e-5, self.dummy_dtype, False, None,
                    self.producer_dequant)
                inputs = inputs + self.feed_forward(dummy_in, inputs_int8=ffn_int8,
                                                    inputs_scale=ffn_scale,
                                                    inputs_dequant=dq[0] if dq else None)
        else:
            inputs = inputs + self.feed_forward(self.feed_forward_norm(inputs))
        return inputs


class RatchetGPT(nn.Module):
    def __init__(self, config: ModelConfig, *, max_code: int | None) -> None:
        super().__init__()
        self.config = config
        self.max_code = max_code
        if max_code is not None and config.ratchet_embedding:
            self.token_embedding = RatchetEmbedding(
                config.vocab_size, config.n_embd, max_code=max_code,
                pressure_threshold=config.pressure_threshold, bucket_low=config.bucket_low,
                bucket_high=config.bucket_high, trainable_scale=config.trainable_scale,
                compile_update=config.compile_update, rms_ema_beta=config.rms_ema_beta,
                pressure_leak_period=config.pressure_leak_period,
            )
        else:
            self.token_embedding = nn.Embedding(config.vocab_size, config.n_embd)
        self.register_buffer("position_encoding", _sinusoidal_positions(config.block_size, config.n_embd))
        self.blocks = nn.ModuleList(TransformerBlock(config, max_code=max_code)
                                    for _ in range(config.n_layer))
        self.final_norm = nn.RMSNorm(config.n_embd)
        self.lm_head = _linear(config, config.n_embd, config.vocab_size, max_code)
        # distinct Philox layer ids for the stochastic rounding of each ratchet layer
        for index, module in enumerate(m for m in self.modules() if isinstance(m, DiscreteRatchetLinear)):
            module.sr_layer = index
        self._step_stats: Tensor | None = None

    def forward(self, tokens: Tensor, targets: Tensor | None = None) -> tuple[Tensor, Tensor | None]:
        if tokens.ndim != 2:
            raise ValueError("tokens must have shape (batch, sequence)")
        sequence_length = tokens.shape[1]
        if sequence_length > self.config.block_size:
            raise ValueError("token sequence exceeds configured block_size")
        if self.training and torch.is_grad_enabled():
            self._assign_stats_slots(tokens.device)
        hidden = self.token_embedding(tokens) + self.position_encoding[:sequence_length]
        for block in self.blocks:
            if self.config.gradient_checkpointing and self.training:
                hidden = torch.utils.checkpoint.checkpoint(block, hidden, use_reentrant=False)
            else:
                hidden = block(hidden)
        normed = self.final_norm(hidden)
        if targets is not None and targets.shape != tokens.shape:
            raise ValueError("targets must have the same shape as tokens")
        if targets is not None and self.config.fused_cross_entropy:
            from .cross_entropy import fused_lm_head_applies, lm_head_cross_entropy

            if fused_lm_head_applies(self.lm_head, normed):
                return lm_head_cross_entropy(self.lm_head, normed, targets,
                                             chunk_rows=self.config.logits_chunk_rows)
        logits = self.lm_head(normed)
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.flatten(0, 1), targets.flatten())
        return logits, loss

    def ratchet_layers(self) -> list[DiscreteRatchetLinear]:
        if getattr(self, "_ratchet_layers", None) is None:
            self._ratchet_layers = [m for m in self.modules() if isinstance(m, DiscreteRatchetLinear)]
        return self._ratchet_layers

    def _assign_stats_slots(self, device: torch.device) -> None:
        """One int64 [layers, 5] buffer per train step collects every fused layer's move counters
        and gradient-rms sum, so the unvalidated model update reduces them in one pass."""
        layers = self.ratchet_layers()
        if device.type != "cuda" or not layers or self._step_stats is not None:
            return
        if not all(l.fuse_backward_update and l._pending_counts is None for l in layers):
            return
        self._step_stats = torch.zeros(len(layers), 5, device=device, dtype=torch.int64)
        for i, layer in enumerate(layers):
            layer._stats_slot = self._step_stats[i]
        if getattr(self, "_out_features_dev", None) is None or self._out_features_dev.device != device:
            self._out_features_dev = torch.tensor([float(max(1, l.out_features)) for l in layers],
                                                  device=device)

    def ratchet_update(self, *, validate: bool = True) -> RatchetUpdateStats:
        layers = self.ratchet_layers()
        buf = self._step_stats
        self._step_stats = None
        if (not validate and buf is not None
                and all(l._stats_slot is not None and l._pending_counts is not None for l in layers)):
            counts = buf[:, :4].sum(dim=0)
            rms = buf[:, 4:].contiguous().view(torch.float32)[:, 0]
            total_weights = 0
            for layer in layers:
                total_weights += layer._pending_stats_total_weights
                layer._reset_pending_stats()
                layer._maybe_leak_pressure()
            return RatchetUpdateStats(
                total_weights=total_weights, positive_moves=counts[0], negative_moves=counts[1],
                blocked_positive_moves=counts[2], blocked_negative_moves=counts[3],
                gradient_rms_mean=(rms / self._out_features_dev).mean())
        per_layer = [module.ratchet_update(validate=validate) for module in layers]
        # counters add over layers; the rms statistic is the mean of the layers' means
        fields = ("total_weights", "positive_moves", "negative_moves", "blocked_positive_moves",
                  "blocked_negative_moves")
        totals = {name: sum(getattr(stats, name) for stats in per_layer) for name in fields}
        rms = [stats.gradient_rms_mean for stats in per_layer]
        combined = RatchetUpdateStats(**totals,
                                      gradient_rms_mean=sum(rms) / len(rms) if rms else 0.0)
        return combined.materialize() if validate else combined

    def discard_pending_gradients(self) -> None:
        for module in self.ratchet_layers():
            module.discard_pending_gradient()


def build_seeded_model(config: ModelConfig, *, max_code: int | None, seed: int) -> RatchetGPT:
    """RatchetGPT(config, max_code) initialised from torch.manual_seed(seed) inside a forked CPU
    RNG, so two calls with one seed give identical models and the caller's generator state is
    unchanged (the reference's seeded-arm helper, model.py:281-285)."""
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        return RatchetGPT(config, max_code=max_code)
