"""CPU fp32 restatement of the reference ratchet GPT train step.

TEST INFRASTRUCTURE AND CPU BASELINE ONLY: tests/ use it as the model-level checker and bench.py
times it as the reported CPU baseline / reference arm.  The product package never imports it.

It restates, in eager torch on the CPU, the reference's fp32 path:
  model.py:23-285      ModelConfig / RatchetGPT module tree and initialisation order
  ratchet.py:18-182    _RatchetMatmul (fp32 mode, fused backward update per row tile)
  ratchet.py:185-301   nibble packing, bucket_pressure, _ratchet_update_core
  ratchet.py:304-403   DiscreteRatchetLinear initialisation
  ratchet.py:487-556   _capture_weight_gradient / _normalize
Pinned against tests/golden/model_tiny.npz (produced by the reference).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor, nn
from torch.nn import functional as F


def pack(code: Tensor, pressure: Tensor, max_code: int) -> Tensor:
    low = (code.to(torch.int16) + max_code) & 0x0F
    high = (pressure.to(torch.int16) + 7) & 0x0F
    return (low | (high << 4)).to(torch.uint8)


def unpack(packed: Tensor, max_code: int) -> tuple[Tensor, Tensor]:
    v = packed.to(torch.int16)
    return ((v & 0x0F) - max_code).to(torch.int8), ((v >> 4) - 7).to(torch.int8)


def update_core(packed: Tensor, z: Tensor, max_code: int, threshold: int, low: float,
                high: float) -> tuple[Tensor, list[Tensor]]:
    mag = z.abs()
    bucket = torch.where(mag >= high, torch.full_like(z, 2, dtype=torch.int16),
                         torch.where(mag >= low, torch.ones_like(z, dtype=torch.int16),
                                     torch.zeros_like(z, dtype=torch.int16)))
    inc = -torch.sign(z).to(torch.int16) * bucket
    code, pressure = unpack(packed, max_code)
    p = pressure.to(torch.int16) + inc
    c = code.to(torch.int16)
    pos_req, neg_req = p >= threshold, p <= -threshold
    pos_mv, neg_mv = pos_req & (c < max_code), neg_req & (c > -max_code)
    c = c + pos_mv.to(torch.int16) - neg_mv.to(torch.int16)
    p = p - pos_req.to(torch.int16) * threshold + neg_req.to(torch.int16) * threshold
    p = p.clamp(-128, 127)
    counts = [pos_mv.sum(), neg_mv.sum(), (pos_req & ~pos_mv).sum(), (neg_req & ~neg_mv).sum()]
    return pack(c.to(torch.int8), p.to(torch.int8), max_code), counts


class RatchetLinearFP32(nn.Module):
    """fp32 ratchet layer with the update fused into backward (reference fuse_backward_update)."""

    def __init__(self, in_features: int, out_features: int, *, max_code: int, threshold: int = 8,
                 low: float = 0.5, high: float = 1.5, eps: float = 1e-8, tile_size: int = 256):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.max_code, self.threshold, self.low, self.high, self.eps = max_code, threshold, low, high, eps
        self.tile_size = tile_size
        ref = torch.empty(out_features, in_features, dtype=torch.float32)
        nn.init.kaiming_uniform_(ref, a=5**0.5)
        scale = (ref.abs().amax(dim=1) / max_code).clamp_min(torch.finfo(torch.float32).eps)
        code = torch.round(ref / scale[:, None]).clamp(-max_code, max_code)
        self.register_buffer("packed", pack(code.to(torch.int8), torch.zeros_like(code, dtype=torch.int8), max_code))
        self.register_buffer("_scale", scale)
        self.moves = torch.zeros(4, dtype=torch.int64)

    def forward(self, x: Tensor) -> Tensor:
        return _FusedFP32.apply(x, self)

    def sink(self, gw: Tensor, start: int, end: int) -> None:
        ms = gw.square().mean(dim=1, keepdim=True)
        z = gw / (ms.sqrt() + self.eps)
        new, counts = update_core(self.packed[start:end], z, self.max_code, self.threshold, self.low, self.high)
        self.packed[start:end] = new
        for i in range(4):
            self.moves[i] += counts[i]


class _FusedFP32(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, layer: RatchetLinearFP32) -> Tensor:
        code, _ = unpack(layer.packed, layer.max_code)
        flat = x.flatten(0, -2)
        ctx.save_for_backward(flat, code, layer._scale.clone())
        ctx.layer, ctx.shape = layer, x.shape
        eff = code.float() * layer._scale[:, None]
        return (flat @ eff.t()).reshape(*x.shape[:-1], code.shape[0])

    @staticmethod
    def backward(ctx, grad: Tensor):
        flat, code, scale = ctx.saved_tensors
        layer = ctx.layer
        g = grad.flatten(0, -2).float()
        grad_input = g @ (code.float() * scale[:, None])
        gt = g.t()
        for start in range(0, code.shape[0], layer.tile_size):
            end = min(start + layer.tile_size, code.shape[0])
            layer.sink(gt[start:end] @ flat, start, end)
        return grad_input.reshape(ctx.shape), None


def _positions(block: int, d: int) -> Tensor:
    pos = torch.arange(block, dtype=torch.float32)[:, None]
    even = torch.arange(0, d, 2, dtype=torch.float32)
    freq = torch.exp(-math.log(10_000.0) * even / d)
    enc = torch.zeros(block, d, dtype=torch.float32)
    enc[:, 0::2] = torch.sin(pos * freq)
    if d > 1:
        enc[:, 1::2] = torch.cos(pos * freq[: enc[:, 1::2].shape[1]])
    return enc


@dataclass(frozen=True)
class Config:
    vocab_size: int
    block_size: int
    n_layer: int
    n_head: int
    n_embd: int
    max_code: int


class Attention(nn.Module):
    def __init__(self, c: Config):
        super().__init__()
        self.qkv = RatchetLinearFP32(c.n_embd, 3 * c.n_embd, max_code=c.max_code)
        self.projection = RatchetLinearFP32(c.n_embd, c.n_embd, max_code=c.max_code)
        self.n_head, self.head = c.n_head, c.n_embd // c.n_head

    def forward(self, x: Tensor) -> Tensor:
        b, t, ch = x.shape
        q, k, v = self.qkv(x).chunk(3, dim=-1)
        h = lambda z: z.view(b, t, self.n_head, self.head).transpose(1, 2)  # noqa: E731
        y = F.scaled_dot_product_attention(h(q), h(k), h(v), is_causal=True)
        return self.projection(y.transpose(1, 2).contiguous().view(b, t, ch))


class MLP(nn.Module):
    def __init__(self, c: Config):
        super().__init__()
        self.expand = RatchetLinearFP32(c.n_embd, 4 * c.n_embd, max_code=c.max_code)
        self.contract = RatchetLinearFP32(4 * c.n_embd, c.n_embd, max_code=c.max_code)

    def forward(self, x: Tensor) -> Tensor:
        return self.contract(F.gelu(self.expand(x)))


class Block(nn.Module):
    def __init__(self, c: Config):
        super().__init__()
        self.attention_norm = nn.RMSNorm(c.n_embd)
        self.attention = Attention(c)
        self.feed_forward_norm = nn.RMSNorm(c.n_embd)
        self.feed_forward = MLP(c)

    def forward(self, x: Tensor) -> Tensor:
        x = x + self.attention(self.attention_norm(x))
        return x + self.feed_forward(self.feed_forward_norm(x))


class RatchetGPTFP32(nn.Module):
    def __init__(self, c: Config):
        super().__init__()
        self.config = c
        self.token_embedding = nn.Embedding(c.vocab_size, c.n_embd)
        self.register_buffer("position_encoding", _positions(c.block_size, c.n_embd))
        self.blocks = nn.ModuleList(Block(c) for _ in range(c.n_layer))
        self.final_norm = nn.RMSNorm(c.n_embd)
        self.lm_head = RatchetLinearFP32(c.n_embd, c.vocab_size, max_code=c.max_code)

    def forward(self, tokens: Tensor, targets: Tensor | None = None):
        x = self.token_embedding(tokens) + self.position_encoding[: tokens.shape[1]]
        for blk in self.blocks:
            x = blk(x)
        logits = self.lm_head(self.final_norm(x))
        loss = None if targets is None else F.cross_entropy(logits.flatten(0, 1), targets.flatten())
        return logits, loss

    def ratchet_layers(self) -> list[RatchetLinearFP32]:
        return [m for m in self.modules() if isinstance(m, RatchetLinearFP32)]


def build_seeded(c: Config, seed: int) -> RatchetGPTFP32:
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        return RatchetGPTFP32(c)


def train_step(model: RatchetGPTFP32, optimizer, tokens: Tensor) -> float:
    """One reference train step: forward, backward (ratchet updates fused), AdamW on support
    parameters (the reference train.py loop, without autocast)."""
    optimizer.zero_grad(set_to_none=True)
    _, loss = model(tokens[:, :-1], tokens[:, 1:])
    loss.backward()
    optimizer.step()
    return float(loss.detach())
