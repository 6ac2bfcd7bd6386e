"""Generates the golden fixtures of tests/golden/ by running the REFERENCE implementation.

Run in a container where the reference project is importable (its src/ directory on sys.path or
given with --reference).  The fixtures pin the CPU oracle (oracle/) to the reference's own
outputs; the CUDA kernels are then checked against the oracle.  Everything here is CPU/fp32
(the reference's eager path), seeded, and small.

Fixtures (npz):
  quant_rows.npz       _quantize_rows_reference (int8_matmul.py:225-239), test shapes of
                       tests/test_int8_matmul.py:20-50 and :93-104 (plain and col-scaled)
  scaled_mm.npz        bf16((A.float() @ B.float()) * ls * rs) (tests/test_int8_matmul.py:172-187)
  update_golden.npz    DiscreteRatchetLinear.apply_normalized_gradient trajectory of
                       tests/test_ratchet.py:196-208 (seed 1234, 6x8, 60 steps, max_code 2/3/4)
  update_random.npz    _normalize + _ratchet_update_core (ratchet.py:265-301, 539-556) on random
                       states and gradients, several shapes / max_code / thresholds / EMA
  config1.npz          single-layer case: one 256x256 quinary fused-backward layer, fp32, 10 steps
  model_tiny.npz       RatchetGPT (model.py) fp32 tiny config, one train step
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _bits_bf16(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


def quant_rows(ref) -> None:
    im = ref["int8_matmul"]
    data = {}
    for dtype in (torch.float32, torch.bfloat16):
        for shape in ((67, 35), (128, 256), (1, 513), (255, 1), (300, 1), (1, 255)):
            torch.manual_seed(7)
            values = torch.randn(shape, dtype=dtype) * 3.0
            q, s = im._quantize_rows_reference(values)
            key = f"{'bf16' if dtype == torch.bfloat16 else 'f32'}_{shape[0]}x{shape[1]}"
            data[f"{key}_x"] = values.float().numpy()
            data[f"{key}_q"] = q.numpy()
            data[f"{key}_s"] = s.numpy()
            col_scale = torch.rand(shape[1], dtype=torch.float32) + 0.01
            qc, sc = im._quantize_rows_reference(values, col_scale)
            data[f"{key}_cs"] = col_scale.numpy()
            data[f"{key}_qc"] = qc.numpy()
            data[f"{key}_sc"] = sc.numpy()
    zeros = torch.zeros(3, 5, dtype=torch.bfloat16)
    qz, sz = im._quantize_rows_reference(zeros)
    data["zeros_q"], data["zeros_s"] = qz.numpy(), sz.numpy()
    np.savez_compressed(OUT / "quant_rows.npz", **data)


def scaled_mm(ref) -> None:
    data = {}
    cases = {"ragged": (67, 35, 53, 20, 8), "aligned": (256, 512, 384, 127, 4),
             "wide": (130, 96, 300, 127, 3)}
    for name, (m, k, n, amax, bmax) in cases.items():
        torch.manual_seed(3)
        lhs = torch.randint(-amax, amax + 1, (m, k), dtype=torch.int8)
        rhs = torch.randint(-bmax, bmax + 1, (k, n), dtype=torch.int8)
        ls = torch.rand(m, dtype=torch.float32) + 0.01
        rs = torch.rand(n, dtype=torch.float32) + 0.01
        expected = ((lhs.float() @ rhs.float()) * ls[:, None] * rs[None, :]).to(torch.bfloat16)
        data[f"{name}_lhs"], data[f"{name}_rhs"] = lhs.numpy(), rhs.numpy()
        data[f"{name}_ls"], data[f"{name}_rs"] = ls.numpy(), rs.numpy()
        data[f"{name}_out"] = expected.float().numpy()
    np.savez_compressed(OUT / "scaled_mm.npz", **data)


def update_golden(ref) -> None:
    rt = ref["ratchet"]
    data = {}
    for max_code in (2, 3, 4):
        torch.manual_seed(1234)
        layer = rt.DiscreteRatchetLinear(8, 6, max_code=max_code, pressure_threshold=8)
        data[f"mc{max_code}_packed0"] = layer.packed.numpy().copy()
        grads, packs, moves = [], [], []
        for _ in range(60):
            g = torch.randn(6, 8) * 2.0
            stats = layer.apply_normalized_gradient(g)
            grads.append(g.numpy().copy())
            packs.append(layer.packed.numpy().copy())
            moves.append([stats.positive_moves, stats.negative_moves,
                          stats.blocked_positive_moves, stats.blocked_negative_moves])
        data[f"mc{max_code}_grads"] = np.stack(grads)
        data[f"mc{max_code}_packs"] = np.stack(packs)
        data[f"mc{max_code}_moves"] = np.asarray(moves, np.int64)
        data[f"mc{max_code}_sums"] = np.asarray(
            [int(layer.code.sum()), int(layer.pressure.sum())], np.int64)
    np.savez_compressed(OUT / "update_golden.npz", **data)


def update_random(ref) -> None:
    rt = ref["ratchet"]
    data = {}
    cases = [
        # rows, cols, max_code, threshold, low, high, beta, grad scale
        (5, 7, 2, 8, 0.5, 1.5, 0.0, 1.0),
        (33, 1030, 3, 4, 0.5, 1.5, 0.0, 1e-3),
        (64, 512, 2, 8, 0.5, 1.5, 0.0, 1e-2),
        (16, 4096, 4, 2, 0.7, 1.3, 0.0, 5.0),
        (9, 9000, 1, 1, 0.5, 1.5, 0.0, 1.0),
        (24, 256, 7, 8, 0.5, 1.5, 0.9, 1.0),
        (12, 100, 3, 3, 0.25, 2.0, 0.5, 1e-4),
    ]
    for idx, (rows, cols, max_code, thr, low, high, beta, gscale) in enumerate(cases):
        torch.manual_seed(100 + idx)
        layer = rt.DiscreteRatchetLinear(cols, rows, max_code=max_code, pressure_threshold=thr,
                                         bucket_low=low, bucket_high=high, rms_ema_beta=beta)
        code = torch.randint(-max_code, max_code + 1, (rows, cols), dtype=torch.int8)
        pressure = torch.randint(-7, 8, (rows, cols), dtype=torch.int8)
        layer.packed.copy_(rt.pack_code_pressure(code, pressure, max_code))
        if beta > 0:
            ema0 = torch.rand(rows) * (gscale ** 2)
            ema0[::3] = 0.0
            layer.rms_ema.copy_(ema0)
            data[f"c{idx}_ema0"] = ema0.numpy().copy()
        grads = torch.randn(rows, cols) * gscale
        grads[0, : min(cols, 3)] = 0.0
        if rows > 2:
            grads[2] = 0.0  # an all-zero row (finite normalisation, no moves)
        packed0 = layer.packed.numpy().copy()
        normalized = layer._normalize(grads, 0, rows)
        new, pos, neg, bpos, bneg = rt._ratchet_update_core(
            layer.packed, normalized, max_code, thr, low, high)
        data[f"c{idx}_meta"] = np.asarray([rows, cols, max_code, thr], np.int64)
        data[f"c{idx}_fmeta"] = np.asarray([low, high, beta], np.float64)
        data[f"c{idx}_grad"] = grads.numpy()
        data[f"c{idx}_packed0"] = packed0
        data[f"c{idx}_normalized"] = normalized.numpy()
        data[f"c{idx}_packed1"] = new.numpy()
        data[f"c{idx}_counts"] = np.asarray([int(pos), int(neg), int(bpos), int(bneg)], np.int64)
        if beta > 0:
            data[f"c{idx}_ema1"] = layer.rms_ema.numpy().copy()
    data["ncases"] = np.asarray(len(cases))
    np.savez_compressed(OUT / "update_random.npz", **data)


def config1(ref) -> None:
    """Single-layer case: X[512,256] ~N(0,1); quinary codes uniform {-2..2} [256,256]; scales
    U(0.01,0.05); pressure 0; grad_out [512,256] ~N(0,1e-2); seed 1337; 10 update steps."""
    rt = ref["ratchet"]
    torch.manual_seed(1337)
    x = torch.randn(512, 256)
    code = torch.randint(-2, 3, (256, 256), dtype=torch.int8)
    scale = torch.rand(256) * 0.04 + 0.01
    grad_out = torch.randn(512, 256) * 1e-2
    layer = rt.DiscreteRatchetLinear(256, 256, max_code=2, fuse_backward_update=True)
    layer.packed.copy_(rt.pack_code_pressure(code, torch.zeros_like(code), 2))
    layer._scale.copy_(scale)
    data = {"x": x.numpy(), "code0": code.numpy(), "scale": scale.numpy(),
            "grad_out": grad_out.numpy()}
    packs, moves, outs, gins = [], [], [], []
    layer.train()
    for _ in range(10):
        inp = x.clone().requires_grad_(True)
        out = layer(inp)
        out.backward(grad_out)
        stats = layer.ratchet_update()
        packs.append(layer.packed.numpy().copy())
        moves.append([stats.positive_moves, stats.negative_moves, stats.blocked_positive_moves,
                      stats.blocked_negative_moves])
        outs.append(out.detach().numpy().copy())
        gins.append(inp.grad.numpy().copy())
    data["packs"] = np.stack(packs)
    data["moves"] = np.asarray(moves, np.int64)
    data["out0"], data["gin0"] = outs[0], gins[0]
    data["sums"] = np.asarray([int(layer.code.sum()), int(layer.pressure.sum()),
                               int(np.asarray(moves)[:, :2].sum())], np.int64)
    np.savez_compressed(OUT / "config1.npz", **data)


def model_tiny(ref) -> None:
    md = ref["model"]
    config = md.ModelConfig(vocab_size=11, block_size=8, n_layer=2, n_head=2, n_embd=16,
                            dropout=0.0)
    model = md.build_seeded_model(config, max_code=3, seed=5)
    model.train()
    gen = torch.Generator().manual_seed(21)
    tokens = torch.randint(0, 11, (3, 9), generator=gen)
    data = {"tokens": tokens.numpy()}
    state0 = {k: v.numpy().copy() for k, v in model.state_dict().items()}
    for k, v in state0.items():
        data[f"state0::{k}"] = v
    logits, loss = model(tokens[:, :8], tokens[:, 1:])
    loss.backward()
    stats = model.ratchet_update()
    data["logits"] = logits.detach().numpy()
    data["loss"] = np.asarray(float(loss))
    data["moves"] = np.asarray([stats.positive_moves, stats.negative_moves,
                                stats.blocked_positive_moves, stats.blocked_negative_moves],
                               np.int64)
    for k, v in model.state_dict().items():
        if k.endswith("packed"):
            data[f"state1::{k}"] = v.numpy().copy()
    data["emb_grad"] = model.token_embedding.weight.grad.numpy()
    np.savez_compressed(OUT / "model_tiny.npz", **data)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("RATCHET_REFERENCE_SRC"),
                        help="directory containing the reference package local_ai_training "
                             "(default: $RATCHET_REFERENCE_SRC)")
    args = parser.parse_args()
    if not args.reference:
        parser.error("give --reference or set RATCHET_REFERENCE_SRC")
    sys.path.insert(0, args.reference)
    import importlib

    ref = {name: importlib.import_module(f"local_ai_training.{name}")
           for name in ("int8_matmul", "ratchet", "model")}
    torch.set_num_threads(1)
    quant_rows(ref)
    scaled_mm(ref)
    update_golden(ref)
    update_random(ref)
    config1(ref)
    model_tiny(ref)
    for path in sorted(OUT.glob("*.npz")):
        print(f"{path.name}: {path.stat().st_size} bytes")


if __name__ == "__main__":
    main()
