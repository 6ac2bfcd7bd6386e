"""CPU: the oracle (oracle/ratchet_oracle.c) against the reference's golden vectors.

The fixtures were produced by the reference itself (tests/golden/make_golden.py).  Integer and
byte results must match exactly; where the reference's torch reduction order differs from the
canonical order shared by the oracle and the CUDA kernels, the number of differing weights is
asserted to stay at (or very near) zero and the normalised values to agree to a few ulps.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import load_golden


# ---------------------------------------------------------------- Philox / stochastic rounding
def test_philox_known_answers():
    # Random123 known-answer vectors for philox4x32-10.
    assert O.philox4x32_10([0, 0, 0, 0], [0, 0]).tolist() == [
        0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert O.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2).tolist() == [
        0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert O.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                           [0xA4093822, 0x299F31D0]).tolist() == [
        0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_sr_uniform_is_in_unit_interval_and_keyed():
    vals = [O.sr_uniform(7, 0, 0, i) for i in range(64)]
    assert all(0.0 <= v < 1.0 for v in vals)
    assert vals != [O.sr_uniform(7, 1, 0, i) for i in range(64)]   # step changes the stream
    assert vals != [O.sr_uniform(7, 0, 3, i) for i in range(64)]   # layer changes the stream
    assert vals != [O.sr_uniform(8, 0, 0, i) for i in range(64)]   # seed changes the stream


def test_stochastic_rounding_is_unbiased_over_a_million_draws():
    # 10^6 draws: one row of 10^6 copies of the same value => the mean of q*scale must match it.
    rng = np.random.default_rng(0)
    for value in (0.3, -1.7, 2.5, 0.01):
        x = np.full((1, 1_000_000), value, np.float32)
        x[0, 0] = 4.0  # fixes the row scale at 4/127
        q, s = O.quantize_rows(x, stochastic=True, seed=int(rng.integers(1 << 40)), step=3, layer=5)
        mean = (q[0, 1:].astype(np.float64) * s[0]).mean()
        # std of one draw <= scale/2 -> 5 sigma over 1e6 draws = 0.0025 scale
        assert abs(mean - value) < 0.0025 * s[0], (value, mean)


# ---------------------------------------------------------------- row quantisation
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("shape", ["67x35", "128x256", "1x513", "255x1", "300x1", "1x255"])
def test_quantize_rows_matches_reference_bit_exact(dtype, shape):
    g = load_golden("quant_rows.npz")
    key = f"{dtype}_{shape}"
    q, s = O.quantize_rows(g[f"{key}_x"])
    np.testing.assert_array_equal(q, g[f"{key}_q"])
    np.testing.assert_array_equal(s, g[f"{key}_s"])
    qc, sc = O.quantize_rows(g[f"{key}_x"], g[f"{key}_cs"])
    np.testing.assert_array_equal(qc, g[f"{key}_qc"])
    np.testing.assert_array_equal(sc, g[f"{key}_sc"])


def test_quantize_zero_rows_stay_finite():
    g = load_golden("quant_rows.npz")
    q, s = O.quantize_rows(np.zeros((3, 5), np.float32))
    np.testing.assert_array_equal(q, g["zeros_q"])
    np.testing.assert_array_equal(s, g["zeros_s"])
    assert np.all(s > 0)


# ---------------------------------------------------------------- scaled int8 GEMM
@pytest.mark.parametrize("case", ["ragged", "aligned", "wide"])
def test_scaled_int8_mm_matches_reference_bit_exact(case):
    g = load_golden("scaled_mm.npz")
    out = O.scaled_int8_mm(g[f"{case}_lhs"], g[f"{case}_rhs"], g[f"{case}_ls"], g[f"{case}_rs"])
    np.testing.assert_array_equal(out, g[f"{case}_out"])


# ---------------------------------------------------------------- nibble packing
def test_pack_unpack_round_trip():
    for max_code in range(1, 8):
        code, pressure = np.meshgrid(np.arange(-max_code, max_code + 1), np.arange(-7, 8),
                                     indexing="ij")
        packed = O.pack_code_pressure(code, pressure, max_code)
        c2, p2 = O.unpack_code_pressure(packed, max_code)
        np.testing.assert_array_equal(c2, code)
        np.testing.assert_array_equal(p2, pressure)


# ---------------------------------------------------------------- ratchet update
def test_bucket_pressure_known_answers():
    # tests/test_ratchet.py:17-22 of the reference
    z = np.array([[-1.5, -1.49, -0.5, -0.49, 0.0, 0.49, 0.5, 1.49, 1.5]], np.float32)
    packed = O.pack_code_pressure(np.zeros_like(z, np.int8), np.zeros_like(z, np.int8), 2)
    out = O.ratchet_update(z, packed, max_code=2, threshold=8, normalize=False)
    _, pressure = O.unpack_code_pressure(out["packed"], 2)
    assert pressure.tolist() == [[2, 1, 1, 0, 0, 0, -1, -1, -2]]


def test_click_with_residual_pressure_and_blocked_move():
    # tests/test_ratchet.py:54-78: from_reference([[1,1]], max_code=2, T=2) -> codes [2, 2]
    packed = O.pack_code_pressure(np.array([[2, 2]]), np.array([[0, 0]]), 2)
    out = O.ratchet_update(np.array([[1.5, 0.5]], np.float32), packed, max_code=2, threshold=2,
                           normalize=False)
    code, pressure = O.unpack_code_pressure(out["packed"], 2)
    assert code.tolist() == [[1, 2]] and pressure.tolist() == [[0, -1]]
    assert out["counts"].tolist() == [0, 1, 0, 0]
    packed = O.pack_code_pressure(np.array([[2]]), np.array([[0]]), 2)
    out = O.ratchet_update(np.array([[-2.0]], np.float32), packed, max_code=2, threshold=2,
                           normalize=False)
    code, pressure = O.unpack_code_pressure(out["packed"], 2)
    assert code.item() == 2 and pressure.item() == 0
    assert out["counts"].tolist() == [0, 0, 1, 0]


@pytest.mark.parametrize("max_code, sums, total", [(2, (15, -32), 59), (3, (14, -32), 62),
                                                   (4, (9, -32), 65)])
def test_update_trajectory_matches_reference_golden(max_code, sums, total):
    g = load_golden("update_golden.npz")
    packed = g[f"mc{max_code}_packed0"]
    moves = 0
    for step in range(60):
        out = O.ratchet_update(g[f"mc{max_code}_grads"][step], packed, max_code=max_code,
                               normalize=False)
        packed = out["packed"]
        np.testing.assert_array_equal(packed, g[f"mc{max_code}_packs"][step])
        np.testing.assert_array_equal(out["counts"], g[f"mc{max_code}_moves"][step])
        moves += int(out["counts"][:2].sum())
    code, pressure = O.unpack_code_pressure(packed, max_code)
    assert (int(code.sum()), int(pressure.sum())) == sums == tuple(g[f"mc{max_code}_sums"])
    assert moves == total


def _random_case(g, idx):
    rows, cols, max_code, thr = (int(v) for v in g[f"c{idx}_meta"])
    low, high, beta = (float(v) for v in g[f"c{idx}_fmeta"])
    return rows, cols, max_code, thr, low, high, beta


@pytest.mark.parametrize("idx", range(7))
def test_normalised_update_matches_reference(idx):
    g = load_golden("update_random.npz")
    rows, cols, max_code, thr, low, high, beta = _random_case(g, idx)
    ema0 = g.get(f"c{idx}_ema0")
    out = O.ratchet_update(g[f"c{idx}_grad"], g[f"c{idx}_packed0"], max_code=max_code,
                           threshold=thr, bucket_low=low, bucket_high=high, rms_ema=ema0,
                           beta=beta)
    # Applying the reference's own normalised values must reproduce its packed state exactly.
    exact = O.ratchet_update(g[f"c{idx}_normalized"], g[f"c{idx}_packed0"], max_code=max_code,
                             threshold=thr, bucket_low=low, bucket_high=high, normalize=False)
    np.testing.assert_array_equal(exact["packed"], g[f"c{idx}_packed1"])
    np.testing.assert_array_equal(exact["counts"], g[f"c{idx}_counts"])
    # With the canonical reduction order the row mean-square may differ from torch's by an ulp;
    # the packed state must still agree on (essentially) every weight.
    mismatched = int((out["packed"] != g[f"c{idx}_packed1"]).sum())
    assert mismatched <= max(1, rows * cols // 100_000), mismatched
    if beta > 0:
        np.testing.assert_allclose(out["rms_ema"], g[f"c{idx}_ema1"], rtol=2e-6, atol=0)


def test_config1_trajectory_counts_match_reference():
    """The single-layer case (fp32 layer, 10 fused steps): the oracle's update fed with the fp32
    grad_weight of each step reproduces the reference's packed trajectory."""
    g = load_golden("config1.npz")
    x, grad_out, scale = g["x"], g["grad_out"], g["scale"]
    packed = O.pack_code_pressure(g["code0"], np.zeros_like(g["code0"]), 2)
    mism_total = 0
    for step in range(10):
        # grad_weight = grad_out^T @ x in fp32 (ratchet.py:154-157); order-free double sum
        gw = (grad_out.T.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)
        out = O.ratchet_update(gw, packed, max_code=2)
        packed = out["packed"]
        mism = int((packed != g["packs"][step]).sum())
        mism_total += mism
        packed = g["packs"][step].copy()  # continue from the reference state
    assert mism_total <= 10, mism_total
    code, pressure = O.unpack_code_pressure(g["packs"][-1], 2)
    assert (int(code.sum()), int(pressure.sum()), int(g["moves"][:, :2].sum())) == tuple(g["sums"])


def test_leak_moves_pressure_toward_zero():
    packed = O.pack_code_pressure(np.array([[1, -2, 0]]), np.array([[5, -2, 0]]), 2)
    out = O.ratchet_leak(packed)
    code, pressure = O.unpack_code_pressure(out, 2)
    assert code.tolist() == [[1, -2, 0]] and pressure.tolist() == [[4, -1, 0]]


def test_nonfinite_rows_are_skipped():
    grad = np.ones((3, 8), np.float32)
    grad[1, 3] = np.nan
    packed = O.pack_code_pressure(np.zeros((3, 8)), np.zeros((3, 8)), 2)
    out = O.ratchet_update(grad, packed, max_code=2)
    assert out["skipped_rows"] == 1
    np.testing.assert_array_equal(out["packed"][1], packed[1])


# ---------------------------------------------------------------- dequant / bf16
def test_bf16_round_matches_torch():
    import torch

    x = (np.random.default_rng(1).standard_normal(10000) * 100).astype(np.float32)
    np.testing.assert_array_equal(O.bf16_round(x), torch.from_numpy(x).bfloat16().float().numpy())


def test_dequant_matches_torch_bf16_product():
    import torch

    rng = np.random.default_rng(2)
    q = rng.integers(-127, 128, (7, 33)).astype(np.int8)
    s = (rng.random(7) * 0.1 + 1e-3).astype(np.float32)
    ref = (torch.from_numpy(q).to(torch.bfloat16) * torch.from_numpy(s)[:, None].to(torch.bfloat16))
    np.testing.assert_array_equal(O.dequant_rows(q, s), ref.float().numpy())


# ---------------------------------------------------------------- model-level fp32 restatement
def test_fp32_model_step_matches_reference_tiny_model():
    """oracle/model_fp32.py (CPU baseline) reproduces the reference RatchetGPT fp32 step:
    identical seeded state, logits, loss and packed states after one fused-update step."""
    import torch

    from oracle.model_fp32 import Config, build_seeded

    g = load_golden("model_tiny.npz")
    model = build_seeded(Config(vocab_size=11, block_size=8, n_layer=2, n_head=2, n_embd=16,
                                max_code=3), seed=5)
    state = model.state_dict()
    for key, value in state.items():
        np.testing.assert_array_equal(value.numpy(), g[f"state0::{key}"], err_msg=key)
    tokens = torch.from_numpy(g["tokens"])
    logits, loss = model(tokens[:, :8], tokens[:, 1:])
    np.testing.assert_allclose(logits.detach().numpy(), g["logits"], rtol=1e-5, atol=1e-6)
    assert abs(float(loss) - float(g["loss"])) < 1e-5
    loss.backward()
    for key, value in model.state_dict().items():
        if key.endswith("packed"):
            np.testing.assert_array_equal(value.numpy(), g[f"state1::{key}"], err_msg=key)
    moves = sum((layer.moves for layer in model.ratchet_layers()), torch.zeros(4, dtype=torch.int64))
    np.testing.assert_array_equal(moves.numpy(), g["moves"])
    np.testing.assert_allclose(model.token_embedding.weight.grad.numpy(), g["emb_grad"], rtol=1e-5, atol=1e-7)
