"""CPU: the C-ABI library loads and exports every symbol include/*.h declares; host-side API
behaviour of the package (construction, buffers, audits, seeded initialisation parity with the
reference, error messages) — no compute calls."""

from __future__ import annotations

import re
import subprocess

import numpy as np
import pytest
import torch
from torch import nn

from tests.conftest import ROOT, load_golden


def _declared_symbols() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"^\s*(?:int|int64_t|const char \*)\s*(rt_[a-z0-9_]+)\s*\(", text, re.M))
    return names


def test_library_exports_every_declared_symbol():
    from local_ai_training_b200 import _build, _lib

    handle = _lib.lib()
    declared = _declared_symbols()
    assert len(declared) >= 18
    for name in declared:
        assert hasattr(handle, name), name
    assert declared == set(_lib.exported_symbols())
    out = subprocess.run(["nm", "-D", "--defined-only", str(_build.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (rt_[a-z0-9_]+)", out))
    assert declared <= exported


def test_library_is_built_for_sm100a_only():
    from local_ai_training_b200 import _build

    assert _build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_status_codes_map_to_reference_exceptions():
    from local_ai_training_b200 import _lib

    # a shape error straight from the library (no GPU work is launched for negative shapes)
    with pytest.raises(ValueError, match="negative shape"):
        _lib.check(_lib.lib().rt_scaled_int8_mm(None, 0, 0, None, 0, 0, None, None, None, 1, 0,
                                                -1, 1, 1, 0, None, 0, None))
    with pytest.raises(TypeError, match="bfloat16 or float32"):
        _lib.check(_lib.lib().rt_scaled_int8_mm(None, 0, 0, None, 0, 0, None, None, None, 7, 0,
                                                1, 1, 1, 0, None, 0, None))
    with pytest.raises(ValueError, match="max_code"):
        _lib.check(_lib.lib().rt_ratchet_update(1, 0, 0, 1, 1, 1, 1, 1, None, 1, 1, None, 0.0, 9,
                                                8, 0.5, 1.5, 1e-8, None, None, None, None, None))


def test_cpu_operands_are_rejected_like_the_reference():
    from local_ai_training_b200 import quantize_columns, quantize_rows, quantize_rows_colscaled, scaled_int8_mm

    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_rows(torch.ones(2, 3))
    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_columns(torch.ones(2, 3))
    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_rows_colscaled(torch.ones(2, 3), torch.ones(3))
    with pytest.raises(RuntimeError, match="requires CUDA"):
        scaled_int8_mm(torch.ones(2, 3, dtype=torch.int8), torch.ones(3, 4, dtype=torch.int8),
                       torch.ones(2), torch.ones(4))


def test_layer_compute_requires_cuda_no_cpu_fallback():
    from local_ai_training_b200 import DiscreteRatchetLinear

    for mode in ("fp32", "bf16", "int8"):
        layer = DiscreteRatchetLinear(8, 4, max_code=2, matmul_mode=mode, fuse_backward_update=True)
        with pytest.raises(RuntimeError, match="CUDA"):
            layer(torch.randn(2, 8))
    layer = DiscreteRatchetLinear(8, 4, max_code=2)
    with pytest.raises(RuntimeError, match="CUDA"):
        layer.apply_normalized_gradient(torch.randn(4, 8))


@pytest.mark.parametrize("max_code", [1, 2, 3, 4, 5, 6, 7])
def test_construction_matches_reference_rules(max_code):
    from local_ai_training_b200 import DiscreteRatchetLinear

    layer = DiscreteRatchetLinear(8, 4, max_code=max_code)
    assert layer.code.abs().max().item() <= max_code
    assert layer.code.dtype == torch.int8 and layer.pressure.dtype == torch.int8
    with pytest.raises(ValueError):
        DiscreteRatchetLinear(8, 4, max_code=8)
    with pytest.raises(ValueError):
        DiscreteRatchetLinear(8, 4, max_code=2, pressure_threshold=128)
    with pytest.raises(ValueError):
        DiscreteRatchetLinear(8, 4, max_code=2, bucket_low=1.0, bucket_high=0.5)


def test_buffers_parameters_and_audit():
    from local_ai_training_b200 import (DiscreteRatchetLinear, audit_no_master_weights,
                                        compare_persistent_footprint)

    for mode in ("fp32", "bf16", "int8"):
        layer = DiscreteRatchetLinear(7, 5, max_code=2, matmul_mode=mode)
        assert dict(layer.named_parameters()) == {}
        assert set(dict(layer.named_buffers())) == {"packed", "_scale"}
    model = nn.Sequential(DiscreteRatchetLinear(256, 128, max_code=2),
                          DiscreteRatchetLinear(128, 64, max_code=3))
    audit = audit_no_master_weights(model)
    assert audit.ratchet_state_bytes == audit.ratchet_weights + (128 + 64) * 4
    assert compare_persistent_footprint(model).reduction_ratio > 10
    bad = nn.Sequential(DiscreteRatchetLinear(3, 2, max_code=2))
    bad[0].register_parameter("master_weight", nn.Parameter(torch.zeros(2, 3)))
    with pytest.raises(RuntimeError, match="master_weight"):
        audit_no_master_weights(bad, raise_on_violation=True)
    ts = DiscreteRatchetLinear(4, 3, max_code=2, trainable_scale=True)
    assert set(dict(ts.named_parameters())) == {"log_scale"}


def test_seeded_model_matches_reference_initialisation():
    """Same module tree, names and RNG consumption as the reference: the seeded tiny model's
    state_dict equals the one the reference built (tests/golden/model_tiny.npz)."""
    from local_ai_training_b200 import ModelConfig, build_seeded_model

    g = load_golden("model_tiny.npz")
    config = ModelConfig(vocab_size=11, block_size=8, n_layer=2, n_head=2, n_embd=16, dropout=0.0)
    model = build_seeded_model(config, max_code=3, seed=5)
    state = model.state_dict()
    ref_keys = {k.split("::", 1)[1] for k in g if k.startswith("state0::")}
    assert set(state) == ref_keys
    for key, value in state.items():
        np.testing.assert_array_equal(value.numpy(), g[f"state0::{key}"], err_msg=key)
    assert len(model.ratchet_layers()) == 2 * 4 + 1


def test_pack_unpack_and_bucket_helpers():
    from local_ai_training_b200 import bucket_pressure, pack_code_pressure, unpack_code_pressure

    z = torch.tensor([-1.5, -1.49, -0.5, -0.49, 0.0, 0.49, 0.5, 1.49, 1.5])
    assert bucket_pressure(z, low=0.5, high=1.5).tolist() == [2, 1, 1, 0, 0, 0, -1, -1, -2]
    for max_code in (2, 3, 4):
        codes = torch.arange(-max_code, max_code + 1, dtype=torch.int8)
        pressures = torch.arange(-7, 8, dtype=torch.int8)
        cg, pg = torch.meshgrid(codes, pressures, indexing="ij")
        c2, p2 = unpack_code_pressure(pack_code_pressure(cg, pg, max_code), max_code)
        assert torch.equal(c2, cg) and torch.equal(p2, pg)


def test_qkv_heads_fn_without_plan_matches_chunk_views():
    """QKVHeadsFn (no quantisation plan): the views `.chunk(3)` + view + transpose give forward,
    and the concatenated gradient backward."""
    from local_ai_training_b200.int8_fused import QKVHeadsFn

    torch.manual_seed(1)
    qkv = torch.randn(2, 16, 3 * 32, requires_grad=True)
    q, k, v = QKVHeadsFn.apply(qkv, 4, None)
    q2, k2, v2 = (t.view(2, 16, 4, 8).transpose(1, 2) for t in qkv.chunk(3, dim=-1))
    for a, b in zip((q, k, v), (q2, k2, v2)):
        assert torch.equal(a, b) and a.stride() == b.stride()
    w = [torch.randn_like(t) for t in (q, k, v)]
    g1, = torch.autograd.grad(sum((a * c).sum() for a, c in zip((q, k, v), w)), qkv)
    g2, = torch.autograd.grad(sum((a * c).sum() for a, c in zip((q2, k2, v2), w)), qkv)
    assert torch.equal(g1, g2)


def test_prequantized_gradient_is_taken_once_and_only_for_its_tensor():
    from local_ai_training_b200.ratchet import (DiscreteRatchetLinear, GradientQuantPlan,
                                                _take_prequantized)

    layer = DiscreteRatchetLinear(16, 8, max_code=2, matmul_mode="int8", int8_backward=True)
    plan = GradientQuantPlan(layer, round_if_fp32=True)
    g = torch.zeros(4, 8)
    q, s, gb = torch.zeros(4, 8, dtype=torch.int8), torch.ones(4), g.to(torch.bfloat16)
    plan.deliver(g, q, s, gb, True)
    assert _take_prequantized(layer._capture_weight_gradient, g.view(4, 8), False) is None
    assert layer._prequant_grad is None  # a mismatch discards it
    plan.deliver(g, q, s, gb, True)
    assert _take_prequantized(layer._capture_weight_gradient, torch.zeros(4, 8), True) is None
    plan.deliver(g, q, s, gb, True)
    got = _take_prequantized(layer._capture_weight_gradient, g.view(4, 8), True)
    assert got is not None and got[0] is q and got[1] is s and got[2] is gb
    assert _take_prequantized(layer._capture_weight_gradient, g.view(4, 8), True) is None
