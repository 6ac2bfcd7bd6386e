"""B200-native (sm_100a) ratchet-linear train step, API-compatible with the reference package
local_ai_training (ratchet.py, int8_matmul.py, int8_fused.py, int8_backward.py, model.py).

The compute lives in libratchet_b200.so (C ABI, include/ratchet_b200.h), loaded through ctypes.
"""

from .int8_matmul import (
    quantize_columns,
    quantize_rows,
    quantize_rows_colscaled,
    scaled_int8_mm,
)
from .model import ModelConfig, RatchetGPT, build_seeded_model
from .ratchet import (
    DiscreteRatchetLinear,
    PersistentFootprint,
    RatchetAuditReport,
    RatchetEmbedding,
    RatchetUpdateStats,
    audit_no_master_weights,
    bucket_pressure,
    compare_persistent_footprint,
    pack_code_pressure,
    unpack_code_pressure,
)

__all__ = [
    "DiscreteRatchetLinear",
    "ModelConfig",
    "PersistentFootprint",
    "RatchetAuditReport",
    "RatchetEmbedding",
    "RatchetGPT",
    "RatchetUpdateStats",
    "audit_no_master_weights",
    "bucket_pressure",
    "build_seeded_model",
    "compare_persistent_footprint",
    "pack_code_pressure",
    "quantize_columns",
    "quantize_rows",
    "quantize_rows_colscaled",
    "scaled_int8_mm",
    "unpack_code_pressure",
]
