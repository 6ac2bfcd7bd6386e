"""Checkpoints of ratchet models, in the reference's format, from single-process or
data-parallel training (reference checkpoint.py:23-106).

Format (unchanged, so checkpoints move between the reference and this package both ways):
`<base>.safetensors` holds `model::<state_dict key>` (the `packed` code|pressure bytes, `_scale`
or `log_scale`, `rms_ema`, support parameters and buffers), `optimizer::<parameter>::<state>`
and `rng::cpu`; `<base>.json` holds format_version, step, max_code, vocabulary,
experiment_config (its matmul_mode is checked on load), tokenizer kind / json.

This package adds `ratchet_sr::<layer>::step` entries: the device step counters of the
stochastic-rounding streams, so that a resumed run draws the same roundings as an uninterrupted
one (the reference draws a fresh host seed per call, covered by `rng::cpu`).  The reference's
loader ignores them; checkpoints without them start the counters at zero.

Data parallel: `RatchetDataParallel` keeps `packed` (code and pressure of every row) and
`rms_ema` replicated on every rank after each step, and the support parameters and their AdamW
state identical, so rank 0's state is the whole model: rank 0 writes, every rank reads.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
from safetensors.torch import load_file, save_file
from torch import Tensor, nn

from .ratchet import DiscreteRatchetLinear

FORMAT_VERSION = 1


def _paths(base_path: str | Path) -> tuple[Path, Path, Path]:
    base = Path(base_path)
    if base.suffix in {".safetensors", ".json"}:
        base = base.with_suffix("")
    return base, base.with_suffix(".safetensors"), base.with_suffix(".json")


def _rank_and_world(group) -> tuple[int, int]:
    if group is not None or (dist.is_available() and dist.is_initialized()):
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def _sr_counters(model: nn.Module) -> dict[str, Tensor]:
    out = {}
    for name, module in model.named_modules():
        if isinstance(module, DiscreteRatchetLinear) and module._sr_step_dev is not None:
            out[f"ratchet_sr::{name}::step"] = module._sr_step_dev.detach().cpu().contiguous()
    return out


def save_checkpoint(
    base_path: str | Path,
    *,
    model: nn.Module,
    optimizer: torch.optim.Optimizer,
    step: int,
    max_code: int,
    vocabulary: tuple[str, ...],
    experiment_config: dict[str, Any],
    tokenizer_kind: str = "char",
    tokenizer_json: str | None = None,
    group: dist.ProcessGroup | None = None,
) -> Path:
    """Writes the checkpoint (rank 0 of `group` under torch.distributed; every rank returns
    after the files exist)."""
    base, tensor_path, metadata_path = _paths(base_path)
    rank, world = _rank_and_world(group)
    if rank == 0:
        base.parent.mkdir(parents=True, exist_ok=True)
        tensors: dict[str, Tensor] = {
            f"model::{name}": tensor.detach().cpu().contiguous()
            for name, tensor in model.state_dict().items()
        }
        for parameter_name, parameter in dict(model.named_parameters()).items():
            for state_name, state_value in optimizer.state.get(parameter, {}).items():
                if not isinstance(state_value, Tensor):
                    state_value = torch.tensor(state_value)
                tensors[f"optimizer::{parameter_name}::{state_name}"] = (
                    state_value.detach().cpu().contiguous())
        tensors.update(_sr_counters(model))
        tensors["rng::cpu"] = torch.get_rng_state()
        save_file(tensors, tensor_path)
        metadata: dict[str, Any] = {
            "format_version": FORMAT_VERSION,
            "step": int(step),
            "max_code": int(max_code),
            "vocabulary": list(vocabulary),
            "experiment_config": experiment_config,
            "tokenizer_kind": tokenizer_kind,
        }
        if tokenizer_json is not None:
            metadata["tokenizer_json"] = tokenizer_json
        metadata_path.write_text(json.dumps(metadata, indent=2, sort_keys=True) + "\n")
    if world > 1:
        dist.barrier(group=group)
    return base


def load_checkpoint(
    base_path: str | Path,
    *,
    model: nn.Module,
    optimizer: torch.optim.Optimizer,
    expected_max_code: int,
    expected_vocabulary: tuple[str, ...],
    expected_matmul_mode: str = "fp32",
) -> dict[str, Any]:
    """Validates the metadata (the reference's checks and messages), then loads the model and
    optimizer state onto the model's devices; every rank of a data-parallel job calls it."""
    _, tensor_path, metadata_path = _paths(base_path)
    metadata = json.loads(metadata_path.read_text())
    if metadata.get("format_version") != FORMAT_VERSION:
        raise ValueError("unsupported checkpoint format version")
    if metadata.get("max_code") != expected_max_code:
        raise ValueError("checkpoint code range does not match requested model")
    if metadata.get("tokenizer_kind", "char") == "char":
        if tuple(metadata.get("vocabulary", ())) != expected_vocabulary:
            raise ValueError("checkpoint vocabulary does not match dataset")
    saved_mode = metadata.get("experiment_config", {}).get("matmul_mode", "fp32")
    if saved_mode != expected_matmul_mode:
        raise ValueError("checkpoint matmul_mode does not match requested run")

    tensors = load_file(tensor_path)
    model_state = {key.removeprefix("model::"): value for key, value in tensors.items()
                   if key.startswith("model::")}
    model.load_state_dict(model_state, strict=True)
    named_parameters = dict(model.named_parameters())
    # an optimizer that is neither capturable nor fused keeps its scalar `step` on the host
    host_steps = {id(p) for group in optimizer.param_groups
                  if not (group.get("capturable") or group.get("fused")) for p in group["params"]}
    optimizer.state.clear()
    for key, value in tensors.items():
        if not key.startswith("optimizer::"):
            continue
        _, parameter_name, state_name = key.split("::", 2)
        if parameter_name not in named_parameters:
            raise ValueError(f"checkpoint optimizer parameter is unknown: {parameter_name}")
        parameter = named_parameters[parameter_name]
        on_host = state_name == "step" and value.ndim == 0 and id(parameter) in host_steps
        optimizer.state[parameter][state_name] = value if on_host else value.to(parameter.device)
    modules = dict(model.named_modules())
    for key, value in tensors.items():
        if not key.startswith("ratchet_sr::"):
            continue
        _, name, _ = key.split("::", 2)
        module = modules.get(name)
        if not isinstance(module, DiscreteRatchetLinear):
            raise ValueError(f"checkpoint stochastic-rounding counter is unknown: {name}")
        module._sr_step_dev = value.to(module.packed.device).clone()
    for module in modules.values():
        if isinstance(module, DiscreteRatchetLinear):
            module._code_mirror = None  # rebuilt from the loaded `packed` on next use
    if "rng::cpu" in tensors:
        torch.set_rng_state(tensors["rng::cpu"])
    return metadata
