"""uint16 token shards on the GPU (reference data.py:238-287).

The reference keeps a tokenised corpus as `<name>.uint16` (little-endian uint16 token ids) plus a
JSON metadata file, loads it into a CPU int64 tensor, and cuts each batch with
`batch_from_starts` (inputs = data[s:s+T], targets = data[s+1:s+T+1] for each start s).  Here the
shard stays uint16 in HBM (2 bytes per token: a billion tokens take 2 GB) and one kernel cuts a
batch's windows and widens them to int64 on the device; only the batch's start offsets cross
from the host.  The schedule of starts is the reference's (seeded torch.randint on the CPU).

Metadata checks and messages follow the reference: token_dtype must be "uint16", the tokenizer
JSON's SHA-256 must match `tokenizer_sha256`, the validation split must leave at least two
tokens on each side.  The tokenizer itself is not rebuilt (text handling is outside this
package); its JSON is returned as read.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import torch
from torch import Tensor

from . import _lib


@dataclass
class TokenShard:
    """A token shard split into train / validation ids, resident on `device` as uint16."""

    train_ids: Tensor        # uint16, on device
    validation_ids: Tensor   # uint16, on device
    tokenizer_json: str
    metadata: dict


def load_token_shard(metadata_path: str | Path, *, validation_fraction: float = 0.1,
                     device: torch.device | str = "cuda") -> TokenShard:
    """Reads the shard described by `metadata_path` (reference data.py:238-264) into device
    memory as uint16 (one host read, one copy)."""
    if not 0 < validation_fraction < 1:
        raise ValueError("validation_fraction must be between zero and one")
    metadata_file = Path(metadata_path)
    metadata = json.loads(metadata_file.read_text())
    if metadata.get("token_dtype") != "uint16":
        raise ValueError("unsupported token shard dtype")
    tokenizer_json = metadata["tokenizer_json"]
    actual_hash = hashlib.sha256(tokenizer_json.encode("utf-8")).hexdigest()
    if actual_hash != metadata["tokenizer_sha256"]:
        raise ValueError("tokenizer hash mismatch")
    tokens_file = metadata_file.with_name(metadata["tokens_file"])
    count = int(metadata["actual_tokens"])
    raw = torch.from_file(str(tokens_file), dtype=torch.uint16, size=count)
    validation_length = int(count * validation_fraction)
    if validation_length < 2 or count - validation_length < 2:
        raise ValueError("token shard is too short for train and validation splits")
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("load_token_shard requires CUDA; the shard lives in device memory")
    ids = raw.pin_memory().to(device, non_blocking=True)
    return TokenShard(train_ids=ids[:-validation_length], validation_ids=ids[-validation_length:],
                      tokenizer_json=tokenizer_json, metadata=metadata)


def make_batch_schedule(*, data_length: int, steps: int, batch_size: int, block_size: int,
                        seed: int) -> Tensor:
    """[steps, batch] window starts on the CPU, the reference's seeded schedule
    (data.py:267-276)."""
    if min(data_length, steps, batch_size, block_size) <= 0:
        raise ValueError("schedule dimensions must be positive")
    high = data_length - block_size
    if high <= 0:
        raise ValueError("data_length must exceed block_size")
    generator = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(0, high, (steps, batch_size), generator=generator)


def batch_from_starts(data: Tensor, starts: Tensor, *, block_size: int) -> tuple[Tensor, Tensor]:
    """(inputs, targets) int64 [batch, block] from a device-resident uint16 shard
    (reference data.py:279-287): one kernel gathers and widens the windows."""
    if data.ndim != 1 or starts.ndim != 1:
        raise ValueError("data and starts must be one-dimensional")
    if data.dtype != torch.uint16 or not data.is_cuda:
        raise TypeError("batch_from_starts takes a CUDA uint16 token shard")
    if starts.numel() and not starts.is_cuda:
        # the host-side range check of the reference, on the host copy of the starts
        if int(starts.max()) + block_size >= data.numel() or int(starts.min()) < 0:
            raise ValueError("batch start exceeds next-token data range")
    starts_dev = starts.to(device=data.device, dtype=torch.int64, non_blocking=True).contiguous()
    batch = starts.numel()
    inputs = torch.empty((batch, block_size), device=data.device, dtype=torch.int64)
    targets = torch.empty_like(inputs)
    if batch == 0:
        return inputs, targets
    _lib.check(_lib.lib().rt_token_windows(
        data.data_ptr(), data.numel(), starts_dev.data_ptr(), batch, block_size,
        inputs.data_ptr(), targets.data_ptr(), _lib.stream_of(data)))
    return inputs, targets
