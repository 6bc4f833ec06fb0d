"""Helpers shared by the schedule builders.

Counterparts of `megakernels/utils.py` in epic-kernel: `assert_div` (:17-19),
`compute_shard_bounds` (:22-37), `trepr` (:103-107) and `get_sm_count`
(:133-135). The safetensors loader and the free-GPU picker of that file are not
part of the decode path (this build runs on synthetic random-init weights).
"""

import os

import torch
from torch import Tensor

# B200 has 148 SMs (2 dies x 74). Used when no CUDA device can be queried, so
# schedules built on a CPU-only host have the same shape as on the GPU.
B200_NUM_SMS = 148


def assert_div(a: int, b: int) -> int:
    assert a % b == 0, f"{a} is not divisible by {b}"
    return a // b


def compute_shard_bounds(tensor_shape, dim: int, num_shards: int, shard_index: int):
    """Slice of `dim` owned by `shard_index` when split as evenly as possible;
    the first `size % num_shards` shards get one extra element."""
    size = tensor_shape[dim]
    base, extra = divmod(size, num_shards)
    start = shard_index * base + min(shard_index, extra)
    stop = start + base + (1 if shard_index < extra else 0)
    return slice(start, stop)


def trepr(t: Tensor) -> str:
    return f"shape={t.shape}, sum={t.sum()}, vals={t}"


def get_sm_count(device) -> int:
    """Number of SMs of `device`.

    `EK_SM_COUNT` overrides it. A CUDA device is queried; anything else (a CPU
    host building schedules for a B200) gets 148.
    """
    override = os.environ.get("EK_SM_COUNT")
    if override:
        return int(override)
    dev = torch.device(device)
    if dev.type == "cuda" and torch.cuda.is_available():
        return torch.cuda.get_device_properties(dev).multi_processor_count
    return B200_NUM_SMS
