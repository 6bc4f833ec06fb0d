"""Small shared types of the decode API.

Mirrors `megakernels/model_types.py:20-60` of epic-kernel: the per-call
`BatchState` bundle handed between embedding, layers and LM head, and the
`ExtraModelConfig` flags that are not part of a Hugging Face config.
"""

from dataclasses import dataclass
from typing import Any

import torch
from torch import Tensor

KV_Cache = tuple[Tensor, Tensor]
DeviceType = torch.device | str


@dataclass
class ModelOutput:
    schedule_id: str
    output_tokens: list[int]
    logprobs: list[float]
    microbatch_index: int | None = None


@dataclass
class BatchState:
    """Tensors flowing through one forward call (batch 1 on the decode path)."""

    input_ids: Tensor
    position_ids: Tensor | None = None
    seq_len: int | None = None
    output_ids: Tensor | None = None
    hidden_states: Tensor | None = None
    position_embeddings: tuple[Tensor, Tensor] | None = None

    kv_indices: Tensor | None = None
    kv_indptr: Tensor | None = None
    kv_last_page_lens: Tensor | None = None
    kv_seqlens: Tensor | None = None
    qo_indptr: Tensor | None = None
    prefill_wrapper: Any | None = None
    decode_wrapper: Any | None = None

    def __post_init__(self):
        if self.seq_len is None:
            self.seq_len = self.input_ids.shape[-1]


@dataclass
class ExtraModelConfig:
    """Flags outside the Hugging Face config (same fields as the reference)."""

    tp_size: int = 1
    tp_rank: int = 0
    tp_group: Any | None = None

    torch_compile: bool = False

    rope_scaling: dict | None = None

    # Permute q/k rows so rotary pairs (i, i + D/2) become adjacent (2i, 2i+1).
    interleave_rope: bool = False

    # KV-cache length; defaults to the config's max_position_embeddings.
    max_len_override: int | None = None

    max_batch_size: int = 1
