"""Instruction base type, word encoding, and the kernel-argument bundle.

Interface of `megakernels/instructions.py` in epic-kernel:
- `BaseGlobals` (:10-69) holds every tensor and constant one decode step reads.
- `Instruction.serialize` (:97-119) turns an instruction into int32 words. Word
  0 is the opcode, then each dataclass field in declaration order. An int or
  bool is one word; a list or tuple is its length followed by its items; None
  is a single 0. A field named `global_idx` is skipped.
- `NoOp` (:122-126) is opcode 0 and pads the per-SM queues.

The encoding must stay word-for-word the same: the megakernel decodes these
words, and instruction tensors built by the reference's scheduler must run
unchanged on this kernel.
"""

from dataclasses import dataclass, fields
from typing import Any

from torch import Tensor

from megakernels.model_types import DeviceType
from megakernels.utils import get_sm_count


@dataclass
class BaseGlobals:
    # model parameters, all layers stacked on a leading layer axis
    qkv_proj_weights: Tensor
    attn_ln_weights: Tensor
    o_proj_weights: Tensor
    mlp_ln_weights: Tensor
    up_proj_weights: Tensor
    gate_proj_weights: Tensor
    down_proj_weights: Tensor
    lm_head_norm_weights: Tensor
    lm_head_weights: Tensor
    k_cache: Tensor
    v_cache: Tensor

    # not stacked per layer
    rope_cos: Tensor
    rope_sin: Tensor

    # model constants
    num_hidden_layers: int
    num_attention_heads: int
    num_kv_heads: int
    head_dim: int
    hidden_size: int
    intermediate_size: int
    vocab_size: int

    attn_scale: float
    rms_norm_eps: float
    device: DeviceType

    hidden_states: Tensor
    barriers: Tensor

    pos_id: int

    def __post_init__(self):
        self.instructions: Tensor | None = None
        self.timings: Tensor | None = None

    def sm_count(self) -> int:
        return get_sm_count(self.device)

    def diff(self, other: "BaseGlobals", skip_kv_cache: bool = False):
        """Print max-abs / mean-relative differences of every activation tensor."""
        out = {}
        for f in fields(self):
            name = f.name
            mine = getattr(self, name)
            if (
                not isinstance(mine, Tensor)
                or "weights" in name
                or name in ("rope_cos", "rope_sin")
                or (skip_kv_cache and "cache" in name)
            ):
                continue
            out[name] = diff_tensors(mine, getattr(other, name), name)
        return out

    def num_total_heads(self) -> int:
        return self.num_attention_heads + self.num_kv_heads * 2


def diff_tensors(a: Tensor, b: Tensor, name: str):
    a = a.float().cpu()
    b = b.float().cpu()
    diff = a - b
    adiff = diff.abs()
    rdiff = 2 * adiff / (a.abs() + b.abs() + 1e-6)
    print(f"{name}: max adiff: {adiff.max()}, mean rdiff: {rdiff.mean()}")
    return diff, adiff, rdiff


@dataclass
class Instruction:
    @classmethod
    def opcode(cls) -> int:
        raise NotImplementedError

    @classmethod
    def prev_opcode(cls) -> int:
        raise NotImplementedError

    @classmethod
    def tags(cls) -> dict[str, Any]:
        return {}

    def serialize(self) -> list[int]:
        words = [self.opcode()]
        for f in fields(self):
            if f.name == "global_idx":
                continue
            value = getattr(self, f.name)
            if value is None:
                words.append(0)
            elif isinstance(value, (list, tuple)):
                words.append(len(value))
                words.extend(int(v) for v in value)
            elif isinstance(value, int):  # bool is an int subclass
                words.append(int(value))
            else:
                raise ValueError(f"Unsupported field type: {value!r}")
        return words


@dataclass
class NoOp(Instruction):
    @classmethod
    def opcode(cls) -> int:
        return 0

    def cost(self, globs) -> float:
        return 0


@dataclass
class PrintInfo:
    layer_filter: list[int] | None = None
    name_filter: list[str] | None = None
    state_filter: list[str] | None = None


@dataclass
class PrintState(Instruction):
    """Host-side debugging aid of the Python interpreter; never sent to the GPU."""

    layer_idx: int
    name: str
    print_info: PrintInfo
