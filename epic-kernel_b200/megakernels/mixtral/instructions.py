"""Mixtral batch-1 decode instructions (opcodes 1-8) and `MixtralGlobals`.

Field order and opcodes follow `megakernels/mixtral/instructions.py` of
epic-kernel (:22-297); the serialized words are the kernel's input format:

| op | class                   | words                                   |
|----|-------------------------|-----------------------------------------|
| 1  | Mixtral_QKV             | layer, start_block, end_block           |
| 2  | Mixtral_PartialAttn     | layer, kv_head, num_partials, partial   |
| 3  | Mixtral_AttnReduction   | layer, head_start, num_partials,        |
|    |                         | is_terminal, len, list..., out_partial  |
| 4  | Mixtral_OProj           | layer, start_block, end_block, red_blk  |
| 5  | RmsRouterUpgate         | layer, start_block, num_blocks          |
| 6  | ExpertDownProjFused     | layer, start_block, end_block, red_blk  |
| 7  | Mixtral_RMS_LM_Head     | start_block, end_block, red_blk         |
| 8  | SpeculativeExpertPredict| layer                                   |
"""

from dataclasses import dataclass
from typing import Optional

from torch import Tensor

from megakernels.instructions import BaseGlobals, Instruction


@dataclass
class MixtralGlobals(BaseGlobals):
    # attention activations
    post_ln_rope_q: Tensor
    attn_out: Tensor
    attn_lse_intermediates: Tensor
    attn_out_intermediates: Tensor

    # MoE activations
    expert_silu_out: Tensor  # [E, I]
    router_normed_hidden: Tensor  # [H]
    logits: Tensor  # [V]

    # router outputs of the current layer (RmsRouterUpgate -> ExpertDownProjFused)
    selected_expert_indices: Tensor  # [k] int32
    selected_expert_scores: Tensor  # [k] bf16

    # SpeculativeExpertPredict output (used for prefetch only)
    predicted_expert_indices: Tensor  # [k] int32

    # MoE weights
    router_weights: Tensor  # [L, E, H]
    expert_gate_weights: Tensor  # [L, E, I, H]
    expert_up_weights: Tensor  # [L, E, I, H]
    expert_down_weights: Tensor  # [L, E, H, I]
    ffn_ln_weights: Tensor  # [L, H]

    num_experts: int
    num_experts_per_tok: int

    skip_attn_reduction: bool

    expert_proj_block_size: int
    down_proj_block_size: int
    o_proj_block_size: int
    lm_head_block_size: int
    matvec_reduction_size: int
    qkv_block_size: int
    attn_kv_block_size: int
    attn_reduction_size: int

    def __post_init__(self):
        super().__post_init__()

    def num_total_heads(self) -> int:
        return self.num_attention_heads + self.num_kv_heads * 2


@dataclass
class Mixtral_QKV(Instruction):
    layer_idx: int
    start_output_block_idx: int
    end_output_block_idx: int

    @classmethod
    def opcode(cls) -> int:
        return 1

    @classmethod
    def prev_opcode(cls) -> int:
        return ExpertDownProjFused.opcode()

    def block_indices(self):
        return list(range(self.start_output_block_idx, self.end_output_block_idx))

    def cost(self, globs: MixtralGlobals) -> float:
        return (self.end_output_block_idx - self.start_output_block_idx) * globs.qkv_block_size * globs.hidden_size


@dataclass
class Mixtral_PartialAttn(Instruction):
    layer_idx: int
    kv_head_idx: int
    num_partials: int
    partial_idx: int

    @classmethod
    def opcode(cls) -> int:
        return 2

    @classmethod
    def prev_opcode(cls) -> int:
        return Mixtral_QKV.opcode()

    def cost(self, globs: MixtralGlobals) -> float:
        return (globs.pos_id + 1) / self.num_partials * globs.head_dim * 2


@dataclass
class Mixtral_AttnReduction(Instruction):
    layer_idx: int
    head_start_idx: int
    num_partials: int
    is_terminal: bool
    reduction_list: list[int]
    output_partial_idx: Optional[int] = None

    @classmethod
    def opcode(cls) -> int:
        return 3

    @classmethod
    def prev_opcode(cls) -> int:
        return Mixtral_PartialAttn.opcode()

    def cost(self, globs: MixtralGlobals) -> float:
        return globs.num_attention_heads // globs.num_kv_heads * self.num_partials * globs.head_dim


@dataclass
class Mixtral_OProj(Instruction):
    layer_idx: int
    start_block_idx: int
    end_block_idx: int
    reduction_block_idx: int

    @classmethod
    def opcode(cls) -> int:
        return 4

    @classmethod
    def prev_opcode(cls) -> int:
        return Mixtral_AttnReduction.opcode()

    def cost(self, globs: MixtralGlobals) -> float:
        return (self.end_block_idx - self.start_block_idx) * globs.o_proj_block_size * globs.hidden_size


@dataclass
class RmsRouterUpgate(Instruction):
    """RMSNorm + router top-k + gate/up rows of the selected experts + SiLU."""

    layer_idx: int
    start_block_idx: int
    num_blocks: int

    @classmethod
    def opcode(cls) -> int:
        return 5

    @classmethod
    def prev_opcode(cls) -> int:
        return Mixtral_OProj.opcode()

    def block_indices(self) -> list[int]:
        return list(range(self.start_block_idx, self.start_block_idx + self.num_blocks))

    def cost(self, globs: MixtralGlobals) -> float:
        return (globs.num_experts * globs.hidden_size
                + self.num_blocks * globs.expert_proj_block_size * globs.hidden_size * 2 * globs.num_experts_per_tok)


@dataclass
class ExpertDownProjFused(Instruction):
    """Down projection of the selected experts, score-weighted into hidden."""

    layer_idx: int
    start_block_idx: int
    end_block_idx: int
    reduction_block_idx: int

    @classmethod
    def opcode(cls) -> int:
        return 6

    @classmethod
    def prev_opcode(cls) -> int:
        return RmsRouterUpgate.opcode()

    def cost(self, globs: MixtralGlobals) -> float:
        return ((self.end_block_idx - self.start_block_idx) * globs.down_proj_block_size
                * globs.intermediate_size * globs.num_experts_per_tok)


@dataclass
class Mixtral_RMS_LM_Head(Instruction):
    start_output_block_idx: int
    end_output_block_idx: int
    reduction_block_idx: int = 0

    @classmethod
    def opcode(cls) -> int:
        return 7

    @classmethod
    def prev_opcode(cls) -> int:
        return ExpertDownProjFused.opcode()

    def cost(self, globs: MixtralGlobals) -> float:
        return (self.end_output_block_idx - self.start_output_block_idx) * globs.lm_head_block_size * globs.hidden_size


@dataclass
class SpeculativeExpertPredict(Instruction):
    """Top-k experts predicted from the pre-attention residual (prefetch hint)."""

    layer_idx: int

    @classmethod
    def opcode(cls) -> int:
        return 8

    @classmethod
    def prev_opcode(cls) -> int:
        return ExpertDownProjFused.opcode()

    def cost(self, globs: MixtralGlobals) -> float:
        return globs.num_experts * globs.hidden_size
