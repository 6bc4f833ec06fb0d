"""Llama batch-1 decode instructions (opcodes 1-7) and their `Globals`.

Fields, order and opcodes follow `megakernels/demos/latency/instructions.py`
of epic-kernel (:9-200), because their serialized words are the kernel's
instruction format:

| op | class                          | words                                  |
|----|--------------------------------|----------------------------------------|
| 1  | LayerNorm_QKV_MatVecRopeAppend | layer, start_block, end_block          |
| 2  | PartialAttention               | layer, kv_head, num_partials, partial  |
| 3  | AttentionReduction             | layer, head_start, num_partials,       |
|    |                                | is_terminal, len, list..., out_partial |
| 4  | O_ProjResidual                 | layer, start_block, end_block, red_blk |
| 5  | LayerNormDoubleMatVecSiLU      | layer, len, block_idxs...              |
| 6  | DownProjResidual               | layer, start_block, end_block, red_blk |
| 7  | RMS_LM_Head                    | start_block, end_block                 |
"""

from dataclasses import dataclass
from typing import Optional

from torch import Tensor

from megakernels.instructions import BaseGlobals, Instruction


@dataclass
class Globals(BaseGlobals):
    # activation buffers
    post_ln_rope_q: Tensor
    attn_out: Tensor
    attn_lse_intermediates: Tensor
    attn_out_intermediates: Tensor
    silu_out: Tensor
    logits: Tensor

    skip_attn_reduction: bool

    # block size constants
    up_gate_proj_block_size: int
    down_proj_block_size: int
    o_proj_block_size: int
    lm_head_block_size: int
    matvec_reduction_size: int
    qkv_block_size: int
    attn_kv_block_size: int
    attn_reduction_size: int


@dataclass
class LayerNorm_QKV_MatVecRopeAppend(Instruction):
    """RMSNorm + rows [start, end) x 16 of W_qkv + RoPE on q/k + KV append."""

    layer_idx: int
    start_output_block_idx: int
    end_output_block_idx: int

    @classmethod
    def opcode(cls) -> int:
        return 1

    @classmethod
    def prev_opcode(cls) -> int:
        return DownProjResidual.opcode()

    def block_indices(self):
        return list(range(self.start_output_block_idx, self.end_output_block_idx))

    def cost(self, globs: Globals):
        return (
            (self.end_output_block_idx - self.start_output_block_idx)
            * globs.qkv_block_size
            * globs.hidden_size
        )


@dataclass
class PartialAttention(Instruction):
    """Attention of one KV head's query group over one slice of the cache."""

    layer_idx: int
    kv_head_idx: int
    num_partials: int
    partial_idx: int

    @classmethod
    def opcode(cls) -> int:
        return 2

    @classmethod
    def prev_opcode(cls) -> int:
        return LayerNorm_QKV_MatVecRopeAppend.opcode()

    def cost(self, globs: Globals):
        return (globs.pos_id + 1) / self.num_partials * globs.head_dim * 2


@dataclass
class AttentionReduction(Instruction):
    """Log-sum-exp merge of the partial attention outputs of one query group."""

    layer_idx: int
    head_start_idx: int
    # number of partitions the attention was split into
    num_partials: int
    is_terminal: bool
    reduction_list: list[int]
    # slot for a non-terminal merge's output
    output_partial_idx: Optional[int] = None

    @classmethod
    def opcode(cls) -> int:
        return 3

    @classmethod
    def prev_opcode(cls) -> int:
        return PartialAttention.opcode()

    def cost(self, globs: Globals):
        gqa_ratio = globs.num_attention_heads // globs.num_kv_heads
        return gqa_ratio * self.num_partials * globs.head_dim


@dataclass
class MatVecAdd(Instruction):
    layer_idx: int
    start_block_idx: int
    end_block_idx: int
    reduction_block_idx: int


@dataclass
class O_ProjResidual(MatVecAdd):
    @classmethod
    def opcode(cls) -> int:
        return 4

    @classmethod
    def prev_opcode(cls) -> int:
        return AttentionReduction.opcode()

    def cost(self, globs: Globals):
        return (
            (self.end_block_idx - self.start_block_idx)
            * globs.o_proj_block_size
            * globs.hidden_size
        )


@dataclass
class LayerNormDoubleMatVecSiLU(Instruction):
    """RMSNorm + up and gate rows of the listed blocks + SiLU(gate) * up."""

    layer_idx: int
    block_idxs: list[int]

    @classmethod
    def opcode(cls) -> int:
        return 5

    @classmethod
    def prev_opcode(cls) -> int:
        return O_ProjResidual.opcode()

    def cost(self, globs: Globals):
        return len(self.block_idxs) * globs.up_gate_proj_block_size * globs.hidden_size * 2


@dataclass
class DownProjResidual(MatVecAdd):
    @classmethod
    def opcode(cls) -> int:
        return 6

    @classmethod
    def prev_opcode(cls) -> int:
        return LayerNormDoubleMatVecSiLU.opcode()

    def cost(self, globs: Globals):
        return (
            (self.end_block_idx - self.start_block_idx)
            * globs.down_proj_block_size
            * globs.hidden_size
        )


@dataclass
class RMS_LM_Head(Instruction):
    start_output_block_idx: int
    end_output_block_idx: int

    @classmethod
    def opcode(cls) -> int:
        return 7

    @classmethod
    def prev_opcode(cls) -> int:
        return DownProjResidual.opcode()

    def cost(self, globs: Globals):
        return (
            (self.end_output_block_idx - self.start_output_block_idx)
            * globs.lm_head_block_size
            * globs.hidden_size
        )
