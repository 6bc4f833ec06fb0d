"""Schedule builder and instruction encoding vs the reference's own output.

The golden fixture holds the instruction words the reference scheduler
(megakernels/demos/latency/scheduler.py) produced for the tiny model at three
positions; ours must be word-for-word identical.
"""

import numpy as np
import pytest
import torch

import cases
from megakernels.demos.latency.instructions import (
    AttentionReduction, LayerNormDoubleMatVecSiLU, PartialAttention,
)
from megakernels.demos.latency.scheduler import LatencyScheduleBuilder, pick_num_attention_partitions
from megakernels.scheduler import (
    INTS_PER_INSTRUCTION, TIMING_SLOTS, assign_to_sms, tensorize_instructions,
)


@pytest.fixture(scope="module")
def tiny():
    return cases.tiny_model()


@pytest.fixture(scope="module")
def golden(golden_dir):
    return np.load(golden_dir / "llama_tiny_step.npz")


def words(instrs):
    out = []
    for ins in instrs:
        w = ins.serialize()
        out.extend(w + [0] * (32 - len(w)))
    return np.array(out, dtype=np.int32)


@pytest.mark.parametrize("pos", cases.TINY_POSITIONS)
def test_instruction_stream_matches_reference(tiny, golden, pos):
    sched = LatencyScheduleBuilder.build(tiny, seq_len=pos)
    np.testing.assert_array_equal(words(sched.get_linear_instructions()), golden[f"p{pos}_words"])
    assert int(sched.globs.skip_attn_reduction) == int(golden[f"p{pos}_skip_attn_reduction"][0])


def test_serialize_layout():
    assert PartialAttention(3, 2, 9, 4).serialize() == [2, 3, 2, 9, 4]
    assert AttentionReduction(1, 8, 3, True, [0, 1, 2], None).serialize() == [3, 1, 8, 3, 1, 3, 0, 1, 2, 0]
    assert LayerNormDoubleMatVecSiLU(0, [5, 153]).serialize() == [5, 0, 2, 5, 153]


def test_partition_count():
    assert pick_num_attention_partitions(1, 0, 8, "cpu") == 1
    assert pick_num_attention_partitions(2049, 0, 8, "cpu") == 9
    assert pick_num_attention_partitions(16385, 0, 8, "cpu") == 18


@pytest.mark.parametrize("mode", ["rr", "zz", "wave", "dag"])
def test_assign_and_tensorize(tiny, mode):
    sched = LatencyScheduleBuilder.build(tiny, seq_len=300)
    queues = assign_to_sms(mode, schedule=sched)
    n = sum(len(q) for q in queues)
    assert n == len(sched.get_linear_instructions())
    tensorize_instructions(sched.globs, queues)
    ins = sched.globs.instructions
    assert ins.dtype == torch.int32 and ins.shape[0] == 148 and ins.shape[2] == INTS_PER_INSTRUCTION
    assert sched.globs.timings.shape == (148, ins.shape[1], TIMING_SLOTS)
    # every non-NoOp word row is one of the schedule's instructions
    assert int((ins[:, :, 0] != 0).sum()) == n
