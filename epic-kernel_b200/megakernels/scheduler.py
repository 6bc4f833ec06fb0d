"""Instruction DAG, SM assignment policies and the instruction tensor.

Same interface and behaviour as `megakernels/scheduler.py` in epic-kernel:
- `DAG_Node`, `Schedule`, `ScheduleBuilder` (:17-92).
- The SM assignment policies `rr`, `zz`, `wave`, `dag` and `pool` (:95-272).
- `tensorize_instructions` (:282-309). It pads every per-SM queue with `NoOp`
  to the longest queue and uploads the queues as an int32 tensor
  `[num_sms, queue_len, 32]`. It also creates the `[num_sms, queue_len, 128]`
  int32 `timings` tensor.

The megakernel walks queue `b` on thread block `b`, in order. A queue may wait
only on instructions that come earlier in the schedule's linear (topological)
order. Every policy here keeps that order within each queue except `wave` and
`dag`. Those two can still only wait on instructions that they placed earlier
in time.
"""

import heapq
from dataclasses import dataclass, field, replace

import torch

from megakernels.instructions import BaseGlobals, Instruction, NoOp

INTS_PER_INSTRUCTION = 32
TIMING_SLOTS = 128


@dataclass(eq=False)
class DAG_Node:
    instruction: Instruction
    dependencies: list["DAG_Node"]

    children: set["DAG_Node"] = field(default_factory=set)
    start_time: float = float("inf")
    end_time: float = float("inf")
    remaining_dependencies: set["DAG_Node"] = field(default_factory=set)
    priority: float = 0

    def earliest_ready_time(self, globs: BaseGlobals) -> float:
        if not self.dependencies:
            return 0
        return max(dep.end_time for dep in self.dependencies)

    def register_with_parents(self):
        for dep in self.dependencies:
            dep.children.add(self)

    def calc_priority(self, globs: BaseGlobals):
        for dep in self.dependencies:
            dep.priority = max(self.priority + dep.instruction.cost(globs), dep.priority)
            dep.calc_priority(globs)


@dataclass
class Schedule:
    globs: BaseGlobals
    dag_nodes: list[DAG_Node]
    end_node: DAG_Node

    def get_linear_instructions(self) -> list[Instruction]:
        # dag_nodes are built in topological order
        return [node.instruction for node in self.dag_nodes]

    def smart_assign_to_sms(self):
        return assign_dag_to_sms(self)

    def round_robin_assign_to_sms(self):
        return round_robin_assign_to_sms(
            self.get_linear_instructions(), self.globs.sm_count()
        )


class ScheduleBuilder:
    @classmethod
    def make_globals(cls, model, seq_len: int = 0):
        raise NotImplementedError

    @classmethod
    def make_dag(cls, globs, stop_after_op: str | None = None, layer_limit: int | None = None):
        raise NotImplementedError

    @classmethod
    def build(
        cls,
        model,
        stop_after_op: str | None = None,
        layer_limit: int | None = None,
        seq_len: int = 0,
    ) -> Schedule:
        globs = cls.make_globals(model, seq_len=seq_len)
        dag_nodes, end_node = cls.make_dag(globs, stop_after_op, layer_limit)
        return Schedule(globs, dag_nodes, end_node)

    @classmethod
    def with_new_globals(cls, schedule: Schedule, model, seq_len: int = 0) -> Schedule:
        return replace(schedule, globs=cls.make_globals(model, seq_len=seq_len))


def assign_dag_to_sms(schedule: Schedule) -> list[list[Instruction]]:
    """List scheduling: the most expensive ready instruction goes to the SM
    that frees up first; children become ready once all parents are placed."""
    nodes = schedule.dag_nodes
    globs = schedule.globs
    for node in nodes:
        node.register_with_parents()
    for node in nodes:
        node.remaining_dependencies = set(node.dependencies)

    sm_count = globs.sm_count()
    queues: list[list[Instruction]] = [[] for _ in range(sm_count)]
    sm_free = [(0, sm) for sm in range(sm_count)]
    heapq.heapify(sm_free)

    index_of = {id(n): i for i, n in enumerate(nodes)}
    ready = [(-n.instruction.cost(globs), index_of[id(n)]) for n in nodes if not n.dependencies]
    heapq.heapify(ready)

    while ready:
        _, idx = heapq.heappop(ready)
        node = nodes[idx]
        sm_time, sm = heapq.heappop(sm_free)
        node.start_time = sm_time
        node.end_time = sm_time + node.instruction.cost(globs)
        queues[sm].append(node.instruction)
        heapq.heappush(sm_free, (node.end_time, sm))
        for child in node.children:
            child.remaining_dependencies.discard(node)
            if not child.remaining_dependencies:
                heapq.heappush(ready, (-child.instruction.cost(globs), index_of[id(child)]))
    return queues


def round_robin_assign_to_sms(instructions: list[Instruction], sm_count: int):
    queues: list[list[Instruction]] = [[] for _ in range(sm_count)]
    for i, ins in enumerate(instructions):
        queues[i % sm_count].append(ins)
    return queues


def zig_zag_assign_to_sms(instructions: list[Instruction], sm_count: int):
    """Round robin that reverses direction every sm_count instructions."""
    queues: list[list[Instruction]] = [[] for _ in range(sm_count)]
    for i, ins in enumerate(instructions):
        k = i % (2 * sm_count)
        sm = k if k < sm_count else 2 * sm_count - 1 - k
        queues[sm].append(ins)
    return queues


def collect_into_waves(instructions: list[Instruction]) -> list[list[Instruction]]:
    """Split the linear order into maximal runs of one opcode."""
    waves: list[list[Instruction]] = []
    for ins in instructions:
        if waves and waves[-1][-1].opcode() == ins.opcode():
            waves[-1].append(ins)
        else:
            waves.append([ins])
    return waves


def wave_assign_to_sms(schedule: Schedule):
    globs = schedule.globs
    sm_count = globs.sm_count()
    queues: list[list[Instruction]] = [[] for _ in range(sm_count)]
    load = [(0, sm) for sm in range(sm_count)]
    heapq.heapify(load)
    for wave in collect_into_waves(schedule.get_linear_instructions()):
        for ins in sorted(wave, key=lambda x: x.cost(globs), reverse=True):
            cost, sm = heapq.heappop(load)
            heapq.heappush(load, (cost + ins.cost(globs), sm))
            queues[sm].append(ins)
    return queues


def pool_assign_to_sms(instructions: list[Instruction], sm_count: int, memory_fraction: float):
    """Memory-pool instructions round-robin over the first share of SMs,
    compute-pool instructions over the rest."""
    memory, compute = [], []
    for ins in instructions:
        pool = ins.tags()["pool"]
        if pool == "memory":
            memory.append(ins)
        elif pool == "compute":
            compute.append(ins)
        else:
            raise ValueError(f"Unknown pool: {pool}")
    mem_sms = round(sm_count * memory_fraction)
    return round_robin_assign_to_sms(memory, mem_sms) + round_robin_assign_to_sms(
        compute, sm_count - mem_sms
    )


def assign_to_sms(
    mode: str,
    schedule: Schedule | None = None,
    instructions: list[Instruction] | None = None,
    sm_count: int | None = None,
    memory_fraction: float | None = None,
):
    if schedule is not None:
        instructions = schedule.get_linear_instructions()
        sm_count = schedule.globs.sm_count()
    if mode == "rr":
        return round_robin_assign_to_sms(instructions, sm_count)
    if mode == "zz":
        return zig_zag_assign_to_sms(instructions, sm_count)
    if mode == "wave":
        return wave_assign_to_sms(schedule)
    if mode == "dag":
        return assign_dag_to_sms(schedule)
    if mode == "pool":
        assert memory_fraction is not None
        return pool_assign_to_sms(instructions, sm_count, memory_fraction=memory_fraction)
    raise ValueError(f"Unknown mode: {mode}")


def serialize_and_pad(instruction: Instruction) -> list[int]:
    words = instruction.serialize()
    assert len(words) <= INTS_PER_INSTRUCTION, (
        f"{type(instruction).__name__} needs {len(words)} words"
    )
    return words + [0] * (INTS_PER_INSTRUCTION - len(words))


def tensorize_instructions(globs: BaseGlobals, instruction_queues: list[list[Instruction]]):
    num_sms = globs.sm_count()
    assert len(instruction_queues) == num_sms, (
        f"{len(instruction_queues)} queues for {num_sms} SMs"
    )
    queue_len = max(1, max(len(q) for q in instruction_queues))
    for q in instruction_queues:
        q.extend([NoOp()] * (queue_len - len(q)))

    globs.attention_reduction_fusable = attention_reduction_fusable(globs, instruction_queues)
    globs.deferrable_down_layers = deferrable_down_layers(instruction_queues)
    globs.lm_head_instructions = sum(1 for q in instruction_queues for ins in q if ins.opcode() == 7)
    globs.expert_predictions = sum(
        1 for q in instruction_queues for ins in q if type(ins).__name__ == "SpeculativeExpertPredict")
    words = [serialize_and_pad(ins) for q in instruction_queues for ins in q]
    globs.instructions = torch.tensor(words, dtype=torch.int32).view(
        num_sms, queue_len, INTS_PER_INSTRUCTION
    ).to(globs.device)
    globs.timings = torch.zeros(
        [num_sms, queue_len, TIMING_SLOTS], dtype=torch.int32, device=globs.device
    )


def attention_reduction_fusable(globs, instruction_queues) -> bool:
    """True when the attention merges of these queues can be done by the last
    PartialAttention (opcode 2) of each KV head instead of by the
    AttentionReduction (opcode 3) instructions: every reduction is terminal
    over all partials of its head group, in order, one per (layer, group), and
    each group's partials are exactly partial_idx 0..P-1 of one P. The engine
    then produces the same outputs and counter values (an engine option; the
    instruction stream itself is unchanged)."""
    heads = getattr(globs, "num_attention_heads", None)
    kv = getattr(globs, "num_kv_heads", None)
    if not heads or not kv:
        return False
    gqa = heads // kv
    reductions, partials = {}, {}
    for q in instruction_queues:
        for ins in q:
            op = ins.opcode()
            if op == 3:
                key = (ins.layer_idx, ins.head_start_idx)
                if (key in reductions or not ins.is_terminal or ins.head_start_idx % gqa
                        or list(ins.reduction_list) != list(range(ins.num_partials))):
                    return False
                reductions[key] = ins.num_partials
            elif op == 2:
                partials.setdefault((ins.layer_idx, ins.kv_head_idx), []).append(
                    (ins.num_partials, ins.partial_idx))
    if not reductions:
        return False
    for (layer, kv_head), parts in partials.items():
        n = parts[0][0]
        if sorted(parts) != [(n, i) for i in range(n)]:
            return False
        if n > 1 and reductions.get((layer, kv_head * gqa)) != n:
            return False
    return len(reductions) == sum(1 for parts in partials.values() if parts[0][0] > 1)


def deferrable_down_layers(instruction_queues) -> int:
    """Number of leading layers l whose DownProjResidual (opcode 6) may leave
    its column-split partials for layer l + 1 to add: the stream holds layer
    l's down projection and layer l + 1's QKV (opcode 1) and O_ProjResidual
    (opcode 4), the two readers of the residual stream that add them."""
    ops = {}
    for q in instruction_queues:
        for ins in q:
            op = ins.opcode()
            if op in (1, 4, 6):
                ops.setdefault(op, set()).add(ins.layer_idx)
    n = 0
    while n in ops.get(6, ()) and n + 1 in ops.get(1, ()) and n + 1 in ops.get(4, ()):
        n += 1
    return n
