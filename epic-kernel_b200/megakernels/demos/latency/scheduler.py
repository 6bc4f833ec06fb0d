"""Llama decode schedule: globals allocation and the per-layer instruction DAG.

Same behaviour as `megakernels/demos/latency/scheduler.py` of epic-kernel, so
that both interpreters see identical instruction streams:
- `pick_num_attention_partitions` (:25-38): ceil(len / 256) slices of the KV
  cache per KV head, capped at sm_count // num_kv_heads (sm_count <= 160).
- `make_globals` (:41-131): activation buffers, fp32 attention intermediates
  `[Hq, sm_count(, D)]`, barriers `[L, 10, Hq + 2 Hkv]`, 16-row blocks and
  `matvec_reduction_size = gcd(I, H)`.
- `schedule_qkv` / `schedule_upgate` / `schedule_downproj` / `schedule_lm_head`
  (:134-248) split the outputs over the SMs, and `make_dag_layer` (:286-428)
  wires the dependencies.
"""

import math

import torch

from megakernels.demos.latency.instructions import (
    AttentionReduction,
    DownProjResidual,
    Globals,
    Instruction,
    LayerNorm_QKV_MatVecRopeAppend,
    LayerNormDoubleMatVecSiLU,
    O_ProjResidual,
    PartialAttention,
    RMS_LM_Head,
)
from megakernels.instructions import NoOp
from megakernels.scheduler import DAG_Node, ScheduleBuilder
from megakernels.utils import assert_div, get_sm_count

# Upper bound the reference applies to the SM count when sizing attention splits.
B200_SM_COUNT = 160
MIN_ATTENTION_CHUNK = 256


def pick_num_attention_partitions(prompt_len: int, ntok: int, num_kv_heads: int, device) -> int:
    full_len = prompt_len + ntok
    num_divisions = math.ceil(full_len / MIN_ATTENTION_CHUNK)
    sm_count = min(get_sm_count(device), B200_SM_COUNT)
    parts = min(num_divisions, sm_count // num_kv_heads)
    assert parts >= 1
    return parts


def make_globals(model, skip_attn_reduction: bool | None = None, seq_len: int = 0) -> Globals:
    config = model.config
    device = model.device
    dtype = model.dtype

    if skip_attn_reduction is None:
        # the DAG is built for pos_id = seq_len, i.e. seq_len + 1 cached tokens
        parts = pick_num_attention_partitions(seq_len + 1, 0, config.num_key_value_heads, device)
        skip_attn_reduction = parts == 1

    def zeros(shape, buffer_dtype=dtype):
        return torch.zeros(shape, device=device, dtype=buffer_dtype)

    sp = model.stacked_params
    max_attn_partitions = get_sm_count(device)
    head_dim = config.head_dim

    barriers = torch.zeros(
        [config.num_hidden_layers, 10, config.num_attention_heads + 2 * config.num_key_value_heads],
        dtype=torch.int32,
        device=device,
    )

    return Globals(
        qkv_proj_weights=sp.qkv_proj,
        o_proj_weights=sp.o_proj,
        attn_ln_weights=sp.attn_ln_weight,
        mlp_ln_weights=sp.mlp_ln_weight,
        up_proj_weights=sp.up_proj,
        gate_proj_weights=sp.gate_proj,
        down_proj_weights=sp.down_proj,
        lm_head_norm_weights=model.lm_head.input_norm.weight,
        lm_head_weights=model.lm_head.lm_head.weight,
        k_cache=model.stacked_kv_cache[0],
        v_cache=model.stacked_kv_cache[1],
        rope_cos=model.model.rope_cos,
        rope_sin=model.model.rope_sin,
        hidden_states=zeros(config.hidden_size),
        post_ln_rope_q=zeros(config.hidden_size),
        attn_out=zeros(config.hidden_size),
        attn_out_intermediates=zeros(
            [config.num_attention_heads, max_attn_partitions, head_dim], torch.float32
        ),
        attn_lse_intermediates=zeros([config.num_attention_heads, max_attn_partitions], torch.float32),
        silu_out=zeros(config.intermediate_size),
        logits=zeros(config.vocab_size),
        pos_id=seq_len,
        attn_scale=1 / math.sqrt(head_dim),
        rms_norm_eps=config.rms_norm_eps,
        skip_attn_reduction=skip_attn_reduction,
        num_hidden_layers=config.num_hidden_layers,
        num_attention_heads=config.num_attention_heads,
        num_kv_heads=config.num_key_value_heads,
        head_dim=head_dim,
        hidden_size=config.hidden_size,
        intermediate_size=config.intermediate_size,
        up_gate_proj_block_size=16,
        down_proj_block_size=16,
        qkv_block_size=16,
        o_proj_block_size=16,
        lm_head_block_size=16,
        matvec_reduction_size=math.gcd(config.intermediate_size, config.hidden_size),
        attn_kv_block_size=16,
        attn_reduction_size=config.num_attention_heads // config.num_key_value_heads,
        vocab_size=config.vocab_size,
        device=device,
        barriers=barriers,
    )


def _even_ranges(num_blocks: int, num_sms: int):
    """[round(i * n / s), round((i + 1) * n / s)) for each SM i."""
    per_sm = num_blocks / num_sms
    return [(round(i * per_sm), round((i + 1) * per_sm)) for i in range(num_sms)]


def schedule_qkv(globs: Globals, layer_idx: int) -> list[LayerNorm_QKV_MatVecRopeAppend]:
    qkv_outdim = (globs.num_attention_heads + 2 * globs.num_kv_heads) * globs.head_dim
    num_blocks = assert_div(qkv_outdim, globs.qkv_block_size)
    sm_count = globs.sm_count()
    assert num_blocks / sm_count > 1
    return [
        LayerNorm_QKV_MatVecRopeAppend(layer_idx, start, end)
        for start, end in _even_ranges(num_blocks, sm_count)
    ]


def schedule_upgate(globs: Globals, layer_idx: int) -> list[Instruction]:
    num_blocks = assert_div(globs.intermediate_size, globs.up_gate_proj_block_size)
    sm_count = globs.sm_count()
    assert num_blocks / sm_count > 1
    # SM i takes blocks i, i + sm_count, i + 2 sm_count, ...
    return [
        LayerNormDoubleMatVecSiLU(layer_idx, list(range(sm, num_blocks, sm_count)))
        for sm in range(sm_count)
    ]


def schedule_downproj(globs: Globals, layer_idx: int) -> list[Instruction]:
    """Jobs (column split, row block) in column-major order are dealt out in
    contiguous runs; a run never crosses into the next column split."""
    num_row_blocks = assert_div(globs.hidden_size, globs.down_proj_block_size)
    num_col_splits = assert_div(globs.intermediate_size, globs.matvec_reduction_size)
    sm_count = globs.sm_count()
    jobs = [(c, b) for c in range(num_col_splits) for b in range(num_row_blocks)]

    out: list[Instruction] = []
    taken = 0
    for sm in range(sm_count):
        per_sm = (len(jobs) - taken) / (sm_count - sm)
        assert per_sm > 1
        run = jobs[taken : taken + round(per_sm)]
        col = run[0][0]
        run = [job for job in run if job[0] == col]
        first = run[0][1]
        assert [job[1] for job in run] == list(range(first, first + len(run)))
        out.append(DownProjResidual(layer_idx, first, first + len(run), col))
        taken += len(run)
    return out


def schedule_lm_head(globs: Globals) -> list[Instruction]:
    num_blocks = assert_div(globs.vocab_size, globs.lm_head_block_size)
    sm_count = globs.sm_count()
    assert num_blocks / sm_count > 1
    return [RMS_LM_Head(start, end) for start, end in _even_ranges(num_blocks, sm_count)]


def make_dag(globs: Globals, stop_after_op: str | None = None, layer_limit: int | None = None):
    nodes: list[DAG_Node] = []
    nlayers = layer_limit if layer_limit is not None else globs.num_hidden_layers

    last_outputs: list[DAG_Node] = []
    for layer_idx in range(nlayers):
        new_nodes, last_outputs = make_dag_layer(globs, layer_idx, last_outputs, stop_after_op)
        nodes.extend(new_nodes)

    if nlayers == globs.num_hidden_layers:
        lm_nodes = [DAG_Node(ins, last_outputs) for ins in schedule_lm_head(globs)]
        nodes.extend(lm_nodes)
        last_outputs = lm_nodes

    return nodes, DAG_Node(NoOp(), last_outputs)


def make_dag_layer(
    globs: Globals,
    layer_idx: int,
    prev_layer_outputs: list[DAG_Node],
    stop_after_op: str | None = None,
):
    parts = pick_num_attention_partitions(globs.pos_id + 1, 0, globs.num_kv_heads, globs.device)
    globs.skip_attn_reduction = parts == 1
    new_nodes: list[DAG_Node] = []

    qkv_nodes = [DAG_Node(ins, prev_layer_outputs) for ins in schedule_qkv(globs, layer_idx)]
    owner_of_block = {}
    for node in qkv_nodes:
        for b in node.instruction.block_indices():
            owner_of_block[b] = node
    new_nodes.extend(qkv_nodes)
    if stop_after_op == "qkv":
        return new_nodes, qkv_nodes

    # each partial waits on the QKV instructions that produced its K and V heads
    blocks_per_head = assert_div(globs.head_dim, globs.qkv_block_size)
    partial_nodes: list[DAG_Node] = []
    for kv_head in range(globs.num_kv_heads):
        k_block = (globs.num_attention_heads + kv_head) * blocks_per_head
        v_block = (globs.num_attention_heads + globs.num_kv_heads + kv_head) * blocks_per_head
        producer_blocks = list(range(k_block, k_block + blocks_per_head)) + list(
            range(v_block, v_block + blocks_per_head)
        )
        deps = list({owner_of_block[b] for b in producer_blocks})
        for p in range(parts):
            partial_nodes.append(DAG_Node(PartialAttention(layer_idx, kv_head, parts, p), deps))
    new_nodes.extend(partial_nodes)
    if stop_after_op == "partial":
        return new_nodes, partial_nodes

    gqa = globs.num_attention_heads // globs.num_kv_heads
    if parts > 1:
        reduction_nodes = []
        for kv_head in range(globs.num_kv_heads):
            ins = AttentionReduction(
                layer_idx=layer_idx,
                head_start_idx=kv_head * gqa,
                num_partials=parts,
                is_terminal=True,
                reduction_list=list(range(parts)),
                output_partial_idx=None,
            )
            deps = [n for n in partial_nodes if n.instruction.kv_head_idx == kv_head]
            reduction_nodes.append(DAG_Node(ins, deps))
        new_nodes.extend(reduction_nodes)
        o_deps = reduction_nodes
    else:
        o_deps = partial_nodes

    num_o_blocks = assert_div(globs.hidden_size, globs.o_proj_block_size)
    o_nodes = [DAG_Node(O_ProjResidual(layer_idx, b, b + 1, 0), o_deps) for b in range(num_o_blocks)]
    new_nodes.extend(o_nodes)
    if stop_after_op == "oproj":
        return new_nodes, o_nodes

    upgate_nodes = [DAG_Node(ins, o_nodes) for ins in schedule_upgate(globs, layer_idx)]
    new_nodes.extend(upgate_nodes)
    if stop_after_op == "upgate":
        return new_nodes, upgate_nodes

    down_nodes = [DAG_Node(ins, upgate_nodes) for ins in schedule_downproj(globs, layer_idx)]
    new_nodes.extend(down_nodes)
    if stop_after_op == "downproj":
        return new_nodes, down_nodes

    assert stop_after_op is None
    return new_nodes, down_nodes


class LatencyScheduleBuilder(ScheduleBuilder):
    @classmethod
    def make_globals(cls, model, seq_len: int = 0):
        return make_globals(model, seq_len=seq_len)

    @classmethod
    def make_dag(cls, globs, stop_after_op: str | None = None, layer_limit: int | None = None):
        return make_dag(globs, stop_after_op, layer_limit)
