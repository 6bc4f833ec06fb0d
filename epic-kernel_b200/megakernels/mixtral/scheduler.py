"""Mixtral decode schedule: globals and the per-layer instruction DAG.

Same behaviour as `megakernels/mixtral/scheduler.py` of epic-kernel:
- `pick_num_attention_partitions` (:24-32) is the Llama rule with a floor of 1.
- `make_globals` (:35-152) uses barriers `[L, 10, max(Hq + 2 Hkv, E)]` and
  16-row blocks.
- `schedule_*` (:159-254): QKV and RmsRouterUpgate split blocks evenly over
  min(sm_count, blocks) SMs; ExpertDownProjFused reduces over all of I; the LM
  head runs hidden / 2048 column splits.
- `make_dag_layer` (:290-418): one SpeculativeExpertPredict per layer, which
  depends on the previous layer's outputs, as QKV does.
"""

import math

import torch

from megakernels.instructions import NoOp
from megakernels.mixtral.instructions import (
    ExpertDownProjFused,
    Mixtral_AttnReduction,
    Mixtral_OProj,
    Mixtral_PartialAttn,
    Mixtral_QKV,
    Mixtral_RMS_LM_Head,
    MixtralGlobals,
    RmsRouterUpgate,
    SpeculativeExpertPredict,
)
from megakernels.scheduler import DAG_Node, ScheduleBuilder
from megakernels.utils import assert_div, get_sm_count

B200_SM_COUNT = 160
LM_HEAD_SPLIT = 2048


def pick_num_attention_partitions(prompt_len: int, ntok: int, num_kv_heads: int, device) -> int:
    num_divisions = math.ceil((prompt_len + ntok) / 256)
    sm_count = min(get_sm_count(device), B200_SM_COUNT)
    return max(1, min(num_divisions, sm_count // num_kv_heads))


def make_globals(model, skip_attn_reduction: bool | None = None, seq_len: int = 0) -> MixtralGlobals:
    config = model.config
    device = model.device
    dtype = model.dtype
    sp = model.stacked_params
    if skip_attn_reduction is None:
        parts = pick_num_attention_partitions(seq_len + 1, 0, config.num_key_value_heads, device)
        skip_attn_reduction = parts == 1

    def buf(shape, buf_dtype=dtype):
        return torch.zeros(shape, device=device, dtype=buf_dtype)

    E = config.num_local_experts
    # = hidden / heads (reference scheduler.py:70); explicit on tensor-parallel shards
    head_dim = getattr(config, "head_dim", config.hidden_size // config.num_attention_heads)
    qdim = config.num_attention_heads * head_dim
    max_parts = get_sm_count(device)
    empty = torch.empty(0, device=device, dtype=dtype)
    return MixtralGlobals(
        qkv_proj_weights=sp.qkv_proj,
        attn_ln_weights=sp.attn_ln_weight,
        o_proj_weights=sp.o_proj,
        mlp_ln_weights=empty,
        up_proj_weights=empty,
        gate_proj_weights=empty,
        down_proj_weights=empty,
        lm_head_norm_weights=model.lm_head.input_norm.weight,
        lm_head_weights=model.lm_head.lm_head.weight,
        k_cache=model.stacked_kv_cache[0],
        v_cache=model.stacked_kv_cache[1],
        rope_cos=model.model.rope_cos,
        rope_sin=model.model.rope_sin,
        num_hidden_layers=config.num_hidden_layers,
        num_attention_heads=config.num_attention_heads,
        num_kv_heads=config.num_key_value_heads,
        head_dim=head_dim,
        hidden_size=config.hidden_size,
        intermediate_size=config.intermediate_size,
        vocab_size=config.vocab_size,
        attn_scale=1.0 / math.sqrt(head_dim),
        rms_norm_eps=config.rms_norm_eps,
        device=device,
        barriers=torch.zeros(
            [config.num_hidden_layers, 10, max(config.num_attention_heads + 2 * config.num_key_value_heads, E)],
            dtype=torch.int32, device=device),
        pos_id=seq_len,
        hidden_states=buf(config.hidden_size),
        post_ln_rope_q=buf(qdim),
        attn_out=buf(qdim),
        attn_out_intermediates=buf([config.num_attention_heads, max_parts, head_dim], torch.float32),
        attn_lse_intermediates=buf([config.num_attention_heads, max_parts], torch.float32),
        expert_silu_out=buf([E, config.intermediate_size]),
        router_normed_hidden=buf(config.hidden_size),
        logits=buf(config.vocab_size),
        selected_expert_indices=torch.zeros(config.num_experts_per_tok, dtype=torch.int32, device=device),
        selected_expert_scores=torch.zeros(config.num_experts_per_tok, dtype=dtype, device=device),
        predicted_expert_indices=torch.zeros(config.num_experts_per_tok, dtype=torch.int32, device=device),
        router_weights=sp.router_weight,
        expert_gate_weights=sp.expert_gate,
        expert_up_weights=sp.expert_up,
        expert_down_weights=sp.expert_down,
        ffn_ln_weights=sp.ffn_ln_weight,
        num_experts=E,
        num_experts_per_tok=config.num_experts_per_tok,
        skip_attn_reduction=skip_attn_reduction,
        expert_proj_block_size=16,
        down_proj_block_size=16,
        o_proj_block_size=16,
        lm_head_block_size=16,
        qkv_block_size=16,
        attn_kv_block_size=16,
        matvec_reduction_size=math.gcd(config.intermediate_size, config.hidden_size),
        attn_reduction_size=config.num_attention_heads // config.num_key_value_heads,
    )


def _ranges(num_blocks: int, sm_count: int):
    n = min(sm_count, num_blocks)
    per = num_blocks / n
    return [(round(i * per), round((i + 1) * per)) for i in range(n)]


def schedule_qkv(globs: MixtralGlobals, layer_idx: int):
    blocks = assert_div((globs.num_attention_heads + 2 * globs.num_kv_heads) * globs.head_dim, globs.qkv_block_size)
    return [Mixtral_QKV(layer_idx, s, e) for s, e in _ranges(blocks, globs.sm_count())]


def schedule_rms_router_upgate(globs: MixtralGlobals, layer_idx: int):
    blocks = assert_div(globs.intermediate_size, globs.expert_proj_block_size)
    return [RmsRouterUpgate(layer_idx, s, e - s) for s, e in _ranges(blocks, globs.sm_count()) if s < e]


def schedule_expert_downproj_fused(globs: MixtralGlobals, layer_idx: int):
    blocks = assert_div(globs.hidden_size, globs.down_proj_block_size)
    return [ExpertDownProjFused(layer_idx, s, e, 0) for s, e in _ranges(blocks, globs.sm_count())]


def schedule_speculative_predict(globs: MixtralGlobals, layer_idx: int):
    return [SpeculativeExpertPredict(layer_idx)]


def schedule_lm_head(globs: MixtralGlobals):
    blocks = assert_div(globs.vocab_size, globs.lm_head_block_size)
    out = []
    for split in range(globs.hidden_size // LM_HEAD_SPLIT):
        out.extend(Mixtral_RMS_LM_Head(s, e, split) for s, e in _ranges(blocks, globs.sm_count()))
    return out


def make_dag(globs: MixtralGlobals, stop_after_op: str | None = None, layer_limit: int | None = None):
    nodes: list[DAG_Node] = []
    nlayers = layer_limit if layer_limit is not None else globs.num_hidden_layers
    last: list[DAG_Node] = []
    for layer_idx in range(nlayers):
        new, last = make_dag_layer(globs, layer_idx, last, stop_after_op)
        nodes.extend(new)
    if nlayers == globs.num_hidden_layers and stop_after_op is None:
        lm = [DAG_Node(ins, last) for ins in schedule_lm_head(globs)]
        nodes.extend(lm)
        last = lm
    return nodes, DAG_Node(NoOp(), last)


def make_dag_layer(globs: MixtralGlobals, layer_idx: int, prev: list[DAG_Node], stop_after_op: str | None = None):
    parts = pick_num_attention_partitions(globs.pos_id + 1, 0, globs.num_kv_heads, globs.device)
    globs.skip_attn_reduction = parts == 1
    new: list[DAG_Node] = []

    qkv = [DAG_Node(ins, prev) for ins in schedule_qkv(globs, layer_idx)]
    owner = {b: n for n in qkv for b in n.instruction.block_indices()}
    new.extend(qkv)
    if getattr(globs, "speculative_prediction", True):
        new.extend(DAG_Node(ins, prev) for ins in schedule_speculative_predict(globs, layer_idx))
    if stop_after_op == "qkv":
        return new, qkv

    bph = globs.head_dim // globs.qkv_block_size
    partials = []
    for kv in range(globs.num_kv_heads):
        kb = (globs.num_attention_heads + kv) * globs.head_dim // globs.qkv_block_size
        vb = (globs.num_attention_heads + globs.num_kv_heads + kv) * globs.head_dim // globs.qkv_block_size
        deps = list({owner[b] for b in list(range(kb, kb + bph)) + list(range(vb, vb + bph))})
        for p in range(parts):
            partials.append(DAG_Node(Mixtral_PartialAttn(layer_idx, kv, parts, p), deps))
    new.extend(partials)
    if stop_after_op == "partial":
        return new, partials

    gqa = globs.num_attention_heads // globs.num_kv_heads
    if parts > 1:
        reds = []
        for kv in range(globs.num_kv_heads):
            ins = Mixtral_AttnReduction(layer_idx, kv * gqa, parts, True, list(range(parts)), None)
            reds.append(DAG_Node(ins, [n for n in partials if n.instruction.kv_head_idx == kv]))
        new.extend(reds)
        o_deps = reds
    else:
        o_deps = partials
    if stop_after_op == "reduction":
        return new, o_deps

    oproj = [DAG_Node(Mixtral_OProj(layer_idx, b, b + 1, 0), o_deps)
             for b in range(assert_div(globs.hidden_size, globs.o_proj_block_size))]
    new.extend(oproj)
    if stop_after_op == "oproj":
        return new, oproj

    upgate = [DAG_Node(ins, oproj) for ins in schedule_rms_router_upgate(globs, layer_idx)]
    new.extend(upgate)
    if stop_after_op in ("router", "expert_upgate", "rms_router_upgate"):
        return new, upgate

    down = [DAG_Node(ins, upgate) for ins in schedule_expert_downproj_fused(globs, layer_idx)]
    new.extend(down)
    if stop_after_op in ("downproj", "expert_downproj", "downproj_fused"):
        return new, down
    assert stop_after_op is None
    return new, down


class MixtralLatencyScheduleBuilder(ScheduleBuilder):
    @classmethod
    def make_globals(cls, model, seq_len: int = 0) -> MixtralGlobals:
        return make_globals(model, seq_len=seq_len)

    @classmethod
    def make_dag(cls, globs, stop_after_op=None, layer_limit=None):
        return make_dag(globs, stop_after_op, layer_limit)


class MixtralNoSpeculationScheduleBuilder(MixtralLatencyScheduleBuilder):
    """The same schedule without SpeculativeExpertPredict instructions (the
    "speculative prediction off" configuration); the engine then prefetches
    no expert weights before the router's choice."""

    @classmethod
    def make_globals(cls, model, seq_len: int = 0) -> MixtralGlobals:
        globs = make_globals(model, seq_len=seq_len)
        globs.speculative_prediction = False
        return globs
