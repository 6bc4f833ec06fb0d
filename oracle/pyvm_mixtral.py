"""CPU oracle for the Mixtral decode path (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this module, and only as the checker.

A restatement in torch-on-CPU of epic-kernel's Mixtral interpreter,
megakernels/mixtral/python_vm.py. Opcodes 1-3 share the Llama restatement
(oracle/pyvm.py); the rest:
- O-proj (:500-519): hidden += bf16(W_o[rows] . attn_out), full hidden.
- RmsRouterUpgate (:525-574): normed = RMSNorm(hidden, ffn_ln) (bf16); router
  logits = W_r.float() @ normed.float(); softmax; top-k; scores renormalised
  (top / sum) and stored as bf16; for each selected expert in top-k order, for
  each block, silu(bf16 gate) * bf16 up -> expert_silu_out[expert].
- ExpertDownProjFused (:581-611): for each selected expert in top-k order, for
  each block, hidden += bf16(float(score) * bf16(W_down[e][rows] . silu[e])).
- Mixtral_RMS_LM_Head (:618-642): logits[rows] += bf16 partial over a
  2048-column window of the RMSNorm'd hidden.
- SpeculativeExpertPredict (:653-668): top-k of the router on the current
  hidden -> predicted_expert_indices (a prefetch hint only).

The reference interpreter rebinds `globs.router_normed_hidden` instead of
writing into it; this oracle writes the normed vector into the buffer, as the
reference's CUDA kernel does.

Pinned against the reference interpreter's own outputs
(tests/golden/mixtral_*.npz, made by tests/golden/make_golden.py).
"""

import torch
import torch.nn.functional as F

from oracle import pyvm
from oracle.pyvm import matvec, rms_norm

QKV, PARTIAL, REDUCTION, OPROJ, ROUTER_UPGATE, DOWN, LM_HEAD, PREDICT = 1, 2, 3, 4, 5, 6, 7, 8
LM_HEAD_SPLIT = 2048


def _bar(g, layer, op):
    return g.barriers[layer, op - 1]


def _expected_down(g):
    return g.num_experts_per_tok * (g.hidden_size // g.down_proj_block_size)


def solve_qkv(g, ins):
    """Mixtral_QKV (python_vm.py:358-418): the Llama arithmetic; the cross-layer
    wait targets ExpertDownProjFused's count (k x H / 16)."""
    saved = pyvm._expected_down
    pyvm._expected_down = _expected_down
    try:
        pyvm.solve_qkv(g, ins)
    finally:
        pyvm._expected_down = saved


def router_topk(g, layer, normed):
    """fp32 router logits, softmax, top-k, renormalised scores (python_vm.py:541-550)."""
    logits = g.router_weights[layer].float() @ normed.float()
    scores = torch.softmax(logits, dim=-1)
    top, idx = torch.topk(scores, g.num_experts_per_tok)
    return top / top.sum(), idx


def solve_oproj(g, ins):
    assert _bar(g, ins.layer_idx, REDUCTION)[0] == g.num_attention_heads
    s, e = ins.start_block_idx * g.o_proj_block_size, ins.end_block_idx * g.o_proj_block_size
    g.hidden_states[s:e] += matvec(g.o_proj_weights[ins.layer_idx][s:e], g.attn_out)
    _bar(g, ins.layer_idx, OPROJ)[0] += ins.end_block_idx - ins.start_block_idx


def solve_router_upgate(g, ins):
    l = ins.layer_idx
    assert _bar(g, l, OPROJ)[0] == g.hidden_size // g.o_proj_block_size
    normed = rms_norm(g.hidden_states, g.ffn_ln_weights[l], g.rms_norm_eps)
    g.router_normed_hidden.copy_(normed)
    top, idx = router_topk(g, l, normed)
    g.selected_expert_indices.copy_(idx.to(torch.int32))
    g.selected_expert_scores.copy_(top.to(g.selected_expert_scores.dtype))
    bs = g.expert_proj_block_size
    for e in g.selected_expert_indices.tolist():
        for b in ins.block_indices():
            s, t = b * bs, (b + 1) * bs
            gate = matvec(g.expert_gate_weights[l, e][s:t], normed)
            up = matvec(g.expert_up_weights[l, e][s:t], normed)
            g.expert_silu_out[e, s:t] = (F.silu(gate) * up).to(g.expert_silu_out.dtype)
    _bar(g, l, ROUTER_UPGATE)[0] += ins.num_blocks


def solve_down(g, ins):
    l = ins.layer_idx
    assert _bar(g, l, ROUTER_UPGATE)[0] == g.intermediate_size // g.expert_proj_block_size
    bs = g.down_proj_block_size
    experts = g.selected_expert_indices.tolist()
    for k in range(g.num_experts_per_tok):
        e = experts[k]
        score = g.selected_expert_scores[k].float()
        for b in range(ins.start_block_idx, ins.end_block_idx):
            s, t = b * bs, (b + 1) * bs
            out = matvec(g.expert_down_weights[l, e][s:t], g.expert_silu_out[e])
            g.hidden_states[s:t] += (score * out).to(g.hidden_states.dtype)
    _bar(g, l, DOWN)[0] += (ins.end_block_idx - ins.start_block_idx) * g.num_experts_per_tok


def solve_lm_head(g, ins):
    assert _bar(g, g.num_hidden_layers - 1, DOWN)[0] == _expected_down(g)
    x = rms_norm(g.hidden_states, g.lm_head_norm_weights, g.rms_norm_eps)
    c0 = ins.reduction_block_idx * LM_HEAD_SPLIT
    bs = g.lm_head_block_size
    for b in range(ins.start_output_block_idx, ins.end_output_block_idx):
        s, t = b * bs, (b + 1) * bs
        g.logits[s:t] += matvec(g.lm_head_weights[s:t, c0 : c0 + LM_HEAD_SPLIT], x[c0 : c0 + LM_HEAD_SPLIT])


def solve_predict(g, ins):
    l = ins.layer_idx
    if l > 0:
        assert _bar(g, l - 1, DOWN)[0] == _expected_down(g)
    normed = rms_norm(g.hidden_states, g.ffn_ln_weights[l], g.rms_norm_eps)
    _, idx = router_topk(g, l, normed)
    g.predicted_expert_indices.copy_(idx.to(torch.int32))
    _bar(g, l, PREDICT)[0] += 1


SOLVERS = {
    QKV: solve_qkv,
    PARTIAL: pyvm.solve_partial,
    REDUCTION: pyvm.solve_reduction,
    OPROJ: solve_oproj,
    ROUTER_UPGATE: solve_router_upgate,
    DOWN: solve_down,
    LM_HEAD: solve_lm_head,
    PREDICT: solve_predict,
}


def interpret(g, instructions):
    for ins in instructions:
        if ins.opcode() == 0:
            continue
        SOLVERS[ins.opcode()](g, ins)
