"""CPU oracle for the Llama decode path (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this module, and only as the checker. The product path (megakernels +
libek.so) never calls it.

A restatement in plain torch-on-CPU of epic-kernel's Python interpreter
("PyVM"), megakernels/demos/latency/python_vm.py. Each instruction updates a
`Globals` bundle exactly as the reference solver does, with the same bf16
rounding points:
- RMSNorm (:50-56): fp32 x * rsqrt(mean(x^2) + eps), rounded to bf16, then
  times the bf16 weight.
- matvec (:29-47): bf16 weights times a bf16 vector, accumulated in fp32 and
  rounded once to bf16. This equals torch's CPU bf16 einsum.
- residual add (:59-80): hidden += bf16(partial), with one bf16 rounding per
  column split, in split order.
- attention (:291-357): fp32. LSE is log2(sum(exp(scores))).
- reduction (:360-401): exp2-weighted merge. A non-terminal merge stores the
  natural log of the denominator, as the reference does.

One deliberate difference from the reference interpreter: O_ProjResidual reduces
over the full hidden dimension. The reference interpreter reduces over
`matvec_reduction_size` columns (python_vm.py:108-117). That differs only when
gcd(I, H) < H, i.e. Llama-3.2-3B, where the reference interpreter drops 2/3 of
W_o. The reference's CUDA kernel and PyTorch model use the full dimension
(demos/low-latency-llama/matvec_adds.cu:202-208, llama.py:289).
`OPROJ_FULL_REDUCTION = False` restores the reference interpreter's behaviour.

Parity of this restatement is pinned against outputs of the reference
interpreter itself, run in the build container (tests/golden/make_golden.py).
"""

import math

import torch
import torch.nn.functional as F

OPROJ_FULL_REDUCTION = True

# opcodes (megakernels/demos/latency/instructions.py)
QKV, PARTIAL, REDUCTION, OPROJ, UPGATE, DOWN, LM_HEAD = 1, 2, 3, 4, 5, 6, 7


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """python_vm.py:50-56."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * xf.to(x.dtype)


def matvec(mat: torch.Tensor, vec: torch.Tensor) -> torch.Tensor:
    """bf16 [o, i] x bf16 [i] -> bf16 [o] with torch's CPU bf16 matrix-vector
    kernel, the op behind the reference's einsum (fp32 accumulation, one
    rounding)."""
    return torch.mv(mat, vec)


def rotate_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x * cos + rot(x) * sin with rot(x)[2i] = -x[2i+1], rot(x)[2i+1] = x[2i]
    (llama.py:136-174). bf16 x, fp32 tables -> fp32."""
    rot = torch.stack((-x[..., 1::2], x[..., 0::2]), dim=-1).reshape(x.shape)
    return x * cos + rot * sin


def _bar(g, layer, op):
    return g.barriers[layer, op - 1]


def _expected_down(g):
    return (g.intermediate_size // g.matvec_reduction_size) * (g.hidden_size // g.down_proj_block_size)


def solve_qkv(g, ins):
    """LayerNorm_QKV_MatVecRopeAppend, python_vm.py:182-262."""
    l = ins.layer_idx
    if l > 0:
        assert _bar(g, l - 1, DOWN)[0] == _expected_down(g)
    x = rms_norm(g.hidden_states, g.attn_ln_weights[l], g.rms_norm_eps)
    D, bs, pos = g.head_dim, g.qkv_block_size, g.pos_id
    k0 = g.num_attention_heads * D
    v0 = k0 + g.num_kv_heads * D
    bars = _bar(g, l, QKV)
    for b in range(ins.start_output_block_idx, ins.end_output_block_idx):
        s, e = b * bs, (b + 1) * bs
        out = matvec(g.qkv_proj_weights[l][s:e], x)
        if s < v0:
            seg = s % D
            out = rotate_interleaved(out, g.rope_cos[pos, seg : seg + bs], g.rope_sin[pos, seg : seg + bs])
        if s < k0:
            g.post_ln_rope_q[s:e] = out
        elif s < v0:
            g.k_cache[l, :, pos].view(-1)[s - k0 : e - k0] = out
        else:
            g.v_cache[l, :, pos].view(-1)[s - v0 : e - v0] = out
        bars[b // (D // bs)] += 1


def partial_token_range(g, num_partials, partial_idx):
    """python_vm.py:306-318."""
    seq = g.pos_id + 1
    total = math.ceil(seq / g.attn_kv_block_size)
    per = math.ceil(total / num_partials)
    b0 = partial_idx * per
    b1 = min(b0 + per, total)
    return b0 * g.attn_kv_block_size, min(b1 * g.attn_kv_block_size, seq)


def solve_partial(g, ins):
    """PartialAttention, python_vm.py:291-357."""
    gqa = g.num_attention_heads // g.num_kv_heads
    bph = g.head_dim // g.qkv_block_size
    l, h = ins.layer_idx, ins.kv_head_idx
    bars = _bar(g, l, QKV)
    for i in range(gqa):
        assert bars[h * gqa + i] == bph
    assert bars[g.num_attention_heads + h] == bph
    assert bars[g.num_attention_heads + g.num_kv_heads + h] == bph
    t0, t1 = partial_token_range(g, ins.num_partials, ins.partial_idx)
    k = g.k_cache[l, 0, t0:t1, h].float()
    v = g.v_cache[l, 0, t0:t1, h].float()
    hs, he = h * gqa, (h + 1) * gqa
    q = g.post_ln_rope_q.view(g.num_attention_heads, -1)[hs:he].float()
    scores = (q @ k.T) * g.attn_scale
    lse = torch.log2(torch.exp(scores).sum(-1))
    out = torch.softmax(scores, dim=-1) @ v
    if g.skip_attn_reduction:
        g.attn_out.view(g.num_attention_heads, -1)[hs:he] = out
        _bar(g, l, REDUCTION)[0] += he - hs
    else:
        g.attn_lse_intermediates[hs:he, ins.partial_idx] = lse
        g.attn_out_intermediates[hs:he, ins.partial_idx] = out
        _bar(g, l, PARTIAL)[hs:he] += 1


def solve_reduction(g, ins):
    """AttentionReduction, python_vm.py:360-401."""
    hs, n = ins.head_start_idx, g.attn_reduction_size
    assert _bar(g, ins.layer_idx, PARTIAL)[hs] == ins.num_partials
    idx = torch.tensor(ins.reduction_list, dtype=torch.long)
    lses = g.attn_lse_intermediates[hs : hs + n][:, idx]
    outs = g.attn_out_intermediates[hs : hs + n][:, idx]
    f = (lses - lses.max(dim=-1, keepdim=True).values).exp2()
    den = f.sum(-1, keepdim=True)
    red = (outs * f.unsqueeze(-1)).sum(dim=1) / den
    if ins.is_terminal:
        g.attn_out.view(g.num_attention_heads, -1)[hs : hs + n] = red
    else:
        g.attn_lse_intermediates[hs : hs + n, ins.output_partial_idx] = den.log().squeeze(-1)
        g.attn_out_intermediates[hs : hs + n, ins.output_partial_idx] = red
    _bar(g, ins.layer_idx, REDUCTION)[0] += n


def _matvec_add(g, mat, vec, ins, block_size, red_size):
    """python_vm.py:59-80."""
    rs, re = ins.reduction_block_idx * red_size, (ins.reduction_block_idx + 1) * red_size
    for b in range(ins.start_block_idx, ins.end_block_idx):
        s, e = b * block_size, (b + 1) * block_size
        g.hidden_states[s:e] += matvec(mat[s:e, rs:re], vec[rs:re])


def solve_oproj(g, ins):
    """O_ProjResidual, python_vm.py:101-120."""
    assert _bar(g, ins.layer_idx, REDUCTION)[0] == g.num_attention_heads
    assert ins.start_block_idx == ins.end_block_idx - 1 and ins.reduction_block_idx == 0
    red = g.hidden_size if OPROJ_FULL_REDUCTION else g.matvec_reduction_size
    _matvec_add(g, g.o_proj_weights[ins.layer_idx], g.attn_out, ins, g.o_proj_block_size, red)
    _bar(g, ins.layer_idx, OPROJ)[0] += ins.end_block_idx - ins.start_block_idx


def solve_down(g, ins):
    """DownProjResidual, python_vm.py:123-139."""
    assert _bar(g, ins.layer_idx, UPGATE)[0] == g.intermediate_size // g.up_gate_proj_block_size
    _matvec_add(g, g.down_proj_weights[ins.layer_idx], g.silu_out, ins, g.down_proj_block_size,
                g.matvec_reduction_size)
    _bar(g, ins.layer_idx, DOWN)[0] += ins.end_block_idx - ins.start_block_idx


def solve_upgate(g, ins):
    """LayerNormDoubleMatVecSiLU, python_vm.py:142-179."""
    l = ins.layer_idx
    assert _bar(g, l, OPROJ)[0] == g.hidden_size // g.o_proj_block_size
    x = rms_norm(g.hidden_states, g.mlp_ln_weights[l], g.rms_norm_eps)
    bs = g.up_gate_proj_block_size
    for b in ins.block_idxs:
        s, e = b * bs, (b + 1) * bs
        up = matvec(g.up_proj_weights[l][s:e], x)
        gate = matvec(g.gate_proj_weights[l][s:e], x)
        g.silu_out[s:e] = F.silu(gate) * up
        _bar(g, l, UPGATE)[0] += 1


def solve_lm_head(g, ins):
    """RMS_LM_Head, python_vm.py:265-288."""
    assert _bar(g, g.num_hidden_layers - 1, DOWN)[0] == _expected_down(g)
    x = rms_norm(g.hidden_states, g.lm_head_norm_weights, g.rms_norm_eps)
    bs = g.lm_head_block_size
    s, e = ins.start_output_block_idx * bs, ins.end_output_block_idx * bs
    g.logits[s:e] = matvec(g.lm_head_weights[s:e], x)


SOLVERS = {
    QKV: solve_qkv,
    PARTIAL: solve_partial,
    REDUCTION: solve_reduction,
    OPROJ: solve_oproj,
    UPGATE: solve_upgate,
    DOWN: solve_down,
    LM_HEAD: solve_lm_head,
}


def interpret(g, instructions):
    """interpret_with_pyvm (megakernels/python_vm.py:83-87): run in list order."""
    for ins in instructions:
        if ins.opcode() == 0:
            continue
        SOLVERS[ins.opcode()](g, ins)


def lm_head_tokens(model, hidden: torch.Tensor):
    """PyVM_Generator's output (generators.py:196-203): the model's PyTorch LM
    head on the final hidden, returning (bf16 logits, argmax)."""
    x = rms_norm(hidden, model.lm_head.input_norm.weight, model.config.rms_norm_eps)
    logits = F.linear(x, model.lm_head.lm_head.weight)
    return logits, int(torch.argmax(logits))


def pyvm_step(model, g, instructions, token: int, pos_id: int):
    """One PyVM_Generator.run (generators.py:182-204): embed, zero barriers,
    interpret, LM head. Returns (logits, next token)."""
    g.hidden_states[:] = model.model.embed_tokens.embed_tokens.weight[token]
    g.barriers.zero_()
    g.pos_id = pos_id
    interpret(g, instructions)
    return lm_head_tokens(model, g.hidden_states)
