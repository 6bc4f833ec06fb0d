"""`mk_mixtral`: drop-in replacement of epic-kernel's pybind module of that
name (demos/mixtral/mixtral.cu:28-94).

Positional signature as in the reference's caller
(megakernels/mixtral/mk.py:42-96): VM tensors, attention weights, expert
weights flattened to [L * E, ...], router [L * E, H], FFN norms, LM head
(norm as [1, H]), 4-D KV caches, rotary tables, activation buffers, router
outputs, then pos_id, attn_scale, rms_norm_eps, skip_attn_reduction, and
`stream=`. Keyword-only options: l2_prefetch_stages (lookahead L2 prefetch,
which also prefetches the predicted experts of expert instructions),
record_timings, timeout_ns, speculative_prefetch_stages (ring stages per
predicted expert L2-prefetched before the router's choice; 0 = off),
tp_lm_instructions (tensor parallel: LM-head
instructions per rank, set by megakernels.mixtral.tp).
"""

import ctypes

import torch

from megakernels import ek
from mk_llama import DEFAULT_CACHE_FLAGS, _need, check, read_status

_BF16 = torch.bfloat16
_cache: dict = {}


def _build(t, l2_prefetch_stages, record_timings, timeout_ns, tp_lm_instructions=0,
           cache_flags=DEFAULT_CACHE_FLAGS, prefetch_gap_ns=0):
    (barriers, instructions, timings, qkv_w, attn_ln_w, o_w, eg, eu, ed, router_w, ffn_ln_w, lm_norm, lm_w,
     k4, v4, cos, sin, hidden, q, attn_out, lse, o_int, esilu, rnormed, logits, sel, scores, pred) = t
    a = ek.EkMixtralArgs()
    a.barriers = _need(barriers, "barriers", torch.int32, 3)
    a.instructions = _need(instructions, "instructions", torch.int32, 3)
    a.timings = _need(timings, "timings", torch.int32, 3) if timings is not None else None
    a.qkv_weights = _need(qkv_w, "qkv_weights", _BF16, 3)
    a.attn_ln_weights = _need(attn_ln_w, "attn_ln_weights", _BF16, 2)
    a.o_weights = _need(o_w, "o_weights", _BF16, 3)
    a.expert_gate_weights = _need(eg, "expert_gate_weights", _BF16, 3)
    a.expert_up_weights = _need(eu, "expert_up_weights", _BF16, 3)
    a.expert_down_weights = _need(ed, "expert_down_weights", _BF16, 3)
    a.router_weights = _need(router_w, "router_weights", _BF16, 2)
    a.ffn_ln_weights = _need(ffn_ln_w, "ffn_ln_weights", _BF16, 2)
    a.lm_head_norm_weights = _need(lm_norm, "lm_head_norm_weights", _BF16)
    a.lm_head_weights = _need(lm_w, "lm_head_weights", _BF16, 2)
    a.k_cache = _need(k4, "k_cache", _BF16, 4)
    a.v_cache = _need(v4, "v_cache", _BF16, 4)
    a.rope_cos = _need(cos, "rope_cos", torch.float32, 2)
    a.rope_sin = _need(sin, "rope_sin", torch.float32, 2)
    a.hidden_states = _need(hidden, "hidden_states", _BF16)
    a.q_post_rope = _need(q, "q_post_rope", _BF16)
    a.attn_out = _need(attn_out, "attn_out", _BF16)
    a.attn_lse_intermediates = _need(lse, "attn_lse_intermediates", torch.float32, 2)
    a.attn_out_intermediates = _need(o_int, "attn_out_intermediates", torch.float32, 3)
    a.expert_silu_out = _need(esilu, "expert_silu_out", _BF16, 2)
    a.router_normed_hidden = _need(rnormed, "router_normed_hidden", _BF16)
    a.logits = _need(logits, "logits", _BF16)
    a.selected_expert_indices = _need(sel, "selected_expert_indices", torch.int32)
    a.selected_expert_scores = _need(scores, "selected_expert_scores", _BF16)
    a.predicted_expert_indices = _need(pred, "predicted_expert_indices", torch.int32)

    E, I = esilu.shape
    L = qkv_w.shape[0]
    H = qkv_w.shape[2]
    D, Hkv = k4.shape[3], k4.shape[2]
    Hq = lse.shape[0]
    V = lm_w.shape[0]
    checks = [
        (qkv_w.shape[1] == (Hq + 2 * Hkv) * D, "qkv_weights shape"),
        (o_w.shape == (L, H, Hq * D), "o_weights shape"),
        (eg.shape == (L * E, I, H) and eu.shape == eg.shape, "expert gate/up shape"),
        (ed.shape == (L * E, H, I), "expert down shape"),
        (router_w.shape == (L * E, H), "router shape"),
        (ffn_ln_w.shape == (L, H) and attn_ln_w.shape == (L, H), "norm shapes"),
        (lm_norm.numel() == H and lm_w.shape[1] == H, "lm head shapes"),
        (k4.shape[0] == L and v4.shape == k4.shape, "kv cache shapes"),
        (cos.shape[1] == D and sin.shape == cos.shape, "rope tables"),
        (hidden.numel() == H and rnormed.numel() == H, "hidden sizes"),
        (sel.numel() == scores.numel() == pred.numel(), "router output sizes"),
        (instructions.shape[2] == 32, "instructions last dim"),
    ]
    for ok, what in checks:
        if not ok:
            raise ValueError(f"mk_mixtral: inconsistent {what}")
    a.num_layers, a.hidden, a.intermediate, a.head_dim = L, H, I, D
    a.num_q_heads, a.num_kv_heads, a.vocab = Hq, Hkv, V
    a.num_experts, a.experts_per_token = E, sel.numel()
    a.kv_len, a.rope_rows, a.max_partials = k4.shape[1], cos.shape[0], lse.shape[1]
    a.barrier_rows, a.barrier_cols = barriers.shape[1], barriers.shape[2]
    a.num_queues, a.queue_len = instructions.shape[0], instructions.shape[1]
    a.l2_prefetch_stages = l2_prefetch_stages
    a.record_timings = int(bool(record_timings))
    a.timeout_ns = int(timeout_ns)
    a.tp_lm_instructions = int(tp_lm_instructions)
    a.cache_flags = int(cache_flags)
    a.prefetch_gap_ns = int(prefetch_gap_ns)
    return a, hidden.device.index


def mk_mixtral(
    barriers, instructions, timings,
    qkv_weights, attn_norm_weights, o_weights,
    expert_gate_weights, expert_up_weights, expert_down_weights, router_weights, ffn_ln_weights,
    lm_head_norm_weights, lm_head_weights,
    k_cache, v_cache, rope_cos, rope_sin,
    hidden_states, q_post_rope, attn_out, attn_lse_intermediates, attn_out_intermediates,
    expert_silu_out, router_normed_hidden, logits,
    selected_expert_indices, selected_expert_scores, predicted_expert_indices,
    pos_id, attn_scale, rms_norm_eps, skip_attn_reduction,
    *, stream=None, l2_prefetch_stages: int = 0, record_timings: bool = False, timeout_ns: int = 0,
    tp_lm_instructions: int = 0, cache_flags: int | None = None, prefetch_gap_ns: int = 0,
    speculative_prefetch_stages: int = 0,
):
    t = (barriers, instructions, timings, qkv_weights, attn_norm_weights, o_weights, expert_gate_weights,
         expert_up_weights, expert_down_weights, router_weights, ffn_ln_weights, lm_head_norm_weights,
         lm_head_weights, k_cache, v_cache, rope_cos, rope_sin, hidden_states, q_post_rope, attn_out,
         attn_lse_intermediates, attn_out_intermediates, expert_silu_out, router_normed_hidden, logits,
         selected_expert_indices, selected_expert_scores, predicted_expert_indices)
    if cache_flags is None:
        cache_flags = DEFAULT_CACHE_FLAGS
    key = (tuple((x.data_ptr(), tuple(x.shape), x.dtype) if x is not None else None for x in t),
           l2_prefetch_stages, bool(record_timings), int(timeout_ns), int(tp_lm_instructions),
           int(cache_flags), int(prefetch_gap_ns))
    hit = _cache.get(key)
    if hit is None:
        hit = _build(t, l2_prefetch_stages, record_timings, timeout_ns, tp_lm_instructions,
                     cache_flags, prefetch_gap_ns)
        if len(_cache) > 64:
            _cache.clear()
        _cache[key] = hit
    args, device = hit
    args.pos_id = int(pos_id)
    args.attn_scale = float(attn_scale)
    args.rms_norm_eps = float(rms_norm_eps)
    args.skip_attn_reduction = int(bool(skip_attn_reduction))
    args.speculative_prefetch_stages = int(speculative_prefetch_stages)
    ctx = ek.context_for(device)
    if stream is None:
        stream = torch.cuda.current_stream(device)
    handle = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    ek.check(ek.load_library().ek_mixtral_decode(ctx.handle, ctypes.byref(args), ctypes.c_void_p(handle)),
             "ek_mixtral_decode")


__all__ = ["mk_mixtral", "check", "read_status"]
