"""Generate the golden fixtures under tests/golden/ by running epic-kernel's
own Python interpreter (the reference "PyVM") on CPU.

Run in the build container, where the reference checkout is importable:

    python tests/golden/make_golden.py --reference /path/to/epic-kernel [--full]

Nothing on the GPU host runs this; the tests read only the committed .npz/.json
outputs. Weights and inputs come from `megakernels.synthetic` (numpy PCG64),
so the GPU host rebuilds the same model bit for bit from the seeds recorded
in each fixture.

The reference needs two shims. `accelerate` is not installed, so a stub with
a no-op `init_empty_weights` is provided. `get_sm_count` queries CUDA, so it
is patched to return 148 (B200).
"""

import argparse
import contextlib
import json
import sys
import time
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "epic-kernel_b200"))

from megakernels.llama import LlamaConfig, LlamaForCausalLM, llama_3_2_1b_config  # noqa: E402
from megakernels.model_types import ExtraModelConfig  # noqa: E402
from megakernels.synthetic import seeded_normal, seeded_randint  # noqa: E402

SM_COUNT = 148


def import_reference(ref_root: Path):
    import transformers  # noqa: F401  (before the accelerate stub)

    acc = types.ModuleType("accelerate")
    acc.init_empty_weights = lambda include_buffers=False: contextlib.nullcontext()
    sys.modules["accelerate"] = acc
    # the reference package is also named `megakernels`: load it under its own
    # name after removing ours from the module cache
    for k in [k for k in sys.modules if k == "megakernels" or k.startswith("megakernels.")]:
        sys.modules["ek_" + k] = sys.modules.pop(k)
    sys.path.insert(0, str(ref_root))
    import megakernels.utils as ru

    ru.get_sm_count = lambda device=None: SM_COUNT
    import megakernels.instructions as ri
    import megakernels.demos.latency.scheduler as rs

    ri.get_sm_count = ru.get_sm_count
    rs.get_sm_count = ru.get_sm_count
    import megakernels.mixtral.scheduler as rms
    import megakernels.mixtral.python_vm as rmvm
    import megakernels.mixtral.model as rmm

    rms.get_sm_count = ru.get_sm_count
    import megakernels.llama as rl
    import megakernels.scheduler as rsch
    import megakernels.demos.latency.python_vm as rvm
    import megakernels.generators as rgen
    import megakernels.python_vm as rpy

    return types.SimpleNamespace(llama=rl, sched=rs, base_sched=rsch, vm=rvm, gen=rgen, pyvm=rpy,
                                 mx_sched=rms, mx_vm=rmvm, mx_model=rmm)


def reference_model(ref, mine: LlamaForCausalLM, max_len: int):
    """The reference's LlamaForCausalLM carrying the same weights as `mine`."""
    from transformers import LlamaConfig as HFConfig

    c = mine.config
    hf = HFConfig(
        hidden_size=c.hidden_size, num_hidden_layers=c.num_hidden_layers,
        num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads,
        head_dim=c.head_dim, intermediate_size=c.intermediate_size, vocab_size=c.vocab_size,
        rms_norm_eps=c.rms_norm_eps, rope_theta=c.rope_theta, rope_scaling=c.rope_scaling,
        max_position_embeddings=c.max_position_embeddings, tie_word_embeddings=c.tie_word_embeddings,
    )
    torch.set_default_dtype(torch.bfloat16)
    try:
        ref_model = ref.llama.LlamaForCausalLM(
            hf, ref.llama.ExtraModelConfig(interleave_rope=True, max_len_override=max_len)
        )
    finally:
        torch.set_default_dtype(torch.float32)
    ref_model.requires_grad_(False)
    # undo our interleave to hand the reference checkpoint-order q/k rows
    D = c.head_dim
    inv = torch.empty(D, dtype=torch.long)
    inv[0::2] = torch.arange(D // 2)
    inv[1::2] = torch.arange(D // 2) + D // 2
    undo = torch.argsort(inv)
    qd, kd = c.num_attention_heads * D, c.num_key_value_heads * D
    sp = mine.stacked_params
    for l, layer in enumerate(ref_model.model.layers):
        a, m = layer.self_attn, layer.mlp
        qkv = sp.qkv_proj[l]
        q = qkv[:qd].view(c.num_attention_heads, D, -1)[:, undo].reshape(qd, -1)
        k = qkv[qd : qd + kd].view(c.num_key_value_heads, D, -1)[:, undo].reshape(kd, -1)
        a.q_proj.weight.copy_(q)
        a.k_proj.weight.copy_(k)
        a.v_proj.weight.copy_(qkv[qd + kd :])
        a.o_proj.weight.copy_(sp.o_proj[l])
        m.up_proj.weight.copy_(sp.up_proj[l])
        m.gate_proj.weight.copy_(sp.gate_proj[l])
        m.down_proj.weight.copy_(sp.down_proj[l])
    ref_model.model.embed_tokens.embed_tokens.weight.copy_(mine.model.embed_tokens.embed_tokens.weight)
    ref_model.lm_head.lm_head.weight.copy_(mine.lm_head.lm_head.weight)
    ref_model.model.interleave_rope()
    ref_model.stack_params()
    ref_model.setup_caches()
    assert torch.equal(ref_model.stacked_params.qkv_proj, sp.qkv_proj), "weight transfer mismatch"
    return ref_model


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().copy()


sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def words_of(instructions):
    return [w for ins in instructions for w in (ins.serialize() + [0] * (32 - len(ins.serialize())))]


def run_tiny(ref, out: dict):
    mine = cases.tiny_model()
    ref_model = reference_model(ref, mine, cases.TINY_MAX_LEN)
    # rotary tables: reference (transformers LlamaRotaryEmbedding) vs ours
    rc = ref_model.model.rope_cos[: cases.TINY_MAX_LEN]
    rs = ref_model.model.rope_sin[: cases.TINY_MAX_LEN]
    out["rope_cos_maxdiff"] = float((rc - mine.model.rope_cos).abs().max())
    out["rope_sin_maxdiff"] = float((rs - mine.model.rope_sin).abs().max())
    arrays = {}
    for pos in cases.TINY_POSITIONS:
        sched = ref.sched.LatencyScheduleBuilder.build(ref_model, seq_len=pos)
        g = sched.globs
        cases.fill_kv(g.k_cache, g.v_cache, pos)
        g.hidden_states[:] = cases.step_hidden(g.hidden_size, pos)
        instrs = sched.get_linear_instructions()
        arrays[f"p{pos}_words"] = np.array(words_of(instrs), dtype=np.int32)
        t = time.time()
        ref.pyvm.interpret_with_pyvm(g, instrs, ref.vm.INSTRUCTION_TO_SOLVER)
        print(f"tiny pos {pos}: {len(instrs)} instructions, {time.time() - t:.1f}s")
        for name in ("hidden_states", "post_ln_rope_q", "attn_out", "silu_out", "logits"):
            arrays[f"p{pos}_{name}"] = bf16_bits(getattr(g, name))
        arrays[f"p{pos}_k_row"] = bf16_bits(g.k_cache[:, 0, pos])
        arrays[f"p{pos}_v_row"] = bf16_bits(g.v_cache[:, 0, pos])
        arrays[f"p{pos}_barriers"] = g.barriers.numpy().copy()
        arrays[f"p{pos}_skip_attn_reduction"] = np.array([int(g.skip_attn_reduction)])
    np.savez_compressed(HERE / "llama_tiny_step.npz", **arrays)


def run_1b_greedy(ref, out: dict, prompt_len=128, ntok=64):

    max_len = 256
    mine = LlamaForCausalLM.random_init(
        llama_3_2_1b_config(), ExtraModelConfig(interleave_rope=True, max_len_override=max_len), seed=0)
    ref_model = reference_model(ref, mine, max_len)
    del mine
    prompt = seeded_randint(prompt_len, ref_model.config.vocab_size, seed=0)
    seq_len = prompt_len + ntok
    sched = ref.sched.LatencyScheduleBuilder.build(ref_model, seq_len=seq_len)
    interp = ref.pyvm.PyVM_Interpreter(ref.vm.INSTRUCTION_TO_SOLVER)
    gen = ref.gen.PyVM_Generator(ref_model, interp, sched)
    g = sched.globs
    tokens, margins, saved = [], [], {}
    t0 = time.time()
    cur = int(prompt[0])
    for pos in range(seq_len - 1):
        # PyVM_Generator.run, but keeping the logits for the fixture
        gen.run(torch.tensor([[cur]]), pos_id=pos)
        normed = ref_model.lm_head.input_norm(g.hidden_states)
        logits = ref_model.lm_head.lm_head(normed).reshape(-1)
        top = torch.topk(logits.float(), 2).values
        nxt = int(torch.argmax(logits))
        margins.append(float(top[0] - top[1]))
        if pos in (prompt_len - 1, seq_len - 2):
            saved[f"logits_pos{pos}"] = bf16_bits(logits)
        if pos + 1 < prompt_len:
            cur = int(prompt[pos + 1])
        else:
            tokens.append(nxt)
            cur = nxt
        if pos % 16 == 0:
            print(f"1b pos {pos}: {time.time() - t0:.0f}s", flush=True)
    saved["prompt"] = prompt.numpy()
    saved["greedy_tokens"] = np.array(tokens, dtype=np.int64)
    saved["top2_margin"] = np.array(margins, dtype=np.float32)
    saved["final_hidden"] = bf16_bits(g.hidden_states)
    np.savez_compressed(HERE / "llama1b_decode192.npz", **saved)
    out["1b_seconds_per_token"] = (time.time() - t0) / (seq_len - 1)
    out["1b_threads"] = torch.get_num_threads()


def reference_mixtral(ref, mine, max_len: int):
    """The reference's MixtralForCausalLM carrying the same weights as `mine`."""
    from transformers import MixtralConfig as HFConfig

    c = mine.config
    hf = HFConfig(hidden_size=c.hidden_size, num_hidden_layers=c.num_hidden_layers,
                  num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads,
                  intermediate_size=c.intermediate_size, num_local_experts=c.num_local_experts,
                  num_experts_per_tok=c.num_experts_per_tok, vocab_size=c.vocab_size,
                  rms_norm_eps=c.rms_norm_eps, rope_theta=c.rope_theta,
                  max_position_embeddings=c.max_position_embeddings, tie_word_embeddings=False)
    torch.set_default_dtype(torch.bfloat16)
    try:
        rm = ref.mx_model.MixtralForCausalLM(
            hf, ref.llama.ExtraModelConfig(interleave_rope=True, max_len_override=max_len))
    finally:
        torch.set_default_dtype(torch.float32)
    rm.requires_grad_(False)
    D = c.head_dim
    inv = torch.empty(D, dtype=torch.long)
    inv[0::2] = torch.arange(D // 2)
    inv[1::2] = torch.arange(D // 2) + D // 2
    undo = torch.argsort(inv)
    qd, kd = c.num_attention_heads * D, c.num_key_value_heads * D
    sp = mine.stacked_params
    for l, blk in enumerate(rm.model.layers):
        a, moe = blk.self_attn, blk.moe
        qkv = sp.qkv_proj[l]
        a.q_proj.weight.copy_(qkv[:qd].view(c.num_attention_heads, D, -1)[:, undo].reshape(qd, -1))
        a.k_proj.weight.copy_(qkv[qd : qd + kd].view(c.num_key_value_heads, D, -1)[:, undo].reshape(kd, -1))
        a.v_proj.weight.copy_(qkv[qd + kd :])
        a.o_proj.weight.copy_(sp.o_proj[l])
        moe.gate.weight.copy_(sp.router_weight[l])
        for e, ex in enumerate(moe.experts):
            ex.w1.weight.copy_(sp.expert_gate[l, e])
            ex.w3.weight.copy_(sp.expert_up[l, e])
            ex.w2.weight.copy_(sp.expert_down[l, e])
    rm.model.embed_tokens.embed_tokens.weight.copy_(mine.model.embed_tokens.embed_tokens.weight)
    rm.lm_head.lm_head.weight.copy_(mine.lm_head.lm_head.weight)
    rm.model.interleave_rope()
    rm.stack_params()
    rm.setup_caches()
    assert torch.equal(rm.stacked_params.qkv_proj, sp.qkv_proj), "weight transfer mismatch"
    assert torch.equal(rm.stacked_params.expert_down, sp.expert_down), "expert transfer mismatch"
    return rm


def run_mixtral(ref, out: dict):
    arrays = {}
    models = {}
    for name, pos in cases.MIXTRAL_CASES:
        if name not in models:
            mine = cases.mixtral_model(name)
            models[name] = (mine, reference_mixtral(ref, mine, cases.MIXTRAL_MAX_LEN))
            rc = models[name][1].model.rope_cos[: cases.MIXTRAL_MAX_LEN]
            out[f"mixtral_{name}_rope_cos_maxdiff"] = float((rc - mine.model.rope_cos).abs().max())
        mine, rm = models[name]
        sched = ref.mx_sched.MixtralLatencyScheduleBuilder.build(rm, seq_len=pos)
        g = sched.globs
        cases.fill_kv(g.k_cache, g.v_cache, pos)
        g.hidden_states[:] = cases.step_hidden(g.hidden_size, pos)
        instrs = sched.get_linear_instructions()
        key = f"{name}_p{pos}"
        arrays[f"{key}_words"] = np.array(words_of(instrs), dtype=np.int32)
        t = time.time()
        ref.pyvm.interpret_with_pyvm(g, instrs, ref.mx_vm.INSTRUCTION_TO_SOLVER)
        print(f"mixtral {key}: {len(instrs)} instructions, {time.time() - t:.1f}s", flush=True)
        for n in ("hidden_states", "post_ln_rope_q", "attn_out", "logits", "expert_silu_out",
                  "selected_expert_scores"):
            arrays[f"{key}_{n}"] = bf16_bits(getattr(g, n))
        for n in ("selected_expert_indices", "predicted_expert_indices", "barriers"):
            arrays[f"{key}_{n}"] = getattr(g, n).numpy().copy()
        arrays[f"{key}_k_row"] = bf16_bits(g.k_cache[:, 0, pos])
        arrays[f"{key}_v_row"] = bf16_bits(g.v_cache[:, 0, pos])
    np.savez_compressed(HERE / "mixtral_step.npz", **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--full", action="store_true", help="also run the 192-step Llama-1B case")
    ap.add_argument("--only", default="", help="llama | mixtral (default: both)")
    args = ap.parse_args()
    ref = import_reference(args.reference)
    info_path = HERE / "golden_info.json"
    out = json.loads(info_path.read_text()) if info_path.exists() else {}
    with torch.no_grad():
        if args.only in ("", "llama"):
            run_tiny(ref, out)
            if args.full:
                run_1b_greedy(ref, out)
        if args.only in ("", "mixtral"):
            run_mixtral(ref, out)
    out["generator"] = "tests/golden/make_golden.py"
    out["sm_count"] = SM_COUNT
    info_path.write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
