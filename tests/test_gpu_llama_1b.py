"""Llama-3.2-1B (full size, random init) on the GPU engine.

- One step at KV length 2048 (9 attention partitions per KV head) against the
  CPU oracle on identical inputs, within the noise-floor bound.
- 192 steps (128 teacher-forced prompt tokens, then 64 greedy tokens) against
  the reference interpreter's own token stream (tests/golden/llama1b_decode192.npz).
"""

import numpy as np
import pytest
import torch

import cases
from gpu_helpers import assert_logits_within_floor, bf16_from_bits, noise_floor, prepare, run_gpu
from megakernels.demos.latency.mk import LatencyMK_Interpreter
from megakernels.demos.latency.scheduler import LatencyScheduleBuilder
from megakernels.generators import MK_Generator
from megakernels.llama import LlamaForCausalLM, llama_3_2_1b_config
from megakernels.model_types import ExtraModelConfig
from megakernels.scheduler import assign_to_sms, tensorize_instructions

pytestmark = pytest.mark.gpu


def test_1b_step_kv2048_vs_oracle():
    pos = 2047
    cfg = llama_3_2_1b_config()
    extra = ExtraModelConfig(interleave_rope=True, max_len_override=2304)
    cpu = LlamaForCausalLM.random_init(cfg, extra, seed=0)
    hidden = cases.step_hidden(cfg.hidden_size, pos)
    ref, alt = noise_floor(cpu, pos, hidden)
    gpu_model = LlamaForCausalLM.random_init(cfg, extra, seed=0, device="cuda")
    s = prepare(gpu_model, pos, hidden)
    assert not s.globs.skip_attn_reduction
    run_gpu(s)
    import mk_llama

    mk_llama.check()
    assert torch.equal(s.globs.barriers.cpu(), ref.globs.barriers)
    mx, rms = assert_logits_within_floor(s.globs.logits, ref.globs.logits, alt.globs.logits)
    print(f"1B kv2048 logits: max/std {mx:.4f} rms/std {rms:.4f}")
    assert int(s.globs.logits.argmax()) == int(ref.globs.logits.argmax())


def test_1b_greedy_tokens_match_reference(golden_dir):
    path = golden_dir / "llama1b_decode192.npz"
    if not path.exists():
        pytest.skip("llama1b_decode192.npz not generated")
    gold = np.load(path)
    prompt = torch.from_numpy(gold["prompt"])
    expected = gold["greedy_tokens"]
    margins = gold["top2_margin"]
    prompt_len, ntok = len(prompt), len(expected)
    model = LlamaForCausalLM.random_init(
        llama_3_2_1b_config(), ExtraModelConfig(interleave_rope=True, max_len_override=256),
        seed=0, device="cuda")
    sched = LatencyScheduleBuilder.build(model, seq_len=prompt_len + ntok)
    tensorize_instructions(sched.globs, assign_to_sms("rr", schedule=sched))
    gen = MK_Generator(model, LatencyMK_Interpreter(), sched)
    toks = []
    cur = int(prompt[0])
    for pos in range(prompt_len + ntok - 1):
        out = gen.run(torch.tensor([[cur]], device="cuda"), pos)
        if pos + 1 < prompt_len:
            cur = int(prompt[pos + 1])
        else:
            cur = int(out)
            toks.append(cur)
    import mk_llama

    mk_llama.check()
    mism = [i for i, (a, b) in enumerate(zip(toks, expected)) if a != b]
    first = mism[0] if mism else None
    assert not mism, (f"greedy tokens differ first at step {first}: {toks[first]} vs {expected[first]} "
                      f"(reference top-2 margin there {margins[prompt_len - 1 + first]:.4f})")
