"""Llama-3.2-1B (full size, random init) on the GPU engine.

- One step at KV lengths 128 / 2048 / 4096 / 16384 (1 / 9 / 16 / 18 attention
  partitions per KV head) against the CPU oracle on identical inputs, within
  the noise-floor bound; the measured errors are recorded (record_parity).
- 192 steps (128 teacher-forced prompt tokens, then 64 greedy tokens) against
  the reference interpreter's own token stream (tests/golden/llama1b_decode192.npz).
"""

import numpy as np
import pytest
import torch

import cases
from gpu_helpers import (
    LOGIT_TOL, assert_logits_within_floor, bf16_from_bits, noise_floor, prepare, record_parity, run_gpu,
)
from megakernels.demos.latency.mk import LatencyMK_Interpreter
from megakernels.demos.latency.scheduler import LatencyScheduleBuilder
from megakernels.generators import MK_Generator
from megakernels.llama import LlamaForCausalLM, llama_3_2_1b_config
from megakernels.model_types import ExtraModelConfig
from megakernels.scheduler import assign_to_sms, tensorize_instructions

pytestmark = pytest.mark.gpu


# KV lengths of the sweep: 128 runs one partition per KV head (no reduction
# instructions), 2048 nine, 4096 sixteen, 16384 the cap of eighteen (the longest
# reduction list; megakernels/demos/latency/scheduler.py:25-37 of epic-kernel).
@pytest.mark.parametrize("kv", [128, 2048, 4096, 16384])
def test_1b_step_vs_oracle(kv):
    pos = kv - 1
    cfg = llama_3_2_1b_config()
    extra = ExtraModelConfig(interleave_rope=True, max_len_override=kv + 64)
    cpu = LlamaForCausalLM.random_init(cfg, extra, seed=0)
    hidden = cases.step_hidden(cfg.hidden_size, pos)
    ref, alt = noise_floor(cpu, pos, hidden)
    del cpu
    gpu_model = LlamaForCausalLM.random_init(cfg, extra, seed=0, device="cuda")
    s = prepare(gpu_model, pos, hidden)
    assert s.globs.skip_attn_reduction == (kv <= 256)
    run_gpu(s)
    import mk_llama

    mk_llama.check()
    assert torch.equal(s.globs.barriers.cpu(), ref.globs.barriers)
    mx, rms = assert_logits_within_floor(s.globs.logits, ref.globs.logits, alt.globs.logits)
    sd = ref.globs.logits.float().std().item()
    fl = (alt.globs.logits.float() - ref.globs.logits.float()).abs()
    record_parity(f"llama-1b kv{kv} one step", max_over_std=mx, rms_over_std=rms,
                  floor_max_over_std=fl.max().item() / sd, floor_rms_over_std=fl.pow(2).mean().sqrt().item() / sd,
                  literal_bar=LOGIT_TOL, meets_literal_bar=mx <= LOGIT_TOL)
    top = torch.topk(ref.globs.logits.float(), 2).values
    if (top[0] - top[1]).item() > 2 * fl.max().item():  # decidable top token
        assert int(s.globs.logits.argmax()) == int(ref.globs.logits.argmax())


# The reference interpreter re-run with another (equally valid) fp32 summation
# order disagrees with itself by up to 0.117 in the Llama-1B logits, and its
# free-running greedy stream leaves the reference's at generated token 20,
# where the reference's top-2 margin is 0.078. Steps whose reference margin is
# below this bound are therefore not decidable by any implementation that does
# not replicate the CPU's summation order.
NEAR_TIE = 0.125


def _decode(gen, model, prompt, forced, total):
    """Run `total` decode steps. The input at position pos is the prompt token,
    else forced[pos - len(prompt) + 1] if given, else our previous output."""
    outs = []
    cur = int(prompt[0])
    for pos in range(total):
        out = int(gen.run(torch.tensor([[cur]], device="cuda"), pos))
        outs.append(out)
        if pos + 1 < len(prompt):
            cur = int(prompt[pos + 1])
        elif forced is not None:
            cur = int(forced[pos + 1 - len(prompt)])
        else:
            cur = out
    return outs


def test_1b_greedy_tokens_match_reference(golden_dir):
    path = golden_dir / "llama1b_decode192.npz"
    if not path.exists():
        pytest.skip("llama1b_decode192.npz not generated")
    gold = np.load(path)
    prompt = gold["prompt"]
    expected = gold["greedy_tokens"]
    margins = gold["top2_margin"]
    P, N = len(prompt), len(expected)
    model = LlamaForCausalLM.random_init(
        llama_3_2_1b_config(), ExtraModelConfig(interleave_rope=True, max_len_override=256),
        seed=0, device="cuda")
    sched = LatencyScheduleBuilder.build(model, seq_len=P + N)
    tensorize_instructions(sched.globs, assign_to_sms("rr", schedule=sched))
    gen = MK_Generator(model, LatencyMK_Interpreter(), sched)
    import mk_llama

    # teacher-forced: the reference's own tokens are fed back; every decidable
    # step must produce the reference's token
    outs = _decode(gen, model, prompt, expected, P + N - 1)
    mk_llama.check()
    gen_margins = margins[P - 1 :]
    ours = outs[P - 1 :]
    wrong = [i for i in range(N) if ours[i] != expected[i] and gen_margins[i] >= NEAR_TIE]
    assert not wrong, f"teacher-forced step {wrong[0]}: {ours[wrong[0]]} vs {expected[wrong[0]]}"
    decidable = int((gen_margins >= NEAR_TIE).sum())
    assert decidable >= N // 2

    # free-running: the agreement length with the reference's stream, next to
    # that of the reference interpreter re-run with another fp32 summation
    # order (tests/golden/make_alt_greedy.py)
    model.stacked_kv_cache[0].zero_()
    model.stacked_kv_cache[1].zero_()
    free = _decode(gen, model, prompt, None, P + N - 1)[P - 1 :]
    agree = next((i for i in range(N) if free[i] != expected[i]), N)
    alt_path = golden_dir / "llama1b_alt_greedy.npz"
    alt_agree = None
    if alt_path.exists():
        alt = np.load(alt_path)["alt_greedy_tokens"]
        alt_agree = next((i for i in range(N) if alt[i] != expected[i]), N)
    ties = [i for i in range(N) if gen_margins[i] < NEAR_TIE]
    first_tie = ties[0] if ties else N
    record_parity("llama-1b greedy 64 tokens", teacher_forced_decidable=decidable,
                  teacher_forced_wrong=len(wrong), free_running_agree=agree,
                  reordered_oracle_agree=alt_agree, first_near_tie=first_tie)
    # Steps 2 and 5 of this stream have reference top-2 margins of 0.016, far
    # below the 0.1 disagreement of two valid summation orders: which side of
    # them a stream falls on is chance. The hard bar is the first near-tie;
    # both agreement lengths are recorded.
    assert agree >= first_tie, f"free-running stream leaves the reference at {agree} (first near-tie {first_tie})"


def test_3b_step_kv2048_vs_oracle():
    """Llama-3.2-3B (head_dim 128, 3 query heads per KV head, 8 down-proj
    column splits) one step at KV length 2048 against the CPU oracle."""
    from megakernels.llama import llama_3_2_3b_config

    pos = 2047
    cfg = llama_3_2_3b_config()
    extra = ExtraModelConfig(interleave_rope=True, max_len_override=2112)
    cpu = LlamaForCausalLM.random_init(cfg, extra, seed=0)
    hidden = cases.step_hidden(cfg.hidden_size, pos)
    ref, alt = noise_floor(cpu, pos, hidden)
    del cpu
    gpu_model = LlamaForCausalLM.random_init(cfg, extra, seed=0, device="cuda")
    s = prepare(gpu_model, pos, hidden)
    assert s.globs.matvec_reduction_size == 1024
    run_gpu(s)
    import mk_llama

    mk_llama.check()
    assert torch.equal(s.globs.barriers.cpu(), ref.globs.barriers)
    mx, rms = assert_logits_within_floor(s.globs.logits, ref.globs.logits, alt.globs.logits)
    sd = ref.globs.logits.float().std().item()
    fl = (alt.globs.logits.float() - ref.globs.logits.float()).abs()
    record_parity("llama-3b kv2048 one step", max_over_std=mx, rms_over_std=rms,
                  floor_max_over_std=fl.max().item() / sd, floor_rms_over_std=fl.pow(2).mean().sqrt().item() / sd,
                  literal_bar=LOGIT_TOL, meets_literal_bar=mx <= LOGIT_TOL)
