"""Dense prefill (`LlamaForCausalLM.prefill`, the reference's prefill branch of
megakernels/llama.py:90-133) against the token-by-token decode of the same
prompt: through the CPU oracle (this file's CPU test) and through the GPU
megakernel (the gpu test). The KV rows the prefill appends must be the ones
the decode writes (layer 0 bit-exact on CPU; deeper layers within bf16
rounding), and the last token's logits within 0.1 x std (max) and 0.03 x std
(RMS): the two paths differ only in summation order."""

import pytest
import torch

import cases
from megakernels.demos.latency.scheduler import LatencyScheduleBuilder

PROMPT = 8


def _ids():
    return torch.randint(0, cases.TINY["vocab_size"], (PROMPT,), generator=torch.Generator().manual_seed(3))


def _compare(la, lb, a, b, exact_layer0):
    sd = lb.float().std().item()
    d = (la.float().cpu() - lb.float().cpu()).abs()
    assert d.max().item() <= 0.1 * sd, f"max |dlogit| {d.max().item() / sd:.4f} std"
    assert d.pow(2).mean().sqrt().item() <= 0.03 * sd
    for l in range(a.config.num_hidden_layers):
        for c in range(2):
            x = a.stacked_kv_cache[c][l, 0, :PROMPT].float().cpu()
            y = b.stacked_kv_cache[c][l, 0, :PROMPT].float().cpu()
            if l == 0 and exact_layer0:
                assert torch.equal(x, y), f"layer 0 {'kv'[c]} rows differ"
            else:
                ulp = torch.exp2(torch.floor(torch.log2(y.abs().clamp_min(1e-30))) - 7)
                assert bool(((x - y).abs() <= 4 * ulp + 2e-2 * y.abs().max()).all()), f"layer {l} {'kv'[c]}"


def test_prefill_matches_oracle_decode_cpu():
    from oracle import pyvm

    a, b = cases.tiny_model("cpu"), cases.tiny_model("cpu")
    ids = _ids()
    la = a.prefill(ids, 0)
    s = LatencyScheduleBuilder.build(b, seq_len=PROMPT)
    instrs = s.get_linear_instructions()
    with torch.no_grad():
        for p in range(PROMPT):
            lb, _ = pyvm.pyvm_step(b, s.globs, instrs, int(ids[p]), p)
    _compare(la, lb, a, b, exact_layer0=True)


def test_prefill_then_offset_prefill_equals_one_prefill_cpu():
    """Prefilling in two chunks (positions 0..4, then 5..7 over the cached
    prefix) gives the same cache and logits as one chunk."""
    a, b = cases.tiny_model("cpu"), cases.tiny_model("cpu")
    ids = _ids()
    la = a.prefill(ids, 0)
    b.prefill(ids[:5], 0)
    lb = b.prefill(ids[5:], 5)
    assert torch.equal(a.stacked_kv_cache[0][:, :, :PROMPT], b.stacked_kv_cache[0][:, :, :PROMPT])
    d = (la.float() - lb.float()).abs().max().item()
    assert d <= 0.05 * lb.float().std().item()


@pytest.mark.gpu
def test_prefill_matches_megakernel_decode_gpu():
    import mk_llama
    from megakernels.demos.latency.mk import LatencyMK_Interpreter
    from megakernels.generators import MK_Generator
    from megakernels.scheduler import assign_to_sms, tensorize_instructions

    a, b = cases.tiny_model("cuda"), cases.tiny_model("cuda")
    ids = _ids().cuda()
    la = a.prefill(ids, 0)
    s = LatencyScheduleBuilder.build(b, seq_len=PROMPT + 4)
    tensorize_instructions(s.globs, assign_to_sms("rr", schedule=s))
    gen = MK_Generator(b, LatencyMK_Interpreter(), s)
    for p in range(PROMPT):
        gen.run(ids[p : p + 1].view(1, 1), p)
    torch.cuda.synchronize()
    mk_llama.check()
    _compare(la, s.globs.logits, a, b, exact_layer0=False)
    # decode continues from the prefilled cache as from the decoded one
    ta = int(MK_Generator(a, LatencyMK_Interpreter(), s).prefill(ids, 0))
    assert ta == int(torch.argmax(s.globs.logits)) or abs(
        float(s.globs.logits.float().topk(2).values.diff().abs())) < 0.1
