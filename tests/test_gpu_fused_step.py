"""The fused token step of the Llama engine (embedding gather and argmax
inside the megakernel) against the unfused path on the same model: identical
logits and hidden state, and the output token equal to torch.argmax of the
logits (first index on ties)."""

import pytest
import torch

import cases
from megakernels.demos.latency.mk import LatencyMK_Interpreter
from megakernels.demos.latency.scheduler import LatencyScheduleBuilder
from megakernels.generators import MK_Generator
from megakernels.scheduler import assign_to_sms, tensorize_instructions

pytestmark = pytest.mark.gpu

POS = 300


@pytest.fixture(scope="module")
def setup():
    torch.cuda.set_device(0)
    model = cases.tiny_model("cuda")
    sched = LatencyScheduleBuilder.build(model, seq_len=POS)
    cases.fill_kv(sched.globs.k_cache, sched.globs.v_cache, POS)
    tensorize_instructions(sched.globs, assign_to_sms("rr", schedule=sched))
    return model, sched


def unfused_step(model, sched, token):
    g = sched.globs
    emb = model.model.embed_tokens.embed_tokens.weight
    g.hidden_states[:] = emb[token]
    g.barriers.zero_()
    g.logits.zero_()
    g.pos_id = POS
    LatencyMK_Interpreter().interpret(g)
    torch.cuda.synchronize()
    return g.logits.clone(), g.hidden_states.clone(), g.barriers.clone()


def fused_step(model, sched, token):
    g = sched.globs
    g.hidden_states.fill_(float("nan"))  # must not be read
    g.logits.fill_(float("nan"))
    gen = MK_Generator(model, LatencyMK_Interpreter(), sched)
    assert gen._fused_step()
    out = gen.run(torch.tensor([[token]], device="cuda"), POS)
    torch.cuda.synchronize()
    return g.logits.clone(), g.hidden_states.clone(), g.barriers.clone(), int(out)


@pytest.mark.parametrize("token", [0, 17, 4095])
def test_fused_step_matches_unfused(setup, token):
    import mk_llama

    model, sched = setup
    lu, hu, bu = unfused_step(model, sched, token)
    lf, hf, bf, tok = fused_step(model, sched, token)
    mk_llama.check()
    assert torch.equal(bu, bf)
    assert torch.equal(hu, hf)
    assert torch.equal(lu, lf)
    assert tok == int(torch.argmax(lu))


def test_fused_argmax_takes_first_of_tied_rows(setup):
    import mk_llama

    model, sched = setup
    lm = model.lm_head.lm_head.weight
    saved = lm.data.clone()
    try:
        # rows 1234 and 77 set to twice the row of the (positive) largest
        # logit: their logits tie as the new maximum, and the earlier row must win
        l0, _, _ = unfused_step(model, sched, 5)
        best = int(torch.argmax(l0))
        assert l0[best] > 0
        lm.data[1234] = saved[best] * 2
        lm.data[77] = saved[best] * 2
        lu, _, _ = unfused_step(model, sched, 5)
        lf, _, _, tok = fused_step(model, sched, 5)
        mk_llama.check()
        assert torch.equal(lu, lf)
        assert lu[77] == lu[1234] == lu.max()
        assert tok == int(torch.argmax(lu)) == 77
    finally:
        lm.data.copy_(saved)


def test_fused_steps_in_a_row(setup):
    """Consecutive fused steps (the output buffer alternates) follow the
    unfused greedy stream."""
    import mk_llama

    model, sched = setup
    gen = MK_Generator(model, LatencyMK_Interpreter(), sched)
    tok = torch.tensor([[3]], device="cuda")
    ref = 3
    for i in range(4):
        lu, _, _ = unfused_step(model, sched, ref)
        ref = int(torch.argmax(lu))
        tok = gen.run(tok, POS).view(1, 1)
        torch.cuda.synchronize()
        assert int(tok) == ref, f"step {i}"
    mk_llama.check()
