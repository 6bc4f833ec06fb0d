"""Mixtral tensor parallel on 2, 4 and 8 GPUs (each case skipped when the box
has fewer GPUs; the small config only splits in two): every rank holds a
shard, the hidden state is all-reduced inside the megakernel over NVLink, and
the result must match the reference interpreter's single-GPU output (router
indices bit-exact, logits and hidden within the noise-floor bound), be
bit-identical on all ranks, and stay so over consecutive launches."""

import os
import sys
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from gpu_helpers import assert_logits_within_floor, bf16_from_bits

pytestmark = pytest.mark.gpu

def _worker(rank, world, name, pos, tmp, paths):
    sys.path[:0] = paths
    import mk_mixtral
    from megakernels.mixtral.scheduler import MixtralLatencyScheduleBuilder
    from megakernels.mixtral.tp import MixtralTPMK_Interpreter, setup_tensor_parallel
    from megakernels.scheduler import assign_to_sms, tensorize_instructions

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"file://{tmp}/init", rank=rank, world_size=world)
    try:
        model = cases.mixtral_shard(name, rank, world, device=f"cuda:{rank}")
        sched = MixtralLatencyScheduleBuilder.build(model, seq_len=pos)
        g = sched.globs
        setup_tensor_parallel(g, rank, world)
        tensorize_instructions(g, assign_to_sms("rr", schedule=sched))
        interp = MixtralTPMK_Interpreter(timeout_ns=2_000_000_000)
        outs = []
        for step in range(2):
            cases.fill_kv_shard(g.k_cache, g.v_cache, pos, rank, world)
            g.hidden_states[:] = cases.step_hidden(g.hidden_size, pos).cuda()
            g.barriers.zero_()
            g.logits.zero_()
            dist.barrier()
            interp.interpret(g)
            torch.cuda.synchronize()
            mk_mixtral.check(rank)
            outs.append({"hidden": g.hidden_states.cpu().clone(), "logits": g.logits.cpu().clone(),
                         "sel": g.selected_expert_indices.cpu().clone()})
            dist.barrier()
        torch.save(outs, f"{tmp}/rank{rank}.pt")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,pos,world", [("small", 300, 2), ("wide", 777, 2), ("wide", 777, 4), ("wide", 777, 8)])
def test_mixtral_tp_matches_single_gpu_reference(golden_dir, name, pos, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    WORLD = world
    from oracle import pyvm, pyvm_mixtral
    from gpu_helpers import _reordered_matvec
    from megakernels.mixtral.scheduler import MixtralLatencyScheduleBuilder

    gold = np.load(golden_dir / "mixtral_step.npz")
    key = f"{name}_p{pos}"
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_worker, args=(WORLD, name, pos, tmp, list(sys.path[:6])), nprocs=WORLD, join=True)
        res = [torch.load(f"{tmp}/rank{r}.pt") for r in range(WORLD)]
    for step in range(2):
        for r in range(1, WORLD):  # all ranks hold the same state
            assert torch.equal(res[r][step]["hidden"], res[0][step]["hidden"])
            assert torch.equal(res[r][step]["logits"], res[0][step]["logits"])
        assert torch.equal(res[0][step]["hidden"], res[0][0]["hidden"])  # launch after launch
        np.testing.assert_array_equal(res[0][step]["sel"].numpy(), gold[f"{key}_selected_expert_indices"])
    # noise floor: the reference interpreter with another summation order
    alt = MixtralLatencyScheduleBuilder.build(cases.mixtral_model(name), seq_len=pos)
    cases.fill_kv(alt.globs.k_cache, alt.globs.v_cache, pos)
    alt.globs.hidden_states[:] = cases.step_hidden(alt.globs.hidden_size, pos)
    saved = pyvm.matvec
    pyvm.matvec = pyvm_mixtral.matvec = _reordered_matvec
    try:
        with torch.no_grad():
            pyvm_mixtral.interpret(alt.globs, alt.get_linear_instructions())
    finally:
        pyvm.matvec = pyvm_mixtral.matvec = saved
    ref_logits = bf16_from_bits(gold[f"{key}_logits"])
    if ref_logits.float().abs().max() > 0:
        assert_logits_within_floor(res[0][0]["logits"], ref_logits, alt.globs.logits)
    ref_h = bf16_from_bits(gold[f"{key}_hidden_states"]).float()
    d = (res[0][0]["hidden"].float() - ref_h).abs()
    f = (alt.globs.hidden_states.float() - ref_h).abs()
    ulp = torch.exp2(torch.floor(torch.log2(ref_h.abs().clamp_min(1e-30))) - 7)
    assert bool((d <= 2 * ulp + max(2e-2 * ref_h.std().item(), 2 * f.max().item())).all())
