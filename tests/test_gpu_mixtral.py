"""GPU parity of the Mixtral decode megakernel (mk_mixtral -> libek.so).

Against the reference interpreter's outputs (tests/golden/mixtral_step.npz):
router top-k indices bit-exact, barrier counters bit-exact, logits and hidden
within max(2e-2 x std, 2 x noise floor). The floor is the reference
interpreter against itself with a different fp32 summation order
(reordered oracle).
"""

import numpy as np
import pytest
import torch

import cases
from gpu_helpers import _reordered_matvec, assert_logits_within_floor, bf16_from_bits
from megakernels.mixtral.mk import MixtralMK_Interpreter
from megakernels.mixtral.scheduler import MixtralLatencyScheduleBuilder
from megakernels.scheduler import assign_to_sms, tensorize_instructions
from oracle import pyvm, pyvm_mixtral

pytestmark = pytest.mark.gpu


def prepare(model, pos, **kw):
    s = MixtralLatencyScheduleBuilder.build(model, seq_len=pos, **kw)
    g = s.globs
    cases.fill_kv(g.k_cache, g.v_cache, pos)
    g.hidden_states[:] = cases.step_hidden(g.hidden_size, pos).to(g.hidden_states.device)
    return s


def run_gpu(s, mode="rr", **options):
    import mk_mixtral

    g = s.globs
    tensorize_instructions(g, assign_to_sms(mode, schedule=s))
    g.barriers.zero_()
    g.logits.zero_()
    MixtralMK_Interpreter(**options).interpret(g)
    torch.cuda.synchronize()
    mk_mixtral.check()


def run_oracle(s, reorder=False):
    saved = pyvm.matvec
    if reorder:
        pyvm.matvec = _reordered_matvec
        pyvm_mixtral.matvec = _reordered_matvec
    try:
        with torch.no_grad():
            pyvm_mixtral.interpret(s.globs, s.get_linear_instructions())
    finally:
        pyvm.matvec = saved
        pyvm_mixtral.matvec = saved


@pytest.fixture(scope="module")
def golden(golden_dir):
    return np.load(golden_dir / "mixtral_step.npz")


@pytest.fixture(scope="module")
def models():
    return {}


def model(models, name, device):
    key = (name, device)
    if key not in models:
        models[key] = cases.mixtral_model(name, device)
    return models[key]


def close_within_floor(mine, ref, alt, name):
    """Each element within two of its own bf16 ulps plus max(2e-2 x std,
    2 x the reordered oracle's largest error)."""
    mine, ref, alt = (t.detach().float().cpu().reshape(-1) for t in (mine, ref, alt))
    d, f = (mine - ref).abs(), (alt - ref).abs()
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - 7)
    bound = 2 * ulp + max(2e-2 * ref.std().item(), 2 * f.max().item())
    excess = (d - bound).max().item()
    assert excess <= 0, f"{name}: error exceeds bound by {excess} (max error {d.max().item()})"


@pytest.mark.parametrize("name,pos", cases.MIXTRAL_CASES)
def test_mixtral_step_vs_reference(models, golden, name, pos):
    key = f"{name}_p{pos}"
    s = prepare(model(models, name, "cuda"), pos)
    run_gpu(s)
    g = s.globs
    np.testing.assert_array_equal(g.barriers.cpu().numpy(), golden[f"{key}_barriers"])
    np.testing.assert_array_equal(g.selected_expert_indices.cpu().numpy(), golden[f"{key}_selected_expert_indices"])
    alt = prepare(model(models, name, "cpu"), pos)
    run_oracle(alt, reorder=True)
    a = alt.globs
    ref_logits = bf16_from_bits(golden[f"{key}_logits"])
    if ref_logits.float().abs().max() > 0:  # the small config has no LM head (hidden < 2048)
        assert_logits_within_floor(g.logits, ref_logits, a.logits)
    for n in ("hidden_states", "post_ln_rope_q", "attn_out"):
        close_within_floor(getattr(g, n), bf16_from_bits(golden[f"{key}_{n}"]), getattr(a, n), n)
    sel = g.selected_expert_indices.cpu().long()
    close_within_floor(g.expert_silu_out[sel], bf16_from_bits(golden[f"{key}_expert_silu_out"])[sel],
                       a.expert_silu_out[sel], "expert_silu_out")
    close_within_floor(g.selected_expert_scores, bf16_from_bits(golden[f"{key}_selected_expert_scores"]),
                       a.selected_expert_scores, "scores")
    # SpeculativeExpertPredict of the last layer: the same router math on the
    # hidden state entering that layer, so its choice is bit-exact too
    np.testing.assert_array_equal(g.predicted_expert_indices.cpu().numpy(),
                                  golden[f"{key}_predicted_expert_indices"])


@pytest.mark.parametrize("stop", ["qkv", "partial", "oproj", "router", "downproj"])
def test_mixtral_one_layer_stages(models, stop):
    pos = 300
    ref = prepare(model(models, "small", "cpu"), pos, layer_limit=1, stop_after_op=stop)
    s = prepare(model(models, "small", "cuda"), pos, layer_limit=1, stop_after_op=stop)
    run_gpu(s)
    run_oracle(ref)
    assert torch.equal(s.globs.barriers.cpu(), ref.globs.barriers)
    if stop in ("router", "downproj"):
        assert torch.equal(s.globs.selected_expert_indices.cpu(), ref.globs.selected_expert_indices)
    for n in ("post_ln_rope_q", "attn_out", "hidden_states", "expert_silu_out"):
        a, b = getattr(s.globs, n).float().cpu(), getattr(ref.globs, n).float()
        assert (a - b).abs().max().item() <= 2e-2 * max(b.std().item(), 1e-3) + 4e-2 * b.abs().max().item(), n


@pytest.mark.parametrize("mode", ["zz", "dag"])
def test_mixtral_policies_bitwise_identical(models, mode):
    pos = 300
    a = prepare(model(models, "small", "cuda"), pos)
    run_gpu(a, "rr", l2_prefetch_stages=32)
    ref = {n: getattr(a.globs, n).clone() for n in ("hidden_states", "barriers", "expert_silu_out")}
    b = prepare(model(models, "small", "cuda"), pos)
    run_gpu(b, mode)
    for n, t in ref.items():
        assert torch.equal(getattr(b.globs, n), t), n
