"""Mixtral: our scheduler and CPU oracle against the reference's own outputs
(tests/golden/mixtral_step.npz, from the reference's Mixtral interpreter)."""

import numpy as np
import pytest
import torch

import cases
from megakernels.mixtral.scheduler import MixtralLatencyScheduleBuilder
from oracle import pyvm_mixtral


def words(instrs):
    out = []
    for ins in instrs:
        w = ins.serialize()
        out.extend(w + [0] * (32 - len(w)))
    return np.array(out, dtype=np.int32)


@pytest.fixture(scope="module")
def golden(golden_dir):
    return np.load(golden_dir / "mixtral_step.npz")


@pytest.fixture(scope="module")
def models():
    return {}


def model(models, name):
    if name not in models:
        models[name] = cases.mixtral_model(name)
    return models[name]


@pytest.mark.parametrize("name,pos", cases.MIXTRAL_CASES)
def test_mixtral_oracle_matches_reference(models, golden, name, pos):
    m = model(models, name)
    key = f"{name}_p{pos}"
    sched = MixtralLatencyScheduleBuilder.build(m, seq_len=pos)
    instrs = sched.get_linear_instructions()
    np.testing.assert_array_equal(words(instrs), golden[f"{key}_words"])
    g = sched.globs
    cases.fill_kv(g.k_cache, g.v_cache, pos)
    g.hidden_states[:] = cases.step_hidden(g.hidden_size, pos)
    with torch.no_grad():
        pyvm_mixtral.interpret(g, instrs)
    np.testing.assert_array_equal(g.barriers.numpy(), golden[f"{key}_barriers"])
    np.testing.assert_array_equal(g.selected_expert_indices.numpy(), golden[f"{key}_selected_expert_indices"])
    np.testing.assert_array_equal(g.predicted_expert_indices.numpy(), golden[f"{key}_predicted_expert_indices"])
    for n in ("hidden_states", "post_ln_rope_q", "attn_out", "logits", "expert_silu_out", "selected_expert_scores"):
        ref = torch.from_numpy(golden[f"{key}_{n}"]).view(torch.bfloat16)
        assert torch.equal(getattr(g, n).reshape(ref.shape), ref), n
