"""Pin the CPU oracle (oracle/pyvm.py) against the reference interpreter's own
outputs (tests/golden/llama_tiny_step.npz, made by make_golden.py)."""

import numpy as np
import pytest
import torch

import cases
from megakernels.demos.latency.scheduler import LatencyScheduleBuilder
from oracle import pyvm


def from_bits(a):
    return torch.from_numpy(a).view(torch.bfloat16).float()


@pytest.fixture(scope="module")
def tiny():
    return cases.tiny_model()


@pytest.mark.parametrize("pos", cases.TINY_POSITIONS)
def test_oracle_matches_reference_interpreter(tiny, golden_dir, pos):
    gold = np.load(golden_dir / "llama_tiny_step.npz")
    sched = LatencyScheduleBuilder.build(tiny, seq_len=pos)
    g = sched.globs
    cases.fill_kv(g.k_cache, g.v_cache, pos)
    g.hidden_states[:] = cases.step_hidden(g.hidden_size, pos)
    with torch.no_grad():
        pyvm.interpret(g, sched.get_linear_instructions())
    np.testing.assert_array_equal(g.barriers.numpy(), gold[f"p{pos}_barriers"])
    for name in ("hidden_states", "post_ln_rope_q", "attn_out", "silu_out", "logits"):
        mine = getattr(g, name).float()
        ref = from_bits(gold[f"p{pos}_{name}"])
        mism = (mine != ref).float().mean().item()
        # same torch CPU ops in the same order: expect bit equality
        assert mism == 0.0, f"{name}: {mism:.2%} of elements differ"
    np.testing.assert_array_equal(g.k_cache[:, 0, pos].view(torch.int16).numpy(), gold[f"p{pos}_k_row"])
    np.testing.assert_array_equal(g.v_cache[:, 0, pos].view(torch.int16).numpy(), gold[f"p{pos}_v_row"])


def test_rope_tables_match_transformers():
    from transformers import LlamaConfig as HF
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    from megakernels.llama import llama_3_2_1b_config, rope_tables

    c = llama_3_2_1b_config()
    hf = HF(hidden_size=c.hidden_size, num_attention_heads=c.num_attention_heads, head_dim=c.head_dim,
            rope_theta=c.rope_theta, rope_scaling=c.rope_scaling,
            max_position_embeddings=c.max_position_embeddings)
    emb = LlamaRotaryEmbedding(config=hf)
    pos = torch.arange(4096).unsqueeze(0)
    cos_ref, sin_ref = emb(torch.empty(0, dtype=torch.float32), pos)
    cos, sin = rope_tables(c.head_dim, c.rope_theta, c.rope_scaling, 4096)
    assert torch.equal(cos, cos_ref[0]) and torch.equal(sin, sin_ref[0])
