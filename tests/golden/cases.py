"""Seeded inputs shared by the golden-fixture generator and the tests.

Everything is drawn with `megakernels.synthetic` (numpy PCG64), so the build
container and the GPU host produce identical bits.
"""

import torch

from megakernels.llama import LLAMA3_ROPE_SCALING, LlamaConfig, LlamaForCausalLM
from megakernels.model_types import ExtraModelConfig
from megakernels.mixtral.model import MixtralConfig, MixtralForCausalLM
from megakernels.synthetic import seeded_normal

# 1B-width, 2-layer, 4096-vocab Llama: small enough for the CPU interpreter,
# wide enough for the reference scheduler's one-block-per-SM assertions.
TINY = dict(
    hidden_size=2048, num_hidden_layers=2, num_attention_heads=32, num_key_value_heads=8,
    head_dim=64, intermediate_size=8192, vocab_size=4096, rope_theta=500000.0,
    rope_scaling=dict(LLAMA3_ROPE_SCALING), max_position_embeddings=131072,
)
TINY_MAX_LEN = 1024
TINY_POSITIONS = (5, 300, 777)

KV_SEED = 1
POISON_SEED = 2
HIDDEN_SEED = 3


def tiny_model(device="cpu") -> LlamaForCausalLM:
    return LlamaForCausalLM.random_init(
        LlamaConfig(**TINY), ExtraModelConfig(interleave_rope=True, max_len_override=TINY_MAX_LEN),
        seed=0, device=device,
    )


def fill_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, pos: int, poison: bool = True):
    """Rows [0, pos) ~ N(0, 1) (seed 1); rows >= pos ~ N(0, 100^2) (seed 2) so
    that a read past the valid range shows up (diff_test.py:129-132 of the
    reference). Caches are [L, 1, T, Hkv, D]."""
    L, B, T, H, D = k_cache.shape
    for i, c in enumerate((k_cache, v_cache)):
        c[:, :, :pos] = seeded_normal((L, B, pos, H, D), KV_SEED, 10 * pos + i).to(c.device)
        if poison and pos < T:
            c[:, :, pos:] = seeded_normal((L, B, T - pos, H, D), POISON_SEED, 10 * pos + i, std=100.0).to(c.device)


def step_hidden(hidden_size: int, pos: int) -> torch.Tensor:
    return seeded_normal((hidden_size,), HIDDEN_SEED, pos)


# Mixtral: FakeModel-like small dims (as the reference's test_mixtral_mk.py),
# and full-width layers (hidden 4096, 8 experts x 14336) with a small vocab.
MIXTRAL_SMALL = dict(hidden_size=512, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                     intermediate_size=1024, num_local_experts=4, num_experts_per_tok=2, vocab_size=256,
                     rope_theta=1e6, max_position_embeddings=32768)
MIXTRAL_WIDE = dict(hidden_size=4096, num_hidden_layers=2, num_attention_heads=32, num_key_value_heads=8,
                    intermediate_size=14336, num_local_experts=8, num_experts_per_tok=2, vocab_size=4096,
                    rope_theta=1e6, max_position_embeddings=32768)
MIXTRAL_MAX_LEN = 1024
MIXTRAL_CASES = (("small", 5), ("small", 300), ("wide", 777))


def mixtral_model(name: str, device="cpu"):
    cfg = MixtralConfig(**(MIXTRAL_SMALL if name == "small" else MIXTRAL_WIDE))
    return MixtralForCausalLM.random_init(
        cfg, ExtraModelConfig(interleave_rope=True, max_len_override=MIXTRAL_MAX_LEN), seed=0, device=device)


def fill_kv_shard(k_cache, v_cache, pos: int, rank: int, world: int):
    """fill_kv for a tensor-parallel shard: the full-model KV draws, sliced to
    this rank's KV heads."""
    L, B, T, h, D = k_cache.shape
    full_k = torch.zeros(L, B, T, h * world, D, dtype=k_cache.dtype)
    full_v = torch.zeros_like(full_k)
    fill_kv(full_k, full_v, pos)
    k_cache.copy_(full_k[:, :, :, rank * h : (rank + 1) * h])
    v_cache.copy_(full_v[:, :, :, rank * h : (rank + 1) * h])


def mixtral_shard(name: str, rank: int, world: int, device="cpu"):
    cfg = MixtralConfig(**(MIXTRAL_SMALL if name == "small" else MIXTRAL_WIDE))
    return MixtralForCausalLM.random_init(
        cfg, ExtraModelConfig(interleave_rope=True, max_len_override=MIXTRAL_MAX_LEN), seed=0, device=device,
        tp=(rank, world))
