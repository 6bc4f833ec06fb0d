"""Mixtral model state for the decode engine: stacked weights, rotary tables,
KV cache.

Attribute layout of `megakernels/mixtral/model.py` in epic-kernel
(`MixtralStackedParams`, :297-306; `stack_params`, :486-565), which the
schedule builder reads: `stacked_params.{qkv_proj, o_proj, attn_ln_weight,
ffn_ln_weight, router_weight [L, E, H], expert_gate / expert_up [L, E, I, H],
expert_down [L, E, H, I]}`, `model.model.rope_cos / rope_sin`,
`model.lm_head.{input_norm.weight, lm_head.weight}`, `stacked_kv_cache`.
head_dim = hidden / num_attention_heads, as the reference computes it.

`random_init` draws N(0, std) weights (norm weights 1). With `host_rng=True`
(default) every tensor comes from `megakernels.synthetic` (numpy PCG64,
identical on every host; used by the parity tests). With `host_rng=False`
the draws use torch's CUDA generator on the target device, because the 46.7 B
parameters of the full model take minutes to draw on a CPU; those weights are
reproducible on the same GPU type and torch version only.
"""

from dataclasses import dataclass

import torch
from torch import Tensor, nn

from megakernels.llama import LlamaEmbeddings, LlamaLMHead, RMSNorm, _Body, interleave_permutation, rope_tables
from megakernels.model_types import ExtraModelConfig
from megakernels.synthetic import seeded_normal


@dataclass
class MixtralConfig:
    hidden_size: int = 4096
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    intermediate_size: int = 14336
    num_local_experts: int = 8
    num_experts_per_tok: int = 2
    vocab_size: int = 32000
    rms_norm_eps: float = 1e-5
    rope_theta: float = 1e6
    rope_scaling: dict | None = None
    max_position_embeddings: int = 32768
    tie_word_embeddings: bool = False
    # set on tensor-parallel shards, whose local head count no longer divides hidden
    head_dim_override: int | None = None

    @property
    def head_dim(self) -> int:
        return self.head_dim_override or self.hidden_size // self.num_attention_heads


@dataclass
class MixtralStackedParams:
    qkv_proj: Tensor
    o_proj: Tensor
    attn_ln_weight: Tensor
    ffn_ln_weight: Tensor
    router_weight: Tensor
    expert_gate: Tensor
    expert_up: Tensor
    expert_down: Tensor


# tensor ids of the synthetic draw: layer l uses 64 l + k
_Q, _K, _V, _O, _ROUTER = 0, 1, 2, 3, 4
_GATE, _UP, _DOWN = 8, 24, 40  # + expert index
_EMBED, _LM = 1_000_000, 1_000_001


class MixtralForCausalLM(nn.Module):
    def __init__(self, config: MixtralConfig, extra_config: ExtraModelConfig | None = None,
                 device="cpu", dtype=torch.bfloat16):
        super().__init__()
        self.config = config
        self.extra_config = extra_config or ExtraModelConfig()
        self.device = torch.device(device)
        self.dtype = dtype
        self.model = _Body(config, dtype)
        self.lm_head = LlamaLMHead(config, dtype)
        self.stacked_params: MixtralStackedParams | None = None
        self.stacked_kv_cache = None

    def max_len(self) -> int:
        return self.extra_config.max_len_override or self.config.max_position_embeddings

    @classmethod
    def random_init(cls, config: MixtralConfig, extra_config: ExtraModelConfig | None = None, seed: int = 0,
                    std: float = 0.02, device="cpu", dtype=torch.bfloat16, host_rng: bool = True,
                    tp: tuple[int, int] | None = None):
        """With `tp=(rank, world)` the model is that rank's tensor-parallel
        shard of the same weights: query/KV heads, expert intermediate rows
        (gate/up rows, down columns) and LM-head vocabulary rows are split
        evenly; router, norms and the embedding are replicated."""
        full = config
        rank, world = tp if tp else (0, 1)
        if world > 1:
            assert full.num_attention_heads % world == 0 and full.num_key_value_heads % world == 0
            assert full.intermediate_size % world == 0 and full.vocab_size % world == 0
            config = MixtralConfig(**{**full.__dict__,
                                      "num_attention_heads": full.num_attention_heads // world,
                                      "num_key_value_heads": full.num_key_value_heads // world,
                                      "intermediate_size": full.intermediate_size // world,
                                      "vocab_size": full.vocab_size // world,
                                      "head_dim_override": full.head_dim})
        m = cls(config, extra_config, device=device, dtype=dtype)
        c = config
        D, H, L, E, I = c.head_dim, c.hidden_size, c.num_hidden_layers, c.num_local_experts, c.intermediate_size
        qd, kd = c.num_attention_heads * D, c.num_key_value_heads * D
        fqd, fkd, fI, fV = full.num_attention_heads * D, full.num_key_value_heads * D, full.intermediate_size, full.vocab_size
        dev = m.device
        gen = None
        if not host_rng:
            gen = torch.Generator(device=dev)
            gen.manual_seed(seed)

        def draw(shape, tid):
            if host_rng:
                return seeded_normal(shape, seed, tid, std, dtype).to(dev)
            return torch.empty(shape, dtype=dtype, device=dev).normal_(0, std, generator=gen)

        def rows(n_full):  # this rank's slice of a split dimension
            n = n_full // world
            return slice(rank * n, (rank + 1) * n)

        # full-shape draws, sliced to this rank's shard (kind from the tensor id)
        def w(shape, tid):
            k = tid % 64 if tid < _EMBED else tid
            if k in (_Q, _K, _V):
                n_full = fqd if k == _Q else fkd
                return draw((n_full, H), tid)[rows(n_full)]
            if k == _O:
                return draw((H, fqd), tid)[:, rows(fqd)].contiguous()
            if _GATE <= k < _DOWN:  # gate and up rows
                return draw((fI, H), tid)[rows(fI)]
            if _DOWN <= k < _DOWN + 16:
                return draw((H, fI), tid)[:, rows(fI)].contiguous()
            if k == _LM:
                return draw((fV, H), tid)[rows(fV)]
            return draw(shape, tid)

        def stacked(shape_fn, tid_fn):
            out = torch.empty((L, E) + shape_fn, dtype=dtype, device=dev)
            for l in range(L):
                for e in range(E):
                    out[l, e] = w(shape_fn, tid_fn(l, e))
            return out

        m.stacked_params = MixtralStackedParams(
            qkv_proj=torch.stack([torch.cat([w((qd, H), 64 * l + _Q), w((kd, H), 64 * l + _K),
                                             w((kd, H), 64 * l + _V)]) for l in range(L)]),
            o_proj=torch.stack([w((H, qd), 64 * l + _O) for l in range(L)]),
            attn_ln_weight=torch.ones(L, H, dtype=dtype, device=dev),
            ffn_ln_weight=torch.ones(L, H, dtype=dtype, device=dev),
            router_weight=torch.stack([w((E, H), 64 * l + _ROUTER) for l in range(L)]),
            expert_gate=stacked((I, H), lambda l, e: 64 * l + _GATE + e),
            expert_up=stacked((I, H), lambda l, e: 64 * l + _UP + e),
            expert_down=stacked((H, I), lambda l, e: 64 * l + _DOWN + e),
        )
        m.model.embed_tokens.embed_tokens.weight.data = draw((fV, H), _EMBED)  # replicated, full vocabulary
        m.lm_head.lm_head.weight.data = w((c.vocab_size, H), _LM)
        m.lm_head.input_norm.weight.data = m.lm_head.input_norm.weight.data.to(dev)
        cos, sin = rope_tables(D, c.rope_theta, c.rope_scaling, m.max_len())
        m.model.rope_cos, m.model.rope_sin = cos.to(dev), sin.to(dev)
        if m.extra_config.interleave_rope:
            perm = interleave_permutation(D).to(dev)
            m.model.rope_cos = m.model.rope_cos[..., perm].contiguous()
            m.model.rope_sin = m.model.rope_sin[..., perm].contiguous()
            heads = c.num_attention_heads + c.num_key_value_heads
            rows = (perm.unsqueeze(0) + D * torch.arange(heads, device=dev).unsqueeze(1)).reshape(-1)
            qkv = m.stacked_params.qkv_proj
            qkv[:, : heads * D] = qkv[:, rows]
        shape = (L, m.extra_config.max_batch_size, m.max_len(), c.num_key_value_heads, D)
        k = torch.zeros(shape, dtype=dtype, device=dev)
        m.stacked_kv_cache = (k, torch.zeros_like(k))
        return m
