"""Llama model state for the decode engine: weights, rotary tables, KV cache.

This mirrors the attribute layout of `megakernels/llama.py` in epic-kernel,
because the schedule builders read these attributes directly:
- `model.stacked_params.{qkv_proj, o_proj, attn_ln_weight, mlp_ln_weight,
  up_proj, gate_proj, down_proj}` are stacked on a leading layer axis
  (`llama.py:713-777`). `qkv_proj[l]` is the q, k and v weights concatenated on
  the row axis.
- `model.model.rope_cos / rope_sin` are fp32 `[max_len, head_dim]` tables.
- `model.lm_head.input_norm.weight` and `model.lm_head.lm_head.weight`.
- `model.stacked_kv_cache` is `(k, v)`, each `[L, 1, max_len, Hkv, D]` bf16
  (`llama.py:552-574`).
- `model.model.embed_tokens(batch_state)` is the token embedding.

With `interleave_rope` (`llama.py:453-475`), rows of q and k are permuted
inside each head so that rotary pairs (i, i + D/2) sit at (2i, 2i + 1). The
tables are permuted the same way, which lets a kernel rotate adjacent pairs.

Weights come from `random_init` (seeded, see `megakernels.synthetic`),
because this engine's configs are random-init architectures. Loading
checkpoints is not part of the decode path.
"""

from dataclasses import dataclass, field
import math

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from megakernels.model_types import BatchState, ExtraModelConfig
from megakernels.synthetic import seeded_normal


@dataclass
class LlamaConfig:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    vocab_size: int
    head_dim: int | None = None
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None
    max_position_embeddings: int = 131072
    tie_word_embeddings: bool = True

    def __post_init__(self):
        if self.head_dim is None:
            self.head_dim = self.hidden_size // self.num_attention_heads


LLAMA3_ROPE_SCALING = {
    "rope_type": "llama3",
    "factor": 32.0,
    "low_freq_factor": 1.0,
    "high_freq_factor": 4.0,
    "original_max_position_embeddings": 8192,
}


def llama_3_2_1b_config(**overrides) -> LlamaConfig:
    cfg = dict(
        hidden_size=2048,
        num_hidden_layers=16,
        num_attention_heads=32,
        num_key_value_heads=8,
        head_dim=64,
        intermediate_size=8192,
        vocab_size=128256,
        rms_norm_eps=1e-5,
        rope_theta=500000.0,
        rope_scaling=dict(LLAMA3_ROPE_SCALING),
        max_position_embeddings=131072,
        tie_word_embeddings=True,
    )
    cfg.update(overrides)
    return LlamaConfig(**cfg)


def llama_3_2_3b_config(**overrides) -> LlamaConfig:
    cfg = dict(
        hidden_size=3072,
        num_hidden_layers=28,
        num_attention_heads=24,
        num_key_value_heads=8,
        head_dim=128,
        intermediate_size=8192,
        vocab_size=128256,
        rms_norm_eps=1e-5,
        rope_theta=500000.0,
        rope_scaling=dict(LLAMA3_ROPE_SCALING),
        max_position_embeddings=131072,
        tie_word_embeddings=True,
    )
    cfg.update(overrides)
    return LlamaConfig(**cfg)


def rope_inv_freq(head_dim: int, theta: float, scaling: dict | None) -> Tensor:
    """Rotary inverse frequencies (fp32), with the llama3 long-context rescale.

    llama3 rule: wavelengths longer than original_len / low_freq_factor are
    divided by `factor`, wavelengths shorter than original_len /
    high_freq_factor are kept, and the band in between blends the two with
    weight (original_len / wavelength - low) / (high - low).
    """
    exponents = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
    inv_freq = 1.0 / (theta**exponents)
    if scaling is None or scaling.get("rope_type", scaling.get("type")) in (None, "default"):
        return inv_freq
    assert scaling.get("rope_type", scaling.get("type")) == "llama3", scaling
    factor = scaling["factor"]
    low = scaling["low_freq_factor"]
    high = scaling["high_freq_factor"]
    orig = scaling["original_max_position_embeddings"]
    wavelen = 2 * math.pi / inv_freq
    scaled = torch.where(wavelen > orig / low, inv_freq / factor, inv_freq)
    blend = (orig / wavelen - low) / (high - low)
    blended = (1 - blend) * scaled / factor + blend * scaled
    in_band = ~(wavelen < orig / high) * ~(wavelen > orig / low)
    return torch.where(in_band, blended, scaled)


def rope_tables(head_dim: int, theta: float, scaling: dict | None, num_positions: int):
    """fp32 cos/sin `[num_positions, head_dim]`, half-split layout (i, i + D/2
    share a frequency)."""
    inv_freq = rope_inv_freq(head_dim, theta, scaling)
    pos = torch.arange(num_positions, dtype=torch.int64).float()
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def interleave_permutation(head_dim: int) -> Tensor:
    """Row order that puts element i at 2i and element i + D/2 at 2i + 1."""
    half = head_dim // 2
    idx = torch.empty(head_dim, dtype=torch.long)
    idx[0::2] = torch.arange(half)
    idx[1::2] = torch.arange(half) + half
    return idx


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float, dtype=torch.bfloat16):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size, dtype=dtype), requires_grad=False)

    def forward(self, x: Tensor) -> Tensor:
        in_dtype = x.dtype
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * xf.to(in_dtype)


class LlamaEmbeddings(nn.Module):
    def __init__(self, vocab_size: int, hidden_size: int, dtype=torch.bfloat16):
        super().__init__()
        self.embed_tokens = nn.Embedding(vocab_size, hidden_size, dtype=dtype)
        self.embed_tokens.weight.requires_grad_(False)

    def forward(self, batch_state: BatchState) -> BatchState:
        batch_state.hidden_states = self.embed_tokens(batch_state.input_ids)
        return batch_state


class LlamaLMHead(nn.Module):
    """Final RMSNorm + vocabulary projection + argmax (the reference's
    `LlamaLMHead`, `llama.py:369-403`)."""

    def __init__(self, config: LlamaConfig, dtype=torch.bfloat16):
        super().__init__()
        self.input_norm = RMSNorm(config.hidden_size, config.rms_norm_eps, dtype)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False, dtype=dtype)
        self.lm_head.weight.requires_grad_(False)

    def forward(self, batch_state: BatchState) -> BatchState:
        logits = self.lm_head(self.input_norm(batch_state.hidden_states))
        batch_state.output_ids = logits.argmax(dim=-1)
        return batch_state


class _Body(nn.Module):
    """Holds `embed_tokens` and the rotary tables (`model.model` in the reference)."""

    def __init__(self, config: LlamaConfig, dtype):
        super().__init__()
        self.embed_tokens = LlamaEmbeddings(config.vocab_size, config.hidden_size, dtype)
        self.rope_cos: Tensor | None = None
        self.rope_sin: Tensor | None = None


@dataclass
class StackedParams:
    qkv_proj: Tensor
    o_proj: Tensor
    attn_ln_weight: Tensor
    mlp_ln_weight: Tensor
    up_proj: Tensor
    gate_proj: Tensor
    down_proj: Tensor


# tensor ids of the synthetic weight draw
_TID_Q, _TID_K, _TID_V, _TID_O, _TID_GATE, _TID_UP, _TID_DOWN = range(7)
_TID_EMBED = 1_000_000
_TID_LM_HEAD = 1_000_001


class LlamaForCausalLM(nn.Module):
    def __init__(self, config: LlamaConfig, extra_config: ExtraModelConfig | None = None,
                 device="cpu", dtype=torch.bfloat16):
        super().__init__()
        self.config = config
        self.extra_config = extra_config or ExtraModelConfig()
        self.device = torch.device(device)
        self.dtype = dtype
        self.model = _Body(config, dtype)
        self.lm_head = LlamaLMHead(config, dtype)
        self.stacked_params: StackedParams | None = None
        self.stacked_kv_cache: tuple[Tensor, Tensor] | None = None

    def max_len(self) -> int:
        return self.extra_config.max_len_override or self.config.max_position_embeddings

    @classmethod
    def random_init(
        cls,
        config: LlamaConfig,
        extra_config: ExtraModelConfig | None = None,
        seed: int = 0,
        std: float = 0.02,
        device="cpu",
        dtype=torch.bfloat16,
    ) -> "LlamaForCausalLM":
        """Weights N(0, std) drawn per tensor from `seed` (norm weights are 1).

        Tensor ids: layer l uses 16 l + {q 0, k 1, v 2, o 3, gate 4, up 5,
        down 6}; the embedding uses 1_000_000 and an untied LM head 1_000_001.
        q/k rows are drawn in the checkpoint (half-split) order and then
        interleaved when `extra_config.interleave_rope` is set, as a loaded
        checkpoint would be.
        """
        m = cls(config, extra_config, device=device, dtype=dtype)
        c = config
        D, H, L = c.head_dim, c.hidden_size, c.num_hidden_layers
        qd, kd = c.num_attention_heads * D, c.num_key_value_heads * D

        def w(shape, tid):
            return seeded_normal(shape, seed, tid, std, dtype)

        qkv, o, gate, up, down = [], [], [], [], []
        for l in range(L):
            base = 16 * l
            qkv.append(torch.cat([w((qd, H), base + _TID_Q), w((kd, H), base + _TID_K),
                                  w((kd, H), base + _TID_V)]))
            o.append(w((H, qd), base + _TID_O))
            gate.append(w((c.intermediate_size, H), base + _TID_GATE))
            up.append(w((c.intermediate_size, H), base + _TID_UP))
            down.append(w((H, c.intermediate_size), base + _TID_DOWN))
        embed = w((c.vocab_size, H), _TID_EMBED)
        lm = embed if c.tie_word_embeddings else w((c.vocab_size, H), _TID_LM_HEAD)

        dev = m.device
        m.stacked_params = StackedParams(
            qkv_proj=torch.stack(qkv).to(dev),
            o_proj=torch.stack(o).to(dev),
            attn_ln_weight=torch.ones(L, H, dtype=dtype, device=dev),
            mlp_ln_weight=torch.ones(L, H, dtype=dtype, device=dev),
            up_proj=torch.stack(up).to(dev),
            gate_proj=torch.stack(gate).to(dev),
            down_proj=torch.stack(down).to(dev),
        )
        del qkv, o, gate, up, down
        m.model.embed_tokens.embed_tokens.weight.data = embed.to(dev)
        if c.tie_word_embeddings:
            m.lm_head.lm_head.weight.data = m.model.embed_tokens.embed_tokens.weight.data
        else:
            m.lm_head.lm_head.weight.data = lm.to(dev)
        m.lm_head.input_norm.weight.data = m.lm_head.input_norm.weight.data.to(dev)

        cos, sin = rope_tables(D, c.rope_theta, c.rope_scaling, m.max_len())
        m.model.rope_cos, m.model.rope_sin = cos.to(dev), sin.to(dev)
        if m.extra_config.interleave_rope:
            m.interleave_rope()
        m.setup_caches()
        return m

    def interleave_rope(self):
        D = self.config.head_dim
        perm = interleave_permutation(D).to(self.device)
        self.model.rope_cos = self.model.rope_cos[..., perm].contiguous()
        self.model.rope_sin = self.model.rope_sin[..., perm].contiguous()
        heads = self.config.num_attention_heads + self.config.num_key_value_heads
        rows = (perm.unsqueeze(0) + D * torch.arange(heads, device=self.device).unsqueeze(1)).reshape(-1)
        qkv = self.stacked_params.qkv_proj
        qkv[:, : heads * D] = qkv[:, rows]

    @torch.no_grad()
    def prefill(self, input_ids: Tensor, start_pos: int = 0) -> Tensor:
        """Run n prompt tokens (positions start_pos .. start_pos + n - 1) through
        the model as dense matrix products with causal attention, append their
        K/V rows to the cache, and return the last token's logits. This is the
        reference's prefill branch (megakernels/llama.py:90-133 of epic-kernel:
        K/V written at the positions, then scaled-dot-product attention with a
        causal mask); the decode megakernel then continues at start_pos + n.
        Rounding follows the decode path: bf16 activations between ops, fp32
        accumulation inside each product, RMSNorm as the interpreter's."""
        c, sp = self.config, self.stacked_params
        k_cache, v_cache = self.stacked_kv_cache
        ids = input_ids.reshape(-1).to(self.device)
        n, D = ids.numel(), c.head_dim
        Hq, Hkv = c.num_attention_heads, c.num_key_value_heads
        end = start_pos + n
        assert n >= 1 and end <= self.max_len(), "prompt beyond the KV cache"
        pos = torch.arange(start_pos, end, device=self.device)
        cos, sin = self.model.rope_cos[pos].unsqueeze(1), self.model.rope_sin[pos].unsqueeze(1)  # [n, 1, D]

        def norm(x, w):
            xf = x.float()
            return w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + c.rms_norm_eps)).to(x.dtype)

        def rope(x):  # [n, heads, D] bf16 -> fp32 rotary -> bf16
            if self.extra_config.interleave_rope:
                rot = torch.stack((-x[..., 1::2], x[..., 0::2]), dim=-1).reshape(x.shape)
            else:
                rot = torch.cat((-x[..., D // 2 :], x[..., : D // 2]), dim=-1)
            return (x * cos + rot * sin).to(x.dtype)

        # causal mask with the cached prefix: query i sees keys 0 .. start_pos + i
        mask = torch.arange(end, device=self.device).unsqueeze(0) <= pos.unsqueeze(1)  # [n, end]
        h = self.model.embed_tokens.embed_tokens.weight[ids]  # [n, H]
        for l in range(c.num_hidden_layers):
            qkv = norm(h, sp.attn_ln_weight[l]) @ sp.qkv_proj[l].T
            q = rope(qkv[:, : Hq * D].view(n, Hq, D))
            k = rope(qkv[:, Hq * D : (Hq + Hkv) * D].view(n, Hkv, D))
            v = qkv[:, (Hq + Hkv) * D :].view(n, Hkv, D)
            k_cache[l, 0, start_pos:end] = k
            v_cache[l, 0, start_pos:end] = v
            keys = k_cache[l, 0, :end].transpose(0, 1).unsqueeze(0)  # [1, Hkv, end, D]
            vals = v_cache[l, 0, :end].transpose(0, 1).unsqueeze(0)
            o = F.scaled_dot_product_attention(q.transpose(0, 1).unsqueeze(0), keys, vals, attn_mask=mask,
                                               scale=1.0 / math.sqrt(D), enable_gqa=True)
            h = h + o[0].transpose(0, 1).reshape(n, Hq * D) @ sp.o_proj[l].T
            x = norm(h, sp.mlp_ln_weight[l])
            up, gate = x @ sp.up_proj[l].T, x @ sp.gate_proj[l].T
            h = h + (F.silu(gate) * up) @ sp.down_proj[l].T
        self.prefill_hidden = h[-1].clone()
        return self.lm_head.lm_head(self.lm_head.input_norm(h[-1]))

    def setup_caches(self):
        shape = (
            self.config.num_hidden_layers,
            self.extra_config.max_batch_size,
            self.max_len(),
            self.config.num_key_value_heads,
            self.config.head_dim,
        )
        k = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.stacked_kv_cache = (k, torch.zeros_like(k))

    def to(self, device=None, dtype=None):  # type: ignore[override]
        raise NotImplementedError("build the model on its target device with random_init(device=...)")
