"""Calling the Mixtral megakernel with a `MixtralGlobals` bundle
(`megakernels/mixtral/mk.py` of epic-kernel, :13-107): expert weights and the
router are viewed as [L * E, ...], the LM-head norm as [1, H], the KV caches
as 4-D, and everything is passed in mk_mixtral's positional order."""

from pathlib import Path

import torch

from megakernels.mixtral.instructions import MixtralGlobals
from megakernels.mk import MK_Interpreter, _add_to_path


def interpret_with_mk(globs: MixtralGlobals, mk_func, **options):
    L, E = globs.num_hidden_layers, globs.num_experts
    mk_func(
        globs.barriers,
        globs.instructions,
        globs.timings,
        globs.qkv_proj_weights,
        globs.attn_ln_weights,
        globs.o_proj_weights,
        globs.expert_gate_weights.reshape(L * E, *globs.expert_gate_weights.shape[2:]),
        globs.expert_up_weights.reshape(L * E, *globs.expert_up_weights.shape[2:]),
        globs.expert_down_weights.reshape(L * E, *globs.expert_down_weights.shape[2:]),
        globs.router_weights.reshape(L * E, -1),
        globs.ffn_ln_weights,
        globs.lm_head_norm_weights.data.unsqueeze(0),
        globs.lm_head_weights.data,
        globs.k_cache.flatten(0, 1),
        globs.v_cache.flatten(0, 1),
        globs.rope_cos,
        globs.rope_sin,
        globs.hidden_states,
        globs.post_ln_rope_q,
        globs.attn_out,
        globs.attn_lse_intermediates,
        globs.attn_out_intermediates,
        globs.expert_silu_out,
        globs.router_normed_hidden,
        globs.logits,
        globs.selected_expert_indices,
        globs.selected_expert_scores,
        globs.predicted_expert_indices,
        globs.pos_id,
        globs.attn_scale,
        globs.rms_norm_eps,
        globs.skip_attn_reduction,
        stream=torch.cuda.current_stream(),
        **options,
    )


class MixtralMK_Interpreter(MK_Interpreter):
    def __init__(self, mk_dir: Path | str | None = None, **options):
        _add_to_path(mk_dir)
        from mk_mixtral import mk_mixtral  # type: ignore

        self.mk_func = mk_mixtral
        self.options = options

    def interpret(self, globs: MixtralGlobals):
        interpret_with_mk(globs, self.mk_func, **stream_options(globs, self.options))


# ring stages per predicted expert prefetched into L2 before the router's choice
SPECULATIVE_PREFETCH_STAGES = 8


def stream_options(globs, options):
    """Engine options that depend on the instruction stream: the speculative
    expert prefetch runs only when the queues hold SpeculativeExpertPredict
    instructions (as `tensorize_instructions` recorded)."""
    opts = dict(options)
    opts.setdefault("speculative_prefetch_stages",
                    SPECULATIVE_PREFETCH_STAGES if getattr(globs, "expert_predictions", 0) else 0)
    return opts
