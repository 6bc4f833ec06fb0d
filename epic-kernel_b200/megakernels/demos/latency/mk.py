"""Calling the Llama megakernel with a `Globals` bundle
(`megakernels/demos/latency/mk.py` of epic-kernel, :11-68): the 5-D KV caches
are viewed as 4-D `[(L * B), T, Hkv, D]` and the tensors passed in the
module's positional order on the current stream."""

from pathlib import Path

import torch

from megakernels.demos.latency.instructions import Globals
from megakernels.mk import MK_Interpreter, _add_to_path


def _positional(globs: Globals):
    """mk_llama's positional arguments for `globs`, in the reference's order."""
    return (globs.barriers, globs.instructions, globs.timings, globs.qkv_proj_weights,
            globs.attn_ln_weights, globs.o_proj_weights, globs.mlp_ln_weights, globs.up_proj_weights,
            globs.gate_proj_weights, globs.down_proj_weights, globs.lm_head_norm_weights.data,
            globs.lm_head_weights.data, globs.k_cache.flatten(0, 1), globs.v_cache.flatten(0, 1),
            globs.rope_cos, globs.rope_sin, globs.hidden_states, globs.post_ln_rope_q, globs.attn_out,
            globs.attn_lse_intermediates, globs.attn_out_intermediates, globs.silu_out, globs.logits,
            globs.pos_id, globs.attn_scale, globs.rms_norm_eps, globs.skip_attn_reduction)


def interpret_with_mk(globs: Globals, mk_func, **options):
    k4 = globs.k_cache.flatten(0, 1)
    v4 = globs.v_cache.flatten(0, 1)
    mk_func(
        globs.barriers,
        globs.instructions,
        globs.timings,
        globs.qkv_proj_weights,
        globs.attn_ln_weights,
        globs.o_proj_weights,
        globs.mlp_ln_weights,
        globs.up_proj_weights,
        globs.gate_proj_weights,
        globs.down_proj_weights,
        globs.lm_head_norm_weights.data,
        globs.lm_head_weights.data,
        k4,
        v4,
        globs.rope_cos,
        globs.rope_sin,
        globs.hidden_states,
        globs.post_ln_rope_q,
        globs.attn_out,
        globs.attn_lse_intermediates,
        globs.attn_out_intermediates,
        globs.silu_out,
        globs.logits,
        globs.pos_id,
        globs.attn_scale,
        globs.rms_norm_eps,
        globs.skip_attn_reduction,
        stream=torch.cuda.current_stream(),
        **options,
    )


def _stream_options(globs, options):
    """Engine options that depend on the instruction stream, as
    `tensorize_instructions` recorded them on `globs` (explicit options win)."""
    opts = dict(options)
    opts.setdefault("fuse_attention_reduction", getattr(globs, "attention_reduction_fusable", False))
    opts.setdefault("deferred_down_layers", getattr(globs, "deferrable_down_layers", 0))
    return opts


class LatencyMK_Interpreter(MK_Interpreter):
    """`options` are passed to every launch (e.g. l2_prefetch_stages)."""

    supports_fused_step = True

    def __init__(self, mk_dir: Path | str | None = None, **options):
        super().__init__(mk_dir)
        self.options = options

    def interpret_step(self, globs: Globals, input_token, embed_weights, output_token):
        """One decode step with the embedding gather and the argmax done inside
        the megakernel (no extra launches): layer 0 reads
        embed_weights[input_token], and the argmax of the logits lands in
        output_token (int64 device tensors)."""
        if input_token.dtype != torch.int64 or output_token.dtype != torch.int64:
            raise ValueError("interpret_step: token tensors must be int64")
        stream = torch.cuda.current_stream()
        key = (id(globs), globs.instructions.data_ptr(), globs.barriers.data_ptr(),
               globs.hidden_states.data_ptr(), globs.k_cache.data_ptr(), globs.logits.data_ptr(),
               embed_weights.data_ptr(), stream.cuda_stream, getattr(globs, "attention_reduction_fusable", False),
               getattr(globs, "deferrable_down_layers", 0))
        prepared = getattr(self, "_prepared", None)
        if prepared is None or prepared[0] != key:
            import mk_llama

            prepared = (key, mk_llama.PreparedStep(
                *_positional(globs), embed_weights=embed_weights,
                lm_head_instructions=getattr(globs, "lm_head_instructions", 0), stream=stream,
                **_stream_options(globs, self.options)))
            self._prepared = prepared
        prepared[1].launch(int(globs.pos_id), input_token, output_token)

    def interpret(self, globs: Globals):
        interpret_with_mk(globs, self.mk_func, **_stream_options(globs, self.options))


class Latency3B_MK_Interpreter(MK_Interpreter):
    def __init__(self, mk_dir: Path | str | None = None, **options):
        _add_to_path(mk_dir)
        from mk_llama_3b import mk_llama_3b  # type: ignore

        self.mk_func = mk_llama_3b
        self.options = options

    def interpret(self, globs: Globals):
        interpret_with_mk(globs, self.mk_func, **_stream_options(globs, self.options))
