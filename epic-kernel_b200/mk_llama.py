"""`mk_llama` / `mk_llama_3b`: drop-in replacements of epic-kernel's pybind
modules of the same names (demos/low-latency-llama/llama_1b.cu:23-47,
llama_3b.cu:26-53).

The positional signature is the reference's (megakernels/demos/latency/mk.py:
18-52): the VM tensors, the weights, the 4-D KV caches, the rotary tables, the
activation buffers, then pos_id, attn_scale, rms_norm_eps,
skip_attn_reduction, and `stream=` as a keyword. Unlike the reference, one
module serves every Llama size, because the model dimensions are read from the
tensor shapes instead of being compiled in.

Extra keyword-only options (defaults match the reference's behaviour):
  l2_prefetch_stages  > 0: 16 KiB weight stages prefetched into L2 ahead of
                      the shared-memory ring while it is full; -1: the next
                      instruction's whole weight range prefetched into L2
                      when an instruction starts loading; -2: a layer's MLP
                      weights prefetched when its attention chain starts;
                      0 = off (default; every mode measured slower on B200)
  timeout_ns          bound of every cross-SM wait (default 1 s)
  record_timings      write start / dependency-ready / end stamps (ns) into
                      timings[q, i, 0..2]
  down_reduction_size columns per DownProjResidual split (default gcd(I, H),
                      as the schedule builder uses)
  cache_flags         EK_CACHE_* bits of include/ek.h (default: weight loads
                      marked evict_first)
  prefetch_gap_ns     pause of the optional MLP-weight prefetcher per 16 KiB
  fuse_attention_reduction
                      the last PartialAttention of each KV head merges the
                      head's partials and AttentionReduction instructions do
                      nothing (only for schedules whose reductions are
                      terminal over all partials in order; the interpreter
                      sets it when `tensorize_instructions` found that)
  deferred_down_layers
                      down projections of layers l < this value leave their
                      column-split partials for layer l + 1 to add (the
                      interpreter passes what `tensorize_instructions` found
                      safe for the stream)
  input_token, embed_weights, output_token, lm_head_instructions
                      fused token step: layer 0 reads embed_weights[input_token]
                      (int64 device scalar) instead of hidden_states, and the
                      argmax of the logits (first index on ties) is written to
                      output_token (int64); lm_head_instructions = number of
                      RMS_LM_Head instructions in the queues

Errors: bad shapes or dtypes raise ValueError before launch; a CUDA launch
failure raises RuntimeError. Device-side failures (timeouts, malformed
instructions) are recorded on the device. Call `check()` after synchronising
to raise them as `megakernels.ek.EngineError`.
"""

import ctypes
import math

import torch

from megakernels import ek

_BF16 = torch.bfloat16
_cache: dict = {}

# EK_CACHE_* bits (include/ek.h). Weight loads are marked evict_first by
# default, so the small cross-SM working set (counters, activations,
# instructions) stays in L2 while 2.5+ GB of weights stream through it.
EK_CACHE_PREFETCH_UPGATE = 1
EK_CACHE_PREFETCH_DOWN = 2
EK_CACHE_PREFETCH_BULK = 4
EK_CACHE_PREFETCH_EVICT_LAST = 8
EK_CACHE_WEIGHTS_EVICT_FIRST = 16
EK_CACHE_KV_EVICT_FIRST = 32
DEFAULT_CACHE_FLAGS = EK_CACHE_WEIGHTS_EVICT_FIRST
EK_OPT_FUSE_ATTENTION_REDUCTION = 1


def _need(t: torch.Tensor, name: str, dtype, ndim: int | None = None):
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name}: expected a tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError(f"{name}: must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name}: dtype {t.dtype}, expected {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name}: {t.dim()}-D, expected {ndim}-D")
    return t.data_ptr()


def _build_args(tensors, l2_prefetch_stages, record_timings, timeout_ns, down_reduction_size,
                cache_flags=None, prefetch_gap_ns=0, fuse_attention_reduction=False,
                deferred_down_layers=0):
    (barriers, instructions, timings, qkv_w, attn_ln_w, o_w, mlp_ln_w, up_w, gate_w, down_w,
     lm_norm_w, lm_w, k4, v4, cos, sin, hidden, q, attn_out, lse, o_int, silu, logits) = tensors
    a = ek.EkLlamaArgs()
    a.barriers = _need(barriers, "barriers", torch.int32, 3)
    a.instructions = _need(instructions, "instructions", torch.int32, 3)
    a.timings = _need(timings, "timings", torch.int32, 3) if timings is not None else None
    a.qkv_weights = _need(qkv_w, "qkv_weights", _BF16, 3)
    a.attn_ln_weights = _need(attn_ln_w, "attn_ln_weights", _BF16, 2)
    a.o_weights = _need(o_w, "o_weights", _BF16, 3)
    a.mlp_ln_weights = _need(mlp_ln_w, "mlp_ln_weights", _BF16, 2)
    a.up_weights = _need(up_w, "up_weights", _BF16, 3)
    a.gate_weights = _need(gate_w, "gate_weights", _BF16, 3)
    a.down_weights = _need(down_w, "down_weights", _BF16, 3)
    a.lm_head_norm_weights = _need(lm_norm_w, "lm_head_norm_weights", _BF16)
    a.lm_head_weights = _need(lm_w, "lm_head_weights", _BF16, 2)
    a.k_cache = _need(k4, "k_cache", _BF16, 4)
    a.v_cache = _need(v4, "v_cache", _BF16, 4)
    a.rope_cos = _need(cos, "rope_cos", torch.float32, 2)
    a.rope_sin = _need(sin, "rope_sin", torch.float32, 2)
    a.hidden_states = _need(hidden, "hidden_states", _BF16)
    a.q_post_rope = _need(q, "q_post_rope", _BF16)
    a.attn_out = _need(attn_out, "attn_out", _BF16)
    a.attn_lse_intermediates = _need(lse, "attn_lse_intermediates", torch.float32, 2)
    a.attn_out_intermediates = _need(o_int, "attn_out_intermediates", torch.float32, 3)
    a.silu_out = _need(silu, "silu_out", _BF16)
    a.logits = _need(logits, "logits", _BF16)

    L, I, H = up_w.shape
    D = k4.shape[3]
    Hkv = k4.shape[2]
    Hq = lse.shape[0]
    V = lm_w.shape[0]
    checks = [
        (qkv_w.shape == (L, (Hq + 2 * Hkv) * D, H), "qkv_weights shape"),
        (o_w.shape == (L, H, Hq * D), "o_weights shape"),
        (gate_w.shape == up_w.shape, "gate_weights shape"),
        (down_w.shape == (L, H, I), "down_weights shape"),
        (attn_ln_w.shape == (L, H) and mlp_ln_w.shape == (L, H), "layernorm weight shapes"),
        (lm_norm_w.numel() == H and lm_w.shape[1] == H, "lm head shapes"),
        (k4.shape[0] == L and v4.shape == k4.shape, "kv cache shapes"),
        (cos.shape[1] == D and sin.shape == cos.shape, "rope table shapes"),
        (hidden.numel() == H and q.numel() == Hq * D and attn_out.numel() == Hq * D, "activation sizes"),
        (o_int.shape[0] == Hq and o_int.shape[1] == lse.shape[1] and o_int.shape[2] == D, "attention intermediates"),
        (silu.numel() == I and logits.numel() == V, "silu_out / logits sizes"),
        (barriers.shape[0] == L, "barriers first dim"),
        (instructions.shape[2] == 32, "instructions last dim"),
        (timings is None or timings.shape[:2] == instructions.shape[:2], "timings shape"),
    ]
    for ok, what in checks:
        if not ok:
            raise ValueError(f"mk_llama: inconsistent {what}")
    devices = {t.device for t in tensors if t is not None}
    if len(devices) != 1:
        raise ValueError(f"mk_llama: tensors on several devices {devices}")

    a.num_layers, a.hidden, a.intermediate, a.head_dim = L, H, I, D
    a.num_q_heads, a.num_kv_heads, a.vocab = Hq, Hkv, V
    a.kv_len = k4.shape[1]
    a.rope_rows = cos.shape[0]
    a.max_partials = lse.shape[1]
    a.barrier_rows, a.barrier_cols = barriers.shape[1], barriers.shape[2]
    a.num_queues, a.queue_len = instructions.shape[0], instructions.shape[1]
    a.down_reduction_size = down_reduction_size or math.gcd(I, H)
    a.oproj_reduction_size = H
    a.l2_prefetch_stages = l2_prefetch_stages
    a.record_timings = int(bool(record_timings))
    a.timeout_ns = int(timeout_ns)
    a.cache_flags = int(DEFAULT_CACHE_FLAGS if cache_flags is None else cache_flags)
    a.prefetch_gap_ns = int(prefetch_gap_ns)
    a.options = EK_OPT_FUSE_ATTENTION_REDUCTION if fuse_attention_reduction else 0
    a.deferred_down_layers = int(deferred_down_layers)
    return a, next(iter(devices)).index


def mk_llama(
    barriers, instructions, timings,
    qkv_proj_weights, attn_ln_weights, o_proj_weights, mlp_ln_weights,
    up_proj_weights, gate_proj_weights, down_proj_weights,
    lm_head_norm_weights, lm_head_weights,
    k_cache, v_cache, rope_cos, rope_sin,
    hidden_states, post_ln_rope_q, attn_out, attn_lse_intermediates, attn_out_intermediates,
    silu_out, logits,
    pos_id, attn_scale, rms_norm_eps, skip_attn_reduction,
    *, stream=None, l2_prefetch_stages: int = 0, record_timings: bool = False,
    timeout_ns: int = 0, down_reduction_size: int = 0,
    cache_flags: int | None = None, prefetch_gap_ns: int = 0, fuse_attention_reduction: bool = False,
    deferred_down_layers: int = 0,
    input_token=None, embed_weights=None, output_token=None, lm_head_instructions: int = 0,
):
    tensors = (barriers, instructions, timings, qkv_proj_weights, attn_ln_weights, o_proj_weights,
               mlp_ln_weights, up_proj_weights, gate_proj_weights, down_proj_weights,
               lm_head_norm_weights, lm_head_weights, k_cache, v_cache, rope_cos, rope_sin,
               hidden_states, post_ln_rope_q, attn_out, attn_lse_intermediates,
               attn_out_intermediates, silu_out, logits)
    if cache_flags is None:
        cache_flags = DEFAULT_CACHE_FLAGS
    key = (tuple((t.data_ptr(), tuple(t.shape), t.dtype) if t is not None else None for t in tensors),
           l2_prefetch_stages, bool(record_timings), int(timeout_ns), down_reduction_size,
           int(cache_flags), int(prefetch_gap_ns), bool(fuse_attention_reduction), int(deferred_down_layers))
    hit = _cache.get(key)
    if hit is None:
        hit = _build_args(tensors, l2_prefetch_stages, record_timings, timeout_ns, down_reduction_size,
                          cache_flags, prefetch_gap_ns, bool(fuse_attention_reduction),
                          int(deferred_down_layers))
        if len(_cache) > 64:
            _cache.clear()
        _cache[key] = hit
    args, device = hit
    args.pos_id = int(pos_id)
    args.attn_scale = float(attn_scale)
    args.rms_norm_eps = float(rms_norm_eps)
    args.skip_attn_reduction = int(bool(skip_attn_reduction))
    # fused token step: per-call device pointers (int64 token ids, embedding table)
    if (input_token is None) != (embed_weights is None):
        raise ValueError("mk_llama: input_token and embed_weights go together")
    args.input_token = _need(input_token, "input_token", torch.int64) if input_token is not None else None
    args.embed_weights = _need(embed_weights, "embed_weights", _BF16, 2) if embed_weights is not None else None
    args.output_token = _need(output_token, "output_token", torch.int64) if output_token is not None else None
    args.lm_head_instructions = int(lm_head_instructions)
    ctx = ek.context_for(device)
    if stream is None:
        stream = torch.cuda.current_stream(device)
    handle = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    ek.check(
        ek.load_library().ek_llama_decode(ctx.handle, ctypes.byref(args), ctypes.c_void_p(handle)),
        "ek_llama_decode",
    )


class PreparedStep:
    """The fused token step's launch with everything but the per-step values
    prepared once: build it from the same positional tensors and options as
    `mk_llama`, then `launch(pos_id, input_token, output_token)` per token.
    Per call it only writes those three fields and calls `ek_llama_decode`
    (no tensor checks or cache lookups); the tensors given at construction must
    stay allocated and in place."""

    def __init__(self, *tensors_and_scalars, embed_weights, lm_head_instructions, stream=None, **options):
        tensors = tensors_and_scalars[:23]
        pos_id, attn_scale, rms_norm_eps, skip_attn_reduction = tensors_and_scalars[23:27]
        opts = dict(options)
        cache_flags = opts.pop("cache_flags", None)
        self.args, self.device = _build_args(
            tensors, opts.pop("l2_prefetch_stages", 0), opts.pop("record_timings", False),
            opts.pop("timeout_ns", 0), opts.pop("down_reduction_size", 0),
            DEFAULT_CACHE_FLAGS if cache_flags is None else cache_flags, opts.pop("prefetch_gap_ns", 0),
            bool(opts.pop("fuse_attention_reduction", False)), int(opts.pop("deferred_down_layers", 0)))
        if opts:
            raise ValueError(f"PreparedStep: unknown options {sorted(opts)}")
        a = self.args
        a.attn_scale = float(attn_scale)
        a.rms_norm_eps = float(rms_norm_eps)
        a.skip_attn_reduction = int(bool(skip_attn_reduction))
        a.embed_weights = _need(embed_weights, "embed_weights", _BF16, 2)
        a.lm_head_instructions = int(lm_head_instructions)
        self.ctx = ek.context_for(self.device)
        self.fn = ek.load_library().ek_llama_decode
        self.args_ref = ctypes.byref(a)
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        self.stream = ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))

    def launch(self, pos_id: int, input_token: torch.Tensor, output_token: torch.Tensor):
        if not (input_token.is_cuda and output_token.is_cuda):
            raise ValueError("PreparedStep.launch: token tensors must be CUDA tensors")
        a = self.args
        a.pos_id = pos_id
        a.input_token = input_token.data_ptr()
        a.output_token = output_token.data_ptr()
        ek.check(self.fn(self.ctx.handle, self.args_ref, self.stream), "ek_llama_decode")


def check(device: int | None = None, clear: bool = True):
    """Synchronise and raise `EngineError` if a launch recorded a device failure."""
    if device is None:
        device = torch.cuda.current_device()
    ek.context_for(device).raise_if_failed(clear)


def read_status(device: int | None = None, clear: bool = False) -> dict:
    if device is None:
        device = torch.cuda.current_device()
    return ek.context_for(device).read_status(clear).as_dict()
