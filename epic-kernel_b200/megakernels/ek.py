"""ctypes binding of the C ABI in `include/ek.h` (libek.so).

The library is built in-tree by `megakernels.build` (or `__graft_entry__.build`).
There is no fallback: if the shared library or a CUDA device is missing, every
call raises.
"""

import ctypes
import os
import threading
from pathlib import Path

import torch

PKG_ROOT = Path(__file__).resolve().parent.parent  # the directory holding mk_llama.py
LIB_PATH = PKG_ROOT / "libek.so"

EK_ABI_VERSION = 2

STATUS_NAMES = {
    0: "ok",
    1: "timeout waiting on a cross-SM counter",
    2: "unknown opcode",
    3: "instruction field out of range",
    4: "load ring stalled",
    5: "weight copy failed its bounds check",
}


class EkStatus(ctypes.Structure):
    _fields_ = [
        ("code", ctypes.c_int32),
        ("sm", ctypes.c_int32),
        ("instr", ctypes.c_int32),
        ("opcode", ctypes.c_int32),
        ("layer", ctypes.c_int32),
        ("observed", ctypes.c_int32),
        ("expected", ctypes.c_int32),
        ("detail", ctypes.c_int32),
    ]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


_P = ctypes.c_void_p
_I = ctypes.c_int32


class EkLlamaArgs(ctypes.Structure):
    _fields_ = [
        ("barriers", _P), ("instructions", _P), ("timings", _P),
        ("qkv_weights", _P), ("attn_ln_weights", _P), ("o_weights", _P), ("mlp_ln_weights", _P),
        ("up_weights", _P), ("gate_weights", _P), ("down_weights", _P),
        ("lm_head_norm_weights", _P), ("lm_head_weights", _P),
        ("k_cache", _P), ("v_cache", _P), ("rope_cos", _P), ("rope_sin", _P),
        ("hidden_states", _P), ("q_post_rope", _P), ("attn_out", _P),
        ("attn_lse_intermediates", _P), ("attn_out_intermediates", _P),
        ("silu_out", _P), ("logits", _P),
        ("num_layers", _I), ("hidden", _I), ("intermediate", _I), ("head_dim", _I),
        ("num_q_heads", _I), ("num_kv_heads", _I), ("vocab", _I),
        ("kv_len", _I), ("rope_rows", _I), ("max_partials", _I),
        ("barrier_rows", _I), ("barrier_cols", _I), ("num_queues", _I), ("queue_len", _I),
        ("pos_id", _I), ("attn_scale", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
        ("skip_attn_reduction", _I),
        ("down_reduction_size", _I), ("oproj_reduction_size", _I),
        ("l2_prefetch_stages", _I), ("record_timings", _I),
        ("timeout_ns", ctypes.c_int64),
        ("cache_flags", _I), ("prefetch_gap_ns", _I),
        ("options", _I), ("deferred_down_layers", _I),
        ("input_token", _P), ("embed_weights", _P), ("output_token", _P), ("lm_head_instructions", _I),
    ]


class EkMixtralArgs(ctypes.Structure):
    _fields_ = [
        ("barriers", _P), ("instructions", _P), ("timings", _P),
        ("qkv_weights", _P), ("attn_ln_weights", _P), ("o_weights", _P),
        ("expert_gate_weights", _P), ("expert_up_weights", _P), ("expert_down_weights", _P),
        ("router_weights", _P), ("ffn_ln_weights", _P),
        ("lm_head_norm_weights", _P), ("lm_head_weights", _P),
        ("k_cache", _P), ("v_cache", _P), ("rope_cos", _P), ("rope_sin", _P),
        ("hidden_states", _P), ("q_post_rope", _P), ("attn_out", _P),
        ("attn_lse_intermediates", _P), ("attn_out_intermediates", _P),
        ("expert_silu_out", _P), ("router_normed_hidden", _P), ("logits", _P),
        ("selected_expert_indices", _P), ("selected_expert_scores", _P), ("predicted_expert_indices", _P),
        ("num_layers", _I), ("hidden", _I), ("intermediate", _I), ("head_dim", _I),
        ("num_q_heads", _I), ("num_kv_heads", _I), ("vocab", _I),
        ("num_experts", _I), ("experts_per_token", _I),
        ("kv_len", _I), ("rope_rows", _I), ("max_partials", _I),
        ("barrier_rows", _I), ("barrier_cols", _I), ("num_queues", _I), ("queue_len", _I),
        ("pos_id", _I), ("attn_scale", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
        ("skip_attn_reduction", _I),
        ("l2_prefetch_stages", _I), ("record_timings", _I),
        ("timeout_ns", ctypes.c_int64),
        ("cache_flags", _I), ("prefetch_gap_ns", _I),
        ("tp_lm_instructions", _I), ("speculative_prefetch_stages", _I),
    ]


_lib = None
_lib_lock = threading.Lock()


def load_library(path: Path | str | None = None) -> ctypes.CDLL:
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        p = Path(path or os.environ.get("EK_LIBRARY", LIB_PATH))
        if not p.exists():
            raise RuntimeError(
                f"{p} not found: build the CUDA engine first (python -m megakernels.build)"
            )
        lib = ctypes.CDLL(str(p))
        lib.ek_abi_version.restype = ctypes.c_int
        lib.ek_last_error.restype = ctypes.c_char_p
        lib.ek_context_create.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
        lib.ek_context_destroy.argtypes = [ctypes.c_void_p]
        lib.ek_context_destroy.restype = None
        lib.ek_llama_decode.argtypes = [ctypes.c_void_p, ctypes.POINTER(EkLlamaArgs), ctypes.c_void_p]
        lib.ek_read_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(EkStatus), ctypes.c_int]
        lib.ek_mixtral_decode.argtypes = [ctypes.c_void_p, ctypes.POINTER(EkMixtralArgs), ctypes.c_void_p]
        lib.ek_tp_setup.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        lib.ek_tp_connect.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        if lib.ek_abi_version() != EK_ABI_VERSION:
            raise RuntimeError(f"{p}: ABI {lib.ek_abi_version()} != expected {EK_ABI_VERSION}")
        _lib = lib
        return lib


def check(rc: int, what: str):
    if rc != 0:
        msg = load_library().ek_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (code {rc}): {msg}")


class EngineError(RuntimeError):
    """A device-side failure recorded by the megakernel."""

    def __init__(self, status: EkStatus):
        self.status = status.as_dict()
        super().__init__(
            f"megakernel: {STATUS_NAMES.get(status.code, status.code)} "
            f"(sm {status.sm}, instruction {status.instr}, opcode {status.opcode}, "
            f"layer {status.layer}, observed {status.observed}, expected {status.expected}, "
            f"detail {status.detail})"
        )


class Context:
    """One engine context per CUDA device (status record + split scratch)."""

    def __init__(self, device: int):
        lib = load_library()
        handle = ctypes.c_void_p()
        check(lib.ek_context_create(device, ctypes.byref(handle)), "ek_context_create")
        self.handle = handle
        self.device = device

    def read_status(self, clear: bool = True) -> EkStatus:
        st = EkStatus()
        check(load_library().ek_read_status(self.handle, ctypes.byref(st), int(clear)), "ek_read_status")
        return st

    def raise_if_failed(self, clear: bool = True):
        st = self.read_status(clear)
        if st.code != 0:
            raise EngineError(st)

    def close(self):
        if self.handle:
            load_library().ek_context_destroy(self.handle)
            self.handle = None


_contexts: dict[int, Context] = {}


def context_for(device: int) -> Context:
    ctx = _contexts.get(device)
    if ctx is None:
        if not torch.cuda.is_available():
            raise RuntimeError("the decode engine needs a CUDA device; none is available")
        ctx = _contexts[device] = Context(device)
    return ctx
