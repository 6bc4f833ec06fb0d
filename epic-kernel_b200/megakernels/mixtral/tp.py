"""Tensor-parallel Mixtral decode: one process per GPU, in-kernel all-reduce.

Set-up, once per model (host side; no counterpart in the reference, whose
megakernel is single-GPU):
1. every rank builds its shard (`MixtralForCausalLM.random_init(tp=(rank, world))`)
   and its schedule as usual;
2. `setup_tensor_parallel(globs, rank, world, group)` allocates the rank's
   symmetric buffer in the engine (`ek_tp_setup`), exchanges the 64-byte CUDA
   IPC handles over `torch.distributed` (any backend; gloo on CPU hosts works),
   opens the peers' buffers (`ek_tp_connect`) and points `globs.logits` at the
   symmetric full-vocabulary logits buffer;
3. decode with `MixtralTPMK_Interpreter` exactly as with one GPU.

The per-layer hidden-state all-reduces and the logits exchange then run inside
the megakernel over NVLink (plain peer stores and release.sys counters); no
NCCL call is on the token path.
"""

import ctypes

import torch
import torch.distributed as dist

from megakernels import ek
from megakernels.mixtral.mk import MixtralMK_Interpreter


class _DevicePointer:
    """A raw device pointer viewed as a torch tensor (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (ptr, False), "version": 3, "strides": None,
        }


def _bf16_view(ptr: int, n: int, device) -> torch.Tensor:
    # expose as int16 (CAI has no bf16 typestr), then reinterpret
    t = torch.as_tensor(_DevicePointer(ptr, (n,), "<i2"), device=device)
    return t.view(torch.bfloat16)


def exchange_handles(handle: bytes, world: int, group=None) -> bytes:
    """All ranks' 64-byte IPC handles concatenated in rank order."""
    assert len(handle) == 64
    out = [None] * world
    dist.all_gather_object(out, handle, group=group)
    assert all(isinstance(h, bytes) and len(h) == 64 for h in out)
    return b"".join(out)


def setup_tensor_parallel(globs, rank: int, world: int, group=None):
    lib = ek.load_library()
    dev = globs.hidden_states.device
    ctx = ek.context_for(dev.index)
    handle = ctypes.create_string_buffer(64)
    logits_ptr = ctypes.c_void_p()
    full_vocab = globs.vocab_size * world
    ek.check(lib.ek_tp_setup(ctx.handle, rank, world, globs.num_hidden_layers, globs.hidden_size,
                             globs.num_experts_per_tok, full_vocab, handle, ctypes.byref(logits_ptr)),
             "ek_tp_setup")
    handles = exchange_handles(handle.raw, world, group)
    ek.check(lib.ek_tp_connect(ctx.handle, handles), "ek_tp_connect")
    globs.logits = _bf16_view(logits_ptr.value, full_vocab, dev)
    globs.logits.zero_()
    torch.cuda.synchronize(dev)
    if group is not None or dist.is_initialized():
        dist.barrier(group=group)
    return globs


def lm_head_instruction_count(globs) -> int:
    """Mixtral_RMS_LM_Head instructions in this rank's queues."""
    return int((globs.instructions[:, :, 0] == 7).sum().item())


class MixtralTPMK_Interpreter(MixtralMK_Interpreter):
    """Launches the tensor-parallel megakernel; `globs` must have been passed
    through setup_tensor_parallel and tensorize_instructions."""

    def interpret(self, globs):
        if not hasattr(globs, "_tp_lm_count"):
            globs._tp_lm_count = lm_head_instruction_count(globs)
        from megakernels.mixtral.mk import interpret_with_mk, stream_options

        interpret_with_mk(globs, self.mk_func, tp_lm_instructions=globs._tp_lm_count,
                          **stream_options(globs, self.options))
