"""The allocation-free entry point `ek_llama_decode_static` (include/ek.h).

It exists for callers that cannot call cudaMalloc while decoding, such as
runtimes that have reserved all device memory up front or allocators that
must not be re-entered. It keeps the engine's scratch in fixed device arrays
inside the library instead of allocating it. This test calls it through the
C ABI twice in a row and checks each result against the regular entry point
(`ek_llama_decode`, via mk_llama) on identical inputs. The kernel is
deterministic, so the bar is bitwise equality, which is tighter than the
parity tolerances of the other GPU tests. This file is collected last so that
a failing run stops only after every other test has run.
"""

import ctypes

import pytest
import torch

import cases
from gpu_helpers import prepare, run_gpu
from megakernels import ek
from megakernels.scheduler import assign_to_sms, tensorize_instructions

pytestmark = pytest.mark.gpu

OUTPUTS = ("hidden_states", "post_ln_rope_q", "attn_out", "silu_out", "logits", "barriers")


def _static_fn():
    lib = ek.load_library()
    fn = lib.ek_llama_decode_static
    fn.argtypes = [ctypes.POINTER(ek.EkLlamaArgs), ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return lib, fn


def _run_static(sched):
    """One decode step through ek_llama_decode_static; returns the EkStatus."""
    import mk_llama

    g = sched.globs
    tensorize_instructions(g, assign_to_sms("rr", schedule=sched))
    g.barriers.zero_()
    tensors = (g.barriers, g.instructions, g.timings, g.qkv_proj_weights, g.attn_ln_weights,
               g.o_proj_weights, g.mlp_ln_weights, g.up_proj_weights, g.gate_proj_weights,
               g.down_proj_weights, g.lm_head_norm_weights.data, g.lm_head_weights.data,
               g.k_cache.flatten(0, 1), g.v_cache.flatten(0, 1), g.rope_cos, g.rope_sin,
               g.hidden_states, g.post_ln_rope_q, g.attn_out, g.attn_lse_intermediates,
               g.attn_out_intermediates, g.silu_out, g.logits)
    args, _ = mk_llama._build_args(tensors, 0, False, 0, 0)
    args.pos_id = g.pos_id
    args.attn_scale = g.attn_scale
    args.rms_norm_eps = g.rms_norm_eps
    args.skip_attn_reduction = int(g.skip_attn_reduction)
    status = torch.zeros(8, dtype=torch.int32, device=g.hidden_states.device)
    lib, fn = _static_fn()
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(ctypes.byref(args), ctypes.c_void_p(stream), ctypes.c_void_p(status.data_ptr()))
    assert rc == 0, lib.ek_last_error().decode()
    torch.cuda.synchronize()
    return status.cpu()


@pytest.mark.parametrize("pos", [300, 777])
def test_static_entry_matches_context_entry_twice(pos):
    model = cases.tiny_model("cuda")
    ref = prepare(model, pos, cases.step_hidden(2048, pos))
    run_gpu(ref)
    import mk_llama

    mk_llama.check()
    expected = {n: getattr(ref.globs, n).clone() for n in OUTPUTS}
    for call in range(2):
        s = prepare(model, pos, cases.step_hidden(2048, pos))
        torch.cuda.synchronize()
        free_before, _ = torch.cuda.mem_get_info()
        status = _run_static(s)
        free_after, _ = torch.cuda.mem_get_info()
        assert free_after == free_before, f"call {call}: device memory changed by {free_before - free_after} B"
        assert int(status[0]) == 0, f"call {call}: device status {status.tolist()}"
        for n in OUTPUTS:
            assert torch.equal(getattr(s.globs, n), expected[n]), f"call {call}: {n} differs"


def test_static_entry_rejects_oversized_model():
    lib, fn = _static_fn()
    a = ek.EkLlamaArgs()
    a.num_layers, a.hidden, a.intermediate = 128, 8192, 28672
    rc = fn(ctypes.byref(a), None, None)
    assert rc == 3  # EK_E_UNSUPPORTED
    assert b"allocation-free" in lib.ek_last_error()
