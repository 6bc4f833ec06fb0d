"""Two host threads, each with its own engine context on one GPU and its own
stream, call ek_llama_decode at the same time on different inputs. The C ABI
keeps no shared host state per call (kernel parameters are staged per call,
the shared-memory opt-in is tracked per device), so every result must equal,
bit for bit, the same step run alone. The two kernels never wait on each
other: each holds all SMs while it runs, so the GPU runs them in turn."""

import ctypes
import threading

import pytest
import torch

import cases
from gpu_helpers import prepare
from megakernels import ek
from megakernels.scheduler import assign_to_sms, tensorize_instructions

pytestmark = pytest.mark.gpu

OUTPUTS = ("hidden_states", "logits", "barriers", "attn_out", "silu_out")
ROUNDS = 4


def _args(sched):
    import mk_llama

    g = sched.globs
    tensors = (g.barriers, g.instructions, g.timings, g.qkv_proj_weights, g.attn_ln_weights,
               g.o_proj_weights, g.mlp_ln_weights, g.up_proj_weights, g.gate_proj_weights,
               g.down_proj_weights, g.lm_head_norm_weights.data, g.lm_head_weights.data,
               g.k_cache.flatten(0, 1), g.v_cache.flatten(0, 1), g.rope_cos, g.rope_sin,
               g.hidden_states, g.post_ln_rope_q, g.attn_out, g.attn_lse_intermediates,
               g.attn_out_intermediates, g.silu_out, g.logits)
    a, _ = mk_llama._build_args(tensors, 0, False, 0, 0)
    a.pos_id = g.pos_id
    a.attn_scale = g.attn_scale
    a.rms_norm_eps = g.rms_norm_eps
    a.skip_attn_reduction = int(g.skip_attn_reduction)
    return a


def _case(model, pos):
    s = prepare(model, pos, cases.step_hidden(2048, pos))
    tensorize_instructions(s.globs, assign_to_sms("rr", schedule=s))
    return s, {n: getattr(s.globs, n).clone() for n in ("hidden_states",)}


def _reset(s, init):
    s.globs.hidden_states.copy_(init["hidden_states"])
    s.globs.barriers.zero_()


def test_two_threads_two_contexts_one_gpu():
    torch.cuda.set_device(0)
    lib = ek.load_library()
    model = cases.tiny_model("cuda")
    cases_ = [_case(model, 300), _case(model, 777)]
    ctxs = []
    for _ in range(2):
        h = ctypes.c_void_p()
        assert lib.ek_context_create(0, ctypes.byref(h)) == 0, lib.ek_last_error()
        ctxs.append(h)
    streams = [torch.cuda.Stream() for _ in range(2)]
    try:
        # serial reference results
        expected = []
        for (s, init), ctx, st in zip(cases_, ctxs, streams):
            with torch.cuda.stream(st):
                _reset(s, init)
                a = _args(s)
                assert lib.ek_llama_decode(ctx, ctypes.byref(a), ctypes.c_void_p(st.cuda_stream)) == 0
                expected.append({n: getattr(s.globs, n).clone() for n in OUTPUTS})
            st.synchronize()
        # concurrent: each thread launches ROUNDS steps on its own context and stream
        errors = []
        results = [[], []]

        def worker(k):
            try:
                s, init = cases_[k]
                a = _args(s)
                with torch.cuda.stream(streams[k]):  # resets, launches and copies in stream order
                    for _ in range(ROUNDS):
                        _reset(s, init)
                        rc = lib.ek_llama_decode(ctxs[k], ctypes.byref(a), ctypes.c_void_p(streams[k].cuda_stream))
                        if rc:
                            errors.append(lib.ek_last_error())
                        results[k].append({n: getattr(s.globs, n).clone() for n in OUTPUTS})
                    streams[k].synchronize()
            except Exception as e:  # noqa: BLE001
                errors.append(repr(e))

        threads = [threading.Thread(target=worker, args=(k,)) for k in range(2)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=120)
        assert not errors, errors
        for k in range(2):
            assert len(results[k]) == ROUNDS
            for r, got in enumerate(results[k]):
                for n in OUTPUTS:
                    assert torch.equal(got[n], expected[k][n]), f"thread {k} round {r}: {n} differs"
        for ctx in ctxs:
            st = ek.EkStatus()
            assert lib.ek_read_status(ctx, ctypes.byref(st), 1) == 0
            assert st.code == 0, st.as_dict()
    finally:
        for ctx in ctxs:
            lib.ek_context_destroy(ctx)
