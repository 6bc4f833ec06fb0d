"""Failure detection on the GPU without faulting it.

Every cross-SM wait in the megakernel is bounded. These tests make a wait run
out (an instruction stream whose producer was removed) or feed a malformed
instruction. Each then checks that the kernel reports the recorded status and
returns, and that the context still runs a correct step afterwards. Nothing
here traps, asserts on the device, or hangs.
"""

from dataclasses import dataclass

import pytest
import torch

import cases
from gpu_helpers import prepare, run_gpu
from megakernels.demos.latency.instructions import O_ProjResidual
from megakernels.demos.latency.mk import LatencyMK_Interpreter
from megakernels.ek import EngineError
from megakernels.instructions import Instruction, NoOp
from megakernels.scheduler import round_robin_assign_to_sms, tensorize_instructions

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_gpu():
    return cases.tiny_model("cuda")


def status_after(sched, instrs, timeout_ns=50_000_000):
    import mk_llama

    g = sched.globs
    tensorize_instructions(g, round_robin_assign_to_sms(instrs, g.sm_count()))
    g.barriers.zero_()
    LatencyMK_Interpreter(timeout_ns=timeout_ns).interpret(g)
    torch.cuda.synchronize()
    with pytest.raises(EngineError) as ei:
        mk_llama.check()
    return ei.value.status


def healthy_step_still_works(tiny_gpu):
    import mk_llama

    s = prepare(tiny_gpu, 300, cases.step_hidden(2048, 300))
    run_gpu(s)
    mk_llama.check()
    assert torch.isfinite(s.globs.logits.float()).all()


def test_missing_producer_times_out(tiny_gpu):
    s = prepare(tiny_gpu, 300, cases.step_hidden(2048, 300))
    instrs = s.get_linear_instructions()
    # drop the first QKV instruction of layer 0: its heads never complete
    instrs = [NoOp() if i == 0 else ins for i, ins in enumerate(instrs)]
    st = status_after(s, instrs)
    assert st["code"] == 1 and st["layer"] == 0
    assert st["observed"] < st["expected"]
    healthy_step_still_works(tiny_gpu)


@dataclass
class Bogus(Instruction):
    x: int

    @classmethod
    def opcode(cls):
        return 42


def test_bad_opcode_reported(tiny_gpu):
    s = prepare(tiny_gpu, 5, cases.step_hidden(2048, 5))
    st = status_after(s, [Bogus(1)] + s.get_linear_instructions())
    assert st["code"] == 2 and st["opcode"] == 42
    healthy_step_still_works(tiny_gpu)


def test_out_of_range_field_reported(tiny_gpu):
    s = prepare(tiny_gpu, 5, cases.step_hidden(2048, 5))
    st = status_after(s, s.get_linear_instructions() + [O_ProjResidual(99, 0, 1, 0)])
    assert st["code"] == 3 and st["expected"] == 1  # word 1 (layer) is out of range
    healthy_step_still_works(tiny_gpu)
