"""Mode -> schedule builder / megakernel interpreter maps
(`megakernels/dispatch.py` of epic-kernel, :20-51).

Modes: "latency" (Llama-3.2-1B), "latency_3b" (Llama-3.2-3B), "mixtral_latency"
(Mixtral-8x7B). The reference's
"throughput" (batch-1024 VM) mode is outside this engine. The CPU reference
interpreter (PyVM) is test infrastructure and lives in `oracle/`, not here.
"""

from pathlib import Path

from megakernels.demos.latency.mk import Latency3B_MK_Interpreter, LatencyMK_Interpreter
from megakernels.demos.latency.scheduler import LatencyScheduleBuilder
from megakernels.mixtral.mk import MixtralMK_Interpreter
from megakernels.mixtral.scheduler import MixtralLatencyScheduleBuilder
from megakernels.mk import MK_Interpreter
from megakernels.scheduler import ScheduleBuilder

BUILDER_MAP = {
    "latency": LatencyScheduleBuilder,
    "latency_3b": LatencyScheduleBuilder,
    "mixtral_latency": MixtralLatencyScheduleBuilder,
}

MK_INTERPRETER_MAP = {
    "latency": LatencyMK_Interpreter,
    "latency_3b": Latency3B_MK_Interpreter,
    "mixtral_latency": MixtralMK_Interpreter,
}


def make_schedule_builder(mode: str) -> ScheduleBuilder:
    return BUILDER_MAP[mode]()


def make_mk_interpreter(mode: str, mk_dir: Path | str | None = None, **options) -> MK_Interpreter:
    return MK_INTERPRETER_MAP[mode](mk_dir, **options)
