"""Shared helpers of the GPU parity tests: run one decode step of a model
through the megakernel (mk_llama via the C ABI) and through the CPU oracle on
identical inputs."""

import json
import os

import torch

import cases
from megakernels.demos.latency.mk import LatencyMK_Interpreter
from megakernels.demos.latency.scheduler import LatencyScheduleBuilder
from megakernels.scheduler import assign_to_sms, tensorize_instructions
from oracle import pyvm


def prepare(model, pos: int, hidden: torch.Tensor, fill=True, **build_kw):
    sched = LatencyScheduleBuilder.build(model, seq_len=pos, **build_kw)
    g = sched.globs
    if fill:
        cases.fill_kv(g.k_cache, g.v_cache, pos)
    g.hidden_states[:] = hidden.to(g.hidden_states.device)
    return sched


def run_gpu(sched, mode="rr", **options):
    g = sched.globs
    tensorize_instructions(g, assign_to_sms(mode, schedule=sched))
    g.barriers.zero_()
    LatencyMK_Interpreter(**options).interpret(g)
    torch.cuda.synchronize()


def run_oracle(sched):
    with torch.no_grad():
        pyvm.interpret(sched.globs, sched.get_linear_instructions())


def bf16_from_bits(a):
    return torch.from_numpy(a).view(torch.bfloat16)


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in bf16 ulps (sign-magnitude bit patterns)."""
    ia = a.to(torch.bfloat16).view(torch.int16).int()
    ib = b.to(torch.bfloat16).view(torch.int16).int()
    ia = torch.where(ia < 0, -32768 - ia, ia)
    ib = torch.where(ib < 0, -32768 - ib, ib)
    return (ia - ib).abs()


def _reordered_matvec(mat, vec):
    return (mat.float() @ vec.float()).to(mat.dtype)


def noise_floor(model_cpu, pos, hidden, **build_kw):
    """Logits of the oracle and of the same oracle with a different fp32
    summation order in every matvec (a second, equally valid rounding of the
    reference interpreter). Their difference is the disagreement any
    implementation that does not replicate the CPU's summation order must be
    allowed."""
    a = prepare(model_cpu, pos, hidden, **build_kw)
    run_oracle(a)
    b = prepare(model_cpu, pos, hidden, **build_kw)
    saved = pyvm.matvec
    pyvm.matvec = _reordered_matvec
    try:
        run_oracle(b)
    finally:
        pyvm.matvec = saved
    return a, b


LOGIT_TOL = 2e-2  # x std(logits), the parity target


def assert_logits_within_floor(mine, ref, alt):
    """max and RMS |mine - ref| must each stay within max(target, 2 x floor),
    where floor = |alt - ref| (alt: reordered-summation oracle)."""
    mine, ref, alt = mine.float().cpu(), ref.float().cpu(), alt.float().cpu()
    sd = ref.std().item()
    d, f = (mine - ref).abs(), (alt - ref).abs()
    max_bound = max(LOGIT_TOL * sd, 2 * f.max().item())
    rms_bound = max(LOGIT_TOL * sd, 2 * f.pow(2).mean().sqrt().item())
    assert d.max().item() <= max_bound, f"max |dlogit| {d.max().item():.4g} > {max_bound:.4g}"
    rms = d.pow(2).mean().sqrt().item()
    assert rms <= rms_bound, f"rms |dlogit| {rms:.4g} > {rms_bound:.4g}"
    return d.max().item() / sd, rms / sd


def record_parity(case: str, **values):
    """Print a parity measurement and, when EK_PARITY_LOG names a file, append
    it there as one JSON line (the source of the committed parity table)."""
    line = {"case": case, **values}
    print("parity", json.dumps(line))
    path = os.environ.get("EK_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(line) + "\n")
