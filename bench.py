"""Batch-1 decode benchmark: Llama-3.2-1B (random-init bf16) at KV length 2048.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--kv 2048] [--model 1b|3b|mixtral] [--prefetch S]

A step is one decode token through `MK_Generator.run`: barrier reset and one
megakernel launch over the whole model (for Llama the embedding gather and
the argmax run inside the megakernel; Mixtral adds them as torch ops). The output token feeds the next step, as in
MK_Generator.generate. Weights (2.47 GB) are far larger than L2 (126 MB), so
no L2 flush is needed between steps.

One JSON line is printed by rank 0:
- `value`: tokens/s with all inputs resident in HBM (device-timed, CUDA events,
  max over ranks). For N > 1 each Llama rank runs an independent replica, so
  the scaling is weak and `value` sums over ranks; Mixtral runs tensor
  parallel over the N GPUs (one token stream, strong scaling, in-kernel
  NVLink all-reduce), so `value` is that stream's tokens/s.
- `e2e`: the same metric through the public API with host buffers. Every step
  copies the input token from pinned host memory and reads the output token
  back to the host.
- `roofline`: HBM-bound. `achieved` is the algorithmic bytes per launch
  (weights read once + KV rows read) over the mean megakernel launch time,
  and `peak` is MEASURED_PEAKS.json hbm_gbs.
- `cpu_baseline`: the CPU oracle (a port of the reference's PyVM) timed on a
  bounded sample on this host.

`--impl reference` times the reference's CPU interpreter path (the oracle
port; the reference's CUDA megakernel cannot be built because its
ThunderKittens dependency is not vendored) on the same workload and metric.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT / "epic-kernel_b200", ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import torch  # noqa: E402

METRIC = "batch-1 decode tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--kv", type=int, default=2048)
    ap.add_argument("--model", default="1b", choices=["1b", "3b", "mixtral"])
    ap.add_argument("--prefetch", type=int, default=0, help="L2 prefetch stages (0 = off)")
    ap.add_argument("--cpu-sample-tokens", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-spec", action="store_true", help="Mixtral: schedule without SpeculativeExpertPredict")
    ap.add_argument("--mixtral-tp-steps", type=int, default=64,
                    help="with --gpus N > 1: also decode Mixtral 8x7B tensor parallel over the N GPUs")
    ap.add_argument("--mixtral-tp-kv", type=int, default=4096)
    ap.add_argument("--per-opcode", action="store_true",
                    help="HBM bandwidth of each instruction type in isolation (one JSON line each)")
    ap.add_argument("--per-opcode-reps", type=int, default=20)
    return ap.parse_args()


def model_config(name):
    from megakernels.llama import llama_3_2_1b_config, llama_3_2_3b_config
    from megakernels.mixtral.model import MixtralConfig

    return {"1b": llama_3_2_1b_config, "3b": llama_3_2_3b_config, "mixtral": MixtralConfig}[name]()


def build_model(name, max_len, device, tp=None):
    from megakernels.llama import LlamaForCausalLM
    from megakernels.mixtral.model import MixtralForCausalLM
    from megakernels.model_types import ExtraModelConfig

    extra = ExtraModelConfig(interleave_rope=True, max_len_override=max_len)
    if name == "mixtral":
        # 46.7 B parameters: drawn on the device (host draws take minutes)
        host = torch.device(device).type == "cpu"
        return MixtralForCausalLM.random_init(model_config(name), extra, seed=0, device=device, host_rng=host,
                                              tp=tp)
    return LlamaForCausalLM.random_init(model_config(name), extra, seed=0, device=device)


def builder_and_interp(name, prefetch, tp=False):
    if name == "mixtral" and tp:
        from megakernels.mixtral.scheduler import MixtralLatencyScheduleBuilder
        from megakernels.mixtral.tp import MixtralTPMK_Interpreter

        return MixtralLatencyScheduleBuilder, MixtralTPMK_Interpreter(l2_prefetch_stages=prefetch)
    if name == "mixtral":
        from megakernels.mixtral.mk import MixtralMK_Interpreter
        from megakernels.mixtral.scheduler import MixtralLatencyScheduleBuilder

        return MixtralLatencyScheduleBuilder, MixtralMK_Interpreter(l2_prefetch_stages=prefetch)
    from megakernels.demos.latency.mk import LatencyMK_Interpreter
    from megakernels.demos.latency.scheduler import LatencyScheduleBuilder

    return LatencyScheduleBuilder, LatencyMK_Interpreter(l2_prefetch_stages=prefetch)


def weight_bytes(model) -> int:
    """Weight bytes one decode step must read: every matrix once; for Mixtral
    only the k active experts of each layer (plus the router)."""
    sp = model.stacked_params
    nbytes = lambda t: t.numel() * t.element_size()  # noqa: E731
    lm = nbytes(model.lm_head.lm_head.weight)
    if hasattr(sp, "expert_gate"):
        c = model.config
        per_expert = (nbytes(sp.expert_gate) + nbytes(sp.expert_up) + nbytes(sp.expert_down)) // c.num_local_experts
        return (nbytes(sp.qkv_proj) + nbytes(sp.o_proj) + nbytes(sp.router_weight)
                + per_expert * c.num_experts_per_tok + lm)
    return sum(nbytes(t) for t in (sp.qkv_proj, sp.o_proj, sp.up_proj, sp.gate_proj, sp.down_proj)) + lm


def kv_bytes_per_token(model) -> int:
    c = model.config
    return c.num_hidden_layers * 2 * c.num_key_value_heads * c.head_dim * 2


def fill_kv(model, kv, rank=0):
    from megakernels.synthetic import seeded_normal

    k, v = model.stacked_kv_cache
    L, B, _, H, D = k.shape
    for i, c in enumerate((k, v)):
        c[:, :, :kv] = seeded_normal((L, B, kv, H, D), 1, 7000 + 16 * rank + i).to(c.device)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def read_profile_traffic(workload):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    f = ROOT / "profiles" / f"decode_kernel_{workload}.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=5)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxes.append(float(f[2]))
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


def cpu_decode_sample(name, kv, tokens):
    """Time `tokens` decode steps of the CPU oracle (a port of the reference
    PyVM) at KV length `kv`. Returns (tokens/s, threads, seconds, note).

    Mixtral (93 GB) does not fit a CPU run here: a 2-layer model of the full
    width is timed and its per-layer cost scaled to 32 layers (the note says
    so); the LM head is timed in full."""
    torch.set_num_threads(os.cpu_count() or 1)
    if name == "mixtral":
        return _cpu_mixtral_sample(kv, tokens)
    from megakernels.demos.latency.scheduler import LatencyScheduleBuilder
    from oracle import pyvm

    model = build_model(name, kv + tokens + 1, "cpu")
    fill_kv(model, kv)
    sched = LatencyScheduleBuilder.build(model, seq_len=kv + tokens)
    instrs = sched.get_linear_instructions()
    tok = 0
    with torch.no_grad():
        pyvm.pyvm_step(model, sched.globs, instrs, tok, kv - 1)  # warm-up (not timed)
        t0 = time.perf_counter()
        for i in range(tokens):
            _, tok = pyvm.pyvm_step(model, sched.globs, instrs, tok, kv + i)
        dt = time.perf_counter() - t0
    note = f"{tokens} decode token(s) of the full model at KV {kv}"
    return tokens / dt, torch.get_num_threads(), dt, note


def _cpu_mixtral_sample(kv, tokens):
    from megakernels.mixtral.model import MixtralConfig, MixtralForCausalLM
    from megakernels.mixtral.scheduler import MixtralLatencyScheduleBuilder
    from megakernels.model_types import ExtraModelConfig
    from oracle import pyvm_mixtral

    full = MixtralConfig()
    layers = 2
    cfg = MixtralConfig(**{**full.__dict__, "num_hidden_layers": layers})
    model = MixtralForCausalLM.random_init(cfg, ExtraModelConfig(interleave_rope=True,
                                                                  max_len_override=kv + tokens + 1), seed=0)
    fill_kv(model, kv)
    sched = MixtralLatencyScheduleBuilder.build(model, seq_len=kv + tokens)
    g = sched.globs
    instrs = sched.get_linear_instructions()
    emb = model.model.embed_tokens.embed_tokens.weight
    with torch.no_grad():
        def step(tok, pos):
            g.hidden_states[:] = emb[tok]
            g.barriers.zero_()
            g.logits.zero_()
            g.pos_id = pos
            pyvm_mixtral.interpret(g, instrs)
            return int(torch.argmax(g.logits))

        tok = step(0, kv - 1)  # warm-up (not timed)
        t0 = time.perf_counter()
        for i in range(tokens):
            tok = step(tok, kv + i)
        dt = time.perf_counter() - t0
    # split the step into layers and LM head: time the LM head alone
    lm = [ins for ins in instrs if ins.opcode() == 7]
    with torch.no_grad():
        t1 = time.perf_counter()
        for ins in lm:
            pyvm_mixtral.SOLVERS[7](g, ins)
        lm_s = time.perf_counter() - t1
    per_layer = (dt / tokens - lm_s) / layers
    per_token = per_layer * full.num_hidden_layers + lm_s
    note = (f"{tokens} decode token(s) of a {layers}-layer full-width Mixtral at KV {kv} "
            f"({dt:.1f} s); per-layer time x {full.num_hidden_layers} layers + LM head, scaled, not measured "
            f"on the 32-layer model (93 GB does not fit host memory)")
    return 1.0 / per_token, torch.get_num_threads(), dt, note


def dist_setup(n):
    if n <= 1 and "RANK" not in os.environ:
        return 0, 1, 0
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", n))
    local = int(os.environ.get("LOCAL_RANK", rank))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29511")
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local))
    else:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    return rank, world, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def workload_name(model, kv):
    return f"mixtral-8x7b-kv{kv}-decode" if model == "mixtral" else f"llama-3.2-{model}-kv{kv}-decode"


def run_reference(args, rank, world):
    if rank != 0:
        return
    samples = max(1, min(args.steps, args.cpu_sample_tokens))
    tps, cores, dt, note = cpu_decode_sample(args.model, args.kv, samples)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": samples, "warmup": 1, "ms_per_step": 1000.0 / tps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02) seed 0; KV N(0,1) seed 1)",
        "config": {"workload": workload_name(args.model, args.kv), "kv_len": args.kv, "batch": 1},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{note}, {dt:.1f} s, CPU port of the reference PyVM (reference CUDA "
                                   f"megakernel unbuildable: ThunderKittens not vendored)"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def decode_leg(model_name, kv, steps, warmup, prefetch, rank, world, local, tp, with_e2e=True, spec=True):
    """Decode `steps` tokens after `warmup` untimed ones through MK_Generator.run
    (device-resident leg), then the same through the public API with host
    buffers (e2e leg). Returns the timings and byte counts."""
    import mk_llama
    from megakernels.generators import MK_Generator
    from megakernels.scheduler import assign_to_sms, tensorize_instructions

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    total = warmup + steps
    max_len = kv + 2 * total + 16
    model = build_model(model_name, max_len, dev, tp=(rank, world) if tp else None)
    fill_kv(model, kv, rank)
    builder, interp = builder_and_interp(model_name, prefetch, tp)
    if model_name == "mixtral" and not spec:
        from megakernels.mixtral.scheduler import MixtralNoSpeculationScheduleBuilder as builder
    sched = builder.build(model, seq_len=kv + 2 * total)
    if tp:
        from megakernels.mixtral.tp import setup_tensor_parallel

        setup_tensor_parallel(sched.globs, rank, world)
    tensorize_instructions(sched.globs, assign_to_sms("rr", schedule=sched))
    gen = MK_Generator(model, interp, sched)
    stream = torch.cuda.current_stream(dev)
    tok = torch.zeros(1, 1, dtype=torch.long, device=dev)
    pos = kv
    out = {}
    with torch.no_grad():
        # ---- device-resident leg: tokens stay on the GPU
        for _ in range(warmup):
            tok = gen.run(tok, pos).view(1, 1)
            pos += 1
        torch.cuda.synchronize()
        mk_llama.check(local)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        kv_lens = []
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            t_start.record(stream)
            for i in range(steps):
                starts[i].record(stream)
                tok = gen.run(tok, pos).view(1, 1)
                ends[i].record(stream)
                kv_lens.append(pos + 1)
                pos += 1
            t_end.record(stream)
            torch.cuda.synchronize()
        barrier(world)
        mk_llama.check(local)
        out["step_ms"] = max_over_ranks(t_start.elapsed_time(t_end) / steps, world)
        out["kernel_ms"] = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
        out["clocks"] = clocks.summary()
        out["alg_bytes"] = weight_bytes(model) + kv_bytes_per_token(model) * statistics.mean(kv_lens)

        if with_e2e:
            # ---- end-to-end leg through the public API with host buffers
            h_in = torch.zeros(1, 1, dtype=torch.long).pin_memory()
            h_out = torch.zeros(1, dtype=torch.long).pin_memory()
            d_in = torch.zeros(1, 1, dtype=torch.long, device=dev)

            def e2e_step(p):
                d_in.copy_(h_in, non_blocking=True)
                h_out.copy_(gen.run(d_in, p).view(-1), non_blocking=True)
                stream.synchronize()
                h_in[0, 0] = h_out[0]  # the host reads the result before the next step

            for _ in range(2):
                e2e_step(pos)
                pos += 1
            barrier(world)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                e2e_step(pos)
                pos += 1
            e1.record(stream)
            torch.cuda.synchronize()
            out["e2e_ms"] = max_over_ranks(e0.elapsed_time(e1) / steps, world)
            mk_llama.check(local)
    del gen, sched, model
    torch.cuda.empty_cache()
    return out


def run_ours(args, rank, world, local):
    tp = args.model == "mixtral" and world > 1  # Mixtral shards; Llama runs replicas
    leg = decode_leg(args.model, args.kv, args.steps, args.warmup, args.prefetch, rank, world, local, tp,
                     spec=not args.no_spec)
    peak, peak_kind = load_peaks()
    achieved = leg["alg_bytes"] / (leg["kernel_ms"] * 1e-3) / 1e9

    # the sharded path on the same GPUs: Mixtral tensor parallel over all ranks
    mixtral_tp = None
    if world > 1 and args.model != "mixtral" and args.mixtral_tp_steps > 0:
        m = decode_leg("mixtral", args.mixtral_tp_kv, args.mixtral_tp_steps, 3, 0, rank, world, local, True)
        ach = m["alg_bytes"] / (m["kernel_ms"] * 1e-3) / 1e9
        mixtral_tp = {"workload": workload_name("mixtral", args.mixtral_tp_kv), "parallelism": f"tp{world}",
                      "steps": args.mixtral_tp_steps, "ms_per_token": m["step_ms"],
                      "tokens_per_s": 1000.0 / m["step_ms"], "e2e_tokens_per_s": 1000.0 / m["e2e_ms"],
                      "ms_per_token_kernel": m["kernel_ms"],
                      "roofline_per_gpu": {"achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                                           "algorithmic_bytes_per_launch": m["alg_bytes"]},
                      "clocks": m["clocks"]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, cores, dt, note = cpu_decode_sample(args.model, args.kv, args.cpu_sample_tokens)
        cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{note} through the CPU port of the reference PyVM ({dt:.1f} s)"}
    if rank != 0:
        return
    workload = workload_name(args.model, args.kv)
    streams = 1 if tp else world  # token streams the job decodes at once
    line = {
        "metric": METRIC, "value": streams * 1000.0 / leg["step_ms"], "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": leg["step_ms"],
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02) seed 0; KV N(0,1) seed 1)",
        "config": {"workload": workload, "kv_len": args.kv, "batch": 1,
                   "parallelism": (f"tp{world}" if tp else f"replicas{world}") if world > 1 else "single",
                   "l2_prefetch_stages": args.prefetch,
                   "speculative_prediction": (not args.no_spec) if args.model == "mixtral" else None,
                   "l2": "no flush: the weights read per step (>= 2.5 GB) exceed the 126 MB L2"},
        "gpu_launches": args.steps,
        "ms_per_token_kernel": leg["kernel_ms"],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": leg["alg_bytes"],
                     "scope": "per GPU: this rank's shard" if tp else "per GPU",
                     "traffic": read_profile_traffic(workload)},
        "clocks": leg["clocks"],
        "e2e": {"value": streams * 1000.0 / leg["e2e_ms"], "unit": "tokens/s",
                "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
        "cpu_baseline": cpu,
    }
    if mixtral_tp is not None:
        line["mixtral_tp"] = mixtral_tp
    print(json.dumps(line), flush=True)


OPCODE_NAMES = {1: "LayerNorm_QKV_MatVecRopeAppend", 2: "PartialAttention", 3: "AttentionReduction",
                4: "O_ProjResidual", 5: "LayerNormDoubleMatVecSiLU", 6: "DownProjResidual", 7: "RMS_LM_Head"}


def run_per_opcode(args, local):
    """Achieved HBM bandwidth per instruction type (Llama or Mixtral): for each opcode, a
    launch whose queues hold only that opcode's instructions of every layer
    (dealt round-robin), with all counters preset so that no instruction waits.
    One JSON line per opcode: bytes the instructions must read, mean launch
    time (CUDA events), GB/s and fraction of the measured HBM peak."""
    import mk_llama
    from megakernels.scheduler import round_robin_assign_to_sms, tensorize_instructions

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    model = build_model(args.model, args.kv + 64, dev)
    fill_kv(model, args.kv)
    builder, interp = builder_and_interp(args.model, args.prefetch)
    sched = builder.build(model, seq_len=args.kv)
    g = sched.globs
    linear = sched.get_linear_instructions()
    c = model.config
    sp = model.stacked_params
    nb = lambda t: t.numel() * t.element_size()  # noqa: E731
    D, kv_rows = c.head_dim, args.kv + 1
    kv_bytes = c.num_hidden_layers * 2 * c.num_key_value_heads * D * 2 * kv_rows
    parts = max(1, sum(1 for i in linear if i.opcode() == 2) // (c.num_hidden_layers * c.num_key_value_heads))
    bytes_of = {1: nb(sp.qkv_proj), 2: kv_bytes, 3: c.num_hidden_layers * c.num_attention_heads * parts * (D + 1) * 4,
                4: nb(sp.o_proj), 7: nb(model.lm_head.lm_head.weight)}
    names = dict(OPCODE_NAMES)
    if args.model == "mixtral":  # the k selected experts of each layer, plus the router
        k, E = c.num_experts_per_tok, c.num_local_experts
        bytes_of[5] = (nb(sp.expert_gate) + nb(sp.expert_up)) * k // E + nb(sp.router_weight)
        bytes_of[6] = nb(sp.expert_down) * k // E
        bytes_of[8] = nb(sp.router_weight)
        names.update({5: "RmsRouterUpgate", 6: "ExpertDownProjFused", 7: "Mixtral_RMS_LM_Head",
                      8: "SpeculativeExpertPredict"})
    else:
        bytes_of[5] = nb(sp.up_proj) + nb(sp.gate_proj)
        bytes_of[6] = nb(sp.down_proj)
    peak, peak_kind = load_peaks()
    reps, warm = args.per_opcode_reps, (0 if args.per_opcode_reps == 1 else 3)
    stream = torch.cuda.current_stream(dev)
    for op in range(1, 9):
        instrs = [i for i in linear if i.opcode() == op]
        if not instrs:
            continue
        tensorize_instructions(g, round_robin_assign_to_sms(instrs, g.sm_count()))
        if op == 6 and args.model != "mixtral":  # as inside a full stream: partials left for the next layer
            g.deferrable_down_layers = c.num_hidden_layers - 1
        times = []
        for it in range(warm + reps):
            g.barriers.fill_(1 << 24)  # every wait is already satisfied
            g.pos_id = args.kv
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            interp.interpret(g)
            e1.record(stream)
            if it >= warm:
                times.append((e0, e1))
        torch.cuda.synchronize()
        mk_llama.check(local)
        us = statistics.mean(a.elapsed_time(b) for a, b in times) * 1e3
        gbs = bytes_of[op] / (us * 1e-6) / 1e9
        print(json.dumps({"per_opcode": op, "name": names[op], "workload": workload_name(args.model, args.kv),
                          "instructions": len(instrs), "layers": c.num_hidden_layers, "bytes": bytes_of[op],
                          "us_per_launch": us, "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak,
                          "peak_kind": peak_kind}), flush=True)


def main():
    args = parse()
    rank, world, local = dist_setup(args.gpus)
    if args.per_opcode:
        if rank == 0:
            run_per_opcode(args, local)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
