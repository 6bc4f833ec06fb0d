"""Host-side logic of Mixtral tensor parallelism, on CPU: shards reassemble to
the full model, and the IPC-handle exchange over torch.distributed (gloo,
world size 2) returns every rank's handle in rank order."""

import os
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from megakernels.mixtral.model import MixtralConfig, MixtralForCausalLM
from megakernels.model_types import ExtraModelConfig


def test_shards_reassemble_full_model():
    cfg = MixtralConfig(**cases.MIXTRAL_SMALL)
    ex = ExtraModelConfig(interleave_rope=True, max_len_override=64)
    full = MixtralForCausalLM.random_init(cfg, ex)
    world = 2
    sh = [MixtralForCausalLM.random_init(cfg, ex, tp=(r, world)) for r in range(world)]
    fp = full.stacked_params
    D = full.config.head_dim
    qd, kd = cfg.num_attention_heads * D, cfg.num_key_value_heads * D
    q = torch.cat([s.stacked_params.qkv_proj[:, : qd // world] for s in sh], 1)
    k = torch.cat([s.stacked_params.qkv_proj[:, qd // world : (qd + kd) // world] for s in sh], 1)
    v = torch.cat([s.stacked_params.qkv_proj[:, (qd + kd) // world :] for s in sh], 1)
    assert torch.equal(torch.cat([q, k, v], 1), fp.qkv_proj)
    assert torch.equal(torch.cat([s.stacked_params.o_proj for s in sh], 2), fp.o_proj)
    assert torch.equal(torch.cat([s.stacked_params.expert_gate for s in sh], 2), fp.expert_gate)
    assert torch.equal(torch.cat([s.stacked_params.expert_up for s in sh], 2), fp.expert_up)
    assert torch.equal(torch.cat([s.stacked_params.expert_down for s in sh], 3), fp.expert_down)
    assert torch.equal(torch.cat([s.lm_head.lm_head.weight for s in sh], 0), full.lm_head.lm_head.weight)
    for s in sh:
        assert torch.equal(s.stacked_params.router_weight, fp.router_weight)
        assert torch.equal(s.model.embed_tokens.embed_tokens.weight, full.model.embed_tokens.embed_tokens.weight)
        assert s.config.head_dim == D
        assert s.stacked_kv_cache[0].shape[3] == cfg.num_key_value_heads // world


def _exchange_worker(rank, world, init_file, out_file):
    import sys

    sys.path[:0] = [p for p in os.environ.get("EK_TEST_PATHS", "").split(os.pathsep) if p]
    from megakernels.mixtral.tp import exchange_handles

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        got = exchange_handles(bytes([rank]) * 64, world)
        if rank == 0:
            with open(out_file, "wb") as f:
                f.write(got)
    finally:
        dist.destroy_process_group()


def test_handle_exchange_gloo_two_ranks():
    import sys

    os.environ["EK_TEST_PATHS"] = os.pathsep.join(sys.path[:4])
    with tempfile.TemporaryDirectory() as d:
        init, out = os.path.join(d, "init"), os.path.join(d, "out")
        mp.spawn(_exchange_worker, args=(2, init, out), nprocs=2, join=True)
        data = open(out, "rb").read()
    assert data == bytes([0]) * 64 + bytes([1]) * 64
