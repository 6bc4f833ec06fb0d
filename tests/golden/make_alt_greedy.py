"""Free-running greedy stream of the Llama-1B oracle with a different (equally
valid) fp32 summation order in every matvec, from the prompt of
llama1b_decode192.npz. It measures how long two correct implementations that
differ only in summation order agree: the GPU engine's stream is required to
match the reference's at least as long as this one does.

    python tests/golden/make_alt_greedy.py   (CPU, about 20 minutes)
"""

import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (ROOT / "epic-kernel_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

from megakernels.demos.latency.scheduler import LatencyScheduleBuilder  # noqa: E402
from megakernels.llama import LlamaForCausalLM, llama_3_2_1b_config  # noqa: E402
from megakernels.model_types import ExtraModelConfig  # noqa: E402
from oracle import pyvm  # noqa: E402


def main():
    gold = np.load(HERE / "llama1b_decode192.npz")
    prompt = gold["prompt"]
    ntok = len(gold["greedy_tokens"])
    P = len(prompt)
    model = LlamaForCausalLM.random_init(
        llama_3_2_1b_config(), ExtraModelConfig(interleave_rope=True, max_len_override=256), seed=0)
    sched = LatencyScheduleBuilder.build(model, seq_len=P + ntok)
    instrs = sched.get_linear_instructions()
    pyvm.matvec = lambda mat, vec: (mat.float() @ vec.float()).to(mat.dtype)
    torch.set_num_threads(torch.get_num_threads())
    cur, out, t0 = int(prompt[0]), [], time.time()
    with torch.no_grad():
        for pos in range(P + ntok - 1):
            _, nxt = pyvm.pyvm_step(model, sched.globs, instrs, cur, pos)
            if pos + 1 < P:
                cur = int(prompt[pos + 1])
            else:
                out.append(nxt)
                cur = nxt
            if pos % 32 == 0:
                print(f"pos {pos}: {time.time() - t0:.0f}s", flush=True)
    np.savez_compressed(HERE / "llama1b_alt_greedy.npz", alt_greedy_tokens=np.array(out, dtype=np.int64))
    ref = gold["greedy_tokens"]
    agree = next((i for i in range(ntok) if out[i] != ref[i]), ntok)
    print(f"reordered-summation oracle agrees with the reference for {agree} of {ntok} tokens")


if __name__ == "__main__":
    main()
