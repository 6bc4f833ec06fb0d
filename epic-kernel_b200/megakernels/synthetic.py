"""Seeded synthetic tensors, reproducible on any host.

Weights N(0, std) and KV-cache contents N(0, 1) are drawn with numpy's PCG64
generator, which gives the same bits on every platform; torch's CPU normal_
may take different vectorised code paths on different CPUs. Each tensor is
drawn in chunks of 2**24 elements. Chunk `c` of the tensor with id `tid` uses
`numpy.random.default_rng([seed, tid, c])`, so the chunks can be drawn on
several threads. Values are drawn in float32, scaled by `std` in float32, then
rounded to the target dtype (bf16 rounds to nearest even).
"""

from concurrent.futures import ThreadPoolExecutor
import os

import numpy as np
import torch

CHUNK = 1 << 24
_THREADS = max(1, min(16, os.cpu_count() or 1))


def _draw(seed: int, tid: int, chunk: int, n: int, std: float) -> np.ndarray:
    a = np.random.default_rng([seed, tid, chunk]).standard_normal(n, dtype=np.float32)
    if std != 1.0:
        a *= np.float32(std)
    return a


def seeded_normal(shape, seed: int, tid: int, std: float = 1.0, dtype=torch.bfloat16) -> torch.Tensor:
    """CPU tensor of `shape` with N(0, std) values, identical on every host."""
    numel = int(np.prod(shape)) if len(shape) else 1
    out = torch.empty(numel, dtype=dtype)
    starts = list(range(0, numel, CHUNK))

    def fill(i_start):
        i, start = i_start
        n = min(CHUNK, numel - start)
        out[start : start + n] = torch.from_numpy(_draw(seed, tid, i, n, std)).to(dtype)

    if len(starts) == 1:
        fill((0, 0))
    else:
        with ThreadPoolExecutor(_THREADS) as ex:
            list(ex.map(fill, enumerate(starts)))
    return out.view(*shape)


def seeded_randint(n: int, high: int, seed: int) -> torch.Tensor:
    """`n` token ids uniform in [0, high), int64."""
    return torch.from_numpy(np.random.default_rng([seed, 999_999]).integers(0, high, n)).long()
