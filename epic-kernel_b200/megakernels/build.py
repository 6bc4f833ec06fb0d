"""Build libek.so in-tree for sm_100a (nvcc, no JIT cache).

    python -m megakernels.build [--force]

The library is written next to mk_llama.py so that it travels with the source
tree and is found by `megakernels.ek`.
"""

import argparse
import os
import shutil
import subprocess
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
CSRC = PKG_ROOT / "csrc"
OUT = PKG_ROOT / "libek.so"
# ek_decode.cu is compiled once per kernel variant (model x prefetch paths),
# so that each kernel carries only the code its model runs.
VARIANTS = [
    ("llama", {"EK_MODEL": 0, "EK_PF": 0}),
    ("llama_pf", {"EK_MODEL": 0, "EK_PF": 1}),
    ("mixtral", {"EK_MODEL": 1, "EK_PF": 0}),
    ("mixtral_pf", {"EK_MODEL": 1, "EK_PF": 1}),
]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMPILE_FLAGS = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC"]
LINK_FLAGS = [*ARCH, "-shared", "-cudart", "static"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps.append(PKG_ROOT.parent / "include" / "ek.h")
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return OUT
    from concurrent.futures import ThreadPoolExecutor

    nvcc = nvcc_path()
    objdir = PKG_ROOT / "_build"
    objdir.mkdir(exist_ok=True)
    jobs = []
    for name, macros in VARIANTS:
        defs = [f"-D{k}={v}" for k, v in macros.items()] + [f"-DEK_NS={name}"]
        jobs.append([nvcc, *COMPILE_FLAGS, *defs, "-c", "-o", str(objdir / f"ek_decode_{name}.o"),
                     str(CSRC / "ek_decode.cu")])
    jobs.append([nvcc, *COMPILE_FLAGS, "-c", "-o", str(objdir / "ek_capi.o"), str(CSRC / "ek_capi.cu")])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True, cwd=PKG_ROOT)

    with ThreadPoolExecutor(max_workers=len(jobs)) as ex:
        list(ex.map(run, jobs))
    tmp = OUT.with_suffix(".so.tmp")
    objs = [str(objdir / f"ek_decode_{n}.o") for n, _ in VARIANTS] + [str(objdir / "ek_capi.o")]
    run([nvcc, *LINK_FLAGS, "-o", str(tmp), *objs])
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True))
