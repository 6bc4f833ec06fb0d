"""The C-ABI library loads and exports every function include/ek.h declares.
No compute call runs here (CPU-only host)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from megakernels import ek
from megakernels.build import build

build()  # no-op when libek.so is newer than its sources

HEADER = Path(__file__).resolve().parent.parent / "include" / "ek.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|void|const char\*)\s+(ek_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("ek_context_create", "ek_context_destroy", "ek_llama_decode", "ek_read_status",
                     "ek_last_error", "ek_abi_version"):
        assert required in names


def test_library_exports_all_declared_symbols():
    lib = ek.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} not exported by {ek.LIB_PATH}"
    assert lib.ek_abi_version() == ek.EK_ABI_VERSION


def _c_layout(struct: str, fields) -> dict:
    """sizeof and offsetof of `struct` as the C compiler lays out include/ek.h."""
    import shutil
    import subprocess
    import tempfile

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = [f'printf("size %zu\\n", sizeof({struct}));']
    lines += [f'printf("{f} %zu\\n", offsetof({struct}, {f}));' for f in fields]
    src = ("#include <stddef.h>\n#include <stdio.h>\n#include \"ek.h\"\nint main(void) {\n"
           + "\n".join(lines) + "\nreturn 0;\n}\n")
    with tempfile.TemporaryDirectory() as d:
        c, exe = Path(d) / "layout.c", Path(d) / "layout"
        c.write_text(src)
        subprocess.run([cc, "-I", str(HEADER.parent), "-o", str(exe), str(c)], check=True)
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.splitlines())}


@pytest.mark.parametrize("struct,cls", [("EkStatus", ek.EkStatus), ("EkLlamaArgs", ek.EkLlamaArgs),
                                        ("EkMixtralArgs", ek.EkMixtralArgs)])
def test_struct_layout_matches_header(struct, cls):
    names = [n for n, _ in cls._fields_]
    c = _c_layout(struct, names)
    assert ctypes.sizeof(cls) == c["size"]
    for n in names:
        assert getattr(cls, n).offset == c[n], n


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_context_create_fails_cleanly_without_gpu():
    lib = ek.load_library()
    h = ctypes.c_void_p()
    rc = lib.ek_context_create(0, ctypes.byref(h))
    assert rc != 0 and not h.value
    assert lib.ek_last_error()


def test_null_arguments_rejected():
    lib = ek.load_library()
    assert lib.ek_llama_decode(None, None, None) == 1
    assert b"NULL" in lib.ek_last_error()
