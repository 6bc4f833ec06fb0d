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


def test_struct_sizes_match_header():
    # EkStatus: 8 int32; EkLlamaArgs: 23 pointers, 22 int32/float fields, padding, int64
    assert ctypes.sizeof(ek.EkStatus) == 32
    expect = 23 * 8 + 22 * 4
    expect = (expect + 7) // 8 * 8 + 8
    assert ctypes.sizeof(ek.EkLlamaArgs) == expect


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
