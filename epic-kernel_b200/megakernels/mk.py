"""Locating the compiled megakernel module (`megakernels/mk.py` of
epic-kernel, :5-17): `mk_dir` is put on sys.path and `mk_llama` imported from
it. For this engine `mk_dir` is the directory holding `mk_llama.py` and
`libek.so` (DEFAULT_MK_DIR)."""

import sys
from pathlib import Path

DEFAULT_MK_DIR = Path(__file__).resolve().parent.parent


def _add_to_path(mk_dir: Path | str | None):
    path = str(Path(mk_dir or DEFAULT_MK_DIR).expanduser().absolute())
    if path not in sys.path:
        sys.path.append(path)


def get_mk_func(mk_dir: Path | str | None = None):
    _add_to_path(mk_dir)
    from mk_llama import mk_llama  # type: ignore

    return mk_llama


class MK_Interpreter:
    def __init__(self, mk_dir: Path | str | None = None):
        self.mk_func = get_mk_func(mk_dir)

    def interpret(self, globs):
        raise NotImplementedError
