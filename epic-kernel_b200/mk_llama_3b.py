"""`mk_llama_3b`: the Llama-3.2-3B entry point of epic-kernel
(demos/low-latency-llama/llama_3b.cu:26-53). The engine reads the model size
from the tensor shapes, so this is the same launcher as `mk_llama`."""

from mk_llama import check, mk_llama, read_status

mk_llama_3b = mk_llama

__all__ = ["mk_llama_3b", "check", "read_status"]
