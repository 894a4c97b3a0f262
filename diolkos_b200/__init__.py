"""diolkos_b200 -- the Diolkos batch-1 Q8_0 LLaMA decode path, B200-native.

The product is ``libdiolkos.so`` (sm_100a CUDA kernels behind the C ABI in include/diolkos.h,
plus the reference-compatible C API: transformer.h, safetensors.h, tensor.h, utils.h, sampler.h,
tokenizer.h).  This package holds its sources (csrc/), its build recipe (build.py), a ctypes
mirror of the C ABI (ops.py, model.py) and the seeded synthetic-checkpoint writer (synth.py).
"""
from . import synth  # noqa: F401  (pure numpy; no GPU needed)

__all__ = ["synth"]
