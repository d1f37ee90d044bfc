"""B200-native EXL3 packed-weight matmul: Python face of the libexl3cu C ABI.

The compute lives in hand-written sm_100a CUDA (``csrc/``) behind
``include/exl3cu.h``; this package binds it for tests, benchmarks and
torch-based callers.  Importing it does not touch the GPU; the first call
loads ``libexl3cu.so`` and fails loudly if it is missing.
"""
from . import format, synthetic  # noqa: F401
from ._lib import (CB_3INST, CB_MCG, CB_MUL1, F16, F32, Exl3Error,  # noqa: F401
                   Exl3InvalidArgument, lib)

__all__ = ["format", "synthetic", "lib", "Exl3Error", "Exl3InvalidArgument", "CB_3INST", "CB_MCG", "CB_MUL1",
           "F16", "F32"]


def __getattr__(name):
    # ops imports torch; load it on first use only
    if name in ("ops", "Exl3Weight"):
        import importlib

        mod = importlib.import_module(".ops", __name__)
        return mod if name == "ops" else mod.Exl3Weight
    if name in ("model", "Exl3Model"):
        import importlib

        mod = importlib.import_module(".model", __name__)
        return mod if name == "model" else mod.Exl3Model
    raise AttributeError(name)
