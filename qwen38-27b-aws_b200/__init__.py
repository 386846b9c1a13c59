"""B200 (sm_100a) implementation of the Qwen3.8 hybrid-decoder step, behind the reference's step API.

The package directory's name is not a Python identifier; import it with
``importlib.import_module("qwen38-27b-aws_b200")``.

Submodules: config (shapes), codec (FP8 formats), weights (synthetic weights and the TP cut),
build (compiles libq38.so), _lib (its ctypes binding), ops (one wrapper per C-ABI call),
step (B200Step / B200Head, the drop-in for the reference's NeuronStep / HeadStep graph).
"""

from . import codec, config, weights  # noqa: F401

__all__ = ["codec", "config", "weights"]
