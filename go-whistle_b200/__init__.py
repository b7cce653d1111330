"""go-whistle_b200: go-whistle's quantized hot path on the NVIDIA B200.

The product is ``libwhistle_b200.so`` (CUDA C++ for sm_100a behind the C ABI
of ``include/whistle_b200.h``). This package is its host side in Python,
mirroring the reference's Go API for the path:

- ``cq``: ``Packed``, ``New``, ``Matrix`` (GEMV, GEMM, Rows, Row, Exact),
  ``GEMMs`` — internal/cq;
- ``needle``: ``QuantizeRow``, ``QuantizeRows``, ``Int8Rows``, ``AttendInt8``,
  ``AttendInt8Spans`` — internal/needle's int8 numerics;
- ``decoder``: ``Decoder`` (the device decode step and greedy loop) and
  ``HeadArgmax`` — internal/decoder;
- ``cact``: the .cact container (``Parse``, ``Open``, ``File``, the writer,
  ``whistle_names``) — internal/cact;
- ``weights``: tensors by name over a .cact file and the decoder's weight
  set loaded from one, a synthetic whistle.cact writer — internal/weights;
- ``synth``: seeded synthetic tensors in the reference's formats;
- ``dp``: data parallelism over independent streams (shards, gathering,
  missing-shard detection).

Import it by its directory name: ``importlib.import_module("go-whistle_b200")``.
"""

from . import _lib, cact, cq, decoder, dp, encoder, needle, synth, weights  # noqa: F401
from ._lib import CQError, CudaError, Panic, WhistleError  # noqa: F401

LIB_PATH = _lib.LIB_PATH


def build(force: bool = False, verbose: bool = False):
    """Compiles libwhistle_b200.so in-tree (nvcc, sm_100a)."""
    import importlib.util
    import sys

    name = __name__ + ".build"
    if name in sys.modules:
        mod = sys.modules[name]
    else:
        spec = importlib.util.spec_from_file_location(name, str(_lib.HERE / "build.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return mod.build(force=force, verbose=verbose)
