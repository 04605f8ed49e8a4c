"""CPU oracle for the IlluminaDepth hot path.

TEST INFRASTRUCTURE ONLY. This package restates the reference's normative CPU
implementation (src/model/reference.ts, src/model/weights.ts,
src/engine/arena.ts, src/model/arch.ts) and, for the shading pass that the
reference only ships as a GPU shader, src/lighting/shade.ts and
src/lighting/composite.ts. It exists to check the CUDA product:

  * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
    import it, and only as the checker or the timed CPU baseline;
  * the product library and its Python host never import it.

Parity pins: the network ops, container and arch table are checked against
fixtures generated from the reference's own Python twin and exporter
(tests/golden/make_golden.py); the PRNG (mulberry32) is integer-exact; the
shading restatement has no reference CPU counterpart to pin against and is
checked against the reference tests' closed forms and invariants.
"""
import ctypes
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build() -> str:
    """Compiles liboracle.so in place (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        from . import _sigs
        _sigs.declare(_lib)
    return _lib
