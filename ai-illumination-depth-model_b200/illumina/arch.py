"""Layer table and cost model: the Python face of src/model/arch.ts.

`buildArchitecture`, `costOf`, `formatCost` and `ILLUMINA_DEPTH_448` keep the
reference's names and meaning; the table itself comes from the native library
(illumina_arch_json), so the runtime and this API cannot drift apart.
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass, field
from functools import lru_cache

from ._lib import check, lib


@dataclass(frozen=True)
class TensorShape:
    h: int
    w: int
    c: int


@dataclass(frozen=True)
class Op:
    kind: str
    name: str
    out: str
    inp: str | None = None
    k: int = 0
    stride: int = 0
    act: str = "linear"
    midAct: str = "linear"
    residual: str | None = None
    coarse: str | None = None
    skip: str | None = None


@dataclass(frozen=True)
class Architecture:
    name: str
    inputSize: int
    mean: tuple
    std: tuple
    tensors: dict = field(default_factory=dict)
    ops: tuple = ()


def _json(fn, size: int) -> dict:
    need = C.c_size_t(0)
    check(fn(size, None, 0, C.byref(need)))
    buf = C.create_string_buffer(need.value)
    check(fn(size, buf, need.value, C.byref(need)))
    return json.loads(buf.value.decode("utf-8"))


@lru_cache(maxsize=None)
def _arch_doc(size: int) -> dict:
    return _json(lib().illumina_arch_json, size)


def buildArchitecture(inputSize: int) -> Architecture:
    """buildArchitecture (arch.ts:191-385). Raises ValueError unless inputSize is a multiple of 32."""
    from ._lib import IlluminaError
    try:
        d = _arch_doc(int(inputSize))
    except IlluminaError as e:
        raise ValueError(str(e)) from None
    tensors = {n: TensorShape(*s) for n, s in d["tensors"].items()}
    ops = tuple(Op(kind=o["kind"], name=o["name"], out=o["out"], inp=o.get("in"), k=o.get("k", 0),
                   stride=o.get("stride", 0), act=o.get("act", "linear"),
                   midAct=o.get("midAct", "linear"), residual=o.get("residual"),
                   coarse=o.get("coarse"), skip=o.get("skip")) for o in d["ops"])
    return Architecture(d["name"], d["inputSize"], tuple(d["mean"]), tuple(d["std"]), tensors, ops)


@dataclass(frozen=True)
class OpCost:
    name: str
    kind: str
    macs: int
    params: int
    outShape: TensorShape


@dataclass(frozen=True)
class ArchCost:
    ops: tuple
    totalMacs: int
    totalParams: int
    dispatches: int
    _naive_vec4: int

    def naiveTensorBytes(self, bytesPerElement: int) -> int:
        return self._naive_vec4 * 4 * bytesPerElement


def costOf(arch: Architecture) -> ArchCost:
    """costOf (arch.ts:415-489)."""
    d = _arch_doc(arch.inputSize)
    ops = tuple(OpCost(c["name"], c["kind"], c["macs"], c["params"], arch.tensors[o.out])
                for c, o in zip(d["cost"], arch.ops))
    naive = sum(s.h * s.w * s.c // 4 for s in arch.tensors.values())
    return ArchCost(ops, d["totalMacs"], d["totalParams"], len(arch.ops), naive)


def formatCost(arch: Architecture) -> str:
    """Human-readable cost report (arch.ts:492-530), without the M1 projection."""
    cost = costOf(arch)
    lines = [f"{arch.name} — {arch.inputSize}×{arch.inputSize}", "",
             f"{'op':<20}{'kind':<13}{'out h×w×c':>16}{'MFLOP':>10}{'params':>10}", "─" * 69]
    for c in cost.ops:
        s = f"{c.outShape.h}×{c.outShape.w}×{c.outShape.c}"
        lines.append(f"{c.name:<20}{c.kind:<13}{s:>16}{c.macs * 2e-6:>10.1f}{c.params:>10}")
    lines += ["─" * 69, f"{'TOTAL':<33}{'':>16}{cost.totalMacs * 2e-6:>10.1f}{cost.totalParams:>10}", "",
              f"dispatches            : {cost.dispatches}",
              f"GFLOP / frame         : {cost.totalMacs * 2e-9:.3f}",
              f"parameters            : {cost.totalParams / 1e6:.2f} M"]
    return "\n".join(lines)


def weightSpecs(arch: Architecture) -> list:
    """weightSpecs (weights.ts:29-63): [(name, shape), ...] in blob order."""
    return [(n, tuple(s)) for n, s in _arch_doc(arch.inputSize)["specs"]]


def __getattr__(name):
    # ILLUMINA_DEPTH_448 (arch.ts:388), built on first access (it needs the library)
    if name == "ILLUMINA_DEPTH_448":
        return buildArchitecture(448)
    raise AttributeError(name)
