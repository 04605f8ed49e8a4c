"""Arena planner: the Python face of src/engine/arena.ts (planArena,
validateArena, opInputs). The plan is computed by the native runtime, the
same code that lays out the device arena.
"""
from __future__ import annotations

from dataclasses import dataclass

from ._lib import lib
from .arch import Architecture, Op, _json


@dataclass(frozen=True)
class ArenaPlan:
    bufferSizes: tuple   # vec4 elements per frame
    assignment: dict     # tensor -> buffer index
    totalBytes: int      # fp32, per frame
    naiveBytes: int


def opInputs(op: Op) -> list:
    """opInputs (arena.ts:19-33)."""
    if op.kind == "preprocess":
        return []
    if op.kind == "conv":
        return [op.inp]
    if op.kind in ("pw", "dwpw"):
        return [op.inp] + ([op.residual] if op.residual else [])
    if op.kind == "lateral":
        return [op.coarse, op.skip]
    return [op.inp]


def planArena(arch: Architecture, exclude=("depth",)) -> ArenaPlan:
    """planArena (arena.ts:57-128) with the runner's exclusion of `depth` (runner.ts:190-192)."""
    if set(exclude) != {"depth"}:
        raise ValueError("planArena: the runtime plans with exclude={'depth'} (runner.ts:190)")
    d = _json(lib().illumina_arena_json, arch.inputSize)
    return ArenaPlan(tuple(d["bufferSizes"]), dict(d["assignment"]), d["totalBytes"], d["naiveBytes"])


def validateArena(arch: Architecture, plan: ArenaPlan, exclude=("depth",)) -> None:
    """validateArena (arena.ts:134-172): raises ValueError on overlapping live ranges."""
    first_write, last_read = {}, {}
    for i, op in enumerate(arch.ops):
        first_write.setdefault(op.out, i)
        for t in opInputs(op):
            last_read[t] = i
    names = [n for n in arch.tensors if n not in exclude]
    for a in names:
        for b in names:
            if a >= b or plan.assignment.get(a) != plan.assignment.get(b):
                continue
            a0 = first_write.get(a, 0)
            a1 = last_read.get(a, a0)
            b0 = first_write.get(b, 0)
            b1 = last_read.get(b, b0)
            if a0 <= b1 and b0 <= a1:
                raise ValueError(f"arena: {a} [{a0}..{a1}] and {b} [{b0}..{b1}] overlap in buffer "
                                 f"{plan.assignment.get(a)}")
    for n in names:
        b = plan.assignment.get(n)
        if b is None:
            raise ValueError(f"arena: {n} was never assigned a buffer")
        s = arch.tensors[n]
        need = s.h * s.w * s.c // 4
        if plan.bufferSizes[b] < need:
            raise ValueError(f"arena: buffer {b} holds {plan.bufferSizes[b]} but {n} needs {need}")
