"""Oracle restatement of the layer table, src/model/arch.ts.

TEST INFRASTRUCTURE ONLY (the checker for the product's own C++ table): only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this.

`build_architecture` follows arch.ts:191-385 op for op; `cost_of` follows
arch.ts:415-489; `weight_specs` follows src/model/weights.ts:29-63.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

ARCH_NAME = "IlluminaDepth-448"
MEAN = (0.485, 0.456, 0.406)
STD = (0.229, 0.224, 0.225)


@dataclass(frozen=True)
class Shape:
    h: int
    w: int
    c: int


@dataclass(frozen=True)
class Op:
    kind: str
    name: str
    out: str
    inp: Optional[str] = None
    k: int = 0
    stride: int = 0
    act: str = "linear"
    mid_act: str = "linear"
    residual: Optional[str] = None
    coarse: Optional[str] = None
    skip: Optional[str] = None


@dataclass
class Architecture:
    name: str
    input_size: int
    mean: tuple
    std: tuple
    tensors: dict = field(default_factory=dict)
    ops: list = field(default_factory=list)


def build_architecture(input_size: int) -> Architecture:
    """arch.ts:191-385."""
    if input_size % 32 != 0:
        raise ValueError(f"inputSize {input_size} must be a multiple of 32")
    tensors: dict[str, Shape] = {}
    ops: list[Op] = []

    def T(name, h, w, c):
        if c % 4 != 0:
            raise ValueError(f"tensor {name}: channel count {c} is not a multiple of 4")
        tensors[name] = Shape(h, w, c)
        return name

    S = input_size
    r = lambda level: S >> level  # noqa: E731

    x0 = T("input", S, S, 4)
    ops.append(Op("preprocess", "preprocess", x0))
    stem = T("stem", r(1), r(1), 16)
    ops.append(Op("conv", "stem", stem, inp=x0, k=3, stride=2, act="hardswish"))
    s0 = T("s0", r(1), r(1), 24)
    ops.append(Op("dwpw", "e1", s0, inp=stem, k=3, stride=1, mid_act="relu6", act="linear"))

    def down_block(prefix, inp, h, w, expand, out, k):
        mid = T(f"{prefix}.mid", h, w, expand)
        ops.append(Op("dwpw", f"{prefix}.dw_expand", mid, inp=inp, k=k, stride=2,
                      mid_act="linear", act="hardswish"))
        o = T(f"{prefix}.out", h, w, out)
        ops.append(Op("pw", f"{prefix}.project", o, inp=mid, act="linear"))
        return o

    def ir_block(prefix, inp, h, w, channels, expand, k):
        mid = T(f"{prefix}.mid", h, w, expand)
        ops.append(Op("pw", f"{prefix}.expand", mid, inp=inp, act="hardswish"))
        o = T(f"{prefix}.out", h, w, channels)
        ops.append(Op("dwpw", f"{prefix}.dw_project", o, inp=mid, k=k, stride=1,
                      mid_act="hardswish", act="linear", residual=inp))
        return o

    t = down_block("e2", s0, r(2), r(2), 96, 32, 3)
    t = ir_block("e3", t, r(2), r(2), 32, 128, 3)
    s1 = t
    t = down_block("e4", s1, r(3), r(3), 128, 56, 5)
    t = ir_block("e5a", t, r(3), r(3), 56, 224, 5)
    t = ir_block("e5b", t, r(3), r(3), 56, 224, 5)
    s2 = t
    t = down_block("e6", s2, r(4), r(4), 224, 104, 5)
    t = ir_block("e7a", t, r(4), r(4), 104, 416, 5)
    t = ir_block("e7b", t, r(4), r(4), 104, 416, 5)
    t = ir_block("e7c", t, r(4), r(4), 104, 416, 5)
    s3 = t
    t = down_block("e8", s3, r(5), r(5), 416, 176, 5)
    t = ir_block("e9a", t, r(5), r(5), 176, 704, 5)
    t = ir_block("e9b", t, r(5), r(5), 176, 704, 5)
    t = ir_block("e9c", t, r(5), r(5), 176, 704, 5)
    bottleneck = t

    d4 = T("d4", r(5), r(5), 96)
    ops.append(Op("pw", "d4.lateral", d4, inp=bottleneck, act="hardswish"))

    def decoder_level(prefix, coarse, skip, h, w, channels, next_channels):
        fused = T(f"{prefix}.fused", h, w, channels)
        ops.append(Op("lateral", f"{prefix}.lateral", fused, coarse=coarse, skip=skip,
                      act="linear"))
        o = T(f"{prefix}.out", h, w, next_channels)
        ops.append(Op("dwpw", f"{prefix}.refine", o, inp=fused, k=3, stride=1,
                      mid_act="hardswish", act="hardswish",
                      residual=fused if channels == next_channels else None))
        return o

    d3 = decoder_level("d3", d4, s3, r(4), r(4), 96, 64)
    d2 = decoder_level("d2", d3, s2, r(3), r(3), 64, 48)
    d1 = decoder_level("d1", d2, s1, r(2), r(2), 48, 32)
    d0 = decoder_level("d0", d1, s0, r(1), r(1), 32, 32)
    low = T("depth_low", r(1), r(1), 4)
    ops.append(Op("head", "head", low, inp=d0))
    full = T("depth", S, S, 4)
    ops.append(Op("bilateralUp", "upsample", full, inp=low))
    return Architecture(ARCH_NAME, S, MEAN, STD, tensors, ops)


def op_inputs(op: Op) -> list:
    """opInputs, src/engine/arena.ts:19-33."""
    if op.kind == "preprocess":
        return []
    if op.kind == "conv":
        return [op.inp]
    if op.kind in ("pw", "dwpw"):
        return [op.inp] + ([op.residual] if op.residual else [])
    if op.kind == "lateral":
        return [op.coarse, op.skip]
    return [op.inp]


def cost_of(arch: Architecture):
    """costOf, arch.ts:415-489. Returns (per-op list of dicts, total MACs, total params)."""
    sh = arch.tensors
    out = []
    for op in arch.ops:
        o = sh[op.out]
        if op.kind in ("preprocess", "bilateralUp"):
            macs, params = 0, 0
        elif op.kind == "conv":
            i = sh[op.inp]
            macs = o.h * o.w * o.c * i.c * op.k * op.k
            params = o.c * i.c * op.k * op.k + o.c
        elif op.kind == "pw":
            i = sh[op.inp]
            macs = o.h * o.w * o.c * i.c
            params = o.c * i.c + o.c
        elif op.kind == "dwpw":
            i = sh[op.inp]
            macs = o.h * o.w * i.c * op.k * op.k + o.h * o.w * o.c * i.c
            params = i.c * op.k * op.k + i.c + o.c * i.c + o.c
        elif op.kind == "lateral":
            s = sh[op.skip]
            c = sh[op.coarse]
            if c.c != o.c:
                raise ValueError(f"{op.name}: coarse tensor has {c.c} channels but the output has {o.c}")
            macs = o.h * o.w * o.c * s.c
            params = o.c * s.c + o.c
        elif op.kind == "head":
            i = sh[op.inp]
            macs = o.h * o.w * i.c
            params = i.c + 1
        else:
            raise ValueError(op.kind)
        out.append({"name": op.name, "kind": op.kind, "macs": macs, "params": params,
                    "out": (o.h, o.w, o.c)})
    return out, sum(c["macs"] for c in out), sum(c["params"] for c in out)


def weight_specs(arch: Architecture) -> list:
    """weightSpecs, src/model/weights.ts:29-63: [(name, shape), ...] in blob order."""
    c = lambda n: arch.tensors[n].c  # noqa: E731
    specs = []
    for op in arch.ops:
        if op.kind == "conv":
            specs += [(f"{op.name}.weight", (c(op.out), c(op.inp), op.k, op.k)),
                      (f"{op.name}.bias", (c(op.out),))]
        elif op.kind == "pw":
            specs += [(f"{op.name}.weight", (c(op.out), c(op.inp))), (f"{op.name}.bias", (c(op.out),))]
        elif op.kind == "dwpw":
            specs += [(f"{op.name}.dw_weight", (c(op.inp), op.k, op.k)),
                      (f"{op.name}.dw_bias", (c(op.inp),)),
                      (f"{op.name}.pw_weight", (c(op.out), c(op.inp))),
                      (f"{op.name}.pw_bias", (c(op.out),))]
        elif op.kind == "lateral":
            specs += [(f"{op.name}.weight", (c(op.out), c(op.skip))), (f"{op.name}.bias", (c(op.out),))]
        elif op.kind == "head":
            specs += [(f"{op.name}.weight", (1, c(op.inp))), (f"{op.name}.bias", (1,))]
    return specs
