"""Command line mirroring the reference's scripts/ref-forward.ts on the B200
path: reads an ntb/1 bundle holding "rgba" (S x S x 4 in [0, 1]) or "input"
(S x S x 4 preprocess output), runs the CUDA forward and writes every
activation forwardReference names (plus "scene_color" for an "rgba" input and
"depth", the joint-bilateral output the reference CLI does not produce) as an
ntb/1 bundle, so a host with Node can diff the two layer by layer.

  python -m illumina.ref_forward --weights synthetic:0 --input in.ntb --out out.ntb --size 448

Options as ref-forward.ts:184-195 (--weights, --input, --out, --dump-weights,
--size, --exposure, --no-srgb), plus --device, --precision and --engine.
Prints one JSON summary line like the reference CLI (:338-347).
"""
from __future__ import annotations

import argparse
import json
import sys

import numpy as np


def _parser():
    ap = argparse.ArgumentParser(prog="python -m illumina.ref_forward", description=__doc__.split("\n\n")[0])
    ap.add_argument("--weights", default="synthetic:1", help=".idm container, or synthetic[:seed] (default synthetic:1)")
    ap.add_argument("--input", default=None, help='bundle holding "rgba" or "input"')
    ap.add_argument("--out", default=None, help="where to write every activation")
    ap.add_argument("--dump-weights", default=None, help="also write the weights actually used (.idm)")
    ap.add_argument("--size", type=int, default=None, help="network size; default: input height")
    ap.add_argument("--exposure", type=float, default=1.0, help="preprocess exposure multiplier (default 1)")
    ap.add_argument("--no-srgb", action="store_true", help='treat "rgba" as already linear')
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--precision", default="f32", choices=["f32", "bf16"])
    ap.add_argument("--engine", default="tensor", choices=["tensor", "simt"])
    return ap


def load_weights(spec: str, arch):
    """loadWeights (ref-forward.ts:256-264)."""
    from .weights import parseWeights, synthesizeWeights
    if spec == "synthetic" or spec.startswith("synthetic:"):
        text = spec[len("synthetic") + 1:]
        try:
            seed = int(text) if text else 1
        except ValueError:
            raise ValueError(f"bad synthetic seed in {spec}") from None
        return synthesizeWeights(arch, seed)
    with open(spec, "rb") as f:
        return parseWeights(f.read(), arch)


def run(argv=None) -> dict:
    from . import bundle as B
    from .arch import buildArchitecture
    from .runner import createDepthModel
    from .weights import serializeWeights

    opts = _parser().parse_args(argv)
    tensors = {}
    if opts.input:
        with open(opts.input, "rb") as f:
            tensors = B.readBundle(f.read(), opts.input)
    size = opts.size
    if size is None:
        probe = tensors.get("rgba", tensors.get("input"))
        if probe is None:
            raise ValueError("--size is required when no --input is given")
        size = int(probe.shape[0])
    arch = buildArchitecture(size)
    weights = load_weights(opts.weights, arch)
    if opts.dump_weights:
        with open(opts.dump_weights, "wb") as f:
            f.write(serializeWeights(arch, weights))
    if not opts.input:
        return {"arch": arch.name, "size": size, "tensors": 0, "dumpedWeights": opts.dump_weights}

    model = createDepthModel(arch, weights=weights, decodeSrgb=not opts.no_srgb, exposure=opts.exposure,
                             device=opts.device, precision=opts.precision, keepIntermediates=True,
                             engine=opts.engine)
    try:
        want = (size, size, 4)
        if "rgba" in tensors:
            rgba = tensors["rgba"]
            if tuple(rgba.shape) != want:
                raise ValueError(f"rgba has shape [{', '.join(map(str, rgba.shape))}], expected [{size}, {size}, 4]")
            depth = model.forward(np.ascontiguousarray(rgba, np.float32)[None])
            out = B.dumpForward(model, include_scene=True)
        elif "input" in tensors:
            given = tensors["input"]
            if tuple(given.shape) != want:
                raise ValueError(f"input has shape [{', '.join(map(str, given.shape))}], expected [{size}, {size}, 4]")
            depth = model.forwardInput(np.ascontiguousarray(given, np.float32)[None])
            out = B.dumpForward(model, include_scene=False)
        else:
            raise ValueError('input bundle contains neither "rgba" nor "input"')
        out["depth"] = depth[0][..., None]
    finally:
        model.destroy()
    if opts.out:
        with open(opts.out, "wb") as f:
            f.write(B.writeBundle(out))
    return {"arch": arch.name, "size": size, "tensors": len(out), "names": list(out), "out": opts.out,
            "dumpedWeights": opts.dump_weights}


def main(argv=None) -> int:
    summary = run(argv)
    sys.stdout.write(json.dumps(summary) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
