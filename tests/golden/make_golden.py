"""Generates the golden fixtures that pin the CPU oracle to the reference.

The reference's normative CPU implementation is TypeScript (no Node on either
machine), so parity is anchored on the reference's own Python code, imported
read-only from a checkout of the reference repository:

  * tools/train/illumina/model.py  -- the PyTorch twin of every op, the layer
    table (build_architecture), cost_of and weight_specs;
  * tools/export/export_idm.py     -- the torch-free .idm container writer.

Run once in a container that has the reference checkout (the GPU box does not):

    python -B tests/golden/make_golden.py --reference <path of the reference checkout>

Outputs (committed, a few hundred KB):
  arch.json        layer table, costs and weight specs at 64 and 448
  idm.json         header + SHA-256 of containers the reference writer produced
                   for the interop pattern (test/interop.test.ts:29-31), f32/f16
  ops.npz          twin outputs (float64) for every per-kernel case of
                   test/kernels.test.ts and test/shapes.test.ts, inputs drawn
                   exactly as those tests draw them (mulberry32 + randomFloats)
  net64.npz        the whole 64x64 network of test/network.test.ts (seed
                   20240819 weights, testImage input): twin intermediates
  preprocess.npz   twin preprocess of the kernels.test.ts preprocess case

The inputs and the seeded weights come from the oracle's own integer-exact
mulberry32 restatement (the twin initialises with the torch RNG), so these
fixtures pin the op semantics; the PRNG itself is pinned by its integer
definition.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import sys
import tempfile

sys.dont_write_bytecode = True
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402

import oracle  # noqa: E402
from oracle import arch as oarch  # noqa: E402
from oracle import weights as owts  # noqa: E402
from tests.golden import cases  # noqa: E402

FULL_LIMIT = 8192  # store whole outputs up to this many elements, else samples


def summarize(name, arr, store):
    a = np.asarray(arr, np.float64).ravel()
    store[f"{name}/sum"] = np.array([a.sum(), (a * a).sum(), np.abs(a).max() if a.size else 0.0])
    if a.size <= FULL_LIMIT:
        store[f"{name}/full"] = a.astype(np.float32)
    else:
        idx = np.linspace(0, a.size - 1, 2048).round().astype(np.int64)
        store[f"{name}/idx"] = idx
        store[f"{name}/val"] = a[idx]


def nhwc(t):
    """[1,C,H,W] torch tensor -> flat channels-last float64."""
    return t[0].permute(1, 2, 0).contiguous().double().numpy().ravel()


def load_reference(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "tools", "train"))
    sys.path.insert(0, os.path.join(ref_root, "tools", "export"))
    from illumina import model as twin  # noqa: F401
    import export_idm  # noqa: F401
    return twin, export_idm


def make_arch(twin, out):
    doc = {}
    for size in (64, 448):
        a = twin.build_architecture(size)
        ops = []
        for op in a.ops:
            d = {"kind": op.kind, "name": op.name, "out": op.out}
            for f in ("inp", "k", "stride", "act", "mid_act", "residual", "coarse", "skip"):
                if hasattr(op, f):
                    d[f] = getattr(op, f)
            ops.append(d)
        tensors = {n: [s.h, s.w, s.c] for n, s in a.tensors.items()}
        per_op, macs, params = twin.cost_of(a)
        doc[str(size)] = {
            "name": a.name, "mean": list(a.mean), "std": list(a.std), "ops": ops,
            "tensors": tensors,
            "cost": [{"name": c.name, "macs": c.macs, "params": c.params} for c in per_op],
            "total_macs": macs, "total_params": params,
            "specs": [[s.name, list(s.shape)] for s in twin.weight_specs(a)],
        }
    with open(os.path.join(out, "arch.json"), "w") as f:
        json.dump(doc, f, indent=0, sort_keys=True)


def make_idm(twin, exp, out):
    a = twin.build_architecture(448)
    specs = twin.weight_specs(a)
    entries = []
    for i, s in enumerate(specs):
        n = math.prod(s.shape)
        vals = [((i * 7919 + j * 31) % 1000) / 1000.0 - 0.5 for j in range(n)]
        entries.append(exp.TensorEntry(name=s.name, shape=tuple(s.shape), values=vals))
    doc = {}
    with tempfile.TemporaryDirectory() as td:
        for dtype in ("f32", "f16"):
            p = os.path.join(td, f"x.{dtype}.idm")
            header = exp.write_container(p, entries, dtype=dtype)
            raw = open(p, "rb").read()
            _, back = exp.read_container(p)
            samples = {s.name: list(back[s.name].values[:8]) for s in specs[::7]}
            doc[dtype] = {"sha256": hashlib.sha256(raw).hexdigest(), "size": len(raw),
                          "header": header, "samples": samples}
    with open(os.path.join(out, "idm.json"), "w") as f:
        json.dump(doc, f)


def make_ops(twin, out):
    import torch
    torch.set_default_dtype(torch.float64)
    store = {}
    for case in cases.all_cases():
        data = cases.draw(case)
        kind = case["kind"]
        name = case["id"]
        with torch.no_grad():
            if kind == "pw":
                h, w, ic, oc = case["h"], case["w"], case["inC"], case["outC"]
                layer = twin.PointwiseLayer(ic, oc, case["act"], with_bn=False).double()
                layer.weight.copy_(torch.from_numpy(data["w"].astype(np.float64).reshape(oc, ic)))
                layer.bias.copy_(torch.from_numpy(data["b"].astype(np.float64)))
                x = torch.from_numpy(data["src"].astype(np.float64).reshape(1, h, w, ic)).permute(0, 3, 1, 2)
                res = None
                if case["residual"]:
                    res = torch.from_numpy(data["res"].astype(np.float64).reshape(1, h, w, oc)).permute(0, 3, 1, 2)
                y = layer(x, res)
            elif kind == "dwpw":
                ic, oc, k, s = case["inC"], case["outC"], case["k"], case["stride"]
                layer = twin.DepthwisePointwiseLayer(ic, oc, k, s, case["midAct"], case["act"],
                                                     with_bn=False).double()
                layer.dw_weight.copy_(torch.from_numpy(data["dw_w"].astype(np.float64).reshape(ic, k, k)))
                layer.dw_bias.copy_(torch.from_numpy(data["dw_b"].astype(np.float64)))
                layer.pw_weight.copy_(torch.from_numpy(data["pw_w"].astype(np.float64).reshape(oc, ic)))
                layer.pw_bias.copy_(torch.from_numpy(data["pw_b"].astype(np.float64)))
                x = torch.from_numpy(data["src"].astype(np.float64).reshape(1, case["inH"], case["inW"], ic)).permute(0, 3, 1, 2)
                res = None
                if case["residual"]:
                    oh, ow = data["outH"], data["outW"]
                    res = torch.from_numpy(data["res"].astype(np.float64).reshape(1, oh, ow, oc)).permute(0, 3, 1, 2)
                y = layer(x, res)
            elif kind == "conv":
                ic, oc, k, s = case["inC"], case["outC"], case["k"], case["stride"]
                layer = twin.ConvLayer(ic, oc, k, s, case["act"], with_bn=False).double()
                layer.weight.copy_(torch.from_numpy(data["w"].astype(np.float64).reshape(oc, ic, k, k)))
                layer.bias.copy_(torch.from_numpy(data["b"].astype(np.float64)))
                x = torch.from_numpy(data["src"].astype(np.float64).reshape(1, case["inH"], case["inW"], ic)).permute(0, 3, 1, 2)
                y = layer(x)
            elif kind == "lateral":
                oc, sc = case["outC"], case["skipC"]
                layer = twin.LateralLayer(sc, oc, case["act"], with_bn=False).double()
                layer.weight.copy_(torch.from_numpy(data["w"].astype(np.float64).reshape(oc, sc)))
                layer.bias.copy_(torch.from_numpy(data["b"].astype(np.float64)))
                co = torch.from_numpy(data["coarse"].astype(np.float64).reshape(1, case["ch"], case["cw"], oc)).permute(0, 3, 1, 2)
                sk = torch.from_numpy(data["skip"].astype(np.float64).reshape(1, 2 * case["ch"], 2 * case["cw"], sc)).permute(0, 3, 1, 2)
                y = layer(co, sk)
            else:
                raise ValueError(kind)
        summarize(name, nhwc(y), store)
    np.savez_compressed(os.path.join(out, "ops.npz"), **store)


def make_net64(twin, out):
    import torch
    torch.set_default_dtype(torch.float64)
    a = oarch.build_architecture(64)
    wts = owts.synthesize_weights(a, cases.NET64_SEED)
    model = twin.build_model(64, with_bn=False).double()
    state = {}
    for n, shape in oarch.weight_specs(a):
        state[n] = torch.from_numpy(wts[n].astype(np.float64).reshape(shape))
    model.load_folded_state_dict(state)
    model.eval()
    rgba = cases.test_image(64).astype(np.float32) / np.float32(255.0)
    rgb = torch.from_numpy(rgba.reshape(64, 64, 4)[..., :3].astype(np.float64)).permute(2, 0, 1)[None]
    with torch.no_grad():
        x, lin = twin.preprocess(rgb)
        _, values = model(x, return_intermediates=True)
    store = {}
    for n, t in values.items():
        summarize(n, nhwc(t), store)
    summarize("scene_linear", nhwc(lin), store)
    np.savez_compressed(os.path.join(out, "net64.npz"), **store)


def make_preprocess(twin, out):
    import torch
    torch.set_default_dtype(torch.float64)
    rgba = cases.preprocess_image(32).astype(np.float32) / np.float32(255.0)
    rgb = torch.from_numpy(rgba.reshape(32, 32, 4)[..., :3].astype(np.float64)).permute(2, 0, 1)[None]
    with torch.no_grad():
        x, lin = twin.preprocess(rgb, exposure=cases.PREPROCESS_EXPOSURE)
    np.savez_compressed(os.path.join(out, "preprocess.npz"), input=nhwc(x), linear=nhwc(lin))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    oracle.build()
    twin, exp = load_reference(args.reference)
    make_arch(twin, args.out)
    make_idm(twin, exp, args.out)
    make_ops(twin, args.out)
    make_net64(twin, args.out)
    make_preprocess(twin, args.out)
    print("golden fixtures written to", args.out)


if __name__ == "__main__":
    main()
