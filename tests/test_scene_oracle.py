"""Procedural scene and depth metrics on the CPU: the oracle restatement
(oracle/scene.c) against the closed forms of the reference's own tests
(test/metrics.test.ts, test/scene.test.ts), and the library's host-side scene
uniforms (illumina_scene_params_*) against the oracle's.
"""
import math

import numpy as np
import pytest

from oracle import scene as OS

N = 64


def _maps(pred_fn, truth_fn):
    pred = np.empty((N, N), np.float32)
    truth = np.empty((N, N, 2), np.float32)
    for y in range(N):
        for x in range(N):
            pred[y, x] = pred_fn(x, y)
            truth[y, x] = truth_fn(x, y)
    return pred, truth


def test_metrics_closed_form_scale_shift():
    """metrics.test.ts:45-78: two groups, LS line through the group means."""
    pred, truth = _maps(lambda x, y: 0.25 if y < 32 else 0.75,
                        lambda x, y: ((4 if y < 16 else 2 if y < 32 else 1 if y < 48 else 2), 1))
    m = OS.evaluate_depth(pred, truth, N, N)
    assert m["samples"] == 4096
    assert m["scale"] == pytest.approx(0.75, abs=1e-12)
    assert m["shift"] == pytest.approx(0.1875, abs=1e-12)
    assert m["absRel"] == pytest.approx(1 / 3, abs=1e-12)
    assert m["rmse"] == pytest.approx(5 / 6, abs=1e-12)
    assert (m["delta1"], m["delta2"], m["delta3"]) == (0, 1, 1)


def test_metrics_affine_perfect_prediction():
    """metrics.test.ts:80-92 (float32 maps here, so the fit is exact to ~1e-7)."""
    z_of = lambda x, y: 1 + ((x + y * N) % 97) * 0.1  # noqa: E731
    pred, truth = _maps(lambda x, y: (1 / z_of(x, y) - 0.2) / 0.5, lambda x, y: (z_of(x, y), 1))
    m = OS.evaluate_depth(pred, truth, N, N)
    assert m["scale"] == pytest.approx(0.5, abs=1e-5)
    assert m["shift"] == pytest.approx(0.2, abs=1e-5)
    assert m["absRel"] < 2e-3
    assert m["delta1"] == 1


def test_metrics_hit_mask_and_window():
    """metrics.test.ts:94-103, plus the depth window (0.05, 25] and the n < 64 early return."""
    pred, truth = _maps(lambda x, y: 0.5, lambda x, y: (2, 1 if y < 32 else 0))
    assert OS.evaluate_depth(pred, truth, N, N)["samples"] == 2048
    pred, truth = _maps(lambda x, y: 0.5, lambda x, y: (0.04 if x < 20 else 30 if x < 40 else 3, 1))
    assert OS.evaluate_depth(pred, truth, N, N)["samples"] == 24 * N
    pred, truth = _maps(lambda x, y: 0.5, lambda x, y: (2, 1 if (x < 7 and y < 9) else 0))
    m = OS.evaluate_depth(pred, truth, N, N)
    assert m["samples"] == 63 and math.isnan(m["absRel"]) and m["delta1"] == 0 and math.isnan(m["scale"])


def test_scene_renders_image_and_truth():
    """scene.test.ts: a non-trivial image and matching ground-truth depth at 64x64, t = 1.5."""
    _, rgba8, truth = OS.render(OS.scene_params(1.5, False), N, N)
    v = rgba8[..., :3].astype(np.float64).mean(-1)
    assert v.mean() > 8 and v.max() > 40 and len(np.unique(rgba8[..., 0])) > 8
    assert (rgba8[..., 3] == 255).all()
    hit = truth[..., 1] > 0.5
    assert hit.sum() > N * N * 0.2
    z = truth[..., 0][hit]
    assert z.min() > 0.1 and z.max() > z.min() * 1.5
    # some sky is missed; the floor along the bottom row is hit
    assert (~hit).any() and hit[-1].all()


def test_scene_uniforms_match_oracle():
    """illumina_scene_params_initial / _update (host code of the library) against the oracle."""
    import ctypes as C
    from illumina import sceneParams
    for t, orbit in [(None, False), (0.0, False), (1.5, False), (7.25, True), (123.4, True)]:
        p = sceneParams(t, orbit)
        got = np.array(list(p.camera) + list(p.focus) + list(p.options), np.float32)
        np.testing.assert_array_equal(got, OS.scene_params(t, orbit))
    assert C.sizeof(type(sceneParams())) == 48
