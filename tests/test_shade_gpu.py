"""Shading + tone-map parity on the GPU (src/lighting/shade.ts,
composite.ts) against the oracle's float32 restatement, plus the reference
lighting tests' closed forms and invariants (test/shading.test.ts,
test/extremes.test.ts, test/frame.test.ts).

Tolerance: the shader has data-dependent branches (contact-shadow thickness
test, integer texel coordinates), so ulp-level differences can flip a branch
on a few pixels. Stated bar: HDR |got-want| <= 1e-3 * (1 + |want|) on at
least 99.5 % of pixels; 8-bit output within 1 level on at least 99.5 % of
pixels and mean absolute difference <= 0.05 levels.
"""
import math

import numpy as np
import pytest

from tests.golden import cases

pytestmark = pytest.mark.gpu

APP_LIGHTS = [  # the three lights main.ts ships with (extremes.test.ts:46-54)
    dict(kind="point", position=(0.9, 0.5, -1.4), color=(1, 0.83, 0.62), intensity=9, radius=7, shadow=1),
    dict(kind="point", position=(-1.2, 0.1, -2.2), color=(0.35, 0.6, 1), intensity=6, radius=8, shadow=0.8),
    dict(kind="spot", position=(0, 1.6, -0.4), direction=(0, -1, -0.35), color=(1, 0.95, 0.9), intensity=22,
         radius=9, innerAngle=0.28, outerAngle=0.52, shadow=1),
]


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _depth64():
    """A real disparity map: the 64x64 network on the test image (oracle)."""
    from oracle import arch as OA
    from oracle import reference as R
    from oracle import weights as OW
    a = OA.build_architecture(64)
    rgb = cases.rgba_bytes_to_planar(cases.test_image(64), 64)
    _, disp = R.forward_frame(a, OW.synthesize_weights(a, 31337), rgb)
    return disp, rgb


def _run_both(torch, depth, dw, dh, albedo, aw, ah, lights, settings, out_w, out_h, steps, frame=0, rows=None):
    from illumina import lighting as L
    from oracle import shade as OS
    d_depth = torch.from_numpy(np.ascontiguousarray(depth, np.float32)).cuda()
    d_alb = torch.from_numpy(np.ascontiguousarray(albedo, np.float32)).cuda()
    hdr = torch.zeros((out_h, out_w, 4), device="cuda")
    rgba = torch.zeros((out_h, out_w, 4), dtype=torch.uint8, device="cuda")
    L.shade(d_depth, dw, dh, d_alb, aw, ah, lights, settings, frame, out_w, out_h, hdr=hdr, rgba8=rgba,
            steps=steps)
    torch.cuda.synchronize()
    s = settings
    sd = dict(fovY=s.fovY, near=s.near, far=s.far, aoStrength=s.aoStrength, shadowStrength=s.shadowStrength,
              volumetric=s.volumetric, exposure=s.exposure, ambient=s.ambient, ambientIntensity=s.ambientIntensity,
              roughness=s.roughness, fogDensity=s.fogDensity, fogColor=s.fogColor, specular=s.specular,
              normalStrength=s.normalStrength, albedoMix=s.albedoMix, contactShadowLength=s.contactShadowLength,
              aoRadiusPixels=s.aoRadiusPixels, toneMap=s.toneMap, contrast=s.contrast, saturation=s.saturation,
              vignette=s.vignette, debug=s.debug)
    P = OS.pack_params(sd, frame, out_w, out_h, dw, dh)
    want_hdr, want_rgba = OS.shade(depth, dw, dh, albedo, aw, ah, OS.pack_lights(lights), P, out_w, out_h,
                                   steps=steps, rows=rows)
    got_hdr, got_rgba = hdr.cpu().numpy(), rgba.cpu().numpy()
    if rows:
        r0, r1 = rows
        return got_hdr[r0:r1], want_hdr[r0:r1], got_rgba[r0:r1], want_rgba[r0:r1]
    return got_hdr, want_hdr, got_rgba, want_rgba


def _assert_close(got_hdr, want_hdr, got_rgba, want_rgba):
    g, w = got_hdr[..., :3], want_hdr[..., :3]
    assert np.isfinite(g).all()
    px_ok = (np.abs(g - w) <= 1e-3 * (1 + np.abs(w))).all(axis=-1)
    assert px_ok.mean() >= 0.995, f"HDR agreement {px_ok.mean():.4f}"
    d = np.abs(got_rgba.astype(np.int32) - want_rgba.astype(np.int32))[..., :3]
    assert (d.max(axis=-1) <= 1).mean() >= 0.995, f"8-bit agreement {(d.max(axis=-1) <= 1).mean():.4f}"
    assert d.mean() <= 0.05, d.mean()


@pytest.mark.parametrize("steps", [(12, 6, 4, 10), (16, 6, 4, 12)])
def test_shade_matches_oracle_64(torch, steps):
    from illumina.lighting import DEFAULT_SETTINGS
    disp, rgb = _depth64()
    out = _run_both(torch, disp, 64, 64, rgb, 64, 64, APP_LIGHTS, DEFAULT_SETTINGS, 64, 64, steps, frame=3)
    _assert_close(*out)


def test_shade_upsampled_render_matches_oracle(torch):
    """Render larger than the depth map (nearest fetch + bilinear albedo), reference constants."""
    from illumina.lighting import DEFAULT_SETTINGS
    disp, rgb = _depth64()
    out = _run_both(torch, disp, 64, 64, rgb, 64, 64, APP_LIGHTS, DEFAULT_SETTINGS, 160, 90, (12, 6, 4, 10))
    _assert_close(*out)


@pytest.mark.parametrize("view", ["depth", "normals", "occlusion", "albedo"])
def test_debug_views_match_oracle(torch, view):
    from illumina.lighting import DEFAULT_SETTINGS
    disp, rgb = _depth64()
    out = _run_both(torch, disp, 64, 64, rgb, 64, 64, APP_LIGHTS, DEFAULT_SETTINGS.with_(debug=view), 64, 64,
                    (12, 6, 4, 10))
    _assert_close(*out)


def test_flat_plane_normals_and_ggx_peak(torch):
    """shading.test.ts: constant disparity -> normal (0,0,1) -> normals view 128,128,255;
    a head-on light at the GGX singularity stays finite."""
    from illumina.lighting import DEFAULT_SETTINGS
    N = 64
    disp = np.full(N * N, 0.5, np.float32)
    alb = np.full((3, N, N), 180 / 255, np.float32)
    near, far = DEFAULT_SETTINGS.near, DEFAULT_SETTINGS.far
    z = 1 / (0.5 * (1 / near - 1 / far) + 1 / far)
    light = [dict(kind="point", position=(0, 0, -z + 1), color=(1, 1, 1), intensity=9, radius=7, shadow=0)]
    for s in [DEFAULT_SETTINGS, DEFAULT_SETTINGS.with_(roughness=0.04, specular=2, exposure=4),
              DEFAULT_SETTINGS.with_(roughness=1, specular=2)]:
        gh, wh, gr, wr = _run_both(torch, disp, N, N, alb, N, N, light, s, N, N, (12, 6, 4, 10))
        assert np.isfinite(gh).all()
        _assert_close(gh, wh, gr, wr)
    gh, wh, gr, wr = _run_both(torch, disp, N, N, alb, N, N, light, DEFAULT_SETTINGS.with_(debug="normals"),
                               N, N, (12, 6, 4, 10))
    c = N // 2
    np.testing.assert_allclose(gh[c, c, :3], [0.5, 0.5, 1.0], atol=1e-6)


RANGES = dict(exposure=(0.1, 4), contrast=(0.6, 1.6), saturation=(0, 2), vignette=(0, 1), near=(0.05, 3),
              far=(2, 60), fovY=(20 * math.pi / 180, 110 * math.pi / 180), normalStrength=(0.1, 4),
              ambientIntensity=(0, 2), shadowStrength=(0, 1), contactShadowLength=(0.05, 4), aoStrength=(0, 1),
              aoRadiusPixels=(2, 48), volumetric=(0, 2), fogDensity=(0, 0.25), roughness=(0.04, 1),
              specular=(0, 2), albedoMix=(0, 1))


def test_no_nan_at_slider_extremes(torch):
    """extremes.test.ts:96-208: every slider at both ends plus adversarial combinations."""
    from illumina import lighting as L
    disp, rgb = _depth64()
    d_depth = torch.from_numpy(disp).cuda()
    d_alb = torch.from_numpy(rgb).cuda()
    hdr = torch.zeros((64, 64, 4), device="cuda")
    base = L.DEFAULT_SETTINGS
    settings = [base.with_(**{k: v}) for k, (lo, hi) in RANGES.items() for v in (lo, hi)]
    settings += [base.with_(roughness=0.04, specular=2, exposure=4),
                 base.with_(roughness=0.04, specular=2, exposure=4, near=0.05, far=2),
                 base.with_(near=3, far=2)]
    bad = []
    for s in settings:
        L.shade(d_depth, 64, 64, d_alb, 64, 64, APP_LIGHTS, s, 0, 64, 64, hdr=hdr)
        torch.cuda.synchronize()
        if not torch.isfinite(hdr).all():
            bad.append(s)
    assert bad == []


def test_render_frame_and_skip_inference(torch):
    """frame.test.ts:305-352: 41 dispatches, and a skipped frame shades the last written depth identically."""
    import illumina
    a = illumina.buildArchitecture(64)
    m = illumina.createDepthModel(a, synthSeed=606)
    rgb = cases.rgba_bytes_to_planar(cases.test_image(64), 64)
    alb = torch.from_numpy(rgb).cuda()
    r = illumina.createRenderer(64, 64, 64, alb, model=m)
    r.setLights(APP_LIGHTS[:1])
    r.update(illumina.DEFAULT_SETTINGS, 0)
    full = illumina.renderFrame(m, r, rgb)
    assert (full.dispatches, full.draws, full.encoders, full.submits) == (41, 1, 1, 1)
    torch.cuda.synchronize()
    lit = r.target.cpu().numpy().copy()
    assert lit[..., :3].mean() > 4 and len(np.unique(lit[..., 0])) > 16
    fresh = m.freshParity()
    skipped = illumina.renderFrame(m, r, skipInference=True)
    assert skipped.dispatches == 1 and m.freshParity() == fresh
    torch.cuda.synchronize()
    np.testing.assert_array_equal(r.target.cpu().numpy(), lit)
    m.destroy()


def test_config4_render_1080p_band_matches_oracle(torch):
    """The relighting-frame geometry: 448 depth, 1920x1080 render, 4 seeded point lights,
    16 contact / 12 volumetric steps; compared on a band of rows (the oracle is scalar)."""
    from illumina.lighting import DEFAULT_SETTINGS
    from illumina.workloads import config4_lights
    import ctypes as C
    from oracle import lib as olib
    disp, _ = _depth64()
    # a smooth 448 disparity: the 64 map bilinearly upsampled
    from oracle import shade as OS
    d448 = OS.resize_bilinear(disp, 64, 64, 448, 448)
    alb = np.empty(3 * 448 * 448, np.float32)
    olib().or_uniform_frame(0, alb.size, alb.ctypes.data_as(C.POINTER(C.c_float)))
    lights = config4_lights(0, 16 / 9, DEFAULT_SETTINGS.fovY)
    out = _run_both(torch, d448, 448, 448, alb.reshape(3, 448, 448), 448, 448, lights, DEFAULT_SETTINGS, 1920,
                    1080, (16, 6, 4, 12), rows=(500, 516))
    _assert_close(*out)
