"""Lighting parameters and the renderer: the Python face of
src/lighting/lights.ts (Light, LightKind, MAX_LIGHTS, packLights) and
src/lighting/renderer.ts (ShadingSettings, DEFAULT_SETTINGS, createRenderer /
Renderer). Shading and the tone-map composite run as one native kernel
(illumina_shade); the HDR target and the 8-bit output are device buffers
(torch tensors) instead of WebGPU textures.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import asdict, dataclass, field, replace

from ._lib import Light, ShadeSteps, ShadingSettingsC, check, lib, ptr, stream_handle

MAX_LIGHTS = 8
LightKind = {"point": 0, "spot": 1, "directional": 2}
DEBUG_IDS = {"lit": 0, "depth": 1, "normals": 2, "occlusion": 3, "albedo": 4}
REFERENCE_STEPS = (12, 6, 4, 10)  # contact, AO dirs, AO steps, volumetric (shade.ts:192, :232-233, :310)


@dataclass(frozen=True)
class LightDescription:
    """LightDescription (lights.ts:151-163)."""
    kind: str
    position: tuple
    color: tuple
    intensity: float
    radius: float | None = None
    innerAngle: float | None = None
    outerAngle: float | None = None
    shadow: float | None = None
    direction: tuple | None = None


def packLights(lights) -> C.Array:
    """packLights (lights.ts:178-206) -> 8 Light structs."""
    lights = [l if isinstance(l, LightDescription) else LightDescription(**l) for l in lights]
    if len(lights) > MAX_LIGHTS:
        raise ValueError(f"packLights: {len(lights)} lights exceeds the maximum of {MAX_LIGHTS}")
    arr = (Light * MAX_LIGHTS)()
    for i in range(MAX_LIGHTS):
        if i >= len(lights):
            arr[i].direction[:] = [0, 0, -1, -1]
            continue
        l = lights[i]
        d = l.direction if l.direction is not None else (0, 0, -1)
        n = math.hypot(*d) or 1
        outer = l.outerAngle if l.outerAngle is not None else math.pi / 5
        inner = min(l.innerAngle if l.innerAngle is not None else math.pi / 8, outer)
        arr[i].position[:] = [l.position[0], l.position[1], l.position[2], 1]
        arr[i].color[:] = [l.color[0], l.color[1], l.color[2], l.intensity]
        arr[i].direction[:] = [d[0] / n, d[1] / n, d[2] / n, math.cos(outer)]
        arr[i].params[:] = [LightKind[l.kind], math.cos(inner), 8 if l.radius is None else l.radius,
                            1 if l.shadow is None else l.shadow]
    return arr


@dataclass(frozen=True)
class ShadingSettings:
    """ShadingSettings (renderer.ts:53-78); defaults are DEFAULT_SETTINGS (:80-103)."""
    fovY: float = 58 * math.pi / 180
    near: float = 0.35
    far: float = 14.0
    aoStrength: float = 0.85
    shadowStrength: float = 0.8
    volumetric: float = 0.35
    exposure: float = 1.15
    ambient: tuple = (0.16, 0.2, 0.3)
    ambientIntensity: float = 0.5
    roughness: float = 0.55
    fogDensity: float = 0.028
    fogColor: tuple = (0.05, 0.07, 0.12)
    specular: float = 0.6
    normalStrength: float = 1.0
    albedoMix: float = 1.0
    contactShadowLength: float = 0.8
    aoRadiusPixels: float = 14.0
    toneMap: str = "aces"
    contrast: float = 1.04
    saturation: float = 1.06
    vignette: float = 0.35
    debug: str = "lit"

    def with_(self, **kw) -> "ShadingSettings":
        return replace(self, **kw)


DEFAULT_SETTINGS = ShadingSettings()


def _settings_c(s: ShadingSettings) -> ShadingSettingsC:
    c = ShadingSettingsC()
    c.fov_y, c.near_m, c.far_m = s.fovY, s.near, s.far
    c.ao_strength, c.shadow_strength, c.volumetric, c.exposure = (s.aoStrength, s.shadowStrength, s.volumetric,
                                                                   s.exposure)
    c.ambient[:] = list(s.ambient)
    c.ambient_intensity, c.roughness, c.fog_density = s.ambientIntensity, s.roughness, s.fogDensity
    c.fog_color[:] = list(s.fogColor)
    c.specular, c.normal_strength, c.albedo_mix = s.specular, s.normalStrength, s.albedoMix
    c.contact_shadow_length, c.ao_radius_pixels = s.contactShadowLength, s.aoRadiusPixels
    c.tone_map = 0 if s.toneMap == "aces" else 1
    c.contrast, c.saturation, c.vignette = s.contrast, s.saturation, s.vignette
    c.debug_view = DEBUG_IDS[s.debug]
    return c


def shade(disparity, dw: int, dh: int, albedo, aw: int, ah: int, lights, settings: ShadingSettings,
          frame: int, out_w: int, out_h: int, hdr=None, rgba8=None, steps=REFERENCE_STEPS,
          disparityChannels: int = 1, stream=None):
    """One shading + composite pass (device buffers; torch tensors or raw addresses)."""
    L = lights if isinstance(lights, C.Array) else packLights(lights)
    st = ShadeSteps(*steps)
    check(lib().illumina_shade(ptr(disparity), dw, dh, disparityChannels, ptr(albedo), aw, ah, L,
                               C.byref(_settings_c(settings)), frame & 0xFFFFFFFF, C.byref(st), out_w, out_h,
                               ptr(hdr), ptr(rgba8), stream_handle(stream)))


class Renderer:
    """Renderer (renderer.ts:105-115): recordShade, recordComposite, setLights, update, resize, hdr, destroy."""

    def __init__(self, width: int, height: int, depthSize: int, albedo, depthSlots, albedoSize=None,
                 steps=REFERENCE_STEPS):
        import torch
        self._torch = torch
        self.width, self.height, self.depthSize = width, height, depthSize
        self.albedo = albedo  # [3, ah, aw] sRGB device tensor
        self.albedoSize = albedoSize or (albedo.shape[2], albedo.shape[1])
        self.depthSlots = depthSlots  # callable parity -> device address of an S x S x 4 slot
        self.steps = steps
        self._lights = packLights([])
        self._settings = DEFAULT_SETTINGS
        self._frame = 0
        self._alloc()

    def _alloc(self):
        t = self._torch
        self.hdr = t.zeros((self.height, self.width, 4), dtype=t.float32, device="cuda")
        self.target = t.zeros((self.height, self.width, 4), dtype=t.uint8, device="cuda")

    def setLights(self, lights):
        self._lights = packLights(lights)

    def update(self, settings: ShadingSettings, frame: int):
        self._settings = settings
        self._frame = frame

    def recordShade(self, parity: int, stream=None, composite: bool = True):
        """Shades from depth slot `parity`; the composite (tone map -> 8-bit) is fused in."""
        aw, ah = self.albedoSize
        shade(self.depthSlots(parity), self.depthSize, self.depthSize, self.albedo, aw, ah, self._lights,
              self._settings, self._frame, self.width, self.height, hdr=self.hdr,
              rgba8=self.target if composite else None, steps=self.steps, disparityChannels=4, stream=stream)

    def recordComposite(self):
        """The composite is fused into recordShade; kept for API parity (no extra dispatch)."""
        return None

    def resize(self, w: int, h: int):
        if w == self.width and h == self.height:
            return
        self.width, self.height = max(1, w), max(1, h)
        self._alloc()

    def destroy(self):
        self.hdr = self.target = None


def createRenderer(width: int, height: int, depthSize: int, albedo, depthTextures=None, model=None,
                   steps=REFERENCE_STEPS) -> Renderer:
    """createRenderer (renderer.ts:123-251). `model` supplies the depth ping-pong slots."""
    if model is not None:
        slots = model.depthSlotPointer
    elif depthTextures is not None:
        slots = lambda parity: ptr(depthTextures[parity])  # noqa: E731
    else:
        raise ValueError("createRenderer needs a model or two depth textures")
    return Renderer(width, height, depthSize, albedo, slots, steps=steps)


__all__ = ["MAX_LIGHTS", "LightKind", "LightDescription", "packLights", "ShadingSettings", "DEFAULT_SETTINGS",
           "Renderer", "createRenderer", "shade", "REFERENCE_STEPS", "asdict", "field"]
