"""IlluminaDepth on B200: the Python host above the native C ABI.

The names mirror the reference's TypeScript API surface for the hot path:

  arch      buildArchitecture, costOf, formatCost, ILLUMINA_DEPTH_448  (src/model/arch.ts)
  weights   weightSpecs, parseWeights, serializeWeights, synthesizeWeights,
            halfToFloat, opWeights                                   (src/model/weights.ts)
  arena     planArena, validateArena, opInputs                       (src/engine/arena.ts)
  runner    createDepthModel -> DepthModel                           (src/model/runner.ts)
  lighting  packLights, ShadingSettings, DEFAULT_SETTINGS,
            createRenderer -> Renderer                               (src/lighting/*.ts)
  frame     renderFrame -> FrameResult                               (src/engine/frame.ts)
  scene     createProceduralScene, renderScenes, evaluateDepth       (src/scene/procedural.ts, metrics.ts)
  ops       per-kernel entry points                                  (src/model/kernels/*.ts)
  bundle    readBundle, writeBundle, dumpForward (ntb/1)             (scripts/ref-forward.ts)
  ref_forward  the ref-forward CLI on the CUDA path: python -m illumina.ref_forward

Everything computes in libillumina.so (CUDA for sm_100a); there is no CPU path.
"""
from ._lib import IlluminaError, lib  # noqa: F401
from .arch import Architecture, TensorShape, buildArchitecture, costOf, formatCost, weightSpecs  # noqa: F401
from .arena import opInputs, planArena, validateArena  # noqa: F401
from .bundle import dumpForward, readBundle, writeBundle  # noqa: F401
from .frame import FrameResult, renderFrame  # noqa: F401
from .lighting import (DEFAULT_SETTINGS, MAX_LIGHTS, LightDescription, LightKind, Renderer,  # noqa: F401
                       ShadingSettings, createRenderer, packLights)
from .runner import DepthModel, createDepthModel, cropTransform  # noqa: F401
from .scene import (DepthMetrics, ProceduralScene, createProceduralScene, evaluateDepth,  # noqa: F401
                    renderScenes, sceneParams)
from .weights import (halfToFloat, opWeights, parseWeights, serializeWeights,  # noqa: F401
                      synthesizeWeights, totalParameters)


def __getattr__(name):
    if name == "ILLUMINA_DEPTH_448":
        return buildArchitecture(448)
    raise AttributeError(name)
