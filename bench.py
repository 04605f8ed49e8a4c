#!/usr/bin/env python
"""IlluminaDepth-448 on B200: batched frames/s (and batch-1 latency) vs roofline.

Workload (one "step"): the whole hot path -- preprocess, 38 convolutions,
head, joint-bilateral upsample -- over one batch of 256 synthetic 3x448x448
fp32 frames (smooth blob images, seeded), with the seeded Kaiming weights
(seed 0). Frames are independent, so N GPUs run N replicas on disjoint frame
ranges with no collective on the data path (weak scaling); only the timing
uses a barrier and a max-reduce.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0). The reference arm times the oracle port of the
reference's CPU forward (src/model/reference.ts) on the host's cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "ai-illumination-depth-model_b200")
for _p in (REPO, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "IlluminaDepth-448 batch-1 µs/frame and batched frames/s at 1/2/4/8 B200 vs roofline"
UNIT = "frames/s"
SIZE = 448
L2_BYTES = 126 * 1024 * 1024


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--precision", default="f32", choices=["f32", "bf16"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip batch-1 latency and bf16 lines")
    ap.add_argument("--only", default=None, choices=["relight", "sweep", "streaming", "bf16"],
                    help="run just one extra measurement on rank 0 and print it (for profiling)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class RankGroup:
    """The only cross-rank operations of a run: a barrier around each timed
    region and a max-reduce of elapsed times (frames are independent, so there
    is no collective on the data path). `backend` is "nccl" on the GPU box
    (tensors on `device`), "gloo" for the CPU tests; world 1 needs no group."""

    def __init__(self, world: int, backend: str = "nccl", device=None, timeout_s: int = 300):
        self.world = world
        self.device = device
        self.pg = False
        if world > 1:
            import datetime
            import torch.distributed as dist
            kw = {"device_id": device} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist
            dist.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=self.device or "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def all_gather(self, t):
        """Rank-ordered concatenation of every rank's equal-sized tensor `t`."""
        if not self.pg:
            return t
        import torch
        import torch.distributed as dist
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t)
        return torch.cat(parts)

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()
            self.pg = False


def frame_seed_base(rank: int, batch: int) -> int:
    """Rank r generates frames with seeds [r*batch, (r+1)*batch): disjoint
    frame ranges, so N ranks process N*batch distinct frames (weak scaling)."""
    return rank * batch


def shard(total: int, rank: int, world: int):
    """Contiguous block of frame indexes [first, first + count) of `rank`."""
    per = total // world
    return rank * per, per


def checksum_digest(sums) -> str:
    """Digest of the per-frame u64 disparity checksums in frame order."""
    import hashlib

    import numpy as np
    return hashlib.sha256(np.ascontiguousarray(sums, dtype=np.uint64).tobytes()).hexdigest()[:16]


def aggregate_frames_per_s(world: int, batch: int, steps: int, ms_max: float) -> float:
    """Whole-job throughput: frames of all ranks over the slowest rank's time."""
    return world * batch * steps / (ms_max / 1000.0)


# ---------------------------------------------------------------------------
# measured peaks, clocks
# ---------------------------------------------------------------------------

def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# algorithmic bytes / FLOPs per op (per frame), from the layer table
# ---------------------------------------------------------------------------

def op_algorithmic(arch, cost, elt=4):
    """{op: (bytes, flops)} per frame: each distinct input and the output once, weights once per launch
    (added by the caller), FLOPs = 2 x MACs (costOf)."""
    t = arch.tensors
    out = {}
    for op, c in zip(arch.ops, cost.ops):
        e = lambda n: t[n].h * t[n].w * t[n].c  # noqa: E731
        if op.kind == "preprocess":
            b = (SIZE * SIZE * 3 + e(op.out)) * 4
        elif op.kind == "bilateralUp":
            low = t[op.inp]
            b = (low.h * low.w + SIZE * SIZE + SIZE * SIZE) * 4  # low-res map, luma guide, output
        elif op.kind == "head":
            b = (e(op.inp) + t[op.out].h * t[op.out].w) * elt
        elif op.kind == "lateral":
            b = (e(op.coarse) + e(op.skip) + e(op.out)) * elt
        else:
            # a residual that is the op's own input (d0.refine) is read once
            ins = [op.inp] + ([op.residual] if op.residual and op.residual != op.inp else [])
            b = (sum(e(n) for n in ins) + e(op.out)) * elt
        out[op.name] = (b, 2 * c.macs)
    return out


def e_in_bytes(arch, name, elt):
    """Bytes per frame of an op's main input (already counted as the previous op's output when fused)."""
    op = next(o for o in arch.ops if o.name == name)
    if not op.inp:
        return 0
    t = arch.tensors[op.inp]
    return t.h * t.w * t.c * elt


def weight_bytes_per_op(arch, specs):
    import numpy as np
    per = {}
    for name, shape in specs:
        op = name.rsplit(".", 1)[0]
        per[op] = per.get(op, 0) + int(np.prod(shape)) * 4
    return per


def load_traffic():
    try:
        with open(os.path.join(REPO, "profiles", "ncu_traffic.json")) as f:
            return json.load(f)
    except Exception:  # noqa: BLE001
        return {}


# ---------------------------------------------------------------------------
# CPU oracle timing (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------

_CPU_FRAMES = {}


def cpu_frames(count: int, threads: int):
    """`count` blob frames (seeds 0..count-1, the device generator's frames of
    rank 0), generated once across the thread pool."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import frames as OF
    missing = [i for i in range(count) if i not in _CPU_FRAMES]
    if missing:
        with ThreadPoolExecutor(max_workers=threads) as ex:
            for i, f in zip(missing, ex.map(lambda k: OF.blob_frame(k, SIZE), missing)):
                _CPU_FRAMES[i] = f.ravel()
    return [_CPU_FRAMES[i] for i in range(count)]


def cpu_oracle_frames_per_s(n_frames: int, threads: int):
    """Times the oracle port of the reference CPU forward (preprocess -> 38 convs -> head ->
    bilateralUp, double accumulation) on `n_frames` 448 blob frames (the benchmark's input)
    across `threads` host threads. Returns (frames/s, seconds)."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import arch as OA
    from oracle import reference as R
    from oracle import weights as OW
    a = OA.build_architecture(SIZE)
    w = OW.synthesize_weights(a, 0)
    frames = cpu_frames(min(n_frames, threads), threads)

    def one(i):
        R.forward_frame(a, w, frames[i % len(frames)])

    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(one, range(n_frames)))
    dt = time.perf_counter() - t0
    return n_frames / dt, dt


def host_threads():
    n = os.cpu_count() or 1
    try:
        n = len(os.sched_getaffinity(0))
    except Exception:  # noqa: BLE001
        pass
    return max(1, min(n, 64))


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    threads = host_threads()
    per_step = threads  # one 448 frame per thread per step (~1 s of CPU each)
    for _ in range(max(0, args.warmup)):
        cpu_oracle_frames_per_s(per_step, threads)
    total_t, total_f = 0.0, 0
    for _ in range(max(1, args.steps)):
        _, dt = cpu_oracle_frames_per_s(per_step, threads)
        total_t += dt
        total_f += per_step
    value = total_f / total_t
    sample = f"{per_step} blob frames of 3x448x448 per step ({threads} threads, one frame each)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total_t / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64-accumulate/f32-store",
        "data": "synthetic",
        "config": {"workload": "illuminadepth448-forward-b256-blobs", "global_batch": args.batch * args.gpus,
                   "input": "3x448x448 fp32", "weights": "synthesizeWeights(seed 0)",
                   "note": "reference CPU path (src/model/reference.ts) as its oracle port; node is absent"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

RELIGHT_W, RELIGHT_H = 1920, 1080
RELIGHT_STEPS = (16, 6, 4, 12)  # contact, AO directions x steps (24 samples), volumetric per light (x4 = 48)


def shade_roofline(shade_ms):
    """The shading kernel against the FP32 CUDA-core rate: algorithmic FLOPs per
    pixel from the op-counting build of the shading restatement (committed in
    profiles/shade_flops_1080p.json, benchmark step counts) over the measured
    time; peak = SMs x 128 FP32 lanes x 2 (FMA) x the measured maximum SM clock."""
    import torch
    try:
        with open(os.path.join(REPO, "profiles", "shade_flops_1080p.json")) as f:
            fpp = float(json.load(f)["benchmark"]["flops_per_pixel"])
    except Exception:  # noqa: BLE001
        return None
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            mhz, src = float(json.load(f)["sm_max_mhz"]), "MEASURED_PEAKS.json sm_max_mhz"
    except Exception:  # noqa: BLE001
        mhz, src = 1965.0, "clocks.max.sm 1965 MHz"
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    peak = sms * 128 * 2 * mhz * 1e6 / 1e12
    achieved = fpp * RELIGHT_W * RELIGHT_H / (shade_ms / 1000.0) / 1e12
    return {"bound": "fp32", "flops_per_pixel": fpp, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "peak_source": f"{sms} SMs x 128 x 2 x {mhz:.0f} MHz ({src})"}


def depth_relight_frame(model, frames, ring, stream, ev0, ev1, reps=60):
    """Depth + relighting frame at batch 1: forward of a uniform 448 frame, its disparity
    bilinearly upsampled to 1920x1080, shaded with 4 seeded point lights (24 AO samples,
    16 contact steps, 12 volumetric steps per light) with the frame's RGB as albedo
    (bilinear, i.e. upsampled), tone-mapped to 8-bit sRGB. Returns ms per frame and
    the shading kernel's share."""
    import torch
    from illumina import _lib
    from illumina import lighting as L
    from illumina.workloads import config4_lights

    lib = _lib.lib()
    d448 = torch.empty((1, SIZE, SIZE), dtype=torch.float32, device="cuda")
    d1080 = torch.empty((RELIGHT_H, RELIGHT_W), dtype=torch.float32, device="cuda")
    rgba8 = torch.empty((RELIGHT_H, RELIGHT_W, 4), dtype=torch.uint8, device="cuda")
    lights = L.packLights(config4_lights(0, RELIGHT_W / RELIGHT_H, L.DEFAULT_SETTINGS.fovY))
    sh = _lib.stream_handle(stream)

    def upsample():
        _lib.check(lib.illumina_resize_bilinear(d448.data_ptr(), SIZE, SIZE, d1080.data_ptr(), RELIGHT_W,
                                                RELIGHT_H, sh))

    def shade(i):
        L.shade(d1080, RELIGHT_W, RELIGHT_H, frames[i % ring], SIZE, SIZE, lights, L.DEFAULT_SETTINGS, i,
                RELIGHT_W, RELIGHT_H, rgba8=rgba8, steps=RELIGHT_STEPS, stream=stream)

    def frame(i):
        model.forward(frames[i % ring:i % ring + 1], disparity=d448, stream=stream)
        upsample()
        shade(i)

    for i in range(5):
        frame(i)
    torch.cuda.synchronize()
    ev0.record(stream)
    for i in range(reps):
        frame(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    frame_ms = ev0.elapsed_time(ev1) / reps
    ev0.record(stream)
    for i in range(reps):
        shade(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    shade_ms = ev0.elapsed_time(ev1) / reps
    return {"ms_per_frame": frame_ms, "shade_ms": shade_ms, "resolution": f"{RELIGHT_W}x{RELIGHT_H}",
            "mpix_per_s_shade": RELIGHT_W * RELIGHT_H / shade_ms / 1e3,
            "shade_roofline": shade_roofline(shade_ms),
            "steps": {"contact": RELIGHT_STEPS[0], "ao_samples": RELIGHT_STEPS[1] * RELIGHT_STEPS[2],
                      "volumetric_per_light": RELIGHT_STEPS[3], "lights": 4},
            "input": "uniform [0,1] 448 frame, batch 1; albedo = the frame's RGB (bilinear)"}


def scene_and_metrics(model, stream, ev0, ev1, batch=64, reps=5):
    """Procedural-scene ground truth at 448 (RGB + exact depth for `batch` frames per
    launch, the orbiting camera of ProceduralScene.update) and evaluateDepth of the
    network's disparity against it, all on the device."""
    import torch
    from illumina import _lib, renderScenes, sceneParams

    lib = _lib.lib()
    batch = min(batch, model.maxBatch)  # the scene frames also go through the model once
    params = [sceneParams(0.25 * i, True) for i in range(batch)]
    rgb = torch.empty((batch, 3, SIZE, SIZE), dtype=torch.float32, device="cuda")
    truth = torch.empty((batch, SIZE, SIZE, 2), dtype=torch.float32, device="cuda")
    disp = torch.empty((batch, SIZE, SIZE), dtype=torch.float32, device="cuda")
    out = torch.empty((batch, 64), dtype=torch.uint8, device="cuda")

    def render():
        renderScenes(params, SIZE, SIZE, rgb=rgb, truth=truth, stream=stream)

    def metrics():
        _lib.check(lib.illumina_evaluate_depth(disp.data_ptr(), 1, truth.data_ptr(), batch, SIZE, SIZE,
                                               out.data_ptr(), _lib.stream_handle(stream)))

    render()
    model.forward(rgb, disparity=disp, stream=stream)
    for _ in range(3):
        render()
        metrics()
    torch.cuda.synchronize()
    res = {}
    for name, fn in (("render", render), ("metrics", metrics)):
        ev0.record(stream)
        for _ in range(reps):
            fn()
        ev1.record(stream)
        torch.cuda.synchronize()
        res[name] = ev0.elapsed_time(ev1) / reps
    return {"render_frames_per_s": batch * 1000.0 / res["render"], "render_ms": res["render"],
            "metrics_ms": res["metrics"], "metrics_gb_per_s": batch * SIZE * SIZE * 12 / res["metrics"] / 1e6,
            "batch": batch, "outputs": "rgb 3x448x448 f32 + truth 448x448x2 f32 per frame"}


def source_sampling(model, stream, ev0, ev1, batch=64, reps=10):
    """8-bit camera frames (1920x1080 RGBA) sampled to the 448 network input with
    the blit's centre crop (cropTransform) folded into makePreprocess's uv
    transform: `batch` frames per launch, device buffers."""
    import torch
    import illumina

    w, h = 1920, 1080
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    src = torch.randint(0, 256, (batch, h, w, 4), dtype=torch.uint8, device="cuda", generator=g)
    frames = torch.empty((batch, 3, SIZE, SIZE), dtype=torch.float32, device="cuda")
    t = illumina.cropTransform(w, h)
    for _ in range(3):
        model.sampleSource(src, t[:2], t[2:], frames=frames, stream=stream)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(reps):
        model.sampleSource(src, t[:2], t[2:], frames=frames, stream=stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / reps
    return {"us_per_frame": 1000.0 * ms / batch, "ms_per_launch": ms, "batch": batch,
            "source": f"{w}x{h} RGBA8, centre crop, bilinear clamp-to-edge", "output": "3x448x448 f32 planar"}


def batch_sweep(model, frames, disp, stream, ev0, ev1, batches=(1, 8, 64, 256), reps=None):
    """Latency and frames/s of one forward at each batch size (device-resident
    blob frames; batch b takes consecutive slices of the 256 generated frames
    in turn, so small batches do not re-read L2-resident inputs)."""
    import torch
    out = []
    n = frames.shape[0]
    for b in batches:
        if b > n:
            continue
        views = [(frames[i:i + b], disp[i:i + b]) for i in range(0, n - b + 1, b)]
        n_reps = reps or max(5, min(200, 2048 // b))
        for k in range(min(len(views), 8) + 3):
            model.forward(views[k % len(views)][0], disparity=views[k % len(views)][1], stream=stream)
        torch.cuda.synchronize()
        ev0.record(stream)
        for k in range(n_reps):
            model.forward(views[k % len(views)][0], disparity=views[k % len(views)][1], stream=stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / n_reps
        out.append({"batch": b, "latency_ms": ms, "frames_per_s": b * 1000.0 / ms, "us_per_frame": 1000.0 * ms / b})
    return out


def streaming_frames(model, rank, world, stream, ranks, total=8192, batch=256):
    """Box-scale streaming: `total` independent uniform frames (seed n for frame n),
    sharded across the ranks in contiguous blocks; each rank generates its frames on
    its device batch by batch, replays the forward graph over batches of `batch` and
    takes per-frame checksums of the disparity (u64 sum of the fp32 bit patterns
    weighted by 2j+1, and a double sum). The only cross-rank step is the final
    gather of the checksums. Returns throughput over the slowest rank's device time,
    a digest of the 8192 u64 checksums in frame order (identical at every rank
    count when every GPU computes the same bits), and a spot check in which rank 0
    recomputes the last rank's last batch itself."""
    import numpy as np
    import torch
    from illumina import _lib

    lib = _lib.lib()
    f0, per = shard(total, rank, world)
    frames = torch.empty((batch, 3, SIZE, SIZE), dtype=torch.float32, device="cuda")
    disp = torch.empty((batch, SIZE, SIZE), dtype=torch.float32, device="cuda")
    h64 = torch.zeros(per, dtype=torch.int64, device="cuda")
    fsum = torch.zeros(per, dtype=torch.float64, device="cuda")
    sh = _lib.stream_handle(stream)

    def one_batch(first, nb, h_out, s_out):
        _lib.check(lib.illumina_generate_frames(0, first, nb, SIZE, frames.data_ptr(), sh))
        model.forward(frames[:nb], disparity=disp[:nb], stream=stream)
        _lib.check(lib.illumina_checksums(disp.data_ptr(), nb, SIZE * SIZE, h_out.data_ptr(), s_out.data_ptr(), sh))

    def run():
        for b0 in range(0, per, batch):
            nb = min(batch, per - b0)
            one_batch(f0 + b0, nb, h64[b0:], fsum[b0:])

    run()  # warm-up: graphs for this batch size
    torch.cuda.synchronize()
    ranks.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run()
    e1.record(stream)
    torch.cuda.synchronize()
    ranks.barrier()
    ms = ranks.max(e0.elapsed_time(e1))
    # the final host gather of per-frame checksums (the workload's only collective)
    gh, gs = ranks.all_gather(h64), ranks.all_gather(fsum)
    res = None
    if rank == 0:
        hosts = gh.cpu().numpy().astype(np.uint64)
        sums = gs.cpu().numpy()
        # rank 0 recomputes the last batch of the last rank on its own GPU
        last = total - min(batch, per)
        nb = total - last
        ch = torch.zeros(nb, dtype=torch.int64, device="cuda")
        cs = torch.zeros(nb, dtype=torch.float64, device="cuda")
        one_batch(last, nb, ch, cs)
        torch.cuda.synchronize()
        spot_ok = bool((ch.cpu().numpy().astype(np.uint64) == hosts[last:]).all())
        res = {"frames": total, "batch": batch, "frames_per_rank": per, "ms": ms,
               "frames_per_s": total * 1000.0 / ms,
               "checksum_digest": checksum_digest(hosts),
               "disparity_mean": float(sums.sum() / (total * SIZE * SIZE)),
               "spot_check": {"frames": [last, total - 1], "recomputed_on_rank0_equal": spot_ok},
               "input": "uniform [0,1] frames, seed n for frame n, generated on each device per batch",
               "timed": "generate + forward (graph replay) + checksums, device time, max over ranks"}
    return res


def bf16_throughput(local_rank, stream, ev0, ev1, batch=256, reps=5):
    """BF16 weights and activations (fp32 accumulation on tcgen05) at batch 256 on uniform
    frames: frames/s on device-resident inputs."""
    import torch
    import illumina
    from illumina import _lib

    arch = illumina.buildArchitecture(SIZE)
    m = illumina.createDepthModel(arch, synthSeed=0, maxBatch=batch, precision="bf16", device=local_rank)
    frames = torch.empty((batch, 3, SIZE, SIZE), dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(0, 0, batch, SIZE, frames.data_ptr(), None))
    disp = torch.empty((batch, SIZE, SIZE), dtype=torch.float32, device="cuda")
    for _ in range(3):
        m.forward(frames, disparity=disp, stream=stream)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(reps):
        m.forward(frames, disparity=disp, stream=stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / reps
    m.destroy()
    del frames, disp
    return {"frames_per_s": batch * 1000.0 / ms, "ms_per_step": ms, "batch": batch,
            "input": "uniform [0,1] frames", "precision": "bf16 weights+activations, fp32 accumulate"}


def run_ours(args, rank, local_rank, world):
    import numpy as np
    import torch

    import illumina
    from illumina import _lib

    torch.cuda.set_device(local_rank)
    ranks = RankGroup(world, "nccl", torch.device("cuda", local_rank))
    barrier, max_over_ranks = ranks.barrier, ranks.max

    B = args.batch
    arch = illumina.buildArchitecture(SIZE)
    cost = illumina.costOf(arch)
    model = illumina.createDepthModel(arch, synthSeed=0, maxBatch=B, precision=args.precision, device=local_rank)
    frames = torch.empty((B, 3, SIZE, SIZE), dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().illumina_generate_frames(1, frame_seed_base(rank, B), B, SIZE, frames.data_ptr(), None))
    disp = torch.empty((B, SIZE, SIZE), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    launches = model.stats.launches

    # ---- device-resident throughput (the value) ----
    for _ in range(max(3, args.warmup)):
        model.forward(frames, disparity=disp, stream=stream)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            model.forward(frames, disparity=disp, stream=stream)
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms)
    value = aggregate_frames_per_s(world, B, args.steps, ms_max)
    ms_per_step = ms_max / args.steps
    stats = model.stats
    launches = stats.launches

    # ---- end to end through the C ABI with host buffers ----
    e2e = e2e_sync = e2e_rgba8 = None
    if not args.no_e2e:
        host_in = torch.empty((B, 3, SIZE, SIZE), dtype=torch.float32, pin_memory=True)
        host_in.copy_(frames.cpu())
        host_out = torch.empty((B, SIZE, SIZE), dtype=torch.float32, pin_memory=True)
        hin, hout = host_in.numpy(), host_out.numpy()
        e_steps = max(3, min(args.steps, 20))
        # the reference's forward is a queue submission plus an asynchronous
        # readback: consecutive steps through illumina_forward_async overlap one
        # step's transfers with the neighbouring steps' graphs; each step still
        # uploads its frames and downloads its disparity inside the timed region
        host_out2 = [host_out, torch.empty((B, SIZE, SIZE), dtype=torch.float32, pin_memory=True)]
        hout2 = [h.numpy() for h in host_out2]
        for i in range(2):
            model.forwardAsync(hin, hout2[i], stream=stream)
        model.sync()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(e_steps):
            model.forwardAsync(hin, hout2[i % 2], stream=stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        model.sync()
        barrier()
        e_ms = max_over_ranks(ev0.elapsed_time(ev1))
        e2e = {"value": aggregate_frames_per_s(world, B, e_steps, e_ms), "unit": UNIT,
               "h2d_bytes_per_step": int(host_in.numel() * 4), "d2h_bytes_per_step": int(host_out.numel() * 4),
               "steps": e_steps,
               "path": "illumina_forward_async (C ABI): pinned host buffers, consecutive steps overlapped",
               "aggregate_pcie_gb_per_s": world * e_steps * (host_in.numel() + host_out.numel()) * 4 / e_ms / 1e6}
        # the synchronous call, one step at a time (frame chunks overlap within a step)
        for _ in range(2):
            model.forward(hin, disparity=hout, stream=stream)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(e_steps):
            model.forward(hin, disparity=hout, stream=stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
        s_ms = max_over_ranks(ev0.elapsed_time(ev1))
        e2e_sync = {"value": aggregate_frames_per_s(world, B, e_steps, s_ms), "unit": UNIT,
                    "h2d_bytes_per_step": int(host_in.numel() * 4), "d2h_bytes_per_step": int(host_out.numel() * 4),
                    "steps": e_steps, "path": "illumina_forward (C ABI), pinned host buffers, synchronous per step",
                    "aggregate_pcie_gb_per_s": world * e_steps * (host_in.numel() + host_out.numel()) * 4 / s_ms / 1e6}
        # the same frames as 8-bit RGBA source images at the network resolution
        # (the reference's input is an rgba8unorm texture): 4 bytes per pixel
        # cross PCIe instead of 12, sampled on the device by the same call
        rgba = torch.empty((B, SIZE, SIZE, 4), dtype=torch.uint8, device="cuda")
        rgba[..., :3] = (frames.permute(0, 2, 3, 1) * 255.0).round().clamp(0, 255).to(torch.uint8)
        rgba[..., 3] = 255
        host_src = torch.empty((B, SIZE, SIZE, 4), dtype=torch.uint8, pin_memory=True)
        host_src.copy_(rgba.cpu())
        hsrc = host_src.numpy()
        del rgba
        for i in range(2):
            model.forwardSourceAsync(hsrc, hout2[i], stream=stream)
        model.sync()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(e_steps):
            model.forwardSourceAsync(hsrc, hout2[i % 2], stream=stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        model.sync()
        barrier()
        r_ms = max_over_ranks(ev0.elapsed_time(ev1))
        e2e_rgba8 = {"value": aggregate_frames_per_s(world, B, e_steps, r_ms), "unit": UNIT,
                     "h2d_bytes_per_step": int(host_src.numel()), "d2h_bytes_per_step": int(host_out.numel() * 4),
                     "steps": e_steps,
                     "path": "illumina_forward_source_async (C ABI): pinned host RGBA8 448x448 frames (the fp32 "
                             "frames x 255, rounded) sampled on the device, disparity to pinned host memory, "
                             "consecutive steps overlapped",
                     "aggregate_pcie_gb_per_s": world * e_steps * (host_src.numel() + host_out.numel() * 4) / r_ms / 1e6}
        del host_in, host_out, host_src, host_out2

    # ---- box-scale streaming: 8192 seeded frames sharded over the ranks ----
    streaming = None
    if not args.no_extras:
        streaming = streaming_frames(model, rank, world, stream, ranks)

    # ---- roofline of the dominant kernel (live CUDA events on the launching stream) ----
    hbm, bf16, peak_src = measured_peaks()
    roofline = None
    per_op = {}
    if rank == 0:
        per_op = model.profile(frames, reps=2)
        alg = op_algorithmic(arch, cost, elt=4 if args.precision == "f32" else 2)
        wbytes = weight_bytes_per_op(arch, illumina.weightSpecs(arch))
        top = max(per_op, key=per_op.get)
        t_s = per_op[top] / 1000.0
        bytes_launch = alg[top][0] * B + wbytes.get(top, 0)
        flops_launch = alg[top][1] * B
        # an op whose successor ran inside its launch (the head folded into
        # d0.refine's epilogue: ~0 time of its own) also does that op's work
        names = [o.name for o in arch.ops]
        nxt = names[names.index(top) + 1] if names.index(top) + 1 < len(names) else None
        if nxt and per_op.get(nxt, 1.0) < 0.02 * per_op[top]:
            bytes_launch += alg[nxt][0] * B - e_in_bytes(arch, nxt, 4 if args.precision == "f32" else 2) * B
            bytes_launch += wbytes.get(nxt, 0)
            flops_launch += alg[nxt][1] * B
        achieved = bytes_launch / t_s / 1e9
        traffic = load_traffic().get(f"{top}@b{B}-{args.precision}")
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "traffic": traffic, "kernel": top, "launch_ms": per_op[top],
                    "algorithmic_bytes": bytes_launch, "flops": flops_launch,
                    "fp32_tflops_achieved": flops_launch / t_s / 1e12,
                    "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                    else "fallback 6.65 TB/s"}

    # ---- extras: batch-1 latency (config 1), the batch sweep (config 2) ----
    extras = {}
    if streaming is not None:
        extras["streaming_8192"] = streaming
    if rank == 0 and not args.no_extras:
        extras["batch_sweep"] = batch_sweep(model, frames, disp, stream, ev0, ev1)
        ring = 64  # 64 x 2.4 MB inputs > L2, so inputs are not cached between iterations
        b1_frames = torch.empty((ring, 3, SIZE, SIZE), dtype=torch.float32, device="cuda")
        _lib.check(_lib.lib().illumina_generate_frames(0, 0, ring, SIZE, b1_frames.data_ptr(), None))
        b1_out = torch.empty((1, SIZE, SIZE), dtype=torch.float32, device="cuda")
        views = [b1_frames[i:i + 1] for i in range(ring)]
        for v in views:
            model.forward(v, disparity=b1_out, stream=stream)
        torch.cuda.synchronize()
        ev0.record(stream)
        reps = 200
        for i in range(reps):
            model.forward(views[i % ring], disparity=b1_out, stream=stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        extras["batch1_us_per_frame"] = 1000.0 * ev0.elapsed_time(ev1) / reps
        extras["depth_relight_1080p"] = depth_relight_frame(model, b1_frames, ring, stream, ev0, ev1)
        extras["scene_448"] = scene_and_metrics(model, stream, ev0, ev1)
        extras["source_1080p"] = source_sampling(model, stream, ev0, ev1)
        del b1_frames
    if rank == 0 and not args.no_extras and args.precision == "f32":
        extras["bf16_b256"] = bf16_throughput(local_rank, stream, ev0, ev1)

    # ---- CPU baseline (rank 0, N=1 only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        n = threads * 2
        fps, dt = cpu_oracle_frames_per_s(n, threads)
        cpu = {"value": fps, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{n} blob frames of 3x448x448 ({dt:.1f} s over {threads} threads); oracle port of "
                         "src/model/reference.ts (double accumulation, f32 storage) + bilateralUp"}

    model.destroy()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
            "config": {"workload": f"illuminadepth448-forward-b{B}-blobs", "model": "IlluminaDepth-448",
                       "global_batch": B * world, "per_gpu_batch": B, "input": "3x448x448 fp32 blob frames",
                       "weights": "synthesizeWeights(seed 0)", "parallelism": f"replicas x{world} (frames sharded)",
                       "l2": f"inputs {B * 3 * SIZE * SIZE * 4 / 1e6:.0f} MB per step > 126 MB L2",
                       "precision": args.precision},
            "e2e": e2e, "e2e_sync": e2e_sync, "e2e_rgba8": e2e_rgba8, "gpu_launches": launches * args.steps, "launches_per_step": launches,
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks.summary(), **extras,
            "per_op_ms": {k: round(v, 4) for k, v in per_op.items()} if per_op else None,
        }
        print(json.dumps(line), flush=True)
    ranks.close()
    return 0


def run_only(args, local_rank):
    """One extra measurement alone (a small command to profile one kernel)."""
    import torch

    import illumina
    from illumina import _lib

    torch.cuda.set_device(local_rank)
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.only == "bf16":
        print(json.dumps({"bf16": bf16_throughput(local_rank, stream, ev0, ev1, batch=args.batch, reps=args.steps)}))
        return 0
    model = illumina.createDepthModel(illumina.buildArchitecture(SIZE), synthSeed=0, maxBatch=args.batch,
                                      precision=args.precision, device=local_rank)
    if args.only == "streaming":
        out = streaming_frames(model, 0, 1, stream, RankGroup(1), total=max(args.batch, 256 * args.steps),
                               batch=args.batch)
    else:
        ring = max(args.batch, 8)
        frames = torch.empty((ring, 3, SIZE, SIZE), dtype=torch.float32, device="cuda")
        _lib.check(_lib.lib().illumina_generate_frames(0 if args.only == "relight" else 1, 0, ring, SIZE,
                                                       frames.data_ptr(), None))
        if args.only == "relight":
            out = depth_relight_frame(model, frames, ring, stream, ev0, ev1, reps=args.steps)
        else:
            disp = torch.empty((ring, SIZE, SIZE), dtype=torch.float32, device="cuda")
            out = batch_sweep(model, frames, disp, stream, ev0, ev1, batches=(args.batch,), reps=args.steps)
    model.destroy()
    print(json.dumps({args.only: out}), flush=True)
    return 0


def main():
    args = parse_args()
    rank, local_rank, world = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.only:
        return run_only(args, local_rank) if rank == 0 else 0
    return run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
