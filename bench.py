"""Benchmark of the frame path on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload WORKLOAD] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1: frames shard across GPUs, no collective)

Workloads (the contract's configs):
  default   the headline, configs[1] SPAN x2 FP16 (a step = one batch of 8 synthetic 1080p frames,
            240 frames a GPU at K = 30), with configs[2] (SPAN x2 FP8 E4M3, key "span_fp8") and
            configs[3] at 3840x2160 (IFNet FP16, 8 frame pairs a step, key "rife_4k") timed in the
            same process, each with its own value, roofline, e2e, clocks and output check;
  span16 / span8 / rife (1080p; --height 2160 --width 3840 for 4K) / rife4k: one of those alone;
  rife425   RIFE 4.25 (the fused RIFE 4.2x plan, KB2_MODEL_RIFE_FUSED, seeded) at 3840x2160;
  chain     configs[4], the full chain: SPAN x2 FP8 on a 1080p stream, then IFNet at 3840x2160 for
            t = 0.2, 0.4, 0.6, 0.8 on every pair, 48-frame chunks dealt round-robin over the ranks,
            every output frame gathered to the host in order (a step = one chunk);
  janai / janai8  the AnimeJaNai unshuffle SPAN b8f64 of a seeded .span8 package (FP16 / E4M3 blocks);
  warp      frames at t = 1/3 from one mid-pair motion (kb2_warp_blend_at), 8 pairs of 1080p;
  kernels   one small pass of every kernel kind (--family to pick one), for the ncu summaries;
  hostcopy  the host traffic of the SPAN x2 e2e leg alone (its pinned uploads and display-pixel
            reads, no compute): the frames/s ceiling the host side sets at this many ranks.

`value` is whole-job frames/s with the inputs resident in HBM, timed with CUDA events on the enqueue
stream (max over ranks). `e2e` is the same through the public C ABI with pinned host frames: the
host->device copy of every step's inputs and the device->host read of every output inside the timed
region, the outputs as the display pixels a player shows (RGB10A2, 4 bytes a pixel: the SPAN engine's
display epilogue, kb2_pack_display after IFNet); `e2e_f16` reads the F16 frames instead. `roofline`
times the dominant kernel with CUDA events on its launching stream during the timed steps. `verify`
checks one output frame of the timed batch against the torch FP32 reference (tests/torch_ref.py).
`--impl reference` times the reference's own FP32 CPU implementation (its IR interpreter, compiled
from the reference sources into oracle/_ref) on the host cores, on bounded crops of the same frames.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "ultimate-anime-videoplayer_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

FRAME_H, FRAME_W = 1080, 1920
FLOP_PER_PX = 777888.0  # canonical SPAN x2: 388,944 MACs per input pixel
CHAIN_TIMES = (0.2, 0.4, 0.6, 0.8)
WORKLOADS = ("default", "span16", "span8", "rife", "rife4k", "rife425", "chain", "janai", "janai8", "warp", "kernels",
             "hostcopy",
             "tiles")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=WORKLOADS, default="default")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--height", type=int, default=None)
    ap.add_argument("--width", type=int, default=None)
    ap.add_argument("--timestep", type=float, default=0.5)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-verify", action="store_true")
    ap.add_argument("--dirty-rows", type=int, default=2,
                    help="--workload tiles: tile rows (of 64 input pixels) recomputed a step by moving tiles")
    ap.add_argument("--family", default="all", help="--workload kernels: all or one of " + ", ".join(
        ("span16", "span8", "rife", "rife425", "warp", "janai", "janai8")))
    a = ap.parse_args()
    if a.workload == "kernels" and "--batch" not in sys.argv:
        a.batch = 1
    if a.workload in ("rife4k", "rife425"):
        a.height, a.width = a.height or 2160, a.width or 3840
    a.height, a.width = a.height or FRAME_H, a.width or FRAME_W
    return a


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region (started before, stopped after)."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model():
    """The host CPU as lscpu names it (model name, sockets, cores a socket)."""
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
    except (OSError, subprocess.TimeoutExpired):
        return None
    info = {}
    for line in out.splitlines():
        if ":" in line:
            k, v = line.split(":", 1)
            info[k.strip()] = v.strip()
    return {"model": info.get("Model name"), "sockets": info.get("Socket(s)"),
            "cores_per_socket": info.get("Core(s) per socket"), "threads_per_core": info.get("Thread(s) per core")}


# ------------------------------------------------------------------------------------------------
# reference CPU implementation (the oracle/_ref build of the reference's own interpreter)
# ------------------------------------------------------------------------------------------------
CROP_H, CROP_W = 24, 48
RIFE_CROP_H, RIFE_CROP_W = 64, 96  # IFNet needs multiples of 32
RIFE42_CROP_H, RIFE42_CROP_W = 64, 128  # RIFE 4.25: multiples of 4 x 8


def reference_sample(threads, frame, flat, crops_per_thread=1, frame_b=None, timestep=0.5, full=None, rife42=False):
    """Each host thread runs the reference's FP32 network on its own crop of the frame (the
    interpreter is single-threaded per call); returns (frames processed, seconds). SPAN when
    frame_b is None, else IFNet (RIFE 4.2x with rife42) on the crop pair; `flat` given as bytes is a
    .span8 package, run by the reference's unshuffle-SPAN forward (src/gpu/span_fp8/forward.cpp:144)."""
    from oracle import ref_lib
    import numpy as np

    rife = frame_b is not None
    ch, cw = crop_of(rife, rife42)
    H, W = frame.shape[1:]
    rng = np.random.default_rng(0)
    jobs = []
    for t in range(threads):
        for _ in range(crops_per_thread):
            y = int(rng.integers(0, H - ch))
            x = int(rng.integers(0, W - cw))
            a = np.ascontiguousarray(frame[None, :, y:y + ch, x:x + cw])
            b = np.ascontiguousarray(frame_b[None, :, y:y + ch, x:x + cw]) if rife else None
            jobs.append((t, a, b))
    done = [0] * threads

    def work(t):
        for tt, a, b in jobs:
            if tt == t:
                if rife42:
                    ref_lib.rife42_forward(a, b, timestep, flat)
                elif rife:
                    ref_lib.ifnet_forward(a, b, timestep, flat)
                elif isinstance(flat, bytes):
                    ref_lib.span8_forward(flat, a)
                else:
                    ref_lib.span_forward(a, flat)
                done[t] += 1

    ts = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    t0 = time.perf_counter()
    for th in ts:
        th.start()
    for th in ts:
        th.join()
    dt = time.perf_counter() - t0
    fh, fw = full if full is not None else (FRAME_H, FRAME_W)
    return sum(done) * ch * cw / float(fh * fw), dt


def crop_of(rife, rife42=False):
    """The crop each reference thread runs: SPAN, IFNet or RIFE 4.25."""
    if rife42:
        return RIFE42_CROP_H, RIFE42_CROP_W
    return (RIFE_CROP_H, RIFE_CROP_W) if rife else (CROP_H, CROP_W)


def janai_package(fp8, H, W, device=0):
    """The seeded b8f64 .span8 package of the janai workloads; FP8: the same contents with activation
    scales derived from the peaks the FP16 engine of the package measures on four seeded frames
    (kb2_span_calibrate; the reference derives them offline the same way, derive.h:42-62)."""
    import numpy as np
    import torch
    import kirari_b200 as kb
    import seeded
    from synth import anime_frames
    p = seeded.span8_init(8, 64, seed=3)
    pkg = seeded.span8_package(p)
    if not fp8:
        return pkg
    e16 = kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, pkg, H, W, max_batch=4, device=device)
    frames = torch.from_numpy(anime_frames(4, H, W, seed=900).astype(np.float16)).cuda()
    peaks = e16.calibrate(frames, n_peaks=1 + 3 * p["blocks"])
    e16.close()
    return seeded.span8_package(seeded.span8_fp8_from_peaks(p, peaks))


def config0_one_thread():
    """configs[0] in full on one host thread: one 1x3x270x480 frame through the reference's FP32
    interpreter (a single call, single-threaded); seconds."""
    import numpy as np
    import seeded
    from oracle import ref_lib
    x = np.random.default_rng(0).random((1, 3, 270, 480), dtype=np.float32)
    t0 = time.perf_counter()
    ref_lib.span_forward(x, seeded.span_flat(seeded.span_init(1)))
    return time.perf_counter() - t0


def cpu_baseline(frame, flat, budget_s=12.0, frame_b=None, timestep=0.5, full=None, with_config0=False,
                 rife42=False):
    from oracle import ref_lib
    if not ref_lib.available():
        return None
    cores = host_cores()
    kw = dict(frame_b=frame_b, timestep=timestep, full=full, rife42=rife42)
    frames, dt = reference_sample(cores, frame, flat, **kw)
    reps = max(1, int(budget_s / max(dt, 1e-3)))
    if reps > 1:
        frames, dt = reference_sample(cores, frame, flat, crops_per_thread=reps, **kw)
    ch, cw = crop_of(frame_b is not None, rife42)
    fh, fw = full if full is not None else (FRAME_H, FRAME_W)
    net = ("RIFE 4.25 pairs" if rife42 else "IFNet pairs" if frame_b is not None else
           "unshuffle SPAN b8f64" if isinstance(flat, bytes) else "SPAN")
    out = {"value": frames / dt, "unit": "frames/s", "cores": cores, "kind": "reference", "cpu": cpu_model(),
           "sample": f"{cores} threads x {reps} {net} crops of {ch}x{cw} px of synthetic {fw}x{fh} frames, "
                     f"reference FP32 IR interpreter (oracle/_ref), scaled by pixels to {fw}x{fh} frames"}
    if with_config0:
        s = config0_one_thread()
        out["config0_one_thread"] = {"seconds": s, "frames_per_s": 1.0 / s,
                                     "sample": "configs[0] in full: one 1x3x270x480 frame, one interpreter call "
                                               "on one host thread"}
    return out


def workload_desc(workload, B, H, W, timestep, steps, world=1):
    """metric, dtype, config of an engine workload (shared by both arms)."""
    if workload == "rife425":
        metric = f"RIFE 4.25 {W}x{H} interpolated frames/s"
        config = {"workload": f"RIFE 4.25 (fused RIFE 4.2x plan, seeded weights) FP16, {B} frame pairs per step, "
                              f"{W}x{H}, t={timestep}",
                  "global_batch": B * world, "frames_per_gpu": B * steps,
                  "parallelism": f"pair-sharded x{world}, no collective",
                  "l2": f"working set > L2: {B} pairs of {W}x{H} FP16 frames and their activations"}
        return metric, "f16", config
    if workload in ("rife", "rife4k"):
        metric = f"RIFE IFNet {W}x{H} interpolated frames/s"
        config = {"workload": f"configs[3] IFNet FP16, {B} frame pairs per step, {W}x{H}, t={timestep}",
                  "global_batch": B * world, "frames_per_gpu": B * steps,
                  "parallelism": f"pair-sharded x{world}, no collective",
                  "l2": f"working set > L2: {B} pairs of {W}x{H} FP16 frames and their activations"}
        return metric, "f16", config
    if workload in ("janai", "janai8"):
        q = workload == "janai8"
        metric = ("SPAN b8f64 unshuffle x2 1080p->2160p frames/s" if (H, W) == (FRAME_H, FRAME_W)
                  else f"SPAN b8f64 unshuffle x2 {W}x{H} frames/s")
        config = {"workload": f"AnimeJaNai unshuffle SPAN b8f64 {'E4M3 blocks' if q else 'FP16'} "
                              f"(.span8 package, seeded), batch {B}, {H}x{W} -> {2 * H}x{2 * W}",
                  "global_batch": B * world, "frames_per_gpu": B * steps,
                  "parallelism": f"frame-sharded x{world}, no collective",
                  "l2": "working set > L2: each layer reads and writes 8 x 66 MB activations (half resolution)"}
        return metric, ("e4m3+f16" if q else "f16"), config
    fp8 = workload == "span8"
    metric = "SPAN x2 1080p->2160p frames/s" if (H, W) == (FRAME_H, FRAME_W) else f"SPAN x2 {W}x{H} frames/s"
    config = {"workload": ("configs[2] SPAN x2 FP8 E4M3" if fp8 else "configs[1] SPAN x2 FP16")
                          + f", batch {B}, {H}x{W} -> {2 * H}x{2 * W}",
              "global_batch": B * world, "frames_per_gpu": B * steps,
              "parallelism": f"frame-sharded x{world}, no collective",
              "l2": "working set > L2: each layer reads and writes 8 x 199 MB activations"}
    return metric, ("e4m3+f16" if fp8 else "f16"), config


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    import numpy as np
    import seeded
    from oracle import ref_lib
    from synth import anime_frame, shifted_pair

    workload = "span16" if args.workload in ("default", "chain") else args.workload
    if workload == "warp":
        return run_warp_reference(args)
    metric, _, config = workload_desc(workload, args.batch, args.height, args.width, args.timestep, args.steps, world)
    config = dict(config, workload=config["workload"] + ", reference FP32 CPU path")
    if not ref_lib.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (reference sources absent)"}))
        return
    rife = workload in ("rife", "rife4k", "rife425")
    rife42 = workload == "rife425"
    if rife:
        fa, fb = shifted_pair(args.height, args.width, 0)
        frame, frame_b = np.ascontiguousarray(fa, np.float32), np.ascontiguousarray(fb, np.float32)
        flat = rife42_flat() if rife42 else seeded.ifnet_flat(seeded.ifnet_init(2))
    elif workload in ("janai", "janai8"):
        # the reference's FP32 forward reads the package's FP16 weights; the E4M3 scales do not enter it
        frame, frame_b = anime_frame(args.height, args.width, 0).astype(np.float32), None
        flat = janai_package(False, args.height, args.width)
    else:
        frame, frame_b = anime_frame(args.height, args.width, 0).astype(np.float32), None
        flat = seeded.span_flat(seeded.span_init(1))
    kw = dict(frame_b=frame_b, timestep=args.timestep, full=(args.height, args.width), rife42=rife42)
    cores = host_cores()
    for _ in range(args.warmup):
        reference_sample(cores, frame, flat, **kw)
    total_frames, total_s = 0.0, 0.0
    for _ in range(args.steps):
        f, dt = reference_sample(cores, frame, flat, **kw)
        total_frames += f
        total_s += dt
    value = total_frames / total_s
    ch, cw = crop_of(rife, rife42)
    line = {"metric": metric, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_s / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference", "config": config,
            "cpu_baseline": {"value": value, "unit": "frames/s", "cores": cores, "kind": "reference",
                             "cpu": cpu_model(),
                             "sample": f"per step: {cores} threads x 1 crop of {ch}x{cw} px, "
                                       f"scaled by pixels to {args.width}x{args.height} frames"},
            "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ------------------------------------------------------------------------------------------------
# this library
# ------------------------------------------------------------------------------------------------
class Dist:
    """The process's rank / device and the two collectives the bench uses (barrier, max-over-ranks)."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.rank, self.local_rank, self.world = dist_env()
        torch.cuda.set_device(self.local_rank)
        if self.world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local_rank))

    def barrier(self):
        import shard
        shard.barrier("cuda")

    def max(self, v):
        import shard
        return shard.max_over_ranks(v, "cuda")

    def close(self):
        import torch.distributed as dist
        if self.world > 1:
            dist.destroy_process_group()


def rife42_flat():
    """The seeded RIFE 4.25 parameter array of the rife425 workload (12 plan floats first)."""
    import seeded
    plan = seeded.RIFE_PLANS["4.25"]
    return seeded.rife_flat(seeded.rife_init(plan), plan)


def calibrated_scales(blob, H, W, B, device):
    """configs[2]'s activation scales: the FP16 engine's peaks over 16 seeded frames (not the timed
    ones), scale = max(peak, 2^-14) * 1.25 / 448 (the reference's derive, derive.h:42-62)."""
    import numpy as np
    import torch
    import kirari_b200 as kb
    import seeded
    from synth import anime_frames
    calib = torch.from_numpy(anime_frames(16, H, W, seed=1000).astype(np.float16)).cuda()
    e16 = kb.Engine(kb.MODEL_SPAN_X2, blob, H, W, max_batch=B, device=device)
    peaks = e16.calibrate(calib)
    e16.close()
    del calib
    return seeded.scales_from_peaks(peaks, floor=2.0 ** -14)


def setup_leg(workload, B, H, W, timestep, D):
    """Engine, host inputs and output shape of an engine workload."""
    import numpy as np
    import kirari_b200 as kb
    import seeded
    import shard
    from synth import anime_frames, shifted_pair

    leg = {"workload": workload, "B": B, "H": H, "W": W, "timestep": timestep,
           "rife": workload in ("rife", "rife4k", "rife425"), "r42": workload == "rife425",
           "janai": workload in ("janai", "janai8"), "fp8": workload == "span8"}
    if leg["janai"]:
        q = workload == "janai8"
        leg["flat"] = janai_package(q, H, W, D.local_rank)
        leg["frames"] = anime_frames(B, H, W, seed=shard.frame_seed(10, D.rank, 0)).astype(np.float16)
        leg["eng"] = kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, leg["flat"], H, W, max_batch=B,
                               precision=kb.PREC_FP8 if q else kb.PREC_FP16, device=D.local_rank)
        leg["host_in"] = [leg["frames"]]
        leg["out_shape"] = (B, 3, 2 * H, 2 * W)
    elif leg["rife"]:
        if leg["r42"]:
            leg["flat"] = rife42_flat()
        else:
            leg["params"] = seeded.ifnet_init(2)
            leg["flat"] = seeded.ifnet_flat(leg["params"])
        # 4 distinct seeded pairs, each used twice in the step's 8 (generating 4K frames is slow on
        # the host); the step's inputs are still 8 x 2 x 49.8 MB at 4K, far above the 126 MB L2
        uniq = min(B, 4)
        pairs = [shifted_pair(H, W, seed=shard.frame_seed(10, D.rank, i)) for i in range(uniq)]
        leg["frames"] = np.ascontiguousarray(np.stack([pairs[i % uniq][0] for i in range(B)]), np.float16)
        leg["frames_b"] = np.ascontiguousarray(np.stack([pairs[i % uniq][1] for i in range(B)]), np.float16)
        model = kb.MODEL_RIFE_FUSED if leg["r42"] else kb.MODEL_IFNET
        leg["eng"] = kb.Engine(model, kb.make_blob(model, leg["flat"]), H, W, max_batch=B, device=D.local_rank)
        leg["eng"].set_timestep(timestep)
        leg["host_in"] = [leg["frames"], leg["frames_b"]]
        leg["out_shape"] = (B, 3, H, W)
    else:
        p = seeded.span_init(1)
        leg["params"] = p
        leg["flat"] = seeded.span_flat(p)
        blob = kb.make_blob(kb.MODEL_SPAN_X2, leg["flat"])
        leg["frames"] = anime_frames(B, H, W, seed=shard.frame_seed(10, D.rank, 0)).astype(np.float16)
        scales = calibrated_scales(blob, H, W, B, D.local_rank) if leg["fp8"] else None
        leg["eng"] = kb.Engine(kb.MODEL_SPAN_X2, blob, H, W, max_batch=B,
                               precision=kb.PREC_FP8 if leg["fp8"] else kb.PREC_FP16, act_scales=scales,
                               device=D.local_rank)
        leg["host_in"] = [leg["frames"]]
        leg["out_shape"] = (B, 3, 2 * H, 2 * W)
    return leg


def verify_leg(leg, d_in, d_out):
    """One output frame of the timed batch (frame 0 of the last step) against the torch FP32
    reference: SPAN on a 64x128 crop with a 24-pixel halo (the network's receptive radius is 20),
    IFNet on the whole padded pair. FP16: max-abs <= 2/255 after clamp; E4M3: PSNR >= 45 dB."""
    import numpy as np
    import torch
    tests_dir = os.path.join(ROOT, "tests")
    if tests_dir not in sys.path:
        sys.path.insert(0, tests_dir)
    import torch_ref

    def clamp01(v):
        return np.clip(np.asarray(v, np.float32), 0.0, 1.0)

    if leg["janai"]:
        return None
    H, W = leg["H"], leg["W"]
    if leg["rife"]:
        a = d_in[0][0:1].float().cpu().numpy()
        b = d_in[1][0:1].float().cpu().numpy()
        al = 64 if leg["r42"] else 32
        hp, wp = -(-H // al) * al, -(-W // al) * al
        top, left = ((hp - H) // 2) & ~1, ((wp - W) // 2) & ~1
        pa = np.zeros((1, 3, hp, wp), np.float32)
        pb = np.zeros((1, 3, hp, wp), np.float32)
        pa[:, :, top:top + H, left:left + W] = a
        pb[:, :, top:top + H, left:left + W] = b
        if leg["r42"]:
            ref = torch_ref.rife42_forward(pa, pb, leg["timestep"], leg["flat"])[0][:, :, top:top + H, left:left + W]
        else:
            ref = torch_ref.ifnet_forward(pa, pb, leg["timestep"], leg["params"])[:, :, top:top + H, left:left + W]
        got = d_out[0:1].float().cpu().numpy()
        err = float(np.max(np.abs(clamp01(got) - clamp01(ref))))
        torch.cuda.empty_cache()
        return {"frame": 0, "region": f"whole {W}x{H} frame",
                "reference": f"torch FP32 {'RIFE 4.25' if leg['r42'] else 'IFNet'} (tests/torch_ref.py)",
                "max_abs_255": err * 255.0, "ok": bool(err <= 2.0 / 255.0)}
    ch, cw, halo = 64, 128, 24
    y0, x0 = max(0, H // 2 - ch // 2), max(0, W // 2 - cw // 2)
    ya, yb = max(0, y0 - halo), min(H, y0 + ch + halo)
    xa, xb = max(0, x0 - halo), min(W, x0 + cw + halo)
    crop = d_in[0][0:1, :, ya:yb, xa:xb].float().cpu().numpy()
    ref = torch_ref.span_forward(crop, leg["params"])
    ref = ref[:, :, 2 * (y0 - ya):2 * (y0 - ya + ch), 2 * (x0 - xa):2 * (x0 - xa + cw)]
    got = d_out[0:1, :, 2 * y0:2 * (y0 + ch), 2 * x0:2 * (x0 + cw)].float().cpu().numpy()
    diff = clamp01(got) - clamp01(ref)
    err = float(np.max(np.abs(diff)))
    mse = float(np.mean(diff.astype(np.float64) ** 2))
    db = float("inf") if mse == 0 else float(10.0 * np.log10(1.0 / mse))
    ok = bool(db >= 45.0) if leg["fp8"] else bool(err <= 2.0 / 255.0)
    out = {"frame": 0, "region": f"{cw}x{ch} input px at ({x0}, {y0}) with a {halo}-px halo",
           "reference": "torch FP32 SPAN (tests/torch_ref.py)", "max_abs_255": err * 255.0, "psnr_db": db, "ok": ok}
    if leg["fp8"]:
        out["note"] = ("with the configs' Kaiming-seeded weights the activations of blocks 1-5 (the E4M3 ones) "
                       "decay below 1e-5, so the output is carried by conv_1 and block 0 (FP16) and matches the "
                       "FP16 leg's here; E4M3 on a network whose every block carries signal is checked by "
                       "tests/test_span_gpu.py::test_fp8_live_blocks_psnr")
    return out


def e2e_leg(leg, D, eng, sh, stream, d_in, steps, warmup, display):
    """The engine driven with pinned host frames: per step the H2D copy of its inputs, the enqueue,
    and the D2H read of every output (display pixels when `display`: the SPAN engine's display
    epilogue, or kb2_pack_display after IFNet), double-buffered across three streams, wall-clock
    timed between barriers (max over ranks)."""
    import numpy as np
    import torch
    import kirari_b200 as kb
    import shard
    B, H, W = leg["B"], leg["H"], leg["W"]
    rife = leg["rife"]
    out_hw = (H, W) if rife else (2 * H, 2 * W)
    frames = leg["frames"]
    if rife:
        # a video stream: pair i is (f_i, f_i+1), so the two input tensors are views one frame apart
        # into a (B + 1)-frame device buffer. Each step uploads its B new frames; the previous step's
        # last frame is copied on the device into slot 0, as a player keeps it.
        h_in = [torch.from_numpy(np.ascontiguousarray(np.concatenate([frames[1:], leg["frames_b"][-1:]]))).pin_memory()]
        d_seq = [torch.empty((B + 1,) + tuple(frames.shape[1:]), dtype=torch.float16, device="cuda") for _ in range(2)]
        for t in d_seq:
            t[0].copy_(d_in[0][0])
            t[1:].copy_(h_in[0].cuda())
        d_ins = [[t[1:]] for t in d_seq]
        views = [[t[:B], t[1:]] for t in d_seq]
    else:
        h_in = [torch.from_numpy(x).pin_memory() for x in leg["host_in"]]
        d_ins = [[torch.empty_like(t) for t in d_in] for _ in range(2)]
        views = d_ins
    span_display = display and not rife
    if span_display:
        eng.set_output_format(kb.DISPLAY_RGB10A2)
        d_outs = [torch.empty((B, 4) + out_hw, dtype=torch.uint8, device="cuda") for _ in range(2)]
    else:
        d_outs = [torch.empty((B, 3) + out_hw, dtype=torch.float16, device="cuda") for _ in range(2)]
    if display and rife:  # the frames packed by kb2_pack_display, as the ring store does
        d_pix = [torch.empty((B,) + out_hw, dtype=torch.int32, device="cuda") for _ in range(2)]
        h_out = [torch.empty((B,) + out_hw, dtype=torch.int32).pin_memory() for _ in range(2)]
        pix_t = [kb.to_kb2_tensor(t) for t in d_outs]
    else:
        d_pix = None
        h_out = [torch.empty(tuple(t.shape), dtype=t.dtype).pin_memory() for t in d_outs]
    s_h2d, s_d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ins2 = [(kb.Tensor * len(v))(*[kb.to_kb2_tensor(t) for t in v]) for v in views]
    outs2 = [(kb.Tensor * 1)(kb.to_kb2_tensor(t)) for t in d_outs]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]

    def pipeline(n_steps):
        for i in range(n_steps):
            k = i % 2
            with torch.cuda.stream(s_h2d):
                if i >= 2:
                    s_h2d.wait_event(ev_free[k])
                if rife:  # carry the previous step's last frame (its upload precedes on this stream)
                    d_seq[k][0].copy_(d_seq[1 - k][B], non_blocking=True)
                for dst, src in zip(d_ins[k], h_in):
                    dst.copy_(src, non_blocking=True)
                ev_in[k].record(s_h2d)
            stream.wait_event(ev_in[k])
            if i >= 2:
                stream.wait_event(ev_free[k])
            eng.enqueue_raw(ins2[k], outs2[k], sh)
            if d_pix is not None:
                rc = kb.lib().kb2_pack_display(sh, kb.ctypes.byref(pix_t[k]), kb.DISPLAY_RGB10A2,
                                               kb.ctypes.c_void_p(d_pix[k].data_ptr()), out_hw[1] * 4)
                if rc != kb.KB2_OK:
                    raise kb.KB2Error(rc, "kb2_pack_display")
            ev_done[k].record(stream)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(ev_done[k])
                h_out[k].copy_(d_pix[k] if d_pix is not None else d_outs[k], non_blocking=True)
                ev_free[k].record(s_d2h)
        torch.cuda.synchronize()

    pipeline(min(2, warmup))
    D.barrier()
    t0 = time.perf_counter()
    pipeline(steps)
    D.barrier()
    e2e_s = D.max(time.perf_counter() - t0)
    if span_display:
        eng.set_output_format(0)
    out_bytes = int(h_out[0].numel() * h_out[0].element_size())
    in_bytes = int(sum(t.numel() * 2 for t in h_in))
    what = ("display pixels (RGB10A2, 4 B/px) from the SPAN engine's display epilogue" if span_display else
            "display pixels (RGB10A2, 4 B/px) packed by kb2_pack_display after the engine" if d_pix is not None else
            "F16 NCHW frames (6 B/px)")
    return {"value": shard.whole_job_rate(B * steps, D.world, e2e_s), "unit": "frames/s",
            "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes,
            "h2d_gbs": in_bytes * steps / e2e_s / 1e9, "d2h_gbs": out_bytes * steps / e2e_s / 1e9,
            "path": "kb2_enqueue with pinned host frames: H2D copy, enqueue, D2H of every output as " + what +
                    ", double-buffered across three streams" +
                    ("; RIFE as a video stream: B new frames uploaded a step, pair i = (f_i, f_i+1) as two views "
                     "of one device buffer, the step's first frame carried on the device" if rife else "")}


def run_leg(workload, args, D, B, H, W, steps, headline):
    """One engine workload: device-resident timing with per-layer events, the roofline of the top
    kernel, the output check, the e2e legs and (rank 0, N = 1) the CPU baseline."""
    import numpy as np
    import torch
    import kirari_b200 as kb
    import shard

    metric, dtype, config = workload_desc(workload, B, H, W, args.timestep, steps, D.world)
    leg = setup_leg(workload, B, H, W, args.timestep, D)
    eng = leg["eng"]
    d_in = [torch.from_numpy(x).cuda() for x in leg["host_in"]]
    d_out = torch.empty(leg["out_shape"], dtype=torch.float16, device="cuda")
    stream = torch.cuda.Stream()
    sh = kb.ctypes.c_void_p(stream.cuda_stream)
    ins = (kb.Tensor * len(d_in))(*[kb.to_kb2_tensor(t) for t in d_in])
    outs = (kb.Tensor * 1)(kb.to_kb2_tensor(d_out))

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            eng.enqueue_raw(ins, outs, sh)
    stream.synchronize()
    eng.check_device(stream)
    eng.read_profile()
    eng.set_profiling(True)
    clocks = ClockSampler(D.local_rank)
    clocks.start()
    D.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        eng.enqueue_raw(ins, outs, sh)
    stop.record(stream)
    stop.synchronize()
    D.barrier()
    clk = clocks.stop()
    eng.set_profiling(False)
    eng.check_device(stream)
    ms = D.max(start.elapsed_time(stop))
    profile = eng.read_profile()
    value = shard.whole_job_rate(B * steps, D.world, ms / 1e3)

    # roofline of the dominant kernel, from its launches inside the timed region
    peaks_json, peak_kind = measured_peaks()
    top_name, top = max(profile.items(), key=lambda kv: kv[1]["total_ms"])
    avg_ms = top["total_ms"] / max(1, top["launches"])
    tflops = top["flops"] / (avg_ms / 1e3) / 1e12
    fp8_top = top_name.endswith(".fp8")
    # the timed region is well under a second of work: the burst peak (MEASURED_PEAKS bf16_tflops)
    peak = float(peaks_json["bf16_tflops"]) * (2.0 if fp8_top else 1.0)
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get(top_name, {}).get(f"{B}x{H}x{W}")
    except (OSError, ValueError):
        pass
    total_flops = sum(v["flops"] * v["launches"] for v in profile.values())
    net_tflops = total_flops / (ms / 1e3) / 1e12
    # the bound is whichever roof is lower for this kernel: its FLOPs at the tensor peak or its
    # algorithmic bytes at the HBM peak (a layer-by-layer 48-channel conv is HBM-bound in both precisions)
    hbm_peak = float(peaks_json["hbm_gbs"])
    hbm_gbs = top["bytes"] / (avg_ms / 1e3) / 1e9
    t_tensor = top["flops"] / (peak * 1e12)
    t_hbm = top["bytes"] / (hbm_peak * 1e9)
    if t_hbm > t_tensor:
        main = {"bound": "hbm", "achieved": hbm_gbs, "peak": hbm_peak, "unit": "GB/s", "frac": hbm_gbs / hbm_peak}
    else:
        main = {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s", "frac": tflops / peak}
    roofline = {**main,
                "traffic": traffic, "kernel": top_name, "launches": top["launches"], "avg_launch_ms": avg_ms,
                "flops_per_launch": top["flops"], "algorithmic_bytes_per_launch": top["bytes"],
                "roof_ms": max(t_tensor, t_hbm) * 1e3, "frac_of_roof": max(t_tensor, t_hbm) / (avg_ms / 1e3),
                "tflops": tflops, "tensor_peak": peak, "tensor_frac": tflops / peak,
                "hbm_gbs": hbm_gbs, "hbm_frac": hbm_gbs / hbm_peak,
                "peak_source": f"{peak_kind} bf16_tflops (burst)" + (" x2 (E4M3)" if fp8_top else "")
                + f", {peak_kind} hbm_gbs",
                "network_tflops": net_tflops, "network_frac": net_tflops / peak}
    layers = {k: {"launches": v["launches"], "ms_per_launch": v["total_ms"] / max(1, v["launches"]),
                  "share": v["total_ms"] / max(1e-9, sum(x["total_ms"] for x in profile.values())),
                  "tflops": v["flops"] / max(1e-12, v["total_ms"] / max(1, v["launches"]) / 1e3) / 1e12,
                  "hbm_gbs": v["bytes"] / max(1e-12, v["total_ms"] / max(1, v["launches"]) / 1e3) / 1e9}
              for k, v in profile.items() if v["launches"] > 0}

    verify = None
    if not args.no_verify and D.rank == 0:
        verify = verify_leg(leg, d_in, d_out)
    e2e = e2e_f16 = None
    if not args.no_e2e:
        e2e = e2e_leg(leg, D, eng, sh, stream, d_in, steps, args.warmup, display=not leg["janai"])
        if not leg["janai"]:
            e2e_f16 = e2e_leg(leg, D, eng, sh, stream, d_in, steps, args.warmup, display=False)
        eng.check_device(stream)
    launches = steps * eng.launches_per_enqueue()
    cpu = None
    if D.rank == 0 and D.world == 1 and not args.no_cpu_baseline and cpu_budget(headline, leg):
        fr = leg["frames"][0].astype(np.float32)
        cpu = cpu_baseline(fr, leg["flat"], frame_b=leg["frames_b"][0].astype(np.float32) if leg["rife"] else None,
                           rife42=leg["r42"],
                           timestep=args.timestep, full=(H, W), with_config0=headline)
    eng.close()
    del d_in, d_out
    torch.cuda.empty_cache()
    return {"metric": metric, "value": value, "unit": "frames/s", "n_gpus": D.world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded anime-like frames, seeded weights)",
            "config": config, "roofline": roofline, "layers": layers, "e2e": e2e, "e2e_f16": e2e_f16,
            "gpu_launches": launches, "clocks": clk, "verify": verify, "cpu_baseline": cpu}


def cpu_budget(headline, leg):
    """Which legs time the reference on the host: the headline, and RIFE (another network). The FP8
    leg runs the same network as the headline, whose reference is the same FP32 interpreter."""
    return headline or leg["rife"] or leg["janai"]


def run_ours(args):
    D = Dist()
    B, H, W = args.batch, args.height, args.width
    if args.workload == "default":
        line = run_leg("span16", args, D, B, FRAME_H, FRAME_W, args.steps, headline=True)
        fp8 = run_leg("span8", args, D, B, FRAME_H, FRAME_W, args.steps, headline=False)
        if fp8["cpu_baseline"] is None and line["cpu_baseline"] is not None:
            fp8["cpu_baseline"] = dict(line["cpu_baseline"], sample="the headline's: the reference's CPU path for "
                                       "this network is the same FP32 interpreter, whatever the GPU precision")
        line["span_fp8"] = fp8
        line["rife_4k"] = run_leg("rife4k", args, D, B, 2160, 3840, args.steps, headline=False)
        line["config"] = dict(line["config"], also=["span_fp8: configs[2] SPAN x2 FP8 E4M3, batch 8, 1080p",
                                                     "rife_4k: configs[3] IFNet FP16 at 3840x2160, 8 pairs"])
    else:
        line = run_leg(args.workload, args, D, B, H, W, args.steps, headline=True)
    if D.rank == 0:
        print(json.dumps(line))
    D.close()


# ------------------------------------------------------------------------------------------------
# the full chain, SPAN FP8 -> IFNet 4K at four instants, chunked over ranks
# ------------------------------------------------------------------------------------------------
def run_chain(args):
    """Per rank, `steps` chunks of 48 source frames (chunk c of the stream on rank c % N, each
    chunk also reading the next chunk's first frame, shard.chunks_for_rank): SPAN x2 FP8 upscales
    the chunk's 49 1080p frames to 3840x2160, then IFNet interpolates its 48 pairs at t = 0.2, 0.4,
    0.6, 0.8. Every output frame (48 upscaled + 192 interpolated a chunk) is packed to RGB10A2 and
    gathered to pinned host memory at its place in the output sequence. `value` counts output 4K
    frames a second with the sources resident and no gather (device events); `e2e` adds the upload
    of the 1080p sources and the gather, overlapped with the next chunk's work on two streams."""
    import numpy as np
    import torch
    import kirari_b200 as kb
    import seeded
    import shard
    from synth import anime_frames

    D = Dist()
    B = args.batch
    H, W = FRAME_H, FRAME_W
    H4, W4 = 2 * H, 2 * W
    chunk = shard.CHAIN_CHUNK
    steps = args.steps
    n_frames = chunk * steps * D.world + 1
    my = shard.chunks_for_rank(n_frames, D.world, D.rank)[:steps]
    src_n = chunk + 1
    # sources: 13 distinct seeded frames cycled (host generation of 49 frames a chunk is slow)
    uniq = anime_frames(13, H, W, seed=shard.frame_seed(20, D.rank, 0)).astype(np.float16)
    src_host = torch.from_numpy(np.ascontiguousarray(uniq[np.arange(src_n) % 13])).pin_memory()
    span_blob = kb.make_blob(kb.MODEL_SPAN_X2, seeded.span_flat(seeded.span_init(1)))
    scales = calibrated_scales(span_blob, H, W, B, D.local_rank)
    span = kb.Engine(kb.MODEL_SPAN_X2, span_blob, H, W, max_batch=B, precision=kb.PREC_FP8, act_scales=scales,
                     device=D.local_rank)
    rife = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, seeded.ifnet_flat(seeded.ifnet_init(2))), H4, W4,
                     max_batch=B, device=D.local_rank)
    src = torch.empty((src_n, 3, H, W), dtype=torch.float16, device="cuda")
    up = torch.empty((src_n, 3, H4, W4), dtype=torch.float16, device="cuda")  # upscaled chunk (RIFE's input)
    mid = torch.empty((B, 3, H4, W4), dtype=torch.float16, device="cuda")    # one batch of interpolated frames
    out_per_chunk = chunk * (1 + len(CHAIN_TIMES))
    pix = [torch.empty((out_per_chunk, H4, W4), dtype=torch.int32, device="cuda") for _ in range(2)]
    # one pinned host buffer a rank (a chunk's 240 RGB10A2 frames, 8 GB): the copy stream writes the
    # chunks into it one after the other, in order, while the next chunk computes into the other pix
    host_ring = torch.empty((out_per_chunk, H4, W4), dtype=torch.int32).pin_memory()
    stream = torch.cuda.Stream()
    s_copy = torch.cuda.Stream()
    sh = kb.ctypes.c_void_p(stream.cuda_stream)
    T = kb.to_kb2_tensor
    L = kb.lib()

    def pack(frames_t, dst):  # F16 frames -> RGB10A2 rows (kb2_pack_display) on `stream`
        t = T(frames_t)
        rc = L.kb2_pack_display(sh, kb.ctypes.byref(t), kb.DISPLAY_RGB10A2, kb.ctypes.c_void_p(dst.data_ptr()),
                                W4 * 4)
        if rc != kb.KB2_OK:
            raise kb.KB2Error(rc, "kb2_pack_display")

    def compute(k):
        """One chunk's work on `stream` into pix[k]; output order: for source frame i of the chunk,
        its upscaled frame, then the 4 instants of pair (i, i + 1)."""
        launches = 0
        for f0 in range(0, src_n, B):
            n = min(B, src_n - f0)
            span.enqueue_raw((kb.Tensor * 1)(T(src[f0:f0 + n])), (kb.Tensor * 1)(T(up[f0:f0 + n])), sh)
            launches += span.launches_per_enqueue()
        # the 48 upscaled frames owned by the chunk, at slots 5 i
        for i in range(chunk):
            pack(up[i:i + 1], pix[k][(1 + len(CHAIN_TIMES)) * i])
        launches += chunk
        for p0 in range(0, chunk, B):
            n = min(B, chunk - p0)
            for j, t in enumerate(CHAIN_TIMES):
                rc = L.kb2_set_timestep(rife.h, kb.ctypes.c_float(t))
                if rc != kb.KB2_OK:
                    raise kb.KB2Error(rc, "kb2_set_timestep")
                rife.enqueue_raw((kb.Tensor * 2)(T(up[p0:p0 + n]), T(up[p0 + 1:p0 + 1 + n])),
                                 (kb.Tensor * 1)(T(mid[:n])), sh)
                launches += rife.launches_per_enqueue()
                for q in range(n):
                    pack(mid[q:q + 1], pix[k][(1 + len(CHAIN_TIMES)) * (p0 + q) + 1 + j])
                launches += n
        return launches

    with torch.cuda.stream(stream):
        src.copy_(src_host, non_blocking=True)
    for w in range(args.warmup):
        compute(w % 2)
    stream.synchronize()
    span.check_device(stream)
    rife.check_device(stream)

    # compute only: sources resident, no gather
    clocks = ClockSampler(D.local_rank)
    clocks.start()
    D.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    launches = 0
    for i in range(len(my)):
        launches += compute(i % 2)
    e1.record(stream)
    e1.synchronize()
    D.barrier()
    clk = clocks.stop()
    ms = D.max(e0.elapsed_time(e1))
    outputs = out_per_chunk * len(my)
    value = shard.whole_job_rate(outputs, D.world, ms / 1e3)

    # end to end: upload each chunk's 49 sources, compute, gather its 240 output frames in order
    e2e = None
    if not args.no_e2e:
        ev_done = [torch.cuda.Event() for _ in range(2)]
        ev_free = [torch.cuda.Event() for _ in range(2)]
        order = []

        def pipeline(chunks):
            for i, c in enumerate(chunks):
                k = i % 2
                with torch.cuda.stream(stream):
                    if i >= 2:
                        stream.wait_event(ev_free[k])
                    src.copy_(src_host, non_blocking=True)
                    compute(k)
                    ev_done[k].record(stream)
                with torch.cuda.stream(s_copy):
                    s_copy.wait_event(ev_done[k])
                    host_ring.copy_(pix[k], non_blocking=True)  # chunk c's frames, in output order
                    ev_free[k].record(s_copy)
                order.append(c.index)
            torch.cuda.synchronize()

        pipeline(my[:min(2, args.warmup)])
        order.clear()
        D.barrier()
        t0 = time.perf_counter()
        pipeline(my)
        D.barrier()
        e2e_s = D.max(time.perf_counter() - t0)
        assert order == [c.index for c in my] and all(b > a for a, b in zip(order, order[1:]))
        e2e = {"value": shard.whole_job_rate(outputs, D.world, e2e_s), "unit": "frames/s",
               "h2d_bytes_per_step": int(src_host.numel() * 2), "d2h_bytes_per_step": int(pix[0].numel() * 4),
               "d2h_gbs": pix[0].numel() * 4 * len(my) / e2e_s / 1e9,
               "path": "per chunk: H2D of its 49 1080p FP16 sources, the chain, D2H of its 240 RGB10A2 4K frames "
                       "into the chunk's slot of a pinned host ring in output order; gather overlapped with the next "
                       "chunk on a second stream"}
    span.close()
    rife.close()
    if D.rank == 0:
        per_gpu = value / D.world
        print(json.dumps({
            "metric": "full chain SPAN x2 FP8 1080p->2160p + RIFE 4K x4 instants, output 4K frames/s",
            "value": value, "unit": "frames/s", "n_gpus": D.world, "steps": len(my), "warmup": args.warmup,
            "ms_per_step": ms / len(my), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3+f16", "data": "synthetic (13 seeded anime-like frames cycled, seeded weights)",
            "config": {"workload": "configs[4]: SPAN x2 FP8 on a 1080p stream, then IFNet FP16 at 3840x2160 at "
                                   "t = 0.2/0.4/0.6/0.8 per pair; 48-frame chunks round-robin over ranks; ordered "
                                   "RGB10A2 gather",
                       "chunk_frames": chunk, "output_frames_per_chunk": out_per_chunk,
                       "source_frames_per_s": value / (1 + len(CHAIN_TIMES)),
                       "parallelism": f"chunk-sharded x{D.world}, no collective", "per_gpu_output_frames_per_s": per_gpu,
                       "l2": "working set > L2: 49 x 49.8 MB upscaled frames a chunk"},
            "e2e": e2e, "gpu_launches": launches, "clocks": clk}))
    D.close()


# ------------------------------------------------------------------------------------------------
# frames at any instant from one mid-pair motion (kb2_warp_blend_at)
# ------------------------------------------------------------------------------------------------
WARP_T = 1.0 / 3.0
WARP_CROP = (96, 160)  # reference arm: frame crops (h, w), their motion window the same size


def warp_inputs(B, H, W, seed):
    """Frames a, b [B,3,H,W] FP16 values, and a RIFE-shaped motion: 4 flow planes + mask on the
    padded plane (multiples of 32) with the frame's window at the rife_window offset; smooth flow
    of a few pixels plus noise."""
    import numpy as np
    from synth import anime_frames
    Hp, Wp = -(-H // 32) * 32, -(-W // 32) * 32
    top, left = ((Hp - H) // 2) & ~1, ((Wp - W) // 2) & ~1
    a = anime_frames(B, H, W, seed=seed).astype(np.float16)
    b = np.roll(a, 3, axis=3)
    rng = np.random.default_rng(seed)
    yy, xx = np.meshgrid(np.linspace(0, 6.28, Hp, dtype=np.float32), np.linspace(0, 6.28, Wp, dtype=np.float32),
                         indexing="ij")
    base = np.stack([np.sin(xx) * 3, np.cos(yy) * 2, -np.sin(xx) * 3, -np.cos(yy) * 2]).astype(np.float32)
    flow = np.ascontiguousarray(np.broadcast_to(base, (B, 4, Hp, Wp)) +
                                rng.standard_normal((B, 4, Hp, Wp), dtype=np.float32) * 0.25, np.float32)
    mask = np.ascontiguousarray(0.5 + 0.4 * np.sin(xx + yy)[None].repeat(B, 0), np.float32)
    return a, b, flow, mask, (left, top, W, H)


def run_warp(args):
    import numpy as np
    import torch

    import kirari_b200 as kb
    import shard

    D = Dist()
    B, H, W = args.batch, args.height, args.width
    a, b, flow, mask, win = warp_inputs(B, H, W, shard.frame_seed(10, D.rank, 0))
    host = [torch.from_numpy(x) for x in (a, b, flow, mask)]
    dev = [x.cuda() for x in host]
    stream = torch.cuda.Stream()
    out = torch.empty_like(dev[0])
    m = kb._motion(dev[2], dev[3], win)
    ta, tb, to = kb.to_kb2_tensor(dev[0]), kb.to_kb2_tensor(dev[1]), kb.to_kb2_tensor(out)
    sh = kb.ctypes.c_void_p(stream.cuda_stream)

    def step(xa, xb, xo, mm):
        rc = kb.lib().kb2_warp_blend_at(sh, kb.ctypes.byref(xa), kb.ctypes.byref(xb), kb.ctypes.byref(mm),
                                        WARP_T, kb.ctypes.byref(xo))
        if rc != kb.KB2_OK:
            raise kb.KB2Error(rc, "kb2_warp_blend_at")

    for _ in range(args.warmup):
        step(ta, tb, to, m)
    stream.synchronize()
    clocks = ClockSampler(D.local_rank)
    clocks.start()
    D.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for e0, e1 in ev:
        e0.record(stream)
        step(ta, tb, to, m)
        e1.record(stream)
    stop.record(stream)
    stop.synchronize()
    D.barrier()
    clk = clocks.stop()
    ms = D.max(start.elapsed_time(stop))
    avg = float(np.mean([e0.elapsed_time(e1) for e0, e1 in ev]))
    value = shard.whole_job_rate(B * args.steps, D.world, ms / 1e3)
    # algorithmic bytes per launch: both frames and the output once (FP16), the 4 flow planes and the
    # mask once over the window (FP32)
    px = B * H * W
    algo = px * (2 * 3 * 2 + 3 * 2 + 5 * 4)
    peaks_json, peak_kind = measured_peaks()
    achieved = algo / (avg / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": float(peaks_json["hbm_gbs"]), "unit": "GB/s",
                "frac": achieved / float(peaks_json["hbm_gbs"]), "traffic": None, "kernel": "warp_blend_at_kernel",
                "launches": args.steps, "avg_launch_ms": avg, "algorithmic_bytes_per_launch": algo,
                "peak_source": f"{peak_kind} hbm_gbs"}
    e2e = None
    if not args.no_e2e:
        pinned = [x.pin_memory() for x in host]
        h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        d = [torch.empty_like(x) for x in dev]
        md = kb._motion(d[2], d[3], win)
        da, db = kb.to_kb2_tensor(d[0]), kb.to_kb2_tensor(d[1])
        D.barrier()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                for dst, src in zip(d, pinned):
                    dst.copy_(src, non_blocking=True)
                step(da, db, to, md)
                h_out.copy_(out, non_blocking=True)
        stream.synchronize()
        D.barrier()
        e2e_s = D.max(time.perf_counter() - t0)
        e2e = {"value": shard.whole_job_rate(B * args.steps, D.world, e2e_s), "unit": "frames/s",
               "h2d_bytes_per_step": int(sum(x.numel() * x.element_size() for x in host)),
               "d2h_bytes_per_step": int(h_out.numel() * 2),
               "path": "kb2_warp_blend_at with pinned host frames and motion: H2D of both frames, the flow and "
                       "the mask, the call, D2H of the frames, serial on one stream"}
    cpu = None
    if D.rank == 0 and D.world == 1 and not args.no_cpu_baseline:
        cpu = warp_reference_sample(a, b, flow, mask, win, budget_s=10.0, full=(H, W))
    if D.rank == 0:
        print(json.dumps({"metric": f"frames synthesised at t=1/3 from a mid-pair motion, {W}x{H}, frames/s",
                          "value": value, "unit": "frames/s", "n_gpus": D.world, "steps": args.steps,
                          "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f16 frames, f32 motion",
                          "data": "synthetic (seeded frames, smooth flow + noise)",
                          "config": {"workload": f"kb2_warp_blend_at, {B} pairs of {W}x{H}, motion planes "
                                                 f"{flow.shape[3]}x{flow.shape[2]}, t=1/3",
                                     "global_batch": B * D.world, "parallelism": f"pair-sharded x{D.world}, no collective",
                                     "l2": "working set > L2: 8 x 12 MB frames x 2 + 8 x 42 MB motion"},
                          "roofline": roofline, "e2e": e2e, "gpu_launches": args.steps, "clocks": clk,
                          "cpu_baseline": cpu}))
    D.close()


def warp_reference_sample(a, b, flow, mask, win, budget_s, full, threads=None):
    """The reference's CPU warp_blend_at (oracle/_ref) on 96x160 crops of the pairs (crop motion =
    the window's same rectangle), one crop per host thread, repeated to about `budget_s` seconds;
    frames/s scaled by pixels to full frames."""
    import numpy as np
    from oracle import ref_lib
    if not ref_lib.available():
        return None
    cores = threads or host_cores()
    ch, cw = WARP_CROP
    H, W = full
    left, top = win[0], win[1]
    rng = np.random.default_rng(0)

    def one(k):
        y = int(rng.integers(0, H - ch))
        x = int(rng.integers(0, W - cw))
        i = k % a.shape[0]
        return (a[i, :, y:y + ch, x:x + cw].astype(np.float32), b[i, :, y:y + ch, x:x + cw].astype(np.float32),
                flow[i][:, top + y:top + y + ch, left + x:left + x + cw], mask[i][top + y:top + y + ch, left + x:left + x + cw])

    def run(reps):
        jobs = [[one(t * reps + r) for r in range(reps)] for t in range(cores)]
        done = [0] * cores

        def work(t):
            for ca, cb, cf, cm in jobs[t]:
                ref_lib.warp_blend_at(ca, cb, cf, cm, (0, 0, cw, ch), WARP_T)
                done[t] += 1

        ts = [threading.Thread(target=work, args=(t,)) for t in range(cores)]
        t0 = time.perf_counter()
        for th in ts:
            th.start()
        for th in ts:
            th.join()
        return sum(done) * ch * cw / float(H * W), time.perf_counter() - t0

    frames, dt = run(1)
    reps = max(1, int(budget_s / max(dt, 1e-3)))
    if reps > 1:
        frames, dt = run(reps)
    return {"value": frames / dt, "unit": "frames/s", "cores": cores, "kind": "reference", "cpu": cpu_model(),
            "sample": f"{cores} threads x {reps} crops of {ch}x{cw} px (and their motion), the reference's CPU "
                      f"warp_blend_at (oracle/_ref), scaled by pixels to {W}x{H} frames"}


def run_warp_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    from oracle import ref_lib
    if not ref_lib.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (reference sources absent)"}))
        return
    B, H, W = args.batch, args.height, args.width
    a, b, flow, mask, win = warp_inputs(min(B, 2), H, W, 10)
    cores = host_cores()
    for _ in range(args.warmup):
        warp_reference_sample(a, b, flow, mask, win, 0.0, (H, W), threads=cores)
    vals = []
    total_s = 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        r = warp_reference_sample(a, b, flow, mask, win, 0.0, (H, W), threads=cores)
        total_s += time.perf_counter() - t0
        vals.append(r["value"])
    value = float(statistics.mean(vals))
    print(json.dumps({"metric": f"frames synthesised at t=1/3 from a mid-pair motion, {W}x{H}, frames/s",
                      "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": 1e3 * total_s / args.steps, "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                      "impl": "reference",
                      "config": {"workload": f"warp_blend_at, {W}x{H}, t=1/3, reference CPU path"},
                      "cpu_baseline": {"value": value, "unit": "frames/s", "cores": cores, "kind": "reference",
                                       "cpu": cpu_model(),
                                       "sample": f"per step: {cores} threads x 1 crop of {WARP_CROP[0]}x{WARP_CROP[1]} "
                                                 f"px, scaled by pixels to {W}x{H} frames"},
                      "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


# ------------------------------------------------------------------------------------------------
# one small pass of every kernel kind, for the per-kernel ncu summaries under profiles/
# ------------------------------------------------------------------------------------------------
KERNEL_FAMILIES = ("span16", "span8", "rife", "rife425", "warp", "janai", "janai8")


def run_kernels(args):
    """Each family runs once, batch `--batch` (1 by default here) at 1920x1080, so that every
    tensor of the SPAN and IFNet paths is larger than L2 while the process holds a few GB: span16
    (the FP16 engine, F16 frames then display pixels), span8 (the E4M3 engine, after one FP16
    calibration pass), rife (IFNet image and motion variants), rife425 (RIFE 4.25 image and motion
    variants), warp (kb2_warp_blend_at bilinear,
    Catmull-Rom and pan-locked, kb2_warp_blend_poses, kb2_flow_max, kb2_pack_display), janai /
    janai8 (the unshuffle SPAN b8f64). Prints one JSON line with each family's kernel launches and
    device time; not a benchmark line."""
    import numpy as np
    import torch
    import kirari_b200 as kb
    import seeded
    from synth import anime_frames, shifted_pair

    D = Dist()
    B, H, W = args.batch, args.height, args.width
    fams = KERNEL_FAMILIES if args.family == "all" else (args.family,)
    stream = torch.cuda.Stream()
    sh = kb.ctypes.c_void_p(stream.cuda_stream)
    report = {}

    def timed(name, fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            launches = fn()
            e1.record(stream)
        e1.synchronize()
        report[name] = {"launches": launches, "ms": e0.elapsed_time(e1)}

    x = torch.from_numpy(anime_frames(B, H, W, seed=7).astype(np.float16)).cuda()
    for fam in fams:
        if fam in ("span16", "span8"):
            blob = kb.make_blob(kb.MODEL_SPAN_X2, seeded.span_flat(seeded.span_init(1)))
            scales = None
            if fam == "span8":
                e16 = kb.Engine(kb.MODEL_SPAN_X2, blob, H, W, max_batch=B)
                scales = seeded.scales_from_peaks(e16.calibrate(x, stream), floor=2.0 ** -14)
                e16.close()
            eng = kb.Engine(kb.MODEL_SPAN_X2, blob, H, W, max_batch=B, act_scales=scales,
                            precision=kb.PREC_FP8 if fam == "span8" else kb.PREC_FP16)
            out = torch.empty((B, 3, 2 * H, 2 * W), dtype=torch.float16, device="cuda")
            timed(fam, lambda: (eng.enqueue([x], [out], stream), eng.launches_per_enqueue())[1])
            if fam == "span16":
                pix = torch.empty((B, 4, 2 * H, 2 * W), dtype=torch.uint8, device="cuda")
                eng.set_output_format(kb.DISPLAY_RGB10A2)
                timed("span16.display", lambda: (eng.enqueue([x], [pix], stream), eng.launches_per_enqueue())[1])
                del pix
            eng.check_device(stream)
            eng.close()
            del out
        elif fam == "rife":
            fa, fb = shifted_pair(H, W, seed=3)
            a = torch.from_numpy(np.ascontiguousarray(np.repeat(fa[None], B, 0), np.float16)).cuda()
            b = torch.from_numpy(np.ascontiguousarray(np.repeat(fb[None], B, 0), np.float16)).cuda()
            eng = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, seeded.ifnet_flat(seeded.ifnet_init(2))), H, W,
                            max_batch=B)
            out = torch.empty((B, 3, H, W), dtype=torch.float16, device="cuda")
            timed("rife", lambda: (eng.enqueue([a, b], [out], stream), eng.launches_per_enqueue())[1])
            timed("rife.motion", lambda: (eng.motion(a, b, stream=stream), eng.launches_per_enqueue())[1])
            eng.check_device(stream)
            eng.close()
        elif fam == "rife425":
            fa, fb = shifted_pair(H, W, seed=3)
            a = torch.from_numpy(np.ascontiguousarray(np.repeat(fa[None], B, 0), np.float16)).cuda()
            b = torch.from_numpy(np.ascontiguousarray(np.repeat(fb[None], B, 0), np.float16)).cuda()
            eng = kb.Engine(kb.MODEL_RIFE_FUSED, kb.make_blob(kb.MODEL_RIFE_FUSED, rife42_flat()), H, W, max_batch=B)
            out = torch.empty((B, 3, H, W), dtype=torch.float16, device="cuda")
            timed("rife425", lambda: (eng.enqueue([a, b], [out], stream), eng.launches_per_enqueue())[1])
            timed("rife425.motion", lambda: (eng.motion(a, b, stream=stream), eng.launches_per_enqueue())[1])
            eng.check_device(stream)
            eng.close()
        elif fam == "warp":
            a, b, flow, mask, win = warp_inputs(B, H, W, 11)
            ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
            tf, tm = torch.from_numpy(flow).cuda(), torch.from_numpy(mask).cuda()
            timed("warp.bilinear", lambda: (kb.warp_blend_at(ta, tb, tf, tm, win, WARP_T, stream=stream), 1)[1])
            timed("warp.catmull_rom", lambda: (kb.warp_blend_at(ta, tb, tf, tm, win, WARP_T, stream=stream, warp=1), 1)[1])
            timed("warp.pan_lock", lambda: (kb.warp_blend_at(ta, tb, tf, tm, win, WARP_T, stream=stream, pan_lock=1), 2)[1])
            timed("warp.poses", lambda: (kb.warp_blend_poses(ta, tb, tf, tm, tf, tm, win, WARP_T, stream=stream), 1)[1])
            timed("flow_max", lambda: (kb.flow_max(tf, tm, win, stream=stream), 1)[1])
            frames = torch.empty((B, 3, 2 * H, 2 * W), dtype=torch.float16, device="cuda").uniform_()
            timed("pack_display", lambda: (kb.pack_display(frames, kb.DISPLAY_RGB10A2_DITHER, stream=stream), 1)[1])
        elif fam in ("janai", "janai8"):
            q = fam == "janai8"
            eng = kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, janai_package(q, H, W), H, W, max_batch=B,
                            precision=kb.PREC_FP8 if q else kb.PREC_FP16)
            out = torch.empty((B, 3, 2 * H, 2 * W), dtype=torch.float16, device="cuda")
            timed(fam, lambda: (eng.enqueue([x], [out], stream), eng.launches_per_enqueue())[1])
            eng.check_device(stream)
            eng.close()
        torch.cuda.empty_cache()
    if D.rank == 0:
        print(json.dumps({"kernels": report, "batch": B, "frame": f"{W}x{H}",
                          "note": "one pass of each kernel kind (profiling aid), not a benchmark line"}))
    D.close()


def run_tiles(args):
    """SPAN x2 FP16 on 8 x 1080p through the engine's partial modes, each timed like the default line:
    whole frames; moving tiles (kb2_next_span_tiles) with `--dirty-rows` tile rows across the frame
    recomputed and the rest kept from the previous output, as in playback where most tiles repeat;
    and configs[2]'s stated processing, 8 row tiles with an 8-row halo (kb2_set_row_tiles). One JSON
    line; `value` is the moving-tiles rate (output frames a second), `modes` has all three."""
    import numpy as np
    import torch

    import kirari_b200 as kb
    import seeded
    import shard
    from synth import anime_frames

    D = Dist()
    B, H, W = args.batch, args.height, args.width
    blob = kb.make_blob(kb.MODEL_SPAN_X2, seeded.span_flat(seeded.span_init(1)))
    eng = kb.Engine(kb.MODEL_SPAN_X2, blob, H, W, max_batch=B, device=D.local_rank)
    stream = torch.cuda.Stream()
    x = torch.from_numpy(anime_frames(B, H, W, seed=shard.frame_seed(10, D.rank, 0)).astype(np.float16)).cuda()
    out = torch.empty((B, 3, 2 * H, 2 * W), dtype=torch.float16, device="cuda")
    grid = eng.span_tile_grid()
    core = np.zeros((grid["rows"], grid["cols"]), np.uint8)
    r0 = max(0, grid["rows"] // 2 - args.dirty_rows // 2)
    core[r0:r0 + args.dirty_rows, :] = 1

    def timed(prepare):
        for _ in range(args.warmup):
            prepare()
            eng.enqueue([x], [out], stream)
        stream.synchronize()
        clocks = ClockSampler(D.local_rank)
        clocks.start()
        D.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            prepare()
            eng.enqueue([x], [out], stream)
        stop.record(stream)
        stop.synchronize()
        D.barrier()
        clk = clocks.stop()
        ms = D.max(start.elapsed_time(stop))
        eng.check_device(stream)
        return {"value": shard.whole_job_rate(B * args.steps, D.world, ms / 1e3), "unit": "frames/s",
                "ms_per_step": ms / args.steps, "clocks": clk}

    whole = timed(lambda: None)
    tiles = timed(lambda: eng.next_span_tiles(core))
    eng.set_row_tiles(8, 8)
    rows = timed(lambda: None)
    eng.set_row_tiles(1, 0)
    launches = args.steps * eng.launches_per_enqueue()
    eng.close()
    frac = float(core.sum()) / core.size
    if D.rank == 0:
        print(json.dumps({
            "metric": "SPAN x2 1080p->2160p frames/s with moving tiles", "value": tiles["value"], "unit": "frames/s",
            "n_gpus": D.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": tiles["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded anime-like frames, seeded weights)",
            "config": {"workload": f"SPAN x2 FP16, {B} x {H}x{W}; moving tiles: {args.dirty_rows} of {grid['rows']} tile "
                                   f"rows ({grid['tile_h']} px) recomputed a step ({100 * frac:.0f} % of the tiles)",
                       "global_batch": B, "tile_grid": grid, "parallelism": "frame-sharded, no collective"},
            "modes": {"whole_frames": whole, "moving_tiles": tiles, "row_tiles_8_halo_8": rows},
            "gpu_launches": launches, "clocks": tiles["clocks"], "e2e": None}))
    D.close()


def run_hostcopy(args):
    """The e2e leg of configs[1] without the engine: per step, on every rank, the H2D copy of B
    1080p F16 NCHW frames from pinned memory and the D2H read of B 3840x2160 RGB10A2 frames into
    pinned memory, on two streams, double-buffered as e2e_leg does; then the D2H reads alone. Wall
    clock between barriers, max over ranks. `value` is the frames/s at which the host side alone
    would carry that leg at this many ranks; an e2e rate near it is bound by host copies, not by
    the GPUs. Not a benchmark of the frame path."""
    import torch
    import shard
    D = Dist()
    B, H, W = args.batch, FRAME_H, FRAME_W
    h_in = torch.empty((B, 3, H, W), dtype=torch.float16).pin_memory()
    d_in = [torch.empty((B, 3, H, W), dtype=torch.float16, device="cuda") for _ in range(2)]
    d_out = [torch.zeros((B, 4, 2 * H, 2 * W), dtype=torch.uint8, device="cuda") for _ in range(2)]
    h_out = [torch.empty((B, 4, 2 * H, 2 * W), dtype=torch.uint8).pin_memory() for _ in range(2)]
    s_h2d, s_d2h = torch.cuda.Stream(), torch.cuda.Stream()
    in_b = h_in.numel() * 2
    out_b = h_out[0].numel()

    def run(n, with_h2d):
        for i in range(n):
            k = i % 2
            if with_h2d:
                with torch.cuda.stream(s_h2d):
                    d_in[k].copy_(h_in, non_blocking=True)
            with torch.cuda.stream(s_d2h):
                h_out[k].copy_(d_out[k], non_blocking=True)
        torch.cuda.synchronize()

    def timed(with_h2d):
        run(max(args.warmup, 3), with_h2d)
        D.barrier()
        t0 = time.perf_counter()
        run(args.steps, with_h2d)
        D.barrier()
        return D.max(time.perf_counter() - t0)

    both = timed(True)
    d2h = timed(False)
    n = D.world
    line = {"metric": "host-copy ceiling of the configs[1] e2e leg (SPAN x2, 1080p in, 4K RGB10A2 out)",
            "value": shard.whole_job_rate(B * args.steps, n, both), "unit": "frames/s", "n_gpus": n,
            "steps": args.steps, "warmup": max(args.warmup, 3), "higher_is_better": True, "scaling": "weak",
            "h2d_bytes_per_step": in_b, "d2h_bytes_per_step": out_b,
            "both_gbs_total": n * (in_b + out_b) * args.steps / both / 1e9,
            "d2h_only_gbs_total": n * out_b * args.steps / d2h / 1e9,
            "d2h_only_frames_per_s": shard.whole_job_rate(B * args.steps, n, d2h),
            "note": "copies only (no compute): pinned H2D of the step's F16 frames and D2H of its display "
                    "pixels on two streams per rank, the e2e leg's buffers and order; not a benchmark line"}
    if D.rank == 0:
        print(json.dumps(line))
    D.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "warp":
        run_warp(args)
    elif args.workload == "chain":
        run_chain(args)
    elif args.workload == "kernels":
        run_kernels(args)
    elif args.workload == "tiles":
        run_tiles(args)
    elif args.workload == "hostcopy":
        run_hostcopy(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
