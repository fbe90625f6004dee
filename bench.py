"""Benchmark of the frame path: SPAN x2 1080p -> 2160p on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload span16|span8|rife|janai|janai8|warp] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1: frames shard across GPUs, no collective)

A step is one batch of 8 synthetic 1080p frames through the engine (the contract's configs[1]:
FP16, batch 8, 240 frames per GPU by default = 30 steps); `--workload span8` is configs[2] (FP8
E4M3), `--workload rife` is configs[3] (IFNet FP16, 8 frame pairs per step at t = 0.5;
`--height 2160 --width 3840` for the 4K interpolation rate), `--workload janai` the AnimeJaNai
unshuffle SPAN b8f64 (8 blocks x 64 channels at half resolution, FP16) read from a seeded .span8
package (the first of the contract's "next" rows), `--workload janai8` the same model from an FP8
package (E4M3 blocks, activation scales calibrated on crops of the frames), `--workload warp` the
frames synthesised at t = 1/3 from one mid-pair motion (`kb2_warp_blend_at`, 8 pairs of 1080p with
a RIFE-shaped motion of 1920x1088 planes). `value` is whole-job frames/s with the
inputs resident in HBM; `e2e` is the same through the public C ABI with pinned host frames, the
host->device copy and the device->host read of every output inside the timed region. `roofline`
times the dominant kernel with CUDA events on its launching stream during the timed steps.
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["span16", "span8", "rife", "janai", "janai8", "warp"], default="span16")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--height", type=int, default=FRAME_H)
    ap.add_argument("--width", type=int, default=FRAME_W)
    ap.add_argument("--timestep", type=float, default=0.5)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


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


# ------------------------------------------------------------------------------------------------
# reference CPU implementation (the oracle/_ref build of the reference's own interpreter)
# ------------------------------------------------------------------------------------------------
CROP_H, CROP_W = 24, 48


RIFE_CROP_H, RIFE_CROP_W = 64, 96  # IFNet needs multiples of 32


def reference_sample(threads, frame, flat, crops_per_thread=1, frame_b=None, timestep=0.5, full=None):
    """Each host thread runs the reference's FP32 network on its own crop of the frame (the
    interpreter is single-threaded per call); returns (frames processed, seconds). SPAN when
    frame_b is None, else IFNet on the crop pair; `flat` given as bytes is a .span8 package, run by
    the reference's unshuffle-SPAN forward (src/gpu/span_fp8/forward.cpp:144)."""
    from oracle import ref_lib
    import numpy as np

    rife = frame_b is not None
    ch, cw = (RIFE_CROP_H, RIFE_CROP_W) if rife else (CROP_H, CROP_W)
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
                if rife:
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


def janai_package(fp8, H, W):
    """The seeded b8f64 .span8 package of the janai workloads; FP8: activation scales calibrated by
    the CPU restatement on four 64x128 crops of seeded frames (the reference derives them offline,
    derive.h:42-62)."""
    import numpy as np
    from oracle import nets
    from synth import anime_frames
    p = nets.span8_init(8, 64, seed=3)
    if fp8:
        crops = anime_frames(4, min(H, 64), min(W, 128), seed=900).astype(np.float16).astype(np.float32)
        p = nets.span8_fp8_package(p, crops)
    return nets.span8_package(p)


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(frame, flat, budget_s=12.0, frame_b=None, timestep=0.5, full=None):
    from oracle import ref_lib
    if not ref_lib.available():
        return None
    cores = host_cores()
    kw = dict(frame_b=frame_b, timestep=timestep, full=full)
    frames, dt = reference_sample(cores, frame, flat, **kw)
    reps = max(1, int(budget_s / max(dt, 1e-3)))
    if reps > 1:
        frames, dt = reference_sample(cores, frame, flat, crops_per_thread=reps, **kw)
    ch, cw = (RIFE_CROP_H, RIFE_CROP_W) if frame_b is not None else (CROP_H, CROP_W)
    fh, fw = full if full is not None else (FRAME_H, FRAME_W)
    net = "IFNet pairs" if frame_b is not None else ("unshuffle SPAN b8f64" if isinstance(flat, bytes) else "SPAN")
    return {"value": frames / dt, "unit": "frames/s", "cores": cores, "kind": "reference",
            "sample": f"{cores} threads x {reps} {net} crops of {ch}x{cw} px of synthetic {fw}x{fh} frames, "
                      f"reference FP32 IR interpreter (oracle/_ref), scaled by pixels to {fw}x{fh} frames"}


def workload_desc(args, world=1):
    """metric, unit, dtype, config of the workload (shared by both arms)."""
    B, H, W = args.batch, args.height, args.width
    if args.workload == "rife":
        metric = f"RIFE IFNet {W}x{H} interpolated frames/s"
        config = {"workload": f"configs[3] IFNet FP16, {B} frame pairs per step, {W}x{H}, t={args.timestep}",
                  "global_batch": B * world, "frames_per_gpu": B * args.steps,
                  "parallelism": f"pair-sharded x{world}, no collective",
                  "l2": "working set > L2: block 3 reads and writes 8 x 67 MB inputs and 8 x 33 MB activations"}
        return metric, "f16", config
    if args.workload in ("janai", "janai8"):
        q = args.workload == "janai8"
        metric = ("SPAN b8f64 unshuffle x2 1080p->2160p frames/s" if (H, W) == (FRAME_H, FRAME_W)
                  else f"SPAN b8f64 unshuffle x2 {W}x{H} frames/s")
        config = {"workload": f"AnimeJaNai unshuffle SPAN b8f64 {'E4M3 blocks' if q else 'FP16'} "
                              f"(.span8 package, seeded), batch {B}, {H}x{W} -> {2 * H}x{2 * W}",
                  "global_batch": B * world, "frames_per_gpu": B * args.steps,
                  "parallelism": f"frame-sharded x{world}, no collective",
                  "l2": "working set > L2: each layer reads and writes 8 x 66 MB activations (half resolution)"}
        return metric, ("e4m3+f16" if q else "f16"), config
    fp8 = args.workload == "span8"
    metric = "SPAN x2 1080p->2160p frames/s" if (H, W) == (FRAME_H, FRAME_W) else f"SPAN x2 {W}x{H} frames/s"
    config = {"workload": ("configs[2] SPAN x2 FP8 E4M3" if fp8 else "configs[1] SPAN x2 FP16")
                          + f", batch {B}, {H}x{W} -> {2 * H}x{2 * W}",
              "global_batch": B * world, "frames_per_gpu": B * args.steps,
              "parallelism": f"frame-sharded x{world}, no collective",
              "l2": "working set > L2: each layer reads and writes 8 x 199 MB activations"}
    return metric, ("e4m3+f16" if fp8 else "f16"), config


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    import numpy as np
    from oracle import nets, ref_lib
    from synth import anime_frame, shifted_pair

    metric, _, config = workload_desc(args, world)
    config = dict(config, workload=config["workload"] + ", reference FP32 CPU path")
    if not ref_lib.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (reference sources absent)"}))
        return
    rife = args.workload == "rife"
    if rife:
        fa, fb = shifted_pair(args.height, args.width, 0)
        frame, frame_b = np.ascontiguousarray(fa, np.float32), np.ascontiguousarray(fb, np.float32)
        flat = nets.ifnet_flat(nets.ifnet_init(2))
    elif args.workload in ("janai", "janai8"):
        frame, frame_b = anime_frame(args.height, args.width, 0).astype(np.float32), None
        flat = janai_package(args.workload == "janai8", args.height, args.width)
    else:
        frame, frame_b = anime_frame(args.height, args.width, 0).astype(np.float32), None
        flat = nets.span_flat(nets.span_init(1))
    kw = dict(frame_b=frame_b, timestep=args.timestep, full=(args.height, args.width))
    cores = host_cores()
    for _ in range(args.warmup):
        reference_sample(cores, frame, flat, **kw)
    total_frames, total_s = 0.0, 0.0
    for _ in range(args.steps):
        f, dt = reference_sample(cores, frame, flat, **kw)
        total_frames += f
        total_s += dt
    value = total_frames / total_s
    ch, cw = (RIFE_CROP_H, RIFE_CROP_W) if rife else (CROP_H, CROP_W)
    line = {"metric": metric, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_s / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference", "config": config,
            "cpu_baseline": {"value": value, "unit": "frames/s", "cores": cores, "kind": "reference",
                             "sample": f"per step: {cores} threads x 1 crop of {ch}x{cw} px, "
                                       f"scaled by pixels to {args.width}x{args.height} frames"},
            "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ------------------------------------------------------------------------------------------------
# this library
# ------------------------------------------------------------------------------------------------
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import kirari_b200 as kb
    from oracle import nets
    from synth import anime_frames, shifted_pair

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))

    import shard

    def barrier():
        shard.barrier("cuda")

    def max_over_ranks(v):
        return shard.max_over_ranks(v, "cuda")

    B, H, W = args.batch, args.height, args.width
    rife = args.workload == "rife"
    fp8 = args.workload == "span8"
    janai = args.workload in ("janai", "janai8")
    metric, dtype, config = workload_desc(args, world)
    if janai:
        q = args.workload == "janai8"
        flat = janai_package(q, H, W)
        frames = anime_frames(B, H, W, seed=shard.frame_seed(10, rank, 0)).astype(np.float16)
        frames_b = None
        eng = kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, flat, H, W, max_batch=B, precision=kb.PREC_FP8 if q else kb.PREC_FP16,
                        device=local_rank)
        host_in = [frames]
        out_shape = (B, 3, 2 * H, 2 * W)
    elif rife:
        p = nets.ifnet_init(2)
        flat = nets.ifnet_flat(p)
        blob = kb.make_blob(kb.MODEL_IFNET, flat)
        pairs = [shifted_pair(H, W, seed=shard.frame_seed(10, rank, i)) for i in range(B)]
        frames = np.ascontiguousarray(np.stack([q[0] for q in pairs]), np.float16)
        frames_b = np.ascontiguousarray(np.stack([q[1] for q in pairs]), np.float16)
        eng = kb.Engine(kb.MODEL_IFNET, blob, H, W, max_batch=B, device=local_rank)
        eng.set_timestep(args.timestep)
        host_in = [frames, frames_b]
        out_shape = (B, 3, H, W)
    else:
        p = nets.span_init(1)
        flat = nets.span_flat(p)
        blob = kb.make_blob(kb.MODEL_SPAN_X2, flat)
        frames = anime_frames(B, H, W, seed=shard.frame_seed(10, rank, 0)).astype(np.float16)
        frames_b = None
        scales = None
        if fp8:
            calib = torch.from_numpy(anime_frames(16, H, W, seed=1000).astype(np.float16)).cuda()
            e16 = kb.Engine(kb.MODEL_SPAN_X2, blob, H, W, max_batch=B, device=local_rank)
            peaks = e16.calibrate(calib)
            e16.close()
            del calib
            scales = nets.span_scales_from_peaks(peaks, floor=2.0 ** -14)
        eng = kb.Engine(kb.MODEL_SPAN_X2, blob, H, W, max_batch=B, precision=kb.PREC_FP8 if fp8 else kb.PREC_FP16,
                        act_scales=scales, device=local_rank)
        host_in = [frames]
        out_shape = (B, 3, 2 * H, 2 * W)
    d_in = [torch.from_numpy(x).cuda() for x in host_in]
    d_out = torch.empty(out_shape, dtype=torch.float16, device="cuda")
    stream = torch.cuda.Stream()
    sh = kb.ctypes.c_void_p(stream.cuda_stream)
    ins = (kb.Tensor * len(d_in))(*[kb.to_kb2_tensor(t) for t in d_in])
    outs = (kb.Tensor * 1)(kb.to_kb2_tensor(d_out))

    # ---- device-resident timing
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            eng.enqueue_raw(ins, outs, sh)
    stream.synchronize()
    eng.check_device(stream)
    eng.read_profile()
    eng.set_profiling(True)
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        eng.enqueue_raw(ins, outs, sh)
    stop.record(stream)
    stop.synchronize()
    barrier()
    clk = clocks.stop()
    eng.set_profiling(False)
    eng.check_device(stream)
    ms = max_over_ranks(start.elapsed_time(stop))
    profile = eng.read_profile()
    value = shard.whole_job_rate(B * args.steps, world, ms / 1e3)

    # ---- roofline of the dominant kernel (measured inside the timed region)
    peaks_json, peak_kind = measured_peaks()
    top_name, top = max(profile.items(), key=lambda kv: kv[1]["total_ms"])
    avg_ms = top["total_ms"] / max(1, top["launches"])
    tflops = top["flops"] / (avg_ms / 1e3) / 1e12
    peak = float(peaks_json["bf16_tflops_sustained"]) * (2.0 if top_name.endswith(".fp8") else 1.0)
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get(top_name, {}).get(f"{B}x{H}x{W}")
    except (OSError, ValueError):
        pass
    total_flops = sum(v["flops"] * v["launches"] for v in profile.values())
    roofline = {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s", "frac": tflops / peak,
                "traffic": traffic, "kernel": top_name, "launches": top["launches"],
                "avg_launch_ms": avg_ms, "flops_per_launch": top["flops"],
                "algorithmic_bytes_per_launch": top["bytes"],
                "peak_source": f"{peak_kind} bf16_tflops_sustained" + (" x2 (E4M3)" if top_name.endswith(".fp8") else ""),
                "network_tflops": (total_flops / (ms / 1e3) / 1e12) if (rife or janai) else
                FLOP_PER_PX * H * W * B * args.steps / (ms / 1e3) / 1e12}
    layers = {k: {"launches": v["launches"], "ms_per_launch": v["total_ms"] / max(1, v["launches"]),
                  "share": v["total_ms"] / max(1e-9, sum(x["total_ms"] for x in profile.values()))}
              for k, v in profile.items()}

    # ---- end to end through the C ABI with host frames (pinned), copies in the timed region
    e2e = None
    if not args.no_e2e:
        if rife:
            # a video stream: pair i is (f_i, f_i+1), so the two input tensors are views one frame
            # apart into a (B + 1)-frame device buffer. Each step uploads its B new frames; the
            # previous step's last frame is copied on the device into slot 0, as a player keeps it.
            h_in = [torch.from_numpy(np.ascontiguousarray(np.concatenate([frames[1:], frames_b[-1:]]))).pin_memory()]
            d_seq = [torch.empty((B + 1,) + tuple(frames.shape[1:]), dtype=torch.float16, device="cuda")
                     for _ in range(2)]
            for t in d_seq:
                t[0].copy_(d_in[0][0])
                t[1:].copy_(h_in[0].cuda())
            d_ins = [[t[1:]] for t in d_seq]  # the H2D target of each step
            pair_views = [[t[:B], t[1:]] for t in d_seq]
        else:
            h_in = [torch.from_numpy(x).pin_memory() for x in host_in]
            d_ins = [[torch.empty_like(t) for t in d_in] for _ in range(2)]
            pair_views = d_ins
        h_out = [torch.empty(out_shape, dtype=torch.float16).pin_memory() for _ in range(2)]
        d_outs = [d_out, torch.empty_like(d_out)]
        s_h2d, s_d2h = torch.cuda.Stream(), torch.cuda.Stream()
        ins2 = [(kb.Tensor * len(d_in))(*[kb.to_kb2_tensor(t) for t in ts]) for ts in pair_views]
        outs2 = [(kb.Tensor * 1)(kb.to_kb2_tensor(t)) for t in d_outs]
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_done = [torch.cuda.Event() for _ in range(2)]
        ev_free = [torch.cuda.Event() for _ in range(2)]

        def pipeline(n_steps):
            for i in range(n_steps):
                k = i % 2
                with torch.cuda.stream(s_h2d):
                    s_h2d.wait_event(ev_free[k]) if i >= 2 else None
                    if rife:  # carry the previous step's last frame (its upload precedes on this stream)
                        d_seq[k][0].copy_(d_seq[1 - k][B], non_blocking=True)
                    for dst, src in zip(d_ins[k], h_in):
                        dst.copy_(src, non_blocking=True)
                    ev_in[k].record(s_h2d)
                stream.wait_event(ev_in[k])
                if i >= 2:
                    stream.wait_event(ev_free[k])
                eng.enqueue_raw(ins2[k], outs2[k], sh)
                ev_done[k].record(stream)
                with torch.cuda.stream(s_d2h):
                    s_d2h.wait_event(ev_done[k])
                    h_out[k].copy_(d_outs[k], non_blocking=True)
                    ev_free[k].record(s_d2h)
            torch.cuda.synchronize()

        pipeline(min(2, args.warmup))
        barrier()
        t0 = time.perf_counter()
        pipeline(args.steps)
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": shard.whole_job_rate(B * args.steps, world, e2e_s), "unit": "frames/s",
               "h2d_bytes_per_step": int(sum(t.numel() * 2 for t in h_in)),
               "d2h_bytes_per_step": int(h_out[0].numel() * 2),
               "path": "kb2_enqueue with pinned host frames: H2D copy, enqueue, D2H of every output frame, "
                       "double-buffered across three streams" +
                       ("; RIFE as a video stream: B new frames uploaded a step, pair i = (f_i, f_i+1) as "
                        "two views of one device buffer, the step's first frame carried on the device"
                        if rife else "")}
        eng.check_device(stream)

    launches = args.steps * eng.launches_per_enqueue()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(frames[0].astype(np.float32), flat,
                           frame_b=frames_b[0].astype(np.float32) if rife else None,
                           timestep=args.timestep, full=(H, W))
    eng.close()
    if rank == 0:
        line = {"metric": metric, "value": value, "unit": "frames/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": dtype, "data": "synthetic (seeded anime-like frames, seeded weights)",
                "config": config, "roofline": roofline, "layers": layers, "e2e": e2e, "gpu_launches": launches,
                "clocks": clk, "cpu_baseline": cpu}
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


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
    import torch.distributed as dist

    import kirari_b200 as kb
    import shard

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    B, H, W = args.batch, args.height, args.width
    a, b, flow, mask, win = warp_inputs(B, H, W, shard.frame_seed(10, rank, 0))
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
    clocks = ClockSampler(local_rank)
    clocks.start()
    shard.barrier("cuda")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for e0, e1 in ev:
        e0.record(stream)
        step(ta, tb, to, m)
        e1.record(stream)
    stop.record(stream)
    stop.synchronize()
    shard.barrier("cuda")
    clk = clocks.stop()
    ms = shard.max_over_ranks(start.elapsed_time(stop), "cuda")
    avg = float(np.mean([e0.elapsed_time(e1) for e0, e1 in ev]))
    value = shard.whole_job_rate(B * args.steps, world, ms / 1e3)
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
        shard.barrier("cuda")
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                for dst, src in zip(d, pinned):
                    dst.copy_(src, non_blocking=True)
                step(da, db, to, md)
                h_out.copy_(out, non_blocking=True)
        stream.synchronize()
        shard.barrier("cuda")
        e2e_s = shard.max_over_ranks(time.perf_counter() - t0, "cuda")
        e2e = {"value": shard.whole_job_rate(B * args.steps, world, e2e_s), "unit": "frames/s",
               "h2d_bytes_per_step": int(sum(x.numel() * x.element_size() for x in host)),
               "d2h_bytes_per_step": int(h_out.numel() * 2),
               "path": "kb2_warp_blend_at with pinned host frames and motion: H2D of both frames, the flow and "
                       "the mask, the call, D2H of the frames, serial on one stream"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = warp_reference_sample(a, b, flow, mask, win, budget_s=10.0, full=(H, W))
    if rank == 0:
        print(json.dumps({"metric": f"frames synthesised at t=1/3 from a mid-pair motion, {W}x{H}, frames/s",
                          "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
                          "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f16 frames, f32 motion",
                          "data": "synthetic (seeded frames, smooth flow + noise)",
                          "config": {"workload": f"kb2_warp_blend_at, {B} pairs of {W}x{H}, motion planes "
                                                 f"{flow.shape[3]}x{flow.shape[2]}, t=1/3",
                                     "global_batch": B * world, "parallelism": f"pair-sharded x{world}, no collective",
                                     "l2": "working set > L2: 8 x 12 MB frames x 2 + 8 x 42 MB motion"},
                          "roofline": roofline, "e2e": e2e, "gpu_launches": args.steps, "clocks": clk,
                          "cpu_baseline": cpu}))
    if world > 1:
        dist.destroy_process_group()


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
    return {"value": frames / dt, "unit": "frames/s", "cores": cores, "kind": "reference",
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
                                       "sample": f"per step: {cores} threads x 1 crop of {WARP_CROP[0]}x{WARP_CROP[1]} "
                                                 f"px, scaled by pixels to {W}x{H} frames"},
                      "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def main():
    args = parse()
    if args.workload == "warp":
        if args.impl == "reference":
            run_warp_reference(args)
        else:
            run_warp(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
