#!/usr/bin/env python
"""Throughput of the segmented separation forward on B200 (HTDemucs; BS-RoFormer with --model).

Metric: audio-seconds separated per second (x realtime), HTDemucs 4-stem
(registry ``htdemucs`` architecture, random init under seed 0), 44.1 kHz
stereo, overlap 0.25, segments batched 32 per forward, fp32. One step is one
pass of ``apply_model`` over one 180 s synthetic track (31 segments). With N
ranks (torchrun) the one track's segments are sharded across the ranks
(contiguous count-balanced runs, at most 32 per forward, so ceil(31 / N) per
rank) and the overlap strips are exchanged with NCCL point-to-point: strong
scaling on the same 180 s of audio. ``--whole-tracks`` instead gives every rank
its own tracks (weak scaling, no data-path collective; with ``--tracks 8
--batch 48 --seconds 240 --precision bf16`` the whole-box sweep's per-rank
share, tails pooled across the rank's tracks).

* ``value``: track resident in HBM before the timed region; K steps timed with
  CUDA events between barriers; max over ranks.
* ``e2e``: the same step through the public API with a pinned host track:
  host->device copy, separation, device->host copy of the stems, per step.
* ``roofline``: the dominant kernel's algorithmic FLOPs per launch over its
  mean launch time (CUDA events around each launch in one extra probed step),
  against the measured peak in MEASURED_PEAKS.json.
* ``cpu_baseline``: the CPU oracle (a restatement of the reference's fp32 CPU
  forward) on a bounded 30 s sample, rank 0 at N=1 only.
* ``split``: (sharded mode) the slowest rank's separation, strip exchange and
  gather times from one extra step with CUDA events around each phase.

The forward is replayed from CUDA graphs (``enable_compiled_core``, the
reference's compiled-core hook) unless ``--no-graphs``; the roofline probe step
runs the same kernels eagerly so each launch can be timed.

``--impl reference`` times that CPU implementation alone on the same 30 s
sample (the reference path runs only on host cores; there is no reference GPU
kernel to run).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import random
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TRACK_SECONDS = 180.0
BATCH = 32
CPU_SAMPLE_SECONDS = 30.0
ROFORMER_TRACK_SECONDS = 300.0
ROFORMER_BATCH = 16
ROFORMER_SEGMENT = 352800  # 8 s at 44.1 kHz
SCNET_BATCH = 8
SIMT_KERNELS = ("unblend_lstm_recurrence", "unblend_conv2d_f32", "unblend_rfft_time", "unblend_irfft_time")
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
METRIC = "audio-sec separated/sec (×realtime), HTDemucs 44.1kHz stereo, 1/2/4/8 B200"


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model", default="htdemucs",
                    choices=["htdemucs", "htdemucs_6s", "bsroformer", "melband", "scnet", "scnet_xl"],
                    help="htdemucs: the headline workload; htdemucs_6s: 6-source HTDemucs (seed 2), bf16, "
                         "shifts=1, 240 s track; bsroformer: BS-RoFormer dim 512 depth 12, 8 s segments, batch 16, "
                         "bf16, 300 s track; scnet / scnet_xl: the registry scnet_small (masked, seed 9) / "
                         "scnet_xl_wide_v5 (seed 10), 11 s segments, batch 8, 180 s track")
    ap.add_argument("--shifts", type=int, default=None, help="random-shift rounds per track")
    ap.add_argument("--stems", default=None,
                    help="comma-separated HTDemucs stems to materialise (default: vocals for htdemucs_6s, "
                         "all stems otherwise)")
    ap.add_argument("--tracks", type=int, default=1,
                    help="tracks per rank and step (e.g. 8 x 240 s bf16 batch 48 per rank for the whole-box sweep)")
    ap.add_argument("--precision", default=None, choices=["fp32", "bf16", "fp32-simt"])
    ap.add_argument("--seconds", type=float, default=None,
                    help="track length per rank (smaller values are for profiling only)")
    ap.add_argument("--batch", type=int, default=None, help="segments per forward")
    ap.add_argument("--whole-tracks", action="store_true",
                    help="N>1: every rank separates its own track(s), no data-path collective (weak scaling); "
                         "default: one track's segments sharded across the ranks with the overlap-strip exchange "
                         "(strong scaling)")
    ap.add_argument("--no-graphs", action="store_true", help="eager launches instead of CUDA-graph replay")
    args = ap.parse_args()
    rof = args.model in ("bsroformer", "melband")
    six = args.model == "htdemucs_6s"
    if args.model.startswith("scnet"):
        if args.precision is None:
            args.precision = "fp32"
        if args.batch is None:
            args.batch = SCNET_BATCH
    if args.precision is None:
        args.precision = "bf16" if rof or six else "fp32"
    if args.shifts is None:
        args.shifts = 1 if six else 0
    if rof and args.precision == "fp32-simt":
        ap.error("fp32-simt is an HTDemucs precision")
    if args.seconds is None:
        args.seconds = ROFORMER_TRACK_SECONDS if rof else (240.0 if six else TRACK_SECONDS)
    if args.batch is None:
        args.batch = ROFORMER_BATCH if rof else BATCH
    return args


def _dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def _peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return {"hbm": d["hbm_gbs"], "bf16": d.get("bf16_tflops_sustained") or d["bf16_tflops"],
                "bf16_burst": d["bf16_tflops"], "src": "measured",
                "kind": "sustained" if d.get("bf16_tflops_sustained") else "burst"}
    return {"hbm": 6650.0, "bf16": 1400.0, "bf16_burst": 1590.0, "src": "fallback", "kind": "sustained"}


def _traffic(key: str, kernel: str):
    """DRAM bytes per launch of `kernel` for workload `key` from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic_per_launch.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 3 and not line.startswith("#") and parts[0] == key and parts[1] == kernel:
            return int(parts[2])
    return None


class Clocks:
    """Samples nvidia-smi clocks / throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = tempfile.mktemp(suffix=".csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sms)}


def cpu_baseline(seconds: float = CPU_SAMPLE_SECONDS) -> dict:
    """The oracle (fp32 CPU restatement of the reference forward) over a bounded sample."""
    import torch

    from oracle.apply_oracle import apply_model as oracle_apply
    from oracle.htdemucs_oracle import htdemucs_forward, segment_length
    from unblend_b200.synth import htdemucs_config, htdemucs_state_dict, synth_track

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    cfg = htdemucs_config("htdemucs")
    sd = htdemucs_state_dict(cfg, 0)
    mix = synth_track(seconds, 1)[None]
    fwd = lambda b: htdemucs_forward(sd, b, cfg)  # noqa: E731
    fwd(mix[..., : segment_length(cfg)])  # warm-up segment
    t0 = time.perf_counter()
    oracle_apply(fwd, mix, 4, segment_length(cfg), cfg["samplerate"], overlap=0.25, chunk_batch_size=BATCH)
    dt = time.perf_counter() - t0
    return {"value": seconds / dt, "unit": "audio-s/s", "cores": cores, "kind": "port",
            "sample": f"oracle apply_model over a {seconds:.0f} s synthetic track (seed 1), fp32, overlap 0.25"}


def cpu_baseline_roformer(seconds: float = 8.0, mel: bool = False) -> dict:
    """The BS-RoFormer (or Mel-Band) oracle, fp32 CPU restatements of the reference forward, over one 8 s segment."""
    import torch

    from oracle.apply_oracle import apply_unshifted
    from oracle.roformer_oracle import bsroformer_forward, melband_forward
    from unblend_b200.synth import (bsroformer_config, bsroformer_state_dict, melband_config, melband_state_dict,
                                    synth_track)

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    if mel:
        cfg = melband_config()
        sd = melband_state_dict(cfg, 6)
        fwd = lambda b: melband_forward(sd, b, cfg, match_length=True)  # noqa: E731
    else:
        cfg = bsroformer_config()
        sd = bsroformer_state_dict(cfg, 3)
        fwd = lambda b: bsroformer_forward(sd, b, cfg)  # noqa: E731
    mix = synth_track(seconds, 1)[None]
    t0 = time.perf_counter()
    apply_unshifted(fwd, mix, 1, ROFORMER_SEGMENT, 0.25, ROFORMER_BATCH)
    dt = time.perf_counter() - t0
    name = "Mel-Band RoFormer" if mel else "BS-RoFormer"
    return {"value": seconds / dt, "unit": "audio-s/s", "cores": cores, "kind": "port",
            "sample": f"{name} oracle over a {seconds:.0f} s synthetic track (one 8 s segment), fp32"}


def cpu_baseline_scnet(xl: bool = False) -> dict:
    """The SCNet oracle (fp32 CPU restatement of the reference forward) over one 11 s segment."""
    import torch

    from oracle.scnet_oracle import scnet_forward
    from unblend_b200.synth import scnet_config, scnet_state_dict, synth_track

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    cfg = scnet_config("scnet_xl_wide_v5" if xl else "scnet_small")
    sd = scnet_state_dict(cfg, 10 if xl else 9)
    seconds = cfg["segment_samples"] / cfg["samplerate"]
    mix = synth_track(seconds, 1)[None]
    t0 = time.perf_counter()
    scnet_forward(sd, mix, cfg)
    dt = time.perf_counter() - t0
    name = "scnet_xl_wide_v5" if xl else "scnet_small"
    return {"value": seconds / dt, "unit": "audio-s/s", "cores": cores, "kind": "port",
            "sample": f"SCNet oracle ({name}) over one {seconds:g} s segment, fp32"}


def run_reference(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    rof = args.model in ("bsroformer", "melband")
    mel = args.model == "melband"
    sc = args.model.startswith("scnet")
    vals = []
    # Each step is one bounded sample, the same one cpu_baseline times in the B200 arm.
    for _ in range(max(1, args.steps)):
        if sc:
            vals.append(cpu_baseline_scnet(xl=args.model == "scnet_xl"))
        else:
            vals.append(cpu_baseline_roformer(mel=mel) if rof else cpu_baseline(CPU_SAMPLE_SECONDS))
    v = statistics.median(x["value"] for x in vals)
    base = dict(vals[0])
    base["value"] = v
    if sc:
        work = f"SCNet ({args.model}) fp32 forward"
    else:
        work = (("Mel-Band RoFormer dim 384 depth 6 fp32 forward" if mel else "BS-RoFormer dim 512 depth 12 fp32 "
                 "forward") if rof else "HTDemucs 4-stem fp32 apply_model")
    work += " on host cores (bounded sample)"
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "dtype": "f32", "data": "synthetic", "vs_baseline": None,
            "config": {"workload": work, "overlap": 0.25},
            "cpu_baseline": base, "e2e": {"value": v, "unit": "audio-s/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    args = _args()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from unblend_b200 import _lib
    from unblend_b200.apply import apply_model
    from unblend_b200.htdemucs import HTDemucsCuda
    from unblend_b200.synth import htdemucs_config, htdemucs_state_dict, synth_track

    world, rank, local = _dist()
    dev = torch.device("cuda", torch.cuda.current_device())
    rof = args.model in ("bsroformer", "melband")
    sc = args.model.startswith("scnet")
    if sc:
        from unblend_b200.scnet import SCNetCuda
        from unblend_b200.synth import scnet_config, scnet_state_dict

        xl = args.model == "scnet_xl"
        scfg = scnet_config("scnet_xl_wide_v5" if xl else "scnet_small")
        model = SCNetCuda(scfg, scnet_state_dict(scfg, 10 if xl else 9), precision=args.precision).to(dev)
        seg_len = scfg["segment_samples"]
    elif args.model == "melband":
        from unblend_b200.roformer import MelBandRoformerCuda
        from unblend_b200.synth import melband_config, melband_state_dict

        rcfg = melband_config()
        model = MelBandRoformerCuda(rcfg, melband_state_dict(rcfg, 6), precision=args.precision).to(dev)
        model.configure_inference(sources=["vocals"], samplerate=44100, segment_samples=ROFORMER_SEGMENT)
        seg_len = ROFORMER_SEGMENT
    elif rof:
        from unblend_b200.roformer import BSRoformerCuda
        from unblend_b200.synth import bsroformer_config, bsroformer_state_dict

        rcfg = bsroformer_config()
        model = BSRoformerCuda(rcfg, bsroformer_state_dict(rcfg, 3), precision=args.precision).to(dev)
        model.configure_inference(sources=["vocals"], samplerate=44100, segment_samples=ROFORMER_SEGMENT)
        seg_len = ROFORMER_SEGMENT
    else:
        name, seed = ("htdemucs_6s", 2) if args.model == "htdemucs_6s" else ("htdemucs", 0)
        cfg = htdemucs_config(name)
        model = HTDemucsCuda(cfg, htdemucs_state_dict(cfg, seed), precision=args.precision).to(dev)
        stems = args.stems or ("vocals" if args.model == "htdemucs_6s" else None)
        if stems:
            model.select_sources(stems.split(","))
        seg_len = model.segment_length
    n_stems = len(model.sources)
    seconds, batch, shifts = args.seconds, args.batch, args.shifts
    split = world > 1 and not args.whole_tracks
    n_tracks = 1 if split else args.tracks
    random.seed(1234 + rank)
    if args.tracks > 1 and not split:
        seeds = [100 + rank * args.tracks + i for i in range(args.tracks)]
    else:
        seeds = [1 if split else 1 + rank]
    tracks = [synth_track(seconds, sd) for sd in seeds]
    track = tracks[0]
    tracks_dev = [t.to(dev) for t in tracks]
    n_seg_track = len(range(0, track.shape[-1], int(0.75 * seg_len)))
    if split:
        # A rank's run of the track is at most ceil(n / N) segments: one forward of that many rows.
        batch = min(batch, -(-n_seg_track // world))
    if not args.no_graphs:
        model.enable_compiled_core()
    if split:
        from unblend_b200.distributed import apply_model_sharded

        step = lambda: apply_model_sharded(model, tracks_dev[0], chunk_batch_size=batch, shifts=shifts,  # noqa: E731
                                           gather=False)
    else:
        from unblend_b200.apply import apply_model_multi

        step = lambda: apply_model_multi(model, tracks_dev, chunk_batch_size=batch, shifts=shifts)  # noqa: E731

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(k):
            fn()
        e.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = s.elapsed_time(e) / k
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    clocks = Clocks(dev.index if world == 1 else local)
    launches0 = _lib.counters["launches"]
    clocks.start()
    ms = timed(step, args.steps)
    clk = clocks.stop()
    launches = _lib.counters["launches"] - launches0

    # End to end through the public API with pinned host tracks.
    hosts = [t.pin_memory() for t in tracks]
    if split:
        def e2e_step():
            # Host track in, full [S, C, L] result back in page-locked host memory on every rank.
            apply_model_sharded(model, hosts[0], device=dev, chunk_batch_size=batch, shifts=shifts, gather=True)
    else:
        def e2e_step():
            apply_model_multi(model, hosts, device=dev, chunk_batch_size=batch, shifts=shifts)
    e2e_step()
    e2e_ms = timed(e2e_step, max(1, args.steps))

    phases = None
    if split:
        # One more step with CUDA events around the separation, strip exchange and gather.
        marks: list = []
        apply_model_sharded(model, tracks_dev[0], chunk_batch_size=batch, shifts=shifts, gather=True,
                            timings=marks)
        torch.cuda.synchronize()
        ev = marks[0]
        ph = torch.tensor([ev["start"].elapsed_time(ev["separated"]), ev["separated"].elapsed_time(ev["exchanged"]),
                           ev["exchanged"].elapsed_time(ev["gathered"])], device=dev)
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
        from unblend_b200.distributed import shard_plan

        plan = shard_plan(track.shape[-1], seg_len, int(0.75 * seg_len), world)
        phases = {"segments_per_rank": [len(p.offsets) for p in plan], "forward_rows": batch,
                  "separate_ms_max": round(float(ph[0]), 3), "strip_exchange_ms_max": round(float(ph[1]), 3),
                  "gather_ms_max": round(float(ph[2]), 3)}

    if not args.no_graphs:
        model.disable_compiled_core()
    # Roofline of the dominant kernel: one probed step with events around each launch.
    _lib.probe = []
    step()
    torch.cuda.synchronize()
    agg: dict = {}
    for name, s, e, work in _lib.probe:
        a = agg.setdefault(name, {"ms": 0.0, "n": 0, "work": 0.0})
        a["ms"] += s.elapsed_time(e)
        a["n"] += 1
        a["work"] += work or 0.0
    _lib.probe = None
    top = max(agg, key=lambda k: agg[k]["ms"])
    peaks = _peaks()
    a = agg[top]
    tflops = a["work"] / (a["ms"] * 1e-3) / 1e12 if a["ms"] > 0 else 0.0
    if top in SIMT_KERNELS:
        # A CUDA-core fp32 kernel: against the nominal FMA rate (148 SMs x 128 FMA x 2 x 1.965 GHz).
        roofline = {"kernel": top, "bound": "fp32-fma", "achieved": round(tflops, 3), "peak": FP32_NOMINAL_TFLOPS,
                    "unit": "TFLOP/s", "frac": round(tflops / FP32_NOMINAL_TFLOPS, 5), "traffic": None,
                    "peak_source": "nominal CUDA-core fp32 FMA rate (no measured figure for it)",
                    "share_of_step": round(a["ms"] / sum(v["ms"] for v in agg.values()), 3),
                    "launches_per_step": a["n"]}
    else:
        roofline = None
    if roofline is None:
        roofline = {"kernel": top, "bound": "tensor", "achieved": round(tflops, 3), "peak": peaks["bf16"],
                    "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16"], 5),
                    "traffic": _traffic(f"{args.model}:{args.precision}:batch{batch}", top),
                    "traffic_unit": "bytes per launch (ncu capture, see profiles/traffic_per_launch.txt)",
                    "peak_source": f"{peaks['src']} bf16 dense ({peaks['kind']}: the kernel is timed inside a "
                                   "seconds-long run)",
                    "frac_of_burst_peak": round(tflops / peaks["bf16_burst"], 5),
                    "share_of_step": round(a["ms"] / sum(v["ms"] for v in agg.values()), 3),
                    "launches_per_step": a["n"]}
    if args.precision == "fp32" and roofline["bound"] == "tensor":
        # fp32 accuracy costs three MMAs per product: kind::f16 at the bf16 rate (bf16 hi / lo
        # operands) or kind::tf32 at half of it (TF32 hi / lo operands).
        bf16x3 = ((top == "unblend_conv2d_tc" and getattr(model, "fp32_split", "") == "bf16x3") or
                  (top == "unblend_attention_tc" and getattr(model, "attention_split", "") == "bf16x3"))
        div = 3 if bf16x3 else 6
        roofline["fp32_split"] = "bf16x3" if bf16x3 else "tf32x3"
        roofline["peak_fp32_3pass"] = round(peaks["bf16"] / div, 1)
        roofline["frac_of_fp32_3pass_peak"] = round(tflops / (peaks["bf16"] / div), 4)

    job_tracks = 1 if split else world * n_tracks
    value = job_tracks * seconds / (ms * 1e-3)
    e2e_value = job_tracks * seconds / (e2e_ms * 1e-3)
    L = track.shape[-1]
    n_seg = len(range(0, L, int(0.75 * seg_len)))
    dtype = {"fp32": "f32", "bf16": "bf16", "fp32-simt": "f32"}[args.precision]
    if sc:
        work = (f"SCNet {'scnet_xl_wide_v5 (seed 10)' if args.model == 'scnet_xl' else 'scnet_small, masked (seed 9)'}, "
                f"{seconds:g} s stereo track, {n_seg} segments of 11 s, overlap 0.25, {batch} segments per launch, "
                f"precision {args.precision}")
    elif rof:
        name = ("Mel-Band RoFormer dim 384 depth 6, 60 mel bands (kim config, seed 6)" if args.model == "melband"
                else "BS-RoFormer dim 512 depth 12 (seed 3)")
        work = (f"{name}, {seconds:g} s stereo track, {n_seg} segments of 8 s, "
                f"overlap 0.25, {batch} segments per launch, precision {args.precision}")
    else:
        label = "HTDemucs 6-stem (seed 2)" if args.model == "htdemucs_6s" else "HTDemucs 4-stem"
        work = (f"{label}, {seconds:g} s stereo track, {n_seg} segments of 7.8 s, "
                f"overlap 0.25, {batch} segments per launch, precision {args.precision}")
        if len(model.sources) < len(model.config["sources"]):
            work += f", stems materialised: {','.join(model.sources)}"
    if shifts:
        work += f", shifts={shifts}"
    if n_tracks > 1:
        work += f", {n_tracks} tracks per rank"
    line = {"metric": METRIC, "value": round(value, 3), "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "strong" if split else "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": {"workload": work,
                       "track_seconds": seconds, "segments_per_launch": batch, "precision": args.precision,
                       "parallelism": (f"one track, segments sharded over {world} ranks + NCCL strip exchange"
                                       if split else f"whole tracks per rank x{world}"),
                       "launch": "eager" if args.no_graphs else "CUDA-graph replay of the forward",
                       "l2": "inputs and activations far larger than L2 (no flush needed)"},
            "e2e": {"value": round(e2e_value, 3), "unit": "audio-s/s", "h2d_bytes_per_step": n_tracks * 2 * L * 4,
                    "d2h_bytes_per_step": n_tracks * n_stems * 2 * L * 4},
            "gpu_launches": launches, "roofline": roofline, "clocks": clk, "split": phases,
            "kernels": {k: {"ms": round(v["ms"], 3), "n": v["n"]} for k, v in sorted(agg.items(), key=lambda kv: -kv[1]["ms"])}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if sc:
            line["cpu_baseline"] = cpu_baseline_scnet(xl=args.model == "scnet_xl")
        else:
            line["cpu_baseline"] = cpu_baseline_roformer(mel=args.model == "melband") if rof else cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
