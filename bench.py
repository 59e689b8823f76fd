#!/usr/bin/env python
"""Benchmark: MNv4-style segmentation net at 160x288, 256 frames per GPU.

One step = one forward pass of the conv graph over a batch of 256 frames
resident in HBM.  Frames shard across GPUs with no
collective on the hot path (weak scaling); the only collective is a
max-reduce of the timings.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --workload rvm [--streams S]
  python bench.py --workload cfg2 | cfg3          # BASELINE configs 2 / 3, one line per shape

Prints one JSON line (rank 0).  ``--workload rvm`` measures the recurrent
matting net instead (144x256, S = 1024 streams sharded across the GPUs, one
step = one frame of every stream, recurrent state resident on the GPU).
``--workload cfg2`` / ``cfg3`` time each conv of the config's sweep as one
launch over its batch and report TFLOP/s against the TF32 tensor peak.
--impl reference times the CPU restatement of ai_engine's ai-cpu path on
all host cores (the Rust reference itself cannot be built here: no Rust
toolchain).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
import zlib

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MNv4-seg 160x288 frames/s at 1/2/4/8 B200; conv GEMM TFLOP/s vs TF32 peak"
UNIT = "frames/s"
BATCH = 256
H, W = 160, 288


# DRAM bytes per frame that each layer's launch moved (dram__bytes_read.sum +
# dram__bytes_write.sum from one ncu capture of an eager step at 128 frames,
# divided by 128; the capture command and the per-layer table sit with the
# ncu summaries under profiles/).  Traffic scales with frames, so the
# roofline's per-launch traffic is this times the batch.
TRAFFIC_PER_FRAME = {
    "stem": 1562008,
    "e1.conv": 1691578,
    "e1.pw": 373514,
    "e2.conv": 371030,
    "e2.pw": 277406,
    "e3.dw5": 184760,
    "e3.exp": 255568,
    "e3.dw5s2": 583264,
    "e3.proj": 139546,
    "e4.0.exp": 70424,
    "e4.0.dw3": 138600,
    "e4.0.proj": 208744,
    "e4.1.exp": 70430,
    "e4.1.dw3": 138618,
    "e4.1.proj": 208742,
    "e5.exp": 71016,
    "e5.dw3": 278970,
    "e5.proj": 278738,
    "e5.0.exp": 95010,
    "e5.0.dw3": 427214,
    "e5.0.proj": 463672,
    "e5.1.exp": 94980,
    "e5.1.dw3": 421550,
    "e5.1.proj": 464198,
    "head960": 299468,
    "fpn.lat16": 697642,
    "fpn.up16": 46396,
    "fpn.lat8": 370550,
    "fpn.up8": 444408,
    "fpn.lat4": 1492144,
    "fpn.smooth4": 867448,
    "fpn.lat2": 2504488,
    "head.pw": 1873088,
    "mask": 46432,
}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


# ------------------------------------------------------------------ clocks ---

class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU during the timed region."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self._h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nv = pynvml
        except Exception as e:  # clocks are reported as unavailable, the bench still runs
            self.error = repr(e)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.004)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._h is not None:
            self._t.join()

    def summary(self):
        if self._h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------- CPU baseline ---

_CPU_MODEL = {}


def cpu_baseline(frames: int, threads: int, min_seconds: float = 0.0, mode: str = "throughput"):
    """ai-cpu restatement: `frames` frames of the same workload per pass,
    passes repeated until at least `min_seconds` have elapsed.  mode
    "throughput": one frame per core; "bands": ai-cpu's own threading, one
    frame at a time with each conv's output rows split over `threads`.
    Returns (frames/s, seconds, frames run)."""
    from ai_engine_b200 import segnet
    from oracle.graph import OracleModel
    if "m" not in _CPU_MODEL:
        g = segnet.build_graph()
        _CPU_MODEL["m"] = OracleModel(g, segnet.init_weights(g), (H, W, 3))
        _CPU_MODEL["x"] = segnet.synthetic_input(max(frames, threads), seed=1)
        _CPU_MODEL["m"].run_batch(_CPU_MODEL["x"][:threads], threads=threads)  # warm-up
    m, x = _CPU_MODEL["m"], _CPU_MODEL["x"]
    if x.shape[0] < frames:
        x = _CPU_MODEL["x"] = segnet.synthetic_input(frames, seed=1)
    done = 0
    t0 = time.perf_counter()
    while True:
        m.run_batch(x[:frames], threads=threads, mode=mode)
        done += frames
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    return done / dt, dt, done


def cpu_model_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference_rvm(args, threads):
    """--impl reference --workload rvm: the oracle chain of the RVM net, one
    stream-frame per core, each step a ~2 s sample."""
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, _, _ = rvm_cpu_baseline(threads, min_seconds=2.0)
        vals.append(v)
    wall = time.perf_counter() - t0
    value = statistics.median(vals)
    return value, wall, {"workload": "RVM-style matting net 144x256 (BASELINE config 5), CPU sample",
                         "h": 144, "w": 256}, "stream-frames (zero recurrent state)"


def run_reference(args, rank):
    """--impl reference: the CPU restatement of ai-cpu on all host cores."""
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    if args.workload in ("cfg2", "cfg3"):
        for label, op, n, ih, iw, split in sweep_shapes(args.workload, args.batch, args.shape):
            rng = np.random.default_rng(zlib.crc32(label.encode()))
            fan_in = op.cin * op.kh * op.kw
            w = (rng.standard_normal(op.cout * fan_in) / np.sqrt(fan_in)).astype(np.float32)
            b = rng.uniform(-0.1, 0.1, op.cout).astype(np.float32)
            gfs, t0 = [], time.perf_counter()
            for _ in range(args.steps):
                gf, fps, done = conv_cpu_baseline(op, ih, iw, w, b, threads, min_seconds=0.5)
                gfs.append(gf)
            value = statistics.median(gfs) / 1000.0
            line = {
                "impl": "reference", "metric": SWEEP_METRIC[args.workload], "value": round(value, 6),
                "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(1000 * (time.perf_counter() - t0) / max(args.steps, 1), 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic",
                "config": {"workload": f"BASELINE {args.workload}: {label}, CPU sample (one frame per step)"},
                "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                                 "sample": f"one frame per step, ai-cpu row bands over {threads} threads, "
                                           f">= 0.5 s per step; {cpu_model_name()}"},
                "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "note": "the Rust reference cannot be built here (no Rust toolchain); this arm runs its C restatement",
            }
            print(json.dumps(line), flush=True)
        return 0
    if getattr(args, "workload", "segnet") == "rvm":
        value, wall, config, what = run_reference_rvm(args, threads)
        line = {
            "impl": "reference", "metric": RVM_METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * wall / max(args.steps, 1), 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config,
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{what}, one per core, ~2 s per step; CPU restatement of crates/ai-cpu "
                                       f"compiled -O3 -ffp-contract=off; {cpu_model_name()}"},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the Rust reference cannot be built here (no Rust toolchain); this arm runs its C restatement",
        }
        print(json.dumps(line), flush=True)
        return 0
    frames = max(threads, 64)
    for _ in range(args.warmup):
        cpu_baseline(threads, threads)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, _, _ = cpu_baseline(frames, threads)
        vals.append(v)
    wall = time.perf_counter() - t0
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * wall / max(args.steps, 1), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "MNv4-style seg net 160x288 (BASELINE config 4), CPU sample", "frames_per_step": frames,
                   "h": H, "w": W},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{frames} frames per step, one frame per core (ai-cpu throughput mode), "
                                   f"CPU restatement of crates/ai-cpu compiled -O3 -ffp-contract=off; "
                                   f"{cpu_model_name()}"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the Rust reference cannot be built here (no Rust toolchain); this arm runs its C restatement",
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------ config 5: RVM net ---

RVM_METRIC = "RVM 144x256 frames/s, 1024 streams x 8 frames"
# DRAM bytes per frame of the config-5 step's dominant launch (ncu at 16
# streams, read + write, divided by 16; the capture's summary sits with the
# ncu summaries under profiles/)
RVM_TRAFFIC_PER_FRAME = {"d0.conv1": 6185696}


def rvm_cpu_baseline(threads: int, min_seconds: float = 10.0):
    """The oracle chain of the RVM net, one stream-frame per core at a time
    (ai-cpu throughput mode), zero recurrent state: (frames/s, s, frames)."""
    import concurrent.futures as cf

    from ai_engine_b200 import rvm
    from oracle.net import OracleNet
    g = rvm.build_graph()
    o = OracleNet(g, rvm.init_weights(g), rvm.inputs(), rvm.STATES, rvm.consts())
    x = rvm.synthetic_frames(threads, 1, seed=1)[0]
    st = o.zero_state(1)
    o.step({"src": x[:1]}, st)  # warm-up
    done = 0
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        while time.perf_counter() - t0 < min_seconds:
            list(ex.map(lambda i: o.step({"src": x[i:i + 1]}, st), range(threads)))
            done += threads
    dt = time.perf_counter() - t0
    return done / dt, dt, done


def run_rvm(args, world, rank, dev):
    """1024 independent streams sharded across the GPUs,
    each GPU stepping its streams' next frame as one batch with the ConvGRU
    state resident in HBM (strong scaling: the stream count is fixed)."""
    import torch
    import torch.distributed as dist

    from ai_engine_b200 import rvm
    from ai_engine_b200.net import NetModel

    if args.streams % world:
        raise SystemExit(f"{args.streams} streams do not split over {world} GPUs")
    n = args.streams // world
    g = rvm.build_graph()
    model = NetModel(g, rvm.init_weights(g), n, rvm.inputs(), rvm.OUTPUTS, rvm.STATES, rvm.consts(),
                     math=args.math, device=dev)
    frames = torch.from_numpy(rvm.synthetic_frames(n, 2, seed=200 + rank)).pin_memory()  # two frames, alternated
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    model.bufs["src"].copy_(frames[0])
    for _ in range(max(args.warmup, 3)):
        model.record()
        model.advance()
    model.capture()
    for _ in range(max(args.warmup, 3)):
        model.replay()
    torch.cuda.synchronize()
    # ---- timed region: K steps replayed from the captured graphs, frames resident
    sampler = ClockSampler(dev.index)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with sampler:
        e0.record(stream)
        for _ in range(args.steps):
            model.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = max_over_ranks(e0.elapsed_time(e1))
    value = n * world * args.steps / (total_ms / 1000.0)
    # ---- per-op eager timing (dominant op)
    recs = [r for r in model.recs if r.node.kind not in ("split", "view")]
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(recs) + 1)]
    evs[0].record(stream)
    for i, r in enumerate(recs):
        model.record(ops=[r])
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    per_op = [evs[i].elapsed_time(evs[i + 1]) for i in range(len(recs))]
    model.advance()
    # ---- end to end through the public API (NetModel.run_pipelined): every
    # step uploads its pinned frame batch and reads fgr + pha back; the
    # copies of neighbouring steps overlap the current step on copy streams
    model.release()
    outs_h = [{"fgr": torch.empty((n, rvm.H, rvm.W, 3)).pin_memory(),
               "pha": torch.empty((n, rvm.H, rvm.W, 1)).pin_memory()} for _ in range(2)]
    fgr_h, pha_h = outs_h[0]["fgr"], outs_h[0]["pha"]
    ins_h = [{"src": frames[k % 2]} for k in range(args.steps)]
    model.run_pipelined([{"src": frames[k]} for k in range(2)], outs_h)  # warm-up (captures the slot graphs)
    torch.cuda.synchronize()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    model.run_pipelined(ins_h, [outs_h[k % 2] for k in range(args.steps)])
    t1.record(stream)
    torch.cuda.synchronize()
    e2e_value = n * world * args.steps / (max_over_ranks(t0.elapsed_time(t1)) / 1000.0)
    act_bytes = sum(b.numel() * 4 for b in model.bufs.values())
    model.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    pk = peaks()
    i = max(range(len(recs)), key=lambda j: per_op[j])
    top = recs[i]
    sec = per_op[i] / 1000.0
    if top.plan is not None:
        fl, by = top.plan.flops, top.plan.min_bytes
    else:
        nd = top.node
        outs = [nd.out]
        by = 4 * n * sum(int(np.prod(model.shapes[t])) for t in (*[x for x in nd.ins if x in model.shapes], *outs))
        fl = 0
    roof = {"bound": "hbm", "achieved": by / sec / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s"}
    ridge = pk["bf16_tflops"] / 2.0 * 1e12 / (pk["hbm_gbs"] * 1e9)
    if top.plan is not None and top.plan.math == "tf32" and fl / max(by, 1) >= ridge:
        roof = {"bound": "tensor", "achieved": fl / sec / 1e12, "peak": pk["bf16_tflops"] / 2.0, "unit": "TFLOP/s"}
    roof["frac"] = round(roof["achieved"] / roof["peak"], 4)
    roof["achieved"] = round(roof["achieved"], 3)
    tpf = RVM_TRAFFIC_PER_FRAME.get(top.node.out)
    roof["traffic"] = int(tpf * n) if tpf is not None else None
    roof["traffic_src"] = "ncu dram bytes at 16 streams, scaled by frames" if tpf is not None else None
    roof["kernel"] = f"{top.node.out} ({top.node.kind}" + (f" {top.plan.kernel}/{top.plan.math})" if top.plan else ")")
    roof["share"] = round(per_op[i] / sum(per_op), 4)
    line = {
        "metric": RVM_METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "tf32" if args.math in ("auto", "tf32") else "f32",
        "data": "synthetic",
        "config": {"workload": "RVM-style matting net 144x256 (BASELINE config 5), ConvGRU state carried",
                   "streams": args.streams, "streams_per_gpu": n, "h": rvm.H, "w": rvm.W,
                   "parallelism": f"streams sharded over {world} GPU(s)", "math": args.math,
                   "l2": f"inputs larger than L2 ({frames[0].numel() * 4 / 1e6:.0f} MB of frames, "
                         f"{act_bytes / 1e9:.1f} GB of activations per step per GPU)",
                   "conv_gflop_per_frame": round(rvm.conv_flops_per_frame() / 1e9, 4)},
        "conv_tflops": round(rvm.conv_flops_per_frame() * n * world / (total_ms / args.steps / 1000.0) / 1e12, 3),
        "roofline": roof,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": int(frames[0].numel() * 4),
                "d2h_bytes_per_step": int((fgr_h.numel() + pha_h.numel()) * 4)},
        "gpu_launches": len(recs) * args.steps,
        "clocks": sampler.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, dt, done = rvm_cpu_baseline(threads)
        line["cpu_baseline"] = {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": f"{done} stream-frames of the same net, one per core, {dt:.1f} s on "
                                          f"{cpu_model_name()}"}
    if args.layers:
        for r, ms in sorted(zip(recs, per_op), key=lambda t: -t[1]):
            kern = f"{r.plan.kernel}/{r.plan.math}" if r.plan is not None else r.node.kind
            print(f"{r.node.out:16s} {kern:14s} {ms * 1000:9.1f} us", file=sys.stderr)
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------- ai_engine's shipped model (segm_r11) ---

SEGM_R11 = os.path.join(ROOT, "tests", "golden", "segm_r11.npz")  # the .sw container, committed as a fixture


def run_segm_r11(args, world, rank, dev):
    """ai_engine's shipped segmentation model web/models/segm_r11_160x288.sw
    (44 ops, real weights) read by the .sw reader and run by the node
    executor: `--batch` frames per GPU (weak scaling), frames resident for
    `value`, pinned host frames in and logits out per step for `e2e`."""
    import torch
    import torch.distributed as dist

    from ai_engine_b200.net import NetModel
    from ai_engine_b200.swfile import load_sw

    sw = load_sw(np.load(SEGM_R11)["sw"].tobytes())
    n = args.batch
    (inp, (h, w, c)), = sw.inputs.items()
    out = sw.outputs[0]
    model = NetModel(sw.nodes, sw.weights, n, sw.inputs, sw.outputs, sw.states, sw.consts, math=args.math, device=dev)
    x = torch.from_numpy(np.random.default_rng(300 + rank).random((n, h, w, c), dtype=np.float32)).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    model.bufs[inp].copy_(x)
    for _ in range(max(args.warmup, 3)):
        model.record()
    model.capture()
    for _ in range(max(args.warmup, 3)):
        model.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(dev.index)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with sampler:
        e0.record(stream)
        for _ in range(args.steps):
            model.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = max_over_ranks(e0.elapsed_time(e1))
    value = n * world * args.steps / (total_ms / 1000.0)
    launches = sum(1 for r in model.recs if r.node.kind not in ("split", "view"))
    # end to end: pinned frames in, logits out, copies overlapping the steps
    model.release()
    oshape = model.tensor(out).shape
    outs = [{out: torch.empty(oshape).pin_memory()} for _ in range(2)]
    model.run_pipelined([{inp: x}] * 2, outs)
    torch.cuda.synchronize()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    model.run_pipelined([{inp: x}] * args.steps, [outs[k % 2] for k in range(args.steps)])
    t1.record(stream)
    torch.cuda.synchronize()
    e2e_value = n * world * args.steps / (max_over_ranks(t0.elapsed_time(t1)) / 1000.0)
    flops = model.conv_flops
    model.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": "segm_r11 160x288 frames/s (ai_engine's shipped .sw model)", "value": round(value, 2), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "tf32" if args.math in ("auto", "tf32") else "f32",
        "data": "synthetic frames, the model's real weights",
        "config": {"workload": "web/models/segm_r11_160x288.sw through the .sw reader and the node executor",
                   "per_gpu_batch": n, "h": h, "w": w, "ops": len(sw.nodes), "math": args.math,
                   "conv_mflop_per_frame": round(flops / n / 1e6, 2)},
        "conv_tflops": round(flops * world / (total_ms / args.steps / 1000.0) / 1e12, 3),
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": int(x.numel() * 4),
                "d2h_bytes_per_step": int(np.prod(oshape) * 4)},
        "gpu_launches": launches * args.steps,
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------- configs 2 and 3: single convs ---

CFG2 = [(16, 16), (32, 64), (64, 128), (128, 256)]          # (Cin, Cout), 3x3 pad 1 at 160x288
CFG3 = [(960, 1280), (1280, 960), (512, 2048)]              # (K, N), 1x1 at 10x18
SWEEP_METRIC = {"cfg2": "conv GEMM TFLOP/s vs TF32 peak (BASELINE config 2: 3x3 implicit GEMM at 160x288)",
                "cfg3": "conv GEMM TFLOP/s vs TF32 peak (BASELINE config 3: split-K 1x1 GEMM at 10x18)"}
L2_BYTES = 126 << 20


def sweep_shapes(which: str, batch: int, only: str = ""):
    """(label, Conv2d, n, ih, iw, split) of the BASELINE config's sweep, in the
    reference's own shape-table spirit (crates/ai-gpu/src/bench.rs:166-260):
    config 2 at `batch` frames for every (Cin, Cout) and stride; config 3 at
    batch 1, 64 and 256 with the auto split, plus batch 1 at every split factor.
    `only`: keep the shapes whose label contains it."""
    return [s for s in _sweep_shapes(which, batch) if only in s[0]]


def _sweep_shapes(which: str, batch: int):
    from ai_engine_b200 import Conv2d
    out = []
    if which == "cfg2":
        for cin, cout in CFG2:
            for s in (1, 2):
                out.append((f"3x3 s{s} {cin}->{cout} B={batch}", Conv2d.same(cin, cout, 3, s, "hardswish"),
                            batch, 160, 288, 0))
    else:
        for k, n in CFG3:
            for b in (256, 64, 1):
                out.append((f"1x1 {k}->{n} B={b} split auto", Conv2d.pointwise(k, n, "none"), b, 10, 18, 0))
            for sp in (1, 4, 8, 16):
                out.append((f"1x1 {k}->{n} B=1 split {sp}", Conv2d.pointwise(k, n, "none"), 1, 10, 18, sp))
    return out


def conv_cpu_baseline(op, ih, iw, w, b, threads, min_seconds=1.5):
    """One frame through the ai-cpu restatement in ai-cpu's own threading
    (row bands over all cores, crates/ai-cpu/src/model.rs:421-441), repeated
    for at least `min_seconds`: (GFLOP/s, frames/s, frames run)."""
    import oracle
    p = oracle.Plan(op, ih, iw, w, b)
    x = np.random.default_rng(5).uniform(-1, 1, (ih, iw, op.cin)).astype(np.float32)
    y = np.empty((p.oh, p.ow, op.cout), np.float32)
    p.run_frame(x, y, threads=threads)  # warm-up
    done, t0 = 0, time.perf_counter()
    while True:
        p.run_frame(x, y, threads=threads)
        done += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    flops = 2 * p.oh * p.ow * op.cout * (op.cin // op.groups) * op.kh * op.kw
    return flops * done / dt / 1e9, done / dt, done


def run_sweep(args, world, rank, dev):
    """BASELINE configs 2 and 3: each shape of the sweep as one conv launch
    over its batch (frames resident in HBM), K launches timed one by one
    with CUDA events on the launching stream, the L2 flushed (a 256 MB
    write) before every launch so that small shapes are not served from L2.
    One JSON line per shape; frames shard across GPUs (each rank runs the
    same shapes on its own batch, weak scaling)."""
    import torch
    import torch.distributed as dist

    from ai_engine_b200.conv import ConvPlan

    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    pk = peaks()
    hbm = pk["hbm_gbs"]
    tf32 = pk["bf16_tflops"] / 2.0            # TF32 dense = half the bf16 rate
    tf32_sus = pk["bf16_tflops_sustained"] / 2.0
    threads = os.cpu_count() or 1

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for label, op, n, ih, iw, split in sweep_shapes(args.workload, args.batch, args.shape):
        rng = np.random.default_rng(zlib.crc32(label.encode()))
        fan_in = op.cin * op.kh * op.kw
        if args.workload == "cfg2":  # Kaiming-normal W, U(-0.1, 0.1) bias
            w = (rng.standard_normal(op.cout * fan_in) * np.sqrt(2.0 / fan_in)).astype(np.float32)
            b = rng.uniform(-0.1, 0.1, op.cout).astype(np.float32)
        else:                        # W ~ N(0, 1/K), no bias
            w = (rng.standard_normal(op.cout * fan_in) / np.sqrt(fan_in)).astype(np.float32)
            b = np.zeros(op.cout, np.float32)
        plan = ConvPlan(op, n, ih, iw, math=args.math, split_k=split, device=dev).load_weights(w, b)
        g = torch.Generator(device=dev)
        g.manual_seed(1000 + rank)
        x = torch.rand((n, ih, iw, op.cin), device=dev, generator=g).mul_(2).sub_(1)
        out = torch.empty(plan.out_shape(), dtype=torch.float32, device=dev)
        for _ in range(max(args.warmup, 3)):
            plan(x, out=out)
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        sampler = ClockSampler(dev.index)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with sampler:
            for e0, e1 in evs:
                flush.zero_()
                e0.record(stream)
                plan(x, out=out)
                e1.record(stream)
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in evs) / len(evs))
        fl, by = plan.flops, plan.min_bytes
        tflops = fl / (ms / 1000.0) / 1e12
        ai = fl / by
        roof_t = min(tf32, ai * hbm / 1000.0)  # TFLOP/s the launch could reach: min(peak, AI x HBM)
        if ai * hbm / 1000.0 >= tf32:
            roof = {"bound": "tensor", "achieved": tflops, "peak": tf32, "unit": "TFLOP/s",
                    "frac_sustained": round(tflops / tf32_sus, 4), "peak_src": pk["src"] + " (TF32 = bf16/2, burst)"}
        else:
            roof = {"bound": "hbm", "achieved": by / (ms / 1000.0) / 1e9, "peak": hbm, "unit": "GB/s",
                    "peak_src": pk["src"]}
        roof["frac"] = round(roof["achieved"] / roof["peak"], 4)
        roof["achieved"] = round(roof["achieved"], 3)
        roof["traffic"] = None
        roof["kernel"] = f"{plan.kernel}/{plan.math}" + (f" split {plan.info.split_k}" if plan.info.split_k > 1 else "")
        # end to end through the public API: pinned input up, the conv, output down, every step
        e2e_steps = min(args.steps, 5)
        xh = torch.empty(x.shape, dtype=torch.float32).pin_memory()
        xh.copy_(x)
        oh_ = torch.empty(out.shape, dtype=torch.float32).pin_memory()
        xd = torch.empty_like(x)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(e2e_steps):
            xd.copy_(xh, non_blocking=True)
            plan(xd, out=out)
            oh_.copy_(out, non_blocking=True)
        t1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(t0.elapsed_time(t1)) / e2e_steps
        line = {
            "metric": SWEEP_METRIC[args.workload], "value": round(tflops * world, 3), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": plan.math,
            "data": "synthetic",
            "config": {"workload": f"BASELINE {args.workload}: {label}", "per_gpu_batch": n, "h": ih, "w": iw,
                       "cin": op.cin, "cout": op.cout, "stride": op.sh, "act": op.act, "math": args.math,
                       "split_k": plan.info.split_k, "flop_per_launch": fl, "min_bytes_per_launch": by,
                       "arith_intensity": round(ai, 2), "l2": "flushed before every timed launch (256 MB write)"},
            "frames_per_s": round(n * world / (ms / 1000.0), 2),
            "of_roofline": round(tflops / roof_t, 4),
            "roofline": roof,
            "e2e": {"value": round(fl * world / (e2e_ms / 1000.0) / 1e12, 4), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": int(x.numel() * 4), "d2h_bytes_per_step": int(out.numel() * 4)},
            "gpu_launches": args.steps,
            "clocks": sampler.summary(),
        }
        if world == 1 and not args.no_cpu_baseline and rank == 0:
            gf, fps, done = conv_cpu_baseline(op, ih, iw, w, b, threads)
            line["cpu_baseline"] = {"value": round(gf / 1000.0, 6), "unit": "TFLOP/s", "cores": threads,
                                    "kind": "port", "gflops": round(gf, 2), "frames_per_s": round(fps, 3),
                                    "sample": f"{done} frame(s) of the same conv, ai-cpu row bands over {threads} "
                                              f"threads, >= 1.5 s on {cpu_model_name()}"}
        if rank == 0:
            print(json.dumps(line), flush=True)
        del plan, x, out, xh, oh_, xd
        torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------- GPU arm ---

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--math", default="auto", choices=["auto", "ffma", "tf32", "fp32_strict"])
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ffma", action="store_true", help="segnet: skip the FP32 FFMA (value_ffma) timing")
    ap.add_argument("--fuse-blocks", type=int, default=None, choices=[0, 1],
                    help="run each small-frame inverted-bottleneck block as one launch (default: Model's)")
    ap.add_argument("--fuse-resize", type=int, default=None, choices=[0, 1],
                    help="fold each resize that only feeds a conv residual into that conv (default: Model's)")
    ap.add_argument("--fuse-stem", type=int, default=None, choices=[0, 1],
                    help="run the 1x1 over the stem's output inside the stem's launch (default: Model's)")
    ap.add_argument("--layers", action="store_true", help="print the per-layer table to stderr")
    ap.add_argument("--workload", default="segnet", choices=["segnet", "rvm", "segm_r11", "cfg2", "cfg3"],
                    help="segnet: BASELINE config 4 (default); rvm: the recurrent matting net of config 5; "
                         "segm_r11: ai_engine's shipped segmentation model (.sw, real weights); "
                         "cfg2 / cfg3: the single-conv sweeps of configs 2 and 3 (one line per shape)")
    ap.add_argument("--streams", type=int, default=1024, help="rvm: video streams over all GPUs")
    ap.add_argument("--shape", default="", help="cfg2 / cfg3: only the shapes whose label contains this")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # each rank's pinned host buffers on its GPU's NUMA node
        from ai_engine_b200.dist import bind_to_gpu_numa
        bind_to_gpu_numa(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if args.workload == "rvm":
        return run_rvm(args, world, rank, dev)
    if args.workload == "segm_r11":
        return run_segm_r11(args, world, rank, dev)
    if args.workload in ("cfg2", "cfg3"):
        return run_sweep(args, world, rank, dev)

    from ai_engine_b200 import segnet
    from ai_engine_b200.conv import resize_bilinear, run_dw_pw, run_mbconv, run_stem_pw
    from ai_engine_b200.graph import Model

    n = args.batch
    g = segnet.build_graph()
    weights = segnet.init_weights(g)  # same weights on every rank (replicas)
    fuse_kw = {} if args.fuse_resize is None else {"fuse": bool(args.fuse_resize)}
    if args.fuse_blocks is not None:
        fuse_kw["fuse_blocks"] = bool(args.fuse_blocks)
    if args.fuse_stem is not None:
        fuse_kw["fuse_stem"] = bool(args.fuse_stem)
    model = Model(g, weights, n, (H, W, 3), math=args.math, device=dev, **fuse_kw)
    x_host = torch.from_numpy(segnet.synthetic_input(n, seed=100 + rank)).pin_memory()
    model.bufs["input"].copy_(x_host)
    stream = torch.cuda.current_stream(dev)
    out_host = torch.empty(model.bufs[model.output].shape, dtype=torch.float32).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- warm-up (eager and captured)
    for _ in range(max(args.warmup, 3)):
        model.record()
    model.capture()
    for _ in range(max(args.warmup, 3)):
        model.infer()
    torch.cuda.synchronize()

    # ---- timed region (value): K steps of the captured batch graph, inputs
    # resident in HBM, CUDA events on the replaying stream
    sampler = ClockSampler(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with sampler:
        e0.record(stream)
        for _ in range(args.steps):
            model.infer()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = max_over_ranks(e0.elapsed_time(e1))
    value = n * world * args.steps / (total_ms / 1000.0)

    # ---- per-op breakdown: the same ops issued eagerly, one CUDA event
    # after each launch on the launching stream (roofline of the top kernel)
    ops = model.ops
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(ops) + 1)] for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for k in range(args.steps):
        ev = evs[k]
        ev[0].record(stream)
        for i, r in enumerate(ops):
            src, out = model.bufs[r.src], model.bufs[r.out]
            if r.kind == "conv":
                r.plan(src, model.bufs[r.res] if r.res else None, out=out)
            elif r.kind == "dwpw":
                run_dw_pw(r.plan, r.head, src, out=out, up=model.bufs[r.up] if r.up else None)
            elif r.kind == "mb":
                run_mbconv(*r.blk, src, res=model.bufs[r.res] if r.res else None, out=out)
            elif r.kind == "stempw":
                run_stem_pw(r.plan, r.head, src, stem_out=out, pw_out=model.bufs[r.out2])
            else:
                resize_bilinear(src, r.size[0], r.size[1], add=model.bufs[r.res] if r.res else None, out=out)
            ev[i + 1].record(stream)
    torch.cuda.synchronize()
    barrier()
    eager_ms = max_over_ranks(evs[0][0].elapsed_time(evs[-1][-1]))
    eager_value = n * world * args.steps / (eager_ms / 1000.0)
    per_op = np.zeros(len(ops))
    for ev in evs:
        for i in range(len(ops)):
            per_op[i] += ev[i].elapsed_time(ev[i + 1])
    per_op /= args.steps

    # ---- end to end through the public API: every step uploads its pinned
    # host frames and reads its mask back (Model.run_pipelined overlaps the
    # copies of neighbouring batches with compute).  Headline (`e2e`):
    # config 4's own f32 frames (12 bytes per pixel); also reported
    # (`e2e_u8`): u8 RGB camera frames (3 bytes per pixel, normalised on the
    # GPU by the graph's first op, as ai_engine's camera pipeline feeds its
    # models).
    outs_host = [out_host, torch.empty_like(out_host).pin_memory()]

    def time_e2e(m, xh):
        m.run_pipelined([xh] * 3, [outs_host[k % 2] for k in range(3)])
        torch.cuda.synchronize()
        barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        m.run_pipelined([xh] * args.steps, [outs_host[k % 2] for k in range(args.steps)])
        t1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(t0.elapsed_time(t1))
        return n * world * args.steps / (ms / 1000.0)

    e2e_f32_value = time_e2e(model, x_host)
    model.release()
    # ---- the same network at the reference's own precision: FP32 FFMA on the
    # CUDA cores for every conv (math "ffma"), timed the same way (graph replay)
    ffma_value = None
    if not args.no_ffma:
        model_ffma = Model(g, weights, n, (H, W, 3), math="ffma", device=dev, **fuse_kw)
        model_ffma.bufs["input"].copy_(x_host)
        model_ffma.capture()
        for _ in range(max(args.warmup, 3)):
            model_ffma.infer()
        torch.cuda.synchronize()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            model_ffma.infer()
        f1.record(stream)
        torch.cuda.synchronize()
        ffma_value = n * world * args.steps / (max_over_ranks(f0.elapsed_time(f1)) / 1000.0)
        model_ffma.release()
        del model_ffma
    model_u8 = Model(g, weights, n, (H, W, 3), math=args.math, input_u8=True, device=dev, **fuse_kw)
    x_host_u8 = torch.from_numpy(np.rint(x_host.numpy() * 255.0).astype(np.uint8)).pin_memory()
    e2e_value = time_e2e(model_u8, x_host_u8)
    model_u8.release()

    # ---- optional output gather (N > 1): every rank's masks into one
    # buffer on rank 0 over NCCL; not part of the hot path, timed apart
    gather = None
    if world > 1:
        from ai_engine_b200.dist import gather_outputs
        mask = model_u8.bufs[model_u8.output]
        gather_outputs(mask, n * world)  # warm-up (allocations, NCCL channels)
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        g0.record(stream)
        for _ in range(reps):
            gather_outputs(mask, n * world)
        g1.record(stream)
        torch.cuda.synchronize()
        gather = {"ms": round(max_over_ranks(g0.elapsed_time(g1)) / reps, 4),
                  "bytes_per_rank": int(mask.numel() * 4), "collective": "all_gather_into_tensor (NCCL)"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    # ---- roofline of the dominant launch
    pk = peaks()
    hbm = pk["hbm_gbs"]
    tf32_peak = pk["bf16_tflops"] / 2.0  # TF32 dense = half the bf16 rate
    layers = []
    for r, ms in zip(ops, per_op):
        if r.kind == "mb":
            # fused block: the expanded tensor and the depthwise output are
            # neither written nor read
            ex, dw, pj = r.blk
            inter = 4 * n * ex.oh * ex.ow * ex.op.cout
            if dw is None:  # expand straight into project: the wide tensor is neither written nor read
                fl, by, kern = ex.flops + pj.flops, ex.min_bytes + pj.min_bytes - 2 * inter, "ex+pj"
            else:
                fl = ex.flops + dw.flops + pj.flops
                by = ex.min_bytes + dw.min_bytes + pj.min_bytes - 4 * inter
                kern = "ex+dw+pj"
            math = "tf32"
        elif r.kind == "dwpw":
            # fused depthwise + 1x1 head: the intermediate is neither written nor read
            inter = 4 * n * r.plan.oh * r.plan.ow * r.plan.op.cout
            fl, by = r.plan.flops + r.head.flops, r.plan.min_bytes + r.head.min_bytes - 2 * inter
            if r.up:  # the half-size source whose resize the kernel adds to its input
                by += 4 * n * int(np.prod(model.shapes[r.up]))
            kern, math = "dw+pw", r.plan.math
        elif r.kind == "stempw":
            # stem + the 1x1 over its output: the 1x1 does not read the stem output back
            inter = 4 * n * r.plan.oh * r.plan.ow * r.plan.op.cout
            fl, by = r.plan.flops + r.head.flops, r.plan.min_bytes + r.head.min_bytes - inter
            kern, math = "stem+pw", "tf32"
        elif r.plan is not None:
            fl, by = r.plan.flops, r.plan.min_bytes
            kern, math = r.plan.kernel, r.plan.math
        else:
            oh, ow = r.size
            c = model.shapes[r.out][2]
            ih, iw, _ = model.shapes[r.src]
            fl, by = 0, 4 * n * c * (ih * iw + oh * ow + (oh * ow if r.res else 0))
            kern, math = "resize", "f32"
        layers.append({"op": r.out, "kernel": kern, "math": math, "ms": float(ms), "flops": int(fl),
                       "bytes": int(by)})
    dom = max(layers, key=lambda l: l["ms"])
    sec = dom["ms"] / 1000.0
    ai = dom["flops"] / max(dom["bytes"], 1)
    ridge = tf32_peak * 1e12 / (hbm * 1e9)
    if dom["kernel"] in ("pw", "igemm") and dom["math"] == "tf32" and ai >= ridge:
        roof = {"bound": "tensor", "achieved": dom["flops"] / sec / 1e12, "peak": tf32_peak, "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": dom["bytes"] / sec / 1e9, "peak": hbm, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    tpf = TRAFFIC_PER_FRAME.get(dom["op"])
    roof["traffic"] = int(tpf * n) if tpf is not None else None
    roof["traffic_src"] = "ncu dram bytes at 128 frames, scaled by frames" if tpf is not None else None
    roof["kernel"] = f"{dom['op']} ({dom['kernel']}/{dom['math']})"
    roof["share"] = dom["ms"] / float(per_op.sum())
    roof["peak_src"] = pk["src"] + (" (TF32 = bf16/2)" if roof["bound"] == "tensor" else "")
    for k in ("achieved", "peak", "frac", "share"):
        roof[k] = round(roof[k], 4)

    conv_flops = sum(l["flops"] for l in layers)
    conv_ms = float(per_op.sum())
    dtype = "tf32" if any(l["math"] == "tf32" for l in layers) else "f32"

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
        "config": {"workload": "MNv4-style seg net 160x288, 256 frames per GPU (BASELINE config 4)",
                   "global_batch": n * world, "per_gpu_batch": n, "h": H, "w": W, "parallelism": f"dp{world}",
                   "math": args.math, "l2": "inputs larger than L2 (141 MB frames, ~2.5 GB activations per step)",
                   "conv_mflop_per_frame": round(conv_flops / n / 1e6, 2)},
        "conv_tflops": round(conv_flops * world / (total_ms / args.steps / 1000.0) / 1e12, 3),
        "roofline": roof,
        "e2e": {"value": round(e2e_f32_value, 2), "unit": UNIT, "h2d_bytes_per_step": int(x_host.numel() * 4),
                "d2h_bytes_per_step": int(out_host.numel() * 4),
                "input": "config 4's f32 U(0,1) frames, uploaded from pinned host memory every step"},
        "e2e_u8": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": int(x_host_u8.numel()),
                   "d2h_bytes_per_step": int(out_host.numel() * 4),
                   "input": "u8 RGB frames (the f32 frames quantised), normalised on the GPU (aie_input_u8)"},
        "value_ffma": None if ffma_value is None else round(ffma_value, 2),
        "eager_value": round(eager_value, 2),
        "gpu_launches": len(ops) * args.steps,
        "clocks": sampler.summary(),
    }
    if gather is not None:
        line["gather"] = gather
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, dt, done = cpu_baseline(2 * threads, threads, min_seconds=10.0)
        vb, dtb, doneb = cpu_baseline(1, threads, min_seconds=4.0, mode="bands")
        line["cpu_baseline"] = {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port",
                                "gflops": round(v * conv_flops / n / 1e9, 2),
                                "sample": f"{done} frames of the same workload, one frame per core (ai-cpu "
                                          f"throughput mode), {dt:.1f} s on {cpu_model_name()}",
                                "aicpu_mode": {"value": round(vb, 3), "unit": UNIT, "threads": threads,
                                               "gflops": round(vb * conv_flops / n / 1e9, 2),
                                               "sample": f"{doneb} frames one at a time, each conv's output rows "
                                                         f"split over {threads} threads (crates/ai-cpu/src/"
                                                         f"model.rs:421-441), {dtb:.1f} s"}}
    if args.layers:
        for l in layers:
            t = l["ms"] / 1000
            print(f"{l['op']:14s} {l['kernel']:7s} {l['math']:11s} {l['ms']*1000:9.1f} us "
                  f"{l['bytes']/t/1e9 if t else 0:8.1f} GB/s {l['flops']/t/1e12 if t else 0:8.2f} TF/s",
                  file=sys.stderr)
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
