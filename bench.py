"""Benchmark of the fused Local Attender (the UPLiFT hot path) on B200.

Workload ("dinov2-s14-448-iters4"): the four Local Attender calls of the
DINOv2-S/14 upsampler at 448 px, iters=4, B=8 images per GPU, bf16:
value 384ch 32^2 -> 64^2 -> 128^2 -> 256^2 -> 512^2 under 64-ch guides,
K=17, each call's output the next call's value.  One step = those four
calls (2.785 output Mpix per GPU).  Synthetic inputs (seed 0, N(0,1)) and a
random-init LocalAttender(64, 17) in bf16.  Inputs are larger than L2
(3.0 GB streamed per step), so no L2 flush is needed between steps.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Prints one JSON line (rank 0).  `value` = output Mpix/s over all ranks with
inputs resident in HBM (device time, max over ranks); `e2e` = the same
metric through LocalAttender.forward with pinned host buffers and the
host<->device copies inside the timed region; `roofline` = algorithmic
HBM bytes / kernel time of the attender kernel vs the measured copy
bandwidth; `cpu_baseline` = the reference algorithm (oracle port, torch
CPU ops) on the host cores on a bounded sample.  Multi-GPU: weak scaling,
each rank runs its own 8 images; no collective on the data path.
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
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Local Attender output Mpix/s (bf16, DINOv2-S/14 448px iters=4 attender chain)"
UNIT = "Mpix/s"
K_NBR = 17
CG = 64
C = 384
B_PER_GPU = 8
LEVELS = [(32, 64), (64, 128), (128, 256), (256, 512)]  # (coarse, fine) sides
ELEM = 2  # bf16 bytes


def algo_bytes_per_pixel(Cg=CG, Cv=C, I=2, s=ELEM):
    """guide read + output write + value read once (amortised over I^2)."""
    return Cg * s + Cv * s + Cv * s / (I * I)


def out_pixels(B=None):
    B = B_PER_GPU if B is None else B
    return sum(B * fo * fo for _, fo in LEVELS)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    """DRAM bytes per step from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "la_tc_kernel_dinov2_448_b8_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_step:"):
            return float(line.split(":", 1)[1])
    return None


REF_ROOT = ROOT / "baseline" / "_ref"


def reference_modules(*names):
    """Submodules of the unmodified reference package, pip-installed under
    baseline/_ref, e.g. reference_modules("uplift", "fast") -> ([uplift.uplift,
    uplift.fast], None); ([], reason) when it is absent or fails to import.
    The package's __init__ imports the feature extractor, which needs
    omegaconf (not installed, and not on the attender's path), so a bare
    package object whose __path__ is the installed directory is registered
    first and the submodules are imported from it as they are."""
    import importlib
    import types
    pkg_dir = REF_ROOT / "uplift"
    if not (pkg_dir / "uplift.py").exists():
        return [], f"reference not installed under {REF_ROOT.relative_to(ROOT)}"
    cur = sys.modules.get("uplift")
    if cur is None or list(getattr(cur, "__path__", [])) != [str(pkg_dir)]:
        pkg = types.ModuleType("uplift")
        pkg.__path__ = [str(pkg_dir)]
        sys.modules["uplift"] = pkg
    try:
        return [importlib.import_module("uplift." + n) for n in names], None
    except Exception as e:  # noqa: BLE001 -- reported, not raised: the bench line still prints
        return [], f"reference import failed: {type(e).__name__}: {e}"[:200]


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device(f"cuda:{local}"))
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def workload_config(world):
    """The `config` object of both arms' JSON lines."""
    return {"workload": "dinov2-s14-448-iters4 Local Attender chain",
            "images_per_gpu": B_PER_GPU, "global_images": B_PER_GPU * world,
            "K": K_NBR, "guide_channels": CG, "value_channels": C, "scale": 2,
            "levels": [f"{c}^2->{f}^2" for c, f in LEVELS],
            "out_mpix_per_step_per_gpu": round(out_pixels() / 1e6, 4),
            "l2": "inputs larger than L2 (3.03 GB algorithmic per step), no flush",
            "parallelism": f"batch-sharded x{world}, no data-path collective"}


def make_inputs(dev, B=None, seed=0):
    """Guides for the four levels and the level-0 value map (bf16, NHWC)."""
    from uplift_b200.attender import LocalAttender
    B = B_PER_GPU if B is None else B
    g = torch.Generator().manual_seed(seed)
    torch.manual_seed(seed)
    la = LocalAttender(CG, K_NBR).to(torch.bfloat16)  # default nn.Conv2d init under seed 0
    value0 = torch.randn(B, C, LEVELS[0][0], LEVELS[0][0], generator=g).to(torch.bfloat16)
    guides = [torch.randn(B, CG, fo, fo, generator=g).to(torch.bfloat16) for _, fo in LEVELS]
    cl = torch.channels_last
    host = dict(value0=value0.contiguous(memory_format=cl), guides=[x.contiguous(memory_format=cl) for x in guides])
    return la, host


def run_ours(args, world, rank, local):
    from uplift_b200 import _native, ops
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    _native.load()
    la, host = make_inputs(torch.device("cpu"), seed=0)
    la = la.to(dev)
    value0 = host["value0"].to(dev)
    guides = [x.to(dev) for x in host["guides"]]
    w = la.conv1.weight.detach().float().reshape(K_NBR, CG).contiguous()
    b = la.conv1.bias.detach().float().contiguous()
    offsets, pn = la.offsets, la.pn
    outs = [torch.empty((B_PER_GPU, C, fo, fo), dtype=torch.bfloat16, device=dev,
                        memory_format=torch.channels_last) for _, fo in LEVELS]
    stream = torch.cuda.current_stream(dev)

    def step(events=None):
        v = value0
        for i, g in enumerate(guides):
            if events is not None:
                events[i][0].record(stream)
            ops.local_attender_raw(g, v, w, b, offsets, pn, out=outs[i])
            if events is not None:
                events[i][1].record(stream)
            v = outs[i]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # one step = four launches on fixed buffers, replayed as a CUDA graph so
    # that host launch latency does not starve the GPU between the short
    # early levels (--eager times plain launches instead)
    graph = None
    if not args.eager:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize(dev)

    # ---- device-resident timing: K steps between a barrier + sync on both sides
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for s in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clk = clocks.stop()
    ms_local = t0.elapsed_time(t1)
    ms_total = max_over_ranks(ms_local, world, dev)
    ms_step = ms_total / args.steps
    mpix_step = out_pixels() / 1e6
    value = world * mpix_step / (ms_step / 1e3)

    # per-level launch durations (events around each eager launch), for the
    # breakdown only
    per_launch = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in LEVELS] for _ in range(args.steps)]
    for s in range(args.steps):
        step(per_launch[s])
    torch.cuda.synchronize(dev)
    kern_ms = [sum(per_launch[s][i][0].elapsed_time(per_launch[s][i][1]) for s in range(args.steps))
               for i in range(len(LEVELS))]
    del graph

    # ---- roofline of the attender kernel (all four launches of a step)
    bpp = algo_bytes_per_pixel()
    algo_bytes_step = out_pixels() * bpp
    # every launch of the step is the attender kernel: achieved = algorithmic
    # bytes of the four launches / device time of the step
    achieved = algo_bytes_step / (ms_step / 1e3) / 1e9
    lvl_px = [B_PER_GPU * fo * fo for _, fo in LEVELS]
    lvl_gbs = [round(px * bpp / (ms / args.steps / 1e3) / 1e9, 1) for px, ms in zip(lvl_px, kern_ms)]
    peak, peak_kind = load_peaks()
    traffic = load_traffic()

    # ---- the reference's own GPU path (Triton) on the same chain
    triton = None
    if not args.no_triton:
        triton = run_triton_reference(dev, stream, la, value0, guides, outs[-1], ms_step)

    # ---- end to end through the public module with pinned host buffers
    e2e = None if args.no_e2e else run_e2e(la, host, dev, stream, world, args, mpix_step)

    # ---- whole upsampler throughput (weak scaling: 8 images per GPU)
    ups = None if args.no_upsampler else run_upsampler(dev, stream, world, rank, args, outsize=1022,
                                                       gather=not args.no_gather)
    models = None if args.no_upsampler else run_model_configs(dev, stream, world, rank, args)

    # ---- fp32 attender configurations (standalone K=9 call, SD1.5-VAE levels)
    fp32 = None if args.no_fp32 else run_fp32_configs(dev, stream, peak)
    glue_rl = None if args.no_upsampler else run_glue_rooflines(dev, stream, peak)
    fused_rs = None if args.no_upsampler else run_fused_resize(dev, stream, peak)

    # ---- attender backward (training) on the same four levels
    bwd = None if args.no_backward else run_backward(dev, stream, peak, B_PER_GPU)

    # ---- the reference's own upsampler (make_fast + torch.compile), N=1 only,
    # after every timing of this repository's kernels (its compile sets global
    # TF32 switches; they are restored)
    ref_ups = None
    if world == 1 and not args.no_upsampler and not args.no_ref_upsampler:
        ref_ups = run_reference_upsampler(dev, stream, True)

    # ---- CPU baseline (rank 0, N=1 only): reference algorithm on host cores
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(la, host)

    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seed 0, N(0,1) guides/values, random-init LocalAttender(64,17) in bf16)",
        "config": workload_config(world),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     # every launch of a step is the attender kernel: achieved = mean launch's
                     # algorithmic bytes / mean launch duration; traffic = the mean launch's
                     # ncu DRAM bytes (read + write) against its algorithmic bytes
                     "traffic": None if traffic is None else round(traffic / len(LEVELS)),
                     "algo_bytes_per_launch": round(algo_bytes_step / len(LEVELS)),
                     "traffic_per_step": traffic, "algo_bytes_per_step": algo_bytes_step,
                     "algo_bytes_per_pixel": bpp,
                     "kernel_ms_per_level_eager": [round(x / args.steps, 4) for x in kern_ms],
                     "gbs_per_level_eager": lvl_gbs,
                     "timing": "CUDA graph of the 4 launches" if not args.eager else "eager launches"},
        "e2e": e2e,
        "gpu_launches": len(LEVELS) * args.steps,
        "clocks": clk,
    }
    if triton is not None:
        result["triton_reference"] = triton
    if ups is not None:
        result["upsampler"] = ups
    if models is not None:
        result["upsampler_other_configs"] = models
    if fp32 is not None:
        result["fp32_configs"] = fp32
    if glue_rl is not None:
        result["glue_rooflines"] = glue_rl
    if fused_rs is not None:
        result["fused_resize"] = fused_rs
    if bwd is not None:
        result["backward"] = bwd
    if ref_ups is not None:
        result["reference_upsampler"] = ref_ups
    if cpu is not None:
        result["cpu_baseline"] = cpu
    result["summary"] = summary(result)
    return result


def summary(r):
    """A short last key: the headline figures of the line, so that a
    truncated tail of the output still carries them."""
    def get(*path):
        x = r
        for p in path:
            if not isinstance(x, dict) or p not in x:
                return None
            x = x[p]
        return x
    return {"n": r["n_gpus"], "attender_Mpix_s": r["value"], "frac": get("roofline", "frac"),
            "e2e_Mpix_s": get("e2e", "value"), "e2e_copy_frac": get("e2e", "copy_roofline", "e2e_frac"),
            "triton_ref_Mpix_s": get("triton_reference", "Mpix_s"),
            "cfg5_img_s": get("upsampler", "img_per_s"),
            "cfg5_ref_compiled_img_s": get("reference_upsampler", "img_per_s"),
            "fused_resize_speedup": get("fused_resize", "speedup"),
            "cfg5_img_s_gather": get("upsampler", "gather", "img_per_s"),
            "cfg3_img_s": get("upsampler_other_configs", "dinov3_splus16_512_b32_bf16", "img_per_s"),
            "cfg4_img_s": get("upsampler_other_configs", "sd15_vae_512_b16_fp32", "img_per_s"),
            "bwd_frac": get("backward", "frac_of_peak_chain")}


def run_triton_reference(dev, stream, la, value0, guides, ours_out, ours_ms_step, steps=10):
    """The reference's own GPU path on the same chain, inputs and weights:
    _TritonAttenderWrapper (cuDNN conv1 + residual_auto, uplift/fast.py:46-64)
    around TritonLocalAttender (F.pad replicate copy, cell-tiled kernel for
    H < 48, NHWC streaming kernel + NCHW copy-back otherwise,
    uplift/kernels/triton_attender.py:317-400), unmodified from the
    baseline/_ref install; eager calls as the reference runs them (its
    module is excluded from compilation), CUDA events, after 3 warm-up
    chains (Triton JIT + autotune).  Reports its Mpix/s beside this
    repository's step time, and the normwise difference of the two final
    outputs (both bf16; different rounding points)."""
    import copy
    mods, why = reference_modules("fast", "kernels.triton_attender")
    if not mods:
        return {"unavailable": why}
    fast_mod, ta = mods
    try:
        wrapper = fast_mod._TritonAttenderWrapper(copy.deepcopy(la.conv1), la.conv_res,
                                                  ta.TritonLocalAttender(K_NBR)).to(dev).eval()

        def chain(ev=None):
            v = value0
            for i, g in enumerate(guides):
                if ev is not None:
                    ev[i][0].record(stream)
                v = wrapper(g, v)
                if ev is not None:
                    ev[i][1].record(stream)
            return v

        with torch.inference_mode():
            for _ in range(3):
                out = chain()
            torch.cuda.synchronize(dev)
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(steps):
                out = chain()
            t1.record(stream)
            torch.cuda.synchronize(dev)
            ms = t0.elapsed_time(t1) / steps
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in guides]
            chain(ev)
            torch.cuda.synchronize(dev)
            lvl = [round(a.elapsed_time(b), 4) for a, b in ev]
        ref = out.float()
        err = ((ours_out.float() - ref).abs().max() / ref.abs().max()).item()
    except Exception as e:  # noqa: BLE001 -- reported in the line
        return {"unavailable": f"reference Triton path failed: {type(e).__name__}: {e}"[:300]}
    mpix = out_pixels() / 1e6
    return {"Mpix_s": round(mpix / (ms / 1e3), 1), "ms_per_step": round(ms, 4), "ms_per_level_eager": lvl,
            "ours_ms_per_step": round(ours_ms_step, 4), "speedup_ours": round(ms / ours_ms_step, 2),
            "normwise_diff_vs_ours": round(err, 5),
            "path": "reference _TritonAttenderWrapper + TritonLocalAttender (baseline/_ref, unmodified), "
                    "eager, bf16, same inputs and weights"}


def run_fused_resize(dev, stream, peak, reps=5, images=8):
    """The last attender call of the 1022 px DINOv2 upsampler (B=8, value
    384 x 584^2, guide 64 x 1168^2, bf16) with the final resize to 1022^2:
    the two launches (attender writes 1168^2, the resize kernel reads it back)
    against uplift_la_forward_resized (one launch, the 1168^2 tensor is never
    stored).  CUDA events, median of `reps`.  Algorithmic bytes of the fused
    call: guide + value once + the 1022^2 output."""
    from uplift_b200 import glue, ops
    from uplift_b200.attender import neighbourhood
    K, B, Cv, side = K_NBR, images, C, 584
    offsets, pn = neighbourhood(K)
    g = torch.Generator(device=dev).manual_seed(5)
    cl = torch.channels_last
    guide = torch.randn(B, CG, 2 * side, 2 * side, generator=g, device=dev).to(torch.bfloat16).contiguous(memory_format=cl)
    value = torch.randn(B, Cv, side, side, generator=g, device=dev).to(torch.bfloat16).contiguous(memory_format=cl)
    w = torch.randn(K, CG, generator=g, device=dev) * 0.1
    b = torch.randn(K, generator=g, device=dev) * 0.1

    def timed(fn):
        fn()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    with torch.cuda.stream(stream):  # the fused call first: it is the first attender launch of a capture
        one = timed(lambda: ops.local_attender_resized_raw(guide, value, w, b, offsets, pn, (1022, 1022)))
        two = timed(lambda: glue.resize_bilinear(ops.local_attender_raw(guide, value, w, b, offsets, pn), (1022, 1022)))
    del guide, value
    torch.cuda.empty_cache()
    algo = B * (2 * side) ** 2 * (CG * ELEM + Cv * ELEM / 4) + B * 1022 * 1022 * Cv * ELEM
    return {"two_launches_ms": round(two, 4), "fused_ms": round(one, 4), "speedup": round(two / one, 3),
            "fused_GB_s": round(algo / one / 1e6, 1), "fused_frac_of_peak": round(algo / one / 1e6 / peak, 4),
            "algo_bytes": int(algo),
            "shape": f"B={B}, value 384x584^2 -> attender 1168^2 -> bilinear 1022^2, bf16, K=17"}


def run_glue_rooflines(dev, stream, peak, reps=5):
    """Achieved HBM bandwidth of the fast-mode glue kernels
    (include/uplift_glue.h) at the shapes of the 1022 px DINOv2 upsampler's
    last level (one micro-batch of 8 images, bf16, channels_last): each
    call timed alone with CUDA events (median of `reps` after a warm call;
    every operand is larger than L2).  Algorithmic bytes: every input
    element read once and every output element written once (in-place
    operands count twice)."""
    from uplift_b200 import glue
    cl = torch.channels_last
    bf = torch.bfloat16
    B, S = 8, 1168

    def t(c, h, w=None):
        return torch.randn(B, c, h, w or h, device=dev, dtype=bf).contiguous(memory_format=cl)

    def timed(fn):
        fn()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    out = {}
    with torch.cuda.stream(stream):
        y, r = t(64, S), t(64, S)
        bias = torch.randn(64, device=dev, dtype=bf)
        ms = timed(lambda: glue.bias_act_(y, bias, True, r))
        out["bias_act_relu_res_64ch_1168"] = (ms, 3 * y.numel() * 2)
        x = t(64, S // 2)
        ms = timed(lambda: glue.upsample_add_(y, x, align_corners=True))
        out["upsample_add_64ch_584to1168"] = (ms, (2 * y.numel() + x.numel()) * 2)
        del x, r
        buf = torch.empty(B, 192, S // 2, S // 2, device=dev, dtype=bf, memory_format=cl)
        skip = t(128, S)
        ms = timed(lambda: glue.nearest_into_(buf[:, 64:], skip))
        out["nearest_into_128ch_1168to584"] = (ms, 2 * B * 128 * (S // 2) ** 2 * 2)
        del buf, skip, y
        a = t(384, S)
        ms = timed(lambda: glue.resize_bilinear(a, (1022, 1022)))
        out["bilinear_384ch_1168to1022"] = (ms, (a.numel() + B * 384 * 1022 * 1022) * 2)
        del a
    torch.cuda.empty_cache()
    return {k: {"ms": round(ms, 4), "GB_s": round(b / ms / 1e6, 1), "frac_of_peak": round(b / ms / 1e6 / peak, 4)}
            for k, (ms, b) in out.items()} | {
        "note": "B=8, bf16, channels_last; single calls, median of 5; algorithmic bytes; "
                "frac against the measured HBM copy peak"}


def run_fp32_configs(dev, stream, peak, reps=20):
    """Device time of the fp32 attender configurations, each call replayed
    `reps` times in a CUDA graph: the standalone call (K=9, value 384x32^2,
    guide 64x64^2, one image; latency-bound, 8.9 MB) and the two attender
    levels of the SD1.5-VAE upsampler (K=17, Cg=512, C=4, B=16; value 64^2
    -> 128^2 and 128^2 -> 256^2).  Algorithmic bytes per output pixel:
    Cg*4 + C*4 + C*4/4.  Random-init LocalAttender in fp32, N(0,1) inputs."""
    from uplift_b200 import _native
    from uplift_b200.attender import LocalAttender

    cases = [("standalone_k9_b1_32to64", 1, 64, 384, 32, 9),
             ("sdvae_k17_b16_64to128", 16, 512, 4, 64, 17),
             ("sdvae_k17_b16_128to256", 16, 512, 4, 128, 17)]
    kernel_names = {_native.KERNEL_SIMT: "la_fwd_kernel", _native.KERNEL_SIMT_STAGED: "la_fwd_staged_kernel",
                    _native.KERNEL_TENSOR_CORE: "la_tc_kernel", _native.KERNEL_TENSOR_CORE_WIDE: "la_tcw_kernel"}
    out = {}
    g = torch.Generator().manual_seed(0)
    side = torch.cuda.Stream(dev)  # graphs are captured off the default stream
    side.wait_stream(stream)
    stream = side
    for name, b, cg, c, h, k in cases:
        torch.manual_seed(0)
        la = LocalAttender(cg, k).to(dev)
        guide = torch.randn(b, cg, 2 * h, 2 * h, generator=g).to(dev).contiguous(memory_format=torch.channels_last)
        value = torch.randn(b, c, h, h, generator=g).to(dev).contiguous(memory_format=torch.channels_last)
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(3):
                la(guide, value)
            kern = _native.last_kernel()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(reps):
                    la(guide, value)
            for _ in range(5):  # warm replays (graph upload, clocks)
                graph.replay()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            times = []
            for _ in range(5):
                ev[0].record(stream)
                graph.replay()
                ev[1].record(stream)
                ev[1].synchronize()
                times.append(ev[0].elapsed_time(ev[1]) / reps)
        del graph
        us = statistics.median(times) * 1e3
        px = b * 4 * h * h
        bpp = cg * 4 + c * 4 + c * 4 / 4
        gbs = px * bpp / (us * 1e-6) / 1e9
        out[name] = {"kernel": kernel_names.get(kern, str(kern)), "us_per_call": round(us, 2),
                     "Mpix_s": round(px / us, 1), "GB_s": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4)}
    out["note"] = ("fp32 storage; CUDA-graph replays of one call, median of 5; bytes = algorithmic "
                   "(guide + output + value once); frac against the measured HBM copy peak")
    return out


def run_backward(dev, stream, peak, images, reps=5):
    """Device time of the attender backward (training; uplift_la_backward:
    dguide, dvalue, dweight, dbias) on the four levels of the chain above,
    bf16, `images` per GPU, random-init LocalAttender(64, 17), N(0,1) guide /
    value / output gradient.  Each level's call (output allocation, the
    zeroing of dW / db and every kernel) is captured in a CUDA graph and
    replayed `reps` times with an L2 flush before each replay (median);
    `ms_eager` is one eager call from the host, median of `reps` (it adds
    the Python wrapper's launch latency).  Algorithmic bytes per output
    pixel: dout + guide read, dguide written ((C + 2 Cg) * 2), the fp32
    softmax workspace written by the dlogit kernel and read once by the dV
    kernel (8 K), value read and dvalue written once per value pixel
    (2 C * 2 / 4); dout's second read (by the dV kernel) is not counted."""
    from uplift_b200 import ops
    from uplift_b200.attender import LocalAttender, neighbourhood

    offsets, pn = neighbourhood(K_NBR)
    torch.manual_seed(0)
    la = LocalAttender(CG, K_NBR).to(dev)
    w = la.conv1.weight.detach().reshape(K_NBR, CG).float()
    b = la.conv1.bias.detach().float()
    g = torch.Generator().manual_seed(0)
    cl = torch.channels_last
    bpp = (C + 2 * CG) * ELEM + 8 * K_NBR + 2 * C * ELEM / 4
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    cap = torch.cuda.Stream(dev)  # graphs are captured off the default stream
    levels, tot_ms, tot_px, tot_eager = [], 0.0, 0, 0.0

    def timed_once(fn):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record(stream)
        fn()
        ev[1].record(stream)
        ev[1].synchronize()
        return ev[0].elapsed_time(ev[1])

    with torch.cuda.stream(stream):
        for co, fo in LEVELS:
            guide = torch.randn(images, CG, fo, fo, generator=g).to(torch.bfloat16).to(dev).contiguous(memory_format=cl)
            value = torch.randn(images, C, co, co, generator=g).to(torch.bfloat16).to(dev).contiguous(memory_format=cl)
            dout = torch.randn(images, C, fo, fo, generator=g).to(torch.bfloat16).to(dev).contiguous(memory_format=cl)

            def call():
                return ops.local_attender_backward_raw(dout, guide, value, w, b, offsets, pn)

            for _ in range(2):
                call()
            eager = []
            for _ in range(reps):
                flush.zero_()
                eager.append(timed_once(call))
            graph = torch.cuda.CUDAGraph()
            cap.wait_stream(stream)
            with torch.cuda.graph(graph, stream=cap):
                outs = call()
            stream.wait_stream(cap)
            graph.replay()
            times = []
            for _ in range(reps):
                flush.zero_()
                times.append(timed_once(graph.replay))
            del graph, outs
            ms = statistics.median(times)
            px = images * fo * fo
            tot_ms += ms
            tot_eager += statistics.median(eager)
            tot_px += px
            levels.append({"level": f"{co}^2->{fo}^2", "ms": round(ms, 4), "ms_eager": round(statistics.median(eager), 4),
                           "Mpix_s": round(px / ms / 1e3, 1), "GB_s": round(px * bpp / ms / 1e6, 1)})
            del guide, value, dout
    del flush
    return {"levels": levels, "ms_chain": round(tot_ms, 4), "ms_chain_eager": round(tot_eager, 4),
            "Mpix_s_chain": round(tot_px / tot_ms / 1e3, 1),
            "frac_of_peak_chain": round(tot_px * bpp / tot_ms / 1e6 / peak, 4), "algo_bytes_per_pixel": bpp,
            "launches_per_level": 2, "dtype": "bf16", "images": images,
            "note": "tensor-core dlogit + tensor-core dV kernels (and the zeroing of dW / db); CUDA-graph "
                    "replay of each level's call, L2 flushed before each, median of 5; frac against the measured "
                    "HBM copy peak"}


def run_e2e(la, host, dev, stream, world, args, mpix_step):
    """The same metric through LocalAttender.forward with pinned host buffers:
    every step copies the level-0 features and the four guides host->device,
    runs the four attender calls and copies the final output device->host,
    all inside the timed region.  As a serving pipeline would, three streams
    overlap step i+1's input copy and step i-1's output copy with step i's
    compute (two slots of device inputs and pinned host outputs; events order
    the slots).  The timed region spans the first input copy to the last
    output copy."""
    # pinned host buffers on the GPU's NUMA node (pages are placed when they
    # are pinned, by the pinning thread)
    with numa_local(dev) as numa:
        h_v0 = host["value0"].pin_memory()
        h_guides = [x.pin_memory() for x in host["guides"]]
        h_outs = [torch.empty((B_PER_GPU, C, LEVELS[-1][1], LEVELS[-1][1]), dtype=torch.bfloat16,
                              memory_format=torch.channels_last).pin_memory() for _ in range(2)]
    h2d = h_v0.numel() * 2 + sum(x.numel() * 2 for x in h_guides)
    d2h = h_outs[0].numel() * 2
    d_v0 = [torch.empty_like(h_v0, device=dev) for _ in range(2)]
    d_guides = [[torch.empty_like(g, device=dev) for g in h_guides] for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_comp = stream
    in_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    started = [False, False]

    def e2e_step(i):
        slot = i & 1
        with torch.cuda.stream(s_in):
            if started[slot]:
                s_in.wait_event(comp_done[slot])  # step i-2 finished reading this slot's inputs
            d_v0[slot].copy_(h_v0, non_blocking=True)
            for d, h in zip(d_guides[slot], h_guides):
                d.copy_(h, non_blocking=True)
            in_done[slot].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_done[slot])
            v = d_v0[slot]
            for g in d_guides[slot]:
                v = la(g, v)
            comp_done[slot].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[slot])
            if started[slot]:
                s_out.wait_event(out_done[slot])
            h_outs[slot].copy_(v, non_blocking=True)
            v.record_stream(s_out)
            out_done[slot].record(s_out)
        started[slot] = True

    with torch.inference_mode():
        for i in range(max(2, min(args.warmup, 3))):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        e_steps = max(2, min(args.steps, 10))
        barrier(world)
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s_in)
        for i in range(e_steps):
            e2e_step(i)
        e1.record(s_out)
        torch.cuda.synchronize(dev)
        barrier(world)
    e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / e_steps
    value = world * mpix_step / (e_ms / 1e3)
    bound = copy_bound(dev, h_v0, h_guides, h_outs[0], world)
    bound_mpix = world * mpix_step / (bound["both_ms"] / 1e3)
    bound.update({"Mpix_s": round(bound_mpix, 2), "e2e_frac": round(value / bound_mpix, 4), "numa": numa})
    return {"value": round(value, 2), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms, 3),
            "api": "uplift_b200.LocalAttender.forward, pinned host buffers",
            "pipelining": "H2D of step i+1 and D2H of step i-1 overlap step i's compute (3 streams, 2 slots)",
            "copy_roofline": bound}


class numa_local:
    """Run a block with the calling thread bound to the CPUs of the GPU's
    NUMA node (from sysfs), so that host memory pinned inside it is placed
    on that node; the previous affinity is restored after.  Yields a short
    description (None when sysfs has no answer)."""

    def __init__(self, dev):
        self.dev = dev
        self.old = None

    def __enter__(self):
        try:
            props = torch.cuda.get_device_properties(self.dev)
            bdf = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            p = Path("/sys/bus/pci/devices") / bdf
            node = int((p / "numa_node").read_text().strip())
            cpus = set()
            for part in (p / "local_cpulist").read_text().strip().split(","):
                a, _, b = part.partition("-")
                cpus.update(range(int(a), int(b or a) + 1))
            cpus &= os.sched_getaffinity(0)
            if not cpus:
                return None
            self.old = os.sched_getaffinity(0)
            os.sched_setaffinity(0, cpus)
            return {"node": node, "cpus": len(cpus), "pci": bdf}
        except (AttributeError, OSError, ValueError, RuntimeError):
            return None

    def __exit__(self, *exc):
        if self.old is not None:
            os.sched_setaffinity(0, self.old)
        return False


def copy_bound(dev, h_v0, h_guides, h_out, world, reps=5):
    """The e2e pipeline's copy roofline: the same pinned host buffers copied
    host->device (level-0 features + four guides) and device->host (final
    output) with nothing else running, both directions at once on two
    streams as the pipeline overlaps them, on every rank at the same time;
    median of `reps`, max over ranks.  Also each direction alone."""
    d_in = [torch.empty_like(h_v0, device=dev)] + [torch.empty_like(x, device=dev) for x in h_guides]
    d_out = torch.empty_like(h_out, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)

    def once(do_in, do_out):
        start, e_in, e_out = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        start.record(cur)
        if do_in:
            s_in.wait_event(start)
            with torch.cuda.stream(s_in):
                for d, h in zip(d_in, [h_v0] + list(h_guides)):
                    d.copy_(h, non_blocking=True)
            e_in.record(s_in)
            cur.wait_event(e_in)
        if do_out:
            s_out.wait_event(start)
            with torch.cuda.stream(s_out):
                h_out.copy_(d_out, non_blocking=True)
            e_out.record(s_out)
            cur.wait_event(e_out)
        end = torch.cuda.Event(enable_timing=True)
        end.record(cur)
        end.synchronize()
        return start.elapsed_time(end)

    res = {}
    for name, a, b in (("both", True, True), ("h2d", True, False), ("d2h", False, True)):
        once(a, b)
        barrier(world)
        ms = statistics.median(once(a, b) for _ in range(reps))
        res[name + "_ms"] = round(max_over_ranks(ms, world, dev), 3)
    h2d = sum(x.numel() * x.element_size() for x in [h_v0] + list(h_guides))
    d2h = h_out.numel() * h_out.element_size()
    res["h2d_GB_s"] = round(h2d / res["h2d_ms"] / 1e6, 1)
    res["d2h_GB_s"] = round(d2h / res["d2h_ms"] / 1e6, 1)
    return res


def run_upsampler(dev, stream, world, rank, args, variant="dinov2-s14", img_px=1022, feat_px=73, iters=4,
                  global_images=64, micro_batch=8, dtype=torch.bfloat16, outsize=None, img_range=(0.0, 1.0),
                  gather=False, gather_micro_batch=2, min_ms=400.0):
    """Whole-upsampler throughput, batch-sharded: the `variant`-shaped UPLiFT
    (random init, eval, channels_last) on images img_px^2 in `img_range`
    with backbone features C x feat_px^2 (N(0,1)), iters, final resize to
    `outsize` (None: none); a global batch of `global_images` split into
    contiguous shards, one per rank, each run in micro-batches of
    `micro_batch` images.  Convolutions are cuDNN, the glue between them and
    the attender are this package's kernels.  Inputs are resident on the
    device (synthetic, seed 1000 + rank).

    Each micro-batch forward is captured once in a CUDA graph and replayed
    (the eager figure, with per-launch host overhead, is reported beside it);
    a pass = every micro-batch of the rank's shard, timed over enough passes
    to last `min_ms`; img/s = global images / max-over-ranks time.

    `gather` (N > 1): a second timing in which every output also travels to
    rank 0 into one preallocated [global, C, H, W] tensor held by rank 0
    only, micro-batch by micro-batch so that the transfer of one overlaps the
    forward of the next (two graph slots; a slot is replayed again only after
    its transfer has read it).  By default the transfers are copy-engine
    copies out of CUDA IPC mappings of the peers' slots (run_gather_ipc,
    micro-batches of the forward's size); --gather-nccl uses NCCL's
    dist.gather in `gather_micro_batch`-image pieces instead (run_gather)."""
    from uplift_b200.configs import get_config
    from uplift_b200.sharding import shard_bounds
    from uplift_b200.uplift import UPLiFT
    from uplift_b200.fast import make_fast
    cfg = get_config(variant)
    torch.manual_seed(0)
    model = UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, dtype=dtype).eval()
    model.enable_iterative(iters)
    # the reference's fast-mode recipe for the convolutions (BatchNorm folded,
    # channels_last), without torch.compile; cuDNN picks its algorithms
    torch.backends.cudnn.benchmark = True
    fast = make_fast(model, compile=False, device=dev)
    lo, hi = shard_bounds(global_images, rank, world)
    g = torch.Generator().manual_seed(1000 + rank)
    mine = hi - lo
    mb = min(micro_batch, max(mine, 1))
    a, b = img_range
    img = (torch.rand(mb, 3, img_px, img_px, generator=g) * (b - a) + a).to(dtype).to(dev)
    feats = torch.randn(mb, cfg.backbone.channel, feat_px, feat_px, generator=g).to(dtype).to(dev)
    img = img.contiguous(memory_format=torch.channels_last)
    feats = feats.contiguous(memory_format=torch.channels_last)
    size = None if outsize is None else [outsize, outsize]
    n_mb = (mine + mb - 1) // mb

    def timed(fn, passes):
        barrier(world)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(passes):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        return max_over_ranks(e0.elapsed_time(e1), world, dev) / passes

    def passes_for(ms_one):  # enough passes for ~min_ms (same count on every rank)
        return int(max(2, min(50, -(-min_ms // max(ms_one, 1e-3)))))

    with torch.inference_mode():
        # eager: warm-up (cuDNN algorithm selection), then timed
        out = fast(img, feats, size)
        torch.cuda.synchronize(dev)

        def eager_pass():
            for _ in range(n_mb):
                fast(img, feats, size)
        ms_eager = timed(eager_pass, 1)
        ms_eager = timed(eager_pass, passes_for(ms_eager))

        # CUDA graph of one micro-batch forward, replayed per micro-batch
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fast(img, feats, size)
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_out = fast(img, feats, size)
        graph.replay()
        torch.cuda.synchronize(dev)

        def graph_pass():
            for _ in range(n_mb):
                graph.replay()
        ms = timed(graph_pass, 1)
        passes = passes_for(ms)
        ms = timed(graph_pass, passes)
        assert static_out.shape[1] == cfg.backbone.channel
        out_shape = tuple(static_out.shape[1:])
        del graph, static_out, out

        gat = None
        if gather and world > 1:
            nccl = getattr(args, "gather_nccl", False)
            gather_micro_batch = getattr(args, "gather_mb", 0) or (gather_micro_batch if nccl else mb)
            if not nccl:
                gat = run_gather_ipc(fast, dev, stream, world, rank, global_images, mine, lo, img, feats, size,
                                     dtype, out_shape, min(gather_micro_batch, mb), timed, passes_for)
            else:
                gat = run_gather(fast, dev, stream, world, rank, global_images, mine, lo, img, feats, size,
                                 dtype, out_shape, min(max(gather_micro_batch, getattr(args, "gather_groups", 1)), mb),
                                 timed, passes_for, getattr(args, "gather_ctas", 0), getattr(args, "gather_groups", 1))
    del fast, model, img, feats
    torch.cuda.empty_cache()
    dt = {torch.bfloat16: "bf16", torch.float32: "fp32"}[dtype]
    shape = f"{outsize}^2 output" if outsize else "no final resize"
    res = {"img_per_s": round(global_images / (ms / 1e3), 2), "ms_per_global_batch": round(ms, 2),
           "img_per_s_eager": round(global_images / (ms_eager / 1e3), 2),
           "global_images": global_images, "images_per_gpu": mine, "micro_batch": mb, "passes": passes,
           "scaling": "strong", "timing": "CUDA-graph replay per micro-batch (eager beside it)",
           "config": f"UPLiFT {variant}, random init, {dt}, img {img_px}^2, feats "
                     f"{cfg.backbone.channel}x{feat_px}^2, iters={iters}, {shape}; make_fast(compile=False)"}
    if gat is not None:
        res["gather"] = gat
    return res


def run_gather(fast, dev, stream, world, rank, global_images, mine, lo, img, feats, size, dtype, out_shape,
               gmb, timed, passes_for, gather_ctas=0, gather_groups=1):
    """Upsampler timing with the final gather of every output to rank 0 (see
    run_upsampler).  Shards are equal (global batch divisible by the world
    size), so every rank issues the same gathers in the same order.

    gather_ctas > 0: the gathers run on their own NCCL communicator capped at
    that many CTAs, and this package's persistent kernels leave as many SMs
    to them (uplift_la_set_max_ctas, set before the graphs are captured: the
    grid is part of them), so that the transfer and the forward share the
    GPU instead of queueing for SMs."""
    import torch.distributed as dist
    from uplift_b200 import _native
    from uplift_b200.sharding import shard_bounds
    C, H, W = out_shape
    bounds = [shard_bounds(global_images, r, world) for r in range(world)]
    if len({hi - lo_ for lo_, hi in bounds}) != 1 or mine % gmb != 0:
        return {"skipped": "unequal shards"}
    # one communicator per concurrent gather: each image of a micro-batch is
    # gathered on its own (round-robin over the groups), so up to
    # gather_groups transfers run at once on separate NCCL streams
    groups = [None]
    if gather_ctas > 0 or gather_groups > 1:
        groups = []
        for _ in range(max(1, gather_groups)):
            opts = dist.ProcessGroupNCCL.Options()
            if gather_ctas > 0:
                opts.config.max_ctas = gather_ctas
            groups.append(dist.new_group(backend="nccl", pg_options=opts))
    if gather_ctas > 0:
        _native.set_max_ctas(max(1, torch.cuda.get_device_properties(dev).multi_processor_count - gather_ctas))
    try:
        full = None
        if rank == 0:
            full = torch.empty((global_images, C, H, W), dtype=dtype, device=dev, memory_format=torch.channels_last)
        n_mb = mine // gmb
        x_img, x_feats = img[:gmb], feats[:gmb]
        pool = torch.cuda.graph_pool_handle()
        graphs, outs = [], []
        for _ in range(2):  # two slots: one is gathered while the other is computed
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                fast(x_img, x_feats, size)
            stream.wait_stream(side)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, pool=pool):
                outs.append(fast(x_img, x_feats, size))
            graphs.append(gr)
        torch.cuda.synchronize(dev)

        def nhwc(t):  # a contiguous view of a channels_last tensor, as NCCL wants it
            return t.permute(0, 2, 3, 1)

        def gather_pass():
            pending = [[], []]
            for j in range(n_mb):
                sl = j & 1
                for w in pending[sl]:
                    w.wait()  # the stream waits until that gather has read the slot
                pending[sl] = []
                graphs[sl].replay()
                per = gmb if len(groups) == 1 else 1
                for i0 in range(0, gmb, per):
                    parts = None
                    if rank == 0:
                        parts = [nhwc(full[lo_ + j * gmb + i0: lo_ + j * gmb + i0 + per]) for lo_, _ in bounds]
                    pending[sl].append(dist.gather(nhwc(outs[sl][i0:i0 + per]), gather_list=parts, dst=0,
                                                   group=groups[(i0 // per) % len(groups)], async_op=True))
            for ws in pending:
                for w in ws:
                    w.wait()
        ms = timed(gather_pass, 1)
        passes = passes_for(ms)
        ms = timed(gather_pass, passes)
        del graphs, outs, full
    finally:
        if gather_ctas > 0:
            _native.set_max_ctas(0)
    elem = 2 if dtype != torch.float32 else 4
    into_root = (world - 1) * mine * C * H * W * elem
    return {"img_per_s": round(global_images / (ms / 1e3), 2), "ms_per_global_batch": round(ms, 2),
            "passes": passes, "gather_micro_batch": gmb,
            "gather_ctas": gather_ctas or "NCCL default (attender on every SM)",
            "gather_groups": len(groups),
            "bytes_into_rank0_per_batch": into_root,
            "rank0_ingress_GB_s": round(into_root / (ms / 1e3) / 1e9, 1),
            "how": "NCCL gather per micro-batch into rank 0's [global, C, H, W] tensor, overlapping the next "
                   "micro-batch's forward (2 CUDA-graph slots); only rank 0 holds the full batch"}


def run_gather_ipc(fast, dev, stream, world, rank, global_images, mine, lo, img, feats, size, dtype, out_shape,
                   gmb, timed, passes_for):
    """The gather of run_gather on the copy engines instead of NCCL
    (uplift_b200.sharding.SlotGather): rank 0 maps every peer's two output
    slots (the outputs of the two graphs) through CUDA IPC and copies each
    micro-batch into its [global, C, H, W] tensor with cudaMemcpyAsync, one
    stream per peer, while the ranks compute the next micro-batch; ordered
    by interprocess events and TCPStore keys."""
    import datetime
    import torch.distributed as dist
    from uplift_b200.sharding import SlotGather, shard_bounds
    C, H, W = out_shape
    bounds = [shard_bounds(global_images, r, world) for r in range(world)]
    if len({hi - lo_ for lo_, hi in bounds}) != 1 or mine % gmb != 0:
        return {"skipped": "unequal shards"}
    # the process group's own rendezvous store (no second port to open),
    # under a prefix of this gather's own; a new TCPStore only without one
    try:
        from torch.distributed.distributed_c10d import _get_default_store
        store = dist.PrefixStore("slotgather/", _get_default_store())
    except Exception:  # noqa: BLE001 -- no default store: open one beside the rendezvous port
        port = int(os.environ.get("MASTER_PORT", "29500")) + 11
        store = dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"), port, world, rank == 0)
    store.set_timeout(datetime.timedelta(seconds=60))
    full = None
    if rank == 0:
        full = torch.empty((global_images, C, H, W), dtype=dtype, device=dev, memory_format=torch.channels_last)
    n_mb = mine // gmb
    x_img, x_feats = img[:gmb], feats[:gmb]
    pool = torch.cuda.graph_pool_handle()
    graphs, outs = [], []
    for _ in range(2):
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fast(x_img, x_feats, size)
        stream.wait_stream(side)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, pool=pool):
            outs.append(fast(x_img, x_feats, size))
        graphs.append(gr)
    torch.cuda.synchronize(dev)
    torch.cuda.set_device(dev)
    sg = SlotGather(outs, full, [b[0] for b in bounds], store, rank, world, stream)
    counter = [0]  # micro-batches so far, across passes

    def gather_pass():
        for i in range(n_mb):
            j = counter[0]
            counter[0] += 1
            sg.before_write(j)
            graphs[j % 2].replay()
            sg.after_write(j, i)
        sg.join()
    ok = True
    try:
        ms = timed(gather_pass, 1)
        passes = passes_for(ms)
        ms = timed(gather_pass, passes)
        # check: every rank's last micro-batch, as copied, against an NCCL
        # gather of the same slot
        last = (counter[0] - 1) % 2
        parts = [torch.empty_like(outs[last]) for _ in range(world)] if rank == 0 else None
        dist.gather(outs[last].permute(0, 2, 3, 1), gather_list=None if parts is None else
                    [t.permute(0, 2, 3, 1) for t in parts], dst=0)
        if rank == 0:
            for r in range(world):
                lo_r = bounds[r][0]
                ok &= bool(torch.equal(full[lo_r + (n_mb - 1) * gmb: lo_r + n_mb * gmb], parts[r]))
    finally:
        torch.cuda.synchronize(dev)
        barrier(world)
        sg.close()
        torch.cuda.synchronize(dev)
        barrier(world)  # rank 0 has unmapped the peers' slots before they are freed
    del graphs, outs, full, sg
    elem = 2 if dtype != torch.float32 else 4
    into_root = (world - 1) * mine * C * H * W * elem
    return {"img_per_s": round(global_images / (ms / 1e3), 2), "ms_per_global_batch": round(ms, 2),
            "passes": passes, "gather_micro_batch": gmb,
            "bytes_into_rank0_per_batch": into_root,
            "rank0_ingress_GB_s": round(into_root / (ms / 1e3) / 1e9, 1),
            "last_micro_batch_equals_nccl_gather": ok,
            "how": "uplift_b200.sharding.SlotGather: rank 0 copies each peer's micro-batch output out of its CUDA "
                   "IPC mapping (cudaMemcpyAsync, one stream per peer), ordered by interprocess events, overlapping "
                   "the next micro-batch's forward; only rank 0 holds the full batch"}


def run_reference_upsampler(dev, stream, compile_model, images=16, micro_batch=8, min_ms=400.0):
    """The reference's own upsampler on the 1022 px DINOv2 configuration
    (config 5: image 1022^2, features 384 x 73^2, iters=4, output 1022^2,
    bf16): its UPLiFT (uplift/uplift.py:538-) built from its shipped
    uplift_dinov2-s14.yaml with random init, wrapped by its make_fast
    (uplift/fast.py:71-133: BatchNorm folding, channels_last, the Triton
    attender, and with `compile_model` torch.compile in its default
    max-autotune mode), unmodified from the baseline/_ref install.  One GPU,
    micro-batches of `micro_batch` images resident on the device; the first
    call (compilation and autotuning) is timed on its own, then passes of
    `images` images are timed with CUDA events for ~`min_ms`.  make_fast
    turns TF32 on globally when it compiles (uplift/fast.py:122-124); the
    previous settings are restored after."""
    import time
    from types import SimpleNamespace
    import yaml
    mods, why = reference_modules("uplift", "fast")
    if not mods:
        return {"unavailable": why}
    up, fastmod = mods

    def ns(d):
        if isinstance(d, dict):
            return SimpleNamespace(**{k: ns(v) for k, v in d.items()})
        if isinstance(d, list):
            return [ns(v) for v in d]
        return d

    cfg = ns(yaml.safe_load(open(REF_ROOT / "uplift" / "configs" / "uplift_dinov2-s14.yaml")))
    tf32 = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    try:
        torch.manual_seed(0)
        model = up.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, dtype=torch.bfloat16).eval()
        model.enable_iterative(4)
        fast = fastmod.make_fast(model, compile=compile_model, warmup=False, device=dev)
        g = torch.Generator().manual_seed(1000)
        img = torch.rand(micro_batch, 3, 1022, 1022, generator=g).to(torch.bfloat16).to(dev)
        feats = torch.randn(micro_batch, cfg.backbone.channel, 73, 73, generator=g).to(torch.bfloat16).to(dev)
        img = img.contiguous(memory_format=torch.channels_last)
        feats = feats.contiguous(memory_format=torch.channels_last)
        n_mb = -(-images // micro_batch)
        with torch.cuda.stream(stream):
            t0 = time.time()
            fast(img, feats, [1022, 1022])
            torch.cuda.synchronize(dev)
            first_s = time.time() - t0
            for _ in range(2):
                fast(img, feats, [1022, 1022])

            def one_pass():
                for _ in range(n_mb):
                    fast(img, feats, [1022, 1022])

            def timed(passes):
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(passes):
                    one_pass()
                e1.record(stream)
                torch.cuda.synchronize(dev)
                return e0.elapsed_time(e1) / passes

            ms = timed(1)
            passes = int(max(2, min(20, -(-min_ms // max(ms, 1e-3)))))
            ms = timed(passes)
    except Exception as e:  # noqa: BLE001 -- reported, not raised: the bench line still prints
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = tf32
    return {"img_per_s": round(n_mb * micro_batch / (ms / 1e3), 2), "ms_per_pass": round(ms, 2),
            "images_per_pass": n_mb * micro_batch, "micro_batch": micro_batch, "passes": passes,
            "first_call_s": round(first_s, 1),
            "path": "reference UPLiFT + make_fast(compile=%s%s) from baseline/_ref, unmodified, bf16, "
                    "random init, eager CUDA-event timing of passes" % (compile_model,
                                                                        ", mode max-autotune" if compile_model else "")}


def run_model_configs(dev, stream, world, rank, args):
    """The other two model configurations, whole upsampler, batch-sharded:
    DINOv3-S+/16 at 512 px (features 384 x 32^2, iters=4, outsize 512,
    bf16, global batch 32; low_mem=True runs the same fused kernel, so one
    line covers both settings) and SD1.5-VAE at 512 px (latent 4 x 64^2,
    iters=2 -> 256^2, fp32, global batch 16)."""
    return {
        "dinov3_splus16_512_b32_bf16": run_upsampler(
            dev, stream, world, rank, args, variant="dinov3-splus16", img_px=512, feat_px=32, iters=4,
            global_images=32, micro_batch=16, dtype=torch.bfloat16, outsize=512),
        "sd15_vae_512_b16_fp32": run_upsampler(
            dev, stream, world, rank, args, variant="sd15-vae", img_px=512, feat_px=64, iters=2,
            global_images=16, micro_batch=8, dtype=torch.float32, outsize=None, img_range=(-1.0, 1.0)),
    }


def cpu_sample_inputs(host, seed=1):
    """Per level: the guide and a value map of one image (level 0: the real
    level-0 features; deeper levels: synthetic N(0,1) maps of the shape the
    chain would feed them)."""
    g = torch.Generator().manual_seed(seed)
    vals = [host["value0"][:1].contiguous()]
    for c, _ in LEVELS[1:]:
        vals.append(torch.randn(1, C, c, c, generator=g).to(torch.bfloat16))
    return [(host["guides"][i][:1].contiguous(), vals[i]) for i in range(len(LEVELS))]


def reference_attender(la):
    """The reference's own LocalAttender (uplift/uplift.py:740-847, from the
    baseline/_ref install) carrying the weights of `la`, in bf16; (None,
    reason) when the install is absent."""
    mods, why = reference_modules("uplift")
    if not mods:
        return None, why
    ref = mods[0].LocalAttender(CG, K_NBR).to(torch.bfloat16).eval()
    with torch.no_grad():
        ref.conv1.weight.copy_(la.conv1.weight.detach().cpu())
        ref.conv1.bias.copy_(la.conv1.bias.detach().cpu())
    return ref, None


def cpu_band_step(la, inputs, band, ref=None):
    """Band `band` of 8 horizontal bands of every level of one image through
    the CPU implementation of the path: the reference's own LocalAttender
    when `ref` is given, else the oracle's restatement of it (torch CPU ops,
    same op order, parallel pooling, bf16).  Each band is computed with its
    +-pn halo rows, so its output equals the whole-image result.  Returns the
    output pixels produced."""
    from oracle import local_attender_oracle as lao
    w = la.conv1.weight.detach().cpu().reshape(K_NBR, CG)
    b = la.conv1.bias.detach().cpu()
    pn = la.pn
    pix = 0
    with torch.inference_mode():
        for (guide, value) in inputs:
            H = value.shape[2]
            h0, h1 = band * H // 8, (band + 1) * H // 8
            lo, hi = max(0, h0 - pn), min(H, h1 + pn)
            g, v = guide[:, :, 2 * lo:2 * hi], value[:, :, lo:hi]
            if ref is not None:
                ref(g, v)
            else:
                lao.local_attender(g, v, w, b, K=K_NBR)
            pix += 2 * (h1 - h0) * guide.shape[3]
    return pix


def cpu_impl(la):
    """(reference module or None, kind, description) of the CPU path timed."""
    ref, why = reference_attender(la)
    if ref is not None:
        return ref, "reference", "the reference's LocalAttender.forward (uplift/uplift.py:801-847, parallel pooling)"
    return None, "port", f"oracle restatement of the reference (torch CPU ops; {why})"


def cpu_baseline(la, host, min_seconds=10.0):
    """Rank 0, N=1: bands 0..7 (= one whole image of the 4-level chain),
    repeated until about `min_seconds` of CPU work, all host threads."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ref, kind, what = cpu_impl(la)
    inputs = cpu_sample_inputs(host)
    cpu_band_step(la, inputs, 4, ref)  # warm-up
    t = time.perf_counter()
    pix, n = 0, 0
    while True:
        pix += cpu_band_step(la, inputs, n % 8, ref)
        n += 1
        sec = time.perf_counter() - t
        if n >= 8 and sec >= min_seconds:
            break
    return {"value": round(pix / 1e6 / sec, 4), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{n} bands of 1/8 image rows x 4 attender levels (= {n / 8:.2f} images of the "
                      f"448px iters=4 chain, {pix} output px) in {sec:.1f} s; {what}, bf16"}


def run_reference(args, world, rank):
    """The reference's CPU implementation of the path, rank 0 only: each step
    = one 1/8-row band of one image through the 4 attender levels (bands
    cycle through the image)."""
    if rank != 0:
        return None
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    la, host = make_inputs(torch.device("cpu"), seed=0)
    ref, kind, what = cpu_impl(la)
    inputs = cpu_sample_inputs(host)
    for i in range(min(args.warmup, 2)):
        cpu_band_step(la, inputs, i % 8, ref)
    pix = 0
    t = time.perf_counter()
    for i in range(args.steps):
        pix += cpu_band_step(la, inputs, i % 8, ref)
    sec = time.perf_counter() - t
    value = pix / 1e6 / sec
    sample = (f"per step 1/8 of the rows of one image through the 4 attender levels "
              f"({pix // max(args.steps, 1)} output px avg); {what}, bf16")
    return {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(sec * 1e3 / max(args.steps, 1), 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(world),
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    global B_PER_GPU
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end pass")
    ap.add_argument("--eager", action="store_true", help="time plain launches instead of a CUDA graph")
    ap.add_argument("--no-upsampler", action="store_true", help="skip the whole-upsampler img/s pass")
    ap.add_argument("--no-fp32", action="store_true", help="skip the fp32 attender configurations")
    ap.add_argument("--only-fp32", action="store_true",
                    help="run only the fp32 attender configurations (profiling captures)")
    ap.add_argument("--no-backward", action="store_true", help="skip the attender backward pass")
    ap.add_argument("--no-triton", action="store_true", help="skip timing the reference's Triton path")
    ap.add_argument("--no-gather", action="store_true", help="skip the upsampler timing with the gather to rank 0")
    ap.add_argument("--only-backward", action="store_true",
                    help="run only the attender backward pass (profiling captures)")
    ap.add_argument("--only-upsampler", action="store_true",
                    help="run only the whole-upsampler pass (profiling captures)")
    ap.add_argument("--only-fused-resize", action="store_true",
                    help="run only the fused attender + final resize timing (profiling captures; --images)")
    ap.add_argument("--gather-ctas", type=int, default=0,
                    help="with --gather-nccl: CTAs for the gather's own communicator, left free by the attender")
    ap.add_argument("--gather-groups", type=int, default=1,
                    help="with --gather-nccl: concurrent communicators (one image per transfer)")
    ap.add_argument("--gather-mb", type=int, default=0,
                    help="N>1: images per gathered micro-batch (0: the forward's micro-batch; 2 with --gather-nccl)")
    ap.add_argument("--gather-nccl", action="store_true",
                    help="N>1: gather with NCCL (dist.gather) instead of the copy engines through CUDA IPC")
    ap.add_argument("--no-ref-upsampler", action="store_true",
                    help="skip timing the reference's own compiled upsampler (N=1)")
    ap.add_argument("--only-reference-upsampler", action="store_true",
                    help="run only the reference's own make_fast upsampler at 1022 px, eager and compiled")
    ap.add_argument("--images", type=int, default=8,
                    help="images per GPU (default 8; smaller only for profiling captures)")
    args = ap.parse_args()
    B_PER_GPU = args.images
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, world, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    world, rank, local = dist_setup()
    try:
        if args.only_fp32:
            dev = torch.device("cuda", local)
            res = {"fp32_configs": run_fp32_configs(dev, torch.cuda.current_stream(dev), load_peaks()[0])}
        elif args.only_backward:
            dev = torch.device("cuda", local)
            res = {"backward": run_backward(dev, torch.cuda.current_stream(dev), load_peaks()[0], B_PER_GPU)}
        elif args.only_fused_resize:
            dev = torch.device("cuda", local)
            res = {"fused_resize": run_fused_resize(dev, torch.cuda.current_stream(dev), load_peaks()[0],
                                                    images=B_PER_GPU)}
        elif args.only_reference_upsampler:
            dev = torch.device("cuda", local)
            st = torch.cuda.current_stream(dev)
            res = {"reference_upsampler": {"eager": run_reference_upsampler(dev, st, False),
                                           "compiled": run_reference_upsampler(dev, st, True)}}
        elif args.only_upsampler:
            dev = torch.device("cuda", local)
            res = {"upsampler": run_upsampler(dev, torch.cuda.current_stream(dev), world, rank, args, outsize=1022,
                                              gather=not args.no_gather)}
        else:
            res = run_ours(args, world, rank, local)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
