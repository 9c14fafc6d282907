#!/usr/bin/env python
"""fwd+bwd SSIM throughput on B200 — one JSON line on rank 0.

Headline workload (per GPU): the 3DGS training-step shape, a 1x3x1080x1920 FP32
render/ground-truth pair (seeded synthetic blob field + 3x3 box blur + noise), padding
"same", window 11, train=True: ``loss = fused_ssim(img1, img2); loss.backward()`` through
the public API. With N GPUs (torchrun) every rank holds its own 1080p pair (weak scaling);
the global mean is formed by the forward kernels publishing their sums to every rank's
mailbox over NVLink and a one-warp gather kernel per rank (no collective call in the step).

Reported:
* value      B*C*H*W/s of all ranks over the max-over-ranks device time of K back-to-back
             steps (Mpix/s, the reference's convention); inputs resident in HBM; 4 rotating
             input pairs (200 MB per rank, > 126 MB L2) so no step starts with its inputs
             in L2. The launch queue is filled before the first timed step (a GPU sleep
             ahead of it), so the figure is the GPU's step rate; ``host_us_per_step`` is the
             host's enqueue cost of one step, measured separately.
* e2e        the same step through the public API with host (pinned) inputs: H2D copy of
             both images, fwd+bwd, D2H of the loss, every step.
* roofline   the dominant kernel timed alone with CUDA events on its stream; achieved =
             algorithmic bytes or FLOPs per launch / launch time.
* batch_2048 the 64x3x2048^2 FP32 batch sharded over the N ranks (64/N images each).
* fp16       FP16 autocast against FP32 on the same configurations (1080p same padding,
             8x3x1024^2 valid padding).
* cpu_baseline  the reference test suite's conv2d SSIM formula (fwd+bwd, FP32, all host
             threads) on the full 1080p frame.

``--impl reference`` prints the reference arm: the same conv2d formula on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd SSIM Mpix/s (FP32, FP16) at 1080p RGB, 1/2/4/8 B200; % of roofline"
SHAPE = (1, 3, 1080, 1920)
N_ROT = 4

# Algorithmic work per channel-pixel (cpx): bytes a kernel must move at minimum, and FP32
# FLOPs (an FMA counts 2) of the separable 11-tap stencils plus the per-pixel epilogue.
FWD_BYTES_F32 = 8 + 12        # read img1, img2; write 3 partials
BWD_BYTES_F32 = 12 + 8 + 4    # read 3 partials, img1, img2; write grad
FWD_FLOPS = 2 * 5 * 2 * 11 + 3 + 30   # 5 moments x 2 passes x 11 MACs, 3 products, epilogue
BWD_FLOPS = 2 * 3 * 2 * 11 + 6        # 3 partial maps x 2 passes x 11 MACs, combine + chain

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the 1080p
# workload's kernels (the column-streaming forward and backward), from one ncu capture of
# this kernel version (ncu flushes L2 before each captured launch: cold-L2 figures).
NCU_TRAFFIC_BYTES = {"fwd": 57.51e6 + 26.33e6, "bwd": 143.76e6 + 13.24e6}
NCU_TRAFFIC_SOURCE = ("ncu --set full --clock-control none -k regex:loss_ -s 4 -c 2 "
                      "python bench.py --steps 50 --warmup 3 --skip-extras")
KERNEL_NAMES = {"fwd": "loss_fwd_kernel (column-streaming forward)",
                "bwd": "loss_bwd_kernel (column-streaming backward)"}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = {"hbm_gbs": 6650.0, "source": "fallback", "sm_max_mhz": 1965.0}
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        peaks.update(hbm_gbs=float(p["hbm_gbs"]), sm_max_mhz=float(p.get("sm_max_mhz", 1965.0)),
                     source="measured")
    return peaks


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ClockSampler:
    """nvidia-smi samples of SM clock and clock-event reasons, written by the nvidia-smi
    process straight to a file (no reader thread in this process), parsed after the run."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        self.file = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
        self.marks = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(gpu_index), "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.file.flush()

    def _rows(self):
        import datetime as dt

        self.file.seek(0)
        rows = []
        for line in self.file.read().splitlines():
            cols = [c.strip() for c in line.split(",")]
            try:
                t = dt.datetime.strptime(cols[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except (ValueError, IndexError):
                continue
            rows.append((t, cols))
        return rows

    def summary(self, t0, t1):
        rows = self._rows()
        inside = [r for t, r in rows if t0 - 0.05 <= t <= t1 + 0.05]
        window = "timed"
        if not inside:
            inside = [r for _, r in rows]
            window = "warmup+timed (timed region shorter than the sampling period)"
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in inside:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except (ValueError, IndexError):
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        try:
            os.unlink(self.file.name)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "window": window}


def cpu_formula_step(a, b):
    """The reference tests' conv2d SSIM (tests/test_ssim.py:34-61) fwd+bwd on the host."""
    from oracle import ssim_oracle as O

    x = a.clone().requires_grad_(True)
    v = O.reference_formula_2d(x, b)
    (1.0 - v).backward()
    return v.item()


def cpu_baseline(steps, budget_s=60.0):
    """Time the CPU formula on the full 1080p frame, all host threads; `steps` is capped so
    the leg stays within about budget_s."""
    from fussim_b200 import synthetic

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    a, b = synthetic.make_pair("rgb_1080p")
    t = time.perf_counter()
    cpu_formula_step(a, b)  # warm (and a probe of the step time)
    probe = time.perf_counter() - t
    steps = int(max(1, min(steps, budget_s / max(probe, 1e-3))))
    t = time.perf_counter()
    for _ in range(steps):
        cpu_formula_step(a, b)
    dt = (time.perf_counter() - t) / steps
    cpx = a.numel()
    return {"value": cpx / dt / 1e6, "unit": "Mpix/s", "cores": threads, "kind": "port",
            "cpu": cpu_model(),
            "sample": f"the full 1x3x1080x1920 pair per step, {steps} steps, conv2d formula "
                      f"fwd+bwd FP32 ({cpx} cpx/step)",
            "ms_per_step": dt * 1e3, "steps": steps}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = cpu_baseline(max(1, args.steps))
    line = {"metric": METRIC, "value": base["value"], "unit": "Mpix/s", "n_gpus": args.gpus,
            "steps": base["steps"], "warmup": args.warmup, "ms_per_step": base["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "1x3x1080x1920 fp32 same train fwd+bwd (host cores)",
                       "global_batch": 1, "window": 11, "padding": "same"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "Mpix/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def event_time(fn, iters, stream=None, prime_us=0.0):
    """Device ms per call of fn over `iters` back-to-back calls (CUDA events on `stream`).
    With prime_us > 0 a GPU sleep of about that long is queued ahead of the first event, so
    the host enqueues the first calls before the GPU starts timing them."""
    s = torch.cuda.current_stream() if stream is None else stream
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if prime_us > 0:
        torch.cuda._sleep(int(prime_us * 2000))  # ~2000 cycles per microsecond
    e0.record(s)
    for i in range(iters):
        fn(i)
    e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters  # ms per call


def host_enqueue_us(fn, iters=30):
    """Host wall time to enqueue one call of fn, with the GPU busy (a long sleep queued
    first) so the launch queue never fills and no call waits for the device."""
    torch.cuda.synchronize()
    torch.cuda._sleep(int(iters * 400 * 2000))  # ~400 us of GPU sleep per call
    t = time.perf_counter()
    for i in range(iters):
        fn(i)
    dt = time.perf_counter() - t
    torch.cuda.synchronize()
    return dt / iters * 1e6


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--skip-extras", action="store_true", help="only the headline number")
    ap.add_argument("--dtype", default="f32", choices=["f32", "f16"],
                    help="f16: the headline step on the same images in FP16 under autocast")
    ap.add_argument("--kernels", default="auto", choices=["auto", "stream", "tile"],
                    help="kernel family of the fused loss (fssim_set_loss_kernels)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch.distributed as dist

    import fussim_b200 as fb
    from fussim_b200 import distributed as fdist
    from fussim_b200 import synthetic
    from fussim_b200.functional import _ensure_cuda_extension

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    ext = _ensure_cuda_extension()
    ext.set_loss_kernels({"stream": 0, "tile": 1, "auto": 2}[args.kernels])
    peaks = load_peaks()
    warm = max(3, args.warmup)
    K = args.steps

    # 4 rotating pairs per rank, generated on the host from rank-specific seeds
    host = [synthetic.make_pair("rgb_1080p", seed=1000 * rank + k) for k in range(N_ROT)]
    half = args.dtype == "f16"
    if half:
        # the same images in FP16 under autocast (headline number only)
        host = [(a.half(), b.half()) for a, b in host]
        args.skip_extras = True
    pairs = [(a.to(dev).requires_grad_(True), b.to(dev)) for a, b in host]
    cpx_rank = pairs[0][0].numel()

    def step(i):
        x, y = pairs[i % N_ROT]
        with torch.autocast("cuda", enabled=half):
            if world > 1:
                v, work = fdist.fused_ssim_dp(x, y, async_op=True)
            else:
                v = fb.fused_ssim(x, y)
        v.backward()
        if world > 1:
            work.wait()
        x.grad = None
        return v

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    host_us = host_enqueue_us(step)
    sampler = ClockSampler(local)
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    ms = event_time(step, K, prime_us=min(K, 100) * 150.0)
    t1 = time.time()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = max_over_ranks(ms)
    time.sleep(0.2)
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    value = world * cpx_rank / (ms * 1e-3) / 1e6

    extras = {}
    if not args.skip_extras:
        if rank == 0:
            extras.update(measure_kernels(ext, pairs, dev, K, warm, peaks, ms))
        if world > 1:
            dist.barrier()
        # every rank takes part in the end-to-end step and in the sharded batch
        extras["e2e"] = measure_e2e(fb, fdist, host, dev, K, warm, world, max_over_ranks)
        if world == 1:
            extras.update(measure_single_gpu(fb, synthetic, pairs, dev, K, warm, ms))
        del pairs
        torch.cuda.empty_cache()
        extras["batch_2048"] = measure_batch_2048(fb, fdist, dev, world, rank, warm, peaks,
                                                  max_over_ranks)
    if world > 1:
        fdist.release_mailboxes()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "Mpix/s", "n_gpus": world, "steps": K,
        "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": args.dtype, "data": "synthetic",
        "config": {"workload": f"1x3x1080x1920 {'fp16 images under autocast' if half else 'fp32'}"
                               ", padding same, window 11, train, fwd+bwd per GPU (public API "
                               "fused_ssim + backward)",
                   "global_batch": world, "shape_per_gpu": list(SHAPE),
                   "parallelism": f"dp{world}" if world > 1 else "none",
                   "l2": "4 rotating input pairs per GPU (200 MB > 126 MB L2)",
                   "timing": "CUDA events around K back-to-back steps, launch queue primed "
                             "by a GPU sleep before the first event; max over ranks",
                   "kernels": args.kernels,
                   "rgb_mpix_per_s": value / 3.0},
        "host_us_per_step": host_us,
        "gpu_launches": 2 * K + (K if world > 1 else 0),
        "clocks": clocks,
    }
    line.update(extras)
    print(json.dumps(line), flush=True)


def measure_kernels(ext, pairs, dev, K, warm, peaks, step_ms):
    """The forward and backward kernels timed alone on this GPU, and their rooflines."""
    out = {}
    C1, C2 = 0.01**2, 0.03**2
    n = pairs[0][0].numel()
    scale = 1.0 / n
    iters = max(20, min(K, 1000))
    dets = [(x.detach(), y) for x, y in pairs]
    parts = [ext.loss_forward(x, y, 11, C1, C2, False, False, True, 1, False, scale)[1]
             for x, y in dets]
    go = torch.ones((), device=dev)

    def fwd(i):
        x, y = dets[i % N_ROT]
        ext.loss_forward(x, y, 11, C1, C2, False, False, True, 1, False, scale)

    def bwd(i):
        x, y = dets[i % N_ROT]
        ext.loss_backward(go, x, y, parts[i % N_ROT], 11, False, scale, 0)

    for i in range(warm):
        fwd(i)
        bwd(i)
    t_f = event_time(fwd, iters, prime_us=3000)
    t_b = event_time(bwd, iters, prime_us=3000)
    hbm = peaks["hbm_gbs"]
    fp32_peak = 148 * 128 * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12  # TFLOP/s, nominal
    kern = {
        "fwd": {"us": t_f * 1e3, "bytes": FWD_BYTES_F32 * n, "flops": FWD_FLOPS * n},
        "bwd": {"us": t_b * 1e3, "bytes": BWD_BYTES_F32 * n, "flops": BWD_FLOPS * n},
    }
    for k in kern.values():
        s = k["us"] * 1e-6
        k["gbs"] = k["bytes"] / s / 1e9
        k["tflops"] = k["flops"] / s / 1e12
        k["t_hbm_us"] = k["bytes"] / (hbm * 1e9) * 1e6
        k["t_fp32_us"] = k["flops"] / (fp32_peak * 1e12) * 1e6
        k["bound"] = "hbm" if k["t_hbm_us"] >= k["t_fp32_us"] else "fp32"
        k["frac"] = max(k["t_hbm_us"], k["t_fp32_us"]) / k["us"]
    dom = max(kern, key=lambda name: kern[name]["us"])
    d = kern[dom]
    if d["bound"] == "hbm":
        roof = {"bound": "hbm", "achieved": d["gbs"], "peak": hbm, "unit": "GB/s",
                "frac": d["gbs"] / hbm}
    else:
        roof = {"bound": "fp32", "achieved": d["tflops"], "peak": fp32_peak, "unit": "TFLOP/s",
                "frac": d["tflops"] / fp32_peak}
    roof["traffic"] = NCU_TRAFFIC_BYTES[dom]
    roof.update(kernel=KERNEL_NAMES[dom], launch_us=d["us"], traffic_unit="bytes per launch",
                traffic_source=NCU_TRAFFIC_SOURCE, algorithmic_bytes=d["bytes"],
                peak_source=("hbm: MEASURED_PEAKS.json (measured)" if peaks["source"] == "measured"
                             else "hbm: fallback") + "; fp32: 148 SMs x 128 lanes x 2 x sm_max_mhz")
    out["roofline"] = roof
    out["kernels"] = kern
    # north-star roofline of the whole step: max(44 B/cpx at HBM peak, FP32 FLOPs at peak)
    t_step_roof = max((FWD_BYTES_F32 + BWD_BYTES_F32) * n / (hbm * 1e9),
                      (FWD_FLOPS + BWD_FLOPS) * n / (fp32_peak * 1e12))
    out["step_roofline"] = {"roof_us": t_step_roof * 1e6, "kernels_us": (t_f + t_b) * 1e3,
                            "api_step_us": step_ms * 1e3,
                            "frac_kernels": t_step_roof * 1e3 / (t_f + t_b),
                            "frac_api_step": t_step_roof * 1e3 / step_ms,
                            "bound": "hbm", "bytes_per_cpx": FWD_BYTES_F32 + BWD_BYTES_F32}
    del parts
    return out


def measure_e2e(fb, fdist, host, dev, K, warm, world, max_over_ranks):
    """The step through the public API from host (pinned) buffers on every rank: H2D of the
    rank's image pair, fwd+bwd (sharded over the ranks), D2H of the loss, every step."""
    pinned = [(a.pin_memory(), b.pin_memory()) for a, b in host]
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    n = host[0][0].numel()
    esize = host[0][0].element_size()

    def e2e(i):
        a_h, b_h = pinned[i % N_ROT]
        x = a_h.to(dev, non_blocking=True).requires_grad_(True)
        y = b_h.to(dev, non_blocking=True)
        v = fdist.fused_ssim_dp(x, y) if world > 1 else fb.fused_ssim(x, y)
        v.backward()
        loss_h.copy_(v.detach(), non_blocking=True)

    e_iters = max(10, min(K, 300))
    for i in range(warm):
        e2e(i)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    t_e = max_over_ranks(event_time(e2e, e_iters))
    return {"value": world * n / (t_e * 1e-3) / 1e6, "unit": "Mpix/s", "ms_per_step": t_e,
            "h2d_bytes_per_step": 2 * n * esize * world, "d2h_bytes_per_step": 4 * world,
            "steps": e_iters, "n_gpus": world}


def measure_single_gpu(fb, synthetic, pairs, dev, K, warm, step_ms):
    """One-GPU legs: the fused 3DGS loss, FP16 against FP32, the CPU baseline."""
    out = {}
    n = pairs[0][0].numel()

    # The 3DGS photometric loss 0.8*L1 + 0.2*(1-SSIM) at 1080p: fused (one forward and one
    # backward kernel) against the same loss composed from fused_ssim and torch's L1.
    def gs_fused(i):
        x, y = pairs[i % N_ROT]
        v = fb.l1_dssim_loss(x, y, lambda_dssim=0.2)
        v.backward()
        x.grad = None

    def gs_composed(i):
        x, y = pairs[i % N_ROT]
        v = 0.8 * (x - y).abs().mean() + 0.2 * (1.0 - fb.fused_ssim(x, y))
        v.backward()
        x.grad = None

    g_iters = max(10, min(K, 300))
    for i in range(warm):
        gs_fused(i)
        gs_composed(i)
    t_gf = event_time(gs_fused, g_iters, prime_us=3000)
    t_gc = event_time(gs_composed, g_iters, prime_us=3000)
    out["l1_dssim_1080p"] = {"workload": "1x3x1080x1920 fp32, 0.8*L1 + 0.2*(1-SSIM), fwd+bwd",
                             "fused_ms_per_step": t_gf, "composed_ms_per_step": t_gc,
                             "fused_value": n / (t_gf * 1e-3) / 1e6, "unit": "Mpix/s"}

    out["fp16"] = measure_fp16(fb, synthetic, pairs, dev, K, warm, step_ms)
    out["cpu_baseline"] = cpu_baseline(steps=3, budget_s=15.0)
    return out


def measure_fp16(fb, synthetic, pairs, dev, K, warm, step_ms_fp32):
    """FP16 autocast against FP32, each pair on the same configuration and inputs."""
    iters = max(10, min(K, 300))

    def run(pp, padding, half):
        def st(i):
            x, y = pp[i % len(pp)]
            with torch.autocast("cuda", enabled=half):
                v = fb.fused_ssim(x, y, padding=padding)
            v.backward()
            x.grad = None

        for i in range(warm):
            st(i)
        return event_time(st, iters, prime_us=3000)

    n1080 = pairs[0][0].numel()
    # FP16 images (the FP16 workload's own dtype): no cast kernel in the step
    p16 = [(x.detach().half().requires_grad_(True), y.half()) for x, y in pairs]
    t16_1080 = run(p16, "same", True)
    del p16
    res = {"1080p_same": {"workload": "1x3x1080x1920, padding same, train, fwd+bwd; FP32 "
                                       "images vs the same images in FP16 under autocast",
                          "fp32_ms": step_ms_fp32, "fp16_ms": t16_1080,
                          "fp32_value": n1080 / (step_ms_fp32 * 1e-3) / 1e6,
                          "fp16_value": n1080 / (t16_1080 * 1e-3) / 1e6,
                          "fp16_over_fp32": step_ms_fp32 / t16_1080}}
    # 8x3x1024^2 blob pairs, valid padding: the same values as FP32 images (FP32 leg) and as
    # FP16 images under autocast (FP16 leg, the workload's own form)
    h = [synthetic.make_pair("fp16_1024_valid", seed=77 + k) for k in range(2)]
    p = [(a.float().to(dev).requires_grad_(True), b.float().to(dev)) for a, b in h]
    n = p[0][0].numel()
    t32 = run(p, "valid", False)
    p = [(a.to(dev).requires_grad_(True), b.to(dev)) for a, b in h]
    t16 = run(p, "valid", True)
    res["8x1024_valid"] = {"workload": "8x3x1024x1024 blob pairs, padding valid, train, fwd+bwd",
                           "fp32_ms": t32, "fp16_ms": t16,
                           "fp32_value": n / (t32 * 1e-3) / 1e6,
                           "fp16_value": n / (t16 * 1e-3) / 1e6, "fp16_over_fp32": t32 / t16}
    del p
    torch.cuda.synchronize()
    return res


def measure_batch_2048(fb, fdist, dev, world, rank, warm, peaks, max_over_ranks):
    """The 64x3x2048^2 FP32 batch (img1 ~ U[0,1], img2 = clamp(img1 + N(0, 0.1^2))) sharded
    over the ranks, 64/N images each, generated on the device outside the timed region."""
    per = 64 // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(4 + 7919 * rank)
    shape = (per, 3, 2048, 2048)
    a = torch.rand(shape, device=dev, generator=gen)
    b = (a + 0.1 * torch.randn(shape, device=dev, generator=gen)).clamp_(0.0, 1.0)
    a.requires_grad_(True)

    def st(i):
        if world > 1:
            v = fdist.fused_ssim_dp(a, b)
        else:
            v = fb.fused_ssim(a, b)
        v.backward()
        a.grad = None

    for i in range(min(warm, 3)):
        st(i)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    iters = 5
    ms = max_over_ranks(event_time(st, iters))
    n_total = 64 * 3 * 2048 * 2048
    hbm = peaks["hbm_gbs"]
    roof_ms = (FWD_BYTES_F32 + BWD_BYTES_F32) * n_total / world / (hbm * 1e9) * 1e3
    del a, b
    torch.cuda.empty_cache()
    return {"workload": "64x3x2048x2048 fp32, padding same, train, fwd+bwd, sharded over "
                        f"{world} GPU(s), {per} images each",
            "value": n_total / (ms * 1e-3) / 1e6, "unit": "Mpix/s", "ms_per_step": ms,
            "steps": iters, "n_gpus": world, "roof_ms_per_gpu": roof_ms,
            "frac_roofline": roof_ms / ms}


if __name__ == "__main__":
    main()
