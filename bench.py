#!/usr/bin/env python
"""fwd+bwd SSIM throughput on B200 — one JSON line on rank 0.

Workload (per GPU): the 3DGS training-step shape, 1x3x1080x1920 FP32 render/ground-truth
pair (seeded synthetic blob field + 3x3 box blur + noise), padding "same", window 11,
train=True: ``loss = fused_ssim(img1, img2); loss.backward()`` through the public API.
With N GPUs (torchrun) every rank holds its own 1080p pair (weak scaling); the global mean
is formed by the forward kernels publishing their sums to every rank's mailbox over NVLink
and a one-warp gather kernel per rank (no collective call in the step).

Reported:
* value      B*C*H*W/s of all ranks over the max-over-ranks device time (Mpix/s, the
             reference's convention); inputs resident in HBM; 4 rotating input pairs
             (200 MB per rank, > 126 MB L2) so no step starts with its inputs in L2.
* e2e        the same step through the public API with host (pinned) inputs: H2D copy of
             both images, fwd+bwd, D2H of the loss, every step.
* roofline   the dominant kernel timed alone with CUDA events on its stream; achieved =
             algorithmic bytes or FLOPs per launch / launch time.
* cpu_baseline  the reference test suite's conv2d SSIM formula (fwd+bwd, FP32, all host
             threads) on a bounded sample of the same workload.
* fp16       the 8x3x1024^2 FP16 'valid' autocast workload on one GPU.

``--impl reference`` prints the reference arm: the conv2d formula on the host cores.
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

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd SSIM Mpix/s (FP32, FP16) at 1080p RGB, 1/2/4/8 B200; % of roofline"
SHAPE = (1, 3, 1080, 1920)
FP16_SHAPE = (8, 3, 1024, 1024)
N_ROT = 4

# Algorithmic work per channel-pixel (cpx): bytes a kernel must move at minimum, and FP32
# FLOPs (an FMA counts 2) of the separable 11-tap stencils plus the per-pixel epilogue.
FWD_BYTES_F32 = 8 + 12        # read img1, img2; write 3 partials
BWD_BYTES_F32 = 12 + 8 + 4    # read 3 partials, img1, img2; write grad
FWD_FLOPS = 2 * 5 * 2 * 11 + 3 + 30   # 5 moments x 2 passes x 11 MACs, 3 products, epilogue
BWD_FLOPS = 2 * 3 * 2 * 11 + 6        # 3 partial maps x 2 passes x 11 MACs, combine + chain

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of each kernel on
# this workload, from one ncu capture (profiles/ssim_fwd_bwd_1080p_fp32.md; the capture
# flushes L2 before each launch, so it is the cold-L2 figure).
NCU_TRAFFIC_BYTES = {"fwd": 60.75e6 + 27.58e6, "bwd": 172.90e6 + 15.77e6}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = {"hbm_gbs": 6650.0, "source": "fallback", "sm_max_mhz": 1965.0}
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        peaks.update(hbm_gbs=float(p["hbm_gbs"]), sm_max_mhz=float(p.get("sm_max_mhz", 1965.0)),
                     source="measured")
    return peaks


class ClockSampler:
    """nvidia-smi samples of SM clock and clock-event reasons, filtered to a time window."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.rows = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(gpu_index), "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [c.strip() for c in line.split(",")]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        inside = [r for t, r in self.rows if t0 <= t <= t1]
        window = "timed"
        if not inside:
            inside = [r for _, r in self.rows]
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


def cpu_baseline(steps, budget_s=20.0):
    """Time the CPU formula on a bounded sample (row band) of the 1080p workload."""
    from fussim_b200 import synthetic

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    a, b = synthetic.make_pair("rgb_1080p")
    # size the sample from one probe on a 120-row band so the whole run stays bounded
    band = 120
    t = time.perf_counter()
    cpu_formula_step(a[:, :, :band], b[:, :, :band])
    per_row = (time.perf_counter() - t) / band
    rows = int(max(32, min(SHAPE[2], budget_s / max(steps, 1) / max(per_row, 1e-9))))
    sa, sb = a[:, :, :rows].contiguous(), b[:, :, :rows].contiguous()
    cpu_formula_step(sa, sb)  # warm
    t = time.perf_counter()
    for _ in range(steps):
        cpu_formula_step(sa, sb)
    dt = (time.perf_counter() - t) / steps
    cpx = sa.numel()
    return {"value": cpx / dt / 1e6, "unit": "Mpix/s", "cores": threads, "kind": "port",
            "sample": f"1x3x{rows}x1920 band of the 1080p pair per step, {steps} steps, "
                      f"conv2d formula fwd+bwd FP32 ({cpx} cpx/step)",
            "ms_per_step": dt * 1e3}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps = max(1, min(args.steps, 50))
    base = cpu_baseline(steps)
    line = {"metric": METRIC, "value": base["value"], "unit": "Mpix/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": base["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "1x3x1080x1920 fp32 same train fwd+bwd (host sample)",
                       "global_batch": 1, "window": 11, "padding": "same"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "Mpix/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def event_time(fn, iters, stream=None):
    s = torch.cuda.current_stream() if stream is None else stream
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(iters):
        fn(i)
    e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters  # ms per call


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--skip-extras", action="store_true", help="only the headline number")
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
    peaks = load_peaks()
    warm = max(3, args.warmup)
    K = args.steps

    # 4 rotating pairs per rank, generated on the host from rank-specific seeds
    host = [synthetic.make_pair("rgb_1080p", seed=1000 * rank + k) for k in range(N_ROT)]
    pairs = [(a.to(dev).requires_grad_(True), b.to(dev)) for a, b in host]
    cpx_rank = pairs[0][0].numel()

    def step(i):
        x, y = pairs[i % N_ROT]
        if world > 1:
            v, work = fdist.fused_ssim_dp(x, y, async_op=True)
            v.backward()
            work.wait()
        else:
            v = fb.fused_ssim(x, y)
            v.backward()
        x.grad = None
        return v

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    ms = event_time(step, K)
    t1 = time.time()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    time.sleep(0.2)
    sampler.stop()
    clocks = sampler.summary(t0, t1)
    value = world * cpx_rank / (ms * 1e-3) / 1e6

    extras = {}
    if rank == 0 and not args.skip_extras:
        extras = measure_extras(ext, fb, synthetic, pairs, host, dev, K, warm, peaks, ms)
    if world > 1:
        fdist.release_mailboxes()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "Mpix/s", "n_gpus": world, "steps": K,
        "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "1x3x1080x1920 fp32, padding same, window 11, train, fwd+bwd "
                               "per GPU (public API fused_ssim + backward)",
                   "global_batch": world, "shape_per_gpu": list(SHAPE),
                   "parallelism": f"dp{world}" if world > 1 else "none",
                   "l2": "4 rotating input pairs per GPU (200 MB > 126 MB L2)",
                   "rgb_mpix_per_s": value / 3.0},
        "gpu_launches": 2 * K,
        "clocks": clocks,
    }
    line.update(extras)
    print(json.dumps(line), flush=True)


def measure_extras(ext, fb, synthetic, pairs, host, dev, K, warm, peaks, step_ms):
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
    t_f = event_time(fwd, iters)
    t_b = event_time(bwd, iters)
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
                "frac": d["gbs"] / hbm, "traffic": None}
    else:
        roof = {"bound": "fp32", "achieved": d["tflops"], "peak": fp32_peak, "unit": "TFLOP/s",
                "frac": d["tflops"] / fp32_peak, "traffic": None}
    roof["traffic"] = NCU_TRAFFIC_BYTES[dom]
    roof.update(kernel=f"ssim_{dom}_kernel", launch_us=d["us"], traffic_unit="bytes per launch",
                algorithmic_bytes=d["bytes"],
                peak_source=("hbm: MEASURED_PEAKS.json (measured)" if peaks["source"] == "measured"
                             else "hbm: fallback") + "; fp32: 148 SMs x 128 lanes x 2 x sm_max_mhz")
    out["roofline"] = roof
    out["kernels"] = kern
    # north-star roofline of the whole step: max(44 B/cpx at HBM peak, FP32 FLOPs at peak)
    t_step_roof = max((FWD_BYTES_F32 + BWD_BYTES_F32) * n / (hbm * 1e9),
                      (FWD_FLOPS + BWD_FLOPS) * n / (fp32_peak * 1e12))
    out["step_roofline"] = {"roof_us": t_step_roof * 1e6, "kernels_us": (t_f + t_b) * 1e3,
                            "frac_kernels": t_step_roof * 1e3 / (t_f + t_b),
                            "frac_api_step": t_step_roof * 1e3 / step_ms,
                            "bound": "hbm", "bytes_per_cpx": FWD_BYTES_F32 + BWD_BYTES_F32}

    # e2e through the public API with host buffers
    pinned = [(a.pin_memory(), b.pin_memory()) for a, b in host]
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e(i):
        a_h, b_h = pinned[i % N_ROT]
        x = a_h.to(dev, non_blocking=True).requires_grad_(True)
        y = b_h.to(dev, non_blocking=True)
        v = fb.fused_ssim(x, y)
        v.backward()
        loss_h.copy_(v.detach(), non_blocking=True)

    e_iters = max(10, min(K, 300))
    for i in range(warm):
        e2e(i)
    torch.cuda.synchronize()
    t_e = event_time(e2e, e_iters)
    out["e2e"] = {"value": n / (t_e * 1e-3) / 1e6, "unit": "Mpix/s", "ms_per_step": t_e,
                  "h2d_bytes_per_step": 2 * n * 4, "d2h_bytes_per_step": 4, "steps": e_iters}

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
    t_gf = event_time(gs_fused, g_iters)
    t_gc = event_time(gs_composed, g_iters)
    out["l1_dssim_1080p"] = {"workload": "1x3x1080x1920 fp32, 0.8*L1 + 0.2*(1-SSIM), fwd+bwd",
                             "fused_ms_per_step": t_gf, "composed_ms_per_step": t_gc,
                             "fused_value": n / (t_gf * 1e-3) / 1e6, "unit": "Mpix/s"}

    # FP16 autocast workload (8x3x1024^2, valid padding) on this GPU
    del parts
    h16 = [synthetic.make_pair("fp16_1024_valid", seed=77 + k) for k in range(N_ROT)]
    p16 = [(a.to(dev).requires_grad_(True), b.to(dev)) for a, b in h16]

    def step16(i):
        x, y = p16[i % N_ROT]
        with torch.autocast("cuda"):
            v = fb.fused_ssim(x, y, padding="valid")
        v.backward()
        x.grad = None

    i16 = max(10, min(K, 300))
    for i in range(warm):
        step16(i)
    t16 = event_time(step16, i16)
    n16 = p16[0][0].numel()
    v16 = n16 / (t16 * 1e-3) / 1e6
    v32 = n / (step_ms * 1e-3) / 1e6
    out["fp16"] = {"workload": "8x3x1024x1024 fp16 inputs, autocast, padding valid, train, "
                               "fwd+bwd", "value": v16, "unit": "Mpix/s", "ms_per_step": t16,
                   "ratio_vs_fp32_1080p": v16 / v32, "steps": i16}
    torch.cuda.synchronize()
    del p16
    # The data-parallel batch config (64x3x2048^2 FP32, U[0,1] + N(0, 0.1^2)) whole on this
    # GPU: 805 M cpx per step, generated on the device outside the timed region.
    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    shape4 = (64, 3, 2048, 2048)
    a4 = torch.rand(shape4, device=dev, generator=gen)
    b4 = (a4 + 0.1 * torch.randn(shape4, device=dev, generator=gen)).clamp_(0.0, 1.0)
    a4.requires_grad_(True)

    def step4(i):
        v = fb.fused_ssim(a4, b4)
        v.backward()
        a4.grad = None

    for i in range(2):
        step4(i)
    t4 = event_time(step4, 5)
    n4 = a4.numel()
    out["batch_2048"] = {"workload": "64x3x2048x2048 fp32, padding same, train, fwd+bwd, whole "
                                     "batch on one GPU", "value": n4 / (t4 * 1e-3) / 1e6,
                         "unit": "Mpix/s", "ms_per_step": t4, "steps": 5,
                         "roof_ms": (FWD_BYTES_F32 + BWD_BYTES_F32) * n4 / (hbm * 1e9) * 1e3}
    out["batch_2048"]["frac_roofline"] = out["batch_2048"]["roof_ms"] / t4
    del a4, b4
    torch.cuda.synchronize()
    out["cpu_baseline"] = cpu_baseline(steps=2, budget_s=15.0)
    return out


if __name__ == "__main__":
    main()
