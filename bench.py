"""Benchmark: batched Householder QR on the five workload configs C1..C5.

Metric (the reference's): QR microseconds per call and TFLOP/s (4 n^3 / 3 per matrix) per
config, and the geometric mean of microseconds per call over the five configs. ``value`` is
that geomean (lower is better). With ``--gpus N`` (under torchrun, one process per GPU) each
config's batch is split into contiguous slices, one per rank -- independent matrices, no
collective on the data path -- and every per-call time is the max over ranks (strong
scaling: the total batch is fixed).

Arms:
  ``--impl ours`` (default)  this repository's C-ABI operator on the GPU;
  ``--impl reference``       the reference's CPU path, ``torch.geqrf`` (LAPACK) on the host
                             cores, rank 0 only.

Timing: W warm-up calls per config, then K timed calls, each bracketed by CUDA events on
the current stream after an L2 flush (a 256 MiB write); ranks barrier before and after.
``e2e`` repeats the measurement through ``custom_kernel_host`` with pinned host input and output
buffers, the host<->device copies inside the timed region.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

from qr_v2_b200_kernel_b200 import gen  # noqa: E402

CONFIG_ORDER = ["C1", "C2", "C3", "C4", "C5"]
# DRAM bytes (read + write) per launch of the dominant kernel kind, from one ncu capture,
# scaled to the bench workload as profiles/panel_kernels.md describes.
MEASURED_TRAFFIC = {("C2", "panel_factor"): 22.3e6}
L2_FLUSH_BYTES = 256 << 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_peaks() -> dict:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        d["source"] = "measured"
        return d
    return dict(FALLBACK_PEAKS)


def tf32x3_peak_tflops(peaks: dict) -> float:
    """tf32x3 ceiling: dense TF32 = half the bf16 rate (datasheet ratio), three passes."""
    return peaks["bf16_tflops"] / 2.0 / 3.0


# ----------------------------------------------------------------------------- distributed
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int):
    if world <= 1:
        return None
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist


def barrier(dist):
    if dist is not None:
        dist.barrier()


def allmax(dist, x: float) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard(batch: int, world: int, rank: int):
    from qr_v2_b200_kernel_b200.sharding import shard_range

    return shard_range(batch, world, rank)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        smax = max((num(r[2]) or 0) for r in rows)
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(rows),
                "power_w_max": max((num(r[3]) or 0) for r in rows)}


# ----------------------------------------------------------------------------- our arm
def l2_flush(buf: torch.Tensor):
    buf.fill_(1)


def time_device(fn, steps: int, warmup: int, flush: torch.Tensor) -> list[float]:
    """Per-call microseconds of ``fn`` (device time via CUDA events, L2 flushed before each)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    stream = torch.cuda.current_stream()
    for _ in range(steps):
        l2_flush(flush)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        e.synchronize()
        out.append(s.elapsed_time(e) * 1e3)
    return out


def run_ours(args, world, rank, local, dist):
    from qr_v2_b200_kernel_b200 import _lib, api, checker, custom_kernel, profile

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = _lib.load()
    peaks = load_peaks()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    names = args.configs
    per = {}
    inputs = {}
    for name in names:
        cfg = gen.CONFIGS[name]
        A_full = gen.config_input(name, device=dev)
        lo, hi = shard(cfg["batch"], world, rank)
        inputs[name] = A_full[lo:hi].contiguous()
        del A_full
        A = inputs[name]
        if A.shape[0] > 0:
            H, tau = custom_kernel(A)
            chk = checker.check(A, H, tau)
            if not chk["ok"]:
                raise RuntimeError(f"{name}: output fails the correctness gate: {chk['message']}")
            per[name] = {"sfr": chk["scaled_factor_residual"], "orth": chk["scaled_orthogonality_residual"]}
            del H, tau
        else:
            per[name] = {}
    torch.cuda.synchronize()

    # ---- device-timed region (inputs resident in HBM) ----
    clocks = ClockSampler(local)
    barrier(dist)
    clocks.start()
    launches0 = lib.qrb200_launch_count()
    for name in names:
        A = inputs[name]
        cfg = gen.CONFIGS[name]
        if A.shape[0] > 0:
            ts = time_device(lambda: custom_kernel(A), args.steps, args.warmup, flush)
            mine = statistics.mean(ts)
        else:
            mine = 0.0
        barrier(dist)
        us = allmax(dist, mine)
        per[name].update({
            "batch": cfg["batch"], "n": cfg["n"], "us_per_call": us,
            "tflops": gen.flops_per_call(cfg["batch"], cfg["n"]) / us / 1e6,
            "matrices_per_s": cfg["batch"] / us * 1e6,
            "hbm_floor_frac": gen.min_hbm_bytes(cfg["batch"], cfg["n"]) / (us * 1e-6) / (peaks["hbm_gbs"] * 1e9),
        })
        per[name]["tf32x3_frac"] = per[name]["tflops"] / tf32x3_peak_tflops(peaks)
    launches = lib.qrb200_launch_count() - launches0
    clk = clocks.stop()
    barrier(dist)

    # ---- end-to-end through custom_kernel with host buffers ----
    e2e_per = {}
    h2d = d2h = 0
    for name in names:
        A = inputs[name]
        cfg = gen.CONFIGS[name]
        if A.shape[0] > 0:
            hA = A.cpu().pin_memory()
            hH = torch.empty(A.shape, dtype=torch.float32).pin_memory()
            htau = torch.empty(A.shape[:2], dtype=torch.float32).pin_memory()

            def e2e_call():
                # Public host-buffer API: copies in, factorisation, copies out, pipelined in
                # batch pieces on separate streams and joined into the current stream.
                api.custom_kernel_host(hA, device=dev, out=(hH, htau))

            ts = time_device(e2e_call, args.steps, max(1, args.warmup), flush)
            mine = statistics.mean(ts)
            h2d += hA.numel() * 4
            d2h += (hH.numel() + htau.numel()) * 4
        else:
            mine = 0.0
        barrier(dist)
        e2e_per[name] = allmax(dist, mine)
    h2d_all = int(allsum(dist, h2d))
    d2h_all = int(allsum(dist, d2h))

    # ---- per-kernel breakdown of the headline config (roofline of the dominant kernel) ----
    roof = None
    kernels = {}
    if rank == 0:
        rname = "C2" if "C2" in names else names[0]
        A = inputs[rname]
        stats = profile.kernel_breakdown(A, steps=max(1, min(3, args.steps)))
        kernels = {rname: stats}
        dom = max(stats, key=lambda s: s["ms"])
        launches_k = max(1, dom["launches"])
        avg_ms = dom["ms"] / launches_k
        bound = dom["bound"]
        if bound == "tensor":
            peak = tf32x3_peak_tflops(peaks)
            ach = dom["flops"] / launches_k / (avg_ms * 1e-3) / 1e12
            unit = "TFLOP/s"
        else:
            peak = peaks["hbm_gbs"]
            ach = dom["bytes"] / launches_k / (avg_ms * 1e-3) / 1e9
            unit = "GB/s"
        roof = {"bound": bound, "kernel": dom["name"], "config": rname, "achieved": ach, "peak": peak,
                "unit": unit, "frac": ach / peak, "traffic": MEASURED_TRAFFIC.get((rname, dom["name"])),
                "peak_source": ("tf32x3 = measured bf16 / 2 / 3" if bound == "tensor" else "measured hbm_gbs")
                + f" ({peaks['source']})",
                "avg_launch_us": avg_ms * 1e3, "launches": dom["launches"]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference(names, args.cpu_budget_s)

    if rank == 0:
        geo = gen.geomean([per[nm]["us_per_call"] for nm in names])
        e2e_geo = gen.geomean([e2e_per[nm] for nm in names])
        line = {
            "metric": "QR us/call geomean over configs C1-C5 (4n^3/3 flop per matrix)",
            "value": geo, "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sum(per[nm]["us_per_call"] for nm in names) / 1e3,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded generators of configs C1-C5)",
            "config": {"workload": "C1..C5 batched QR, " + ",".join(
                f"{nm}=b{gen.CONFIGS[nm]['batch']}xn{gen.CONFIGS[nm]['n']}" for nm in names),
                "l2": "flushed by a 256 MiB write before every timed call",
                "parallelism": f"batch-sharded over {world} GPU(s), no collective"},
            "per_config": per,
            "e2e": {"value": e2e_geo, "unit": "us", "h2d_bytes_per_step": h2d_all,
                    "d2h_bytes_per_step": d2h_all,
                    "per_config_us": e2e_per},
            "gpu_launches": int(launches),
            "roofline": roof,
            "kernels": kernels,
            "clocks": clk,
            "cpu_baseline": cpu,
            "impl": "ours",
        }
        print(json.dumps(line), flush=True)


def allsum(dist, x: float) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU reference
def cpu_reference(names, budget_s: float, steps: int = 1, warmup: int = 0) -> dict:
    """Time torch.geqrf (LAPACK) on the host cores on a bounded sample of each config.

    Each config is timed on ``s`` of its matrices (s chosen so the whole measurement stays
    within ``budget_s``) and scaled linearly to the full batch (matrices are independent).
    """
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    per = {}
    samples = []
    per_cfg_budget = budget_s / max(1, len(names))
    for name in names:
        cfg = gen.CONFIGS[name]
        b, n = cfg["batch"], cfg["n"]
        # first probe with one matrix to size the sample
        A1 = gen.config_input(name, device="cpu", batch=1)
        t0 = time.perf_counter()
        torch.geqrf(A1)
        one = max(time.perf_counter() - t0, 1e-6)
        s = int(max(1, min(b, per_cfg_budget / one / max(1, steps + warmup))))
        A = gen.config_input(name, device="cpu", batch=s)
        for _ in range(warmup):
            torch.geqrf(A)
        ts = []
        for _ in range(steps):
            t0 = time.perf_counter()
            torch.geqrf(A)
            ts.append(time.perf_counter() - t0)
        t = statistics.median(ts)
        per[name] = {"us_per_call": t / s * b * 1e6, "sample_matrices": s, "batch": b, "n": n}
        samples.append(f"{name}:{s}/{b}")
    geo = gen.geomean([per[nm]["us_per_call"] for nm in names])
    return {"value": geo, "unit": "us", "cores": threads, "kind": "reference",
            "sample": "torch.geqrf (LAPACK sgeqrf) on " + ", ".join(samples)
                      + " matrices per config, scaled linearly to the full batch",
            "per_config": per, "torch_threads": torch.get_num_threads()}


def run_reference(args, world, rank):
    if rank != 0:
        return
    t0 = time.perf_counter()
    cpu = cpu_reference(args.configs, args.cpu_budget_s, steps=args.steps, warmup=min(1, args.warmup))
    names = args.configs
    line = {
        "metric": "QR us/call geomean over configs C1-C5 (4n^3/3 flop per matrix)",
        "value": cpu["value"], "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sum(cpu["per_config"][nm]["us_per_call"] for nm in names) / 1e3,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded generators of configs C1-C5)",
        "config": {"workload": "C1..C5 batched QR, " + ",".join(
            f"{nm}=b{gen.CONFIGS[nm]['batch']}xn{gen.CONFIGS[nm]['n']}" for nm in names),
            "parallelism": "host CPU, all cores"},
        "impl": "reference",
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "per_config": cpu["per_config"],
        "e2e": {"value": cpu["value"], "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--configs", default=",".join(CONFIG_ORDER))
    ap.add_argument("--cpu-budget-s", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.configs = [c.strip() for c in args.configs.split(",") if c.strip()]
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    dist = init_dist(world, local)
    try:
        run_ours(args, world, rank, local, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
