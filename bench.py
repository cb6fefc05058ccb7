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
                             cores, rank 0 only;
  ``--impl triton``          the reference's own GPU submission (``submission.py``, Triton +
                             cuSOLVER), unmodified, staged under ``baseline/_ref/`` by
                             ``__graft_entry__.build()``; run in its own process because importing
                             it flips global TF32 flags. The ``ours`` arm runs it as a
                             subprocess at N = 1 and reports it under ``triton_submission``.

Timing: W warm-up calls per config, then K timed calls, each bracketed by CUDA events on
the current stream after an L2 flush (a 256 MiB write); ranks barrier before and after.
``e2e`` repeats the measurement through ``custom_kernel_host`` with pinned host input and output
buffers, the host<->device copies inside the timed region. ``per_case`` times the reference's
12 scored cases (``harness/lab.py:33-46``) the same way; the Triton arm times them too, so
both report the reference's own leaderboard geomean on the same box.
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
# DRAM bytes (read + write) per launch of the dominant kernel kind, from one ncu capture of its
# launches (`ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum
# --clock-control none -k regex:panel_owner_kernel -c 16` over one call of
# `python -m qr_v2_b200_kernel_b200.run --config C2 --batch 160 --calls 1`): the 16 owner-panel
# launches of one call read 90.05 MB in total and wrote 0 (their writes stay in L2) at batch
# 160; per launch, scaled by the matrices processed to batch 640: 22.51 MB (the algorithmic
# panel read + write is 44.6 MB per launch on average).
MEASURED_TRAFFIC = {("C2", "panel_factor"): 22.51e6}
L2_FLUSH_BYTES = 256 << 20
TRITON_REF_DIR = os.path.join(REPO, "baseline", "_ref")
TRITON_REF_FILE = os.path.join(TRITON_REF_DIR, "submission.py")
REFERENCE_SOURCE = "/root/reference/submission.py"


def stage_triton_reference(src: str = REFERENCE_SOURCE) -> str | None:
    """Copy the reference's GPU submission, unmodified, into the git-ignored ``baseline/_ref/``.

    Runs where the reference tree is present (the build container); the staged copy travels
    with the repository snapshot to the GPU box. Returns the staged path or None.
    """
    if not os.path.exists(src):
        return TRITON_REF_FILE if os.path.exists(TRITON_REF_FILE) else None
    os.makedirs(TRITON_REF_DIR, exist_ok=True)
    data = open(src, "rb").read()
    if not os.path.exists(TRITON_REF_FILE) or open(TRITON_REF_FILE, "rb").read() != data:
        with open(TRITON_REF_FILE + ".tmp", "wb") as f:
            f.write(data)
        os.replace(TRITON_REF_FILE + ".tmp", TRITON_REF_FILE)
    return TRITON_REF_FILE


def case_label(c: dict) -> str:
    return f"b{c['batch']}_n{c['n']}_cond{c['cond']}_{c.get('case', 'dense')}"


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
        self.skip = 0

    def _rows(self) -> list:
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        return rows

    def start(self):
        """Start sampling every 25 ms and return once the first sample is written (at most 5 s),
        so that the sampler is running when the timed region begins; samples taken before that
        are left out of the summary (a multi-GPU timed region can be shorter than 0.1 s)."""
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "25"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 5.0 and self.proc.poll() is None:
            n = len(self._rows())
            if n > 0:
                self.skip = n
                break
            time.sleep(0.01)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = self._rows()
        os.unlink(self.path)
        # Samples taken inside the timed region; if it ended before the next sample, the one
        # written just before it began.
        rows = rows[self.skip:] or rows[-1:]
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


# ----------------------------------------------------------------------------- timing
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


def allsum(dist, x: float) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------- our arm
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
    _lib.check_last_status("a timed call")

    # ---- end-to-end through custom_kernel with host buffers ----
    e2e_per = {}
    h2d = d2h = 0
    for name in names:
        A = inputs[name]
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

    # ---- the reference's 12 scored cases (harness/lab.py:33-46), same timing ----
    per_case = {}
    if not args.no_cases:
        for c in gen.REFERENCE_BENCH_CASES:
            A_full = gen.generate_input(**c, device=dev)
            lo, hi = shard(c["batch"], world, rank)
            A = A_full[lo:hi].contiguous()
            del A_full
            entry = {"batch": c["batch"], "n": c["n"], "cond": c["cond"], "case": c.get("case", "dense")}
            if A.shape[0] > 0:
                H, tau = custom_kernel(A)
                chk = checker.check(A, H, tau)
                entry.update(ok=chk["ok"], sfr=chk.get("scaled_factor_residual"))
                del H, tau
                mine = statistics.mean(time_device(lambda: custom_kernel(A), args.steps, args.warmup, flush))
            else:
                mine = 0.0
            barrier(dist)
            entry["us_per_call"] = allmax(dist, mine)
            per_case[case_label(c)] = entry
            del A
        _lib.check_last_status("a timed call")

    # ---- per-kernel breakdowns: roofline of C2's dominant kernel, latency of C5's panel chain ----
    roof = None
    latency = None
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
        if "C5" in names and inputs["C5"].shape[0] > 0:
            st5 = profile.kernel_breakdown(inputs["C5"], steps=1)
            kernels["C5"] = st5
            cl = next((s for s in st5 if s["name"] == "panel_cluster"), None)
            mhz = clk.get("sm_mhz") or peaks.get("sm_max_mhz") or 1965.0
            if cl is not None and cl["launches"] > 0:
                avg_us = cl["ms"] / cl["launches"] * 1e3
                latency = {"kernel": "panel_cluster", "config": "C5", "bound": "latency",
                           "avg_launch_us": avg_us, "launches": cl["launches"],
                           "reflectors_per_launch": 32, "sm_mhz": mhz,
                           "cycles_per_reflector": avg_us * mhz / 32.0,
                           "note": "serial profile (one stream); cycles = CUDA-event time x median SM clock"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference(names, {nm: inputs[nm].cpu() for nm in names}, steps=5, warmup=1,
                            budget_s=args.cpu_budget_s)
        cpu["inputs"] = "the GPU arm's inputs, copied to the host"

    triton = None
    if rank == 0 and world == 1 and not args.no_triton:
        triton = triton_subprocess(args)

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
            "per_case": per_case,
            "per_case_geomean_us": gen.geomean([v["us_per_call"] for v in per_case.values()]) if per_case else None,
            "gpu_launches": int(launches),
            "roofline": roof,
            "latency": latency,
            "kernels": kernels,
            "clocks": clk,
            "cpu_baseline": cpu,
            "triton_submission": triton,
            "impl": "ours",
        }
        print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- CPU reference
def physical_cores() -> int:
    try:
        import psutil

        return int(psutil.cpu_count(logical=False) or os.cpu_count() or 1)
    except Exception:
        return os.cpu_count() or 1


def cpu_reference(names, inputs: dict, steps: int = 5, warmup: int = 1, budget_s: float = 60.0) -> dict:
    """Time torch.geqrf (LAPACK sgeqrf, the reference's CPU path) on the host's physical cores.

    Per config: ``warmup`` untimed calls, then the median of ``steps`` timed calls (wall clock)
    of one batched call. A config whose full batch would not fit its share of ``budget_s`` is
    timed on its first ``s`` matrices and scaled linearly to the full batch (matrices are
    independent; the sample is reported).
    """
    threads = physical_cores()
    torch.set_num_threads(threads)
    per = {}
    samples = []
    per_cfg_budget = budget_s / max(1, len(names))
    for name in names:
        A = inputs[name]
        b, n = int(A.shape[0]), int(A.shape[-1])
        t0 = time.perf_counter()
        torch.geqrf(A[:1])
        one = max(time.perf_counter() - t0, 1e-6)
        s = int(max(1, min(b, per_cfg_budget / one / max(1, steps + warmup))))
        As = A[:s].contiguous()
        for _ in range(warmup):
            torch.geqrf(As)
        ts = []
        for _ in range(steps):
            t0 = time.perf_counter()
            torch.geqrf(As)
            ts.append(time.perf_counter() - t0)
        t = statistics.median(ts)
        per[name] = {"us_per_call": t / s * b * 1e6, "sample_matrices": s, "batch": b, "n": n,
                     "timed_calls": steps, "warmup_calls": warmup}
        samples.append(f"{name}:{s}/{b}")
    geo = gen.geomean([per[nm]["us_per_call"] for nm in names])
    pinfo = [ln.strip() for ln in torch.__config__.parallel_info().splitlines() if ln.strip()][:8]
    return {"value": geo, "unit": "us", "cores": threads, "kind": "reference",
            "sample": "torch.geqrf (LAPACK sgeqrf), median of " + str(steps) + " calls after " + str(warmup)
                      + " warm-up, on " + ", ".join(samples) + " matrices per config (scaled to the full batch)",
            "per_config": per, "torch_threads": torch.get_num_threads(), "logical_cpus": os.cpu_count(),
            "parallel_info": pinfo}


def run_reference(args, world, rank):
    if rank != 0:
        return
    t0 = time.perf_counter()
    names = args.configs
    inputs = {nm: gen.config_input(nm, device="cpu") for nm in names}
    cpu = cpu_reference(names, inputs, steps=max(1, args.steps), warmup=max(1, min(1, args.warmup)),
                        budget_s=args.cpu_budget_s)
    line = {
        "metric": "QR us/call geomean over configs C1-C5 (4n^3/3 flop per matrix)",
        "value": cpu["value"], "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sum(cpu["per_config"][nm]["us_per_call"] for nm in names) / 1e3,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded generators of configs C1-C5, CPU generator)",
        "config": {"workload": "C1..C5 batched QR, " + ",".join(
            f"{nm}=b{gen.CONFIGS[nm]['batch']}xn{gen.CONFIGS[nm]['n']}" for nm in names),
            "parallelism": "host CPU, physical cores"},
        "impl": "reference",
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "per_config": cpu["per_config"],
        "parallel_info": cpu["parallel_info"],
        "e2e": {"value": cpu["value"], "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- Triton arm
def triton_subprocess(args) -> dict:
    """Run ``bench.py --impl triton`` in its own process (the submission flips global TF32 flags
    on import) and return its JSON line, or an ``unavailable`` record."""
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "triton", "--steps", str(args.steps),
           "--warmup", str(args.warmup), "--configs", ",".join(args.configs)]
    if args.no_cases:
        cmd.append("--no-cases")
    env = dict(os.environ)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=args.triton_timeout_s, env=env)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"Triton arm exceeded {args.triton_timeout_s} s"}
    for line in reversed(res.stdout.strip().splitlines()):
        if line.startswith("{"):
            try:
                return json.loads(line)
            except ValueError:
                break
    return {"unavailable": f"Triton arm exited {res.returncode}: " + (res.stderr.strip().splitlines() or [""])[-1][:300]}


def run_triton(args, world, rank):
    """Time the reference's GPU submission, unmodified, through its own ``custom_kernel``.

    Procedure of the reference's harness (``harness/gpu_bench.py:164-170``, ``harness/eval.py:
    202-211``): a full warm-up pass over every workload first (Triton compilation and autotuning
    fall outside the timing), then per workload the mean of K calls, each after a 256 MiB L2
    flush, timed with CUDA events. Inputs are this benchmark's own (same seeds and generators as
    the ``ours`` arm). Each workload's output goes once through the FP64 gate.
    """
    if rank != 0:
        return
    if not os.path.exists(TRITON_REF_FILE):
        print(json.dumps({"impl": "triton", "unavailable": "baseline/_ref/submission.py not staged (run "
                          "__graft_entry__.build() where the reference tree is present)"}), flush=True)
        return
    import importlib.util

    from qr_v2_b200_kernel_b200 import checker

    t0 = time.perf_counter()
    spec = importlib.util.spec_from_file_location("reference_submission", TRITON_REF_FILE)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    kernel = mod.custom_kernel
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    work = [(nm, lambda nm=nm: gen.config_input(nm, device=dev)) for nm in args.configs]
    if not args.no_cases:
        work += [(case_label(c), lambda c=c: gen.generate_input(**c, device=dev)) for c in gen.REFERENCE_BENCH_CASES]
    for _, make in work:  # full warm-up pass
        A = make()
        for _ in range(max(1, args.warmup)):
            kernel(A)
        torch.cuda.synchronize()
        del A
    warm_s = time.perf_counter() - t0
    per = {}
    for label, make in work:
        A = make()
        H, tau = kernel(A)
        chk = checker.check(A, H, tau)
        del H, tau
        ts = time_device(lambda: kernel(A), args.steps, 0, flush)
        us = statistics.mean(ts)
        per[label] = {"us_per_call": us, "ok": chk["ok"], "sfr": chk.get("scaled_factor_residual"),
                      "batch": int(A.shape[0]), "n": int(A.shape[-1])}
        del A
    cfg_names = [nm for nm in args.configs]
    case_names = [lb for lb, _ in work if lb not in cfg_names]
    line = {
        "impl": "triton", "source": "reference submission.py (unmodified copy in baseline/_ref)",
        "value": gen.geomean([per[nm]["us_per_call"] for nm in cfg_names]), "unit": "us",
        "per_config": {nm: per[nm] for nm in cfg_names},
        "per_case": {lb: per[lb] for lb in case_names},
        "per_case_geomean_us": gen.geomean([per[lb]["us_per_call"] for lb in case_names]) if case_names else None,
        "steps": args.steps, "warmup_pass_s": warm_s, "wall_s": time.perf_counter() - t0,
        "tf32_flags_after_import": bool(torch.backends.cuda.matmul.allow_tf32),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "triton"], default="ours")
    ap.add_argument("--configs", default=",".join(CONFIG_ORDER))
    ap.add_argument("--cpu-budget-s", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-triton", action="store_true")
    ap.add_argument("--no-cases", action="store_true")
    ap.add_argument("--triton-timeout-s", type=float, default=900.0)
    args = ap.parse_args()
    args.configs = [c.strip() for c in args.configs.split(",") if c.strip()]
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.impl == "triton":
        run_triton(args, world, rank)
        return
    dist = init_dist(world, local)
    try:
        run_ours(args, world, rank, local, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
