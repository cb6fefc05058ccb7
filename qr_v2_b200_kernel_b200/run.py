"""Run the QR operator on one workload config, for profiling and quick timing.

    python -m qr_v2_b200_kernel_b200.run --config C2 [--batch 160] [--calls 2] [--check] [--breakdown]

Builds the config's seeded input on the GPU, makes ``--calls`` calls of ``custom_kernel``
and prints the CUDA-event time of the last one. ``--breakdown`` prints the per-kernel
totals of one profiled call.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import checker, custom_kernel, gen, profile


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="C2", choices=sorted(gen.CONFIGS))
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--n", type=int, default=None)
    ap.add_argument("--calls", type=int, default=2)
    ap.add_argument("--check", action="store_true")
    ap.add_argument("--breakdown", action="store_true")
    a = ap.parse_args()
    A = gen.config_input(a.config, device="cuda", batch=a.batch, n=a.n)
    b, n = int(A.shape[0]), int(A.shape[-1])
    us = None
    for _ in range(a.calls):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        H, tau = custom_kernel(A)
        e.record()
        e.synchronize()
        us = s.elapsed_time(e) * 1e3
    out = {"config": a.config, "batch": b, "n": n, "us_last_call": us,
           "tflops": gen.flops_per_call(b, n) / us / 1e6 if us else None}
    if a.check:
        r = checker.check(A, H, tau)
        out.update(ok=r["ok"], scaled_factor_residual=r.get("scaled_factor_residual"),
                   scaled_orthogonality_residual=r.get("scaled_orthogonality_residual"))
    if a.breakdown:
        out["kernels"] = profile.kernel_breakdown(A, steps=1)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
