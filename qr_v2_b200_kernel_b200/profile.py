"""Per-kernel timing of one QR call through ``qrb200_profile_geqrf_f32`` (CUDA events).

Used by bench.py for the live roofline of the dominant kernel: each launch is bracketed by
an event pair on the launching stream, so per-kind totals are device durations.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .api import _workspace, workspace_bytes


def kernel_breakdown(A: torch.Tensor, steps: int = 1) -> list[dict]:
    """Average per-call totals for each kernel kind over ``steps`` profiled calls."""
    lib = _lib.load()
    batch, n = int(A.shape[0]), int(A.shape[-1])
    H = torch.empty_like(A)
    tau = torch.empty((batch, n), dtype=torch.float32, device=A.device)
    stream = torch.cuda.current_stream(A.device).cuda_stream
    ws = _workspace(A.device, workspace_bytes(batch, n))
    agg: dict[str, dict] = {}
    for _ in range(steps):
        stats = (_lib.KernelStat * 16)()
        cnt = ctypes.c_int(0)
        st = lib.qrb200_profile_geqrf_f32(
            ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(H.data_ptr()), ctypes.c_void_p(tau.data_ptr()),
            batch, n, n * n, ctypes.c_void_p(ws.data_ptr() if ws is not None else 0),
            ws.numel() if ws is not None else 0, ctypes.c_void_p(stream), stats, 16, ctypes.byref(cnt))
        _lib.check(st, "profile_geqrf_f32")
        for i in range(cnt.value):
            s = stats[i]
            name = s.name.decode()
            d = agg.setdefault(name, dict(name=name, launches=0, ms=0.0, flops=0.0, bytes=0.0,
                                          bound="tensor" if s.tensor_bound else "hbm"))
            d["launches"] += s.launches
            d["ms"] += s.ms
            d["flops"] += s.flops
            d["bytes"] += s.bytes
    out = []
    total = sum(d["ms"] for d in agg.values()) or 1.0
    for d in agg.values():
        for key in ("launches", "ms", "flops", "bytes"):
            d[key] = d[key] / steps
        d["share"] = d["ms"] / (total / steps)
        out.append(d)
    return sorted(out, key=lambda d: -d["ms"])
