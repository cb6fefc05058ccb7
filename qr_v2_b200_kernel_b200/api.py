"""``custom_kernel(data) -> (H, tau)``: the reference's operator API over the qrb200 C ABI.

Mirrors ``submission.custom_kernel`` (Raymondlol/qr-v2-b200-kernel ``submission.py:560-596``)
as the harness calls it (``harness/eval.py:189-211``):

* input: a ``(batch, n, n)`` float32 CUDA tensor; it is never modified;
* output: fresh ``H (batch, n, n)`` and ``tau (batch, n)`` float32 tensors on the input's
  device, in the ``torch.geqrf`` layout (R = triu(H), unit-lower reflectors below the
  diagonal), all finite for finite input (``harness/reference.py:175-204``);
* the work is enqueued on the current torch CUDA stream of the input's device with no host
  synchronisation, so CUDA events recorded around the call on that stream time it
  (``harness/eval.py:205-210``);
* errors raise: ``TypeError``/``ValueError`` for a wrong argument, ``RuntimeError`` for a
  non-CUDA input (there is no CPU path) and :class:`QRB200Error` for a failing C-ABI call.
  The reference instead falls back to ``torch.geqrf`` (``submission.py:572-596``); this
  operator never falls back.

Unlike the reference (``submission.py:50-55``) importing this module changes no global torch
flag.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

__all__ = ["custom_kernel", "geqrf", "workspace_bytes"]

_ws_lock = threading.Lock()
_ws_cache: dict[tuple[int, int], torch.Tensor] = {}


def workspace_bytes(batch: int, n: int) -> int:
    """Scratch bytes one call needs for ``(batch, n)``."""
    return int(_lib.load().qrb200_workspace_bytes(int(batch), int(n)))


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor | None:
    """Callee-owned scratch, cached per (device, stream) and grown on demand.

    Calls on one stream are ordered, so they may share it; another stream gets its own.
    """
    if nbytes == 0:
        return None
    key = (device.index, stream)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
        return buf


def geqrf(A: torch.Tensor, H: torch.Tensor, tau: torch.Tensor) -> None:
    """Factor ``A`` into caller-provided ``H`` and ``tau`` (same device, contiguous float32)."""
    lib = _lib.load()
    batch, n = int(A.shape[0]), int(A.shape[-1])
    if batch == 0 or n == 0:
        return
    abs_ = int(A.stride(0)) if batch > 1 else n * n
    with torch.cuda.device(A.device):
        stream = torch.cuda.current_stream(A.device).cuda_stream
        need = workspace_bytes(batch, n)
        ws = _workspace(A.device, stream, need)
        st = lib.qrb200_geqrf_f32(
            ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(H.data_ptr()), ctypes.c_void_p(tau.data_ptr()),
            batch, n, abs_,
            ctypes.c_void_p(ws.data_ptr() if ws is not None else 0),
            ws.numel() if ws is not None else 0,
            ctypes.c_void_p(stream))
    _lib.check(st, "geqrf_f32")


def custom_kernel(data: torch.Tensor):
    """Batched Householder QR: ``(batch, n, n)`` float32 CUDA -> ``(H, tau)``."""
    A = data
    if not isinstance(A, torch.Tensor):
        raise TypeError("custom_kernel expects a torch.Tensor")
    if A.dim() != 3 or A.shape[-1] != A.shape[-2]:
        raise ValueError(f"expected a (batch, n, n) tensor, got shape {tuple(A.shape)}")
    if A.dtype != torch.float32:
        raise TypeError(f"expected torch.float32, got {A.dtype}")
    if not A.is_cuda:
        raise RuntimeError("qrb200 runs on CUDA tensors only (no CPU fallback)")
    batch, n = int(A.shape[0]), int(A.shape[-1])
    if A.stride(-1) != 1 or A.stride(-2) != n or (batch > 1 and A.stride(0) < n * n):
        A = A.contiguous()
    H = torch.empty((batch, n, n), dtype=torch.float32, device=A.device)
    tau = torch.empty((batch, n), dtype=torch.float32, device=A.device)
    geqrf(A, H, tau)
    return H, tau
