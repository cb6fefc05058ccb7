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
  non-CUDA input (there is no CPU path) and :class:`QRB200Error` for a failing C-ABI call or
  for a device-side wait that expired in an earlier call on the same device (checked at the
  start of every call from a mapped host word, without synchronising).
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

__all__ = ["custom_kernel", "custom_kernel_host", "geqrf", "workspace_bytes", "householder_product", "ormqr"]

_ws_lock = threading.Lock()


def workspace_bytes(batch: int, n: int) -> int:
    """Scratch bytes one call needs for ``(batch, n)``."""
    return int(_lib.load().qrb200_workspace_bytes(int(batch), int(n)))


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """Callee-owned scratch for one call, from the torch caching allocator on the current stream.

    The tensor is released when the call returns (after the work is enqueued); the allocator
    hands its block only to later work on the same stream, or to another stream once this
    stream's work is done, so scratch is never shared by unordered calls. After the first call
    of a shape this is a cache hit, not a device allocation.
    """
    if nbytes == 0:
        return None
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _check_operands(A: torch.Tensor, H: torch.Tensor, tau: torch.Tensor) -> tuple[int, int, int]:
    """Validate :func:`geqrf`'s operands before any pointer reaches the C ABI."""
    for name, t in (("A", A), ("H", H), ("tau", tau)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.dtype != torch.float32:
            raise TypeError(f"{name} must be torch.float32, got {t.dtype}")
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor (qrb200 has no CPU path)")
        if t.device != A.device:
            raise ValueError(f"{name} is on {t.device}, A on {A.device}")
    if A.dim() != 3 or A.shape[-1] != A.shape[-2]:
        raise ValueError(f"A must be (batch, n, n), got {tuple(A.shape)}")
    batch, n = int(A.shape[0]), int(A.shape[-1])
    if tuple(H.shape) != (batch, n, n) or not H.is_contiguous():
        raise ValueError(f"H must be a contiguous ({batch}, {n}, {n}) tensor, got {tuple(H.shape)}")
    if tuple(tau.shape) != (batch, n) or not tau.is_contiguous():
        raise ValueError(f"tau must be a contiguous ({batch}, {n}) tensor, got {tuple(tau.shape)}")
    if batch > 0 and n > 0 and (A.stride(-1) != 1 or A.stride(-2) != n or (batch > 1 and A.stride(0) < n * n)):
        raise ValueError("A must have unit column stride, row stride n and batch stride >= n*n")
    abs_ = int(A.stride(0)) if batch > 1 else n * n
    return batch, n, abs_


def geqrf(A: torch.Tensor, H: torch.Tensor, tau: torch.Tensor) -> None:
    """Factor ``A`` into caller-provided ``H`` and ``tau``.

    ``A``: (batch, n, n) float32 CUDA, rows contiguous (unit column stride, row stride n, any
    batch stride >= n*n); ``H`` (batch, n, n) and ``tau`` (batch, n): contiguous float32 on A's
    device. Raises ``TypeError``/``ValueError``/``RuntimeError`` for bad operands before
    anything is launched, :class:`QRB200Error` for a failing C-ABI call or a device-side wait
    that expired in an earlier call on this device.
    """
    batch, n, abs_ = _check_operands(A, H, tau)
    lib = _lib.load()
    if batch == 0 or n == 0:
        return
    with torch.cuda.device(A.device):
        _lib.check_last_status()
        stream = torch.cuda.current_stream(A.device).cuda_stream
        need = workspace_bytes(batch, n)
        ws = _workspace(A.device, need)
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


def _check_factors(H: torch.Tensor, tau: torch.Tensor) -> tuple[int, int]:
    """(H, tau) as :func:`custom_kernel` returns them: contiguous float32 CUDA, n % 4 == 0."""
    for name, t in (("H", H), ("tau", tau)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.dtype != torch.float32:
            raise TypeError(f"{name} must be torch.float32, got {t.dtype}")
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor (qrb200 has no CPU path)")
    if H.dim() != 3 or H.shape[-1] != H.shape[-2]:
        raise ValueError(f"H must be (batch, n, n), got {tuple(H.shape)}")
    batch, n = int(H.shape[0]), int(H.shape[-1])
    if tuple(tau.shape) != (batch, n):
        raise ValueError(f"tau must be ({batch}, {n}), got {tuple(tau.shape)}")
    if tau.device != H.device:
        raise ValueError(f"tau is on {tau.device}, H on {H.device}")
    if n % 4 != 0:
        raise ValueError("the tensor-core Q application needs n % 4 == 0")
    return batch, n


def householder_product(H: torch.Tensor, tau: torch.Tensor) -> torch.Tensor:
    """``Q = H_0 H_1 ... H_{n-1}`` of square factors: ``torch.linalg.householder_product(H, tau)``
    on the B200 (the reference's checker step, ``harness/reference.py:206``).

    ``H`` (batch, n, n) and ``tau`` (batch, n) float32 CUDA as :func:`custom_kernel` returns
    them; n % 4 == 0. Returns a fresh (batch, n, n) tensor; enqueued on the current stream.
    """
    batch, n = _check_factors(H, tau)
    Q = torch.empty((batch, n, n), dtype=torch.float32, device=H.device)
    if batch == 0 or n == 0:
        return Q
    H, tau = H.contiguous(), tau.contiguous()
    lib = _lib.load()
    with torch.cuda.device(H.device):
        _lib.check_last_status()
        stream = torch.cuda.current_stream(H.device).cuda_stream
        need = int(lib.qrb200_apply_workspace_bytes(batch, n, n))
        ws = _workspace(H.device, need)
        st = lib.qrb200_orgqr_f32(ctypes.c_void_p(H.data_ptr()), ctypes.c_void_p(tau.data_ptr()),
                                  ctypes.c_void_p(Q.data_ptr()), batch, n, ctypes.c_void_p(ws.data_ptr()), need,
                                  ctypes.c_void_p(stream))
    _lib.check(st, "orgqr_f32")
    return Q


def ormqr(H: torch.Tensor, tau: torch.Tensor, C: torch.Tensor, transpose: bool = False) -> torch.Tensor:
    """``Q^T C`` (``transpose=True``) or ``Q C`` for ``Q`` of the factors ``(H, tau)``:
    ``torch.ormqr(H, tau, C, left=True, transpose=transpose)`` on the B200.

    ``C``: (batch, n, nrhs) float32 on H's device, nrhs % 4 == 0. Returns a new tensor (C is not
    modified); enqueued on the current stream. Least squares: ``R x = (Q^T b)[:n]``.
    """
    batch, n = _check_factors(H, tau)
    if not isinstance(C, torch.Tensor) or C.dtype != torch.float32:
        raise TypeError("C must be a float32 torch.Tensor")
    if C.device != H.device:
        raise ValueError(f"C is on {C.device}, H on {H.device}")
    if C.dim() != 3 or int(C.shape[0]) != batch or int(C.shape[1]) != n:
        raise ValueError(f"C must be ({batch}, {n}, nrhs), got {tuple(C.shape)}")
    nrhs = int(C.shape[2])
    if nrhs % 4 != 0:
        raise ValueError("the tensor-core Q application needs nrhs % 4 == 0")
    out = C.contiguous().clone()
    if batch == 0 or n == 0 or nrhs == 0:
        return out
    H, tau = H.contiguous(), tau.contiguous()
    lib = _lib.load()
    with torch.cuda.device(H.device):
        _lib.check_last_status()
        stream = torch.cuda.current_stream(H.device).cuda_stream
        need = int(lib.qrb200_apply_workspace_bytes(batch, n, nrhs))
        ws = _workspace(H.device, need)
        st = lib.qrb200_ormqr_f32(ctypes.c_void_p(H.data_ptr()), ctypes.c_void_p(tau.data_ptr()),
                                  ctypes.c_void_p(out.data_ptr()), batch, n, nrhs, 1 if transpose else 0,
                                  ctypes.c_void_p(ws.data_ptr()), need, ctypes.c_void_p(stream))
    _lib.check(st, "ormqr_f32")
    return out


_chunk_streams: dict[int, list] = {}


def _host_chunks(batch: int, n: int) -> int:
    """Pieces a host-buffer call is cut into, by input size: one below 32 MB (the copies are
    short), two below 192 MB, four below 512 MB, else eight; at most one per matrix. Each piece
    runs on its own stream with its own look-ahead streams, so the pieces' factorisations
    overlap one another as well as the copies, and the call ends one piece's factorisation and
    copy-out after the last input byte arrives (measured on B200: C4 e2e 9.97 -> 8.27 ms with
    two pieces, C5 14.8 -> 13.3 ms, C3 11.0 -> 10.0 ms with four, C2 17.8 -> 16.3 ms with eight;
    more pieces than that lost: C3 10.0 ms with eight, C4 10.3 ms with four)."""
    nbytes = 4 * batch * n * n
    k = 1 if nbytes < (32 << 20) else (2 if nbytes < (192 << 20) else (4 if nbytes < (512 << 20) else 8))
    return max(1, min(k, batch))


def _streams(device: torch.device, count: int) -> list:
    with _ws_lock:
        ss = _chunk_streams.setdefault(device.index, [])
        while len(ss) < count:
            ss.append(torch.cuda.Stream(device=device))
        return ss[:count]


def custom_kernel_host(data: torch.Tensor, device=None, out=None, chunks: int | None = None):
    """Batched QR of a host-resident ``(batch, n, n)`` float32 tensor, results back on the host.

    The batch is cut into up to eight contiguous pieces, each on its own CUDA stream of
    ``device`` (default: the current device): copy in, factor (:func:`custom_kernel`), copy out,
    so the copies of one piece overlap the factorisations of the others, and the pieces'
    factorisations overlap one another (use pinned host memory for that). Every matrix is factored exactly as :func:`custom_kernel` would factor it (a
    matrix's arithmetic does not depend on its batch), so the results agree bit for bit.

    ``out`` may pass preallocated host tensors ``(H, tau)`` (pinned, ``(batch, n, n)`` and
    ``(batch, n)``); otherwise pinned ones are allocated. The call returns once the work is
    enqueued: the results are ready after the device's current stream is synchronised (all
    pieces are joined back into it).
    """
    A = data
    if not isinstance(A, torch.Tensor):
        raise TypeError("custom_kernel_host expects a torch.Tensor")
    if A.dim() != 3 or A.shape[-1] != A.shape[-2]:
        raise ValueError(f"expected a (batch, n, n) tensor, got shape {tuple(A.shape)}")
    if A.dtype != torch.float32:
        raise TypeError(f"expected torch.float32, got {A.dtype}")
    if A.is_cuda:
        raise ValueError("custom_kernel_host takes a host tensor; use custom_kernel for device tensors")
    if not torch.cuda.is_available():
        raise RuntimeError("qrb200 needs a CUDA device (no CPU fallback)")
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if dev.type != "cuda":
            raise ValueError(f"device must be a CUDA device, got {dev}")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
    batch, n = int(A.shape[0]), int(A.shape[-1])
    if out is None:
        H_host = torch.empty((batch, n, n), dtype=torch.float32, pin_memory=True)
        tau_host = torch.empty((batch, n), dtype=torch.float32, pin_memory=True)
    else:
        H_host, tau_host = out
        if tuple(H_host.shape) != (batch, n, n) or tuple(tau_host.shape) != (batch, n):
            raise ValueError("out tensors have the wrong shape")
    if batch == 0 or n == 0:
        return H_host, tau_host
    A = A.contiguous()
    k = max(1, min(int(chunks) if chunks else _host_chunks(batch, n), batch))
    bounds = [(batch * i // k, batch * (i + 1) // k) for i in range(k)]
    with torch.cuda.device(dev):
        if k == 1:  # nothing to overlap: stay on the current stream
            H, tau = custom_kernel(A.to(dev, non_blocking=True))
            H_host.copy_(H, non_blocking=True)
            tau_host.copy_(tau, non_blocking=True)
            return H_host, tau_host
        cur = torch.cuda.current_stream(dev)
        streams = _streams(dev, k)
        for s in streams:
            s.wait_stream(cur)
        for s, (lo, hi) in zip(streams, bounds):
            with torch.cuda.stream(s):
                dA = A[lo:hi].to(dev, non_blocking=True)
                H, tau = custom_kernel(dA)
                H_host[lo:hi].copy_(H, non_blocking=True)
                tau_host[lo:hi].copy_(tau, non_blocking=True)
            # dA, H and tau were allocated on s and are used only there, so the caching
            # allocator hands their memory to later work on s only.
        for s in streams:
            cur.wait_stream(s)
    return H_host, tau_host
