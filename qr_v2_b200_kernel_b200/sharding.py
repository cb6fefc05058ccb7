"""Batch sharding of the QR over several GPUs of one node: host-side split and gather only.

Matrices are independent, so the batch is cut into contiguous slices, one per GPU, and no
collective touches the data path. Two ways to drive it:

* one process per GPU (torchrun): each rank factors ``shard_range(batch, world, rank)`` of
  the batch; ``gather_shards`` (a ``torch.distributed`` all-gather) is only needed when every
  rank wants the whole result;
* one process, several GPUs: ``custom_kernel_multi(A, devices)`` copies each slice to its
  device, enqueues the factorisation on that device's current stream and copies the results
  back to ``A``'s device (peer copies over NVLink when ``A`` is on a GPU).

Per-matrix results are bitwise identical to a single-GPU call: the kernels' work split depends
only on the matrix order, never on the batch size.
"""

from __future__ import annotations

import torch

__all__ = ["shard_range", "custom_kernel_multi", "gather_shards"]


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of the batch for ``rank`` (ceil split; trailing ranks may be empty)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("need 0 <= rank < world")
    per = -(-batch // world) if batch > 0 else 0
    lo = min(batch, rank * per)
    hi = min(batch, lo + per)
    return lo, hi


def custom_kernel_multi(A: torch.Tensor, devices: list[int] | None = None):
    """Factor ``A`` (batch, n, n) with its batch spread over ``devices``; returns (H, tau) on A's device."""
    from .api import custom_kernel

    if devices is None:
        devices = list(range(torch.cuda.device_count()))
    if not devices:
        raise RuntimeError("no CUDA device available (no CPU fallback)")
    batch, n = int(A.shape[0]), int(A.shape[-1])
    out_dev = A.device
    H = torch.empty((batch, n, n), dtype=torch.float32, device=out_dev)
    tau = torch.empty((batch, n), dtype=torch.float32, device=out_dev)
    pending = []
    for r, dev in enumerate(devices):
        lo, hi = shard_range(batch, len(devices), r)
        if hi <= lo:
            continue
        with torch.cuda.device(dev):
            a = A[lo:hi].to(f"cuda:{dev}", non_blocking=True)
            h, t = custom_kernel(a)
            pending.append((lo, hi, h, t))
    for lo, hi, h, t in pending:
        H[lo:hi].copy_(h, non_blocking=True)
        tau[lo:hi].copy_(t, non_blocking=True)
    return H, tau


def gather_shards(local: torch.Tensor, batch: int, group=None) -> torch.Tensor:
    """All-gather per-rank slices (cut by ``shard_range``) into the full batch on every rank."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    per = -(-batch // world)
    shape = (per,) + tuple(local.shape[1:])
    padded = torch.zeros(shape, dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat(parts, dim=0)[:batch]
