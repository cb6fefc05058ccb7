"""qr_v2_b200_kernel_b200 -- batched Householder QR on B200 (sm_100a).

Public API (the reference's drop-in operator, ``submission.py:560-596``)::

    from qr_v2_b200_kernel_b200 import custom_kernel
    H, tau = custom_kernel(A)          # A: (batch, n, n) float32 CUDA tensor
    H, tau = custom_kernel_host(A)     # A on the host: copies overlapped with the factorisation
    Q = householder_product(H, tau)    # explicit Q (sorgqr), on the tensor cores
    X = ormqr(H, tau, B, transpose=True)   # Q^T B (sormqr)

Helpers: ``gen`` (seeded inputs), ``checker`` (the FP64 correctness gate),
``sharding`` (host-side batch split over several GPUs).
"""

from .api import custom_kernel, custom_kernel_host, geqrf, householder_product, ormqr, workspace_bytes  # noqa: F401

__version__ = "0.1.0"
