"""FP64 correctness gate for ``(H, tau)``, the reference's criteria restated with torch ops.

Follows ``harness/reference.py:189-273`` (Raymondlol/qr-v2-b200-kernel):

* ``Q = householder_product(H, tau)`` in FP32 (as the reference does), R = triu(H);
* per matrix ``||R - Q^T A||_1 <= 20 n eps32 ||A||_1`` (factor residual);
* batch max ``||Q^T Q - I||_1 <= 100 n eps32`` (orthogonality);
* informational reconstruction ``||QR - A||_1`` and ``||tril(Q^T A, -1)||_1``.

``compare_diag_r`` adds the R-diagonal agreement with ``torch.geqrf`` up to sign, within
the factor bound. Matrices are processed in chunks so an 8 x 2048^2 or 2 x 4096^2 batch
fits in device memory in FP64. This module checks results; it is not on the product path.
"""

from __future__ import annotations

import torch

EPS32 = torch.finfo(torch.float32).eps
FACTOR_RTOL_FACTOR = 20.0
ORTH_RTOL_FACTOR = 100.0


def _l1(x: torch.Tensor) -> torch.Tensor:
    return torch.linalg.matrix_norm(x, ord=1, dim=(-2, -1))


def _chunk(batch: int, n: int) -> int:
    return max(1, min(batch, (1 << 27) // max(1, n * n)))


def check(A: torch.Tensor, H: torch.Tensor, tau: torch.Tensor) -> dict:
    """Return a dict with ``ok``, ``message`` and the scaled residuals (reference names)."""
    batch, n, _ = A.shape
    out = dict(batch=batch, n=n, ok=False, message="")
    if not isinstance(H, torch.Tensor) or H.shape != (batch, n, n) or H.dtype != torch.float32:
        out["message"] = "H shape/dtype"
        return out
    if not isinstance(tau, torch.Tensor) or tau.shape != (batch, n) or tau.dtype != torch.float32:
        out["message"] = "tau shape/dtype"
        return out
    if H.device != A.device or tau.device != A.device:
        out["message"] = "device"
        return out
    if not (torch.isfinite(H).all() and torch.isfinite(tau).all()):
        out["message"] = "H or tau contains NaN or Inf"
        return out
    denom = EPS32 * max(n, 1)
    f_scaled, orth, recon, tri = [], [], [], []
    f_fail = []
    cs = _chunk(batch, n)
    eye = torch.eye(n, device=A.device, dtype=torch.float64)
    for b0 in range(0, batch, cs):
        a = A[b0:b0 + cs].double()
        q = torch.linalg.householder_product(H[b0:b0 + cs], tau[b0:b0 + cs]).double()
        r = torch.triu(H[b0:b0 + cs]).double()
        proj = q.transpose(-1, -2) @ a
        fres = _l1(r - proj)
        fscale = _l1(a)
        f_fail.append(fres > FACTOR_RTOL_FACTOR * n * EPS32 * fscale)
        f_scaled.append(fres / (denom * fscale.clamp_min(1e-30)))
        orth.append(_l1(q.transpose(-1, -2) @ q - eye).amax())
        recon.append((_l1(q @ r - a) / (denom * fscale.clamp_min(1e-30))).amax())
        tri.append((_l1(torch.tril(proj, diagonal=-1)) / (denom * fscale.clamp_min(1e-30))).amax())
        del a, q, r, proj
    f_scaled = torch.cat(f_scaled)
    f_fail = torch.cat(f_fail)
    orth_res = torch.stack(orth).amax()
    out.update(
        scaled_factor_residual=float(f_scaled.amax()),
        scaled_factor_residual_per_matrix=f_scaled.cpu(),
        scaled_orthogonality_residual=float(orth_res / denom),
        scaled_reconstruction_residual=float(torch.stack(recon).amax()),
        scaled_triangular_residual=float(torch.stack(tri).amax()),
    )
    if bool(f_fail.any()):
        worst = int(f_scaled.argmax())
        out["message"] = f"R - Q^T A too large: matrix={worst}, scaled={float(f_scaled[worst]):.3g}"
        return out
    if float(orth_res) > ORTH_RTOL_FACTOR * n * EPS32:
        out["message"] = f"Q not orthogonal enough: scaled={out['scaled_orthogonality_residual']:.3g}"
        return out
    out["ok"] = True
    out["message"] = (f"scaled_factor_residual={out['scaled_factor_residual']:.3g}; "
                      f"scaled_orthogonality_residual={out['scaled_orthogonality_residual']:.3g}")
    return out


def compare_diag_r(A: torch.Tensor, H: torch.Tensor, H_ref: torch.Tensor) -> dict:
    """|diag R| of ``H`` vs ``H_ref`` (e.g. torch.geqrf), scaled like the factor residual.

    ``scaled = max_i | |R_ii| - |Rref_ii| | / (n eps32 ||A||_1)``; passing means it stays
    within the factor bound of 20.
    """
    n = A.shape[-1]
    d = torch.diagonal(H, dim1=-2, dim2=-1).double().abs()
    dr = torch.diagonal(H_ref, dim1=-2, dim2=-1).double().abs()
    scale = _l1(A.double()).clamp_min(1e-30) * EPS32 * max(n, 1)
    scaled = ((d - dr).abs().amax(dim=-1) / scale)
    return dict(ok=bool((scaled <= FACTOR_RTOL_FACTOR).all()), scaled_max=float(scaled.amax()))
