"""Seeded synthetic inputs: the reference's test-case generators and the five benchmark configs.

Two families live here.

1. ``generate_input(batch, n, cond, seed, case)`` reproduces the competition generator the
   reference is graded on (``harness/reference.py:132-149`` with the per-case transforms of
   ``:37-97`` and the heterogeneous "mixed" batch of ``:100-129``). The draw order is kept
   identical so that, on the same device type, the tensors are bit-for-bit the reference's
   (pinned on CPU by ``tests/test_generators.py`` against ``tests/golden/``).

2. ``config_input(name)`` builds the five benchmark workloads C1..C5 (batch, n, structure):
   dense Gaussian C1/C2/C5, the rank-deficient clustered-spectrum C3 and the row-scaled /
   near-collinear C4. These have no counterpart in the reference; the constants are the
   workload definition.

Everything is generated with a ``torch.Generator`` on the requested device, stored as
contiguous float32 (orthogonal factors are formed in float64 first).
"""

from __future__ import annotations

import math

import torch

__all__ = ["generate_input", "config_input", "CONFIGS", "REFERENCE_BENCH_CASES", "REFERENCE_TEST_CASES"]

_F32_EPS = torch.finfo(torch.float32).eps

# Heterogeneous-batch profile table and weights (harness/reference.py:33-36): the labels
# index this tuple, so order and weights must match the reference for identical draws.
MIXED_PROFILES = ("dense", "rankdef", "nearrank", "clustered", "band", "rowscale", "nearcollinear")
MIXED_WEIGHTS = (6.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0)


def _col_scale(a: torch.Tensor, cond: int) -> torch.Tensor:
    """Geometric column scaling 1 .. 10^-cond (harness/reference.py:16-22)."""
    if not cond:
        return a.contiguous()
    n = a.shape[-1]
    return a * torch.logspace(0.0, -float(cond), n, device=a.device, dtype=torch.float32)


def _case(a: torch.Tensor, case: str, cond: int, gen: torch.Generator) -> torch.Tensor:
    """One conditioning profile applied to a drawn base batch (harness/reference.py:37-97)."""
    m, n = a.shape[0], a.shape[-1]
    dev = a.device
    f32 = torch.float32
    if case == "dense":
        return _col_scale(a, cond)
    if case == "upper":
        a = torch.triu(a)
        a.diagonal(dim1=-2, dim2=-1).add_(torch.linspace(1.0, 0.25, n, device=dev, dtype=f32))
        return _col_scale(a, cond)
    if case == "diagonal":
        d = torch.randn((m, n), device=dev, dtype=f32, generator=gen)
        mag = torch.logspace(0.0, -float(max(cond, 2)), n, device=dev, dtype=f32)
        return torch.diag_embed(d.sign().clamp(min=0.0).mul(2.0).sub(1.0) * mag)
    if case == "rankdef":
        a[:, :, max(1, (3 * n) // 4):] = 0.0
        return _col_scale(a, cond)
    if case == "nearrank":
        r = max(1, (3 * n) // 4)
        tail = n - r
        if tail > 0:
            noise = torch.randn((m, n, tail), device=dev, dtype=f32, generator=gen)
            a[:, :, r:] = a[:, :, :tail] + 1.0e-5 * noise
        return _col_scale(a, cond)
    if case == "clustered":
        s = torch.ones((n,), device=dev, dtype=f32)
        s[n // 2:] = 4.0 * _F32_EPS
        if n >= 8:
            s[max(0, n // 2 - 2):min(n, n // 2 + 2)] = torch.sqrt(torch.tensor(_F32_EPS, device=dev))
        return a * s
    if case == "band":
        bw = max(2, min(32, n // 32))
        idx = torch.arange(n, device=dev)
        a = a * ((idx[:, None] - idx[None, :]).abs() <= bw)
        a.diagonal(dim1=-2, dim2=-1).add_(torch.linspace(1.0, 0.5, n, device=dev, dtype=f32))
        return _col_scale(a, cond)
    if case == "nearcollinear":
        base = torch.randn((m, n, 1), device=dev, dtype=f32, generator=gen)
        noise = torch.randn((m, n, n), device=dev, dtype=f32, generator=gen)
        return _col_scale(base.expand(m, n, n) + 1.0e-4 * noise, cond)
    if case == "rowscale":
        s = torch.logspace(0.0, -float(max(cond, 4)), n, device=dev, dtype=f32)
        return s.reshape(1, n, 1) * a
    raise ValueError(f"unknown QR test case: {case}")


def _mixed(a: torch.Tensor, cond: int, gen: torch.Generator) -> torch.Tensor:
    """Per-matrix random profile assignment (harness/reference.py:100-129)."""
    m = a.shape[0]
    dev = a.device
    labels = torch.multinomial(torch.tensor(MIXED_WEIGHTS, dtype=torch.float32, device=dev), m,
                               replacement=True, generator=gen)
    if m >= 2:
        dense = labels == 0
        if not bool(dense.any()):
            labels[int(torch.randint(0, m, (1,), device=dev, generator=gen))] = 0
        elif bool(dense.all()):
            pos = int(torch.randint(0, m, (1,), device=dev, generator=gen))
            labels[pos] = int(torch.randint(1, len(MIXED_PROFILES), (1,), device=dev, generator=gen))
    for k, prof in enumerate(MIXED_PROFILES):
        sel = labels == k
        if bool(sel.any()):
            a[sel] = _case(a[sel], prof, cond, gen)
    return a


def generate_input(batch: int, n: int, cond: int, seed: int, case: str = "dense",
                   device: str | torch.device | None = None) -> torch.Tensor:
    """The reference's seeded test input (harness/reference.py:132-149) as (batch, n, n) fp32."""
    if batch <= 0 or n <= 0 or cond < 0:
        raise ValueError("batch and n must be positive and cond non-negative")
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    case = case.lower()
    a = torch.randn((batch, n, n), device=device, dtype=torch.float32, generator=gen)
    a = _mixed(a, cond, gen) if case == "mixed" else _case(a, case, cond, gen)
    return a.contiguous()


# The reference's 12 scored cases (harness/lab.py:33-46) and 22 correctness cases
# (harness/lab.py:48-71); used as extra stress cases by the tests.
REFERENCE_BENCH_CASES = [
    dict(batch=20, n=32, cond=1, seed=43214),
    dict(batch=40, n=176, cond=1, seed=423011),
    dict(batch=40, n=352, cond=1, seed=123456),
    dict(batch=640, n=512, cond=2, seed=1029),
    dict(batch=60, n=1024, cond=2, seed=75342),
    dict(batch=8, n=2048, cond=1, seed=224466),
    dict(batch=2, n=4096, cond=1, seed=32412),
    dict(batch=640, n=512, cond=2, seed=770001, case="mixed"),
    dict(batch=60, n=1024, cond=2, seed=770002, case="mixed"),
    dict(batch=640, n=512, cond=0, seed=770003, case="rankdef"),
    dict(batch=640, n=512, cond=0, seed=770004, case="clustered"),
    dict(batch=60, n=1024, cond=0, seed=770005, case="nearrank"),
]
REFERENCE_TEST_CASES = [
    dict(batch=20, n=32, cond=1, seed=53124),
    dict(batch=40, n=176, cond=1, seed=3321),
    dict(batch=40, n=352, cond=1, seed=1200),
    dict(batch=16, n=512, cond=2, seed=32523),
    dict(batch=4, n=1024, cond=2, seed=4327),
    dict(batch=1, n=4096, cond=1, seed=75342),
    dict(batch=16, n=512, cond=4, seed=32524, case="dense"),
    dict(batch=16, n=512, cond=0, seed=32525, case="rankdef"),
    dict(batch=16, n=512, cond=0, seed=32526, case="clustered"),
    dict(batch=16, n=512, cond=0, seed=32527, case="band"),
    dict(batch=16, n=512, cond=0, seed=32528, case="rowscale"),
    dict(batch=16, n=512, cond=0, seed=32529, case="nearcollinear"),
    dict(batch=4, n=1024, cond=4, seed=4328, case="dense"),
    dict(batch=4, n=1024, cond=0, seed=4329, case="rankdef"),
    dict(batch=4, n=1024, cond=0, seed=4330, case="nearrank"),
    dict(batch=4, n=1024, cond=0, seed=4331, case="clustered"),
    dict(batch=2, n=2048, cond=2, seed=224466, case="dense"),
    dict(batch=2, n=2048, cond=0, seed=224467, case="rankdef"),
    dict(batch=1, n=4096, cond=0, seed=75343, case="upper"),
    dict(batch=16, n=512, cond=2, seed=32530, case="mixed"),
    dict(batch=4, n=1024, cond=2, seed=4332, case="mixed"),
    dict(batch=2, n=2048, cond=2, seed=224468, case="mixed"),
]


# ----------------------------------------------------------------------------------------
# The five benchmark workloads.
# ----------------------------------------------------------------------------------------
CONFIGS = {
    "C1": dict(batch=8, n=128, kind="gaussian", seed=0),
    "C2": dict(batch=640, n=512, kind="gaussian", seed=1),
    "C3": dict(batch=64, n=1024, kind="lowrank_cluster", seed=2),
    "C4": dict(batch=8, n=2048, kind="rowscale_collinear", seed=3),
    "C5": dict(batch=2, n=4096, kind="gaussian", seed=5),
}


def haar_orthogonal(batch: int, n: int, gen: torch.Generator, device) -> torch.Tensor:
    """Haar-distributed orthogonal matrices (float64): QR of a Gaussian with diag(R) > 0.

    On a CUDA device (n % 4 == 0) the QR is this repository's own: ``custom_kernel`` on the
    Gaussian (drawn in float64, factored in float32) and Q from ``householder_product``, both
    on the B200, so benchmark set-up does not leave the GPU or call cuSOLVER. Q is then
    orthogonal to float32 accuracy; ``U diag(s) V^T`` built from such factors has the singular
    values ``s (1 + O(n eps32))`` (relative perturbations), so the spectrum's zeros, cluster and
    decay are kept. On the CPU: float64 ``torch.linalg.qr``.
    """
    g = torch.randn((batch, n, n), device=device, dtype=torch.float64, generator=gen)
    dev = torch.device(device)
    if dev.type == "cuda" and n % 4 == 0:
        from .api import custom_kernel, householder_product

        H, tau = custom_kernel(g.float())
        q = householder_product(H, tau).double()
        r_diag = torch.diagonal(H, dim1=-2, dim2=-1).double()
    else:
        q, r = torch.linalg.qr(g)
        r_diag = torch.diagonal(r, dim1=-2, dim2=-1)
    d = torch.sign(r_diag)
    d = torch.where(d == 0, torch.ones_like(d), d)
    return q * d.unsqueeze(-2)


def lowrank_cluster_spectrum(n: int, gen: torch.Generator, device) -> torch.Tensor:
    """C3 singular values (float64, length n).

    s_i = 10^(-6 i / n) for the first 7n/8 indices; of the last n/8 the first half is a
    cluster at 1e-3 (1 + 0.01 U(-1, 1)) and the rest are exactly zero.
    """
    k = (7 * n) // 8
    s = torch.zeros(n, dtype=torch.float64, device=device)
    i = torch.arange(k, dtype=torch.float64, device=device)
    s[:k] = torch.pow(10.0, -6.0 * i / n)
    tail = n - k
    nclu = tail // 2
    if nclu > 0:
        jit = torch.rand(nclu, dtype=torch.float64, device=device, generator=gen) * 2.0 - 1.0
        s[k:k + nclu] = 1.0e-3 * (1.0 + 0.01 * jit)
    return s


def _lowrank_cluster(batch: int, n: int, gen: torch.Generator, device) -> torch.Tensor:
    u = haar_orthogonal(batch, n, gen, device)
    v = haar_orthogonal(batch, n, gen, device)
    s = lowrank_cluster_spectrum(n, gen, device)
    a = (u * s.unsqueeze(-2)) @ v.transpose(-1, -2)
    return a.to(torch.float32).contiguous()


def _rowscale(batch: int, n: int, gen: torch.Generator, device) -> torch.Tensor:
    """Rows of an iid N(0,1) matrix times 10^u, u ~ U(-4, 4) per row."""
    a = torch.randn((batch, n, n), device=device, dtype=torch.float32, generator=gen)
    u = torch.rand((batch, n, 1), device=device, dtype=torch.float32, generator=gen) * 8.0 - 4.0
    return (a * torch.pow(10.0, u)).contiguous()


def _collinear(a: torch.Tensor, gen: torch.Generator, ncols: int = 16) -> torch.Tensor:
    """Near-collinear variant: the last ``ncols`` columns = column 0 + 1e-6 N(0,1)."""
    b, n, _ = a.shape
    k = min(ncols, n - 1)
    noise = torch.randn((b, n, k), device=a.device, dtype=torch.float32, generator=gen)
    a = a.clone()
    a[:, :, n - k:] = a[:, :, :1] + 1.0e-6 * noise
    return a.contiguous()


def config_input(name: str, device: str | torch.device | None = None, batch: int | None = None,
                 n: int | None = None) -> torch.Tensor:
    """Benchmark workload ``name`` in {C1..C5}; ``batch``/``n`` override for reduced tests.

    C4 mixes its two variants in one batch: the first half row-scaled (seed 3), the second
    half row-scaled then near-collinear (seed 4).
    """
    cfg = CONFIGS[name]
    batch = cfg["batch"] if batch is None else batch
    n = cfg["n"] if n is None else n
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    gen = torch.Generator(device=device)
    gen.manual_seed(cfg["seed"])
    kind = cfg["kind"]
    if kind == "gaussian":
        return torch.randn((batch, n, n), device=device, dtype=torch.float32, generator=gen)
    if kind == "lowrank_cluster":
        return _lowrank_cluster(batch, n, gen, device)
    if kind == "rowscale_collinear":
        h = batch - batch // 2
        a0 = _rowscale(h, n, gen, device)
        gen4 = torch.Generator(device=device)
        gen4.manual_seed(4)
        a1 = _collinear(_rowscale(batch - h, n, gen4, device), gen4)
        return torch.cat([a0, a1], dim=0).contiguous()
    raise ValueError(kind)


def flops_per_call(batch: int, n: int) -> float:
    """Algorithmic FLOP count of one batched call: 4 n^3 / 3 per matrix."""
    return batch * 4.0 * n ** 3 / 3.0


def min_hbm_bytes(batch: int, n: int) -> float:
    """HBM floor of one call: read A, write H and tau (fp32)."""
    return batch * (8.0 * n * n + 4.0 * n)


def geomean(xs) -> float:
    xs = list(xs)
    return math.exp(sum(math.log(x) for x in xs) / len(xs))
