"""Input generators: bit-exact with the reference generator on CPU; benchmark configs' structure."""

import numpy as np
import pytest
import torch

from qr_v2_b200_kernel_b200 import gen


def test_reference_generator_bit_exact(golden):
    z, meta = golden
    for c in meta["cases"]:
        a = gen.generate_input(**c["args"], device="cpu")
        assert np.array_equal(a.numpy(), z[c["key"] + "_A"]), c["args"]


def test_reference_case_lists():
    assert len(gen.REFERENCE_BENCH_CASES) == 12 and len(gen.REFERENCE_TEST_CASES) == 22
    with pytest.raises(ValueError):
        gen.generate_input(1, 4, 0, 0, case="nope", device="cpu")


def test_config_shapes_small():
    for name in ("C1", "C2", "C5"):
        a = gen.config_input(name, device="cpu", batch=2, n=16)
        assert a.shape == (2, 16, 16) and a.dtype == torch.float32 and a.is_contiguous()


def test_lowrank_cluster_spectrum():
    n = 64
    g = torch.Generator().manual_seed(2)
    s = gen.lowrank_cluster_spectrum(n, g, "cpu")
    k = 7 * n // 8
    assert torch.allclose(s[:k], torch.pow(10.0, -6.0 * torch.arange(k, dtype=torch.float64) / n))
    clu = s[k:k + (n - k) // 2]
    assert ((clu > 0.99e-3) & (clu < 1.01e-3)).all()
    assert (s[k + (n - k) // 2:] == 0).all()
    a = gen.config_input("C3", device="cpu", batch=2, n=n)
    sv = torch.linalg.svdvals(a.double())[0]
    ref = torch.sort(s, descending=True).values
    # the cluster's +-1% jitter comes from the config's own generator state, hence atol 2e-5
    assert torch.allclose(sv, ref, rtol=1e-3, atol=2e-5)
    assert (sv[-(n - k - (n - k) // 2):] < 1e-6).all()  # exact zeros up to float32 rounding


def test_rowscale_collinear():
    a = gen.config_input("C4", device="cpu", batch=4, n=64)
    assert a.shape == (4, 64, 64)
    rn = a.abs().amax(dim=-1)
    ratio = rn.amax(dim=-1) / rn.amin(dim=-1)
    assert (ratio > 1e3).all()  # rows span several decades
    d = (a[2:, :, -16:] - a[2:, :, :1]).abs().amax(dim=1) / a[2:, :, :1].abs().amax(dim=1)
    assert (d < 1e-4).all()  # second half: last 16 columns nearly equal column 0
    d0 = (a[:2, :, -16:] - a[:2, :, :1]).abs().amax()
    assert d0 > 1.0


def test_flops_and_bytes():
    assert gen.flops_per_call(640, 512) == pytest.approx(1.1453e11, rel=1e-3)
    assert gen.min_hbm_bytes(640, 512) == pytest.approx(1.342e9, rel=2e-3)
    assert gen.geomean([1, 100]) == pytest.approx(10.0)
