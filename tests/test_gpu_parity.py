"""CUDA path parity: the C-ABI operator against the oracle, the golden fixtures and the
reference correctness gate (harness/reference.py:189-273), on the B200.

Tolerances (floating point, from the north-star criteria):
* gate: per matrix ||triu(H) - Q^T A||_1 <= 20 n eps32 ||A||_1 and ||Q^T Q - I||_1 <= 100 n eps32;
* |diag R| vs torch.geqrf and vs the oracle within the factor bound (scaled <= 20);
* elementwise H vs the oracle / LAPACK within 20 n eps32 ||A||_1 on well-conditioned inputs.
"""

import numpy as np
import pytest
import torch

import oracle
from qr_v2_b200_kernel_b200 import checker, custom_kernel, gen

pytestmark = pytest.mark.gpu

WELL_CONDITIONED = {"dense", "band", "upper", "diagonal", "rowscale", "clustered"}


def _run(A):
    A_copy = A.clone()
    H, tau = custom_kernel(A)
    torch.cuda.synchronize()
    assert torch.equal(A, A_copy), "input was modified"
    return H, tau


def _assert_gate(A, H, tau, what=""):
    res = checker.check(A, H, tau)
    assert res["ok"], (what, res["message"])
    return res


def _assert_diag(A, H, what=""):
    Hg, _ = torch.geqrf(A)
    d = checker.compare_diag_r(A, H, Hg)
    assert d["ok"], (what, d)


def test_golden_fixtures(golden):
    z, meta = golden
    for c in meta["cases"]:
        k = c["key"]
        A = torch.from_numpy(z[k + "_A"]).cuda()
        H, tau = _run(A)
        _assert_gate(A, H, tau, c["args"])
        Hn, taun = H.cpu().numpy(), tau.cpu().numpy()
        n = A.shape[-1]
        dl = np.abs(np.abs(np.diagonal(Hn, axis1=1, axis2=2)) - np.abs(np.diagonal(z[k + "_H_lapack"], axis1=1, axis2=2)))
        sc = np.abs(z[k + "_A"]).sum(axis=-2).max(axis=-1)[:, None] * n * oracle.EPS32
        assert (dl / np.maximum(sc, 1e-30)).max() <= 20.0, c["args"]
        if c["args"].get("case", "dense") in WELL_CONDITIONED:
            tol = 20.0 * n * oracle.EPS32 * sc.max() / (n * oracle.EPS32)
            assert np.abs(Hn - z[k + "_H_ref"]).max() <= tol, c["args"]
            assert np.abs(taun - z[k + "_tau_lapack"]).max() <= 1e-4, c["args"]


@pytest.mark.parametrize("n", [1, 2, 3, 17, 31, 32, 33, 63, 64, 65, 96, 127, 128, 129, 200, 255, 256, 257, 300])
def test_against_oracle_sizes(n):
    rng = np.random.default_rng(1000 + n)
    b = 3
    A_np = rng.standard_normal((b, n, n)).astype(np.float32)
    A = torch.from_numpy(A_np).cuda()
    H, tau = _run(A)
    Ho, tauo = oracle.geqrf_blocked(A_np)
    ok, info = oracle.check(A_np, H.cpu().numpy(), tau.cpu().numpy())
    assert ok, info
    scale = np.abs(A_np).sum(axis=-2).max(axis=-1)[:, None, None]
    d = np.abs(H.cpu().numpy() - Ho) / scale
    assert d.max() <= 20.0 * n * oracle.EPS32, d.max()
    assert np.abs(tau.cpu().numpy() - tauo).max() <= 1e-4


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C4", "C5"])
def test_benchmark_configs_full_size(name):
    A = gen.config_input(name, device="cuda")
    H, tau = _run(A)
    _assert_gate(A, H, tau, name)
    _assert_diag(A, H, name)


@pytest.mark.parametrize("idx", range(12))
def test_reference_scored_cases_full_batch(idx):
    """The reference's 12 scored cases (harness/lab.py:33-46) at their real batch, including
    mixed@640 n = 512, the case its authors found binding against the gate margin, which a
    batch-16 probe misses: gate on every matrix and |diag R| against torch.geqrf."""
    c = gen.REFERENCE_BENCH_CASES[idx]
    A = gen.generate_input(**c, device="cuda")
    H, tau = _run(A)
    res = _assert_gate(A, H, tau, c)
    print(c, res["message"])
    _assert_diag(A, H, c)


@pytest.mark.parametrize("batch,n", [(2, 512), (1, 1536)])
def test_against_oracle_two_level_and_cluster_sizes(batch, n):
    """Elementwise against the CPU restatement at a two-level size (n = 512: owner panels,
    narrow FP32 and 128-wide tcgen05 updates) and a single-level size with cluster panels
    (n = 1536: 16-, 8- and 4-CTA cluster panels above 512 rows, factor-warp panels below).
    Tolerance: the factor bound, |H - H_oracle| <= 20 n eps32 ||A||_1 elementwise."""
    rng = np.random.default_rng(77 + n)
    A_np = rng.standard_normal((batch, n, n)).astype(np.float32)
    A = torch.from_numpy(A_np).cuda()
    H, tau = _run(A)
    Ho, tauo = oracle.geqrf_blocked(A_np)
    scale = np.abs(A_np).sum(axis=-2).max(axis=-1)[:, None, None]
    d = np.abs(H.cpu().numpy() - Ho) / scale
    print(f"n={n}: max |H - H_oracle| / ||A||_1 = {d.max():.3g} (bound {20.0 * n * oracle.EPS32:.3g}); "
          f"max |tau - tau_oracle| = {np.abs(tau.cpu().numpy() - tauo).max():.3g}")
    assert d.max() <= 20.0 * n * oracle.EPS32, d.max()
    assert np.abs(tau.cpu().numpy() - tauo).max() <= 1e-3


def test_geqrf_rejects_bad_operands_before_launch():
    from qr_v2_b200_kernel_b200 import geqrf

    A = torch.randn(2, 64, 64, device="cuda")
    H = torch.empty_like(A)
    tau = torch.empty(2, 64, device="cuda")
    geqrf(A, H, tau)
    with pytest.raises(TypeError):
        geqrf(A, H.double(), tau)
    with pytest.raises(ValueError):
        geqrf(A, torch.empty(2, 64, 63, device="cuda"), tau)
    with pytest.raises(ValueError):
        geqrf(A, H, torch.empty(2, 63, device="cuda"))
    with pytest.raises(ValueError):
        geqrf(A, torch.empty(2, 64, 128, device="cuda")[:, :, :64], tau)  # non-contiguous H
    with pytest.raises(ValueError):
        geqrf(A.transpose(1, 2), H, tau)  # A rows not contiguous
    with pytest.raises(RuntimeError):
        geqrf(A, H.cpu(), tau)
    if torch.cuda.device_count() > 1:
        with pytest.raises(ValueError):
            geqrf(A, H.to("cuda:1"), tau)


@pytest.mark.parametrize("idx", range(22))
def test_reference_test_cases(idx):
    c = gen.REFERENCE_TEST_CASES[idx]
    A = gen.generate_input(**c, device="cuda")
    H, tau = _run(A)
    _assert_gate(A, H, tau, c)


def test_edge_matrices():
    n = 96
    g = torch.Generator().manual_seed(96)
    cases = {
        "zero": torch.zeros(2, n, n),
        "identity": torch.eye(n).expand(2, n, n).clone(),
        "neg_identity": -torch.eye(n).expand(2, n, n).clone(),
        "zero_column": torch.randn(2, n, n, generator=g).index_fill_(2, torch.tensor([5, 40]), 0.0),
        "rank_one": torch.randn(2, n, 1, generator=g) @ torch.randn(2, 1, n, generator=g),
        "tiny": torch.randn(2, n, n, generator=g) * 1e-20,
        "huge": torch.randn(2, n, n, generator=g) * 1e15,
    }
    for name, A in cases.items():
        A = A.float().cuda().contiguous()
        H, tau = _run(A)
        assert torch.isfinite(H).all() and torch.isfinite(tau).all(), name
        _assert_gate(A, H, tau, name)
    # the zero matrix: every reflector is the identity
    H, tau = _run(torch.zeros(1, 40, 40, device="cuda"))
    assert (tau == 0).all() and (H == 0).all()


@pytest.mark.parametrize("n", [96, 200, 600, 1536])
def test_tiny_scale_keeps_q_orthogonal(n):
    """Entries near 1e-20 square into fp32's subnormal range (fewer than 24 bits), which left
    tau inconsistent with its vector on short column tails; the rescaled reflector keeps Q
    orthogonal. n = 96: whole-matrix kernel; 200: owner panels; 600: cluster panels (tails of
    513+ rows, whose sums stay accurate at 1e-20) and owner panels; 1536: cluster and
    factor-warp panels. Much smaller entries are out of range: the panels form tail-by-column
    dot products before normalising the tail (as the reference panel does), and below about
    1e-22 those products underflow."""
    g = torch.Generator().manual_seed(n)
    A = (torch.randn(3, n, n, generator=g) * 1e-20).cuda()
    H, tau = _run(A)
    assert torch.isfinite(H).all() and torch.isfinite(tau).all()
    _assert_gate(A, H, tau, n)


def test_noncontiguous_and_batch_views():
    base = torch.randn(6, 160, 160, device="cuda")
    At = base.transpose(1, 2)  # non-contiguous view
    H, tau = _run(At)
    _assert_gate(At.contiguous(), H, tau, "transposed")
    sub = base[1:4]  # contiguous sub-batch with an offset
    H2, tau2 = _run(sub)
    H3, tau3 = _run(sub.clone())
    assert torch.equal(H2, H3) and torch.equal(tau2, tau3)


def test_deterministic_and_batch_independent():
    A = gen.config_input("C2", device="cuda", batch=12)
    H1, t1 = _run(A)
    H2, t2 = _run(A)
    assert torch.equal(H1, H2) and torch.equal(t1, t2)
    # a matrix's result does not depend on its batch neighbours
    H3, t3 = _run(A[5:6].contiguous())
    assert torch.equal(H3[0], H1[5]) and torch.equal(t3[0], t1[5])


def test_runs_on_current_stream():
    A = gen.config_input("C3", device="cuda", batch=4)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        H, tau = custom_kernel(A)
    s.synchronize()
    _assert_gate(A, H, tau, "side stream")


def _profiled(A):
    """The same factorisation through qrb200_profile_geqrf_f32 (every launch on the caller's
    stream, one after another: no look-ahead)."""
    import ctypes

    from qr_v2_b200_kernel_b200 import _lib

    lib = _lib.load()
    b, n, _ = A.shape
    H = torch.empty_like(A)
    tau = torch.empty((b, n), device=A.device)
    need = lib.qrb200_workspace_bytes(b, n)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=A.device)
    stats = (_lib.KernelStat * 16)()
    cnt = ctypes.c_int(0)
    st = lib.qrb200_profile_geqrf_f32(A.data_ptr(), H.data_ptr(), tau.data_ptr(), b, n, n * n, ws.data_ptr(), need,
                                      torch.cuda.current_stream().cuda_stream, stats, 16, ctypes.byref(cnt))
    assert st == 0
    return H, tau


@pytest.mark.parametrize("batch,n", [(3, 384), (4, 512), (2, 1000), (2, 1024), (1, 1536)])
def test_lookahead_schedule_matches_serial_schedule(batch, n):
    # The look-ahead cuts each update (128-column tiles of the two-level schedule; the next
    # panel's 32 columns of the single-level schedule, n >= 1024) and runs part of it on a
    # second stream; the serial schedule makes the same cuts, so results agree bit for bit.
    A = torch.randn(batch, n, n, device="cuda")
    H, tau = _run(A)
    Hs, taus = _profiled(A)
    torch.cuda.synchronize()
    assert torch.equal(H, Hs) and torch.equal(tau, taus)


def test_concurrent_calls_from_host_threads():
    import threading

    As = [torch.randn(3, 512, 512, device="cuda") for _ in range(4)]
    ref = [_run(A) for A in As]
    out = [None] * len(As)
    errors = []

    def worker(i):
        try:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.default_stream())
            with torch.cuda.stream(s):
                for _ in range(3):
                    out[i] = custom_kernel(As[i])
            s.synchronize()
        except Exception as e:  # surfaced below
            errors.append(e)

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(len(As))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors
    for (H, tau), (Hr, taur) in zip(out, ref):
        assert torch.equal(H, Hr) and torch.equal(tau, taur)


def test_error_paths_on_gpu():
    from qr_v2_b200_kernel_b200._lib import QRB200Error

    with pytest.raises(QRB200Error):
        custom_kernel(torch.zeros(1, 4097, 4097, device="cuda"))
    H, tau = custom_kernel(torch.zeros(0, 8, 8, device="cuda"))
    assert H.shape == (0, 8, 8) and tau.shape == (0, 8)


@pytest.mark.parametrize("batch,n,chunks", [(96, 256, None), (5, 200, None), (7, 96, 3)])
def test_host_api_matches_device_api(batch, n, chunks):
    # The host-buffer entry point cuts the batch into pieces on separate streams; a matrix's
    # arithmetic does not depend on its batch, so the result equals the device call bit for bit.
    from qr_v2_b200_kernel_b200 import custom_kernel_host

    A = torch.randn(batch, n, n)
    H, tau = custom_kernel(A.cuda())
    Hh, tauh = custom_kernel_host(A.pin_memory(), chunks=chunks)
    torch.cuda.synchronize()
    assert torch.equal(H.cpu(), Hh) and torch.equal(tau.cpu(), tauh)
