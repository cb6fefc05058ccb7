"""qrb200_geqrf_f32_noalloc (static device scratch) against qrb200_geqrf_f32, both via the C ABI.

The no-alloc entry runs the same kernels as qrb200_geqrf_f32 with the library's static scratch
in place of a caller workspace, so results must agree bit for bit. Two calls in a row on
different inputs check that nothing depends on the scratch's earlier contents; the caller
workspace of the comparison call is filled with NaN for the same reason. This file is named to
be collected last, so it also runs after every other GPU test in the same process.
"""

import ctypes

import pytest
import torch

from qr_v2_b200_kernel_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _existing(lib, A):
    b, n, _ = A.shape
    H = torch.empty_like(A)
    tau = torch.empty((b, n), dtype=A.dtype, device=A.device)
    need = lib.qrb200_workspace_bytes(b, n)
    ws = torch.full((max(need, 4) // 4,), float("nan"), dtype=torch.float32, device=A.device)
    st = lib.qrb200_geqrf_f32(_ptr(A), _ptr(H), _ptr(tau), b, n, n * n, _ptr(ws), need, _stream())
    assert st == _lib.QRB200_OK, lib.qrb200_status_string(st)
    return H, tau


def _noalloc(lib, A):
    b, n, _ = A.shape
    H = torch.full_like(A, float("nan"))
    tau = torch.full((b, n), float("nan"), dtype=A.dtype, device=A.device)
    st = lib.qrb200_geqrf_f32_noalloc(_ptr(A), _ptr(H), _ptr(tau), b, n, n * n, _stream())
    assert st == _lib.QRB200_OK, lib.qrb200_status_string(st)
    return H, tau


def _max_batch(lib, n):
    b = 0
    while lib.qrb200_workspace_bytes(b + 1, n) <= _lib.NOALLOC_SCRATCH_BYTES:
        b += 1
    return b


# n <= 128 (no scratch), single-level (n % 4 != 0), two-level, and the largest batches that fit
# (batch None = the largest).
SHAPES = [(5, 96), (3, 200), (4, 256), (2, 512), (1, 1000), (None, 512), (None, 1024), (1, 4096)]


@pytest.mark.parametrize("batch,n", SHAPES)
def test_noalloc_matches_workspace_entry_two_calls(lib, batch, n):
    if batch is None:
        batch = _max_batch(lib, n)
        assert batch >= 8
    assert lib.qrb200_workspace_bytes(batch, n) <= _lib.NOALLOC_SCRATCH_BYTES
    g = torch.Generator(device="cuda").manual_seed(1000 * n + batch)
    for call in range(2):
        A = torch.randn((batch, n, n), generator=g, device="cuda", dtype=torch.float32)
        A0 = A.clone()
        H_ref, tau_ref = _existing(lib, A)
        H, tau = _noalloc(lib, A)
        torch.cuda.synchronize()
        assert torch.equal(A, A0), "input modified"
        assert torch.equal(H, H_ref), f"call {call}: H differs"
        assert torch.equal(tau, tau_ref), f"call {call}: tau differs"
    st = ctypes.c_int(-1)
    assert lib.qrb200_device_status(ctypes.byref(st)) == _lib.QRB200_OK and st.value == 0


def test_noalloc_launches_the_same_kernels(lib):
    A = torch.randn((2, 512, 512), device="cuda")
    _noalloc(lib, A)  # first call per device does the one-time symbol lookup
    c0 = lib.qrb200_launch_count()
    _existing(lib, A)
    c1 = lib.qrb200_launch_count()
    _noalloc(lib, A)
    c2 = lib.qrb200_launch_count()
    torch.cuda.synchronize()
    assert c2 - c1 == c1 - c0 > 0


def test_noalloc_rejects_problems_beyond_the_static_scratch(lib):
    for b, n in [(2, 4096), (_max_batch(lib, 512) + 1, 512), (_max_batch(lib, 1024) + 1, 1024)]:
        assert lib.qrb200_workspace_bytes(b, n) > _lib.NOALLOC_SCRATCH_BYTES
        A = torch.randn((b, n, n), device="cuda")
        H = torch.zeros_like(A)
        tau = torch.zeros((b, n), device="cuda")
        c0 = lib.qrb200_launch_count()
        st = lib.qrb200_geqrf_f32_noalloc(_ptr(A), _ptr(H), _ptr(tau), b, n, n * n, _stream())
        assert st == _lib.QRB200_ERR_SCRATCH_LIMIT
        assert b"static scratch" in lib.qrb200_status_string(st)
        assert lib.qrb200_launch_count() == c0  # nothing launched
        torch.cuda.synchronize()
        assert not H.any() and not tau.any()
