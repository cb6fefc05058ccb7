"""C-ABI library: loads, exports every symbol include/qrb200.h declares, host-side checks.

No kernel runs here (CPU-only): only calls that return before touching the device.
"""

import ctypes
import os
import re

import pytest

from qr_v2_b200_kernel_b200 import _lib, build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_symbols():
    text = open(os.path.join(REPO, "include", "qrb200.h")).read()
    return sorted(set(re.findall(r"\b(qrb200_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_the_binding_table():
    assert _header_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_header_symbol(lib):
    for name in _header_symbols():
        assert hasattr(lib, name), name


def test_status_strings_and_version(lib):
    assert lib.qrb200_version() >= 100
    for st in range(7):
        assert lib.qrb200_status_string(st)
    assert lib.qrb200_status_string(0) == b"ok"


def test_workspace_query(lib):
    assert lib.qrb200_workspace_bytes(0, 128) == 0
    assert lib.qrb200_workspace_bytes(8, 64) == 0  # single-CTA path needs no scratch
    assert lib.qrb200_workspace_bytes(640, 512) > 0
    assert lib.qrb200_workspace_bytes(2, 4096) % 256 == 0
    assert lib.qrb200_workspace_bytes(1, 1 << 20) == 0  # unsupported order


def test_argument_errors_before_any_device_work(lib):
    p = ctypes.c_void_p(16)
    f = lib.qrb200_geqrf_f32
    assert f(p, p, p, -1, 8, 64, None, 0, None) == _lib.QRB200_ERR_ARG
    assert f(p, p, p, 1, -8, 64, None, 0, None) == _lib.QRB200_ERR_ARG
    assert f(None, p, p, 1, 8, 64, None, 0, None) == _lib.QRB200_ERR_ARG
    assert f(p, p, p, 2, 8, 63, None, 0, None) == _lib.QRB200_ERR_ARG  # batch stride < n*n
    assert f(p, p, p, 1, 1 << 20, 1 << 40, None, 0, None) == _lib.QRB200_ERR_ARG
    assert f(p, p, p, 0, 8, 64, None, 0, None) == _lib.QRB200_OK  # empty batch: no-op
    assert f(p, p, p, 4, 0, 0, None, 0, None) == _lib.QRB200_OK


def test_device_status_null_pointer(lib):
    assert lib.qrb200_device_status(None) == _lib.QRB200_ERR_ARG


def test_operator_rejects_bad_inputs_on_cpu():
    import torch

    from qr_v2_b200_kernel_b200 import custom_kernel

    with pytest.raises(RuntimeError):
        custom_kernel(torch.zeros(2, 4, 4))  # CPU tensor: no fallback
    with pytest.raises(TypeError):
        custom_kernel(torch.zeros(2, 4, 4, dtype=torch.float64))
    with pytest.raises(ValueError):
        custom_kernel(torch.zeros(2, 4, 5))
    with pytest.raises(TypeError):
        custom_kernel([[1.0]])


def test_noalloc_entry_host_checks(lib):
    p = ctypes.c_void_p(16)
    f = lib.qrb200_geqrf_f32_noalloc
    assert f(p, p, p, -1, 8, 64, None) == _lib.QRB200_ERR_ARG
    assert f(None, p, p, 1, 8, 64, None) == _lib.QRB200_ERR_ARG
    assert f(p, p, p, 1, 1 << 20, 1 << 40, None) == _lib.QRB200_ERR_ARG
    assert f(p, p, p, 70000, 512, 512 * 512, None) == _lib.QRB200_ERR_ARG  # batch limit, not scratch
    assert f(p, p, p, 0, 512, 512 * 512, None) == _lib.QRB200_OK
    # beyond the static scratch: rejected before any device call
    assert lib.qrb200_workspace_bytes(2, 4096) > _lib.NOALLOC_SCRATCH_BYTES >= lib.qrb200_workspace_bytes(1, 4096)
    assert f(p, p, p, 2, 4096, 4096 * 4096, None) == _lib.QRB200_ERR_SCRATCH_LIMIT


def test_host_api_rejects_bad_inputs_on_cpu():
    import torch

    from qr_v2_b200_kernel_b200 import custom_kernel_host
    from qr_v2_b200_kernel_b200.api import _host_chunks

    with pytest.raises(TypeError):
        custom_kernel_host([[1.0]])
    with pytest.raises(ValueError):
        custom_kernel_host(torch.zeros(2, 3, 4))
    with pytest.raises(TypeError):
        custom_kernel_host(torch.zeros(2, 3, 3, dtype=torch.float64))
    # pieces by input size: one below 32 MB, two below 192 MB, else four; at most one per matrix
    assert _host_chunks(8, 128) == 1  # C1: 0.5 MB
    assert _host_chunks(8, 2048) == 2 and _host_chunks(2, 4096) == 2  # C4, C5: 134 MB
    assert _host_chunks(64, 1024) == 4 and _host_chunks(640, 512) == 8  # C3: 268 MB, C2: 671 MB
    assert _host_chunks(1, 4096) == 1  # never more pieces than matrices


def test_geqrf_rejects_bad_operands_on_cpu():
    import torch

    from qr_v2_b200_kernel_b200 import geqrf

    A = torch.zeros(2, 4, 4)
    with pytest.raises(TypeError):
        geqrf([[1.0]], A, torch.zeros(2, 4))
    with pytest.raises(TypeError):
        geqrf(A.double(), A, torch.zeros(2, 4))
    with pytest.raises(RuntimeError):
        geqrf(A, A.clone(), torch.zeros(2, 4))  # host tensors: no CPU path


def test_status_entries_without_a_device(lib):
    # No CUDA device here: the status read fails with a CUDA error instead of touching memory.
    import torch

    if torch.cuda.is_available():
        pytest.skip("needs a host without a GPU")
    assert lib.qrb200_last_status(None) == _lib.QRB200_ERR_CUDA


def test_apply_entries_host_checks(lib):
    p = ctypes.c_void_p(16)
    assert lib.qrb200_apply_workspace_bytes(2, 512, 64) > 0
    assert lib.qrb200_apply_workspace_bytes(2, 512, 64) % 256 == 0
    assert lib.qrb200_apply_workspace_bytes(0, 512, 64) == 0
    assert lib.qrb200_apply_workspace_bytes(1, 8192, 8) == 0  # unsupported order
    f = lib.qrb200_ormqr_f32
    assert f(p, p, p, 1, 30, 8, 1, None, 0, None) == _lib.QRB200_ERR_ARG  # n % 4 != 0
    assert f(p, p, p, 1, 32, 6, 1, None, 0, None) == _lib.QRB200_ERR_ARG  # nrhs % 4 != 0
    assert f(None, p, p, 1, 32, 8, 0, None, 0, None) == _lib.QRB200_ERR_ARG
    assert f(ctypes.c_void_p(20), p, p, 1, 32, 8, 0, None, 0, None) == _lib.QRB200_ERR_ARG  # unaligned H
    assert f(p, p, p, 0, 32, 8, 1, None, 0, None) == _lib.QRB200_OK  # empty batch: no-op
    g = lib.qrb200_orgqr_f32
    assert g(p, p, p, 1, 5000, None, 0, None) == _lib.QRB200_ERR_ARG
    assert g(p, p, p, -1, 32, None, 0, None) == _lib.QRB200_ERR_ARG
    assert g(p, p, p, 3, 0, None, 0, None) == _lib.QRB200_OK
