"""Device-side failure reporting on the B200, without faulting or hanging the GPU.

Every wait inside the kernels is bounded; a wait that runs out records its site in a device word
and in a mapped pinned host word. The test hook ``qrb200_selftest_wait_timeout`` makes one warp
wait, with a short poll limit, on a barrier that nothing completes (nothing else is in flight),
so the wait runs out through the same reporting path as the factorisation kernels. The operator
then raises ``QRB200Error(QRB200_ERR_TIMEOUT)`` at its next call on the device, and the device
stays usable.
"""

import ctypes

import pytest
import torch

from qr_v2_b200_kernel_b200 import _lib, custom_kernel
from qr_v2_b200_kernel_b200._lib import QRB200Error

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _clear(lib):
    st = ctypes.c_int(0)
    assert lib.qrb200_device_status(ctypes.byref(st)) == _lib.QRB200_OK
    return st.value


def test_expired_wait_is_reported_then_raised_and_cleared():
    lib = _lib.load()
    A = torch.randn(2, 256, 256, device="cuda")
    H0, tau0 = custom_kernel(A)
    torch.cuda.synchronize()
    _clear(lib)
    site = ctypes.c_int(-1)
    assert lib.qrb200_last_status(ctypes.byref(site)) == _lib.QRB200_OK and site.value == 0

    # a wait that runs out: seen through the host word without a CUDA call, cleared by the read
    assert lib.qrb200_selftest_wait_timeout(2000, _stream()) == _lib.QRB200_OK
    torch.cuda.synchronize()
    assert lib.qrb200_last_status(ctypes.byref(site)) == _lib.QRB200_ERR_TIMEOUT and site.value == 4
    assert lib.qrb200_last_status(ctypes.byref(site)) == _lib.QRB200_OK and site.value == 0
    assert _clear(lib) == _lib.QRB200_ERR_TIMEOUT  # the device word saw it too
    assert _clear(lib) == _lib.QRB200_OK

    # the operator raises at its next call, then works again with the same result
    assert lib.qrb200_selftest_wait_timeout(2000, _stream()) == _lib.QRB200_OK
    torch.cuda.synchronize()
    with pytest.raises(QRB200Error) as ei:
        custom_kernel(A)
    assert ei.value.status == _lib.QRB200_ERR_TIMEOUT
    _clear(lib)
    H1, tau1 = custom_kernel(A)
    torch.cuda.synchronize()
    assert torch.equal(H0, H1) and torch.equal(tau0, tau1)
    assert lib.qrb200_last_status(None) == _lib.QRB200_OK
    assert _clear(lib) == _lib.QRB200_OK
