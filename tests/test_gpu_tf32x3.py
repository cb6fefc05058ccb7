"""Accuracy of the 3xTF32 tcgen05 GEMMs of the 128-wide trailing update against FP64.

``qrb200_diag_wide_update_f32`` runs the three tensor-core products of one wide compact-WY
update on their own: W^T = C^T V (``tc_vtc128``), W'^T = W^T Tt^T (``tc_tw128``) and
C -= V W' (``tc_upd128``), V the unit lower trapezoid of H[:, :128], C = H[:, 128:], Tt a given
128 x 128 matrix (the schedule passes the block factor T transposed). The result is compared
with C - V Tt V^T C in FP64. Tolerance: the largest error relative to |V| |Tt| |V|^T |C| (the
magnitude of the subtracted product, elementwise) must stay below 1e-5, where one TF32 pass
(10-bit mantissa) would sit near 5e-4; the measured value is printed.
"""

import ctypes

import pytest
import torch

from qr_v2_b200_kernel_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,n", [(3, 512), (2, 1024), (4, 260)])
def test_wide_update_matches_fp64(batch, n):
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(n)
    H = torch.randn((batch, n, n), device="cuda", generator=g)
    Tt = torch.randn((batch, 128, 128), device="cuda", generator=g)
    H0 = H.clone()
    need = lib.qrb200_workspace_bytes(batch, n)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    st = lib.qrb200_diag_wide_update_f32(ctypes.c_void_p(H.data_ptr()), ctypes.c_void_p(Tt.data_ptr()), batch, n,
                                         ctypes.c_void_p(ws.data_ptr()), need,
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.QRB200_OK
    torch.cuda.synchronize()
    Hd = H0.double()
    V = torch.tril(Hd[:, :, :128], diagonal=-1)
    V[:, torch.arange(128), torch.arange(128)] = 1.0
    C = Hd[:, :, 128:]
    Td = Tt.double()
    W = V.transpose(-1, -2) @ C
    ref = C - V @ (Td @ W)
    mag = V.abs() @ (Td.abs() @ (V.abs().transpose(-1, -2) @ C.abs()))
    err = ((H[:, :, 128:].double() - ref).abs() / mag.clamp_min(1e-30)).max().item()
    print(f"3xTF32 wide update batch={batch} n={n}: max error / |V||Tt||V^T||C| = {err:.3g}")
    assert err < 1e-5, err
    assert torch.equal(H[:, :, :128], H0[:, :, :128])
