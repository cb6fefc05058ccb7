"""Q from the factorisation on the B200: ``householder_product`` (sorgqr) and ``ormqr`` (sormqr).

The reference builds Q with ``torch.linalg.householder_product`` in its checker
(``harness/reference.py:206``); these replace it (and ``torch.ormqr``) with the blocked
compact-WY kernels. Tolerances (FP32, from the reference's orthogonality criterion): Q against
torch's householder_product within ||Q - Q_torch||_1 <= 100 n eps32, Q^T Q - I within the same
bound, and ``ormqr`` against the FP64 product with torch's Q within 100 n eps32 ||C||_1.
"""

import pytest
import torch

from qr_v2_b200_kernel_b200 import custom_kernel, gen, householder_product, ormqr

pytestmark = pytest.mark.gpu

EPS = torch.finfo(torch.float32).eps


def _l1(x):
    return torch.linalg.matrix_norm(x, ord=1, dim=(-2, -1))


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C4", "C5"])
def test_householder_product_matches_torch_at_the_configs(name):
    A = gen.config_input(name, device="cuda")
    H, tau = custom_kernel(A)
    Q = householder_product(H, tau)
    n = A.shape[-1]
    bound = 100.0 * n * EPS
    for b0 in range(0, A.shape[0], 64):
        Qt = torch.linalg.householder_product(H[b0:b0 + 64], tau[b0:b0 + 64]).double()
        Qo = Q[b0:b0 + 64].double()
        diff = _l1(Qo - Qt).max().item()
        orth = _l1(Qo.transpose(-1, -2) @ Qo - torch.eye(n, device="cuda", dtype=torch.float64)).max().item()
        assert diff <= bound, (name, diff / (n * EPS))
        assert orth <= bound, (name, orth / (n * EPS))
    # the factorisation through our Q passes the reference's factor criterion
    Ad, Qd = A[:8].double(), Q[:8].double()
    fres = _l1(torch.triu(H[:8]).double() - Qd.transpose(-1, -2) @ Ad) / _l1(Ad)
    assert fres.max().item() <= 20.0 * n * EPS


@pytest.mark.parametrize("n", [4, 32, 100, 128, 132, 260, 516])
def test_householder_product_small_and_ragged_orders(n):
    A = torch.randn(3, n, n, device="cuda")
    H, tau = custom_kernel(A)
    Q = householder_product(H, tau)
    Qt = torch.linalg.householder_product(H, tau)
    assert (_l1((Q - Qt).double()).max() <= 100.0 * n * EPS).item()


def test_householder_product_of_identity_reflectors():
    # tau = 0 everywhere (zero matrix): Q = I exactly
    H, tau = custom_kernel(torch.zeros(2, 64, 64, device="cuda"))
    Q = householder_product(H, tau)
    assert torch.equal(Q, torch.eye(64, device="cuda").expand(2, 64, 64))


@pytest.mark.parametrize("batch,n,nrhs", [(4, 512, 64), (2, 1024, 8), (1, 2048, 256), (3, 200, 12)])
def test_ormqr_both_directions(batch, n, nrhs):
    A = torch.randn(batch, n, n, device="cuda")
    C = torch.randn(batch, n, nrhs, device="cuda")
    H, tau = custom_kernel(A)
    Qt = torch.linalg.householder_product(H, tau).double()
    QtC = ormqr(H, tau, C, transpose=True)
    QC = ormqr(H, tau, C, transpose=False)
    Cd = C.double()
    bound = 100.0 * n * EPS * _l1(Cd)
    assert (_l1(QtC.double() - Qt.transpose(-1, -2) @ Cd) <= bound).all()
    assert (_l1(QC.double() - Qt @ Cd) <= bound).all()
    # round trip Q (Q^T C) = C, and C itself untouched
    back = ormqr(H, tau, QtC, transpose=False)
    assert (_l1(back.double() - Cd) <= bound).all()
    # least squares: R x = (Q^T b)[:n] solves A x = b
    x = torch.linalg.solve_triangular(torch.triu(H).double(), QtC.double(), upper=True)
    res = _l1(A.double() @ x - Cd) / (_l1(A.double()) * _l1(x))
    assert (res <= 20.0 * n * EPS).all()


def test_apply_q_argument_errors():
    H, tau = custom_kernel(torch.randn(2, 64, 64, device="cuda"))
    with pytest.raises(ValueError):
        ormqr(H, tau, torch.randn(2, 64, 6, device="cuda"))  # nrhs % 4 != 0
    with pytest.raises(ValueError):
        ormqr(H, tau, torch.randn(2, 60, 8, device="cuda"))
    with pytest.raises(TypeError):
        householder_product(H.double(), tau)
    H2, tau2 = custom_kernel(torch.randn(1, 30, 30, device="cuda"))
    with pytest.raises(ValueError):
        householder_product(H2, tau2)  # n % 4 != 0
