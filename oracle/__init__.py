"""CPU oracle (test infrastructure only; never imported by the product package).

See ``oracle.householder`` for what it restates and how it is pinned.
"""

from .householder import (  # noqa: F401
    EPS32,
    block_size,
    build_v,
    check,
    form_t,
    geqrf_blocked,
    householder_product,
    larfg,
    panel_factor,
)
