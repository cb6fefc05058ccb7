"""Generate the golden fixtures in this directory from the reference itself.

Runs ONLY where the reference checkout is present (its path is the first CLI argument or
``$QR_REFERENCE_ROOT``). For every case it records:

* ``A``            -- the reference generator's input (``harness/reference.py:132-149``, CPU),
* ``H_ref, tau_ref`` -- the reference's own CPU path, ``submission.custom_kernel`` on CPU
  tensors, which runs the eager blocked compact-WY ``_factor_custom`` (``submission.py:560-564``),
* ``H_lapack, tau_lapack`` -- ``torch.geqrf`` on CPU (the reference's ``ref_kernel``,
  ``harness/reference.py:152-154``),
* the reference checker's verdict and scaled residuals for both
  (``harness/reference.py:189-273``).

Usage:  python tests/golden/make_golden.py <reference-root>
Writes: tests/golden/golden.npz and tests/golden/golden_meta.json
"""

from __future__ import annotations

import importlib.util
import json
import os
import re
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    dict(batch=4, n=32, cond=1, seed=53124, case="dense"),
    dict(batch=2, n=64, cond=2, seed=32523, case="dense"),
    dict(batch=2, n=48, cond=0, seed=32525, case="rankdef"),
    dict(batch=2, n=64, cond=0, seed=4330, case="nearrank"),
    dict(batch=2, n=64, cond=0, seed=32526, case="clustered"),
    dict(batch=2, n=64, cond=0, seed=32527, case="band"),
    dict(batch=2, n=64, cond=0, seed=32528, case="rowscale"),
    dict(batch=2, n=64, cond=0, seed=32529, case="nearcollinear"),
    dict(batch=2, n=40, cond=0, seed=75343, case="upper"),
    dict(batch=2, n=33, cond=0, seed=7, case="diagonal"),
    dict(batch=8, n=40, cond=2, seed=32530, case="mixed"),
    dict(batch=2, n=128, cond=1, seed=0, case="dense"),
    dict(batch=1, n=176, cond=1, seed=3321, case="dense"),
    dict(batch=3, n=1, cond=0, seed=11, case="dense"),
    dict(batch=3, n=2, cond=0, seed=12, case="dense"),
    dict(batch=2, n=3, cond=0, seed=13, case="dense"),
    dict(batch=2, n=17, cond=0, seed=14, case="dense"),
]


def _load(ref_root: str):
    sys.path.insert(0, os.path.join(ref_root, "harness"))
    import reference  # noqa: E402  (the reference's harness module)

    spec = importlib.util.spec_from_file_location("ref_submission", os.path.join(ref_root, "submission.py"))
    sub = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sub)
    return reference, sub


def _residuals(msg: str) -> dict:
    return {k: float(v) for k, v in re.findall(r"(scaled_\w+)=([0-9.eE+-]+)", msg or "")}


def main() -> int:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QR_REFERENCE_ROOT", "")
    if not ref_root or not os.path.isdir(ref_root):
        print("usage: make_golden.py <reference-root>", file=sys.stderr)
        return 2
    torch.manual_seed(0)
    reference, sub = _load(ref_root)
    arrays, meta = {}, []
    for i, c in enumerate(CASES):
        a = reference.generate_input(**c)
        assert a.device.type == "cpu"
        h_ref, tau_ref = sub.custom_kernel(a.clone())
        h_lp, tau_lp = torch.geqrf(a.clone())
        ok_ref, msg_ref = reference.check_implementation(a, (h_ref, tau_ref))
        ok_lp, msg_lp = reference.check_implementation(a, (h_lp, tau_lp))
        key = f"c{i:02d}"
        arrays[f"{key}_A"] = a.numpy()
        arrays[f"{key}_H_ref"] = h_ref.numpy()
        arrays[f"{key}_tau_ref"] = tau_ref.numpy()
        arrays[f"{key}_H_lapack"] = h_lp.numpy()
        arrays[f"{key}_tau_lapack"] = tau_lp.numpy()
        meta.append(dict(key=key, args=c, ref_ok=bool(ok_ref), ref_check=_residuals(msg_ref),
                         lapack_ok=bool(ok_lp), lapack_check=_residuals(msg_lp)))
        print(key, c, ok_ref, ok_lp)
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(dict(source="Raymondlol/qr-v2-b200-kernel harness/reference.py + submission.py (CPU)",
                       torch=torch.__version__, cases=meta), f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
