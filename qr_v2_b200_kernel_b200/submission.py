"""Drop-in ``submission`` module: ``from submission import custom_kernel`` works unchanged.

The reference harness imports the operator as ``from submission import custom_kernel``
(``harness/eval.py:131``, ``:189``). Put this package on ``sys.path`` and alias this module
as ``submission``, or copy the one import below into a
``submission.py`` of your own.
"""

from qr_v2_b200_kernel_b200.api import custom_kernel  # noqa: F401
