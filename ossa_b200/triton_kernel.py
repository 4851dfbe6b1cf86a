"""Import-path compatibility for ``ossa.triton_kernel`` (ossa/triton_kernel.py).

Code written against the reference imports ``topk_attention`` and
``HAS_TRITON`` from this module path; both resolve to the sm_100a
implementation in :mod:`ossa_b200.topk_attention`.  No Triton is used.
"""

from .topk_attention import HAS_TRITON, topk_attention

__all__ = ["HAS_TRITON", "topk_attention"]
