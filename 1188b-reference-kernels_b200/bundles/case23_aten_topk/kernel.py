"""Drop-in for kernel_results/case23_aten_topk/kernel.py:14-25.

Row-wise top-k of fp32 scores: values[t,:], indices[t,:] =
topk(input[t,:], k, largest=True, sorted=True), ties to the lower index
(kernel_cases/case23_ref_aten_topk.py:47-62). Unsupported arguments raise
ValueError, as in the reference bundle.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402

MAX_K = 16


def kernel_function(input, k=8, dim=1, largest=True, sorted=True):
    if not largest:
        raise ValueError("only largest=True is supported")
    if dim not in (1, -1):
        raise ValueError("only dim=1 is supported")
    if input.dim() != 2:
        raise ValueError(f"expected 2D input, got {input.dim()}D")
    n = int(input.shape[1])
    k = min(int(k), n)
    if k > MAX_K:
        raise ValueError(f"k={k} exceeds the {MAX_K} supported by this kernel")
    return moe_b200.topk(input, k)
