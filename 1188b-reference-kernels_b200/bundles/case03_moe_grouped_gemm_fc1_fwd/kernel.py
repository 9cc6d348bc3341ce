"""Drop-in for the grouped GEMM forward of
kernel_cases/case03_moe_grouped_gemm_fc1_fwd.py:57-64 (and the G=1 case10):
out = cat_i(x[seg_i] @ w[i].T), x [T,K] bf16, w [G,N,K] bf16 -> [T,N] bf16.
Segments default to the reference's uniform group_sizes (:43-46); pass
m_splits for the ragged per-expert counts of a real routing.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(x, w, m_splits=None):
    return moe_b200.grouped_gemm(x, w, m_splits)
