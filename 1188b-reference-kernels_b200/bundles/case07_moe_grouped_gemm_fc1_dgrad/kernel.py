"""Grouped dgrad of the fc1 GEMM: dx [T,K] = cat_g(dy[seg_g] @ w[g]) with dy
[T,N] bf16 and the forward weight w [G,N,K] bf16 as it is (kernel_cases/
case07_moe_grouped_gemm_fc1_dgrad.py:49-64, "NN" layout; case13/case19 are the one-group
form). Uniform splits by default, as the reference's group_sizes. The weight
is staged MN-major on the tensor cores; fp32 accumulation, bf16 out.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(dy, w, m_splits=None):
    return moe_b200.grouped_gemm(dy, w, m_splits, w_layout="KN")
