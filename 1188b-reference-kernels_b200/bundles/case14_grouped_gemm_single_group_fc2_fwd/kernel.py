"""Drop-in for kernel_cases/case14_grouped_gemm_single_group_fc2_fwd.py:57-64:
the fc2 grouped GEMM with one group, out [T,N] = x [T,K] @ w[0].T for x [T,K]
bf16, w [1,N,K] bf16 (fp32 accumulation, bf16 out). Any G works, with the
reference's uniform group_sizes (:43-46) unless m_splits is given.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(x, w, m_splits=None):
    return moe_b200.grouped_gemm(x, w, m_splits)
