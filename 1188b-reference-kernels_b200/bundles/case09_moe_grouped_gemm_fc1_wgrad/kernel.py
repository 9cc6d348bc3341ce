"""Grouped wgrad of the fc1 GEMM: dW [G,N,K] = stack_g(dy[seg_g].T @ x[seg_g])
from dy [T,N] and x [T,K] bf16 (kernel_cases/case09_moe_grouped_gemm_fc1_wgrad.py:49-64, "TN"), fp32
accumulation, bf16 out. The reference Model splits T uniformly over
NUM_GROUPS = 40 (its group_sizes); num_groups / m_splits select another split.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402

NUM_GROUPS = 40


def kernel_function(dy, x, num_groups=NUM_GROUPS, m_splits=None):
    if m_splits is None:
        base, rem = divmod(dy.shape[0], num_groups)
        m_splits = [base + (1 if i < rem else 0) for i in range(num_groups)]
    return moe_b200.grouped_wgrad(dy, x, m_splits)
