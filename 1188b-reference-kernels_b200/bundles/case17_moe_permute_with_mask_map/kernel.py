"""Drop-in for kernel_results/case17_moe_permute_with_mask_map/kernel.py:4-6.

(x [T,H] bf16, row_id_map [T,E] int64, probs [T,E]) ->
(out [R,H] bf16, permuted_probs [R] fp32) with R = max(row_id_map) + 1, the
contract of kernel_cases/case17_moe_permute_with_mask_map.py:58-71.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(x, row_id_map, probs):
    return moe_b200.permute(x, row_id_map, probs)
