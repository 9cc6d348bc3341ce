"""Permute without probs (deep_ep <bf16,false> form), the contract of
kernel_cases/case30_ref_moe_permute_mask_kernel.py:44-58."""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(grad, row_id_map):
    out, _ = moe_b200.permute_trans(grad, row_id_map, None)
    return out
