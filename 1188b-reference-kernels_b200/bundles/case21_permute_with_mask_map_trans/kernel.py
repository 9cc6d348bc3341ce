"""Permute without probs over the expert-major map, the contract of
kernel_cases/case21_ref_permute_with_mask_map_trans.py:52-68."""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(inp, row_id_map):
    out, _ = moe_b200.permute_trans(inp, row_id_map, None)
    return out
