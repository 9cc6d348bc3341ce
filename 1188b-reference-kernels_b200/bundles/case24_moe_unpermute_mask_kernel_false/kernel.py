"""Unweighted unpermute with an int32 expert-major map (deep_ep FusedCombine),
the contract of kernel_cases/case24_ref_moe_unpermute_mask_kernel_false.py:
45-68: returns (fp32 sum [T,H], bf16 store [T,H])."""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(grad_in, row_id_map):
    if int(row_id_map.numel()) and int(row_id_map.max()) >= grad_in.shape[0]:
        raise ValueError("row_id_map points past grad_in")
    out, acc = moe_b200.unpermute(grad_in, row_id_map, return_acc=True)
    return acc, out
