"""Permute with probs over the expert-major map (deep_ep FusedDispatch form).

Same contract as reference_permute_mask_with_probs,
kernel_cases/case22_ref_moe_permute_mask_kernel_true.py:47-69:
(inp [T,H] bf16, row_id_map [E,T] int64/int32, probs [T,E] fp32) ->
(out [R,H], permuted_probs [R]) with R = max + 1; empty map -> empty outputs.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(inp, row_id_map, probs):
    return moe_b200.permute_trans(inp, row_id_map, probs)
