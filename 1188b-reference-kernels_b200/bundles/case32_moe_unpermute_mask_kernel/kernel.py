"""deep_ep dispatch backward with an int32 [E,T] map: (acc [T,H] fp32,
grad_x [T,H] bf16, grad_probs [T,E] fp32) from (grad_in [R,H] bf16,
row_id_map [E,T] int32, prob_grad [R] fp32) — the signature and results of
kernel_cases/case32_ref_moe_unpermute_mask_kernel.py reference_unpermute_mask
(:47-79): unweighted fp32 sum of the routed rows (ascending expert), stored
bf16, and the prob gradient gathered onto [token, expert].
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(grad_in, row_id_map, prob_grad):
    return moe_b200.permute_backward(grad_in, row_id_map, prob_grad, return_acc=True)
