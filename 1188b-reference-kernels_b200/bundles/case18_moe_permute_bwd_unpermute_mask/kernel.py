"""Backward of the permute (int64 [E,T] map): (dact [T,H] bf16, dprobs [T,E] fp32)
from (dperm_act [R,H] bf16, dpp [R] fp32, row_id_map [E,T] int64) — the
signature and results of kernel_cases/case18_moe_permute_bwd_unpermute_mask.py
Model.forward (:56-70): dact[t] = bf16(sum over e of fp32 rows, ascending e),
dprobs[t,e] = dpp[row_id_map[e,t]] where routed, else 0.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(dperm_act, dpp, row_id_map):
    return moe_b200.permute_backward(dperm_act, row_id_map, dpp)
