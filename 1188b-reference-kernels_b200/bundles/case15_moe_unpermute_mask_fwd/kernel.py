"""Drop-in for kernel_results/case15_moe_unpermute_mask_fwd/kernel.py:4-5.

(pin [R,H] bf16, row_id_map [E,T] int64) -> out [T,H] bf16, the unweighted
fp32 sum of kernel_cases/case15_moe_unpermute_mask_fwd.py:58-64, accumulated
in ascending expert order (deterministic, bit-identical to the CPU reference).
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(pin, row_id_map):
    return moe_b200.unpermute(pin, row_id_map)
