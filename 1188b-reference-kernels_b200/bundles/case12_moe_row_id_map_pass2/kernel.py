"""Drop-in for kernel_results/case12_moe_row_id_map_pass2/kernel.py:4-6.

routing_map [T,E] bool -> (row_id_map [E,T] int64, row_id_map [T,E] int64),
the output order of kernel_cases/case12_moe_row_id_map_pass2.py:53-61.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(routing_map):
    r = moe_b200.row_id_map(routing_map, align=1)
    return r.map_et, r.map_te
