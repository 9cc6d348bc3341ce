"""One expert's fc1 GEMM, out [M,N] = inp [M,K] @ weight [N,K].T in bf16 with
fp32 accumulation (kernel_cases/case35_ref_musa_asm_bf16_gemm_nt_256x384.py:
41-48 is the fp32 golden; tolerance :66-75). Runs the grouped kernel with G=1.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(inp, weight):
    return moe_b200.grouped_gemm(inp, weight.unsqueeze(0), [inp.shape[0]])
