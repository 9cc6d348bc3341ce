"""One expert's fc1 dgrad GEMM, out [M,N] = grad_output [M,K] @ weight [K,N]
in bf16 with fp32 accumulation ("NN", _GroupedLinearBackward;
kernel_cases/case37_ref_musa_asm_bf16_gemm_nn_256x384.py:46-48 is the fp32
golden, :66-75 the tolerance). Runs the grouped dgrad kernel with G=1 (the
weight staged MN-major on the tensor cores).
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(grad_output, weight):
    return moe_b200.grouped_gemm(grad_output, weight.unsqueeze(0), [grad_output.shape[0]],
                                 w_layout="KN")
