"""Router gate GEMM, logits [M,N] fp32 = inp [M,K] bf16 @ weight [N,K] bf16 .T
with fp32 accumulation and an unrounded fp32 store
(kernel_cases/case38_ref_musa_asm_bf16_ssgemm_nt_320x256.py:51-59 is the
golden, reference_fp32; M=16384, K=8192, N=320 at the traced shape). Runs the
grouped tcgen05 kernel with one group and the fp32 epilogue.
"""
import sys
from pathlib import Path

_PKG = str(Path(__file__).resolve().parents[2])
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import moe_b200  # noqa: E402


def kernel_function(inp, weight):
    return moe_b200.router_logits(inp, weight)
