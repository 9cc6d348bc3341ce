"""Seeded input generators shared by the golden-fixture script and the tests.

All inputs are torch CPU draws from explicit seeds, so they are identical on
every machine running the same torch build; fixtures store a SHA-256 of each
regenerated input to detect a different RNG.
"""
from __future__ import annotations

import torch

# The reference's full-shape cases draw their activations with these seeds
# (kernel_cases/case17_moe_permute_with_mask_map.py:83-84,
#  kernel_cases/case15_moe_unpermute_mask_fwd.py:74-75).
CASE17_SEED = 20261114
CASE15_SEED = 20261113


def case17_x(tokens: int = 16384, hidden: int = 8192) -> torch.Tensor:
    g = torch.Generator().manual_seed(CASE17_SEED)
    return torch.randn(tokens, hidden, generator=g).to(torch.bfloat16)


def case15_pin(rows: int, hidden: int = 8192) -> torch.Tensor:
    g = torch.Generator().manual_seed(CASE15_SEED)
    return torch.randn(rows, hidden, generator=g).to(torch.bfloat16)


CASE18_SEED = 20261118


def case18_inputs(tokens: int = 4096, hidden: int = 8192, experts: int = 320, topk: int = 8):
    """Seeded draws in the form of case18's get_inputs (kernel_cases/case18_moe_
    permute_bwd_unpermute_mask.py:77-84): random top-k routing [T,E] bool,
    N(0,1) gradients of the permuted rows [T*k,H] bf16 and of the permuted
    probs [T*k] fp32."""
    g = torch.Generator().manual_seed(CASE18_SEED)
    rm = torch.zeros(tokens, experts, dtype=torch.bool)
    idx = torch.argsort(torch.rand(tokens, experts, generator=g), dim=-1)[:, :topk]
    rm.scatter_(1, idx, True)
    dperm = torch.randn(tokens * topk, hidden, generator=g).to(torch.bfloat16)
    dpp = torch.randn(tokens * topk, generator=g, dtype=torch.float32)
    return rm, dperm, dpp


def _randn(seed: int, m: int, n: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(m, n, generator=g, dtype=torch.float32)


def topk_cases() -> dict:
    """Top-k edge suite modelled on the reference's top-k test categories:
    several seeds at the traced shape, other shapes and k, heavy ties,
    all-zero, all-negative and -inf columns."""
    cases = {}
    for s in (0, 1, 7):
        cases[f"seed{s}"] = (_randn(s, 16384, 320), 8)
    for m, n, k in ((1, 320, 8), (17, 320, 8), (1000, 320, 8), (16384, 320, 1), (16384, 320, 4),
                    (256, 64, 8), (128, 33, 8), (64, 16, 3), (512, 256, 8), (300, 1000, 16)):
        cases[f"shape_{m}x{n}_k{k}"] = (_randn(m + n + k, m, n), k)
    g = torch.Generator().manual_seed(3)
    cases["ties"] = (torch.randint(0, 5, (4096, 320), generator=g).float(), 8)
    cases["zeros"] = (torch.zeros(64, 320), 8)
    g = torch.Generator().manual_seed(5)
    cases["negative"] = (-torch.rand(512, 320, generator=g), 8)
    x = _randn(6, 64, 320)
    x[:, :40] = float("-inf")
    cases["neg_inf_cols"] = (x, 8)
    x = _randn(9, 64, 320)
    x[:, 300:] = float("-inf")
    x[::2, 5] = float("-inf")
    cases["neg_inf_tail"] = (x, 8)
    return cases
