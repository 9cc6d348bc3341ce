"""The MoE expert-layer forward as the reference's own PyTorch CPU code
expresses it -- TEST INFRASTRUCTURE / CPU BASELINE ONLY.

A restatement, in torch on the CPU, of the reference cases' Model.forward
chain for this path, op for op, so that the timed CPU baseline runs the
reference's algorithm with the reference's kind of torch calls (bf16
torch.mm per expert, index_select / index_copy_ / index_add_) on all host
cores. Only bench.py's cpu_baseline and --impl reference legs and tests/ may
import it; the product never does. Where the reference has no code for a
step (the softmax router with renormalisation, SwiGLU, the weighted
combine) the restatement is the build's own, as in oracle/moe_oracle.py.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def route(logits: torch.Tensor, bias: torch.Tensor, k: int):
    """Top-k by a full stable descending sort per row (kernel_cases/
    case23_ref_aten_topk.py:47-62, reference_topk), softmax gates of the
    selected experts renormalised (no reference code); returns the bool
    routing map [T,E] and the dense gates [T,E] fp32."""
    lb = logits + bias[None, :]
    idx = torch.sort(lb, dim=1, descending=True, stable=True).indices[:, :k]
    p = torch.softmax(lb, dim=1).gather(1, idx)
    p = p / p.sum(dim=1, keepdim=True)
    rmap = torch.zeros_like(lb, dtype=torch.bool).scatter_(1, idx, True)
    probs = torch.zeros_like(lb).scatter_(1, idx, p)
    return rmap, probs


def make_row_id_map(routing_map: torch.Tensor) -> torch.Tensor:
    """Per-expert cumsum over tokens plus exclusive expert offsets, -1 where
    not routed (kernel_cases/case12_moe_row_id_map_pass2.py:43-50)."""
    mask = routing_map.to(torch.int64)
    within = torch.cumsum(mask, dim=0) - 1
    counts = mask.sum(dim=0)
    offset = torch.cumsum(counts, dim=0) - counts
    return torch.where(mask > 0, within + offset[None, :], torch.full_like(within, -1))


def permute(x: torch.Tensor, row_te: torch.Tensor, num_out: int) -> torch.Tensor:
    """out[row[t,e]] = x[t] (kernel_cases/case17_moe_permute_with_mask_map.py:
    58-71: index_select of the source tokens, index_copy_ into the rows)."""
    t, e = row_te.shape
    dst = row_te.reshape(-1)
    keep = dst >= 0
    tok = torch.arange(t).repeat_interleave(e)[keep]
    out = x.new_zeros((num_out, x.shape[1]))
    out.index_copy_(0, dst[keep], x.index_select(0, tok))
    return out


def grouped_mm(x: torch.Tensor, w, sizes) -> torch.Tensor:
    """cat over groups of x[seg] @ w[g].T in bf16 (kernel_cases/
    case03_moe_grouped_gemm_fc1_fwd.py:57-64, case04…:57-64); w[g] is
    fetched per group, so a sample needs only the experts it reaches."""
    outs, off = [], 0
    for g, m in enumerate(sizes):
        if m:
            outs.append(torch.mm(x[off:off + m], w(g).t()))
        off += m
    return torch.cat(outs, dim=0)


def swiglu(y: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up in fp32, bf16 out (SwiGLU; no reference code)."""
    g, u = y.float().chunk(2, dim=-1)
    return (F.silu(g) * u).to(y.dtype)


def combine(y: torch.Tensor, row_te: torch.Tensor, probs: torch.Tensor) -> torch.Tensor:
    """out[t] = bf16(sum over e of probs[t,e] * y[row[t,e]]) with an fp32
    index_add_ (kernel_cases/case15_moe_unpermute_mask_fwd.py:58-64, here
    weighted by the gates; no reference code for the weights)."""
    row_et = row_te.t()
    valid = row_et >= 0
    src = row_et[valid]
    e_idx, t_idx = valid.nonzero(as_tuple=True)
    w = probs[t_idx, e_idx][:, None]
    out = torch.zeros(row_te.shape[0], y.shape[1], dtype=torch.float32)
    out.index_add_(0, t_idx, y.index_select(0, src).float() * w)
    return out.to(y.dtype)


def layer(x, logits, bias, w1, w2, k: int):
    """router -> row_id_map -> permute -> fc1 -> SwiGLU -> fc2 -> weighted
    combine. w1(e) [2F,H] and w2(e) [H,F] bf16 return expert e's weights."""
    rmap, probs = route(logits, bias, k)
    row_te = make_row_id_map(rmap)
    sizes = rmap.sum(dim=0).tolist()
    xp = permute(x, row_te, int(sum(sizes)))
    h = swiglu(grouped_mm(xp, w1, sizes))
    y = grouped_mm(h, w2, sizes)
    return combine(y, row_te, probs)
