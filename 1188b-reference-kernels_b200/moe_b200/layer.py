"""Single-GPU MoE expert-layer forward built from the sm_100a kernels.

    logits (+bias) -> router top-k (softmax gates, renormalised)
                   -> row_id_map (both layouts, per-expert counts on device)
                   -> permute x into the expert-major buffer
                   -> fc1 grouped GEMM with fused SwiGLU
                   -> fc2 grouped GEMM
                   -> prob-weighted combine back to token order

This is the chain the reference traces (router topk case23 -> row_id_map
case12 -> permute case17 -> fc1 case03 -> SwiGLU -> fc2 case04 -> unpermute
case15/case24), with the combine weighted by the router gates. Every stage
runs on the current CUDA stream with no host synchronisation: with top-k
routing and no token dropping the permuted buffer always has T*k rows, and
the per-expert row counts stay on the device.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import ops


@dataclass
class MoEWeights:
    """Expert FFN weights in the reference "[out,in]" layout.

    w1 [E, 2F, H]: rows [0,F) gate, [F,2F) up (fc1, case03 layout)
    w2 [E, H, F]: fc2 (case04 layout)
    """
    w1: torch.Tensor
    w2: torch.Tensor

    @property
    def num_experts(self) -> int:
        return self.w1.shape[0]

    @property
    def hidden(self) -> int:
        return self.w1.shape[2]

    @property
    def ffn(self) -> int:
        return self.w2.shape[2]

    @staticmethod
    def random(num_experts: int, hidden: int, ffn: int, device, seed: int = 0,
               std: float = 0.02) -> "MoEWeights":
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        w1 = torch.empty((num_experts, 2 * ffn, hidden), dtype=torch.bfloat16, device=device)
        w2 = torch.empty((num_experts, hidden, ffn), dtype=torch.bfloat16, device=device)
        w1.normal_(0.0, std, generator=g)
        w2.normal_(0.0, std, generator=g)
        return MoEWeights(w1, w2)


class MoELayer:
    """Forward of one MoE expert layer on one GPU (inputs already on device)."""

    def __init__(self, weights: MoEWeights, topk: int = 8, renorm: bool = True,
                 expert_bias: Optional[torch.Tensor] = None):
        self.w = weights
        self.k = int(topk)
        self.renorm = renorm
        self.bias = expert_bias
        e = weights.num_experts
        self.plan = ops.GroupedGemmPlan(e, weights.w1.device)
        self.events = None  # optional dict name -> torch.cuda.Event for stage timing

    def _ev(self, name: str):
        if self.events is not None:
            self.events[name].record()

    def forward(self, x: torch.Tensor, logits: torch.Tensor, return_intermediates: bool = False):
        t, h = x.shape
        e = self.w.num_experts
        if logits.shape != (t, e):
            raise ValueError(f"logits must be [{t},{e}]")
        if h != self.w.hidden:
            raise ValueError(f"x hidden {h} != weights hidden {self.w.hidden}")
        self._ev("start")
        r = ops.router_topk(logits, self.k, "softmax", self.renorm, self.bias, outputs="maps")
        rim = ops.row_id_map(r.routing_map, align=1)
        self._ev("routing")
        rows = t * self.k
        xp, _ = ops.permute(x, rim.map_te, None, num_out=rows)
        self._ev("permute")
        self.plan.from_splits(rim.counts, 1)
        hmid = ops.grouped_gemm(xp, self.w.w1, epilogue="swiglu", plan=self.plan)
        self._ev("fc1")
        y = ops.grouped_gemm(hmid, self.w.w2, plan=self.plan)
        self._ev("fc2")
        out = ops.unpermute(y, rim.map_et, r.probs, probs_mode="dense")
        self._ev("combine")
        if return_intermediates:
            return out, dict(routing=r, rim=rim, xp=xp, h=hmid, y=y)
        return out

    __call__ = forward
