"""Expert-parallel MoE layer: experts sharded evenly across the ranks of one
node, tokens data-parallel, NCCL all-to-all over NVLink for dispatch and
combine (the traced deep_ep FusedDispatch / FusedCombine hop,
kernel_cases/case22_ref_moe_permute_mask_kernel_true.py:3-6 and
case24_ref_moe_unpermute_mask_kernel_false.py:3-6, named but not present in
the reference).

Rank r owns experts [r*E_loc, (r+1)*E_loc). Because the permuted buffer is
expert-major, the rows bound for rank d are one contiguous block, so the
dispatch is a single all_to_all_single of the permuted buffer:

  1. route, row_id_map, permute locally (expert-major rows)
  2. all-to-all of the per-expert counts ([G, E_loc] int32), then one
     device->host read of the split sizes (the only host sync)
  3. all-to-all of the rows into a local receive buffer laid out as
     (source rank, local expert) segments
  4. fc1+SwiGLU and fc2 grouped GEMMs over those segments, grouped
     expert-major so each local weight matrix is streamed once
  5. all-to-all of the results back (same splits, reversed), which restores
     the local expert-major row order, then the weighted combine.

The collective plumbing (EPDispatcher) is device-agnostic so its protocol
can be tested with gloo on CPU; the layer itself runs only on CUDA.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import ops
from .layer import MoEWeights


class EPDispatcher:
    """Split-size exchange and row all-to-alls for one expert-parallel group."""

    def __init__(self, num_experts: int, group: Optional[dist.ProcessGroup] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split evenly over {self.world} ranks")
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world

    def local_range(self) -> Tuple[int, int]:
        return self.rank * self.local_experts, (self.rank + 1) * self.local_experts

    def exchange_counts(self, counts: torch.Tensor):
        """counts [E] int32 (this rank's tokens per global expert) ->
        (send_splits, recv_splits, recv_counts [G*E_loc] int32 in (src, expert) order)."""
        c = counts.to(torch.int32).contiguous()
        recv = torch.empty_like(c)
        dist.all_to_all_single(recv, c, group=self.group)
        both = torch.stack([c.view(self.world, self.local_experts).sum(1, dtype=torch.int64),
                            recv.view(self.world, self.local_experts).sum(1, dtype=torch.int64)])
        both = both.cpu()  # the one host sync of the forward
        send_splits = [int(v) for v in both[0]]
        recv_splits = [int(v) for v in both[1]]
        return send_splits, recv_splits, recv

    def _rows_a2a(self, src: torch.Tensor, in_splits: List[int], out_splits: List[int],
                  out: Optional[torch.Tensor]) -> torch.Tensor:
        if src.dim() != 2 or src.shape[0] != sum(in_splits):
            raise ValueError(f"rows {tuple(src.shape)} do not match split sizes {in_splits}")
        if out is None:
            out = src.new_empty((sum(out_splits), src.shape[1]))
        # Rows travel as raw bytes: every backend moves uint8, and the copy is
        # bit-exact whatever the element type.
        dist.all_to_all_single(out.view(torch.uint8), src.contiguous().view(torch.uint8),
                               output_split_sizes=out_splits, input_split_sizes=in_splits,
                               group=self.group)
        return out

    def dispatch(self, xp: torch.Tensor, send_splits: List[int], recv_splits: List[int],
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Sends each destination rank its block of expert-major rows."""
        return self._rows_a2a(xp, send_splits, recv_splits, out)

    def combine(self, y: torch.Tensor, send_splits: List[int], recv_splits: List[int],
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Inverse of dispatch: returns rows to their source ranks, in the
        source's original (expert-major) order."""
        return self._rows_a2a(y, recv_splits, send_splits, out)


def ep_group_table(recv_counts, num_src: int, num_w: int):
    """Host restatement of the device group table for a receive buffer of
    (source rank, local expert) segments, groups ordered expert-major:
    returns (row_start, rows, widx) lists. The device planner
    (moe_grouped_gemm_plan_ep) builds the same table on the GPU."""
    c = [int(v) for v in recv_counts]
    pos, acc = [], 0
    for v in c:
        pos.append(acc)
        acc += v
    starts, rows, widx = [], [], []
    for e in range(num_w):
        for s in range(num_src):
            f = s * num_w + e
            starts.append(pos[f])
            rows.append(c[f])
            widx.append(e)
    return starts, rows, widx


class MoELayerEP:
    """Expert-parallel forward; this rank holds the weights of its local experts.

    weights.w1 [E_loc, 2F, H], weights.w2 [E_loc, H, F].
    """

    def __init__(self, local_weights: MoEWeights, num_experts: int, topk: int = 8,
                 renorm: bool = True, expert_bias: Optional[torch.Tensor] = None,
                 group: Optional[dist.ProcessGroup] = None):
        self.disp = EPDispatcher(num_experts, group)
        if local_weights.num_experts != self.disp.local_experts:
            raise ValueError("local weights do not match num_experts / world size")
        self.w = local_weights
        self.k = int(topk)
        self.renorm = renorm
        self.bias = expert_bias
        self.plan = ops.GroupedGemmPlan(self.disp.world * self.disp.local_experts,
                                        local_weights.w1.device)
        self.events = None  # optional dict of CUDA events for stage timing

    def _ev(self, name: str):
        if self.events is not None:
            self.events[name].record()

    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        t, h = x.shape
        e = self.disp.num_experts
        if logits.shape != (t, e):
            raise ValueError(f"logits must be [{t},{e}]")
        self._ev("start")
        r = ops.router_topk(logits, self.k, "softmax", self.renorm, self.bias, outputs="maps")
        rim = ops.row_id_map(r.routing_map, align=1)
        xp, _ = ops.permute(x, rim.map_te, None, num_out=t * self.k)
        self._ev("local_dispatch")
        send, recv, recv_counts = self.disp.exchange_counts(rim.counts)
        xr = self.disp.dispatch(xp, send, recv)
        self._ev("a2a_dispatch")
        self.plan.from_ep_counts(recv_counts, self.disp.world, self.disp.local_experts)
        hmid = ops.grouped_gemm(xr, self.w.w1, epilogue="swiglu", plan=self.plan)
        self._ev("fc1")
        y = ops.grouped_gemm(hmid, self.w.w2, plan=self.plan)
        self._ev("fc2")
        yb = self.disp.combine(y, send, recv)
        self._ev("a2a_combine")
        out = ops.unpermute(yb, rim.map_et, r.probs, probs_mode="dense")
        self._ev("combine")
        return out

    __call__ = forward
