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
                 expert_bias: Optional[torch.Tensor] = None,
                 placement: Optional[torch.Tensor] = None):
        """placement (optional int32 [E] permutation): weights[c] is model expert
        placement[c]; routing, permuted rows and the combine order follow slots."""
        self.w = weights
        self.k = int(topk)
        self.renorm = renorm
        self.bias = expert_bias
        self.placement = placement
        e = weights.num_experts
        self.plan = ops.GroupedGemmPlan(e, weights.w1.device)
        self.events = None  # optional dict name -> torch.cuda.Event for stage timing

    def _ev(self, name: str):
        if self.events is not None:
            self.events[name].record()

    def forward(self, x: torch.Tensor, logits: Optional[torch.Tensor] = None,
                return_intermediates: bool = False,
                router_weight: Optional[torch.Tensor] = None,
                save_for_backward: bool = False):
        """logits [T,E] fp32, or router_weight [E,H] bf16: then the router gate
        GEMM and the router run as one kernel (ops.router_gemm_topk) where it
        covers the shape, else as ops.router_logits + ops.router_topk.

        save_for_backward: return (out, ctx) with what backward() needs; fc1
        then keeps its gate|up output (GEMM with a plain epilogue followed by
        the SwiGLU kernel, the same bits as the fused epilogue)."""
        t, h = x.shape
        e = self.w.num_experts
        if h != self.w.hidden:
            raise ValueError(f"x hidden {h} != weights hidden {self.w.hidden}")
        if logits is None:
            if router_weight is None:
                raise ValueError("pass logits or router_weight")
            if router_weight.shape != (e, h):
                raise ValueError(f"router_weight must be [{e},{h}]")
        elif logits.shape != (t, e):
            raise ValueError(f"logits must be [{t},{e}]")
        self._ev("start")
        # outputs="all": the [T,k] expert list lets the permute read k map
        # entries per token instead of scanning the whole map row
        if logits is None and self.placement is None and ops.router_gemm_fusable(
                x, router_weight, self.k):
            r = ops.router_gemm_topk(x, router_weight, self.k, "softmax", self.renorm, self.bias,
                                     outputs="all")
        else:
            if logits is None:
                logits = ops.router_logits(x, router_weight)
            r = ops.router_topk(logits, self.k, "softmax", self.renorm, self.bias, outputs="all",
                                placement=self.placement)
        rim = ops.row_id_map(r.routing_map, align=1, want_et=False)
        self._ev("routing")
        rows = t * self.k
        xp, _ = ops.permute(x, rim.map_te, None, num_out=rows, experts=r.topk_idx)
        self._ev("permute")
        self.plan.from_splits(rim.counts, 1)
        y1 = None
        if save_for_backward:
            y1 = ops.grouped_gemm(xp, self.w.w1, plan=self.plan)
            hmid = ops.swiglu(y1)
        else:
            hmid = ops.grouped_gemm(xp, self.w.w1, epilogue="swiglu", plan=self.plan)
        self._ev("fc1")
        y = ops.grouped_gemm(hmid, self.w.w2, plan=self.plan)
        self._ev("fc2")
        out = ops.unpermute(y, rim.map_te, r.probs, probs_mode="dense", token_major=True)
        self._ev("combine")
        if return_intermediates or save_for_backward:
            return out, dict(routing=r, rim=rim, xp=xp, y1=y1, h=hmid, y=y)
        return out

    __call__ = forward

    def backward(self, grad_out: torch.Tensor, ctx: dict):
        """Backward of one forward(..., save_for_backward=True), given the
        output gradient grad_out [T,H] bf16. Returns (grad_x [T,H] bf16,
        grad_probs [T,E] fp32 (the gradient of the dense gate matrix, zero
        where a token is not routed; columns in slot order when the layer has
        a placement), dw1 [E,2F,H] bf16, dw2 [E,H,F] bf16).

        The chain, every GEMM grouped by expert on the forward's row layout:
        combine backward -> fc2 dgrad (dh = dy2 @ W2[e]) and wgrad
        (dW2[e] = dy2^T @ h) -> SwiGLU backward -> fc1 dgrad (dxp = dy1 @
        W1[e]) and wgrad (dW1[e] = dy1^T @ xp) -> permute backward (grad_x[t]
        = sum over the token's experts of dxp rows). The router's own backward
        (through softmax, top-k and renormalisation) is the caller's."""
        if ctx.get("y1") is None:
            raise ValueError("ctx must come from forward(..., save_for_backward=True)")
        r, rim = ctx["routing"], ctx["rim"]
        t, h = ctx["xp"].shape[0] // self.k, ctx["xp"].shape[1]
        if grad_out.shape != (t, h):
            raise ValueError(f"grad_out must be [{t},{h}]")
        # The group table of this forward's routing (another forward since may
        # have replaced the layer's); the wgrad takes the same device counts,
        # so the backward never waits for the GPU.
        self.plan.from_splits(rim.counts, 1)
        dy2, grad_probs = ops.combine_backward(grad_out, ctx["y"], rim.map_te, r.probs)
        dh = ops.grouped_gemm(dy2, self.w.w2, plan=self.plan, w_layout="KN")
        dw2 = ops.grouped_wgrad(dy2, ctx["h"], rim.counts)
        dy1 = ops.swiglu_backward(ctx["y1"], dh)
        dxp = ops.grouped_gemm(dy1, self.w.w1, plan=self.plan, w_layout="KN")
        dw1 = ops.grouped_wgrad(dy1, ctx["xp"], rim.counts)
        grad_x = ops.unpermute(dxp, rim.map_te, None, token_major=True)
        return grad_x, grad_probs, dw1, dw2


def moe_layer_fwd(x: torch.Tensor, logits: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                  topk: int = 8, renorm: bool = True,
                  expert_bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Functional form of MoELayer: one expert-layer forward, x [T,H] bf16,
    logits [T,E] fp32, w1 [E,2F,H], w2 [E,H,F] bf16 -> [T,H] bf16."""
    return MoELayer(MoEWeights(w1, w2), topk=topk, renorm=renorm, expert_bias=expert_bias)(x, logits)


class HostPipeline:
    """Runs layer steps whose inputs and outputs live in pinned host memory.

    Each submitted step copies its x and logits host->device on an upload
    stream, runs the layer on the compute stream once its upload has landed,
    and copies the output device->host on a download stream. Uploads of the
    next step and the download of the previous one overlap the current step's
    kernels (the copy engines are independent of the SMs), so a stream of
    steps runs at the pace of the slowest of the three. `depth` device buffer
    slots are cycled; a slot is reused only after the step that read it.
    """

    def __init__(self, layer, tokens: int, hidden: int, num_experts: int, device,
                 depth: int = 2):
        self.layer = layer
        self.depth = depth
        self.dev = torch.device(device)
        self.x = [torch.empty((tokens, hidden), dtype=torch.bfloat16, device=self.dev)
                  for _ in range(depth)]
        self.lg = [torch.empty((tokens, num_experts), dtype=torch.float32, device=self.dev)
                   for _ in range(depth)]
        self.up = torch.cuda.Stream(self.dev)
        self.down = torch.cuda.Stream(self.dev)
        self.compute = torch.cuda.current_stream(self.dev)
        self.uploaded = [torch.cuda.Event() for _ in range(depth)]
        self.consumed = [torch.cuda.Event() for _ in range(depth)]
        self.done = [torch.cuda.Event() for _ in range(depth)]
        self._used = [False] * depth
        self._n = 0

    def _upload(self, s: int, x_host: torch.Tensor, logits_host: torch.Tensor) -> None:
        with torch.cuda.stream(self.up):
            if self._used[s]:
                self.up.wait_event(self.consumed[s])
            self.x[s].copy_(x_host, non_blocking=True)
            self.lg[s].copy_(logits_host, non_blocking=True)
            self.uploaded[s].record(self.up)
        self._used[s] = True

    def _compute_download(self, s: int, out_host: torch.Tensor) -> torch.cuda.Event:
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(self.uploaded[s])
            out = self.layer(self.x[s], self.lg[s])
            self.consumed[s].record(self.compute)
        with torch.cuda.stream(self.down):
            self.down.wait_event(self.consumed[s])
            out_host.copy_(out, non_blocking=True)
            out.record_stream(self.down)
            self.done[s].record(self.down)
        return self.done[s]

    def submit(self, x_host: torch.Tensor, logits_host: torch.Tensor,
               out_host: torch.Tensor) -> torch.cuda.Event:
        """Enqueues one step; returns the event that marks its output on the host."""
        s = self._n % self.depth
        self._n += 1
        self._upload(s, x_host, logits_host)
        return self._compute_download(s, out_host)

    def run(self, steps) -> None:
        """Runs a sequence of (x_host, logits_host, out_host) steps, queueing the
        upload of step i+1 before step i's kernels, so the upload overlaps even
        layers that synchronise with the host mid-forward (the expert-parallel
        layer reads its split sizes)."""
        steps = list(steps)
        if not steps:
            return
        slots = []
        for i, (xh, lh, _) in enumerate(steps):
            if i == 0:
                s = self._n % self.depth
                self._n += 1
                self._upload(s, xh, lh)
                slots.append(s)
            if i + 1 < len(steps):
                s = self._n % self.depth
                self._n += 1
                self._upload(s, steps[i + 1][0], steps[i + 1][1])
                slots.append(s)
            self._compute_download(slots[i], steps[i][2])

    def synchronize(self) -> None:
        self.down.synchronize()
