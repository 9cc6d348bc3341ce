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

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib

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


def balanced_placement(load: Sequence[float], world: int) -> List[int]:
    """Expert placement with exactly E/world experts per rank and balanced load.

    Greedy longest-processing-time: experts in decreasing load go to the rank
    with the least load that still has a free slot. Returns the model expert
    ids in slot order (rank r owns slots [r*E/world, (r+1)*E/world)), each
    rank's experts in ascending id order.
    """
    e = len(load)
    if e % world:
        raise ValueError(f"{e} experts do not split evenly over {world} ranks")
    per = e // world
    order = sorted(range(e), key=lambda i: (-float(load[i]), i))
    bins = [[] for _ in range(world)]
    tot = [0.0] * world
    for i in order:
        d = min((r for r in range(world) if len(bins[r]) < per), key=lambda r: (tot[r], r))
        bins[d].append(i)
        tot[d] += float(load[i])
    return [i for b in bins for i in sorted(b)]


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


@dataclass
class ExchangePlan:
    """Split sizes and row offsets of one EP exchange, seen from one rank.

    blk[s][d] = rows rank s sends to rank d (its tokens routed to d's experts).
    """
    send: List[int]       # rows this rank sends to each d (its xp block for d)
    recv: List[int]       # rows this rank receives from each s
    send_off: List[int]   # start of the block for d in this rank's xp
    recv_off: List[int]   # start of the rows from s in this rank's receive buffer
    dst_off: List[int]    # where this rank's block starts in d's receive buffer
    back_off: List[int]   # where the results for s start in s's return buffer


def exchange_plan(counts_all: Sequence[Sequence[int]], rank: int, local_experts: int) -> ExchangePlan:
    """Host computation of every split and offset from the gathered [G, E]
    per-expert token counts (row s = rank s's counts for all E experts)."""
    g = len(counts_all)
    el = local_experts
    blk = [[int(sum(counts_all[s][d * el:(d + 1) * el])) for d in range(g)] for s in range(g)]

    def prefix(v):
        out, acc = [], 0
        for x in v:
            out.append(acc)
            acc += x
        return out

    send = blk[rank]
    recv = [blk[s][rank] for s in range(g)]
    dst_off = [sum(blk[s][d] for s in range(rank)) for d in range(g)]
    back_off = [sum(blk[s][d] for d in range(rank)) for s in range(g)]
    return ExchangePlan(send, recv, prefix(send), prefix(recv), dst_off, back_off)


class ExpertMajorLayout:
    """Receive layout of the fused transport, seen from one rank.

    Every owner stores its local experts one after another, and inside each
    expert the rows of source 0, 1, ... in order, so each local expert is one
    contiguous GEMM group.
    """

    def __init__(self, deltas: List[int], splits: List[int], recv_rows: List[int]):
        self.deltas = deltas        # [E]: row in the owner's buffer = this rank's permuted row + deltas[e]
        self.splits = splits        # [E_loc]: rows this rank receives per local expert
        self.recv_rows = recv_rows  # [G]: rows every rank receives


def expert_major_layout(counts_all: Sequence[Sequence[int]], rank: int,
                        local_experts: int) -> ExpertMajorLayout:
    """Row shifts and group sizes of the expert-major receive layout from the
    gathered [G, E] per-expert counts (row s = rank s's counts). This rank's
    permuted rows of expert e start at the prefix of its own counts; in the
    owner's buffer they start after the owner's lower experts and after the
    rows of expert e from lower-numbered sources."""
    import numpy as np
    c = np.asarray(counts_all, dtype=np.int64)
    g, e = c.shape
    el = int(local_experts)
    if e != g * el:
        raise ValueError("counts do not match world size x local experts")
    tot = c.sum(axis=0).reshape(g, el)                  # rows per expert, by owner
    blk = (np.cumsum(tot, axis=1) - tot).reshape(-1)    # expert's block start in its owner
    before = c[:rank].sum(axis=0)                       # rows of lower sources, per expert
    src_start = np.cumsum(c[rank]) - c[rank]
    deltas = blk + before - src_start
    return ExpertMajorLayout([int(v) for v in deltas], [int(v) for v in tot[rank]],
                             [int(v) for v in tot.sum(axis=1)])


def pull_group_table(counts_all: Sequence[Sequence[int]], rank: int, local_experts: int):
    """Group table of the pull dispatch on `rank` from the gathered [G, E]
    per-expert counts: for group g = le * G + s (local expert le, source s),
    the first receive row, the row count and the source's first permuted row
    of that expert. The receive rows are those of expert_major_layout (the
    push dispatch's): source s's rows of expert e land at its permuted row +
    deltas_s[e]. Returns three lists of G * local_experts ints."""
    import numpy as np
    c = np.asarray(counts_all, dtype=np.int64)
    g, e = c.shape
    el = int(local_experts)
    if e != g * el:
        raise ValueError("counts do not match world size x local experts")
    mine = c[:, rank * el:(rank + 1) * el]                        # [G sources, E_loc]
    src_start = (np.cumsum(c, axis=1) - c)[:, rank * el:(rank + 1) * el]
    cnt = mine.T.reshape(-1)                                       # le-major, then source
    start = np.cumsum(cnt) - cnt
    src0 = src_start.T.reshape(-1)
    return [int(v) for v in start], [int(v) for v in cnt], [int(v) for v in src0]


class EPPeerExchange:
    """Row exchange through peer-mapped buffers and the copy engines.

    Every rank registers a receive buffer (capacity world*T*k rows) and a
    return buffer (T*k rows) once, with CUDA IPC. Dispatch: each rank copies
    its block for rank d straight into d's receive buffer; combine: each rank
    copies the results for rank s straight into s's return buffer. One copy
    per peer, on parallel side streams, then a one-element NCCL all-reduce as
    a stream-ordered barrier so no rank reads a buffer before every copy into
    it has finished. Buffers are reused across forwards without double
    buffering: a rank can only start the next dispatch after the previous
    combine, which needs every peer's GEMMs of the previous step.
    """

    def __init__(self, num_experts: int, tokens: int, hidden: int, topk: int,
                 device: torch.device, group: Optional[dist.ProcessGroup] = None,
                 fused: bool = False, dedup: bool = False, pull: bool = False):
        """fused=False: receive + return buffers, rows moved by copy engines.
        fused=True: receive + fc2-output buffers; the dispatch kernel stores
        rows into the peers' receive buffers and the combine kernel loads the
        results from the peers' fc2 outputs. dedup=True (with fused): a token
        row crosses NVLink once per destination rank into that rank's staging
        rows, and each rank expands them into its receive buffer."""
        self.fused = fused
        self.dedup = bool(dedup and fused)
        self.pull = bool(pull and fused and not self.dedup)
        self.topk = int(topk)
        self.tokens = int(tokens)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split evenly over {self.world} ranks")
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world
        self.rows_cap = tokens * topk
        self.row_bytes = hidden * 2
        self.device = torch.device(device)
        self.recv_cap = self.world * self.rows_cap
        self.recv_buf = torch.empty((self.recv_cap, hidden), dtype=torch.bfloat16,
                                    device=self.device)
        self.side = [torch.cuda.Stream(self.device) for _ in range(self.world)]
        self.flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._opened: List[int] = []
        self.peer_recv = self._share(self.recv_buf)
        if fused:
            self.y_buf = torch.empty((self.recv_cap, hidden), dtype=torch.bfloat16,
                                     device=self.device)
            self.peer_y = self._share(self.y_buf)
        if self.pull:
            # this rank's staged token rows and permuted row -> token index,
            # read by the receivers of the pull dispatch
            self.xs_buf = torch.empty((self.tokens, hidden), dtype=torch.bfloat16,
                                      device=self.device)
            self.inv_buf = torch.empty((self.rows_cap,), dtype=torch.int32, device=self.device)
            self.peer_xs = self._share(self.xs_buf)
            self.peer_inv = self._share(self.inv_buf)
        if self.dedup:
            rows = self.world * self.tokens
            self.stage_buf = torch.empty((rows, hidden), dtype=torch.bfloat16, device=self.device)
            self.stage_meta = torch.empty((rows, self.local_experts), dtype=torch.int32,
                                          device=self.device)
            self.stage_count = torch.zeros(self.world, dtype=torch.int32, device=self.device)
            self.peer_stage = self._share(self.stage_buf)
            self.peer_meta = self._share(self.stage_meta)
            self.peer_count = self._share(self.stage_count)
        else:
            self.ret_buf = torch.empty((self.rows_cap, hidden), dtype=torch.bfloat16,
                                       device=self.device)
            self.peer_ret = self._share(self.ret_buf)

    def _share(self, t: torch.Tensor) -> List[int]:
        lib = _lib.load()
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        _lib.call("moe_ipc_get_handle", t.data_ptr(), handle, ctypes.byref(off))
        mine = (bytes(handle.raw), int(off.value))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=self.group)
        ptrs = []
        for r, (h, o) in enumerate(allh):
            if r == self.rank:
                ptrs.append(t.data_ptr())
                continue
            base = ctypes.c_void_p(0)
            _lib.call("moe_ipc_open_handle", ctypes.create_string_buffer(h, 64), ctypes.byref(base))
            self._opened.append(base.value)
            ptrs.append(base.value + o)
        del lib
        return ptrs

    def _gather_counts(self, counts: torch.Tensor) -> torch.Tensor:
        c = counts.to(torch.int32).contiguous()
        allc = torch.empty((self.world * self.num_experts,), dtype=torch.int32, device=c.device)
        dist.all_gather_into_tensor(allc, c, group=self.group)
        return allc.view(self.world, self.num_experts)

    def exchange_counts(self, counts: torch.Tensor):
        """All-gathers the per-expert counts; returns (plan, recv_counts [G*E_loc]
        int32 on the device in (source, local expert) order)."""
        m = self._gather_counts(counts)
        e0 = self.rank * self.local_experts
        recv_counts = m[:, e0:e0 + self.local_experts].contiguous().view(-1)
        host = m.cpu().tolist()  # the one host sync of the forward
        return exchange_plan(host, self.rank, self.local_experts), recv_counts

    def expert_major(self, counts: torch.Tensor):
        """All-gathers the per-expert counts (the one host sync of the forward);
        returns (layout, [G][E] counts on the host, device int64 [E] row shifts)."""
        host = self._gather_counts(counts).cpu().tolist()
        lay = expert_major_layout(host, self.rank, self.local_experts)
        if max(lay.recv_rows) > self.recv_cap:
            raise ValueError("exchange exceeds a receive buffer")
        deltas = torch.tensor(lay.deltas, dtype=torch.int64).to(self.device, non_blocking=True)
        return lay, host, deltas

    def _copies(self, jobs):
        main = torch.cuda.current_stream(self.device)
        ready = torch.cuda.Event()
        ready.record(main)
        done = []
        for i, (dst, src, nbytes) in enumerate(jobs):
            if nbytes == 0:
                continue
            st = self.side[i % len(self.side)]
            st.wait_event(ready)
            _lib.call("moe_copy_async", dst, src, nbytes, st.cuda_stream)
            ev = torch.cuda.Event()
            ev.record(st)
            done.append(ev)
        for ev in done:
            main.wait_event(ev)
        dist.all_reduce(self.flag, group=self.group)  # every rank's copies have landed

    def dispatch(self, xp: torch.Tensor, plan: ExchangePlan) -> torch.Tensor:
        if xp.shape[0] != sum(plan.send) or sum(plan.recv) > self.recv_buf.shape[0]:
            raise ValueError("rows do not match the exchanged counts or exceed the buffer")
        rb = self.row_bytes
        base = xp.data_ptr()
        jobs = [(self.peer_recv[d] + plan.dst_off[d] * rb, base + plan.send_off[d] * rb,
                 plan.send[d] * rb) for d in range(self.world)]
        self._copies(jobs)
        return self.recv_buf[:sum(plan.recv)]

    def combine(self, y: torch.Tensor, plan: ExchangePlan) -> torch.Tensor:
        if y.shape[0] != sum(plan.recv):
            raise ValueError("result rows do not match the received rows")
        rb = self.row_bytes
        base = y.data_ptr()
        jobs = [(self.peer_ret[s] + plan.back_off[s] * rb, base + plan.recv_off[s] * rb,
                 plan.recv[s] * rb) for s in range(self.world)]
        self._copies(jobs)
        return self.ret_buf[:sum(plan.send)]

    def barrier(self) -> None:
        """Stream-ordered barrier: returns (on the device) once every rank's
        earlier work on its stream has finished."""
        dist.all_reduce(self.flag, group=self.group)

    def fused_dispatch(self, x: torch.Tensor, map_te: torch.Tensor, deltas: torch.Tensor,
                       nsend: int, nrecv: int) -> torch.Tensor:
        """Permutes x straight into the owners' receive buffers (row of expert
        e at its permuted row + deltas[e]), then barriers."""
        t, h = x.shape
        bases = (ctypes.c_int64 * self.world)(*self.peer_recv)
        _lib.call("moe_ep_dispatch", x.data_ptr(), map_te.data_ptr(), bases, deltas.data_ptr(),
                  self.world, self.local_experts, self.recv_cap, t, h, self.num_experts, nsend,
                  torch.cuda.current_stream(self.device).cuda_stream)
        self.barrier()
        return self.recv_buf[:nrecv]

    def dispatch_range(self, x: torch.Tensor, map_te: torch.Tensor, deltas: torch.Tensor,
                       nsend: int, local_lo: int, local_hi: int, max_ctas: int) -> None:
        """One chunk of the fused dispatch on the current stream, no barrier:
        the rows of every (t, e) whose local expert index e % E_loc is in
        [local_lo, local_hi), stored straight into the owners' receive
        buffers by a persistent kernel of at most max_ctas CTAs."""
        t, h = x.shape
        bases = (ctypes.c_int64 * self.world)(*self.peer_recv)
        _lib.call("moe_ep_dispatch_range", x.data_ptr(), map_te.data_ptr(), bases,
                  deltas.data_ptr(), self.world, self.local_experts, self.recv_cap, t, h,
                  self.num_experts, nsend, int(local_lo), int(local_hi), int(max_ctas),
                  torch.cuda.current_stream(self.device).cuda_stream)

    def fused_dispatch_pull(self, x: torch.Tensor, map_te: torch.Tensor, counts_all,
                            nsend: int, nrecv: int) -> torch.Tensor:
        """Stages x and the permuted-row -> token index of this rank, barriers,
        then loads this rank's receive rows from their sources (the rows of
        the push dispatch, in the same places)."""
        t, h = x.shape
        if t > self.tokens:
            raise ValueError(f"{t} tokens exceed the staging capacity of {self.tokens}")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.call("moe_ep_pull_stage", x.data_ptr(), map_te.data_ptr(), t, h, self.num_experts,
                  nsend, self.xs_buf.data_ptr(), self.inv_buf.data_ptr(), stream)
        start, cnt, src0 = pull_group_table(counts_all, self.rank, self.local_experts)
        table = torch.tensor(start + cnt + src0, dtype=torch.int32).pin_memory().to(
            self.device, non_blocking=True)
        self.barrier()  # every rank's staged rows and index are in place
        n = self.world
        arr = lambda v: (ctypes.c_int64 * n)(*v)  # noqa: E731
        _lib.call("moe_ep_dispatch_pull", arr(self.peer_xs), arr(self.peer_inv), n, self.tokens,
                  self.rows_cap, table.data_ptr(), len(start), self.recv_buf.data_ptr(), nrecv,
                  self.recv_cap, h, stream)
        return self.recv_buf[:nrecv]

    def fused_dispatch_dedup(self, x: torch.Tensor, map_te: torch.Tensor, deltas: torch.Tensor,
                             nsend: int, nrecv: int) -> torch.Tensor:
        """Token rows once per destination rank into the peers' staging rows
        (own experts straight into the receive buffer), barrier, then this
        rank's expansion of its staging rows into the receive buffer."""
        t, h = x.shape
        if t > self.tokens:
            raise ValueError(f"{t} tokens exceed the staging capacity of {self.tokens}")
        n = self.world
        arr = lambda v: (ctypes.c_int64 * n)(*v)  # noqa: E731
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.call("moe_ep_dispatch_dedup", x.data_ptr(), map_te.data_ptr(), arr(self.peer_recv),
                  deltas.data_ptr(), arr(self.peer_stage), arr(self.peer_meta),
                  arr(self.peer_count), n, self.rank, self.local_experts, self.recv_cap, t, h,
                  self.num_experts, nsend, stream)
        self.barrier()
        _lib.call("moe_ep_expand", self.stage_buf.data_ptr(), self.stage_meta.data_ptr(),
                  self.stage_count.data_ptr(), self.recv_buf.data_ptr(), n, self.rank,
                  self.local_experts, self.tokens, self.recv_cap, h, stream)
        return self.recv_buf[:nrecv]

    def fused_combine(self, map_te: torch.Tensor, probs: Optional[torch.Tensor],
                      deltas: torch.Tensor, nsend: int, tokens: int, hidden: int) -> torch.Tensor:
        """Weighted combine reading every result row from the rank that made it
        (call after every rank's fc2 wrote into y_buf and barrier())."""
        bases = (ctypes.c_int64 * self.world)(*self.peer_y)
        out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=self.device)
        _lib.call("moe_ep_combine", bases, deltas.data_ptr(), self.world, self.local_experts,
                  self.recv_cap, map_te.data_ptr(), None if probs is None else probs.data_ptr(),
                  out.data_ptr(), tokens, hidden, self.num_experts, nsend,
                  torch.cuda.current_stream(self.device).cuda_stream)
        return out

    def close(self) -> None:
        if self._opened:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            for b in self._opened:
                _lib.call("moe_ipc_close_handle", b)
            self._opened = []


class MoELayerEP:
    """Expert-parallel forward; this rank holds the weights of its local experts.

    weights.w1 [E_loc, 2F, H], weights.w2 [E_loc, H, F].
    """

    def __init__(self, local_weights: MoEWeights, num_experts: int, topk: int = 8,
                 renorm: bool = True, expert_bias: Optional[torch.Tensor] = None,
                 group: Optional[dist.ProcessGroup] = None, transport: str = "nccl",
                 tokens: Optional[int] = None, placement: Optional[torch.Tensor] = None,
                 overlap_chunks: int = 1):
        """transport "nccl": all_to_all_single of counts and rows; "peer": IPC-mapped
        buffers filled by copy-engine pushes; "fused": the dispatch and combine
        kernels store / load rows in the peers' buffers directly; "fused_dedup":
        as "fused", with each token row sent once per destination rank and
        expanded there; "fused_pull": as "fused", with each receiver loading
        its rows from the sources' staged rows instead of the sources storing
        them. "peer" and "fused*" need `tokens`, the per-rank T. placement (int32 [E] permutation):
        slot c is model expert placement[c]; this rank holds the weights of
        slots [rank*E_loc, (rank+1)*E_loc) (e.g. from balanced_placement).

        overlap_chunks (transport "fused" only): C > 1 splits every rank's local
        experts into C contiguous chunks. Chunk c's rows are dispatched and
        barriered on a side stream; chunk c's fc1/fc2 run on the caller's
        stream once its barrier has passed, while chunk c+1's rows already
        cross NVLink. The dispatch kernel is persistent with about one small
        CTA per SM, so it fits beside the GEMM's CTAs; the two kernels share
        no data and never wait on each other on the device. The output is the
        same, bit for bit, as with C = 1 (same receive rows, same GEMM
        groups, same combine)."""
        self.placement = placement
        self.disp = EPDispatcher(num_experts, group)
        self.peer = None
        self.fused = transport in ("fused", "fused_dedup", "fused_pull")
        if transport in ("peer", "fused", "fused_dedup", "fused_pull"):
            if tokens is None:
                raise ValueError(f"transport='{transport}' needs the per-rank token count")
            self.peer = EPPeerExchange(num_experts, tokens, local_weights.hidden, topk,
                                       local_weights.w1.device, group, fused=self.fused,
                                       dedup=transport == "fused_dedup",
                                       pull=transport == "fused_pull")
        elif transport != "nccl":
            raise ValueError("transport must be 'nccl', 'peer', 'fused', 'fused_dedup' or "
                             "'fused_pull'")
        if local_weights.num_experts != self.disp.local_experts:
            raise ValueError("local weights do not match num_experts / world size")
        self.w = local_weights
        self.k = int(topk)
        self.renorm = renorm
        self.bias = expert_bias
        # fused: one group per local expert (expert-major receive layout);
        # otherwise one group per (source rank, local expert).
        groups = self.disp.local_experts * (1 if self.fused else self.disp.world)
        self.plan = ops.GroupedGemmPlan(groups, local_weights.w1.device)
        self._deltas = None
        self.events = None  # optional dict of CUDA events for stage timing
        self.chunks = int(overlap_chunks)
        if self.chunks < 1 or self.chunks > self.disp.local_experts:
            raise ValueError(f"overlap_chunks must be in [1, {self.disp.local_experts}]")
        if self.chunks > 1 and transport != "fused":
            raise ValueError("overlap_chunks > 1 needs transport='fused'")
        self._bounds = self.chunk_bounds(self.disp.local_experts, self.chunks)
        self._chunk_plans = [ops.GroupedGemmPlan(hi - lo, local_weights.w1.device)
                             for lo, hi in self._bounds] if self.chunks > 1 else []
        self._comm = None
        self._sms = 0
        self.last_recv_rows = 0  # rows this rank's experts received in the last forward

    def _ev(self, name: str):
        if self.events is not None:
            self.events[name].record()

    def forward(self, x: torch.Tensor, logits: torch.Tensor, save_for_backward: bool = False):
        """One expert-parallel forward of this rank's tokens x [T,H] with router
        logits [T,E]. save_for_backward (transports "fused" and "fused_dedup"):
        returns (out, ctx) for backward(); fc1 then keeps
        its gate|up output, and the received rows are copied out of the
        receive buffer, which the backward reuses for the fc2 gradient rows."""
        t, h = x.shape
        e = self.disp.num_experts
        if logits.shape != (t, e):
            raise ValueError(f"logits must be [{t},{e}]")
        if save_for_backward and not self.fused:
            raise ValueError("save_for_backward needs transport 'fused' or 'fused_dedup'")
        self._ev("start")
        r = ops.router_topk(logits, self.k, "softmax", self.renorm, self.bias, outputs="maps",
                            placement=self.placement)
        rim = ops.row_id_map(r.routing_map, align=1, want_et=False)
        if self.fused:
            return self._forward_fused(x, r, rim, save_for_backward)
        xp, _ = ops.permute(x, rim.map_te, None, num_out=t * self.k)
        self._ev("local_dispatch")
        if self.peer is not None:
            plan, recv_counts = self.peer.exchange_counts(rim.counts)
            xr = self.peer.dispatch(xp, plan)
        else:
            send, recv, recv_counts = self.disp.exchange_counts(rim.counts)
            xr = self.disp.dispatch(xp, send, recv)
        self._ev("a2a_dispatch")
        self.plan.from_ep_counts(recv_counts, self.disp.world, self.disp.local_experts)
        self.last_recv_rows = int(xr.shape[0])
        hmid = ops.grouped_gemm(xr, self.w.w1, epilogue="swiglu", plan=self.plan)
        self._ev("fc1")
        y = ops.grouped_gemm(hmid, self.w.w2, plan=self.plan)
        self._ev("fc2")
        if self.peer is not None:
            yb = self.peer.combine(y, plan)
        else:
            yb = self.disp.combine(y, send, recv)
        self._ev("a2a_combine")
        out = ops.unpermute(yb, rim.map_te, r.probs, probs_mode="dense", token_major=True)
        self._ev("combine")
        return out

    def _forward_fused(self, x, r, rim, save=False):
        t, h = x.shape
        self._ev("local_dispatch")
        lay, host, deltas = self.peer.expert_major(rim.counts)
        self._deltas = deltas  # read by both fused kernels of this forward
        nsend = int(sum(host[self.peer.rank]))
        nrecv = int(sum(lay.splits))
        self.last_recv_rows = nrecv
        ctx = None
        if self.chunks > 1:
            saved = self._chunked_experts(x, rim.map_te, deltas, nsend, lay.splits, save)
            if save:
                ctx = dict(routing=r, rim=rim, deltas=deltas, splits=list(lay.splits),
                           nsend=nsend, xr=self.peer.recv_buf[:nrecv].clone(), y1=saved[0],
                           h=saved[1], tokens=t)
        else:
            if self.peer.dedup:
                xr = self.peer.fused_dispatch_dedup(x, rim.map_te, deltas, nsend, nrecv)
            elif self.peer.pull:
                xr = self.peer.fused_dispatch_pull(x, rim.map_te, host, nsend, nrecv)
            else:
                xr = self.peer.fused_dispatch(x, rim.map_te, deltas, nsend, nrecv)
            self._ev("a2a_dispatch")
            self.plan.from_splits(torch.tensor(lay.splits, dtype=torch.int32))
            if save:
                y1 = ops.grouped_gemm(xr, self.w.w1, plan=self.plan)
                hmid = ops.swiglu(y1)  # the fused SwiGLU epilogue's bits
                ctx = dict(routing=r, rim=rim, deltas=deltas, splits=list(lay.splits),
                           nsend=nsend, xr=xr.clone(), y1=y1, h=hmid, tokens=t)
            else:
                hmid = ops.grouped_gemm(xr, self.w.w1, epilogue="swiglu", plan=self.plan)
            self._ev("fc1")
            ops.grouped_gemm(hmid, self.w.w2, plan=self.plan, out=self.peer.y_buf[:xr.shape[0]])
        self._ev("fc2")
        self.peer.barrier()
        self._ev("a2a_combine")
        out = self.peer.fused_combine(rim.map_te, r.probs, deltas, nsend, t, h)
        self._ev("combine")
        return (out, ctx) if save else out

    def backward(self, grad_out: torch.Tensor, ctx: dict):
        """Backward of one forward(..., save_for_backward=True) of this rank's
        tokens; call it on every rank, before the layer's next forward (the
        fc2 outputs it reads stay in the peer-shared output buffers only until
        then). Returns (grad_x [T,H] bf16, grad_probs [T,E] fp32 in slot
        order, dw1 [E_loc,2F,H], dw2 [E_loc,H,F]) -- the gradients of this
        rank's tokens and of this rank's experts, the same bits as
        MoELayer.backward on all ranks' tokens with all experts.

          1. combine backward over NVLink (moe_ep_combine_backward): gate
             gradients from the owners' fc2 rows, fc2 gradient rows stored
             into the owners' receive buffers at the forward's rows; barrier;
          2. on the local experts, grouped by the forward's expert-major
             receive layout: fc2 dgrad and wgrad, SwiGLU backward, fc1 dgrad
             (written into the peer-shared output buffer) and wgrad; barrier;
          3. permute backward: grad_x[t] = the unweighted fused combine of the
             fc1 dgrad rows, read back from their owners."""
        if ctx is None or "xr" not in ctx:
            raise ValueError("ctx must come from forward(..., save_for_backward=True)")
        t = ctx["tokens"]
        h = self.w.hidden
        if grad_out.shape != (t, h) or grad_out.dtype != torch.bfloat16:
            raise ValueError(f"grad_out must be bf16 [{t},{h}]")
        r, rim, deltas = ctx["routing"], ctx["rim"], ctx["deltas"]
        nsend = ctx["nsend"]
        nrecv = ctx["xr"].shape[0]
        peer = self.peer
        e = self.disp.num_experts
        go = grad_out.contiguous()
        grad_probs = torch.empty((t, e), dtype=torch.float32, device=go.device)
        n = peer.world
        arr = lambda v: (ctypes.c_int64 * n)(*v)  # noqa: E731
        _lib.call("moe_ep_combine_backward", go.data_ptr(), rim.map_te.data_ptr(),
                  r.probs.data_ptr(), arr(peer.peer_y), arr(peer.peer_recv), deltas.data_ptr(),
                  n, self.disp.local_experts, peer.recv_cap, grad_probs.data_ptr(), t, h, e,
                  nsend, torch.cuda.current_stream(go.device).cuda_stream)
        peer.barrier()
        dy2 = peer.recv_buf[:nrecv]
        sp = torch.tensor(ctx["splits"], dtype=torch.int32).pin_memory().to(go.device,
                                                                            non_blocking=True)
        self.plan.from_splits(sp)
        dh = ops.grouped_gemm(dy2, self.w.w2, plan=self.plan, w_layout="KN")
        dw2 = ops.grouped_wgrad(dy2, ctx["h"], sp)
        dy1 = ops.swiglu_backward(ctx["y1"], dh)
        ops.grouped_gemm(dy1, self.w.w1, plan=self.plan, w_layout="KN",
                         out=peer.y_buf[:nrecv])
        dw1 = ops.grouped_wgrad(dy1, ctx["xr"], sp)
        peer.barrier()
        grad_x = peer.fused_combine(rim.map_te, None, deltas, nsend, t, h)
        return grad_x, grad_probs, dw1, dw2

    @staticmethod
    def chunk_bounds(local_experts: int, chunks: int):
        """[lo, hi) local-expert ranges of the overlap chunks: contiguous, in
        order, sizes differing by at most one."""
        el = int(local_experts)
        return [(el * c // chunks, el * (c + 1) // chunks) for c in range(chunks)]

    def _chunked_experts(self, x, map_te, deltas, nsend, splits, save=False):
        """Dispatch (side stream) and fc1/fc2 (caller's stream) chunk by chunk
        of the local experts; see overlap_chunks. Stage events: a2a_dispatch
        when chunk 0 is ready, fc1 after the last chunk's fc1. With save, fc1
        keeps its gate|up output: returns (y1 [rows,2F], h [rows,F])."""
        dev = x.device
        main = torch.cuda.current_stream(dev)
        if self._comm is None:
            self._comm = torch.cuda.Stream(dev)
            self._sms = torch.cuda.get_device_properties(dev).multi_processor_count
        comm = self._comm
        starts = [0]
        for v in splits:
            starts.append(starts[-1] + int(v))
        # Group sizes of every chunk on the device up front, so no chunk's
        # plan waits on a host copy between the GEMM launches.
        sp = torch.tensor([int(v) for v in splits], dtype=torch.int32).pin_memory().to(
            dev, non_blocking=True)
        comm.wait_stream(main)
        for tt in (x, map_te, deltas):
            tt.record_stream(comm)
        ready = []
        with torch.cuda.stream(comm):
            for lo, hi in self._bounds:
                self.peer.dispatch_range(x, map_te, deltas, nsend, lo, hi, self._sms)
                self.peer.barrier()  # every rank's rows of this chunk have landed
                ev = torch.cuda.Event()
                ev.record(comm)
                ready.append(ev)
        last = len(self._bounds) - 1
        y1 = h = None
        if save:
            f = self.w.ffn
            y1 = torch.empty((starts[-1], 2 * f), dtype=torch.bfloat16, device=dev)
            h = torch.empty((starts[-1], f), dtype=torch.bfloat16, device=dev)
        for c, (lo, hi) in enumerate(self._bounds):
            main.wait_event(ready[c])
            if c == 0:
                self._ev("a2a_dispatch")
            r0, r1 = starts[lo], starts[hi]
            hm = None
            if r1 > r0:
                plan = self._chunk_plans[c].from_splits(sp[lo:hi])
                if save:
                    ops.grouped_gemm(self.peer.recv_buf[r0:r1], self.w.w1[lo:hi], plan=plan,
                                     out=y1[r0:r1])
                    hm = ops.swiglu(y1[r0:r1], out=h[r0:r1])
                else:
                    hm = ops.grouped_gemm(self.peer.recv_buf[r0:r1], self.w.w1[lo:hi],
                                          epilogue="swiglu", plan=plan)
            if c == last:
                self._ev("fc1")
            if hm is not None:
                ops.grouped_gemm(hm, self.w.w2[lo:hi], plan=plan, out=self.peer.y_buf[r0:r1])
        return (y1, h) if save else None

    def device_error(self) -> int:
        """First non-zero device error word of this layer's grouped-GEMM
        plans (0: none). Synchronises."""
        for p in [self.plan] + self._chunk_plans:
            v = p.device_error()
            if v:
                return v
        return 0

    __call__ = forward

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
