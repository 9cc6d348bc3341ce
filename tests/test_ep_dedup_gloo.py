"""The deduplicated expert-parallel dispatch (transport "fused_dedup") as a
host restatement on gloo CPU ranks, world size 2, 4 and 8.

On the GPU, ep_dispatch_dedup_kernel stores each token row once per
destination rank: rows for this rank's own experts go straight into its
receive buffer at (permuted row + deltas[e]); for every other rank d the row
goes once into d's staging rows for this source, at a slot taken from d's
per-source counter, together with a table row holding, for each of d's local
experts, the receive row it belongs to (-1 if the token is not routed
there). After a barrier, ep_expand_kernel on d copies every staged row to the
receive rows its table lists. The receive buffer must come out exactly as the
plain fused dispatch lays it out (expert_major_layout: a token row of expert e
at its permuted row + deltas[e] in the owner's buffer).

Here the same three steps run on the host with the staging rows, tables and
counters moved between ranks by gloo all-to-alls. Slots are handed out in a
shuffled token order, since the kernel's atomics give no order. The check is
against the receive buffers that every source's plain fused stores would
produce, bit for bit, with every receive row written exactly once.
"""
import os
import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import GOLDEN, PKG, ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _routing(world, t, e, k, h, seed):
    """Every rank's tokens (bf16 bits) and [T,E] row maps, from one seed."""
    from oracle import moe_oracle as orc
    rng = np.random.default_rng(seed)
    bias = (-1.5 * np.log(rng.permutation(e) + 1.0)).astype(np.float32)
    xs, tes, counts = [], [], []
    for _ in range(world):
        xs.append(orc.f32_to_bf16(rng.standard_normal((t, h), dtype=np.float32)))
        _, _, rmap, _ = orc.router(rng.standard_normal((t, e), dtype=np.float32), k, bias)
        _, te, c, _ = orc.row_id_map(rmap)
        tes.append(te)
        counts.append(c)
    return xs, tes, np.stack(counts)


def _dedup_stage(x, te, deltas, world, rank, el, t, order):
    """Source side of the dedup dispatch (ep_dispatch_dedup_kernel): returns
    the rows for this rank's own receive buffer [(row, token)], and per
    destination d the staged token rows and their table rows, in slot order."""
    own, stage, meta = [], [[] for _ in range(world)], [[] for _ in range(world)]
    counter = [0] * world  # d's counter for this source
    for tok in order:
        dest = np.where(te[tok] >= 0, te[tok] + deltas, -1)
        for d in range(world):
            rows = dest[d * el:(d + 1) * el]
            if not (rows >= 0).any():
                continue
            if d == rank:
                own += [(int(r), tok) for r in rows if r >= 0]
                continue
            slot = counter[d]
            counter[d] += 1
            assert slot < t  # the kernel skips a slot beyond T (a valid map never gets there)
            stage[d].append(x[tok])
            meta[d].append(rows.astype(np.int32))
    return own, stage, meta


def _worker(rank, world, port, q):
    for p in (str(PKG), str(ROOT), str(GOLDEN)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=20))
        from moe_b200.ep import expert_major_layout
        t, h, e, k = 40, 16, 32, 4
        el = e // world
        xs, tes, counts = _routing(world, t, e, k, h, seed=world)
        # counts are all-gathered on the GPU path; here every rank derives them
        # from the shared seed and checks the gathered copy matches.
        got = [torch.empty(e, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(got, torch.from_numpy(counts[rank].astype(np.int64)))
        assert np.array_equal(torch.stack(got).numpy(), counts)
        lay = expert_major_layout(counts.tolist(), rank, el)
        deltas = np.asarray(lay.deltas, dtype=np.int64)
        cap = world * t * k
        order = np.random.default_rng(100 + rank).permutation(t)
        own, stage, meta = _dedup_stage(xs[rank], tes[rank], deltas, world, rank, el, t, order)

        # exchange: per-destination slot counts, then staged rows and tables
        nsend = torch.tensor([len(stage[d]) for d in range(world)], dtype=torch.int64)
        nrecv = torch.empty_like(nsend)
        dist.all_to_all_single(nrecv, nsend)
        # rows travel as raw bytes, as the NCCL path's row exchange does
        rows_out = torch.from_numpy(np.ascontiguousarray(np.concatenate(
            [np.asarray(stage[d], np.uint16).reshape(-1, h) for d in range(world)])).view(np.uint8))
        meta_out = torch.from_numpy(np.concatenate(
            [np.asarray(meta[d], np.int32).reshape(-1, el) for d in range(world)]))
        rows_in = torch.empty((int(nrecv.sum()), 2 * h), dtype=torch.uint8)
        meta_in = torch.empty((int(nrecv.sum()), el), dtype=torch.int32)
        dist.all_to_all_single(rows_in, rows_out, nrecv.tolist(), nsend.tolist())
        dist.all_to_all_single(meta_in, meta_out, nrecv.tolist(), nsend.tolist())

        # receiver: own rows, then the expansion (ep_expand_kernel)
        recv = np.zeros((cap, h), np.uint16)
        writes = np.zeros(cap, np.int64)
        for r, tok in own:
            recv[r] = xs[rank][tok]
            writes[r] += 1
        rin = rows_in.numpy().view(np.uint16)  # [rows, h]
        for i, mrow in enumerate(meta_in.numpy()):
            for rr in mrow:
                if 0 <= rr < cap:
                    recv[rr] = rin[i]
                    writes[rr] += 1

        # expected: every source's plain fused stores (row of (t, e) at its
        # permuted row + that source's deltas[e], in the owner's buffer)
        want = np.zeros((cap, h), np.uint16)
        for s in range(world):
            ds = np.asarray(expert_major_layout(counts.tolist(), s, el).deltas, np.int64)
            ti, ei = np.nonzero(tes[s] >= 0)
            mine = ei // el == rank
            want[tes[s][ti[mine], ei[mine]] + ds[ei[mine]]] = xs[s][ti[mine]]
        n = sum(lay.splits)
        ok = (np.array_equal(recv, want) and np.all(writes[:n] == 1) and np.all(writes[n:] == 0)
              and n == lay.recv_rows[rank])
        # one NVLink crossing per (token, destination rank) instead of per (token, expert)
        crossings = int(nsend.sum())
        plain = int(sum(((tes[rank][:, d * el:(d + 1) * el] >= 0).sum())
                        for d in range(world) if d != rank))
        q.put((rank, bool(ok), crossings, plain))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        q.put((rank, "error", type(exc).__name__, str(exc)[:300], traceback.format_exc()[-800:]))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_dedup_dispatch_fills_the_expert_major_receive_rows(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=180) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            raise AssertionError("rank did not exit")
    for r in res:
        assert r[1] is True, r
        assert r[2] <= r[3], r  # dedup never sends more rows than the plain dispatch
