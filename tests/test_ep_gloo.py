"""Expert-parallel host logic on CPU with gloo ranks (world size 2 and 4).

The dispatcher (count exchange, split sizes, row all-to-alls) is the same
code the NCCL path runs; the expert math here is the CPU oracle, so these
tests check the data movement: the EP layer output must equal the
single-process oracle layer bit for bit. Failure cases (a rank that leaves,
rows that do not match their counts) must end in an error, not a hang.
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


def _problem(t_per_rank, world, h, e, f, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(world * t_per_rank, h, generator=g).to(torch.bfloat16)
    lg = torch.randn(world * t_per_rank, e, generator=g)
    bias = -1.5 * torch.log(torch.randperm(e, generator=g).float() + 1)
    w1 = (torch.randn(e, 2 * f, h, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(e, h, f, generator=g) * 0.05).to(torch.bfloat16)
    return x, lg, bias, w1, w2


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _worker(rank, world, port, mode, q):
    for p in (str(PKG), str(ROOT), str(GOLDEN)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=8))
        from moe_b200.ep import EPDispatcher, ep_group_table
        from oracle import moe_oracle as orc
        t, h, e, f, k = 24, 32, 8, 16, 3
        x, lg, bias, w1, w2 = _problem(t, world, h, e, f, k)
        sl = slice(rank * t, (rank + 1) * t)
        xl, lgl = x[sl], lg[sl]
        disp = EPDispatcher(e)
        e0, e1 = disp.local_range()
        # local routing + permute (oracle stands in for the kernels)
        _, _, rmap, probs = orc.router(lgl.numpy(), k, bias.numpy())
        et, te, counts, n = orc.row_id_map(rmap)
        xp, _ = orc.permute(_bits(xl), te, None, n)
        xp_t = torch.from_numpy(xp.view(np.int16)).view(torch.bfloat16)
        if mode == "leave" and rank == 1:
            dist.destroy_process_group()
            q.put((rank, "left"))
            return
        send, recv, recv_counts = disp.exchange_counts(torch.from_numpy(counts))
        if mode == "bad_rows" and rank == 1:
            xp_t = xp_t[:-1]  # rows no longer match the counts just exchanged
        xr = disp.dispatch(xp_t, send, recv)
        # local experts over (src, expert) segments, expert-major table
        starts, rows, widx = ep_group_table(recv_counts.tolist(), world, e1 - e0)
        xr_b = _bits(xr)
        hmid = orc.grouped_gemm(xr_b, _bits(w1[e0:e1])[widx], rows, "swiglu", row_starts=starts)
        y = orc.grouped_gemm(hmid, _bits(w2[e0:e1])[widx], rows, row_starts=starts)
        y_t = torch.from_numpy(y.view(np.int16)).view(torch.bfloat16)
        yb = disp.combine(y_t, send, recv)
        _, out = orc.unpermute(_bits(yb), et, probs, "dense")
        # reference: the whole layer in one process
        ref = orc.moe_layer(_bits(x), lg.numpy(), _bits(w1), _bits(w2), k, bias.numpy())
        q.put((rank, bool(np.array_equal(out, ref[sl])), send, recv))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        q.put((rank, "error", type(exc).__name__, str(exc)[:300], traceback.format_exc()[-800:]))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = []
    for _ in range(world):
        res.append(q.get(timeout=120))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            raise AssertionError("rank did not exit")
    return sorted(res, key=lambda r: r[0])


@pytest.mark.parametrize("world", [2, 4])
def test_ep_layer_matches_single_process(world):
    res = _run(world, "ok")
    for r in res:
        assert r[1] is True, r
    # every rank's received rows equal what the others sent it
    sends = {r[0]: r[2] for r in res}
    recvs = {r[0]: r[3] for r in res}
    for d in range(world):
        assert recvs[d] == [sends[s][d] for s in range(world)]


def test_ep_rank_leaving_gives_error_not_hang():
    res = _run(2, "leave")
    assert res[1][1] == "left"
    assert res[0][1] == "error", res[0]


def test_ep_rows_not_matching_counts_are_rejected():
    res = _run(2, "bad_rows")
    assert res[1][1] == "error" and res[1][2] == "ValueError", res[1]
    assert res[0][1] == "error", res[0]  # its peer times out instead of hanging
