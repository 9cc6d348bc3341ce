"""Expert-parallel layer on 2 (or 4) GPUs over NCCL, against the single-GPU layer.

Each output element is accumulated in the same K order by the same kernel on
either path, and the combine adds experts in ascending order on both, so the
EP result must equal the single-GPU result bit for bit. Needs >= 2 GPUs (4
and 8 for the wider cases); skipped on hosts with fewer.
"""
import os
import socket
import sys
import traceback
from datetime import timedelta

import pytest
import torch

from conftest import GOLDEN, PKG, ROOT

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(world, t, h, e, f, routing):
    g = torch.Generator().manual_seed(11 + world)
    x = torch.randn(world * t, h, generator=g).to(torch.bfloat16)
    lg = torch.randn(world * t, e, generator=g)
    bias = torch.zeros(e)
    if routing == "zipf":
        bias = -1.5 * torch.log(torch.randperm(e, generator=g).float() + 1)
    w1 = (torch.randn(e, 2 * f, h, generator=g) * 0.03).to(torch.bfloat16)
    w2 = (torch.randn(e, h, f, generator=g) * 0.03).to(torch.bfloat16)
    return x, lg, bias, w1, w2


def _worker(rank, world, port, routing, transport, q, placed=False, chunks=1):
    for p in (str(PKG), str(ROOT), str(GOLDEN)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        import moe_b200
        from moe_b200.ep import MoELayerEP
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        t, h, e, f, k = 256, 1024, 16, 256, 4
        x, lg, bias, w1, w2 = _problem(world, t, h, e, f, routing)
        el = e // world
        sl = slice(rank * t, (rank + 1) * t)
        pl = torch.arange(e, dtype=torch.int32)
        if placed:
            from moe_b200.ep import balanced_placement
            load = torch.bincount(torch.topk(lg + bias, k, dim=1).indices.reshape(-1), minlength=e)
            pl = torch.tensor(balanced_placement(load.tolist(), world), dtype=torch.int32)
        w1, w2 = w1[pl.long()], w2[pl.long()]  # slot order
        local = moe_b200.MoEWeights(w1[rank * el:(rank + 1) * el].to(dev).contiguous(),
                                    w2[rank * el:(rank + 1) * el].to(dev).contiguous())
        layer = MoELayerEP(local, e, topk=k, expert_bias=bias.to(dev), transport=transport,
                           tokens=t, placement=pl.to(dev) if placed else None,
                           overlap_chunks=chunks)
        out = layer(x[sl].to(dev), lg[sl].to(dev))
        out2 = layer(x[sl].to(dev), lg[sl].to(dev))  # buffers reused across forwards
        assert torch.equal(out, out2)
        outs = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(outs, out)
        err = layer.device_error()
        ok = None
        if rank == 0:
            full = moe_b200.MoELayer(moe_b200.MoEWeights(w1.to(dev), w2.to(dev)), topk=k,
                                     expert_bias=bias.to(dev),
                                     placement=pl.to(dev) if placed else None)
            ref = full(x.to(dev), lg.to(dev))
            ok = bool(torch.equal(torch.cat(outs), ref))
        layer.close()
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        q.put((rank, ok, err))
    except Exception as exc:
        q.put((rank, "error", f"{type(exc).__name__}: {exc}", traceback.format_exc()[-1500:]))


@pytest.mark.parametrize("world,routing,transport", [(2, "uniform", "nccl"), (2, "zipf", "nccl"),
                                                     (2, "zipf", "peer"), (2, "uniform", "peer"),
                                                     (2, "zipf", "fused"), (2, "uniform", "fused"),
                                                     (4, "zipf", "peer"), (4, "uniform", "nccl"),
                                                     (4, "zipf", "fused"), (4, "uniform", "fused"),
                                                     (2, "zipf", "fused+placed"),
                                                     (4, "zipf", "fused+placed"),
                                                     (8, "zipf", "fused+placed"),
                                                     (8, "uniform", "nccl"),
                                                     (2, "zipf", "fused_dedup"),
                                                     (4, "uniform", "fused_dedup"),
                                                     (4, "zipf", "fused_dedup+placed"),
                                                     (8, "zipf", "fused_dedup+placed"),
                                                     (2, "zipf", "fused+overlap2"),
                                                     (2, "uniform", "fused+placed+overlap3"),
                                                     (4, "zipf", "fused+placed+overlap2"),
                                                     (8, "zipf", "fused+placed+overlap2")])
def test_ep_equals_single_gpu(world, routing, transport):
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    parts = transport.split("+")
    placed = "placed" in parts
    chunks = int(next((p[len("overlap"):] for p in parts if p.startswith("overlap")), 1))
    tr = parts[0]
    procs = [ctx.Process(target=_worker, args=(r, world, port, routing, tr, q, placed, chunks))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    for r in res:
        assert r[1] != "error", r
        assert r[2] == 0, r
    assert res[0][1] is True


def _bwd_worker(rank, world, port, transport, q, chunks=1):
    for p in (str(PKG), str(ROOT), str(GOLDEN)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        import moe_b200
        from moe_b200.ep import MoELayerEP, balanced_placement
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        t, h, e, f, k = 256, 1024, 16, 256, 4
        x, lg, bias, w1, w2 = _problem(world, t, h, e, f, "zipf")
        g = torch.Generator().manual_seed(99)
        go = torch.randn(world * t, h, generator=g).to(torch.bfloat16)
        el = e // world
        sl = slice(rank * t, (rank + 1) * t)
        load = torch.bincount(torch.topk(lg + bias, k, dim=1).indices.reshape(-1), minlength=e)
        pl = torch.tensor(balanced_placement(load.tolist(), world), dtype=torch.int32)
        w1, w2 = w1[pl.long()], w2[pl.long()]  # slot order
        local = moe_b200.MoEWeights(w1[rank * el:(rank + 1) * el].to(dev).contiguous(),
                                    w2[rank * el:(rank + 1) * el].to(dev).contiguous())
        layer = MoELayerEP(local, e, topk=k, expert_bias=bias.to(dev), transport=transport,
                           tokens=t, placement=pl.to(dev), overlap_chunks=chunks)
        out, ctx = layer.forward(x[sl].to(dev), lg[sl].to(dev), save_for_backward=True)
        gx, gp, dw1, dw2 = layer.backward(go[sl].to(dev), ctx)
        err = layer.device_error() + moe_b200.grouped_wgrad_device_error(dev)
        full = moe_b200.MoELayer(moe_b200.MoEWeights(w1.to(dev), w2.to(dev)), topk=k,
                                 expert_bias=bias.to(dev), placement=pl.to(dev))
        ref_out, rctx = full.forward(x.to(dev), lg.to(dev), save_for_backward=True)
        rgx, rgp, rdw1, rdw2 = full.backward(go.to(dev), rctx)
        es = slice(rank * el, (rank + 1) * el)
        same = {"out": torch.equal(out, ref_out[sl]), "grad_x": torch.equal(gx, rgx[sl]),
                "grad_probs": torch.equal(gp, rgp[sl]),
                "dw1": torch.equal(dw1.view(torch.int16), rdw1[es].view(torch.int16)),
                "dw2": torch.equal(dw2.view(torch.int16), rdw2[es].view(torch.int16))}
        layer.close()
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        q.put((rank, same, err))
    except Exception as exc:
        q.put((rank, "error", f"{type(exc).__name__}: {exc}", traceback.format_exc()[-1500:]))


@pytest.mark.parametrize("world,transport", [(2, "fused"), (2, "fused_dedup"), (4, "fused"),
                                             (8, "fused"), (2, "fused+overlap3"),
                                             (8, "fused+overlap2")])
def test_ep_backward_equals_single_gpu(world, transport):
    """MoELayerEP.backward (combine backward over NVLink, grouped dgrad/wgrad
    on the receive rows, permute backward as the unweighted fused combine)
    against MoELayer.backward on all ranks' tokens with all experts (same
    placement): output, grad_x, grad_probs and every local expert's dW1/dW2
    bit for bit."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    tr, _, ov = transport.partition("+overlap")
    procs = [ctx.Process(target=_bwd_worker, args=(r, world, port, tr, q, int(ov or 1)))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    for r in res:
        assert r[1] != "error", r
        assert r[2] == 0, r
        assert all(r[1].values()), r
