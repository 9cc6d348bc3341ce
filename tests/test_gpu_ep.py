"""Expert-parallel layer on 2, 4 and 8 GPUs, against the single-GPU layer.

Each output element is accumulated in the same K order by the same kernel on
either path, and the combine adds experts in ascending order on both, so the
EP result must equal the single-GPU result bit for bit, forward and backward.
One group of processes per world size (one per GPU, NCCL) runs every variant
of that size in turn -- transport, routing, expert placement, overlap chunks
-- so the process start and NCCL set-up are paid once per world size. Needs
>= 2 GPUs (4 and 8 for the wider cases); skipped on hosts with fewer.
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

# (routing, transport[+placed][+overlapN]) per world size
FORWARD = {
    2: [("uniform", "nccl"), ("zipf", "nccl"), ("zipf", "peer"), ("uniform", "peer"),
        ("zipf", "fused"), ("uniform", "fused"), ("zipf", "fused+placed"),
        ("zipf", "fused_dedup"), ("zipf", "fused+overlap2"),
        ("uniform", "fused+placed+overlap3"), ("zipf", "fused_pull+placed"),
        ("uniform", "fused_pull")],
    4: [("zipf", "peer"), ("uniform", "nccl"), ("zipf", "fused"), ("uniform", "fused"),
        ("zipf", "fused+placed"), ("uniform", "fused_dedup"), ("zipf", "fused_dedup+placed"),
        ("zipf", "fused+placed+overlap2"), ("zipf", "fused_pull+placed")],
    8: [("zipf", "fused+placed"), ("uniform", "nccl"), ("zipf", "fused_dedup+placed"),
        ("zipf", "fused+placed+overlap2"), ("zipf", "fused_pull+placed")],
}
BACKWARD = {2: ["fused", "fused_dedup", "fused+overlap3", "fused_pull"], 4: ["fused", "fused_pull"],
            8: ["fused", "fused+overlap2", "fused_pull"]}


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


def _parse(variant):
    parts = variant.split("+")
    chunks = int(next((p[len("overlap"):] for p in parts if p.startswith("overlap")), 1))
    return parts[0], "placed" in parts, chunks


def _forward_case(world, rank, dev, routing, variant):
    """EP forward (twice: buffers are reused) vs the single-GPU layer on all
    ranks' tokens; returns (equal on rank 0 or None, device error)."""
    import torch.distributed as dist
    import moe_b200
    from moe_b200.ep import MoELayerEP, balanced_placement
    transport, placed, chunks = _parse(variant)
    t, h, e, f, k = 256, 1024, 16, 256, 4
    x, lg, bias, w1, w2 = _problem(world, t, h, e, f, routing)
    el = e // world
    sl = slice(rank * t, (rank + 1) * t)
    pl = torch.arange(e, dtype=torch.int32)
    if placed:
        load = torch.bincount(torch.topk(lg + bias, k, dim=1).indices.reshape(-1), minlength=e)
        pl = torch.tensor(balanced_placement(load.tolist(), world), dtype=torch.int32)
    w1, w2 = w1[pl.long()], w2[pl.long()]  # slot order
    local = moe_b200.MoEWeights(w1[rank * el:(rank + 1) * el].to(dev).contiguous(),
                                w2[rank * el:(rank + 1) * el].to(dev).contiguous())
    layer = MoELayerEP(local, e, topk=k, expert_bias=bias.to(dev), transport=transport,
                       tokens=t, placement=pl.to(dev) if placed else None,
                       overlap_chunks=chunks)
    out = layer(x[sl].to(dev), lg[sl].to(dev))
    out2 = layer(x[sl].to(dev), lg[sl].to(dev))
    outs = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(outs, out)
    err = layer.device_error()
    ok = None
    if rank == 0:
        full = moe_b200.MoELayer(moe_b200.MoEWeights(w1.to(dev), w2.to(dev)), topk=k,
                                 expert_bias=bias.to(dev),
                                 placement=pl.to(dev) if placed else None)
        ok = bool(torch.equal(torch.cat(outs), full(x.to(dev), lg.to(dev))))
    ok2 = bool(torch.equal(out, out2))
    layer.close()
    return (None if ok is None else ok and ok2), (0 if ok2 else -1) + err


def _backward_case(world, rank, dev, variant):
    """EP forward with save_for_backward + backward vs the single-GPU
    backward on all ranks' tokens (same placement): output, grad_x,
    grad_probs and the local experts' dW1/dW2 bit for bit."""
    import moe_b200
    from moe_b200.ep import MoELayerEP, balanced_placement
    transport, _, chunks = _parse(variant)
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
    return all(same.values()), err, same


def _worker(rank, world, port, q):
    for p in (str(PKG), str(ROOT), str(GOLDEN)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    res = {}
    try:
        import torch.distributed as dist
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        for routing, variant in FORWARD[world]:
            res[("fwd", routing, variant)] = _forward_case(world, rank, dev, routing, variant)
            dist.barrier(device_ids=[rank])
        for variant in BACKWARD[world]:
            res[("bwd", "zipf", variant)] = _backward_case(world, rank, dev, variant)
            dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as exc:
        q.put((rank, {"error": f"{type(exc).__name__}: {exc}",
                      "trace": traceback.format_exc()[-1500:], "done": list(res)}))


_RESULTS = {}


def _results(world):
    """Every variant of one world size, run once per session."""
    if world not in _RESULTS:
        import torch.multiprocessing as mp
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
        for p in procs:
            p.start()
        res = sorted((q.get(timeout=900) for _ in range(world)), key=lambda r: r[0])
        for p in procs:
            p.join(timeout=120)
        _RESULTS[world] = res
    return _RESULTS[world]


def _need(world):
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_forward_equals_single_gpu(world):
    """Every forward variant of this world size: NCCL all-to-all, copy-engine
    peer copies, fused dispatch/combine kernels on peer memory (push, pull
    and deduplicated dispatch), balanced placement and the chunked comm/GEMM
    overlap, each equal to the single-GPU layer bit for bit."""
    _need(world)
    for rank, res in _results(world):
        assert "error" not in res, (rank, res)
        for key, (ok, err) in ((k, v) for k, v in res.items() if k[0] == "fwd"):
            assert err == 0, (rank, key, err)
            if rank == 0:
                assert ok is True, key


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_backward_equals_single_gpu(world):
    """MoELayerEP.backward (combine backward over NVLink, grouped dgrad/wgrad
    on the receive rows, permute backward as the unweighted fused combine)
    against MoELayer.backward on all ranks' tokens with all experts (same
    placement): output, grad_x, grad_probs and every local expert's dW1/dW2
    bit for bit, for the fused, deduplicated and overlapped forwards."""
    _need(world)
    for rank, res in _results(world):
        assert "error" not in res, (rank, res)
        for key, (ok, err, same) in ((k, v) for k, v in res.items() if k[0] == "bwd"):
            assert err == 0, (rank, key, err)
            assert ok, (rank, key, same)
