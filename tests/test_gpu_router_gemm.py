"""GPU parity of the fused router (gate GEMM + softmax/top-k in one kernel).

Parity chain: the fused kernel's logits are the router gate GEMM (checked
against the case38 golden and against float64 sums within the GEMM rounding
bound), and its routing outputs must equal, bit for bit, the standalone
router kernel (moe_router_topk, itself pinned to the oracle and the case23
edge suite) run on those same logits. The oracle router then checks indices
exactly and gates within rtol 1e-5 on the same logits.
"""
import numpy as np
import pytest
import torch

from conftest import from_u16, u16
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(dev, t, h, e, seed, wscale=0.05):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(e, h, generator=g) * wscale).to(torch.bfloat16).to(dev)
    return x, w


def _check_against_router(moe_b200, x, w, k, score, renorm, bias):
    r, lg = moe_b200.router_gemm_topk(x, w, k, score, renorm, bias, outputs="all",
                                      return_logits=True)
    ref = moe_b200.router_topk(lg, k, score, renorm, bias, outputs="all")
    assert torch.equal(r.topk_idx, ref.topk_idx)
    for a, b in ((r.topk_vals, ref.topk_vals), (r.probs, ref.probs)):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    assert torch.equal(r.routing_map, ref.routing_map)
    # maps-only call: same maps, no logits written
    r2 = moe_b200.router_gemm_topk(x, w, k, score, renorm, bias, outputs="maps")
    assert torch.equal(r2.routing_map, ref.routing_map)
    assert torch.equal(r2.probs.view(torch.int32), ref.probs.view(torch.int32))
    return r, lg


def _logits_bound_check(x, w, lg, rows=None):
    xs = orc.bf16_to_f32(u16(x)).astype(np.float64)
    ws = orc.bf16_to_f32(u16(w)).astype(np.float64)
    got = lg.cpu().numpy().astype(np.float64)
    if rows is not None:
        xs, got = xs[rows], got[rows]
    exact = xs @ ws.T
    bound = 1e-5 * (np.abs(xs) @ np.abs(ws).T) + 1e-30
    err = np.abs(got - exact)
    assert (err <= bound).all(), (err.max(), (err / bound).max())


@pytest.mark.parametrize("t,h,e,k", [(1, 64, 32, 1), (100, 200, 64, 8), (128, 512, 256, 8),
                                     (300, 1024, 320, 8), (777, 256, 512, 16),
                                     (1000, 136, 96, 6), (257, 4096, 256, 16)])
@pytest.mark.parametrize("score,renorm", [("softmax", True), ("softmax", False),
                                          ("logits", True), ("logits", False)])
def test_fused_router_equals_router_on_its_logits(cuda_dev, t, h, e, k, score, renorm):
    import moe_b200
    x, w = _inputs(cuda_dev, t, h, e, seed=t + h + e + k)
    g = torch.Generator().manual_seed(e)
    bias = (torch.randn(e, generator=g) * 0.5).to(cuda_dev) if (t % 2) else None
    r, lg = _check_against_router(moe_b200, x, w, k, score, renorm, bias)
    _logits_bound_check(x, w, lg)
    # oracle router on the same logits: indices exact, gates rtol 1e-5
    vals, idx, rmap, probs = orc.router(lg.cpu().numpy(), k,
                                        None if bias is None else bias.cpu().numpy(),
                                        score, renorm)
    assert np.array_equal(r.topk_idx.cpu().numpy(), idx)
    assert np.array_equal(r.routing_map.cpu().numpy(), rmap)
    np.testing.assert_allclose(r.topk_vals.cpu().numpy(), vals, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(r.probs.cpu().numpy(), probs, rtol=1e-5, atol=1e-7)
    assert moe_b200.router_device_error(cuda_dev) == 0


@pytest.mark.parametrize("e,k,renorm", [(96, 8, True), (320, 8, False), (256, 16, True)])
def test_fused_router_several_tiles_per_pair(cuda_dev, e, k, renorm):
    """More 256-token tiles than CTA pairs (40000 tokens: 157 tiles), so each
    pair walks several tiles: accumulator reuse (one accumulator at E=320, two
    at E<=256) and the per-quadrant list hand-over across tiles."""
    import moe_b200
    t, h = 40000, 512
    x, w = _inputs(cuda_dev, t, h, e, seed=e + k)
    g = torch.Generator().manual_seed(3)
    bias = (torch.randn(e, generator=g) * 0.5).to(cuda_dev)
    _, lg = _check_against_router(moe_b200, x, w, k, "softmax", renorm, bias)
    rows = np.unique(np.concatenate([[0, 255, 256, t // 2, t - 1],
                                     np.random.default_rng(4).integers(0, t, 59)]))
    _logits_bound_check(x, w, lg, rows)
    assert moe_b200.router_device_error(cuda_dev) == 0


def test_fused_router_case38_golden(cuda_dev, golden):
    """Logits-only call vs the reference's reference_fp32 golden (case38)."""
    import moe_b200
    z = golden("gemm_swiglu.npz")
    x, w = from_u16(z["c38_x"], cuda_dev), from_u16(z["c38_w"], cuda_dev)
    _, lg = moe_b200.router_gemm_topk(x, w, 8, outputs="none", return_logits=True)
    np.testing.assert_allclose(lg.cpu().numpy(), z["c38_y"], rtol=1e-5, atol=1e-4)
    # same logits as the grouped-GEMM router path within the GEMM rounding bound
    _logits_bound_check(x, w, moe_b200.router_logits(x, w))
    _logits_bound_check(x, w, lg)


def test_fused_router_ties_and_specials(cuda_dev):
    """Duplicate weight rows give bit-equal logits (ties -> lower expert);
    a -inf / +inf / NaN bias entry ranks as the standalone router ranks it."""
    import moe_b200
    t, h, e, k = 256, 128, 64, 8
    x, w = _inputs(cuda_dev, t, h, e, seed=11)
    w[5] = w[3]
    w[40] = w[3]
    w[17] = w[60]
    for bias in (None,
                 torch.zeros(e, device=cuda_dev),
                 torch.tensor([float("-inf")] * 4 + [0.0] * (e - 4), device=cuda_dev),
                 torch.tensor([0.0] * (e - 1) + [float("inf")], device=cuda_dev),
                 torch.tensor([0.0] * 7 + [float("nan")] + [0.0] * (e - 8), device=cuda_dev)):
        for score in ("softmax", "logits"):
            _check_against_router(moe_b200, x, w, k, score, True, bias)
    r, _ = moe_b200.router_gemm_topk(x, w, k, outputs="all", return_logits=True)
    idx = r.topk_idx.cpu().numpy()
    for row in idx:  # where both tied experts are chosen, the lower id comes first
        p3, p5 = np.where(row == 3)[0], np.where(row == 5)[0]
        if p3.size and p5.size:
            assert p3[0] < p5[0]


def test_fused_router_reference_shape(cuda_dev):
    """case38's traced shape (16384 x 8192 x 320, N(0,1) inputs) with the
    layer's routing (softmax, top-8, renormalised): routing equals the
    standalone router on the fused logits; sampled logit rows within the
    GEMM rounding bound of float64 sums."""
    import moe_b200
    m, kk, n = 16384, 8192, 320
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    x = torch.randn(m, kk, device=cuda_dev, generator=g).to(torch.bfloat16)
    w = torch.randn(n, kk, device=cuda_dev, generator=g).to(torch.bfloat16)
    r, lg = _check_against_router(moe_b200, x, w, 8, "softmax", True, None)
    rows = np.unique(np.concatenate([[0, m // 2, m - 1],
                                     np.random.default_rng(2).integers(0, m, 29)]))
    _logits_bound_check(x, w, lg, rows)
    assert moe_b200.router_device_error(cuda_dev) == 0


def test_fused_router_empty_and_errors(cuda_dev):
    import moe_b200
    x, w = _inputs(cuda_dev, 0, 64, 32, seed=1)
    r = moe_b200.router_gemm_topk(x, w, 4, outputs="all")
    assert r.topk_idx.shape == (0, 4) and r.probs.shape == (0, 32)
    x, w = _inputs(cuda_dev, 16, 64, 48, seed=1)  # E not a multiple of 32
    assert not moe_b200.ops.router_gemm_fusable(x, w, 4)
    with pytest.raises(moe_b200.MoeError):
        moe_b200.router_gemm_topk(x, w, 4)
    x, w = _inputs(cuda_dev, 16, 64, 64, seed=1)
    with pytest.raises(moe_b200.MoeError):
        moe_b200.router_gemm_topk(x, w, 17)
    with pytest.raises(ValueError):
        moe_b200.router_gemm_topk(x, w, 4, outputs="none")
