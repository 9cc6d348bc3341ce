"""End-to-end parity of the single-GPU MoE expert layer against the CPU oracle.

Routing, maps and permuted rows are exact; the layer output (two bf16 GEMMs
and a weighted combine) is within rtol 2e-2 / atol 1e-2.
"""
import numpy as np
import pytest
import torch

from conftest import u16
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t,h,e,f,k,zipf", [(256, 256, 16, 128, 4, False),
                                            (512, 1024, 64, 256, 8, True),
                                            (1024, 7168, 32, 2048, 8, True)])
def test_layer_vs_oracle(cuda_dev, t, h, e, f, k, zipf):
    import moe_b200
    g = torch.Generator().manual_seed(t + h + e)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    lg = torch.randn(t, e, generator=g)
    bias = None
    if zipf:
        bias = -1.5 * torch.log(torch.randperm(e, generator=g).float() + 1)
    w1 = (torch.randn(e, 2 * f, h, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(e, h, f, generator=g) * 0.02).to(torch.bfloat16)
    layer = moe_b200.MoELayer(moe_b200.MoEWeights(w1.to(cuda_dev), w2.to(cuda_dev)), topk=k,
                              expert_bias=None if bias is None else bias.to(cuda_dev))
    out, mid = layer.forward(x.to(cuda_dev), lg.to(cuda_dev), return_intermediates=True)
    assert layer.plan.device_error() == 0
    # exact stages
    _, _, rmap, probs = orc.router(lg.numpy(), k, None if bias is None else bias.numpy())
    et, te, counts, n = orc.row_id_map(rmap)
    np.testing.assert_array_equal(mid["rim"].map_te.cpu().numpy(), te)
    xp, _ = orc.permute(u16(x), te, None, n)
    np.testing.assert_array_equal(u16(mid["xp"]), xp)
    # end-to-end tolerance
    tokens = np.arange(t) if t * h <= 1 << 20 else np.unique(
        np.random.default_rng(0).integers(0, t, 96))
    ref = orc.moe_layer(u16(x), lg.numpy(), u16(w1), u16(w2), k,
                        None if bias is None else bias.numpy(), tokens=tokens)
    got = orc.bf16_to_f32(u16(out)[tokens])
    np.testing.assert_allclose(got, orc.bf16_to_f32(ref), rtol=2e-2, atol=1e-2)


def test_host_pipeline_matches_direct_calls(cuda_dev):
    """Overlapped host->device->host steps give the same outputs as direct calls."""
    import moe_b200
    t, h, e, f, k = 384, 512, 16, 256, 4
    g = torch.Generator().manual_seed(9)
    w1 = (torch.randn(e, 2 * f, h, generator=g) * 0.03).to(torch.bfloat16).to(cuda_dev)
    w2 = (torch.randn(e, h, f, generator=g) * 0.03).to(torch.bfloat16).to(cuda_dev)
    layer = moe_b200.MoELayer(moe_b200.MoEWeights(w1, w2), topk=k)
    xs = [torch.randn(t, h, generator=g).to(torch.bfloat16).pin_memory() for _ in range(5)]
    lgs = [torch.randn(t, e, generator=g).pin_memory() for _ in range(5)]
    outs = [torch.empty(t, h, dtype=torch.bfloat16).pin_memory() for _ in range(5)]
    pipe = moe_b200.HostPipeline(layer, t, h, e, cuda_dev, depth=2)
    for i in range(5):
        pipe.submit(xs[i], lgs[i], outs[i])
    pipe.synchronize()
    for i in range(5):
        ref = layer(xs[i].to(cuda_dev), lgs[i].to(cuda_dev)).cpu()
        assert torch.equal(outs[i], ref), i
    outs2 = [torch.empty(t, h, dtype=torch.bfloat16).pin_memory() for _ in range(5)]
    pipe.run([(xs[i], lgs[i], outs2[i]) for i in range(5)])
    pipe.synchronize()
    for i in range(5):
        assert torch.equal(outs2[i], outs[i]), i


def test_layer_with_placement(cuda_dev):
    """Placed layer (weights in slot order) vs the oracle with the same placement."""
    import moe_b200
    t, h, e, f, k = 512, 512, 32, 256, 8
    g = torch.Generator().manual_seed(21)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    lg = torch.randn(t, e, generator=g)
    bias = -1.5 * torch.log(torch.randperm(e, generator=g).float() + 1)
    w1 = (torch.randn(e, 2 * f, h, generator=g) * 0.03).to(torch.bfloat16)
    w2 = (torch.randn(e, h, f, generator=g) * 0.03).to(torch.bfloat16)
    pl = torch.randperm(e, generator=g).to(torch.int32)
    layer = moe_b200.MoELayer(moe_b200.MoEWeights(w1[pl.long()].to(cuda_dev),
                                                  w2[pl.long()].to(cuda_dev)),
                              topk=k, expert_bias=bias.to(cuda_dev), placement=pl.to(cuda_dev))
    out, mid = layer.forward(x.to(cuda_dev), lg.to(cuda_dev), return_intermediates=True)
    _, _, rmap, _ = orc.router(lg.numpy(), k, bias.numpy(), placement=pl.numpy())
    _, te, _, _ = orc.row_id_map(rmap)
    np.testing.assert_array_equal(mid["rim"].map_te.cpu().numpy(), te)
    ref = orc.moe_layer(u16(x), lg.numpy(), u16(w1[pl.long()]), u16(w2[pl.long()]), k,
                        bias.numpy(), placement=pl.numpy())
    np.testing.assert_allclose(orc.bf16_to_f32(u16(out)), orc.bf16_to_f32(ref), rtol=2e-2,
                               atol=1e-2)


def test_layer_from_hidden_with_router_gemm(cuda_dev):
    """router_weight path: the fused router (gate GEMM + top-k in one kernel)
    then the same layer; equals feeding its logits in, bit for bit, and the
    logits match the fp32 oracle and the grouped-GEMM router logits."""
    import moe_b200
    t, h, e, f, k = 512, 1024, 64, 256, 8
    g = torch.Generator().manual_seed(5)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16).to(cuda_dev)
    rw = (torch.randn(e, h, generator=g) * 0.05).to(torch.bfloat16).to(cuda_dev)
    w1 = (torch.randn(e, 2 * f, h, generator=g) * 0.02).to(torch.bfloat16).to(cuda_dev)
    w2 = (torch.randn(e, h, f, generator=g) * 0.02).to(torch.bfloat16).to(cuda_dev)
    layer = moe_b200.MoELayer(moe_b200.MoEWeights(w1, w2), topk=k)
    out = layer(x, router_weight=rw)
    _, lg = moe_b200.router_gemm_topk(x, rw, k, outputs="none", return_logits=True)
    for logits in (lg, moe_b200.router_logits(x, rw)):
        np.testing.assert_allclose(logits.cpu().numpy(), orc.router_logits(u16(x), u16(rw)),
                                   rtol=1e-5, atol=1e-4)
    assert torch.equal(out, layer(x, lg))
    with pytest.raises(ValueError):
        layer(x)


def test_functional_layer_equals_module(cuda_dev):
    """moe_layer_fwd (functional form) == MoELayer, bit for bit."""
    import moe_b200
    t, h, e, f, k = 256, 512, 16, 128, 4
    g = torch.Generator().manual_seed(8)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16).to(cuda_dev)
    lg = torch.randn(t, e, generator=g).to(cuda_dev)
    w1 = (torch.randn(e, 2 * f, h, generator=g) * 0.02).to(torch.bfloat16).to(cuda_dev)
    w2 = (torch.randn(e, h, f, generator=g) * 0.02).to(torch.bfloat16).to(cuda_dev)
    a = moe_b200.moe_layer_fwd(x, lg, w1, w2, topk=k)
    b = moe_b200.MoELayer(moe_b200.MoEWeights(w1, w2), topk=k)(x, lg)
    assert torch.equal(a, b)
