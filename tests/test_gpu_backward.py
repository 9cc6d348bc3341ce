"""GPU parity of the layer backward: the combine and SwiGLU backward kernels
against the oracle (pinned to torch.autograd in tests/test_oracle_backward.py),
and MoELayer.backward against the oracle's chain with the same bf16
roundings."""
import numpy as np
import pytest
import torch

from conftest import u16
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def _rand_bf16(g, *shape, std=1.0):
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


@pytest.mark.parametrize("t,h,e,k", [(1, 8, 4, 1), (100, 200, 16, 4), (513, 7168, 64, 8),
                                     (64, 130, 8, 2), (5, 7, 4, 2)])
def test_combine_backward_vs_oracle(cuda_dev, t, h, e, k):
    import moe_b200
    g = torch.Generator().manual_seed(t + h + e)
    logits = torch.randn(t, e, generator=g)
    _, _, rmap, probs = orc.router(logits.numpy(), k)
    _, map_te, _, rows_n = orc.row_id_map(rmap)
    rows = _rand_bf16(g, rows_n, h)
    go = _rand_bf16(g, t, h)
    gr, gp = moe_b200.combine_backward(go.to(cuda_dev), rows.to(cuda_dev),
                                       torch.from_numpy(map_te).to(cuda_dev),
                                       torch.from_numpy(probs).to(cuda_dev))
    ref_r, ref_p = orc.combine_backward(u16(go), u16(rows), map_te, probs)
    assert np.array_equal(u16(gr), ref_r)  # bf16(p * g): one rounding, bit-exact
    np.testing.assert_allclose(gp.cpu().numpy(), ref_p, rtol=1e-5, atol=1e-5 * np.sqrt(h))


@pytest.mark.parametrize("m,f", [(1, 8), (300, 2048), (77, 136)])
def test_swiglu_backward_vs_oracle(cuda_dev, m, f):
    import moe_b200
    g = torch.Generator().manual_seed(m + f)
    y = _rand_bf16(g, m, 2 * f, std=2.0)
    dh = _rand_bf16(g, m, f)
    dy = moe_b200.swiglu_backward(y.to(cuda_dev), dh.to(cuda_dev))
    ref = orc.bf16_to_f32(orc.swiglu_backward(u16(y), u16(dh)))
    got = orc.bf16_to_f32(u16(dy))
    # expf differs from numpy's exp by a few fp32 ulp: at most one bf16 ulp here
    assert (np.abs(got - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-30).all()
    assert (got == ref).mean() > 0.99


def test_layer_backward_vs_oracle(cuda_dev):
    import moe_b200
    t, h, e, f, k = 256, 512, 16, 128, 4
    g = torch.Generator().manual_seed(9)
    x = _rand_bf16(g, t, h)
    lg = torch.randn(t, e, generator=g)
    w1 = _rand_bf16(g, e, 2 * f, h, std=0.05)
    w2 = _rand_bf16(g, e, h, f, std=0.05)
    go = _rand_bf16(g, t, h)
    layer = moe_b200.MoELayer(moe_b200.MoEWeights(w1.to(cuda_dev), w2.to(cuda_dev)), topk=k)
    out, ctx = layer.forward(x.to(cuda_dev), lg.to(cuda_dev), save_for_backward=True)
    # same output bits as the fused-SwiGLU forward
    assert torch.equal(out, layer(x.to(cuda_dev), lg.to(cuda_dev)))
    # another forward in between (different routing) must not disturb ctx
    layer(x.to(cuda_dev), torch.randn(t, e, generator=g).to(cuda_dev))
    gx, gp, dw1, dw2 = layer.backward(go.to(cuda_dev), ctx)
    torch.cuda.synchronize()
    assert layer.plan.device_error() == 0
    rx, rp, rw1, rw2 = orc.moe_layer_backward(u16(x), lg.numpy(), u16(w1), u16(w2), k, u16(go))

    def close(got, ref, tag):
        # the device and the oracle differ only in GEMM summation order, and
        # the bf16 roundings that follow can move an element by an ulp
        scale = np.abs(ref).max() + 1e-6
        err = np.abs(got - ref).max()
        assert err <= 2e-2 * scale, (tag, err, scale)

    close(orc.bf16_to_f32(u16(gx)), orc.bf16_to_f32(rx), "grad_x")
    close(gp.cpu().numpy(), rp, "grad_probs")
    close(orc.bf16_to_f32(u16(dw1)), orc.bf16_to_f32(rw1), "dw1")
    close(orc.bf16_to_f32(u16(dw2)), orc.bf16_to_f32(rw2), "dw2")
    with pytest.raises(ValueError):
        layer.backward(go.to(cuda_dev), dict(ctx, y1=None))
