"""CPU: the oracle's backward of the weighted combine, of SwiGLU and of the
whole layer, pinned to torch.autograd (no reference code exists for these
three; the reference covers the permute backward and the grouped dgrad and
wgrad, which tests/test_oracle_golden.py pins to its Model outputs)."""
import numpy as np
import torch

from oracle import moe_oracle as orc


def _bf16(g, *shape, std=1.0):
    t = (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)
    return t, t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _ulp_close(got_u16, ref_f32, frac=0.999):
    got = orc.bf16_to_f32(got_u16)
    ok = np.abs(got - ref_f32) <= np.abs(ref_f32) * 2.0 ** -7 + 1e-6
    assert ok.mean() >= frac, ok.mean()


def test_combine_backward_matches_autograd():
    g = torch.Generator().manual_seed(1)
    t, h, e, k = 24, 64, 10, 3
    logits = torch.randn(t, e, generator=g)
    _, _, rmap, probs = orc.router(logits.numpy(), k)
    _, map_te, _, rows_n = orc.row_id_map(rmap)
    rows_t, rows_u = _bf16(g, rows_n, h)
    go_t, go_u = _bf16(g, t, h)
    grad_rows, grad_probs = orc.combine_backward(go_u, rows_u, map_te, probs)
    # autograd of out[t] = sum_e probs[t,e] * rows[map[t,e]]
    r = rows_t.float().requires_grad_()
    p = torch.from_numpy(probs).requires_grad_()
    mt = torch.from_numpy(map_te)
    out = torch.zeros(t, h)
    for ti in range(t):
        for ei in range(e):
            if mt[ti, ei] >= 0:
                out[ti] = out[ti] + p[ti, ei] * r[mt[ti, ei]]
    out.backward(go_t.float())
    _ulp_close(grad_rows, r.grad.numpy())
    np.testing.assert_allclose(grad_probs, p.grad.numpy(), rtol=1e-5, atol=1e-5)


def test_swiglu_backward_matches_autograd():
    g = torch.Generator().manual_seed(2)
    m, f = 33, 40
    y_t, y_u = _bf16(g, m, 2 * f, std=2.0)
    d_t, d_u = _bf16(g, m, f)
    dy = orc.swiglu_backward(y_u, d_u)
    yf = y_t.float().requires_grad_()
    gate, up = yf.chunk(2, -1)
    (torch.nn.functional.silu(gate) * up).backward(d_t.float())
    _ulp_close(dy, yf.grad.numpy(), frac=0.995)


def test_layer_backward_matches_autograd():
    """Whole layer: the oracle chain (bf16 at every GEMM and elementwise
    output, like the device) against autograd of the same layer in fp32."""
    g = torch.Generator().manual_seed(3)
    t, h, e, f, k = 48, 64, 6, 32, 2
    x_t, x_u = _bf16(g, t, h)
    logits = torch.randn(t, e, generator=g)
    w1_t, w1_u = _bf16(g, e, 2 * f, h, std=0.1)
    w2_t, w2_u = _bf16(g, e, h, f, std=0.1)
    go_t, go_u = _bf16(g, t, h)
    gx, gp, dw1, dw2 = orc.moe_layer_backward(x_u, logits.numpy(), w1_u, w2_u, k, go_u)

    _, idx, _, probs = orc.router(logits.numpy(), k)
    xf = x_t.float().requires_grad_()
    w1f = w1_t.float().requires_grad_()
    w2f = w2_t.float().requires_grad_()
    pf = torch.from_numpy(probs).requires_grad_()
    out = torch.zeros(t, h)
    for ti in range(t):
        for ei in idx[ti]:
            y1 = w1f[ei] @ xf[ti]
            hh = torch.nn.functional.silu(y1[:f]) * y1[f:]
            out[ti] = out[ti] + pf[ti, ei] * (w2f[ei] @ hh)
    out.backward(go_t.float())

    def close(got, ref, tag):
        scale = np.abs(ref).max() + 1e-6
        assert np.abs(got - ref).max() <= 3e-2 * scale, (tag, np.abs(got - ref).max(), scale)

    close(orc.bf16_to_f32(gx), xf.grad.numpy(), "grad_x")
    close(gp, pf.grad.numpy(), "grad_probs")
    close(orc.bf16_to_f32(dw1), w1f.grad.numpy(), "dw1")
    close(orc.bf16_to_f32(dw2), w2f.grad.numpy(), "dw2")
