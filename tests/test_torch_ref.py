"""The torch CPU restatement of the reference's layer chain (oracle/torch_ref.py),
which bench.py times as the CPU baseline, pinned like the numpy oracle: its
row_id_map, permute and unweighted combine reproduce the reference goldens
exactly, and its whole layer matches the numpy oracle within the GEMM
tolerance (bf16 torch.mm vs fp32 numpy accumulation)."""
import numpy as np
import torch

from conftest import from_u16, u16
from oracle import moe_oracle as orc
from oracle import torch_ref as tr


def test_row_id_map_matches_case12_golden(golden):
    z = golden("case12_row_id_map.npz")
    for i in range(5):
        te = tr.make_row_id_map(torch.from_numpy(z[f"s{i}_rmap"]))
        np.testing.assert_array_equal(te.numpy(), z[f"s{i}_te"])


def test_permute_matches_case17_golden(golden):
    z = golden("case17_permute.npz")
    out = tr.permute(from_u16(z["s_x"], "cpu"), torch.from_numpy(z["s_map"]),
                     int(z["s_map"].max()) + 1)
    np.testing.assert_array_equal(u16(out), z["s_out"])


def test_unweighted_combine_matches_case15_golden(golden):
    z = golden("case15_unpermute.npz")
    row_te = torch.from_numpy(z["s_map"]).t().contiguous()
    ones = (row_te >= 0).float()
    out = tr.combine(from_u16(z["s_pin"], "cpu"), row_te, ones)
    np.testing.assert_array_equal(u16(out), z["s_out"])


def test_layer_matches_numpy_oracle():
    t, h, e, f, k = 160, 256, 16, 128, 4
    g = torch.Generator().manual_seed(3)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    lg = torch.randn(t, e, generator=g)
    bias = -1.5 * torch.log(torch.randperm(e, generator=g).float() + 1)
    w1 = (torch.randn(e, 2 * f, h, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(e, h, f, generator=g) * 0.05).to(torch.bfloat16)
    rmap, probs = tr.route(lg, bias, k)
    _, _, rmap_o, probs_o = orc.router(lg.numpy(), k, bias.numpy())
    np.testing.assert_array_equal(rmap.numpy(), rmap_o)
    np.testing.assert_allclose(probs.numpy(), probs_o, rtol=1e-5, atol=1e-7)
    out = tr.layer(x, lg, bias, lambda i: w1[i], lambda i: w2[i], k)
    ref = orc.moe_layer(u16(x), lg.numpy(), u16(w1), u16(w2), k, bias.numpy())
    np.testing.assert_allclose(orc.bf16_to_f32(u16(out)),
                               orc.bf16_to_f32(ref), rtol=2e-2, atol=1e-2)
