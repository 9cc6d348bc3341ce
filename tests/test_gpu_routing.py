"""GPU parity of the routing stage: top-k, fused router, row_id_map.

Bit-exact against the reference's golden outputs (indices, maps) and the CPU
oracle; gate weights within rtol 1e-5.
"""
import hashlib

import numpy as np
import pytest
import torch

import inputs as gi
from conftest import load_bundle
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def sha(t) -> str:
    a = t.detach().contiguous().cpu()
    return hashlib.sha256(a.numpy().tobytes()).hexdigest()


# ------------------------------------------------------------------ a1 top-k
def test_topk_small_kat(cuda_dev, golden):
    z = golden("case23_topk.npz")
    k23 = load_bundle("case23_aten_topk")
    v, i = k23.kernel_function(torch.from_numpy(z["small_in"]).to(cuda_dev), 2)
    assert v.dtype == torch.float32 and i.dtype == torch.int64 and v.device == cuda_dev
    np.testing.assert_array_equal(v.cpu().numpy(), z["small_v"])
    np.testing.assert_array_equal(i.cpu().numpy(), z["small_i"])


def test_topk_edge_suite_exact(cuda_dev, golden):
    z = golden("case23_topk.npz")
    k23 = load_bundle("case23_aten_topk")
    for name, (x, k) in gi.topk_cases().items():
        v, i = k23.kernel_function(x.to(cuda_dev), k)
        i = i.cpu().numpy()
        np.testing.assert_array_equal(i, z[f"{name}_i"].astype(np.int64), err_msg=name)
        vals = v.cpu().numpy()
        np.testing.assert_array_equal(vals, np.take_along_axis(x.numpy(), i, axis=1),
                                      err_msg=name)
        if f"{name}_v" in z:
            np.testing.assert_array_equal(vals, z[f"{name}_v"], err_msg=name)


def test_topk_nan_ranks_first(cuda_dev):
    x = torch.tensor([[1.0, float("nan"), 3.0, 2.0, float("nan")]])
    v, i = load_bundle("case23_aten_topk").kernel_function(x.to(cuda_dev), 3)
    ref_v, ref_i = orc.topk(x.numpy(), 3)
    np.testing.assert_array_equal(i.cpu().numpy(), ref_i)
    tv, ti = torch.topk(x, 3)
    np.testing.assert_array_equal(i.cpu().numpy(), ti.numpy())


def test_topk_bad_arguments(cuda_dev):
    k23 = load_bundle("case23_aten_topk")
    x = torch.randn(4, 32, device=cuda_dev)
    with pytest.raises(ValueError):
        k23.kernel_function(x, 8, largest=False)
    with pytest.raises(ValueError):
        k23.kernel_function(x, 8, dim=0)
    with pytest.raises(ValueError):
        k23.kernel_function(x, 17)
    with pytest.raises(ValueError):
        k23.kernel_function(torch.randn(4, 32), 8)  # CPU tensor: no CPU path


@pytest.mark.parametrize("t,e,k", [(4096, 64, 8), (8192, 256, 8), (1000, 320, 8), (333, 33, 5)])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_softmax_topk(cuda_dev, t, e, k, renorm):
    g = torch.Generator().manual_seed(t + e + k)
    lg = torch.randn(t, e, generator=g)
    bias = -1.5 * torch.log(torch.randperm(e, generator=g).float() + 1)
    import moe_b200
    r = moe_b200.router_topk(lg.to(cuda_dev), k, "softmax", renorm, bias.to(cuda_dev))
    gates, idx, rmap, probs = orc.router(lg.numpy(), k, bias.numpy(), "softmax", renorm)
    np.testing.assert_array_equal(r.topk_idx.cpu().numpy(), idx)
    np.testing.assert_allclose(r.topk_vals.cpu().numpy(), gates, rtol=1e-5, atol=1e-7)
    np.testing.assert_array_equal(r.routing_map.cpu().numpy(), rmap)
    np.testing.assert_allclose(r.probs.cpu().numpy(), probs, rtol=1e-5, atol=1e-7)


def test_router_raw_logits_matches_topk(cuda_dev):
    import moe_b200
    x = torch.randn(2048, 256, generator=torch.Generator().manual_seed(1))
    r = moe_b200.router_topk(x.to(cuda_dev), 8, "logits", renorm=False)
    v, i = orc.topk(x.numpy(), 8)
    np.testing.assert_array_equal(r.topk_idx.cpu().numpy(), i)
    np.testing.assert_array_equal(r.topk_vals.cpu().numpy(), v)


# ------------------------------------------------------------------ a3 row_id_map
def test_row_id_map_small_exact(cuda_dev, golden):
    z = golden("case12_row_id_map.npz")
    k12 = load_bundle("case12_moe_row_id_map_pass2")
    for i in range(5):
        et, te = k12.kernel_function(torch.from_numpy(z[f"s{i}_rmap"]).to(cuda_dev))
        assert et.dtype == torch.int64 and te.dtype == torch.int64
        np.testing.assert_array_equal(et.cpu().numpy(), z[f"s{i}_et"])
        np.testing.assert_array_equal(te.cpu().numpy(), z[f"s{i}_te"])


def test_row_id_map_full_reference_shape(cuda_dev, golden):
    z = golden("case12_row_id_map.npz")
    t, e = z["full_shape"]
    rm = np.unpackbits(z["full_rmap_packed"], axis=1)[:, :e].astype(bool)
    et, te = load_bundle("case12_moe_row_id_map_pass2").kernel_function(
        torch.from_numpy(rm).to(cuda_dev))
    assert sha(et) == str(z["full_sha_et"])
    assert sha(te) == str(z["full_sha_te"])


@pytest.mark.parametrize("t,e,align", [(16384, 256, 1), (8192, 256, 128), (777, 1000, 16),
                                       (1, 5, 1), (65, 300, 8)])
def test_row_id_map_vs_oracle(cuda_dev, t, e, align):
    import moe_b200
    g = torch.Generator().manual_seed(t * 7 + e)
    rm = torch.rand(t, e, generator=g) < 0.04
    r = moe_b200.row_id_map(rm.to(cuda_dev), align=align)
    et, te, counts, num_out = orc.row_id_map(rm.numpy(), align)
    np.testing.assert_array_equal(r.map_et.cpu().numpy(), et)
    np.testing.assert_array_equal(r.map_te.cpu().numpy(), te)
    np.testing.assert_array_equal(r.counts.cpu().numpy(), counts)
    assert int(r.num_out.item()) == num_out


def test_row_id_map_empty_tokens(cuda_dev):
    import moe_b200
    r = moe_b200.row_id_map(torch.zeros(0, 16, dtype=torch.bool, device=cuda_dev))
    assert r.map_et.shape == (16, 0) and r.map_te.shape == (0, 16)
    assert int(r.num_out.item()) == 0
    assert int(r.counts.abs().sum().item()) == 0


def test_router_to_row_id_map_chain_cfg1(cuda_dev):
    """BASELINE cfg1 routing: T=4096, E=64, softmax top-8 -> maps, bit-exact."""
    import moe_b200
    g = torch.Generator().manual_seed(1)
    lg = torch.randn(4096, 64, generator=g)
    r = moe_b200.router_topk(lg.to(cuda_dev), 8, "softmax", renorm=False)
    m = moe_b200.row_id_map(r.routing_map)
    _, _, rmap, _ = orc.router(lg.numpy(), 8, None, "softmax", False)
    et, te, counts, num_out = orc.row_id_map(rmap)
    assert num_out == 4096 * 8
    np.testing.assert_array_equal(m.map_te.cpu().numpy(), te)
    np.testing.assert_array_equal(m.map_et.cpu().numpy(), et)


@pytest.mark.parametrize("t,e,k", [(2048, 256, 8), (333, 64, 4)])
def test_router_with_placement(cuda_dev, t, e, k):
    """Placed router: slot c reads model expert placement[c]; maps exact vs oracle."""
    import moe_b200
    g = torch.Generator().manual_seed(e + k)
    lg = torch.randn(t, e, generator=g)
    bias = -1.5 * torch.log(torch.randperm(e, generator=g).float() + 1)
    pl = torch.randperm(e, generator=g).to(torch.int32)
    r = moe_b200.router_topk(lg.to(cuda_dev), k, "softmax", True, bias.to(cuda_dev),
                             placement=pl.to(cuda_dev))
    gates, idx, rmap, probs = orc.router(lg.numpy(), k, bias.numpy(), "softmax", True,
                                         placement=pl.numpy())
    np.testing.assert_array_equal(r.topk_idx.cpu().numpy(), idx)
    np.testing.assert_array_equal(r.routing_map.cpu().numpy(), rmap)
    np.testing.assert_allclose(r.probs.cpu().numpy(), probs, rtol=1e-5, atol=1e-7)
    # the same experts as the unplaced router, named by slot
    r0 = moe_b200.router_topk(lg.to(cuda_dev), k, "softmax", True, bias.to(cuda_dev))
    model_ids = pl.to(cuda_dev).long()[r.topk_idx]
    assert torch.equal(torch.sort(model_ids, 1).values, torch.sort(r0.topk_idx, 1).values)
