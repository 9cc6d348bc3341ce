"""GPU parity of permute (dispatch) and unpermute (combine).

Permute is a pure copy and the combine accumulates in ascending expert order
with one fp32 rounding per operation, so both must match the reference /
oracle bit for bit.
"""
import hashlib

import numpy as np
import pytest
import torch

import inputs as gi
from conftest import from_u16, load_bundle, u16
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def sha(t) -> str:
    a = t.detach().contiguous().cpu()
    if a.dtype == torch.bfloat16:
        a = a.view(torch.int16)
    return hashlib.sha256(a.numpy().tobytes()).hexdigest()


# ------------------------------------------------------------------ a4 permute
def test_permute_small_exact(cuda_dev, golden):
    z = golden("case17_permute.npz")
    k17 = load_bundle("case17_moe_permute_with_mask_map")
    out, pp = k17.kernel_function(from_u16(z["s_x"], cuda_dev),
                                  torch.from_numpy(z["s_map"]).to(cuda_dev),
                                  torch.from_numpy(z["s_probs"]).to(cuda_dev))
    np.testing.assert_array_equal(u16(out), z["s_out"])
    np.testing.assert_array_equal(pp.cpu().numpy(), z["s_pp"])


def test_permute_full_reference_shape(cuda_dev, golden):
    """case17 at its own shape (T=16384, H=8192, E=320, R=86016), SHA-256 equal."""
    z = golden("case17_permute.npz")
    t, h, e = (int(v) for v in z["full_shape"])
    x = gi.case17_x(t, h)
    assert sha(x) == str(z["full_sha_x"]), "torch RNG differs from the fixture's"
    routed = np.unpackbits(z["full_rmap_packed"], axis=1)[:, :e].astype(bool)
    probs = np.zeros((t, e), dtype=np.float32)
    probs[routed] = z["full_probs_routed"]
    rm = load_bundle("case12_moe_row_id_map_pass2").kernel_function(
        torch.from_numpy(routed).to(cuda_dev))[1]
    out, pp = load_bundle("case17_moe_permute_with_mask_map").kernel_function(
        x.to(cuda_dev), rm, torch.from_numpy(probs).to(cuda_dev))
    assert out.shape[0] == int(z["full_num_out"])
    assert sha(out) == str(z["full_sha_out"])
    assert sha(pp) == str(z["full_sha_pp"])


def test_permute_trans_kats(cuda_dev, golden):
    z = golden("kats_permute_unpermute.npz")
    inp = from_u16(z["k22_inp"], cuda_dev)
    mp = torch.from_numpy(z["k22_map"]).to(cuda_dev)
    pr = torch.from_numpy(z["k22_probs"]).to(cuda_dev)
    out, pp = load_bundle("case22_moe_permute_mask_kernel_true").kernel_function(inp, mp, pr)
    np.testing.assert_array_equal(u16(out), z["k22_out"])
    np.testing.assert_array_equal(pp.cpu().numpy(), z["k22_pp"])
    for case, key in (("case21_permute_with_mask_map_trans", "k21_out"),
                      ("case30_moe_permute_mask_kernel", "k30_out")):
        o = load_bundle(case).kernel_function(inp, mp)
        np.testing.assert_array_equal(u16(o), z[key])
        o32 = load_bundle(case).kernel_function(inp, mp.to(torch.int32))
        np.testing.assert_array_equal(u16(o32), z[key])
    out, pp = load_bundle("case22_moe_permute_mask_kernel_true").kernel_function(
        from_u16(z["m22_x"], cuda_dev), torch.from_numpy(z["m22_map"]).to(cuda_dev),
        torch.from_numpy(z["m22_probs"]).to(cuda_dev))
    np.testing.assert_array_equal(u16(out), z["m22_out"])
    np.testing.assert_array_equal(pp.cpu().numpy(), z["m22_pp"])


def test_permute_empty_map(cuda_dev):
    inp = torch.randn(5, 16, device=cuda_dev).to(torch.bfloat16)
    mp = torch.full((3, 5), -1, dtype=torch.int64, device=cuda_dev)
    pr = torch.zeros(5, 3, device=cuda_dev)
    out, pp = load_bundle("case22_moe_permute_mask_kernel_true").kernel_function(inp, mp, pr)
    assert out.shape == (0, 16) and pp.shape == (0,)


def test_permute_sparse_map_zero_fills_unwritten_rows(cuda_dev):
    import moe_b200
    x = torch.randn(4, 8, device=cuda_dev).to(torch.bfloat16)
    mp = torch.tensor([[0, -1], [-1, 5], [2, -1], [-1, -1]], dtype=torch.int64, device=cuda_dev)
    out, _ = moe_b200.permute(x, mp)
    ref, _ = orc.permute(u16(x), mp.cpu().numpy(), None, 6)
    np.testing.assert_array_equal(u16(out), ref)


@pytest.mark.parametrize("t,h,e,k", [(4096, 2048, 64, 8), (1000, 7168, 256, 8), (333, 8, 33, 3),
                                     (64, 12288, 16, 2), (17, 16384, 8, 8)])
def test_permute_chain_vs_oracle(cuda_dev, t, h, e, k):
    """Router -> row_id_map -> permute (BASELINE cfg1 first), bit-exact."""
    import moe_b200
    g = torch.Generator().manual_seed(t + h)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    lg = torch.randn(t, e, generator=g)
    r = moe_b200.router_topk(lg.to(cuda_dev), k, "softmax", renorm=False)
    m = moe_b200.row_id_map(r.routing_map)
    out, pp = moe_b200.permute(x.to(cuda_dev), m.map_te, r.probs, num_out=t * k)
    _, _, rmap, probs = orc.router(lg.numpy(), k, None, "softmax", False)
    _, te, _, n = orc.row_id_map(rmap)
    ref, ref_pp = orc.permute(u16(x), te, probs, n)
    np.testing.assert_array_equal(u16(out), ref)
    np.testing.assert_allclose(pp.cpu().numpy(), ref_pp, rtol=1e-5, atol=1e-7)
    # the same rows through the [E,T] map
    out2, _ = moe_b200.permute_trans(x.to(cuda_dev), m.map_et, None, num_out=t * k)
    np.testing.assert_array_equal(u16(out2), ref)


def test_permute_paths_give_the_same_bits(cuda_dev):
    """The bulk-copy permute (MOE_PERMUTE_BULK=1: rows staged in shared memory
    by bulk TMA loads and written by bulk TMA stores), the register-staged
    kernel with 16-byte vectors (the default) and with 32-byte vectors
    (MOE_PERMUTE_V32=1), each in a fresh process, give the same bits, for the
    token-major map with probs and the [E,T] int32 map, with fewer tokens
    than CTAs and with many tokens per CTA; the device error word stays 0."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    code = r'''
import sys, hashlib, torch
sys.path[:0] = [sys.argv[1], sys.argv[2], sys.argv[3]]
import moe_b200
from moe_b200 import _lib
from ctypes import byref, c_int32
dev = torch.device("cuda", 0)
out = []
for t, h, e, k in ((3, 7168, 16, 4), (20000, 1024, 64, 8), (2500, 16384, 32, 2)):
    g = torch.Generator().manual_seed(t)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16).to(dev)
    lg = torch.randn(t, e, generator=g).to(dev)
    r = moe_b200.router_topk(lg, k, "softmax", renorm=True)
    m = moe_b200.row_id_map(r.routing_map)
    a, pa = moe_b200.permute(x, m.map_te, r.probs, num_out=t * k)
    b, _ = moe_b200.permute_trans(x, m.map_et.to(torch.int32), None, num_out=t * k)
    for v in (a.view(torch.int16), pa, b.view(torch.int16)):
        out.append(hashlib.sha256(v.cpu().numpy().tobytes()).hexdigest())
err = c_int32(-1)
assert _lib.load().moe_permute_check(None, byref(err)) == 0 and err.value == 0
print(" ".join(out))
'''
    res = {}
    for flag, envs in (("1", {"MOE_PERMUTE_BULK": "1"}), ("0", {}),
                       ("v32", {"MOE_PERMUTE_V32": "1"})):
        env = dict(os.environ, **envs)
        r = subprocess.run([sys.executable, "-c", code, str(ROOT / "1188b-reference-kernels_b200"),
                            str(ROOT), str(ROOT / "tests")], env=env, capture_output=True,
                           text=True, timeout=300)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        res[flag] = r.stdout.split()
    assert res["1"] == res["0"] == res["v32"]


@pytest.mark.parametrize("t,h,e,k", [(4096, 7168, 256, 8), (333, 1024, 64, 4), (7, 8, 16, 2)])
def test_permute_from_expert_list_equals_map_permute(cuda_dev, t, h, e, k):
    """moe_permute_topk (destinations read from the router's [T,k] expert list,
    in selection order or shuffled) gives the same rows and permuted probs as
    the map-scanning permute, and both equal the oracle."""
    import moe_b200
    g = torch.Generator().manual_seed(t + k)
    x = torch.randn(t, h, generator=g).to(torch.bfloat16).to(cuda_dev)
    lg = torch.randn(t, e, generator=g).to(cuda_dev)
    r = moe_b200.router_topk(lg, k, "softmax", renorm=True, outputs="all")
    m = moe_b200.row_id_map(r.routing_map)
    a, pa = moe_b200.permute(x, m.map_te, r.probs, num_out=t * k)
    b, pb = moe_b200.permute(x, m.map_te, r.probs, num_out=t * k, experts=r.topk_idx)
    perm = torch.argsort(torch.rand(t, k, generator=g), dim=1).to(cuda_dev)
    c, pc = moe_b200.permute(x, m.map_te, r.probs, num_out=t * k,
                             experts=torch.gather(r.topk_idx, 1, perm))
    assert torch.equal(a, b) and torch.equal(a, c)
    assert torch.equal(pa, pb) and torch.equal(pa, pc)
    ref, _ = orc.permute(u16(x), m.map_te.cpu().numpy(), None, t * k)
    np.testing.assert_array_equal(u16(b), ref)


# ------------------------------------------------------------------ a6-a8 unpermute
def test_unpermute_small_exact(cuda_dev, golden):
    z = golden("case15_unpermute.npz")
    out = load_bundle("case15_moe_unpermute_mask_fwd").kernel_function(
        from_u16(z["s_pin"], cuda_dev), torch.from_numpy(z["s_map"]).to(cuda_dev))
    np.testing.assert_array_equal(u16(out), z["s_out"])


def test_unpermute_kats_int32(cuda_dev, golden):
    z = golden("kats_permute_unpermute.npz")
    k24 = load_bundle("case24_moe_unpermute_mask_kernel_false")
    acc, out = k24.kernel_function(from_u16(z["k24_in"], cuda_dev),
                                   torch.from_numpy(z["k24_map"]).to(cuda_dev))
    np.testing.assert_array_equal(acc.cpu().numpy(), z["k24_acc"])
    np.testing.assert_array_equal(u16(out), z["k24_out"])
    acc, out = k24.kernel_function(from_u16(z["m24_in"], cuda_dev),
                                   torch.from_numpy(z["m24_map"]).to(cuda_dev))
    np.testing.assert_array_equal(acc.cpu().numpy(), z["m24_acc"])
    np.testing.assert_array_equal(u16(out), z["m24_out"])
    with pytest.raises(ValueError):
        k24.kernel_function(from_u16(z["k24_in"][:1], cuda_dev),
                            torch.from_numpy(z["k24_map"]).to(cuda_dev))


def test_unpermute_full_reference_shape(cuda_dev, golden):
    """case15 at its own shape (R=86016, H=8192, E=320), SHA-256 equal."""
    z = golden("case15_unpermute.npz")
    t, h, e = (int(v) for v in z["full_shape"])
    pin = gi.case15_pin(int(z["full_rows"]), h)
    assert sha(pin) == str(z["full_sha_pin"]), "torch RNG differs from the fixture's"
    routed = np.unpackbits(z["full_rmap_packed"], axis=1)[:, :e].astype(bool)
    et = load_bundle("case12_moe_row_id_map_pass2").kernel_function(
        torch.from_numpy(routed).to(cuda_dev))[0]
    out = load_bundle("case15_moe_unpermute_mask_fwd").kernel_function(pin.to(cuda_dev), et)
    assert sha(out) == str(z["full_sha_out"])


def test_weighted_combine_golden(cuda_dev, golden):
    import moe_b200
    z = golden("router_combine.npz")
    out, acc = moe_b200.unpermute(from_u16(z["w_pin"], cuda_dev),
                                  torch.from_numpy(z["w_map_et"]).to(cuda_dev),
                                  torch.from_numpy(z["w_probs"]).to(cuda_dev), "dense",
                                  return_acc=True)
    np.testing.assert_array_equal(acc.cpu().numpy(), z["w_acc"])
    np.testing.assert_array_equal(u16(out), z["w_out"])
    w = moe_b200.unpermute_weighted(from_u16(z["w_pin"], cuda_dev),
                                    torch.from_numpy(z["w_map_et"]).to(cuda_dev),
                                    torch.from_numpy(z["w_probs"]).to(cuda_dev))
    np.testing.assert_array_equal(u16(w), z["w_out"])


@pytest.mark.parametrize("t,h,e,k,mode", [(8192, 7168, 256, 8, "dense"),
                                          (8192, 7168, 256, 8, "permuted"),
                                          (257, 2048, 64, 6, "dense"), (100, 16384, 16, 4, None),
                                          (31, 72, 300, 16, "dense")])
def test_combine_vs_oracle(cuda_dev, t, h, e, k, mode):
    """BASELINE cfg2 (T=8192, H=7168, E=256, renormalised probs) and others;
    checked bit-exact on a token subset at full size."""
    import moe_b200
    g = torch.Generator().manual_seed(t * 3 + e)
    lg = torch.randn(t, e, generator=g)
    r = moe_b200.router_topk(lg.to(cuda_dev), k, "softmax", renorm=True)
    m = moe_b200.row_id_map(r.routing_map)
    rows = t * k
    pin = torch.randn(rows, h, generator=g).to(torch.bfloat16)
    probs = None
    if mode == "dense":
        probs = r.probs
    elif mode == "permuted":
        _, probs = moe_b200.permute(torch.zeros(t, 8, dtype=torch.bfloat16, device=cuda_dev),
                                    m.map_te, r.probs, num_out=rows)
    out, acc = moe_b200.unpermute(pin.to(cuda_dev), m.map_et, probs,
                                  mode or "dense", return_acc=True)
    tokens = np.unique(np.concatenate([np.arange(min(t, 64)), np.arange(max(0, t - 64), t),
                                       np.random.default_rng(0).integers(0, t, 128)]))
    p_np = None if probs is None else probs.cpu().numpy()
    ref_acc, ref = orc.unpermute(u16(pin), m.map_et.cpu().numpy(), p_np, mode or "dense",
                                 tokens=tokens)
    np.testing.assert_array_equal(acc.cpu().numpy()[tokens], ref_acc)
    np.testing.assert_array_equal(u16(out)[tokens], ref)
    # token-major map: same sums, same bits
    out_tm, acc_tm = moe_b200.unpermute(pin.to(cuda_dev), m.map_te, probs, mode or "dense",
                                        return_acc=True, token_major=True)
    assert torch.equal(out_tm, out) and torch.equal(acc_tm, acc)


def test_permute_unpermute_round_trip_full_size(cuda_dev):
    """Size-independent property at the full layer shape: with unit rows the
    unweighted combine of a permute is k * x exactly (k = 8 is a power of 2)."""
    import moe_b200
    t, h, e, k = 16384, 7168, 256, 8
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    x = torch.randn(t, h, device=cuda_dev, generator=g).to(torch.bfloat16)
    lg = torch.randn(t, e, device=cuda_dev, generator=g)
    r = moe_b200.router_topk(lg, k, "softmax", renorm=True)
    m = moe_b200.row_id_map(r.routing_map)
    xp, _ = moe_b200.permute(x, m.map_te, None, num_out=t * k)
    back = moe_b200.unpermute(xp, m.map_et)
    assert torch.equal(back, (x.float() * k).to(torch.bfloat16))
    # weighted with renormalised gates returns x up to rounding
    back_w = moe_b200.unpermute(xp, m.map_et, r.probs, "dense")
    torch.testing.assert_close(back_w.float(), x.float(), rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("h", [1, 2, 3, 4, 6, 12, 1030])
def test_odd_hidden_sizes(cuda_dev, h):
    """Rows that are not a multiple of 8 elements take the 4- or 2-byte path."""
    import moe_b200
    g = torch.Generator().manual_seed(h)
    t, e, k = 37, 12, 3
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    lg = torch.randn(t, e, generator=g)
    _, _, rmap, probs = orc.router(lg.numpy(), k, None, "softmax", True)
    et, te, _, n = orc.row_id_map(rmap)
    out, pp = moe_b200.permute(x.to(cuda_dev), torch.from_numpy(te).to(cuda_dev),
                               torch.from_numpy(probs).to(cuda_dev), num_out=n)
    ref, ref_pp = orc.permute(u16(x), te, probs, n)
    np.testing.assert_array_equal(u16(out), ref)
    np.testing.assert_array_equal(pp.cpu().numpy(), ref_pp)
    pin = torch.randn(n, h, generator=g).to(torch.bfloat16)
    o, acc = moe_b200.unpermute(pin.to(cuda_dev), torch.from_numpy(et).to(cuda_dev),
                                torch.from_numpy(probs).to(cuda_dev), "dense", return_acc=True)
    ref_acc, ref_o = orc.unpermute(u16(pin), et, probs, "dense")
    np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
    np.testing.assert_array_equal(u16(o), ref_o)
    # a row view that starts 2 bytes into an allocation (unaligned for 16-byte vectors)
    xs = torch.randn(t * h + 1, generator=g).to(torch.bfloat16).to(cuda_dev)[1:].view(t, h)
    out2, _ = moe_b200.permute(xs, torch.from_numpy(te).to(cuda_dev), None, num_out=n)
    ref2, _ = orc.permute(u16(xs), te, None, n)
    np.testing.assert_array_equal(u16(out2), ref2)


# ------------------------------------------------------------------ f3 permute backward
def test_permute_backward_goldens(cuda_dev, golden):
    """case18 bundle (int64 map) small; case32 bundle (int32 map) on its KAT and
    a medium run: bit-exact sums, bf16 outputs and gathered prob gradients."""
    z = golden("permute_bwd.npz")
    k18 = load_bundle("case18_moe_permute_bwd_unpermute_mask")
    dact, dprobs = k18.kernel_function(from_u16(z["s18_dperm"], cuda_dev),
                                       torch.from_numpy(z["s18_dpp"]).to(cuda_dev),
                                       torch.from_numpy(z["s18_map"]).to(cuda_dev))
    assert dact.dtype == torch.bfloat16 and dprobs.dtype == torch.float32
    np.testing.assert_array_equal(u16(dact), z["s18_dact"])
    np.testing.assert_array_equal(dprobs.cpu().numpy(), z["s18_dprobs"])
    k32 = load_bundle("case32_moe_unpermute_mask_kernel")
    for tag in ("k32", "m32"):
        acc, out, gp = k32.kernel_function(from_u16(z[f"{tag}_in"], cuda_dev),
                                           torch.from_numpy(z[f"{tag}_map"]).to(cuda_dev),
                                           torch.from_numpy(z[f"{tag}_pg"]).to(cuda_dev))
        np.testing.assert_array_equal(acc.cpu().numpy(), z[f"{tag}_acc"], err_msg=tag)
        np.testing.assert_array_equal(u16(out), z[f"{tag}_out"], err_msg=tag)
        np.testing.assert_array_equal(gp.cpu().numpy(), z[f"{tag}_gp"], err_msg=tag)


def test_permute_backward_full_reference_shape(cuda_dev, golden):
    """case18 at its own shape (T=4096, H=8192, E=320, top-8), SHA-256 equal."""
    z = golden("permute_bwd.npz")
    t, h, e, k = (int(v) for v in z["full_shape"])
    rm, dperm, dpp = gi.case18_inputs(t, h, e, k)
    assert sha(dperm) == str(z["full_sha_dperm"]), "torch RNG differs from the fixture's"
    et = load_bundle("case12_moe_row_id_map_pass2").kernel_function(rm.to(cuda_dev))[0]
    dact, dprobs = load_bundle("case18_moe_permute_bwd_unpermute_mask").kernel_function(
        dperm.to(cuda_dev), dpp.to(cuda_dev), et)
    assert sha(dact) == str(z["full_sha_dact"])
    assert sha(dprobs) == str(z["full_sha_dprobs"])


def test_permute_backward_bad_arguments(cuda_dev):
    import moe_b200
    g = torch.zeros(8, 16, dtype=torch.bfloat16, device=cuda_dev)
    m = torch.full((4, 2), -1, dtype=torch.int64, device=cuda_dev)
    with pytest.raises(ValueError):
        moe_b200.permute_backward(g, m, torch.zeros(7, device=cuda_dev))  # wrong length
    with pytest.raises(ValueError):
        moe_b200.permute_backward(g.float(), m)
    gx, gp = moe_b200.permute_backward(g, m)  # nothing routed: zeros, no prob grad
    assert gp is None and int(gx.view(torch.int16).abs().sum()) == 0
