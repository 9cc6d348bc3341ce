"""Pins the CPU oracle (oracle/moe_oracle.py) to the reference's own outputs.

The golden fixtures were produced by running the reference case files
(tests/golden/make_golden.py). Integer / copy paths must match bit for bit;
GEMM paths within the reference's bf16 GEMM tolerance.
"""
import hashlib

import numpy as np
import pytest
import torch

import inputs as gi
from oracle import moe_oracle as orc


def sha(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.contiguous()
        if a.dtype == torch.bfloat16:
            a = a.view(torch.int16)
        a = a.numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bits_to_tensor(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


# ------------------------------------------------------------------ bf16 rounding
def test_bf16_round_trip_matches_torch():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(100000, generator=g) * torch.exp(torch.randn(100000, generator=g) * 10)
    x = torch.cat([x, torch.tensor([0.0, -0.0, float("inf"), float("-inf"), 1e-40, 3.4e38])])
    ref = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(orc.f32_to_bf16(x.numpy()), ref)
    back = orc.bf16_to_f32(ref)
    np.testing.assert_array_equal(back, x.to(torch.bfloat16).float().numpy())


# ------------------------------------------------------------------ a3 row_id_map
def test_row_id_map_small_exact(golden):
    z = golden("case12_row_id_map.npz")
    for i in range(5):
        et, te, counts, num_out = orc.row_id_map(z[f"s{i}_rmap"])
        np.testing.assert_array_equal(et, z[f"s{i}_et"])
        np.testing.assert_array_equal(te, z[f"s{i}_te"])
        assert num_out == int(z[f"s{i}_rmap"].sum())


def test_row_id_map_full_reference_shape(golden):
    z = golden("case12_row_id_map.npz")
    t, e = z["full_shape"]
    rm = np.unpackbits(z["full_rmap_packed"], axis=1)[:, :e].astype(bool)
    et, te, counts, num_out = orc.row_id_map(rm)
    assert num_out == 86016
    assert sha(et) == str(z["full_sha_et"])
    assert sha(te) == str(z["full_sha_te"])


def test_row_id_map_align_pads_segments():
    g = np.random.default_rng(0)
    rm = g.random((50, 7)) < 0.3
    et, te, counts, num_out = orc.row_id_map(rm, align=16)
    starts = [te[:, e][te[:, e] >= 0].min() for e in range(7) if counts[e]]
    assert all(s % 16 == 0 for s in starts)
    assert num_out == int(sum(-(-c // 16) * 16 for c in counts))


# ------------------------------------------------------------------ a4/a5 permute
def test_permute_small_exact(golden):
    z = golden("case17_permute.npz")
    out, pp = orc.permute(z["s_x"], z["s_map"], z["s_probs"], int(z["s_map"].max()) + 1)
    np.testing.assert_array_equal(out, z["s_out"])
    np.testing.assert_array_equal(pp, z["s_pp"])


@pytest.mark.slow
def test_permute_full_reference_shape(golden):
    z = golden("case17_permute.npz")
    t, h, e = z["full_shape"]
    x = gi.case17_x(int(t), int(h))
    assert sha(x) == str(z["full_sha_x"]), "torch RNG differs from the fixture's"
    routed = np.unpackbits(z["full_rmap_packed"], axis=1)[:, :e].astype(bool)
    _, te, _, num_out = orc.row_id_map(routed)
    probs = np.zeros((t, e), dtype=np.float32)
    probs[routed] = z["full_probs_routed"]
    xb = x.view(torch.int16).numpy().view(np.uint16)
    out, pp = orc.permute(xb, te, probs, num_out)
    assert sha(out.view(np.int16)) == str(z["full_sha_out"])
    assert sha(pp) == str(z["full_sha_pp"])


def test_permute_kats(golden):
    z = golden("kats_permute_unpermute.npz")
    out, pp = orc.permute_trans(z["k22_inp"], z["k22_map"], z["k22_probs"])
    np.testing.assert_array_equal(out, z["k22_out"])
    np.testing.assert_array_equal(pp, z["k22_pp"])
    out21, _ = orc.permute_trans(z["k22_inp"], z["k22_map"], None)
    np.testing.assert_array_equal(out21, z["k21_out"])
    np.testing.assert_array_equal(out21, z["k30_out"])
    # the hidden row is not scaled by the prob (case22 negative check)
    scaled = orc.f32_to_bf16(orc.bf16_to_f32(z["k22_inp"][0]) * 10)
    assert not np.array_equal(out[0], scaled)
    out, pp = orc.permute_trans(z["m22_x"], z["m22_map"], z["m22_probs"])
    np.testing.assert_array_equal(out, z["m22_out"])
    np.testing.assert_array_equal(pp, z["m22_pp"])


# ------------------------------------------------------------------ a6-a8 unpermute
def test_unpermute_small_exact(golden):
    z = golden("case15_unpermute.npz")
    acc, out = orc.unpermute(z["s_pin"], z["s_map"])
    np.testing.assert_array_equal(out, z["s_out"])


def test_unpermute_kats(golden):
    z = golden("kats_permute_unpermute.npz")
    acc, out = orc.unpermute(z["k24_in"], z["k24_map"])
    np.testing.assert_array_equal(acc, z["k24_acc"])
    np.testing.assert_array_equal(out, z["k24_out"])
    acc, out = orc.unpermute(z["m24_in"], z["m24_map"])
    np.testing.assert_array_equal(acc, z["m24_acc"])
    np.testing.assert_array_equal(out, z["m24_out"])


@pytest.mark.slow
def test_unpermute_full_reference_shape(golden):
    z = golden("case15_unpermute.npz")
    t, h, e = (int(v) for v in z["full_shape"])
    pin = gi.case15_pin(int(z["full_rows"]), h)
    assert sha(pin) == str(z["full_sha_pin"]), "torch RNG differs from the fixture's"
    routed = np.unpackbits(z["full_rmap_packed"], axis=1)[:, :e].astype(bool)
    et, _, _, _ = orc.row_id_map(routed)
    _, out = orc.unpermute(pin.view(torch.int16).numpy().view(np.uint16), et)
    assert sha(out.view(np.int16)) == str(z["full_sha_out"])


def test_weighted_combine_matches_torch_restatement(golden):
    z = golden("router_combine.npz")
    acc, out = orc.unpermute(z["w_pin"], z["w_map_et"], z["w_probs"], "dense")
    np.testing.assert_array_equal(acc, z["w_acc"])
    np.testing.assert_array_equal(out, z["w_out"])
    # permuted-probs mode gives the same sums
    _, te, _, n = orc.row_id_map(z["w_map_et"].T >= 0)
    pp = np.zeros(n, np.float32)
    pp[te[te >= 0]] = z["w_probs"][te >= 0]
    acc2, _ = orc.unpermute(z["w_pin"], z["w_map_et"], pp, "permuted")
    np.testing.assert_array_equal(acc2, z["w_acc"])


# ------------------------------------------------------------------ a1 top-k / router
def test_topk_small_kat(golden):
    z = golden("case23_topk.npz")
    v, i = orc.topk(z["small_in"], 2)
    np.testing.assert_array_equal(v, z["small_v"])
    np.testing.assert_array_equal(i, z["small_i"])


def test_topk_edge_suite(golden):
    z = golden("case23_topk.npz")
    for name, (x, k) in gi.topk_cases().items():
        assert sha(x) == str(z[f"{name}_sha_in"]), f"{name}: torch RNG differs"
        v, i = orc.topk(x.numpy(), k)
        np.testing.assert_array_equal(i, z[f"{name}_i"].astype(np.int64), err_msg=name)
        if f"{name}_v" in z:
            np.testing.assert_array_equal(v, z[f"{name}_v"], err_msg=name)
        np.testing.assert_array_equal(v, np.take_along_axis(x.numpy(), i, axis=1))


def test_router_matches_torch_restatement(golden):
    z = golden("router_combine.npz")
    gates, idx, rmap, probs = orc.router(z["r_logits"], 8, z["r_bias"], "softmax", renorm=False)
    np.testing.assert_array_equal(idx, z["r_idx"])
    np.testing.assert_allclose(gates, z["r_gates"], rtol=2e-6, atol=1e-9)
    gates, idx, rmap, probs = orc.router(z["r_logits"], 8, z["r_bias"], "softmax", renorm=True)
    np.testing.assert_allclose(gates, z["r_gates_renorm"], rtol=2e-6, atol=1e-9)
    assert rmap.sum() == 8 * rmap.shape[0]
    np.testing.assert_allclose(probs.sum(1), 1.0, rtol=1e-6)


# ------------------------------------------------------------------ a9-a11 GEMM
def _gemm_close(got_u16, ref_f32):
    """Reference bf16 GEMM tolerance: kernel_cases/case35_...:66-75."""
    got = orc.bf16_to_f32(got_u16)
    diff = np.abs(got - ref_f32)
    max_rel = (diff / np.maximum(np.abs(ref_f32), 1.0)).max()
    max_abs = diff.max()
    assert not (max_rel > 2e-2 and max_abs > 2e-1), (max_rel, max_abs)


def test_grouped_gemm_against_reference_models(golden):
    z = golden("gemm_swiglu.npz")
    for tag in ("c03", "c04", "c10", "c14"):
        y = orc.grouped_gemm(z[f"{tag}_x"], z[f"{tag}_w"], z[f"{tag}_splits"])
        ref = orc.bf16_to_f32(z[f"{tag}_y"])
        _gemm_close(y, ref)
        # bf16 outputs agree to within one bf16 ulp of each other
        rel = np.abs(orc.bf16_to_f32(y) - ref) / np.maximum(np.abs(ref), 1e-3)
        assert rel.max() <= 2 ** -7, tag


def test_single_expert_gemm_fp32_golden(golden):
    z = golden("gemm_swiglu.npz")
    y = orc.grouped_gemm(z["c35_x"], z["c35_w"][None], [z["c35_x"].shape[0]])
    _gemm_close(y, z["c35_y"])


def test_single_expert_nn_gemm_fp32_golden(golden):
    """case37: out = grad_output @ weight ("NN"), the one-group dgrad form."""
    z = golden("gemm_swiglu.npz")
    y = orc.grouped_gemm(z["c37_x"], z["c37_w"][None], [z["c37_x"].shape[0]], w_layout="KN")
    _gemm_close(y, z["c37_y"])


def test_grouped_dgrad_against_reference_models(golden):
    """case07/08 (groups) and case13/19 (one group): dx = dy[seg] @ w[g]."""
    z = golden("gemm_swiglu.npz")
    for tag in ("c07", "c08", "c13", "c19"):
        y = orc.grouped_gemm(z[f"{tag}_dy"], z[f"{tag}_w"], z[f"{tag}_splits"], w_layout="KN")
        _gemm_close(y, orc.bf16_to_f32(z[f"{tag}_dx"]))


def test_grouped_wgrad_against_reference_models(golden):
    """case05 (fc2) and case09 (fc1): dW[g] = dy[seg].T @ x[seg]."""
    z = golden("gemm_swiglu.npz")
    for tag in ("c05", "c09"):
        y = orc.grouped_wgrad(z[f"{tag}_dy"], z[f"{tag}_x"], z[f"{tag}_splits"])
        assert y.shape == z[f"{tag}_dw"].shape
        _gemm_close(y, orc.bf16_to_f32(z[f"{tag}_dw"]))


def test_router_gemm_fp32_golden(golden):
    """case38 reference_fp32 (router gate GEMM, fp32 out) at N = 320 experts:
    both sides accumulate in fp32 and differ only in summation order."""
    z = golden("gemm_swiglu.npz")
    y = orc.router_logits(z["c38_x"], z["c38_w"])
    assert y.dtype == np.float32 and y.shape == z["c38_y"].shape == (80, 320)
    np.testing.assert_allclose(y, z["c38_y"], rtol=1e-5, atol=1e-4)


def test_permute_backward_goldens(golden):
    """case18 Model (int64 map) small, case32 KAT and medium (int32 map): the
    fp32 sums, the bf16 outputs and the gathered prob gradients, bit for bit."""
    z = golden("permute_bwd.npz")
    acc, out, gp = orc.permute_backward(z["s18_dperm"], z["s18_map"], z["s18_dpp"])
    np.testing.assert_array_equal(out, z["s18_dact"])
    np.testing.assert_array_equal(gp, z["s18_dprobs"])
    for tag in ("k32", "m32"):
        acc, out, gp = orc.permute_backward(z[f"{tag}_in"], z[f"{tag}_map"], z[f"{tag}_pg"])
        np.testing.assert_array_equal(acc, z[f"{tag}_acc"], err_msg=tag)
        np.testing.assert_array_equal(out, z[f"{tag}_out"], err_msg=tag)
        np.testing.assert_array_equal(gp, z[f"{tag}_gp"], err_msg=tag)


def test_permute_backward_full_reference_shape(golden):
    """case18 at its own shape (T=4096, H=8192, E=320, top-8), SHA-256 equal."""
    z = golden("permute_bwd.npz")
    t, h, e, k = (int(v) for v in z["full_shape"])
    rm, dperm, dpp = gi.case18_inputs(t, h, e, k)
    assert sha(dperm) == str(z["full_sha_dperm"]) and sha(dpp) == str(z["full_sha_dpp"])
    assert (np.unpackbits(z["full_rmap_packed"], axis=1)[:, :e].astype(bool) == rm.numpy()).all()
    et, _, _, _ = orc.row_id_map(rm.numpy())
    _, out, gp = orc.permute_backward(dperm.view(torch.int16).numpy().view(np.uint16), et,
                                      dpp.numpy())
    assert hashlib.sha256(out.tobytes()).hexdigest() == str(z["full_sha_dact"])
    assert hashlib.sha256(gp.tobytes()).hexdigest() == str(z["full_sha_dprobs"])


def test_swiglu_matches_torch_restatement(golden):
    z = golden("gemm_swiglu.npz")
    h = orc.swiglu(z["swiglu_y"])
    ref = orc.bf16_to_f32(z["swiglu_h"])
    got = orc.bf16_to_f32(h)
    assert (np.abs(got - ref) <= np.abs(ref) * 2 ** -8 + 1e-6).all()


def test_uniform_group_sizes():
    assert orc.group_sizes(4096, 40)[:2] == [103, 103]
    assert sum(orc.group_sizes(4096, 40)) == 4096
