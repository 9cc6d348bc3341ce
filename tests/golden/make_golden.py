"""Generates the golden fixtures in this directory from the reference's own code.

Run once, in a checkout that has the reference corpus, with its root given
explicitly:

    python tests/golden/make_golden.py --reference-root <path-to-reference>

It imports the reference case files (plain PyTorch, CPU) from
<root>/kernel_cases, runs their Model.forward / reference_* functions on
seeded inputs and saves inputs and outputs as compressed .npz files. Large
inputs that are pure seeded torch draws are not stored; the tests regenerate
them with ``tests/golden/inputs.py`` and the fixture holds a SHA-256 of the
regenerated input so that a different torch RNG is reported as such.

Nothing at test time reads the reference; only these fixtures travel.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import inputs as gi  # noqa: E402


def sha(t) -> str:
    if isinstance(t, torch.Tensor):
        t = t.contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        a = t.numpy()
    else:
        a = np.ascontiguousarray(t)
    return hashlib.sha256(a.tobytes()).hexdigest()


def load_case(root: Path, name: str):
    path = root / "kernel_cases" / f"{name}.py"
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def save(name: str, **arrays) -> None:
    path = HERE / name
    np.savez_compressed(path, **arrays)
    print(f"wrote {path.name}: {path.stat().st_size / 1024:.1f} KiB")


def gen_case12(root: Path) -> None:
    c12 = load_case(root, "case12_moe_row_id_map_pass2")
    model = c12.Model()
    out = {}
    # Full reference shape: the reference's own seeded routing map.
    (rm,) = c12.get_inputs()
    et, te = model(rm)
    out["full_rmap_packed"] = np.packbits(rm.numpy(), axis=1)
    out["full_shape"] = np.array(rm.shape)
    out["full_sha_et"] = np.array(sha(et))
    out["full_sha_te"] = np.array(sha(te))
    # Small exact cases (own seeded maps, reference function output).
    for i, (t, e, p) in enumerate([(37, 13, 0.3), (64, 8, 0.5), (130, 64, 0.125), (5, 3, 0.0),
                                   (300, 320, 6 / 320)]):
        g = torch.Generator().manual_seed(100 + i)
        m = torch.rand(t, e, generator=g) < p
        a, b = model(m)
        out[f"s{i}_rmap"] = m.numpy()
        out[f"s{i}_et"] = a.numpy()
        out[f"s{i}_te"] = b.numpy()
    save("case12_row_id_map.npz", **out)


def gen_case17(root: Path) -> None:
    c17 = load_case(root, "case17_moe_permute_with_mask_map")
    x, row_id_map, probs = c17.get_inputs()
    model = c17.Model(*c17.get_init_inputs())
    o, pp = model(x, row_id_map, probs)
    routed = row_id_map >= 0
    x_mine = gi.case17_x()
    assert torch.equal(x_mine.view(torch.int16), x.view(torch.int16)), "x regeneration differs"
    out = {
        "full_rmap_packed": np.packbits(routed.numpy(), axis=1),
        "full_shape": np.array([x.shape[0], x.shape[1], row_id_map.shape[1]]),
        "full_probs_routed": probs[routed].numpy(),
        "full_sha_x": np.array(sha(x)),
        "full_sha_out": np.array(sha(o)),
        "full_sha_pp": np.array(sha(pp)),
        "full_num_out": np.array(o.shape[0]),
    }
    # Small case with the same structure.
    g = torch.Generator().manual_seed(17)
    t, h, e = 96, 64, 16
    xs = torch.randn(t, h, generator=g).to(torch.bfloat16)
    rm = torch.rand(t, e, generator=g) < 0.3
    mp = c17.make_row_id_map(rm)
    pr = torch.rand(t, e, generator=g) * rm
    ms = c17.Model(e, int(rm.sum()))
    so, spp = ms(xs, mp, pr)
    out.update(s_x=bits(xs), s_map=mp.numpy(), s_probs=pr.numpy(), s_out=bits(so),
               s_pp=spp.numpy())
    save("case17_permute.npz", **out)


def gen_case15(root: Path) -> None:
    c15 = load_case(root, "case15_moe_unpermute_mask_fwd")
    pin, row_id_map = c15.get_inputs()
    model = c15.Model(*c15.get_init_inputs())
    o = model(pin, row_id_map)
    pin_mine = gi.case15_pin(pin.shape[0])
    assert torch.equal(pin_mine.view(torch.int16), pin.view(torch.int16)), "pin regen differs"
    out = {
        "full_rmap_packed": np.packbits((row_id_map >= 0).t().contiguous().numpy(), axis=1),
        "full_shape": np.array([row_id_map.shape[1], pin.shape[1], row_id_map.shape[0]]),
        "full_sha_pin": np.array(sha(pin)),
        "full_sha_out": np.array(sha(o)),
        "full_rows": np.array(pin.shape[0]),
    }
    g = torch.Generator().manual_seed(15)
    t, h, e = 80, 48, 12
    rm = torch.rand(t, e, generator=g) < 0.4
    mp = c15.make_row_id_map_trans(rm)
    r = int(rm.sum())
    ps = torch.randn(r, h, generator=g).to(torch.bfloat16)
    so = c15.Model(e)(ps, mp)
    out.update(s_pin=bits(ps), s_map=mp.numpy(), s_out=bits(so))
    save("case15_unpermute.npz", **out)


def gen_kats(root: Path) -> None:
    """Known-answer inputs of case21/22/24/30 and medium-size reference runs."""
    c21 = load_case(root, "case21_ref_permute_with_mask_map_trans")
    c22 = load_case(root, "case22_ref_moe_permute_mask_kernel_true")
    c24 = load_case(root, "case24_ref_moe_unpermute_mask_kernel_false")
    c30 = load_case(root, "case30_ref_moe_permute_mask_kernel")
    out = {}
    # case22 KAT inputs (kernel_cases/case22...:106-134)
    inp = torch.arange(2 * 4, dtype=torch.bfloat16).reshape(2, 4) + 1
    mp = torch.tensor([[0, -1], [-1, 2], [1, -1], [-1, -1]], dtype=torch.int64)
    pr = torch.tensor([[10.0, 0.0, 20.0, 0.0], [0.0, 30.0, 0.0, 0.0]])
    o, pp = c22.reference_permute_mask_with_probs(inp, mp, pr)
    out.update(k22_inp=bits(inp), k22_map=mp.numpy(), k22_probs=pr.numpy(), k22_out=bits(o),
               k22_pp=pp.numpy())
    o21 = c21.reference_permute_with_mask_map_trans(inp, mp)
    o30 = c30.reference_permute_mask(inp, mp)
    out.update(k21_out=bits(o21), k30_out=bits(o30))
    # case24 KAT (kernel_cases/case24...:87-102)
    gin = torch.tensor([[4, 1], [4, 1], [7, 0]], dtype=torch.bfloat16)
    mp24 = torch.tensor([[0, -1], [-1, 2], [1, -1], [-1, -1]], dtype=torch.int32)
    acc, st = c24.reference_unpermute_mask(gin, mp24)
    out.update(k24_in=bits(gin), k24_map=mp24.numpy(), k24_acc=acc.numpy(), k24_out=bits(st))
    # medium: the reference map generators at reduced size
    for tag, mod in (("m22", c22), ("m24", c24)):
        m = mod.make_row_id_map(num_tokens=257, num_experts=32, topk=8)
        out[f"{tag}_map"] = m.numpy()
    g = torch.Generator().manual_seed(22)
    x22 = torch.randn(257, 64, generator=g).to(torch.bfloat16)
    p22 = c22.make_probs(c22.make_row_id_map(num_tokens=257, num_experts=32, topk=8), seed=1)
    o22, pp22 = c22.reference_permute_mask_with_probs(
        x22, c22.make_row_id_map(num_tokens=257, num_experts=32, topk=8), p22)
    out.update(m22_x=bits(x22), m22_probs=p22.numpy(), m22_out=bits(o22), m22_pp=pp22.numpy())
    g = torch.Generator().manual_seed(24)
    m24 = c24.make_row_id_map(num_tokens=257, num_experts=32, topk=8)
    gi24 = torch.randn(257 * 8, 64, generator=g).to(torch.bfloat16)
    a24, s24 = c24.reference_unpermute_mask(gi24, m24)
    out.update(m24_in=bits(gi24), m24_acc=a24.numpy(), m24_out=bits(s24))
    save("kats_permute_unpermute.npz", **out)


def gen_case23(root: Path) -> None:
    c23 = load_case(root, "case23_ref_aten_topk")
    out = {}
    small = torch.tensor([[0.1, 0.5, 0.3, 0.2], [4.0, 1.0, 3.0, 2.0]], dtype=torch.float32)
    v, i = c23.reference_topk(small, k=2)
    out.update(small_in=small.numpy(), small_v=v.numpy(), small_i=i.numpy())
    cases = gi.topk_cases()
    for name, (x, k) in cases.items():
        v, i = c23.reference_topk(x, k=k)
        out[f"{name}_sha_in"] = np.array(sha(x))
        out[f"{name}_k"] = np.array(k)
        if v.numel() <= 8192:  # large cases: values are checked as input[indices]
            out[f"{name}_v"] = v.numpy()
        out[f"{name}_i"] = i.numpy().astype(np.int16)
    save("case23_topk.npz", **out)


def gen_gemm(root: Path) -> None:
    c03 = load_case(root, "case03_moe_grouped_gemm_fc1_fwd")
    c04 = load_case(root, "case04_moe_grouped_gemm_fc2_fwd")
    c35 = load_case(root, "case35_ref_musa_asm_bf16_gemm_nt_256x384")
    out = {}
    for tag, mod, (g_, t_, n_, k_) in (("c03", c03, (4, 300, 128, 128)),
                                       ("c04", c04, (3, 130, 256, 64)),
                                       ("c10", c03, (1, 200, 256, 128))):
        gen = torch.Generator().manual_seed(3 + g_)
        x = torch.randn(t_, k_, generator=gen).to(torch.bfloat16)
        w = (torch.randn(g_, n_, k_, generator=gen) * 0.05).to(torch.bfloat16)
        y = mod.Model(g_, t_)(x, w)
        out.update({f"{tag}_x": bits(x), f"{tag}_w": bits(w), f"{tag}_y": bits(y),
                    f"{tag}_splits": np.array(mod.group_sizes(t_, g_))})
    gen = torch.Generator().manual_seed(35)
    inp = torch.randn(96, 512, generator=gen).to(torch.bfloat16)
    wt = torch.randn(256, 512, generator=gen).to(torch.bfloat16)
    out.update(c35_x=bits(inp), c35_w=bits(wt), c35_y=c35.reference_fp32(inp, wt).numpy())
    # Grouped dgrad (dy @ w[g], "NN"): case07/08 with several groups, case13/19 with one.
    for tag, name, (g_, t_, n_, k_) in (
            ("c07", "case07_moe_grouped_gemm_fc1_dgrad", (4, 300, 128, 192)),
            ("c08", "case08_moe_grouped_gemm_fc2_dgrad", (3, 200, 192, 128)),
            ("c13", "case13_grouped_gemm_single_group_fc1_dgrad", (1, 200, 128, 128)),
            ("c19", "case19_grouped_gemm_single_group_fc2_dgrad", (1, 100, 256, 64))):
        mod = load_case(root, name)
        gen = torch.Generator().manual_seed(7 + g_ + n_)
        dy = torch.randn(t_, n_, generator=gen).to(torch.bfloat16)
        w = (torch.randn(g_, n_, k_, generator=gen) * 0.05).to(torch.bfloat16)
        dx = mod.Model(g_, t_)(dy, w)
        out.update({f"{tag}_dy": bits(dy), f"{tag}_w": bits(w), f"{tag}_dx": bits(dx),
                    f"{tag}_splits": np.array(mod.group_sizes(t_, g_))})
    # Grouped wgrad (dy[seg].T @ x[seg], "TN"): case05 (fc2) and case09 (fc1).
    for tag, name, (g_, t_, n_, k_) in (
            ("c05", "case05_moe_grouped_gemm_fc2_wgrad", (3, 200, 192, 128)),
            ("c09", "case09_moe_grouped_gemm_fc1_wgrad", (4, 300, 128, 192))):
        mod = load_case(root, name)
        gen = torch.Generator().manual_seed(5 + g_ + n_)
        dy = torch.randn(t_, n_, generator=gen).to(torch.bfloat16)
        xw = torch.randn(t_, k_, generator=gen).to(torch.bfloat16)
        dw = mod.Model(g_, t_)(dy, xw)
        out.update({f"{tag}_dy": bits(dy), f"{tag}_x": bits(xw), f"{tag}_dw": bits(dw),
                    f"{tag}_splits": np.array(mod.group_sizes(t_, g_))})
    # Router gate GEMM (fp32 out) at the traced N = 320 experts, small M and K.
    c38 = load_case(root, "case38_ref_musa_asm_bf16_ssgemm_nt_320x256")
    gen = torch.Generator().manual_seed(38)
    inp = torch.randn(80, 512, generator=gen).to(torch.bfloat16)
    wt = torch.randn(c38.N, 512, generator=gen).to(torch.bfloat16)
    out.update(c38_x=bits(inp), c38_w=bits(wt), c38_y=c38.reference_fp32(inp, wt).numpy())
    # One-group fc2 forward (case14's own Model) and the single NN GEMM of case37.
    c14 = load_case(root, "case14_grouped_gemm_single_group_fc2_fwd")
    gen = torch.Generator().manual_seed(14)
    x = torch.randn(150, 96, generator=gen).to(torch.bfloat16)
    w = (torch.randn(1, 192, 96, generator=gen) * 0.05).to(torch.bfloat16)
    out.update(c14_x=bits(x), c14_w=bits(w), c14_y=bits(c14.Model(1, 150)(x, w)),
               c14_splits=np.array(c14.group_sizes(150, 1)))
    c37 = load_case(root, "case37_ref_musa_asm_bf16_gemm_nn_256x384")
    gen = torch.Generator().manual_seed(37)
    go = torch.randn(72, 320, generator=gen).to(torch.bfloat16)
    wt = torch.randn(320, 256, generator=gen).to(torch.bfloat16)
    out.update(c37_x=bits(go), c37_w=bits(wt), c37_y=c37.reference_fp32(go, wt).numpy())
    # Build-only ops (no reference code): torch fp32 restatements pin the numpy oracle.
    gen = torch.Generator().manual_seed(8)
    y = torch.randn(64, 2 * 96, generator=gen).to(torch.bfloat16)
    gte, up = y.float().chunk(2, -1)
    h = (torch.nn.functional.silu(gte) * up).to(torch.bfloat16)
    out.update(swiglu_y=bits(y), swiglu_h=bits(h))
    save("gemm_swiglu.npz", **out)


def gen_permute_bwd(root: Path) -> None:
    """Backward of the permute: case18 Model (int64 map) at its own shape and
    small, case32 reference_unpermute_mask (int32 map) on its KAT and medium."""
    c18 = load_case(root, "case18_moe_permute_bwd_unpermute_mask")
    c32 = load_case(root, "case32_ref_moe_unpermute_mask_kernel")
    rm, dperm, dpp = gi.case18_inputs()
    row = c18.make_row_id_map_trans(rm)
    dact, dprobs = c18.Model(rm.shape[1])(dperm, dpp, row)
    out = {"full_rmap_packed": np.packbits(rm.numpy(), axis=1),
           "full_shape": np.array([rm.shape[0], dperm.shape[1], rm.shape[1], 8]),
           "full_sha_dperm": np.array(sha(dperm)), "full_sha_dpp": np.array(sha(dpp)),
           "full_sha_dact": np.array(sha(dact)), "full_sha_dprobs": np.array(sha(dprobs))}
    rm_s, dperm_s, dpp_s = gi.case18_inputs(tokens=48, hidden=64, experts=12, topk=3)
    row_s = c18.make_row_id_map_trans(rm_s)
    da, dp = c18.Model(12)(dperm_s, dpp_s, row_s)
    out.update(s18_dperm=bits(dperm_s), s18_dpp=dpp_s.numpy(), s18_map=row_s.numpy(),
               s18_dact=bits(da), s18_dprobs=dp.numpy())
    # case32 known answer (its _check_sum_and_prob_grad inputs) and a medium run
    gin = torch.tensor([[4, 1], [4, 1], [7, 0]], dtype=torch.bfloat16)
    kmap = torch.tensor([[0, -1], [-1, 2], [1, -1], [-1, -1]], dtype=torch.int32)
    kpg = torch.tensor([10.0, 20.0, 30.0])
    acc, stored, gathered = c32.reference_unpermute_mask(gin, kmap, kpg)
    out.update(k32_in=bits(gin), k32_map=kmap.numpy(), k32_pg=kpg.numpy(), k32_acc=acc.numpy(),
               k32_out=bits(stored), k32_gp=gathered.numpy())
    mmap = c32.make_row_id_map(num_tokens=100, num_experts=24, topk=5)
    r = int(mmap.max()) + 1
    g = torch.Generator().manual_seed(32)
    gin = torch.randn(r, 128, generator=g).to(torch.bfloat16)
    pg = torch.randn(r, generator=g)
    acc, stored, gathered = c32.reference_unpermute_mask(gin, mmap, pg)
    out.update(m32_in=bits(gin), m32_map=mmap.numpy(), m32_pg=pg.numpy(), m32_acc=acc.numpy(),
               m32_out=bits(stored), m32_gp=gathered.numpy())
    save("permute_bwd.npz", **out)


def gen_router_combine() -> None:
    """Torch fp32 restatements of the build-only router and weighted combine."""
    out = {}
    g = torch.Generator().manual_seed(4)
    lg = torch.randn(257, 64, generator=g)
    bias = -1.5 * torch.log(torch.randperm(64, generator=g).float() + 1)
    z = lg + bias
    p = torch.softmax(z, dim=-1)
    _, idx = torch.sort(z, dim=1, descending=True, stable=True)
    idx = idx[:, :8]
    gates = torch.gather(p, 1, idx)
    gates_n = gates / gates.sum(-1, keepdim=True)
    out.update(r_logits=lg.numpy(), r_bias=bias.numpy(), r_idx=idx.numpy(), r_gates=gates.numpy(),
               r_gates_renorm=gates_n.numpy())
    # weighted combine: sum over experts ascending of probs * row, fp32
    t, e, h = 50, 16, 40
    rm = torch.zeros(t, e, dtype=torch.bool)
    sel = torch.argsort(torch.rand(t, e, generator=g), dim=1)[:, :4]
    rm.scatter_(1, sel, True)
    mask = rm.long()
    within = torch.cumsum(mask, 0) - 1
    cnt = mask.sum(0)
    off = torch.cumsum(cnt, 0) - cnt
    row = torch.where(mask > 0, within + off[None], torch.full_like(within, -1))
    r = int(rm.sum())
    pin = torch.randn(r, h, generator=g).to(torch.bfloat16)
    probs = torch.rand(t, e, generator=g) * rm
    acc = torch.zeros(t, h)
    for ee in range(e):
        m = row[:, ee] >= 0
        acc[m] = acc[m] + probs[m, ee][:, None] * pin[row[m, ee]].float()
    out.update(w_map_et=row.t().contiguous().numpy(), w_pin=bits(pin), w_probs=probs.numpy(),
               w_acc=acc.numpy(), w_out=bits(acc.to(torch.bfloat16)))
    save("router_combine.npz", **out)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=True, type=Path)
    args = ap.parse_args()
    torch.set_num_threads(8)
    gen_case12(args.reference_root)
    gen_case17(args.reference_root)
    gen_case15(args.reference_root)
    gen_kats(args.reference_root)
    gen_case23(args.reference_root)
    gen_gemm(args.reference_root)
    gen_router_combine()
    gen_permute_bwd(args.reference_root)


if __name__ == "__main__":
    main()
