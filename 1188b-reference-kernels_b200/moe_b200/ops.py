"""Torch-facing wrappers of the C ABI: one function per hot-path operator.

Each wrapper validates shapes and dtypes, allocates outputs with torch (the
caller's device and current stream), and calls the sm_100a kernel through
``_lib.call``. Inputs must be CUDA tensors: there is no CPU path.

Reference interfaces mirrored (kernel_results/<case>/binding.cpp):
  topk            <- case23_aten_topk/binding.cpp:6-26 (topk_forward)
  row_id_map      <- case12_moe_row_id_map_pass2/binding.cpp:13-36
  permute         <- case17_moe_permute_with_mask_map/binding.cpp:8-32
  unpermute       <- case15_moe_unpermute_mask_fwd/binding.cpp:11-22
"""
from __future__ import annotations

from ctypes import byref, c_int32, c_size_t
from typing import NamedTuple, Optional, Sequence, Union

import torch

from . import _lib

__all__ = [
    "topk", "router_topk", "RouterOutput", "row_id_map", "RowIdMap", "permute",
    "permute_trans", "permute_device_error", "unpermute", "unpermute_weighted", "grouped_gemm", "GroupedGemmPlan",
    "grouped_wgrad", "grouped_wgrad_device_error", "swiglu", "router_logits", "router_gemm_topk", "router_gemm_fusable",
    "router_device_error", "permute_backward", "combine_backward", "swiglu_backward",
]


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _need_cuda(name: str, t: Optional[torch.Tensor]) -> None:
    if t is not None and not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the MoE B200 ops have no CPU path)")


def _need_dtype(name: str, t: torch.Tensor, *dtypes: torch.dtype) -> None:
    if t.dtype not in dtypes:
        raise ValueError(f"{name} must be {' or '.join(map(str, dtypes))}, got {t.dtype}")


def _workspace(nbytes: int, dev: torch.device) -> torch.Tensor:
    # The caching allocator returns blocks aligned to at least 512 bytes.
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)


# --------------------------------------------------------------------------- a1
def topk(input: torch.Tensor, k: int = 8):
    """Row-wise top-k (largest, sorted, ties -> lower index) of fp32 [M,N].

    Same contract as kernel_cases/case23_ref_aten_topk.py:47-62 (reference_topk).
    Returns (values fp32 [M,k], indices int64 [M,k]).
    """
    _need_cuda("input", input)
    _need_dtype("input", input, torch.float32)
    if input.dim() != 2:
        raise ValueError(f"expected 2D input, got {input.dim()}D")
    x = input.contiguous()
    m, n = x.shape
    values = torch.empty((m, k), dtype=torch.float32, device=x.device)
    indices = torch.empty((m, k), dtype=torch.int64, device=x.device)
    _lib.call("moe_topk_f32", _p(x), _p(values), _p(indices), m, n, int(k), _stream(x.device))
    return values, indices


class RouterOutput(NamedTuple):
    topk_vals: torch.Tensor    # [T,k] fp32 gate weights in selection order
    topk_idx: torch.Tensor     # [T,k] int64 expert ids
    routing_map: torch.Tensor  # [T,E] bool
    probs: torch.Tensor        # [T,E] fp32, gate at routed pairs, 0 elsewhere


def router_topk(logits: torch.Tensor, k: int, score: str = "softmax", renorm: bool = True,
                bias: Optional[torch.Tensor] = None, outputs: str = "all",
                placement: Optional[torch.Tensor] = None) -> RouterOutput:
    """Fused router: (logits + bias) -> top-k -> gates -> routing map + probs.

    score="softmax": gates are softmax probabilities (renormalised over the k
    selected experts when renorm). score="logits": gates are the raw logits
    (case23 semantics). The selection follows the logits, which orders the
    experts exactly as their softmax probabilities do.
    outputs="all" or "maps" (skip topk_vals/topk_idx).
    placement (int32 [E] permutation on the device): output column c is
    model expert placement[c] (see moe_router_topk_placed).
    """
    _need_cuda("logits", logits)
    _need_dtype("logits", logits, torch.float32)
    if logits.dim() != 2:
        raise ValueError("logits must be [T,E]")
    if score not in ("softmax", "logits"):
        raise ValueError("score must be 'softmax' or 'logits'")
    lg = logits.contiguous()
    t, e = lg.shape
    dev = lg.device
    if bias is not None:
        _need_cuda("bias", bias)
        _need_dtype("bias", bias, torch.float32)
        if bias.shape != (e,):
            raise ValueError(f"bias must be [{e}]")
        bias = bias.contiguous()
    tv = ti = None
    if outputs == "all":
        tv = torch.empty((t, k), dtype=torch.float32, device=dev)
        ti = torch.empty((t, k), dtype=torch.int64, device=dev)
    rmap = torch.empty((t, e), dtype=torch.bool, device=dev)
    probs = torch.empty((t, e), dtype=torch.float32, device=dev)
    if placement is None:
        _lib.call("moe_router_topk", _p(lg), _p(bias), t, e, int(k),
                  1 if score == "softmax" else 0, 1 if renorm else 0, _p(tv), _p(ti), _p(rmap),
                  _p(probs), _stream(dev))
    else:
        _need_cuda("placement", placement)
        _need_dtype("placement", placement, torch.int32)
        if placement.shape != (e,):
            raise ValueError(f"placement must be [{e}]")
        pl = placement.contiguous()
        _lib.call("moe_router_topk_placed", _p(lg), _p(bias), _p(pl), t, e, int(k),
                  1 if score == "softmax" else 0, 1 if renorm else 0, _p(tv), _p(ti), _p(rmap),
                  _p(probs), _stream(dev))
    return RouterOutput(tv, ti, rmap, probs)


# --------------------------------------------------------------------------- a3
class RowIdMap(NamedTuple):
    map_et: Optional[torch.Tensor]  # [E,T] int64
    map_te: Optional[torch.Tensor]  # [T,E] int64
    counts: torch.Tensor            # [E] int32 tokens per expert
    num_out: torch.Tensor           # [1] int64 total (padded) rows, on device


def row_id_map(routing_map: torch.Tensor, align: int = 1, want_et: bool = True,
               want_te: bool = True) -> RowIdMap:
    """routing_map [T,E] bool -> expert-major row-id maps (both layouts).

    align=1 reproduces kernel_cases/case12_moe_row_id_map_pass2.py:43-50
    exactly; align>1 starts every expert segment on a multiple of align.
    """
    _need_cuda("routing_map", routing_map)
    _need_dtype("routing_map", routing_map, torch.bool, torch.uint8)
    if routing_map.dim() != 2:
        raise ValueError("routing_map must be [T,E]")
    rm = routing_map.contiguous()
    t, e = rm.shape
    dev = rm.device
    ws_bytes = c_size_t(0)
    _lib.call("moe_row_id_map_workspace_size", t, e, byref(ws_bytes))
    ws = _workspace(ws_bytes.value, dev)
    map_et = torch.empty((e, t), dtype=torch.int64, device=dev) if want_et else None
    map_te = torch.empty((t, e), dtype=torch.int64, device=dev) if want_te else None
    counts = torch.empty((e,), dtype=torch.int32, device=dev)
    num_out = torch.empty((1,), dtype=torch.int64, device=dev)
    _lib.call("moe_row_id_map", _p(rm), t, e, int(align), _p(map_et), _p(map_te), _p(counts),
              _p(num_out), _p(ws), ws_bytes.value, _stream(dev))
    return RowIdMap(map_et, map_te, counts, num_out)


# --------------------------------------------------------------------------- a4/a5
def _map_stats(row_id_map: torch.Tensor):
    """(max+1, number of valid entries) with one device->host sync."""
    valid = row_id_map >= 0
    stats = torch.stack([row_id_map.max().to(torch.int64) + 1, valid.sum().to(torch.int64)])
    r, n = (int(v) for v in stats.cpu())
    return max(r, 0), n


def _permute_outputs(x, probs, num_out, dense):
    alloc = torch.empty if dense else torch.zeros
    out = alloc((num_out, x.shape[1]), dtype=x.dtype, device=x.device)
    pp = None
    if probs is not None:
        pp = alloc((num_out,), dtype=torch.float32, device=x.device)
    return out, pp


def permute(x: torch.Tensor, row_id_map: torch.Tensor, probs: Optional[torch.Tensor] = None,
            num_out: Optional[int] = None, experts: Optional[torch.Tensor] = None):
    """out[row_id_map[t,e]] = x[t]; permuted_probs[row_id_map[t,e]] = probs[t,e].

    row_id_map is the token-major [T,E] int64 map (case17). When num_out is
    None it is max(row_id_map)+1, found with one host sync as the reference
    binding does (kernel_results/case17_moe_permute_with_mask_map/binding.cpp:24).
    experts (optional [T,k] int64, e.g. RouterOutput.topk_idx): the experts of
    each token; the kernel then reads only those k map entries per token
    (moe_permute_topk), with the same result.
    Returns (out [num_out,H], permuted_probs [num_out] or None).
    """
    for n_, t_ in (("x", x), ("row_id_map", row_id_map), ("probs", probs)):
        _need_cuda(n_, t_)
    if x.dim() != 2 or row_id_map.dim() != 2 or row_id_map.shape[0] != x.shape[0]:
        raise ValueError(f"shapes x {tuple(x.shape)} row_id_map {tuple(row_id_map.shape)}")
    if x.element_size() != 2:
        raise ValueError("x must be a 2-byte type (bf16/fp16)")
    _need_dtype("row_id_map", row_id_map, torch.int64)
    t, e = row_id_map.shape
    xc = x.contiguous()
    mc = row_id_map.contiguous()
    pc = None
    if probs is not None:
        if probs.shape != (t, e):
            raise ValueError(f"probs {tuple(probs.shape)} expected {(t, e)}")
        pc = probs.contiguous().to(torch.float32)
    dense = True
    if num_out is None:
        num_out, nvalid = _map_stats(mc) if mc.numel() else (0, 0)
        dense = nvalid >= num_out
    out, pp = _permute_outputs(xc, pc, int(num_out), dense)
    if experts is not None and xc.shape[1] % 8 == 0 and (xc.data_ptr() | out.data_ptr()) % 16 == 0:
        _need_cuda("experts", experts)
        _need_dtype("experts", experts, torch.int64)
        if experts.dim() != 2 or experts.shape[0] != t:
            raise ValueError(f"experts must be [{t},k]")
        ec = experts.contiguous()
        _lib.call("moe_permute_topk", _p(xc), _p(mc), _p(ec), ec.shape[1], _p(pc), _p(out),
                  _p(pp), t, xc.shape[1], e, int(num_out), _stream(xc.device))
        return out, pp
    _lib.call("moe_permute_mask_map", _p(xc), _p(mc), _p(pc), _p(out), _p(pp), t, xc.shape[1], e,
              int(num_out), _stream(xc.device))
    return out, pp


def permute_device_error(device) -> int:
    """Error word of the bulk-copy permute on this device (0: none, 1: a row
    load timed out), cleared after reading. Synchronises the current stream."""
    dev = torch.device(device)
    if dev.index is None:
        dev = torch.device(dev.type, torch.cuda.current_device())
    v = c_int32(0)
    with torch.cuda.device(dev):
        _lib.load().moe_permute_check(_stream(dev), byref(v))
    return int(v.value)


def permute_trans(x: torch.Tensor, row_id_map: torch.Tensor, probs: Optional[torch.Tensor] = None,
                  num_out: Optional[int] = None):
    """Permute with the expert-major [E,T] map (int64 or int32), case22/21/30."""
    for n_, t_ in (("x", x), ("row_id_map", row_id_map), ("probs", probs)):
        _need_cuda(n_, t_)
    if row_id_map.dim() != 2 or x.dim() != 2 or row_id_map.shape[1] != x.shape[0]:
        raise ValueError(f"shapes inp {tuple(x.shape)} row_id_map {tuple(row_id_map.shape)}")
    if x.element_size() != 2:
        raise ValueError("x must be a 2-byte type (bf16/fp16)")
    _need_dtype("row_id_map", row_id_map, torch.int64, torch.int32)
    e, t = row_id_map.shape
    xc = x.contiguous()
    mc = row_id_map.contiguous()
    pc = None
    if probs is not None:
        if probs.shape != (t, e):
            raise ValueError(f"probs {tuple(probs.shape)} expected {(t, e)}")
        pc = probs.contiguous().to(torch.float32)
    dense = True
    if num_out is None:
        num_out, nvalid = _map_stats(mc) if mc.numel() else (0, 0)
        dense = nvalid >= num_out
    out, pp = _permute_outputs(xc, pc, int(num_out), dense)
    bits = 64 if mc.dtype == torch.int64 else 32
    _lib.call("moe_permute_mask_map_trans", _p(xc), _p(mc), bits, _p(pc), _p(out), _p(pp), t,
              xc.shape[1], e, int(num_out), _stream(xc.device))
    return out, pp


# --------------------------------------------------------------------------- a6-a8
def unpermute(pin: torch.Tensor, row_id_map: torch.Tensor, probs: Optional[torch.Tensor] = None,
              probs_mode: str = "dense", return_acc: bool = False, token_major: bool = False):
    """out[t] = bf16(sum over e ascending of w * pin[row_id_map[e,t]]), fp32 accumulation.

    w = 1 without probs (case15 / case24); w = probs[t,e] for probs_mode
    "dense" ([T,E]); w = probs[row] for probs_mode "permuted" ([rows]).
    token_major=True takes the [T,E] int64 map instead of [E,T] (same result).
    Returns out (and the fp32 accumulator when return_acc).
    """
    for n_, t_ in (("pin", pin), ("row_id_map", row_id_map), ("probs", probs)):
        _need_cuda(n_, t_)
    if row_id_map.dim() != 2 or pin.dim() != 2:
        raise ValueError(f"shapes pin {tuple(pin.shape)} row_id_map {tuple(row_id_map.shape)}")
    _need_dtype("pin", pin, torch.bfloat16)
    _need_dtype("row_id_map", row_id_map, torch.int64, torch.int32)
    if token_major:
        _need_dtype("row_id_map", row_id_map, torch.int64)
        t, e = row_id_map.shape
    else:
        e, t = row_id_map.shape
    pc = pin.contiguous()
    mc = row_id_map.contiguous()
    mode = -1
    prc = None
    if probs is not None:
        prc = probs.contiguous().to(torch.float32)
        if probs_mode == "dense":
            if prc.shape != (t, e):
                raise ValueError(f"probs {tuple(prc.shape)} expected {(t, e)}")
            mode = 0
        elif probs_mode == "permuted":
            if prc.shape != (pc.shape[0],):
                raise ValueError(f"permuted probs must be [{pc.shape[0]}]")
            mode = 1
        else:
            raise ValueError("probs_mode must be 'dense' or 'permuted'")
    out = torch.empty((t, pc.shape[1]), dtype=pc.dtype, device=pc.device)
    acc = torch.empty((t, pc.shape[1]), dtype=torch.float32, device=pc.device) if return_acc else None
    if token_major:
        _lib.call("moe_unpermute_mask_token_major", _p(pc), _p(mc), _p(prc),
                  mode if mode >= 0 else 0, _p(out), _p(acc), t, pc.shape[1], e, pc.shape[0],
                  _stream(pc.device))
    else:
        bits = 64 if mc.dtype == torch.int64 else 32
        _lib.call("moe_unpermute_mask", _p(pc), _p(mc), bits, _p(prc), mode if mode >= 0 else 0,
                  _p(out), _p(acc), t, pc.shape[1], e, pc.shape[0], _stream(pc.device))
    return (out, acc) if return_acc else out


# --------------------------------------------------------------------------- a9-a11
class GroupedGemmPlan:
    """Device-side group table for moe_grouped_gemm (reusable across calls)."""

    def __init__(self, num_groups: int, device: torch.device):
        self.num_groups = int(num_groups)
        nb = c_size_t(0)
        _lib.call("moe_grouped_gemm_workspace_size", self.num_groups, byref(nb))
        self.nbytes = nb.value
        self.workspace = _workspace(self.nbytes, device)
        self.workspace[:256].zero_()  # error word reads 0 before the first plan
        self.device = device

    def from_splits(self, m_splits: torch.Tensor, align: int = 1) -> "GroupedGemmPlan":
        ms = m_splits.to(device=self.device, dtype=torch.int32).contiguous()
        if ms.numel() != self.num_groups:
            raise ValueError(f"m_splits has {ms.numel()} entries, plan has {self.num_groups}")
        self._keep = ms
        _lib.call("moe_grouped_gemm_plan_splits", _p(ms), self.num_groups, int(align),
                  _p(self.workspace), self.nbytes, _stream(self.device))
        return self

    def from_ep_counts(self, counts: torch.Tensor, num_src: int, num_w: int) -> "GroupedGemmPlan":
        c = counts.to(device=self.device, dtype=torch.int32).contiguous()
        if c.numel() != num_src * num_w or num_src * num_w != self.num_groups:
            raise ValueError("counts must be [num_src * num_w]")
        self._keep = c
        _lib.call("moe_grouped_gemm_plan_ep", _p(c), int(num_src), int(num_w),
                  _p(self.workspace), self.nbytes, _stream(self.device))
        return self

    def device_error(self) -> int:
        v = c_int32(0)
        lib = _lib.load()
        lib.moe_grouped_gemm_check(_p(self.workspace), self.nbytes, _stream(self.device), byref(v))
        return int(v.value)


def grouped_gemm(x: torch.Tensor, w: torch.Tensor,
                 m_splits: Union[None, Sequence[int], torch.Tensor] = None,
                 epilogue: str = "none", align: int = 1,
                 plan: Optional[GroupedGemmPlan] = None,
                 out: Optional[torch.Tensor] = None, w_layout: str = "NK") -> torch.Tensor:
    """out = cat_g(x[seg_g] @ w[g].T) on tcgen05 tensor cores (bf16, fp32 accumulate).

    x [rows,K] bf16, w [G,N,K] bf16 ("[out,in]" as in case03/case04). With
    epilogue="swiglu", w holds [gate|up] (N=2F) and the result is
    silu(gate)*up, [rows,F]; with epilogue="fp32" the result is the fp32
    accumulator, [rows,N] float32. m_splits defaults to the uniform split of
    kernel_cases/case03_moe_grouped_gemm_fc1_fwd.py:43-46. A prebuilt plan
    (device group table) skips the planning launch.

    w_layout="KN": w is [G,K,N] and out = cat_g(x[seg_g] @ w[g]) — the
    grouped dgrad dx = dy @ W of kernel_cases/case07/08_moe_grouped_gemm_fc*_
    dgrad.py:49-64 (case13/19 with one group), with the forward weight tensor
    as it is; the weight operand is staged MN-major (no transposed copy).
    """
    for n_, t_ in (("x", x), ("w", w)):
        _need_cuda(n_, t_)
        _need_dtype(n_, t_, torch.bfloat16)
    if w_layout not in ("NK", "KN"):
        raise ValueError("w_layout must be 'NK' (w [G,N,K]) or 'KN' (w [G,K,N])")
    kdim = 2 if w_layout == "NK" else 1
    if x.dim() != 2 or w.dim() != 3 or x.shape[1] != w.shape[kdim]:
        raise ValueError(f"shapes x {tuple(x.shape)} w {tuple(w.shape)} ({w_layout})")
    if w_layout == "KN" and epilogue == "swiglu":
        raise ValueError("the SwiGLU epilogue needs w_layout 'NK'")
    codes = {"none": 0, "swiglu": 1, "fp32": 2}
    if epilogue not in codes:
        raise ValueError("epilogue must be 'none', 'swiglu' or 'fp32'")
    xc = x.contiguous()
    wc = w.contiguous()
    rows, k = xc.shape
    g = wc.shape[0]
    n = wc.shape[1] if w_layout == "NK" else wc.shape[2]
    dev = xc.device
    if plan is None:
        if m_splits is None:
            base, rem = divmod(rows, g)
            m_splits = [base + (1 if i < rem else 0) for i in range(g)]
        if isinstance(m_splits, torch.Tensor):
            ms = m_splits
        else:
            if len(m_splits) != g:
                raise ValueError(f"m_splits has {len(m_splits)} entries for {g} groups")
            if align == 1 and sum(int(v) for v in m_splits) > rows:
                raise ValueError("sum(m_splits) exceeds x rows")
            ms = torch.tensor([int(v) for v in m_splits], dtype=torch.int32)
        plan = GroupedGemmPlan(g, dev).from_splits(ms, align)
    n_out = n // 2 if epilogue == "swiglu" else n
    odt = torch.float32 if epilogue == "fp32" else torch.bfloat16
    if out is None:
        out = torch.empty((rows, n_out), dtype=odt, device=dev)
    elif out.dtype != odt or tuple(out.shape) != (rows, n_out) or not out.is_contiguous() \
            or out.device != dev:
        raise ValueError(f"out must be a contiguous {odt} [{rows},{n_out}] tensor on {dev}")
    _lib.call("moe_grouped_gemm" if w_layout == "NK" else "moe_grouped_gemm_nn", _p(xc), _p(wc),
              _p(out), rows, plan.num_groups, g, n, k, codes[epilogue], _p(plan.workspace),
              plan.nbytes, _stream(dev))
    return out


def unpermute_weighted(pin: torch.Tensor, row_id_map: torch.Tensor,
                       probs: torch.Tensor) -> torch.Tensor:
    """Prob-weighted combine: out[t] = bf16(sum over e ascending of
    probs[t,e] * fp32(pin[row_id_map[e,t]])), probs dense [T,E] fp32 — the
    unweighted unpermute of kernel_cases/case15_moe_unpermute_mask_fwd.py:
    58-64 with each source row scaled by its gate (no reference code)."""
    return unpermute(pin, row_id_map, probs, probs_mode="dense")


def permute_backward(grad_permuted: torch.Tensor, row_id_map: torch.Tensor,
                     permuted_probs_grad: Optional[torch.Tensor] = None,
                     return_acc: bool = False):
    """Backward of the permute with an [E,T] map (int64 or int32).

    grad_x[t] = bf16(sum over e ascending of fp32(grad_permuted[row_id_map[e,t]]))
    and, with permuted_probs_grad [rows] fp32, grad_probs[t,e] =
    permuted_probs_grad[row_id_map[e,t]] for a routed (t,e), else 0 —
    kernel_cases/case18_moe_permute_bwd_unpermute_mask.py:56-70 (int64 map)
    and case32_ref_moe_unpermute_mask_kernel.py:47-79 (int32 map, which also
    returns the fp32 sums). One kernel: the unweighted combine that also
    gathers the prob gradient while it reads the map.

    Returns (grad_x, grad_probs), with the fp32 sums first when return_acc:
    (acc, grad_x, grad_probs); grad_probs is None without permuted_probs_grad.
    """
    for n_, t_ in (("grad_permuted", grad_permuted), ("row_id_map", row_id_map),
                   ("permuted_probs_grad", permuted_probs_grad)):
        _need_cuda(n_, t_)
    if row_id_map.dim() != 2 or grad_permuted.dim() != 2:
        raise ValueError(f"shapes grad_permuted {tuple(grad_permuted.shape)} "
                         f"row_id_map {tuple(row_id_map.shape)}")
    _need_dtype("grad_permuted", grad_permuted, torch.bfloat16)
    _need_dtype("row_id_map", row_id_map, torch.int64, torch.int32)
    e, t = row_id_map.shape
    gc = grad_permuted.contiguous()
    mc = row_id_map.contiguous()
    rows, h = gc.shape
    pg = None
    gp = None
    if permuted_probs_grad is not None:
        _need_dtype("permuted_probs_grad", permuted_probs_grad, torch.float32)
        if permuted_probs_grad.shape != (rows,):
            raise ValueError(f"permuted_probs_grad must be [{rows}]")
        pg = permuted_probs_grad.contiguous()
        gp = torch.empty((t, e), dtype=torch.float32, device=gc.device)
    gx = torch.empty((t, h), dtype=gc.dtype, device=gc.device)
    acc = torch.empty((t, h), dtype=torch.float32, device=gc.device) if return_acc else None
    _lib.call("moe_permute_backward", _p(gc), _p(mc), 64 if mc.dtype == torch.int64 else 32,
              _p(pg), _p(gx), _p(acc), _p(gp), t, h, e, rows, _stream(gc.device))
    return (acc, gx, gp) if return_acc else (gx, gp)


def combine_backward(grad_out: torch.Tensor, rows: torch.Tensor, row_id_map: torch.Tensor,
                     probs: torch.Tensor):
    """Backward of the prob-weighted combine out[t] = sum_e probs[t,e] *
    rows[row_id_map[t,e]] (token-major [T,E] int64 map, dense probs [T,E]):
    grad_rows[row_id_map[t,e]] = bf16(probs[t,e] * grad_out[t]) and
    grad_probs[t,e] = <grad_out[t], rows[row_id_map[t,e]]> (fp32), 0 where the
    token is not routed. Returns (grad_rows [R,H] bf16, grad_probs [T,E] fp32).
    Rows no token references stay uninitialised."""
    for n_, t_ in (("grad_out", grad_out), ("rows", rows), ("row_id_map", row_id_map),
                   ("probs", probs)):
        _need_cuda(n_, t_)
    _need_dtype("grad_out", grad_out, torch.bfloat16)
    _need_dtype("rows", rows, torch.bfloat16)
    _need_dtype("row_id_map", row_id_map, torch.int64)
    _need_dtype("probs", probs, torch.float32)
    if grad_out.dim() != 2 or rows.dim() != 2 or rows.shape[1] != grad_out.shape[1]:
        raise ValueError(f"shapes grad_out {tuple(grad_out.shape)} rows {tuple(rows.shape)}")
    t, h = grad_out.shape
    if row_id_map.shape[0] != t or probs.shape != row_id_map.shape:
        raise ValueError("row_id_map and probs must both be [T,E]")
    e = row_id_map.shape[1]
    go, rc, mc, pc = (v.contiguous() for v in (grad_out, rows, row_id_map, probs))
    grad_rows = torch.empty_like(rc)
    grad_probs = torch.empty((t, e), dtype=torch.float32, device=go.device)
    _lib.call("moe_combine_backward", _p(go), _p(rc), _p(mc), _p(pc), _p(grad_rows),
              _p(grad_probs), t, h, e, rc.shape[0], _stream(go.device))
    return grad_rows, grad_probs


def swiglu_backward(y: torch.Tensor, dh: torch.Tensor) -> torch.Tensor:
    """Backward of h = silu(g) * u for y = [g | u] [M,2F] bf16 and dh [M,F]
    bf16: returns dy = [dh * u * silu'(g) | dh * silu(g)] [M,2F] bf16."""
    _need_cuda("y", y)
    _need_cuda("dh", dh)
    _need_dtype("y", y, torch.bfloat16)
    _need_dtype("dh", dh, torch.bfloat16)
    if y.dim() != 2 or dh.dim() != 2 or y.shape[0] != dh.shape[0] or y.shape[1] != 2 * dh.shape[1]:
        raise ValueError(f"shapes y {tuple(y.shape)} dh {tuple(dh.shape)}")
    yc, dc = y.contiguous(), dh.contiguous()
    dy = torch.empty_like(yc)
    _lib.call("moe_swiglu_backward", _p(yc), _p(dc), _p(dy), yc.shape[0], dc.shape[1],
              _stream(yc.device))
    return dy


def grouped_wgrad(dy: torch.Tensor, x: torch.Tensor,
                  m_splits: Union[Sequence[int], torch.Tensor],
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dW[g] = dy[seg_g]^T @ x[seg_g] on tcgen05 tensor cores, [G,N,K] bf16.

    dy [rows,N] and x [rows,K] bf16 (the forward's output gradient and input,
    groups contiguous in order), fp32 accumulation; an empty group gives
    zeros. The torch.mm(dy[seg].t(), x[seg]) loop of kernel_cases/
    case05_moe_grouped_gemm_fc2_wgrad.py:49-64 / case09_moe_grouped_gemm_fc1_
    wgrad.py:49-64. m_splits: a CUDA int tensor (e.g. the expert counts of
    row_id_map; used where it is, no host sync) or host counts (G <= 4096).
    The group table and per-group tensor maps are built on the device.
    """
    for n_, t_ in (("dy", dy), ("x", x)):
        _need_cuda(n_, t_)
        _need_dtype(n_, t_, torch.bfloat16)
    if dy.dim() != 2 or x.dim() != 2 or dy.shape[0] != x.shape[0]:
        raise ValueError(f"shapes dy {tuple(dy.shape)} x {tuple(x.shape)}")
    on_dev = isinstance(m_splits, torch.Tensor) and m_splits.is_cuda
    if on_dev:
        ms = m_splits.to(dtype=torch.int32).contiguous()
        if ms.dim() != 1 or ms.numel() == 0 or ms.device != dy.device:
            raise ValueError("device m_splits must be a 1-D tensor on dy's device")
        g = ms.numel()
    else:
        if isinstance(m_splits, torch.Tensor):
            m_splits = m_splits.tolist()
        splits = [int(v) for v in m_splits]
        if any(v < 0 for v in splits) or sum(splits) > dy.shape[0] or not splits:
            raise ValueError("m_splits must be >= 0 and sum to at most the rows")
        g = len(splits)
    dyc, xc = dy.contiguous(), x.contiguous()
    n, k = dyc.shape[1], xc.shape[1]
    dev = dyc.device
    if out is None:
        out = torch.empty((g, n, k), dtype=torch.bfloat16, device=dev)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (g, n, k) or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous bf16 [{g},{n},{k}] tensor")
    nb = c_size_t(0)
    _lib.call("moe_grouped_wgrad_workspace_size", g, byref(nb))
    ws = _workspace(nb.value, dev)
    if on_dev:
        _lib.call("moe_grouped_wgrad_dev", _p(dyc), _p(xc), _p(out), dyc.shape[0], g, n, k,
                  _p(ms), _p(ws), nb.value, _stream(dev))
    else:
        host = (c_int32 * g)(*splits)
        _lib.call("moe_grouped_wgrad", _p(dyc), _p(xc), _p(out), dyc.shape[0], g, n, k, host,
                  _p(ws), nb.value, _stream(dev))
    _WGRAD_ERR[dev] = ws  # the error word of the last call on this device
    return out  # ws returns to torch's allocator, reused only after this stream's work


# Workspace of the last grouped_wgrad per device (its first word is the
# device error word, see grouped_wgrad_device_error).
_WGRAD_ERR: dict = {}


def grouped_wgrad_device_error(device) -> int:
    """Error code the last grouped_wgrad on this device left (0: none;
    4: a negative count or counts summing past the rows). Syncs."""
    dev = torch.device(device)
    if dev.index is None:
        dev = torch.device(dev.type, torch.cuda.current_device())
    ws = _WGRAD_ERR.get(dev)
    if ws is None:
        return 0
    v = c_int32(0)
    _lib.load().moe_grouped_gemm_check(_p(ws), ws.numel(), _stream(dev), byref(v))
    return int(v.value)


def router_logits(x: torch.Tensor, weight: torch.Tensor,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Router gate GEMM: logits [T,E] fp32 = x [T,H] bf16 @ weight [E,H] bf16 ^T,
    accumulated in fp32 on the tensor cores and stored unrounded.

    Replaces kernel_cases/case38_ref_musa_asm_bf16_ssgemm_nt_320x256.py:51-59
    (reference_fp32, the TN muDNN GEMM of Megatron's router gate). It is the
    grouped GEMM with one group and the fp32 epilogue.
    """
    for n_, t_ in (("x", x), ("weight", weight)):
        _need_cuda(n_, t_)
        _need_dtype(n_, t_, torch.bfloat16)
    if x.dim() != 2 or weight.dim() != 2 or x.shape[1] != weight.shape[1]:
        raise ValueError(f"shapes x {tuple(x.shape)} weight {tuple(weight.shape)}")
    key = (x.device, x.shape[0])
    plan = _ROUTER_PLANS.get(key)
    if plan is None:
        if len(_ROUTER_PLANS) >= 64:
            _ROUTER_PLANS.clear()
        plan = GroupedGemmPlan(1, x.device).from_splits(torch.tensor([x.shape[0]], dtype=torch.int32))
        torch.cuda.current_stream(x.device).synchronize()  # table ready for every stream
        _ROUTER_PLANS[key] = plan
    return grouped_gemm(x, weight.unsqueeze(0), epilogue="fp32", plan=plan, out=out)


# One-group plans of router_logits, by (device, rows): the table depends only
# on the row count, so repeated calls skip the planning launch.
_ROUTER_PLANS: dict = {}

# Device error words of router_gemm_topk, one zeroed int32 per device.
_ROUTER_ERR: dict = {}


def _router_err(dev: torch.device) -> torch.Tensor:
    if dev.index is None:
        dev = torch.device(dev.type, torch.cuda.current_device())
    e = _ROUTER_ERR.get(dev)
    if e is None:
        e = torch.zeros(1, dtype=torch.int32, device=dev)
        _ROUTER_ERR[dev] = e
    return e


def router_device_error(device) -> int:
    """Error code left by router_gemm_topk on this device (0: none). Syncs."""
    dev = torch.device(device)
    if dev.index is None:
        dev = torch.device(dev.type, torch.cuda.current_device())
    e = _ROUTER_ERR.get(dev)
    return 0 if e is None else int(e.item())


def router_gemm_fusable(x: torch.Tensor, weight: torch.Tensor, k: int) -> bool:
    """Whether router_gemm_topk covers this shape (E a multiple of 32 up to
    512, H a multiple of 8, k <= min(E, 16))."""
    e, h = weight.shape[0], weight.shape[1]
    return e % 32 == 0 and 32 <= e <= 512 and h % 8 == 0 and 1 <= k <= min(e, 16)


def router_gemm_topk(x: torch.Tensor, weight: torch.Tensor, k: int, score: str = "softmax",
                     renorm: bool = True, bias: Optional[torch.Tensor] = None,
                     outputs: str = "maps", return_logits: bool = False):
    """Router gate GEMM and router in one kernel: logits = x @ weight^T (fp32
    accumulation on the tensor cores), then router_topk(logits, k, score,
    renorm, bias) without the logits round trip through HBM; the routing
    outputs are bit-identical to router_topk on the same logits.

    Replaces kernel_cases/case38_ref_musa_asm_bf16_ssgemm_nt_320x256.py:51-59
    followed by the softmax/top-k router. x [T,H] bf16, weight [E,H] bf16.
    outputs="maps" (routing map + probs), "all" (+ topk_vals/topk_idx) or
    "none" (only the logits, which then must be requested).
    Returns RouterOutput, or (RouterOutput, logits) with return_logits.
    """
    for n_, t_ in (("x", x), ("weight", weight)):
        _need_cuda(n_, t_)
        _need_dtype(n_, t_, torch.bfloat16)
    if x.dim() != 2 or weight.dim() != 2 or x.shape[1] != weight.shape[1]:
        raise ValueError(f"shapes x {tuple(x.shape)} weight {tuple(weight.shape)}")
    if score not in ("softmax", "logits"):
        raise ValueError("score must be 'softmax' or 'logits'")
    if outputs not in ("maps", "all", "none"):
        raise ValueError("outputs must be 'maps', 'all' or 'none'")
    if outputs == "none" and not return_logits:
        raise ValueError("outputs='none' needs return_logits=True")
    xc, wc = x.contiguous(), weight.contiguous()
    t, e = xc.shape[0], wc.shape[0]
    dev = xc.device
    if bias is not None:
        _need_cuda("bias", bias)
        _need_dtype("bias", bias, torch.float32)
        if bias.shape != (e,):
            raise ValueError(f"bias must be [{e}]")
        bias = bias.contiguous()
    tv = ti = rmap = probs = None
    if outputs == "all":
        tv = torch.empty((t, k), dtype=torch.float32, device=dev)
        ti = torch.empty((t, k), dtype=torch.int64, device=dev)
    if outputs in ("all", "maps"):
        rmap = torch.empty((t, e), dtype=torch.bool, device=dev)
        probs = torch.empty((t, e), dtype=torch.float32, device=dev)
    logits = torch.empty((t, e), dtype=torch.float32, device=dev) if return_logits else None
    _lib.call("moe_router_gemm_topk", _p(xc), _p(wc), _p(bias), t, xc.shape[1], e, int(k),
              1 if score == "softmax" else 0, 1 if renorm else 0, _p(logits), _p(tv), _p(ti),
              _p(rmap), _p(probs), _p(_router_err(dev)), _stream(dev))
    r = RouterOutput(tv, ti, rmap, probs)
    return (r, logits) if return_logits else r


def swiglu(y: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """h = silu(y[:, :F]) * y[:, F:] for y [M,2F] bf16 (gate|up order);
    into `out` (contiguous bf16 [M,F]) when given."""
    _need_cuda("y", y)
    _need_dtype("y", y, torch.bfloat16)
    if y.dim() != 2 or y.shape[1] % 2:
        raise ValueError("y must be [M,2F]")
    yc = y.contiguous()
    m, f2 = yc.shape
    if out is None:
        h = torch.empty((m, f2 // 2), dtype=yc.dtype, device=yc.device)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (m, f2 // 2) or \
            not out.is_contiguous() or out.device != yc.device:
        raise ValueError(f"out must be a contiguous bf16 [{m},{f2 // 2}] tensor on {yc.device}")
    else:
        h = out
    _lib.call("moe_swiglu", _p(yc), _p(h), m, f2 // 2, _stream(yc.device))
    return h
