"""CPU oracle for the MoE expert-layer forward path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference algorithms of the hot path so
that the CUDA kernels can be checked against them. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it, and only as the checker or the timed CPU
baseline; the product (``1188b-reference-kernels_b200``) never calls it.

bf16 tensors are carried as uint16 bit patterns. Float arithmetic is fp32
with one IEEE rounding per operation, so the integer / copy paths and the
combine are bit-exact against the kernels; GEMM-based paths are compared
within the tolerance stated in each test.

Parity pins: every function here is checked against golden vectors produced
by the reference's own Python code (``tests/golden/make_golden.py``) in
``tests/test_oracle_golden.py``. The softmax/renormalisation router, the
weighted combine and SwiGLU have no reference implementation (they are named
but not computed by the reference); their restatements are pinned only by
torch fp32 equivalents in the same golden script.
"""
from __future__ import annotations

import numpy as np

# --------------------------------------------------------------------------- bf16


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN stays NaN).

    Same rounding as torch's float->bfloat16 cast; written from the IEEE
    definition (add half an ulp of the truncated format plus the tie bit).
    """
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16))
    r = r.astype(np.uint16)
    if nan.any():
        r = np.where(nan, ((u >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16), r)
    return r


# --------------------------------------------------------------------------- a1 top-k


def topk(inp: np.ndarray, k: int):
    """Row-wise top-k by a full stable descending sort, then the first k.

    kernel_cases/case23_ref_aten_topk.py:47-62 (reference_topk): values
    descending, equal values keep ascending column order; NaN ranks first
    (torch.sort descending order).
    """
    x = np.asarray(inp, dtype=np.float32)
    if x.ndim != 2:
        raise ValueError("expected 2D input")
    m, n = x.shape
    if not 1 <= k <= n:
        raise ValueError(f"k={k} out of range for N={n}")
    cols = np.broadcast_to(np.arange(n), x.shape)
    isnum = ~np.isnan(x)
    neg = np.where(isnum, -x, 0.0).astype(np.float32)
    order = np.lexsort((cols, neg, isnum), axis=-1)[:, :k]
    vals = np.take_along_axis(x, order, axis=1)
    return vals, order.astype(np.int64)


def router(logits: np.ndarray, k: int, bias: np.ndarray | None = None, score: str = "softmax",
           renorm: bool = True, placement: np.ndarray | None = None):
    """Router: softmax over experts, top-k, optional renormalisation.

    No reference function computes this (the reference's router case23 is the
    top-k alone, kernel_cases/case23_ref_aten_topk.py:47-62). Restated as
    p = softmax(l); selection = top-k order of l (softmax is monotone, so
    this is the top-k of p with ties broken by l); gates = p[sel] / sum.
    Returns (gates [T,k], idx [T,k], routing_map [T,E] bool, probs [T,E]).
    """
    lg = np.asarray(logits, dtype=np.float32)
    if bias is not None:
        lg = (lg + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    if placement is not None:  # slot c holds model expert placement[c]
        lg = np.ascontiguousarray(lg[:, np.asarray(placement)])
    _, idx = topk(lg, k)
    if score == "softmax":
        m = lg.max(axis=1, keepdims=True)
        ex = np.exp(lg - m, dtype=np.float32)
        p = ex / ex.sum(axis=1, keepdims=True, dtype=np.float32)
    else:
        p = lg
    gates = np.take_along_axis(p, idx, axis=1).astype(np.float32)
    if renorm:
        gates = (gates / gates.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    t, e = lg.shape
    rmap = np.zeros((t, e), dtype=bool)
    np.put_along_axis(rmap, idx, True, axis=1)
    probs = np.zeros((t, e), dtype=np.float32)
    np.put_along_axis(probs, idx, gates, axis=1)
    return gates, idx, rmap, probs


# --------------------------------------------------------------------------- a3 row_id_map


def row_id_map(routing_map: np.ndarray, align: int = 1):
    """routing_map [T,E] bool -> (row_id_map [E,T], row_id_map [T,E]) int64.

    kernel_cases/case12_moe_row_id_map_pass2.py:43-50 (make_row_id_map) and
    :53-61 (Model returns the transposed and the token-major map):
    row[t,e] = offset[e] + cumsum_t(mask[:,e]) - 1 where routed, else -1,
    offset = exclusive cumsum of per-expert counts (padded to `align`; the
    reference is align = 1).
    """
    mask = np.asarray(routing_map).astype(np.int64)
    within = np.cumsum(mask, axis=0) - 1
    counts = mask.sum(axis=0)
    padded = ((counts + align - 1) // align) * align
    offset = np.cumsum(padded) - padded
    row = np.where(mask > 0, within + offset[None, :], -1).astype(np.int64)
    return np.ascontiguousarray(row.T), row, counts.astype(np.int32), int(padded.sum())


# --------------------------------------------------------------------------- a4/a5 permute


def permute(x_u16: np.ndarray, row_te: np.ndarray, probs: np.ndarray | None, num_out: int):
    """out[row[t,e]] = x[t]; pp[row[t,e]] = probs[t,e] (zeros elsewhere).

    kernel_cases/case17_moe_permute_with_mask_map.py:58-71 (Model.forward).
    """
    row = np.asarray(row_te)
    t_idx, e_idx = np.nonzero(row >= 0)
    dst = row[t_idx, e_idx]
    out = np.zeros((num_out, x_u16.shape[1]), dtype=x_u16.dtype)
    out[dst] = x_u16[t_idx]
    pp = None
    if probs is not None:
        pp = np.zeros((num_out,), dtype=np.float32)
        pp[dst] = np.asarray(probs, dtype=np.float32)[t_idx, e_idx]
    return out, pp


def permute_trans(x_u16: np.ndarray, row_et: np.ndarray, probs: np.ndarray | None,
                  num_out: int | None = None):
    """Same scatter with the expert-major [E,T] map; num_out = max + 1.

    kernel_cases/case22_ref_moe_permute_mask_kernel_true.py:47-69 and the
    no-probs variants case21_ref_permute_with_mask_map_trans.py:52-68,
    case30_ref_moe_permute_mask_kernel.py:44-58.
    """
    row = np.asarray(row_et).astype(np.int64)
    e_idx, t_idx = np.nonzero(row >= 0)
    dst = row[e_idx, t_idx]
    if num_out is None:
        num_out = int(dst.max()) + 1 if dst.size else 0
    out = np.zeros((num_out, x_u16.shape[1]), dtype=x_u16.dtype)
    out[dst] = x_u16[t_idx]
    pp = None
    if probs is not None:
        pp = np.zeros((num_out,), dtype=np.float32)
        pp[dst] = np.asarray(probs, dtype=np.float32)[t_idx, e_idx]
    return out, pp


# --------------------------------------------------------------------------- a6-a8 unpermute


def unpermute(pin_u16: np.ndarray, row_et: np.ndarray, probs: np.ndarray | None = None,
              probs_mode: str = "dense", tokens: np.ndarray | None = None):
    """acc[t] = sum over e ascending of w * pin[row[e,t]] in fp32; out = bf16(acc).

    Unweighted: kernel_cases/case15_moe_unpermute_mask_fwd.py:58-64 (index_add_
    of rows ordered by nonzero() of the [E,T] map, i.e. ascending expert per
    token, into zeros) and case24_ref_moe_unpermute_mask_kernel_false.py:45-68.
    Weighted (no reference; the build's restatement): w = probs[t,e] (dense)
    or probs[row] (permuted), product and sum rounded separately in fp32.
    `tokens` restricts the computation to a subset of token ids.
    Returns (acc fp32 [T',H], out bf16 bits [T',H]).
    """
    row = np.asarray(row_et).astype(np.int64)
    e_n, t_n = row.shape
    if tokens is None:
        tokens = np.arange(t_n)
    sub = row[:, tokens]
    acc = np.zeros((len(tokens), pin_u16.shape[1]), dtype=np.float32)
    for e in range(e_n):
        src = sub[e]
        m = src >= 0
        if not m.any():
            continue
        xs = bf16_to_f32(pin_u16[src[m]])
        if probs is None:
            acc[m] = acc[m] + xs
        else:
            if probs_mode == "dense":
                w = np.asarray(probs, dtype=np.float32)[tokens[m], e]
            else:
                w = np.asarray(probs, dtype=np.float32)[src[m]]
            acc[m] = acc[m] + (w[:, None] * xs).astype(np.float32)
    return acc, f32_to_bf16(acc)


# --------------------------------------------------------------------------- a9-a11 GEMM


def permute_backward(grad_u16: np.ndarray, row_et: np.ndarray, pgrad: np.ndarray | None = None):
    """Backward of the permute with an [E,T] map: the unweighted unpermute of
    the row gradients and the prob gradient gathered onto [token, expert].

    kernel_cases/case18_moe_permute_bwd_unpermute_mask.py:56-70 (int64 map)
    and case32_ref_moe_unpermute_mask_kernel.py:47-79 (int32 map): acc[t] =
    sum over e ascending of fp32 rows, out = bf16(acc), grad_probs[t,e] =
    pgrad[row[e,t]] where routed, else 0.
    Returns (acc fp32, out bf16 bits, grad_probs fp32 [T,E] or None).
    """
    acc, out = unpermute(grad_u16, row_et)
    gp = None
    if pgrad is not None:
        row = np.asarray(row_et).astype(np.int64)
        gp = np.zeros((row.shape[1], row.shape[0]), dtype=np.float32)
        m = row >= 0
        gp.T[m] = np.asarray(pgrad, dtype=np.float32)[row[m]]
    return acc, out, gp


def group_sizes(total: int, groups: int):
    """Uniform split, kernel_cases/case03_moe_grouped_gemm_fc1_fwd.py:43-46."""
    base, rem = divmod(total, groups)
    return [base + (1 if i < rem else 0) for i in range(groups)]


def swiglu_f32(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """silu(g) * u in fp32 (no reference; SwiGLU is only named upstream)."""
    g = g.astype(np.float32)
    s = (g / (np.float32(1.0) + np.exp(-g, dtype=np.float32))).astype(np.float32)
    return (s * u.astype(np.float32)).astype(np.float32)


def swiglu(y_u16: np.ndarray) -> np.ndarray:
    """h = bf16(silu(gate) * up) with gate, up = y.chunk(2, -1)."""
    f = y_u16.shape[1] // 2
    return f32_to_bf16(swiglu_f32(bf16_to_f32(y_u16[:, :f]), bf16_to_f32(y_u16[:, f:])))


def grouped_gemm(x_u16: np.ndarray, w_u16: np.ndarray, m_splits, epilogue: str = "none",
                 row_starts=None, w_layout: str = "NK"):
    """out = cat_g(x[seg_g] @ w[g].T) in fp32, rounded to bf16.

    kernel_cases/case03_moe_grouped_gemm_fc1_fwd.py:57-64 and
    case04_moe_grouped_gemm_fc2_fwd.py:57-64 (torch.mm per group, bf16 out);
    fp32 accumulation as in case35_ref_musa_asm_bf16_gemm_nt_256x384.py:41-48.
    epilogue "swiglu": the fc1 output is rounded to bf16, then SwiGLU.
    Rows outside every group are left as zeros. w_u16 may also be a sequence
    of per-group float32 matrices (used by the CPU timing baseline).
    w_layout "KN": w[g] is [K,N] and out = x @ w[g] — the grouped dgrad of
    kernel_cases/case07/08_moe_grouped_gemm_fc*_dgrad.py:49-64 (case13/19
    with one group): torch.mm(dy[seg], w[g]), fp32 accumulation, bf16 out.
    """
    n = w_u16[0].shape[0] if w_layout == "NK" else w_u16[0].shape[1]
    n_out = n // 2 if epilogue == "swiglu" else n
    out = np.zeros((x_u16.shape[0], n_out), dtype=np.uint16)
    off = 0
    for g, m in enumerate(m_splits):
        m = int(m)
        start = off if row_starts is None else int(row_starts[g])
        if m > 0:
            xs = bf16_to_f32(x_u16[start:start + m])
            ws = w_u16[g] if w_u16[g].dtype == np.float32 else bf16_to_f32(w_u16[g])
            y = f32_to_bf16(xs @ (ws.T if w_layout == "NK" else ws))
            out[start:start + m] = swiglu(y) if epilogue == "swiglu" else y
        off = start + m
    return out


def grouped_wgrad(dy_u16: np.ndarray, x_u16: np.ndarray, m_splits) -> np.ndarray:
    """dW[g] = dy[seg_g]^T @ x[seg_g] in fp32, rounded to bf16; [G,N,K] bits.

    kernel_cases/case05_moe_grouped_gemm_fc2_wgrad.py:49-64 and
    case09_moe_grouped_gemm_fc1_wgrad.py:49-64 (torch.mm(dy[seg].t(), x[seg]),
    stacked); a group without rows gives zeros.
    """
    n, k = dy_u16.shape[1], x_u16.shape[1]
    out = np.zeros((len(m_splits), n, k), dtype=np.uint16)
    off = 0
    for g, m in enumerate(m_splits):
        m = int(m)
        if m > 0:
            out[g] = f32_to_bf16(bf16_to_f32(dy_u16[off:off + m]).T @ bf16_to_f32(x_u16[off:off + m]))
        off += m
    return out


def combine_backward(grad_out_u16: np.ndarray, rows_u16: np.ndarray, row_te: np.ndarray,
                     probs: np.ndarray):
    """Backward of the prob-weighted combine out[t] = sum_e probs[t,e] *
    rows[row_te[t,e]] (no reference kernel; the chain rule of the build's
    weighted combine, as torch.autograd forms it):
    grad_rows[r] = bf16(probs[t,e] * grad_out[t]) for r = row_te[t,e],
    grad_probs[t,e] = <grad_out[t], rows[r]> (fp32; 0 where not routed).
    Returns (grad_rows bf16 bits [R,H], grad_probs fp32 [T,E])."""
    g = bf16_to_f32(grad_out_u16)
    rows = bf16_to_f32(rows_u16)
    t, e = row_te.shape
    grad_rows = np.zeros(rows_u16.shape, np.uint16)
    grad_probs = np.zeros((t, e), np.float32)
    ti, ei = np.nonzero(row_te >= 0)
    r = row_te[ti, ei]
    p = probs[ti, ei].astype(np.float32)[:, None]
    grad_rows[r] = f32_to_bf16((p * g[ti]).astype(np.float32))
    grad_probs[ti, ei] = np.einsum("ij,ij->i", g[ti].astype(np.float64),
                                   rows[r].astype(np.float64)).astype(np.float32)
    return grad_rows, grad_probs


def swiglu_backward(y_u16: np.ndarray, dh_u16: np.ndarray) -> np.ndarray:
    """Backward of h = silu(g) * u, y = [g | u]: dg = dh * u * silu'(g),
    du = dh * silu(g), silu'(g) = s (1 + g (1 - s)), s = sigmoid(g); fp32
    from bf16 inputs, bf16 out (no reference; SwiGLU is only named upstream)."""
    f = dh_u16.shape[1]
    g = bf16_to_f32(y_u16[:, :f])
    u = bf16_to_f32(y_u16[:, f:])
    d = bf16_to_f32(dh_u16)
    den = (np.float32(1.0) + np.exp(-g, dtype=np.float32)).astype(np.float32)
    sig = (np.float32(1.0) / den).astype(np.float32)
    silu = (g / den).astype(np.float32)
    dsilu = (sig * (np.float32(1.0) + g * (np.float32(1.0) - sig))).astype(np.float32)
    dg = (d * u * dsilu).astype(np.float32)
    du = (d * silu).astype(np.float32)
    return np.concatenate([f32_to_bf16(dg), f32_to_bf16(du)], axis=1)


def moe_layer_backward(x_u16, logits, w1_u16, w2_u16, k, grad_out_u16, bias=None, renorm=True):
    """Backward of moe_layer for the output gradient grad_out, with the same
    bf16 roundings as the device chain (every GEMM output and every
    elementwise result rounded to bf16): combine backward -> fc2 dgrad and
    wgrad -> SwiGLU backward -> fc1 dgrad and wgrad -> permute backward.
    Returns (grad_x bf16 bits [T,H], grad_probs fp32 [T,E], dw1 bf16 bits
    [E,2F,H], dw2 bf16 bits [E,H,F])."""
    _, _, rmap, probs = router(logits, k, bias, "softmax", renorm)
    map_et, map_te, counts, num_out = row_id_map(rmap)
    xp, _ = permute(x_u16, map_te, None, num_out)
    y1 = grouped_gemm(xp, w1_u16, counts)
    h = swiglu(y1)
    y = grouped_gemm(h, w2_u16, counts)
    dy2, grad_probs = combine_backward(grad_out_u16, y, map_te, probs)
    dh = grouped_gemm(dy2, w2_u16, counts, w_layout="KN")
    dw2 = grouped_wgrad(dy2, h, counts)
    dy1 = swiglu_backward(y1, dh)
    dxp = grouped_gemm(dy1, w1_u16, counts, w_layout="KN")
    dw1 = grouped_wgrad(dy1, xp, counts)
    _, grad_x, _ = permute_backward(dxp, map_et)
    return grad_x, grad_probs, dw1, dw2


def router_logits(x_u16: np.ndarray, w_u16: np.ndarray) -> np.ndarray:
    """Router gate GEMM, logits fp32 = x @ w.T accumulated in fp32, unrounded.

    kernel_cases/case38_ref_musa_asm_bf16_ssgemm_nt_320x256.py:51-59
    (reference_fp32: inp.float().matmul(weight.float().t())).
    """
    return bf16_to_f32(x_u16) @ bf16_to_f32(w_u16).T


# --------------------------------------------------------------------------- layer


def moe_layer(x_u16, logits, w1_u16, w2_u16, k, bias=None, renorm=True, tokens=None,
              placement=None):
    """Full expert-layer forward: router -> row_id_map -> permute -> fc1+SwiGLU
    -> fc2 -> weighted combine. Returns out bf16 bits [T',H] for `tokens`.
    With a placement, w1/w2 are in slot order (w[c] = model expert placement[c])."""
    t = x_u16.shape[0]
    e = w1_u16.shape[0]
    _, _, rmap, probs = router(logits, k, bias, "softmax", renorm, placement)
    map_et, map_te, counts, num_out = row_id_map(rmap)
    xp, _ = permute(x_u16, map_te, None, num_out)
    h = grouped_gemm(xp, w1_u16, counts, "swiglu")
    y = grouped_gemm(h, w2_u16, counts)
    _, out = unpermute(y, map_et, probs, "dense", tokens=tokens)
    return out


def moe_layer_tokens(x_u16, probs, tokens, w1_of, w2_of):
    """The layer output of `tokens` only, computed from each token's own rows.

    The same chain as moe_layer for the selected tokens: for every expert e a
    token is routed to (probs[t,e] != 0, ascending e, which is the combine's
    order), y1 = bf16(x[t] @ w1[e].T), h = bf16(silu(gate) * up), y =
    bf16(h @ w2[e].T), then acc = acc + probs[t,e] * y in fp32 and out =
    bf16(acc) -- kernel_cases/case17…:58-71 (permute) -> case03…:57-64 (fc1)
    -> case04…:57-64 (fc2) -> case15…:58-64 (combine, weighted). A GEMM row
    depends only on its own input row, so this equals the grouped chain up to
    fp32 summation order inside each dot product. w1_of(e) / w2_of(e) return
    expert e's weights as bf16 bits ([2F,H] / [H,F]); each expert is fetched
    once, so a full-size layer can be checked on a few tokens without holding
    every expert's weights on the host.
    Returns out bf16 bits [len(tokens), H].
    """
    tokens = np.asarray(tokens, dtype=np.int64)
    p = np.asarray(probs, dtype=np.float32)[tokens]
    h_dim = x_u16.shape[1]
    ys = {}
    for e in np.unique(np.nonzero(p)[1]):
        sel = np.nonzero(p[:, e])[0]
        xs = bf16_to_f32(x_u16[tokens[sel]])
        w1 = bf16_to_f32(w1_of(int(e)))
        f = w1.shape[0] // 2
        y1 = bf16_to_f32(f32_to_bf16(xs @ w1.T))
        hm = bf16_to_f32(f32_to_bf16(swiglu_f32(y1[:, :f], y1[:, f:])))
        y = bf16_to_f32(f32_to_bf16(hm @ bf16_to_f32(w2_of(int(e))).T))
        for i, s in enumerate(sel):
            ys[(int(s), int(e))] = y[i]
    acc = np.zeros((len(tokens), h_dim), dtype=np.float32)
    for i in range(len(tokens)):
        for e in np.nonzero(p[i])[0]:  # ascending expert order
            acc[i] = acc[i] + (p[i, e] * ys[(i, int(e))]).astype(np.float32)
    return f32_to_bf16(acc)
