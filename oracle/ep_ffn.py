"""CPU oracle for the expert-parallel MoE FFN -- TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's pre-timed ``ep_parity`` self-check use it, as the checker.

The reference has no distributed code: expert parallelism is an addition of this build.  Its
correct result is the single-process MoE FFN over ALL ranks' tokens: every routed copy (token t of
rank r, slot j) goes through expert idx[t, j] with the reference's kernel chain
(oracle.moe_ffn.kernel_chain, the roundings of csrc/grouped_mm_kernel.cuh:130-143 and the SwiGLU
visitors), and a token's output is sum_j w[t, j] * y(copy).  Backward: the copy's output gradient is
bf16(w[t, j] * g[t]); dx[t] sums its copies' dx in fp32; d w[t, j] = <y(copy), g[t]> in fp32; the
weight and bias gradients of expert e sum over every rank's copies routed to it.
"""

from __future__ import annotations

import torch

from .moe_ffn import kernel_chain


def ep_reference(xs, idxs, ws, gs, w_up, b_up, w_down, b_down):
    """xs/idxs/ws/gs: per-rank [T, H] bf16 tokens, [T, k] expert ids, [T, k] router weights (or None),
    [T, H] output gradients.  w_up..b_down: all E experts' weights (CPU).  Returns
    {"out": [per-rank [T, H]], "dx": [...], "dw_router": [...], "dw_up", "db_up", "dw_down", "db_down"}."""
    E = w_up.shape[0]
    k = idxs[0].shape[1]
    T = [x.shape[0] for x in xs]
    x_all = torch.cat(xs, 0)
    idx_all = torch.cat(idxs, 0).reshape(-1).to(torch.int64)
    w_all = torch.cat([w.float() if w is not None else torch.ones(t, k) for w, t in zip(ws, T)], 0).reshape(-1)
    g_all = torch.cat(gs, 0).float()
    order = torch.argsort(idx_all, stable=True)
    tok = torch.div(order, k, rounding_mode="floor")
    counts = torch.bincount(idx_all, minlength=E)
    offs = torch.cumsum(counts, 0).to(torch.int32)
    rows = x_all[tok]
    g_rows = (g_all[tok] * w_all[order].unsqueeze(1)).to(torch.bfloat16)
    r = kernel_chain(rows, w_up, b_up, w_down, b_down, offs, g_rows)
    y = r["out"]
    n_tok = x_all.shape[0]
    out = torch.zeros(n_tok, x_all.shape[1]).index_add_(0, tok, y * w_all[order].unsqueeze(1))
    dx = torch.zeros(n_tok, x_all.shape[1]).index_add_(0, tok, r["dx"])
    dw_sorted = (y * g_all[tok]).sum(1)
    dw_router = torch.empty_like(dw_sorted)
    dw_router[order] = dw_sorted
    dw_router = dw_router.view(n_tok, k)
    res = {"out": [], "dx": [], "dw_router": []}
    start = 0
    for t in T:
        res["out"].append(out[start:start + t])
        res["dx"].append(dx[start:start + t])
        res["dw_router"].append(dw_router[start:start + t])
        start += t
    for key in ("dw_up", "db_up", "dw_down", "db_down"):
        res[key] = r[key]
    return res
