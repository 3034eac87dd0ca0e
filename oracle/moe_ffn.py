"""CPU oracle for the MoE FFN grouped-GEMM path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg may import this
module, and only as the checker or the timed CPU baseline.  The product path never calls it.

Two restatements of Butterfingrz/CuTe-MoE-Train's math (paths relative to
cutlass_op/bf16_grouped_mm/), both in float32 torch on the CPU over bf16-rounded inputs:

``kernel_chain``  the reference's operator chain with bf16 roundings exactly where its kernels
                  round:  aux = bf16(x@W_up[e] + b_up[e])            csrc/grouped_mm_kernel.cuh:130-143
                          swiglu = bf16(SwiGLU(aux))                 csrc/grouped_mm_swiglu_visitor.cuh:295-334
                          out = bf16(swiglu@W_down[e] + b_down[e])   custom_op.py:579-601
                  backward as routed by custom_op.py:630-687 and 467-520:
                          dW_down = bf16(swiglu^T g), db_down = bf16(sum g)     custom_op.py:661-667, 79-101
                          grad_aux = bf16(SwiGLU_bwd(g@W_down^T, aux))         csrc/grouped_mm_swiglu_bwd_visitor.cuh:35-68
                          dx = bf16(grad_aux@W_up^T), dW_up = bf16(x^T grad_aux),
                          db_up = bf16(sum grad_aux)                            custom_op.py:508-518
``fp32_composition``  the primary oracle of the E=8, H=2048, I=1024 CPU case: a plain per-expert
                  fp32 composition (matmul + bias + clamp + sigmoid) differentiated by torch autograd, with no
                  intermediate rounding.

Parity pin: the reference ships no tests or golden vectors.  tests/golden/make_golden.py runs the
reference's own Python layer (its __init__.py + custom_op.py, unmodified: the autograd routing,
the fused-only contract, _segment_sum_rows) over a CPU stand-in for its three CUDA kernels that
mimics their arithmetic (bf16 SwiGLU with tanh), and commits the outputs; tests check this oracle
against them.  The CUDA kernels of the reference cannot run here (sm_90a only; the CUTLASS fork
they need is an empty submodule), so kernel-level numerics are pinned only through that stand-in.
"""

from __future__ import annotations

import torch

ALPHA = 1.702
LIMIT = 7.0


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def segments(offs: torch.Tensor) -> list[tuple[int, int]]:
    """[start, end) rows of each group from int32 cumulative ends (custom_op.py:86-94)."""
    ends = [int(v) for v in offs.tolist()]
    out, prev = [], 0
    for e in ends:
        out.append((prev, e))
        prev = e
    return out


def swiglu_fwd(aux: torch.Tensor, alpha: float = ALPHA, limit: float = LIMIT) -> torch.Tensor:
    """Clamped SwiGLU on interleaved columns: even = gate, odd = up.

    csrc/grouped_mm_swiglu_visitor.cuh:309-334: g = min(gate, limit), u = clamp(up, -limit, limit),
    out = g * sigmoid(alpha * g) * (u + 1).
    """
    gate = aux[..., 0::2]
    up = aux[..., 1::2]
    g = torch.clamp(gate, max=limit)
    u = torch.clamp(up, min=-limit, max=limit)
    return g * torch.sigmoid(alpha * g) * (u + 1.0)


def swiglu_bwd(grad_s: torch.Tensor, aux: torch.Tensor, alpha: float = ALPHA, limit: float = LIMIT) -> torch.Tensor:
    """Gradient w.r.t. the interleaved aux (csrc/grouped_mm_swiglu_bwd_visitor.cuh:35-68)."""
    gate = aux[..., 0::2]
    up = aux[..., 1::2]
    gc = torch.clamp(gate, max=limit)
    uc = torch.clamp(up, min=-limit, max=limit)
    sig = torch.sigmoid(alpha * gc)
    d_gate = grad_s * (uc + 1.0) * sig * (1.0 + alpha * gc * (1.0 - sig))
    d_up = grad_s * gc * sig
    d_gate = torch.where(gate <= limit, d_gate, torch.zeros_like(d_gate))
    d_up = torch.where((up >= -limit) & (up <= limit), d_up, torch.zeros_like(d_up))
    out = torch.empty_like(aux)
    out[..., 0::2] = d_gate
    out[..., 1::2] = d_up
    return out


def grouped_linear(a, w, offs, bias=None):
    """Ragged-M: out[rows(e)] = a[rows(e)] @ w[e] (+ bias[e]), fp32 accumulate, one bf16 rounding."""
    out = torch.zeros(a.shape[0], w.shape[-1], dtype=torch.float32)
    for e, (s, t) in enumerate(segments(offs)):
        if t > s:
            y = a[s:t].float() @ w[e].float()
            if bias is not None:
                y = y + bias[e].float()
            out[s:t] = y
    return _bf16(out)


def grouped_wgrad(a, g, offs):
    """Ragged-K: dW[e] = a[rows(e)]^T @ g[rows(e)] and db[e] = sum g[rows(e)] (zeros for empty groups)."""
    E = offs.numel()
    dw = torch.zeros(E, a.shape[1], g.shape[1], dtype=torch.float32)
    db = torch.zeros(E, g.shape[1], dtype=torch.float32)
    for e, (s, t) in enumerate(segments(offs)):
        if t > s:
            dw[e] = a[s:t].float().t() @ g[s:t].float()
            db[e] = g[s:t].float().sum(0)
    return _bf16(dw), _bf16(db)


def kernel_chain(x, w_up, b_up, w_down, b_down, offs, grad_out, alpha=ALPHA, limit=LIMIT):
    """Forward + backward of the fused MoE FFN, rounded like the reference's kernel chain."""
    aux = grouped_linear(x, w_up, offs, b_up)
    swiglu = _bf16(swiglu_fwd(aux, alpha, limit))
    out = grouped_linear(swiglu, w_down, offs, b_down)
    g = grad_out.float()
    dw_down, db_down = grouped_wgrad(swiglu, _bf16(g), offs)
    gs = torch.zeros(x.shape[0], w_down.shape[1], dtype=torch.float32)
    for e, (s, t) in enumerate(segments(offs)):
        if t > s:
            gs[s:t] = _bf16(g[s:t]) @ w_down[e].float().t()
    grad_aux = _bf16(swiglu_bwd(gs, aux, alpha, limit))
    n_rows = int(offs[-1]) if offs.numel() else 0
    grad_aux[n_rows:] = 0.0
    dx = grouped_linear(grad_aux, w_up.transpose(-2, -1), offs)
    dw_up, db_up = grouped_wgrad(x, grad_aux, offs)
    return {
        "swiglu_out": swiglu, "aux": aux, "out": out, "grad_aux": grad_aux,
        "dx": dx, "dw_up": dw_up, "db_up": db_up, "dw_down": dw_down, "db_down": db_down,
    }


def fp32_composition(x, w_up, b_up, w_down, b_down, offs, grad_out, alpha=ALPHA, limit=LIMIT):
    """Plain fp32 per-expert composition with torch autograd (no intermediate rounding)."""
    leaves = [t.detach().float().clone().requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
    xf, wu, bu, wd, bd = leaves
    rows = []
    for e, (s, t) in enumerate(segments(offs)):
        if t > s:
            h = xf[s:t] @ wu[e] + bu[e]
            rows.append(swiglu_fwd(h, alpha, limit) @ wd[e] + bd[e])
    n_rows = int(offs[-1]) if offs.numel() else 0
    if not rows:
        z = [torch.zeros_like(t) for t in leaves]
        return {"out": xf.new_zeros(0, w_down.shape[-1]), "dx": z[0], "dw_up": z[1], "db_up": z[2],
                "dw_down": z[3], "db_down": z[4]}
    out = torch.cat(rows, 0)
    (out * grad_out.float()[:n_rows]).sum().backward()
    grads = [t.grad if t.grad is not None else torch.zeros_like(t) for t in leaves]
    return {
        "out": out.detach(), "dx": grads[0], "dw_up": grads[1], "db_up": grads[2],
        "dw_down": grads[3], "db_down": grads[4],
    }


# ---------------------------------------------------------------------------------------- checker

def rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max|got - ref| / max|ref| in float64 (0 when both are all zero)."""
    g, r = got.detach().cpu().double(), ref.detach().cpu().double()
    den = r.abs().max().item() if r.numel() else 0.0
    num = (g - r).abs().max().item() if r.numel() else 0.0
    if den == 0.0:
        return 0.0 if num == 0.0 else float("inf")
    return num / den


def cosine(got: torch.Tensor, ref: torch.Tensor) -> float:
    """Cosine similarity computed in float64 (fp32 cosine can exceed 1 on large tensors)."""
    g, r = got.detach().cpu().double().flatten(), ref.detach().cpu().double().flatten()
    ng, nr = g.norm().item(), r.norm().item()
    if ng == 0.0 and nr == 0.0:
        return 1.0
    if ng == 0.0 or nr == 0.0:
        return 0.0
    return float((g @ r).item() / (ng * nr))


REL_TOL = 1e-2
COS_TOL = 0.9999


def check(name: str, got: torch.Tensor, ref: torch.Tensor, rel_tol: float = REL_TOL, cos_tol: float = COS_TOL) -> dict:
    """Return {'name', 'rel', 'cos', 'ok'} with the tolerances stated by the spec."""
    assert tuple(got.shape) == tuple(ref.shape), f"{name}: shape {tuple(got.shape)} != {tuple(ref.shape)}"
    r, c = rel_err(got, ref), cosine(got, ref)
    return {"name": name, "rel": r, "cos": c, "ok": (r <= rel_tol) and (c >= cos_tol)}
