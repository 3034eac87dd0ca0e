"""The general `grouped_mm::mm` layouts (ragged-M, ragged-K, ragged-N, batched; row- and column-major
operands) against a plain fp32 torch reference of the same op, forward and backward.

Tolerance: max|err|/max|ref| <= 1e-2 and float64 cosine >= 0.9999 (bf16 output, fp32 accumulation).
"""

from __future__ import annotations

import pytest
import torch

from oracle import moe_ffn as O

pytestmark = pytest.mark.gpu


def _m():
    import cutlass_op.bf16_grouped_mm as m

    return m


def _col(t):
    """Same values, column-major in the last two dims."""
    return t.transpose(-2, -1).contiguous().transpose(-2, -1)


def _lay(t, col):
    return _col(t) if col else t.contiguous()


def _segs(offs):
    prev = 0
    for e, end in enumerate(offs.tolist()):
        yield e, prev, end
        prev = end


def _ref(a, b, offs, bias):
    """fp32 reference of grouped_mm for every rank combination (csrc/grouped_mm_common.cuh:90-140)."""
    a, b = a.float().cpu(), b.float().cpu()
    bias = bias.float().cpu() if bias is not None else None
    if a.dim() == 2 and b.dim() == 3:
        out = torch.zeros(a.shape[0], b.shape[2])
        for e, s, t in _segs(offs):
            out[s:t] = a[s:t] @ b[e] + (bias[e] if bias is not None else 0)
        return out
    if a.dim() == 2 and b.dim() == 2:
        out = torch.zeros(offs.numel(), a.shape[0], b.shape[1])
        for e, s, t in _segs(offs):
            out[e] = a[:, s:t] @ b[s:t]
        return out
    if a.dim() == 3 and b.dim() == 2:
        out = torch.zeros(a.shape[1], b.shape[1])
        for e, s, t in _segs(offs):
            out[:, s:t] = a[e] @ b[:, s:t] + (bias[e, : t - s] if bias is not None else 0)
        return out
    return a @ b + (bias[:, None, :] if bias is not None else 0)


def _check(name, got, ref):
    r = O.check(name, got.float().cpu(), ref)
    assert r["ok"], f"{name}: rel={r['rel']:.3e} cos={r['cos']:.7f}"


def _rand(*shape, seed):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)


CASES = [
    # name, a shape, b shape, offs, bias shape or None
    ("ragged_m", (304, 64), (4, 64, 48), [70, 70, 201, 304], (4, 48)),
    ("ragged_k", (40, 304), (304, 56), [64, 64, 190, 304], None),
    ("ragged_n", (3, 72, 64), (64, 208), [40, 40, 208], (3, 208)),
    ("ragged_n_m_odd", (3, 36, 64), (64, 96), [16, 48, 96], None),
    ("batched", (3, 56, 64), (3, 64, 40), None, (3, 40)),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("a_col", [False, True], ids=["a_row", "a_col"])
@pytest.mark.parametrize("b_col", [False, True], ids=["b_row", "b_col"])
def test_layouts_forward_backward(case, a_col, b_col):
    name, ash, bsh, offs_l, bias_sh = case
    if name == "ragged_n_m_odd" and a_col:
        pytest.skip("a column-major [E, 36, 64] has a 72-byte stride: rejected like the reference (16-byte rule)")
    m = _m()
    a0, b0 = _rand(*ash, seed=1), _rand(*bsh, seed=2)
    bias0 = (_rand(*bias_sh, seed=3) * 0.1).to(torch.bfloat16) if bias_sh else None
    offs = torch.tensor(offs_l, dtype=torch.int32) if offs_l is not None else None
    a = _lay(a0.cuda(), a_col).requires_grad_(True)
    b = _lay(b0.cuda(), b_col).requires_grad_(True)
    bias = bias0.cuda().requires_grad_(True) if bias0 is not None else None
    out = m.grouped_mm(a, b, offs.cuda() if offs is not None else None, bias)
    ref_out = _ref(a0, b0, offs, bias0)
    if name.startswith("ragged_n"):  # columns past offs[-1] belong to no group
        ref_out = ref_out[:, : offs_l[-1]]
        out_cmp = out[:, : offs_l[-1]]
    elif name == "ragged_m":
        ref_out, out_cmp = ref_out[: offs_l[-1]], out[: offs_l[-1]]
    else:
        out_cmp = out
    _check(f"{name}:out", out_cmp, ref_out)

    g = _rand(*out.shape, seed=4)
    out.backward(g.cuda())
    torch.cuda.synchronize()
    m.check_device_status()
    # fp32 autograd of the reference composition
    af, bf = a0.float().requires_grad_(True), b0.float().requires_grad_(True)
    biasf = bias0.float().requires_grad_(True) if bias0 is not None else None
    rf = _ref_autograd(af, bf, offs, biasf)
    rf.backward(g.float())
    _check(f"{name}:grad_a", a.grad, af.grad)
    _check(f"{name}:grad_b", b.grad, bf.grad)
    if bias is not None:
        _check(f"{name}:grad_bias", bias.grad, biasf.grad)


def _ref_autograd(a, b, offs, bias):
    """Differentiable fp32 version of _ref (same math, torch autograd)."""
    if a.dim() == 2 and b.dim() == 3:
        parts = [a[s:t] @ b[e] + (bias[e] if bias is not None else 0) for e, s, t in _segs(offs)]
        used = torch.cat(parts, 0)
        return torch.cat([used, a.new_zeros(a.shape[0] - used.shape[0], b.shape[2])], 0)
    if a.dim() == 2 and b.dim() == 2:
        return torch.stack([a[:, s:t] @ b[s:t] for e, s, t in _segs(offs)], 0)
    if a.dim() == 3 and b.dim() == 2:
        parts = [a[e] @ b[:, s:t] + (bias[e, : t - s] if bias is not None else 0) for e, s, t in _segs(offs)]
        used = torch.cat(parts, 1)
        return torch.cat([used, a.new_zeros(a.shape[1], b.shape[1] - used.shape[1])], 1)
    return a @ b + (bias[:, None, :] if bias is not None else 0)
