"""FP8 (e4m3, row-wise scales) forward operators against an fp32 reference on the dequantised inputs.

The reference multiplies exactly the values the kernel multiplies (the e4m3 inputs times their fp32
scales), so the only differences are fp32 summation order and the bf16 output rounding.  Tolerance:
max|err|/max|ref| <= 1e-2 and float64 cosine >= 0.9999.
"""

from __future__ import annotations

import os

import pytest
import torch

from oracle import moe_ffn as O

pytestmark = pytest.mark.gpu


def _case(E, K, N, counts, seed):
    g = torch.Generator().manual_seed(seed)
    M = sum(counts)
    x = torch.randn(M, K, generator=g)
    w = torch.randn(E, K, N, generator=g) / K ** 0.5
    b = (torch.randn(E, N, generator=g) * 0.02).to(torch.bfloat16)
    offs = torch.cumsum(torch.tensor(counts, dtype=torch.int64), 0).to(torch.int32)
    return x, w, b, offs


def _check(name, got, ref):
    r = O.check(name, got.float().cpu(), ref.float().cpu())
    assert r["ok"], f"{name}: rel={r['rel']:.3e} cos={r['cos']:.7f}"


@pytest.mark.parametrize("cg", ["1", "2"])
@pytest.mark.parametrize("E,K,N,counts", [
    (4, 256, 192, [70, 0, 131, 5]),
    (3, 320, 256, [600, 513, 700]),
    (2, 2880, 512, [1029, 640]),
])
def test_fp8_mm_and_swiglu(cg, E, K, N, counts, monkeypatch):
    import cutlass_op.bf16_grouped_mm as m
    from cutlass_op.bf16_grouped_mm import fp8

    monkeypatch.setenv("MGF_CTA_GROUP", cg)
    x, w, b, offs = _case(E, K, N, counts, seed=E * 7 + K)
    qx, sx = fp8.quantize_rows(x.cuda())
    qw, sw = fp8.quantize_weights(w.cuda())
    xd, wd = fp8.dequantize_rows(qx, sx).cpu(), fp8.dequantize_weights(qw, sw).cpu()
    rows = int(offs[-1])
    out = fp8.grouped_mm_fp8(qx, qw, offs.cuda(), sx, sw, b.cuda())
    ref = O.grouped_linear(xd, wd, offs, b)
    _check("mm_fp8", out[:rows], ref[:rows])
    s, aux = fp8.grouped_mm_swiglu_fp8(qx, qw, offs.cuda(), sx, sw, b.cuda())
    torch.cuda.synchronize()
    m.check_device_status()
    _check("aux", aux[:rows], ref[:rows])
    _check("swiglu", s[:rows], O._bf16(O.swiglu_fwd(ref))[:rows])


def test_fp8_rejects_bad_layouts():
    from cutlass_op.bf16_grouped_mm import fp8

    qx = torch.zeros(32, 64, dtype=torch.float8_e4m3fn, device="cuda")
    qw_mn = torch.zeros(2, 64, 32, dtype=torch.float8_e4m3fn, device="cuda")  # unit stride along N: rejected
    offs = torch.tensor([16, 32], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="unit stride along K"):
        fp8.grouped_mm_fp8(qx, qw_mn, offs, torch.ones(32, device="cuda"), torch.ones(2, 32, device="cuda"))


@pytest.mark.parametrize("cg", ["1", "2"])
@pytest.mark.parametrize("E,H,I,counts", [(4, 256, 192, [70, 0, 131, 5]), (2, 2880, 256, [1029, 640])])
def test_fp8_swiglu_bwd(cg, E, H, I, counts, monkeypatch):
    """e4m3 down-proj dgrad + SwiGLU backward against the fp32 SwiGLU backward of the dequantised GEMM."""
    import cutlass_op.bf16_grouped_mm as m
    from cutlass_op.bf16_grouped_mm import fp8

    monkeypatch.setenv("MGF_CTA_GROUP", cg)
    g = torch.Generator().manual_seed(E + H)
    M = sum(counts)
    gout = torch.randn(M, H, generator=g)
    w_down = torch.randn(E, I, H, generator=g) / I ** 0.5
    aux = (torch.randn(M, 2 * I, generator=g) * 3).to(torch.bfloat16)
    offs = torch.cumsum(torch.tensor(counts, dtype=torch.int64), 0).to(torch.int32)
    qg, sg = fp8.quantize_rows(gout.cuda())
    qw, sw = fp8.quantize_weights(w_down.cuda().transpose(-2, -1))
    got = fp8.grouped_mm_swiglu_bwd_fp8(qg, qw, offs.cuda(), aux.cuda(), sg, sw)
    torch.cuda.synchronize()
    m.check_device_status()
    # the kernel feeds the fp32 accumulator (not a bf16-rounded one) into the SwiGLU backward
    gs32 = torch.zeros(M, I)
    for e, (s0, s1) in enumerate(O.segments(offs)):
        gs32[s0:s1] = fp8.dequantize_rows(qg, sg).cpu()[s0:s1] @ fp8.dequantize_weights(qw, sw).cpu()[e]
    ref = O._bf16(O.swiglu_bwd(gs32, aux.float()))
    rows = int(offs[-1])
    _check("swiglu_bwd_fp8", got[:rows], ref[:rows])


@pytest.mark.parametrize("m_,n,counts", [
    (192, 320, [70, 0, 131, 5, 1, 129, 256]),   # ones row inside the last m tile, an n tail
    (256, 256, [300, 7, 0, 129]),               # m % 128 == 0: the ones row gets its own m tile
    (2880, 5760, [1029, 0, 640, 1]),            # GPT-OSS widths
])
def test_fp8_wgrad_bias(m_, n, counts, monkeypatch):
    """e4m3 ragged-K weight + bias gradient against fp32 on the per-column-dequantised operands;
    empty groups give exact zeros.  The 128-row and the 256-row single-CTA tiles give the same bits."""
    import cutlass_op.bf16_grouped_mm as m
    from cutlass_op.bf16_grouped_mm import fp8

    g = torch.Generator().manual_seed(m_ + n)
    M = sum(counts)
    a = torch.randn(M, m_, generator=g)
    b = torch.randn(M, n, generator=g) * torch.linspace(0.1, 3.0, n)
    offs = torch.cumsum(torch.tensor(counts, dtype=torch.int64), 0).to(torch.int32)
    qa, sa = fp8.quantize_cols(a.cuda())
    qb, sb = fp8.quantize_cols(b.cuda())
    forms = {}
    for form in ("0", "1"):
        monkeypatch.setenv("MGF_WGRAD_M256", form)
        forms[form] = fp8.grouped_mm_wgrad_fp8(qa, qb, offs.cuda(), sa, sb)
        torch.cuda.synchronize()
        m.check_device_status()
    assert torch.equal(forms["0"][0], forms["1"][0]) and torch.equal(forms["0"][1], forms["1"][1])
    dw, db = forms["1"]
    ad, bd = fp8.dequantize_cols(qa, sa).cpu(), fp8.dequantize_cols(qb, sb).cpu()
    ref_w, ref_b = O.grouped_wgrad(ad, bd, offs)
    for e, (s0, s1) in enumerate(O.segments(offs)):
        if s1 == s0:
            assert torch.count_nonzero(dw[e]) == 0 and torch.count_nonzero(db[e]) == 0
        else:
            _check(f"dW[{e}]", dw[e], ref_w[e])
            _check(f"db[{e}]", db[e], ref_b[e])


def test_fp8_ffn_tracks_the_bf16_oracle():
    """grouped_mm_ffn_fp8 (every forward and backward GEMM in e4m3) against the bf16 oracle chain:
    e4m3 keeps ~3 significant bits less than bf16, so the tolerance here is max|err|/max|ref| <= 0.1
    and float64 cosine >= 0.995 on the output and all five gradients."""
    import cutlass_op.bf16_grouped_mm as m
    from cutlass_op.bf16_grouped_mm import fp8
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    x, w_up, b_up, w_down, b_down, offs, gout = small_case(4, 256, 128, [96, 0, 131, 29], seed=12)
    leaves = [t.cuda().clone().requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
    out = fp8.grouped_mm_ffn_fp8(leaves[0], leaves[1], leaves[3], offs.cuda(), leaves[2], leaves[4])
    out.backward(gout.cuda())
    torch.cuda.synchronize()
    m.check_device_status()
    ref = O.kernel_chain(x, w_up, b_up, w_down, b_down, offs, gout)
    got = dict(zip(["out", "dx", "dw_up", "db_up", "dw_down", "db_down"], [out.detach()] + [t.grad for t in leaves]))
    rows = int(offs[-1])
    for k, v in got.items():
        a, b = v.float().cpu(), ref[k]
        if k in ("out", "dx"):
            a, b = a[:rows], b[:rows]
        r = O.check(k, a, b, rel_tol=0.1, cos_tol=0.995)
        assert r["ok"], r
    for k in ("dw_up", "db_up", "dw_down", "db_down"):
        assert torch.count_nonzero(got[k][1]) == 0


@pytest.mark.parametrize("shape", [(1029, 2880), (7, 64), (0, 128), (640, 5760)])
def test_fused_quantisers_match_the_formula(shape):
    """The fused e4m3 quantisers (rows, columns, weights in both layouts) give the torch formula's
    scales and codes bit for bit on bf16 inputs."""
    from cutlass_op.bf16_grouped_mm import fp8

    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=g) * torch.linspace(0.01, 30.0, shape[1])).to(torch.bfloat16).cuda()
    for fn in (fp8.quantize_rows, fp8.quantize_cols):
        q, s = fn(x)
        qr, sr = fn(x, native=False)
        assert torch.equal(s, sr), fn.__name__
        assert torch.equal(q.view(torch.uint8), qr.view(torch.uint8)), fn.__name__
    if shape[0]:
        w = x[: min(shape[0], 256)].reshape(1, -1, shape[1]).repeat(3, 1, 1)
        for ww in (w, w.transpose(1, 2).contiguous().transpose(1, 2), w.transpose(1, 2)):
            q, s = fp8.quantize_weights(ww)
            qr, sr = fp8.quantize_weights(ww, native=False)
            assert torch.equal(s, sr)
            assert q.stride(1) == 1 and torch.equal(q.view(torch.uint8), qr.view(torch.uint8))


@pytest.mark.parametrize("shape", [(3, 136, 40), (2, 2880, 5760), (4, 70, 264), (1, 1, 8)])
def test_fused_both_axes_weight_quantiser_matches_two_calls(shape):
    """quantize_weights_both(w) gives exactly quantize_weights(w) and quantize_weights(w^T): the same
    codes and scales bit for bit, k and n tails included."""
    from cutlass_op.bf16_grouped_mm import fp8

    E, K, N = shape
    g = torch.Generator().manual_seed(E * K + N)
    w = (torch.randn(E, K, N, generator=g) * torch.linspace(0.01, 4.0, N)).to(torch.bfloat16).cuda()
    q, s, q_t, s_t = fp8.quantize_weights_both(w)
    r, rs = fp8.quantize_weights(w)
    r_t, rs_t = fp8.quantize_weights(w.transpose(-2, -1))
    torch.cuda.synchronize()
    assert q.shape == r.shape and q_t.shape == r_t.shape
    assert torch.equal(q.view(torch.uint8), r.view(torch.uint8)) and torch.equal(s, rs)
    assert torch.equal(q_t.view(torch.uint8), r_t.view(torch.uint8)) and torch.equal(s_t, rs_t)


@pytest.mark.parametrize("shape", [(1029, 2880), (7, 64), (0, 128), (640, 5760), (300, 40)])
def test_fused_rows_cols_quantiser_matches_two_calls(shape):
    """quantize_rows_cols(x) gives exactly quantize_rows(x) and quantize_cols(x), bit for bit."""
    from cutlass_op.bf16_grouped_mm import fp8

    g = torch.Generator().manual_seed(shape[0] + shape[1])
    x = (torch.randn(*shape, generator=g) * torch.linspace(0.05, 6.0, shape[1])).to(torch.bfloat16).cuda()
    q_r, s_r, q_c, s_c = fp8.quantize_rows_cols(x)
    r_r, rs_r = fp8.quantize_rows(x)
    r_c, rs_c = fp8.quantize_cols(x)
    torch.cuda.synchronize()
    assert torch.equal(q_r.view(torch.uint8), r_r.view(torch.uint8)) and torch.equal(s_r, rs_r)
    assert torch.equal(q_c.view(torch.uint8), r_c.view(torch.uint8)) and torch.equal(s_c, rs_c)
