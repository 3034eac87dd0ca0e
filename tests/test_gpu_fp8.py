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
