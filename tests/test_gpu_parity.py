"""GPU parity of the sm_100a kernels against the CPU oracle (tolerance: max|err|/max|ref| <= 1e-2
and float64 cosine >= 0.9999 on every output and gradient; group boundaries exact)."""

from __future__ import annotations

import pytest
import torch

from oracle import moe_ffn as O

pytestmark = pytest.mark.gpu

REL, COS = 1e-2, 0.9999


def _lib():
    import cutlass_op.bf16_grouped_mm as m

    return m


def _assert_close(name, got, ref, rel=REL, cos=COS):
    r = O.check(name, got.float().cpu(), ref.float().cpu(), rel, cos)
    assert r["ok"], f"{name}: rel={r['rel']:.3e} cos={r['cos']:.7f}"


def _run_chain(x, w_up, b_up, w_down, b_down, offs, gout, dev="cuda"):
    m = _lib()
    leaves = [t.to(dev).clone().requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
    xl, wu, bu, wd, bd = leaves
    offs_d = offs.to(dev)
    s, aux = m.grouped_mm_swiglu(xl, wu, offs=offs_d, bias=bu, swiglu_alpha=1.702, swiglu_limit=7.0)
    out = m.grouped_mm_downproj(s, wd, offs=offs_d, bias=bd, aux_biased_acc=aux, swiglu_alpha=1.702,
                                swiglu_limit=7.0)
    out.backward(gout.to(dev))
    torch.cuda.synchronize()
    m.check_device_status()
    return {
        "swiglu_out": s.detach(), "aux": aux.detach(), "out": out.detach(), "dx": xl.grad,
        "dw_up": wu.grad, "db_up": bu.grad, "dw_down": wd.grad, "db_down": bd.grad,
    }


KEYS = ["swiglu_out", "aux", "out", "dx", "dw_up", "db_up", "dw_down", "db_down"]


def _compare_chain(got, ref, offs, keys=KEYS):
    rows = int(offs[-1]) if offs.numel() else 0
    for k in keys:
        g, r = got[k], ref[k]
        if k in ("swiglu_out", "aux", "out", "dx"):
            g, r = g[:rows], r[:rows]
        _assert_close(k, g, r)


@pytest.mark.parametrize("case", ["mixed_empty", "odd_sizes", "single_expert", "leading_trailing_empty", "all_empty"])
def test_chain_vs_golden(golden, case):
    c = golden["cases"][case]
    i = c["inputs"]
    got = _run_chain(i["x"], i["w_up"], i["b_up"], i["w_down"], i["b_down"], i["offs"], i["grad_out"])
    _compare_chain(got, c["outputs"], i["offs"])
    # empty experts: weight and bias gradients are exact zeros
    for e, n in enumerate(c["counts"]):
        if n == 0:
            for k in ("dw_up", "db_up", "dw_down", "db_down"):
                assert torch.count_nonzero(got[k][e]).item() == 0, f"{k}[{e}] not zero for an empty expert"


def test_config1_vs_oracle():
    from cutlass_op.bf16_grouped_mm.workloads import config1

    x, w_up, b_up, w_down, b_down, offs = config1()
    gout = torch.ones(x.shape[0], x.shape[1], dtype=torch.bfloat16)  # loss = out.sum()
    got = _run_chain(x, w_up, b_up, w_down, b_down, offs, gout)
    ref = O.kernel_chain(x, w_up, b_up, w_down, b_down, offs, gout)
    _compare_chain(got, ref, offs)
    fp = O.fp32_composition(x, w_up, b_up, w_down, b_down, offs, gout)
    for k in ("out", "dx", "dw_up", "db_up", "dw_down", "db_down"):
        _assert_close("fp32:" + k, got[k], fp[k])


@pytest.mark.parametrize(
    "E,H,I,counts",
    [
        (3, 136, 40, [70, 0, 131]),        # n and k tails (N=80, 136), m tail with the ones row at 8
        (2, 128, 64, [129, 255]),          # m % 128 == 0: extra bias-gradient tile
        (4, 256, 192, [1, 7, 129, 300]),   # forced sizes 1, 7, 129
        (6, 384, 96, [0, 0, 513, 0, 64, 0]),
    ],
)
@pytest.mark.parametrize("cg", ["auto", "1", "2"])
def test_chain_shapes(E, H, I, counts, cg, monkeypatch):
    """Every launch of the chain with the default CTA policy, forced single CTAs and forced pairs
    (ragged-K pairs included)."""
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    if cg != "auto":
        monkeypatch.setenv("MGF_CTA_GROUP", cg)

    x, w_up, b_up, w_down, b_down, offs, gout = small_case(E, H, I, counts, seed=E * 1000 + H)
    got = _run_chain(x, w_up, b_up, w_down, b_down, offs, gout)
    ref = O.kernel_chain(x, w_up, b_up, w_down, b_down, offs, gout)
    _compare_chain(got, ref, offs)


def test_plain_grouped_mm_autograd():
    """grouped_mm (ragged-M with bias) forward and all three gradients."""
    m = _lib()
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    x, w, b, _, _, offs, _ = small_case(4, 192, 96, [33, 0, 190, 64], seed=7)
    xl, wl, bl = (t.cuda().clone().requires_grad_(True) for t in (x, w, b))
    out = m.grouped_mm(xl, wl, offs=offs.cuda(), bias=bl)
    g = torch.randn(out.shape, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    out.backward(g.cuda())
    ref_out = O.grouped_linear(x, w, offs, b)
    _assert_close("out", out, ref_out)
    ref_dx = O.grouped_linear(g, w.transpose(-2, -1), offs)
    ref_dw, ref_db = O.grouped_wgrad(x, g, offs)
    _assert_close("dx", xl.grad, ref_dx)
    _assert_close("dw", wl.grad, ref_dw)
    _assert_close("db", bl.grad, ref_db)


def test_batched_grouped_mm():
    m = _lib()
    g = torch.Generator().manual_seed(11)
    a = torch.randn(3, 100, 64, generator=g).to(torch.bfloat16)
    bm = torch.randn(3, 64, 48, generator=g).to(torch.bfloat16)
    out = m.grouped_mm(a.cuda(), bm.cuda())
    ref = (a.float() @ bm.float()).to(torch.bfloat16)
    _assert_close("bmm", out, ref)


def test_fused_only_contract():
    """A gradient reaching swiglu_out directly raises, as in the reference."""
    m = _lib()
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    x, w_up, b_up, _, _, offs, _ = small_case(2, 64, 32, [10, 20], seed=3)
    xl = x.cuda().requires_grad_(True)
    s, aux = m.grouped_mm_swiglu(xl, w_up.cuda(), offs.cuda(), b_up.cuda())
    with pytest.raises(RuntimeError, match="fused-only"):
        s.float().sum().backward()


def test_config5_style_fine_grained_groups():
    """Config 5's structure at small widths: 256 experts, top-8, Zipf(1.3) plus forced groups of
    0, 1, 7 and 129 rows -- most groups tiny or empty."""
    from cutlass_op.bf16_grouped_mm.workloads import config5_counts, small_case

    counts = config5_counts(96, 256, 8, seed=3)
    assert sorted(counts.tolist()).count(0) >= 1 and 129 in counts.tolist() and 7 in counts.tolist()
    x, w_up, b_up, w_down, b_down, offs, gout = small_case(256, 64, 32, counts.tolist(), seed=5)
    got = _run_chain(x, w_up, b_up, w_down, b_down, offs, gout)
    ref = O.kernel_chain(x, w_up, b_up, w_down, b_down, offs, gout)
    _compare_chain(got, ref, offs)


@pytest.mark.parametrize("counts", [[70, 0, 131, 5], [0, 0, 0, 0], [256, 1, 0, 300]])
def test_ffn_recompute_equals_stored_aux(counts):
    """store_aux=False (aux recomputed in backward) gives the stored-aux results bit for bit, and both
    match the oracle."""
    from cutlass_op.bf16_grouped_mm import grouped_mm_ffn
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    x, w_up, b_up, w_down, b_down, offs, gout = small_case(4, 192, 96, counts, seed=sum(counts) + 1)
    res = {}
    for store_aux in (True, False):
        leaves = [t.cuda().clone().requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
        out = grouped_mm_ffn(leaves[0], leaves[1], leaves[3], offs.cuda(), leaves[2], leaves[4], store_aux=store_aux)
        out.backward(gout.cuda())
        torch.cuda.synchronize()
        res[store_aux] = [out.detach()] + [t.grad for t in leaves]
    _lib().check_device_status()
    names = ["out", "dx", "dw_up", "db_up", "dw_down", "db_down"]
    rows = int(offs[-1])
    for name, a, b in zip(names, res[True], res[False]):
        if name in ("out", "dx"):
            a, b = a[:rows], b[:rows]
        assert torch.equal(a, b), f"{name}: recompute differs from stored aux"
    ref = O.kernel_chain(x, w_up, b_up, w_down, b_down, offs, gout)
    got = dict(zip(names, res[False]))
    _compare_chain(got, ref, offs, keys=names)


def test_reference_binding_functions_match_the_operators():
    """`_ext._grouped_mm_swiglu_cuda` / `_grouped_mm_swiglu_bwd_cuda` write into the caller's buffers
    exactly what the operators return (store_aux on and off; the packed fp32 views of the reference)."""
    m = _lib()
    from cutlass_op.bf16_grouped_mm import _ext
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    x, w_up, b_up, w_down, b_down, offs, gout = small_case(3, 128, 64, [70, 0, 131], seed=21)
    x, w_up, b_up, w_down, offs, gout = (t.cuda() for t in (x, w_up, b_up, w_down, offs, gout))
    s_ref, aux_ref = m.grouped_mm_swiglu(x, w_up, offs, b_up)
    M, I = x.shape[0], w_up.shape[2] // 2
    s_out = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    aux_out = torch.empty(M, 2 * I, dtype=torch.bfloat16, device="cuda")
    _ext._grouped_mm_swiglu_cuda(x, w_up, offs, b_up, aux_out, s_out, 1.702, 7.0, True)
    rows = int(offs[-1])
    assert torch.equal(s_out[:rows], s_ref[:rows]) and torch.equal(aux_out[:rows], aux_ref[:rows])
    s_only = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    _ext._grouped_mm_swiglu_cuda(x, w_up, offs, b_up, None, s_only, 1.702, 7.0, False)
    assert torch.equal(s_only[:rows], s_ref[:rows])
    g_ref = torch.ops.grouped_mm.mm_swiglu_bwd(gout, w_down.cuda().transpose(-2, -1), offs, aux_ref, 1.702, 7.0)
    g_packed = torch.empty(M, I, dtype=torch.float32, device="cuda")
    _ext._grouped_mm_swiglu_bwd_cuda(gout, w_down.cuda().transpose(-2, -1), offs, aux_ref.view(torch.float32),
                                     g_packed, 1.702, 7.0)
    torch.cuda.synchronize()
    m.check_device_status()
    assert torch.equal(g_packed.view(torch.bfloat16)[:rows], g_ref[:rows])
    out = _ext._grouped_mm_cuda(s_ref, w_down.cuda(), offs, None, None)
    assert torch.equal(out[:rows], m.grouped_mm(s_ref, w_down.cuda(), offs)[:rows])


def test_rows_past_offs_end_are_never_written():
    """offs[-1] < rows of the buffers: the in-place binding functions leave every row at or past
    offs[-1] untouched (NaN-prefilled here) in swiglu_out, aux_out and the packed grad_aux."""
    m = _lib()
    from cutlass_op.bf16_grouped_mm import _ext
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    x, w_up, b_up, w_down, b_down, offs, gout = small_case(3, 128, 64, [70, 0, 131], seed=23)
    M, I = x.shape[0] + 77, w_up.shape[2] // 2    # 77 rows past offs[-1]
    xp = torch.cat([x, torch.randn(77, x.shape[1]).to(torch.bfloat16)]).cuda()
    gp = torch.cat([gout, torch.randn(77, gout.shape[1]).to(torch.bfloat16)]).cuda()
    w_up, b_up, w_down, offs = (t.cuda() for t in (w_up, b_up, w_down, offs))
    rows = int(offs[-1])
    nan = float("nan")
    s_out = torch.full((M, I), nan, dtype=torch.bfloat16, device="cuda")
    aux_out = torch.full((M, 2 * I), nan, dtype=torch.bfloat16, device="cuda")
    _ext._grouped_mm_swiglu_cuda(xp, w_up, offs, b_up, aux_out, s_out, 1.702, 7.0, True)
    g_packed = torch.full((M, 2 * I), nan, dtype=torch.bfloat16, device="cuda").view(torch.float32)
    _ext._grouped_mm_swiglu_bwd_cuda(gp, w_down.transpose(-2, -1), offs, aux_out.view(torch.float32), g_packed,
                                     1.702, 7.0)
    torch.cuda.synchronize()
    m.check_device_status()
    assert torch.isnan(s_out[rows:].float()).all() and torch.isnan(aux_out[rows:].float()).all()
    assert torch.isnan(g_packed.view(torch.bfloat16)[rows:].float()).all()
    assert not torch.isnan(s_out[:rows].float()).any() and not torch.isnan(aux_out[:rows].float()).any()
    assert not torch.isnan(g_packed.view(torch.bfloat16)[:rows].float()).any()
    ref = O.kernel_chain(x, *(t.cpu() for t in (w_up, b_up, w_down)), b_down, offs.cpu(), gout)
    for name, got in (("swiglu_out", s_out), ("aux", aux_out), ("grad_aux", g_packed.view(torch.bfloat16))):
        r = O.check(name, got[:rows].float().cpu(), ref[name][:rows])
        assert r["ok"], r


def test_group_range_launches_equal_one_launch():
    """Two launches over the expert ranges [0, h) and [h, E) of one offs array (group_begin), writing
    into the same outputs, give the single launch's results bit for bit (single CTAs and pairs)."""
    import os

    _lib()
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    for cg in ("1", "2"):
        os.environ["MGF_CTA_GROUP"] = cg
        try:
            x, w_up, b_up, _, _, offs, _ = small_case(6, 256, 128, [300, 0, 517, 41, 600, 1], seed=41)
            x, w_up, b_up, offs = (t.cuda() for t in (x, w_up, b_up, offs))
            s_ref, aux_ref = torch.ops.grouped_mm.mm_swiglu(x, w_up, offs, b_up, 1.702, 7.0)
            M, I = x.shape[0], w_up.shape[2] // 2
            s = torch.full((M, I), float("nan"), dtype=torch.bfloat16, device="cuda")
            aux = torch.full((M, 2 * I), float("nan"), dtype=torch.bfloat16, device="cuda")
            h = 3
            torch.ops.grouped_mm.swiglu_range_into(x, w_up[:h], offs[:h], b_up[:h], aux, s, 1.702, 7.0, True, 0)
            torch.ops.grouped_mm.swiglu_range_into(x, w_up, offs, b_up, aux, s, 1.702, 7.0, True, h)
            torch.cuda.synchronize()
            assert torch.equal(s, s_ref) and torch.equal(aux, aux_ref), cg
        finally:
            del os.environ["MGF_CTA_GROUP"]


def test_backward_range_launches_equal_one_launch():
    """The weight + bias gradient (ragged-K) and the dgrad + SwiGLU backward split into the expert
    ranges [0, h) and [h, E) (group_begin) equal the single launches bit for bit, empty groups included."""
    _lib()
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    x, w_up, b_up, w_down, b_down, offs, gout = small_case(6, 256, 128, [300, 0, 517, 41, 600, 1], seed=43)
    x, w_up, b_up, w_down, offs, gout = (t.cuda() for t in (x, w_up, b_up, w_down, offs, gout))
    s, aux = torch.ops.grouped_mm.mm_swiglu(x, w_up, offs, b_up, 1.702, 7.0)
    h = 3
    dw_ref, db_ref = torch.ops.grouped_mm.mm_wgrad_bias(s.transpose(-2, -1), gout, offs)
    E, I, H = w_down.shape
    dw = torch.full((E, I, H), float("nan"), dtype=torch.bfloat16, device="cuda")
    db = torch.full((E, H), float("nan"), dtype=torch.bfloat16, device="cuda")
    torch.ops.grouped_mm.wgrad_bias_into(s.transpose(-2, -1), gout, offs[:h], dw[:h], db[:h], 0)
    torch.ops.grouped_mm.wgrad_bias_into(s.transpose(-2, -1), gout, offs, dw, db, h)
    ga_ref = torch.ops.grouped_mm.mm_swiglu_bwd(gout, w_down.transpose(-2, -1), offs, aux, 1.702, 7.0)
    ga = torch.full_like(aux, float("nan"))
    w_t = w_down.transpose(-2, -1)
    torch.ops.grouped_mm.swiglu_bwd_range_into(gout, w_t[:h], offs[:h], aux, ga, 1.702, 7.0, 0)
    torch.ops.grouped_mm.swiglu_bwd_range_into(gout, w_t, offs, aux, ga, 1.702, 7.0, h)
    torch.cuda.synchronize()
    assert torch.equal(dw, dw_ref) and torch.equal(db, db_ref.to(db.dtype))
    assert torch.equal(ga, ga_ref)


@pytest.mark.parametrize("m,n,counts", [
    (256, 128, [300, 0, 517, 41, 600, 1]),   # average above the small-K threshold
    (136, 80, [70, 0, 131, 5]),              # m and n tails, the ones row inside the last tile
    (128, 64, [129, 255, 0]),                # m % 128 == 0: the ones row in a tile of its own
    (384, 256, [1, 7, 129, 0, 64, 33, 200]),
    (200, 2240, [50, 0, 130, 7]),            # BN = 256, last n tile 192 wide: a warp half of one 64-col chunk
    (72, 448, [3, 260, 0, 64]),              # BN = 128, last n tile 64 wide; m tail inside a warp's rows
])
def test_wgrad_staging_forms_equal(m, n, counts, monkeypatch):
    """The ragged-K weight + bias gradient stored as 32 x 32 chunks and in the wide small-K form
    (one TMA store of all a warp's chunks per tile) give the same bits, and match the oracle."""
    _lib()
    g = torch.Generator().manual_seed(m + n)
    rows = sum(counts)
    a = torch.randn(rows, m, generator=g).to(torch.bfloat16)
    b = torch.randn(rows, n, generator=g).to(torch.bfloat16)
    offs = torch.tensor(counts).cumsum(0).to(torch.int32)
    out = {}
    for form in ("0", "1"):
        monkeypatch.setenv("MGF_WGRAD_SMALL_K", form)
        dw, db = torch.ops.grouped_mm.mm_wgrad_bias(a.cuda().t(), b.cuda(), offs.cuda())
        torch.cuda.synchronize()
        out[form] = (dw.cpu(), db.cpu())
    assert torch.equal(out["0"][0], out["1"][0]) and torch.equal(out["0"][1], out["1"][1])
    ref_dw, ref_db = O.grouped_wgrad(a, b, offs)
    _assert_close("dw", out["1"][0], ref_dw)
    _assert_close("db", out["1"][1], ref_db)


@pytest.mark.parametrize("m,n,counts", [
    (2880, 2880, [300, 0, 517, 1000]),   # last 256-row tile holds 64 rows + the ones row: upper half skipped
    (384, 512, [700, 0, 900]),           # the ones row opens the upper half of the last tile
    (512, 256, [400, 300]),              # m % 256 == 0: the bias-gradient row in a tile of its own
    (200, 2304, [333, 290, 0, 411]),     # one tile, both halves partly filled
])
def test_wgrad_256_row_tiles_equal_128_row_tiles(m, n, counts, monkeypatch):
    """The weight + bias gradient with 256-row single-CTA tiles (two accumulators sharing each B
    stage) gives the same bits as 128-row tiles, and matches the oracle."""
    _lib()
    g = torch.Generator().manual_seed(m * 3 + n)
    rows = sum(counts)
    a = torch.randn(rows, m, generator=g).to(torch.bfloat16)
    b = torch.randn(rows, n, generator=g).to(torch.bfloat16)
    offs = torch.tensor(counts).cumsum(0).to(torch.int32)
    monkeypatch.setenv("MGF_CTA_GROUP", "1")
    out = {}
    for form in ("0", "1"):
        monkeypatch.setenv("MGF_WGRAD_M256", form)
        dw, db = torch.ops.grouped_mm.mm_wgrad_bias(a.cuda().t(), b.cuda(), offs.cuda())
        torch.cuda.synchronize()
        out[form] = (dw.cpu(), db.cpu())
    assert torch.equal(out["0"][0], out["1"][0]) and torch.equal(out["0"][1], out["1"][1])
    ref_dw, ref_db = O.grouped_wgrad(a, b, offs)
    _assert_close("dw", out["1"][0], ref_dw)
    _assert_close("db", out["1"][1], ref_db)
