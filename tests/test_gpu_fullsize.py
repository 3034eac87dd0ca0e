"""Parity at the full fwd+bwd benchmark size (E=32, H=I=2880, 24576 tokens top-4 Zipf(1.1), two empty
experts, 98304 routed rows): one fwd+bwd through the wrappers, then spot checks against the oracle's
rounding chain on slices the CPU computes in seconds -- sampled rows of out and dx from every
non-empty expert, sampled columns of both weight gradients and the full bias gradients of the
smallest and of the largest expert (the longest ragged-K accumulation, where the dynamic tile
counter and long fp32 sums matter), and exact zeros for the empty experts.

A second test does the same at the fine-grained shape E=256, H=7168, I=2048, 4096 tokens top-8
(Zipf(1.3) with forced groups of 0, 1, 7 and 129 rows): sampled rows of out and dx, and the FULL
weight and bias gradients of the 1-, 7- and 129-row experts.

Tolerance: max|err|/max|ref| <= 1e-2 and float64 cosine >= 0.9999 on every checked slice.
"""

from __future__ import annotations

import pytest
import torch

from oracle import moe_ffn as O

pytestmark = pytest.mark.gpu

ALPHA, LIMIT = 1.702, 7.0


def _check(name, got, ref):
    r = O.check(name, got.float().cpu(), ref.float().cpu())
    assert r["ok"], f"{name}: rel={r['rel']:.3e} cos={r['cos']:.7f}"


def test_cfg3_full_size_spot_checks():
    import cutlass_op.bf16_grouped_mm as m
    from cutlass_op.bf16_grouped_mm.workloads import MoEShape, make_weights_device, offs_from_counts, zipf_routing

    E, H, I = 32, 2880, 2880
    counts = zipf_routing(24576, E, 4, 1.1, seed=0, zero_experts=2)
    offs = offs_from_counts(counts)
    M = int(counts.sum())
    dev = torch.device("cuda")
    x = torch.randn(M, H, generator=torch.Generator(device=dev).manual_seed(1), device=dev).to(torch.bfloat16)
    w_up, b_up, w_down, b_down = make_weights_device(MoEShape(E, H, I), seed=2, device=dev)
    leaves = [t.clone().requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
    xl, wu, bu, wd, bd = leaves
    s, aux = m.grouped_mm_swiglu(xl, wu, offs.to(dev), bu, ALPHA, LIMIT)
    out = m.grouped_mm_downproj(s, wd, offs.to(dev), bd, aux, ALPHA, LIMIT)
    out.sum().backward()  # grad_out = ones
    torch.cuda.synchronize()
    m.check_device_status()

    ends = offs.tolist()
    starts = [0] + ends[:-1]
    wu_c, bu_c, wd_c, bd_c = (t.detach().cpu() for t in (w_up, b_up, w_down, b_down))
    g = torch.Generator().manual_seed(5)
    # sampled rows of every non-empty expert: out and dx through the oracle's rounding chain
    rows = []
    for e in range(E):
        if ends[e] > starts[e]:
            rows += torch.randint(starts[e], ends[e], (4,), generator=g).tolist()
    rows_t = torch.tensor(rows)
    exp_of = torch.bucketize(rows_t, torch.tensor(ends), right=True)
    xr = x[rows_t.to(dev)].cpu()
    ref_out, ref_dx = [], []
    for i, e in enumerate(exp_of.tolist()):
        a = O._bf16(xr[i:i + 1].float() @ wu_c[e].float() + bu_c[e].float())
        sw = O._bf16(O.swiglu_fwd(a))
        ref_out.append(O._bf16(sw @ wd_c[e].float() + bd_c[e].float()))
        gs = torch.ones(1, H) @ wd_c[e].float().t()
        ga = O._bf16(O.swiglu_bwd(gs, a))
        ref_dx.append(O._bf16(ga @ wu_c[e].float().t()))
    _check("out rows", out.detach()[rows_t.to(dev)], torch.cat(ref_out))
    _check("dx rows", xl.grad[rows_t.to(dev)], torch.cat(ref_dx))

    # the smallest and the largest expert: sampled weight-gradient columns and both bias gradients
    nonempty = [e for e in range(E) if ends[e] > starts[e]]
    for e in (min(nonempty, key=lambda j: ends[j] - starts[j]), max(nonempty, key=lambda j: ends[j] - starts[j])):
        xe = x[starts[e]:ends[e]].float().cpu()
        a = O._bf16(xe @ wu_c[e].float() + bu_c[e].float())
        sw = O._bf16(O.swiglu_fwd(a))
        ge = torch.ones(ends[e] - starts[e], H)
        ga = O._bf16(O.swiglu_bwd(ge @ wd_c[e].float().t(), a))
        cols_h = torch.randint(0, H, (16,), generator=g)
        cols_2i = torch.randint(0, 2 * I, (16,), generator=g)
        tag = f"expert {e} ({ends[e] - starts[e]} rows)"
        _check(f"dW_down cols {tag}", wd.grad[e][:, cols_h.to(dev)], O._bf16(sw.t() @ ge[:, cols_h]))
        _check(f"dW_up cols {tag}", wu.grad[e][:, cols_2i.to(dev)], O._bf16(xe.t() @ ga[:, cols_2i]))
        _check(f"db_down {tag}", bd.grad[e], O._bf16(ge.sum(0)))
        _check(f"db_up {tag}", bu.grad[e], O._bf16(ga.sum(0)))
    for j in range(E):
        if ends[j] == starts[j]:
            for name, t in (("dW_up", wu.grad[j]), ("db_up", bu.grad[j]), ("dW_down", wd.grad[j]), ("db_down", bd.grad[j])):
                assert torch.count_nonzero(t).item() == 0, f"{name}[{j}] of an empty expert is not zero"


def test_cfg5_full_width_spot_checks():
    """E=256, H=7168 (112 K-blocks in the up-projection), I=2048 (2I = 4096, whole 256-column tiles),
    4096 tokens top-8 with forced groups of 0, 1, 7 and 129 rows, random output gradient."""
    import cutlass_op.bf16_grouped_mm as m
    from cutlass_op.bf16_grouped_mm.workloads import MoEShape, config5_counts, make_weights_device, offs_from_counts

    E, H, I = 256, 7168, 2048
    counts = config5_counts(4096, E, 8, seed=0)
    for sz in (0, 1, 7, 129):
        assert sz in counts.tolist()
    offs = offs_from_counts(counts)
    M = int(counts.sum())
    dev = torch.device("cuda")
    gd = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(M, H, generator=gd, device=dev).to(torch.bfloat16)
    gout = torch.randn(M, H, generator=gd, device=dev).to(torch.bfloat16)
    w_up, b_up, w_down, b_down = make_weights_device(MoEShape(E, H, I), seed=12, device=dev)
    leaves = [t.clone().requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
    xl, wu, bu, wd, bd = leaves
    s, aux = m.grouped_mm_swiglu(xl, wu, offs.to(dev), bu, ALPHA, LIMIT)
    out = m.grouped_mm_downproj(s, wd, offs.to(dev), bd, aux, ALPHA, LIMIT)
    out.backward(gout)
    torch.cuda.synchronize()
    m.check_device_status()

    ends = offs.tolist()
    starts = [0] + ends[:-1]
    sizes = [b - a for a, b in zip(starts, ends)]
    g = torch.Generator().manual_seed(13)
    forced = [sizes.index(sz) for sz in (1, 7, 129)]
    biggest = max(range(E), key=lambda j: sizes[j])
    sampled = sorted(set(forced + [biggest] + torch.randperm(E, generator=g)[:24].tolist()))
    for e in sampled:
        if sizes[e] == 0:
            for name, t in (("dW_up", wu.grad[e]), ("db_up", bu.grad[e]), ("dW_down", wd.grad[e]),
                            ("db_down", bd.grad[e])):
                assert torch.count_nonzero(t).item() == 0, f"{name}[{e}] of an empty expert is not zero"
            continue
        full = e in forced
        rows = torch.arange(starts[e], ends[e]) if full else \
            torch.randint(starts[e], ends[e], (min(4, sizes[e]),), generator=g)
        rd = rows.to(dev)
        wu_e, bu_e, wd_e, bd_e = (t[e].detach().float().cpu() for t in (w_up, b_up, w_down, b_down))
        xr, gr = x[rd].float().cpu(), gout[rd].float().cpu()
        a = O._bf16(xr @ wu_e + bu_e)
        sw = O._bf16(O.swiglu_fwd(a))
        ga = O._bf16(O.swiglu_bwd(gr @ wd_e.t(), a))
        tag = f"expert {e} ({sizes[e]} rows)"
        _check(f"out {tag}", out.detach()[rd], O._bf16(sw @ wd_e + bd_e))
        _check(f"dx {tag}", xl.grad[rd], O._bf16(ga @ wu_e.t()))
        if full:  # every row of the group: the whole weight and bias gradients
            _check(f"dW_up {tag}", wu.grad[e], O._bf16(xr.t() @ ga))
            _check(f"db_up {tag}", bu.grad[e], O._bf16(ga.sum(0)))
            _check(f"dW_down {tag}", wd.grad[e], O._bf16(sw.t() @ gr))
            _check(f"db_down {tag}", bd.grad[e], O._bf16(gr.sum(0)))
