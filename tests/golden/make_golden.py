"""Generate tests/golden/moe_ffn_golden.pt from the reference's own Python layer.

Run in the build container (the reference is mounted read-only at REF_ROOT; nothing at test time
reads it):

    python tests/golden/make_golden.py REF_ROOT

It loads Butterfingrz/CuTe-MoE-Train's ``cutlass_op/bf16_grouped_mm/__init__.py`` and
``custom_op.py`` unmodified under the module name ``ref_bf16_grouped_mm`` and injects a CPU
stand-in for its compiled ``_ext`` module.  The reference's autograd routing, fused-only contract,
ZeroTensor handling and ``_segment_sum_rows`` therefore run as written; only the three CUDA entry
points are restated here, with the reference kernels' arithmetic:

* ``_grouped_mm_cuda``: fp32 accumulate + bias, one bf16 rounding (csrc/grouped_mm_kernel.cuh:130-143);
  ragged-K outputs of empty groups are written as zeros.
* ``_grouped_mm_swiglu_cuda``: aux = bf16(acc + bias); SwiGLU evaluated in bf16 arithmetic with a
  bf16 tanh, step by step as csrc/grouped_mm_swiglu_visitor.cuh:309-334.
* ``_grouped_mm_swiglu_bwd_cuda``: fp32 SwiGLU backward on (gate, up) pairs with tanh-based
  sigmoid (csrc/grouped_mm_swiglu_bwd_visitor.cuh:35-68).

The ops it registers live in the ``grouped_mm`` namespace, so this script must not run in a
process that also loads this repository's native operators.
"""

from __future__ import annotations

import importlib.util
import math
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "moe_ffn_golden.pt"

CASES = [
    # name, E, H, I, tokens per expert, seed, grad
    ("mixed_empty", 4, 64, 32, [16, 0, 37, 11], 1, "randn"),
    ("odd_sizes", 3, 128, 64, [1, 7, 129], 2, "randn"),
    ("single_expert", 1, 64, 64, [200], 3, "randn"),
    ("leading_trailing_empty", 5, 64, 48, [0, 33, 64, 5, 0], 4, "ones"),
    ("all_empty", 2, 64, 32, [0, 0], 5, "randn"),
]


def _bf(t):
    return t.to(torch.bfloat16)


def _segments(offs):
    prev = 0
    for e, end in enumerate(offs.tolist()):
        yield e, prev, int(end)
        prev = int(end)


def _stub_ext():
    m = types.ModuleType("ref_bf16_grouped_mm._ext")

    def _grouped_mm_cuda(mat_a, mat_b, offs, bias, out_dtype):
        a2, b2 = mat_a.dim() == 2, mat_b.dim() == 2
        if a2 and not b2:
            n = mat_b.shape[-1]
            out = torch.zeros(mat_a.shape[0], n, dtype=torch.bfloat16)
            for e, s, t in _segments(offs):
                if t > s:
                    y = mat_a[s:t].float() @ mat_b[e].float()
                    if bias is not None:
                        y = y + bias[e].float()
                    out[s:t] = _bf(y)
            return out
        if a2 and b2:
            E = offs.numel()
            out = torch.zeros(E, mat_a.shape[0], mat_b.shape[1], dtype=torch.bfloat16)
            for e, s, t in _segments(offs):
                if t > s:
                    out[e] = _bf(mat_a[:, s:t].float() @ mat_b[s:t].float())
            return out
        y = mat_a.float() @ mat_b.float()
        if bias is not None:
            y = y + bias.float().unsqueeze(-2)
        return _bf(y)

    def _grouped_mm_swiglu_cuda(mat_a, mat_b, offs, bias, aux_out, swiglu_out, alpha, limit, store_aux):
        aux = _grouped_mm_cuda(mat_a, mat_b, offs, bias, None)
        if store_aux:
            aux_out.copy_(aux)
        bf = torch.bfloat16
        g = aux[:, 0::2]
        u = aux[:, 1::2]
        lim = torch.tensor(limit).to(bf)
        g = torch.minimum(g, lim)
        u = torch.maximum(torch.minimum(u, lim), -lim)
        ag = _bf(torch.tensor(alpha * 0.5).to(bf).float() * g.float())
        t = _bf(torch.tanh(ag.float()))
        s = _bf(t.float() * 0.5 + 0.5)
        gs = _bf(g.float() * s.float())
        res = _bf(gs.float() * u.float() + gs.float())
        rows = int(offs[-1]) if offs.numel() else 0
        swiglu_out[:rows] = res[:rows]

    def _grouped_mm_swiglu_bwd_cuda(grad_output, down_w_t, offs, aux_packed, grad_packed, alpha, limit):
        aux = aux_packed.view(torch.bfloat16).float()
        grad = grad_packed.view(torch.bfloat16)
        for e, s, t in _segments(offs):
            if t <= s:
                continue
            gs = grad_output[s:t].float() @ down_w_t[e].float()
            gate = aux[s:t, 0::2]
            up = aux[s:t, 1::2]
            gc = torch.clamp(gate, max=limit)
            uc = torch.clamp(up, min=-limit, max=limit)
            sig = 0.5 * torch.tanh(0.5 * alpha * gc) + 0.5
            glu = gc * sig
            dg = gs * (uc + 1.0) * sig * (1.0 + alpha * gc * (1.0 - sig))
            du = gs * glu
            dg = dg * (gate <= limit).float()
            du = du * ((up >= -limit) & (up <= limit)).float()
            grad[s:t, 0::2] = _bf(dg)
            grad[s:t, 1::2] = _bf(du)

    m._grouped_mm_cuda = _grouped_mm_cuda
    m._grouped_mm_swiglu_cuda = _grouped_mm_swiglu_cuda
    m._grouped_mm_swiglu_bwd_cuda = _grouped_mm_swiglu_bwd_cuda
    return m


def load_reference(ref_root: Path):
    pkg_dir = ref_root / "cutlass_op" / "bf16_grouped_mm"
    sys.modules["ref_bf16_grouped_mm._ext"] = _stub_ext()
    spec = importlib.util.spec_from_file_location(
        "ref_bf16_grouped_mm", pkg_dir / "__init__.py", submodule_search_locations=[str(pkg_dir)]
    )
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_bf16_grouped_mm"] = mod
    spec.loader.exec_module(mod)
    return mod


def make_inputs(E, H, I, counts, seed, grad):
    # Same draw order as cutlass_op/bf16_grouped_mm/workloads.py::small_case.
    g = torch.Generator().manual_seed(seed)
    M = int(sum(counts))
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w_up = (torch.randn(E, H, 2 * I, generator=g) / math.sqrt(H)).to(torch.bfloat16)
    b_up = (torch.randn(E, 2 * I, generator=g) * 0.02).to(torch.bfloat16)
    w_down = (torch.randn(E, I, H, generator=g) / math.sqrt(I)).to(torch.bfloat16)
    b_down = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    gout = torch.ones(M, H).to(torch.bfloat16) if grad == "ones" else torch.randn(M, H, generator=g).to(torch.bfloat16)
    offs = torch.cumsum(torch.tensor(counts, dtype=torch.int64), 0).to(torch.int32)
    return x, w_up, b_up, w_down, b_down, offs, gout


def run_reference(ref, x, w_up, b_up, w_down, b_down, offs, gout):
    leaves = [t.clone().requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
    xl, wu, bu, wd, bd = leaves
    swiglu_out, aux = ref.grouped_mm_swiglu(xl, wu, offs=offs, bias=bu, swiglu_alpha=1.702, swiglu_limit=7.0)
    out = ref.grouped_mm_downproj(swiglu_out, wd, offs=offs, bias=bd, aux_biased_acc=aux,
                                  swiglu_alpha=1.702, swiglu_limit=7.0)
    (out.float() * gout.float()).sum().backward()
    return {
        "swiglu_out": swiglu_out.detach(), "aux": aux.detach(), "out": out.detach(),
        "dx": xl.grad, "dw_up": wu.grad, "db_up": bu.grad, "dw_down": wd.grad, "db_down": bd.grad,
    }


def main():
    if len(sys.argv) < 2:
        raise SystemExit("usage: python tests/golden/make_golden.py REF_ROOT  (the reference project's root)")
    ref_root = Path(sys.argv[1])
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = load_reference(ref_root)
    fixtures = {"cases": {}, "generator": "tests/golden/make_golden.py", "alpha": 1.702, "limit": 7.0}
    for name, E, H, I, counts, seed, grad in CASES:
        inp = make_inputs(E, H, I, counts, seed, grad)
        outs = run_reference(ref, *inp)
        fixtures["cases"][name] = {
            "E": E, "H": H, "I": I, "counts": counts, "seed": seed, "grad": grad,
            "inputs": dict(zip(["x", "w_up", "b_up", "w_down", "b_down", "offs", "grad_out"], inp)),
            "outputs": {k: (v.to(torch.bfloat16) if v is not None else None) for k, v in outs.items()},
        }
        print(f"{name}: M={sum(counts)} done")
    torch.save(fixtures, OUT)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
