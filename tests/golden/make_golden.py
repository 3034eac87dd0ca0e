"""Generate tests/golden/moe_ffn_golden.pt from the reference's own Python layer.

Run in the build container (the reference is mounted read-only at REF_ROOT; nothing at test time
reads it):

    python tests/golden/make_golden.py REF_ROOT

It loads Butterfingrz/CuTe-MoE-Train's ``cutlass_op/bf16_grouped_mm/__init__.py`` and
``custom_op.py`` unmodified under the module name ``ref_bf16_grouped_mm`` and injects a CPU
stand-in for its compiled ``_ext`` module (oracle/ref_ext_cpu.py).  The reference's autograd
routing, fused-only contract, ZeroTensor handling and ``_segment_sum_rows`` therefore run as
written; only the three CUDA entry points are restated, with the reference kernels' arithmetic:

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

import math
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))  # the repository root, for oracle/
OUT = HERE / "moe_ffn_golden.pt"

CASES = [
    # name, E, H, I, tokens per expert, seed, grad
    ("mixed_empty", 4, 64, 32, [16, 0, 37, 11], 1, "randn"),
    ("odd_sizes", 3, 128, 64, [1, 7, 129], 2, "randn"),
    ("single_expert", 1, 64, 64, [200], 3, "randn"),
    ("leading_trailing_empty", 5, 64, 48, [0, 33, 64, 5, 0], 4, "ones"),
    ("all_empty", 2, 64, 32, [0, 0], 5, "randn"),
]


def load_reference(ref_root: Path):
    from oracle.ref_ext_cpu import load_reference_layer

    return load_reference_layer(ref_root / "cutlass_op" / "bf16_grouped_mm")


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
