"""CPU stand-in for the reference's compiled `_ext` module -- TEST INFRASTRUCTURE ONLY.

Only tests/, tests/golden/make_golden.py and bench.py's reference / cpu_baseline legs use this
module, as the checker or the timed CPU baseline; the product path never imports it.

Butterfingrz/CuTe-MoE-Train's Python layer (cutlass_op/bf16_grouped_mm/__init__.py and
custom_op.py) calls three pybind functions of its CUDA extension (csrc/binding.cu:120-148).  The
extension needs sm_90a and an un-vendored CUTLASS fork, so it cannot be built anywhere here.  This
module restates the three functions on the CPU with the kernels' arithmetic, so the reference's own,
unmodified Python layer (autograd routing, fused-only contract, ZeroTensor handling,
_segment_sum_rows) can run on top of it:

* ``_grouped_mm_cuda``: fp32 accumulate + bias, one bf16 rounding (csrc/grouped_mm_kernel.cuh:130-143);
  ragged-K outputs of empty groups are written as zeros.
* ``_grouped_mm_swiglu_cuda``: aux = bf16(acc + bias); SwiGLU evaluated in bf16 arithmetic with a
  bf16 tanh, step by step as csrc/grouped_mm_swiglu_visitor.cuh:309-334.
* ``_grouped_mm_swiglu_bwd_cuda``: fp32 SwiGLU backward on (gate, up) pairs with tanh-based
  sigmoid (csrc/grouped_mm_swiglu_bwd_visitor.cuh:35-68).

``load_reference_layer`` imports the reference's two Python files from a directory (the git-ignored
staged copy ``baseline/_ref/group_gemm`` written by baseline/stage_reference.py, or the reference
checkout itself) under a private module name with a given `_ext`.  The layer registers operators
in the ``grouped_mm`` namespace, so it must not be loaded into a process that also loads this
repository's native operators.
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import torch


def _bf(t):
    return t.to(torch.bfloat16)


def _segments(offs):
    prev = 0
    for e, end in enumerate(offs.tolist()):
        yield e, prev, int(end)
        prev = int(end)


def make_module(name: str = "ref_bf16_grouped_mm._ext") -> types.ModuleType:
    """A module object with the three entry points of the reference's `_ext`, computed on the CPU."""
    m = types.ModuleType(name)

    def _grouped_mm_cuda(mat_a, mat_b, offs=None, bias=None, out_dtype=None):
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

    def _grouped_mm_swiglu_cuda(mat_a, mat_b, offs, bias, aux_out=None, swiglu_out=None, swiglu_alpha=1.702,
                                swiglu_limit=7.0, store_aux=True):
        aux = _grouped_mm_cuda(mat_a, mat_b, offs, bias, None)
        if store_aux:
            aux_out.copy_(aux)
        bf = torch.bfloat16
        g = aux[:, 0::2]
        u = aux[:, 1::2]
        lim = torch.tensor(swiglu_limit).to(bf)
        g = torch.minimum(g, lim)
        u = torch.maximum(torch.minimum(u, lim), -lim)
        ag = _bf(torch.tensor(swiglu_alpha * 0.5).to(bf).float() * g.float())
        t = _bf(torch.tanh(ag.float()))
        s = _bf(t.float() * 0.5 + 0.5)
        gs = _bf(g.float() * s.float())
        res = _bf(gs.float() * u.float() + gs.float())
        rows = int(offs[-1]) if offs.numel() else 0
        swiglu_out[:rows] = res[:rows]

    def _grouped_mm_swiglu_bwd_cuda(grad_output, down_w_t, offs, aux_packed, grad_gate_up_packed, swiglu_alpha,
                                    swiglu_limit):
        alpha, limit = swiglu_alpha, swiglu_limit
        aux = aux_packed.view(torch.bfloat16).float()
        grad = grad_gate_up_packed.view(torch.bfloat16)
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


def load_reference_layer(pkg_dir: Path, ext: types.ModuleType | None = None,
                         modname: str = "ref_bf16_grouped_mm") -> types.ModuleType:
    """Import the reference's __init__.py + custom_op.py from `pkg_dir`, unmodified, as `modname`,
    with `ext` (default: the CPU stand-in) as its `_ext` submodule."""
    pkg_dir = Path(pkg_dir)
    for f in ("__init__.py", "custom_op.py"):
        if not (pkg_dir / f).is_file():
            raise FileNotFoundError(f"reference layer file missing: {pkg_dir / f}")
    sys.modules[f"{modname}._ext"] = ext if ext is not None else make_module(f"{modname}._ext")
    spec = importlib.util.spec_from_file_location(modname, pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[modname] = mod
    spec.loader.exec_module(mod)
    return mod
