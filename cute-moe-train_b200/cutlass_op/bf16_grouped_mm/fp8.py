"""Forward-only FP8 (e4m3) variants of the ragged-M grouped GEMMs: ``grouped_mm::mm_fp8`` (+ bias) and
``grouped_mm::mm_swiglu_fp8`` (+ bias + clamped SwiGLU, returning ``(swiglu_out, aux_biased_acc)``).

The reference lists FP8 on its roadmap (README.md:99-102) without fixing a recipe; this one is
row-wise scaling: every token row of A has an fp32 scale, every output column of every expert's B has
one, the tensor cores accumulate e4m3 x e4m3 products in fp32 (``tcgen05.mma kind::f8f6f4``), and the
epilogue multiplies the accumulator by ``scale_a[row] * scale_b[e, col]`` before the bf16 bias and
SwiGLU -- the same epilogues, and the same bf16 outputs, as the bf16 operators.

B is taken as ``[E, K, N]`` with unit stride along K, i.e. the transpose of a contiguous [E, N, K]
tensor (``quantize_weights`` produces it).  Gradients are not defined for these operators.
"""

from __future__ import annotations

import torch

from . import _ext  # noqa: F401  (registers the operators)
from .custom_op import _padded
from .optimer import timed

E4M3_MAX = 448.0


@torch.library.register_fake("grouped_mm::mm_fp8")
def _mm_fp8_fake(mat_a, mat_b, offs, scale_a, scale_b, bias):
    n = mat_b.size(-1)
    return torch.empty_strided((mat_a.size(0), n), (_padded(n, torch.bfloat16), 1), dtype=torch.bfloat16,
                               device=mat_a.device)


@torch.library.register_fake("grouped_mm::mm_swiglu_fp8")
def _mm_swiglu_fp8_fake(mat_a, mat_b, offs, scale_a, scale_b, bias, swiglu_alpha, swiglu_limit):
    n = mat_b.size(-1)
    m = mat_a.size(0)
    s = torch.empty_strided((m, n // 2), (_padded(n // 2, torch.bfloat16), 1), dtype=torch.bfloat16,
                            device=mat_a.device)
    aux = torch.empty_strided((m, n), (_padded(n, torch.bfloat16), 1), dtype=torch.bfloat16, device=mat_a.device)
    return s, aux


def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[M, K] -> (e4m3 [M, K] with a 16-byte row pitch, fp32 [M] scales): x ~= q * scale[:, None]."""
    amax = x.detach().abs().amax(dim=1).float().clamp_min(1e-12)
    scale = amax / E4M3_MAX
    k = x.shape[1]
    kp = (k + 15) // 16 * 16
    q = torch.empty_strided((x.shape[0], k), (kp, 1), dtype=torch.float8_e4m3fn, device=x.device)
    q.copy_((x.float() / scale[:, None]).clamp_(-E4M3_MAX, E4M3_MAX))
    return q, scale.contiguous()


def quantize_weights(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[E, K, N] -> (e4m3 [E, K, N] view with unit stride along K, fp32 [E, N] scales):
    w[e, :, n] ~= q[e, :, n] * scale[e, n]."""
    amax = w.detach().abs().amax(dim=1).float().clamp_min(1e-12)  # [E, N]
    scale = amax / E4M3_MAX
    e, k, n = w.shape
    kp = (k + 15) // 16 * 16
    qt = torch.zeros((e, n, kp), dtype=torch.float8_e4m3fn, device=w.device)[:, :, :k]  # [E, N, K]
    qt.copy_((w.float() / scale[:, None, :]).clamp_(-E4M3_MAX, E4M3_MAX).transpose(1, 2))
    return qt.transpose(1, 2), scale.contiguous()


def dequantize_rows(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() * scale[:, None]


def dequantize_weights(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() * scale[:, None, :]


def grouped_mm_fp8(mat_a: torch.Tensor, mat_b: torch.Tensor, offs: torch.Tensor, scale_a: torch.Tensor,
                   scale_b: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """Ragged-M e4m3 grouped GEMM with row-wise scales (+ per-expert bf16 bias) -> bf16 [total_M, N]."""
    with timed("fp8_mm"):
        return torch.ops.grouped_mm.mm_fp8(mat_a, mat_b, offs, scale_a, scale_b, bias)


def grouped_mm_swiglu_fp8(mat_a: torch.Tensor, mat_b: torch.Tensor, offs: torch.Tensor, scale_a: torch.Tensor,
                          scale_b: torch.Tensor, bias: torch.Tensor, swiglu_alpha: float = 1.702,
                          swiglu_limit: float = 7.0) -> tuple[torch.Tensor, torch.Tensor]:
    """e4m3 up-projection + bias + clamped SwiGLU -> (swiglu_out [total_M, I], aux_biased_acc [total_M, 2I])."""
    with timed("fp8_up_swiglu_fwd"):
        return torch.ops.grouped_mm.mm_swiglu_fp8(mat_a, mat_b, offs, scale_a, scale_b, bias, swiglu_alpha,
                                                  swiglu_limit)
