"""FP8 (e4m3) variants of all four fused epilogues of the MoE FFN, and the FFN with autograd on them.

The reference lists FP8 on its roadmap (README.md:99-102) without fixing a recipe; this one scales
per row for the ragged-M GEMMs and per feature column for the ragged-K weight gradients:

* ``grouped_mm::mm_fp8`` (+ bias) and ``grouped_mm::mm_swiglu_fp8`` (+ bias + clamped SwiGLU):
  every token row of A has an fp32 scale, every output column of every expert's B has one, the tensor
  cores accumulate e4m3 x e4m3 products in fp32 (``tcgen05.mma kind::f8f6f4``) and the epilogue
  multiplies the accumulator by ``scale_a[row] * scale_b[e, col]`` before the bf16 bias and SwiGLU;
* ``grouped_mm::mm_swiglu_bwd_fp8``: the down-proj dgrad with the same row / column scales, the
  dequantised accumulator going into the SwiGLU backward against the bf16 aux;
* ``grouped_mm::mm_wgrad_fp8``: the ragged-K weight gradient (+ bias gradient) over token rows.  The
  contraction runs over tokens, so a per-token scale cannot be factored out; both operands are scaled
  per feature column instead (``quantize_cols``: one scale per column over all tokens), and the
  epilogue multiplies by ``scale_a[i] * scale_b[j]`` (the bias-gradient row by ``scale_b[j]``).

B of the ragged-M operators is ``[E, K, N]`` with unit stride along K, i.e. the transpose of a
contiguous [E, N, K] tensor (``quantize_weights`` produces it).  ``grouped_mm_ffn_fp8`` chains them
into the fused MoE FFN with autograd: forward ``x -> mm_swiglu_fp8 -> mm_fp8``, backward
``mm_wgrad_fp8`` (down), ``mm_swiglu_bwd_fp8``, ``mm_fp8`` (up dgrad), ``mm_wgrad_fp8`` (up); every
output and gradient is bf16, every GEMM operand is quantised right before its GEMM.
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


@torch.library.register_fake("grouped_mm::mm_swiglu_bwd_fp8")
def _mm_swiglu_bwd_fp8_fake(grad_output, down_w_t, offs, aux_biased_acc, scale_a, scale_b, swiglu_alpha,
                            swiglu_limit):
    n = 2 * down_w_t.size(-1)
    return torch.empty_strided((grad_output.size(0), n), (_padded(n, torch.bfloat16), 1), dtype=torch.bfloat16,
                               device=grad_output.device)


@torch.library.register_fake("grouped_mm::mm_wgrad_fp8")
def _mm_wgrad_fp8_fake(mat_a, mat_b, offs, scale_a, scale_b, bias_grad):
    e, m, n = offs.size(0), mat_a.size(0), mat_b.size(1)
    pn = _padded(n, torch.bfloat16)
    dw = torch.empty_strided((e, m, n), (m * pn, pn, 1), dtype=torch.bfloat16, device=mat_a.device)
    db = torch.empty((e, n), dtype=torch.bfloat16, device=mat_a.device) if bias_grad else \
        torch.empty(0, dtype=torch.bfloat16, device=mat_a.device)
    return dw, db


@torch.library.register_fake("grouped_mm::mm_swiglu_fp8")
def _mm_swiglu_fp8_fake(mat_a, mat_b, offs, scale_a, scale_b, bias, swiglu_alpha, swiglu_limit):
    n = mat_b.size(-1)
    m = mat_a.size(0)
    s = torch.empty_strided((m, n // 2), (_padded(n // 2, torch.bfloat16), 1), dtype=torch.bfloat16,
                            device=mat_a.device)
    aux = torch.empty_strided((m, n), (_padded(n, torch.bfloat16), 1), dtype=torch.bfloat16, device=mat_a.device)
    return s, aux


def _native(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0


def quantize_rows(x: torch.Tensor, native: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """[M, K] -> (e4m3 [M, K] with a 16-byte row pitch, fp32 [M] scales): x ~= q * scale[:, None].
    bf16 CUDA inputs go through the fused kernel (grouped_mm::fp8_quantize_rows); the torch expression
    below is the same formula (used for other dtypes, and by the tests as the reference)."""
    if native and _native(x) and x.stride(-1) == 1:
        with timed("fp8_quantize"):
            return torch.ops.grouped_mm.fp8_quantize_rows(x.detach())
    amax = x.detach().abs().amax(dim=1).float().clamp_min(1e-12)
    scale = amax / torch.full_like(amax, E4M3_MAX)  # true division, as the kernels
    k = x.shape[1]
    kp = (k + 15) // 16 * 16
    q = torch.empty_strided((x.shape[0], k), (kp, 1), dtype=torch.float8_e4m3fn, device=x.device)
    q.copy_((x.float() / scale[:, None]).clamp_(-E4M3_MAX, E4M3_MAX))
    return q, scale.contiguous()


def quantize_weights(w: torch.Tensor, native: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """[E, K, N] -> (e4m3 [E, K, N] view with unit stride along K, fp32 [E, N] scales):
    w[e, :, n] ~= q[e, :, n] * scale[e, n]."""
    if native and w.is_cuda and w.dtype == torch.bfloat16 and (w.stride(2) == 1 or w.stride(1) == 1):
        with timed("fp8_quantize"):
            return torch.ops.grouped_mm.fp8_quantize_weights(w.detach())
    amax = w.detach().abs().amax(dim=1).float().clamp_min(1e-12)  # [E, N]
    scale = amax / torch.full_like(amax, E4M3_MAX)  # true division, as the kernels
    e, k, n = w.shape
    kp = (k + 15) // 16 * 16
    qt = torch.zeros((e, n, kp), dtype=torch.float8_e4m3fn, device=w.device)[:, :, :k]  # [E, N, K]
    qt.copy_((w.float() / scale[:, None, :]).clamp_(-E4M3_MAX, E4M3_MAX).transpose(1, 2))
    return qt.transpose(1, 2), scale.contiguous()


def quantize_weights_both(w: torch.Tensor, native: bool = True):
    """[E, K, N] -> (quantize_weights(w), quantize_weights(w^T)) as (q, scale, q_t, scale_t): the forward's
    K-major B operand and the dgrad's, bit-identical to the two calls; with unit stride along N the fused
    kernel reads w twice instead of four times (grouped_mm::fp8_quantize_weights_both)."""
    if native and w.is_cuda and w.dtype == torch.bfloat16 and w.stride(2) == 1 and w.shape[2] % 8 == 0 \
            and w.stride(1) % 8 == 0 and w.stride(0) % 8 == 0 and w.data_ptr() % 16 == 0:
        with timed("fp8_quantize"):
            return torch.ops.grouped_mm.fp8_quantize_weights_both(w.detach())
    q, s = quantize_weights(w, native)
    q_t, s_t = quantize_weights(w.transpose(-2, -1), native)
    return q, s, q_t, s_t


def quantize_cols(x: torch.Tensor, native: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """[M, K] -> (e4m3 [M, K] with a 16-byte row pitch, fp32 [K] scales): x ~= q * scale[None, :]
    (one scale per feature column over all rows: the weight-gradient operands)."""
    if native and _native(x) and x.stride(-1) == 1:
        with timed("fp8_quantize"):
            return torch.ops.grouped_mm.fp8_quantize_cols(x.detach())
    amax = (x.detach().abs().amax(dim=0).float() if x.shape[0] else
            torch.zeros(x.shape[1], device=x.device)).clamp_min(1e-12)
    scale = amax / torch.full_like(amax, E4M3_MAX)  # true division, as the kernels
    k = x.shape[1]
    kp = (k + 15) // 16 * 16
    q = torch.empty_strided((x.shape[0], k), (kp, 1), dtype=torch.float8_e4m3fn, device=x.device)
    q.copy_((x.float() / scale[None, :]).clamp_(-E4M3_MAX, E4M3_MAX))
    return q, scale.contiguous()


def quantize_rows_cols(x: torch.Tensor, native: bool = True):
    """[M, K] -> (quantize_rows(x), quantize_cols(x)) as (q_r, s_r, q_c, s_c), bit-identical to the two
    calls; the fused kernel (grouped_mm::fp8_quantize_rows_cols) reads x twice instead of three times."""
    if native and _native(x) and x.stride(-1) == 1:
        with timed("fp8_quantize"):
            return torch.ops.grouped_mm.fp8_quantize_rows_cols(x.detach())
    q_r, s_r = quantize_rows(x, native)
    q_c, s_c = quantize_cols(x, native)
    return q_r, s_r, q_c, s_c


def dequantize_cols(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() * scale[None, :]


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


def grouped_mm_swiglu_bwd_fp8(grad_output: torch.Tensor, down_w_t: torch.Tensor, offs: torch.Tensor,
                              aux_biased_acc: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                              swiglu_alpha: float = 1.702, swiglu_limit: float = 7.0) -> torch.Tensor:
    """e4m3 down-proj dgrad + SwiGLU backward -> grad_aux bf16 [total_M, 2I] (interleaved)."""
    with timed("fp8_down_dgrad_swiglu_bwd"):
        return torch.ops.grouped_mm.mm_swiglu_bwd_fp8(grad_output, down_w_t, offs, aux_biased_acc, scale_a, scale_b,
                                                      swiglu_alpha, swiglu_limit)


def grouped_mm_wgrad_fp8(a_cols: torch.Tensor, b_cols: torch.Tensor, offs: torch.Tensor, scale_a: torch.Tensor,
                         scale_b: torch.Tensor, bias_grad: bool = True) -> tuple[torch.Tensor, torch.Tensor | None]:
    """e4m3 ragged-K weight gradient: a_cols e4m3 [total, m] and b_cols e4m3 [total, n] (row-major token rows,
    per-column scales from quantize_cols) -> (dW bf16 [E, m, n], db bf16 [E, n] or None)."""
    with timed("fp8_wgrad_bias"):
        dw, db = torch.ops.grouped_mm.mm_wgrad_fp8(a_cols.transpose(0, 1), b_cols, offs, scale_a, scale_b, bias_grad)
    return dw, (db if bias_grad else None)


class _FFNFp8(torch.autograd.Function):
    """The fused MoE FFN with every GEMM in e4m3 (see the module docstring for the recipe)."""

    @staticmethod
    def forward(ctx, x, w_up, b_up, w_down, b_down, offs, alpha, limit):
        qx, sx = quantize_rows(x)
        # both axes of each weight at once: the forward's operand now, the dgrad's kept for backward
        qwu, swu, qwut, swut = quantize_weights_both(w_up)
        s, aux = grouped_mm_swiglu_fp8(qx, qwu, offs, sx, swu, b_up, alpha, limit)
        qs, ss = quantize_rows(s)
        qwd, swd, qwdt, swdt = quantize_weights_both(w_down)
        out = grouped_mm_fp8(qs, qwd, offs, ss, swd, b_down)
        ctx.save_for_backward(x, qwut, swut, qwdt, swdt, s, aux, offs)
        ctx.alpha, ctx.limit = alpha, limit
        return out

    @staticmethod
    def backward(ctx, g):
        x, qwut, swut, qwdt, swdt, s, aux, offs = ctx.saved_tensors
        g = g.contiguous()
        # down-proj weight + bias gradients over token rows (per-column scales)
        qs_c, ss_c = quantize_cols(s)
        qg, sg, qg_c, sg_c = quantize_rows_cols(g)  # rows for the dgrad below, columns here
        g_wd, g_bd = grouped_mm_wgrad_fp8(qs_c, qg_c, offs, ss_c, sg_c)
        # down-proj dgrad + SwiGLU backward (row scales for grad_out, column scales for W_down^T)
        grad_aux = grouped_mm_swiglu_bwd_fp8(qg, qwdt, offs, aux, sg, swdt, ctx.alpha, ctx.limit)
        # up-proj dgrad and weight + bias gradients
        qga, sga, qga_c, sga_c = quantize_rows_cols(grad_aux)
        g_x = grouped_mm_fp8(qga, qwut, offs, sga, swut, None)
        qx_c, sx_c = quantize_cols(x)
        g_wu, g_bu = grouped_mm_wgrad_fp8(qx_c, qga_c, offs, sx_c, sga_c)
        return g_x, g_wu, g_bu, g_wd, g_bd, None, None, None


def grouped_mm_ffn_fp8(x: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, offs: torch.Tensor,
                       b_up: torch.Tensor, b_down: torch.Tensor, swiglu_alpha: float = 1.702,
                       swiglu_limit: float = 7.0) -> torch.Tensor:
    """The MoE FFN (up-proj + bias + clamped SwiGLU, down-proj + bias) with every GEMM of its forward and
    backward in e4m3; bf16 inputs, parameters, output and gradients."""
    return _FFNFp8.apply(x, w_up, b_up, w_down, b_down, offs, swiglu_alpha, swiglu_limit)
