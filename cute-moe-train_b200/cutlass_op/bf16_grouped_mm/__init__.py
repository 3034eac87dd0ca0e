"""B200 (sm_100a) grouped GEMM for the MoE FFN, with autograd.

Drop-in for Butterfingrz/CuTe-MoE-Train's ``cutlass_op.bf16_grouped_mm`` (``__init__.py:9-114``):
the same three wrappers with the same arguments and defaults, over the same ``grouped_mm::*``
operators.  Importing the package loads the native libraries and registers autograd.
"""

from __future__ import annotations

import torch

from . import custom_op as _custom_op
from ._ext import check_device_status, device_status  # noqa: F401
from .optimer import OpTimer, timed  # noqa: F401
from .custom_op import (  # noqa: F401
    grouped_mm_downproj_forward,
    grouped_mm_forward,
    grouped_mm_swiglu_forward,
)


def grouped_mm(
    mat_a: torch.Tensor,
    mat_b: torch.Tensor,
    offs: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Grouped matrix multiplication with autograd support.

    mat_a [total_M, K] x mat_b [E, K, N] with ``offs`` (int32 cumulative row ends) is the MoE
    ragged-M case; 2D x 2D is ragged-K (output [E, M, N]); 3D x 3D is a batched GEMM.  ``bias``
    [E, N] is added per group.  ``out_dtype`` must be None or the input dtype (bf16).
    """
    return torch.ops.grouped_mm.mm(mat_a, mat_b, offs, bias, _custom_op.dtype_to_int(out_dtype))


def grouped_mm_swiglu(
    mat_a: torch.Tensor,
    mat_b: torch.Tensor,
    offs: torch.Tensor,
    bias: torch.Tensor,
    swiglu_alpha: float = 1.702,
    swiglu_limit: float = 7.0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused grouped GEMM + bias + clamped SwiGLU (GPT-OSS form), one kernel launch.

    Args:
        mat_a: [total_M, K] bf16 ragged token rows, grouped by expert.
        mat_b: [E, K, 2*I] bf16 weights with gate/up columns interleaved (even = gate, odd = up).
        offs: [E] int32 cumulative token offsets per expert.
        bias: [E, 2*I] bf16, interleaved like mat_b.
        swiglu_alpha, swiglu_limit: activation parameters.

    Returns:
        (swiglu_out [total_M, I], aux_biased_acc [total_M, 2*I]).  The backward is fused-only:
        ``aux_biased_acc`` must be handed to :func:`grouped_mm_downproj`, which routes the
        gradient back through it; a gradient reaching ``swiglu_out`` directly raises.
    """
    with timed("up_swiglu_fwd"):
        return torch.ops.grouped_mm.mm_swiglu(mat_a, mat_b, offs, bias, swiglu_alpha, swiglu_limit)


def grouped_mm_downproj(
    mat_a: torch.Tensor,
    mat_b: torch.Tensor,
    offs: torch.Tensor,
    bias: torch.Tensor | None,
    aux_biased_acc: torch.Tensor,
    swiglu_alpha: float = 1.702,
    swiglu_limit: float = 7.0,
) -> torch.Tensor:
    """Down-projection grouped GEMM (+ bias) whose backward emits the SwiGLU input gradient.

    Forward equals ``grouped_mm(mat_a, mat_b, offs=offs, bias=bias)``.  Backward computes
    ``grad_aux = SwiGLU_bwd(grad_out @ mat_b^T, aux_biased_acc)`` in one fused launch.
    """
    with timed("down_fwd"):
        return torch.ops.grouped_mm.mm_downproj(
            mat_a, mat_b, offs, bias, aux_biased_acc, swiglu_alpha, swiglu_limit
        )


def grouped_mm_ffn(
    x: torch.Tensor,
    w_up: torch.Tensor,
    w_down: torch.Tensor,
    offs: torch.Tensor,
    b_up: torch.Tensor,
    b_down: torch.Tensor | None = None,
    swiglu_alpha: float = 1.702,
    swiglu_limit: float = 7.0,
    store_aux: bool = True,
) -> torch.Tensor:
    """The whole MoE expert FFN: ``grouped_mm_downproj(grouped_mm_swiglu(x, w_up) ...)``.

    ``store_aux=True`` keeps ``aux_biased_acc`` [total_M, 2*I] from the forward for the backward,
    like the two wrappers chained.  ``store_aux=False`` is the reference binding's recompute mode:
    the forward does not write aux and the backward recomputes it with one more grouped GEMM
    (same results, bit for bit; 4*M*H*I more FLOPs per step, rows x 2I x 2 bytes less memory).
    """
    return _custom_op.GroupedFFN.apply(x, w_up, b_up, w_down, b_down, offs, swiglu_alpha, swiglu_limit, store_aux)


# The reference's exports; grouped_mm_ffn is an addition, imported by name.
__all__ = [
    "grouped_mm",
    "grouped_mm_downproj",
    "grouped_mm_swiglu",
]
