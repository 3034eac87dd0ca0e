"""Shape inference and autograd for the `grouped_mm::*` operators.

The operators themselves (schemas and CUDA implementations) are registered in C++
(csrc/torch_ops.cpp) over the C ABI of include/moe_gemm.h.  This module gives them fake-tensor
shape inference and autograd with the same contract as Butterfingrz/CuTe-MoE-Train
(cutlass_op/bf16_grouped_mm/custom_op.py):

* ``grouped_mm::mm`` (custom_op.py:139-335): grouped GEMM with optional bias; backward computes
  both dgrads with ``mm`` and, new here, the weight and bias gradients of the ragged-M case in one
  fused launch (``grouped_mm::mm_wgrad_bias``) instead of a GEMM plus ``_segment_sum_rows``.
* ``grouped_mm::mm_swiglu`` (custom_op.py:400-526): fused up-projection + bias + clamped SwiGLU
  returning ``(swiglu_out, aux_biased_acc)``.  Backward is fused-only: it accepts the gradient of
  ``aux_biased_acc`` produced by ``mm_downproj``'s backward and raises if a gradient reaches
  ``swiglu_out`` directly.
* ``grouped_mm::mm_swiglu_bwd`` (custom_op.py:534-571): opaque down-proj dgrad + SwiGLU backward.
* ``grouped_mm::mm_downproj`` (custom_op.py:579-693): down-projection whose backward emits
  ``grad_aux`` for ``mm_swiglu`` instead of a gradient for ``swiglu_out``.
* ``grouped_mm::mm_swiglu_noaux`` and :class:`GroupedFFN`: the ``store_aux=False`` recompute path
  of the reference's binding (csrc/binding.cu:36-63) as a whole-FFN autograd function.
"""

from __future__ import annotations

import torch

from . import _ext  # noqa: F401  (loads the native libraries and registers the operators)
from .optimer import timed

# c10::ScalarType codes accepted by the `out_dtype: int` argument (-1 means "same as mat_a").
_SCALAR_TYPE_CODE = {torch.float16: 5, torch.float32: 6, torch.bfloat16: 15}
_CODE_SCALAR_TYPE = {v: k for k, v in _SCALAR_TYPE_CODE.items()}


def dtype_to_int(dtype: torch.dtype | None) -> int:
    if dtype is None:
        return -1
    if dtype not in _SCALAR_TYPE_CODE:
        raise RuntimeError(f"grouped_mm: unsupported out_dtype {dtype}")
    return _SCALAR_TYPE_CODE[dtype]


def _dtype_from_int(out_dtype: int) -> torch.dtype | None:
    return None if out_dtype == -1 else _CODE_SCALAR_TYPE[out_dtype]


def _padded(n: int, dtype: torch.dtype) -> int:
    align = 16 // torch.empty((), dtype=dtype).element_size()
    return (n + align - 1) // align * align


def _out_shape(mat_a: torch.Tensor, mat_b: torch.Tensor, offs: torch.Tensor | None) -> tuple[int, ...]:
    """Output shape of grouped_mm for the four input-rank combinations (custom_op.py:12-37)."""
    a2, b2 = mat_a.dim() == 2, mat_b.dim() == 2
    if (a2 or b2) and offs is None:
        raise RuntimeError("grouped_mm: `offs` must be provided when at least one input is 2D (ragged/grouped path).")
    if a2 and b2:
        return (offs.size(0), mat_a.size(0), mat_b.size(1))
    if a2:
        return (mat_a.size(0), mat_b.size(-1))
    if b2:
        return (mat_a.size(1), mat_b.size(1))
    return (mat_a.size(0), mat_a.size(1), mat_b.size(-1))


def _empty_out(mat_a, mat_b, offs, out_dtype: int) -> torch.Tensor:
    """Output with the 16-byte padded last-dim stride of csrc/cutlass_utils.cuh:51-63."""
    dtype = _dtype_from_int(out_dtype) or mat_a.dtype
    shape = _out_shape(mat_a, mat_b, offs)
    last = _padded(shape[-1], dtype)
    if len(shape) == 2:
        strides = (last, 1)
    else:
        strides = (shape[1] * last, last, 1)
    return torch.empty_strided(shape, strides, dtype=dtype, device=mat_a.device)


def _has_effective_grad(grad: torch.Tensor | None) -> bool:
    """True only for a usable gradient: not None, not empty, not a ZeroTensor (custom_op.py:384-397)."""
    if grad is None or grad.numel() == 0:
        return False
    is_zero = getattr(torch, "_is_zerotensor", None)
    if is_zero is not None:
        try:
            if bool(is_zero(grad)):
                return False
        except Exception:  # pragma: no cover
            pass
    return True


def segment_sum_rows(grad: torch.Tensor, offs: torch.Tensor) -> torch.Tensor:
    """Per-group row sums with fp32 accumulation (custom_op.py:79-101).

    Only used when a bias gradient is requested without the weight gradient; the common path
    gets it from the fused ``grouped_mm::mm_wgrad_bias`` launch.
    """
    total_m, n = grad.shape
    groups = offs.numel()
    acc = torch.zeros((groups, n), dtype=torch.float32, device=grad.device)
    rows = torch.arange(total_m, device=grad.device, dtype=torch.int64)
    gid = torch.bucketize(rows, offs.to(torch.int64), right=True)
    keep = gid < groups  # rows past offs[-1] belong to no group
    acc.index_add_(0, gid[keep], grad[keep].to(torch.float32))
    return acc.to(grad.dtype)


def segment_sum_cols(grad: torch.Tensor, offs: torch.Tensor) -> torch.Tensor:
    """Bias gradient of the ragged-N layout (custom_op.py:104-131): column sums of ``grad`` [M, total_N]
    in fp32, placed at [group, column - group start] of an [E, total_N] result."""
    groups = offs.numel()
    total_n = grad.shape[1]
    col_sum = grad.sum(dim=0, dtype=torch.float32)
    cols = torch.arange(total_n, device=grad.device, dtype=torch.int64)
    ends = offs.to(torch.int64)
    gid = torch.bucketize(cols, ends, right=True)
    starts = torch.cat([ends.new_zeros(1), ends[:-1]])
    keep = gid < groups  # columns past offs[-1] belong to no group
    acc = torch.zeros((groups, total_n), dtype=torch.float32, device=grad.device)
    acc[gid[keep], cols[keep] - starts[gid[keep]]] = col_sum[keep]
    return acc.to(grad.dtype)


def _is_col_major(t: torch.Tensor) -> bool:
    d = t.dim()
    return t.stride(d - 2) == 1 and t.stride(d - 1) == t.size(d - 2)


# ============================================================================ grouped_mm::mm


@torch.library.register_fake("grouped_mm::mm")
def _mm_fake(mat_a, mat_b, offs, bias, out_dtype):
    return _empty_out(mat_a, mat_b, offs, out_dtype)


def _mm_setup_context(ctx, inputs, output):  # noqa: ARG001
    mat_a, mat_b, offs, bias, out_dtype = inputs
    ctx.has_offs = offs is not None
    ctx.has_bias = bias is not None
    saved = [mat_a, mat_b]
    if offs is not None:
        saved.append(offs)
    ctx.save_for_backward(*saved)
    if bias is not None:
        ctx.bias_shape = bias.shape
        ctx.bias_dtype = bias.dtype
    ctx.out_dtype = int(out_dtype)


def _mm_backward(ctx, grad_out):
    saved = ctx.saved_tensors
    mat_a, mat_b = saved[0], saved[1]
    offs = saved[2] if ctx.has_offs else None
    need_a, need_b = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    need_bias = ctx.needs_input_grad[3] and ctx.has_bias

    if not grad_out.numel():
        return (
            torch.zeros_like(mat_a) if need_a else None,
            torch.zeros_like(mat_b) if need_b else None,
            None,
            torch.zeros(ctx.bias_shape, dtype=ctx.bias_dtype, device=mat_a.device) if need_bias else None,
            None,
        )
    grad_out = grad_out.contiguous()
    ga = gb = gbias = None
    a2, b2 = mat_a.dim() == 2, mat_b.dim() == 2

    if a2 and not b2:
        # ragged-M: out[rows(e)] = a[rows(e)] @ b[e] (+ bias[e])
        if need_a:
            with timed("mm_dgrad"):
                ga = torch.ops.grouped_mm.mm(grad_out, mat_b.transpose(-2, -1), offs, None, -1)
        if need_b and need_bias:
            with timed("mm_wgrad_bias"):
                gb, gbias = torch.ops.grouped_mm.mm_wgrad_bias(mat_a.transpose(-2, -1), grad_out, offs)
            gbias = gbias.to(ctx.bias_dtype)
        elif need_b:
            gb = torch.ops.grouped_mm.mm(mat_a.transpose(-2, -1), grad_out, offs, None, -1)
        elif need_bias:
            gbias = segment_sum_rows(grad_out, offs).to(ctx.bias_dtype)
    elif a2 and b2:
        # ragged-K: out[e] = a[:, rows(e)] @ b[rows(e)]; both gradients are ragged-M GEMMs.
        if need_a:
            # grad_a[:, rows(e)] = grad_out[e] @ b[rows(e)]^T  ==  (b[rows(e)] @ grad_out[e]^T)^T
            ga = torch.ops.grouped_mm.mm(mat_b, grad_out.transpose(-2, -1), offs, None, -1).transpose(-2, -1)
        if need_b:
            gb = torch.ops.grouped_mm.mm(mat_a.transpose(-2, -1), grad_out, offs, None, -1)
        if need_bias:
            raise RuntimeError("grouped_mm: bias is not supported on the ragged-K path")
    elif not a2 and not b2:
        if need_a:
            ga = torch.ops.grouped_mm.mm(grad_out, mat_b.transpose(-2, -1).contiguous(), None, None, -1)
        if need_b:
            gb = torch.ops.grouped_mm.mm(mat_a.transpose(-2, -1).contiguous(), grad_out, None, None, -1)
        if need_bias:
            gbias = grad_out.sum(dim=-2, dtype=torch.float32).to(grad_out.dtype)
    else:
        # ragged-N: out[:, cols(e)] = a[e] @ b[:, cols(e)] (+ bias[e, local col]), custom_op.py:263-330
        if need_a:
            ga = torch.ops.grouped_mm.mm(grad_out, mat_b.transpose(-2, -1), offs, None, -1)
        if need_b:
            gb = torch.ops.grouped_mm.mm(mat_a.transpose(-2, -1), grad_out, offs, None, -1)
        if need_bias:
            gbias = segment_sum_cols(grad_out, offs).to(ctx.bias_dtype)
    return ga, gb, None, gbias, None


torch.library.register_autograd("grouped_mm::mm", _mm_backward, setup_context=_mm_setup_context)


# ============================================================================ grouped_mm::mm_wgrad_bias


@torch.library.register_fake("grouped_mm::mm_wgrad_bias")
def _wgrad_bias_fake(mat_a, mat_b, offs):
    e, m, n = offs.size(0), mat_a.size(0), mat_b.size(1)
    last = _padded(n, mat_a.dtype)
    dw = torch.empty_strided((e, m, n), (m * last, last, 1), dtype=mat_a.dtype, device=mat_a.device)
    db = torch.empty((e, n), dtype=mat_a.dtype, device=mat_a.device)
    return dw, db


# ============================================================================ grouped_mm::mm_swiglu


@torch.library.register_fake("grouped_mm::mm_swiglu")
def _swiglu_fake(mat_a, mat_b, offs, bias, swiglu_alpha, swiglu_limit):
    total_m, n_full = mat_a.size(0), mat_b.size(-1)
    half = n_full // 2
    swiglu_out = torch.empty_strided(
        (total_m, half), (_padded(half, torch.bfloat16), 1), dtype=torch.bfloat16, device=mat_a.device
    )
    return swiglu_out, _empty_out(mat_a, mat_b, offs, -1)


def _swiglu_setup_context(ctx, inputs, output):  # noqa: ARG001
    mat_a, mat_b, offs, bias, _alpha, _limit = inputs
    # Unused output gradients stay None instead of materialised zeros.
    ctx.set_materialize_grads(False)
    # The bias value is not needed for backward (only its gradient is produced).
    ctx.save_for_backward(mat_a, mat_b, offs)
    ctx.bias_shape = bias.shape
    ctx.bias_dtype = bias.dtype


def _swiglu_backward(ctx, grad_swiglu, grad_aux):
    mat_a, mat_b, offs = ctx.saved_tensors
    if _has_effective_grad(grad_swiglu):
        raise RuntimeError(
            "grouped_mm::mm_swiglu backward received grad_swiglu, which is unsupported in fused-only mode. "
            "Ensure swiglu_out is consumed only by grouped_mm::mm_downproj."
        )
    if grad_aux is None:
        raise RuntimeError(
            "grouped_mm::mm_swiglu backward requires grad_aux from grouped_mm::mm_downproj (got grad_aux=None). "
            "Fused-only mode does not support standalone backward through swiglu_out."
        )
    need_a, need_b, need_bias = ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.needs_input_grad[3]
    if not _has_effective_grad(grad_aux):
        return (
            torch.zeros_like(mat_a) if need_a else None,
            torch.zeros_like(mat_b) if need_b else None,
            None,
            torch.zeros(ctx.bias_shape, dtype=ctx.bias_dtype, device=mat_a.device) if need_bias else None,
            None,
            None,
        )
    grad_gate_up = grad_aux.contiguous()
    ga = gb = gbias = None
    if need_a:
        with timed("up_dgrad"):
            ga = torch.ops.grouped_mm.mm(grad_gate_up, mat_b.transpose(-2, -1), offs, None, -1)
    if need_b and need_bias:
        with timed("up_wgrad_bias"):
            gb, gbias = torch.ops.grouped_mm.mm_wgrad_bias(mat_a.transpose(-2, -1), grad_gate_up, offs)
        gbias = gbias.to(ctx.bias_dtype)
    elif need_b:
        gb = torch.ops.grouped_mm.mm(mat_a.transpose(-2, -1), grad_gate_up, offs, None, -1)
    elif need_bias:
        gbias = segment_sum_rows(grad_gate_up, offs).to(ctx.bias_dtype)
    return ga, gb, None, gbias, None, None


torch.library.register_autograd("grouped_mm::mm_swiglu", _swiglu_backward, setup_context=_swiglu_setup_context)


# ============================================================================ grouped_mm::mm_swiglu_bwd


@torch.library.register_fake("grouped_mm::mm_swiglu_bwd")
def _swiglu_bwd_fake(grad_out, down_w_t, offs, aux_biased_acc, swiglu_alpha, swiglu_limit):
    return torch.empty_like(aux_biased_acc)


# ============================================================================ grouped_mm::mm_downproj


@torch.library.register_fake("grouped_mm::mm_downproj")
def _downproj_fake(mat_a, mat_b, offs, bias, aux_biased_acc, swiglu_alpha, swiglu_limit):
    return _empty_out(mat_a, mat_b, offs, -1)


def _downproj_setup_context(ctx, inputs, output):  # noqa: ARG001
    mat_a, mat_b, offs, bias, aux_biased_acc, swiglu_alpha, swiglu_limit = inputs
    ctx.save_for_backward(mat_a, mat_b, offs, aux_biased_acc)
    ctx.has_bias = bias is not None
    if bias is not None:
        ctx.bias_shape = bias.shape
        ctx.bias_dtype = bias.dtype
    ctx.swiglu_alpha = swiglu_alpha
    ctx.swiglu_limit = swiglu_limit


def _downproj_backward(ctx, grad_out):
    mat_a, mat_b, offs, aux_biased_acc = ctx.saved_tensors
    need_a, need_b = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    need_bias = ctx.needs_input_grad[3] and ctx.has_bias
    need_aux = ctx.needs_input_grad[4]

    if not grad_out.numel():
        return (
            (None if need_aux else torch.zeros_like(mat_a)) if need_a else None,
            torch.zeros_like(mat_b) if need_b else None,
            None,
            torch.zeros(ctx.bias_shape, dtype=ctx.bias_dtype, device=mat_a.device) if need_bias else None,
            torch.zeros_like(aux_biased_acc) if need_aux else None,
            None,
            None,
        )
    grad_out = grad_out.contiguous()
    ga = gb = gbias = gaux = None
    if need_b and need_bias:
        with timed("down_wgrad_bias"):
            gb, gbias = torch.ops.grouped_mm.mm_wgrad_bias(mat_a.transpose(-2, -1), grad_out, offs)
        gbias = gbias.to(ctx.bias_dtype)
    elif need_b:
        gb = torch.ops.grouped_mm.mm(mat_a.transpose(-2, -1), grad_out, offs, None, -1)
    elif need_bias:
        gbias = segment_sum_rows(grad_out, offs).to(ctx.bias_dtype)
    if need_aux:
        with timed("down_dgrad_swiglu_bwd"):
            gaux = torch.ops.grouped_mm.mm_swiglu_bwd(
                grad_out, mat_b.transpose(-2, -1), offs, aux_biased_acc, ctx.swiglu_alpha, ctx.swiglu_limit
            )
    # With the aux route active the plain dgrad of mat_a is skipped: mm_swiglu's backward
    # consumes grad_aux directly (custom_op.py:681-685).
    if need_a and not need_aux:
        ga = torch.ops.grouped_mm.mm(grad_out, mat_b.transpose(-2, -1), offs, None, -1)
    return ga, gb, None, gbias, gaux, None, None


torch.library.register_autograd(
    "grouped_mm::mm_downproj", _downproj_backward, setup_context=_downproj_setup_context
)

# ============================================================================ grouped_mm::mm_swiglu_noaux


@torch.library.register_fake("grouped_mm::mm_swiglu_noaux")
def _swiglu_noaux_fake(mat_a, mat_b, offs, bias, swiglu_alpha, swiglu_limit):
    half = mat_b.size(-1) // 2
    return torch.empty_strided(
        (mat_a.size(0), half), (_padded(half, torch.bfloat16), 1), dtype=torch.bfloat16, device=mat_a.device
    )


# ============================================================================ whole FFN, aux optional


class GroupedFFN(torch.autograd.Function):
    """Up-projection + bias + SwiGLU -> down-projection + bias, with autograd.

    ``store_aux=True`` is exactly ``grouped_mm_swiglu`` followed by ``grouped_mm_downproj``.
    ``store_aux=False`` is the recompute path of the reference's binding
    (``_grouped_mm_swiglu_cuda(..., store_aux=False)``, csrc/binding.cu:36-63): the forward writes
    no ``aux_biased_acc`` (saving rows x 2I bf16 of memory between forward and backward) and the
    backward rebuilds it with one ragged-M GEMM + bias before the fused SwiGLU backward.  The
    rebuilt aux equals the stored one bit for bit: the same tiles accumulate in the same order and
    round once.
    """

    @staticmethod
    def forward(ctx, x, w_up, b_up, w_down, b_down, offs, swiglu_alpha, swiglu_limit, store_aux):
        if store_aux:
            with timed("up_swiglu_fwd"):
                s, aux = torch.ops.grouped_mm.mm_swiglu(x, w_up, offs, b_up, swiglu_alpha, swiglu_limit)
        else:
            with timed("up_swiglu_fwd"):
                s = torch.ops.grouped_mm.mm_swiglu_noaux(x, w_up, offs, b_up, swiglu_alpha, swiglu_limit)
            aux = None
        with timed("down_fwd"):
            out = torch.ops.grouped_mm.mm(s, w_down, offs, b_down, -1)
        ctx.store_aux = bool(store_aux)
        ctx.has_b_down = b_down is not None
        ctx.alpha, ctx.limit = swiglu_alpha, swiglu_limit
        ctx.save_for_backward(x, w_up, b_up, w_down, s, offs, *( [aux] if store_aux else []))
        if b_down is not None:
            ctx.b_down_shape, ctx.b_down_dtype = b_down.shape, b_down.dtype
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, w_up, b_up, w_down, s, offs = ctx.saved_tensors[:6]
        need = ctx.needs_input_grad
        need_x, need_wu, need_bu, need_wd, need_bd = need[0], need[1], need[2], need[3], need[4] and ctx.has_b_down
        if not grad_out.numel():
            z = lambda t, n: torch.zeros_like(t) if n else None  # noqa: E731
            bd = torch.zeros(ctx.b_down_shape, dtype=ctx.b_down_dtype, device=x.device) if need_bd else None
            return z(x, need_x), z(w_up, need_wu), z(b_up, need_bu), z(w_down, need_wd), bd, None, None, None, None
        grad_out = grad_out.contiguous()
        g_wd = g_bd = None
        if need_wd and need_bd:
            with timed("down_wgrad_bias"):
                g_wd, g_bd = torch.ops.grouped_mm.mm_wgrad_bias(s.transpose(-2, -1), grad_out, offs)
            g_bd = g_bd.to(ctx.b_down_dtype)
        elif need_wd:
            g_wd = torch.ops.grouped_mm.mm(s.transpose(-2, -1), grad_out, offs, None, -1)
        elif need_bd:
            g_bd = segment_sum_rows(grad_out, offs).to(ctx.b_down_dtype)
        g_x = g_wu = g_bu = None
        if need_x or need_wu or need_bu:
            if ctx.store_aux:
                aux = ctx.saved_tensors[6]
            else:
                with timed("up_recompute_aux"):
                    aux = torch.ops.grouped_mm.mm(x, w_up, offs, b_up, -1)
            with timed("down_dgrad_swiglu_bwd"):
                grad_aux = torch.ops.grouped_mm.mm_swiglu_bwd(
                    grad_out, w_down.transpose(-2, -1), offs, aux, ctx.alpha, ctx.limit
                )
            del aux
            if need_x:
                with timed("up_dgrad"):
                    g_x = torch.ops.grouped_mm.mm(grad_aux, w_up.transpose(-2, -1), offs, None, -1)
            if need_wu and need_bu:
                with timed("up_wgrad_bias"):
                    g_wu, g_bu = torch.ops.grouped_mm.mm_wgrad_bias(x.transpose(-2, -1), grad_aux, offs)
                g_bu = g_bu.to(b_up.dtype)
            elif need_wu:
                g_wu = torch.ops.grouped_mm.mm(x.transpose(-2, -1), grad_aux, offs, None, -1)
            elif need_bu:
                g_bu = segment_sum_rows(grad_aux, offs).to(b_up.dtype)
        return g_x, g_wu, g_bu, g_wd, g_bd, None, None, None, None


# ============================================================================ into-output forms


@torch.library.register_fake("grouped_mm::swiglu_into")
def _swiglu_into_fake(mat_a, mat_b, offs, bias, aux_out, swiglu_out, swiglu_alpha, swiglu_limit, store_aux):
    return None


@torch.library.register_fake("grouped_mm::swiglu_bwd_into")
def _swiglu_bwd_into_fake(grad_output, down_w_t, offs, aux_packed, grad_gate_up_packed, swiglu_alpha, swiglu_limit):
    return None


# ============================================================================ EP row movement


@torch.library.register_fake("grouped_mm::gather_rows")
def _gather_rows_fake(src, idx, scale):
    return src.new_empty((idx.numel(), src.shape[1]))


@torch.library.register_fake("grouped_mm::combine_rows")
def _combine_rows_fake(rows, pos, weights, k):
    return rows.new_empty((pos.numel() // k, rows.shape[1]))


# Names the reference module exports (custom_op.py:139, 400, 579): the registered operators.
grouped_mm_forward = torch.ops.grouped_mm.mm
grouped_mm_swiglu_forward = torch.ops.grouped_mm.mm_swiglu
grouped_mm_swiglu_bwd_forward = torch.ops.grouped_mm.mm_swiglu_bwd
grouped_mm_downproj_forward = torch.ops.grouped_mm.mm_downproj

# ... and its autograd pieces and helpers (custom_op.py:12-131, 190-330, 353-397, 467-693), for code
# that imports them: this module's equivalents under the reference's names.
grouped_mm_setup_context = _mm_setup_context
grouped_mm_backward = _mm_backward
grouped_mm_swiglu_setup_context = _swiglu_setup_context
grouped_mm_swiglu_backward = _swiglu_backward
grouped_mm_downproj_setup_context = _downproj_setup_context
grouped_mm_downproj_backward = _downproj_backward
_segment_sum_rows = segment_sum_rows
_segment_sum_cols = segment_sum_cols  # groups columns exactly like the forward's bias (see segment_sum_cols)
_infer_grouped_mm_out_shape = _out_shape
_empty_grouped_mm_output = _empty_out


def _infer_grouped_mm_out_strides(out_shape, out_dtype, *, a_is_2d: bool, b_is_2d: bool) -> tuple[int, ...]:
    """Row-major strides with the last dimension padded to 16 bytes; 2D output for ragged-M / ragged-N."""
    last = _padded(out_shape[-1], out_dtype)
    if a_is_2d != b_is_2d:
        return (last, 1)
    return (out_shape[1] * last, last, 1)


def _empty_swiglu_output(mat_a, mat_b, offs=None) -> torch.Tensor:
    """swiglu_out [total_M, I] bf16 with the 16-byte padded row stride."""
    half = mat_b.size(-1) // 2
    return torch.empty_strided((mat_a.size(0), half), (_padded(half, torch.bfloat16), 1), dtype=torch.bfloat16,
                               device=mat_a.device)


def _as_packed_fp32(tensor_bf16: torch.Tensor, *, tensor_name: str) -> torch.Tensor:
    """The fp32 [..., I] view of interleaved bf16 (gate, up) pairs [..., 2I]."""
    if tensor_bf16.dtype != torch.bfloat16:
        raise RuntimeError(f"{tensor_name} must be bfloat16, got {tensor_bf16.dtype}")
    if tensor_bf16.size(-1) % 2 or tensor_bf16.stride(-1) != 1 or tensor_bf16.stride(-2) % 2:
        raise RuntimeError(f"{tensor_name} must be row-major with an even last dimension and row stride")
    return tensor_bf16.view(torch.float32)
