"""ctypes binding of libmoe_gemm.so that replaces the reference's compiled `_ext` module.

Butterfingrz/CuTe-MoE-Train's custom_op.py:5 imports three pybind functions from its CUDA extension
(csrc/binding.cu:120-148).  A maintainer who wants the reference's own Python layer to run on the
B200 kernels saves this file as ``cutlass_op/bf16_grouped_mm/_ext.py`` of the reference package (or
registers it as that module) and points ``MGF_LIBRARY`` at libmoe_gemm.so; nothing else changes.
It binds only the C ABI of include/moe_gemm.h -- no torch operator library is loaded, so it can sit
in a process that imports the reference package (which registers the ``grouped_mm`` namespace).

Covered: the MoE layouts the reference's custom_op.py uses -- ragged-M 2D x 3D with a row-major or
K-major B (+ bias), ragged-K 2D x 2D (weight gradients), the fused bias + SwiGLU forward (with
``store_aux``) and the fused dgrad + SwiGLU backward on the packed fp32 views.  Other layouts raise.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

_DEFAULT_LIB = Path(__file__).resolve().parent / "cutlass_op" / "bf16_grouped_mm" / "libmoe_gemm.so"
_lib = ctypes.CDLL(os.environ.get("MGF_LIBRARY", str(_DEFAULT_LIB)))

MGF_EPI_BIAS, MGF_EPI_SWIGLU, MGF_EPI_SWIGLU_BWD, MGF_EPI_WGRAD = 0, 1, 2, 3


class MgfGemmDesc(ctypes.Structure):  # include/moe_gemm.h: mgf_gemm_desc
    _fields_ = [("epilogue", ctypes.c_int32), ("num_groups", ctypes.c_int32),
                ("total_rows", ctypes.c_int64), ("m", ctypes.c_int64), ("n", ctypes.c_int64),
                ("k", ctypes.c_int64), ("a", ctypes.c_void_p), ("lda", ctypes.c_int64),
                ("b", ctypes.c_void_p), ("ldb", ctypes.c_int64), ("ldb_batch", ctypes.c_int64),
                ("b_mn_major", ctypes.c_int32), ("offs", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("bias_stride", ctypes.c_int64), ("d", ctypes.c_void_p), ("ldd", ctypes.c_int64),
                ("ldd_batch", ctypes.c_int64), ("d2", ctypes.c_void_p), ("ldd2", ctypes.c_int64),
                ("aux", ctypes.c_void_p), ("ld_aux", ctypes.c_int64), ("swiglu_alpha", ctypes.c_float),
                ("swiglu_limit", ctypes.c_float), ("store_aux", ctypes.c_int32),
                ("sm_carveout", ctypes.c_int32), ("workspace", ctypes.c_void_p),
                ("bias_per_row", ctypes.c_int32), ("ab_type", ctypes.c_int32),
                ("scale_a", ctypes.c_void_p), ("scale_b", ctypes.c_void_p), ("scale_b_stride", ctypes.c_int64),
                ("d_row_ptrs", ctypes.c_void_p), ("group_begin", ctypes.c_int32)]


_lib.mgf_grouped_gemm_launch.argtypes = [ctypes.POINTER(MgfGemmDesc), ctypes.c_void_p]
_lib.mgf_grouped_gemm_launch.restype = ctypes.c_int
_lib.mgf_status_string.restype = ctypes.c_char_p
_lib.mgf_status_string.argtypes = [ctypes.c_int]
_lib.mgf_last_error_detail.restype = ctypes.c_char_p
_lib.mgf_gemm_desc_size.restype = ctypes.c_size_t
if ctypes.sizeof(MgfGemmDesc) != _lib.mgf_gemm_desc_size():
    raise ImportError("ctypes_ext: MgfGemmDesc does not match the library's mgf_gemm_desc")


def _launch(desc: MgfGemmDesc, device: torch.device) -> None:
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream().cuda_stream
        rc = _lib.mgf_grouped_gemm_launch(ctypes.byref(desc), ctypes.c_void_p(stream))
    if rc != 0:
        raise RuntimeError(f"mgf_grouped_gemm_launch: {_lib.mgf_status_string(rc).decode()} "
                           f"{_lib.mgf_last_error_detail().decode()}")


def _ragged_m(epi, a, b, offs, bias, d, d2=None, aux=None, alpha=1.702, limit=7.0, store_aux=True):
    k_major = b.stride(-2) == 1 and b.stride(-1) != 1   # e.g. W.transpose(-2, -1)
    g = MgfGemmDesc(epilogue=epi, num_groups=offs.numel(), total_rows=a.size(0), n=b.size(2), k=a.size(1),
                    a=a.data_ptr(), lda=a.stride(0), b=b.data_ptr(),
                    ldb=b.stride(2) if k_major else b.stride(1), ldb_batch=b.stride(0),
                    b_mn_major=0 if k_major else 1, offs=offs.data_ptr(), d=d.data_ptr(), ldd=d.stride(0),
                    swiglu_alpha=alpha, swiglu_limit=limit, store_aux=int(store_aux))
    if bias is not None:
        g.bias, g.bias_stride = bias.data_ptr(), bias.stride(0)
    if d2 is not None:
        g.d2, g.ldd2 = d2.data_ptr(), d2.stride(0)
    if aux is not None:
        g.aux, g.ld_aux = aux.data_ptr(), aux.stride(0)
    _launch(g, a.device)


def _grouped_mm_cuda(mat_a, mat_b, offs=None, bias=None, out_dtype=None):
    """csrc/binding.cu:13-34 for the MoE layouts: ragged-M (2D x 3D) and ragged-K (2D x 2D)."""
    if offs is None or offs.dtype != torch.int32:
        raise RuntimeError("ctypes_ext._grouped_mm_cuda: the MoE layouts need int32 offs")
    if mat_a.dim() == 2 and mat_b.dim() == 3:
        out = torch.empty(mat_a.size(0), mat_b.size(2), dtype=torch.bfloat16, device=mat_a.device)
        _ragged_m(MGF_EPI_BIAS, mat_a, mat_b, offs, bias, out)
        return out
    if mat_a.dim() == 2 and mat_b.dim() == 2 and mat_a.stride(0) == 1 and bias is None:
        # ragged-K: mat_a is the transposed view of a row-major [total, m] matrix, mat_b row-major
        E, M, N = offs.numel(), mat_a.size(0), mat_b.size(1)
        out = torch.empty(E, M, N, dtype=torch.bfloat16, device=mat_a.device)
        ws = torch.zeros(1, dtype=torch.int32, device=mat_a.device)  # the dynamic tile counter
        g = MgfGemmDesc(epilogue=MGF_EPI_WGRAD, num_groups=E, total_rows=mat_a.size(1), m=M, n=N,
                        a=mat_a.data_ptr(), lda=mat_a.stride(1), b=mat_b.data_ptr(), ldb=mat_b.stride(0),
                        offs=offs.data_ptr(), d=out.data_ptr(), ldd=out.stride(1), ldd_batch=out.stride(0),
                        workspace=ws.data_ptr())
        _launch(g, mat_a.device)
        return out
    raise RuntimeError(f"ctypes_ext._grouped_mm_cuda: layout {mat_a.dim()}D x {mat_b.dim()}D with these strides "
                       "is not bound here (use the grouped_mm torch operators)")


def _grouped_mm_swiglu_cuda(mat_a, mat_b, offs, bias, aux_out=None, swiglu_out=None, swiglu_alpha=1.702,
                            swiglu_limit=7.0, store_aux=True):
    """csrc/binding.cu:39-64: aux_out = bf16(x W + b) (when store_aux), swiglu_out = SwiGLU(aux)."""
    d = aux_out if (store_aux and aux_out is not None) else swiglu_out
    _ragged_m(MGF_EPI_SWIGLU, mat_a, mat_b, offs, bias, d, d2=swiglu_out, alpha=swiglu_alpha,
              limit=swiglu_limit, store_aux=bool(store_aux and aux_out is not None))


def _grouped_mm_swiglu_bwd_cuda(grad_output, down_w_t, offs, aux_packed, grad_gate_up_packed, swiglu_alpha,
                                swiglu_limit):
    """csrc/binding.cu:68-118: grad_gate_up = SwiGLU_bwd(grad_output W_down^T, aux) on packed fp32 views."""
    aux = aux_packed.view(torch.bfloat16)
    grad = grad_gate_up_packed.view(torch.bfloat16)
    _ragged_m(MGF_EPI_SWIGLU_BWD, grad_output, down_w_t, offs, None, grad, aux=aux, alpha=swiglu_alpha,
              limit=swiglu_limit)
