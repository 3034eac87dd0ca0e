"""The allocation-free weight-gradient entry point, called through the C ABI.

Callers that cannot allocate device memory when they launch (a runtime with a fixed, up-front
memory plan, or a host program binding the C ABI that only holds the buffers it was given) use
mgf_grouped_gemm_launch_noalloc: the ragged-K weight-gradient kernel then takes its zero-filled tile
counter from a static array inside the library instead of a caller-provided workspace.  This test
checks that entry point against the regular one (the grouped_mm::mm_wgrad_bias operator, which
passes a freshly zeroed workspace) on two calls in a row -- the second call must not see the first
call's counter.  It lives in its own file, collected last, and also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import moe_ffn as O

pytestmark = pytest.mark.gpu


class MgfGemmDesc(ctypes.Structure):
    """include/moe_gemm.h: mgf_gemm_desc."""

    _fields_ = [("epilogue", ctypes.c_int32), ("num_groups", ctypes.c_int32), ("total_rows", ctypes.c_int64),
                ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64), ("a", ctypes.c_void_p),
                ("lda", ctypes.c_int64), ("b", ctypes.c_void_p), ("ldb", ctypes.c_int64),
                ("ldb_batch", ctypes.c_int64), ("b_mn_major", ctypes.c_int32), ("offs", ctypes.c_void_p),
                ("bias", ctypes.c_void_p), ("bias_stride", ctypes.c_int64), ("d", ctypes.c_void_p),
                ("ldd", ctypes.c_int64), ("ldd_batch", ctypes.c_int64), ("d2", ctypes.c_void_p),
                ("ldd2", ctypes.c_int64), ("aux", ctypes.c_void_p), ("ld_aux", ctypes.c_int64),
                ("swiglu_alpha", ctypes.c_float), ("swiglu_limit", ctypes.c_float), ("store_aux", ctypes.c_int32),
                ("sm_carveout", ctypes.c_int32), ("workspace", ctypes.c_void_p), ("bias_per_row", ctypes.c_int32),
                ("ab_type", ctypes.c_int32), ("scale_a", ctypes.c_void_p), ("scale_b", ctypes.c_void_p),
                ("scale_b_stride", ctypes.c_int64), ("d_row_ptrs", ctypes.c_void_p), ("group_begin", ctypes.c_int32)]


MGF_EPI_WGRAD = 3


def _lib():
    from cutlass_op.bf16_grouped_mm import _ext

    lib = _ext.lib
    lib.mgf_grouped_gemm_launch_noalloc.argtypes = [ctypes.POINTER(MgfGemmDesc), ctypes.c_void_p]
    lib.mgf_grouped_gemm_launch_noalloc.restype = ctypes.c_int
    lib.mgf_last_error_detail.restype = ctypes.c_char_p
    return lib


def _noalloc_wgrad(x, g, offs):
    """dW [E, m, n] and db [E, n] for dW[e] = x[rows(e)]^T g[rows(e)], via the no-alloc entry point."""
    lib = _lib()
    E, m, n = offs.numel(), x.shape[1], g.shape[1]
    dw = torch.full((E, m, n), float("nan"), dtype=torch.bfloat16, device=x.device)
    db = torch.full((E, n), float("nan"), dtype=torch.bfloat16, device=x.device)
    desc = MgfGemmDesc(epilogue=MGF_EPI_WGRAD, num_groups=E, total_rows=x.shape[0], m=m, n=n, a=x.data_ptr(),
                       lda=x.stride(0), b=g.data_ptr(), ldb=g.stride(0), offs=offs.data_ptr(), d=dw.data_ptr(),
                       ldd=dw.stride(1), ldd_batch=dw.stride(0), d2=db.data_ptr(), ldd2=db.stride(0),
                       swiglu_alpha=1.702, swiglu_limit=7.0)
    rc = lib.mgf_grouped_gemm_launch_noalloc(ctypes.byref(desc), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, (rc, lib.mgf_last_error_detail())
    return dw, db


def test_noalloc_wgrad_matches_regular_entry_point_twice():
    from cutlass_op.bf16_grouped_mm import check_device_status

    gen = torch.Generator().manual_seed(42)
    counts = [300, 0, 129, 1, 700, 64]
    M, H, N = sum(counts), 256, 384
    x = torch.randn(M, H, generator=gen).to(torch.bfloat16).cuda()
    offs = torch.cumsum(torch.tensor(counts), 0).to(torch.int32).cuda()
    for call in range(2):
        g = torch.randn(M, N, generator=gen).to(torch.bfloat16).cuda()
        ref_dw, ref_db = torch.ops.grouped_mm.mm_wgrad_bias(x.t(), g, offs)
        dw, db = _noalloc_wgrad(x, g, offs)
        torch.cuda.synchronize()
        check_device_status()
        for name, got, ref in (("dw", dw, ref_dw), ("db", db, ref_db)):
            r = O.check(f"call{call}:{name}", got.float().cpu(), ref.float().cpu())
            assert r["ok"], r
        assert torch.count_nonzero(dw[1]).item() == 0 and torch.count_nonzero(db[1]).item() == 0


def test_noalloc_rejects_other_epilogues_and_workspace():
    lib = _lib()
    desc = MgfGemmDesc(epilogue=0, num_groups=1)
    assert lib.mgf_grouped_gemm_launch_noalloc(ctypes.byref(desc), None) != 0
    assert b"MGF_EPI_WGRAD" in lib.mgf_last_error_detail()
    desc = MgfGemmDesc(epilogue=MGF_EPI_WGRAD, num_groups=1, workspace=16)
    assert lib.mgf_grouped_gemm_launch_noalloc(ctypes.byref(desc), None) != 0
    assert b"workspace" in lib.mgf_last_error_detail()
