"""Loader for the native libraries of the MoE FFN grouped-GEMM path.

`libmoe_gemm.so` holds the sm_100a kernels behind the C ABI of include/moe_gemm.h;
`_grouped_mm_ops.so` registers the `grouped_mm::*` torch operators on top of it.  Both are built
in-tree by cute-moe-train_b200/build.py.  There is no fallback: if a library is missing the
import fails with the command that builds it.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libmoe_gemm.so"
OPS_PATH = _HERE / "_grouped_mm_ops.so"

# Device status bits (include/moe_gemm.h).
DEV_WAIT_TIMEOUT = 0x1
DEV_BAD_OFFS = 0x2
DEV_ROW_OUT_OF_RANGE = 0x4


def _require(path: Path) -> None:
    if not path.exists():
        raise ImportError(
            f"{path.name} is not built; run `python cute-moe-train_b200/build.py` "
            "(or __graft_entry__.build()) first. This path has no CPU fallback."
        )


_require(LIB_PATH)
_require(OPS_PATH)
# Load the C-ABI library first (global symbols) so the ops library resolves against this copy.
lib = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_GLOBAL)
lib.mgf_version.restype = ctypes.c_int
lib.mgf_status_string.restype = ctypes.c_char_p
lib.mgf_status_string.argtypes = [ctypes.c_int]
lib.mgf_device_status.restype = ctypes.c_int
lib.mgf_device_status.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]
lib.mgf_ipc_open.restype = ctypes.c_int
lib.mgf_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
lib.mgf_ipc_get_handle.restype = ctypes.c_int
lib.mgf_ipc_get_handle.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]
lib.mgf_ipc_close.restype = ctypes.c_int
lib.mgf_ipc_close.argtypes = [ctypes.c_void_p]
torch.ops.load_library(str(OPS_PATH))


def ipc_handle(ptr: int) -> tuple[bytes, int]:
    """(64-byte IPC handle of the allocation holding device address `ptr`, ptr's offset in it)."""
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_int64(0)
    rc = lib.mgf_ipc_get_handle(ctypes.c_void_p(ptr), buf, ctypes.byref(off))
    if rc != 0:
        raise RuntimeError(f"mgf_ipc_get_handle failed: {lib.mgf_status_string(rc).decode()}")
    return buf.raw, int(off.value)


def ipc_open(handle: bytes) -> int:
    """Map a peer's CUDA IPC allocation into the current device's context; returns its base address."""
    if len(handle) != 64:
        raise RuntimeError(f"ipc_open: expected a 64-byte cudaIpcMemHandle_t, got {len(handle)} bytes")
    out = ctypes.c_void_p()
    rc = lib.mgf_ipc_open(handle, ctypes.byref(out))
    if rc != 0:
        raise RuntimeError(f"mgf_ipc_open failed: {lib.mgf_status_string(rc).decode()}")
    return int(out.value)


def ipc_close(base: int) -> None:
    lib.mgf_ipc_close(ctypes.c_void_p(base))


def device_status(device: int | None = None, clear: bool = True) -> int:
    """Synchronise `device` and return its kernel status bits (0 = clean); clears them by default."""
    if device is None:
        device = torch.cuda.current_device()
    out = ctypes.c_uint32(0)
    rc = lib.mgf_device_status(int(device), ctypes.byref(out), 1 if clear else 0)
    if rc != 0:
        raise RuntimeError(f"mgf_device_status failed: {lib.mgf_status_string(rc).decode()}")
    return int(out.value)


def check_device_status(device: int | None = None) -> None:
    """Raise RuntimeError if a kernel on `device` recorded a problem since the last check."""
    st = device_status(device, clear=True)
    if st:
        what = []
        if st & DEV_WAIT_TIMEOUT:
            what.append("a pipeline wait ran out and the kernel stopped early")
        if st & DEV_BAD_OFFS:
            what.append("offs was not non-decreasing within [0, total rows]")
        if st & DEV_ROW_OUT_OF_RANGE:
            what.append("a gather/combine/push row index fell outside its buffer (row skipped)")
        raise RuntimeError("grouped_mm device status: " + "; ".join(what))


# ------------------------------------------------------------------------ the reference binding's API
# Butterfingrz/CuTe-MoE-Train exposes three functions from its compiled `_ext` module
# (cutlass_op/bf16_grouped_mm/csrc/binding.cu:121-145); its custom_op.py calls them, and so may code
# that imports `_ext` directly.  Same names, arguments, defaults and in-place outputs here.

def _grouped_mm_cuda(mat_a: torch.Tensor, mat_b: torch.Tensor, offs: torch.Tensor | None = None,
                     bias: torch.Tensor | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Grouped GEMM (+ per-group bias); returns a new output (csrc/binding.cu:13-34)."""
    from .custom_op import dtype_to_int

    return torch.ops.grouped_mm.mm(mat_a, mat_b, offs, bias, dtype_to_int(out_dtype))


def _grouped_mm_swiglu_cuda(mat_a: torch.Tensor, mat_b: torch.Tensor, offs: torch.Tensor, bias: torch.Tensor,
                            aux_out: torch.Tensor | None = None, swiglu_out: torch.Tensor | None = None,
                            swiglu_alpha: float = 1.702, swiglu_limit: float = 7.0, store_aux: bool = True) -> None:
    """Fused GEMM + bias + SwiGLU into the caller's `swiglu_out` (and `aux_out` when store_aux)
    (csrc/binding.cu:36-63)."""
    if swiglu_out is None:
        raise TypeError("_grouped_mm_swiglu_cuda: swiglu_out is required")
    torch.ops.grouped_mm.swiglu_into(mat_a, mat_b, offs, bias, aux_out, swiglu_out, swiglu_alpha, swiglu_limit,
                                     store_aux)


def _grouped_mm_swiglu_bwd_cuda(grad_output: torch.Tensor, down_w_t: torch.Tensor, offs: torch.Tensor,
                                aux_packed: torch.Tensor, grad_gate_up_packed: torch.Tensor,
                                swiglu_alpha: float, swiglu_limit: float) -> None:
    """Fused down-proj dgrad + SwiGLU backward into `grad_gate_up_packed` (fp32 [M, I] views of bf16
    pairs, csrc/binding.cu:68-118)."""
    torch.ops.grouped_mm.swiglu_bwd_into(grad_output, down_w_t, offs, aux_packed, grad_gate_up_packed,
                                         swiglu_alpha, swiglu_limit)
