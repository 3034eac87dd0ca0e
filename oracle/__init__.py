"""CPU oracle of the MoE FFN grouped-GEMM path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline / reference leg,
as the checker or the timed CPU baseline; the product path (cute-moe-train_b200/) never imports
it and fails loudly when its CUDA libraries are missing.  Parity is pinned against outputs of the
reference's own Python layer (tests/golden/, made by tests/golden/make_golden.py); the reference's
CUDA kernels cannot run here, so kernel-level numerics are pinned through that CPU stand-in only.
"""
