"""Drop-in package path of the reference (`cutlass_op.bf16_grouped_mm`) for the B200 build."""
