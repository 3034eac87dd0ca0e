"""Operator schemas, wrapper signatures and fake-tensor shape inference (no GPU needed)."""

from __future__ import annotations

import inspect

import pytest
import torch


def _pkg():
    import cutlass_op.bf16_grouped_mm as m

    return m


REF_SCHEMAS = {
    "mm": "grouped_mm::mm(Tensor mat_a, Tensor mat_b, Tensor? offs, Tensor? bias, int out_dtype) -> Tensor",
    "mm_swiglu": "grouped_mm::mm_swiglu(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor bias, float swiglu_alpha, "
                 "float swiglu_limit) -> (Tensor, Tensor)",
    "mm_swiglu_bwd": "grouped_mm::mm_swiglu_bwd(Tensor grad_out, Tensor down_w_t, Tensor offs, Tensor aux_biased_acc, "
                     "float swiglu_alpha, float swiglu_limit) -> Tensor",
    "mm_downproj": "grouped_mm::mm_downproj(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor? bias, "
                   "Tensor aux_biased_acc, float swiglu_alpha, float swiglu_limit) -> Tensor",
}


@pytest.mark.parametrize("op", sorted(REF_SCHEMAS))
def test_schema_matches_reference(op):
    _pkg()
    schema = str(getattr(torch.ops.grouped_mm, op).default._schema)
    assert schema == REF_SCHEMAS[op]


def test_wrapper_signatures_and_defaults():
    m = _pkg()
    s = inspect.signature(m.grouped_mm_swiglu)
    assert list(s.parameters) == ["mat_a", "mat_b", "offs", "bias", "swiglu_alpha", "swiglu_limit"]
    assert s.parameters["swiglu_alpha"].default == 1.702 and s.parameters["swiglu_limit"].default == 7.0
    s = inspect.signature(m.grouped_mm_downproj)
    assert list(s.parameters) == ["mat_a", "mat_b", "offs", "bias", "aux_biased_acc", "swiglu_alpha", "swiglu_limit"]
    s = inspect.signature(m.grouped_mm)
    assert list(s.parameters) == ["mat_a", "mat_b", "offs", "bias", "out_dtype"]
    assert set(m.__all__) == {"grouped_mm", "grouped_mm_downproj", "grouped_mm_swiglu"}


def _meta(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, dtype=dtype, device="meta")


def test_fake_shapes_ffn():
    m = _pkg()
    E, H, I, M = 8, 2048, 1024, 864
    x, wu, bu = _meta(M, H), _meta(E, H, 2 * I), _meta(E, 2 * I)
    wd, bd = _meta(E, I, H), _meta(E, H)
    offs = _meta(E, dtype=torch.int32)
    s, aux = m.grouped_mm_swiglu(x, wu, offs, bu)
    assert s.shape == (M, I) and aux.shape == (M, 2 * I) and s.stride() == (I, 1)
    out = m.grouped_mm_downproj(s, wd, offs, bd, aux)
    assert out.shape == (M, H)
    g = torch.ops.grouped_mm.mm_swiglu_bwd(out, wd.transpose(-2, -1), offs, aux, 1.702, 7.0)
    assert g.shape == aux.shape
    dw, db = torch.ops.grouped_mm.mm_wgrad_bias(x.transpose(0, 1), aux, offs)
    assert dw.shape == (E, H, 2 * I) and db.shape == (E, 2 * I)


def test_fake_shapes_grouped_mm_variants():
    m = _pkg()
    offs = _meta(4, dtype=torch.int32)
    assert m.grouped_mm(_meta(100, 64), _meta(4, 64, 40), offs).shape == (100, 40)
    # padded row stride for N not a multiple of 8 (16-byte rule)
    assert m.grouped_mm(_meta(100, 64), _meta(4, 64, 36), offs).stride() == (40, 1)
    assert m.grouped_mm(_meta(64, 100), _meta(100, 40), offs).shape == (4, 64, 40)
    assert m.grouped_mm(_meta(3, 10, 64), _meta(3, 64, 40)).shape == (3, 10, 40)


def test_out_dtype_codes():
    from cutlass_op.bf16_grouped_mm.custom_op import _dtype_from_int, dtype_to_int

    assert dtype_to_int(None) == -1
    assert _dtype_from_int(dtype_to_int(torch.bfloat16)) == torch.bfloat16


def test_cpu_tensors_rejected_loudly():
    """No CPU fallback: CPU inputs raise instead of computing."""
    m = _pkg()
    x = torch.zeros(8, 16, dtype=torch.bfloat16)
    w = torch.zeros(1, 16, 32, dtype=torch.bfloat16)
    with pytest.raises((RuntimeError, NotImplementedError)):
        m.grouped_mm_swiglu(x, w, torch.tensor([8], dtype=torch.int32), torch.zeros(1, 32, dtype=torch.bfloat16))


def test_zipf_routing_properties():
    from cutlass_op.bf16_grouped_mm.workloads import offs_from_counts, zipf_routing

    c = zipf_routing(24576, 32, 4, 1.1, seed=0, zero_experts=2)
    assert int(c.sum()) == 24576 * 4
    assert int((c == 0).sum()) >= 2
    assert int(c.max()) <= 24576  # without replacement: at most one copy of a token per expert
    assert any(int(v) % 128 for v in c)
    offs = offs_from_counts(c)
    assert offs.dtype == torch.int32 and int(offs[-1]) == 24576 * 4
    assert torch.equal(zipf_routing(24576, 32, 4, 1.1, seed=0, zero_experts=2), c)


def test_config5_forced_group_sizes():
    from cutlass_op.bf16_grouped_mm.workloads import config5_counts

    for tokens in (64, 96, 4096):
        c = config5_counts(tokens, 256, 8, seed=1)
        assert int(c.sum()) == tokens * 8 and int(c.min()) >= 0
        for sz in (0, 1, 7, 129):
            assert sz in c.tolist()


def test_recompute_path_shapes():
    """store_aux=False: mm_swiglu_noaux returns swiglu_out only; the whole-FFN function runs its
    forward on meta tensors with and without aux."""
    from cutlass_op.bf16_grouped_mm import grouped_mm_ffn

    _pkg()
    assert "mm_swiglu_noaux(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor bias, float swiglu_alpha, " \
           "float swiglu_limit) -> Tensor" in str(torch.ops.grouped_mm.mm_swiglu_noaux.default._schema)
    E, H, I, M = 4, 256, 128, 300
    x, wu, bu = _meta(M, H), _meta(E, H, 2 * I), _meta(E, 2 * I)
    wd, bd = _meta(E, I, H), _meta(E, H)
    offs = _meta(E, dtype=torch.int32)
    s = torch.ops.grouped_mm.mm_swiglu_noaux(x, wu, offs, bu, 1.702, 7.0)
    assert s.shape == (M, I)
    for store_aux in (True, False):
        assert grouped_mm_ffn(x, wu, wd, offs, bu, bd, store_aux=store_aux).shape == (M, H)


def test_segment_sum_cols_groups_columns_like_the_forward():
    """Ragged-N bias gradient: column c of group e (start(e) <= c < end(e)) lands at [e, c - start(e)];
    columns past offs[-1] belong to no group."""
    from cutlass_op.bf16_grouped_mm.custom_op import segment_sum_cols

    g = torch.randn(5, 10)
    offs = torch.tensor([3, 3, 8], dtype=torch.int32)
    got = segment_sum_cols(g, offs)
    ref = torch.zeros(3, 10)
    ref[0, :3] = g[:, 0:3].sum(0)
    ref[2, :5] = g[:, 3:8].sum(0)
    assert torch.allclose(got, ref, atol=1e-6)


def test_fake_shape_ragged_n():
    m = _pkg()
    offs = _meta(3, dtype=torch.int32)
    out = m.grouped_mm(_meta(3, 72, 64), _meta(64, 208), offs)
    assert out.shape == (72, 208)


def test_fp8_ops_registered_and_shapes():
    from cutlass_op.bf16_grouped_mm import fp8

    _pkg()
    E, K, N, M = 4, 256, 128, 300
    a = torch.empty(M, K, dtype=torch.float8_e4m3fn, device="meta")
    b = torch.empty(E, N, K, dtype=torch.float8_e4m3fn, device="meta").transpose(1, 2)
    offs = _meta(E, dtype=torch.int32)
    sa, sb = _meta(M, dtype=torch.float32), _meta(E, N, dtype=torch.float32)
    assert fp8.grouped_mm_fp8(a, b, offs, sa, sb).shape == (M, N)
    s, aux = fp8.grouped_mm_swiglu_fp8(a, b, offs, sa, sb, _meta(E, N))
    assert s.shape == (M, N // 2) and aux.shape == (M, N)


def test_fp8_quantizers_round_trip():
    """Row-wise e4m3 quantisation keeps every element within e4m3's relative step of its value."""
    from cutlass_op.bf16_grouped_mm import fp8

    g = torch.Generator().manual_seed(0)
    x = torch.randn(37, 72, generator=g)
    q, s = fp8.quantize_rows(x)
    assert q.dtype == torch.float8_e4m3fn and q.stride(0) % 16 == 0 and s.shape == (37,)
    err = (fp8.dequantize_rows(q, s) - x).abs()
    assert (err <= x.abs() * 2 ** -3 + s[:, None] * 2 ** -6).all()
    w = torch.randn(3, 72, 40, generator=g)
    qw, sw = fp8.quantize_weights(w)
    assert qw.shape == (3, 72, 40) and qw.stride(1) == 1 and sw.shape == (3, 40)
    errw = (fp8.dequantize_weights(qw, sw) - w).abs()
    assert (errw <= w.abs() * 2 ** -3 + sw[:, None, :] * 2 ** -6).all()


def test_reference_binding_functions():
    """The reference's compiled `_ext` functions exist with its argument names and defaults
    (csrc/binding.cu:121-145)."""
    from cutlass_op.bf16_grouped_mm import _ext

    s = inspect.signature(_ext._grouped_mm_cuda)
    assert list(s.parameters) == ["mat_a", "mat_b", "offs", "bias", "out_dtype"]
    assert all(s.parameters[k].default is None for k in ("offs", "bias", "out_dtype"))
    s = inspect.signature(_ext._grouped_mm_swiglu_cuda)
    assert list(s.parameters) == ["mat_a", "mat_b", "offs", "bias", "aux_out", "swiglu_out", "swiglu_alpha",
                                  "swiglu_limit", "store_aux"]
    assert s.parameters["aux_out"].default is None and s.parameters["store_aux"].default is True
    s = inspect.signature(_ext._grouped_mm_swiglu_bwd_cuda)
    assert list(s.parameters) == ["grad_output", "down_w_t", "offs", "aux_packed", "grad_gate_up_packed",
                                  "swiglu_alpha", "swiglu_limit"]


def test_reference_module_names_present():
    """Every module-level function / name the reference's custom_op.py defines exists here."""
    import cutlass_op.bf16_grouped_mm.custom_op as c

    names = ["grouped_mm_forward", "grouped_mm_swiglu_forward", "grouped_mm_swiglu_bwd_forward",
             "grouped_mm_downproj_forward", "grouped_mm_setup_context", "grouped_mm_backward",
             "grouped_mm_swiglu_setup_context", "grouped_mm_swiglu_backward", "grouped_mm_downproj_setup_context",
             "grouped_mm_downproj_backward", "_segment_sum_rows", "_segment_sum_cols", "_infer_grouped_mm_out_shape",
             "_infer_grouped_mm_out_strides", "_empty_grouped_mm_output", "_empty_swiglu_output", "_as_packed_fp32",
             "_dtype_from_int", "_has_effective_grad"]
    assert [n for n in names if not hasattr(c, n)] == []
    assert c._infer_grouped_mm_out_strides((10, 36), torch.bfloat16, a_is_2d=True, b_is_2d=False) == (40, 1)
    assert c._infer_grouped_mm_out_strides((3, 10, 36), torch.bfloat16, a_is_2d=True, b_is_2d=True) == (400, 40, 1)
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    assert c._as_packed_fp32(x, tensor_name="x").shape == (4, 4)


def test_segment_sum_rows_matches_a_loop():
    """Ragged-M bias gradient (custom_op.py:79-101): fp32 row sums per group; rows past offs[-1] and
    empty groups contribute nothing."""
    from cutlass_op.bf16_grouped_mm.custom_op import segment_sum_rows

    g = torch.randn(11, 6, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    offs = torch.tensor([4, 4, 9], dtype=torch.int32)  # group 1 empty, rows 9-10 in no group
    got = segment_sum_rows(g, offs)
    ref = torch.zeros(3, 6)
    ref[0] = g[0:4].float().sum(0)
    ref[2] = g[4:9].float().sum(0)
    assert got.dtype == torch.bfloat16 and torch.equal(got, ref.to(torch.bfloat16))
