// torch.library registration of the `grouped_mm` operator namespace on top of the C ABI in
// moe_gemm.h.  Schemas, argument meaning, output allocation (16-byte padded row stride) and the
// error messages follow Butterfingrz/CuTe-MoE-Train (paths relative to cutlass_op/bf16_grouped_mm/):
//   grouped_mm::mm            custom_op.py:139-149, csrc/binding.cu:13-34, csrc/cutlass_utils.cuh:26-147
//   grouped_mm::mm_swiglu     custom_op.py:400-435, csrc/binding.cu:39-64
//   grouped_mm::mm_swiglu_bwd custom_op.py:534-558, csrc/binding.cu:68-118
//   grouped_mm::mm_downproj   custom_op.py:579-601
// Shape inference (fake tensors) and autograd are registered from Python, like the reference.
// Every launch goes on the current CUDA stream; nothing here synchronises or reads offs on the host.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstring>

#include "moe_gemm.h"

namespace {

using at::Tensor;

void check_launch(int rc, const char* what) {
  TORCH_CHECK(rc == MGF_OK, what, ": ", mgf_status_string(rc), " (status ", rc, ") ", mgf_last_error_detail());
}

int64_t padded(int64_t n) { return (n + 7) / 8 * 8; }

// csrc/cutlass_utils.cuh:66-81: one of the last two strides is 1 and the other a multiple of
// 16 bytes; returns true when the matrix is column-major (stride(-2) == 1).
bool check_strides_transposed(const Tensor& mat, const char* name) {
  const auto st = mat.strides();
  const auto sz = mat.sizes();
  const int end = mat.dim() - 1;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(mat.data_ptr()) % 16 == 0, name,
              ": expected data_ptr to be aligned to 16 bytes");
  if (st[end - 1] == 1 && st[end] >= std::max<int64_t>(1, sz[end - 1])) {
    TORCH_CHECK(st[end] % 8 == 0, name, ": strides should be multiple of 16 bytes");
    return true;
  }
  if (st[end] == 1 && st[end - 1] >= std::max<int64_t>(1, sz[end])) {
    TORCH_CHECK(st[end - 1] % 8 == 0, name, ": strides should be multiple of 16 bytes");
    return false;
  }
  TORCH_CHECK(false, "Invalid strides/sizes, got ", mat.strides(), " for strides and ", mat.sizes(), " for sizes");
  return false;
}

void check_offs(const Tensor& offs, const Tensor& ref) {
  TORCH_CHECK(offs.dim() == 1, "offs has to be 1D");
  TORCH_CHECK(offs.scalar_type() == at::kInt, "Offsets have to be int32");
  TORCH_CHECK(offs.is_contiguous(), "offs must be contiguous");
  TORCH_CHECK(offs.device() == ref.device(), "All tensors must be on the same device");
  TORCH_CHECK(offs.numel() >= 1 && offs.numel() <= 1024, "group count must be in [1, 1024], got ", offs.numel());
}

void check_bias(const Tensor& bias, int64_t groups, int64_t n) {
  TORCH_CHECK(bias.scalar_type() == at::kBFloat16, "Bias must be BFloat16, got ", bias.scalar_type());
  TORCH_CHECK(bias.dim() == 2, "Bias must be 2D [group_count, N] for per-group bias, got ", bias.dim(), "D");
  TORCH_CHECK(bias.size(0) == groups, "Bias first dimension must match group_count, expected ", groups, " got ",
              bias.size(0));
  TORCH_CHECK(bias.size(1) == n, "Bias second dimension must match N dimension, expected ", n, " got ", bias.size(1));
  TORCH_CHECK(bias.is_contiguous(), "Bias must be contiguous");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(bias.data_ptr()) % 16 == 0,
              "Bias data pointer must be 16-byte aligned for TMA transfers");
  TORCH_CHECK(bias.size(1) % 8 == 0, "Bias N dimension must be multiple of 8 elements (16 bytes), got ",
              bias.size(1));
}

mgf_gemm_desc base_desc() {
  mgf_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.swiglu_alpha = 1.702f;
  d.swiglu_limit = 7.0f;
  d.sm_carveout = 0;
  return d;
}

int sm_carveout_for(const Tensor& t) {
  // Honour PyTorch's SM carve-out knob (the reference reads it at
  // csrc/grouped_mm_kernel.cuh:355-356) so collectives can keep SMs free.
  auto c = at::globalContext()._SMCarveout_EXPERIMENTAL();
  (void)t;
  return c.has_value() ? static_cast<int>(*c) : 0;
}

// Ragged-M launch: A [total_rows, k] row-major, B [E, k, n] (either major), D [total_rows, n].
void launch_ragged_m(int epi, const Tensor& a, const Tensor& b, const Tensor& offs, const Tensor* bias,
                     const Tensor& d, const Tensor* d2, const Tensor* aux, double alpha, double limit,
                     bool store_aux, const char* what, bool bias_per_row = false, int64_t group_begin = 0) {
  const bool b_col_major = check_strides_transposed(b, "mat_b");
  mgf_gemm_desc g = base_desc();
  g.epilogue = epi;
  g.num_groups = static_cast<int32_t>(offs.numel());
  g.total_rows = a.size(0);
  g.k = a.size(1);
  g.n = b.size(2);
  g.a = a.data_ptr();
  g.lda = a.stride(0);
  g.b = b.data_ptr();
  g.b_mn_major = b_col_major ? 0 : 1;
  g.ldb = b_col_major ? b.stride(2) : b.stride(1);
  g.ldb_batch = b.stride(0);
  g.offs = offs.data_ptr<int32_t>();
  if (bias != nullptr) {
    g.bias = bias->data_ptr();
    g.bias_stride = bias->stride(0);
  }
  g.d = d.data_ptr();
  g.ldd = d.stride(0);
  if (d2 != nullptr) {
    g.d2 = d2->data_ptr();
    g.ldd2 = d2->stride(0);
  }
  if (aux != nullptr) {
    g.aux = aux->data_ptr();
    g.ld_aux = aux->stride(0);
  }
  g.swiglu_alpha = static_cast<float>(alpha);
  g.swiglu_limit = static_cast<float>(limit);
  g.store_aux = store_aux ? 1 : 0;
  g.bias_per_row = bias_per_row ? 1 : 0;
  g.group_begin = static_cast<int32_t>(group_begin);
  g.sm_carveout = sm_carveout_for(a);
  check_launch(mgf_grouped_gemm_launch(&g, at::cuda::getCurrentCUDAStream().stream()), what);
}

// Ragged-K launch: mat_a [M, total_K] is the transposed view (stride(0) == 1) of a row-major
// [total_K, M] matrix, mat_b [total_K, N] is row-major; returns (D [E, M, N], db [E, N] or undefined).
std::tuple<Tensor, Tensor> ragged_k_launch(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs,
                                           bool bias_grad, const char* what, const Tensor* out_in = nullptr,
                                           const Tensor* db_in = nullptr, int64_t group_begin = 0) {
  TORCH_CHECK(mat_a.stride(0) == 1, what,
              ": ragged-K needs mat_a as a transposed row-major matrix (stride(0) == 1)");
  TORCH_CHECK(mat_b.stride(1) == 1, what, ": ragged-K needs a row-major mat_b");
  TORCH_CHECK(mat_a.size(1) == mat_b.size(0), "contraction dimension of mat_a and mat_b must match");
  const int64_t E = offs.size(0), M = mat_a.size(0), N = mat_b.size(1);
  Tensor out = out_in != nullptr ? *out_in : at::empty_strided({E, M, N}, {M * padded(N), padded(N), 1}, mat_a.options());
  Tensor db = db_in != nullptr ? *db_in : Tensor();
  mgf_gemm_desc g = base_desc();
  g.epilogue = MGF_EPI_WGRAD;
  g.num_groups = static_cast<int32_t>(E);
  g.total_rows = mat_a.size(1);
  g.m = M;
  g.n = N;
  g.a = mat_a.data_ptr();
  g.lda = mat_a.stride(1);
  g.b = mat_b.data_ptr();
  g.ldb = mat_b.stride(0);
  g.offs = offs.data_ptr<int32_t>();
  g.d = out.data_ptr();
  g.ldd = out.stride(1);
  g.ldd_batch = out.stride(0);
  // dynamic tile counter of the ragged-K schedule (zero-filled, one per launch)
  Tensor workspace = at::zeros({1}, mat_a.options().dtype(at::kInt));
  g.workspace = workspace.data_ptr<int32_t>();
  if (bias_grad) {
    if (!db.defined()) db = at::empty({E, N}, mat_a.options());
    g.d2 = db.data_ptr();
    g.ldd2 = db.stride(0);
  }
  g.group_begin = static_cast<int32_t>(group_begin);
  g.sm_carveout = sm_carveout_for(mat_a);
  check_launch(mgf_grouped_gemm_launch(&g, at::cuda::getCurrentCUDAStream().stream()), what);
  return {out, db};
}

// In-place forms over a range of groups, for launches split by expert range (group_begin): the weight
// + bias gradient into dW [E, m, n] (unit column stride, rows padded to 16 bytes) and db [E, n], and the
// down-proj dgrad + SwiGLU backward into grad_aux [M, 2I].
void wgrad_bias_into_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs, const Tensor& dw,
                          const Tensor& db, int64_t group_begin) {
  TORCH_CHECK(mat_a.is_cuda() && mat_b.is_cuda() && mat_a.scalar_type() == at::kBFloat16 &&
                  mat_b.scalar_type() == at::kBFloat16 && dw.scalar_type() == at::kBFloat16 &&
                  db.scalar_type() == at::kBFloat16,
              "grouped_mm_wgrad_bias: bf16 CUDA tensors");
  check_offs(offs, mat_a);
  const int64_t E = offs.size(0);
  TORCH_CHECK(dw.dim() == 3 && dw.size(0) == E && dw.size(1) == mat_a.size(0) && dw.size(2) == mat_b.size(1) &&
                  dw.stride(2) == 1 && dw.stride(1) % 8 == 0 && dw.stride(0) % 8 == 0,
              "grouped_mm_wgrad_bias: dw must be [E, m, n] with unit column stride and 16-byte row pitch");
  TORCH_CHECK(db.dim() == 2 && db.size(0) == E && db.size(1) == mat_b.size(1) && db.stride(1) == 1 &&
                  db.stride(0) % 8 == 0,
              "grouped_mm_wgrad_bias: db must be [E, n] row-major");
  TORCH_CHECK(group_begin >= 0 && group_begin <= E, "grouped_mm_wgrad_bias: group_begin out of range");
  const c10::cuda::CUDAGuard guard(mat_a.device());
  ragged_k_launch(mat_a, mat_b, offs, true, "grouped_mm_wgrad_bias", &dw, &db, group_begin);
}

// Layout normalisation for the general `grouped_mm::mm` layouts the kernels do not read directly
// (the reference's CUTLASS kernel takes row- and column-major A and B on every path,
// csrc/grouped_mm_kernel.cuh:94-486).  These are explicit device copies into a layout the kernels
// take, off the MoE hot path; the MoE layouts never copy.
//
// A copy of the last two dims of `t` in row-major order with the row pitch padded to 8 elements.
Tensor row_major_padded(const Tensor& t) {
  const int64_t r = t.size(-2), c = t.size(-1);
  if (t.stride(-1) == 1 && t.stride(-2) % 8 == 0 && t.stride(-2) >= c &&
      (t.dim() == 2 || t.stride(0) == r * t.stride(-2)) && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0)
    return t;
  std::vector<int64_t> sizes(t.sizes().begin(), t.sizes().end());
  std::vector<int64_t> strides(t.dim());
  strides[t.dim() - 1] = 1;
  strides[t.dim() - 2] = padded(c);
  if (t.dim() == 3) strides[0] = r * padded(c);
  Tensor out = at::empty_strided(sizes, strides, t.options());
  out.copy_(t);
  return out;
}
// The same, column-major (a transposed view of a padded row-major copy of t^T).
Tensor col_major_padded(const Tensor& t) { return row_major_padded(t.transpose(-2, -1)).transpose(-2, -1); }

// ---------------------------------------------------------------- grouped_mm::mm
Tensor mm_cuda(const Tensor& mat_a, const Tensor& mat_b, const std::optional<Tensor>& offs,
               const std::optional<Tensor>& bias, int64_t out_dtype) {
  TORCH_CHECK(mat_a.is_cuda() && mat_b.is_cuda(), "grouped_mm: inputs must be CUDA tensors");
  const c10::cuda::CUDAGuard guard(mat_a.device());
  TORCH_CHECK(mat_a.dim() == 2 || mat_a.dim() == 3, "mat_a has to be 2 or 3d");
  TORCH_CHECK(mat_b.dim() == 2 || mat_b.dim() == 3, "mat_b has to be 2 or 3d");
  const bool a2 = mat_a.dim() == 2, b2 = mat_b.dim() == 2;
  if (!a2 || !b2)
    TORCH_CHECK(mat_a.size(-1) == mat_b.size(-2), "contraction dimension of mat_a and mat_b must match");
  TORCH_CHECK(offs.has_value() == (a2 || b2),
              "Have to provide offsets if there is a 2d matrix, or no offset if both matrices are 3d");
  if (out_dtype != -1)
    TORCH_CHECK(static_cast<c10::ScalarType>(out_dtype) == mat_a.scalar_type(),
                "Grouped gemm output dtype must match `mat_a` dtype");
  TORCH_CHECK(mat_a.scalar_type() == at::kBFloat16 && mat_b.scalar_type() == at::kBFloat16,
              "grouped_mm CUDA kernel currently supports only BFloat16 inputs/output. Got mat_a=",
              mat_a.scalar_type(), ", mat_b=", mat_b.scalar_type());
  const bool a_col = check_strides_transposed(mat_a, "mat_a");
  check_strides_transposed(mat_b, "mat_b");
  if (offs.has_value()) check_offs(*offs, mat_a);

  if (a2 && !b2) {
    // ragged-M: out [total_M, N]
    TORCH_CHECK(offs->size(0) == mat_b.size(0), "matrix batch sizes have to match");
    const Tensor a = a_col ? row_major_padded(mat_a) : mat_a;
    const int64_t N = mat_b.size(2);
    if (bias.has_value()) check_bias(*bias, mat_b.size(0), N);
    Tensor out = at::empty_strided({mat_a.size(0), N}, {padded(N), 1}, mat_a.options());
    launch_ragged_m(MGF_EPI_BIAS, a, mat_b, *offs, bias.has_value() ? &*bias : nullptr, out, nullptr, nullptr,
                    1.702, 7.0, false, "grouped_mm");
    return out;
  }
  if (a2 && b2) {
    TORCH_CHECK(!bias.has_value(), "grouped_mm: bias is not supported on the ragged-K path");
    // the kernel reads A as the transposed view of a row-major [total_K, M] and B row-major
    const Tensor a = (mat_a.stride(0) == 1) ? mat_a : col_major_padded(mat_a);
    const Tensor b = (mat_b.stride(1) == 1) ? mat_b : row_major_padded(mat_b);
    return std::get<0>(ragged_k_launch(a, b, *offs, false, "grouped_mm"));
  }
  if (!a2 && !b2) {
    // batched: [B, M, K] x [B, K, N] -> [B, M, N]; run as ragged-M with equal groups.
    TORCH_CHECK(mat_a.size(0) == mat_b.size(0), "batched dimension has to match");
    const Tensor a = row_major_padded(mat_a);
    const int64_t B = mat_a.size(0), M = mat_a.size(1), N = mat_b.size(2);
    if (bias.has_value()) check_bias(*bias, B, N);
    Tensor out = at::empty_strided({B, M, N}, {M * padded(N), padded(N), 1}, mat_a.options());
    TORCH_CHECK(B >= 1 && B <= 1024, "group count must be in [1, 1024]");
    Tensor boffs = at::arange(1, B + 1, mat_a.options().dtype(at::kInt)).mul_(static_cast<int>(M));
    Tensor a_flat = a.view({B * M, a.size(2)}).narrow(0, 0, B * M);
    Tensor out_flat = out.view({B * M, padded(N)}).narrow(1, 0, N);
    launch_ragged_m(MGF_EPI_BIAS, a_flat, mat_b, boffs, bias.has_value() ? &*bias : nullptr, out_flat, nullptr,
                    nullptr, 1.702, 7.0, false, "grouped_mm");
    return out;
  }
  // ragged-N: mat_a [E, M, K] x mat_b [K, total_N], groups along N (csrc/grouped_mm_common.cuh:107-118):
  // out[:, cols(e)] = mat_a[e] @ mat_b[:, cols(e)] + bias[e, col - start(e)].  Run as the ragged-M
  // GEMM of the transposed problem, out^T[cols(e), :] = mat_b^T[cols(e), :] @ mat_a[e]^T, whose bias is
  // per row, then transposed into the row-major [M, total_N] output.
  TORCH_CHECK(offs->size(0) == mat_a.size(0), "matrix batch sizes have to match");
  const int64_t E = mat_a.size(0), M = mat_a.size(1), total_n = mat_b.size(1);
  if (bias.has_value()) check_bias(*bias, E, total_n);
  const Tensor at_rows = row_major_padded(mat_b.transpose(0, 1));  // [total_N, K]
  // mat_a^T as B of the ragged-M GEMM: [E, K, M] (either major); M padded to a multiple of 8 with
  // zero rows when needed so the kernel's n-extent stays in bounds
  Tensor a3 = mat_a;
  const int64_t Mp = padded(M);
  if (Mp != M || !(mat_a.stride(-1) == 1 || mat_a.stride(-2) == 1)) {
    a3 = at::zeros({E, Mp, mat_a.size(2)}, mat_a.options());
    a3.narrow(1, 0, M).copy_(mat_a);
  } else if (mat_a.stride(-1) == 1) {
    a3 = row_major_padded(mat_a);
  } else {
    a3 = col_major_padded(mat_a);
  }
  const Tensor bt = a3.transpose(-2, -1);  // [E, K, Mp]
  Tensor out_t = at::empty_strided({total_n, Mp}, {Mp, 1}, mat_a.options());
  launch_ragged_m(MGF_EPI_BIAS, at_rows, bt, *offs, bias.has_value() ? &*bias : nullptr, out_t, nullptr, nullptr,
                  1.702, 7.0, false, "grouped_mm", /*bias_per_row=*/true);
  Tensor out = at::empty_strided({M, total_n}, {padded(total_n), 1}, mat_a.options());
  out.copy_(out_t.narrow(1, 0, M).transpose(0, 1));
  return out;
}

// ---------------------------------------------------------------- grouped_mm::mm_swiglu
// store_aux = false is the reference binding's `_grouped_mm_swiglu_cuda(..., store_aux=False)`
// (csrc/binding.cu:36-63): only swiglu_out is written and the returned aux is undefined.
std::tuple<Tensor, Tensor> swiglu_launch(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs,
                                         const Tensor& bias, double alpha, double limit, bool store_aux) {
  TORCH_CHECK(mat_a.is_cuda() && mat_b.is_cuda(), "grouped_mm_swiglu: inputs must be CUDA tensors");
  const c10::cuda::CUDAGuard guard(mat_a.device());
  TORCH_CHECK(mat_a.dim() == 2 && mat_b.dim() == 3, "grouped_mm_swiglu requires mat_a 2D and mat_b 3D (ragged-M path)");
  TORCH_CHECK(mat_a.scalar_type() == at::kBFloat16 && mat_b.scalar_type() == at::kBFloat16,
              "grouped_mm_swiglu requires BFloat16 inputs");
  TORCH_CHECK(bias.scalar_type() == at::kBFloat16, "bias must be BFloat16");
  TORCH_CHECK(offs.scalar_type() == at::kInt, "offs must be int32");
  TORCH_CHECK(mat_a.size(1) == mat_b.size(1), "contraction dimension of mat_a and mat_b must match");
  TORCH_CHECK(!check_strides_transposed(mat_a, "mat_a"), "grouped_mm_swiglu requires a row-major mat_a");
  check_offs(offs, mat_a);
  TORCH_CHECK(offs.size(0) == mat_b.size(0), "matrix batch sizes have to match");
  const int64_t N = mat_b.size(2);
  TORCH_CHECK(N % 16 == 0, "grouped_mm_swiglu: 2*I must be a multiple of 16, got ", N);
  check_bias(bias, mat_b.size(0), N);
  const int64_t M = mat_a.size(0);
  Tensor swiglu_out = at::empty_strided({M, N / 2}, {padded(N / 2), 1}, mat_a.options());
  if (!store_aux) {
    // the kernel writes no aux row; swiglu_out stands in as the (unwritten) aux destination
    launch_ragged_m(MGF_EPI_SWIGLU, mat_a, mat_b, offs, &bias, swiglu_out, &swiglu_out, nullptr, alpha, limit,
                    false, "grouped_mm_swiglu_noaux");
    return {swiglu_out, Tensor()};
  }
  Tensor aux_out = at::empty_strided({M, N}, {padded(N), 1}, mat_a.options());
  launch_ragged_m(MGF_EPI_SWIGLU, mat_a, mat_b, offs, &bias, aux_out, &swiglu_out, nullptr, alpha, limit, true,
                  "grouped_mm_swiglu");
  return {swiglu_out, aux_out};
}

std::tuple<Tensor, Tensor> mm_swiglu_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs,
                                          const Tensor& bias, double alpha, double limit) {
  return swiglu_launch(mat_a, mat_b, offs, bias, alpha, limit, true);
}

// ---------------------------------------------------------------- into-output forms (the reference binding)
// csrc/binding.cu:36-63 `_grouped_mm_swiglu_cuda(mat_a, mat_b, offs, bias, aux_out, swiglu_out, alpha,
// limit, store_aux)`: the caller allocates swiglu_out [M, I] (and aux_out [M, 2I] when store_aux);
// the launch writes them in place.
void swiglu_range_into_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs, const Tensor& bias,
                            const std::optional<Tensor>& aux_out, const Tensor& swiglu_out, double alpha,
                            double limit, bool store_aux, int64_t group_begin) {
  TORCH_CHECK(mat_a.is_cuda() && mat_b.is_cuda(), "grouped_mm_swiglu: inputs must be CUDA tensors");
  const c10::cuda::CUDAGuard guard(mat_a.device());
  TORCH_CHECK(mat_a.dim() == 2 && mat_b.dim() == 3, "grouped_mm_swiglu requires mat_a 2D and mat_b 3D (ragged-M path)");
  TORCH_CHECK(mat_a.scalar_type() == at::kBFloat16 && mat_b.scalar_type() == at::kBFloat16,
              "grouped_mm_swiglu requires BFloat16 inputs");
  TORCH_CHECK(bias.scalar_type() == at::kBFloat16, "bias must be BFloat16");
  TORCH_CHECK(offs.scalar_type() == at::kInt, "offs must be int32");
  if (store_aux) {
    TORCH_CHECK(aux_out.has_value(), "grouped_mm_swiglu(store_aux=True) requires aux_out tensor");
    TORCH_CHECK(aux_out->scalar_type() == at::kBFloat16, "aux_out must be BFloat16");
  }
  TORCH_CHECK(mat_a.size(1) == mat_b.size(1), "contraction dimension of mat_a and mat_b must match");
  TORCH_CHECK(!check_strides_transposed(mat_a, "mat_a"), "grouped_mm_swiglu requires a row-major mat_a");
  check_offs(offs, mat_a);
  TORCH_CHECK(offs.size(0) == mat_b.size(0), "matrix batch sizes have to match");
  const int64_t M = mat_a.size(0), N = mat_b.size(2);
  TORCH_CHECK(N % 16 == 0, "grouped_mm_swiglu: 2*I must be a multiple of 16, got ", N);
  check_bias(bias, mat_b.size(0), N);
  TORCH_CHECK(swiglu_out.scalar_type() == at::kBFloat16 && swiglu_out.dim() == 2 && swiglu_out.size(0) == M &&
                  swiglu_out.size(1) == N / 2 && swiglu_out.stride(1) == 1,
              "swiglu_out must be a row-major bf16 [M, I]");
  if (store_aux)
    TORCH_CHECK(aux_out->dim() == 2 && aux_out->size(0) == M && aux_out->size(1) == N && aux_out->stride(1) == 1,
                "aux_out must be a row-major bf16 [M, 2*I]");
  TORCH_CHECK(group_begin >= 0 && group_begin <= offs.size(0), "grouped_mm_swiglu: group_begin out of range");
  launch_ragged_m(MGF_EPI_SWIGLU, mat_a, mat_b, offs, &bias, store_aux ? *aux_out : swiglu_out, &swiglu_out, nullptr,
                  alpha, limit, store_aux, "grouped_mm_swiglu", false, group_begin);
}

void swiglu_into_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs, const Tensor& bias,
                      const std::optional<Tensor>& aux_out, const Tensor& swiglu_out, double alpha, double limit,
                      bool store_aux) {
  swiglu_range_into_cuda(mat_a, mat_b, offs, bias, aux_out, swiglu_out, alpha, limit, store_aux, 0);
}

// csrc/binding.cu:68-118 `_grouped_mm_swiglu_bwd_cuda(grad_output, down_w_t, offs, aux_packed,
// grad_gate_up_packed, alpha, limit)`: aux and the result are the fp32 [M, I] views of bf16 (gate, up)
// pairs; the result is written in place.
void swiglu_bwd_into_cuda(const Tensor& grad_output, const Tensor& down_w_t, const Tensor& offs,
                          const Tensor& aux_packed, const Tensor& grad_packed, double alpha, double limit) {
  TORCH_CHECK(grad_output.dim() == 2, "grad_output must be 2D [M, H]");
  TORCH_CHECK(down_w_t.dim() == 3, "down_w_t must be 3D [E, H, I]");
  TORCH_CHECK(aux_packed.dim() == 2, "aux_packed must be 2D [M, I]");
  TORCH_CHECK(grad_packed.dim() == 2, "grad_gate_up_packed must be 2D [M, I]");
  TORCH_CHECK(offs.dim() == 1, "offs must be 1D [E]");
  TORCH_CHECK(grad_output.scalar_type() == at::kBFloat16 && down_w_t.scalar_type() == at::kBFloat16,
              "_grouped_mm_swiglu_bwd_cuda requires bf16 grad_output and down_w_t");
  TORCH_CHECK(aux_packed.scalar_type() == at::kFloat, "aux_packed must be float32");
  TORCH_CHECK(grad_packed.scalar_type() == at::kFloat, "grad_gate_up_packed must be float32");
  TORCH_CHECK(offs.scalar_type() == at::kInt, "offs must be int32");
  TORCH_CHECK(grad_output.size(0) == aux_packed.size(0) && aux_packed.sizes() == grad_packed.sizes(),
              "Expected [M, I] packed tensors with matching shape");
  TORCH_CHECK(down_w_t.size(0) == offs.size(0), "down_w_t.shape[0] must match offs.size(0)");
  TORCH_CHECK(grad_output.size(1) == down_w_t.size(1), "grad_output.shape[1] must match down_w_t.shape[1] (H)");
  TORCH_CHECK(down_w_t.size(2) == aux_packed.size(1), "down_w_t.shape[2] must match aux_packed.shape[1] (I)");
  TORCH_CHECK(grad_output.device() == down_w_t.device() && down_w_t.device() == offs.device() &&
                  offs.device() == aux_packed.device() && aux_packed.device() == grad_packed.device(),
              "All tensors must be on the same device");
  TORCH_CHECK(aux_packed.stride(1) == 1 && grad_packed.stride(1) == 1, "packed tensors must be row-major");
  const c10::cuda::CUDAGuard guard(grad_output.device());
  if (grad_output.numel() == 0) return;
  const Tensor aux = aux_packed.view(at::kBFloat16);  // [M, 2I]
  const Tensor grad = grad_packed.view(at::kBFloat16);
  launch_ragged_m(MGF_EPI_SWIGLU_BWD, grad_output.contiguous(), down_w_t, offs, nullptr, grad, nullptr, &aux, alpha,
                  limit, false, "grouped_mm_swiglu_bwd");
}

void swiglu_bwd_range_into_cuda(const Tensor& grad_output, const Tensor& down_w_t, const Tensor& offs,
                                const Tensor& aux, const Tensor& grad_aux, double alpha, double limit,
                                int64_t group_begin) {
  TORCH_CHECK(grad_output.is_cuda() && grad_output.dim() == 2 && grad_output.stride(1) == 1 &&
                  grad_output.scalar_type() == at::kBFloat16 && down_w_t.dim() == 3 &&
                  down_w_t.scalar_type() == at::kBFloat16,
              "grouped_mm_swiglu_bwd: bf16 grad_output [M, H] row-major and down_w_t [E, H, I]");
  check_offs(offs, grad_output);
  TORCH_CHECK(down_w_t.size(0) == offs.size(0) && grad_output.size(1) == down_w_t.size(1),
              "grouped_mm_swiglu_bwd: shapes");
  TORCH_CHECK(aux.scalar_type() == at::kBFloat16 && grad_aux.scalar_type() == at::kBFloat16 && aux.dim() == 2 &&
                  grad_aux.dim() == 2 && aux.size(0) == grad_output.size(0) && grad_aux.size(0) == aux.size(0) &&
                  aux.size(1) == 2 * down_w_t.size(2) && grad_aux.size(1) == aux.size(1) && aux.stride(1) == 1 &&
                  grad_aux.stride(1) == 1,
              "grouped_mm_swiglu_bwd: aux and grad_aux must be row-major bf16 [M, 2*I]");
  TORCH_CHECK(group_begin >= 0 && group_begin <= offs.size(0), "grouped_mm_swiglu_bwd: group_begin out of range");
  const c10::cuda::CUDAGuard guard(grad_output.device());
  if (grad_output.size(0) == 0) return;
  launch_ragged_m(MGF_EPI_SWIGLU_BWD, grad_output, down_w_t, offs, nullptr, grad_aux, nullptr, &aux, alpha, limit,
                  false, "grouped_mm_swiglu_bwd", false, group_begin);
}

// ---------------------------------------------------------------- grouped_mm::mm_swiglu_noaux
Tensor mm_swiglu_noaux_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs, const Tensor& bias,
                            double alpha, double limit) {
  return std::get<0>(swiglu_launch(mat_a, mat_b, offs, bias, alpha, limit, false));
}

// ---------------------------------------------------------------- grouped_mm::mm_swiglu_bwd
Tensor mm_swiglu_bwd_cuda(const Tensor& grad_out_in, const Tensor& down_w_t, const Tensor& offs,
                          const Tensor& aux_biased_acc, double alpha, double limit) {
  TORCH_CHECK(grad_out_in.is_cuda(), "grouped_mm_swiglu_bwd: inputs must be CUDA tensors");
  const c10::cuda::CUDAGuard guard(grad_out_in.device());
  if (grad_out_in.numel() == 0) return at::zeros_like(aux_biased_acc);
  Tensor grad_out = grad_out_in.contiguous();
  TORCH_CHECK(grad_out.dim() == 2, "grad_output must be 2D [M, H]");
  TORCH_CHECK(down_w_t.dim() == 3, "down_w_t must be 3D [E, H, I]");
  TORCH_CHECK(aux_biased_acc.dim() == 2, "aux_biased_acc must be 2D [M, 2*I]");
  TORCH_CHECK(grad_out.scalar_type() == at::kBFloat16 && down_w_t.scalar_type() == at::kBFloat16,
              "_grouped_mm_swiglu_bwd_cuda requires bf16 grad_output and down_w_t");
  TORCH_CHECK(aux_biased_acc.scalar_type() == at::kBFloat16, "aux_biased_acc must be bfloat16, got ",
              aux_biased_acc.scalar_type());
  TORCH_CHECK(aux_biased_acc.size(-1) % 2 == 0, "aux_biased_acc.shape[-1] must be even for bf16 pair packing");
  TORCH_CHECK(aux_biased_acc.stride(-1) == 1, "aux_biased_acc must have stride(-1) == 1 for packed view");
  TORCH_CHECK(aux_biased_acc.stride(-2) % 2 == 0, "aux_biased_acc.stride(-2) must be even for packed fp32 reinterpretation");
  check_offs(offs, grad_out);
  TORCH_CHECK(grad_out.size(0) == aux_biased_acc.size(0), "Expected [M, I] packed tensors with matching shape");
  TORCH_CHECK(down_w_t.size(0) == offs.size(0), "down_w_t.shape[0] must match offs.size(0)");
  TORCH_CHECK(grad_out.size(1) == down_w_t.size(1), "grad_output.shape[1] must match down_w_t.shape[1] (H)");
  TORCH_CHECK(down_w_t.size(2) * 2 == aux_biased_acc.size(1), "down_w_t.shape[2] must match aux_packed.shape[1] (I)");
  TORCH_CHECK(grad_out.device() == down_w_t.device() && down_w_t.device() == aux_biased_acc.device(),
              "All tensors must be on the same device");
  Tensor grad_aux = at::empty_like(aux_biased_acc, at::MemoryFormat::Contiguous);
  TORCH_CHECK(grad_aux.stride(0) == aux_biased_acc.size(1), "grad_aux layout");
  launch_ragged_m(MGF_EPI_SWIGLU_BWD, grad_out, down_w_t, offs, nullptr, grad_aux, nullptr, &aux_biased_acc, alpha,
                  limit, false, "grouped_mm_swiglu_bwd");
  return grad_aux;
}

// ---------------------------------------------------------------- grouped_mm::mm_downproj
Tensor mm_downproj_cuda(const Tensor& mat_a, const Tensor& mat_b, const std::optional<Tensor>& offs,
                        const std::optional<Tensor>& bias, const Tensor& /*aux_biased_acc*/, double /*alpha*/,
                        double /*limit*/) {
  TORCH_CHECK(offs.has_value(), "grouped_mm::mm_downproj requires offs for ragged-M path");
  TORCH_CHECK(mat_a.dim() == 2 && mat_b.dim() == 3, "grouped_mm::mm_downproj requires mat_a 2D and mat_b 3D");
  return mm_cuda(mat_a, mat_b, offs, bias, -1);
}

// ---------------------------------------------------------------- grouped_mm::mm_fp8 / mm_swiglu_fp8
// Forward-only e4m3 variants of the ragged-M launches (BIAS and SWIGLU epilogues): mat_a [total_M, K]
// row-major e4m3 with per-row fp32 scales scale_a [total_M]; mat_b [E, K, N] e4m3 with unit stride
// along K (the transpose of a contiguous [E, N, K]) with per-(expert, column) scales scale_b [E, N].
// The accumulator is dequantised in fp32 (acc * scale_a[row] * scale_b[e, col]) before the bf16 bias
// and the epilogue; outputs are bf16 exactly as in mm / mm_swiglu.
void launch_ragged_m_f8(int epi, const Tensor& a, const Tensor& b, const Tensor& offs, const Tensor& scale_a,
                        const Tensor& scale_b, const Tensor* bias, const Tensor& d, const Tensor* d2, double alpha,
                        double limit, bool store_aux, const char* what, const Tensor* aux = nullptr) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && scale_a.is_cuda() && scale_b.is_cuda(), what,
              ": inputs must be CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && b.scalar_type() == at::kFloat8_e4m3fn, what,
              ": mat_a and mat_b must be float8_e4m3fn");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 3, what, ": requires mat_a 2D and mat_b 3D (ragged-M path)");
  TORCH_CHECK(a.size(1) == b.size(1), "contraction dimension of mat_a and mat_b must match");
  TORCH_CHECK(a.stride(1) == 1 && a.stride(0) % 16 == 0, what, ": mat_a must be row-major with a 16-byte row pitch");
  TORCH_CHECK(b.stride(1) == 1 && b.stride(2) % 16 == 0 && b.stride(0) % 16 == 0, what,
              ": mat_b must have unit stride along K (mat_b[e] = W[e].t() of a contiguous [E, N, K])");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              what, ": data pointers must be 16-byte aligned");
  check_offs(offs, a);
  TORCH_CHECK(offs.size(0) == b.size(0), "matrix batch sizes have to match");
  const int64_t N = b.size(2);
  TORCH_CHECK(scale_a.scalar_type() == at::kFloat && scale_a.dim() == 1 && scale_a.size(0) == a.size(0) &&
                  scale_a.is_contiguous(),
              what, ": scale_a must be a contiguous float32 [total_M]");
  TORCH_CHECK(scale_b.scalar_type() == at::kFloat && scale_b.dim() == 2 && scale_b.size(0) == b.size(0) &&
                  scale_b.size(1) == N && scale_b.stride(1) == 1 && scale_b.stride(0) % 4 == 0,
              what, ": scale_b must be a float32 [E, N] with unit column stride");
  mgf_gemm_desc g = base_desc();
  g.epilogue = epi;
  g.ab_type = MGF_AB_E4M3;
  g.num_groups = static_cast<int32_t>(offs.numel());
  g.total_rows = a.size(0);
  g.k = a.size(1);
  g.n = N;
  g.a = a.data_ptr();
  g.lda = a.stride(0);
  g.b = b.data_ptr();
  g.b_mn_major = 0;
  g.ldb = b.stride(2);
  g.ldb_batch = b.stride(0);
  g.offs = offs.data_ptr<int32_t>();
  g.scale_a = scale_a.data_ptr<float>();
  g.scale_b = scale_b.data_ptr<float>();
  g.scale_b_stride = scale_b.stride(0);
  if (bias != nullptr) {
    g.bias = bias->data_ptr();
    g.bias_stride = bias->stride(0);
  }
  g.d = d.data_ptr();
  g.ldd = d.stride(0);
  if (d2 != nullptr) {
    g.d2 = d2->data_ptr();
    g.ldd2 = d2->stride(0);
  }
  if (aux != nullptr) {
    g.aux = aux->data_ptr();
    g.ld_aux = aux->stride(0);
  }
  g.swiglu_alpha = static_cast<float>(alpha);
  g.swiglu_limit = static_cast<float>(limit);
  g.store_aux = store_aux ? 1 : 0;
  g.sm_carveout = sm_carveout_for(a);
  check_launch(mgf_grouped_gemm_launch(&g, at::cuda::getCurrentCUDAStream().stream()), what);
}

// e4m3 down-proj dgrad + SwiGLU backward: grad_aux = SwiGLU_bwd(dequant(grad_output @ down_w_t), aux),
// grad_output e4m3 [M, H] with row scales, down_w_t e4m3 [E, H, I] with unit stride along H and
// per-(expert, column) scales; aux and grad_aux bf16 [M, 2I] interleaved (gate, up).
Tensor mm_swiglu_bwd_fp8_cuda(const Tensor& grad_output, const Tensor& down_w_t, const Tensor& offs, const Tensor& aux,
                              const Tensor& scale_a, const Tensor& scale_b, double alpha, double limit) {
  const c10::cuda::CUDAGuard guard(grad_output.device());
  const int64_t I = down_w_t.size(2);
  TORCH_CHECK(aux.is_cuda() && aux.dim() == 2 && aux.scalar_type() == at::kBFloat16 && aux.stride(1) == 1 &&
                  aux.size(0) == grad_output.size(0) && aux.size(1) == 2 * I,
              "grouped_mm_swiglu_bwd_fp8: aux_biased_acc must be bf16 [M, 2*I] row-major");
  TORCH_CHECK(I % 8 == 0, "grouped_mm_swiglu_bwd_fp8: I must be a multiple of 8");
  Tensor grad = at::empty_strided({grad_output.size(0), 2 * I}, {padded(2 * I), 1}, aux.options());
  launch_ragged_m_f8(MGF_EPI_SWIGLU_BWD, grad_output, down_w_t, offs, scale_a, scale_b, nullptr, grad, nullptr, alpha,
                     limit, false, "grouped_mm_swiglu_bwd_fp8", &aux);
  return grad;
}

// e4m3 ragged-K weight gradient with the fused bias gradient: mat_a e4m3 [m, total] (the transposed
// view of a row-major [total, m]), mat_b e4m3 [total, n] row-major; per-feature fp32 scales
// scale_a [m] and scale_b [n]; dW[e] = (mat_a[:, rows(e)] @ mat_b[rows(e)]) * scale_a[:, None] * scale_b
// and db[e] = column sums of mat_b[rows(e)] * scale_b, both bf16.
std::tuple<Tensor, Tensor> mm_wgrad_fp8_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs,
                                             const Tensor& scale_a, const Tensor& scale_b, bool bias_grad) {
  const char* what = "grouped_mm_wgrad_fp8";
  const c10::cuda::CUDAGuard guard(mat_a.device());
  TORCH_CHECK(mat_a.scalar_type() == at::kFloat8_e4m3fn && mat_b.scalar_type() == at::kFloat8_e4m3fn, what,
              ": mat_a and mat_b must be float8_e4m3fn");
  TORCH_CHECK(mat_a.dim() == 2 && mat_b.dim() == 2 && mat_a.stride(0) == 1 && mat_b.stride(1) == 1, what,
              ": mat_a must be the transposed view of a row-major [total, m] and mat_b row-major [total, n]");
  TORCH_CHECK(mat_a.stride(1) % 16 == 0 && mat_b.stride(0) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(mat_a.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(mat_b.data_ptr()) % 16 == 0,
              what, ": 16-byte aligned bases and row pitches");
  TORCH_CHECK(mat_a.size(1) == mat_b.size(0), "contraction dimension of mat_a and mat_b must match");
  check_offs(offs, mat_b);
  const int64_t E = offs.size(0), M = mat_a.size(0), N = mat_b.size(1);
  TORCH_CHECK(N % 8 == 0, what, ": n must be a multiple of 8");
  TORCH_CHECK(scale_a.is_cuda() && scale_a.scalar_type() == at::kFloat && scale_a.is_contiguous() &&
                  scale_a.numel() == M && scale_b.is_cuda() && scale_b.scalar_type() == at::kFloat &&
                  scale_b.is_contiguous() && scale_b.numel() == N,
              what, ": scale_a [m] and scale_b [n] contiguous float32");
  auto opts = scale_a.options().dtype(at::kBFloat16);
  Tensor out = at::empty_strided({E, M, N}, {M * padded(N), padded(N), 1}, opts);
  Tensor db;
  mgf_gemm_desc g = base_desc();
  g.epilogue = MGF_EPI_WGRAD;
  g.ab_type = MGF_AB_E4M3;
  g.num_groups = static_cast<int32_t>(E);
  g.total_rows = mat_a.size(1);
  g.m = M;
  g.n = N;
  g.a = mat_a.data_ptr();
  g.lda = mat_a.stride(1);
  g.b = mat_b.data_ptr();
  g.ldb = mat_b.stride(0);
  g.offs = offs.data_ptr<int32_t>();
  g.scale_a = scale_a.data_ptr<float>();
  g.scale_b = scale_b.data_ptr<float>();
  g.d = out.data_ptr();
  g.ldd = out.stride(1);
  g.ldd_batch = out.stride(0);
  Tensor workspace = at::zeros({1}, offs.options());
  g.workspace = workspace.data_ptr<int32_t>();
  if (bias_grad) {
    db = at::empty({E, N}, opts);
    g.d2 = db.data_ptr();
    g.ldd2 = db.stride(0);
  }
  g.sm_carveout = sm_carveout_for(mat_b);
  check_launch(mgf_grouped_gemm_launch(&g, at::cuda::getCurrentCUDAStream().stream()), what);
  return {out, db};
}

Tensor mm_fp8_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs, const Tensor& scale_a,
                   const Tensor& scale_b, const std::optional<Tensor>& bias) {
  const c10::cuda::CUDAGuard guard(mat_a.device());
  const int64_t N = mat_b.size(2);
  if (bias.has_value()) check_bias(*bias, mat_b.size(0), N);
  TORCH_CHECK(N % 8 == 0, "grouped_mm_fp8: N must be a multiple of 8");
  Tensor out = at::empty_strided({mat_a.size(0), N}, {padded(N), 1}, mat_a.options().dtype(at::kBFloat16));
  launch_ragged_m_f8(MGF_EPI_BIAS, mat_a, mat_b, offs, scale_a, scale_b, bias.has_value() ? &*bias : nullptr, out,
                     nullptr, 1.702, 7.0, false, "grouped_mm_fp8");
  return out;
}

std::tuple<Tensor, Tensor> mm_swiglu_fp8_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs,
                                              const Tensor& scale_a, const Tensor& scale_b, const Tensor& bias,
                                              double alpha, double limit) {
  const c10::cuda::CUDAGuard guard(mat_a.device());
  const int64_t N = mat_b.size(2);
  TORCH_CHECK(N % 16 == 0, "grouped_mm_swiglu_fp8: 2*I must be a multiple of 16, got ", N);
  check_bias(bias, mat_b.size(0), N);
  const int64_t M = mat_a.size(0);
  auto opts = mat_a.options().dtype(at::kBFloat16);
  Tensor swiglu_out = at::empty_strided({M, N / 2}, {padded(N / 2), 1}, opts);
  Tensor aux_out = at::empty_strided({M, N}, {padded(N), 1}, opts);
  launch_ragged_m_f8(MGF_EPI_SWIGLU, mat_a, mat_b, offs, scale_a, scale_b, &bias, aux_out, &swiglu_out, alpha, limit,
                     true, "grouped_mm_swiglu_fp8");
  return {swiglu_out, aux_out};
}

// ---------------------------------------------------------------- grouped_mm::mm_wgrad_bias
// Weight gradient of a ragged-M layer fused with its bias gradient: for every group e,
// dW[e] = mat_a[:, rows(e)] @ mat_b[rows(e), :] and db[e] = sum over rows(e) of mat_b (fp32
// accumulation, one bf16 rounding).  Replaces the separate `_segment_sum_rows` pass of the
// reference (custom_op.py:79-101, called at custom_op.py:516-518 and 666-667).
std::tuple<Tensor, Tensor> mm_wgrad_bias_cuda(const Tensor& mat_a, const Tensor& mat_b, const Tensor& offs) {
  TORCH_CHECK(mat_a.is_cuda() && mat_b.is_cuda(), "grouped_mm_wgrad_bias: inputs must be CUDA tensors");
  const c10::cuda::CUDAGuard guard(mat_a.device());
  TORCH_CHECK(mat_a.dim() == 2 && mat_b.dim() == 2, "grouped_mm_wgrad_bias requires 2D mat_a and mat_b");
  TORCH_CHECK(mat_a.scalar_type() == at::kBFloat16 && mat_b.scalar_type() == at::kBFloat16,
              "grouped_mm_wgrad_bias requires BFloat16 inputs");
  check_strides_transposed(mat_a, "mat_a");
  check_strides_transposed(mat_b, "mat_b");
  check_offs(offs, mat_a);
  const Tensor a = (mat_a.stride(0) == 1) ? mat_a : col_major_padded(mat_a);
  const Tensor b = (mat_b.stride(1) == 1) ? mat_b : row_major_padded(mat_b);
  return ragged_k_launch(a, b, offs, true, "grouped_mm_wgrad_bias");
}

// ---------------------------------------------------------------- expert-parallel row movement
void check_rows(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.scalar_type() == at::kBFloat16 && t.stride(1) == 1,
              name, " must be a row-major 2D bf16 CUDA tensor");
}

Tensor gather_rows_cuda(const Tensor& src, const Tensor& idx_in, const std::optional<Tensor>& scale_in) {
  check_rows(src, "src");
  const c10::cuda::CUDAGuard guard(src.device());
  Tensor idx = idx_in.to(at::kLong).contiguous();
  Tensor out = at::empty({idx.numel(), src.size(1)}, src.options());
  Tensor scale;
  if (scale_in.has_value()) {
    scale = scale_in->to(at::kFloat).contiguous();
    TORCH_CHECK(scale.numel() == idx.numel(), "gather_rows: scale must have one entry per row");
  }
  check_launch(mgf_gather_rows(src.data_ptr(), src.stride(0), src.size(0), idx.data_ptr<int64_t>(),
                               scale.defined() ? scale.data_ptr<float>() : nullptr, idx.numel(), src.size(1),
                               out.data_ptr(), out.stride(0), at::cuda::getCurrentCUDAStream().stream()),
               "gather_rows");
  return out;
}

Tensor combine_rows_cuda(const Tensor& rows, const Tensor& pos_in, const std::optional<Tensor>& w_in, int64_t k) {
  check_rows(rows, "rows");
  const c10::cuda::CUDAGuard guard(rows.device());
  TORCH_CHECK(k >= 1 && pos_in.numel() % k == 0, "combine_rows: pos must hold k entries per output row");
  Tensor pos = pos_in.to(at::kLong).contiguous();
  const int64_t n_out = pos.numel() / k;
  Tensor out = at::empty({n_out, rows.size(1)}, rows.options());
  Tensor w;
  if (w_in.has_value()) {
    w = w_in->to(at::kFloat).contiguous();
    TORCH_CHECK(w.numel() == pos.numel(), "combine_rows: one weight per (row, slot)");
  }
  check_launch(mgf_combine_rows(rows.data_ptr(), rows.stride(0), rows.size(0), pos.data_ptr<int64_t>(),
                                w.defined() ? w.data_ptr<float>() : nullptr, n_out, static_cast<int32_t>(k),
                                rows.size(1), out.data_ptr(), out.stride(0), at::cuda::getCurrentCUDAStream().stream()),
               "combine_rows");
  return out;
}

// Rows of src pushed into other ranks' IPC-mapped buffers (see mgf_push_rows).
void push_rows_cuda(const Tensor& src, const std::optional<Tensor>& src_idx, const std::optional<Tensor>& scale,
                    const std::optional<Tensor>& n_dev, const Tensor& dst_rank, const Tensor& dst_row,
                    const Tensor& peer_bases, int64_t dst_rows, int64_t ld_dst, int64_t n_max,
                    const std::optional<Tensor>& flag_bases, const std::optional<Tensor>& counter, int64_t seq,
                    int64_t rank, const std::optional<Tensor>& rotate) {
  check_rows(src, "src");
  const c10::cuda::CUDAGuard guard(src.device());
  TORCH_CHECK(dst_rank.scalar_type() == at::kLong && dst_row.scalar_type() == at::kLong &&
                  peer_bases.scalar_type() == at::kLong && dst_rank.is_contiguous() && dst_row.is_contiguous() &&
                  peer_bases.is_contiguous(),
              "push_rows: dst_rank, dst_row and peer_bases must be contiguous int64");
  TORCH_CHECK(dst_rank.numel() >= n_max && dst_row.numel() >= n_max, "push_rows: index arrays shorter than n_max");
  const int64_t* si = nullptr;
  if (src_idx.has_value()) {
    TORCH_CHECK(src_idx->scalar_type() == at::kLong && src_idx->is_contiguous() && src_idx->numel() >= n_max,
                "push_rows: src_idx must be contiguous int64 with n_max entries");
    si = src_idx->data_ptr<int64_t>();
  }
  const float* sc = nullptr;
  if (scale.has_value()) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->is_contiguous() && scale->numel() >= n_max,
                "push_rows: scale must be contiguous float32 with n_max entries");
    sc = scale->data_ptr<float>();
  }
  const int32_t* nd = nullptr;
  if (n_dev.has_value()) {
    TORCH_CHECK(n_dev->scalar_type() == at::kInt && n_dev->numel() >= 1, "push_rows: n_dev must be int32");
    nd = n_dev->data_ptr<int32_t>();
  }
  if (rotate.has_value())
    TORCH_CHECK(rotate->is_cuda() && rotate->scalar_type() == at::kLong && rotate->numel() >= 1,
                "push_rows: rotate must be an int64 device scalar");
  const unsigned long long* fb = nullptr;
  unsigned long long* ctr = nullptr;
  if (flag_bases.has_value()) {
    TORCH_CHECK(counter.has_value() && flag_bases->scalar_type() == at::kLong && flag_bases->is_contiguous() &&
                    flag_bases->numel() == peer_bases.numel() && counter->scalar_type() == at::kLong &&
                    counter->numel() >= 1,
                "push_rows: flag_bases must be int64 [world] and counter an int64 device word");
    fb = reinterpret_cast<const unsigned long long*>(flag_bases->data_ptr<int64_t>());
    ctr = reinterpret_cast<unsigned long long*>(counter->data_ptr<int64_t>());
  }
  check_launch(mgf_push_rows(src.data_ptr(), src.stride(0), src.size(0), si, sc, n_max, nd,
                             dst_rank.data_ptr<int64_t>(), dst_row.data_ptr<int64_t>(),
                             reinterpret_cast<const unsigned long long*>(peer_bases.data_ptr<int64_t>()),
                             peer_bases.numel(), dst_rows, ld_dst, src.size(1), fb, ctr,
                             static_cast<unsigned long long>(seq), rank,
                             rotate.has_value() ? rotate->data_ptr<int64_t>() : nullptr,
                             at::cuda::getCurrentCUDAStream().stream()),
               "push_rows");
}

// Ragged-M GEMM + bias whose output rows go to per-row addresses (mgf_gemm_desc.d_row_ptrs), e.g.
// straight into the source ranks' combine buffers.
void mm_scatter_cuda(const Tensor& a, const Tensor& b, const Tensor& offs, const std::optional<Tensor>& bias,
                     const Tensor& row_ptrs) {
  TORCH_CHECK(a.is_cuda() && a.dim() == 2 && b.dim() == 3 && a.scalar_type() == at::kBFloat16 &&
                  b.scalar_type() == at::kBFloat16,
              "mm_scatter: mat_a [rows, k] and mat_b [E, k, n] bf16 CUDA tensors");
  TORCH_CHECK(a.stride(1) == 1, "mm_scatter: mat_a must be row-major");
  TORCH_CHECK(offs.scalar_type() == at::kInt && offs.dim() == 1 && offs.size(0) == b.size(0),
              "mm_scatter: offs must be int32 [E]");
  TORCH_CHECK(row_ptrs.scalar_type() == at::kLong && row_ptrs.is_contiguous() && row_ptrs.numel() >= a.size(0),
              "mm_scatter: row_ptrs must be contiguous int64 with one address per row");
  if (bias.has_value()) check_bias(*bias, b.size(0), b.size(2));
  const c10::cuda::CUDAGuard guard(a.device());
  const bool b_col_major = check_strides_transposed(b, "mat_b");
  mgf_gemm_desc g = base_desc();
  g.epilogue = MGF_EPI_BIAS;
  g.num_groups = static_cast<int32_t>(offs.numel());
  g.total_rows = a.size(0);
  g.k = a.size(1);
  g.n = b.size(2);
  g.a = a.data_ptr();
  g.lda = a.stride(0);
  g.b = b.data_ptr();
  g.b_mn_major = b_col_major ? 0 : 1;
  g.ldb = b_col_major ? b.stride(2) : b.stride(1);
  g.ldb_batch = b.stride(0);
  g.offs = offs.data_ptr<int32_t>();
  if (bias.has_value()) {
    g.bias = bias->data_ptr();
    g.bias_stride = bias->stride(0);
  }
  g.d_row_ptrs = row_ptrs.data_ptr<int64_t>();
  g.sm_carveout = sm_carveout_for(a);
  check_launch(mgf_grouped_gemm_launch(&g, at::cuda::getCurrentCUDAStream().stream()), "mm_scatter");
}

void signal_flags_cuda(const Tensor& flag_bases, int64_t rank, int64_t seq) {
  TORCH_CHECK(flag_bases.is_cuda() && flag_bases.scalar_type() == at::kLong && flag_bases.is_contiguous(),
              "signal_flags: flag_bases must be a contiguous int64 CUDA tensor");
  const c10::cuda::CUDAGuard guard(flag_bases.device());
  check_launch(mgf_signal_flags(reinterpret_cast<const unsigned long long*>(flag_bases.data_ptr<int64_t>()),
                                flag_bases.numel(), rank, static_cast<unsigned long long>(seq),
                                at::cuda::getCurrentCUDAStream().stream()),
               "signal_flags");
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> ep_sort_cuda(const Tensor& ids_in, int64_t num_experts,
                                                                int64_t topk) {
  TORCH_CHECK(ids_in.is_cuda(), "ep_sort: expert ids must be a CUDA tensor");
  const c10::cuda::CUDAGuard guard(ids_in.device());
  Tensor ids = ids_in.reshape(-1).to(at::kLong).contiguous();
  const int64_t n = ids.numel();
  auto opt = ids.options();
  Tensor order = at::empty({n}, opt), inv = at::empty({n}, opt), tok = at::empty({n}, opt),
         es = at::empty({n}, opt), counts = at::empty({num_experts}, opt);
  Tensor ws = at::empty({mgf_ep_sort_workspace_words(n, static_cast<int32_t>(num_experts))}, opt.dtype(at::kInt));
  check_launch(mgf_ep_sort(ids.data_ptr<int64_t>(), n, static_cast<int32_t>(num_experts),
                           static_cast<int32_t>(topk), ws.data_ptr<int32_t>(), order.data_ptr<int64_t>(),
                           inv.data_ptr<int64_t>(),
                           tok.data_ptr<int64_t>(), es.data_ptr<int64_t>(), counts.data_ptr<int64_t>(),
                           at::cuda::getCurrentCUDAStream().stream()),
               "ep_sort");
  return {order, inv, tok, es, counts};
}

std::vector<Tensor> ep_routes_cuda(const Tensor& c_all_in, const Tensor& e_sorted, int64_t rank, int64_t cap,
                                   const std::optional<Tensor>& ret_bases, const std::optional<Tensor>& gret_bases,
                                   int64_t row_bytes) {
  TORCH_CHECK(c_all_in.is_cuda() && c_all_in.dim() == 2, "ep_routes: c_all must be a [world, E] CUDA tensor");
  const c10::cuda::CUDAGuard guard(c_all_in.device());
  Tensor c_all = c_all_in.to(at::kLong).contiguous();
  const int64_t world = c_all.size(0), E = c_all.size(1), n = e_sorted.numel();
  TORCH_CHECK(e_sorted.scalar_type() == at::kLong && e_sorted.is_contiguous(), "ep_routes: e_sorted must be int64");
  auto opt = c_all.options();
  Tensor ws = at::empty({mgf_ep_routes_workspace_words(static_cast<int32_t>(world), static_cast<int32_t>(E))},
                        opt.dtype(at::kInt));
  Tensor dst_rank = at::empty({n}, opt), dst_row = at::empty({n}, opt);
  Tensor src_rank = at::empty({cap}, opt), src_pos = at::empty({cap}, opt);
  Tensor ptr_ret, ptr_gret;
  const unsigned long long* rb = nullptr;
  const unsigned long long* gb = nullptr;
  if (ret_bases.has_value()) {
    TORCH_CHECK(ret_bases->scalar_type() == at::kLong && ret_bases->numel() == world, "ep_routes: ret_bases [world]");
    ptr_ret = at::empty({cap}, opt);
    rb = reinterpret_cast<const unsigned long long*>(ret_bases->data_ptr<int64_t>());
  }
  if (gret_bases.has_value()) {
    TORCH_CHECK(gret_bases->scalar_type() == at::kLong && gret_bases->numel() == world,
                "ep_routes: gret_bases [world]");
    ptr_gret = at::empty({cap}, opt);
    gb = reinterpret_cast<const unsigned long long*>(gret_bases->data_ptr<int64_t>());
  }
  Tensor offs = at::empty({E / world}, opt.dtype(at::kInt)), n_recv = at::empty({1}, opt.dtype(at::kInt));
  check_launch(mgf_ep_routes(c_all.data_ptr<int64_t>(), static_cast<int32_t>(world), static_cast<int32_t>(E),
                             e_sorted.data_ptr<int64_t>(), n, static_cast<int32_t>(rank), cap, rb, gb, row_bytes,
                             ws.data_ptr<int32_t>(), dst_rank.data_ptr<int64_t>(), dst_row.data_ptr<int64_t>(),
                             src_rank.data_ptr<int64_t>(), src_pos.data_ptr<int64_t>(),
                             ptr_ret.defined() ? ptr_ret.data_ptr<int64_t>() : nullptr,
                             ptr_gret.defined() ? ptr_gret.data_ptr<int64_t>() : nullptr, offs.data_ptr<int32_t>(),
                             n_recv.data_ptr<int32_t>(), at::cuda::getCurrentCUDAStream().stream()),
               "ep_routes");
  return {dst_rank, dst_row, src_rank, src_pos, offs, n_recv,
          ptr_ret.defined() ? ptr_ret : at::empty({0}, opt), ptr_gret.defined() ? ptr_gret : at::empty({0}, opt)};
}

// ---------------------------------------------------------------- e4m3 quantisers
int64_t pad16(int64_t n) { return (n + 15) / 16 * 16; }

std::tuple<Tensor, Tensor> fp8_quantize_rows_cuda(const Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1,
              "fp8_quantize_rows: x must be a row-major bf16 [rows, cols] CUDA tensor");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t rows = x.size(0), cols = x.size(1);
  Tensor q = at::empty_strided({rows, cols}, {pad16(cols), 1}, x.options().dtype(at::kFloat8_e4m3fn));
  Tensor scale = at::empty({rows}, x.options().dtype(at::kFloat));
  check_launch(mgf_fp8_quantize_rows(x.data_ptr(), rows, cols, x.stride(0), q.data_ptr(), q.stride(0),
                                     scale.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()),
               "fp8_quantize_rows");
  return {q, scale};
}

std::tuple<Tensor, Tensor> fp8_quantize_cols_cuda(const Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1,
              "fp8_quantize_cols: x must be a row-major bf16 [rows, cols] CUDA tensor");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t rows = x.size(0), cols = x.size(1);
  Tensor q = at::empty_strided({rows, cols}, {pad16(cols), 1}, x.options().dtype(at::kFloat8_e4m3fn));
  Tensor scale = at::empty({cols}, x.options().dtype(at::kFloat));
  check_launch(mgf_fp8_quantize_cols(x.data_ptr(), rows, cols, rows > 0 ? x.stride(0) : 8, q.data_ptr(), q.stride(0),
                                     scale.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()),
               "fp8_quantize_cols");
  return {q, scale};
}

// Both scalings of one activation (see mgf_fp8_quantize_rows_cols): fp8_quantize_rows(x) and
// fp8_quantize_cols(x) from two passes.
std::tuple<Tensor, Tensor, Tensor, Tensor> fp8_quantize_rows_cols_cuda(const Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1,
              "fp8_quantize_rows_cols: x must be a row-major bf16 [rows, cols] CUDA tensor");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t rows = x.size(0), cols = x.size(1);
  Tensor q_r = at::empty_strided({rows, cols}, {pad16(cols), 1}, x.options().dtype(at::kFloat8_e4m3fn));
  Tensor s_r = at::empty({rows}, x.options().dtype(at::kFloat));
  Tensor q_c = at::empty_strided({rows, cols}, {pad16(cols), 1}, x.options().dtype(at::kFloat8_e4m3fn));
  Tensor s_c = at::empty({cols}, x.options().dtype(at::kFloat));
  check_launch(mgf_fp8_quantize_rows_cols(x.data_ptr(), rows, cols, rows > 0 ? x.stride(0) : 8, q_r.data_ptr(),
                                          q_r.stride(0), s_r.data_ptr<float>(), q_c.data_ptr(), q_c.stride(0),
                                          s_c.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()),
               "fp8_quantize_rows_cols");
  return {q_r, s_r, q_c, s_c};
}

std::tuple<Tensor, Tensor> fp8_quantize_weights_cuda(const Tensor& w) {
  TORCH_CHECK(w.is_cuda() && w.dim() == 3 && w.scalar_type() == at::kBFloat16 && (w.stride(2) == 1 || w.stride(1) == 1),
              "fp8_quantize_weights: w must be a bf16 [E, K, N] CUDA tensor with unit stride along K or N");
  const c10::cuda::CUDAGuard guard(w.device());
  const int64_t E = w.size(0), K = w.size(1), N = w.size(2), kp = pad16(K);
  Tensor qt = at::empty({E, N, kp}, w.options().dtype(at::kFloat8_e4m3fn));
  Tensor scale = at::empty({E, N}, w.options().dtype(at::kFloat));
  check_launch(mgf_fp8_quantize_weights(w.data_ptr(), E, K, N, w.stride(0), w.stride(1), w.stride(2), qt.data_ptr(),
                                        kp, scale.data_ptr<float>(), at::cuda::getCurrentCUDAStream().stream()),
               "fp8_quantize_weights");
  return {qt.as_strided({E, K, N}, {N * kp, 1, kp}), scale};
}

// Both quantisations of one weight in two passes (see mgf_fp8_quantize_weights_both): the results of
// fp8_quantize_weights(w) and of fp8_quantize_weights(w.transpose(-2, -1)).
std::tuple<Tensor, Tensor, Tensor, Tensor> fp8_quantize_weights_both_cuda(const Tensor& w) {
  TORCH_CHECK(w.is_cuda() && w.dim() == 3 && w.scalar_type() == at::kBFloat16 && w.stride(2) == 1,
              "fp8_quantize_weights_both: w must be a bf16 [E, K, N] CUDA tensor with unit stride along N");
  const c10::cuda::CUDAGuard guard(w.device());
  const int64_t E = w.size(0), K = w.size(1), N = w.size(2), kpa = pad16(K), kpb = pad16(N);
  Tensor qa = at::empty({E, N, kpa}, w.options().dtype(at::kFloat8_e4m3fn));
  Tensor sa = at::empty({E, N}, w.options().dtype(at::kFloat));
  Tensor qb = at::empty({E, K, kpb}, w.options().dtype(at::kFloat8_e4m3fn));
  Tensor sb = at::empty({E, K}, w.options().dtype(at::kFloat));
  check_launch(mgf_fp8_quantize_weights_both(w.data_ptr(), E, K, N, w.stride(0), w.stride(1), qa.data_ptr(), kpa,
                                             sa.data_ptr<float>(), qb.data_ptr(), kpb, sb.data_ptr<float>(),
                                             at::cuda::getCurrentCUDAStream().stream()),
               "fp8_quantize_weights_both");
  return {qa.as_strided({E, K, N}, {N * kpa, 1, kpa}), sa, qb.as_strided({E, N, K}, {K * kpb, 1, kpb}), sb};
}

// Wait on the current stream until every slot of this rank's flag array reaches seq (see mgf_wait_flags).
void wait_flags_cuda(const Tensor& flags, int64_t seq, int64_t timeout_ns) {
  TORCH_CHECK(flags.is_cuda() && flags.scalar_type() == at::kLong && flags.is_contiguous(),
              "wait_flags: flags must be a contiguous int64 CUDA tensor");
  const c10::cuda::CUDAGuard guard(flags.device());
  check_launch(mgf_wait_flags(reinterpret_cast<const unsigned long long*>(flags.data_ptr<int64_t>()), flags.numel(),
                              static_cast<unsigned long long>(seq), timeout_ns,
                              at::cuda::getCurrentCUDAStream().stream()),
               "wait_flags");
}

}  // namespace

TORCH_LIBRARY(grouped_mm, m) {
  m.def("mm(Tensor mat_a, Tensor mat_b, Tensor? offs, Tensor? bias, int out_dtype) -> Tensor");
  m.def(
      "mm_swiglu(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor bias, float swiglu_alpha, float swiglu_limit)"
      " -> (Tensor, Tensor)");
  m.def(
      "mm_swiglu_bwd(Tensor grad_out, Tensor down_w_t, Tensor offs, Tensor aux_biased_acc, float swiglu_alpha,"
      " float swiglu_limit) -> Tensor");
  m.def(
      "mm_downproj(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor? bias, Tensor aux_biased_acc,"
      " float swiglu_alpha, float swiglu_limit) -> Tensor");
  m.def(
      "mm_swiglu_noaux(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor bias, float swiglu_alpha,"
      " float swiglu_limit) -> Tensor");
  m.def("mm_wgrad_bias(Tensor mat_a, Tensor mat_b, Tensor offs) -> (Tensor, Tensor)");
  m.def(
      "swiglu_into(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor bias, Tensor(a!)? aux_out, Tensor(b!) swiglu_out,"
      " float swiglu_alpha, float swiglu_limit, bool store_aux) -> ()");
  m.def(
      "swiglu_range_into(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor bias, Tensor(a!)? aux_out,"
      " Tensor(b!) swiglu_out, float swiglu_alpha, float swiglu_limit, bool store_aux, int group_begin) -> ()");
  m.def(
      "swiglu_bwd_range_into(Tensor grad_output, Tensor down_w_t, Tensor offs, Tensor aux_biased_acc,"
      " Tensor(a!) grad_aux, float swiglu_alpha, float swiglu_limit, int group_begin) -> ()");
  m.def("wgrad_bias_into(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor(a!) dw, Tensor(b!) db, int group_begin) -> ()");
  m.def(
      "swiglu_bwd_into(Tensor grad_output, Tensor down_w_t, Tensor offs, Tensor aux_packed,"
      " Tensor(a!) grad_gate_up_packed, float swiglu_alpha, float swiglu_limit) -> ()");
  m.def("mm_fp8(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor scale_a, Tensor scale_b, Tensor? bias) -> Tensor");
  m.def(
      "mm_swiglu_fp8(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor scale_a, Tensor scale_b, Tensor bias,"
      " float swiglu_alpha, float swiglu_limit) -> (Tensor, Tensor)");
  m.def(
      "mm_swiglu_bwd_fp8(Tensor grad_output, Tensor down_w_t, Tensor offs, Tensor aux_biased_acc, Tensor scale_a,"
      " Tensor scale_b, float swiglu_alpha, float swiglu_limit) -> Tensor");
  m.def(
      "mm_wgrad_fp8(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor scale_a, Tensor scale_b, bool bias_grad)"
      " -> (Tensor, Tensor)");
  m.def("gather_rows(Tensor src, Tensor idx, Tensor? scale) -> Tensor");
  m.def("combine_rows(Tensor rows, Tensor pos, Tensor? weights, int k) -> Tensor");
  m.def(
      "push_rows(Tensor src, Tensor? src_idx, Tensor? scale, Tensor? n_dev, Tensor dst_rank, Tensor dst_row,"
      " Tensor peer_bases, int dst_rows, int ld_dst, int n_max, Tensor? flag_bases=None, Tensor? counter=None,"
      " int seq=0, int rank=0, Tensor? rotate=None) -> ()");
  m.def("wait_flags(Tensor flags, int seq, int timeout_ns) -> ()");
  m.def("fp8_quantize_rows(Tensor x) -> (Tensor, Tensor)");
  m.def("fp8_quantize_cols(Tensor x) -> (Tensor, Tensor)");
  m.def("fp8_quantize_weights(Tensor w) -> (Tensor, Tensor)");
  m.def("fp8_quantize_weights_both(Tensor w) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("fp8_quantize_rows_cols(Tensor x) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("signal_flags(Tensor flag_bases, int rank, int seq) -> ()");
  m.def("mm_scatter(Tensor mat_a, Tensor mat_b, Tensor offs, Tensor? bias, Tensor row_ptrs) -> ()");
  m.def("ep_sort(Tensor expert_ids, int num_experts, int topk) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def(
      "ep_routes(Tensor c_all, Tensor e_sorted, int rank, int cap, Tensor? ret_bases, Tensor? gret_bases,"
      " int row_bytes) -> Tensor[]");
}

TORCH_LIBRARY_IMPL(grouped_mm, CUDA, m) {
  m.impl("mm", &mm_cuda);
  m.impl("mm_swiglu", &mm_swiglu_cuda);
  m.impl("mm_swiglu_noaux", &mm_swiglu_noaux_cuda);
  m.impl("swiglu_into", &swiglu_into_cuda);
  m.impl("swiglu_range_into", &swiglu_range_into_cuda);
  m.impl("swiglu_bwd_range_into", &swiglu_bwd_range_into_cuda);
  m.impl("wgrad_bias_into", &wgrad_bias_into_cuda);
  m.impl("swiglu_bwd_into", &swiglu_bwd_into_cuda);
  m.impl("mm_swiglu_bwd", &mm_swiglu_bwd_cuda);
  m.impl("mm_wgrad_bias", &mm_wgrad_bias_cuda);
  m.impl("mm_fp8", &mm_fp8_cuda);
  m.impl("mm_swiglu_fp8", &mm_swiglu_fp8_cuda);
  m.impl("mm_swiglu_bwd_fp8", &mm_swiglu_bwd_fp8_cuda);
  m.impl("mm_wgrad_fp8", &mm_wgrad_fp8_cuda);
  m.impl("gather_rows", &gather_rows_cuda);
  m.impl("combine_rows", &combine_rows_cuda);
  m.impl("push_rows", &push_rows_cuda);
  m.impl("wait_flags", &wait_flags_cuda);
  m.impl("fp8_quantize_rows", &fp8_quantize_rows_cuda);
  m.impl("fp8_quantize_cols", &fp8_quantize_cols_cuda);
  m.impl("fp8_quantize_weights", &fp8_quantize_weights_cuda);
  m.impl("fp8_quantize_weights_both", &fp8_quantize_weights_both_cuda);
  m.impl("fp8_quantize_rows_cols", &fp8_quantize_rows_cols_cuda);
  m.impl("signal_flags", &signal_flags_cuda);
  m.impl("mm_scatter", &mm_scatter_cuda);
  m.impl("ep_sort", &ep_sort_cuda);
  m.impl("ep_routes", &ep_routes_cuda);
  m.impl("mm_downproj",
         [](const Tensor& a, const Tensor& b, const Tensor& offs, const std::optional<Tensor>& bias,
            const Tensor& aux, double alpha, double limit) {
           return mm_downproj_cuda(a, b, offs, bias, aux, alpha, limit);
         });
}
