// e4m3 quantisers of the FP8 MoE FFN: bf16 -> float8_e4m3fn with fp32 scales, scale = amax / 448
// (max(amax, 1e-12)), q = saturate_to_e4m3(x / scale), round to nearest even.
//
//   rows     one scale per row of a [rows, cols] matrix (the ragged-M A operands): one warp per row,
//            16-byte loads, the row read twice (amax, then quantise; the second pass hits L1/L2);
//   cols     one scale per column (the ragged-K weight-gradient operands): per-column amax by an
//            atomicMax on the fp32 bit patterns of |x| (non-negative floats order like their bits),
//            then an elementwise pass;
//   weights  [E, K, N] (any strides) -> e4m3 [E, N, K] with K contiguous (the K-major B operand) and
//            one scale per (e, n): the same two passes over 32 x 32 tiles, the second transposing
//            through shared memory so that both the read and the write are coalesced;
//   rows + cols  both scalings of one activation (the backward's grad_out and grad_aux feed a dgrad by
//            rows and a weight gradient by columns): one read for both amax sets, one read for both
//            code sets, instead of three;
//   weights, both axes  [E, K, N] with unit stride along n -> the K-major codes above AND the codes of
//            w^T (one scale per (e, k), n contiguous: the dgrad's B operand) from two passes instead of
//            four: one read for both amax sets, one read for both code sets.
// These replace chains of eager torch ops (abs, amax, divide, clamp, copy, transpose) that cost more
// than the e4m3 GEMMs they feed.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "moe_gemm.h"

namespace mgf {
namespace {

constexpr float kE4M3Max = 448.0f;

__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float scale_of(float amax) { return fmaxf(amax, 1e-12f) / kE4M3Max; }

__global__ void __launch_bounds__(256) quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                         int64_t cols, int64_t ldx, uint8_t* __restrict__ q,
                                                         int64_t ldq, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + row * ldx;
  const int64_t nv = cols / 8;  // whole 16-byte vectors; cols % 8 == 0 is checked by the host
  float amax = 0.0f;
  for (int64_t v = lane; v < nv; v += 32) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr) + v);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float s = scale_of(amax);
  if (lane == 0) scale[row] = s;
  uint8_t* qr = q + row * ldq;
  for (int64_t v = lane; v < nv; v += 32) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr) + v);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    uint32_t w[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float2 a = __bfloat1622float2(h[2 * j]);
      const float2 b = __bfloat1622float2(h[2 * j + 1]);
      w[j] = static_cast<uint32_t>(to_e4m3(a.x / s)) | (static_cast<uint32_t>(to_e4m3(a.y / s)) << 8) |
             (static_cast<uint32_t>(to_e4m3(b.x / s)) << 16) | (static_cast<uint32_t>(to_e4m3(b.y / s)) << 24);
    }
    *reinterpret_cast<uint2*>(qr + v * 8) = make_uint2(w[0], w[1]);
  }
}

// column amax: a block covers 8 * 32 columns (one 16-byte vector per thread) and kRowsPerBlock rows;
// the eight row lanes are reduced in shared memory, then one atomicMax per column and block
constexpr int kRowsPerBlock = 1024;

__global__ void __launch_bounds__(256) col_amax_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                       int64_t cols, int64_t ldx, unsigned int* __restrict__ amax) {
  __shared__ float red[8][256];
  const int lane = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t v = static_cast<int64_t>(blockIdx.x) * 32 + lane;  // vector index along cols
  const int64_t r_begin = static_cast<int64_t>(blockIdx.y) * kRowsPerBlock;
  const int64_t r_end = r_begin + kRowsPerBlock < rows ? r_begin + kRowsPerBlock : rows;
  float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (v * 8 < cols) {
    for (int64_t r = r_begin + ty; r < r_end; r += 8) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(x + r * ldx) + v);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        m[2 * j] = fmaxf(m[2 * j], fabsf(f.x));
        m[2 * j + 1] = fmaxf(m[2 * j + 1], fabsf(f.y));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[ty][lane * 8 + j] = m[j];
  __syncthreads();
  const int c = threadIdx.x;  // column within the block
  float mm = red[0][c];
#pragma unroll
  for (int t = 1; t < 8; ++t) mm = fmaxf(mm, red[t][c]);
  const int64_t col = static_cast<int64_t>(blockIdx.x) * 256 + c;
  if (col < cols) atomicMax(amax + col, __float_as_uint(mm));
}

// Rows + cols amax: the col_amax_kernel tiling; each warp's row (256 columns of it) is also reduced
// across the lanes and sent to the row's amax with one atomicMax per row and block.
__global__ void __launch_bounds__(256) rowcol_amax_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                          int64_t cols, int64_t ldx, unsigned int* __restrict__ amax_c,
                                                          unsigned int* __restrict__ amax_r) {
  __shared__ float red[8][256];
  const int lane = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t v = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const int64_t r_begin = static_cast<int64_t>(blockIdx.y) * kRowsPerBlock;
  const int64_t r_end = r_begin + kRowsPerBlock < rows ? r_begin + kRowsPerBlock : rows;
  const bool in = v * 8 < cols;
  float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int64_t r = r_begin + ty; r < r_end; r += 8) {  // warp-uniform
    float rm = 0.0f;
    if (in) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(x + r * ldx) + v);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        m[2 * j] = fmaxf(m[2 * j], fabsf(f.x));
        m[2 * j + 1] = fmaxf(m[2 * j + 1], fabsf(f.y));
        rm = fmaxf(rm, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) rm = fmaxf(rm, __shfl_xor_sync(0xffffffffu, rm, off));
    if (lane == 0) atomicMax(amax_r + r, __float_as_uint(rm));
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[ty][lane * 8 + j] = m[j];
  __syncthreads();
  const int c = threadIdx.x;
  float mm = red[0][c];
#pragma unroll
  for (int t = 1; t < 8; ++t) mm = fmaxf(mm, red[t][c]);
  const int64_t col = static_cast<int64_t>(blockIdx.x) * 256 + c;
  if (col < cols) atomicMax(amax_c + col, __float_as_uint(mm));
}

// Rows + cols codes: one 8-element vector per thread, both code sets from one read.
__global__ void __launch_bounds__(256) quant_rows_cols_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                              int64_t cols, int64_t ldx,
                                                              const float* __restrict__ s_r, uint8_t* __restrict__ q_r,
                                                              int64_t ldq_r, const float* __restrict__ s_c,
                                                              uint8_t* __restrict__ q_c, int64_t ldq_c) {
  const int64_t nv = cols / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * nv) return;
  const int64_t r = i / nv, v = i - r * nv;
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(x + r * ldx) + v);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float sr = __ldg(s_r + r);
  const float4 s0 = __ldg(reinterpret_cast<const float4*>(s_c + v * 8));
  const float4 s1 = __ldg(reinterpret_cast<const float4*>(s_c + v * 8) + 1);
  const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  uint32_t wr[2], wc[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float2 a = __bfloat1622float2(h[2 * j]);
    const float2 b = __bfloat1622float2(h[2 * j + 1]);
    wr[j] = static_cast<uint32_t>(to_e4m3(a.x / sr)) | (static_cast<uint32_t>(to_e4m3(a.y / sr)) << 8) |
            (static_cast<uint32_t>(to_e4m3(b.x / sr)) << 16) | (static_cast<uint32_t>(to_e4m3(b.y / sr)) << 24);
    wc[j] = static_cast<uint32_t>(to_e4m3(a.x / sv[4 * j])) | (static_cast<uint32_t>(to_e4m3(a.y / sv[4 * j + 1])) << 8) |
            (static_cast<uint32_t>(to_e4m3(b.x / sv[4 * j + 2])) << 16) |
            (static_cast<uint32_t>(to_e4m3(b.y / sv[4 * j + 3])) << 24);
  }
  *reinterpret_cast<uint2*>(q_r + r * ldq_r + v * 8) = make_uint2(wr[0], wr[1]);
  *reinterpret_cast<uint2*>(q_c + r * ldq_c + v * 8) = make_uint2(wc[0], wc[1]);
}

__global__ void amax_to_scale_kernel(float* __restrict__ s, int64_t n) {  // in place: amax bits -> scale
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) s[i] = scale_of(__uint_as_float(reinterpret_cast<unsigned int*>(s)[i]));
}

__global__ void __launch_bounds__(256) quant_cols_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                         int64_t cols, int64_t ldx, const float* __restrict__ scale,
                                                         uint8_t* __restrict__ q, int64_t ldq) {
  const int64_t nv = cols / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * nv) return;
  const int64_t r = i / nv, v = i - r * nv;
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(x + r * ldx) + v);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float4 s0 = __ldg(reinterpret_cast<const float4*>(scale + v * 8));
  const float4 s1 = __ldg(reinterpret_cast<const float4*>(scale + v * 8) + 1);
  const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  uint32_t w[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float2 a = __bfloat1622float2(h[2 * j]);
    const float2 b = __bfloat1622float2(h[2 * j + 1]);
    w[j] = static_cast<uint32_t>(to_e4m3(a.x / sv[4 * j])) | (static_cast<uint32_t>(to_e4m3(a.y / sv[4 * j + 1])) << 8) |
           (static_cast<uint32_t>(to_e4m3(b.x / sv[4 * j + 2])) << 16) |
           (static_cast<uint32_t>(to_e4m3(b.y / sv[4 * j + 3])) << 24);
  }
  *reinterpret_cast<uint2*>(q + r * ldq + v * 8) = make_uint2(w[0], w[1]);
}

// Weights, per-(e, n) amax over k: one block per expert and strip of 32 columns, no atomics.
// N_FAST: the input's unit stride is along n (lanes walk n, the 8 warps split k); else along k
// (each warp takes 4 of the 32 columns, its lanes walk k).  Writes the scale directly.
template <bool N_FAST>
__global__ void __launch_bounds__(256) w_amax_kernel(const __nv_bfloat16* __restrict__ w, int64_t K, int64_t N,
                                                     int64_t s_e, int64_t s_k, int64_t s_n,
                                                     float* __restrict__ scale) {
  __shared__ float red[8][32];
  const int64_t e = blockIdx.y, n0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const __nv_bfloat16* we = w + e * s_e;
  if (N_FAST) {
    const int64_t n = n0 + lane;
    float m = 0.0f;
    if (n < N)
      for (int64_t k = wid; k < K; k += 8) m = fmaxf(m, fabsf(__bfloat162float(we[k * s_k + n * s_n])));
    red[wid][lane] = m;
    __syncthreads();
    if (wid == 0) {
#pragma unroll
      for (int t = 1; t < 8; ++t) m = fmaxf(m, red[t][lane]);
      if (n < N) scale[e * N + n] = scale_of(m);
    }
  } else {
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + wid * 4 + j;
      if (n >= N) break;
      float m = 0.0f;
      for (int64_t k = lane; k < K; k += 32) m = fmaxf(m, fabsf(__bfloat162float(we[k * s_k + n * s_n])));
#pragma unroll
      for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (lane == 0) scale[e * N + n] = scale_of(m);
    }
  }
}

template <bool N_FAST>
__global__ void __launch_bounds__(256) w_quant_kernel(const __nv_bfloat16* __restrict__ w, int64_t K, int64_t N,
                                                      int64_t s_e, int64_t s_k, int64_t s_n,
                                                      const float* __restrict__ scale, uint8_t* __restrict__ q,
                                                      int64_t ldq) {
  __shared__ float tile[32][33];
  const int64_t e = blockIdx.z, k0 = static_cast<int64_t>(blockIdx.y) * 32, n0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int j = ty; j < 32; j += 8) {
    const int64_t k = k0 + (N_FAST ? j : tx), n = n0 + (N_FAST ? tx : j);
    float v = 0.0f;
    if (k < K && n < N) v = __bfloat162float(w[e * s_e + k * s_k + n * s_n]);
    if (N_FAST) tile[j][tx] = v; else tile[tx][j] = v;
  }
  __syncthreads();
  // output q[e][n][k], k contiguous: threadIdx.x walks k
  for (int j = ty; j < 32; j += 8) {
    const int64_t n = n0 + j, k = k0 + tx;
    if (n < N && k < K) q[(e * N + n) * ldq + k] = to_e4m3(tile[tx][j] / __ldg(scale + e * N + n));
  }
}

// Vectorised weight kernels (16-byte loads along the contiguous dimension, 16-byte code stores along
// k); used when the contiguous extent and the other strides are multiples of 8 elements and the base is
// 16-byte aligned, which is the case for every weight layout of the FFN.
template <bool N_FAST>
__global__ void __launch_bounds__(256) w_amax_vec_kernel(const __nv_bfloat16* __restrict__ w, int64_t K, int64_t N,
                                                         int64_t s_e, int64_t s_k, int64_t s_n,
                                                         float* __restrict__ scale) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t e = blockIdx.y;
  const __nv_bfloat16* we = w + e * s_e;
  if (N_FAST) {  // a block: 256 columns (8 per lane), the 8 warps split k
    __shared__ float red[8][256];
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 256 + lane * 8;
    float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (n0 < N) {
      for (int64_t k = wid; k < K; k += 8) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(we + k * s_k + n0));
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          m[2 * j] = fmaxf(m[2 * j], fabsf(f.x));
          m[2 * j + 1] = fmaxf(m[2 * j + 1], fabsf(f.y));
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) red[wid][lane * 8 + j] = m[j];
    __syncthreads();
    float mm = red[0][threadIdx.x];
#pragma unroll
    for (int t = 1; t < 8; ++t) mm = fmaxf(mm, red[t][threadIdx.x]);
    const int64_t n = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
    if (n < N) scale[e * N + n] = scale_of(mm);
  } else {  // a block: 32 columns, 4 per warp; lanes walk k in 8-element vectors
    for (int j = 0; j < 4; ++j) {
      const int64_t n = static_cast<int64_t>(blockIdx.x) * 32 + wid * 4 + j;
      if (n >= N) break;
      const __nv_bfloat16* row = we + n * s_n;
      float m = 0.0f;
      for (int64_t k8 = lane; k8 < K / 8; k8 += 32) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row) + k8);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (lane == 0) scale[e * N + n] = scale_of(m);
    }
  }
}

// 64 (k) x 64 (n) tile: 16-byte loads along the contiguous input dimension into shared memory, then
// every thread writes 16 consecutive k codes of one n (q[e][n][k], k contiguous) as one 16-byte store.
template <bool N_FAST>
__global__ void __launch_bounds__(256) w_quant_vec_kernel(const __nv_bfloat16* __restrict__ w, int64_t K, int64_t N,
                                                          int64_t s_e, int64_t s_k, int64_t s_n,
                                                          const float* __restrict__ scale, uint8_t* __restrict__ q,
                                                          int64_t ldq) {
  __shared__ float tile[64][65];  // [k][n]
  const int64_t e = blockIdx.z, k0 = static_cast<int64_t>(blockIdx.y) * 64, n0 = static_cast<int64_t>(blockIdx.x) * 64;
  const __nv_bfloat16* we = w + e * s_e;
  for (int it = threadIdx.x; it < 512; it += 256) {  // 64 lines x 8 vectors of 8
    const int line = it >> 3, vec = it & 7;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int64_t kk = N_FAST ? k0 + line : k0 + vec * 8;  // first k of the vector
    const int64_t nn = N_FAST ? n0 + vec * 8 : n0 + line;   // first n of the vector
    if (kk < K && nn < N) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(we + kk * s_k + nn * s_n));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 v = __bfloat1622float2(h[j]);
        f[2 * j] = v.x;
        f[2 * j + 1] = v.y;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (N_FAST) tile[line][vec * 8 + j] = f[j];
      else tile[vec * 8 + j][line] = f[j];
    }
  }
  __syncthreads();
  const int nl = threadIdx.x >> 2, kq = (threadIdx.x & 3) * 16;  // 64 n x 4 groups of 16 k
  const int64_t n = n0 + nl, k = k0 + kq;
  if (n >= N || k >= K) return;
  const float s = __ldg(scale + e * N + n);
  uint32_t wds[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t wv = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) wv |= static_cast<uint32_t>(to_e4m3(tile[kq + 4 * g + b][nl] / s)) << (8 * b);
    wds[g] = wv;
  }
  uint8_t* dst = q + (e * N + n) * ldq + k;
  if (k + 16 <= K) {
    *reinterpret_cast<uint4*>(dst) = make_uint4(wds[0], wds[1], wds[2], wds[3]);
  } else {
    for (int i = 0; i < K - k; ++i) dst[i] = static_cast<uint8_t>(wds[i >> 2] >> (8 * (i & 3)));
  }
}

// Both-axes amax: a block covers 256 columns (8 per lane) and 128 k rows (16 per warp); per-column
// maxima over the block's rows and per-row maxima over its columns go out as atomicMax on the fp32
// bit patterns of |w| (non-negative floats order like their bits).
__global__ void __launch_bounds__(256) w_amax_both_kernel(const __nv_bfloat16* __restrict__ w, int64_t K, int64_t N,
                                                          int64_t s_e, int64_t s_k, unsigned int* __restrict__ amax_n,
                                                          unsigned int* __restrict__ amax_k) {
  __shared__ float red[8][256];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t e = blockIdx.z, k0 = static_cast<int64_t>(blockIdx.y) * 128;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 256 + lane * 8;
  const __nv_bfloat16* we = w + e * s_e;
  float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < 16; ++i) {
    const int64_t k = k0 + wid + 8 * i;  // warp-uniform
    if (k >= K) break;
    float rm = 0.0f;
    if (n0 < N) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(we + k * s_k + n0));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        m[2 * j] = fmaxf(m[2 * j], fabsf(f.x));
        m[2 * j + 1] = fmaxf(m[2 * j + 1], fabsf(f.y));
        rm = fmaxf(rm, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) rm = fmaxf(rm, __shfl_xor_sync(0xffffffffu, rm, off));
    if (lane == 0) atomicMax(amax_k + e * K + k, __float_as_uint(rm));
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[wid][lane * 8 + j] = m[j];
  __syncthreads();
  float mm = red[0][threadIdx.x];
#pragma unroll
  for (int t = 1; t < 8; ++t) mm = fmaxf(mm, red[t][threadIdx.x]);
  const int64_t n = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (n < N) atomicMax(amax_n + e * N + n, __float_as_uint(mm));
}

// Both-axes codes from one 64 (k) x 64 (n) tile in shared memory: q_a[e][n][k] (k contiguous, scale per
// (e, n)), written as in w_quant_vec_kernel, and q_b[e][k][n] (n contiguous, scale per (e, k)): every
// thread writes 16 consecutive n codes of one k as one 16-byte store.
__global__ void __launch_bounds__(256) w_quant_both_kernel(const __nv_bfloat16* __restrict__ w, int64_t K, int64_t N,
                                                           int64_t s_e, int64_t s_k, const float* __restrict__ sa,
                                                           uint8_t* __restrict__ qa, int64_t ldqa,
                                                           const float* __restrict__ sb, uint8_t* __restrict__ qb,
                                                           int64_t ldqb) {
  __shared__ float tile[64][65];  // [k][n]
  const int64_t e = blockIdx.z, k0 = static_cast<int64_t>(blockIdx.y) * 64, n0 = static_cast<int64_t>(blockIdx.x) * 64;
  const __nv_bfloat16* we = w + e * s_e;
  for (int it = threadIdx.x; it < 512; it += 256) {  // 64 k lines x 8 vectors of 8 n
    const int line = it >> 3, vec = it & 7;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int64_t kk = k0 + line, nn = n0 + vec * 8;
    if (kk < K && nn < N) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(we + kk * s_k + nn));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 v = __bfloat1622float2(h[j]);
        f[2 * j] = v.x;
        f[2 * j + 1] = v.y;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) tile[line][vec * 8 + j] = f[j];
  }
  __syncthreads();
  {  // q_a: 64 n x 4 groups of 16 k
    const int nl = threadIdx.x >> 2, kq = (threadIdx.x & 3) * 16;
    const int64_t n = n0 + nl, k = k0 + kq;
    if (n < N && k < K) {
      const float s = __ldg(sa + e * N + n);
      uint32_t wds[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t wv = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) wv |= static_cast<uint32_t>(to_e4m3(tile[kq + 4 * g + b][nl] / s)) << (8 * b);
        wds[g] = wv;
      }
      uint8_t* dst = qa + (e * N + n) * ldqa + k;
      if (k + 16 <= K) *reinterpret_cast<uint4*>(dst) = make_uint4(wds[0], wds[1], wds[2], wds[3]);
      else for (int i = 0; i < K - k; ++i) dst[i] = static_cast<uint8_t>(wds[i >> 2] >> (8 * (i & 3)));
    }
  }
  {  // q_b: 64 k x 4 groups of 16 n
    const int kl = threadIdx.x >> 2, nq = (threadIdx.x & 3) * 16;
    const int64_t k = k0 + kl, n = n0 + nq;
    if (k < K && n < N) {
      const float s = __ldg(sb + e * K + k);
      uint32_t wds[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t wv = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) wv |= static_cast<uint32_t>(to_e4m3(tile[kl][nq + 4 * g + b] / s)) << (8 * b);
        wds[g] = wv;
      }
      uint8_t* dst = qb + (e * K + k) * ldqb + n;
      if (n + 16 <= N) *reinterpret_cast<uint4*>(dst) = make_uint4(wds[0], wds[1], wds[2], wds[3]);
      else for (int i = 0; i < N - n; ++i) dst[i] = static_cast<uint8_t>(wds[i >> 2] >> (8 * (i & 3)));
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace mgf

extern "C" int mgf_fp8_quantize_rows(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq,
                                     float* scale, void* stream) {
  using namespace mgf;
  if (rows < 0 || cols < 0 || (rows > 0 && (x == nullptr || q == nullptr || scale == nullptr)))
    return MGF_ERR_INVALID_ARGUMENT;
  if (rows == 0) return MGF_OK;
  if (cols % 8 || ldx % 8 || ldq % 8 || !aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u)) return MGF_ERR_ALIGNMENT;
  const int64_t blocks = (rows * 32 + 255) / 256;
  quant_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), rows, cols, ldx, static_cast<uint8_t*>(q), ldq, scale);
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int mgf_fp8_quantize_cols(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq,
                                     float* scale, void* stream) {
  using namespace mgf;
  if (rows < 0 || cols < 0 || (cols > 0 && scale == nullptr) || (rows > 0 && (x == nullptr || q == nullptr)))
    return MGF_ERR_INVALID_ARGUMENT;
  if (cols == 0) return MGF_OK;
  if (cols % 8 || ldx % 8 || ldq % 8 || !aligned16(x) || !aligned16(scale) || (reinterpret_cast<uintptr_t>(q) & 7u))
    return MGF_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scale, 0, sizeof(float) * cols, st) != cudaSuccess) return MGF_ERR_CUDA;
  if (rows > 0) {
    const dim3 grid(static_cast<unsigned>((cols / 8 + 31) / 32), static_cast<unsigned>((rows + kRowsPerBlock - 1) / kRowsPerBlock));
    col_amax_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, ldx,
                                          reinterpret_cast<unsigned int*>(scale));
  }
  amax_to_scale_kernel<<<static_cast<unsigned>((cols + 255) / 256), 256, 0, st>>>(scale, cols);
  if (rows > 0) {
    const int64_t items = rows * (cols / 8);
    quant_cols_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), rows, cols, ldx, scale, static_cast<uint8_t*>(q), ldq);
  }
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int mgf_fp8_quantize_weights(const void* w, int64_t E, int64_t K, int64_t N, int64_t s_e, int64_t s_k,
                                        int64_t s_n, void* q, int64_t ldq, float* scale, void* stream) {
  using namespace mgf;
  if (E < 0 || K < 0 || N < 0 || ldq < K) return MGF_ERR_INVALID_ARGUMENT;
  if (E == 0 || N == 0) return MGF_OK;
  if (w == nullptr || q == nullptr || scale == nullptr) return MGF_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool n_fast = s_n == 1;
  const __nv_bfloat16* wp = static_cast<const __nv_bfloat16*>(w);
  const int64_t fast_extent = n_fast ? N : K;
  const int64_t slow_stride = n_fast ? s_k : s_n;
  const bool vec = aligned16(w) && fast_extent % 8 == 0 && slow_stride % 8 == 0 && s_e % 8 == 0 &&
                   (n_fast || s_k == 1) && ldq % 16 == 0 && (reinterpret_cast<uintptr_t>(q) & 15u) == 0;
  if (vec) {
    const dim3 agrid(static_cast<unsigned>(n_fast ? (N + 255) / 256 : (N + 31) / 32), static_cast<unsigned>(E));
    if (n_fast) w_amax_vec_kernel<true><<<agrid, 256, 0, st>>>(wp, K, N, s_e, s_k, s_n, scale);
    else w_amax_vec_kernel<false><<<agrid, 256, 0, st>>>(wp, K, N, s_e, s_k, s_n, scale);
    if (K > 0) {
      const dim3 grid(static_cast<unsigned>((N + 63) / 64), static_cast<unsigned>((K + 63) / 64), static_cast<unsigned>(E));
      if (n_fast) w_quant_vec_kernel<true><<<grid, 256, 0, st>>>(wp, K, N, s_e, s_k, s_n, scale, static_cast<uint8_t*>(q), ldq);
      else w_quant_vec_kernel<false><<<grid, 256, 0, st>>>(wp, K, N, s_e, s_k, s_n, scale, static_cast<uint8_t*>(q), ldq);
    }
  } else {
    const dim3 agrid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>(E));
    if (n_fast) w_amax_kernel<true><<<agrid, 256, 0, st>>>(wp, K, N, s_e, s_k, s_n, scale);
    else w_amax_kernel<false><<<agrid, 256, 0, st>>>(wp, K, N, s_e, s_k, s_n, scale);
    if (K > 0) {
      const dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((K + 31) / 32), static_cast<unsigned>(E));
      if (n_fast) w_quant_kernel<true><<<grid, 256, 0, st>>>(wp, K, N, s_e, s_k, s_n, scale, static_cast<uint8_t*>(q), ldq);
      else w_quant_kernel<false><<<grid, 256, 0, st>>>(wp, K, N, s_e, s_k, s_n, scale, static_cast<uint8_t*>(q), ldq);
    }
  }
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int mgf_fp8_quantize_weights_both(const void* w, int64_t E, int64_t K, int64_t N, int64_t s_e, int64_t s_k,
                                             void* qa, int64_t ldqa, float* sa, void* qb, int64_t ldqb, float* sb,
                                             void* stream) {
  using namespace mgf;
  if (E < 0 || K < 0 || N < 0 || ldqa < K || ldqb < N) return MGF_ERR_INVALID_ARGUMENT;
  if (E == 0) return MGF_OK;
  if (w == nullptr || qa == nullptr || qb == nullptr || sa == nullptr || sb == nullptr) return MGF_ERR_INVALID_ARGUMENT;
  if (!aligned16(w) || N % 8 || s_k % 8 || s_e % 8 || ldqa % 16 || ldqb % 16 || !aligned16(qa) || !aligned16(qb) ||
      !aligned16(sa) || !aligned16(sb))
    return MGF_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(sa, 0, sizeof(float) * E * N, st) != cudaSuccess ||
      cudaMemsetAsync(sb, 0, sizeof(float) * E * K, st) != cudaSuccess)
    return MGF_ERR_CUDA;
  const __nv_bfloat16* wp = static_cast<const __nv_bfloat16*>(w);
  if (K > 0 && N > 0) {
    const dim3 agrid(static_cast<unsigned>((N + 255) / 256), static_cast<unsigned>((K + 127) / 128), static_cast<unsigned>(E));
    w_amax_both_kernel<<<agrid, 256, 0, st>>>(wp, K, N, s_e, s_k, reinterpret_cast<unsigned int*>(sa),
                                              reinterpret_cast<unsigned int*>(sb));
  }
  if (N > 0) amax_to_scale_kernel<<<static_cast<unsigned>((E * N + 255) / 256), 256, 0, st>>>(sa, E * N);
  if (K > 0) amax_to_scale_kernel<<<static_cast<unsigned>((E * K + 255) / 256), 256, 0, st>>>(sb, E * K);
  if (K > 0 && N > 0) {
    const dim3 grid(static_cast<unsigned>((N + 63) / 64), static_cast<unsigned>((K + 63) / 64), static_cast<unsigned>(E));
    w_quant_both_kernel<<<grid, 256, 0, st>>>(wp, K, N, s_e, s_k, sa, static_cast<uint8_t*>(qa), ldqa, sb,
                                              static_cast<uint8_t*>(qb), ldqb);
  }
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int mgf_fp8_quantize_rows_cols(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q_r,
                                          int64_t ldq_r, float* s_r, void* q_c, int64_t ldq_c, float* s_c,
                                          void* stream) {
  using namespace mgf;
  if (rows < 0 || cols < 0 || (cols > 0 && s_c == nullptr) || (rows > 0 && (s_r == nullptr)) ||
      (rows > 0 && cols > 0 && (x == nullptr || q_r == nullptr || q_c == nullptr)))
    return MGF_ERR_INVALID_ARGUMENT;
  if (cols % 8 || ldx % 8 || ldq_r % 8 || ldq_c % 8 || (rows > 0 && cols > 0 && !aligned16(x)) ||
      (cols > 0 && !aligned16(s_c)) || (reinterpret_cast<uintptr_t>(q_r) & 7u) || (reinterpret_cast<uintptr_t>(q_c) & 7u))
    return MGF_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((cols > 0 && cudaMemsetAsync(s_c, 0, sizeof(float) * cols, st) != cudaSuccess) ||
      (rows > 0 && cudaMemsetAsync(s_r, 0, sizeof(float) * rows, st) != cudaSuccess))
    return MGF_ERR_CUDA;
  if (rows > 0 && cols > 0) {
    const dim3 grid(static_cast<unsigned>((cols / 8 + 31) / 32), static_cast<unsigned>((rows + kRowsPerBlock - 1) / kRowsPerBlock));
    rowcol_amax_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, ldx,
                                             reinterpret_cast<unsigned int*>(s_c), reinterpret_cast<unsigned int*>(s_r));
  }
  if (cols > 0) amax_to_scale_kernel<<<static_cast<unsigned>((cols + 255) / 256), 256, 0, st>>>(s_c, cols);
  if (rows > 0) amax_to_scale_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, st>>>(s_r, rows);
  if (rows > 0 && cols > 0) {
    const int64_t items = rows * (cols / 8);
    quant_rows_cols_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), rows, cols, ldx, s_r, static_cast<uint8_t*>(q_r), ldq_r, s_c,
        static_cast<uint8_t*>(q_c), ldq_c);
  }
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}
