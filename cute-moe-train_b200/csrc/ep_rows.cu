// Row movement kernels of the expert-parallel MoE FFN (dispatch / combine around the grouped GEMMs).
//
//   gather:  dst[i]  = scale[i] * src[idx[i]]                          (scale optional)
//   combine: out[t]  = sum_j w[t*k + j] * rows[pos[t*k + j]]  for j < k  (fp32 sum, one bf16 rounding)
//
// Dispatch is a gather (token copies in expert order), combine sums a token's k expert outputs.
// Each is the other's backward: d(gather)/d(src) is a combine over the copies of each source row,
// d(combine)/d(rows) is a gather of the token gradients.  Both are HBM-bound: one warp per row,
// 16-byte vector loads/stores, a grid of a few waves over the 148 SMs.  The reference has no
// distributed code; these serve the expert-parallel mode this build adds.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "moe_gemm.h"

namespace mgf {
namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(32 * kWarpsPerBlock) gather_rows_kernel(
    const __nv_bfloat16* __restrict__ src, int64_t ld_src, int64_t n_src, const int64_t* __restrict__ idx,
    const float* __restrict__ scale, int64_t n_rows, int64_t row_vec, __nv_bfloat16* __restrict__ dst,
    int64_t ld_dst, unsigned int* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t i = warp0; i < n_rows; i += nwarps) {
    const int64_t s = __ldg(idx + i);
    if (s < 0 || s >= n_src) {  // a wrong plan: report it, leave the output row as it was
      if (lane == 0) atomicOr(status, MGF_DEV_ROW_OUT_OF_RANGE);
      continue;
    }
    const uint4* sp = reinterpret_cast<const uint4*>(src + s * ld_src);
    uint4* dp = reinterpret_cast<uint4*>(dst + i * ld_dst);
    if (scale == nullptr) {
      for (int64_t v = lane; v < row_vec; v += 32) dp[v] = __ldg(sp + v);
    } else {
      const float f = __ldg(scale + i);
      for (int64_t v = lane; v < row_vec; v += 32) {
        const uint4 a = __ldg(sp + v);
        dp[v] = make_uint4(pack(f * lo(a.x), f * hi(a.x)), pack(f * lo(a.y), f * hi(a.y)),
                           pack(f * lo(a.z), f * hi(a.z)), pack(f * lo(a.w), f * hi(a.w)));
      }
    }
  }
}

__global__ void __launch_bounds__(32 * kWarpsPerBlock) combine_rows_kernel(
    const __nv_bfloat16* __restrict__ rows, int64_t ld_rows, int64_t n_rows, const int64_t* __restrict__ pos,
    const float* __restrict__ w, int64_t n_out, int k, int64_t row_vec, __nv_bfloat16* __restrict__ out,
    int64_t ld_out, unsigned int* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = warp0; t < n_out; t += nwarps) {
    bool bad = false;
    for (int j = lane; j < k; j += 32) {
      const int64_t r = __ldg(pos + t * k + j);
      bad |= (r < 0 || r >= n_rows);
    }
    if (__any_sync(0xffffffffu, bad)) {  // a wrong plan: report it, leave the output row as it was
      if (lane == 0) atomicOr(status, MGF_DEV_ROW_OUT_OF_RANGE);
      continue;
    }
    uint4* op = reinterpret_cast<uint4*>(out + t * ld_out);
    for (int64_t v = lane; v < row_vec; v += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < k; ++j) {
        const int64_t r = __ldg(pos + t * k + j);
        const float f = (w != nullptr) ? __ldg(w + t * k + j) : 1.0f;
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(rows + r * ld_rows) + v);
        acc[0] += f * lo(a.x); acc[1] += f * hi(a.x);
        acc[2] += f * lo(a.y); acc[3] += f * hi(a.y);
        acc[4] += f * lo(a.z); acc[5] += f * hi(a.z);
        acc[6] += f * lo(a.w); acc[7] += f * hi(a.w);
      }
      op[v] = make_uint4(pack(acc[0], acc[1]), pack(acc[2], acc[3]), pack(acc[4], acc[5]), pack(acc[6], acc[7]));
    }
  }
}

// Rows written straight into other GPUs' memory (NVLink peer stores through CUDA IPC mappings):
// dst_rank[i]'s buffer (peer_bases[dst_rank[i]]) row dst_row[i] = scale[i] * src[src_idx[i]].
// The row count is n_max, or *n_dev when given (a device-side count, never read by the host).
//
// Completion signal (sig.flag_bases != nullptr): every block fences its stores system-wide and
// counts itself on sig.counter; the last block of the launch then writes sig.seq into slot
// sig.rank of every rank's flag array (a release store over NVLink) and resets the counter for the
// next launch.  A reader waits for seq in all slots of its own flag array (wait_flags_kernel):
// then every source's rows have landed.  This replaces a collective barrier between the pushes
// and the kernels that read them.
struct PushSignal {
  const unsigned long long* flag_bases;  // device [world]: address of each rank's flag array
  unsigned long long* counter;           // device: blocks of this launch that finished (starts at 0)
  unsigned long long seq;
  int64_t rank;
};

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(32 * kWarpsPerBlock) push_rows_kernel(
    const __nv_bfloat16* __restrict__ src, int64_t ld_src, const int64_t* __restrict__ src_idx,
    const float* __restrict__ scale, int64_t n_max, const int32_t* __restrict__ n_dev,
    const int64_t* __restrict__ dst_rank, const int64_t* __restrict__ dst_row,
    const unsigned long long* __restrict__ peer_bases, int64_t world, int64_t dst_rows, int64_t ld_dst,
    int64_t row_vec, int64_t n_src, unsigned int* __restrict__ status, PushSignal sig,
    const int64_t* __restrict__ rotate) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  int64_t n = n_max;
  if (n_dev != nullptr) {
    const int64_t c = __ldg(n_dev);
    n = c < n ? (c > 0 ? c : 0) : n;
  }
  // rotation: row slot j handles entry (j + *rotate) mod n, so that ranks whose entries are sorted by
  // destination start on different destinations instead of all writing to rank 0 first
  int64_t rot = 0;
  if (rotate != nullptr && n > 0) {
    rot = __ldg(rotate) % n;
    if (rot < 0) rot += n;
  }
  for (int64_t j = warp0; j < n; j += nwarps) {
    int64_t i = j + rot;
    if (i >= n) i -= n;
    const int64_t s = src_idx != nullptr ? __ldg(src_idx + i) : i;
    const int64_t r = __ldg(dst_rank + i);
    const int64_t row = __ldg(dst_row + i);
    if (r < 0 || r >= world || row < 0 || row >= dst_rows || s < 0 || s >= n_src) {
      // never store outside a peer buffer nor read outside src; report the skipped row
      if (lane == 0) atomicOr(status, MGF_DEV_ROW_OUT_OF_RANGE);
      continue;
    }
    __nv_bfloat16* dbase = reinterpret_cast<__nv_bfloat16*>(peer_bases[r]);
    const uint4* sp = reinterpret_cast<const uint4*>(src + s * ld_src);
    uint4* dp = reinterpret_cast<uint4*>(dbase + row * ld_dst);
    if (scale == nullptr) {
      for (int64_t v = lane; v < row_vec; v += 32) dp[v] = __ldg(sp + v);
    } else {
      const float f = __ldg(scale + i);
      for (int64_t v = lane; v < row_vec; v += 32) {
        const uint4 a = __ldg(sp + v);
        dp[v] = make_uint4(pack(f * lo(a.x), f * hi(a.x)), pack(f * lo(a.y), f * hi(a.y)),
                           pack(f * lo(a.z), f * hi(a.z)), pack(f * lo(a.w), f * hi(a.w)));
      }
    }
  }
  // make the peer stores visible system-wide before the signal (or the stream's next operation)
  __threadfence_system();
  if (sig.flag_bases == nullptr) return;
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(sig.counter, 1ull) == static_cast<unsigned long long>(gridDim.x) - 1ull;
  __syncthreads();
  if (!last) return;
  __threadfence_system();  // every block's stores (fenced before its count) precede the flags
  for (int64_t r = threadIdx.x; r < world; r += blockDim.x) {
    unsigned long long* flags = reinterpret_cast<unsigned long long*>(sig.flag_bases[r]);
    st_release_sys_u64(flags + sig.rank, sig.seq);
  }
  if (threadIdx.x == 0) *sig.counter = 0ull;  // the next launch is stream-ordered after this one
}

// Wait until every slot s < world of this rank's flag array holds a value >= seq (all sources
// finished the push with that sequence number), at most timeout_ns; on time-out record
// MGF_DEV_WAIT_TIMEOUT and return (the kernels that follow then read incomplete data, which the
// status check reports).  One block; thread s polls slot s.
__global__ void wait_flags_kernel(const unsigned long long* __restrict__ flags, int64_t world, unsigned long long seq,
                                  int64_t timeout_ns, unsigned int* __restrict__ status) {
  const uint64_t t0 = globaltimer_ns();
  for (int64_t s = threadIdx.x; s < world; s += blockDim.x) {
    uint32_t it = 0;
    while (ld_acquire_sys_u64(flags + s) < seq) {
      if ((++it & 63u) == 0 && globaltimer_ns() - t0 > static_cast<uint64_t>(timeout_ns)) {
        atomicOr(status, MGF_DEV_WAIT_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

int grid_for(int64_t rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap = static_cast<int64_t>(sms) * 8;  // 8 resident blocks per SM, grid-stride beyond
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// The device status word lives in the GEMM translation unit (moe_gemm_sm100.cu); its device
// address for the current device comes from there.
unsigned int* status_word_address();

}  // namespace mgf

extern "C" int mgf_gather_rows(const void* src, int64_t ld_src, int64_t n_src, const int64_t* idx,
                               const float* scale, int64_t n_rows, int64_t row_elems, void* dst, int64_t ld_dst,
                               void* stream) {
  using namespace mgf;
  if (n_rows < 0 || row_elems < 0 || n_src < 0) return MGF_ERR_INVALID_ARGUMENT;
  if (n_rows == 0 || row_elems == 0) return MGF_OK;
  if (src == nullptr || idx == nullptr || dst == nullptr) return MGF_ERR_INVALID_ARGUMENT;
  if (row_elems % 8 || ld_src % 8 || ld_dst % 8 || !aligned16(src) || !aligned16(dst)) return MGF_ERR_ALIGNMENT;
  unsigned int* status = status_word_address();
  if (status == nullptr) return MGF_ERR_CUDA;
  gather_rows_kernel<<<grid_for(n_rows), 32 * kWarpsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), ld_src, n_src, idx, scale, n_rows, row_elems / 8,
      static_cast<__nv_bfloat16*>(dst), ld_dst, status);
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int mgf_combine_rows(const void* rows, int64_t ld_rows, int64_t n_rows, const int64_t* pos,
                                const float* weights, int64_t n_out, int32_t k, int64_t row_elems, void* out,
                                int64_t ld_out, void* stream) {
  using namespace mgf;
  if (n_out < 0 || row_elems < 0 || k < 0 || n_rows < 0) return MGF_ERR_INVALID_ARGUMENT;
  if (n_out == 0 || row_elems == 0) return MGF_OK;
  if (out == nullptr || (k > 0 && (rows == nullptr || pos == nullptr))) return MGF_ERR_INVALID_ARGUMENT;
  if (row_elems % 8 || ld_rows % 8 || ld_out % 8 || !aligned16(rows) || !aligned16(out)) return MGF_ERR_ALIGNMENT;
  unsigned int* status = status_word_address();
  if (status == nullptr) return MGF_ERR_CUDA;
  combine_rows_kernel<<<grid_for(n_out), 32 * kWarpsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(rows), ld_rows, n_rows, pos, weights, n_out, k, row_elems / 8,
      static_cast<__nv_bfloat16*>(out), ld_out, status);
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int mgf_push_rows(const void* src, int64_t ld_src, int64_t n_src, const int64_t* src_idx,
                             const float* scale, int64_t n_max, const int32_t* n_dev, const int64_t* dst_rank,
                             const int64_t* dst_row, const unsigned long long* peer_bases, int64_t world, int64_t dst_rows, int64_t ld_dst,
                             int64_t row_elems, const unsigned long long* flag_bases,
                             unsigned long long* counter, unsigned long long seq, int64_t rank,
                             const int64_t* rotate, void* stream) {
  using namespace mgf;
  if (n_max < 0 || row_elems < 0 || n_src < 0) return MGF_ERR_INVALID_ARGUMENT;
  if (flag_bases != nullptr && (counter == nullptr || rank < 0 || rank >= world)) return MGF_ERR_INVALID_ARGUMENT;
  const PushSignal sig{flag_bases, counter, seq, rank};
  if (n_max == 0 || row_elems == 0) n_max = 0;  // nothing to move, but a signal still goes out
  if (n_max == 0 && flag_bases == nullptr) return MGF_OK;
  if (src == nullptr || dst_rank == nullptr || dst_row == nullptr || peer_bases == nullptr)
    return MGF_ERR_INVALID_ARGUMENT;
  if (row_elems % 8 || ld_src % 8 || ld_dst % 8 || !aligned16(src)) return MGF_ERR_ALIGNMENT;
  unsigned int* status = status_word_address();
  if (status == nullptr) return MGF_ERR_CUDA;
  push_rows_kernel<<<grid_for(n_max), 32 * kWarpsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), ld_src, src_idx, scale, n_max, n_dev, dst_rank, dst_row, peer_bases,
      world, dst_rows, ld_dst, row_elems / 8, n_src, status, sig, rotate);
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

// Export an IPC handle for the allocation holding `ptr`: the 64-byte cudaIpcMemHandle_t of the
// allocation base and the byte offset of `ptr` inside it (the base is found with the driver's
// cuMemGetAddressRange, reached through cudaGetDriverEntryPoint).
extern "C" int mgf_ipc_get_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return MGF_ERR_INVALID_ARGUMENT;
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range_fn = nullptr;
  if (range_fn == nullptr) {
    void* fp = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fp, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return MGF_ERR_CUDA;
    range_fn = reinterpret_cast<RangeFn>(fp);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return MGF_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return MGF_ERR_CUDA;
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MGF_OK;
}

// CUDA IPC mapping of another process's device allocation into THIS device's context (the calling
// thread's current device), with peer access enabled lazily: kernels on this device may then store
// to the peer allocation over NVLink.  `handle` is the 64-byte cudaIpcMemHandle_t of the peer's
// allocation base.
extern "C" int mgf_ipc_open(const void* handle, void** base_out) {
  if (handle == nullptr || base_out == nullptr) return MGF_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MGF_ERR_CUDA;
  *base_out = p;
  return MGF_OK;
}

extern "C" int mgf_ipc_close(void* base) {
  if (base == nullptr) return MGF_ERR_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int mgf_wait_flags(const unsigned long long* flags, int64_t world, unsigned long long seq,
                              int64_t timeout_ns, void* stream) {
  using namespace mgf;
  if (flags == nullptr || world <= 0 || world > 1024 || timeout_ns <= 0) return MGF_ERR_INVALID_ARGUMENT;
  unsigned int* status = status_word_address();
  if (status == nullptr) return MGF_ERR_CUDA;
  const int threads = world <= 32 ? 32 : (world <= 256 ? 256 : 1024);
  wait_flags_kernel<<<1, threads, 0, static_cast<cudaStream_t>(stream)>>>(flags, world, seq, timeout_ns, status);
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

// ============================================================================ expert-parallel plan
//
// The device-side plan of the peer transport, three launches and no host synchronisation:
//   ep_sort      a stable counting sort of this rank's T*k routed copies by expert id (one block):
//                order / inverse / token of every sorted copy, and the per-expert counts that the
//                caller all-gathers into c_all [world, E];
//   ep_tables    prefix sums of c_all (one block) into a small int32 workspace;
//   ep_routes    elementwise: for sorted copy p its owner rank and row in the owner's receive
//                buffer; for row j of this rank's receive buffer its source rank and sorted
//                position there, the row's addresses in the sources' `ret` / `gret` buffers (for
//                the scatter epilogues), the int32 offs of the local experts and the row count.
// Owner row layout: local expert-major, then source rank, then the source's copies in sorted order.

namespace mgf {
namespace {

// Stable counting sort in three launches.  Copies are cut into blocks of 1024 (32 warps x 32);
// ep_hist counts each block's copies per expert, ep_scan turns the [block][expert] counts into
// exclusive starts (expert-major, then block), ep_scatter ranks every copy inside its block (warp
// by warp, lane by lane: the original order) and writes it to start + rank.
constexpr int kSortBlock = 1024;

__device__ __forceinline__ int clamp_expert(int64_t r, int E, bool& bad) {
  if (r < 0 || r >= E) {
    bad = true;
    return r < 0 ? 0 : E - 1;
  }
  return static_cast<int>(r);
}

__global__ void __launch_bounds__(kSortBlock) ep_hist_kernel(const int64_t* __restrict__ ids, int64_t n, int E,
                                                            int* __restrict__ bhist, unsigned int* __restrict__ status) {
  extern __shared__ int h[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kSortBlock + threadIdx.x;
  bool bad = false;
  if (i < n) atomicAdd(&h[clamp_expert(__ldg(ids + i), E, bad)], 1);
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(status, MGF_DEV_ROW_OUT_OF_RANGE);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) bhist[static_cast<int64_t>(blockIdx.x) * E + e] = h[e];
}

__global__ void __launch_bounds__(1024) ep_scan_kernel(int* __restrict__ bhist, int nblocks, int E,
                                                       int64_t* __restrict__ counts) {
  extern __shared__ int tot[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {  // exclusive over blocks, per expert
    int run = 0;
    for (int b = 0; b < nblocks; ++b) {
      const int c = bhist[static_cast<int64_t>(b) * E + e];
      bhist[static_cast<int64_t>(b) * E + e] = run;
      run += c;
    }
    tot[e] = run;
    counts[e] = run;
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // exclusive prefix of the totals over experts (in place)
    const int lane = threadIdx.x;
    int carry = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + lane;
      const int v = e < E ? tot[e] : 0;
      int inc = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += o;
      }
      if (e < E) tot[e] = carry + inc - v;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
  }
  __syncthreads();
  for (int64_t idx = threadIdx.x; idx < static_cast<int64_t>(nblocks) * E; idx += blockDim.x)
    bhist[idx] += tot[idx % E];
}

__global__ void __launch_bounds__(kSortBlock) ep_scatter_kernel(const int64_t* __restrict__ ids, int64_t n, int E,
                                                               int k, const int* __restrict__ bstart,
                                                               int64_t* __restrict__ order, int64_t* __restrict__ inv,
                                                               int64_t* __restrict__ token,
                                                               int64_t* __restrict__ e_sorted) {
  extern __shared__ int wh[];  // [32 warps][E]: copies of each expert in the block's earlier warps
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int idx = threadIdx.x; idx < 32 * E; idx += blockDim.x) wh[idx] = 0;
  __syncthreads();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kSortBlock + threadIdx.x;
  const bool v = i < n;
  bool bad = false;
  const int e = v ? clamp_expert(__ldg(ids + i), E, bad) : -1;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
  if (v && lane == 31 - __clz(peers)) wh[warp * E + e] = __popc(peers);
  __syncthreads();
  for (int c = threadIdx.x; c < E; c += blockDim.x) {  // exclusive over warps, per expert
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int x = wh[w * E + c];
      wh[w * E + c] = run;
      run += x;
    }
  }
  __syncthreads();
  if (v) {
    const int64_t pos = bstart[static_cast<int64_t>(blockIdx.x) * E + e] + wh[warp * E + e] + rank_in_warp;
    order[pos] = i;
    inv[i] = pos;
    token[pos] = i / k;
    e_sorted[pos] = e;
  }
}

// Workspace (int32) layout written by ep_tables_kernel, read by ep_routes_kernel.
struct RouteTables {
  int E, world, rank, e_local;
  int* pos;      // [world][E] first sorted copy of expert e on source s (exclusive prefix over e)
  int* dst0;     // [E] owner row of this rank's first copy of expert e: base[e] + before_rank[e]
  int* seg_end;  // [e_local * world] inclusive prefix of this rank's (local expert, source) segments
};

__host__ __device__ inline RouteTables route_tables(int* ws, int E, int world, int rank, int e_local) {
  RouteTables t{E, world, rank, e_local, ws, ws + world * E, ws + world * E + E};
  return t;
}

__global__ void ep_tables_kernel(const int64_t* __restrict__ c_all, RouteTables t) {
  const int E = t.E, world = t.world;
  for (int s = threadIdx.x; s < world; s += blockDim.x) {  // per-source exclusive prefix over experts
    int run = 0;
    for (int e = 0; e < E; ++e) {
      t.pos[s * E + e] = run;
      run += static_cast<int>(c_all[s * E + e]);
    }
  }
  for (int o = threadIdx.x; o < world; o += blockDim.x) {  // per-owner rows of each expert
    int base = 0;
    for (int e = o * t.e_local; e < (o + 1) * t.e_local; ++e) {
      int tot = 0, before = 0;
      for (int s = 0; s < world; ++s) {
        const int c = static_cast<int>(c_all[s * E + e]);
        if (s < t.rank) before += c;
        tot += c;
      }
      t.dst0[e] = base + before;
      base += tot;
    }
  }
  if (threadIdx.x == 0) {
    int run = 0;
    for (int el = 0; el < t.e_local; ++el)
      for (int s = 0; s < world; ++s) {
        run += static_cast<int>(c_all[s * E + t.rank * t.e_local + el]);
        t.seg_end[el * world + s] = run;
      }
  }
}

__global__ void ep_routes_kernel(const int64_t* __restrict__ e_sorted, int64_t n, int64_t cap, RouteTables t,
                                 const unsigned long long* __restrict__ ret_bases,
                                 const unsigned long long* __restrict__ gret_bases, int64_t row_bytes,
                                 int64_t* __restrict__ dst_rank, int64_t* __restrict__ dst_row,
                                 int64_t* __restrict__ src_rank, int64_t* __restrict__ src_pos,
                                 int64_t* __restrict__ ptr_ret, int64_t* __restrict__ ptr_gret,
                                 int32_t* __restrict__ offs, int32_t* __restrict__ n_recv) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int S = t.e_local * t.world;
  if (i < n) {
    const int e = static_cast<int>(e_sorted[i]);
    dst_rank[i] = e / t.e_local;
    dst_row[i] = t.dst0[e] + (i - t.pos[t.rank * t.E + e]);
  }
  if (i < cap) {
    const int total = t.seg_end[S - 1];
    if (i >= total) {
      src_rank[i] = -1;
      src_pos[i] = -1;
      if (ptr_ret) ptr_ret[i] = 0;
      if (ptr_gret) ptr_gret[i] = 0;
    } else {
      int lo = 0, hi = S - 1;  // first segment whose end is > i
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (t.seg_end[mid] > i) hi = mid; else lo = mid + 1;
      }
      const int el = lo / t.world, s = lo - el * t.world;
      const int seg_start = lo == 0 ? 0 : t.seg_end[lo - 1];
      const int64_t sp = t.pos[s * t.E + t.rank * t.e_local + el] + (i - seg_start);
      src_rank[i] = s;
      src_pos[i] = sp;
      if (ptr_ret) ptr_ret[i] = static_cast<int64_t>(ret_bases[s] + sp * row_bytes);
      if (ptr_gret) ptr_gret[i] = static_cast<int64_t>(gret_bases[s] + sp * row_bytes);
    }
  }
  if (i < t.e_local) offs[i] = t.seg_end[i * t.world + t.world - 1];
  if (i == 0) n_recv[0] = t.seg_end[S - 1];
}

__global__ void signal_flags_kernel(const unsigned long long* __restrict__ flag_bases, int64_t world, int64_t rank,
                                    unsigned long long seq) {
  __threadfence_system();  // the stream's earlier kernels (e.g. a scatter epilogue's peer stores) precede the flags
  for (int64_t r = threadIdx.x; r < world; r += blockDim.x) {
    unsigned long long* flags = reinterpret_cast<unsigned long long*>(flag_bases[r]);
    st_release_sys_u64(flags + rank, seq);
  }
}

}  // namespace
}  // namespace mgf

extern "C" int64_t mgf_ep_sort_workspace_words(int64_t n, int32_t num_experts) {
  const int64_t nb = (n + mgf::kSortBlock - 1) / mgf::kSortBlock;
  return (nb > 0 ? nb : 1) * num_experts;
}

extern "C" int mgf_ep_sort(const int64_t* expert_ids, int64_t n, int32_t num_experts, int32_t topk,
                           int32_t* workspace, int64_t* order, int64_t* inv_order, int64_t* copy_token,
                           int64_t* e_sorted, int64_t* counts, void* stream) {
  using namespace mgf;
  if (n < 0 || n > INT32_MAX || num_experts < 1 || num_experts > 1024 || topk < 1) return MGF_ERR_INVALID_ARGUMENT;
  if (counts == nullptr || workspace == nullptr ||
      (n > 0 && (expert_ids == nullptr || order == nullptr || inv_order == nullptr || copy_token == nullptr ||
                 e_sorted == nullptr)))
    return MGF_ERR_INVALID_ARGUMENT;
  unsigned int* status = status_word_address();
  if (status == nullptr) return MGF_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nb = static_cast<int>((n + kSortBlock - 1) / kSortBlock);
  const int smem_h = num_experts * static_cast<int>(sizeof(int));
  const int smem_w = 32 * num_experts * static_cast<int>(sizeof(int));
  if (cudaFuncSetAttribute(ep_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_w) != cudaSuccess)
    return MGF_ERR_CUDA;
  if (nb > 0) ep_hist_kernel<<<nb, kSortBlock, smem_h, st>>>(expert_ids, n, num_experts, workspace, status);
  ep_scan_kernel<<<1, 1024, smem_h, st>>>(workspace, nb, num_experts, counts);
  if (nb > 0)
    ep_scatter_kernel<<<nb, kSortBlock, smem_w, st>>>(expert_ids, n, num_experts, topk, workspace, order,
                                                      inv_order, copy_token, e_sorted);
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int64_t mgf_ep_routes_workspace_words(int32_t world, int32_t num_experts) {
  return static_cast<int64_t>(world) * num_experts + num_experts + num_experts;
}

extern "C" int mgf_ep_routes(const int64_t* c_all, int32_t world, int32_t num_experts, const int64_t* e_sorted,
                             int64_t n, int32_t rank, int64_t cap, const unsigned long long* ret_bases,
                             const unsigned long long* gret_bases, int64_t row_bytes, int32_t* workspace,
                             int64_t* dst_rank, int64_t* dst_row, int64_t* src_rank, int64_t* src_pos,
                             int64_t* ptr_ret, int64_t* ptr_gret, int32_t* offs, int32_t* n_recv, void* stream) {
  using namespace mgf;
  if (world < 1 || num_experts < 1 || num_experts % world || rank < 0 || rank >= world || n < 0 || cap < 1 ||
      n > INT32_MAX || cap > INT32_MAX || c_all == nullptr || workspace == nullptr || offs == nullptr ||
      n_recv == nullptr || src_rank == nullptr || src_pos == nullptr ||
      (n > 0 && (e_sorted == nullptr || dst_rank == nullptr || dst_row == nullptr)))
    return MGF_ERR_INVALID_ARGUMENT;
  if ((ptr_ret != nullptr && ret_bases == nullptr) || (ptr_gret != nullptr && gret_bases == nullptr))
    return MGF_ERR_INVALID_ARGUMENT;
  const int e_local = num_experts / world;
  const RouteTables t = route_tables(workspace, num_experts, world, rank, e_local);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ep_tables_kernel<<<1, 32, 0, st>>>(c_all, t);
  int64_t items = n > cap ? n : cap;
  if (items < e_local) items = e_local;
  const int64_t blocks = (items + 255) / 256;
  ep_routes_kernel<<<static_cast<unsigned>(blocks > 0 ? blocks : 1), 256, 0, st>>>(
      e_sorted, n, cap, t, ret_bases, gret_bases, row_bytes, dst_rank, dst_row, src_rank, src_pos, ptr_ret,
      ptr_gret, offs, n_recv);
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}

extern "C" int mgf_signal_flags(const unsigned long long* flag_bases, int64_t world, int64_t rank,
                                unsigned long long seq, void* stream) {
  using namespace mgf;
  if (flag_bases == nullptr || world < 1 || world > 1024 || rank < 0 || rank >= world) return MGF_ERR_INVALID_ARGUMENT;
  signal_flags_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag_bases, world, rank, seq);
  return cudaGetLastError() == cudaSuccess ? MGF_OK : MGF_ERR_CUDA;
}
