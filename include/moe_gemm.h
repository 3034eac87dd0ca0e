/*
 * moe_gemm.h -- C ABI of the B200 (sm_100a) MoE FFN grouped-GEMM library (libmoe_gemm.so).
 *
 * One launcher runs every GEMM of the MoE FFN forward and backward.  A call describes one
 * grouped GEMM over E experts whose token rows are delimited by `offs` (int32 cumulative
 * end offsets, on the device) and picks one of four fused epilogues.  All pointers are
 * device pointers; nothing here allocates, synchronises the host or reads `offs` on the host.
 *
 * Reference interfaces this ABI replaces (Butterfingrz/CuTe-MoE-Train,
 * paths relative to cutlass_op/bf16_grouped_mm/):
 *   MGF_EPI_BIAS            <- csrc/binding.cu:13-34  `_grouped_mm_cuda` (ragged-M, bias optional)
 *                              and csrc/grouped_mm_kernel.cuh:478 `bf16bf16_grouped_mm`
 *   MGF_EPI_SWIGLU          <- csrc/binding.cu:39-64  `_grouped_mm_swiglu_cuda`
 *                              and csrc/grouped_mm_kernel.cuh:1365 `bf16bf16_grouped_mm_swiglu`
 *   MGF_EPI_SWIGLU_BWD      <- csrc/binding.cu:68-118 `_grouped_mm_swiglu_bwd_cuda`
 *                              and csrc/grouped_mm_kernel.cuh:854 `bf16bf16_grouped_mm_swiglu_bwd`
 *   MGF_EPI_WGRAD           <- the ragged-K (2D x 2D) branch of `_grouped_mm_cuda`
 *                              (csrc/grouped_mm_kernel.cuh:224-226, csrc/grouped_mm_common.cuh:120-133)
 *                              fused with custom_op.py:79-101 `_segment_sum_rows` (bias gradient)
 *
 * Error behaviour: host-side argument errors return a negative MGF_ERR_* code and launch
 * nothing (the torch layer turns them into RuntimeError, like the reference's TORCH_CHECKs).
 * Device-side problems (malformed offs, a pipeline wait that ran out) never trap: the kernel
 * records a bit in a device status word that mgf_device_status() reads.
 */
#ifndef MOE_GEMM_H_
#define MOE_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Epilogue selector. */
enum mgf_epilogue {
  MGF_EPI_BIAS = 0,       /* D = bf16(A*B[e] + bias[e])           (bias may be NULL)          */
  MGF_EPI_SWIGLU = 1,     /* aux = bf16(A*B[e] + bias[e]); D2 = swiglu(aux) (gate/up interleaved) */
  MGF_EPI_SWIGLU_BWD = 2, /* D = swiglu_bwd(A*B[e], aux): interleaved (d_gate, d_up) pairs     */
  MGF_EPI_WGRAD = 3       /* ragged-K: D[e] = A[g]^T-view * B[g]; D2[e] = column sums of B[g]  */
};

/* Status codes returned by the host entry points. */
enum mgf_status {
  MGF_OK = 0,
  MGF_ERR_INVALID_ARGUMENT = -1,
  MGF_ERR_UNSUPPORTED_LAYOUT = -2,
  MGF_ERR_ALIGNMENT = -3,
  MGF_ERR_TOO_MANY_GROUPS = -4,
  MGF_ERR_CUDA = -5,
  MGF_ERR_NO_DEVICE_SUPPORT = -6
};

/* Device status bits recorded by the kernels (read with mgf_device_status). */
#define MGF_DEV_WAIT_TIMEOUT 0x1u  /* a pipeline wait ran out; the kernel stopped early        */
#define MGF_DEV_BAD_OFFS 0x2u      /* offs not non-decreasing or beyond the row extent; clamped */
#define MGF_DEV_ROW_OUT_OF_RANGE 0x4u /* a row index of gather/combine/push fell outside its buffer;
                                         that row was skipped (left unwritten)                    */

/*
 * One grouped GEMM.  Matrix layouts are given as element strides of bf16 tensors.
 *
 * Ragged-M epilogues (BIAS, SWIGLU, SWIGLU_BWD):
 *   A    : [total_rows, k] row-major (stride lda, unit stride along k); rows of group e are
 *          offs[e-1]..offs[e]-1.
 *   B    : [E, k, n] with batch stride ldb_batch; b_mn_major=1 means unit stride along n
 *          (row stride ldb), b_mn_major=0 means unit stride along k (column stride ldb).
 *   D    : [total_rows, n_out] row-major, stride ldd (n_out = n, or the aux tensor for SWIGLU).
 *   D2   : SWIGLU only: swiglu_out [total_rows, n/2], stride ldd2.
 *   aux  : SWIGLU_BWD only: [total_rows, 2n] interleaved (gate, up), stride ld_aux; D is then
 *          grad_aux [total_rows, 2n] with stride ldd.
 * Ragged-K epilogue (WGRAD):
 *   A    : [total_rows, m] row-major (stride lda): the GEMM uses its transpose per group.
 *   B    : [total_rows, n] row-major (stride ldb).
 *   D    : [E, m, n] bf16, row stride ldd, batch stride ldd_batch.  Empty groups get zeros.
 *   D2   : optional [E, n] bf16 bias gradient (stride ldd2 between groups): column sums of B.
 * Extents: n a multiple of 8 (whole 16-byte output units); k (ragged-M) and m (ragged-K) any
 * positive value.  Every base pointer 16-byte aligned and every row / batch stride a multiple of
 * 8 elements (the TMA rule); reads past k, m, n or total_rows return zeros.
 */
typedef struct mgf_gemm_desc {
  int32_t epilogue;      /* enum mgf_epilogue */
  int32_t num_groups;    /* E (1..1024) */
  int64_t total_rows;    /* extent of the ragged dimension (tokens) */
  int64_t m, n, k;       /* fixed GEMM extents (m unused for ragged-M, k unused for ragged-K) */
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  int64_t ldb_batch;
  int32_t b_mn_major;
  const int32_t* offs;   /* device int32 [E] cumulative end offsets */
  const void* bias;      /* device bf16 [E, n] or NULL */
  int64_t bias_stride;
  void* d;
  int64_t ldd;
  int64_t ldd_batch;
  void* d2;
  int64_t ldd2;
  const void* aux;
  int64_t ld_aux;
  float swiglu_alpha;
  float swiglu_limit;
  int32_t store_aux;     /* SWIGLU: 1 = also write aux (D) */
  int32_t sm_carveout;   /* SMs left free for concurrent work (collectives); 0 = use all */
  int32_t* workspace;    /* WGRAD: device int32[1], zero-filled before the call: the dynamic tile
                            counter (tiles of a ragged-K launch cost in proportion to their group's
                            size; handing them out in order keeps the CTAs on neighbouring tiles).
                            NULL = static tile striding.  One workspace per launch in flight. */
  int32_t bias_per_row;  /* BIAS, ragged-M only: 0 = bias[e, col] added to every row (the MoE case);
                            1 = bias[e, row - group start] added to every column of a row (the
                            transposed form of the reference's ragged-N bias, csrc/grouped_mm_common.cuh:107-118) */
  int32_t ab_type;       /* enum mgf_ab_type: element type of A and B.  MGF_AB_E4M3 (8-bit float).
                            Ragged-M (BIAS, SWIGLU, SWIGLU_BWD; B with unit stride along k): the
                            accumulator is scaled by scale_a[row] * scale_b[e * scale_b_stride + col]
                            before the bias / SwiGLU / SwiGLU backward.  Ragged-K (WGRAD): A and B are
                            the same row-major token layouts as for bf16, with per-feature scales:
                            D[e][i][j] = acc * scale_a[i] * scale_b[j], the bias gradient acc * scale_b[j]
                            (scale_b_stride unused).  lda / ldb / ldb_batch then count bytes
                            (multiples of 16). */
  const float* scale_a;  /* E4M3: device fp32 [total_rows] (ragged-M) or [m] (ragged-K) */
  const float* scale_b;  /* E4M3: device fp32 [E, n] (ragged-M) or [n] (ragged-K) */
  int64_t scale_b_stride;
  const int64_t* d_row_ptrs; /* BIAS (bf16) only, NULL = off.  Scatter mode: output row r is written
                            at the address d_row_ptrs[r] (device int64 [total_rows]; any address this
                            device can store to, e.g. a peer GPU's IPC-mapped buffer; 0 = row not
                            written; 16-byte aligned, 32-byte aligned for whole-sector stores)
                            instead of d + r * ldd (d and ldd are then unused).  The expert-parallel
                            combine writes each expert output straight into its source rank's buffer
                            this way, fusing the transfer into the GEMM epilogue. */
  int32_t group_begin;   /* groups 0 .. group_begin-1 are skipped (no tile computed, nothing written --
                            for WGRAD not even the zeros of empty groups); 0 = all.  Lets a caller run a grouped GEMM in two launches
                            over the expert ranges [0, g) and [g, E) of one offs array, e.g. while the
                            rows of the second range are still arriving. */
} mgf_gemm_desc;

enum mgf_ab_type { MGF_AB_BF16 = 0, MGF_AB_E4M3 = 1 };

/* Launch one grouped GEMM on `stream` (a cudaStream_t; NULL = legacy default stream).
 * Replaces: csrc/binding.cu:13-148 (the three pybind entry points) + the dispatch in
 * csrc/grouped_mm_kernel.cuh:390-486, 760-864, 1267-1390. */
int mgf_grouped_gemm_launch(const mgf_gemm_desc* desc, void* stream);

/* Allocation-free variant of the ragged-K weight-gradient launch (MGF_EPI_WGRAD only).
 * No counterpart in the reference.  For callers that cannot allocate device memory when they
 * launch (a runtime with a fixed, up-front memory plan; a host program that binds this ABI and
 * only holds the buffers it was given): the zero-filled tile counter normally passed as
 * desc->workspace comes instead from a 256-byte static device array inside the library (64 int32
 * words, 1 used per call; held by every GPU that loads the library until exit).  desc->workspace
 * must be NULL.  The call clears the word it uses on `stream` before the kernel; all calls share
 * the array, so calls that overlap on the GPU race and must not be issued.  Each call looks up
 * the array's address on the calling device (so it stays right after a device reset); the first
 * call on a device should come before any stream capture.  Allocates
 * nothing (no cudaMalloc/cudaFree).  Same return codes as mgf_grouped_gemm_launch. */
int mgf_grouped_gemm_launch_noalloc(const mgf_gemm_desc* desc, void* stream);

/* Expert-parallel row movement (no counterpart in the reference, which has no distributed code).
 * bf16 rows of row_elems elements (a multiple of 8), row strides ld_* in elements (multiples of 8),
 * 16-byte aligned bases, int64 device index arrays, optional fp32 device scales (NULL = 1).
 *   mgf_gather_rows:  dst[i] = scale[i] * src[idx[i]],                     i < n_rows
 *   mgf_combine_rows: out[t] = sum_{j<k} weights[t*k+j] * rows[pos[t*k+j]], t < n_out (fp32 sum)
 * n_src / n_rows is the row count of src / rows: an index outside [0, n_src) leaves its output
 * row unwritten (combine: any of the token's k indices) and sets MGF_DEV_ROW_OUT_OF_RANGE.
 * Dispatch gathers token copies into expert order; combine sums each token's k expert outputs;
 * each is the other's backward. */
int mgf_gather_rows(const void* src, int64_t ld_src, int64_t n_src, const int64_t* idx, const float* scale,
                    int64_t n_rows, int64_t row_elems, void* dst, int64_t ld_dst, void* stream);
int mgf_combine_rows(const void* rows, int64_t ld_rows, int64_t n_rows, const int64_t* pos, const float* weights,
                     int64_t n_out, int32_t k, int64_t row_elems, void* out, int64_t ld_out, void* stream);

/* Expert-parallel push over NVLink peer memory (no counterpart in the reference): for i < n rows
 * (n = n_max, or *n_dev when n_dev is non-NULL -- a device-side count), write
 * scale[i] * src[src_idx[i]] (src_idx NULL = i, scale NULL = 1) to row dst_row[i] of the buffer at
 * peer_bases[dst_rank[i]] (device array of `world` base addresses, one per rank, from CUDA IPC
 * mappings; each buffer dst_rows rows of stride ld_dst).  Rows whose rank or destination row falls
 * outside [0, world) x [0, dst_rows), or whose source row falls outside [0, n_src), are skipped and
 * set MGF_DEV_ROW_OUT_OF_RANGE.  Plain peer stores, no multicast.
 * Completion signal (flag_bases non-NULL): when all of the launch's stores are visible, `seq` is
 * written (release, system scope) into slot `rank` of every rank's flag array (flag_bases: device
 * array of `world` addresses of uint64 [world] flag arrays, IPC-mapped); `counter` is a zeroed
 * device uint64 of this rank that the launch uses and leaves at zero.  Readers then call
 * mgf_wait_flags on their own flag array instead of a collective barrier.
 * rotate (optional device int64): entries are visited starting at index *rotate (mod n), so that ranks
 * whose entries are sorted by destination do not all write to the same rank at the same time. */
int mgf_push_rows(const void* src, int64_t ld_src, int64_t n_src, const int64_t* src_idx, const float* scale,
                  int64_t n_max, const int32_t* n_dev, const int64_t* dst_rank, const int64_t* dst_row,
                  const unsigned long long* peer_bases, int64_t world, int64_t dst_rows, int64_t ld_dst,
                  int64_t row_elems, const unsigned long long* flag_bases, unsigned long long* counter,
                  unsigned long long seq, int64_t rank, const int64_t* rotate, void* stream);

/* Wait on `stream` until flags[s] >= seq for every s < world (every rank's push with sequence
 * number seq has landed here), at most timeout_ns; a wait that runs out records
 * MGF_DEV_WAIT_TIMEOUT in the device status word and returns.  One small kernel, no host sync
 * (no counterpart in the reference). */
int mgf_wait_flags(const unsigned long long* flags, int64_t world, unsigned long long seq, int64_t timeout_ns,
                   void* stream);

/* Signal on `stream`: after every earlier operation of the stream (e.g. a scatter-epilogue GEMM
 * that stored rows into peers' buffers), write seq into slot `rank` of every rank's flag array
 * (flag_bases as for mgf_push_rows).  Readers use mgf_wait_flags.  No counterpart in the reference. */
int mgf_signal_flags(const unsigned long long* flag_bases, int64_t world, int64_t rank, unsigned long long seq,
                     void* stream);

/* Device-side plan of the expert-parallel peer transport (no counterpart in the reference; no host
 * synchronisation).  mgf_ep_sort: stable counting sort of n routed copies (expert_ids int64 [n], copy
 * i = token i / topk) by expert: order[p] (copy at sorted position p), inv_order[copy], copy_token[p],
 * e_sorted[p], counts[E] (int64); workspace: int32 [mgf_ep_sort_workspace_words(n, E)] device scratch.
 * Out-of-range ids are clamped and set MGF_DEV_ROW_OUT_OF_RANGE.
 * mgf_ep_routes: from the all-gathered count matrix c_all [world, E] (int64) and this rank's e_sorted:
 * dst_rank / dst_row [n] (owner rank and row of each sorted copy in the owner's receive buffer: local
 * expert-major, then source rank, then sorted order), src_rank / src_pos [cap] (source rank and its
 * sorted position of each receive row; -1 past the received rows), optional ptr_ret / ptr_gret [cap]
 * (ret_bases[src] + src_pos * row_bytes and the same in gret_bases; 0 past the received rows: the row
 * addresses of the scatter epilogues), offs [E / world] (int32) and n_recv [1] (int32).  workspace:
 * int32 [mgf_ep_routes_workspace_words(world, E)] device scratch. */
int64_t mgf_ep_sort_workspace_words(int64_t n, int32_t num_experts);
int mgf_ep_sort(const int64_t* expert_ids, int64_t n, int32_t num_experts, int32_t topk, int32_t* workspace,
                int64_t* order, int64_t* inv_order, int64_t* copy_token, int64_t* e_sorted, int64_t* counts,
                void* stream);
int64_t mgf_ep_routes_workspace_words(int32_t world, int32_t num_experts);
int mgf_ep_routes(const int64_t* c_all, int32_t world, int32_t num_experts, const int64_t* e_sorted, int64_t n,
                  int32_t rank, int64_t cap, const unsigned long long* ret_bases,
                  const unsigned long long* gret_bases, int64_t row_bytes, int32_t* workspace, int64_t* dst_rank,
                  int64_t* dst_row, int64_t* src_rank, int64_t* src_pos, int64_t* ptr_ret, int64_t* ptr_gret,
                  int32_t* offs, int32_t* n_recv, void* stream);

/* e4m3 quantisers of the FP8 path (no counterpart in the reference, which has no FP8): bf16 in,
 * float8_e4m3fn out, fp32 scales = max(amax, 1e-12) / 448, q = saturate(x / scale), round to nearest.
 *   rows:    x [rows, cols] (row stride ldx) -> q [rows, cols] (row stride ldq), scale [rows];
 *   cols:    the same with one scale per column, scale [cols];
 *   weights: w [E, K, N] with element strides s_e, s_k, s_n (s_n == 1 or s_k == 1 read coalesced)
 *            -> q [E, N, K] with K contiguous (row stride ldq >= K), scale [E, N].
 * cols, ldx and ldq multiples of 8, x 16-byte aligned.  Each a few kernels on `stream`, no host sync. */
int mgf_fp8_quantize_rows(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq, float* scale,
                          void* stream);
int mgf_fp8_quantize_cols(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq, float* scale,
                          void* stream);
/* Both scalings of one [rows, cols] activation in two passes: (q_r, s_r) as mgf_fp8_quantize_rows and
 * (q_c, s_c) as mgf_fp8_quantize_cols give, bit-identical (no counterpart in the reference). */
int mgf_fp8_quantize_rows_cols(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q_r, int64_t ldq_r,
                               float* s_r, void* q_c, int64_t ldq_c, float* s_c, void* stream);
int mgf_fp8_quantize_weights(const void* w, int64_t E, int64_t K, int64_t N, int64_t s_e, int64_t s_k, int64_t s_n,
                             void* q, int64_t ldq, float* scale, void* stream);
/* Both axes of one weight [E, K, N] (unit stride along n, n % 8 == 0, 16-byte aligned strides and
 * bases) in two passes: qa [E, N, ldqa] / sa [E, N] as mgf_fp8_quantize_weights gives for w, and
 * qb [E, K, ldqb] / sb [E, K] as it gives for w^T (codes n-contiguous, one scale per (e, k));
 * bit-identical to the two calls (no counterpart in the reference). */
int mgf_fp8_quantize_weights_both(const void* w, int64_t E, int64_t K, int64_t N, int64_t s_e, int64_t s_k, void* qa,
                                  int64_t ldqa, float* sa, void* qb, int64_t ldqb, float* sb, void* stream);

/* Map a peer process's device allocation (its 64-byte cudaIpcMemHandle_t) into the context of
 * the calling thread's current device, peer access enabled, for mgf_push_rows destinations
 * (no counterpart in the reference).  mgf_ipc_close unmaps it. */
int mgf_ipc_open(const void* handle, void** base_out);
/* The 64-byte IPC handle of the allocation containing device pointer `ptr`, and ptr's byte offset
 * in it (what a peer passes to mgf_ipc_open, then adds the offset). */
int mgf_ipc_get_handle(const void* ptr, void* handle_out, int64_t* offset_out);
int mgf_ipc_close(void* base);

/* Read (and optionally clear) the device status word of `device`.  Synchronises that
 * device; meant for tests and debugging, never called on the hot path. */
int mgf_device_status(int device, uint32_t* status_out, int clear);

/* Human-readable text for a mgf_status code. */
const char* mgf_status_string(int status);

/* Text of the last CUDA / driver error seen by mgf_grouped_gemm_launch on this host thread
 * ("" when the last call succeeded). */
const char* mgf_last_error_detail(void);

/* Library ABI version (major * 100 + minor). */
int mgf_version(void);

/* sizeof(mgf_gemm_desc) as compiled into the library, for bindings that declare the struct
 * themselves (ctypes, cffi) to check their layout against. */
size_t mgf_gemm_desc_size(void);

#ifdef __cplusplus
}
#endif

#endif /* MOE_GEMM_H_ */
