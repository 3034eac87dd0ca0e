// B200 (sm_100a) grouped GEMM for the MoE FFN path: persistent ragged-M / ragged-K tile
// scheduler, TMA-fed tcgen05 UMMA with fp32 accumulators in TMEM (double-buffered so the
// epilogue of tile i overlaps the mainloop of tile i+1, except in the 256-row ragged-K form),
// and four fused epilogues:
//   MGF_EPI_BIAS        D = bf16(acc + bias[e])                     (down-proj fwd, dgrads)
//   MGF_EPI_SWIGLU      aux = bf16(acc + bias[e]), D2 = clamped SwiGLU(aux)  (up-proj fwd)
//   MGF_EPI_SWIGLU_BWD  D = SwiGLU_bwd(acc, aux)                    (down-proj dgrad)
//   MGF_EPI_WGRAD       D[e] = A[g]^T B[g] over ragged K, D2[e] = column sums of B[g]
//
// Semantics follow Butterfingrz/CuTe-MoE-Train (paths relative to cutlass_op/bf16_grouped_mm/):
//   bias epilogue          csrc/grouped_mm_kernel.cuh:130-143 (fp32 acc + bias, one bf16 rounding)
//   SwiGLU forward         csrc/grouped_mm_swiglu_visitor.cuh:295-334 (gate = even column,
//                          up = odd column, min() on gate, two-sided clamp on up,
//                          out = g*sigmoid(alpha*g)*(u+1), computed from the bf16-rounded aux)
//   SwiGLU backward        csrc/grouped_mm_swiglu_bwd_visitor.cuh:35-68
//   ragged-K weight grad   csrc/grouped_mm_common.cuh:120-133
//   bias gradient          custom_op.py:79-101 (_segment_sum_rows, fp32 accumulation)
//
// Warp roles (320 threads, one CTA per SM):
//   warp 0      TMA producer (one elected thread)
//   warp 1      TMEM allocator + UMMA issuer; for ragged-K it also patches the K tail of the
//               last stage (zero rows past the group end) and writes the bias-gradient "ones" row
//   warps 2..9  epilogue (two warpgroups, each half of the tile's columns): TMEM -> registers ->
//               fused math -> predicated 16/32-byte global stores (ragged-M) or per-warp 32 x 32
//               TMA tile stores from shared memory (ragged-K)
//
// CTA pairs (CG = 2, cluster of two, cta_group::2 MMAs on 256-row tiles) for ragged-M launches whose
// groups are large; single CTAs (128-row tiles) otherwise.  Ragged-K runs single CTAs in one of
// three forms: 256-row tiles (MH = 2: two 128-row accumulators over all of TMEM share each B stage,
// no TMEM double buffer) for longer groups, one wide TMA store per warp and tile (OB = 4) for short
// groups, 128-row tiles with 32 x 32 stores otherwise.  F8 = true is the e4m3 variant of every
// epilogue (kind::f8f6f4, row / column scales applied in the epilogue).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>

#include "moe_gemm.h"
#include "ptx.cuh"

namespace mgf {

__device__ unsigned int g_status;

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kMaxGroups = 1024;
constexpr int kEpiGroups = 2;                 // epilogue warpgroups, each owns half of the columns
constexpr int kNumEpiWarps = 4 * kEpiGroups;
constexpr int kThreads = 64 + 32 * kNumEpiWarps;
constexpr int kRing = 4;                      // tile ids in flight between the producer and the consumers
constexpr uint64_t kWaitLimitNs = 1500ull * 1000ull * 1000ull;  // 1.5 s per pipeline wait
constexpr uint64_t kDrainLimitNs = 100ull * 1000ull * 1000ull;

// OB: 2 KB output staging slices per epilogue warp (ragged-K TMA-store epilogue).  OB = 1: one
// 32 x 32 store per chunk.  OB = 4 (short groups): a warp stages all its chunks of a tile (32 rows x
// up to 128 columns) and stores them with one TMA store, 4x fewer store operations per tile, at the
// price of a pipeline stage that tiles of a few K stages do not need.
// MH: 128-row accumulators per CTA (2: the 256-row single-CTA weight gradient, both TMEM halves).
template <int BN, int CG, bool B_MN, int OB = 1, int MH = 1>
struct TileCfg {
  static constexpr int A_BYTES = BM * BK * 2 * MH;                   // this CTA's 128 (or 256) rows of A
  static constexpr int BNC = BN / CG;                                // this CTA's columns of B
  static constexpr int B_CHUNKS = (BNC + 63) / 64;                   // 64-column chunks (MN-major / ragged-K)
  static constexpr int B_BYTES = B_MN ? B_CHUNKS * 8192 : BNC * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SCHED_BYTES = 3 * 4 * (kMaxGroups + 1);
  static constexpr int OUT_CHUNK_BYTES = BM * 32 * 2;                // one 128 x 32 bf16 output chunk
  static constexpr int OUT_BYTES = kEpiGroups * OUT_CHUNK_BYTES * OB;  // TMA-store staging (ragged-K)
  static constexpr int OUT_OFFSET = (BAR_BYTES + SCHED_BYTES + 1023) / 1024 * 1024;  // after the stages
  static constexpr int BUDGET = 227 * 1024 - 1024 - OUT_OFFSET - OUT_BYTES;
  static constexpr int STAGES = (BUDGET / STAGE_BYTES) > 8 ? 8 : (BUDGET / STAGE_BYTES);
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + OUT_OFFSET + OUT_BYTES;
  static_assert(STAGES >= 3, "pipeline depth");
  static_assert((3 * STAGES + 5 + 4 * kRing) * 8 + 8 + 8 * kRing <= BAR_BYTES, "barrier area");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

struct Params {
  int epi;
  int E;
  int64_t total_rows;
  int m, n, k;
  int n_tiles;
  int m_tiles;        // ragged-K: tiles along m per group (incl. the extra bias-grad tile)
  int m_tiles_real;   // ragged-K: ceil(m / tile rows)
  int bias_grad;      // ragged-K: write D2
  int a_chunked, b_chunked;  // ragged-K: tmA / tmB are 3D {64, rows, 64-column chunks}: one box per stage
  const int32_t* offs;
  const __nv_bfloat16* bias;
  int64_t bias_stride;
  int bias_per_row;   // BIAS: bias[e, row - group start] added along the row
  int bke;            // elements of K per pipeline stage (64 bf16 or 128 e4m3: 128 bytes)
  const float* scale_a;  // e4m3: per-row scale of A
  const float* scale_b;  // e4m3: per-(group, column) scale of B
  int64_t scale_b_stride;
  __nv_bfloat16* d;
  int64_t ldd, ldd_batch;
  __nv_bfloat16* d2;
  int64_t ldd2;
  const __nv_bfloat16* aux;
  int64_t ld_aux;
  float alpha, limit;
  int store_aux;
  int aux_v8;         // aux base 32-byte aligned and row pitch a multiple of 32 bytes
  int d_v8, d2_v8;    // the same for the ragged-M outputs d and d2
  int stall_test;     // test hook: the producer hands out no tiles, so every consumer wait runs out
  int* tile_counter;  // zero-filled device counter: dynamic tile order; nullptr = static striding
  const long long* d_rows;  // BIAS scatter mode: destination address of every output row (0 = none)
  int group_begin;          // ragged-M: groups below this index have no tiles (their rows are not touched)
  int small_k;              // ragged-K bf16, single CTAs: one wide TMA store per warp and tile, one stage fewer
  int m256;                 // ragged-K single CTAs, BN 256: 256-row tiles (two accumulators share B)
};

struct TileInfo {
  int e;
  int m_blk, n_blk;
  int row0, row_end;      // ragged-M: global rows of this tile / group end
  int k_start, k_end;     // ragged-K: token range of the group
  int nk;                 // number of BK blocks
};

struct SchedSmem {
  int* prefix;     // [E+1] tile prefix
  int* seg_start;  // [E]
  int* seg_end;    // [E]
};

template <bool CLUSTER = false>
__device__ __forceinline__ bool try_wait_sel(uint32_t bar, uint32_t parity) {
  if constexpr (CLUSTER) return ptx::mbar_try_wait_cluster(bar, parity);
  return ptx::mbar_try_wait(bar, parity);
}

// Wait for phase `parity` of an mbarrier for at most `limit_ns`.  CLUSTER = true acquires at
// cluster scope (barriers that the peer CTA of a pair also arrives on).
template <bool CLUSTER = false>
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                             uint64_t limit_ns = kWaitLimitNs) {
  if (try_wait_sel<CLUSTER>(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    if (try_wait_sel<CLUSTER>(bar, parity)) return true;
    if ((++it & 127u) == 0) {
      if (*abort_flag) return false;
      if (ptx::globaltimer_ns() - t0 > limit_ns) {
        *abort_flag = 1;
        atomicOr(&g_status, MGF_DEV_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}


#ifndef MGF_AUX_NOALLOC
#define MGF_AUX_NOALLOC 1
#endif
// One chunk of aux words (32 packed (gate, up) pairs = 128 bytes of one row) as four 32-byte loads;
// words past n read as zero.  Each sector is requested once, so nothing relies on L1 reuse.
// v8 = false (aux rows only 16-byte aligned): eight 16-byte loads.
__device__ __forceinline__ void load_aux_chunk(const __nv_bfloat16* row, int col0, int n, bool valid, bool v8,
                                               uint4 (&aw)[8]) {
  const uint4* ap = reinterpret_cast<const uint4*>(row + 2 * col0);
  if (!v8) {
#pragma unroll
    for (int g = 0; g < 8; ++g) aw[g] = (valid && col0 + 4 * g < n) ? __ldg(ap + g) : make_uint4(0, 0, 0, 0);
    return;
  }
#pragma unroll
  for (int g = 0; g < 8; g += 2) {
    if (valid && col0 + 4 * g < n) {
      if (MGF_AUX_NOALLOC) ptx::ld_nc_v8_noalloc(ap + g, aw[g], aw[g + 1]);
      else ptx::ld_nc_v8(ap + g, aw[g], aw[g + 1]);
    } else {
      aw[g] = make_uint4(0, 0, 0, 0);
      aw[g + 1] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Store the first `nvalid` of NU 16-byte units of one output row; pairs of units go out as one
// 32-byte store when v8 (the row and its 32-byte pairs aligned).
template <int NU>
__device__ __forceinline__ void store_units(void* dst, const uint4 (&u)[NU], int nvalid, bool v8) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int g = 0; g < NU; g += 2) {
    if (v8 && g + 1 < nvalid) {
      ptx::st_v8(d + g, u[g], u[g + 1]);
    } else {
      if (g < nvalid) d[g] = u[g];
      if (g + 1 < nvalid) d[g + 1] = u[g + 1];
    }
  }
}

template <int TM, bool RAGGED_K>
__device__ __forceinline__ void decode_tile(int t, const Params& p, const SchedSmem& s, TileInfo& ti) {
  int lo = 0, hi = p.E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s.prefix[mid] <= t) lo = mid; else hi = mid;
  }
  ti.e = lo;
  const int local = t - s.prefix[lo];
  if constexpr (!RAGGED_K) {
    // n fastest: the CTAs at work share a few row blocks and the expert's whole weight slab
    ti.m_blk = local / p.n_tiles;
    ti.n_blk = local - ti.m_blk * p.n_tiles;
  } else {
    // m fastest: the CTAs at work share a few column blocks of B (the gradient) and all of A
    // (the activations) for the group's tokens, which stays resident in L2 across windows
    ti.n_blk = local / p.m_tiles;
    ti.m_blk = local - ti.n_blk * p.m_tiles;
  }
  if constexpr (!RAGGED_K) {
    ti.row0 = s.seg_start[lo] + ti.m_blk * TM;
    ti.row_end = s.seg_end[lo];
    ti.k_start = 0;
    ti.k_end = p.k;
    ti.nk = (p.k + p.bke - 1) / p.bke;
  } else {
    ti.row0 = 0;
    ti.row_end = 0;
    ti.k_start = s.seg_start[lo];
    ti.k_end = s.seg_end[lo];
    ti.nk = (ti.k_end - ti.k_start + p.bke - 1) / p.bke;  // K rows per stage: 64 (bf16) or 128 (e4m3)
  }
}

// Clamp every group's [start, end) into [0, total_rows] and build the tile prefix.  Malformed
// offs (decreasing, negative, or past total_rows) are reported through g_status, never by a
// trap; the clamped segments keep every access in bounds.  Run by one warp.
template <int TM, bool RAGGED_K>
__device__ void build_schedule(const Params& p, const SchedSmem& s, int lane) {
  int running = 0;
  bool bad = false;
  const long long tr = p.total_rows;
  for (int base = 0; base < p.E; base += 32) {
    const int e = base + lane;
    int cnt = 0;
    if (e < p.E) {
      const long long raw_prev = e == 0 ? 0 : (long long)__ldg(p.offs + e - 1);
      const long long raw_end = (long long)__ldg(p.offs + e);
      if (raw_end < raw_prev || raw_end > tr || raw_prev < 0) bad = true;
      const long long sp = raw_prev < 0 ? 0 : (raw_prev > tr ? tr : raw_prev);
      const long long ep = raw_end < sp ? sp : (raw_end > tr ? tr : raw_end);
      s.seg_start[e] = (int)sp;
      s.seg_end[e] = (int)ep;
      if constexpr (!RAGGED_K) {
        cnt = e < p.group_begin ? 0 : (int)((ep - sp + TM - 1) / TM) * p.n_tiles;
      } else {
        cnt = e < p.group_begin ? 0 : p.m_tiles * p.n_tiles;
      }
    }
    int inc = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += o;
    }
    if (e < p.E) s.prefix[e + 1] = running + inc;
    running += __shfl_sync(0xffffffffu, inc, 31);
  }
  if (lane == 0) s.prefix[0] = 0;
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(&g_status, MGF_DEV_BAD_OFFS);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// sigma(z) = 0.5 * tanh(z / 2) + 0.5, the form the reference's SwiGLU visitors use
// (csrc/grouped_mm_swiglu_visitor.cuh:309-334, csrc/grouped_mm_swiglu_bwd_visitor.cuh:35-68), on the
// hardware tanh approximation (one MUFU operation; max relative error about 2^-11, below bf16's 2^-8).
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float sigmoidf_fast(float z) { return fmaf(0.5f, tanh_approx(0.5f * z), 0.5f); }

// SwiGLU forward on one (gate, up) pair of bf16-rounded values.
__device__ __forceinline__ float swiglu_fwd(float g, float u, float alpha, float limit) {
  const float gc = fminf(g, limit);
  const float uc = fmaxf(fminf(u, limit), -limit);
  return gc * sigmoidf_fast(alpha * gc) * (uc + 1.0f);
}

// SwiGLU backward for one packed (gate, up) word of aux; returns packed (d_gate, d_up).
__device__ __forceinline__ uint32_t swiglu_bwd_word(float gs, uint32_t aux_word, float alpha, float limit) {
  const float g = bf16_lo(aux_word);
  const float u = bf16_hi(aux_word);
  const float gc = fminf(g, limit);
  const float uc = fmaxf(fminf(u, limit), -limit);
  const float sig = sigmoidf_fast(alpha * gc);
  float d_gate = gs * (uc + 1.0f) * sig * (1.0f + alpha * gc * (1.0f - sig));
  float d_up = gs * gc * sig;
  d_gate = (g <= limit) ? d_gate : 0.0f;
  d_up = (u >= -limit && u <= limit) ? d_up : 0.0f;
  return pack_bf16x2(d_gate, d_up);
}

// Zero the K rows valid_k..end_k-1 (past the group end, up to the last row the MMAs read) in this
// CTA's A and B chunks of one stage (each K row is one 128-byte line of a 64-column chunk, whatever
// the swizzle) and set the bias-gradient "ones" row of A for the valid K rows.  Run by one warp; the
// caller fences the writes to the async proxy.
template <int A_CHUNKS, int B_CHUNKS>
__device__ __forceinline__ void patch_ragged_k_stage(uint8_t* sA, int valid_k, int end_k, int ones_local,
                                                     int lane) {
  constexpr int kChunks = A_CHUNKS + B_CHUNKS;
  // 16-byte unit u of a chunk is K row u / 8 (8 units per 128-byte row): clear units
  // 8*valid_k..8*end_k-1 of every chunk, the same unit of all chunks per iteration (8 KB apart).
  for (int u = valid_k * 8 + lane; u < end_k * 8; u += 32) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) *reinterpret_cast<uint4*>(sA + c * 8192 + u * 16) = make_uint4(0, 0, 0, 0);
  }
  if (ones_local >= 0) {
    // The A feature row past m reads as zero (TMA out-of-bounds fill); 1.0 in its valid K rows makes
    // accumulator row `ones_local` the column sums of B.  128-byte swizzle: 16-byte unit ^= row % 8.
    const int c1 = ones_local >> 6, mm = ones_local & 63;
    for (int kr = lane; kr < valid_k; kr += 32) {
      const int off = c1 * 8192 + kr * 128 + (((mm >> 3) ^ (kr & 7)) << 4) + (mm & 7) * 2;
      *reinterpret_cast<uint16_t*>(sA + off) = 0x3F80u;
    }
  }
}

// e4m3 variant: every operand chunk of a stage is 128 elements (128 bytes) wide and 128 K rows
// deep (16 KB); clear the K rows past the group end and put e4m3 1.0 (0x38) into the ones row.
template <int CHUNKS>
__device__ __forceinline__ void patch_ragged_k_stage_f8(uint8_t* sA, int valid_k, int end_k, int ones_local,
                                                        int lane) {
  for (int u = valid_k * 8 + lane; u < end_k * 8; u += 32) {
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) *reinterpret_cast<uint4*>(sA + c * 16384 + u * 16) = make_uint4(0, 0, 0, 0);
  }
  if (ones_local >= 0) {  // A chunks hold 128 features each; 128-byte swizzle: 16-byte unit ^= row % 8
    const int mm = ones_local & 127;
    for (int kr = lane; kr < valid_k; kr += 32) {
      const int off = (ones_local >> 7) * 16384 + kr * 128 + ((((mm >> 4) ^ (kr & 7))) << 4) + (mm & 15);
      sA[off] = 0x38u;
    }
  }
}

// CG = 1: one CTA per 128 x BN tile.  CG = 2: a cluster of two CTAs per 256 x BN tile; the even
// CTA issues tcgen05.mma.cta_group::2 over both CTAs' shared memory (each CTA holds 128 rows of A
// and BN/2 columns of B) and both CTAs' TMEM (each holds its 128 rows of the accumulator).
// Stages whose odd-CTA half must be patched first (ragged-K tails, the ones row) are "relayed":
// the odd CTA counts their bytes on its own barrier, patches, then arrives on the even CTA's
// patch_done barrier; every other stage counts both CTAs' bytes directly on the even CTA's barrier.
template <int BN, int EPI, bool A_MN, bool B_MN, int CG, bool F8 = false, int OB = 1, int MH = 1>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmD, const Params p) {
  using Cfg = TileCfg<BN, CG, B_MN, OB, MH>;
  static_assert(MH == 1 || (EPI == MGF_EPI_WGRAD && CG == 1 && OB == 1 && BN == 256),
                "256-row tiles: single-CTA weight gradient, BN = 256");
  static_assert(OB == 1 || (EPI == MGF_EPI_WGRAD && OB == 4 && CG == 1 && !F8 && BN != 192),
                "wide output staging: bf16 single-CTA weight gradient, 64-column-aligned warp halves");
  constexpr bool RAGGED_K = (EPI == MGF_EPI_WGRAD);
  constexpr int KR = (RAGGED_K && F8) ? 128 : BK;  // ragged-K: token rows per stage
  constexpr int KMMA = F8 ? 32 : 16;                // K rows (elements) of one MMA instruction
  constexpr int kMmaPerStage = 4;                   // 128 bytes of K per stage / 32 bytes per instruction
  static_assert(!RAGGED_K || KR / KMMA == kMmaPerStage, "ragged-K stage depth");
  static_assert(!(RAGGED_K && F8) || (CG == 1 && (BN == 128 || BN == 256)), "e4m3 weight gradient: single CTA");
  constexpr int STAGES = Cfg::STAGES;
  constexpr int MMA_M = BM * CG;  // rows of one MMA (both CTAs of a pair)
  constexpr int TM = MMA_M * MH;  // rows of a tile
  constexpr int BNC = BN / CG;  // B columns held by one CTA

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;
  uint64_t* drain_bar = bars + 2 * STAGES + 4;
  uint64_t* ring_full = bars + 2 * STAGES + 5;
  uint64_t* ring_empty = bars + 2 * STAGES + 5 + kRing;
  uint64_t* patch_done = bars + 2 * STAGES + 5 + 2 * kRing;
  uint64_t* mbox_full = bars + 3 * STAGES + 5 + 2 * kRing;   // odd CTA: tile id posted by the leader
  uint64_t* mbox_empty = bars + 3 * STAGES + 5 + 3 * kRing;  // leader: the odd CTA took the id
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 5 + 4 * kRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* ring_ids = reinterpret_cast<volatile int*>(tmem_holder + 2);
  volatile int* mbox_ids = ring_ids + kRing;
  int* sched = reinterpret_cast<int*>(smem + STAGES * Cfg::STAGE_BYTES + Cfg::BAR_BYTES);
  uint8_t* out_stage = smem + STAGES * Cfg::STAGE_BYTES + Cfg::OUT_OFFSET;  // 1024-aligned
  SchedSmem ss{sched, sched + (kMaxGroups + 1), sched + 2 * (kMaxGroups + 1)};

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = (CG == 2) ? ptx::cluster_ctarank() : 0u;
  const bool leader = crank == 0;
  const int unit = (CG == 2) ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int num_units = (CG == 2) ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(ptx::smem_u32(&full_bar[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&empty_bar[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&patch_done[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(ptx::smem_u32(&tfull_bar[b]), 1);
      ptx::mbar_init(ptx::smem_u32(&tempty_bar[b]), kNumEpiWarps * CG);
    }
    ptx::mbar_init(ptx::smem_u32(drain_bar), 1);
    for (int j = 0; j < kRing; ++j) {
      ptx::mbar_init(ptx::smem_u32(&ring_full[j]), 1);
      ptx::mbar_init(ptx::smem_u32(&ring_empty[j]), 1 + kNumEpiWarps);
      ptx::mbar_init(ptx::smem_u32(&mbox_full[j]), 1);
      ptx::mbar_init(ptx::smem_u32(&mbox_empty[j]), 1);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      ptx::tmem_alloc_pair(ptx::smem_u32(tmem_holder), Cfg::TMEM_COLS);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(ptx::smem_u32(tmem_holder), Cfg::TMEM_COLS);
      ptx::tmem_relinquish();
    }
  }
  if (warp == 2) build_schedule<TM, RAGGED_K>(p, ss, lane);
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) ptx::cluster_sync();  // barriers of both CTAs initialised before any remote use
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total_tiles = ss.prefix[p.E];

  // Shared::cluster address of a barrier in the even CTA (identity for CG = 1).
  auto leader_addr = [&](const void* ptr) -> uint32_t {
    const uint32_t a = ptx::smem_u32(ptr);
    if constexpr (CG == 2) return ptx::mapa_shared(a, 0);
    return a;
  };
  // Does the odd CTA of a ragged-K pair hold the ones row of this tile?
  auto odd_has_ones = [&](const TileInfo& ti) -> bool {
    if constexpr (CG == 2 && RAGGED_K) {
      const int o = p.m - ti.m_blk * TM - BM;
      return p.bias_grad && o >= 0 && o < BM;
    }
    return false;
  };
  // Stages relayed through the odd CTA (CG = 2, ragged-K): those it must patch before the MMA.
  auto relayed = [&](const TileInfo& ti, int kb, bool odd_ones) -> bool {
    if constexpr (CG == 2 && RAGGED_K) {
      const int valid_k = min(KR, ti.k_end - (ti.k_start + kb * KR));
      return valid_k < KR || odd_ones;
    }
    return false;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      constexpr uint32_t kLoadBytes = Cfg::STAGE_BYTES;  // bytes landing in this CTA per stage
      uint32_t stage = 0, phase = 0;
      uint32_t issued_parity[STAGES];
      bool outstanding[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) { outstanding[s] = false; issued_parity[s] = 0; }
      bool ok = true;
      // The producer picks the tile sequence (static striding, or an atomic counter when the
      // launch has one) and hands every tile id to the MMA and epilogue warps through the ring.
      // A pair with a counter: the even CTA claims each tile and posts its id into the odd CTA's
      // mailbox (a remote store, then a release arrive on the odd CTA's barrier).
      const bool forwarded = (CG == 2) && (p.tile_counter != nullptr);
      int t = unit;
      uint32_t rslot = 0, rphase = 0;
      uint32_t mslot = 0, mphase = 0;
      while (ok && !p.stall_test) {
        if (!wait_bounded(ptx::smem_u32(&ring_empty[rslot]), rphase ^ 1, abort_flag)) { ok = false; break; }
        if (forwarded) {
          if (leader) {
            if (!wait_bounded<true>(ptx::smem_u32(&mbox_empty[mslot]), mphase ^ 1, abort_flag)) { ok = false; break; }
            ptx::st_cluster_u32(ptx::mapa_shared(ptx::smem_u32(const_cast<int*>(&mbox_ids[mslot])), 1),
                                static_cast<uint32_t>(t < total_tiles ? t : -1));
            ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(&mbox_full[mslot]), 1));
          } else {
            if (!wait_bounded<true>(ptx::smem_u32(&mbox_full[mslot]), mphase, abort_flag)) { ok = false; break; }
            t = mbox_ids[mslot];
            ptx::mbar_arrive_cluster(leader_addr(&mbox_empty[mslot]));
          }
          if (++mslot == kRing) { mslot = 0; mphase ^= 1; }
        }
        const int tt = (t >= 0 && t < total_tiles) ? t : -1;
        ring_ids[rslot] = tt;
        ptx::mbar_arrive(ptx::smem_u32(&ring_full[rslot]));
        if (++rslot == kRing) { rslot = 0; rphase ^= 1; }
        if (tt < 0) break;
        TileInfo ti;
        decode_tile<TM, RAGGED_K>(t, p, ss, ti);
        const bool odd_ones = odd_has_ones(ti);
        const int nb0 = ti.n_blk * BN + static_cast<int>(crank) * BNC;  // this CTA's first B column
        for (int kb = 0; kb < ti.nk; ++kb) {
          if (!wait_bounded(ptx::smem_u32(&empty_bar[stage]), phase ^ 1, abort_flag)) { ok = false; break; }
          const uint32_t own_full = ptx::smem_u32(&full_bar[stage]);
          uint32_t fb = own_full;
          if constexpr (CG == 2) {
            const bool relay = relayed(ti, kb, odd_ones);
            if (leader) {
              ptx::mbar_arrive_expect_tx(own_full, relay ? kLoadBytes : 2 * kLoadBytes);
            } else if (relay) {
              ptx::mbar_arrive_expect_tx(own_full, kLoadBytes);
            } else {
              fb = leader_addr(&full_bar[stage]);
            }
          } else {
            ptx::mbar_arrive_expect_tx(own_full, kLoadBytes);
          }
          const uint32_t sA = ptx::smem_u32(stage_base + stage * Cfg::STAGE_BYTES);
          const uint32_t sB = sA + Cfg::A_BYTES;
          auto load2 = [&](uint32_t dst, const CUtensorMap* tm, int x, int y) {
            if constexpr (CG == 2) ptx::tma_load_2d_pair(dst, tm, fb, x, y);
            else ptx::tma_load_2d(dst, tm, fb, x, y);
          };
          auto load3 = [&](uint32_t dst, const CUtensorMap* tm, int x, int y, int z) {
            if constexpr (CG == 2) ptx::tma_load_3d_pair(dst, tm, fb, x, y, z);
            else ptx::tma_load_3d(dst, tm, fb, x, y, z);
          };
          if constexpr (!RAGGED_K) {
            constexpr int BKE = F8 ? 128 : BK;  // K elements per stage (128 bytes of a row)
            load2(sA, &tmA, kb * BKE, ti.row0 + static_cast<int>(crank) * BM);
            if constexpr (B_MN) {
#pragma unroll
              for (int c = 0; c < Cfg::B_CHUNKS; ++c) load3(sB + c * 8192, &tmB, nb0 + 64 * c, kb * BK, ti.e);
            } else {
              load3(sB, &tmB, kb * BKE, nb0, ti.e);
            }
          } else if constexpr (F8) {
            // e4m3 token rows: one {128 features, 128 rows} box per 128 columns of A and of B
            const int kr = ti.k_start + kb * KR;
            const int m0 = ti.m_blk * TM;
#pragma unroll
            for (int h = 0; h < MH; ++h) load2(sA + h * 16384, &tmA, m0 + h * BM, kr);
#pragma unroll
            for (int c = 0; c < BNC / 128; ++c) load2(sB + c * 16384, &tmB, nb0 + 128 * c, kr);
          } else {
            const int kr = ti.k_start + kb * BK;
            const int m0 = ti.m_blk * TM + static_cast<int>(crank) * BM;
            if (p.a_chunked) {
#pragma unroll
              for (int h = 0; h < MH; ++h) load3(sA + h * (BM / 64) * 8192, &tmA, 0, kr, (m0 + h * BM) >> 6);
            } else {
#pragma unroll
              for (int c = 0; c < MH * BM / 64; ++c) load2(sA + c * 8192, &tmA, m0 + 64 * c, kr);
            }
            if (p.b_chunked) {
              load3(sB, &tmB, 0, kr, nb0 >> 6);
            } else {
#pragma unroll
              for (int c = 0; c < Cfg::B_CHUNKS; ++c) load2(sB + c * 8192, &tmB, nb0 + 64 * c, kr);
            }
          }
          outstanding[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        // (claiming the next id at the start of the tile instead was measured: each CTA then holds two
        // tiles, the window of tiles in work widens, DRAM reads of the weight gradients grow by 10%
        // and they run 10-15% slower)
        if (p.tile_counter == nullptr) t += num_units;
        else if (leader) t = num_units + atomicAdd(p.tile_counter, 1);  // the odd CTA reads its mailbox
      }
      if (!ok && CG == 1) {
        // Stopped early: let the copies already in flight land before the CTA exits.  (A pair waits
        // for its copies at the final cluster barrier.)
        for (int s = 0; s < STAGES; ++s)
          if (outstanding[s]) wait_bounded(ptx::smem_u32(&full_bar[s]), issued_parity[s], abort_flag, kDrainLimitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (even CTA) /
    //                                                              ragged-K stage patcher (odd CTA)
    constexpr uint32_t idesc =
        F8 ? ptx::make_idesc_e4m3(MMA_M, BN, A_MN, B_MN) : ptx::make_idesc_bf16(MMA_M, BN, A_MN, B_MN);
    // MN-major operands: chunks of 128 bytes along M / N are 8 KB apart (bf16: 64 K rows per chunk)
    // or 16 KB apart (e4m3 weight gradient: 128 K rows); one instruction advances 16 (bf16) or 32
    // (e4m3) K rows of 128 bytes.  K-major: 16-byte units, 32 bytes of K per instruction.
    constexpr uint32_t mn_lbo = (RAGGED_K && F8) ? 16384u : 8192u;
    constexpr uint32_t mn_kstep = ((F8 ? 32u : 16u) * 128u) >> 4;
    constexpr uint32_t a_lbo = A_MN ? mn_lbo : 16u;
    constexpr uint32_t b_lbo = B_MN ? mn_lbo : 16u;
    constexpr uint32_t a_kstep = A_MN ? mn_kstep : (16u * 2u) >> 4;
    constexpr uint32_t b_kstep = B_MN ? mn_kstep : (16u * 2u) >> 4;
    const bool issuer = (CG == 1) || leader;
    uint32_t stage = 0, phase = 0;
    uint32_t relay_bits = 0;  // per-stage phase of patch_done (even CTA) / own full (odd CTA) on relayed stages
    bool ok = true;
    bool issued_any = false;
    uint32_t rslot = 0, rphase = 0;
    for (int it = 0; ok; ++it) {
      ok = __all_sync(0xffffffffu, wait_bounded(ptx::smem_u32(&ring_full[rslot]), rphase, abort_flag));
      if (!ok) break;
      const int t = ring_ids[rslot];
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&ring_empty[rslot]));
      if (++rslot == kRing) { rslot = 0; rphase ^= 1; }
      if (t < 0) break;
      if (!issuer && !RAGGED_K) continue;  // the odd CTA of a ragged-M pair has nothing to do here
      TileInfo ti;
      decode_tile<TM, RAGGED_K>(t, p, ss, ti);
      const bool odd_ones = odd_has_ones(ti);
      // two TMEM accumulators in turn; a 256-row tile (MH = 2) fills both, one tile at a time
      const int buf = MH == 2 ? 0 : (it & 1);
      const uint32_t tph = MH == 2 ? (it & 1) : ((it >> 1) & 1);
      // MH = 2: the second 128-row half is multiplied only if it holds rows of dW or the ones row
      const bool hi_half = MH == 2 && ti.m_blk * TM + BM < p.m + (p.bias_grad ? 1 : 0);
      if (issuer) {
        ok = __all_sync(0xffffffffu,
                        wait_bounded<CG == 2>(ptx::smem_u32(&tempty_bar[buf]), tph ^ 1, abort_flag));
        if (!ok) break;
        ptx::tc_fence_after();
      }
      const uint32_t d_tmem = tmem_base + buf * BN;
      int ones_local = -1;  // this CTA's A row that carries the bias-gradient ones
      if constexpr (RAGGED_K) {
        if (p.bias_grad) {
          const int o = p.m - ti.m_blk * TM - static_cast<int>(crank) * BM;
          if (o >= 0 && o < BM * MH) ones_local = o;
        }
      }
      for (int kb = 0; kb < ti.nk; ++kb) {
        uint8_t* sA_ptr = stage_base + stage * Cfg::STAGE_BYTES;
        const bool relay = relayed(ti, kb, odd_ones);
        if (!issuer) {
          // odd CTA of a ragged-K pair: patch the relayed stages, then release them to the leader
          if (relay) {
            const uint32_t par = (relay_bits >> stage) & 1u;
            relay_bits ^= 1u << stage;
            ok = __all_sync(0xffffffffu, wait_bounded(ptx::smem_u32(&full_bar[stage]), par, abort_flag));
            if (!ok) break;
            const int valid_k = min(KR, ti.k_end - (ti.k_start + kb * KR));
            patch_ragged_k_stage<BM / 64, Cfg::B_CHUNKS>(sA_ptr, valid_k, KR, ones_local, lane);
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive_cluster(leader_addr(&patch_done[stage]));
          }
          __syncwarp();
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
          continue;
        }
        ok = __all_sync(0xffffffffu, wait_bounded<CG == 2>(ptx::smem_u32(&full_bar[stage]), phase, abort_flag));
        if (!ok) break;
        if (relay) {
          const uint32_t par = (relay_bits >> stage) & 1u;
          relay_bits ^= 1u << stage;
          ok = __all_sync(0xffffffffu, wait_bounded<true>(ptx::smem_u32(&patch_done[stage]), par, abort_flag));
          if (!ok) break;
        }
        ptx::tc_fence_after();
        // MMAs of this stage: all of them, except in the short-group form (OB = 4), whose tail
        // stage stops at the instruction holding the group's last token row, so that only the
        // rows up to that instruction's end need clearing.
        int n_mma = kMmaPerStage;
        if constexpr (RAGGED_K) {
          const int valid_k = min(KR, ti.k_end - (ti.k_start + kb * KR));
          int end_k = KR;
          if constexpr (OB == 4) {
            n_mma = (valid_k + KMMA - 1) / KMMA;
            end_k = n_mma * KMMA;
          }
          if (valid_k < end_k || ones_local >= 0) {
            if constexpr (F8) patch_ragged_k_stage_f8<MH + BNC / 128>(sA_ptr, valid_k, end_k, ones_local, lane);
            else patch_ragged_k_stage<MH * BM / 64, Cfg::B_CHUNKS>(sA_ptr, valid_k, end_k, ones_local, lane);
            ptx::fence_proxy_async_smem();
          }
          __syncwarp();
        }
        if (lane == 0) {
          const uint32_t sA = ptx::smem_u32(sA_ptr);
          const uint32_t sB = sA + Cfg::A_BYTES;
          const uint64_t adesc = ptx::make_smem_desc_sw128(sA, a_lbo, 1024);
          const uint64_t bdesc = ptx::make_smem_desc_sw128(sB, b_lbo, 1024);
#pragma unroll
          for (int kk = 0; kk < kMmaPerStage; ++kk) {
            if (OB == 4 && kk >= n_mma) break;
            // one instruction consumes 32 bytes of every K-major row: K = 16 bf16 or K = 32 e4m3
            if constexpr (CG == 2 && F8) {
              ptx::umma_f8_pair(d_tmem, adesc + kk * a_kstep, bdesc + kk * b_kstep, idesc, (kb | kk) != 0 ? 1u : 0u);
            } else if constexpr (CG == 2) {
              ptx::umma_bf16_pair(d_tmem, adesc + kk * a_kstep, bdesc + kk * b_kstep, idesc, (kb | kk) != 0 ? 1u : 0u);
            } else if constexpr (F8) {
              ptx::umma_f8(d_tmem, adesc + kk * a_kstep, bdesc + kk * b_kstep, idesc, (kb | kk) != 0 ? 1u : 0u);
              if (MH == 2 && hi_half)  // rows 128..255: the second 16 KB A chunk, BN TMEM columns on
                ptx::umma_f8(d_tmem + BN, ptx::make_smem_desc_sw128(sA + 16384, a_lbo, 1024) + kk * a_kstep,
                             bdesc + kk * b_kstep, idesc, (kb | kk) != 0 ? 1u : 0u);
            } else {
              ptx::umma_bf16(d_tmem, adesc + kk * a_kstep, bdesc + kk * b_kstep, idesc, (kb | kk) != 0 ? 1u : 0u);
              if (MH == 2 && hi_half)  // rows 128..255: A half two chunks on, accumulator BN columns on
                ptx::umma_bf16(d_tmem + BN, ptx::make_smem_desc_sw128(sA + (BM / 64) * 8192, a_lbo, 1024) + kk * a_kstep,
                               bdesc + kk * b_kstep, idesc, (kb | kk) != 0 ? 1u : 0u);
            }
          }
          if constexpr (CG == 2) ptx::umma_commit_pair(ptx::smem_u32(&empty_bar[stage]), 0x3);
          else ptx::umma_commit(ptx::smem_u32(&empty_bar[stage]));
          issued_any = true;
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (issuer && lane == 0) {
        if (ti.nk > 0) {
          if constexpr (CG == 2) ptx::umma_commit_pair(ptx::smem_u32(&tfull_bar[buf]), 0x3);
          else ptx::umma_commit(ptx::smem_u32(&tfull_bar[buf]));
        } else {
          // empty group (ragged-K): nothing to multiply, the epilogues write zeros
          ptx::mbar_arrive(ptx::smem_u32(&tfull_bar[buf]));
          if constexpr (CG == 2) ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(&tfull_bar[buf]), 1));
        }
      }
      __syncwarp();
    }
    if (!ok && issuer && lane == 0 && issued_any) {
      // Stopped early: wait for the UMMAs already issued before TMEM is released.
      if constexpr (CG == 2) ptx::umma_commit_pair(ptx::smem_u32(drain_bar), 0x1);
      else ptx::umma_commit(ptx::smem_u32(drain_bar));
      wait_bounded(ptx::smem_u32(drain_bar), 0, abort_flag, kDrainLimitNs);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue warps
    // Two warpgroups; each reads all 128 TMEM lanes (warp w owns lanes 32*(w%4)..+31, i.e. 32
    // tile rows) for its half of the tile's columns.
    const int q = warp & 3;
    const int wg = (warp - 2) >> 2;
    constexpr int kChunks = BN / 32 / kEpiGroups;
    const int c_begin = wg * kChunks;
    const int r = q * 32 + lane;
    const uint32_t tempty_leader[2] = {leader_addr(&tempty_bar[0]), leader_addr(&tempty_bar[1])};
    uint32_t rslot = 0, rphase = 0;
    for (int it = 0;; ++it) {
      if (!__all_sync(0xffffffffu, wait_bounded(ptx::smem_u32(&ring_full[rslot]), rphase, abort_flag))) break;
      const int t = ring_ids[rslot];
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&ring_empty[rslot]));
      if (++rslot == kRing) { rslot = 0; rphase ^= 1; }
      if (t < 0) break;
      TileInfo ti;
      decode_tile<TM, RAGGED_K>(t, p, ss, ti);
      const int buf = MH == 2 ? 0 : (it & 1);
      const uint32_t tph = MH == 2 ? (it & 1) : ((it >> 1) & 1);
      const int n0 = ti.n_blk * BN;

      if constexpr (!RAGGED_K) {
        const int crow0 = ti.row0 + static_cast<int>(crank) * BM;  // first row of this CTA's half
        const int grow = crow0 + r;
        const bool warp_active = crow0 + q * 32 < ti.row_end;
        const bool valid = grow < ti.row_end;
        // SwiGLU backward: the aux words do not depend on the accumulator, so the first chunk's
        // loads are issued before waiting for the mainloop.
        uint4 aw[8];
        if constexpr (EPI == MGF_EPI_SWIGLU_BWD) {
          load_aux_chunk(p.aux + (int64_t)grow * p.ld_aux, n0 + c_begin * 32, p.n, valid, p.aux_v8, aw);
        }
        if (!__all_sync(0xffffffffu, wait_bounded(ptx::smem_u32(&tfull_bar[buf]), tph, abort_flag))) break;
        ptx::tc_fence_after();
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
        // output row of D: row `grow` of d, or (scatter mode) the address d_rows[grow] -- possibly in
        // another GPU's memory -- with 0 meaning "no destination"; 32-byte stores only where aligned
        __nv_bfloat16* drow = p.d + (int64_t)grow * p.ldd;
        bool dv8 = p.d_v8;
        if (p.d_rows != nullptr) {
          drow = valid ? reinterpret_cast<__nv_bfloat16*>(__ldg(p.d_rows + grow)) : nullptr;
          dv8 = p.d_v8 && (reinterpret_cast<uintptr_t>(drow) & 31u) == 0;
        }
        if (warp_active) {
#pragma unroll 1
          for (int c = c_begin; c < c_begin + kChunks; ++c) {
            const int col0 = n0 + c * 32;
            if (col0 >= p.n) break;
            uint32_t v[32];
            ptx::tmem_ld_32x32b_x32(tbase + c * 32, v);
            ptx::tmem_ld_wait();
            if (!valid) continue;
            if constexpr (EPI == MGF_EPI_BIAS || EPI == MGF_EPI_SWIGLU) {
              float f[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
              if constexpr (F8) {
                // dequantise: row scale of A times the group's column scales of B (fp32), then bias
                const float sa = __ldg(p.scale_a + grow);
                const float4* sp = reinterpret_cast<const float4*>(p.scale_b + (int64_t)ti.e * p.scale_b_stride + col0);
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                  if (col0 + 4 * g < p.n) {
                    const float4 sb = __ldg(sp + g);
                    f[4 * g] *= sa * sb.x;
                    f[4 * g + 1] *= sa * sb.y;
                    f[4 * g + 2] *= sa * sb.z;
                    f[4 * g + 3] *= sa * sb.w;
                  }
                }
              }
              if (EPI == MGF_EPI_BIAS && p.bias_per_row) {
                const float bv = __bfloat162float(p.bias[(int64_t)ti.e * p.bias_stride + (grow - ti.row0 + ti.m_blk * TM)]);
#pragma unroll
                for (int j = 0; j < 32; ++j) f[j] += bv;
              } else if (p.bias != nullptr) {
                const uint4* bp = reinterpret_cast<const uint4*>(p.bias + (int64_t)ti.e * p.bias_stride + col0);
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                  if (col0 + 8 * g < p.n) {
                    const uint4 bw = __ldg(bp + g);
                    const uint32_t w[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                      f[8 * g + 2 * h] += bf16_lo(w[h]);
                      f[8 * g + 2 * h + 1] += bf16_hi(w[h]);
                    }
                  }
                }
              }
              uint32_t packed[16];
#pragma unroll
              for (int h = 0; h < 16; ++h) packed[h] = pack_bf16x2(f[2 * h], f[2 * h + 1]);
              if (EPI == MGF_EPI_BIAS || p.store_aux) {
                uint4 u[4];
#pragma unroll
                for (int g = 0; g < 4; ++g) u[g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
                if (drow != nullptr) store_units<4>(drow + col0, u, (p.n - col0) >> 3, dv8);
              }
              if constexpr (EPI == MGF_EPI_SWIGLU) {
                uint32_t so[8];
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                  const float a0 = swiglu_fwd(bf16_lo(packed[2 * h]), bf16_hi(packed[2 * h]), p.alpha, p.limit);
                  const float a1 =
                      swiglu_fwd(bf16_lo(packed[2 * h + 1]), bf16_hi(packed[2 * h + 1]), p.alpha, p.limit);
                  so[h] = pack_bf16x2(a0, a1);
                }
                const uint4 u[2] = {make_uint4(so[0], so[1], so[2], so[3]), make_uint4(so[4], so[5], so[6], so[7])};
                store_units<2>(p.d2 + (int64_t)grow * p.ldd2 + (col0 >> 1), u, (p.n - col0) >> 4, p.d2_v8);
              }
            } else if constexpr (EPI == MGF_EPI_SWIGLU_BWD) {
              if constexpr (F8) {
                // dequantise the accumulator (grad_s) before the SwiGLU backward: scale_a of the row
                // times the group's column scales of B
                const float sa = __ldg(p.scale_a + grow);
                const float4* sp = reinterpret_cast<const float4*>(p.scale_b + (int64_t)ti.e * p.scale_b_stride + col0);
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                  if (col0 + 4 * g < p.n) {
                    const float4 sb = __ldg(sp + g);
                    v[4 * g] = __float_as_uint(__uint_as_float(v[4 * g]) * (sa * sb.x));
                    v[4 * g + 1] = __float_as_uint(__uint_as_float(v[4 * g + 1]) * (sa * sb.y));
                    v[4 * g + 2] = __float_as_uint(__uint_as_float(v[4 * g + 2]) * (sa * sb.z));
                    v[4 * g + 3] = __float_as_uint(__uint_as_float(v[4 * g + 3]) * (sa * sb.w));
                  }
                }
              }
              uint4 cur[8];
#pragma unroll
              for (int g = 0; g < 8; ++g) cur[g] = aw[g];
              // prefetch the next chunk's aux words while this chunk is computed and stored
              const int ncol0 = col0 + 32;
              if (c + 1 < c_begin + kChunks && ncol0 < p.n) load_aux_chunk(p.aux + (int64_t)grow * p.ld_aux, ncol0, p.n, true, p.aux_v8, aw);
              // two 16-byte units (8 GEMM columns) at a time: computed, then stored
              uint4* gp = reinterpret_cast<uint4*>(p.d + (int64_t)grow * p.ldd + 2 * col0);
              const int nvalid = (p.n - col0) >> 2;
#pragma unroll
              for (int g = 0; g < 8; g += 2) {
                if (g < nvalid) {
                  uint4 o[2];
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    o[h].x = swiglu_bwd_word(__uint_as_float(v[4 * (g + h) + 0]), cur[g + h].x, p.alpha, p.limit);
                    o[h].y = swiglu_bwd_word(__uint_as_float(v[4 * (g + h) + 1]), cur[g + h].y, p.alpha, p.limit);
                    o[h].z = swiglu_bwd_word(__uint_as_float(v[4 * (g + h) + 2]), cur[g + h].z, p.alpha, p.limit);
                    o[h].w = swiglu_bwd_word(__uint_as_float(v[4 * (g + h) + 3]), cur[g + h].w, p.alpha, p.limit);
                  }
                  // n % 8 == 0 and g even: unit g valid implies unit g + 1 valid
                  if (p.d_v8) ptx::st_v8(gp + g, o[0], o[1]);
                  else {
                    gp[g] = o[0];
                    gp[g + 1] = o[1];
                  }
                }
              }
            }
          }
        }
      } else {
        if (!__all_sync(0xffffffffu, wait_bounded(ptx::smem_u32(&tfull_bar[buf]), tph, abort_flag))) break;
        ptx::tc_fence_after();
        // one pass per 128-row accumulator (MH = 2: rows 128..255 sit BN TMEM columns on)
        for (int h = 0; h < MH; ++h) {
          const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + (buf + h) * BN;
          // ragged-K weight gradient: rows are output features m0 + r.  dW [E, m, n] is dense, so each
          // warp stages its 32 rows x 32 columns in its own shared-memory slice and lane 0 stores it
          // with one TMA tile store (clipped at m and n by the tensor map); no cross-warp sync.
          const int m0 = ti.m_blk * TM + static_cast<int>(crank) * BM + h * BM;
          if (h > 0 && m0 >= p.m + (p.bias_grad ? 1 : 0)) break;  // MH = 2: an empty second half
          int ones_r = -1;
          if (p.bias_grad && p.m - m0 >= 0 && p.m - m0 < BM) ones_r = p.m - m0;
          const bool row_bias = (r == ones_r);
          const bool warp_rows = m0 + q * 32 < p.m;  // this warp holds rows of dW
          const bool warp_active = warp_rows || (ones_r >= q * 32 && ones_r < q * 32 + 32);
          uint8_t* const slices = out_stage + (warp - 2) * OB * (32 * 64);
          if (OB == 4 && warp_active) {
            // wide form: the TMEM loads of two chunks are issued before one wait; the chunks go into
            // one slab {64 columns, 32 rows, 64-column chunks} (128-byte swizzle: chunk j is 64-column
            // chunk j / 2, 16-byte units 4 * (j % 2) + g, each at unit ^ (row & 7) within its row's
            // 128 bytes) and out with one TMA store
            if (warp_rows) {
              if (lane == 0) ptx::bulk_wait_read_all();  // the previous tile's store has read the slab
              __syncwarp();
            }
  #pragma unroll
            for (int jb = 0; jb < kChunks; jb += 2) {
              if (n0 + (c_begin + jb) * 32 >= p.n) break;
              uint32_t v[2][32];
              if (ti.nk > 0) {
  #pragma unroll
                for (int u = 0; u < 2; ++u)
                  if (jb + u < kChunks && n0 + (c_begin + jb + u) * 32 < p.n)
                    ptx::tmem_ld_32x32b_x32(tbase + (c_begin + jb + u) * 32, v[u]);
                ptx::tmem_ld_wait();
              }
  #pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int j = jb + u;
                const int col0 = n0 + (c_begin + j) * 32;
                if (j >= kChunks || col0 >= p.n) break;
                uint32_t packed[16];
  #pragma unroll
                for (int h = 0; h < 16; ++h)
                  packed[h] = ti.nk > 0 ? pack_bf16x2(__uint_as_float(v[u][2 * h]), __uint_as_float(v[u][2 * h + 1])) : 0u;
                if (warp_rows) {
                  uint8_t* row_base = slices + (j >> 1) * 4096 + lane * 128;
  #pragma unroll
                  for (int g = 0; g < 4; ++g)
                    *reinterpret_cast<uint4*>(row_base + (((4 * (j & 1) + g) ^ (lane & 7)) << 4)) =
                        make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
                }
                if (row_bias) {
                  uint4* dp = reinterpret_cast<uint4*>(p.d2 + (int64_t)ti.e * p.ldd2 + col0);
  #pragma unroll
                  for (int g = 0; g < 4; ++g)
                    if (col0 + 8 * g < p.n)
                      dp[g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
                }
              }
            }
            // one store of the warp's chunks (clipped at m, and at the last 64-column chunk of n)
            const int col_first = n0 + c_begin * 32;
            if (warp_rows && col_first < p.n) {
              ptx::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                ptx::tma_store_4d(&tmD, ptx::smem_u32(slices), 0, m0 + q * 32, col_first / 64, ti.e);
                ptx::bulk_commit();
              }
            }
          } else if (warp_active) {
  #pragma unroll 1
            for (int c = c_begin; c < c_begin + kChunks; ++c) {
              const int col0 = n0 + c * 32;
              if (col0 >= p.n) break;
              uint32_t packed[16];
              if (ti.nk > 0) {
                uint32_t v[32];
                ptx::tmem_ld_32x32b_x32(tbase + c * 32, v);
                ptx::tmem_ld_wait();
                if constexpr (F8) {
                  // per-feature scales: scale_a of this row's feature (1 for the bias-gradient row),
                  // scale_b of each column
                  const float rs = row_bias ? 1.0f : (m0 + r < p.m ? __ldg(p.scale_a + m0 + r) : 0.0f);
                  const float4* sp = reinterpret_cast<const float4*>(p.scale_b + col0);
  #pragma unroll
                  for (int g = 0; g < 8; ++g) {
                    const float4 sb = (col0 + 4 * g < p.n) ? __ldg(sp + g) : make_float4(0.f, 0.f, 0.f, 0.f);
                    v[4 * g] = __float_as_uint(__uint_as_float(v[4 * g]) * (rs * sb.x));
                    v[4 * g + 1] = __float_as_uint(__uint_as_float(v[4 * g + 1]) * (rs * sb.y));
                    v[4 * g + 2] = __float_as_uint(__uint_as_float(v[4 * g + 2]) * (rs * sb.z));
                    v[4 * g + 3] = __float_as_uint(__uint_as_float(v[4 * g + 3]) * (rs * sb.w));
                  }
                }
  #pragma unroll
                for (int h = 0; h < 16; ++h) packed[h] = pack_bf16x2(__uint_as_float(v[2 * h]), __uint_as_float(v[2 * h + 1]));
              } else {
  #pragma unroll
                for (int h = 0; h < 16; ++h) packed[h] = 0u;
              }
              if (warp_rows) {
                const uint32_t slice_u32 = ptx::smem_u32(slices);
                if (lane == 0) ptx::bulk_wait_read_all();  // the slice's previous store has read it
                __syncwarp();
                // 64-byte swizzle (matches the tensor map): 16-byte unit g of row `lane` at g ^ ((lane >> 1) & 3)
  #pragma unroll
                for (int g = 0; g < 4; ++g)
                  *reinterpret_cast<uint4*>(slices + lane * 64 + ((g ^ ((lane >> 1) & 3)) << 4)) =
                      make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
                ptx::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                  ptx::tma_store_3d(&tmD, slice_u32, col0, m0 + q * 32, ti.e);
                  ptx::bulk_commit();
                }
              }
              if (row_bias) {
                uint4* dp = reinterpret_cast<uint4*>(p.d2 + (int64_t)ti.e * p.ldd2 + col0);
  #pragma unroll
                for (int g = 0; g < 4; ++g)
                  if (col0 + 8 * g < p.n)
                    dp[g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
              }
            }
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2) ptx::mbar_arrive_cluster(tempty_leader[buf]);
        else ptx::mbar_arrive(ptx::smem_u32(&tempty_bar[buf]));
      }
    }
  }

  if constexpr (RAGGED_K) {
    if (warp >= 2 && lane == 0) ptx::bulk_wait_all();  // this warp's tile stores are complete
  }
  ptx::tc_fence_before();
  __syncthreads();
  // A pair leaves together: the peer may still signal this CTA's barriers until both are done.
  if constexpr (CG == 2) ptx::cluster_sync();
  if (warp == 1) {
    ptx::tc_fence_after();
    if constexpr (CG == 2) ptx::tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else ptx::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ============================================================================ host side

static thread_local char g_last_error[256] = "";

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

static bool encode_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                        const uint32_t* box, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B,
                        CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return false;
  if (rank < 1 || rank > 4) return false;
  cuuint64_t d[4];
  cuuint64_t s[3];
  cuuint32_t b[4];
  cuuint32_t e[4] = {1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
  const CUresult r = fn(m, dtype, rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(g_last_error, sizeof(g_last_error), "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
    return false;
  }
  return true;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
};

static DeviceInfo device_info(int dev) {
  static DeviceInfo cache[64];
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (dev < 0 || dev >= 64) return DeviceInfo{};
  if (cache[dev].sms == 0) {
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
  }
  return cache[dev];
}

static void record_error(const char* what, cudaError_t e) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, cudaGetErrorString(e));
}

static bool debug_sync() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("MGF_DEBUG_SYNC");
    v = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

template <int BN, int EPI, bool A_MN, bool B_MN, int CG, bool F8 = false, int OB = 1, int MH = 1>
static int launch_inst(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tD, const Params& p,
                       int grid_in, cudaStream_t st) {
  int grid = grid_in;
  auto kern = grouped_gemm_kernel<BN, EPI, A_MN, B_MN, CG, F8, OB, MH>;
  constexpr int smem = TileCfg<BN, CG, B_MN, OB, MH>::SMEM_BYTES;
  static std::mutex mu;
  static bool attr_done[64] = {};
  static int max_clusters[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MGF_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    std::lock_guard<std::mutex> g(mu);
    if (!attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) {
        record_error("cudaFuncSetAttribute", e);
        return MGF_ERR_CUDA;
      }
      if (CG == 2) {
        // Persistent pairs: never launch more clusters than can be resident at once, or the extra
        // ones would start only after others finished their whole share of tiles.
        cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = 1 << 30;
        cudaGetLastError();
        max_clusters[dev] = n;
      }
      attr_done[dev] = true;
    }
  }
  if (CG == 2 && grid / 2 > max_clusters[dev]) grid = 2 * max_clusters[dev];
  // A non-sticky error left by an unrelated runtime call would otherwise be reported as ours.
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess && debug_sync()) fprintf(stderr, "[mgf] cleared pre-existing error: %s\n", cudaGetErrorString(e));
  if constexpr (CG == 1) {
    kern<<<grid, kThreads, smem, st>>>(tA, tB, tD, p);
    e = cudaGetLastError();
  } else {
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    e = cudaLaunchKernelEx(&cfg, kern, tA, tB, tD, p);
  }
  if (e != cudaSuccess) {
    record_error("kernel launch", e);
    return MGF_ERR_CUDA;
  }
  if (debug_sync()) {
    e = cudaStreamSynchronize(st);
    fprintf(stderr, "[mgf] BN=%d CG=%d epi=%d a_mn=%d b_mn=%d grid=%d E=%d rows=%lld m=%d n=%d k=%d -> %s\n", BN, CG,
            EPI, int(A_MN), int(B_MN), grid, p.E, (long long)p.total_rows, p.m, p.n, p.k, cudaGetErrorString(e));
    if (e != cudaSuccess) {
      record_error("kernel execution", e);
      return MGF_ERR_CUDA;
    }
  }
  return MGF_OK;
}

template <int BN, int CG>
static int dispatch_epi(int epi, bool b_mn, bool f8, const CUtensorMap& tA, const CUtensorMap& tB,
                        const CUtensorMap& tD, const Params& p, int grid, cudaStream_t st) {
  if (f8) {  // e4m3: ragged-M epilogues with both operands K-major; the ragged-K weight gradient
    if (epi == MGF_EPI_WGRAD) {
      if constexpr (CG == 1 && BN == 256)
        if (p.m256) return launch_inst<256, MGF_EPI_WGRAD, true, true, 1, true, 1, 2>(tA, tB, tD, p, grid, st);
      if constexpr (CG == 1 && (BN == 128 || BN == 256))
        return launch_inst<BN, MGF_EPI_WGRAD, true, true, 1, true>(tA, tB, tD, p, grid, st);
      return MGF_ERR_INVALID_ARGUMENT;
    }
    if (b_mn) return MGF_ERR_INVALID_ARGUMENT;
    if (epi == MGF_EPI_BIAS) return launch_inst<BN, MGF_EPI_BIAS, false, false, CG, true>(tA, tB, tD, p, grid, st);
    if (epi == MGF_EPI_SWIGLU) return launch_inst<BN, MGF_EPI_SWIGLU, false, false, CG, true>(tA, tB, tD, p, grid, st);
    if (epi == MGF_EPI_SWIGLU_BWD)
      return launch_inst<BN, MGF_EPI_SWIGLU_BWD, false, false, CG, true>(tA, tB, tD, p, grid, st);
    return MGF_ERR_INVALID_ARGUMENT;
  }
  switch (epi) {
    case MGF_EPI_BIAS:
      return b_mn ? launch_inst<BN, MGF_EPI_BIAS, false, true, CG>(tA, tB, tD, p, grid, st)
                  : launch_inst<BN, MGF_EPI_BIAS, false, false, CG>(tA, tB, tD, p, grid, st);
    case MGF_EPI_SWIGLU:
      return b_mn ? launch_inst<BN, MGF_EPI_SWIGLU, false, true, CG>(tA, tB, tD, p, grid, st)
                  : launch_inst<BN, MGF_EPI_SWIGLU, false, false, CG>(tA, tB, tD, p, grid, st);
    case MGF_EPI_SWIGLU_BWD:
      return b_mn ? launch_inst<BN, MGF_EPI_SWIGLU_BWD, false, true, CG>(tA, tB, tD, p, grid, st)
                  : launch_inst<BN, MGF_EPI_SWIGLU_BWD, false, false, CG>(tA, tB, tD, p, grid, st);
    case MGF_EPI_WGRAD:
      if constexpr (CG == 1 && BN != 192)
        if (p.small_k) return launch_inst<BN, MGF_EPI_WGRAD, true, true, 1, false, 4>(tA, tB, tD, p, grid, st);
      if constexpr (CG == 1 && BN == 256)
        if (p.m256) return launch_inst<256, MGF_EPI_WGRAD, true, true, 1, false, 1, 2>(tA, tB, tD, p, grid, st);
      return launch_inst<BN, MGF_EPI_WGRAD, true, true, CG>(tA, tB, tD, p, grid, st);
    default:
      return MGF_ERR_INVALID_ARGUMENT;
  }
}

// CTA pair (cta_group::2, 256-row tiles) or single CTA (128-row tiles).  Pairs halve the B bytes
// each SM streams per FLOP; their 256-row tiles waste more rows at group ends, so small groups stay
// on single CTAs.  MGF_CTA_GROUP=1|2 forces a choice (the tests exercise both).
constexpr int64_t kSmallKTokens = 256;  // average tokens per group at or below which small_k applies

static int pick_cta_group(bool ragged_k, int64_t total_rows, int num_groups, int64_t m) {
  const char* env = getenv("MGF_CTA_GROUP");
  if (env != nullptr && (env[0] == '1' || env[0] == '2')) return env[0] - '0';
  (void)m;
  if (!ragged_k) return (total_rows / num_groups >= 512) ? 2 : 1;
  // Ragged-K pairs measured slower than single CTAs with the dynamic tile order (B200, cfg3 shapes:
  // 2.5 vs 2.07 ms and 4.8 vs 4.06 ms): m = 2880 wastes 6.7% of a 256-row tile and pairs must use
  // static striding.  MGF_CTA_GROUP=2 still selects them.
  return 1;
}

// N tile: 256 unless it pads n by more than 1/8, else the candidate with the least padding.
// Measured on B200 at the GPT-OSS shapes: 256-column tiles beat 192-column ones on every launch of
// the step (fwd+bwd 14.4 vs 16.2 ms) even where 256 pads n = 2880 to 3072 -- per FLOP they read
// fewer A bytes from shared memory and issue fewer, larger UMMAs.  MGF_BN forces a choice.
static int pick_bn(int64_t n) {
  const char* env = getenv("MGF_BN");
  if (env != nullptr) {
    const int v = atoi(env);
    if (v == 128 || v == 192 || v == 256) return v;
  }
  if ((n + 255) / 256 * 256 - n <= n / 8) return 256;
  const int cands[2] = {192, 128};
  int best = 192;
  int64_t best_pad = -1;
  for (int c : cands) {
    const int64_t pad = (n + c - 1) / c * c - n;
    if (best_pad < 0 || pad < best_pad) {
      best = c;
      best_pad = pad;
    }
  }
  return best;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace mgf

using namespace mgf;

extern "C" int mgf_version(void) { return 101; }

extern "C" size_t mgf_gemm_desc_size(void) { return sizeof(mgf_gemm_desc); }

extern "C" const char* mgf_last_error_detail(void) { return g_last_error; }

extern "C" const char* mgf_status_string(int status) {
  switch (status) {
    case MGF_OK: return "ok";
    case MGF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MGF_ERR_UNSUPPORTED_LAYOUT: return "unsupported layout";
    case MGF_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case MGF_ERR_TOO_MANY_GROUPS: return "number of groups outside 1..1024";
    case MGF_ERR_CUDA: return "CUDA runtime error";
    case MGF_ERR_NO_DEVICE_SUPPORT: return "device is not sm_100 (B200)";
    default: return "unknown status";
  }
}

namespace mgf {
// Device address of g_status on the current device, for the kernels of the other translation units
// (the expert-parallel row movement) that report into the same word.
unsigned int* status_word_address() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
  return static_cast<unsigned int*>(p);
}
}  // namespace mgf

extern "C" int mgf_device_status(int device, uint32_t* status_out, int clear) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return MGF_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return MGF_ERR_CUDA;
  int rc = MGF_OK;
  unsigned int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpyFromSymbol(&v, g_status, sizeof(v)) != cudaSuccess) {
    rc = MGF_ERR_CUDA;
  } else {
    if (status_out) *status_out = v;
    if (clear) {
      const unsigned int zero = 0;
      if (cudaMemcpyToSymbol(g_status, &zero, sizeof(zero)) != cudaSuccess) rc = MGF_ERR_CUDA;
    }
  }
  cudaSetDevice(prev);
  return rc;
}

extern "C" int mgf_grouped_gemm_launch(const mgf_gemm_desc* desc, void* stream) {
  if (desc == nullptr) return MGF_ERR_INVALID_ARGUMENT;
  const mgf_gemm_desc& g = *desc;
  if (g.num_groups < 1 || g.num_groups > kMaxGroups) return MGF_ERR_TOO_MANY_GROUPS;
  if (g.epilogue < MGF_EPI_BIAS || g.epilogue > MGF_EPI_WGRAD) return MGF_ERR_INVALID_ARGUMENT;
  if (g.total_rows < 0 || g.total_rows > INT32_MAX) return MGF_ERR_INVALID_ARGUMENT;
  const bool ragged_k = g.epilogue == MGF_EPI_WGRAD;
  // Ragged-M with no rows has nothing to write.  Ragged-K with no rows still writes zeros for
  // every group (A and B, possibly NULL, are then never read).
  if (!ragged_k && g.total_rows == 0) return MGF_OK;
  const bool no_rows = g.total_rows == 0;
  const bool scatter = g.d_row_ptrs != nullptr;
  if (scatter && (g.epilogue != MGF_EPI_BIAS || g.ab_type != MGF_AB_BF16)) return MGF_ERR_INVALID_ARGUMENT;
  if (g.offs == nullptr || (g.d == nullptr && !scatter)) return MGF_ERR_INVALID_ARGUMENT;
  if (!no_rows && (g.a == nullptr || g.b == nullptr)) return MGF_ERR_INVALID_ARGUMENT;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MGF_ERR_CUDA;
  g_last_error[0] = 0;
  // Tensor maps are encoded through the driver API, which needs a current context on this host
  // thread.  Threads that only made runtime calls so far (autograd's backward workers) may have
  // none; cudaSetDevice binds the device's primary context.
  static thread_local int bound_dev = -1;
  if (bound_dev != dev) {
    if (cudaSetDevice(dev) != cudaSuccess) return MGF_ERR_CUDA;
    bound_dev = dev;
  }
  const DeviceInfo di = device_info(dev);
  if (di.major != 10) return MGF_ERR_NO_DEVICE_SUPPORT;

  Params p{};
  p.epi = g.epilogue;
  p.E = g.num_groups;
  p.total_rows = g.total_rows;
  p.offs = g.offs;
  p.bias = static_cast<const __nv_bfloat16*>(g.bias);
  p.bias_stride = g.bias_stride;
  p.bias_per_row = (g.epilogue == MGF_EPI_BIAS && g.bias != nullptr && g.bias_per_row) ? 1 : 0;
  p.d = static_cast<__nv_bfloat16*>(g.d);
  p.ldd = g.ldd;
  p.ldd_batch = g.ldd_batch;
  p.d2 = static_cast<__nv_bfloat16*>(g.d2);
  p.ldd2 = g.ldd2;
  p.aux = static_cast<const __nv_bfloat16*>(g.aux);
  p.ld_aux = g.ld_aux;
  auto v8_ok = [](const void* ptr, int64_t ld) {
    return ptr != nullptr && (reinterpret_cast<uintptr_t>(ptr) & 31u) == 0 && (ld % 16) == 0;
  };
  p.aux_v8 = v8_ok(g.aux, g.ld_aux) ? 1 : 0;
  p.d_v8 = v8_ok(g.d, g.ldd) ? 1 : 0;
  p.d_rows = reinterpret_cast<const long long*>(g.d_row_ptrs);
  if (g.group_begin < 0 || g.group_begin > g.num_groups) return MGF_ERR_INVALID_ARGUMENT;
  p.group_begin = g.group_begin;
  if (scatter) p.d_v8 = (g.n % 16) == 0 ? 1 : 0;  // per-row address alignment is checked in the kernel
  p.d2_v8 = v8_ok(g.d2, g.ldd2) ? 1 : 0;
  p.alpha = g.swiglu_alpha;
  p.limit = g.swiglu_limit;
  p.store_aux = g.store_aux;

  // Every row stride must be a multiple of 8 bf16 (16 bytes) and every base 16-byte aligned:
  // TMA needs it for A and B, the epilogue's 16-byte vector stores need it for the outputs.
  auto stride_ok = [](int64_t s) { return s > 0 && (s % 8) == 0; };
  if (!aligned16(g.a) || !aligned16(g.b) || !aligned16(g.d)) return MGF_ERR_ALIGNMENT;
  if (!scatter && !stride_ok(g.ldd)) return MGF_ERR_ALIGNMENT;
  const bool f8 = g.ab_type == MGF_AB_E4M3;
  if (g.ab_type != MGF_AB_BF16 && !f8) return MGF_ERR_INVALID_ARGUMENT;
  const int esz = f8 ? 1 : 2;  // bytes per A / B element
  auto ab_stride_ok = [esz](int64_t s) { return s > 0 && (s * esz) % 16 == 0; };
  if (!no_rows && (!ab_stride_ok(g.lda) || !ab_stride_ok(g.ldb))) return MGF_ERR_ALIGNMENT;
  if (f8) {
    if ((!ragged_k && g.b_mn_major) || g.scale_a == nullptr || g.scale_b == nullptr || g.bias_per_row)
      return MGF_ERR_INVALID_ARGUMENT;
    if (!aligned16(g.scale_b) || (!ragged_k && ((g.scale_b_stride % 4) != 0 || g.scale_b_stride < 0)))
      return MGF_ERR_ALIGNMENT;
  }
  p.bke = f8 ? 128 : BK;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.scale_b_stride = g.scale_b_stride;

  CUtensorMap tA, tB, tD;
  int bn, n_tiles, cg = 1;
  int64_t tiles_upper;
  if (!ragged_k) {
    // k: any (TMA reads zeros past it; the row pitches carry the 16-byte rule); n: whole 16-byte
    // output units
    if (g.n <= 0 || g.k <= 0 || (g.n % 8) != 0) return MGF_ERR_INVALID_ARGUMENT;
    if (g.n > INT32_MAX || g.k > INT32_MAX) return MGF_ERR_INVALID_ARGUMENT;
    if (!ab_stride_ok(g.ldb_batch)) return MGF_ERR_ALIGNMENT;
    if (g.bias != nullptr && (!aligned16(g.bias) || !stride_ok(g.bias_stride))) return MGF_ERR_ALIGNMENT;
    if (g.epilogue == MGF_EPI_SWIGLU) {
      if (g.bias == nullptr || g.d2 == nullptr || (g.n % 16) != 0) return MGF_ERR_INVALID_ARGUMENT;
      if (!aligned16(g.d2) || !stride_ok(g.ldd2)) return MGF_ERR_ALIGNMENT;
    }
    if (g.epilogue == MGF_EPI_SWIGLU_BWD) {
      if (g.aux == nullptr) return MGF_ERR_INVALID_ARGUMENT;
      if (!aligned16(g.aux) || !stride_ok(g.ld_aux)) return MGF_ERR_ALIGNMENT;
    }
    p.m = 0;
    p.n = static_cast<int>(g.n);
    p.k = static_cast<int>(g.k);
    bn = pick_bn(g.n);
    n_tiles = static_cast<int>((g.n + bn - 1) / bn);
    p.n_tiles = n_tiles;
    if (g.total_rows == 0) return MGF_OK;  // nothing to compute, outputs have no rows
    cg = pick_cta_group(false, g.total_rows, g.num_groups, 0);
    // one stage = 128 bytes of K per row: 64 bf16 or 128 e4m3 elements
    const CUtensorMapDataType abt = f8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint32_t bke = static_cast<uint32_t>(p.bke);
    const uint64_t dA[2] = {static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.total_rows)};
    const uint64_t sA[1] = {static_cast<uint64_t>(g.lda) * esz};
    const uint32_t bA[2] = {bke, 128};
    if (!encode_bf16(&tA, g.a, 2, dA, sA, bA, CU_TENSOR_MAP_SWIZZLE_128B, abt)) return MGF_ERR_CUDA;
    tD = tA;  // unused by the ragged-M epilogues
    const uint64_t sB[2] = {static_cast<uint64_t>(g.ldb) * esz, static_cast<uint64_t>(g.ldb_batch) * esz};
    if (f8) {
      const uint64_t dB[3] = {static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.num_groups)};
      const uint32_t bB[3] = {bke, static_cast<uint32_t>(bn / cg), 1};
      if (!encode_bf16(&tB, g.b, 3, dB, sB, bB, CU_TENSOR_MAP_SWIZZLE_128B, abt)) return MGF_ERR_CUDA;
    } else if (g.b_mn_major) {
      const uint64_t dB[3] = {static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.num_groups)};
      const uint32_t bB[3] = {64, 64, 1};
      if (!encode_bf16(&tB, g.b, 3, dB, sB, bB)) return MGF_ERR_CUDA;
    } else {
      const uint64_t dB[3] = {static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.num_groups)};
      const uint32_t bB[3] = {64, static_cast<uint32_t>(bn / cg), 1};
      if (!encode_bf16(&tB, g.b, 3, dB, sB, bB)) return MGF_ERR_CUDA;
    }
    tiles_upper = (g.total_rows / (BM * cg) + g.num_groups) * static_cast<int64_t>(n_tiles);
  } else {
    if (g.m <= 0 || g.n <= 0 || (g.n % 8) != 0) return MGF_ERR_INVALID_ARGUMENT;  // m: any (A rows are 16-byte aligned by lda)
    if (g.m > INT32_MAX || g.n > INT32_MAX) return MGF_ERR_INVALID_ARGUMENT;
    if (!stride_ok(g.ldd_batch)) return MGF_ERR_ALIGNMENT;
    if (g.d2 != nullptr && (!aligned16(g.d2) || !stride_ok(g.ldd2))) return MGF_ERR_ALIGNMENT;
    p.m = static_cast<int>(g.m);
    p.n = static_cast<int>(g.n);
    p.k = 0;
    bn = f8 ? (g.n <= 128 ? 128 : 256) : pick_bn(g.n);  // e4m3: whole 128-column chunks of B
    n_tiles = static_cast<int>((g.n + bn - 1) / bn);
    p.n_tiles = n_tiles;
    cg = f8 ? 1 : pick_cta_group(true, g.total_rows, g.num_groups, g.m);
    // Short groups (a few K stages per tile): the tile time is its dW store epilogue, so each warp
    // stores its 32 rows x BN/2 columns with one TMA store (the wide form; n a multiple of 64 so
    // that 64-column chunks never cross a row end).  MGF_WGRAD_SMALL_K=0|1 forces the choice.
    if (!f8 && cg == 1 && bn != 192 && (g.n % 64) == 0) {
      const char* env = getenv("MGF_WGRAD_SMALL_K");
      if (env != nullptr && (env[0] == '0' || env[0] == '1')) p.small_k = env[0] - '0';
      else p.small_k = (g.total_rows / g.num_groups <= kSmallKTokens) ? 1 : 0;
    }
    // Longer groups, BN = 256, single CTAs, m > 128: 256-row tiles, two 128-row accumulators over
    // all of TMEM sharing each B stage -- a third fewer operand bytes per output at the price of
    // the TMEM double buffer (measured on cfg3: up / down wgrad 2.86 / 1.50 -> 2.56 / 1.32 ms).
    // MGF_WGRAD_M256=0|1 forces the choice.
    if (cg == 1 && bn == 256 && !p.small_k) {
      const char* env = getenv("MGF_WGRAD_M256");
      p.m256 = (env != nullptr && (env[0] == '0' || env[0] == '1')) ? env[0] - '0' : (g.m > BM ? 1 : 0);
    }
    const int tm = BM * cg * (p.m256 ? 2 : 1);
    p.m_tiles_real = static_cast<int>((g.m + tm - 1) / tm);
    p.bias_grad = g.d2 != nullptr ? 1 : 0;
    p.m_tiles = p.m_tiles_real + ((p.bias_grad && (g.m % tm) == 0) ? 1 : 0);
    const uint32_t box[2] = {64, 64};
    if (!no_rows && f8) {
      // e4m3 token rows (row pitches in bytes): {128 features, 128 rows} boxes of A and B
      const uint32_t box8[2] = {128, 128};
      const uint64_t dA[2] = {static_cast<uint64_t>(g.m), static_cast<uint64_t>(g.total_rows)};
      const uint64_t sA[1] = {static_cast<uint64_t>(g.lda)};
      const uint64_t dB[2] = {static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.total_rows)};
      const uint64_t sB[1] = {static_cast<uint64_t>(g.ldb)};
      if (!encode_bf16(&tA, g.a, 2, dA, sA, box8, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_DATA_TYPE_UINT8) ||
          !encode_bf16(&tB, g.b, 2, dB, sB, box8, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_DATA_TYPE_UINT8))
        return MGF_ERR_CUDA;
      p.a_chunked = p.b_chunked = 0;
    } else if (!no_rows) {
      // Where the feature count is a multiple of 64, a stage's 64-column chunks of an operand come
      // in one 3D box: {64 features, 64 rows, chunks}, the chunk dimension 128 bytes apart (TMA
      // clips it at the last chunk, so the m / n tails still read as zeros).  Otherwise one 2D box
      // per chunk, clipped at m / n.
      const uint32_t boxA3[3] = {64, 64, static_cast<uint32_t>(BM / 64)};
      const uint32_t boxB3[3] = {64, 64, static_cast<uint32_t>((bn / cg + 63) / 64)};
      p.a_chunked = (g.m % 64) == 0 ? 1 : 0;
      // (each CTA's first column, n_blk * BN + crank * BN / CG, must start a chunk: not so for
      // CTA pairs with BN = 192, whose halves are 96 columns wide)
      p.b_chunked = ((g.n % 64) == 0 && ((bn / cg) % 64) == 0) ? 1 : 0;
      if (p.a_chunked) {
        const uint64_t dA[3] = {64, static_cast<uint64_t>(g.total_rows), static_cast<uint64_t>(g.m / 64)};
        const uint64_t sA[2] = {static_cast<uint64_t>(g.lda) * 2, 128};
        if (!encode_bf16(&tA, g.a, 3, dA, sA, boxA3)) return MGF_ERR_CUDA;
      } else {
        const uint64_t dA[2] = {static_cast<uint64_t>(g.m), static_cast<uint64_t>(g.total_rows)};
        const uint64_t sA[1] = {static_cast<uint64_t>(g.lda) * 2};
        if (!encode_bf16(&tA, g.a, 2, dA, sA, box)) return MGF_ERR_CUDA;
      }
      if (p.b_chunked) {
        const uint64_t dB[3] = {64, static_cast<uint64_t>(g.total_rows), static_cast<uint64_t>(g.n / 64)};
        const uint64_t sB[2] = {static_cast<uint64_t>(g.ldb) * 2, 128};
        if (!encode_bf16(&tB, g.b, 3, dB, sB, boxB3)) return MGF_ERR_CUDA;
      } else {
        const uint64_t dB[2] = {static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.total_rows)};
        const uint64_t sB[1] = {static_cast<uint64_t>(g.ldb) * 2};
        if (!encode_bf16(&tB, g.b, 2, dB, sB, box)) return MGF_ERR_CUDA;
      }
    } else {
      // Never dereferenced (every group is empty): well-formed maps over the output buffer.
      const uint64_t dz[2] = {8, 1};
      const uint64_t sz[1] = {16};
      if (!encode_bf16(&tA, g.d, 2, dz, sz, box) || !encode_bf16(&tB, g.d, 2, dz, sz, box)) return MGF_ERR_CUDA;
    }
    tiles_upper = static_cast<int64_t>(p.m_tiles) * n_tiles * g.num_groups;
    const uint64_t sD[2] = {static_cast<uint64_t>(g.ldd) * 2, static_cast<uint64_t>(g.ldd_batch) * 2};
    if (p.small_k) {
      // dW as {64 columns, m rows, n / 64 chunks, E}: boxes {64, 32, BN / 128, 1}, 128-byte swizzle
      const uint64_t dD[4] = {64, static_cast<uint64_t>(g.m), static_cast<uint64_t>(g.n / 64),
                              static_cast<uint64_t>(g.num_groups)};
      const uint64_t sD4[3] = {sD[0], 128, sD[1]};
      const uint32_t bD[4] = {64, 32, static_cast<uint32_t>(bn / 128), 1};
      if (!encode_bf16(&tD, g.d, 4, dD, sD4, bD, CU_TENSOR_MAP_SWIZZLE_128B)) return MGF_ERR_CUDA;
    } else {
      // dW [E, m, n] for the epilogue's TMA tile stores: 32 x 32 boxes, 64-byte swizzle
      const uint64_t dD[3] = {static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.m), static_cast<uint64_t>(g.num_groups)};
      const uint32_t bD[3] = {32, 32, 1};
      if (!encode_bf16(&tD, g.d, 3, dD, sD, bD, CU_TENSOR_MAP_SWIZZLE_64B)) return MGF_ERR_CUDA;
    }
  }

  int sms = di.sms - (g.sm_carveout > 0 ? g.sm_carveout : 0);
  if (sms < cg) sms = cg;
  const int units = sms / cg;  // CTAs (CG = 1) or CTA pairs (CG = 2) resident at once
  const int64_t launch_units = tiles_upper < units ? tiles_upper : units;
  if (launch_units <= 0) return MGF_OK;
  const int grid = static_cast<int>(launch_units) * cg;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool b_mn = ragged_k ? true : (g.b_mn_major != 0);
  // The dynamic tile counter serves single CTAs only: both CTAs of a pair must walk the same tile
  // sequence, which static striding gives them.
  p.tile_counter = (g.epilogue == MGF_EPI_WGRAD) ? g.workspace : nullptr;
  // Test hook for the bounded waits: with MGF_TEST_STALL_PRODUCER=1 the kernel does no work and
  // every consumer wait gives up after its limit, setting MGF_DEV_WAIT_TIMEOUT.  Nothing is in flight
  // when they give up, so the context stays usable; tests use it to exercise that path on a GPU.
  {
    const char* env = getenv("MGF_TEST_STALL_PRODUCER");
    p.stall_test = (env != nullptr && env[0] == '1') ? 1 : 0;
  }
  if (cg == 2) {
    switch (bn) {
      case 256: return dispatch_epi<256, 2>(g.epilogue, b_mn, f8, tA, tB, tD, p, grid, st);
      case 192: return dispatch_epi<192, 2>(g.epilogue, b_mn, f8, tA, tB, tD, p, grid, st);
      default: return dispatch_epi<128, 2>(g.epilogue, b_mn, f8, tA, tB, tD, p, grid, st);
    }
  }
  switch (bn) {
    case 256: return dispatch_epi<256, 1>(g.epilogue, b_mn, f8, tA, tB, tD, p, grid, st);
    case 192: return dispatch_epi<192, 1>(g.epilogue, b_mn, f8, tA, tB, tD, p, grid, st);
    default: return dispatch_epi<128, 1>(g.epilogue, b_mn, f8, tA, tB, tD, p, grid, st);
  }
}

// ============================================================================ allocation-free entry point
//
// Some callers cannot allocate device memory at the point where they launch: a runtime that lays out
// every device buffer once up front (a fixed memory plan with no allocator on the step path), or a
// host program that binds this C ABI directly and only holds the buffers it was handed.  Such a
// caller can still pass its inputs and outputs, but has nowhere to get the zero-filled int32 tile
// counter that the ragged-K weight-gradient launch (MGF_EPI_WGRAD) wants as `workspace`.
// mgf_grouped_gemm_launch_noalloc runs that launch with the counter taken from the array below
// instead.  The array lives in the library's device image, so every GPU that loads the library holds
// its 256 bytes until the process exits.
//
// Limits and rules:
//  * only MGF_EPI_WGRAD descriptors, with desc->workspace == NULL (the entry point supplies it);
//  * the launch needs one int32 word; a launch needing more than kNoAllocScratchWords words would be
//    rejected with MGF_ERR_INVALID_ARGUMENT and a message in mgf_last_error_detail();
//  * every call shares the one array and it keeps the last call's contents, so each call clears the
//    word it uses (cudaMemsetAsync on `stream`) before the kernel; calls that overlap on the GPU
//    (different streams, no ordering between them) race on the counter and must not be issued;
//  * each call looks up the array's device address afresh (cudaGetSymbolAddress with the calling
//    device current), so the address stays right after a cudaDeviceReset reloads the module; while
//    `stream` is capturing no lookup is made and the last address found on that device is reused,
//    so make the first call on each device before any stream capture.
//  * nothing here calls cudaMalloc, cudaFree or any allocating routine.

namespace mgf {

constexpr int kNoAllocScratchWords = 64;
static __device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocScratchWords];

static int32_t* noalloc_scratch_address(int dev, bool capturing) {
  static int32_t* cached[64] = {};
  static std::mutex mu;
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (capturing) return cached[dev];  // no runtime lookups inside a capture
  // The symbol's host-side name is only a stand-in: the device address must come from the
  // runtime, with this device current.
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) {
    record_error("cudaGetSymbolAddress(g_noalloc_scratch)", e);
    return nullptr;
  }
  cached[dev] = static_cast<int32_t*>(ptr);
  return cached[dev];
}

}  // namespace mgf

extern "C" int mgf_grouped_gemm_launch_noalloc(const mgf_gemm_desc* desc, void* stream) {
  if (desc == nullptr) return MGF_ERR_INVALID_ARGUMENT;
  g_last_error[0] = 0;
  if (desc->epilogue != MGF_EPI_WGRAD) {
    snprintf(g_last_error, sizeof(g_last_error),
             "mgf_grouped_gemm_launch_noalloc: only MGF_EPI_WGRAD launches use scratch; use mgf_grouped_gemm_launch");
    return MGF_ERR_INVALID_ARGUMENT;
  }
  if (desc->workspace != nullptr) {
    snprintf(g_last_error, sizeof(g_last_error),
             "mgf_grouped_gemm_launch_noalloc: desc->workspace must be NULL (the static scratch is used)");
    return MGF_ERR_INVALID_ARGUMENT;
  }
  const int words_needed = 1;  // the dynamic tile counter
  if (words_needed > kNoAllocScratchWords) {
    snprintf(g_last_error, sizeof(g_last_error),
             "mgf_grouped_gemm_launch_noalloc: launch needs %d scratch words, the static scratch holds %d",
             words_needed, kNoAllocScratchWords);
    return MGF_ERR_INVALID_ARGUMENT;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MGF_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return MGF_ERR_CUDA;
  int32_t* scratch = noalloc_scratch_address(dev, cap != cudaStreamCaptureStatusNone);
  if (scratch == nullptr) {
    if (g_last_error[0] == 0)
      snprintf(g_last_error, sizeof(g_last_error),
               "mgf_grouped_gemm_launch_noalloc: first call on this device made during stream capture");
    return MGF_ERR_CUDA;
  }
  const cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(int32_t) * words_needed, st);
  if (e != cudaSuccess) {
    record_error("cudaMemsetAsync(static scratch)", e);
    return MGF_ERR_CUDA;
  }
  mgf_gemm_desc d = *desc;
  d.workspace = scratch;
  return mgf_grouped_gemm_launch(&d, stream);
}
