// Device kernels of the B200 grouped FP8 x MXFP4 MoE GEMM.
//
//   cdg_sf_atom_kernel      weight scales [E, N, K/32] -> 128x4 scale-factor atoms (weight-load time)
//   cdg_psum_rows_kernel    psum-form m_indices -> one group id per row
//   cdg_prep_kernel         per 128-row block: plan (expert, rows, class) + oracle-faithful split of the
//                           activations into two e4m3 planes (hi, lo) and their UE8M0 scale atoms;
//                           the last CTA orders the blocks of each class into work lists
//   cdg_gemm_kernel<TOK>    persistent tcgen05 block-scaled GEMM over one class of blocks
//   cdg_generic_kernel      exact SIMT path for blocks/layouts the tensor-core kernel does not take
//
// Layout facts shared by the host code live in cdg_layout.h.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>

#include "cdg_layout.h"
#include "cdg_ptx.cuh"
#include "cdg_split.cuh"

namespace cdg {

// =====================================================================================
// Scale-factor atoms.
// One atom holds the UE8M0 scales of 128 rows x 4 consecutive 32-wide K blocks (512 B):
// byte (r, c) of a [rows, kb] matrix goes to atom (r/128, c/4), offset
// (r%32)*16 + ((r%128)/32)*4 + c%4; missing rows/columns read 127 (scale 1.0).
// This is the order in which tcgen05.cp.32x128b.warpx4 feeds the MMA's scale
// columns, and the reorder of consumer_deep_gemm/gemm.py:76-116.
// =====================================================================================
__global__ void cdg_sf_atom_kernel(const uint8_t* __restrict__ src, int64_t src_stride_e, int64_t src_stride_n,
                                   uint32_t* __restrict__ dst, int E, int N, int KB32) {
  const int n_tiles = (N + 127) / 128;
  const int k_tiles = (KB32 + 3) / 4;
  const int64_t words_per_e = static_cast<int64_t>(n_tiles) * k_tiles * 128;
  const int64_t total = words_per_e * E;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(w / words_per_e);
    const int64_t rem = w - e * words_per_e;
    const int atom = static_cast<int>(rem >> 7);
    const int j = static_cast<int>(rem & 127);
    const int mt = atom / k_tiles, kt = atom - mt * k_tiles;
    const int row = mt * 128 + (j & 3) * 32 + (j >> 2);
    uint32_t v = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int col = kt * 4 + b;
      uint32_t byte = 127u;
      if (row < N && col < KB32) byte = src[e * src_stride_e + row * src_stride_n + col];
      v |= byte << (8 * b);
    }
    dst[w] = v;
  }
}

// UE8M0 code of a float weight scale.  A positive power of two 2^(c-127), c in [0, 254], is
// exact (*exact = true): c is its FP32 exponent field (2^-127, a subnormal, is code 0).  Any
// other value gets the reference's rounding, clamp(round(log2(s)) + 127, 0, 255) with s
// clamped below at the smallest normal float (consumer_deep_gemm/gemm.py:62-73): for a normal
// s = m * 2^e, m in [1, 2), round(log2(s)) is e + 1 when m >= sqrt(2) (m * m >= 2, exact in
// double), else e.  NaN gets 255.
__device__ __forceinline__ uint32_t float_scale_code(float s, bool* exact) {
  const uint32_t bits = __float_as_uint(s);
  const uint32_t ex = (bits >> 23) & 0xFFu, man = bits & 0x7FFFFFu;
  if (!(bits >> 31) && man == 0 && ex >= 1 && ex <= 254) {
    *exact = true;
    return ex;
  }
  *exact = false;
  if (bits == 0x00400000u) {  // 2^-127
    *exact = true;
    return 0;
  }
  if (s != s) return 255;
  if (!(s >= 1.17549435e-38f)) return 1;  // zero, negative or subnormal: log2 of the smallest normal
  if (ex == 255) return 255;              // +inf
  const double m = 1.0 + static_cast<double>(man) * (1.0 / 8388608.0);
  const int r = static_cast<int>(ex) - 127 + (m * m >= 2.0 ? 1 : 0);
  return static_cast<uint32_t>(min(max(r + 127, 0), 255));
}

// Float weight scales [E, N, KB32] -> the same atoms as cdg_sf_atom_kernel, each byte
// float_scale_code(s); sets *inexact when any scale of the tensor is not a power of two.
__global__ void cdg_sf_atom_f32_kernel(const float* __restrict__ src, int64_t src_stride_e, int64_t src_stride_n,
                                       uint32_t* __restrict__ dst, int E, int N, int KB32, int* inexact) {
  const int n_tiles = (N + 127) / 128;
  const int k_tiles = (KB32 + 3) / 4;
  const int64_t words_per_e = static_cast<int64_t>(n_tiles) * k_tiles * 128;
  const int64_t total = words_per_e * E;
  bool all_exact = true;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(w / words_per_e);
    const int64_t rem = w - e * words_per_e;
    const int atom = static_cast<int>(rem >> 7);
    const int j = static_cast<int>(rem & 127);
    const int mt = atom / k_tiles, kt = atom - mt * k_tiles;
    const int row = mt * 128 + (j & 3) * 32 + (j >> 2);
    uint32_t v = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int col = kt * 4 + b;
      uint32_t byte = 127u;
      if (row < N && col < KB32) {
        bool ex = true;
        byte = float_scale_code(src[e * src_stride_e + row * src_stride_n + col], &ex);
        all_exact = all_exact && ex;
      }
      v |= byte << (8 * b);
    }
    dst[w] = v;
  }
  if (!all_exact) atomicOr(inexact, 1);
}

// =====================================================================================
// psum form: m_indices[g] is the cumulative end row of group g (group g owns rows
// [end[g-1], end[g]) with end[-1] = 0).  Later groups win where ranges overlap, as
// in the reference's per-group index_copy_ (consumer_deep_gemm/gemm.py:318-324, 358-367).
// =====================================================================================
// masked form: counts[g] rows of group g start at row g*S (S = M / G); where a count
// exceeds S the rows run on into the next block and later groups win, as in the
// reference's sequential per-group copies (consumer_deep_gemm/gemm.py:541-551).
template <typename IdT>
__global__ void cdg_masked_rows_kernel(const IdT* __restrict__ counts, int G, int S, int M,
                                       int32_t* __restrict__ row_ids) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= M) return;
  int32_t id = -1;
  const int top = S > 0 ? min(G - 1, r / S) : G - 1;
  for (int g = top; g >= 0; --g) {
    if (static_cast<int64_t>(r) < static_cast<int64_t>(g) * S + static_cast<int64_t>(counts[g])) {
      id = g;
      break;
    }
  }
  row_ids[r] = id;
}

template <typename IdT>
__global__ void cdg_psum_rows_kernel(const IdT* __restrict__ ends, int G, int M, int32_t* __restrict__ row_ids) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= M) return;
  int32_t id = -1;
  int64_t start = 0;
  for (int g = 0; g < G; ++g) {
    const int64_t end = static_cast<int64_t>(ends[g]);
    if (r >= start && r < end) id = g;
    start = end;
  }
  row_ids[r] = id;
}

// =====================================================================================
// Prep: block plan + activation split.
//
// For a row r with valid expert id and a K block kb (128 wide) the reference's
// activation value is x = bf16(bf16(a[r,k]) * bf16(sa[r,kb])) (gemm.py:44-48).
// Let 2^E bound |bf16(sa[r,kb])| over all K blocks of the row (E = frexp exponent
// of the largest).  Every x / 2^E is then a BF16 number below 448 in magnitude,
// which splits exactly into hi = e4m3(x/2^E) and lo = e4m3(x/2^E - hi) whenever
// |x/2^E| >= 2^-2 (smaller elements lose at most 2^-10 * 2^E).  The tensor core
// multiplies both planes with the weights (activation scale factor 1), and the
// epilogue multiplies the FP32 sum by 2^E, exactly: sum_k (hi+lo) * w * 2^E = sum_k x * w.
// =====================================================================================
struct PrepArgs {
  const uint8_t* a;  // e4m3 [M, K]
  int64_t a_row_stride;
  const float* sa;  // [M, K/128] FP32, or int32 words of 4 UE8M0 scales (sa_packed)
  int64_t sa_stride_m, sa_stride_k;
  int sa_packed;
  const void* ids;  // per-row group ids (int32 or int64)
  int M, K, E;
  int nblk;
  TileMap tm;              // rows of each block
  uint8_t* hilo;           // [2][nblk*128][K]
  uint8_t* tok_code;       // [M][tok_code_pitch(K)] UE8M0 code of each direct-class row's activation scale
  int pair_wide;           // wide blocks run on the CTA-pair path (token tiles of the planes kernel, or
                           // of the direct kernel when their scales are all powers of two)
  int32_t* row_exp;        // [nblk*128] exponent E of each routed row's activation planes
  int4* blk_info;          // [nblk] {expert (-1 none, -2 several), rows spanned, class, 0}
  uint4* blk_mask;         // [nblk] bit r set when row r of the block has the block's expert
  int* ctrl;               // control words (zeroed by the host before launch)
  int4* lists;             // [kNumClasses][nblk] {block, expert, rows spanned, 0}
  int4* plane_tiles;       // [2*nblk] tiles of cdg_gemm_planes_kernel (pair_wide only):
                           // {first plane row, rows, expert, 1 on the last tile of a run}
  int4* direct_tiles;      // [nblk] tiles of cdg_gemm_direct_kernel, the same form
  const int* sf_inexact;   // float weight scales: set when one is not a power of two, and the
                           // exact SIMT kernel then takes every block (nullptr: not consulted)
  int planes_given;        // the caller passed the activation planes and row exponents: plan the
                           // blocks only (no plane split, no direct class)
};

// 2^(e-127) exactly, e in [0, 255] (255 gives +inf as in the reference's FP32 pow).
__device__ __forceinline__ float ue8m0_to_f32(uint32_t e) {
  return e == 0 ? __uint_as_float(0x00400000u) : __uint_as_float(e << 23);
}

// UE8M0 code of an activation scale 2^s with s in [-117, 118], or -1.  In that range
// every e4m3 value times 2^s (magnitudes 2^-9 .. 448) is a normal BF16 number, so
// BF16 dequantisation of the row is exact and equals the product the tensor core forms
// from the e4m3 value and the scale factor.
__device__ __forceinline__ int pow2_code(float v) {
  const uint32_t bits = __float_as_uint(v);
  const uint32_t e = bits >> 23;  // sign bit 0 for positive values
  return ((bits & 0x7FFFFFu) == 0 && e >= 10 && e <= 245) ? static_cast<int>(e) : -1;
}

// Activation scale of row r, 128-wide K block kb: FP32, or UE8M0 packed four to a word.
// (Read-only loads: the scales are an input of the call, never written by it.)
__device__ __forceinline__ float load_sa(const float* sa, int packed, int64_t sm, int64_t sk, int64_t r, int64_t kb) {
  if (!packed) return __ldg(sa + r * sm + kb * sk);
  const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(sa) + r * sm + (kb >> 2) * sk);
  return ue8m0_to_f32((w >> (8 * (kb & 3))) & 0xFFu);
}

// Group id of row r; a null id vector means every row belongs to group 0.
__device__ __forceinline__ int64_t load_id(const void* ids, int is64, int r) {
  if (!ids) return 0;
  return is64 ? static_cast<const int64_t*>(ids)[r] : static_cast<int64_t>(static_cast<const int32_t*>(ids)[r]);
}

__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}

// Grid: (nblk, ceil(K / kPrepK)).  CTA (b, y) converts K columns [y*kPrepK, (y+1)*kPrepK)
// of block b; CTA (b, 0) also publishes the block's plan, and the last of those
// orders the blocks of each class into lists.
constexpr int kPrepK = 1024;
constexpr int kContBits = 16384;  // blocks whose run-continuation bits the last prep CTA keeps in shared memory

template <typename IdT>
__global__ void __launch_bounds__(256) cdg_prep_kernel(PrepArgs p) {
  __shared__ int s_min_id, s_max_id, s_max_row;
  __shared__ int s_last, s_nv, s_pow2, s_exp_bad;
  __shared__ int64_t s_prev_id;  // id of the row before the block (-1 for the first block)
  __shared__ uint8_t s_vrow[128];  // the block's rows that carry its expert (compacted)
  __shared__ int s_id[128];
  __shared__ uint32_t s_mask[4];
  __shared__ float s_scale[128][kPrepK / 128];
  __shared__ int s_exp[128];
  __shared__ float s_inv[128];              // 2^-E of each row
  __shared__ uint32_t s_smax_bits[128];     // bits of the largest finite |bf16(sa)| of each row
  constexpr int kScan = kNumClasses + 2;    // last CTA: per-class block counts, plane and direct tiles
  __shared__ int s_warp_sum[8][kScan];      // last CTA: the scan's per-warp totals (256 threads)
  __shared__ uint32_t s_cont[kContBits / 32];  // last CTA: which blocks continue a run (bitmask)
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_min_id = 0x7fffffff;
    s_max_id = -1;
    s_max_row = -1;
    s_nv = 0;
    s_pow2 = 1;
    s_exp_bad = 0;
  }
  if (tid < 4) s_mask[tid] = 0u;
  if (tid < 128) s_smax_bits[tid] = 0u;
  int row0, nrows;
  p.tm.rows(b, row0, nrows);
  __syncthreads();
  if (tid < 128) {
    const int r = row0 + tid;
    int id = -1;
    if (tid < nrows) {
      const int64_t v = load_id(p.ids, sizeof(IdT) == 8, r);
      id = (v >= 0 && v < p.E) ? static_cast<int>(v) : -1;
    }
    s_id[tid] = id;
    if (id >= 0) {
      atomicMin(&s_min_id, id);
      atomicMax(&s_max_id, id);
      atomicMax(&s_max_row, tid);
    }
  } else if (tid == 128) {
    // read alongside the block's own ids (the class rule below needs it)
    s_prev_id = row0 > 0 ? load_id(p.ids, sizeof(IdT) == 8, row0 - 1) : -1;
  }
  __syncthreads();
  const int eff = s_max_row + 1;
  int cls, expert;
  if (eff == 0) {
    cls = kClassZero;
    expert = -1;
  } else if (s_min_id != s_max_id) {
    cls = kClassIrregular;
    expert = -2;
  } else {
    cls = eff <= kTinyTok ? kClassTiny : eff <= kNarrowTok ? kClassNarrow : kClassWide;
    expert = s_min_id;
    // The last block of an expert that spans several blocks joins its wide blocks on the
    // CTA-pair path: the wide kernels trim the MMA to the block's rows, and they read the
    // expert's weights from L2 right after its other blocks did, where the tiny and narrow
    // kernels would stream them from HBM again.
    if (cls != kClassWide && p.pair_wide && row0 > 0 && s_prev_id == static_cast<int64_t>(expert)) cls = kClassWide;
    // float weight scales that are not all powers of two: the tensor cores' UE8M0 scale
    // factors cannot hold them, the exact SIMT kernel takes the block
    if (p.sf_inexact && __ldcg(p.sf_inexact)) {
      cls = kClassIrregular;
      expert = -2;
    }
  }
  if (p.planes_given && cls == kClassIrregular) {
    // planes given by the caller: the exact SIMT kernel has no e4m3 rows to read, and a block
    // holding rows of several experts breaks the caller's promise of 128-aligned groups; the
    // block is left out (written as zeros unless rows outside groups are skipped) and reported
    cls = kClassZero;
    expert = -1;
    if (tid == 0 && blockIdx.y == 0) {
      atomicOr(&p.ctrl[kCtrlStatus], kStatusBadIndex);
      atomicOr(&g_sticky_status[0], kStatusBadIndex);
    }
  }

  if (cls == kClassTiny || cls == kClassNarrow || cls == kClassWide) {
    if (tid < 128 && s_id[tid] == expert) {
      atomicOr(&s_mask[tid >> 5], 1u << (tid & 31));
      s_vrow[atomicAdd(&s_nv, 1)] = static_cast<uint8_t>(tid);
    }
  }
  if (!p.planes_given && (cls == kClassTiny || cls == kClassNarrow || cls == kClassWide)) {
    const int ntok = (eff + 15) & ~15;
    const int K = p.K;
    const int kb_count = K / 128;
    const int kb0 = blockIdx.y * (kPrepK / 128);
    const int kbn = min(kPrepK / 128, kb_count - kb0);
    // (1) per routed row: the exponent E with |bf16(sa[r,kb])| < 2^E for every K block of
    //     the row (frexp exponent of the largest scale); and the BF16-rounded scales of
    //     this CTA's K blocks, kept from the same pass.  The (row, K block) scales are read
    //     by all threads at once, the K block fastest unless the scales are stored row-fastest
    //     (MN-major).
    {
      const bool mn_major = !p.sa_packed && p.sa_stride_m == 1;
      const int items = ntok * kb_count;
      bool pow2 = true;
      // kU items per thread per round: their loads are all issued before any is used
      constexpr int kU = 8;
      for (int it0 = tid; it0 < items; it0 += kU * blockDim.x) {
        float sraw[kU];
        int rrs[kU], kbs[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int it = it0 + u * blockDim.x;
          const int rr = mn_major ? it % ntok : it / kb_count;
          const int kb = mn_major ? it / ntok : it % kb_count;
          const bool mine = it < items && s_id[rr] == expert;
          rrs[u] = mine ? rr : -1;
          kbs[u] = kb;
          sraw[u] = mine ? load_sa(p.sa, p.sa_packed, p.sa_stride_m, p.sa_stride_k, row0 + rr, kb) : 1.0f;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          if (rrs[u] < 0) continue;
          const float sbf = __bfloat162float(__float2bfloat16_rn(sraw[u]));
          // non-negative floats order as their bit patterns
          if (isfinite(sbf)) atomicMax(&s_smax_bits[rrs[u]], __float_as_uint(fabsf(sbf)));
          pow2 = pow2 && pow2_code(sraw[u]) >= 0;
          const int kl = kbs[u] - kb0;
          if (kl >= 0 && kl < kbn) s_scale[rrs[u]][kl] = sbf;  // this CTA's K blocks (routed rows only)
        }
      }
      if (!pow2) atomicAnd(&s_pow2, 0);
      __syncthreads();
    }
    if (tid < ntok) {
      int emax = 0;
      if (s_id[tid] == expert) {
        const float smax = __uint_as_float(s_smax_bits[tid]);
        if (smax > 0.0f) frexpf(smax, &emax);
        // 2^E must be a UE8M0 scale factor (and a normal FP32 factor in the epilogue)
        if (emax < -126 || emax > 127) atomicOr(&s_exp_bad, 1);
      }
      s_exp[tid] = emax;
      s_inv[tid] = ldexpf(1.0f, -emax);
      if (blockIdx.y == 0) p.row_exp[b * 128 + tid] = emax;
    }
    __syncthreads();
  }
  if (s_exp_bad) {
    // a row exponent outside the scale-factor range: the exact SIMT kernel takes the block
    cls = kClassIrregular;
    expert = -2;
  }
  if (!p.planes_given && (cls == kClassTiny || cls == kClassNarrow || cls == kClassWide)) {
    const int K = p.K;
    const int kb_count = K / 128;
    const int kb0 = blockIdx.y * (kPrepK / 128);
    const int kbn = min(kPrepK / 128, kb_count - kb0);
    const int64_t plane = static_cast<int64_t>(p.nblk) * 128 * K;
    // Direct class: a wide block (CTA-pair path) whose routed rows' scales are all powers
    // of two.  The reference's bf16(bf16(a) * bf16(2^s)) is then the exact product a * 2^s,
    // which the tensor core forms itself from the raw e4m3 rows with 2^s as scale factor: no
    // planes, one MMA per K slice.  The UE8M0 code of every row of the block (127 for rows
    // without its expert) goes to tok_code (row major, one byte per K block), for this CTA's
    // K blocks.
    const bool direct = cls == kClassWide && p.pair_wide && s_pow2;
    if (direct) {
      const int pitch = tok_code_pitch(K);
#pragma unroll 4
      for (int it = tid; it < kbn * nrows; it += blockDim.x) {
        const int rr = it / kbn, kl = it - rr * kbn;
        int code = 127;
        if (s_id[rr] == expert)
          code = pow2_code(load_sa(p.sa, p.sa_packed, p.sa_stride_m, p.sa_stride_k, row0 + rr, kb0 + kl));
        p.tok_code[static_cast<int64_t>(row0 + rr) * pitch + kb0 + kl] = static_cast<uint8_t>(code);
      }
    }
    if (direct) {
      cls = kClassWideDirect;
    } else {
    // (2) activation planes of the rows that carry the block's expert, one 16-byte chunk
    //     per item; consecutive threads read consecutive chunks of a row (coalesced).
    //     Other rows of the planes are not written: whatever they hold only reaches
    //     accumulator columns the epilogue replaces by zeros.
    const int chunks = kbn * 8;
    const int nv = s_nv;
    for (int it = tid; it < nv * chunks; it += blockDim.x) {
      const int rr = s_vrow[it / chunks];
      const int c = it % chunks;
      const int kl = c >> 3;
      const int r = row0 + rr;
      const int64_t col = static_cast<int64_t>(kb0) * 128 + c * 16;
      uint4 hi4, lo4;
      split_planes16(*reinterpret_cast<const uint4*>(p.a + r * p.a_row_stride + col), s_scale[rr][kl], s_inv[rr], hi4,
                     lo4);
      uint8_t* dst = p.hilo + (static_cast<int64_t>(b) * 128 + rr) * K + col;
      *reinterpret_cast<uint4*>(dst) = hi4;
      *reinterpret_cast<uint4*>(dst + plane) = lo4;
    }
    }
  }
  if (blockIdx.y != 0) return;

  // Publish the plan (thread 0 orders its own store before the ticket), then the
  // last block to arrive orders each class's blocks (block order = expert order
  // in the contiguous layout, which keeps blocks of one expert adjacent).
  __syncthreads();
  if (tid == 0) {
    p.blk_info[b] = make_int4(expert, eff, cls, 0);
    p.blk_mask[b] = make_uint4(s_mask[0], s_mask[1], s_mask[2], s_mask[3]);
    __threadfence();
    s_last = (atomicAdd(&p.ctrl[kCtrlTicket], 1) == p.nblk - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int per = (p.nblk + blockDim.x - 1) / blockDim.x;
  const int lo = min(p.nblk, tid * per), hi = min(p.nblk, lo + per);
  // Tiles of the planes kernel: a run is a maximal sequence of wide blocks of one expert
  // whose rows follow each other, every block but the last full (128 routed rows spanned).
  // A run of S rows is cut into the fewest tiles, n = ceil(S / kPlanesTileTok), of
  // T = ceil16(S / n) rows each (the last one shorter): a tile costs the kernel about the
  // same time at any width, so fewer tiles is faster, and equal widths spread the MMA work.
  auto continues_g = [&](int i) -> bool {  // block i extends the run of block i - 1 (same class)
    if (i == 0) return false;
    const int4 a = __ldcg(&p.blk_info[i - 1]), c = __ldcg(&p.blk_info[i]);
    if ((c.z != kClassWide && c.z != kClassWideDirect) || a.z != c.z || a.x != c.x || a.y != 128) return false;
    int r0a, na, r0c, nc;
    p.tm.rows(i - 1, r0a, na);
    p.tm.rows(i, r0c, nc);
    return na == 128 && r0c == r0a + 128;
  };
  // The "continues" bit of every block, computed once by all threads (independent loads) into a
  // shared bitmask, so that the run walks below read shared memory instead of chaining global
  // loads (up to kContBits blocks; beyond, the bits are recomputed from global memory).
  const bool cached = p.nblk <= kContBits;
  if (cached) {
    for (int w = tid; w < (p.nblk + 31) / 32; w += blockDim.x) s_cont[w] = 0u;
    __syncthreads();
    for (int i = tid; i < p.nblk; i += blockDim.x)
      if (continues_g(i)) atomicOr(&s_cont[i >> 5], 1u << (i & 31));
    __syncthreads();
  }
  auto continues = [&](int i) -> bool {
    return cached ? ((s_cont[i >> 5] >> (i & 31)) & 1u) != 0u : continues_g(i);
  };
  auto run_span = [&](int i) -> int {  // rows spanned by the run that starts at block i
    int j = i;
    while (j + 1 < p.nblk && continues(j + 1)) ++j;
    return 128 * (j - i) + __ldcg(&p.blk_info[j].y);
  };
  static_assert(kPlanesTileTok % 16 == 0, "tile cuts at multiples of 16 rows");
  // per thread (its blocks [lo, hi)): blocks of each class, then plane tiles, then direct tiles
  int cnt[kScan] = {};
  for (int i = lo; i < hi; ++i) {
    const int c = __ldcg(&p.blk_info[i].z);
    cnt[c]++;
    if (p.pair_wide && c == kClassWide && !continues(i))
      cnt[kNumClasses] += (run_span(i) + kPlanesTileTok - 1) / kPlanesTileTok;
    if (p.pair_wide && c == kClassWideDirect && !continues(i))
      cnt[kNumClasses + 1] += (run_span(i) + kDirectTileTok - 1) / kDirectTileTok;
  }
  // Exclusive scan of the eight counts over the 256 threads (in block order): shuffles within
  // each warp, then the eight warp totals.
  const int lane = tid & 31, warp = tid >> 5;
  int incl[kScan];
#pragma unroll
  for (int k = 0; k < kScan; ++k) incl[k] = cnt[k];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int k = 0; k < kScan; ++k) {
      const int v = __shfl_up_sync(0xffffffffu, incl[k], o);
      if (lane >= o) incl[k] += v;
    }
  }
  if (lane == 31) {
#pragma unroll
    for (int k = 0; k < kScan; ++k) s_warp_sum[warp][k] = incl[k];
  }
  __syncthreads();
  if (tid < kScan) {  // thread k: exclusive scan of value k over the warps, and its total
    int run = 0;
    for (int w = 0; w < 8; ++w) {
      const int v = s_warp_sum[w][tid];
      s_warp_sum[w][tid] = run;
      run += v;
    }
    p.ctrl[tid < kNumClasses ? kCtrlCount0 + tid : tid == kNumClasses ? kCtrlPlaneTiles : kCtrlDirectTiles] = run;
  }
  __syncthreads();
  int pos[kNumClasses];
#pragma unroll
  for (int c = 0; c < kNumClasses; ++c) pos[c] = s_warp_sum[warp][c] + incl[c] - cnt[c];
  int tpos = s_warp_sum[warp][kNumClasses] + incl[kNumClasses] - cnt[kNumClasses];
  int dpos = s_warp_sum[warp][kNumClasses + 1] + incl[kNumClasses + 1] - cnt[kNumClasses + 1];
  for (int i = lo; i < hi; ++i) {
    const int c = __ldcg(&p.blk_info[i].z);
    const int4 info = __ldcg(&p.blk_info[i]);
    p.lists[c * p.nblk + pos[c]++] = make_int4(i, info.x, info.y, 0);
    if (p.pair_wide && c == kClassWide && !continues(i)) {
      const int span = run_span(i);
      const int n = (span + kPlanesTileTok - 1) / kPlanesTileTok;
      const int tile = ((span + n - 1) / n + 15) & ~15;
      for (int k = 0; k < n; ++k) {
        const int o = k * tile;
        const int e = k + 1 == n ? span : o + tile;
        p.plane_tiles[tpos++] = make_int4(i * 128 + o, e - o, info.x, k + 1 == n ? 1 : 0);
      }
    }
    if (p.pair_wide && c == kClassWideDirect && !continues(i)) {
      const int span = run_span(i);
      const int n = (span + kDirectTileTok - 1) / kDirectTileTok;
      const int tile = ((span + n - 1) / n + 15) & ~15;
      for (int k = 0; k < n; ++k) {
        const int o = k * tile;
        const int e = k + 1 == n ? span : o + tile;
        p.direct_tiles[dpos++] = make_int4(i * 128 + o, e - o, info.x, k + 1 == n ? 1 : 0);
      }
    }
  }
}

// =====================================================================================
// Persistent tcgen05 grouped GEMM, weights as the MMA's M side ("swap AB").
//
// A work tile is (128-row block of one expert, 128 output columns).  Per K step
// of 128 the producer issues three copies into one pipeline stage: the weight
// tile [128 n x 128 k] (TMA, 16U4_ALIGN16B type: packed E2M1 in global memory,
// one byte per element in shared memory, 128-byte swizzle), one 3-D TMA box
// holding both activation planes [hi TOK rows; lo TOK rows], and the weights'
// 512-byte scale atom (bulk copy).  The activation scale factor is the constant
// 1.0 (the planes carry the per-row power of two, applied by the epilogue).  One
// thread issues tcgen05.cp of the weight atom and, per 32-wide K slice,
// tcgen05.mma.kind::mxf8f6f4.block_scale: once over the stacked planes
// (N = 2*TOK) for TOK <= 32, or once per plane (N = ntok) for TOK = 128, into a
// TMEM accumulator of 128 lanes (n) x tokens.  Each tcgen05 instruction holds
// the tensor pipe ~45 cycles, so the issue stream per K step (1 cp, 4 or 8 MMAs,
// 1 commit) is kept minimal.  Four epilogue warps drain TMEM, add the hi and lo parts, cast to
// BF16 and store D[row, n]; rows of the block without the block's id, and blocks
// without any, are written as zeros.
//
// Warp roles: 0 = TMA producer, 1 = MMA issuer (also owns TMEM), 2-3 idle,
// 4-7 = epilogue.
// =====================================================================================
struct GemmArgs {
  const int4* blk_info;
  const uint4* blk_mask;
  const int* ctrl;
  const int4* list;       // blocks of this kernel's class, in order: {block, expert, rows spanned, 0}
  const int4* direct_list;  // tiles of cdg_gemm_direct_kernel (their token atoms: write_direct_atoms)
  const int4* zero_list;  // all-padding blocks (zero-filled by the kernel with do_zero_blocks)
  const uint32_t* sfw_atoms;  // [E][N/128][K/128][128] words
  const int32_t* row_exp;     // [nblk*128] per-row exponent of the activation planes
  const uint8_t* tok_code;    // [M][tok_code_pitch(K)] UE8M0 activation scale codes of direct-class rows
  uint32_t* tok_atoms;        // [direct tile][K/512][2][128] token scale atoms (write_direct_atoms)
  __nv_bfloat16* d;
  int64_t d_row_stride;
  int M, N, K, E, nblk;
  TileMap tm;            // rows of each block
  int count_slot;        // ctrl index of this class's block count
  int do_zero_blocks;
  int fill_rest;          // 1: zero the block's rows past its last routed row
  int* status;
  const uint64_t* d_rows;  // optional: D row r goes to the address d_rows[r] (not written when 0)
};

// Start of D row r: d + r * d_row_stride, or the address the row table lists (nullptr: the row
// is not written; an address that is not 16-byte aligned is not written either and raises
// kStatusBadIndex).
__device__ __forceinline__ __nv_bfloat16* d_row(const GemmArgs& p, int64_t r) {
  if (p.d_rows) {
    const uint64_t a = __ldg(p.d_rows + r);
    if (a & 15) {
      atomicOr(p.status, kStatusBadIndex);
      atomicOr(&g_sticky_status[0], kStatusBadIndex);
      return nullptr;
    }
    return reinterpret_cast<__nv_bfloat16*>(a);
  }
  return p.d + r * p.d_row_stride;
}

// Token scale atoms of the direct tiles, written by the kernel that runs before
// cdg_gemm_direct_kernel (the planes kernel, all its threads).  For tile i (list order) and
// scale stage st of four K steps, the 1024 bytes at tok_atoms + (i * stages + st) * 256 words:
// token slot n (0..255) at word (n/128)*128 + (n%32)*4 + (n%128)/32, the 4-byte word of its
// row's codes for the stage's K steps (byte j = K step j), 127 (scale 1) for slots past the
// tile.
__device__ __forceinline__ void write_direct_atoms(const GemmArgs& p) {
  const int count = __ldcg(&p.ctrl[kCtrlDirectTiles]);
  const int pitch = tok_code_pitch(p.K);
  const int stages = pitch / 4;
  const int items = count * 256;
  for (int it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += gridDim.x * blockDim.x) {
    const int i = it >> 8, n = it & 255;
    const int4 cur = __ldcg(&p.direct_list[i]);
    int brow0, bn;
    p.tm.rows(cur.x >> 7, brow0, bn);
    const int row = brow0 + (cur.x & 127) + n;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p.tok_code + static_cast<int64_t>(row) * pitch);
    uint32_t* dst = p.tok_atoms + static_cast<int64_t>(i) * stages * 256 + (n >> 7) * 128 + (n & 31) * 4 + ((n & 127) >> 5);
#pragma unroll 4
    for (int st = 0; st < stages; ++st) dst[st * 256] = n < cur.y ? __ldcg(src + st) : 0x7F7F7F7Fu;
  }
}

template <int TOK>
struct GemmSmem {
  static constexpr int kStages = TOK <= 16 ? 10 : TOK <= 32 ? 8 : 4;
  static constexpr int kW = 128 * 128;                   // weight tile, bytes per stage
  static constexpr int kA = TOK * 128;                   // one activation plane, bytes per stage
  static constexpr int kStageBytes = kW + 2 * kA + 1024;  // + weight scale atom (512 B, padded)
  static constexpr int kOneAtom = kStages * kStageBytes;  // constant activation scale atom (all 127)
  static constexpr int kBarOffset = kOneAtom + 512;
  static constexpr int kBytes = kBarOffset + 256 + 1024;  // + barriers + alignment slack
};

template <int TOK>
__global__ void __launch_bounds__(256, 1)
    cdg_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                    GemmArgs p) {
  using L = GemmSmem<TOK>;
  constexpr int S = L::kStages;
  // TOK <= 32: the two planes are stacked along N ([hi rows; lo rows], N = 2*TOK), so one
  // MMA per K slice covers both; TOK = 128: one MMA per plane (N = ntok).
  constexpr bool kStacked = TOK <= 32;
  constexpr uint32_t kAccCols = 128;  // TMEM columns per accumulator stage

  grid_dependency_wait();  // the block plan comes from the previous kernel of the stream
  grid_launch_dependents();
  const int n_tiles = p.N / 128;
  const int k_steps = p.K / 128;
  const int count = __ldcg(&p.ctrl[p.count_slot]);
  const int zero_count = p.do_zero_blocks ? __ldcg(&p.ctrl[kCtrlCount0 + kClassZero]) : 0;
  const int reg_tiles = count * n_tiles;
  const int total_tiles = reg_tiles + zero_count * n_tiles;
  if (total_tiles == 0) return;  // nothing of this class in the call: leave before any set-up

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto stage_w = [&](int s) { return smem + s * L::kStageBytes; };
  auto stage_a = [&](int s) { return smem + s * L::kStageBytes + L::kW; };  // [hi TOK rows][lo TOK rows]
  auto stage_sf = [&](int s) { return smem + s * L::kStageBytes + L::kW + 2 * L::kA; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;       // [S] stage landed
  uint64_t* empty = bars + S;  // [S] stage consumed
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tfull + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kTmemCols = 512;
  // Weight scale-factor columns, double-buffered by K-step parity so that the copy
  // for step kb+1 does not overwrite what the MMAs of step kb still read; the
  // activation scale factor is the constant 1.0 (byte 127), copied once.
  constexpr uint32_t kSfwCol = 256, kSfSetCols = 4, kSfaCol = 264;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_a);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 128);
    }
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2) {
    reinterpret_cast<uint32_t*>(smem + L::kOneAtom)[lane] = 0x7F7F7F7Fu;
    reinterpret_cast<uint32_t*>(smem + L::kOneAtom)[lane + 32] = 0x7F7F7F7Fu;
    reinterpret_cast<uint32_t*>(smem + L::kOneAtom)[lane + 64] = 0x7F7F7F7Fu;
    reinterpret_cast<uint32_t*>(smem + L::kOneAtom)[lane + 96] = 0x7F7F7F7Fu;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to tcgen05.cp
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      // the next tile's list entry is loaded one tile ahead, off the issue path
      int4 next = blockIdx.x < reg_tiles ? __ldg(&p.list[blockIdx.x / n_tiles]) : make_int4(0, 0, 0, 0);
      for (int t = blockIdx.x; t < reg_tiles && ok; t += gridDim.x) {
        const int4 cur = next;
        if (t + static_cast<int>(gridDim.x) < reg_tiles) next = __ldg(&p.list[(t + gridDim.x) / n_tiles]);
        const int blk = cur.x;
        const int nt = t % n_tiles;
        const int expert = cur.y;
        const int wrow = expert * p.N + nt * 128;
        const uint32_t* sfw_tile = p.sfw_atoms + (static_cast<int64_t>(expert) * n_tiles + nt) * k_steps * 128;
        for (int kb = 0; kb < k_steps; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], 128u * 64u + 2u * L::kA + 512u);
          tma_load_2d(stage_w(stage), &tmap_w, &full[stage], kb * 128, wrow);
          tma_load_3d(stage_a(stage), &tmap_a, &full[stage], kb * 128, blk * 128, 0);
          bulk_load(stage_sf(stage), sfw_tile + kb * 128, 512, &full[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: wait (bounded) until the copies of every stage issued so far landed.
      if (!ok) {
        for (int s = 0; s < S; ++s) mbar_wait(&full[s], 0, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      const uint32_t sfa_t = tmem_base + kSfaCol;
      tc_cp_sf_atom(sfa_t, smem_desc_sf(smem_u32(smem + L::kOneAtom)));
      int4 next = blockIdx.x < reg_tiles ? __ldg(&p.list[blockIdx.x / n_tiles]) : make_int4(0, 0, 0, 0);
      for (int t = blockIdx.x; t < reg_tiles && ok; t += gridDim.x, ++local) {
        const int4 cur = next;
        if (t + static_cast<int>(gridDim.x) < reg_tiles) next = __ldg(&p.list[(t + gridDim.x) / n_tiles]);
        const uint32_t ntok = static_cast<uint32_t>((cur.z + 15) & ~15);
        const uint32_t n_mma = kStacked ? 2u * TOK : ntok;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        for (int kb = 0; kb < k_steps; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sfw_t = tmem_base + kSfwCol + (kb & 1) * kSfSetCols;
          tc_cp_sf_atom(sfw_t, smem_desc_sf(smem_u32(stage_sf(stage))));
          const uint32_t w_addr = smem_u32(stage_w(stage));
          const uint32_t a_addr = smem_u32(stage_a(stage));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t wd = smem_desc_sw128(w_addr + k * 32);
            const uint32_t idesc = idesc_mxf8f6f4(/*a=E2M1*/ 5, /*b=E4M3*/ 0, 128, n_mma, k, k);
            const uint32_t accumulate = (kb | k) != 0 ? 1u : 0u;
            tc_mma_mxf8f6f4(d_tmem, wd, smem_desc_sw128(a_addr + k * 32), idesc, accumulate, sfw_t, sfa_t);
            if (!kStacked)
              tc_mma_mxf8f6f4(d_tmem, wd, smem_desc_sw128(a_addr + L::kA + k * 32), idesc, 1u, sfw_t, sfa_t);
          }
          tc_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int tid = threadIdx.x - 128;
    int local = 0;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      const bool regular = t < reg_tiles;
      const int blk = regular ? __ldg(&p.list[t / n_tiles]).x : __ldg(&p.zero_list[(t - reg_tiles) / n_tiles]).x;
      const int nt = t % n_tiles;
      int row0, nrows;
      p.tm.rows(blk, row0, nrows);
      int zero_from = 0;
      if (regular) {
        const int4 info = p.blk_info[blk];
        const uint4 mask = p.blk_mask[blk];
        const int ntok = (info.y + 15) & ~15;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        ++local;
        // 2^E of the tile's rows, loaded before the accumulator wait: lane l holds rows l + 32k
        float row_sc[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          row_sc[k] = __uint_as_float(
              static_cast<uint32_t>(min(max(__ldg(p.row_exp + blk * 128 + k * 32 + lane) + 127, 1), 254)) << 23);
        if (!mbar_wait(&tfull[acc], acc_phase, p.status)) { ok = false; break; }
        tc_fence_after();
        const int n = nt * 128 + q * 32 + lane;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kAccCols;
        for (int j0 = 0; j0 < ntok; j0 += 16) {
          const int kq = j0 >> 5;  // which of the 32-row groups this chunk lies in
          const float my_scale = kq == 0 ? row_sc[0] : kq == 1 ? row_sc[1] : kq == 2 ? row_sc[2] : row_sc[3];
          uint32_t v[16];
          tmem_ld16(taddr + j0, v);
          if (kStacked) {
            uint32_t w[16];
            tmem_ld16(taddr + TOK + j0, w);  // the lo-plane columns of the same tokens
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
          } else {
            tmem_ld_wait();
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int r = row0 + j0 + j;
            const int rb = j0 + j;
            const uint32_t word = rb < 32 ? mask.x : rb < 64 ? mask.y : rb < 96 ? mask.z : mask.w;
            const float sc = __shfl_sync(0xffffffffu, my_scale, (j0 & 31) + j);
            if (rb < nrows) {
              const float x = ((word >> (rb & 31)) & 1u) ? __uint_as_float(v[j]) * sc : 0.0f;
              __nv_bfloat16* rp = d_row(p, r);
              if (rp) rp[n] = __float2bfloat16_rn(x);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        zero_from = ntok;
      }
      // zero rows [zero_from, 128) of this block, columns [nt*128, nt*128+128), 16 B per store
      const int rows = p.fill_rest ? nrows - zero_from : 0;
      const uint4 z = make_uint4(0, 0, 0, 0);
      for (int c = tid; c < rows * 16; c += 128) {
        const int r = row0 + zero_from + (c >> 4);
        __nv_bfloat16* rp = d_row(p, r);
        if (rp) *reinterpret_cast<uint4*>(rp + nt * 128 + (c & 15) * 8) = z;
      }
    }
  }

  if (p.d_rows) __threadfence_system();  // rows stored into other GPUs' memory
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// =====================================================================================
// Generic exact path (SIMT).  One CTA per (128-row block, 256 output columns).
// Follows the reference's arithmetic element by element: activations as
// bf16(bf16(a) * bf16(sa)) for e4m3, unchanged for BF16/FP32 (gemm.py:31-52);
// weights as bf16(e2m1 * scale) with scale 2^(e-127) or a float (gemm.py:147-187);
// FP32 accumulation; result cast to D's dtype.  Rows whose id is outside [0, E)
// are written as zeros.  Used for the blocks the tensor-core kernel does not take
// (rows of several experts in one 128-row block) and for inputs outside its
// envelope (K or N not multiples of 128, BF16/FP32 activations, float weight
// scales, FP32 output).
// =====================================================================================
struct GenericArgs {
  const void* a;
  int a_dtype;  // CDG_DTYPE_*
  int64_t a_row_stride;
  const float* sa;
  int64_t sa_stride_m, sa_stride_k;
  int sa_block_k;   // K columns per scale (FP32 scales); 128 for packed UE8M0
  int sa_packed;    // 1: sa holds int32 words of 4 UE8M0 scales
  const uint8_t* b;  // packed [E][N][K/2]
  int64_t b_stride_e, b_stride_n;
  const void* sb;
  int sb_dtype;   // CDG_DTYPE_UE8M0 or CDG_DTYPE_F32
  int sb_atoms;   // 1: sb is in the 128x4 atom layout of cdg_sf_atom_kernel (UE8M0 only)
  int64_t sb_stride_e, sb_stride_n;
  const void* ids;
  int ids_is_64;
  void* d;
  int d_dtype;  // CDG_DTYPE_BF16 or CDG_DTYPE_F32
  int64_t d_row_stride;
  int M, N, K, E;
  int nblk;
  TileMap tm;        // rows of each block
  const int4* list;  // nullptr: every block; else the listed blocks ({block, ...})
  const int* count;  // number of listed blocks (device)
  const uint64_t* d_rows;  // optional row table, as in GemmArgs (BF16 output)
};

__constant__ float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(256) cdg_generic_kernel(GenericArgs p) {
  extern __shared__ float s_row[];  // K floats: the dequantised activation row
  grid_dependency_wait();  // the block list comes from the previous kernel of the stream
  const int n_chunks = (p.N + 255) / 256;
  const int units = (p.list ? __ldcg(p.count) : p.nblk) * n_chunks;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int bi = u / n_chunks;
    const int blk = p.list ? p.list[bi].x : bi;
    const int n = (u % n_chunks) * 256 + threadIdx.x;
    int row0, nrows;
    p.tm.rows(blk, row0, nrows);
    for (int r = row0; r < row0 + nrows; ++r) {
      const int64_t id = load_id(p.ids, p.ids_is_64, r);
      const bool valid = id >= 0 && id < p.E;
      if (valid) {
        __syncthreads();
        for (int k = threadIdx.x; k < p.K; k += blockDim.x) {
          float x;
          if (p.a_dtype == CDG_DTYPE_E4M3) {
            const uint8_t raw = static_cast<const uint8_t*>(p.a)[r * p.a_row_stride + k];
            const float s = bf16r(load_sa(p.sa, p.sa_packed, p.sa_stride_m, p.sa_stride_k, r, k / p.sa_block_k));
            x = bf16r(e4m3_to_f32(raw) * s);
          } else if (p.a_dtype == CDG_DTYPE_BF16) {
            x = __bfloat162float(static_cast<const __nv_bfloat16*>(p.a)[r * p.a_row_stride + k]);
          } else {
            x = static_cast<const float*>(p.a)[r * p.a_row_stride + k];
          }
          s_row[k] = x;
        }
        __syncthreads();
      }
      if (n >= p.N) continue;
      float acc = 0.0f;
      if (valid) {
        const uint8_t* wrow = p.b + id * p.b_stride_e + static_cast<int64_t>(n) * p.b_stride_n;
        for (int k = 0; k < p.K; k += 2) {
          const uint8_t byte = __ldg(wrow + (k >> 1));
          float sc;
          const int kb = k >> 5;
          if (p.sb_atoms) {
            const int64_t atom = (id * ((p.N + 127) / 128) + n / 128) * ((p.K / 32 + 3) / 4) + (kb >> 2);
            const uint8_t e = static_cast<const uint8_t*>(p.sb)[atom * 512 + (n & 31) * 16 + ((n & 127) >> 5) * 4 +
                                                                (kb & 3)];
            sc = ue8m0_to_f32(e);
          } else if (p.sb_dtype == CDG_DTYPE_UE8M0) {
            const uint8_t e = static_cast<const uint8_t*>(p.sb)[id * p.sb_stride_e + n * p.sb_stride_n + kb];
            sc = ue8m0_to_f32(e);
          } else {
            sc = static_cast<const float*>(p.sb)[id * p.sb_stride_e + n * p.sb_stride_n + kb];
          }
          acc = fmaf(s_row[k], bf16r(kE2M1[byte & 15] * sc), acc);
          if (k + 1 < p.K) acc = fmaf(s_row[k + 1], bf16r(kE2M1[byte >> 4] * sc), acc);
        }
      }
      if (p.d_rows) {
        const uint64_t a = __ldg(p.d_rows + r);
        if (a & 15) {
          atomicOr(&g_sticky_status[0], kStatusBadIndex);
        } else if (a) {
          reinterpret_cast<__nv_bfloat16*>(a)[n] = __float2bfloat16_rn(acc);
        }
      } else if (p.d_dtype == CDG_DTYPE_BF16) {
        static_cast<__nv_bfloat16*>(p.d)[r * p.d_row_stride + n] = __float2bfloat16_rn(acc);
      } else {
        static_cast<float*>(p.d)[r * p.d_row_stride + n] = acc;
      }
    }
  }
  if (p.d_rows) __threadfence_system();  // rows stored into other GPUs' memory
}

}  // namespace cdg
