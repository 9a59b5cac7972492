// CTA-pair tcgen05 kernel for the direct class: wide blocks (more than 32 routed rows of one
// expert, or the tail block of an expert spanning several blocks) whose activation scales are
// all powers of two.
//
// A cluster of two CTAs computes a pair tile: 256 weight rows of one expert (CTA r holds
// output-column tile 2*pt + r) x the block's tokens, with tcgen05.mma.cta_group::2
// (M = 256, weights as the MMA's A operand: "swap AB").  The tokens are the MMA's N side:
// N = 2h, h = the block's routed span halved and rounded up to 16; CTA 0 holds tokens
// [0, h), CTA 1 tokens [h, 2h) of every K step, the e4m3 rows of A themselves (one MMA per
// 32-wide K slice).  The reference's bf16(bf16(a) * bf16(2^s)) is then the exact product
// a * 2^s, which the tensor core forms from the raw rows with 2^s as the MMA's B scale factor:
// the prep kernel writes a 512-byte UE8M0 atom per (block, K step), so the accumulator holds
// the final values and the epilogue only converts and stores.
//
// Pipeline: a stage holds kKS = 2 K steps (weights, tokens, weight and token scale atoms of
// each), so the MMA issuer waits on one barrier per two K steps.  The scale atoms reach TMEM
// through a second thread (tcgen05.cp into the stage's own TMEM scale columns, then a commit
// to the stage's `sfready` barrier), so the MMA warp issues nothing but MMAs and commits; the
// MMA loop runs on the whole warp with each instruction issued by its elected lane.  A
// stage's scale columns are free again when its data lands the next time: the producer
// refills a stage only after the MMAs that read it completed.
//
// Epilogue (four warps per CTA, warp q owns TMEM lanes 32q..32q+31 = output columns):
// tcgen05.ld 16x256b hands each thread two adjacent tokens of one column; packed to
// bf16x2 these are the fragments of 8x8 [column][token] matrices, and stmatrix.trans
// stores their transposes, i.e. [token][8 columns] 16-byte rows of D, into a swizzled
// per-warp staging tile; the warp then writes the staged D rows with 16-byte stores
// (rows past the block's end skipped, rows without the block's expert written as zeros).
//
// Warp roles per CTA: 0 = TMA producer, 1 = MMA issuer (even CTA) and TMEM owner,
// 2 = scale-factor copier (even CTA), 3 idle, 4-7 = epilogue.  All waits are bounded
// (kStatusTimeout).
#pragma once

#include "cdg_kernels.cuh"

namespace cdg {

struct WideSmem {
  static constexpr int kKS = 2;                    // K steps per stage
  static constexpr int kW = 128 * 128;             // weight tile per K step (E2M1 unpacked to bytes)
  static constexpr int kA = 64 * 128;              // 64 token rows per K step
  static constexpr int kStep = kW + kA;            // operand bytes per K step
  static constexpr int kStages = 4;
  static constexpr int kStageBytes = kKS * kStep;
  static constexpr int kSfRing = kStages * kStageBytes;            // [stage][kKS] weight scale atoms
  static constexpr int kTsfRing = kSfRing + kStages * kKS * 512;   // [stage][kKS] token scale atoms
  static constexpr int kStaging = kTsfRing + kStages * kKS * 512;  // 4 warps x [16 tokens][32 columns] bf16
  static constexpr int kBarOffset = kStaging + 4 * 1024;
  static constexpr int kBarBytes = (3 * kStages + 5) * 8 + 16;  // full, empty, sfready, tfull[2], tempty[2], done; TMEM
  static constexpr int kBytes = kBarOffset + kBarBytes + 1024;  // + alignment slack
  static_assert(kBytes <= 232448, "shared memory per CTA");
  static_assert(kStep % 1024 == 0, "K steps must stay 1024-byte aligned for SW128 tiles");
  // bytes one CTA's copies of one K step add to the even CTA's `full` barrier
  static constexpr uint32_t kTxPerStep = 128u * 64u + kA + 512u + 512u;
  // TMEM: two 128-column accumulators, then [stage][kKS] 4-column weight scale sets and
  // [stage][kKS] 4-column token scale sets
  static constexpr uint32_t kSfwCol = 256;
  static constexpr uint32_t kTsfCol = kSfwCol + kStages * kKS * 4;
  static_assert(kTsfCol + kStages * kKS * 4 <= 512, "TMEM columns");
  static constexpr int kThreads = 256;
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    cdg_gemm_wide_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_sfw, const __grid_constant__ CUtensorMap tmap_tsf,
                         GemmArgs p) {
  using L = WideSmem;
  constexpr int S = L::kStages;
  constexpr int KS = L::kKS;
  constexpr uint32_t kTmemCols = 512;

  grid_dependency_wait();  // the block plan comes from the previous kernel of the stream
  grid_launch_dependents();
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int n_tiles = p.N / 128;
  const int n_pt = p.N / 256;  // pair tiles per block
  const int k_steps = p.K / 128;
  const int count = __ldcg(&p.ctrl[p.count_slot]);
  const int tiles = count * n_pt;
  if (tiles == 0) return;  // both CTAs of the pair read the same count and leave together

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto step_w = [&](int s, int u) { return smem + s * L::kStageBytes + u * L::kStep; };
  auto step_a = [&](int s, int u) { return smem + s * L::kStageBytes + u * L::kStep + L::kW; };
  auto step_sfw = [&](int s, int u) { return smem + L::kSfRing + (s * KS + u) * 512; };
  auto step_tsf = [&](int s, int u) { return smem + L::kTsfRing + (s * KS + u) * 512; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;           // [S] even CTA: both CTAs' copies of a stage landed
  uint64_t* empty = bars + S;      // [S] stage consumed (multicast by the MMA commit)
  uint64_t* sfready = bars + 2 * S;  // [S] even CTA: the stage's scale atoms are in TMEM
  uint64_t* tfull = bars + 3 * S;  // [2] accumulator complete
  uint64_t* tempty = tfull + 2;    // [2] even CTA: all 256 epilogue threads of the pair drained it
  uint64_t* done = tempty + 2;     // even CTA: every MMA completed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_sfw);
    prefetch_tmap(&tmap_tsf);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sfready[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 256);
    }
    mbar_init(done, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised before any copy or commit reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool ok = true;

  // Tokens per CTA of a block spanning `rows` rows: half, rounded up to 16 (N = 2h, a
  // multiple of 32).
  auto wide_half = [](int rows) { return (((rows + 1) >> 1) + 15) & ~15; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t full0 = cluster_addr(&full[0], 0);
      int4 next = pair < tiles ? __ldg(&p.list[pair / n_pt]) : make_int4(0, 0, 0, 0);
      for (int t = pair; t < tiles && ok; t += npairs) {
        const int4 cur = next;
        if (t + npairs < tiles) next = __ldg(&p.list[(t + npairs) / n_pt]);
        const int blk = cur.x;
        const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
        const int wrow = cur.y * p.N + nt * 128;
        const int atom0 = (cur.y * n_tiles + nt) * k_steps;
        int row0, nrows;
        p.tm.rows(blk, row0, nrows);
        const int a_row = row0 + static_cast<int>(rank) * wide_half(cur.z);  // rows of A itself
        for (int kb0 = 0; kb0 < k_steps; kb0 += KS) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1, p.status,
                                 wait_code(1, static_cast<int>(rank), stage, phase ^ 1, kb0))) {
            ok = false;
            break;
          }
          const int n = k_steps - kb0 < KS ? k_steps - kb0 : KS;
          const uint32_t fb = full0 + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2u * static_cast<uint32_t>(n) * L::kTxPerStep);
          for (int u = 0; u < n; ++u) {
            const int kb = kb0 + u;
            tma_load_2d_pair(step_w(stage, u), &tmap_w, fb, kb * 128, wrow);
            tma_load_2d_pair(step_a(stage, u), &tmap_a, fb, kb * 128, a_row);
            tma_load_2d_pair(step_sfw(stage, u), &tmap_sfw, fb, 0, atom0 + kb);
            tma_load_2d_pair(step_tsf(stage, u), &tmap_tsf, fb, 0, blk * k_steps + kb);
          }
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA, whole warp)
    if (rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      int4 next = pair < tiles ? __ldg(&p.list[pair / n_pt]) : make_int4(0, 0, 0, 0);
      for (int t = pair; t < tiles && ok; t += npairs, ++local) {
        const int4 cur = next;
        if (t + npairs < tiles) next = __ldg(&p.list[(t + npairs) / n_pt]);
        const uint32_t n_mma = 2u * static_cast<uint32_t>(wide_half(cur.z));
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_cluster_warp(&tempty[acc], acc_phase ^ 1, p.status, wait_code(2, 0, acc, acc_phase ^ 1, local))) {
          ok = false;
          break;
        }
        const uint32_t d_tmem = tmem_base + acc * 128;
        uint32_t idk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) idk[k] = idesc_mxf8f6f4(/*a=E2M1*/ 5, /*b=E4M3*/ 0, 256, n_mma, k, k);
        for (int kb0 = 0; kb0 < k_steps; kb0 += KS) {
          if (!mbar_wait_cta_warp(&sfready[stage], phase, p.status, wait_code(3, 0, stage, phase, kb0))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int n = k_steps - kb0 < KS ? k_steps - kb0 : KS;
          for (int u = 0; u < n; ++u) {
            const uint32_t sfw_t = tmem_base + L::kSfwCol + (stage * KS + u) * 4;
            const uint32_t tsf_t = tmem_base + L::kTsfCol + (stage * KS + u) * 4;
            const uint64_t wd0 = smem_desc_sw128(smem_u32(step_w(stage, u)));
            const uint64_t ad0 = smem_desc_sw128(smem_u32(step_a(stage, u)));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // descriptor start addresses are in 16-byte units: +32 bytes per K slice
              tc_mma_mxf8f6f4_pair_warp(d_tmem, wd0 + 2 * k, ad0 + 2 * k, idk[k],
                                        (kb0 + u != 0 || k != 0) ? 1u : 0u, sfw_t, tsf_t);
            }
          }
          tc_commit_pair_warp(&empty[stage], 0x3);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair_warp(&tfull[acc], 0x3);
      }
      // Every MMA (and its TMEM writes in both CTAs) completes before teardown.
      tc_commit_pair_warp(done, 0x1);
      mbar_wait_cluster_warp(done, 0, p.status, wait_code(5, 0, 0, 0, 0));
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ scale-factor copier (even CTA, whole warp)
    if (rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < tiles && ok; t += npairs) {
        for (int kb0 = 0; kb0 < k_steps; kb0 += KS) {
          if (!mbar_wait_cta_warp(&full[stage], phase, p.status, wait_code(6, 0, stage, phase, kb0))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int n = k_steps - kb0 < KS ? k_steps - kb0 : KS;
          for (int u = 0; u < n; ++u) {
            tc_cp_sf_atom_pair_warp(tmem_base + L::kSfwCol + (stage * KS + u) * 4,
                                    smem_desc_sf(smem_u32(step_sfw(stage, u))));
            tc_cp_sf_atom_pair_warp(tmem_base + L::kTsfCol + (stage * KS + u) * 4,
                                    smem_desc_sf(smem_u32(step_tsf(stage, u))));
          }
          tc_commit_pair_warp(&sfready[stage], 0x1);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int tid = threadIdx.x - 128;
    const uint32_t tempty0 = cluster_addr(&tempty[0], 0);
    uint8_t* wst = smem + L::kStaging + q * 1024;  // [16 tokens][4 x 16-byte column chunks], swizzled
    const uint32_t wst_u32 = smem_u32(wst);
    // stmatrix row addresses: thread 8k + i gives row i of matrix k, i.e. token i + 8*(k/2),
    // column chunk (k%2) (+2 for the second 16-lane half); chunk c of row r sits at c ^ ((r/2)%4)
    const int sm_row = (lane & 7) + 8 * (lane >> 4);
    const int sm_chunk = (lane >> 3) & 1;
    const uint32_t sm_addr0 = wst_u32 + sm_row * 64 + ((sm_chunk ^ ((sm_row >> 1) & 3)) << 4);
    const uint32_t sm_addr1 = wst_u32 + sm_row * 64 + (((sm_chunk + 2) ^ ((sm_row >> 1) & 3)) << 4);
    int local = 0;
    for (int t = pair; t < tiles && ok; t += npairs, ++local) {
      const int blk = __ldg(&p.list[t / n_pt]).x;
      const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
      int row0, nrows;
      p.tm.rows(blk, row0, nrows);
      const int4 info = p.blk_info[blk];
      const uint4 mask = p.blk_mask[blk];
      const int ntok = (info.y + 15) & ~15;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_cluster(&tfull[acc], acc_phase, p.status,
                             wait_code(4, static_cast<int>(rank), acc, acc_phase, local))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * 128;
      __nv_bfloat16* dcol = p.d + nt * 128 + q * 32;
      for (int j0 = 0; j0 < ntok; j0 += 16) {
        uint32_t lo[8], hi[8];
        tmem_ld_16x256b_x2(taddr + j0, lo);                  // lanes 0-15 of the quadrant
        tmem_ld_16x256b_x2(taddr + (16u << 16) + j0, hi);    // lanes 16-31
        tmem_ld_wait();
        uint32_t m[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          __nv_bfloat162 a = __floats2bfloat162_rn(__uint_as_float(lo[2 * k]), __uint_as_float(lo[2 * k + 1]));
          __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(hi[2 * k]), __uint_as_float(hi[2 * k + 1]));
          m[k] = *reinterpret_cast<uint32_t*>(&a);
          m[4 + k] = *reinterpret_cast<uint32_t*>(&b);
        }
        // matrices: (columns 0-7 | 8-15, tokens 0-7 | 8-15) of each 16-lane half
        stmatrix_x4_trans(sm_addr0, m[0], m[1], m[2], m[3]);
        stmatrix_x4_trans(sm_addr1, m[4], m[5], m[6], m[7]);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int vi = lane + 32 * i, rr = vi >> 2, part = vi & 3;
          const int tok = j0 + rr;
          if (tok < nrows) {
            const uint32_t word = tok < 32 ? mask.x : tok < 64 ? mask.y : tok < 96 ? mask.z : mask.w;
            uint4 v = make_uint4(0, 0, 0, 0);
            if ((word >> (tok & 31)) & 1u)
              v = *reinterpret_cast<const uint4*>(wst + rr * 64 + ((part ^ ((rr >> 1) & 3)) << 4));
            *reinterpret_cast<uint4*>(dcol + static_cast<int64_t>(row0 + tok) * p.d_row_stride + part * 8) = v;
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      if (rank == 0)
        mbar_arrive(&tempty[acc]);
      else
        mbar_arrive_cluster(tempty0 + acc * 8);
      // rows of the block past its last routed row
      const int rows = p.fill_rest ? nrows - ntok : 0;
      const uint4 z = make_uint4(0, 0, 0, 0);
      for (int c = tid; c < rows * 16; c += 128) {
        const int r = row0 + ntok + (c >> 4);
        *reinterpret_cast<uint4*>(p.d + static_cast<int64_t>(r) * p.d_row_stride + nt * 128 + (c & 15) * 8) = z;
      }
    }
  }

  tc_fence_before();
  const int any_fail = __syncthreads_or(!ok);
  cluster_sync();  // no CTA releases TMEM or exits while its pair still uses it
  if (any_fail) {
    // after a timeout, copies issued before it still land: give them time before exit
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 200000ull) __nanosleep(20000);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace cdg
