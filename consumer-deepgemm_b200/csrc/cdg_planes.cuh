// CTA-pair tcgen05 kernel for wide blocks carried by activation planes (blocks with more
// than 32 routed rows of one expert whose activation scales are not all powers of two,
// and the tail blocks of experts that span several blocks).
//
// Work is cut by tokens, not by blocks: the prep kernel joins consecutive wide blocks of
// one expert into runs and cuts each run into tiles of up to kPlanesTileTok = 112 rows (a
// tile may cross a block boundary; the planes, row exponents and D rows of a run are
// contiguous).  A cluster of two CTAs computes a pair tile: 256 weight rows of the expert
// (CTA r holds output-column tile 2*pt + r) x the tile's tokens, with
// tcgen05.mma.cta_group::2 (M = 256, weights as the MMA's A operand: "swap AB").
//
// The token operand is the two e4m3 planes hi, lo of the BF16-dequantised rows (each row
// divided by 2^E, E per row from the prep kernel), stacked in the MMA's N dimension so that
// one MMA per 32-wide K slice covers both: each CTA holds h tokens (CTA 0 the tile's tokens
// [0, h), CTA 1 [h, 2h), h = half the tile rounded up to 8) as groups of 8 tokens, each
// group 8 hi rows followed by its 8 lo rows, N = 4h <= 224.  A 4-D view of the planes array
// brings that order straight from the stacked [hi rows][lo rows] layout in global memory.
// Accumulator column 16g + j (j < 8) then holds the hi part and 16g + 8 + j the lo part of
// token 8g + j; the epilogue adds them and multiplies by 2^E.  The token scale factor of the
// MMA is the constant 1.0 (eight TMEM columns of UE8M0 127, written once).
//
// Issue rate.  A single thread needs ~50 cycles to issue one tcgen05.mma (measured, with
// the issuing loop run by the whole warp and the instruction by its elected lane), while an
// M = 256, N = 128 MMA of K = 32 takes ~64 cycles of tensor pipe: two MMAs per K slice of
// N = 128 (one per plane) kept the pipe ~70% busy.  One MMA of N = 224 per K slice gives the
// issuer room for its waits.  TMEM then holds two accumulators of 224 columns (the epilogue
// drains one while the MMAs fill the other), the weight scale ring and the constant token
// scale columns: 504 of 512 columns.  (Tiles of 128 tokens, N = 256, leave room for one
// accumulator only; the tensor pipe then idled while the epilogue drained it.)
//
// Scale factors.  The weight scale atoms travel in their own ring (3 stages of 4 K steps,
// against 3 operand stages of 2), loaded by a producer thread of their own and copied to
// TMEM by a third thread (tcgen05.cp) as soon as the MMAs that used the TMEM slot last
// completed.  Their copies therefore enter the tensor pipe well ahead of the MMAs that read
// them; loaded together with the operands, the copy of stage s+1 sat behind the MMAs of
// stage s and the issuer waited for it every stage.
//
// Warp roles per CTA: 0 = operand TMA producer, 1 = MMA issuer (even CTA, whole warp) and
// TMEM owner, 2 = scale-factor copier (even CTA, whole warp), 3 = scale-atom TMA producer,
// 4-11 = epilogue (two warps per TMEM lane quadrant, each taking every other group of 8
// tokens).  All waits are bounded (kStatusTimeout).
#pragma once

#include "cdg_kernels.cuh"

namespace cdg {

#ifndef CDG_PLANES_KS
#define CDG_PLANES_KS 2
#endif
#ifndef CDG_PLANES_STAGES
#define CDG_PLANES_STAGES 3
#endif
#ifndef CDG_PLANES_KSF
#define CDG_PLANES_KSF 4
#endif
#ifndef CDG_PLANES_SF_STAGES
#define CDG_PLANES_SF_STAGES 3
#endif
#ifndef CDG_PLANES_EPI_WARPS
#define CDG_PLANES_EPI_WARPS 8
#endif

struct PlanesSmem {
  static constexpr int kKS = CDG_PLANES_KS;       // K steps per operand stage
  static constexpr int kKSF = CDG_PLANES_KSF;     // K steps per scale-atom stage
  static constexpr int kW = 128 * 128;            // weight tile per K step (E2M1 unpacked to bytes)
  static constexpr int kA = kPlanesTileTok * 128;  // 56 tokens x 2 planes per K step
  static constexpr int kStep = kW + kA;
  static constexpr int kStages = CDG_PLANES_STAGES;
  static constexpr int kSfStages = CDG_PLANES_SF_STAGES;
  static constexpr int kStageBytes = kKS * kStep;
  static constexpr int kSfRing = kStages * kStageBytes;              // [kSfStages][kKSF] weight scale atoms
  static constexpr int kConstSf = kSfRing + kSfStages * kKSF * 512;  // 512 bytes of UE8M0 127
  static constexpr int kEpiWarps = CDG_PLANES_EPI_WARPS;             // kEpiSets per TMEM lane quadrant
  static constexpr int kEpiSets = kEpiWarps / 4;
  static_assert(kEpiWarps % 4 == 0, "whole sets of four quadrant warps");
  static constexpr int kStaging = kConstSf + 512;                    // kEpiWarps x [8 tokens][32 columns] bf16
  static constexpr int kBarOffset = kStaging + kEpiWarps * 512;
  // full, empty; sffull, sfready, sftfree; tfull[2], tempty[2], done
  static constexpr int kNumBars = 2 * kStages + 3 * kSfStages + 5;
  static constexpr int kBarBytes = kNumBars * 8 + 16;                // + TMEM address
  static constexpr int kBytes = kBarOffset + kBarBytes + 1024;      // + alignment slack
  static_assert(kBytes <= 232448, "shared memory per CTA");
  static_assert(kStep % 1024 == 0, "K steps must stay 1024-byte aligned for SW128 tiles");
  static_assert(kKSF % kKS == 0, "an operand stage lies in one scale-atom stage");
  // bytes one CTA's operand copies of one K step add to the even CTA's `full` barrier
  static constexpr uint32_t kTxPerStep = 128u * 64u + kA;
  // TMEM: two accumulators of 2 x kPlanesTileTok columns, the weight scale ring, eight
  // constant token scale columns
  static constexpr uint32_t kAccCols = 2 * kPlanesTileTok;
  static constexpr uint32_t kSfwCol = 2 * kAccCols;
  static constexpr uint32_t kConstCol = kSfwCol + kSfStages * kKSF * 4;
  static_assert(kConstCol + 8 <= 512, "TMEM columns");
  static constexpr int kThreads = 128 + 32 * kEpiWarps;
};

// Tensor maps of the planes, one per box height: m[g - 1] brings g groups of 8 tokens.
struct PlaneMaps {
  CUtensorMap m[kPlanesTileTok / 16];
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PlanesSmem::kThreads, 1)
    cdg_gemm_planes_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ PlaneMaps tmaps_a,
                           const __grid_constant__ CUtensorMap tmap_sfw, GemmArgs p) {
  using L = PlanesSmem;
  constexpr int S = L::kStages;
  constexpr int RS = L::kSfStages;
  constexpr int KS = L::kKS;
  constexpr int KSF = L::kKSF;
  constexpr uint32_t kTmemCols = 512;

  grid_dependency_wait();  // the tile list comes from the previous kernel of the stream
  grid_launch_dependents();
  write_direct_atoms(p);  // for cdg_gemm_direct_kernel, which runs next
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int n_tiles = p.N / 128;
  const int n_pt = p.N / 256;  // pair tiles per token tile
  const int k_steps = p.K / 128;
  const int count = __ldcg(&p.ctrl[p.count_slot]);
  const int tiles = count * n_pt;
  if (tiles == 0) return;  // both CTAs of the pair read the same count and leave together

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto step_w = [&](int s, int u) { return smem + s * L::kStageBytes + u * L::kStep; };
  auto step_a = [&](int s, int u) { return smem + s * L::kStageBytes + u * L::kStep + L::kW; };
  auto step_sfw = [&](int s, int u) { return smem + L::kSfRing + (s * KSF + u) * 512; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;                // [S] even CTA: both CTAs' operand copies of a stage landed
  uint64_t* empty = bars + S;           // [S] stage consumed (multicast by the MMA commit)
  uint64_t* sffull = bars + 2 * S;      // [RS] even CTA: both CTAs' scale atoms of a stage landed
  uint64_t* sfready = sffull + RS;      // [RS] the stage's scale atoms are in TMEM (multicast)
  uint64_t* sftfree = sfready + RS;     // [RS] even CTA: the MMAs that read the TMEM slot completed
  uint64_t* tfull = sftfree + RS;       // [2] accumulator complete (multicast)
  uint64_t* tempty = tfull + 2;         // [2] even CTA: all epilogue threads of the pair drained it
  uint64_t* done = tempty + 2;          // even CTA: every MMA completed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    for (int g = 0; g < kPlanesTileTok / 16; ++g) prefetch_tmap(&tmaps_a.m[g]);
    prefetch_tmap(&tmap_sfw);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(&sffull[s], 1);
      mbar_init(&sfready[s], 1);
      mbar_init(&sftfree[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 2 * 32 * L::kEpiWarps);
    }
    mbar_init(done, 1);
    fence_mbarrier_init();
  }
  if (warp == 2) {  // the constant token scale factors, read by tcgen05.cp (async proxy)
    uint4* c = reinterpret_cast<uint4*>(smem + L::kConstSf);
    c[lane] = make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    fence_proxy_async_shared();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers and constant atoms ready before any copy or commit reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool ok = true;

  // Tokens per CTA of a tile of `rows` rows: half, rounded up to a group of 8 (N = 4h).
  auto tile_half = [](int rows) { return (((rows + 1) >> 1) + 7) & ~7; };

  if (warp == 0) {
    // ------------------------------------------------------------ operand TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t full0 = cluster_addr(&full[0], 0);
      int4 next = pair < tiles ? __ldg(&p.list[pair / n_pt]) : make_int4(0, 0, 0, 0);
      for (int t = pair; t < tiles && ok; t += npairs) {
        const int4 cur = next;
        if (t + npairs < tiles) next = __ldg(&p.list[(t + npairs) / n_pt]);
        const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
        const int wrow = cur.z * p.N + nt * 128;
        // plane rows of this CTA's tokens, in groups of 8; a box of just the tile's groups
        const int grp = (cur.x + static_cast<int>(rank) * tile_half(cur.y)) >> 3;
        const int ng_cta = tile_half(cur.y) >> 3;
        const CUtensorMap* tmap_a = &tmaps_a.m[ng_cta - 1];
        const uint32_t tx_step = 128u * 64u + static_cast<uint32_t>(ng_cta) * 2048u;
        for (int kb0 = 0; kb0 < k_steps; kb0 += KS) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1, p.status,
                                 wait_code(1, static_cast<int>(rank), stage, phase ^ 1, kb0))) {
            ok = false;
            break;
          }
          const int n = k_steps - kb0 < KS ? k_steps - kb0 : KS;
          const uint32_t fb = full0 + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2u * static_cast<uint32_t>(n) * tx_step);
          for (int u = 0; u < n; ++u) {
            const int kb = kb0 + u;
            tma_load_2d_pair(step_w(stage, u), &tmap_w, fb, kb * 128, wrow);
            tma_load_4d_pair(step_a(stage, u), tmap_a, fb, kb * 128, 0, 0, grp);
          }
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ scale-atom TMA producer (both CTAs)
    if (lane == 0) {
      int sfs = 0;
      uint32_t sfphase = 0;
      const uint32_t sffull0 = cluster_addr(&sffull[0], 0);
      int4 next = pair < tiles ? __ldg(&p.list[pair / n_pt]) : make_int4(0, 0, 0, 0);
      for (int t = pair; t < tiles && ok; t += npairs) {
        const int4 cur = next;  // read a tile ahead: the load stays off the tile boundary
        if (t + npairs < tiles) next = __ldg(&p.list[(t + npairs) / n_pt]);
        const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
        const int atom0 = (cur.z * n_tiles + nt) * k_steps;
        for (int kb0 = 0; kb0 < k_steps; kb0 += KSF) {
          // the copies out of this slot (RS stages ago) completed
          if (!mbar_wait_cluster(&sfready[sfs], sfphase ^ 1, p.status,
                                 wait_code(7, static_cast<int>(rank), sfs, sfphase ^ 1, kb0))) {
            ok = false;
            break;
          }
          const int n = k_steps - kb0 < KSF ? k_steps - kb0 : KSF;
          const uint32_t fb = sffull0 + sfs * 8;
          if (rank == 0) mbar_arrive_expect_tx(&sffull[sfs], 2u * static_cast<uint32_t>(n) * 512u);
          for (int u = 0; u < n; ++u) tma_load_2d_pair(step_sfw(sfs, u), &tmap_sfw, fb, 0, atom0 + kb0 + u);
          if (++sfs == RS) { sfs = 0; sfphase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA, whole warp)
    if (rank == 0) {
      // All 512 columns are allocated, so the TMEM base address is 0 and the MMA operands below
      // are compile-time constants plus warp-uniform offsets (operands the compiler cannot prove
      // warp-uniform, e.g. loaded from memory, made the issuing loop measurably slower).  Any
      // other base is reported as an error and the kernel leaves without issuing.
      if (tmem_base != 0u) {
        record_timeout(p.status, wait_code(15, 0, 0, 0, 0));  // role 15: unexpected TMEM base
        ok = false;
      }
      constexpr uint32_t const_sf = L::kConstCol;
      tc_cp_sf_atom_pair_warp(const_sf, smem_desc_sf(smem_u32(smem + L::kConstSf)));
      tc_cp_sf_atom_pair_warp(const_sf + 4, smem_desc_sf(smem_u32(smem + L::kConstSf)));
      int stage = 0, sfs = 0;
      uint32_t phase = 0, sfphase = 0;
      int local = 0;
      int4 next = pair < tiles ? __ldg(&p.list[pair / n_pt]) : make_int4(0, 0, 0, 0);
      for (int t = pair; t < tiles && ok; t += npairs, ++local) {
        const int4 cur = next;  // read a tile ahead: the load stays off the tile boundary
        if (t + npairs < tiles) next = __ldg(&p.list[(t + npairs) / n_pt]);
        const uint32_t n_mma = __shfl_sync(0xffffffffu, 4u * static_cast<uint32_t>(tile_half(cur.y)), 0);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_cluster_warp(&tempty[acc], acc_phase ^ 1, p.status, wait_code(2, 0, acc, acc_phase ^ 1, local))) {
          ok = false;
          break;
        }
        const uint32_t d_tmem = acc * L::kAccCols;
        uint32_t idk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) idk[k] = idesc_mxf8f6f4(/*a=E2M1*/ 5, /*b=E4M3*/ 0, 256, n_mma, k, 0);
        for (int kb0 = 0; kb0 < k_steps; kb0 += KS) {
          const int sub = kb0 % KSF;  // K step offset within the scale-atom stage
          if (sub == 0 && !mbar_wait_cta_warp(&sfready[sfs], sfphase, p.status, wait_code(3, 1, sfs, sfphase, kb0))) {
            ok = false;
            break;
          }
          if (!mbar_wait_cta_warp(&full[stage], phase, p.status, wait_code(3, 0, stage, phase, kb0))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int n = k_steps - kb0 < KS ? k_steps - kb0 : KS;
          for (int u = 0; u < n; ++u) {
            const uint32_t sfw_t = L::kSfwCol + (sfs * KSF + sub + u) * 4;
            const uint64_t wd0 = smem_desc_sw128(smem_u32(step_w(stage, u)));
            const uint64_t ad0 = smem_desc_sw128(smem_u32(step_a(stage, u)));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // descriptor start addresses are in 16-byte units: +32 bytes per K slice
              tc_mma_mxf8f6f4_pair_warp(d_tmem, wd0 + 2 * k, ad0 + 2 * k, idk[k],
                                        (kb0 + u != 0 || k != 0) ? 1u : 0u, sfw_t, const_sf);
            }
          }
          tc_commit_pair_warp(&empty[stage], 0x3);
          if (++stage == S) { stage = 0; phase ^= 1; }
          if (sub + KS >= KSF || kb0 + KS >= k_steps) {  // last operand stage of the scale-atom stage
            tc_commit_pair_warp(&sftfree[sfs], 0x1);
            if (++sfs == RS) { sfs = 0; sfphase ^= 1; }
          }
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
      int sfs = 0;
      uint32_t sfphase = 0;
      for (int t = pair; t < tiles && ok; t += npairs) {
        for (int kb0 = 0; kb0 < k_steps; kb0 += KSF) {
          if (!mbar_wait_cluster_warp(&sffull[sfs], sfphase, p.status, wait_code(6, 0, sfs, sfphase, kb0)) ||
              !mbar_wait_cluster_warp(&sftfree[sfs], sfphase ^ 1, p.status, wait_code(6, 1, sfs, sfphase ^ 1, kb0))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int n = k_steps - kb0 < KSF ? k_steps - kb0 : KSF;
          for (int u = 0; u < n; ++u)
            tc_cp_sf_atom_pair_warp(tmem_base + L::kSfwCol + (sfs * KSF + u) * 4,
                                    smem_desc_sf(smem_u32(step_sfw(sfs, u))));
          tc_commit_pair_warp(&sfready[sfs], 0x3);
          if (++sfs == RS) { sfs = 0; sfphase ^= 1; }
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;            // TMEM lane quadrant this warp may access
    const int half = (warp - 4) >> 2;  // this warp's token groups: half, half + kEpiSets, ...
    constexpr int kSets = L::kEpiSets;
    const int tid = threadIdx.x - 128;
    constexpr int kEpiThreads = 32 * L::kEpiWarps;
    const uint32_t tempty0 = cluster_addr(&tempty[0], 0);
    uint8_t* wst = smem + L::kStaging + (warp - 4) * 512;  // [8 tokens][4 x 16-byte column chunks], swizzled
    const uint32_t wst_u32 = smem_u32(wst);
    // stmatrix row addresses: thread 8k + i gives row i (token i) of the transpose of matrix
    // k (output columns 8k..8k+7 of the warp's 32); chunk c of row r sits at c ^ ((r/2)%4)
    const int sm_row = lane & 7;
    const int sm_chunk = lane >> 3;
    const uint32_t sm_addr = wst_u32 + sm_row * 64 + ((sm_chunk ^ ((sm_row >> 1) & 3)) << 4);
    const int ld_tok = lane >> 2, ld_part = lane & 3;  // the 16-byte piece of D this thread stores
    const uint8_t* ld_src = wst + ld_tok * 64 + ((ld_part ^ ((ld_tok >> 1) & 3)) << 4);
    const int c = 2 * (lane & 3);                       // tokens c, c+1 of each group (tcgen05.ld 16x256b)
    constexpr int kGroups = (kPlanesTileTok / 8 + kSets - 1) / kSets;  // groups per warp (of 2h / 8 <= 14)
    int local = 0;
    for (int t = pair; t < tiles && ok; t += npairs, ++local) {
      const int4 cur = __ldg(&p.list[t / n_pt]);
      const int pr0 = cur.x;  // first plane row of the tile
      const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
      const int ng = tile_half(cur.y) >> 2;  // groups of 8 tokens in the tile (2h tokens)
      const int b0 = pr0 >> 7;
      int brow0, bn;
      p.tm.rows(b0, brow0, bn);
      const int drow0 = brow0 + (pr0 & 127);  // D rows of a run follow its plane rows
      // loaded before the accumulator is ready, so that their latency stays off the drain:
      // the exponents of this thread's tokens (c, c+1 of each of its groups) and the row
      // masks of the (at most two) blocks the tile touches
      int2 ev[kGroups];
#pragma unroll
      for (int j = 0; j < kGroups; ++j) {
        const int g = half + kSets * j;
        ev[j] = g < ng ? __ldg(reinterpret_cast<const int2*>(p.row_exp + pr0 + g * 8 + c)) : make_int2(0, 0);
      }
      const uint4 m0 = __ldg(p.blk_mask + b0);
      const uint4 m1 = b0 + 1 < p.nblk ? __ldg(p.blk_mask + b0 + 1) : make_uint4(0, 0, 0, 0);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_cluster(&tfull[acc], acc_phase, p.status,
                             wait_code(4, static_cast<int>(rank), acc, acc_phase, local))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * L::kAccCols;
      const int dcol = nt * 128 + q * 32 + ld_part * 8;
#pragma unroll
      for (int j0 = 0; j0 < kGroups; j0 += 2) {
        if (half + kSets * j0 < ng) {
          uint32_t ra[2][8], rb[2][8];  // lanes 0-15 and 16-31 of the quadrant, two groups
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int g = half + kSets * (j0 + i);
            if (j0 + i < kGroups && g < ng) {
              tmem_ld_16x256b_x2(taddr + g * 16, ra[i]);
              tmem_ld_16x256b_x2(taddr + (16u << 16) + g * 16, rb[i]);
            }
          }
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int j = j0 + i;
            const int g = half + kSets * j;
            if (j < kGroups && g < ng) {
              const float s0 = __uint_as_float(static_cast<uint32_t>(min(max(ev[j].x + 127, 1), 254)) << 23);
              const float s1 = __uint_as_float(static_cast<uint32_t>(min(max(ev[j].y + 127, 1), 254)) << 23);
              uint32_t frag[4];
#pragma unroll
              for (int m = 0; m < 4; ++m) {
                // lanes 0-15 (m = 0, 1) or 16-31 (m = 2, 3), row l (even m) or l+8; registers
                // 0,1 / 2,3 hold the hi parts of tokens c, c+1 and 4,5 / 6,7 the lo parts
                const uint32_t* v = (m < 2 ? ra[i] : rb[i]) + 2 * (m & 1);
                const float x0 = (__uint_as_float(v[0]) + __uint_as_float(v[4])) * s0;
                const float x1 = (__uint_as_float(v[1]) + __uint_as_float(v[5])) * s1;
                __nv_bfloat162 b = __floats2bfloat162_rn(x0, x1);
                frag[m] = *reinterpret_cast<uint32_t*>(&b);
              }
              stmatrix_x4_trans(sm_addr, frag[0], frag[1], frag[2], frag[3]);
              __syncwarp();
              const int tok = g * 8 + ld_tok;
              if (tok < cur.y) {  // tokens past the tile belong to the next tile of the run
                const int pr = pr0 + tok;
                const uint4 mk = (pr >> 7) == b0 ? m0 : m1;
                const int wi = (pr >> 5) & 3;
                const uint32_t word = wi == 0 ? mk.x : wi == 1 ? mk.y : wi == 2 ? mk.z : mk.w;
                uint4 v = make_uint4(0, 0, 0, 0);
                if ((word >> (pr & 31)) & 1u) v = *reinterpret_cast<const uint4*>(ld_src);
                __nv_bfloat16* rp = d_row(p, static_cast<int64_t>(drow0 + tok));
                if (rp) *reinterpret_cast<uint4*>(rp + dcol) = v;
              }
              __syncwarp();
            }
          }
        }
      }
      tc_fence_before();
      if (rank == 0)
        mbar_arrive(&tempty[acc]);
      else
        mbar_arrive_cluster(tempty0 + acc * 8);
      // after the last tile of a run: the rows of its last block past the run
      if (cur.w && p.fill_rest) {
        const int pe = pr0 + cur.y;  // plane row after the run
        const int bl = (pe - 1) >> 7;
        int lrow0, ln;
        p.tm.rows(bl, lrow0, ln);
        const int r_first = lrow0 + (pe - bl * 128);
        const int rows = lrow0 + ln - r_first;
        const uint4 z = make_uint4(0, 0, 0, 0);
        for (int cc = tid; cc < rows * 16; cc += kEpiThreads) {
          const int r = r_first + (cc >> 4);
          __nv_bfloat16* rp = d_row(p, r);
          if (rp) *reinterpret_cast<uint4*>(rp + nt * 128 + (cc & 15) * 8) = z;
        }
      }
    }
  }

  if (p.d_rows) __threadfence_system();  // rows stored into other GPUs' memory
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
