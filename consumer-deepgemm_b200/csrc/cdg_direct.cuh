// CTA-pair tcgen05 kernel for the direct class: wide blocks (more than 32 routed rows of one
// expert, or the tail block of an expert spanning several blocks) whose activation scales are
// all powers of two.  The reference's bf16(bf16(a) * bf16(2^s)) is then the exact product
// a * 2^s, which the tensor core forms itself from the raw e4m3 rows of A with 2^s as the
// MMA's token scale factor: the accumulator holds the final values, one MMA per 32-wide K
// slice, and the epilogue only converts and stores.
//
// Work is cut by tokens, as in cdg_gemm_planes_kernel: the prep kernel joins consecutive
// direct blocks of one expert into runs and cuts each run into tiles of up to
// kDirectTileTok = 224 rows (a tile may cross block boundaries; the rows of a run are
// contiguous in A and D).  A cluster of two CTAs computes a pair tile: 256 weight rows of the
// expert (CTA r holds output-column tile 2*pt + r) x the tile's tokens, with
// tcgen05.mma.cta_group::2 (M = 256, weights as the MMA's A operand: "swap AB").  CTA 0 holds
// tokens [0, h), CTA 1 [h, 2h) (h = half the tile rounded up to 8, N = 2h <= 224), brought
// by one 2-D box of 8g rows of A per K step (one tensor map per g = h / 8).
//
// Token scale factors.  The prep kernel writes one UE8M0 code per (row, 128-wide K block),
// row major with four K blocks per aligned 32-bit word; the planes kernel, which runs just
// before this one, then writes (write_direct_atoms), per tile and scale stage of kKSF = 4 K
// steps, two 512-byte scale atoms (tokens 0-127 and
// 128-255: token n at byte (n%32)*16 + ((n%128)/32)*4 of atom n/128) whose byte j is the
// code of K step j of the stage.  One 8-column TMEM set then holds the token scales of four
// K steps and the MMA of K step j selects byte j (b_sf_id).  The token atoms and the weight
// scale atoms (one per K step, byte = 32-wide K slice) travel by TMA in a shared-memory ring
// of their own, and a copier thread moves them into TMEM (tcgen05.cp) as soon as the MMAs
// that used the TMEM slot last completed.  TMEM holds two scale stages, the shared-memory
// ring four, so the loads run well ahead of the copies.  (Atoms built inside this kernel
// from the per-row codes put the codes' global-load latency on the scale ring's critical
// path: the MMA issuer then waited for its scale stage about a third of the time.)
//
// TMEM: two accumulators of 224 columns (the epilogue drains one while the MMAs fill the
// other), 2 slots x 4 K steps x 4 weight scale columns, 2 slots x 8 token scale columns:
// 496 of 512 columns.
//
// Warp roles per CTA: 0 = operand TMA producer, 1 = MMA issuer (even CTA, whole warp) and
// TMEM owner, 2 = scale-factor copier (even CTA, whole warp), 3 = scale-atom TMA producer,
// 4-11 = epilogue (two warps per TMEM lane quadrant, each taking every other 16-token
// chunk).  All waits are bounded (kStatusTimeout).
#pragma once

#include "cdg_kernels.cuh"

namespace cdg {

struct DirectSmem {
  static constexpr int kKS = 2;                   // K steps per operand stage
  static constexpr int kKSF = 4;                  // K steps per scale-atom stage (bytes of a token scale word)
  static constexpr int kW = 128 * 128;            // weight tile per K step (E2M1 unpacked to bytes)
  static constexpr int kA = kDirectTileTok / 2 * 128;  // 112 token rows per K step
  static constexpr int kStep = kW + kA;
  static constexpr int kStages = 3;
  static constexpr int kSfStages = 4;   // scale stages in shared memory
  static constexpr int kSfSlots = 2;    // scale stages in TMEM
  static constexpr int kStageBytes = kKS * kStep;
  static constexpr int kSfRing = kStages * kStageBytes;              // [kSfStages][kKSF] weight scale atoms
  static constexpr int kTsfRing = kSfRing + kSfStages * kKSF * 512;  // [kSfStages][2] token scale atoms
  static constexpr int kEpiWarps = 8;                                // two per TMEM lane quadrant
  static constexpr int kStaging = kTsfRing + kSfStages * 2 * 512;    // kEpiWarps x [16 tokens][32 columns] bf16
  static constexpr int kBarOffset = kStaging + kEpiWarps * 1024;
  // full, empty; sffull, sfsfree; sfready, sftfree; tfull[2], tempty[2], done
  static constexpr int kNumBars = 2 * kStages + 2 * kSfStages + 2 * kSfSlots + 5;
  static constexpr int kBarBytes = kNumBars * 8 + 16;                // + TMEM address
  static constexpr int kBytes = kBarOffset + kBarBytes + 1024;      // + alignment slack
  static_assert(kBytes <= 232448, "shared memory per CTA");
  static_assert(kStep % 1024 == 0, "K steps must stay 1024-byte aligned for SW128 tiles");
  static_assert(kKSF % kKS == 0, "an operand stage lies in one scale-atom stage");
  static_assert(kKSF == 4, "a token scale word holds the codes of four K steps");
  // TMEM: two accumulators of kDirectTileTok columns, the weight and token scale rings
  static constexpr uint32_t kAccCols = kDirectTileTok;
  static constexpr uint32_t kSfwCol = 2 * kAccCols;
  static constexpr uint32_t kTsfCol = kSfwCol + kSfSlots * kKSF * 4;
  static_assert(kTsfCol + kSfSlots * 8 <= 512, "TMEM columns");
  static constexpr int kThreads = 128 + 32 * kEpiWarps;
};

// Tensor maps of A, one per box height: m[g - 1] brings 8g rows.
struct DirectMaps {
  CUtensorMap m[kDirectTileTok / 16];
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(DirectSmem::kThreads, 1)
    cdg_gemm_direct_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ DirectMaps tmaps_a,
                           const __grid_constant__ CUtensorMap tmap_sfw, const __grid_constant__ CUtensorMap tmap_tsf,
                           GemmArgs p) {
  using L = DirectSmem;
  constexpr int S = L::kStages;
  constexpr int SR = L::kSfStages;
  constexpr int RS = L::kSfSlots;
  constexpr int KS = L::kKS;
  constexpr int KSF = L::kKSF;
  constexpr uint32_t kTmemCols = 512;

  grid_dependency_wait();  // the tile list and the token codes come from the previous kernel of the stream
  grid_launch_dependents();
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
  auto step_tsf = [&](int s) { return smem + L::kTsfRing + s * 1024; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;                // [S] even CTA: both CTAs' operand copies of a stage landed
  uint64_t* empty = bars + S;           // [S] stage consumed (multicast by the MMA commit)
  uint64_t* sffull = bars + 2 * S;      // [SR] even CTA: both CTAs' scale atoms of a stage are in place
  uint64_t* sfsfree = sffull + SR;      // [SR] the copies out of the shared-memory stage completed (multicast)
  uint64_t* sfready = sfsfree + SR;     // [RS] even CTA: the TMEM slot holds its scale stage
  uint64_t* sftfree = sfready + RS;     // [RS] even CTA: the MMAs that read the TMEM slot completed
  uint64_t* tfull = sftfree + RS;       // [2] accumulator complete (multicast)
  uint64_t* tempty = tfull + 2;         // [2] even CTA: all epilogue threads of the pair drained it
  uint64_t* done = tempty + 2;          // even CTA: every MMA completed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    for (int g = 0; g < kDirectTileTok / 16; ++g) prefetch_tmap(&tmaps_a.m[g]);
    prefetch_tmap(&tmap_sfw);
    prefetch_tmap(&tmap_tsf);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < SR; ++s) {
      mbar_init(&sffull[s], 1);
      mbar_init(&sfsfree[s], 1);
    }
    for (int s = 0; s < RS; ++s) {
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
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers ready before any copy or commit reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool ok = true;

  // Tokens per CTA of a tile of `rows` rows: half, rounded up to 8 (N = 2h).
  auto tile_half = [](int rows) { return (((rows + 1) >> 1) + 7) & ~7; };
  // First row of A (and D) of a tile whose first block-relative row is `br`.
  auto tile_row0 = [&](int br) {
    int brow0, bn;
    p.tm.rows(br >> 7, brow0, bn);
    return brow0 + (br & 127);
  };

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
        const int h = tile_half(cur.y);
        const int arow = tile_row0(cur.x) + static_cast<int>(rank) * h;  // rows of A itself
        const CUtensorMap* tmap_a = &tmaps_a.m[(h >> 3) - 1];
        const uint32_t tx_step = 128u * 64u + static_cast<uint32_t>(h) * 128u;
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
            tma_load_2d_pair(step_a(stage, u), tmap_a, fb, kb * 128, arow);
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
      const int stages = (k_steps + KSF - 1) / KSF;
      int next = pair < tiles ? __ldg(&p.list[pair / n_pt]).z : 0;
      for (int t = pair; t < tiles && ok; t += npairs) {
        const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
        const int expert = next;  // read a tile ahead: the load stays off the tile boundary
        if (t + npairs < tiles) next = __ldg(&p.list[(t + npairs) / n_pt]).z;
        const int atom0 = (expert * n_tiles + nt) * k_steps;
        const int tatom0 = (t / n_pt) * stages * 2;  // the tile's token atoms, two per stage
        for (int kb0 = 0, st = 0; kb0 < k_steps; kb0 += KSF, ++st) {
          // the copies out of this stage (SR stages ago) completed
          if (!mbar_wait_cluster(&sfsfree[sfs], sfphase ^ 1, p.status,
                                 wait_code(7, static_cast<int>(rank), sfs, sfphase ^ 1, kb0))) {
            ok = false;
            break;
          }
          const int n = k_steps - kb0 < KSF ? k_steps - kb0 : KSF;
          const uint32_t fb = sffull0 + sfs * 8;
          if (rank == 0) mbar_arrive_expect_tx(&sffull[sfs], 2u * (static_cast<uint32_t>(n) * 512u + 1024u));
          for (int u = 0; u < n; ++u) tma_load_2d_pair(step_sfw(sfs, u), &tmap_sfw, fb, 0, atom0 + kb0 + u);
          tma_load_2d_pair(step_tsf(sfs), &tmap_tsf, fb, 0, tatom0 + 2 * st);
          if (++sfs == SR) { sfs = 0; sfphase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA, whole warp)
    if (rank == 0) {
      // All 512 columns are allocated, so the TMEM base address is 0 and the MMA operands below
      // are compile-time constants plus warp-uniform offsets.  Any other base is reported as an
      // error and the kernel leaves without issuing.
      if (tmem_base != 0u) {
        record_timeout(p.status, wait_code(15, 0, 0, 0, 0));  // role 15: unexpected TMEM base
        ok = false;
      }
      int stage = 0, sfs = 0;
      uint32_t phase = 0, sfphase = 0;
      int local = 0;
      int4 next = pair < tiles ? __ldg(&p.list[pair / n_pt]) : make_int4(0, 0, 0, 0);
      for (int t = pair; t < tiles && ok; t += npairs, ++local) {
        const int4 cur = next;  // read a tile ahead: the load stays off the tile boundary
        if (t + npairs < tiles) next = __ldg(&p.list[(t + npairs) / n_pt]);
        const uint32_t n_mma = __shfl_sync(0xffffffffu, 2u * static_cast<uint32_t>(tile_half(cur.y)), 0);
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
          const uint32_t tsf_t = L::kTsfCol + sfs * 8;
          for (int u = 0; u < n; ++u) {
            const uint32_t sfw_t = L::kSfwCol + (sfs * KSF + sub + u) * 4;
            const uint32_t bsf = static_cast<uint32_t>(sub + u) << 4;  // b_sf_id: byte of this K step
            const uint64_t wd0 = smem_desc_sw128(smem_u32(step_w(stage, u)));
            const uint64_t ad0 = smem_desc_sw128(smem_u32(step_a(stage, u)));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // descriptor start addresses are in 16-byte units: +32 bytes per K slice
              tc_mma_mxf8f6f4_pair_warp(d_tmem, wd0 + 2 * k, ad0 + 2 * k, idk[k] | bsf,
                                        (kb0 + u != 0 || k != 0) ? 1u : 0u, sfw_t, tsf_t);
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
      int ss = 0, ts = 0;  // shared-memory stage, TMEM slot
      uint32_t ssphase = 0, tsphase = 0;
      for (int t = pair; t < tiles && ok; t += npairs) {
        for (int kb0 = 0; kb0 < k_steps; kb0 += KSF) {
          if (!mbar_wait_cluster_warp(&sffull[ss], ssphase, p.status, wait_code(6, 0, ss, ssphase, kb0)) ||
              !mbar_wait_cluster_warp(&sftfree[ts], tsphase ^ 1, p.status, wait_code(6, 1, ts, tsphase ^ 1, kb0))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int n = k_steps - kb0 < KSF ? k_steps - kb0 : KSF;
          for (int u = 0; u < n; ++u)
            tc_cp_sf_atom_pair_warp(tmem_base + L::kSfwCol + (ts * KSF + u) * 4,
                                    smem_desc_sf(smem_u32(step_sfw(ss, u))));
          tc_cp_sf_atom_pair_warp(tmem_base + L::kTsfCol + ts * 8, smem_desc_sf(smem_u32(step_tsf(ss))));
          tc_cp_sf_atom_pair_warp(tmem_base + L::kTsfCol + ts * 8 + 4, smem_desc_sf(smem_u32(step_tsf(ss) + 512)));
          tc_commit_pair_warp(&sfready[ts], 0x1);
          tc_commit_pair_warp(&sfsfree[ss], 0x3);
          if (++ss == SR) { ss = 0; ssphase ^= 1; }
          if (++ts == RS) { ts = 0; tsphase ^= 1; }
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;            // TMEM lane quadrant this warp may access
    const int half = (warp - 4) >> 2;  // this warp's 16-token chunks: half, half + 2, ...
    const int tid = threadIdx.x - 128;
    constexpr int kEpiThreads = 32 * L::kEpiWarps;
    const uint32_t tempty0 = cluster_addr(&tempty[0], 0);
    uint8_t* wst = smem + L::kStaging + (warp - 4) * 1024;  // [16 tokens][4 x 16-byte column chunks], swizzled
    const uint32_t wst_u32 = smem_u32(wst);
    // stmatrix row addresses: thread 8k + i gives row i of matrix k, i.e. token i + 8*(k/2),
    // column chunk (k%2) (+2 for the second 16-lane half); chunk c of row r sits at c ^ ((r/2)%4)
    const int sm_row = (lane & 7) + 8 * (lane >> 4);
    const int sm_chunk = (lane >> 3) & 1;
    const uint32_t sm_addr0 = wst_u32 + sm_row * 64 + ((sm_chunk ^ ((sm_row >> 1) & 3)) << 4);
    const uint32_t sm_addr1 = wst_u32 + sm_row * 64 + (((sm_chunk + 2) ^ ((sm_row >> 1) & 3)) << 4);
    int local = 0;
    for (int t = pair; t < tiles && ok; t += npairs, ++local) {
      const int4 cur = __ldg(&p.list[t / n_pt]);
      const int br0 = cur.x;  // block-relative row of the tile's first token
      const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
      const int nchunk = tile_half(cur.y) >> 3;  // 16-token chunks of the accumulator (2h tokens)
      const int b0 = br0 >> 7;
      const int drow0 = tile_row0(br0);  // D rows of a run follow its block-relative rows
      // row masks of the (at most three) blocks the tile touches, loaded before the
      // accumulator is ready
      uint4 mk[3];
#pragma unroll
      for (int i = 0; i < 3; ++i) mk[i] = b0 + i < p.nblk ? __ldg(p.blk_mask + b0 + i) : make_uint4(0, 0, 0, 0);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_cluster(&tfull[acc], acc_phase, p.status,
                             wait_code(4, static_cast<int>(rank), acc, acc_phase, local))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * L::kAccCols;
      const int dcol = nt * 128 + q * 32;
      for (int c0 = half; c0 < nchunk; c0 += 4) {
        uint32_t ra[2][8], rb[2][8];  // lanes 0-15 and 16-31 of the quadrant, chunks c0 and c0 + 2
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (c0 + 2 * i < nchunk) {
            tmem_ld_16x256b_x2(taddr + (c0 + 2 * i) * 16, ra[i]);
            tmem_ld_16x256b_x2(taddr + (16u << 16) + (c0 + 2 * i) * 16, rb[i]);
          }
        }
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int j0 = (c0 + 2 * i) * 16;
          if (c0 + 2 * i < nchunk) {
            uint32_t m[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              __nv_bfloat162 a = __floats2bfloat162_rn(__uint_as_float(ra[i][2 * k]), __uint_as_float(ra[i][2 * k + 1]));
              __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(rb[i][2 * k]), __uint_as_float(rb[i][2 * k + 1]));
              m[k] = *reinterpret_cast<uint32_t*>(&a);
              m[4 + k] = *reinterpret_cast<uint32_t*>(&b);
            }
            // matrices: (columns 0-7 | 8-15, tokens 0-7 | 8-15) of each 16-lane half
            stmatrix_x4_trans(sm_addr0, m[0], m[1], m[2], m[3]);
            stmatrix_x4_trans(sm_addr1, m[4], m[5], m[6], m[7]);
            __syncwarp();
#pragma unroll
            for (int s = 0; s < 2; ++s) {
              const int vi = lane + 32 * s, rr = vi >> 2, part = vi & 3;
              const int tok = j0 + rr;
              if (tok < cur.y) {  // tokens past the tile belong to the next tile of the run
                const int br = br0 + tok;
                const int bi = (br >> 7) - b0;
                const uint4 w4 = bi == 0 ? mk[0] : bi == 1 ? mk[1] : mk[2];
                const int wi = (br >> 5) & 3;
                const uint32_t word = wi == 0 ? w4.x : wi == 1 ? w4.y : wi == 2 ? w4.z : w4.w;
                uint4 v = make_uint4(0, 0, 0, 0);
                if ((word >> (br & 31)) & 1u)
                  v = *reinterpret_cast<const uint4*>(wst + rr * 64 + ((part ^ ((rr >> 1) & 3)) << 4));
                __nv_bfloat16* rp = d_row(p, static_cast<int64_t>(drow0 + tok));
                if (rp) *reinterpret_cast<uint4*>(rp + dcol + part * 8) = v;
              }
            }
            __syncwarp();
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
        const int be = br0 + cur.y;  // block-relative row after the run
        const int bl = (be - 1) >> 7;
        int lrow0, ln;
        p.tm.rows(bl, lrow0, ln);
        const int r_first = lrow0 + (be - bl * 128);
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
