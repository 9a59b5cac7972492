// CTA-pair variant of the tcgen05 grouped GEMM (tcgen05.mma.cta_group::2, M = 256).
//
// A cluster of two CTAs (one TPC) computes a pair tile: 256 weight rows (two
// adjacent 128-row output-column tiles of one expert, one per CTA) x the tokens of
// one 128-row block.  One MMA instruction, issued by the even CTA, covers both SMs'
// weight tiles.
//
// At decode sizes (N <= 64 per MMA) the cost is instruction issue, not math: one
// thread issuing cp + 4 MMAs + commit per K step and waiting on an mbarrier every
// step sustains ~475-530 cycles per step (measured), two issuing threads ~270 and
// four ~160, the tensor pipe interleaving their streams.  So the K steps are dealt
// round-robin to NI issuing warps (K step i of the CTA's sequence to issuer i % NI,
// which with a stage ring of a multiple of NI stages means each issuer owns fixed
// stages), each accumulating into its own TMEM partial sum (a fixed assignment, so
// results are deterministic); the epilogue adds the partials.
//
// Operands per pipeline stage (K step of 128), in each CTA's own shared memory:
//   * its weight tile [128 n x 128 k] (TMA, packed E2M1 unpacked to bytes, SW128);
//   * its half of the MMA's B operand (N rows split between the CTAs): CTA 0 holds the hi
//     plane's TOK token rows and CTA 1 the lo plane's, one MMA per K slice with N = 2*TOK;
//     TMEM columns [0, TOK) then hold the hi part and [TOK, 2*TOK) the lo part of each token;
//   * its weights' 512-byte scale atom (TMA, 2-D view of the atom array).
// Every copy of both CTAs completes on the even CTA's `full` barrier (cta_group::2
// form of the TMA load, no multicast); the MMA commits arrive on the `empty` and
// `tfull` barriers of both CTAs (tcgen05.commit multicast); each epilogue thread of
// both CTAs drains its own TMEM lanes (its CTA's 128 output columns) and arrives on
// the even CTA's `tempty` barrier.  All waits are bounded (kStatusTimeout).  Wide
// blocks (more than 32 rows) run the token-tile kernels instead (cdg_gemm_planes_kernel,
// cdg_gemm_direct_kernel).
//
// Warp roles per CTA: 0 = TMA producer of the weight tiles, 1..NI = MMA issuers (even CTA;
// warp 1 also owns TMEM), then four epilogue warps (4-7, or 5-8 when NI = 4), then the TMA
// producer of the activation planes and weight scale atoms (8 or 9).
#pragma once

#include "cdg_kernels.cuh"

namespace cdg {

template <int TOK, int NI>
struct PairSmem {
  static_assert(TOK == 16 || TOK == 32, "tiny and narrow blocks");
  // A multiple of NI: stage s is always consumed by issuer s % NI, in order, so an
  // issuer never waits on a stage use whose predecessor it did not consume itself.
  static constexpr int kStages = NI == 4 ? 12 : 10;
  static_assert(kStages % NI == 0, "stage ring must split evenly over the issuers");
  static constexpr int kW = 128 * 128;             // weight tile, bytes per stage
  static constexpr int kA = TOK * 128;             // one plane's rows, bytes per stage
  static constexpr int kStageBytes = kW + kA;      // operand tiles (1024-byte multiple)
  static constexpr int kSfRing = kStages * kStageBytes;  // then one 512-byte weight scale atom per stage
  static constexpr int kOneAtom = kSfRing + kStages * 512;  // constant activation scale atom
  // narrow tiles: per epilogue warp a [16 rows x 32 columns] BF16 staging tile, so that D
  // leaves as 16-byte row segments instead of 2-byte column elements
  static constexpr bool kStagedStores = TOK > 16;
  static constexpr int kStaging = kOneAtom + 512;
  static constexpr int kStagingBytes = kStagedStores ? 4 * 16 * 32 * 2 : 0;
  static constexpr int kBarOffset = kStaging + kStagingBytes;
  static constexpr int kBarBytes = (2 * kStages + 4 + NI) * 8 + 16;  // barriers + TMEM address
  static constexpr int kBytes = kBarOffset + kBarBytes + 1024;          // + alignment slack
  static_assert(kBytes <= 232448, "shared memory per CTA");
  // bytes one CTA's copies of one stage add to the even CTA's `full` barrier
  static constexpr uint32_t kTxPerCta = 128u * 64u + kA + 512u;
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned for SW128 tiles");
  // TMEM: per accumulator buffer NI partials of kPartCols columns; two buffers; then
  // per issuer two 4-column weight scale sets; then per issuer the constant activation
  // scale set (each issuer copies its own, so no issuer reads another's TMEM writes).
  static constexpr uint32_t kPartCols = 2 * TOK;
  static constexpr uint32_t kAccCols = NI * kPartCols;
  static constexpr uint32_t kSfwCol = 2 * kAccCols;
  static constexpr uint32_t kSfaCol = kSfwCol + 8 * NI;
  static_assert(kSfaCol + 4 * NI <= 512, "TMEM columns");
  static constexpr int kEpiWarp0 = NI < 4 ? 4 : NI + 1;
  static constexpr int kActWarp = kEpiWarp0 + 4;  // second TMA producer: activation plane + scale atom
  static constexpr int kThreads = (kActWarp + 1) * 32;
};

template <int TOK, int NI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairSmem<TOK, NI>::kThreads, 1)
    cdg_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_sf, GemmArgs p) {
  using L = PairSmem<TOK, NI>;
  constexpr int S = L::kStages;
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
  const int zero_count = p.do_zero_blocks ? __ldcg(&p.ctrl[kCtrlCount0 + kClassZero]) : 0;
  const int reg_tiles = count * n_pt;
  const int total_tiles = reg_tiles + zero_count * n_pt;
  if (total_tiles == 0) return;  // both CTAs of the pair read the same counts and leave together

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto stage_w = [&](int s) { return smem + s * L::kStageBytes; };
  auto stage_a = [&](int s) { return smem + s * L::kStageBytes + L::kW; };
  auto stage_sf = [&](int s) { return smem + L::kSfRing + s * 512; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;       // [S] (even CTA's count both CTAs' copies)
  uint64_t* empty = bars + S;  // [S] stage consumed (multicast by the MMA commit)
  uint64_t* tfull = bars + 2 * S;  // [2] all NI partials of an accumulator buffer complete
  uint64_t* tempty = tfull + 2;    // [2] even CTA: all 256 epilogue threads of the pair drained
  uint64_t* done = tempty + 2;     // [NI] even CTA: every MMA of issuer j completed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + NI);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_sf);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], NI);
      mbar_init(&tempty[s], 256);
    }
    for (int j = 0; j < NI; ++j) mbar_init(&done[j], 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == L::kEpiWarp0) {
    uint32_t* one = reinterpret_cast<uint32_t*>(smem + L::kOneAtom);
    one[lane] = one[lane + 32] = one[lane + 64] = one[lane + 96] = 0x7F7F7F7Fu;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised before any copy or commit reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t full0 = cluster_addr(&full[0], 0);
      // the next tile's list entry is loaded one tile ahead, off the issue path
      int4 next = pair < reg_tiles ? __ldg(&p.list[pair / n_pt]) : make_int4(0, 0, 0, 0);
      for (int t = pair; t < reg_tiles && ok; t += npairs) {
        const int4 cur = next;
        if (t + npairs < reg_tiles) next = __ldg(&p.list[(t + npairs) / n_pt]);
        const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
        const int wrow = cur.y * p.N + nt * 128;
        for (int kb = 0; kb < k_steps; ++kb) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1, p.status,
                                 wait_code(1, static_cast<int>(rank), stage, phase ^ 1, kb))) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + stage * 8;
          // this stage's weight tile; the activation plane and the weight scale atom come from
          // the second producer (warp kActWarp), onto the same barrier
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2u * L::kTxPerCta);
          tma_load_2d_pair(stage_w(stage), &tmap_w, fb, kb * 128, wrow);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == L::kActWarp) {
    // ------------------------------------------------------------ second TMA producer (both CTAs)
    // A single thread issuing all three copies of a K step held the decode kernel at the rate it
    // issues them (its time followed the SM clock); the copies of a stage are split over two.
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t full0 = cluster_addr(&full[0], 0);
      int4 next = pair < reg_tiles ? __ldg(&p.list[pair / n_pt]) : make_int4(0, 0, 0, 0);
      for (int t = pair; t < reg_tiles && ok; t += npairs) {
        const int4 cur = next;  // read a tile ahead: the load stays off the tile boundary
        if (t + npairs < reg_tiles) next = __ldg(&p.list[(t + npairs) / n_pt]);
        const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
        const int atom0 = (cur.y * n_tiles + nt) * k_steps;
        const int a_row = cur.x * 128;
        for (int kb = 0; kb < k_steps; ++kb) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1, p.status,
                                 wait_code(1, static_cast<int>(rank), stage, phase ^ 1, kb))) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + stage * 8;
          tma_load_3d_pair(stage_a(stage), &tmap_a, fb, kb * 128, a_row, static_cast<int>(rank));
          tma_load_2d_pair(stage_sf(stage), &tmap_sf, fb, 0, atom0 + kb);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp >= 1 && warp <= NI) {
    // ------------------------------------------------------------ MMA issuers (even CTA)
    // Issuer j takes the K steps i (counted over all tiles of this CTA) with i % NI == j,
    // into partial sum j.
    const int j = warp - 1;
    if (lane == 0 && rank == 0) {
      int local = 0;
      int seq = 0;  // K steps of all earlier tiles
      const uint32_t sfa_t = tmem_base + L::kSfaCol + 4 * j;
      tc_cp_sf_atom_pair(sfa_t, smem_desc_sf(smem_u32(smem + L::kOneAtom)));
      int n_own = 0;  // K steps this issuer has taken (weight scale set parity)
      for (int t = pair; t < reg_tiles && ok; t += npairs, ++local, seq += k_steps) {
        constexpr uint32_t n_mma = 2u * TOK;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, p.status, wait_code(2, j, acc, acc_phase ^ 1, local))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * L::kAccCols + j * L::kPartCols;
        const int kb0 = (j - seq % NI + NI) % NI;  // this issuer's first K step of the tile
        for (int kb = kb0; kb < k_steps; kb += NI, ++n_own) {
          const int i = seq + kb;
          const int stage = i % S;
          const uint32_t phase = static_cast<uint32_t>(i / S) & 1u;
          if (!mbar_wait_cluster(&full[stage], phase, p.status, wait_code(3, j, stage, phase, i))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfw_t = tmem_base + L::kSfwCol + j * 8 + (n_own & 1) * 4;
          tc_cp_sf_atom_pair(sfw_t, smem_desc_sf(smem_u32(stage_sf(stage))));
          const uint32_t w_addr = smem_u32(stage_w(stage));
          const uint32_t a_addr = smem_u32(stage_a(stage));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t wd = smem_desc_sw128(w_addr + k * 32);
            const uint32_t idesc = idesc_mxf8f6f4(/*a=E2M1*/ 5, /*b=E4M3*/ 0, 256, n_mma, k, k);
            const uint32_t accumulate = (kb != kb0 || k != 0) ? 1u : 0u;
            tc_mma_mxf8f6f4_pair(d_tmem, wd, smem_desc_sw128(a_addr + k * 32), idesc, accumulate, sfw_t, sfa_t);
          }
          tc_commit_pair(&empty[stage], 0x3);
        }
        if (!ok) break;
        tc_commit_pair(&tfull[acc], 0x3);
      }
      // Every MMA (and its TMEM writes in both CTAs) completes before teardown.
      tc_commit_pair(&done[j], 0x1);
      mbar_wait_cluster(&done[j], 0, p.status, wait_code(5, j, 0, 0, 0));
    }
  } else if (warp >= L::kEpiWarp0) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int tid = threadIdx.x - L::kEpiWarp0 * 32;
    const int parts = NI < k_steps ? NI : k_steps;  // partial sums holding K steps
    int seq = 0;  // K steps of the earlier regular tiles (which issuers hold partials)
    const uint32_t tempty0 = cluster_addr(&tempty[0], 0);
    int local = 0;
    for (int t = pair; t < total_tiles && ok; t += npairs) {
      const bool regular = t < reg_tiles;
      const int blk = regular ? __ldg(&p.list[t / n_pt]).x : __ldg(&p.zero_list[(t - reg_tiles) / n_pt]).x;
      const int nt = 2 * (t % n_pt) + static_cast<int>(rank);
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
        const int first = seq % NI;  // issuer of the tile's first K step
        seq += k_steps;
        // 2^E of the tile's rows, loaded before the accumulator wait: lane l holds rows l + 32k
        float row_sc[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          row_sc[k] = __uint_as_float(
              static_cast<uint32_t>(min(max(__ldg(p.row_exp + blk * 128 + k * 32 + lane) + 127, 1), 254)) << 23);
        if (!mbar_wait_cluster(&tfull[acc], acc_phase, p.status,
                               wait_code(4, static_cast<int>(rank), acc, acc_phase, local - 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int n = nt * 128 + q * 32 + lane;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * L::kAccCols;
        for (int j0 = 0; j0 < ntok; j0 += 16) {
          const int kq = j0 >> 5;  // which of the 32-row groups this chunk lies in
          const float my_scale = kq == 0 ? row_sc[0] : kq == 1 ? row_sc[1] : kq == 2 ? row_sc[2] : row_sc[3];
          uint32_t v[16];
          tmem_ld16(taddr + first * L::kPartCols + j0, v);
          {
            uint32_t w[16];
            tmem_ld16(taddr + first * L::kPartCols + TOK + j0, w);  // lo-plane columns of the same tokens
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
            for (int x = 1; x < parts; ++x) {  // the other issuers' partial sums, in K order
              const int pj = (first + x) % NI;
              uint32_t h[16];
              tmem_ld16(taddr + pj * L::kPartCols + j0, h);
              tmem_ld16(taddr + pj * L::kPartCols + TOK + j0, w);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j)
                v[j] = __float_as_uint(__uint_as_float(v[j]) + (__uint_as_float(h[j]) + __uint_as_float(w[j])));
            }
          }
          if (L::kStagedStores) {
            // this warp's 32 columns x 16 rows through shared memory: each lane then stores two
            // 16-byte row segments (rows past the block's end are skipped)
            __nv_bfloat16* wst = reinterpret_cast<__nv_bfloat16*>(smem + L::kStaging) + q * 16 * 32;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int rb = j0 + j;
              const uint32_t word = rb < 32 ? mask.x : rb < 64 ? mask.y : rb < 96 ? mask.z : mask.w;
              const float sc = __shfl_sync(0xffffffffu, my_scale, (j0 & 31) + j);
              const float x = ((word >> (rb & 31)) & 1u) ? __uint_as_float(v[j]) * sc : 0.0f;
              wst[j * 32 + lane] = __float2bfloat16_rn(x);
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int vi = lane + 32 * i, rr = vi >> 2, part = vi & 3;
              if (j0 + rr < nrows) {
                __nv_bfloat16* rp = d_row(p, row0 + j0 + rr);
                if (rp)
                  *reinterpret_cast<uint4*>(rp + nt * 128 + q * 32 + part * 8) =
                      *reinterpret_cast<const uint4*>(wst + rr * 32 + part * 8);
              }
            }
            __syncwarp();
          } else {
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
        }
        tc_fence_before();
        if (rank == 0)
          mbar_arrive(&tempty[acc]);
        else
          mbar_arrive_cluster(tempty0 + acc * 8);
        zero_from = ntok;
      }
      const int rows = p.fill_rest ? nrows - zero_from : 0;
      const uint4 z = make_uint4(0, 0, 0, 0);
      if (p.d_rows == nullptr) {  // the common case, without the row table's per-store branch
        __nv_bfloat16* base = p.d + static_cast<int64_t>(row0 + zero_from) * p.d_row_stride + nt * 128;
        for (int c = tid; c < rows * 16; c += 128)
          *reinterpret_cast<uint4*>(base + (c >> 4) * p.d_row_stride + (c & 15) * 8) = z;
      } else {
        for (int c = tid; c < rows * 16; c += 128) {
          const int r = row0 + zero_from + (c >> 4);
          __nv_bfloat16* rp = d_row(p, r);
          if (rp) *reinterpret_cast<uint4*>(rp + nt * 128 + (c & 15) * 8) = z;
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
