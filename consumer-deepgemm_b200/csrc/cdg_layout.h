// Internal layout constants shared by the host launcher and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>

#include "cdg_b200.h"

namespace cdg {

// Classes of 128-row blocks, decided by cdg_prep_kernel.
enum : int {
  kClassTiny = 0,       // one expert, rows within the first kTinyTok   -> cdg_gemm_kernel<16>
  kClassNarrow = 1,     // one expert, rows within the first kNarrowTok -> cdg_gemm_kernel<32>
  kClassWide = 2,       // one expert, more rows                        -> cdg_gemm_kernel<128>
  kClassZero = 3,       // no row with a valid id                       -> zero fill (tiny kernel)
  kClassIrregular = 4,  // rows of two or more experts                  -> cdg_generic_kernel
  kClassWideDirect = 5, // a wide block whose activation scales are all powers of two: the raw
                        // e4m3 rows with their scales as UE8M0 MMA scale factors (one plane)
  kNumClasses = 6,
};
constexpr int kTinyTok = 16;
constexpr int kNarrowTok = 32;
// Tokens per tile of cdg_gemm_planes_kernel: runs of consecutive wide blocks of one expert
// are cut into tiles of this many rows (two accumulators of N = 2 x 112 fill TMEM).
constexpr int kPlanesTileTok = 112;
// Tokens per tile of cdg_gemm_direct_kernel (one plane: N = 224).
constexpr int kDirectTileTok = 224;
// Bytes per row of the direct class's activation scale codes: one per 128-wide K block,
// rounded up to 4 so that four consecutive K blocks of a row are one aligned 32-bit word.
__host__ __device__ constexpr int tok_code_pitch(int K) { return ((K / 128) + 3) & ~3; }

// Control words at the start of the workspace (int32 slots, zeroed before each call).
enum : int {
  kCtrlTicket = 0,
  kCtrlCount0 = 1,  // kCtrlCount0 + class = number of blocks in that class
  kCtrlPlaneTiles = 7,  // number of tiles in the planes kernel's tile list
  kCtrlStatus = 8,  // device status bits (kStatus*); kCtrlStatus + 1: code of the first wait that gave up
  kCtrlDirectTiles = 10,  // number of tiles in the direct kernel's tile list
  kCtrlSfInexact = 11,    // set when a float weight scale of the call is not a power of two
  kCtrlWords = 64,
};

constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Row ranges of the 128-row work tiles ("blocks").  The rows of A form `nseg`
// segments of `seg_rows` rows (the per-group blocks of the masked layout; a single
// segment of all M rows otherwise), each cut into ceil(seg_rows / 128) tiles that
// never cross a segment boundary, followed by the rows past the last segment in
// plain 128-row tiles.  Block b of the kernels covers rows [row0, row0 + n) of A
// and D; its activation planes and row exponents stay at rows [b*128, b*128 + n).
struct TileMap {
  int M = 0, seg_rows = 0, tiles_per_seg = 0, nseg = 0;

  __host__ __device__ static TileMap contiguous(int M) {
    TileMap t;
    t.M = M;
    t.seg_rows = M;
    t.tiles_per_seg = (M + 127) / 128;
    t.nseg = M > 0 ? 1 : 0;
    return t;
  }
  // M rows in G groups of M / G rows each (rows past G * (M / G) form the tail).
  __host__ __device__ static TileMap masked(int M, int G) {
    TileMap t;
    t.M = M;
    t.seg_rows = G > 0 ? M / G : 0;
    t.tiles_per_seg = (t.seg_rows + 127) / 128;
    t.nseg = t.seg_rows > 0 ? G : 0;
    return t;
  }
  __host__ __device__ int tail_start() const { return nseg * seg_rows; }
  __host__ __device__ int tiles() const { return nseg * tiles_per_seg + (M - tail_start() + 127) / 128; }
  __host__ __device__ void rows(int b, int& row0, int& n) const {
    const int seg_tiles = nseg * tiles_per_seg;
    if (b < seg_tiles) {
      const int s = b / tiles_per_seg, j = b - s * tiles_per_seg;
      row0 = s * seg_rows + j * 128;
      n = seg_rows - j * 128 < 128 ? seg_rows - j * 128 : 128;
    } else {
      row0 = tail_start() + (b - seg_tiles) * 128;
      n = M - row0 < 128 ? M - row0 : 128;
    }
  }
};

// Workspace regions of one GEMM call.
struct WorkspaceLayout {
  size_t ctrl = 0, blk_info = 0, blk_mask = 0, lists = 0, plane_tiles = 0, direct_tiles = 0, row_ids = 0, row_exp = 0,
         hilo = 0, tok_code = 0, tok_atoms = 0, sfw_atoms = 0, total = 0;

  static WorkspaceLayout make(int64_t M, int64_t nblk, int64_t K, int64_t N, int64_t E, bool fast, bool row_ids,
                              bool sfw_from_rows, bool planes_given = false) {
    WorkspaceLayout w;
    size_t off = 0;
    w.ctrl = off;
    off = align_up(off + kCtrlWords * 4, 1024);
    w.blk_info = off;
    off = align_up(off + static_cast<size_t>(nblk) * 16, 1024);
    w.blk_mask = off;
    off = align_up(off + static_cast<size_t>(nblk) * 16, 1024);
    w.lists = off;
    off = align_up(off + static_cast<size_t>(nblk) * 16 * kNumClasses, 1024);
    w.plane_tiles = off;  // at most one tile per 112 rows of a run plus one per run: 2 per block
    off = align_up(off + static_cast<size_t>(nblk) * 2 * 16, 1024);
    w.direct_tiles = off;  // tiles of up to 224 rows: at most one per block
    off = align_up(off + static_cast<size_t>(nblk) * 16, 1024);
    if (row_ids) {
      w.row_ids = off;
      off = align_up(off + static_cast<size_t>(M) * 4, 1024);
    }
    if (fast) {
      if (!planes_given) {  // otherwise the caller's planes and row exponents are used
        w.row_exp = off;
        off = align_up(off + static_cast<size_t>(nblk) * 128 * 4, 1024);
        w.hilo = off;
        off = align_up(off + static_cast<size_t>(2) * nblk * 128 * K, 1024);
      }
      w.tok_code = off;  // [M][tok_code_pitch(K)] UE8M0 activation scale codes of the direct class's rows
      off = align_up(off + static_cast<size_t>(tok_code_pitch(K)) * static_cast<size_t>(M), 1024);
      w.tok_atoms = off;  // [direct tile][K/512 scale stage][2][128] words: token scale atoms
      off = align_up(off + static_cast<size_t>(nblk) * (tok_code_pitch(K) / 4) * 1024, 1024);
      if (sfw_from_rows) {
        w.sfw_atoms = off;
        off = align_up(off + static_cast<size_t>(E) * ((N + 127) / 128) * (K / 128) * 512, 1024);
      }
    }
    w.total = off;
    return w;
  }
};

}  // namespace cdg
