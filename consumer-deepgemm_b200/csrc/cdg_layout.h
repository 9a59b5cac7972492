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
  kNumClasses = 5,
};
constexpr int kTinyTok = 16;
constexpr int kNarrowTok = 32;

// Control words at the start of the workspace (int32 slots, zeroed before each call).
enum : int {
  kCtrlTicket = 0,
  kCtrlCount0 = 1,  // kCtrlCount0 + class = number of blocks in that class
  kCtrlStatus = 8,  // device status bits (kStatus*)
  kCtrlWords = 64,
};

constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Workspace regions of one GEMM call.
struct WorkspaceLayout {
  size_t ctrl = 0, blk_info = 0, blk_mask = 0, lists = 0, row_ids = 0, row_exp = 0, hilo = 0, sfw_atoms = 0, total = 0;

  static WorkspaceLayout make(int64_t M, int64_t K, int64_t N, int64_t E, bool fast, bool psum, bool sfw_from_rows) {
    WorkspaceLayout w;
    const int64_t nblk = (M + 127) / 128;
    size_t off = 0;
    w.ctrl = off;
    off = align_up(off + kCtrlWords * 4, 1024);
    w.blk_info = off;
    off = align_up(off + static_cast<size_t>(nblk) * 16, 1024);
    w.blk_mask = off;
    off = align_up(off + static_cast<size_t>(nblk) * 16, 1024);
    w.lists = off;
    off = align_up(off + static_cast<size_t>(nblk) * 4 * kNumClasses, 1024);
    if (psum) {
      w.row_ids = off;
      off = align_up(off + static_cast<size_t>(M) * 4, 1024);
    }
    if (fast) {
      w.row_exp = off;
      off = align_up(off + static_cast<size_t>(nblk) * 128 * 4, 1024);
      w.hilo = off;
      off = align_up(off + static_cast<size_t>(2) * nblk * 128 * K, 1024);
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
