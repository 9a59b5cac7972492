// Kernels around the grouped GEMM for a mixture-of-experts layer, and the
// bookkeeping of expert parallelism (experts sharded over ranks, token rows
// exchanged with all-to-all collectives issued by the host).
//
//   cdg_quant_fp8_rows        BF16/FP32 rows -> e4m3 + FP32 scale per 128 columns
//   cdg_silu_mul_quant_fp8    [gate | up] BF16 rows -> e4m3(silu(gate) * up) + scales
//   cdg_ep_count              routed rows per expert
//   cdg_ep_pack               routed rows -> send buffer grouped by destination rank
//   cdg_ep_permute            received rows -> 128-aligned contiguous layout per local expert
//   cdg_ep_quant_pack_fixed   BF16 rows -> quantised packed rows in fixed-capacity regions
//                             with per-expert count headers (exchange without host sync)
//   cdg_ep_permute_fixed      fixed-capacity receive buffer -> contiguous layout
//   cdg_ep_unpermute          GEMM rows -> received order
//   cdg_ep_combine            returned rows -> weighted top-k sum per token
//   cdg_ep_unpermute_combine  both in one pass, for a layer without an exchange
//
// Row order inside a destination or an expert group comes from atomics and is
// not deterministic; every row is computed independently and returned to its
// (token, slot) place, so results are.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "cdg_b200.h"
#include "cdg_split.cuh"

namespace cdg {
namespace {

__device__ __forceinline__ float load_f(const void* p, int dtype, int64_t i) {
  return dtype == CDG_DTYPE_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i])
                                 : static_cast<const float*>(p)[i];
}

__device__ __forceinline__ int64_t load_idx(const void* p, int dtype, int64_t i) {
  return dtype == CDG_DTYPE_I64 ? static_cast<const int64_t*>(p)[i]
                                : static_cast<int64_t>(static_cast<const int32_t*>(p)[i]);
}

// Bytes of one dispatched row: [e4m3 data H][FP32 scales H/128][int32 local expert][pad to 16].
__host__ __device__ __forceinline__ int64_t packed_row_bytes(int64_t H) { return (H + 4 * (H / 128) + 4 + 15) / 16 * 16; }

// Bytes of one row of the peer-memory exchange: [e4m3 data H][FP32 scales H/128][int32
// source token][topk x int32: the local expert of the token's slot j, or -1 when slot j goes
// to another rank][pad to 16].  A token sends one such row to each rank that owns at least
// one of its experts; the receiver expands it into every listed expert's group.
__host__ __device__ __forceinline__ int64_t p2p_row_bytes(int64_t H, int64_t topk) {
  return (H + 4 * (H / 128) + 4 + 4 * topk + 15) / 16 * 16;
}

// Exchange window of one rank: [0, 512) dispatch flags int32[ranks], [512, 1024) return
// flags int32[ranks], [1024, 1028) status, [1028, 1032) the number of completed exchanges
// (the step counter: a step's epoch is its value + 1); from 4096 the receive regions
// [2 parity][ranks source][1 + tokens rows][row bytes] (row 0 of a region is a header:
// int32 per-local-expert slot counts, then the number of rows), then (256-aligned) the
// return rows [2 parity][tokens * topk][H] BF16, indexed by this rank's own slot t * topk + j.
struct Window {
  int64_t ranks, tokens, topk, H, rb;
  static constexpr int64_t kDispatchFlags = 0, kReturnFlags = 512, kStatus = 1024, kEpoch = 1028, kRecv = 4096;
  __host__ __device__ int64_t region(int64_t parity, int64_t src) const {
    return kRecv + (parity * ranks + src) * (tokens + 1) * rb;
  }
  __host__ __device__ int64_t ret_base() const { return (region(2, 0) + 255) / 256 * 256; }
  __host__ __device__ int64_t ret_parity(int64_t parity) const { return ret_base() + parity * tokens * topk * H * 2; }
  __host__ __device__ int64_t bytes() const { return ret_parity(2); }
};

__host__ __device__ inline Window make_window(int64_t ranks, int64_t tokens, int64_t topk, int64_t H) {
  return Window{ranks, tokens, topk, H, p2p_row_bytes(H, topk)};
}

// What the peer-memory exchange kernels need: every rank's window (device array), this
// rank's window and index, and the window layout.  The step's epoch (flag value and buffer
// parity) is read from the own window's counter, so the kernels take no per-step host
// argument and a whole exchange step can be captured in a CUDA graph.
struct PeerStep {
  const uint64_t* peers = nullptr;
  uint8_t* own = nullptr;
  Window win{};
  int me = 0;
  __device__ int32_t epoch() const { return *reinterpret_cast<const volatile int32_t*>(own + Window::kEpoch) + 1; }
};

// ---- cross-GPU flags of the peer-memory exchange (system scope: the writer is another GPU)
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bound of every wait on another rank's flag, per device (cdg_ep_set_wait_timeout_ns).
constexpr uint64_t kPeerWaitNs = 2000000000ull;  // 2 s
__device__ uint64_t g_peer_wait_ns = kPeerWaitNs;

// Sticky per-device record of the exchange's device-side errors ([0] status bits, [1] the first
// wait code); cdg_device_status() reads it together with the GEMM's.
__device__ int g_ep_sticky_status[2];

// Wait codes of the peer waits: role 8 = dispatch flag (permute), 9 = return flag (combine),
// then the source rank whose flag did not arrive.
__device__ __forceinline__ int peer_wait_code(int role, int src) {
  return static_cast<int>((static_cast<uint32_t>(role & 15) << 28) | static_cast<uint32_t>(src & 0xFFFF));
}

// Thread 0 of the CTA waits until flags[0 .. n) all reach `epoch` (bounded by
// g_peer_wait_ns); the CTA then proceeds only if they did.  A wait that gives up sets bit 0
// of *status (the window's status word) and the sticky per-device record.
__device__ bool wait_peer_flags(const int32_t* flags, int n, int32_t epoch, int32_t* status, int role) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t limit = *reinterpret_cast<volatile uint64_t*>(&g_peer_wait_ns);
    const uint64_t t0 = now_ns();
    for (int i = 0; i < n && ok; ++i) {
      while (ld_acquire_sys(flags + i) < epoch) {
        if (now_ns() - t0 > limit) {
          atomicOr(status, 1);
          atomicOr(&g_ep_sticky_status[0], 1);
          atomicCAS(&g_ep_sticky_status[1], 0, peer_wait_code(role, i));
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Quantise one 128-wide block held by a warp (4 values per lane) to e4m3 (FP32 arithmetic,
// round to nearest even; amax clamped at 1e-12).
// pow2 == 0: the per_block_cast_to_fp8 recipe, scale = amax / 448, q = e4m3(x / amax * 448).
// pow2 != 0: the UE8M0 recipe (DeepGEMM's per-token cast with use_ue8m0 on SM100): scale =
//   amax / 448 rounded up to a power of two (exactly: next exponent unless the mantissa is
//   zero), q = e4m3(x / scale).  Such scales make the GEMM take its direct class.
// quant_block_values returns the lane's four codes (one 32-bit word) and the block's scale;
// quant_block_warp stores them.
__device__ __forceinline__ uint32_t quant_block_values(const float (&v)[4], int pow2, float& scale) {
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-12f);
  uint32_t sb = __float_as_uint(amax / 448.0f);
  if (sb & 0x007FFFFFu) sb = (sb & 0xFF800000u) + 0x00800000u;
  const float s2 = __uint_as_float(sb);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float y = pow2 ? v[i] / s2 : v[i] / amax * 448.0f;
    packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3)) << (8 * i);
  }
  scale = pow2 ? s2 : amax / 448.0f;
  return packed;
}

// The same block quantisation with one division per block instead of one per element: the
// scale is the one above, the codes take x * (448 / amax) (FP32 recipe) or x * (1 / s)
// (power-of-two recipe, where it equals x / s exactly).  For the FP32 recipe the code can
// differ from e4m3(x / amax * 448) only where the two roundings fall on opposite sides of an
// e4m3 rounding point (a 1-in-2^18 event); used where the input is itself computed (SiLU-mul).
__device__ __forceinline__ uint32_t quant_block_values_mul(const float (&v)[4], int pow2, float& scale) {
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-12f);
  uint32_t sb = __float_as_uint(amax / 448.0f);
  if (sb & 0x007FFFFFu) sb = (sb & 0xFF800000u) + 0x00800000u;
  const float s2 = __uint_as_float(sb);
  const float r = pow2 ? 1.0f / s2 : 448.0f / amax;
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(v[i] * r, __NV_SATFINITE, __NV_E4M3)) << (8 * i);
  scale = pow2 ? s2 : amax / 448.0f;
  return packed;
}

// silu(g) * u in FP32 with the fast exponential and the fast (two-instruction) division:
// g / (1 + e^-g) * u.  For g below about -88 the divisor is infinite and the result 0, the
// limit.  The SiLU-mul kernels are issue-bound (77% of issue slots busy), and the correctly
// rounded reciprocal's extra instructions cost them about a fifth of their time (the c4
// layer's SiLU-mul step: 1.06 -> 0.83 ms); the results differ in the last bit of a few
// values, which moves an e4m3 code by one step in a small fraction of cases.
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

__device__ __forceinline__ void quant_block_warp_mul(const float (&v)[4], uint8_t* q, float* scale_out, int lane,
                                                     int pow2) {
  float scale;
  reinterpret_cast<uint32_t*>(q)[lane] = quant_block_values_mul(v, pow2, scale);
  if (lane == 0) *scale_out = scale;
}

__device__ __forceinline__ void quant_block_warp(const float (&v)[4], uint8_t* q, float* scale_out, int lane,
                                                 int pow2) {
  float scale;
  reinterpret_cast<uint32_t*>(q)[lane] = quant_block_values(v, pow2, scale);
  if (lane == 0) *scale_out = scale;
}

// One warp per (row, 128-column block).
__global__ void quant_rows_kernel(const void* x, int x_dtype, int64_t x_stride, int64_t M, int64_t K, uint8_t* q,
                                  int64_t q_stride, float* s, int64_t s_stride_m, int64_t s_stride_k, int pow2) {
  const int64_t kb_count = K / 128;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= M * kb_count) return;
  const int64_t r = w / kb_count, kb = w - r * kb_count;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = load_f(x, x_dtype, r * x_stride + kb * 128 + lane * 4 + i);
  quant_block_warp(v, q + r * q_stride + kb * 128, s + r * s_stride_m + kb * s_stride_k, lane, pow2);
}

// Four values of a 128-column block for lane `lane` (BF16 or FP32 row, 16-byte aligned).
__device__ __forceinline__ void load_block4(const void* x, int x_dtype, int64_t base, float (&v)[4]) {
  if (x_dtype == CDG_DTYPE_BF16) {
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(x) + base));
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  } else {
    const float4 f = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(x) + base));
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  }
}

// One warp quantises row x[row_off .. row_off + H) (quant_block_values: the
// per_block_cast_to_fp8 or power-of-two recipe, bit for bit) into codes[H] and scales[H/128]
// in shared memory; the loads of eight 128-column blocks are issued before the first is used.
__device__ __forceinline__ void warp_quant_row(const void* x, int x_dtype, int64_t row_off, int64_t H, uint8_t* codes,
                                               float* scales, int lane, int pow2) {
  const int64_t nkb = H / 128;
  for (int64_t kb0 = 0; kb0 < nkb; kb0 += 8) {
    float v[8][4];
#pragma unroll
    for (int b = 0; b < 8; ++b)
      if (kb0 + b < nkb) load_block4(x, x_dtype, row_off + (kb0 + b) * 128 + lane * 4, v[b]);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (kb0 + b < nkb) {
        float sc;
        reinterpret_cast<uint32_t*>(codes + (kb0 + b) * 128)[lane] = quant_block_values(v[b], pow2, sc);
        if (lane == 0) scales[kb0 + b] = sc;
      }
    }
  }
}

// The row exponent E of the activation planes (cdg_split.cuh) from a row's nkb FP32 scales,
// by the whole warp: the frexp exponent of the largest finite |bf16(s)|, clamped to the range
// the MMA scale factors take (scales produced by the 1x128 recipe from finite BF16/FP32 rows
// always lie inside it).
__device__ __forceinline__ int warp_plane_exponent(const float* scales, int64_t nkb, int lane) {
  float m = 0.0f;
  for (int64_t kb = lane; kb < nkb; kb += 32) {
    const float sb = fabsf(bf16_round(scales[kb]));
    if (isfinite(sb)) m = fmaxf(m, sb);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  bool in_range = true;
  const int e = plane_exponent(m, &in_range);
  return e < -126 ? -126 : e > 127 ? 127 : e;
}

// Shared-memory stage of one quantised row: codes, then scales, 16-byte aligned.
__host__ __device__ __forceinline__ int64_t row_stage_bytes(int64_t H) { return (H + 4 * (H / 128) + 15) / 16 * 16; }

constexpr int kP2pWarps = 4;  // tokens per CTA of the peer dispatch, one warp each

// Quantise and lay out for the grouped GEMM in one pass, when there is no exchange (one rank).
// Warp w of CTA c takes token t = c * kP2pWarps + w; lane j < topk claims slot j's row in
// the contiguous layout (row expert_off[e] + a per-expert counter, e = topk_ids[t, j] in
// [0, E)); the warp quantises the token's row once into shared memory (warp_quant_row, the
// same bits as per_block_cast_to_fp8 or the power-of-two recipe) and copies the codes
// (16-byte stores) and scales into every claimed row.  perm_pos[t*topk + j] is that row and
// send_index[t*topk + j] the slot itself (-1 for skipped slots), the form the combine step
// reads.  fill: [E] counters, zeroed by the host.
// Planes form (planes != nullptr; A and SA unused): each claimed row gets the row's two e4m3
// planes (planes[0][row], planes[1][row], plane stride M_pad * H) and row_exp[row] = E, the
// split the GEMM's prep kernel would make of the codes and scales (cdg_split.cuh).
__global__ void __launch_bounds__(kP2pWarps * 32) ep_quant_dispatch_local_kernel(
    const void* x, int x_dtype, int64_t x_stride, const void* ids, int ids_dtype, int64_t T, int64_t topk, int64_t E,
    int64_t H, const int64_t* expert_off, int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices,
    int32_t* perm_pos, int32_t* send_index, int pow2, uint8_t* planes = nullptr, int32_t* row_exp = nullptr,
    int64_t M_pad = 0) {
  constexpr int kMaxTopk = 32;
  extern __shared__ __align__(16) uint8_t local_stage[];
  __shared__ int64_t s_row[kP2pWarps][kMaxTopk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kP2pWarps + warp;
  if (t >= T) return;  // warp-uniform; no block-wide barrier follows
  if (lane < topk) {
    const int64_t i = t * topk + lane;
    const int64_t e = load_idx(ids, ids_dtype, i);
    int64_t row = -1;
    if (e >= 0 && e < E) {
      row = expert_off[e] + atomicAdd(&fill[e], 1);
      m_indices[row] = static_cast<int32_t>(e);
    }
    s_row[warp][lane] = row;
    perm_pos[i] = static_cast<int32_t>(row);
    send_index[i] = row >= 0 ? static_cast<int32_t>(i) : -1;
  }
  uint8_t* stage = local_stage + warp * row_stage_bytes(H);
  const float* scales = reinterpret_cast<const float*>(stage + H);
  warp_quant_row(x, x_dtype, t * x_stride, H, stage, reinterpret_cast<float*>(stage + H), lane, pow2);
  __syncwarp();
  if (planes) {
    const int e = warp_plane_exponent(scales, H / 128, lane);
    const float inv = ldexpf(1.0f, -e);
    const int64_t plane = M_pad * H;
    for (int64_t c = lane; c < H / 16; c += 32) {
      uint4 hi, lo;
      split_planes16(reinterpret_cast<const uint4*>(stage)[c], bf16_round(scales[c >> 3]), inv, hi, lo);
      for (int j = 0; j < topk; ++j) {
        const int64_t row = s_row[warp][j];
        if (row < 0) continue;
        reinterpret_cast<uint4*>(planes + row * H)[c] = hi;
        reinterpret_cast<uint4*>(planes + plane + row * H)[c] = lo;
      }
    }
    if (lane < topk && s_row[warp][lane] >= 0) row_exp[s_row[warp][lane]] = e;
    return;
  }
  for (int j = 0; j < topk; ++j) {
    const int64_t row = s_row[warp][j];
    if (row < 0) continue;
    for (int64_t c = lane; c < H / 16; c += 32)
      reinterpret_cast<uint4*>(A + row * H)[c] = reinterpret_cast<const uint4*>(stage)[c];
    for (int64_t c = lane; c < H / 128; c += 32) SA[row * (H / 128) + c] = scales[c];
  }
}

// One warp per (row, kSiluBlocks 128-column blocks of the output); gate = columns [0, I),
// up = [I, 2I); rows 8-byte aligned.  The lane's four gate and four up values of each block
// arrive as one 8-byte load each, all of the warp's blocks issued before any is used, and the
// row's m_indices entry is loaded alongside (a padding row's values are read and dropped), so
// that a warp waits for memory once.
constexpr int kSiluBlocks = 4;
__global__ void __launch_bounds__(256) silu_mul_quant_vec_kernel(const __nv_bfloat16* in, int64_t in_stride,
                                                                 int64_t M, int64_t I, const int32_t* m_indices,
                                                                 uint8_t* q, int64_t q_stride, float* s,
                                                                 int64_t s_stride_m, int64_t s_stride_k, int pow2) {
  const int64_t kb_count = I / 128;
  const int64_t chunks = (kb_count + kSiluBlocks - 1) / kSiluBlocks;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= M * chunks) return;
  const int64_t r = w / chunks, kb0 = (w - r * chunks) * kSiluBlocks;
  const int nb = kb_count - kb0 < kSiluBlocks ? static_cast<int>(kb_count - kb0) : kSiluBlocks;
  const int32_t id = m_indices ? __ldg(m_indices + r) : 0;
  const __nv_bfloat16* gp = in + r * in_stride + kb0 * 128 + lane * 4;
  uint2 g2[kSiluBlocks], u2[kSiluBlocks];
#pragma unroll
  for (int b = 0; b < kSiluBlocks; ++b) {
    if (b < nb) {
      g2[b] = __ldg(reinterpret_cast<const uint2*>(gp + b * 128));
      u2[b] = __ldg(reinterpret_cast<const uint2*>(gp + I + b * 128));
    }
  }
  if (id < 0) return;  // padding row: never read by the next GEMM
#pragma unroll
  for (int b = 0; b < kSiluBlocks; ++b) {
    if (b < nb) {
      const float2 g01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&g2[b].x));
      const float2 g23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&g2[b].y));
      const float2 u01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u2[b].x));
      const float2 u23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u2[b].y));
      const float gv[4] = {g01.x, g01.y, g23.x, g23.y}, uv[4] = {u01.x, u01.y, u23.x, u23.y};
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = silu_mul(gv[i], uv[i]);
      quant_block_warp_mul(v, q + r * q_stride + (kb0 + b) * 128, s + r * s_stride_m + (kb0 + b) * s_stride_k,
                           lane, pow2);
    }
  }
}

// The 16-byte path (rows and codes 16-byte aligned): one warp per (row, four 128-column blocks
// of the output), eight lanes per block and sixteen columns per lane: two 16-byte loads of gate
// values, two of up values, one 16-byte store of codes, the block's amax over its eight lanes in
// three shuffles, and two conversions to e4m3 per instruction.  A grid of a few CTAs per SM
// strides over the items; a row whose m_indices entry is negative is skipped before any of its
// values is read.  Same arithmetic as the paths above (silu_mul, quant_block_values_mul).
// KB: the row's 128-column blocks when known at compile time (0: from I); the warp's (row,
// chunk) split is then a shift instead of a 64-bit division.
template <int KB>
__global__ void __launch_bounds__(256) silu_mul_quant_16b_kernel(const __nv_bfloat16* in, int64_t in_stride,
                                                                 int64_t M, int64_t I, const int32_t* m_indices,
                                                                 uint8_t* q, int64_t q_stride, float* s,
                                                                 int64_t s_stride_m, int64_t s_stride_k, int pow2) {
  if (KB) I = KB * 128;
  const int64_t kb_count = I / 128;
  const int64_t chunks = (kb_count + 3) / 4;
  const int64_t items = M * chunks;
  const int lane = threadIdx.x & 31, sub = lane & 7, blk = lane >> 3;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < items;
       w += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int64_t r = w / chunks;
    const int64_t kb = (w - r * chunks) * 4 + blk;
    if (m_indices && __ldg(m_indices + r) < 0) continue;  // padding row (warp-uniform): never read by the next GEMM
    const bool on = kb < kb_count;
    const int64_t col = kb * 128 + sub * 16;
    uint4 raw[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    if (on) {
      const uint4* gp = reinterpret_cast<const uint4*>(in + r * in_stride + col);
      const uint4* up = reinterpret_cast<const uint4*>(in + r * in_stride + I + col);
      raw[0] = __ldg(gp);
      raw[1] = __ldg(gp + 1);
      raw[2] = __ldg(up);
      raw[3] = __ldg(up + 1);
    }
    float v[16];
    float amax = 0.0f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t gw[4] = {raw[h].x, raw[h].y, raw[h].z, raw[h].w};
      const uint32_t uw[4] = {raw[2 + h].x, raw[2 + h].y, raw[2 + h].z, raw[2 + h].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 g2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[i]));
        const float2 u2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uw[i]));
        v[h * 8 + 2 * i] = silu_mul(g2.x, u2.x);
        v[h * 8 + 2 * i + 1] = silu_mul(g2.y, u2.y);
        amax = fmaxf(amax, fmaxf(fabsf(v[h * 8 + 2 * i]), fabsf(v[h * 8 + 2 * i + 1])));
      }
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));  // the block's 8 lanes
    amax = fmaxf(amax, 1e-12f);
    uint32_t sb = __float_as_uint(amax / 448.0f);
    if (sb & 0x007FFFFFu) sb = (sb & 0xFF800000u) + 0x00800000u;
    const float s2 = __uint_as_float(sb);
    const float rcp = pow2 ? 1.0f / s2 : 448.0f / amax;
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i] * rcp, v[4 * i + 1] * rcp), __NV_SATFINITE,
                                                   __NV_E4M3);
      const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i + 2] * rcp, v[4 * i + 3] * rcp),
                                                   __NV_SATFINITE, __NV_E4M3);
      packed[i] = (lo & 0xFFFFu) | (hi << 16);
    }
    if (on) {
      *reinterpret_cast<uint4*>(q + r * q_stride + col) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      if (sub == 0) s[r * s_stride_m + kb * s_stride_k] = pow2 ? s2 : amax / 448.0f;
    }
  }
}

// Planes form of the SiLU-mul requant (16-byte aligned rows): one warp per row.  The row's
// codes and scales are formed as in silu_mul_quant_16b_kernel (the same bits) into shared
// memory, then the row is split into the GEMM's two e4m3 planes (cdg_split.cuh):
// planes[0][r], planes[1][r] (plane stride M * I) and row_exp[r].  Rows whose m_indices entry
// is negative are skipped.
// KB: the row's 128-column blocks when known at compile time (0: from I), so that the common
// widths run fully unrolled loops (the kernel is issue-bound).
template <int KB>
__global__ void __launch_bounds__(256) silu_mul_quant_planes_kernel(const __nv_bfloat16* in, int64_t in_stride,
                                                                    int64_t M, int64_t I, const int32_t* m_indices,
                                                                    uint8_t* planes, int32_t* row_exp) {
  extern __shared__ __align__(16) uint8_t act_stage[];
  if (KB) I = KB * 128;
  const int64_t kb_count = I / 128;
  const int64_t chunks = (kb_count + 3) / 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane & 7, blk = lane >> 3;
  uint8_t* codes = act_stage + warp * row_stage_bytes(I);
  float* scales = reinterpret_cast<float*>(codes + I);
  const int64_t plane = M * I;
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < M;
       r += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    if (m_indices && __ldg(m_indices + r) < 0) continue;  // warp-uniform
    for (int64_t ch = 0; ch < chunks; ++ch) {
      const int64_t kb = ch * 4 + blk;
      const bool on = kb < kb_count;
      const int64_t col = kb * 128 + sub * 16;
      uint4 raw[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      if (on) {
        const uint4* gp = reinterpret_cast<const uint4*>(in + r * in_stride + col);
        const uint4* up = reinterpret_cast<const uint4*>(in + r * in_stride + I + col);
        raw[0] = __ldg(gp);
        raw[1] = __ldg(gp + 1);
        raw[2] = __ldg(up);
        raw[3] = __ldg(up + 1);
      }
      float v[16];
      float amax = 0.0f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t gw[4] = {raw[h].x, raw[h].y, raw[h].z, raw[h].w};
        const uint32_t uw[4] = {raw[2 + h].x, raw[2 + h].y, raw[2 + h].z, raw[2 + h].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 g2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[i]));
          const float2 u2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uw[i]));
          v[h * 8 + 2 * i] = silu_mul(g2.x, u2.x);
          v[h * 8 + 2 * i + 1] = silu_mul(g2.y, u2.y);
          amax = fmaxf(amax, fmaxf(fabsf(v[h * 8 + 2 * i]), fabsf(v[h * 8 + 2 * i + 1])));
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      amax = fmaxf(amax, 1e-12f);
      const float rcp = 448.0f / amax;
      uint32_t packed[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i] * rcp, v[4 * i + 1] * rcp), __NV_SATFINITE,
                                                     __NV_E4M3);
        const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i + 2] * rcp, v[4 * i + 3] * rcp),
                                                     __NV_SATFINITE, __NV_E4M3);
        packed[i] = (lo & 0xFFFFu) | (hi << 16);
      }
      if (on) {
        *reinterpret_cast<uint4*>(codes + col) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        if (sub == 0) scales[kb] = amax / 448.0f;
      }
    }
    __syncwarp();
    const int e = warp_plane_exponent(scales, kb_count, lane);
    const float inv = ldexpf(1.0f, -e);
    for (int64_t c = lane; c < I / 16; c += 32) {
      uint4 hi, lo;
      split_planes16(reinterpret_cast<const uint4*>(codes)[c], bf16_round(scales[c >> 3]), inv, hi, lo);
      reinterpret_cast<uint4*>(planes + r * I)[c] = hi;
      reinterpret_cast<uint4*>(planes + plane + r * I)[c] = lo;
    }
    if (lane == 0) row_exp[r] = e;
    __syncwarp();  // the stage is rewritten for the next row
  }
}

// The same for rows that are not 8-byte aligned: one warp per (row, 128-column block), one
// 2-byte load per value.
__global__ void silu_mul_quant_kernel(const __nv_bfloat16* in, int64_t in_stride, int64_t M, int64_t I,
                                      const int32_t* m_indices, uint8_t* q, int64_t q_stride, float* s,
                                      int64_t s_stride_m, int64_t s_stride_k, int pow2) {
  const int64_t kb_count = I / 128;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= M * kb_count) return;
  const int64_t r = w / kb_count, kb = w - r * kb_count;
  if (m_indices && m_indices[r] < 0) return;  // padding row: never read by the next GEMM
  const __nv_bfloat16* gp = in + r * in_stride + kb * 128 + lane * 4;
  float gv[4], uv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    gv[i] = __bfloat162float(gp[i]);
    uv[i] = __bfloat162float(gp[I + i]);
  }
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = silu_mul(gv[i], uv[i]);
  quant_block_warp_mul(v, q + r * q_stride + kb * 128, s + r * s_stride_m + kb * s_stride_k, lane, pow2);
}

// Per-CTA histogram in shared memory (when E fits), then one global atomic per CTA and expert:
// the global counters of a few hundred experts see a few hundred atomics each instead of one
// per routed slot.  With `offsets` (and `ticket`, zeroed by the host), the last CTA also writes
// the start row of each expert's group in the 128-aligned contiguous layout,
// offsets[e] = sum over e' < e of ceil128(cnt[e']).
constexpr int kCountSmemExperts = 4096;
__global__ void ep_count_kernel(const void* ids, int ids_dtype, int64_t n, int64_t E, int32_t* cnt,
                                int64_t* offsets = nullptr, int32_t* ticket = nullptr) {
  __shared__ int32_t s_cnt[kCountSmemExperts];
  __shared__ int64_t s_part[1024];
  __shared__ int s_last;
  const bool local = E <= kCountSmemExperts;
  if (local)
    for (int64_t e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = load_idx(ids, ids_dtype, i);
    if (e >= 0 && e < E) atomicAdd(local ? &s_cnt[e] : &cnt[e], 1);
  }
  if (local) {
    __syncthreads();
    for (int64_t e = threadIdx.x; e < E; e += blockDim.x)
      if (s_cnt[e]) atomicAdd(&cnt[e], s_cnt[e]);
  }
  if (!offsets) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // exclusive scan of the aligned counts: a contiguous run of experts per thread, then the
  // threads' totals in shared memory
  const int64_t per = (E + blockDim.x - 1) / blockDim.x;
  const int64_t e0 = (E < static_cast<int64_t>(threadIdx.x) * per ? E : static_cast<int64_t>(threadIdx.x) * per);
  const int64_t e1 = E < e0 + per ? E : e0 + per;
  int64_t tot = 0;
  for (int64_t e = e0; e < e1; ++e) tot += (__ldcg(&cnt[e]) + 127) / 128 * 128;
  s_part[threadIdx.x] = tot;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t run = 0;
    for (int t = 0; t < static_cast<int>(blockDim.x); ++t) {
      const int64_t v = s_part[t];
      s_part[t] = run;
      run += v;
    }
  }
  __syncthreads();
  int64_t off = s_part[threadIdx.x];
  for (int64_t e = e0; e < e1; ++e) {
    offsets[e] = off;
    off += (__ldcg(&cnt[e]) + 127) / 128 * 128;
  }
}


// One warp per routed (token, slot): copies the token's e4m3 row and scales into one packed row.
__global__ void ep_pack_kernel(const uint8_t* xq, int64_t xq_stride, const float* xs, int64_t xs_stride, const void* ids,
                               int ids_dtype, int64_t T, int64_t topk, int64_t E, int64_t e_per_rank, int64_t H,
                               const int64_t* send_off, int32_t* fill, uint8_t* out_rows, int32_t* send_index) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= T * topk) return;
  const int64_t e = load_idx(ids, ids_dtype, w);
  int64_t row = -1;
  if (e >= 0 && e < E) {
    const int64_t dest = e / e_per_rank;
    int slot = 0;
    if (lane == 0) slot = atomicAdd(&fill[dest], 1);
    row = send_off[dest] + __shfl_sync(0xffffffffu, slot, 0);
  }
  if (lane == 0) send_index[w] = static_cast<int32_t>(row);
  if (row < 0) return;
  const int64_t t = w / topk;
  uint8_t* out = out_rows + row * packed_row_bytes(H);
  const uint4* src = reinterpret_cast<const uint4*>(xq + t * xq_stride);
  uint4* dst = reinterpret_cast<uint4*>(out);
  for (int64_t c = lane; c < H / 16; c += 32) dst[c] = src[c];
  float* out_s = reinterpret_cast<float*>(out + H);
  for (int64_t c = lane; c < H / 128; c += 32) out_s[c] = xs[t * xs_stride + c];
  if (lane == 0) *reinterpret_cast<int32_t*>(out + H + 4 * (H / 128)) = static_cast<int32_t>(e % e_per_rank);
}

// One warp per received packed row.
__global__ void ep_permute_kernel(const uint8_t* rows, int64_t R, int64_t H, const int64_t* expert_off, int32_t* fill,
                                  uint8_t* A, float* SA, int32_t* m_indices, int32_t* perm_pos) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= R) return;
  const uint8_t* in = rows + w * packed_row_bytes(H);
  const int e = *reinterpret_cast<const int32_t*>(in + H + 4 * (H / 128));
  int slot = 0;
  if (lane == 0) slot = atomicAdd(&fill[e], 1);
  const int64_t pos = expert_off[e] + __shfl_sync(0xffffffffu, slot, 0);
  const uint4* src = reinterpret_cast<const uint4*>(in);
  uint4* dst = reinterpret_cast<uint4*>(A + pos * H);
  for (int64_t c = lane; c < H / 16; c += 32) dst[c] = src[c];
  const float* rs = reinterpret_cast<const float*>(in + H);
  for (int64_t c = lane; c < H / 128; c += 32) SA[pos * (H / 128) + c] = rs[c];
  if (lane == 0) {
    m_indices[pos] = e;
    perm_pos[w] = static_cast<int32_t>(pos);
  }
}

// Fixed-capacity exchange layout: per destination rank a region of 1 + cap packed rows.
// Row 0 of a region is a header holding, as int32, the number of rows the sender
// routed to each of the destination's local experts; rows 1 .. n follow (n = the sum of
// the header), the rest of the region is unused.  The receive buffer has the same
// layout per source rank, so the counts arrive with the rows in one all-to-all.
constexpr int kFixedMaxExperts = 1024, kFixedMaxRanks = 256;

// One CTA of 4 warps per routed (token, slot): thread 0 takes the row's slot in the
// destination's region, then the warps quantise the token's row (per_block_cast_to_fp8
// recipe, 128-column blocks dealt round-robin to the warps) straight into it.
// Per-destination, per-local-expert counts go to `scratch`; the last CTA writes them into
// the region headers.  scratch (zeroed by the host): [ranks] fill, [ranks * E_local]
// counts, [1] ticket.
__global__ void __launch_bounds__(128) ep_quant_pack_fixed_kernel(const void* x, int x_dtype, int64_t x_stride,
                                                                  const void* ids, int ids_dtype, int64_t T,
                                                                  int64_t topk, int64_t E, int64_t e_per_rank,
                                                                  int64_t ranks, int64_t H, int64_t cap,
                                                                  int32_t* scratch, uint8_t* out_rows,
                                                                  int32_t* send_index, int pow2) {
  __shared__ int s_last;
  __shared__ int64_t s_row, s_e;
  int32_t* fill = scratch;
  int32_t* cnt = scratch + ranks;
  int32_t* ticket = cnt + ranks * e_per_rank;
  const int64_t w = blockIdx.x;  // the (token, slot) of this CTA
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rb = packed_row_bytes(H);
  if (threadIdx.x == 0) {
    int64_t row = -1;
    const int64_t e = w < T * topk ? load_idx(ids, ids_dtype, w) : -1;
    if (e >= 0 && e < E) {
      const int64_t dest = e / e_per_rank;
      const int slot = atomicAdd(&fill[dest], 1);
      atomicAdd(&cnt[dest * e_per_rank + e % e_per_rank], 1);
      if (slot < cap) row = dest * (cap + 1) + 1 + slot;
    }
    if (w < T * topk) send_index[w] = static_cast<int32_t>(row);
    s_row = row;
    s_e = e;
  }
  __syncthreads();
  const int64_t row = s_row;
  auto row_ptr = [&](int64_t r) -> uint8_t* { return out_rows + r * rb; };
  if (row >= 0) {
    const int64_t t = w / topk;
    uint8_t* out = row_ptr(row);
    float* out_s = reinterpret_cast<float*>(out + H);
    for (int64_t kb = warp; kb < H / 128; kb += blockDim.x / 32) {
      float v[4];
      const int64_t base = t * x_stride + kb * 128 + lane * 4;
      if (x_dtype == CDG_DTYPE_BF16) {
        const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(x) + base);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
        const float2 f0 = __bfloat1622float2(h2[0]), f1 = __bfloat1622float2(h2[1]);
        v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
      } else {
        const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + base);
        v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
      }
      quant_block_warp(v, out + kb * 128, out_s + kb, lane, pow2);
    }
    if (threadIdx.x == 0) *reinterpret_cast<int32_t*>(out + H + 4 * (H / 128)) = static_cast<int32_t>(s_e % e_per_rank);
  }
  // the last CTA to finish writes the region headers; every thread fences its own row
  // stores before the CTA takes its ticket
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int64_t i = threadIdx.x; i < ranks * e_per_rank; i += blockDim.x) {
    const int64_t d = i / e_per_rank, e = i - d * e_per_rank;
    reinterpret_cast<int32_t*>(row_ptr(d * (cap + 1)))[e] = __ldcg(&cnt[i]);
  }
}

// Every CTA first derives, in shared memory, each source's row count and the 128-aligned
// offsets of the local experts' groups (exclusive scan of the per-expert totals over all
// sources, read from the region headers); then one warp per slot places valid rows as
// ep_permute_kernel does.
__global__ void __launch_bounds__(256) ep_permute_fixed_kernel(const uint8_t* rows, int64_t ranks, int64_t cap,
                                                               int64_t H, int64_t E_local, int32_t* fill, uint8_t* A,
                                                               float* SA, int32_t* m_indices, int32_t* perm_pos) {
  __shared__ int64_t s_off[kFixedMaxExperts];
  __shared__ int32_t s_nsrc[kFixedMaxRanks];
  __shared__ int64_t s_warp_sum[8];
  const int tid = threadIdx.x;
  const int64_t rb = packed_row_bytes(H);
  auto header = [&](int64_t r) { return reinterpret_cast<const int32_t*>(rows + r * (cap + 1) * rb); };
  // per-expert aligned totals, 4 consecutive experts per thread, then a block scan
  int64_t part[4];
  int64_t run = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t e = tid * 4 + i;
    int64_t tot = 0;
    if (e < E_local)
      for (int64_t r = 0; r < ranks; ++r) tot += header(r)[e];
    part[i] = (tot + 127) / 128 * 128;
    run += part[i];
  }
  const int lane = tid & 31, warp = tid >> 5;
  int64_t incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp_sum[warp] = incl;
  for (int64_t r = tid; r < ranks; r += blockDim.x) {
    int32_t n = 0;
    for (int64_t e = 0; e < E_local; ++e) n += header(r)[e];
    s_nsrc[r] = n;
  }
  __syncthreads();
  int64_t base = 0;
  for (int w = 0; w < warp; ++w) base += s_warp_sum[w];
  int64_t off = base + incl - run;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t e = tid * 4 + i;
    if (e < E_local) s_off[e] = off;
    off += part[i];
  }
  __syncthreads();
  const int64_t R = ranks * (cap + 1);
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + tid) >> 5; w < R;
       w += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int64_t src = w / (cap + 1), slot = w - src * (cap + 1) - 1;
    if (slot < 0 || slot >= s_nsrc[src]) {
      if (lane == 0) perm_pos[w] = -1;
      continue;
    }
    const uint8_t* in = rows + w * rb;
    const int e = *reinterpret_cast<const int32_t*>(in + H + 4 * (H / 128));
    int slot_e = 0;
    if (lane == 0) slot_e = atomicAdd(&fill[e], 1);
    const int64_t pos = s_off[e] + __shfl_sync(0xffffffffu, slot_e, 0);
    const uint4* src4 = reinterpret_cast<const uint4*>(in);
    uint4* dst = reinterpret_cast<uint4*>(A + pos * H);
    for (int64_t c = lane; c < H / 16; c += 32) dst[c] = src4[c];
    const float* rs = reinterpret_cast<const float*>(in + H);
    for (int64_t c = lane; c < H / 128; c += 32) SA[pos * (H / 128) + c] = rs[c];
    if (lane == 0) {
      m_indices[pos] = e;
      perm_pos[w] = static_cast<int32_t>(pos);
    }
  }
}

// ---------------------------------------------------------------- peer-memory exchange
// Peer dispatch.  Warp w of CTA c takes token t = c * kP2pWarps + w; lane j holds the token's
// slot j.  The slots are grouped by destination rank (__match_any_sync): the token sends one
// row to each rank that owns any of its experts.  The CTA counts its rows per destination in
// shared memory and claims them from the global counter with one atomic per destination.  The
// warp quantises the token's row once into shared memory, then stores it with 16-byte stores
// into each destination's region of this rank (over NVLink for the other GPUs), followed by
// the token index and, per slot, its local expert (or -1 when the slot goes elsewhere).
// send_index[t * topk + j] is the slot itself (where the combine finds its returned row), or
// -1 for a slot whose expert lies outside [0, E).  Per-destination, per-local-expert slot
// counts go to `scratch`; the last CTA writes each destination's header (those counts and
// the number of rows) and raises this rank's flag there.
// scratch (zeroed by the host): [ranks] rows per destination, [ranks * E_local] counts, [1] ticket.
__global__ void __launch_bounds__(kP2pWarps * 32) ep_dispatch_p2p_kernel(const void* x, int x_dtype, int64_t x_stride,
                                                                        const void* ids, int ids_dtype, int64_t T,
                                                                        int64_t E, int64_t e_per_rank,
                                                                        int32_t* scratch, int32_t* send_index, int pow2,
                                                                        PeerStep ps) {
  extern __shared__ __align__(16) uint8_t p2p_stage[];
  __shared__ int s_cnt[kFixedMaxRanks];
  __shared__ int s_base[kFixedMaxRanks];
  __shared__ int s_last;
  const int64_t ranks = ps.win.ranks, topk = ps.win.topk, H = ps.win.H, rb = ps.win.rb;
  const int32_t epoch = ps.epoch();
  int32_t* fill = scratch;
  int32_t* cnt = scratch + ranks;
  int32_t* ticket = cnt + ranks * e_per_rank;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kP2pWarps + warp;
  const bool live = t < T;
  for (int i = threadIdx.x; i < ranks; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  int64_t e = -1;
  int dest = -1;
  if (live && lane < topk) {
    const int64_t v = load_idx(ids, ids_dtype, t * topk + lane);
    if (v >= 0 && v < E) {
      e = v;
      dest = static_cast<int>(v / e_per_rank);
    }
    send_index[t * topk + lane] = dest >= 0 ? static_cast<int32_t>(t * topk + lane) : -1;
  }
  const unsigned same = __match_any_sync(0xffffffffu, dest);  // lanes sending to the same rank
  const bool lead = dest >= 0 && lane == __ffs(same) - 1;
  int local = 0;
  if (lead) local = atomicAdd(&s_cnt[dest], 1);
  if (dest >= 0) atomicAdd(&cnt[dest * e_per_rank + e % e_per_rank], 1);
  __syncthreads();
  for (int i = threadIdx.x; i < ranks; i += blockDim.x) s_base[i] = s_cnt[i] ? atomicAdd(&fill[i], s_cnt[i]) : 0;
  uint8_t* stage = p2p_stage + warp * row_stage_bytes(H);
  if (live) warp_quant_row(x, x_dtype, t * x_stride, H, stage, reinterpret_cast<float*>(stage + H), lane, pow2);
  __syncthreads();  // s_base complete; the warp's stage written
  const int64_t region = ps.win.region(epoch & 1, ps.me);
  for (unsigned leaders = __ballot_sync(0xffffffffu, lead); leaders; leaders &= leaders - 1) {
    const int l = __ffs(leaders) - 1;
    const int d = __shfl_sync(0xffffffffu, dest, l);
    const int64_t r = s_base[d] + __shfl_sync(0xffffffffu, local, l);
    uint8_t* out = reinterpret_cast<uint8_t*>(ps.peers[d]) + region + (1 + r) * rb;
    for (int64_t c = lane; c < H / 16; c += 32)
      reinterpret_cast<uint4*>(out)[c] = reinterpret_cast<const uint4*>(stage)[c];
    for (int64_t c = lane; c < H / 128; c += 32)
      reinterpret_cast<float*>(out + H)[c] = reinterpret_cast<const float*>(stage + H)[c];
    int32_t* tail = reinterpret_cast<int32_t*>(out + H + 4 * (H / 128));
    if (lane == 0) tail[0] = static_cast<int32_t>(t);
    if (lane < topk) tail[1 + lane] = dest == d ? static_cast<int32_t>(e % e_per_rank) : -1;
  }
  // the last CTA writes the headers and raises the flags; every thread fences its own peer
  // stores before the CTA takes its ticket
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int64_t i = threadIdx.x; i < ranks * (e_per_rank + 1); i += blockDim.x) {
    const int64_t d = i / (e_per_rank + 1), k = i - d * (e_per_rank + 1);
    int32_t* hdr = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ps.peers[d]) + region);
    hdr[k] = k < e_per_rank ? __ldcg(&cnt[d * e_per_rank + k]) : __ldcg(&fill[d]);
  }
  __threadfence_system();
  __syncthreads();
  for (int64_t d = threadIdx.x; d < ranks; d += blockDim.x)
    st_release_sys(reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ps.peers[d]) + Window::kDispatchFlags) + ps.me,
                   epoch);
}

// Peer permute.  Waits (bounded) until every source raised its flag for the step, derives the
// local experts' 128-aligned group offsets from the region headers (exclusive scan of the
// per-expert totals over all sources), then one warp per received row (region src, row r
// below the header's row count) reads the row once and writes it into the group of each of
// its slots' local experts: A, SA, m_indices, and ret_slot[pos] = src * cap + t * topk + j
// (cap = tokens * topk), the place in the source's window where the return step sends GEMM
// row pos.  With ret_rows (and ps.peers) set, ret_rows[pos] also gets that place's address
// (the source's window, return rows of the step's parity, slot t * topk + j): the row table of
// an FC2 GEMM that stores its rows straight into the sources' windows (cdg_gemm_args.d_rows).
// A wait that gives up places nothing (m_indices and ret_slot keep the -1, ret_rows the 0 the
// host wrote).  fill: [E_local] counters, zeroed by the host.
// Planes form (planes != nullptr; A and SA unused): each placed row is written as the GEMM's two
// e4m3 planes (plane stride M_pad * H) with row_exp[pos] = E (cdg_split.cuh).
__global__ void __launch_bounds__(256) ep_permute_p2p_kernel(int64_t E_local, int32_t* fill, uint8_t* A, float* SA,
                                                             int32_t* m_indices, int32_t* ret_slot, uint64_t* ret_rows,
                                                             PeerStep ps, uint8_t* planes = nullptr,
                                                             int32_t* row_exp = nullptr, int64_t M_pad = 0) {
  constexpr int kMaxTopk = 32;
  __shared__ int64_t s_off[kFixedMaxExperts];
  __shared__ int32_t s_tot[kFixedMaxExperts];
  __shared__ int32_t s_nrows[kFixedMaxRanks];
  __shared__ int64_t s_warp_sum[8];
  __shared__ int64_t s_pos[8][kMaxTopk];
  const int64_t ranks = ps.win.ranks, tokens = ps.win.tokens, topk = ps.win.topk, H = ps.win.H, rb = ps.win.rb;
  const int64_t cap = tokens * topk;
  const int32_t epoch = ps.epoch();
  const int64_t ret_off = ps.win.ret_parity(epoch & 1);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (!wait_peer_flags(reinterpret_cast<const int32_t*>(ps.own + Window::kDispatchFlags), static_cast<int>(ranks),
                       epoch, reinterpret_cast<int32_t*>(ps.own + Window::kStatus), 8))
    return;
  auto header = [&](int64_t src) {
    return reinterpret_cast<const int32_t*>(ps.own + ps.win.region(epoch & 1, src));
  };
  int64_t part[4];
  int64_t run = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t e = tid * 4 + i;
    int64_t tot = 0;
    if (e < E_local) {
      for (int64_t r = 0; r < ranks; ++r) tot += header(r)[e];
      s_tot[e] = static_cast<int32_t>(tot);
    }
    part[i] = (tot + 127) / 128 * 128;
    run += part[i];
  }
  int64_t incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp_sum[warp] = incl;
  for (int64_t r = tid; r < ranks; r += blockDim.x) s_nrows[r] = header(r)[E_local];
  __syncthreads();
  int64_t base = 0;
  for (int w = 0; w < warp; ++w) base += s_warp_sum[w];
  int64_t off = base + incl - run;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t e = tid * 4 + i;
    if (e < E_local) s_off[e] = off;
    off += part[i];
  }
  __syncthreads();
  const int64_t R = ranks * tokens;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + tid) >> 5; w < R;
       w += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int64_t src = w / tokens, r = w - src * tokens;
    if (r >= s_nrows[src]) continue;  // warp-uniform
    const uint8_t* in = ps.own + ps.win.region(epoch & 1, src) + (1 + r) * rb;
    const int32_t* tail = reinterpret_cast<const int32_t*>(in + H + 4 * (H / 128));
    int64_t pos = -1;
    if (lane < topk) {
      const int32_t el = tail[1 + lane];
      const int32_t t = tail[0];
      if (el >= 0 && el < E_local) {
        const int32_t k = atomicAdd(&fill[el], 1);
        if (k < s_tot[el] && t >= 0 && t < tokens) {  // inside the expert's group as the headers sized it
          pos = s_off[el] + k;
          m_indices[pos] = el;
          const int64_t slot = static_cast<int64_t>(t) * topk + lane;
          ret_slot[pos] = static_cast<int32_t>(src * cap + slot);
          if (ret_rows) {  // a missing window (address 0) leaves the row unreturned rather than misdirected
            const uint64_t base = ps.peers[src];
            ret_rows[pos] = base ? base + ret_off + slot * H * 2 : 0;
          }
        } else {
          atomicOr(reinterpret_cast<int32_t*>(ps.own + Window::kStatus), 2);
          atomicOr(&g_ep_sticky_status[0], 2);
          atomicCAS(&g_ep_sticky_status[1], 0, peer_wait_code(10, static_cast<int>(src)));
        }
      }
      s_pos[warp][lane] = pos;
    }
    __syncwarp();
    if (planes) {
      const float* rs = reinterpret_cast<const float*>(in + H);
      const int e = warp_plane_exponent(rs, H / 128, lane);
      const float inv = ldexpf(1.0f, -e);
      const int64_t plane = M_pad * H;
      for (int64_t c = lane; c < H / 16; c += 32) {
        uint4 hi, lo;
        split_planes16(reinterpret_cast<const uint4*>(in)[c], bf16_round(rs[c >> 3]), inv, hi, lo);
        for (int j = 0; j < topk; ++j) {
          const int64_t p = s_pos[warp][j];
          if (p < 0) continue;
          reinterpret_cast<uint4*>(planes + p * H)[c] = hi;
          reinterpret_cast<uint4*>(planes + plane + p * H)[c] = lo;
        }
      }
      if (lane < topk && s_pos[warp][lane] >= 0) row_exp[s_pos[warp][lane]] = e;
      __syncwarp();
      continue;
    }
    for (int64_t c = lane; c < H / 16; c += 32) {
      const uint4 v = reinterpret_cast<const uint4*>(in)[c];
      for (int j = 0; j < topk; ++j) {
        const int64_t p = s_pos[warp][j];
        if (p >= 0) reinterpret_cast<uint4*>(A + p * H)[c] = v;
      }
    }
    for (int64_t c = lane; c < H / 128; c += 32) {
      const float v = reinterpret_cast<const float*>(in + H)[c];
      for (int j = 0; j < topk; ++j) {
        const int64_t p = s_pos[warp][j];
        if (p >= 0) SA[p * (H / 128) + c] = v;
      }
    }
    __syncwarp();
  }
}

// Peer return: one warp per GEMM row pos < rows whose ret_slot is set; the row goes straight to
// its source's window (return rows of the step's parity) at the source's slot index.  Entries
// that decode to a rank or slot outside the window are skipped.  The last CTA raises this
// rank's flag in every source window.  scratch: [1] ticket, zeroed by the host.
__global__ void __launch_bounds__(256) ep_return_p2p_kernel(const __nv_bfloat16* Y, int64_t y_stride, int64_t rows,
                                                            const int32_t* ret_slot, PeerStep ps, int32_t* scratch) {
  __shared__ int s_last;
  const int64_t ranks = ps.win.ranks, H = ps.win.H, cap = ps.win.tokens * ps.win.topk;
  const int32_t epoch = ps.epoch();
  const int64_t ret_off = ps.win.ret_parity(epoch & 1);
  const int lane = threadIdx.x & 31;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < rows;
       w += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int32_t rs = ret_slot[w];
    if (rs < 0) continue;
    const int64_t src = rs / cap, idx = rs - src * cap;
    if (src >= ranks) continue;
    const uint4* from = reinterpret_cast<const uint4*>(Y + w * y_stride);
    uint4* to = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(ps.peers[src]) + ret_off +
                                         idx * H * static_cast<int64_t>(sizeof(__nv_bfloat16)));
    for (int64_t c = lane; c < H / 8; c += 32) to[c] = from[c];
  }
  __threadfence_system();  // each thread's peer stores before the CTA takes its ticket
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(scratch, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  for (int64_t r = threadIdx.x; r < ranks; r += blockDim.x)
    st_release_sys(reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ps.peers[r]) + Window::kReturnFlags) + ps.me,
                   epoch);
}

// One warp per row: out[i, :] = Y[perm_pos[i], :]; rows with perm_pos -1 are left as they are.
__global__ void ep_unpermute_kernel(const __nv_bfloat16* Y, int64_t y_stride, const int32_t* perm_pos, int64_t R,
                                    int64_t H, __nv_bfloat16* out) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= R || perm_pos[w] < 0) return;
  const uint4* src = reinterpret_cast<const uint4*>(Y + static_cast<int64_t>(perm_pos[w]) * y_stride);
  uint4* dst = reinterpret_cast<uint4*>(out + w * H);
  for (int64_t c = lane; c < H / 8; c += 32) dst[c] = src[c];
}

// One CTA per token; y[t, :] = bf16(sum_j w[t, j] * rows[row(send_index[t*k + j]), :]) in FP32,
// slots in order (an fmaf per slot), where row(i) = perm_pos[i] when perm_pos is given (the
// rows are then read where the grouped GEMM left them, fusing the unpermute) and i otherwise;
// slots whose index or row is -1 add nothing.  VEC: each thread reads and writes 8 columns
// at a time (16-byte accesses; H a multiple of 8, rows and y 16-byte aligned).
// Peer variant (ps.own != nullptr; `rows` unused): the returned rows are the own window's
// return rows for the step's parity, indexed by slot; first waits until every rank returned
// its rows (a wait that gives up writes the token's output as zeros); the last CTA then
// advances the window's step counter (scratch: [2] tickets, zeroed by the host).  With
// ps.peers set, the first CTA to run first raises this rank's return flag in every rank's
// window: the rows this rank owes were stored into the windows by the FC2 GEMM before this
// kernel (its epilogue stores through a row table, ending with a system-scope fence).
constexpr int kCombineMaxTopk = 32;

template <bool VEC>
__global__ void ep_combine_kernel(const __nv_bfloat16* rows, int64_t row_stride, const int32_t* perm_pos,
                                  const int32_t* send_index, const float* topk_w, int64_t T, int64_t topk, int64_t H,
                                  __nv_bfloat16* y, PeerStep ps = PeerStep{}, int32_t* scratch = nullptr) {
  int32_t epoch = 0;
  bool ok = true;
  if (ps.own) {
    epoch = ps.epoch();
    rows = reinterpret_cast<const __nv_bfloat16*>(ps.own + ps.win.ret_parity(epoch & 1));
    if (ps.peers && threadIdx.x == 0 && atomicAdd(scratch + 1, 1) == 0) {
      // a ticket rather than blockIdx 0: the CTA that raises is one that runs, whichever order
      // the CTAs start in (the others wait for these flags too)
      __threadfence_system();
      for (int64_t r = 0; r < ps.win.ranks; ++r)
        st_release_sys(
            reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ps.peers[r]) + Window::kReturnFlags) + ps.me, epoch);
    }
    ok = wait_peer_flags(reinterpret_cast<const int32_t*>(ps.own + Window::kReturnFlags),
                         static_cast<int>(ps.win.ranks), epoch, reinterpret_cast<int32_t*>(ps.own + Window::kStatus), 9);
    if (!ok && blockIdx.x < T) {
      // some rank's rows did not come back: the token's output is written as zeros (the
      // window's status word and cdg_device_status() report the timeout)
      for (int64_t c = threadIdx.x; c < H; c += blockDim.x) y[blockIdx.x * H + c] = __float2bfloat16_rn(0.0f);
    }
  }
  __shared__ int64_t s_row[kCombineMaxTopk];
  __shared__ float s_w[kCombineMaxTopk];
  const int64_t t = blockIdx.x;
  if (ok && t < T) {
    if (threadIdx.x < topk) {
      const int32_t i = send_index[t * topk + threadIdx.x];
      const int32_t r = (i >= 0 && perm_pos) ? perm_pos[i] : i;
      s_row[threadIdx.x] = r;
      s_w[threadIdx.x] = topk_w[t * topk + threadIdx.x];
    }
    __syncthreads();
    if (VEC) {
      for (int64_t c8 = threadIdx.x; c8 < H / 8; c8 += blockDim.x) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        // slots in batches of eight: the batch's loads are all issued before the first is used
        for (int64_t j0 = 0; j0 < topk; j0 += 8) {
          uint4 v[8];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int64_t r = j0 + jj < topk ? s_row[j0 + jj] : -1;
            // L2 loads: in the peer variant the rows were written by other GPUs while this kernel waited
            v[jj] = r >= 0 ? __ldcg(reinterpret_cast<const uint4*>(rows + r * row_stride + c8 * 8)) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            if (j0 + jj >= topk || s_row[j0 + jj] < 0) continue;
            const float wj = s_w[j0 + jj];
            const uint32_t vw[4] = {v[jj].x, v[jj].y, v[jj].z, v[jj].w};
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) {
              const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vw[q2]));
              acc[2 * q2] = fmaf(wj, f.x, acc[2 * q2]);
              acc[2 * q2 + 1] = fmaf(wj, f.y, acc[2 * q2 + 1]);
            }
          }
        }
        uint32_t o[4];
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * q2], acc[2 * q2 + 1]);
          o[q2] = *reinterpret_cast<uint32_t*>(&b);
        }
        *reinterpret_cast<uint4*>(y + t * H + c8 * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    } else {
      for (int64_t c = threadIdx.x; c < H; c += blockDim.x) {
        float acc = 0.0f;
        for (int64_t j = 0; j < topk; ++j) {
          const int64_t r = s_row[j];
          if (r >= 0) acc = fmaf(s_w[j], __bfloat162float(rows[r * row_stride + c]), acc);
        }
        y[t * H + c] = __float2bfloat16_rn(acc);
      }
    }
  }
  if (!ps.own) return;
  // every CTA read its rows (and every rank finished the step); the last advances the counter
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(scratch, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) *reinterpret_cast<volatile int32_t*>(ps.own + Window::kEpoch) = epoch;
}

// Weight-row gathers of transform_weights_for_mega_moe: destination row n of a group
// takes source row src_row(n).  kind bit 0: gate/up interleave in granules of 8 rows
// (rows [q*16, q*16+8) from the gate half, [q*16+8, q*16+16) from the up half);
// bit 1: within every 128 rows, the [4 x 32] -> [32 x 4] transpose of scale rows that
// tcgen05.cp's 32x128b.warpx4 pattern expects (applied after the interleave).
__host__ __device__ __forceinline__ int64_t mega_src_row(int64_t n, int64_t N, int kind) {
  if (kind & 2) {
    const int64_t blk = n / 128, r = n - blk * 128;
    n = blk * 128 + (r % 4) * 32 + r / 4;
  }
  if (kind & 1) {
    const int64_t half = N / 2, q = n / 16, rem = n - q * 16;
    n = (rem / 8) * half + q * 8 + rem % 8;
  }
  return n;
}

// One warp per (group, destination row); 16-byte copies when rows allow them.
__global__ void mega_rows_kernel(const uint8_t* src, uint8_t* dst, int64_t G, int64_t N, int64_t row_bytes,
                                 int64_t stride_g, int64_t stride_n, int kind) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= G * N) return;
  const int64_t g = w / N, n = w - g * N;
  const uint8_t* from = src + g * stride_g + mega_src_row(n, N, kind) * stride_n;
  uint8_t* to = dst + (g * N + n) * row_bytes;
  if (row_bytes % 16 == 0 && reinterpret_cast<uintptr_t>(from) % 16 == 0 && reinterpret_cast<uintptr_t>(to) % 16 == 0) {
    for (int64_t c = lane; c < row_bytes / 16; c += 32)
      reinterpret_cast<uint4*>(to)[c] = reinterpret_cast<const uint4*>(from)[c];
  } else {
    for (int64_t c = lane; c < row_bytes; c += 32) to[c] = from[c];
  }
}

unsigned warp_grid(int64_t warps) { return static_cast<unsigned>((warps * 32 + 255) / 256); }

// SM count of the current device (looked up at each call: a cheap attribute query).
int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return n > 0 ? n : 148;
}



int launched() { return cudaGetLastError() == cudaSuccess ? CDG_OK : CDG_ERR_CUDA; }

}  // namespace
}  // namespace cdg

extern "C" {

int cdg_quant_fp8_rows(const void* x, int32_t x_dtype, int64_t x_stride, int64_t M, int64_t K, uint8_t* q,
                       int64_t q_stride, float* s, int64_t s_stride_m, int64_t s_stride_k, int32_t scale_fmt,
                       cdg_stream_t stream) {
  if (M < 0 || K <= 0 || K % 128 || (M > 0 && (!x || !q || !s))) return CDG_ERR_INVALID_ARGUMENT;
  if (scale_fmt != CDG_SCALE_FP32 && scale_fmt != CDG_SCALE_POW2) return CDG_ERR_INVALID_ARGUMENT;
  if (x_dtype != CDG_DTYPE_BF16 && x_dtype != CDG_DTYPE_F32) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(q) % 4 || q_stride % 4) return CDG_ERR_ALIGNMENT;
  if (M == 0) return CDG_OK;
  cdg::quant_rows_kernel<<<cdg::warp_grid(M * (K / 128)), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, x_dtype, x_stride, M, K, q, q_stride, s, s_stride_m, s_stride_k, scale_fmt);
  return cdg::launched();
}

int cdg_silu_mul_quant_fp8(const void* in, int64_t in_stride, int64_t M, int64_t I, const int32_t* m_indices,
                           uint8_t* q, int64_t q_stride, float* s, int64_t s_stride_m, int64_t s_stride_k,
                           int32_t scale_fmt, cdg_stream_t stream) {
  if (M < 0 || I <= 0 || I % 128 || (M > 0 && (!in || !q || !s))) return CDG_ERR_INVALID_ARGUMENT;
  if (scale_fmt != CDG_SCALE_FP32 && scale_fmt != CDG_SCALE_POW2) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(q) % 4 || q_stride % 4) return CDG_ERR_ALIGNMENT;
  if (M == 0) return CDG_OK;
  const bool vec = reinterpret_cast<uintptr_t>(in) % 8 == 0 && in_stride % 4 == 0;
  const bool wide = reinterpret_cast<uintptr_t>(in) % 16 == 0 && in_stride % 8 == 0 &&
                    reinterpret_cast<uintptr_t>(q) % 16 == 0 && q_stride % 16 == 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const __nv_bfloat16* h = static_cast<const __nv_bfloat16*>(in);
  if (wide) {
    const int64_t warps = M * ((I / 128 + 3) / 4);
    const unsigned grid =
        static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, int64_t(cdg::sm_count()) * 16)));
    auto kernel = I == 2048 ? cdg::silu_mul_quant_16b_kernel<16>
                  : I == 1024 ? cdg::silu_mul_quant_16b_kernel<8>
                              : cdg::silu_mul_quant_16b_kernel<0>;
    kernel<<<grid, 256, 0, st>>>(h, in_stride, M, I, m_indices, q, q_stride, s, s_stride_m, s_stride_k, scale_fmt);
  } else if (vec) {
    const int64_t chunks = (I / 128 + cdg::kSiluBlocks - 1) / cdg::kSiluBlocks;
    cdg::silu_mul_quant_vec_kernel<<<cdg::warp_grid(M * chunks), 256, 0, st>>>(
        h, in_stride, M, I, m_indices, q, q_stride, s, s_stride_m, s_stride_k, scale_fmt);
  } else {
    cdg::silu_mul_quant_kernel<<<cdg::warp_grid(M * (I / 128)), 256, 0, st>>>(
        h, in_stride, M, I, m_indices, q, q_stride, s, s_stride_m, s_stride_k, scale_fmt);
  }
  return cdg::launched();
}

int cdg_ep_count(const void* topk_ids, int32_t ids_dtype, int64_t n, int64_t E, int32_t* counts, cdg_stream_t stream) {
  if (n < 0 || E <= 0 || !counts || (n > 0 && !topk_ids)) return CDG_ERR_INVALID_ARGUMENT;
  if (ids_dtype != CDG_DTYPE_I32 && ids_dtype != CDG_DTYPE_I64) return CDG_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(counts, 0, E * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (n == 0) return CDG_OK;
  // a few CTAs per SM, each over many slots (its histogram is flushed once)
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n + 2047) / 2048, int64_t(cdg::sm_count()) * 2));
  cdg::ep_count_kernel<<<blocks, 256, 0, st>>>(topk_ids, ids_dtype, n, E, counts);
  return cdg::launched();
}

int cdg_ep_count_offsets(const void* topk_ids, int32_t ids_dtype, int64_t n, int64_t E, int32_t* counts,
                         int64_t* expert_off, int32_t* scratch, cdg_stream_t stream) {
  if (n < 0 || E <= 0 || !counts || !expert_off || !scratch || (n > 0 && !topk_ids)) return CDG_ERR_INVALID_ARGUMENT;
  if (ids_dtype != CDG_DTYPE_I32 && ids_dtype != CDG_DTYPE_I64) return CDG_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(counts, 0, E * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemsetAsync(scratch, 0, sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  const unsigned blocks =
      static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((n + 2047) / 2048, int64_t(cdg::sm_count()) * 2)));
  cdg::ep_count_kernel<<<blocks, 256, 0, st>>>(topk_ids, ids_dtype, n, E, counts, expert_off, scratch);
  return cdg::launched();
}

int64_t cdg_ep_row_bytes(int64_t H) { return H > 0 && H % 128 == 0 ? cdg::packed_row_bytes(H) : 0; }

int cdg_ep_pack(const uint8_t* xq, int64_t xq_stride, const float* xs, int64_t xs_stride, const void* topk_ids,
                int32_t ids_dtype, int64_t T, int64_t topk, int64_t E, int64_t ranks, int64_t H,
                const int64_t* send_off, int32_t* fill, uint8_t* out_rows, int32_t* send_index, cdg_stream_t stream) {
  if (T < 0 || topk <= 0 || E <= 0 || ranks <= 0 || E % ranks || H <= 0 || H % 128) return CDG_ERR_INVALID_ARGUMENT;
  if (ids_dtype != CDG_DTYPE_I32 && ids_dtype != CDG_DTYPE_I64) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(xq) % 16 || xq_stride % 16 || reinterpret_cast<uintptr_t>(out_rows) % 16)
    return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fill, 0, ranks * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (T == 0) return CDG_OK;
  cdg::ep_pack_kernel<<<cdg::warp_grid(T * topk), 256, 0, st>>>(xq, xq_stride, xs, xs_stride, topk_ids, ids_dtype, T,
                                                                topk, E, E / ranks, H, send_off, fill, out_rows,
                                                                send_index);
  return cdg::launched();
}

int cdg_ep_permute(const uint8_t* recv_rows, int64_t R, int64_t H, int64_t E_local, const int64_t* expert_off,
                   int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices, int64_t M_pad, int32_t* perm_pos,
                   cdg_stream_t stream) {
  if (R < 0 || H <= 0 || H % 128 || E_local <= 0 || M_pad < 0) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(recv_rows) % 16 || reinterpret_cast<uintptr_t>(A) % 16) return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fill, 0, E_local * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemsetAsync(m_indices, 0xFF, M_pad * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (R == 0) return CDG_OK;
  cdg::ep_permute_kernel<<<cdg::warp_grid(R), 256, 0, st>>>(recv_rows, R, H, expert_off, fill, A, SA, m_indices,
                                                            perm_pos);
  return cdg::launched();
}

int64_t cdg_ep_fixed_scratch_ints(int64_t ranks, int64_t E) {
  return ranks > 0 && E > 0 && E % ranks == 0 ? ranks + E + 1 : 0;
}

int cdg_ep_quant_pack_fixed(const void* x, int32_t x_dtype, int64_t x_stride, const void* topk_ids, int32_t ids_dtype,
                            int64_t T, int64_t topk, int64_t E, int64_t ranks, int64_t H, int64_t cap, int32_t* scratch,
                            uint8_t* out_rows, int32_t* send_index, int32_t scale_fmt, cdg_stream_t stream) {
  if (T < 0 || topk <= 0 || E <= 0 || ranks <= 0 || ranks > cdg::kFixedMaxRanks || E % ranks || H <= 0 || H % 128 ||
      cap < 0 || E / ranks > cdg::kFixedMaxExperts || !scratch || !out_rows)
    return CDG_ERR_INVALID_ARGUMENT;
  if (scale_fmt != CDG_SCALE_FP32 && scale_fmt != CDG_SCALE_POW2) return CDG_ERR_INVALID_ARGUMENT;
  if (4 * (E / ranks) > cdg::packed_row_bytes(H)) return CDG_ERR_INVALID_ARGUMENT;  // header fits a row
  if (x_dtype != CDG_DTYPE_BF16 && x_dtype != CDG_DTYPE_F32) return CDG_ERR_INVALID_ARGUMENT;
  if (ids_dtype != CDG_DTYPE_I32 && ids_dtype != CDG_DTYPE_I64) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(out_rows) % 16) return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, cdg_ep_fixed_scratch_ints(ranks, E) * sizeof(int32_t), st) != cudaSuccess)
    return CDG_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(x) % 16 || x_stride % 4) return CDG_ERR_ALIGNMENT;  // vector loads of 4 values
  const unsigned grid = T * topk > 0 ? static_cast<unsigned>(T * topk) : 1u;
  cdg::ep_quant_pack_fixed_kernel<<<grid, 128, 0, st>>>(x, x_dtype, x_stride, topk_ids, ids_dtype, T, topk, E, E / ranks,
                                                        ranks, H, cap, scratch, out_rows, send_index, scale_fmt);
  return cdg::launched();
}

int cdg_ep_permute_fixed(const uint8_t* recv_rows, int64_t ranks, int64_t cap, int64_t H, int64_t E_local,
                         int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices, int64_t M_pad, int32_t* perm_pos,
                         cdg_stream_t stream) {
  if (ranks <= 0 || ranks > cdg::kFixedMaxRanks || cap < 0 || H <= 0 || H % 128 || E_local <= 0 ||
      E_local > cdg::kFixedMaxExperts || M_pad < ranks * cap + 127 * E_local)
    return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(recv_rows) % 16 || reinterpret_cast<uintptr_t>(A) % 16) return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fill, 0, E_local * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemsetAsync(m_indices, 0xFF, M_pad * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  const int64_t R = ranks * (cap + 1);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((R + 7) / 8, 1184));
  cdg::ep_permute_fixed_kernel<<<grid, 256, 0, st>>>(recv_rows, ranks, cap, H, E_local, fill, A, SA, m_indices,
                                                     perm_pos);
  return cdg::launched();
}

int cdg_ep_unpermute(const void* Y, int64_t y_stride, const int32_t* perm_pos, int64_t R, int64_t H, void* out,
                     cdg_stream_t stream) {
  if (R < 0 || H <= 0 || H % 8) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(Y) % 16 || y_stride % 8 || reinterpret_cast<uintptr_t>(out) % 16)
    return CDG_ERR_ALIGNMENT;
  if (R == 0) return CDG_OK;
  cdg::ep_unpermute_kernel<<<cdg::warp_grid(R), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(Y), y_stride, perm_pos, R, H, static_cast<__nv_bfloat16*>(out));
  return cdg::launched();
}

namespace cdg {
namespace {
int launch_combine(const void* rows, int64_t row_stride, const int32_t* perm_pos, const int32_t* send_index,
                   const float* topk_w, int64_t T, int64_t topk, int64_t H, void* y, cudaStream_t st) {
  if (T < 0 || topk <= 0 || topk > kCombineMaxTopk || H <= 0 || row_stride < H) return CDG_ERR_INVALID_ARGUMENT;
  if (T == 0) return CDG_OK;
  const bool vec = H % 8 == 0 && row_stride % 8 == 0 && reinterpret_cast<uintptr_t>(rows) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(y) % 16 == 0;
  auto kernel = vec ? ep_combine_kernel<true> : ep_combine_kernel<false>;
  kernel<<<static_cast<unsigned>(T), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(rows), row_stride, perm_pos,
                                                   send_index, topk_w, T, topk, H, static_cast<__nv_bfloat16*>(y),
                                                   PeerStep{}, nullptr);
  return launched();
}
}  // namespace
}  // namespace cdg

int cdg_ep_combine(const void* rows, const int32_t* send_index, const float* topk_w, int64_t T, int64_t topk,
                   int64_t H, void* y, cdg_stream_t stream) {
  return cdg::launch_combine(rows, H, nullptr, send_index, topk_w, T, topk, H, y,
                             reinterpret_cast<cudaStream_t>(stream));
}

int cdg_ep_quant_dispatch_local(const void* x, int32_t x_dtype, int64_t x_stride, const void* topk_ids,
                                int32_t ids_dtype, int64_t T, int64_t topk, int64_t E, int64_t H,
                                const int64_t* expert_off, int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices,
                                int64_t M_pad, int32_t* perm_pos, int32_t* send_index, int32_t scale_fmt,
                                cdg_stream_t stream) {
  if (T < 0 || topk <= 0 || topk > 32 || E <= 0 || H <= 0 || H % 128 || M_pad < 0 || !fill || !expert_off ||
      (T > 0 && (!x || !topk_ids || !A || !SA || !m_indices || !perm_pos || !send_index)))
    return CDG_ERR_INVALID_ARGUMENT;
  if (scale_fmt != CDG_SCALE_FP32 && scale_fmt != CDG_SCALE_POW2) return CDG_ERR_INVALID_ARGUMENT;
  if (x_dtype != CDG_DTYPE_BF16 && x_dtype != CDG_DTYPE_F32) return CDG_ERR_INVALID_ARGUMENT;
  if (ids_dtype != CDG_DTYPE_I32 && ids_dtype != CDG_DTYPE_I64) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(x) % 16 || x_stride % 4 || reinterpret_cast<uintptr_t>(A) % 16)
    return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fill, 0, E * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (M_pad > 0 && cudaMemsetAsync(m_indices, 0xFF, M_pad * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (T == 0) return CDG_OK;
  const size_t smem = static_cast<size_t>(cdg::kP2pWarps * cdg::row_stage_bytes(H));
  if (smem > 200 * 1024) return CDG_ERR_UNSUPPORTED;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(cdg::ep_quant_dispatch_local_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return CDG_ERR_CUDA;
  const unsigned grid = static_cast<unsigned>((T + cdg::kP2pWarps - 1) / cdg::kP2pWarps);
  cdg::ep_quant_dispatch_local_kernel<<<grid, cdg::kP2pWarps * 32, smem, st>>>(
      x, x_dtype, x_stride, topk_ids, ids_dtype, T, topk, E, H, expert_off, fill, A, SA, m_indices, perm_pos,
      send_index, scale_fmt);
  return cdg::launched();
}

int cdg_ep_quant_dispatch_local_planes(const void* x, int32_t x_dtype, int64_t x_stride, const void* topk_ids,
                                       int32_t ids_dtype, int64_t T, int64_t topk, int64_t E, int64_t H,
                                       const int64_t* expert_off, int32_t* fill, uint8_t* planes, int32_t* row_exp,
                                       int32_t* m_indices, int64_t M_pad, int32_t* perm_pos, int32_t* send_index,
                                       cdg_stream_t stream) {
  if (T < 0 || topk <= 0 || topk > 32 || E <= 0 || H <= 0 || H % 128 || M_pad < 0 || M_pad % 128 || !fill ||
      !expert_off || (T > 0 && (!x || !topk_ids || !planes || !row_exp || !m_indices || !perm_pos || !send_index)))
    return CDG_ERR_INVALID_ARGUMENT;
  if (x_dtype != CDG_DTYPE_BF16 && x_dtype != CDG_DTYPE_F32) return CDG_ERR_INVALID_ARGUMENT;
  if (ids_dtype != CDG_DTYPE_I32 && ids_dtype != CDG_DTYPE_I64) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(x) % 16 || x_stride % 4 || reinterpret_cast<uintptr_t>(planes) % 16)
    return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fill, 0, E * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (M_pad > 0 && cudaMemsetAsync(m_indices, 0xFF, M_pad * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (T == 0) return CDG_OK;
  const size_t smem = static_cast<size_t>(cdg::kP2pWarps * cdg::row_stage_bytes(H));
  if (smem > 200 * 1024) return CDG_ERR_UNSUPPORTED;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(cdg::ep_quant_dispatch_local_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return CDG_ERR_CUDA;
  const unsigned grid = static_cast<unsigned>((T + cdg::kP2pWarps - 1) / cdg::kP2pWarps);
  cdg::ep_quant_dispatch_local_kernel<<<grid, cdg::kP2pWarps * 32, smem, st>>>(
      x, x_dtype, x_stride, topk_ids, ids_dtype, T, topk, E, H, expert_off, fill, nullptr, nullptr, m_indices,
      perm_pos, send_index, CDG_SCALE_FP32, planes, row_exp, M_pad);
  return cdg::launched();
}

int cdg_silu_mul_quant_planes(const void* in, int64_t in_stride, int64_t M, int64_t I, const int32_t* m_indices,
                              uint8_t* planes, int32_t* row_exp, cdg_stream_t stream) {
  if (M < 0 || I <= 0 || I % 128 || (M > 0 && (!in || !planes || !row_exp))) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(in) % 16 || in_stride % 8 || reinterpret_cast<uintptr_t>(planes) % 16)
    return CDG_ERR_ALIGNMENT;
  if (M == 0) return CDG_OK;
  const size_t smem = 8 * static_cast<size_t>(cdg::row_stage_bytes(I));
  if (smem > 200 * 1024) return CDG_ERR_UNSUPPORTED;
  auto kernel = I == 2048 ? cdg::silu_mul_quant_planes_kernel<16>
                : I == 1024 ? cdg::silu_mul_quant_planes_kernel<8>
                            : cdg::silu_mul_quant_planes_kernel<0>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return CDG_ERR_CUDA;
  const unsigned grid =
      static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((M + 7) / 8, int64_t(cdg::sm_count()) * 8)));
  kernel<<<grid, 256, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(in), in_stride, M, I, m_indices, planes, row_exp);
  return cdg::launched();
}

int cdg_ep_unpermute_combine(const void* Y, int64_t y_stride, const int32_t* perm_pos, const int32_t* send_index,
                             const float* topk_w, int64_t T, int64_t topk, int64_t H, void* y, cdg_stream_t stream) {
  if (!perm_pos) return CDG_ERR_INVALID_ARGUMENT;
  return cdg::launch_combine(Y, y_stride, perm_pos, send_index, topk_w, T, topk, H, y,
                             reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------- peer-memory exchange
namespace cdg {
namespace {
// Shapes the peer exchange takes: ranks <= 128, topk <= 32, H a multiple of 128, every slot
// index of a window (ranks * tokens * topk) an int32, the header (E_local counts and the row
// count) inside one row.
bool p2p_shape_ok(int64_t ranks, int64_t tokens, int64_t topk, int64_t H) {
  return ranks > 0 && ranks <= 128 && tokens >= 0 && topk > 0 && topk <= 32 && H > 0 && H % 128 == 0 &&
         ranks * tokens * topk < (int64_t(1) << 31);
}

PeerStep make_step(const uint64_t* peers, void* window, int32_t me, int64_t ranks, int64_t tokens, int64_t topk,
                   int64_t H) {
  PeerStep ps;
  ps.peers = peers;
  ps.own = static_cast<uint8_t*>(window);
  ps.win = make_window(ranks, tokens, topk, H);
  ps.me = me;
  return ps;
}
}  // namespace
}  // namespace cdg

extern "C" {

size_t cdg_ep_window_bytes(int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H) {
  if (!cdg::p2p_shape_ok(ranks, max_tokens, topk, H)) return 0;
  return static_cast<size_t>(cdg::make_window(ranks, max_tokens, topk, H).bytes());
}

int cdg_ep_window_create(size_t bytes, void** window, void* ipc_handle) {
  if (!bytes || !window || !ipc_handle) return CDG_ERR_INVALID_ARGUMENT;
  *window = nullptr;
  if (cudaMalloc(window, bytes) != cudaSuccess) return CDG_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(*window, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, *window) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(*window);
    *window = nullptr;
    return CDG_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  return CDG_OK;
}

int cdg_ep_window_open(const void* ipc_handle, void** window) {
  if (!ipc_handle || !window) return CDG_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(window, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? CDG_OK : CDG_ERR_CUDA;
}

int cdg_ep_window_close(void* window, int32_t opened) {
  if (!window) return CDG_OK;
  return (opened ? cudaIpcCloseMemHandle(window) : cudaFree(window)) == cudaSuccess ? CDG_OK : CDG_ERR_CUDA;
}

int cdg_ep_window_status(const void* window, cdg_stream_t stream) {
  if (!window) return CDG_ERR_INVALID_ARGUMENT;
  int32_t word = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&word, static_cast<const uint8_t*>(window) + cdg::Window::kStatus, 4, cudaMemcpyDeviceToHost,
                      st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return CDG_ERR_CUDA;
  return (word & 1) ? CDG_ERR_DEVICE_TIMEOUT : word ? CDG_ERR_DEVICE_INDEX : CDG_OK;
}

int cdg_ep_dispatch_p2p(const void* x, int32_t x_dtype, int64_t x_stride, const void* topk_ids, int32_t ids_dtype,
                        int64_t T, int64_t topk, int64_t E, int64_t ranks, int64_t H, int64_t max_tokens,
                        const uint64_t* peers, void* window, int32_t me, int32_t* scratch, int32_t* send_index,
                        int32_t scale_fmt, cdg_stream_t stream) {
  if (!cdg::p2p_shape_ok(ranks, max_tokens, topk, H) || T < 0 || T > max_tokens || E <= 0 || E % ranks ||
      E / ranks > cdg::kFixedMaxExperts || !scratch || !peers || !window || me < 0 || me >= ranks ||
      (T > 0 && (!x || !topk_ids || !send_index)))
    return CDG_ERR_INVALID_ARGUMENT;
  if (scale_fmt != CDG_SCALE_FP32 && scale_fmt != CDG_SCALE_POW2) return CDG_ERR_INVALID_ARGUMENT;
  const cdg::Window win = cdg::make_window(ranks, max_tokens, topk, H);
  if (4 * (E / ranks + 1) > win.rb) return CDG_ERR_INVALID_ARGUMENT;  // the header fits a row
  if (x_dtype != CDG_DTYPE_BF16 && x_dtype != CDG_DTYPE_F32) return CDG_ERR_INVALID_ARGUMENT;
  if (ids_dtype != CDG_DTYPE_I32 && ids_dtype != CDG_DTYPE_I64) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(x) % 16 || x_stride % 4) return CDG_ERR_ALIGNMENT;
  const size_t smem = static_cast<size_t>(cdg::kP2pWarps * cdg::row_stage_bytes(H));
  if (smem > 200 * 1024) return CDG_ERR_UNSUPPORTED;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(cdg::ep_dispatch_p2p_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem)) != cudaSuccess)
    return CDG_ERR_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, cdg_ep_fixed_scratch_ints(ranks, E) * sizeof(int32_t), st) != cudaSuccess)
    return CDG_ERR_CUDA;
  const cdg::PeerStep ps = cdg::make_step(peers, window, me, ranks, max_tokens, topk, H);
  const unsigned grid = T > 0 ? static_cast<unsigned>((T + cdg::kP2pWarps - 1) / cdg::kP2pWarps) : 1u;
  cdg::ep_dispatch_p2p_kernel<<<grid, cdg::kP2pWarps * 32, smem, st>>>(x, x_dtype, x_stride, topk_ids, ids_dtype, T, E,
                                                                       E / ranks, scratch, send_index, scale_fmt, ps);
  return cdg::launched();
}

int cdg_ep_permute_p2p(void* window, int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H, int64_t E_local,
                       int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices, int64_t M_pad, int32_t* ret_slot,
                       const uint64_t* peers, uint64_t* ret_rows, cdg_stream_t stream) {
  if (!window || !cdg::p2p_shape_ok(ranks, max_tokens, topk, H) || E_local <= 0 ||
      E_local > cdg::kFixedMaxExperts || M_pad < ranks * max_tokens * topk + 127 * E_local || !fill || !A || !SA ||
      !m_indices || !ret_slot || (ret_rows && !peers))
    return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(A) % 16) return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fill, 0, E_local * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemsetAsync(m_indices, 0xFF, M_pad * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemsetAsync(ret_slot, 0xFF, M_pad * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (ret_rows && cudaMemsetAsync(ret_rows, 0, M_pad * sizeof(uint64_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  const cdg::PeerStep ps = cdg::make_step(peers, window, 0, ranks, max_tokens, topk, H);
  const int64_t R = ranks * max_tokens;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((R + 7) / 8, 1184)));
  cdg::ep_permute_p2p_kernel<<<grid, 256, 0, st>>>(E_local, fill, A, SA, m_indices, ret_slot, ret_rows, ps);
  return cdg::launched();
}

int cdg_ep_permute_p2p_planes(void* window, int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H,
                              int64_t E_local, int32_t* fill, uint8_t* planes, int32_t* row_exp, int32_t* m_indices,
                              int64_t M_pad, int32_t* ret_slot, const uint64_t* peers, uint64_t* ret_rows,
                              cdg_stream_t stream) {
  if (!window || !cdg::p2p_shape_ok(ranks, max_tokens, topk, H) || E_local <= 0 ||
      E_local > cdg::kFixedMaxExperts || M_pad < ranks * max_tokens * topk + 127 * E_local || M_pad % 128 || !fill ||
      !planes || !row_exp || !m_indices || !ret_slot || (ret_rows && !peers))
    return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(planes) % 16) return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fill, 0, E_local * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemsetAsync(m_indices, 0xFF, M_pad * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemsetAsync(ret_slot, 0xFF, M_pad * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (ret_rows && cudaMemsetAsync(ret_rows, 0, M_pad * sizeof(uint64_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  const cdg::PeerStep ps = cdg::make_step(peers, window, 0, ranks, max_tokens, topk, H);
  const int64_t R = ranks * max_tokens;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((R + 7) / 8, 1184)));
  cdg::ep_permute_p2p_kernel<<<grid, 256, 0, st>>>(E_local, fill, nullptr, nullptr, m_indices, ret_slot, ret_rows, ps,
                                                   planes, row_exp, M_pad);
  return cdg::launched();
}

int cdg_ep_return_p2p(const void* Y, int64_t y_stride, int64_t y_rows, const int32_t* ret_slot, int64_t M_pad,
                      int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H, const uint64_t* peers, void* window,
                      int32_t me, int32_t* scratch, cdg_stream_t stream) {
  if (!cdg::p2p_shape_ok(ranks, max_tokens, topk, H) || !peers || !window || !scratch || !ret_slot || me < 0 ||
      me >= ranks || y_rows < 0 || M_pad < 0 || y_stride < H || (y_rows > 0 && !Y))
    return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(Y) % 16 || y_stride % 8) return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  const cdg::PeerStep ps = cdg::make_step(peers, window, me, ranks, max_tokens, topk, H);
  const int64_t rows = std::min(M_pad, y_rows);
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, 1184)));
  cdg::ep_return_p2p_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(Y), y_stride, rows, ret_slot, ps,
                                                  scratch);
  return cdg::launched();
}

int cdg_ep_combine_p2p(void* window, const int32_t* send_index, const float* topk_w, int64_t T, int64_t topk,
                       int64_t H, int64_t ranks, int64_t max_tokens, const uint64_t* peers, int32_t me,
                       int32_t* scratch, void* y, cdg_stream_t stream) {
  if (!window || !scratch || !cdg::p2p_shape_ok(ranks, max_tokens, topk, H) || T < 0 || T > max_tokens ||
      topk > cdg::kCombineMaxTopk || (T > 0 && (!send_index || !topk_w || !y)) || (peers && (me < 0 || me >= ranks)))
    return CDG_ERR_INVALID_ARGUMENT;
  if (H % 8 || reinterpret_cast<uintptr_t>(y) % 16) return CDG_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, 2 * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  const cdg::PeerStep ps = cdg::make_step(peers, window, peers ? me : 0, ranks, max_tokens, topk, H);
  const unsigned grid = T > 0 ? static_cast<unsigned>(T) : 1u;
  cdg::ep_combine_kernel<true><<<grid, 256, 0, st>>>(nullptr, H, nullptr, send_index, topk_w, T, topk, H,
                                                     static_cast<__nv_bfloat16*>(y), ps, scratch);
  return cdg::launched();
}

int cdg_ep_set_wait_timeout_ns(uint64_t ns) {
  if (ns > 60ull * 1000000000ull) return CDG_ERR_INVALID_ARGUMENT;
  const uint64_t v = ns ? ns : cdg::kPeerWaitNs;
  return cudaMemcpyToSymbol(cdg::g_peer_wait_ns, &v, sizeof(v)) == cudaSuccess ? CDG_OK : CDG_ERR_CUDA;
}

}  // extern "C"

namespace cdg {
// The exchange kernels' half of cdg_device_status(): reads (after the device is idle) and
// optionally clears this unit's sticky record on the current device.
int ep_sticky_status(int clear, int32_t* out) {
  if (cudaDeviceSynchronize() != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemcpyFromSymbol(out, g_ep_sticky_status, 2 * sizeof(int32_t)) != cudaSuccess) return CDG_ERR_CUDA;
  if (clear) {
    const int32_t z[2] = {0, 0};
    if (cudaMemcpyToSymbol(g_ep_sticky_status, z, sizeof(z)) != cudaSuccess) return CDG_ERR_CUDA;
  }
  return CDG_OK;
}
}  // namespace cdg

extern "C" {

// ---------------------------------------------------------------- MegaMoE weight layout
int cdg_mega_moe_transform_rows(const void* src, int64_t stride_g, int64_t stride_n, void* dst, int64_t G, int64_t N,
                                int64_t row_bytes, int32_t kind, cdg_stream_t stream) {
  if (!src || !dst || G < 0 || N <= 0 || row_bytes <= 0 || kind < 0 || kind > 3 || stride_n < row_bytes ||
      stride_g < stride_n * N)
    return CDG_ERR_INVALID_ARGUMENT;
  if ((kind & 1) && (N % 16)) return CDG_ERR_INVALID_ARGUMENT;   // gate and up halves of whole granules
  if ((kind & 2) && (N % 128)) return CDG_ERR_INVALID_ARGUMENT;  // whole 128-row blocks
  if (G == 0) return CDG_OK;
  cdg::mega_rows_kernel<<<cdg::warp_grid(G * N), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), G, N, row_bytes, stride_g, stride_n, kind);
  return cdg::launched();
}

}  // extern "C"
