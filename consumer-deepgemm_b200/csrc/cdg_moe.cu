// Kernels around the grouped GEMM for a mixture-of-experts layer, and the
// bookkeeping of expert parallelism (experts sharded over ranks, token rows
// exchanged with all-to-all collectives issued by the host).
//
//   cdg_quant_fp8_rows        BF16/FP32 rows -> e4m3 + FP32 scale per 128 columns
//   cdg_silu_mul_quant_fp8    [gate | up] BF16 rows -> e4m3(silu(gate) * up) + scales
//   cdg_ep_count              routed rows per expert
//   cdg_ep_pack               routed rows -> send buffer grouped by destination rank
//   cdg_ep_permute            received rows -> 128-aligned contiguous layout per local expert
//   cdg_ep_unpermute          GEMM rows -> received order
//   cdg_ep_combine            returned rows -> weighted top-k sum per token
//
// Row order inside a destination or an expert group comes from atomics and is
// not deterministic; every row is computed independently and returned to its
// (token, slot) place, so results are.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "cdg_b200.h"

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

// Quantise one 128-wide block held by a warp (4 values per lane) to e4m3 with the
// per_block_cast_to_fp8 recipe: amax clamped at 1e-12, scale = amax / 448,
// q = e4m3(x / amax * 448) (FP32 arithmetic, round to nearest even).
__device__ __forceinline__ void quant_block_warp(const float (&v)[4], uint8_t* q, float* scale_out, int lane) {
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-12f);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float y = v[i] / amax * 448.0f;
    packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3)) << (8 * i);
  }
  reinterpret_cast<uint32_t*>(q)[lane] = packed;
  if (lane == 0) *scale_out = amax / 448.0f;
}

// One warp per (row, 128-column block).
__global__ void quant_rows_kernel(const void* x, int x_dtype, int64_t x_stride, int64_t M, int64_t K, uint8_t* q,
                                  int64_t q_stride, float* s, int64_t s_stride_m, int64_t s_stride_k) {
  const int64_t kb_count = K / 128;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= M * kb_count) return;
  const int64_t r = w / kb_count, kb = w - r * kb_count;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = load_f(x, x_dtype, r * x_stride + kb * 128 + lane * 4 + i);
  quant_block_warp(v, q + r * q_stride + kb * 128, s + r * s_stride_m + kb * s_stride_k, lane);
}

// One warp per (row, 128-column block of the output); gate = columns [0, I), up = [I, 2I).
__global__ void silu_mul_quant_kernel(const __nv_bfloat16* in, int64_t in_stride, int64_t M, int64_t I,
                                      const int32_t* m_indices, uint8_t* q, int64_t q_stride, float* s,
                                      int64_t s_stride_m, int64_t s_stride_k) {
  const int64_t kb_count = I / 128;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= M * kb_count) return;
  const int64_t r = w / kb_count, kb = w - r * kb_count;
  if (m_indices && m_indices[r] < 0) return;  // padding row: never read by the next GEMM
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t c = kb * 128 + lane * 4 + i;
    const float g = __bfloat162float(in[r * in_stride + c]);
    const float u = __bfloat162float(in[r * in_stride + I + c]);
    v[i] = g / (1.0f + expf(-g)) * u;
  }
  quant_block_warp(v, q + r * q_stride + kb * 128, s + r * s_stride_m + kb * s_stride_k, lane);
}

__global__ void ep_count_kernel(const void* ids, int ids_dtype, int64_t n, int64_t E, int32_t* cnt) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = load_idx(ids, ids_dtype, i);
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
}

// Bytes of one dispatched row: [e4m3 data H][FP32 scales H/128][int32 local expert][pad to 16].
__host__ __device__ __forceinline__ int64_t packed_row_bytes(int64_t H) { return (H + 4 * (H / 128) + 4 + 15) / 16 * 16; }

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

// One warp per row: out[i, :] = Y[perm_pos[i], :].
__global__ void ep_unpermute_kernel(const __nv_bfloat16* Y, int64_t y_stride, const int32_t* perm_pos, int64_t R,
                                    int64_t H, __nv_bfloat16* out) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= R) return;
  const uint4* src = reinterpret_cast<const uint4*>(Y + static_cast<int64_t>(perm_pos[w]) * y_stride);
  uint4* dst = reinterpret_cast<uint4*>(out + w * H);
  for (int64_t c = lane; c < H / 8; c += 32) dst[c] = src[c];
}

// One CTA per token; y[t, :] = bf16(sum_j w[t, j] * rows[send_index[t*k + j], :]) in FP32, slots in order.
__global__ void ep_combine_kernel(const __nv_bfloat16* rows, const int32_t* send_index, const float* topk_w, int64_t T,
                                  int64_t topk, int64_t H, __nv_bfloat16* y) {
  const int64_t t = blockIdx.x;
  if (t >= T) return;
  for (int64_t c = threadIdx.x; c < H; c += blockDim.x) {
    float acc = 0.0f;
    for (int64_t j = 0; j < topk; ++j) {
      const int32_t r = send_index[t * topk + j];
      if (r >= 0) acc = fmaf(topk_w[t * topk + j], __bfloat162float(rows[static_cast<int64_t>(r) * H + c]), acc);
    }
    y[t * H + c] = __float2bfloat16_rn(acc);
  }
}

unsigned warp_grid(int64_t warps) { return static_cast<unsigned>((warps * 32 + 255) / 256); }

int launched() { return cudaGetLastError() == cudaSuccess ? CDG_OK : CDG_ERR_CUDA; }

}  // namespace
}  // namespace cdg

extern "C" {

int cdg_quant_fp8_rows(const void* x, int32_t x_dtype, int64_t x_stride, int64_t M, int64_t K, uint8_t* q,
                       int64_t q_stride, float* s, int64_t s_stride_m, int64_t s_stride_k, cdg_stream_t stream) {
  if (M < 0 || K <= 0 || K % 128 || (M > 0 && (!x || !q || !s))) return CDG_ERR_INVALID_ARGUMENT;
  if (x_dtype != CDG_DTYPE_BF16 && x_dtype != CDG_DTYPE_F32) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(q) % 4 || q_stride % 4) return CDG_ERR_ALIGNMENT;
  if (M == 0) return CDG_OK;
  cdg::quant_rows_kernel<<<cdg::warp_grid(M * (K / 128)), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, x_dtype, x_stride, M, K, q, q_stride, s, s_stride_m, s_stride_k);
  return cdg::launched();
}

int cdg_silu_mul_quant_fp8(const void* in, int64_t in_stride, int64_t M, int64_t I, const int32_t* m_indices,
                           uint8_t* q, int64_t q_stride, float* s, int64_t s_stride_m, int64_t s_stride_k,
                           cdg_stream_t stream) {
  if (M < 0 || I <= 0 || I % 128 || (M > 0 && (!in || !q || !s))) return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(q) % 4 || q_stride % 4) return CDG_ERR_ALIGNMENT;
  if (M == 0) return CDG_OK;
  cdg::silu_mul_quant_kernel<<<cdg::warp_grid(M * (I / 128)), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(in), in_stride, M, I, m_indices, q, q_stride, s, s_stride_m, s_stride_k);
  return cdg::launched();
}

int cdg_ep_count(const void* topk_ids, int32_t ids_dtype, int64_t n, int64_t E, int32_t* counts, cdg_stream_t stream) {
  if (n < 0 || E <= 0 || !counts || (n > 0 && !topk_ids)) return CDG_ERR_INVALID_ARGUMENT;
  if (ids_dtype != CDG_DTYPE_I32 && ids_dtype != CDG_DTYPE_I64) return CDG_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(counts, 0, E * sizeof(int32_t), st) != cudaSuccess) return CDG_ERR_CUDA;
  if (n == 0) return CDG_OK;
  const unsigned blocks = static_cast<unsigned>(n < 256 * 1024 ? (n + 255) / 256 : 1024);
  cdg::ep_count_kernel<<<blocks, 256, 0, st>>>(topk_ids, ids_dtype, n, E, counts);
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

int cdg_ep_combine(const void* rows, const int32_t* send_index, const float* topk_w, int64_t T, int64_t topk,
                   int64_t H, void* y, cdg_stream_t stream) {
  if (T < 0 || topk <= 0 || H <= 0) return CDG_ERR_INVALID_ARGUMENT;
  if (T == 0) return CDG_OK;
  cdg::ep_combine_kernel<<<static_cast<unsigned>(T), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(rows), send_index, topk_w, T, topk, H, static_cast<__nv_bfloat16*>(y));
  return cdg::launched();
}

}  // extern "C"
