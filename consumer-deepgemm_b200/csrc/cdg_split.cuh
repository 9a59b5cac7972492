// The split of e4m3 activations with FP32 1x128 scales into the two e4m3 planes the tensor
// cores read, shared by the GEMM's prep kernel and the MoE layer's quantising steps (which
// write the planes themselves, CDG_DTYPE_E4M3_PLANES).
//
// The reference dequantises activations to BF16: x = bf16(bf16(a) * bf16(s))
// (consumer_deep_gemm/gemm.py:44-48).  With E the frexp exponent of the largest finite
// |bf16(s)| of the row, every v = x / 2^E is a BF16 number of magnitude < 448 and splits into
// hi = e4m3(v) and lo = e4m3(v - hi), exactly when |v| >= 2^-2; the tensor core multiplies
// both planes with the weights and the epilogue scales the sum by 2^E.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>

namespace cdg {

// The row exponent of the planes from the largest finite |bf16(s)| of the row (0 when every
// scale is zero), and whether it lies in the range the MMA's scale factors and the epilogue's
// FP32 factor take ([-126, 127]).
__device__ __forceinline__ int plane_exponent(float smax, bool* in_range) {
  int e = 0;
  if (smax > 0.0f) frexpf(smax, &e);
  *in_range = e >= -126 && e <= 127;
  return e;
}

// Sixteen e4m3 codes (one 16-byte chunk of a row) with their block's BF16 scale `sbf` and the
// row's 2^-E `inv` -> the chunk of each plane.  Two elements per conversion instruction.
//   * v = bf16(a * (sbf * 2^-E)) equals bf16(a * sbf) * 2^-E: a * sbf is exact in FP32 (4 + 8
//     significant bits) and scaling by a power of two commutes with the rounding (outside
//     BF16's subnormal range, which no scale of one row reaches relative to the row's largest);
//   * lo = e4m3(v - hi) with the difference taken in f16x2: v and hi are f16 numbers whenever
//     |v| >= 2^-17, and below that hi and lo are both zero either way, so the difference is
//     exact and lo is the same code as from FP32.
__device__ __forceinline__ void split_planes16(const uint4 raw, float sbf, float inv, uint4& hi4, uint4& lo4) {
  const float sp = sbf * inv;
  const uint32_t in[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t hw[4] = {0u, 0u, 0u, 0u}, lw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __nv_fp8x2_storage_t a2 = static_cast<__nv_fp8x2_storage_t>(in[i >> 1] >> (16 * (i & 1)));
    const float2 af = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(a2, __NV_E4M3)));
    const float2 v = __bfloat1622float2(__floats2bfloat162_rn(__fmul_rn(af.x, sp), __fmul_rn(af.y, sp)));
    const __nv_fp8x2_storage_t h = __nv_cvt_float2_to_fp8x2(v, __NV_SATFINITE, __NV_E4M3);
    const __half2 d = __hsub2(__float22half2_rn(v), __half2(__nv_cvt_fp8x2_to_halfraw2(h, __NV_E4M3)));
    const __nv_fp8x2_storage_t l = __nv_cvt_halfraw2_to_fp8x2(static_cast<__half2_raw>(d), __NV_SATFINITE, __NV_E4M3);
    hw[i >> 1] |= static_cast<uint32_t>(h) << (16 * (i & 1));
    lw[i >> 1] |= static_cast<uint32_t>(l) << (16 * (i & 1));
  }
  hi4 = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  lo4 = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// BF16 rounding of a scale, as the reference's dequant applies it.
__device__ __forceinline__ float bf16_round(float s) { return __bfloat162float(__float2bfloat16_rn(s)); }

}  // namespace cdg
