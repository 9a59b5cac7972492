// consumer_deep_gemm._C: the PyTorch binding of libcdg_b200.so.
//
// Mirrors the reference's pybind module (csrc/bindings.cpp:133-148): the same
// tuple arguments, the same shape/dtype checks (csrc/bindings.cpp:50-101), but
// every call ends in the C ABI of cdg_b200.h on the current CUDA stream with a
// workspace taken from PyTorch's caching allocator.  There is no host fallback:
// CPU tensors are rejected.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <string>
#include <vector>

#include "cdg_b200.h"

namespace py = pybind11;

namespace {

void check_status(int st, const char* what) {
  if (st == CDG_OK) return;
  const std::string msg = std::string(what) + ": " + cdg_status_string(st);
  if (st == CDG_ERR_INVALID_ARGUMENT || st == CDG_ERR_ALIGNMENT) throw std::invalid_argument(msg);
  if (st == CDG_ERR_UNSUPPORTED) throw std::runtime_error(msg + " (not implemented by this build)");
  TORCH_CHECK(false, msg);
}

int32_t dtype_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kFloat8_e4m3fn: return CDG_DTYPE_E4M3;
    case torch::kBFloat16: return CDG_DTYPE_BF16;
    case torch::kFloat32: return CDG_DTYPE_F32;
    case torch::kUInt8: return CDG_DTYPE_UE8M0;
    case torch::kInt32: return CDG_DTYPE_I32;
    case torch::kInt64: return CDG_DTYPE_I64;
    default: return 0;
  }
}

void check_cuda(const torch::Tensor& t, const char* name, const torch::Device& dev) {
  TORCH_CHECK(t.defined(), name, " must be defined");
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor (this build has no CPU path)");
  TORCH_CHECK(t.device() == dev, name, " must be on ", dev, ", got ", t.device());
}

// Fill the C-ABI argument block from already-normalised tensors (see gemm.py).
//   a: [M,K] e4m3/bf16/f32;  sa: [M,C] f32 or undefined;  b: [E,N,K/2] uint8
//   sfb: [E,N,K/32] uint8/f32 or int32 atoms [E,N/128,K/128,128];  d: [M,N] bf16/f32
cdg_gemm_args make_args(const torch::Tensor& a, const c10::optional<torch::Tensor>& sa, const torch::Tensor& b,
                        const torch::Tensor& sfb, const torch::Tensor& d, const c10::optional<torch::Tensor>& ids,
                        int64_t flags, bool masked = false) {
  const auto dev = a.device();
  check_cuda(a, "a", dev);
  check_cuda(b, "b", dev);
  check_cuda(sfb, "b scale", dev);
  check_cuda(d, "d", dev);
  TORCH_CHECK_VALUE(a.dim() == 2, "a must be [M, K], got dim ", a.dim());
  TORCH_CHECK_VALUE(b.dim() == 3, "b must be [G, N, K/2] packed FP4, got dim ", b.dim());
  TORCH_CHECK_VALUE(d.dim() == 2, "d must be [M, N], got dim ", d.dim());
  TORCH_CHECK_VALUE(a.stride(1) == 1 && d.stride(1) == 1, "a and d must have unit stride along their last dim");
  TORCH_CHECK_VALUE(b.is_contiguous(), "b must be contiguous");
  TORCH_CHECK_VALUE(b.scalar_type() == torch::kUInt8 || b.scalar_type() == torch::kInt8,
                    "b must be int8/uint8 packed FP4, got ", b.scalar_type());
  const int64_t M = a.size(0), K = a.size(1), E = b.size(0), N = b.size(1);
  TORCH_CHECK_VALUE(b.size(2) * 2 == K, "b packed K must equal a K/2, got b.size(2)=", b.size(2), " and a K=", K);
  TORCH_CHECK_VALUE(d.size(0) == M, "d M must match a M");
  TORCH_CHECK_VALUE(d.size(1) == N, "d N must match b N");

  cdg_gemm_args g{};
  g.a = a.data_ptr();
  g.a_dtype = dtype_code(a);
  TORCH_CHECK_VALUE(g.a_dtype == CDG_DTYPE_E4M3 || g.a_dtype == CDG_DTYPE_BF16 || g.a_dtype == CDG_DTYPE_F32,
                    "a must be FP8/BF16/FP32, got ", a.scalar_type());
  g.a_row_stride = a.stride(0);
  if (g.a_dtype == CDG_DTYPE_E4M3) {
    TORCH_CHECK_VALUE(sa.has_value(), "FP8 a needs its scale");
    const auto& s = *sa;
    check_cuda(s, "a scale", dev);
    TORCH_CHECK_VALUE((s.scalar_type() == torch::kFloat32 || s.scalar_type() == torch::kInt32) && s.dim() == 2 &&
                          s.size(0) == M,
                      "a scale must be float32 [M, K/128] or int32 [M, ceil(K/512)] (packed UE8M0)");
    g.sa = static_cast<const float*>(s.data_ptr());
    g.sa_dtype = s.scalar_type() == torch::kInt32 ? CDG_DTYPE_UE8M0_X4 : CDG_DTYPE_F32;
    g.sa_stride_m = s.stride(0);
    g.sa_stride_k = s.stride(1);
    g.sa_cols = static_cast<int32_t>(s.size(1));
  }
  g.b = b.data_ptr();
  g.b_stride_e = b.stride(0);
  g.b_stride_n = b.stride(1);
  g.sfb = sfb.data_ptr();
  if (sfb.scalar_type() == torch::kInt32) {
    const int64_t NT = (N + 127) / 128, KT = (K / 32 + 3) / 4;
    TORCH_CHECK_VALUE(sfb.is_contiguous() && sfb.dim() == 4 && sfb.size(0) == E && sfb.size(1) == NT &&
                          sfb.size(2) == KT && sfb.size(3) == 128,
                      "transformed b scale must be int32 [E, N/128, K/128, 128]");
    g.sfb_dtype = CDG_DTYPE_UE8M0;
    g.sfb_layout = CDG_SF_ATOMS;
  } else {
    TORCH_CHECK_VALUE(sfb.dim() == 3 && sfb.size(0) == E && sfb.size(1) == N && sfb.stride(2) == 1,
                      "b scale must be [G, N, K/32] with unit last stride");
    TORCH_CHECK_VALUE(sfb.size(2) == (K + 31) / 32, "b scale must have ceil(K/32) columns");
    g.sfb_dtype = dtype_code(sfb);
    TORCH_CHECK_VALUE(g.sfb_dtype == CDG_DTYPE_UE8M0 || g.sfb_dtype == CDG_DTYPE_F32,
                      "b scale must be uint8 (UE8M0) or float32, got ", sfb.scalar_type());
    g.sfb_layout = CDG_SF_ROW_MAJOR;
    g.sfb_stride_e = sfb.stride(0);
    g.sfb_stride_n = sfb.stride(1);
  }
  if (ids.has_value()) {
    const auto& t = *ids;
    check_cuda(t, "m_indices", dev);
    TORCH_CHECK_VALUE(t.dim() == 1 && t.is_contiguous(), "m_indices must be a contiguous 1D tensor");
    g.m_indices_dtype = dtype_code(t);
    TORCH_CHECK_VALUE(g.m_indices_dtype == CDG_DTYPE_I32 || g.m_indices_dtype == CDG_DTYPE_I64,
                      "m_indices must be int32/int64, got ", t.scalar_type());
    if (masked) {
      TORCH_CHECK_VALUE(t.numel() == E, "masked_m length must be G, got ", t.numel(), ", G=", E);
    } else {
      TORCH_CHECK_VALUE(t.numel() == M || t.numel() == E, "m_indices length must be M or G, got ", t.numel(),
                        ", M=", M, ", G=", E);
    }
    g.m_indices = t.data_ptr();
    g.m_indices_len = t.numel();
    g.index_form = masked ? CDG_INDEX_MASKED : t.numel() == M ? CDG_INDEX_PER_ROW : CDG_INDEX_PSUM;
  } else {
    TORCH_CHECK_VALUE(E == 1, "m_indices is required when b has multiple groups");
    g.index_form = CDG_INDEX_NONE;
  }
  g.d = d.data_ptr();
  g.d_dtype = dtype_code(d);
  TORCH_CHECK_VALUE(g.d_dtype == CDG_DTYPE_BF16 || g.d_dtype == CDG_DTYPE_F32, "d must be BF16/FP32, got ",
                    d.scalar_type());
  g.d_row_stride = d.stride(0);
  g.M = M;
  g.N = N;
  g.K = K;
  g.E = E;
  g.flags = static_cast<int32_t>(flags);
  return g;
}

// D through a row table (cdg_gemm_args.d_rows): int64 [M] addresses on the device; `d` then only
// gives the shape and dtype (an expanded [1, N] BF16 view will do) and is not written.
void set_d_rows(cdg_gemm_args& g, const c10::optional<torch::Tensor>& d_rows) {
  if (!d_rows.has_value()) return;
  const auto& t = *d_rows;
  TORCH_CHECK_VALUE(t.is_cuda() && t.scalar_type() == torch::kInt64 && t.is_contiguous() && t.numel() == g.M,
                    "d_rows: contiguous int64 [M] row addresses on the device");
  TORCH_CHECK_VALUE(g.d_dtype == CDG_DTYPE_BF16, "d_rows needs a BF16 output");
  g.d_rows = reinterpret_cast<const uint64_t*>(t.data_ptr<int64_t>());
  g.d = nullptr;
  g.d_row_stride = g.N;
}

void grouped_gemm(const torch::Tensor& a, const c10::optional<torch::Tensor>& sa, const torch::Tensor& b,
                  const torch::Tensor& sfb, const torch::Tensor& d, const c10::optional<torch::Tensor>& ids,
                  int64_t flags, bool masked, const c10::optional<torch::Tensor>& d_rows) {
  cdg_gemm_args g = make_args(a, sa, b, sfb, d, ids, flags, masked);
  set_d_rows(g, d_rows);
  const c10::cuda::CUDAGuard guard(a.device());
  const size_t ws_bytes = cdg_grouped_fp8_fp4_workspace_bytes(&g);
  TORCH_CHECK(ws_bytes > 0, "invalid GEMM arguments");
  // 1024 bytes of slack so the workspace can start on a 1024-byte boundary.
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes + 1024)}, a.options().dtype(torch::kUInt8));
  auto* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 1023) & ~uintptr_t(1023));
  const auto stream = at::cuda::getCurrentCUDAStream(a.get_device()).stream();
  if (masked)
    check_status(cdg_grouped_fp8_fp4_gemm_nt_masked(&g, base, ws_bytes, reinterpret_cast<cdg_stream_t>(stream)),
                 "m_grouped_fp8_fp4_gemm_nt_masked");
  else
    check_status(cdg_grouped_fp8_fp4_gemm_nt_contiguous(&g, base, ws_bytes, reinterpret_cast<cdg_stream_t>(stream)),
                 "m_grouped_fp8_fp4_gemm_nt_contiguous");
}

cdg_stream_t cur_stream(const torch::Tensor& t);

// The GEMM on activations given as e4m3 planes [2, M, K] (uint8) with int32 row exponents [M]
// (CDG_DTYPE_E4M3_PLANES): the form the MoE layer's own quantising steps write.
void grouped_gemm_planes(const torch::Tensor& planes, const torch::Tensor& row_exp, const torch::Tensor& b,
                         const torch::Tensor& sfb, const torch::Tensor& d, const torch::Tensor& ids, int64_t flags,
                         const c10::optional<torch::Tensor>& d_rows) {
  TORCH_CHECK_VALUE(planes.is_cuda() && planes.dim() == 3 && planes.size(0) == 2 && planes.is_contiguous() &&
                        planes.scalar_type() == torch::kUInt8,
                    "planes: contiguous uint8 [2, M, K] on the device");
  const int64_t M = planes.size(1);
  TORCH_CHECK_VALUE(row_exp.is_cuda() && row_exp.scalar_type() == torch::kInt32 && row_exp.is_contiguous() &&
                        row_exp.numel() == M,
                    "row exponents: contiguous int32 [M]");
  // the argument block of the hi plane as an e4m3 [M, K] operand, then switched to the planes form
  const torch::Tensor hi = planes.select(0, 0).view(torch::kFloat8_e4m3fn);
  cdg_gemm_args g = make_args(hi, row_exp.view({M, 1}), b, sfb, d, ids, flags);
  g.a_dtype = CDG_DTYPE_E4M3_PLANES;
  g.sa = reinterpret_cast<const float*>(row_exp.data_ptr());
  g.sa_dtype = CDG_DTYPE_I32;
  g.sa_stride_m = 1;
  g.sa_stride_k = 1;
  g.sa_cols = 1;
  set_d_rows(g, d_rows);
  const c10::cuda::CUDAGuard guard(planes.device());
  const size_t ws_bytes = cdg_grouped_fp8_fp4_workspace_bytes(&g);
  TORCH_CHECK_VALUE(ws_bytes > 0, "invalid GEMM arguments for the planes form");
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes + 1024)}, planes.options());
  auto* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 1023) & ~uintptr_t(1023));
  check_status(cdg_grouped_fp8_fp4_gemm_nt_contiguous(&g, base, ws_bytes, cur_stream(planes)),
               "m_grouped_fp8_fp4_gemm_nt_contiguous (planes)");
}

int64_t can_implement(const torch::Tensor& a, const c10::optional<torch::Tensor>& sa, const torch::Tensor& b,
                      const torch::Tensor& sfb, const torch::Tensor& d, const c10::optional<torch::Tensor>& ids) {
  const cdg_gemm_args g = make_args(a, sa, b, sfb, d, ids, 0);
  return cdg_can_implement(&g);
}

torch::Tensor transform_sf_atoms(const torch::Tensor& sf) {
  TORCH_CHECK(sf.is_cuda(), "scale must be a CUDA tensor");
  TORCH_CHECK_VALUE(sf.dim() == 3 && sf.scalar_type() == torch::kUInt8 && sf.stride(2) == 1,
                    "scale must be uint8 [E, N, K/32] with unit last stride");
  const c10::cuda::CUDAGuard guard(sf.device());
  const int64_t E = sf.size(0), N = sf.size(1), KB = sf.size(2);
  auto out = torch::empty({E, (N + 127) / 128, (KB + 3) / 4, 128}, sf.options().dtype(torch::kInt32));
  const auto stream = at::cuda::getCurrentCUDAStream(sf.get_device()).stream();
  check_status(cdg_transform_sf(sf.data_ptr<uint8_t>(), sf.stride(0), sf.stride(1), E, N, KB,
                                reinterpret_cast<uint8_t*>(out.data_ptr()), reinterpret_cast<cdg_stream_t>(stream)),
               "transform_sf_into_required_layout");
  return out;
}

cdg_stream_t cur_stream(const torch::Tensor& t) {
  return reinterpret_cast<cdg_stream_t>(at::cuda::getCurrentCUDAStream(t.get_device()).stream());
}

// ------------------------------------------------------------------ MoE layer / expert parallelism
std::vector<torch::Tensor> quant_fp8_rows(const torch::Tensor& x, bool ue8m0) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "x must be a CUDA [M, K] tensor with unit last stride");
  TORCH_CHECK_VALUE(x.scalar_type() == torch::kBFloat16 || x.scalar_type() == torch::kFloat32, "x must be BF16/FP32");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t M = x.size(0), K = x.size(1);
  auto q = torch::empty({M, K}, x.options().dtype(torch::kFloat8_e4m3fn));
  auto s = torch::empty({M, K / 128}, x.options().dtype(torch::kFloat32));
  check_status(cdg_quant_fp8_rows(x.data_ptr(), dtype_code(x), x.stride(0), M, K,
                                  reinterpret_cast<uint8_t*>(q.data_ptr()), K, s.data_ptr<float>(), K / 128, 1,
                                  ue8m0 ? CDG_SCALE_POW2 : CDG_SCALE_FP32, cur_stream(x)),
               "quant_fp8_rows");
  return {q, s};
}

std::vector<torch::Tensor> silu_mul_quant(const torch::Tensor& h, const c10::optional<torch::Tensor>& m_indices,
                                          bool ue8m0) {
  TORCH_CHECK(h.is_cuda() && h.dim() == 2 && h.stride(1) == 1 && h.scalar_type() == torch::kBFloat16,
              "h must be a CUDA BF16 [M, 2I] tensor with unit last stride");
  const c10::cuda::CUDAGuard guard(h.device());
  const int64_t M = h.size(0), I = h.size(1) / 2;
  auto q = torch::empty({M, I}, h.options().dtype(torch::kFloat8_e4m3fn));
  auto s = torch::empty({M, I / 128}, h.options().dtype(torch::kFloat32));
  const int32_t* ids = nullptr;
  if (m_indices.has_value()) {
    TORCH_CHECK(m_indices->scalar_type() == torch::kInt32 && m_indices->numel() == M, "m_indices must be int32 [M]");
    ids = m_indices->data_ptr<int32_t>();
  }
  check_status(cdg_silu_mul_quant_fp8(h.data_ptr(), h.stride(0), M, I, ids, reinterpret_cast<uint8_t*>(q.data_ptr()),
                                      I, s.data_ptr<float>(), I / 128, 1, ue8m0 ? CDG_SCALE_POW2 : CDG_SCALE_FP32,
                                      cur_stream(h)),
               "silu_mul_quant");
  return {q, s};
}

torch::Tensor ep_count(const torch::Tensor& ids, int64_t E) {
  TORCH_CHECK(ids.is_cuda() && ids.is_contiguous(), "topk ids must be a contiguous CUDA tensor");
  const c10::cuda::CUDAGuard guard(ids.device());
  auto cnt = torch::empty({E}, ids.options().dtype(torch::kInt32));
  check_status(cdg_ep_count(ids.data_ptr(), dtype_code(ids), ids.numel(), E, cnt.data_ptr<int32_t>(), cur_stream(ids)),
               "ep_count");
  return cnt;
}

std::vector<torch::Tensor> ep_count_offsets(const torch::Tensor& ids, int64_t E) {
  TORCH_CHECK(ids.is_cuda() && ids.is_contiguous(), "topk ids must be a contiguous CUDA tensor");
  const c10::cuda::CUDAGuard guard(ids.device());
  auto cnt = torch::empty({E}, ids.options().dtype(torch::kInt32));
  auto off = torch::empty({E}, ids.options().dtype(torch::kInt64));
  auto scratch = torch::empty({1}, ids.options().dtype(torch::kInt32));
  check_status(cdg_ep_count_offsets(ids.data_ptr(), dtype_code(ids), ids.numel(), E, cnt.data_ptr<int32_t>(),
                                    off.data_ptr<int64_t>(), scratch.data_ptr<int32_t>(), cur_stream(ids)),
               "ep_count_offsets");
  return {cnt, off};
}

// Returns (packed rows uint8 [R, cdg_ep_row_bytes(H)], send_index [T*topk]).
std::vector<torch::Tensor> ep_pack(const torch::Tensor& xq, const torch::Tensor& xs, const torch::Tensor& ids,
                                   int64_t E, int64_t ranks, const torch::Tensor& send_off, int64_t rows) {
  TORCH_CHECK(xq.is_cuda() && xq.dim() == 2 && xq.is_contiguous(), "xq must be contiguous [T, H]");
  TORCH_CHECK(xs.is_contiguous() && ids.is_contiguous() && ids.dim() == 2, "xs and topk ids must be contiguous");
  TORCH_CHECK(send_off.scalar_type() == torch::kInt64 && send_off.numel() == ranks, "send_off must be int64 [ranks]");
  const c10::cuda::CUDAGuard guard(xq.device());
  const int64_t T = xq.size(0), H = xq.size(1), topk = ids.size(1);
  auto out = torch::empty({rows, cdg_ep_row_bytes(H)}, xq.options().dtype(torch::kUInt8));
  auto send_index = torch::empty({T * topk}, ids.options().dtype(torch::kInt32));
  auto fill = torch::empty({ranks}, ids.options().dtype(torch::kInt32));
  check_status(cdg_ep_pack(reinterpret_cast<const uint8_t*>(xq.data_ptr()), H, xs.data_ptr<float>(), H / 128,
                           ids.data_ptr(), dtype_code(ids), T, topk, E, ranks, H, send_off.data_ptr<int64_t>(),
                           fill.data_ptr<int32_t>(), out.data_ptr<uint8_t>(), send_index.data_ptr<int32_t>(),
                           cur_stream(xq)),
               "ep_pack");
  return {out, send_index};
}

// Returns (A e4m3 [M_pad, H], SA [M_pad, H/128], m_indices [M_pad], perm_pos [R]).
std::vector<torch::Tensor> ep_permute(const torch::Tensor& rows, int64_t H, int64_t E_local,
                                      const torch::Tensor& expert_off, int64_t M_pad) {
  TORCH_CHECK(rows.is_cuda() && rows.dim() == 2 && rows.is_contiguous() && rows.scalar_type() == torch::kUInt8 &&
                  rows.size(1) == cdg_ep_row_bytes(H),
              "received rows must be contiguous packed rows");
  TORCH_CHECK(expert_off.scalar_type() == torch::kInt64 && expert_off.numel() == E_local, "expert_off: int64 [E]");
  const c10::cuda::CUDAGuard guard(rows.device());
  const int64_t R = rows.size(0);
  auto i32 = rows.options().dtype(torch::kInt32);
  auto A = torch::empty({M_pad, H}, rows.options().dtype(torch::kFloat8_e4m3fn));
  auto SA = torch::ones({M_pad, H / 128}, rows.options().dtype(torch::kFloat32));
  auto mi = torch::empty({M_pad}, i32);
  auto pos = torch::empty({R}, i32);
  auto fill = torch::empty({E_local}, i32);
  check_status(cdg_ep_permute(rows.data_ptr<uint8_t>(), R, H, E_local, expert_off.data_ptr<int64_t>(),
                              fill.data_ptr<int32_t>(), reinterpret_cast<uint8_t*>(A.data_ptr()), SA.data_ptr<float>(),
                              mi.data_ptr<int32_t>(), M_pad, pos.data_ptr<int32_t>(), cur_stream(rows)),
               "ep_permute");
  return {A, SA, mi, pos};
}

// One rank: quantise + contiguous layout in one pass -> (A, SA, m_indices, perm_pos, send_index).
std::vector<torch::Tensor> silu_mul_quant_planes(const torch::Tensor& h, const torch::Tensor& m_indices) {
  TORCH_CHECK(h.is_cuda() && h.dim() == 2 && h.stride(1) == 1 && h.scalar_type() == torch::kBFloat16,
              "h must be a CUDA BF16 [M, 2I] tensor with unit last stride");
  TORCH_CHECK(m_indices.scalar_type() == torch::kInt32 && m_indices.numel() == h.size(0), "m_indices must be int32 [M]");
  const c10::cuda::CUDAGuard guard(h.device());
  const int64_t M = h.size(0), I = h.size(1) / 2;
  auto planes = torch::empty({2, M, I}, h.options().dtype(torch::kUInt8));
  auto row_exp = torch::empty({M}, h.options().dtype(torch::kInt32));
  check_status(cdg_silu_mul_quant_planes(h.data_ptr(), h.stride(0), M, I, m_indices.data_ptr<int32_t>(),
                                         planes.data_ptr<uint8_t>(), row_exp.data_ptr<int32_t>(), cur_stream(h)),
               "silu_mul_quant_planes");
  return {planes, row_exp};
}

std::vector<torch::Tensor> ep_quant_dispatch_local_planes(const torch::Tensor& x, const torch::Tensor& ids, int64_t E,
                                                          const torch::Tensor& expert_off, int64_t M_pad) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "x must be a CUDA [T, H] tensor with unit last stride");
  TORCH_CHECK(ids.is_cuda() && ids.is_contiguous() && ids.dim() == 2 && ids.size(0) == x.size(0),
              "topk ids must be contiguous [T, topk]");
  TORCH_CHECK(expert_off.is_cuda() && expert_off.scalar_type() == torch::kInt64 && expert_off.numel() == E,
              "expert_off: int64 [E] on the device");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), topk = ids.size(1);
  auto i32 = ids.options().dtype(torch::kInt32);
  auto planes = torch::empty({2, M_pad, H}, x.options().dtype(torch::kUInt8));
  auto row_exp = torch::empty({M_pad}, i32);
  auto mi = torch::empty({M_pad}, i32);
  auto pos = torch::empty({T * topk}, i32);
  auto send_index = torch::empty({T * topk}, i32);
  auto fill = torch::empty({E}, i32);
  check_status(cdg_ep_quant_dispatch_local_planes(x.data_ptr(), dtype_code(x), x.stride(0), ids.data_ptr(),
                                                  dtype_code(ids), T, topk, E, H, expert_off.data_ptr<int64_t>(),
                                                  fill.data_ptr<int32_t>(), planes.data_ptr<uint8_t>(),
                                                  row_exp.data_ptr<int32_t>(), mi.data_ptr<int32_t>(), M_pad,
                                                  pos.data_ptr<int32_t>(), send_index.data_ptr<int32_t>(), cur_stream(x)),
               "ep_quant_dispatch_local_planes");
  return {planes, row_exp, mi, pos, send_index};
}

std::vector<torch::Tensor> ep_quant_dispatch_local(const torch::Tensor& x, const torch::Tensor& ids, int64_t E,
                                                   const torch::Tensor& expert_off, int64_t M_pad, bool ue8m0) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "x must be a CUDA [T, H] tensor with unit last stride");
  TORCH_CHECK(ids.is_cuda() && ids.is_contiguous() && ids.dim() == 2 && ids.size(0) == x.size(0),
              "topk ids must be contiguous [T, topk]");
  TORCH_CHECK(expert_off.is_cuda() && expert_off.scalar_type() == torch::kInt64 && expert_off.numel() == E,
              "expert_off: int64 [E] on the device");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), topk = ids.size(1);
  auto i32 = ids.options().dtype(torch::kInt32);
  auto A = torch::empty({M_pad, H}, x.options().dtype(torch::kFloat8_e4m3fn));
  auto SA = torch::ones({M_pad, H / 128}, x.options().dtype(torch::kFloat32));
  auto mi = torch::empty({M_pad}, i32);
  auto pos = torch::empty({T * topk}, i32);
  auto send_index = torch::empty({T * topk}, i32);
  auto fill = torch::empty({E}, i32);
  check_status(cdg_ep_quant_dispatch_local(x.data_ptr(), dtype_code(x), x.stride(0), ids.data_ptr(), dtype_code(ids), T,
                                           topk, E, H, expert_off.data_ptr<int64_t>(), fill.data_ptr<int32_t>(),
                                           reinterpret_cast<uint8_t*>(A.data_ptr()), SA.data_ptr<float>(),
                                           mi.data_ptr<int32_t>(), M_pad, pos.data_ptr<int32_t>(),
                                           send_index.data_ptr<int32_t>(), ue8m0 ? CDG_SCALE_POW2 : CDG_SCALE_FP32,
                                           cur_stream(x)),
               "ep_quant_dispatch_local");
  return {A, SA, mi, pos, send_index};
}

// Fixed-capacity send buffer: (packed rows uint8 [ranks*(cap+1), row_bytes], send_index [T*topk]).
std::vector<torch::Tensor> ep_quant_pack_fixed(const torch::Tensor& x, const torch::Tensor& ids, int64_t E,
                                               int64_t ranks, int64_t cap, bool ue8m0) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "x must be a CUDA [T, H] tensor with unit last stride");
  TORCH_CHECK(ids.is_cuda() && ids.is_contiguous() && ids.dim() == 2 && ids.size(0) == x.size(0),
              "topk ids must be contiguous [T, topk]");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), topk = ids.size(1);
  auto out = torch::empty({ranks * (cap + 1), cdg_ep_row_bytes(H)}, x.options().dtype(torch::kUInt8));
  auto send_index = torch::empty({T * topk}, ids.options().dtype(torch::kInt32));
  auto scratch = torch::empty({std::max<int64_t>(cdg_ep_fixed_scratch_ints(ranks, E), 1)},
                              ids.options().dtype(torch::kInt32));
  check_status(cdg_ep_quant_pack_fixed(x.data_ptr(), dtype_code(x), x.stride(0), ids.data_ptr(), dtype_code(ids), T,
                                       topk, E, ranks, H, cap, scratch.data_ptr<int32_t>(), out.data_ptr<uint8_t>(),
                                       send_index.data_ptr<int32_t>(), ue8m0 ? CDG_SCALE_POW2 : CDG_SCALE_FP32,
                                       cur_stream(x)),
               "ep_quant_pack_fixed");
  return {out, send_index};
}

// Fixed-capacity receive buffer -> (A, SA, m_indices, perm_pos).
std::vector<torch::Tensor> ep_permute_fixed(const torch::Tensor& rows, int64_t H, int64_t E_local, int64_t ranks,
                                            int64_t cap, int64_t M_pad) {
  TORCH_CHECK(rows.is_cuda() && rows.dim() == 2 && rows.is_contiguous() && rows.scalar_type() == torch::kUInt8 &&
                  rows.size(1) == cdg_ep_row_bytes(H) && rows.size(0) == ranks * (cap + 1),
              "received rows must be a contiguous fixed-capacity buffer [ranks*(cap+1), row_bytes]");
  const c10::cuda::CUDAGuard guard(rows.device());
  auto i32 = rows.options().dtype(torch::kInt32);
  auto A = torch::empty({M_pad, H}, rows.options().dtype(torch::kFloat8_e4m3fn));
  auto SA = torch::empty({M_pad, H / 128}, rows.options().dtype(torch::kFloat32));
  auto mi = torch::empty({M_pad}, i32);
  auto pos = torch::empty({rows.size(0)}, i32);
  auto fill = torch::empty({E_local}, i32);
  check_status(cdg_ep_permute_fixed(rows.data_ptr<uint8_t>(), ranks, cap, H, E_local, fill.data_ptr<int32_t>(),
                                    reinterpret_cast<uint8_t*>(A.data_ptr()), SA.data_ptr<float>(),
                                    mi.data_ptr<int32_t>(), M_pad, pos.data_ptr<int32_t>(), cur_stream(rows)),
               "ep_permute_fixed");
  return {A, SA, mi, pos};
}

// [G, N, ...] row gather of transform_weights_for_mega_moe; returns a new contiguous tensor.
torch::Tensor mega_moe_transform_rows(const torch::Tensor& t, int64_t kind) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 3 && t.stride(2) == 1, "expects a CUDA [G, N, X] tensor with unit last stride");
  const c10::cuda::CUDAGuard guard(t.device());
  auto out = torch::empty(t.sizes(), t.options());
  const int64_t es = t.element_size();
  check_status(cdg_mega_moe_transform_rows(t.data_ptr(), t.stride(0) * es, t.stride(1) * es, out.data_ptr(), t.size(0),
                                           t.size(1), t.size(2) * es, static_cast<int32_t>(kind), cur_stream(t)),
               "transform_weights_for_mega_moe");
  return out;
}

// ------------------------------------------------------------------ peer-memory exchange
py::tuple ep_window_create(int64_t bytes) {
  void* w = nullptr;
  char handle[64];
  check_status(cdg_ep_window_create(static_cast<size_t>(bytes), &w, handle), "ep_window_create");
  return py::make_tuple(reinterpret_cast<uint64_t>(w), py::bytes(handle, 64));
}

uint64_t ep_window_open(const py::bytes& handle) {
  std::string h = handle;
  TORCH_CHECK_VALUE(h.size() == 64, "an exchange window handle is 64 bytes");
  void* w = nullptr;
  check_status(cdg_ep_window_open(h.data(), &w), "ep_window_open");
  return reinterpret_cast<uint64_t>(w);
}

torch::Tensor ep_dispatch_p2p(const torch::Tensor& x, const torch::Tensor& ids, int64_t E, int64_t ranks,
                              int64_t max_tokens, const torch::Tensor& peers, uint64_t window, int64_t me, bool ue8m0) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "x must be a CUDA [T, H] tensor with unit last stride");
  TORCH_CHECK(ids.is_cuda() && ids.is_contiguous() && ids.dim() == 2 && ids.size(0) == x.size(0),
              "topk ids must be contiguous [T, topk]");
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == torch::kInt64 && peers.numel() == ranks,
              "peers: int64 [ranks] window addresses on the device");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), topk = ids.size(1);
  auto send_index = torch::empty({T * topk}, ids.options().dtype(torch::kInt32));
  auto scratch = torch::empty({std::max<int64_t>(cdg_ep_fixed_scratch_ints(ranks, E), 1)},
                              ids.options().dtype(torch::kInt32));
  check_status(cdg_ep_dispatch_p2p(x.data_ptr(), dtype_code(x), x.stride(0), ids.data_ptr(), dtype_code(ids), T, topk,
                                   E, ranks, H, max_tokens,
                                   reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()),
                                   reinterpret_cast<void*>(window), static_cast<int32_t>(me),
                                   scratch.data_ptr<int32_t>(), send_index.data_ptr<int32_t>(),
                                   ue8m0 ? CDG_SCALE_POW2 : CDG_SCALE_FP32, cur_stream(x)),
               "ep_dispatch_p2p");
  return send_index;
}

// Optional row table of a fused return: uint64 [M_pad] when `peers` is given, else an empty tensor.
std::pair<const uint64_t*, torch::Tensor> ret_rows_for(const c10::optional<torch::Tensor>& peers, int64_t M_pad,
                                                       const torch::Tensor& like) {
  if (!peers.has_value()) return {nullptr, torch::empty({0}, like.options().dtype(torch::kInt64))};
  TORCH_CHECK(peers->is_cuda() && peers->scalar_type() == torch::kInt64 && peers->is_contiguous(),
              "peers: int64 window addresses on the device");
  return {reinterpret_cast<const uint64_t*>(peers->data_ptr<int64_t>()),
          torch::empty({M_pad}, like.options().dtype(torch::kInt64))};
}

std::vector<torch::Tensor> ep_permute_p2p(uint64_t window, int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H,
                                          int64_t E_local, int64_t M_pad, const torch::Tensor& like,
                                          const c10::optional<torch::Tensor>& peers) {
  const c10::cuda::CUDAGuard guard(like.device());
  auto i32 = like.options().dtype(torch::kInt32);
  auto A = torch::empty({M_pad, H}, like.options().dtype(torch::kFloat8_e4m3fn));
  auto SA = torch::empty({M_pad, H / 128}, like.options().dtype(torch::kFloat32));
  auto mi = torch::empty({M_pad}, i32);
  auto ret_slot = torch::empty({M_pad}, i32);
  auto fill = torch::empty({E_local}, i32);
  auto [pp, ret_rows] = ret_rows_for(peers, M_pad, like);
  check_status(cdg_ep_permute_p2p(reinterpret_cast<void*>(window), ranks, max_tokens, topk, H, E_local,
                                  fill.data_ptr<int32_t>(), reinterpret_cast<uint8_t*>(A.data_ptr()),
                                  SA.data_ptr<float>(), mi.data_ptr<int32_t>(), M_pad, ret_slot.data_ptr<int32_t>(),
                                  pp, pp ? reinterpret_cast<uint64_t*>(ret_rows.data_ptr<int64_t>()) : nullptr,
                                  cur_stream(like)),
               "ep_permute_p2p");
  return {A, SA, mi, ret_slot, ret_rows};
}

std::vector<torch::Tensor> ep_permute_p2p_planes(uint64_t window, int64_t ranks, int64_t max_tokens, int64_t topk,
                                                 int64_t H, int64_t E_local, int64_t M_pad, const torch::Tensor& like,
                                                 const c10::optional<torch::Tensor>& peers) {
  const c10::cuda::CUDAGuard guard(like.device());
  auto i32 = like.options().dtype(torch::kInt32);
  auto planes = torch::empty({2, M_pad, H}, like.options().dtype(torch::kUInt8));
  auto row_exp = torch::empty({M_pad}, i32);
  auto mi = torch::empty({M_pad}, i32);
  auto ret_slot = torch::empty({M_pad}, i32);
  auto fill = torch::empty({E_local}, i32);
  auto [pp, ret_rows] = ret_rows_for(peers, M_pad, like);
  check_status(cdg_ep_permute_p2p_planes(reinterpret_cast<void*>(window), ranks, max_tokens, topk, H, E_local,
                                         fill.data_ptr<int32_t>(), planes.data_ptr<uint8_t>(),
                                         row_exp.data_ptr<int32_t>(), mi.data_ptr<int32_t>(), M_pad,
                                         ret_slot.data_ptr<int32_t>(), pp,
                                         pp ? reinterpret_cast<uint64_t*>(ret_rows.data_ptr<int64_t>()) : nullptr,
                                         cur_stream(like)),
               "ep_permute_p2p_planes");
  return {planes, row_exp, mi, ret_slot, ret_rows};
}

void ep_return_p2p(const torch::Tensor& Y, const torch::Tensor& ret_slot, int64_t ranks, int64_t max_tokens,
                   int64_t topk, const torch::Tensor& peers, uint64_t window, int64_t me) {
  TORCH_CHECK(Y.is_cuda() && Y.dim() == 2 && Y.stride(1) == 1 && Y.scalar_type() == torch::kBFloat16, "Y: BF16 rows");
  TORCH_CHECK(ret_slot.is_cuda() && ret_slot.scalar_type() == torch::kInt32 && ret_slot.is_contiguous(),
              "ret_slot: int32, one entry per GEMM row");
  const c10::cuda::CUDAGuard guard(Y.device());
  auto scratch = torch::empty({1}, ret_slot.options());
  check_status(cdg_ep_return_p2p(Y.data_ptr(), Y.stride(0), Y.size(0), ret_slot.data_ptr<int32_t>(), ret_slot.numel(),
                                 ranks, max_tokens, topk, Y.size(1),
                                 reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()),
                                 reinterpret_cast<void*>(window), static_cast<int32_t>(me), scratch.data_ptr<int32_t>(),
                                 cur_stream(Y)),
               "ep_return_p2p");
}

torch::Tensor ep_combine_p2p(uint64_t window, const torch::Tensor& send_index, const torch::Tensor& topk_w,
                             int64_t ranks, int64_t max_tokens, int64_t H, const c10::optional<torch::Tensor>& peers,
                             int64_t me) {
  TORCH_CHECK(topk_w.is_cuda() && topk_w.scalar_type() == torch::kFloat32 && topk_w.is_contiguous() &&
                  topk_w.dim() == 2 && send_index.numel() == topk_w.numel(),
              "topk weights: FP32 [T, topk] matching send_index");
  const c10::cuda::CUDAGuard guard(topk_w.device());
  const int64_t T = topk_w.size(0), topk = topk_w.size(1);
  auto y = torch::empty({T, H}, topk_w.options().dtype(torch::kBFloat16));
  auto scratch = torch::empty({2}, send_index.options());
  const uint64_t* pp = nullptr;
  if (peers.has_value()) {
    TORCH_CHECK(peers->is_cuda() && peers->scalar_type() == torch::kInt64 && peers->is_contiguous(),
                "peers: int64 window addresses on the device");
    pp = reinterpret_cast<const uint64_t*>(peers->data_ptr<int64_t>());
  }
  check_status(cdg_ep_combine_p2p(reinterpret_cast<void*>(window), send_index.data_ptr<int32_t>(),
                                  topk_w.data_ptr<float>(), T, topk, H, ranks, max_tokens, pp, static_cast<int32_t>(me),
                                  scratch.data_ptr<int32_t>(), y.data_ptr(), cur_stream(topk_w)),
               "ep_combine_p2p");
  return y;
}

torch::Tensor ep_unpermute(const torch::Tensor& Y, const torch::Tensor& perm_pos) {
  TORCH_CHECK(Y.is_cuda() && Y.dim() == 2 && Y.stride(1) == 1 && Y.scalar_type() == torch::kBFloat16, "Y: BF16 rows");
  const c10::cuda::CUDAGuard guard(Y.device());
  const int64_t R = perm_pos.numel(), H = Y.size(1);
  auto out = torch::empty({R, H}, Y.options());
  check_status(cdg_ep_unpermute(Y.data_ptr(), Y.stride(0), perm_pos.data_ptr<int32_t>(), R, H, out.data_ptr(),
                                cur_stream(Y)),
               "ep_unpermute");
  return out;
}

torch::Tensor ep_combine(const torch::Tensor& rows, const torch::Tensor& send_index, const torch::Tensor& topk_w) {
  TORCH_CHECK(rows.is_cuda() && rows.is_contiguous() && rows.scalar_type() == torch::kBFloat16, "rows: BF16");
  TORCH_CHECK(topk_w.scalar_type() == torch::kFloat32 && topk_w.is_contiguous() && topk_w.dim() == 2, "topk_w: f32");
  const c10::cuda::CUDAGuard guard(rows.device());
  const int64_t T = topk_w.size(0), topk = topk_w.size(1), H = rows.size(1);
  auto y = torch::empty({T, H}, rows.options());
  check_status(cdg_ep_combine(rows.data_ptr(), send_index.data_ptr<int32_t>(), topk_w.data_ptr<float>(), T, topk, H,
                              y.data_ptr(), cur_stream(rows)),
               "ep_combine");
  return y;
}

torch::Tensor ep_unpermute_combine(const torch::Tensor& Y, const torch::Tensor& perm_pos, const torch::Tensor& send_index,
                                   const torch::Tensor& topk_w) {
  TORCH_CHECK(Y.is_cuda() && Y.dim() == 2 && Y.stride(1) == 1 && Y.scalar_type() == torch::kBFloat16, "Y: BF16 rows");
  TORCH_CHECK(topk_w.scalar_type() == torch::kFloat32 && topk_w.is_contiguous() && topk_w.dim() == 2, "topk_w: f32");
  TORCH_CHECK(perm_pos.scalar_type() == torch::kInt32 && send_index.scalar_type() == torch::kInt32, "int32 indices");
  const c10::cuda::CUDAGuard guard(Y.device());
  const int64_t T = topk_w.size(0), topk = topk_w.size(1), H = Y.size(1);
  auto y = torch::empty({T, H}, Y.options());
  check_status(cdg_ep_unpermute_combine(Y.data_ptr(), Y.stride(0), perm_pos.data_ptr<int32_t>(),
                                        send_index.data_ptr<int32_t>(), topk_w.data_ptr<float>(), T, topk, H,
                                        y.data_ptr(), cur_stream(Y)),
               "ep_unpermute_combine");
  return y;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 grouped FP8 x MXFP4 MoE GEMM (binding of libcdg_b200.so)";
  m.def("is_available", []() { return true; });
  m.def("build_info", []() { return std::string(cdg_build_info()); });
  m.def("mk_alignment_for_contiguous_layout", []() { return cdg_mk_alignment_for_contiguous_layout(); });
  m.def("grouped_gemm", &grouped_gemm, py::arg("a"), py::arg("sa"), py::arg("b"), py::arg("sfb"), py::arg("d"),
        py::arg("m_indices"), py::arg("flags") = 0, py::arg("masked") = false, py::arg("d_rows") = py::none());
  m.def("grouped_gemm_planes", &grouped_gemm_planes, py::arg("planes"), py::arg("row_exp"), py::arg("b"),
        py::arg("sfb"), py::arg("d"), py::arg("m_indices"), py::arg("flags") = 0, py::arg("d_rows") = py::none());
  m.def("can_implement", &can_implement, py::arg("a"), py::arg("sa"), py::arg("b"), py::arg("sfb"), py::arg("d"),
        py::arg("m_indices"));
  m.def("transform_sf_atoms", &transform_sf_atoms, py::arg("sf"));
  m.def(
      "set_profile_events",
      [](uint64_t start, uint64_t stop) {
        check_status(cdg_set_profile_events(reinterpret_cast<void*>(start), reinterpret_cast<void*>(stop)),
                     "set_profile_events");
      },
      py::arg("start"), py::arg("stop"));
  m.def("quant_fp8_rows", &quant_fp8_rows, py::arg("x"), py::arg("ue8m0") = false);
  m.def("silu_mul_quant", &silu_mul_quant, py::arg("h"), py::arg("m_indices") = py::none(),
        py::arg("ue8m0") = false);
  m.def("ep_count", &ep_count, py::arg("topk_ids"), py::arg("num_experts"));
  m.def("ep_count_offsets", &ep_count_offsets, py::arg("topk_ids"), py::arg("num_experts"));
  m.def("ep_pack", &ep_pack, py::arg("xq"), py::arg("xs"), py::arg("topk_ids"), py::arg("num_experts"),
        py::arg("ranks"), py::arg("send_off"), py::arg("rows"));
  m.def("ep_permute", &ep_permute, py::arg("rows"), py::arg("hidden"), py::arg("local_experts"),
        py::arg("expert_off"), py::arg("m_pad"));
  m.def("ep_quant_pack_fixed", &ep_quant_pack_fixed, py::arg("x"), py::arg("topk_ids"), py::arg("num_experts"),
        py::arg("ranks"), py::arg("cap"), py::arg("ue8m0") = false);
  m.def("ep_quant_dispatch_local", &ep_quant_dispatch_local, py::arg("x"), py::arg("topk_ids"),
        py::arg("num_experts"), py::arg("expert_off"), py::arg("m_pad"), py::arg("ue8m0") = false);
  m.def("ep_permute_fixed", &ep_permute_fixed, py::arg("rows"), py::arg("hidden"), py::arg("local_experts"),
        py::arg("ranks"), py::arg("cap"), py::arg("m_pad"));
  m.def("mega_moe_transform_rows", &mega_moe_transform_rows, py::arg("t"), py::arg("kind"));
  m.def(
      "ep_window_bytes",
      [](int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H) {
        return cdg_ep_window_bytes(ranks, max_tokens, topk, H);
      },
      py::arg("ranks"), py::arg("max_tokens"), py::arg("topk"), py::arg("hidden"));
  m.def("ep_window_create", &ep_window_create, py::arg("bytes"));
  m.def("ep_window_open", &ep_window_open, py::arg("handle"));
  m.def(
      "ep_window_close",
      [](uint64_t w, bool opened) {
        check_status(cdg_ep_window_close(reinterpret_cast<void*>(w), opened ? 1 : 0), "ep_window_close");
      },
      py::arg("window"), py::arg("opened"));
  m.def(
      "ep_window_status",
      [](uint64_t w) {
        return cdg_ep_window_status(reinterpret_cast<void*>(w),
                                    reinterpret_cast<cdg_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
      },
      py::arg("window"));
  m.def("ep_dispatch_p2p", &ep_dispatch_p2p, py::arg("x"), py::arg("topk_ids"), py::arg("num_experts"),
        py::arg("ranks"), py::arg("max_tokens"), py::arg("peers"), py::arg("window"), py::arg("me"),
        py::arg("ue8m0") = false);
  m.def("ep_permute_p2p_planes", &ep_permute_p2p_planes, py::arg("window"), py::arg("ranks"), py::arg("max_tokens"),
        py::arg("topk"), py::arg("hidden"), py::arg("local_experts"), py::arg("m_pad"), py::arg("like"),
        py::arg("peers") = py::none());
  m.def("ep_quant_dispatch_local_planes", &ep_quant_dispatch_local_planes, py::arg("x"), py::arg("topk_ids"),
        py::arg("num_experts"), py::arg("expert_off"), py::arg("m_pad"));
  m.def("silu_mul_quant_planes", &silu_mul_quant_planes, py::arg("h"), py::arg("m_indices"));
  m.def("ep_permute_p2p", &ep_permute_p2p, py::arg("window"), py::arg("ranks"), py::arg("max_tokens"),
        py::arg("topk"), py::arg("hidden"), py::arg("local_experts"), py::arg("m_pad"), py::arg("like"),
        py::arg("peers") = py::none());
  m.def("ep_return_p2p", &ep_return_p2p, py::arg("y"), py::arg("ret_slot"), py::arg("ranks"), py::arg("max_tokens"),
        py::arg("topk"), py::arg("peers"), py::arg("window"), py::arg("me"));
  m.def("ep_combine_p2p", &ep_combine_p2p, py::arg("window"), py::arg("send_index"), py::arg("topk_w"),
        py::arg("ranks"), py::arg("max_tokens"), py::arg("hidden"), py::arg("peers") = py::none(),
        py::arg("me") = 0);
  m.def("ep_row_bytes", [](int64_t H) { return cdg_ep_row_bytes(H); }, py::arg("hidden"));
  m.def(
      "ep_set_wait_timeout_ns",
      [](uint64_t ns) { check_status(cdg_ep_set_wait_timeout_ns(ns), "ep_set_wait_timeout_ns"); }, py::arg("ns"));
  m.def(
      "device_status",
      [](bool clear) {
        int32_t where = 0;
        const int st = cdg_device_status(clear ? 1 : 0, &where);
        if (st != CDG_OK && st != CDG_ERR_DEVICE_TIMEOUT && st != CDG_ERR_DEVICE_INDEX)
          check_status(st, "device_status");
        return py::make_tuple(st, where);
      },
      py::arg("clear") = true);
  m.def(
      "set_num_sms", [](int64_t n) { check_status(cdg_set_num_sms(static_cast<int32_t>(n)), "set_num_sms"); },
      py::arg("num_sms"));
  m.def("get_num_sms", []() { return cdg_get_num_sms(); });
  m.def("set_pdl", [](bool v) { check_status(cdg_set_pdl(v ? 1 : 0), "set_pdl"); }, py::arg("enable"));
  m.def("get_pdl", []() { return cdg_get_pdl() != 0; });
  m.def("ep_unpermute", &ep_unpermute, py::arg("y"), py::arg("perm_pos"));
  m.def("ep_combine", &ep_combine, py::arg("rows"), py::arg("send_index"), py::arg("topk_w"));
  m.def("ep_unpermute_combine", &ep_unpermute_combine, py::arg("y"), py::arg("perm_pos"), py::arg("send_index"),
        py::arg("topk_w"));
}
