// Host side of libcdg_b200.so: argument checks, workspace carving, TMA
// descriptors and kernel launches behind the C ABI declared in cdg_b200.h.
//
// No call here blocks the host or copies device data to the host (except
// cdg_read_device_status and cdg_device_status, diagnostics).  The state kept between
// calls: a per-device, initialise-once record (SM count, compute capability, kernel
// attributes), the resolved driver entry point for tensor-map encoding, the process-wide
// SM limit of cdg_set_num_sms, and on the device the sticky error record the bounded waits
// write (g_sticky_status).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>

#include "cdg_b200.h"
#include "cdg_kernels.cuh"
#include "cdg_pair.cuh"
#include "cdg_planes.cuh"
#include "cdg_direct.cuh"
#include "cdg_layout.h"

namespace cdg {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

struct DeviceInfo {
  int sm_count = 0;
  int cc_major = 0;
  bool ok = false;
};

constexpr int kMaxDevices = 64;

const DeviceInfo& device_info(int dev) {
  static DeviceInfo infos[kMaxDevices];
  static std::once_flag flags[kMaxDevices];
  std::call_once(flags[dev], [dev] {
    DeviceInfo& d = infos[dev];
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return;
    if (cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return;
    if (d.cc_major == 10) {
      if (cudaFuncSetAttribute(cdg_gemm_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               GemmSmem<16>::kBytes) != cudaSuccess)
        return;
      if (cudaFuncSetAttribute(cdg_gemm_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               GemmSmem<32>::kBytes) != cudaSuccess)
        return;
      if (cudaFuncSetAttribute(cdg_gemm_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               GemmSmem<128>::kBytes) != cudaSuccess)
        return;
      if (cudaFuncSetAttribute(cdg_gemm_pair_kernel<16, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               PairSmem<16, 4>::kBytes) != cudaSuccess)
        return;
      if (cudaFuncSetAttribute(cdg_gemm_pair_kernel<32, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               PairSmem<32, 2>::kBytes) != cudaSuccess)
        return;
      if (cudaFuncSetAttribute(cdg_gemm_planes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               PlanesSmem::kBytes) != cudaSuccess)
        return;
      if (cudaFuncSetAttribute(cdg_gemm_direct_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               DirectSmem::kBytes) != cudaSuccess)
        return;
      if (cudaFuncSetAttribute(cdg_generic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
          cudaSuccess)
        return;
    }
    d.ok = true;
  });
  return infos[dev];
}

// SMs the persistent GEMM kernels may use (cdg_set_num_sms; 0 = all of the device's), and
// whether the GEMM kernels are launched with programmatic stream serialization (cdg_set_pdl).
std::atomic<int> g_num_sms{0};
std::atomic<int> g_pdl{1};

int usable_sms(const DeviceInfo& di) {
  const int n = g_num_sms.load(std::memory_order_relaxed);
  return n > 0 && n < di.sm_count ? n : di.sm_count;
}

// Optional events recorded around the tensor-core GEMM launches (per host thread).
thread_local cudaEvent_t t_prof_start = nullptr;
thread_local cudaEvent_t t_prof_stop = nullptr;

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Shape/dtype validation shared by every entry point; does not look at alignment.
int validate(const cdg_gemm_args* g) {
  if (!g) return CDG_ERR_INVALID_ARGUMENT;
  if (g->M < 0 || g->N <= 0 || g->K <= 0 || g->E <= 0) return CDG_ERR_INVALID_ARGUMENT;
  if (g->M > (int64_t(1) << 31) - 256 || g->N > (int64_t(1) << 24) || g->K > (int64_t(1) << 20) ||
      g->E > (int64_t(1) << 20))
    return CDG_ERR_UNSUPPORTED;
  if (g->K % 2) return CDG_ERR_INVALID_ARGUMENT;
  if (g->M > 0 && (!g->a || (!g->d && !g->d_rows))) return CDG_ERR_INVALID_ARGUMENT;
  if (g->d_rows && g->d_dtype != CDG_DTYPE_BF16) return CDG_ERR_INVALID_ARGUMENT;
  if (!g->b || !g->sfb) return CDG_ERR_INVALID_ARGUMENT;
  if (g->a_dtype != CDG_DTYPE_E4M3 && g->a_dtype != CDG_DTYPE_BF16 && g->a_dtype != CDG_DTYPE_F32 &&
      g->a_dtype != CDG_DTYPE_E4M3_PLANES)
    return CDG_ERR_INVALID_ARGUMENT;
  if (g->a_dtype == CDG_DTYPE_E4M3_PLANES) {
    // [2][M][K] planes and int32 row exponents, 128-aligned per-row groups
    if (!g->sa || g->sa_dtype != CDG_DTYPE_I32 || g->a_row_stride != g->K || g->M % 128 ||
        g->index_form != CDG_INDEX_PER_ROW)
      return CDG_ERR_INVALID_ARGUMENT;
  } else if (g->sa_dtype != 0 && g->sa_dtype != CDG_DTYPE_F32 && g->sa_dtype != CDG_DTYPE_UE8M0_X4) {
    return CDG_ERR_INVALID_ARGUMENT;
  }
  if (g->a_dtype == CDG_DTYPE_E4M3) {
    if (!g->sa || g->sa_cols <= 0) return CDG_ERR_INVALID_ARGUMENT;
    if (g->sa_dtype == CDG_DTYPE_UE8M0_X4) {
      // one scale per 128-wide K block, four to a word
      if (g->sa_cols != ((g->K + 127) / 128 + 3) / 4) return CDG_ERR_INVALID_ARGUMENT;
    } else {
      // Same rule as the reference: sa_cols > 1 gives blocks of K / sa_cols;
      // a single column is one scale per row only when K fits one 128 block.
      if (g->sa_cols == 1 && g->K > 128) return CDG_ERR_UNSUPPORTED;
      if (g->sa_cols > 1 && (g->K % g->sa_cols)) return CDG_ERR_INVALID_ARGUMENT;
    }
  } else if (g->sa_dtype == CDG_DTYPE_UE8M0_X4) {
    return CDG_ERR_INVALID_ARGUMENT;  // packed scales belong to e4m3 activations
  }
  if (g->sfb_dtype != CDG_DTYPE_UE8M0 && g->sfb_dtype != CDG_DTYPE_F32) return CDG_ERR_INVALID_ARGUMENT;
  if (g->sfb_layout != CDG_SF_ROW_MAJOR && g->sfb_layout != CDG_SF_ATOMS) return CDG_ERR_INVALID_ARGUMENT;
  if (g->sfb_layout == CDG_SF_ATOMS && (g->sfb_dtype != CDG_DTYPE_UE8M0 || g->K % 128 || g->N % 128))
    return CDG_ERR_INVALID_ARGUMENT;
  if (g->d_dtype != CDG_DTYPE_BF16 && g->d_dtype != CDG_DTYPE_F32) return CDG_ERR_INVALID_ARGUMENT;
  if (g->a_row_stride < g->K || g->d_row_stride < g->N) return CDG_ERR_INVALID_ARGUMENT;
  if (g->b_stride_n < g->K / 2 || g->b_stride_e < g->b_stride_n * g->N) return CDG_ERR_INVALID_ARGUMENT;
  switch (g->index_form) {
    case CDG_INDEX_NONE:
      if (g->E != 1) return CDG_ERR_INVALID_ARGUMENT;
      break;
    case CDG_INDEX_PER_ROW:
      if (!g->m_indices && g->M > 0) return CDG_ERR_INVALID_ARGUMENT;
      if (g->m_indices_len != g->M) return CDG_ERR_INVALID_ARGUMENT;
      break;
    case CDG_INDEX_PSUM:
    case CDG_INDEX_MASKED:
      if (!g->m_indices || g->m_indices_len != g->E) return CDG_ERR_INVALID_ARGUMENT;
      break;
    default:
      return CDG_ERR_INVALID_ARGUMENT;
  }
  if (g->index_form != CDG_INDEX_NONE && g->m_indices_dtype != CDG_DTYPE_I32 && g->m_indices_dtype != CDG_DTYPE_I64)
    return CDG_ERR_INVALID_ARGUMENT;
  return CDG_OK;
}

// True when the tensor-core kernel can run these (validated) arguments.
bool fast_path(const cdg_gemm_args* g) {
  if (g->flags & CDG_FLAG_FORCE_GENERIC) return false;
  // float weight scales go through the tensor cores as UE8M0 codes: exactly when they are powers of
  // two (decided on the device; otherwise the exact SIMT kernel takes every block), or rounded
  // with CDG_FLAG_ROUND_SFB
  const bool sfb_ok = g->sfb_dtype == CDG_DTYPE_UE8M0 || (g->sfb_dtype == CDG_DTYPE_F32 &&
                                                          g->sfb_layout == CDG_SF_ROW_MAJOR);
  const bool planes = g->a_dtype == CDG_DTYPE_E4M3_PLANES;
  if ((g->a_dtype != CDG_DTYPE_E4M3 && !planes) || !sfb_ok || g->d_dtype != CDG_DTYPE_BF16) return false;
  const bool packed = g->sa_dtype == CDG_DTYPE_UE8M0_X4;
  if (g->K % 128 || g->N % 128 || (!planes && !packed && g->sa_cols != g->K / 128)) return false;
  if (g->a_row_stride % 16 || !aligned(g->a, 16)) return false;
  if (g->b_stride_n != g->K / 2 || g->b_stride_e != g->b_stride_n * g->N || !aligned(g->b, 32)) return false;
  if (g->d_row_stride % 8 || !aligned(g->d, 16)) return false;
  if (g->sfb_layout == CDG_SF_ATOMS && !aligned(g->sfb, 16)) return false;
  return true;
}

bool sfw_needs_transform(const cdg_gemm_args* g) { return g->sfb_layout == CDG_SF_ROW_MAJOR; }

TileMap tile_map(const cdg_gemm_args* g) {
  return g->index_form == CDG_INDEX_MASKED ? TileMap::masked(static_cast<int>(g->M), static_cast<int>(g->E))
                                           : TileMap::contiguous(static_cast<int>(g->M));
}

WorkspaceLayout layout_for(const cdg_gemm_args* g) {
  const bool fast = fast_path(g);
  return WorkspaceLayout::make(g->M, tile_map(g).tiles(), g->K, g->N, g->E, fast,
                               g->index_form == CDG_INDEX_PSUM || g->index_form == CDG_INDEX_MASKED,
                               fast && sfw_needs_transform(g), g->a_dtype == CDG_DTYPE_E4M3_PLANES);
}

int launch_sf_atoms_f32(const float* sf, int64_t se, int64_t sn, int64_t E, int64_t N, int64_t KB, uint32_t* out,
                        int* inexact, cudaStream_t stream, int sm_count) {
  const int64_t words = E * ((N + 127) / 128) * ((KB + 3) / 4) * 128;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((words + threads - 1) / threads, int64_t(sm_count) * 32);
  if (blocks <= 0) return CDG_OK;
  cdg_sf_atom_f32_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      sf, se, sn, out, static_cast<int>(E), static_cast<int>(N), static_cast<int>(KB), inexact);
  return cudaGetLastError() == cudaSuccess ? CDG_OK : CDG_ERR_CUDA;
}

int launch_sf_atoms(const uint8_t* sf, int64_t se, int64_t sn, int64_t E, int64_t N, int64_t KB, uint32_t* out,
                    cudaStream_t stream, int sm_count) {
  const int64_t words = E * ((N + 127) / 128) * ((KB + 3) / 4) * 128;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((words + threads - 1) / threads, int64_t(sm_count) * 32);
  if (blocks <= 0) return CDG_OK;
  cdg_sf_atom_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(sf, se, sn, out, static_cast<int>(E),
                                                                           static_cast<int>(N), static_cast<int>(KB));
  return cudaGetLastError() == cudaSuccess ? CDG_OK : CDG_ERR_CUDA;
}

// Activation planes: 3-D view [2 planes][nblk*128 rows][K] e4m3 bytes; one box brings
// `tok` rows of `planes` planes, landing as [hi tok rows][lo tok rows] in shared memory.
int make_plane_tmap(EncodeTiledFn enc, const cdg_gemm_args* g, uint8_t* hilo, int64_t nblk, uint32_t tok,
                    CUtensorMap* ta, uint32_t planes = 2) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(g->K), static_cast<cuuint64_t>(nblk * 128), 2};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(g->K), static_cast<cuuint64_t>(nblk * 128 * g->K)};
  cuuint32_t box[3] = {128, tok, planes};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, hilo, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? CDG_OK
             : CDG_ERR_CUDA;
}

int make_tmaps(const cdg_gemm_args* g, uint8_t* hilo, int64_t nblk, CUtensorMap* tw, CUtensorMap* ta16,
               CUtensorMap* ta32, CUtensorMap* ta128) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return CDG_ERR_CUDA;
  {
    // Weights: [E*N rows, K] packed E2M1, unpacked into one byte per element in shared memory.
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(g->K), static_cast<cuuint64_t>(g->E * g->N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(g->K / 2)};
    cuuint32_t box[2] = {128, 128};
    cuuint32_t estr[2] = {1, 1};
    if (enc(tw, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void*>(g->b), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return CDG_ERR_CUDA;
  }
  int st = make_plane_tmap(enc, g, hilo, nblk, 16, ta16);
  if (st == CDG_OK) st = make_plane_tmap(enc, g, hilo, nblk, 32, ta32);
  if (st == CDG_OK) st = make_plane_tmap(enc, g, hilo, nblk, 128, ta128);
  return st;
}

// Tensor maps of the CTA-pair kernels: one plane of TOK rows per CTA (tiny, narrow), and
// the weight scale atoms as a 2-D array [atoms][128 words] read one 512-byte atom per box.
int make_pair_tmaps(const cdg_gemm_args* g, uint8_t* hilo, int64_t nblk, const uint32_t* sfw, CUtensorMap* p16,
                    CUtensorMap* p32, CUtensorMap* tsf) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return CDG_ERR_CUDA;
  int st = make_plane_tmap(enc, g, hilo, nblk, 16, p16, 1);
  if (st == CDG_OK) st = make_plane_tmap(enc, g, hilo, nblk, 32, p32, 1);
  if (st != CDG_OK) return st;
  const int64_t atoms = g->E * (g->N / 128) * (g->K / 128);
  cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(atoms)};
  cuuint64_t strides[1] = {512};
  cuuint32_t box[2] = {128, 1};
  cuuint32_t estr[2] = {1, 1};
  return enc(tsf, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(sfw), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? CDG_OK
             : CDG_ERR_CUDA;
}

// Tensor maps of cdg_gemm_planes_kernel: a 4-D view (K, token % 8, plane, token / 8) of the
// stacked planes [2][nblk*128][K], so that a box of g token groups (one map per g = 1..7, the
// groups of a CTA's half tile) lands in shared memory as [group][plane][8 rows] -- 8 hi rows,
// then the same tokens' 8 lo rows, per group.
int make_planes_tmap(const cdg_gemm_args* g, uint8_t* hilo, int64_t nblk, PlaneMaps* maps) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return CDG_ERR_CUDA;
  const cuuint64_t K = static_cast<cuuint64_t>(g->K);
  cuuint64_t dims[4] = {K, 8, 2, static_cast<cuuint64_t>(nblk * 16)};
  cuuint64_t strides[3] = {K, static_cast<cuuint64_t>(nblk * 128) * K, 8 * K};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  for (int gi = 0; gi < kPlanesTileTok / 16; ++gi) {
    cuuint32_t box[4] = {128, 8, 2, static_cast<cuuint32_t>(gi + 1)};
    if (enc(&maps->m[gi], CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, hilo, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return CDG_ERR_CUDA;
  }
  return CDG_OK;
}

// Tensor maps of cdg_gemm_direct_kernel: A itself ([M rows][K] e4m3), a box of 8g rows per
// map (g = 1..14, the rows of a CTA's half tile), and the token scale atoms
// ([tiles * K/512 * 2][128 words], two 512-byte atoms per box).
int make_direct_tmaps(const cdg_gemm_args* g, uint32_t* tok_atoms, int64_t nblk, DirectMaps* maps,
                      CUtensorMap* tsf) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return CDG_ERR_CUDA;
  {
    cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(nblk * (tok_code_pitch(static_cast<int>(g->K)) / 4) * 2)};
    cuuint64_t strides[1] = {512};
    cuuint32_t box[2] = {128, 2};
    cuuint32_t estr[2] = {1, 1};
    if (enc(tsf, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, tok_atoms, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return CDG_ERR_CUDA;
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(g->K), static_cast<cuuint64_t>(g->M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(g->a_row_stride)};
  cuuint32_t estr[2] = {1, 1};
  for (int gi = 0; gi < kDirectTileTok / 16; ++gi) {
    cuuint32_t box[2] = {128, static_cast<cuuint32_t>(8 * (gi + 1))};
    if (enc(&maps->m[gi], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(g->a), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return CDG_ERR_CUDA;
  }
  return CDG_OK;
}

// Launch with programmatic stream serialization: the kernel may be scheduled while
// the previous kernel of the stream drains and waits for it on the device
// (griddepcontrol.wait), which hides the launch gap between the GEMM's kernels.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl.load(std::memory_order_relaxed) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int run(const cdg_gemm_args* g, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  int st = validate(g);
  if (st != CDG_OK) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CDG_ERR_CUDA;
  const DeviceInfo& di = device_info(dev);
  if (!di.ok) return CDG_ERR_CUDA;
  if (di.cc_major != 10) return CDG_ERR_NO_SM100;
  if (g->M == 0) return CDG_OK;

  const WorkspaceLayout wl = layout_for(g);
  if (!workspace || workspace_bytes < wl.total) return CDG_ERR_WORKSPACE;
  if (!aligned(workspace, 1024)) return CDG_ERR_ALIGNMENT;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* ctrl = reinterpret_cast<int*>(ws + wl.ctrl);
  if (cudaMemsetAsync(ctrl, 0, kCtrlWords * 4, stream) != cudaSuccess) return CDG_ERR_CUDA;

  const TileMap tm = tile_map(g);
  const int64_t nblk = tm.tiles();
  const void* ids = g->index_form == CDG_INDEX_NONE ? nullptr : g->m_indices;
  int ids_dtype = g->m_indices_dtype;
  if (g->index_form == CDG_INDEX_PSUM || g->index_form == CDG_INDEX_MASKED) {
    int32_t* rows = reinterpret_cast<int32_t*>(ws + wl.row_ids);
    const unsigned blocks = static_cast<unsigned>((g->M + 255) / 256);
    const int G = static_cast<int>(g->E), M = static_cast<int>(g->M);
    if (g->index_form == CDG_INDEX_MASKED) {
      if (ids_dtype == CDG_DTYPE_I64)
        cdg_masked_rows_kernel<int64_t><<<blocks, 256, 0, stream>>>(static_cast<const int64_t*>(ids), G,
                                                                     tm.seg_rows, M, rows);
      else
        cdg_masked_rows_kernel<int32_t><<<blocks, 256, 0, stream>>>(static_cast<const int32_t*>(ids), G,
                                                                     tm.seg_rows, M, rows);
    } else if (ids_dtype == CDG_DTYPE_I64) {
      cdg_psum_rows_kernel<int64_t><<<blocks, 256, 0, stream>>>(static_cast<const int64_t*>(ids), G, M, rows);
    } else {
      cdg_psum_rows_kernel<int32_t><<<blocks, 256, 0, stream>>>(static_cast<const int32_t*>(ids), G, M, rows);
    }
    ids = rows;
    ids_dtype = CDG_DTYPE_I32;
  }
  int4* lists = reinterpret_cast<int4*>(ws + wl.lists);
  int4* blk_info = reinterpret_cast<int4*>(ws + wl.blk_info);
  uint4* blk_mask = reinterpret_cast<uint4*>(ws + wl.blk_mask);

  GenericArgs ga{};
  ga.a = g->a;
  ga.a_dtype = g->a_dtype;
  ga.a_row_stride = g->a_row_stride;
  ga.sa = g->sa;
  ga.sa_stride_m = g->sa_stride_m;
  ga.sa_stride_k = g->sa_stride_k;
  ga.sa_packed = g->sa_dtype == CDG_DTYPE_UE8M0_X4;
  ga.sa_block_k = g->a_dtype == CDG_DTYPE_E4M3 && !ga.sa_packed
                      ? (g->sa_cols > 1 ? static_cast<int>(g->K / g->sa_cols) : 128)
                      : 128;
  ga.b = static_cast<const uint8_t*>(g->b);
  ga.b_stride_e = g->b_stride_e;
  ga.b_stride_n = g->b_stride_n;
  ga.sb = g->sfb;
  ga.sb_dtype = g->sfb_dtype;
  ga.sb_atoms = g->sfb_layout == CDG_SF_ATOMS;
  ga.sb_stride_e = g->sfb_stride_e;
  ga.sb_stride_n = g->sfb_stride_n;
  ga.d = g->d;
  ga.d_dtype = g->d_dtype;
  ga.d_row_stride = g->d_row_stride;
  ga.d_rows = g->d_rows;
  ga.M = static_cast<int>(g->M);
  ga.N = static_cast<int>(g->N);
  ga.K = static_cast<int>(g->K);
  ga.E = static_cast<int>(g->E);
  ga.nblk = static_cast<int>(nblk);
  ga.tm = tm;
  const size_t generic_smem = static_cast<size_t>(g->K) * 4;
  if (generic_smem > 200 * 1024) return CDG_ERR_UNSUPPORTED;
  const int64_t generic_units = nblk * ((g->N + 255) / 256);

  const bool planes_in = g->a_dtype == CDG_DTYPE_E4M3_PLANES;
  if (planes_in && !fast_path(g)) return CDG_ERR_UNSUPPORTED;  // planes run on the tensor cores only
  if (!fast_path(g)) {
    ga.ids = ids;
    ga.ids_is_64 = ids_dtype == CDG_DTYPE_I64;
    ga.list = nullptr;
    ga.count = nullptr;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(generic_units, int64_t(usable_sms(di)) * 8));
    cdg_generic_kernel<<<grid, 256, generic_smem, stream>>>(ga);
    return cudaGetLastError() == cudaSuccess ? CDG_OK : CDG_ERR_CUDA;
  }

  // ---------------------------------------------------------------- tensor-core path
  const uint32_t* sfw = static_cast<const uint32_t*>(g->sfb);
  const bool float_sfb = g->sfb_dtype == CDG_DTYPE_F32;
  if (sfw_needs_transform(g)) {
    uint32_t* out = reinterpret_cast<uint32_t*>(ws + wl.sfw_atoms);
    if (float_sfb)
      st = launch_sf_atoms_f32(static_cast<const float*>(g->sfb), g->sfb_stride_e, g->sfb_stride_n, g->E, g->N,
                               g->K / 32, out, ctrl + kCtrlSfInexact, stream, di.sm_count);
    else
      st = launch_sf_atoms(static_cast<const uint8_t*>(g->sfb), g->sfb_stride_e, g->sfb_stride_n, g->E, g->N,
                           g->K / 32, out, stream, di.sm_count);
    if (st != CDG_OK) return st;
    sfw = out;
  }
  uint8_t* hilo = planes_in ? static_cast<uint8_t*>(const_cast<void*>(g->a)) : ws + wl.hilo;
  int32_t* row_exp = planes_in ? reinterpret_cast<int32_t*>(const_cast<float*>(g->sa))
                               : reinterpret_cast<int32_t*>(ws + wl.row_exp);

  PrepArgs pa{};
  pa.a = static_cast<const uint8_t*>(g->a);
  pa.a_row_stride = g->a_row_stride;
  pa.sa = g->sa;
  pa.sa_stride_m = g->sa_stride_m;
  pa.sa_stride_k = g->sa_stride_k;
  pa.sa_packed = g->sa_dtype == CDG_DTYPE_UE8M0_X4;
  pa.ids = ids;
  pa.M = static_cast<int>(g->M);
  pa.K = static_cast<int>(g->K);
  pa.E = static_cast<int>(g->E);
  pa.nblk = static_cast<int>(nblk);
  pa.tm = tm;
  pa.hilo = hilo;
  pa.row_exp = row_exp;
  pa.blk_info = blk_info;
  pa.blk_mask = blk_mask;
  pa.ctrl = ctrl;
  pa.lists = lists;
  pa.plane_tiles = reinterpret_cast<int4*>(ws + wl.plane_tiles);
  const int sms = usable_sms(di);
  const bool pair_path = g->N % 256 == 0 && !(g->flags & CDG_FLAG_SINGLE_CTA) && sms >= 2;
  uint8_t* tok_code = ws + wl.tok_code;
  pa.tok_code = tok_code;
  pa.direct_tiles = reinterpret_cast<int4*>(ws + wl.direct_tiles);
  pa.pair_wide = pair_path ? 1 : 0;
  pa.sf_inexact = float_sfb && !(g->flags & CDG_FLAG_ROUND_SFB) ? ctrl + kCtrlSfInexact : nullptr;
  pa.planes_given = planes_in ? 1 : 0;
  const dim3 prep_grid(static_cast<unsigned>(nblk),
                       planes_in ? 1u : static_cast<unsigned>((g->K + kPrepK - 1) / kPrepK));
  if (ids_dtype == CDG_DTYPE_I64)
    cdg_prep_kernel<int64_t><<<prep_grid, 256, 0, stream>>>(pa);
  else
    cdg_prep_kernel<int32_t><<<prep_grid, 256, 0, stream>>>(pa);
  if (cudaGetLastError() != cudaSuccess) return CDG_ERR_CUDA;

  CUtensorMap tw, ta16, ta32, ta128;
  st = make_tmaps(g, hilo, nblk, &tw, &ta16, &ta32, &ta128);
  if (st != CDG_OK) return st;

  GemmArgs ka{};
  ka.blk_info = blk_info;
  ka.blk_mask = blk_mask;
  ka.ctrl = ctrl;
  ka.sfw_atoms = sfw;
  ka.row_exp = row_exp;
  ka.tok_code = tok_code;
  ka.tok_atoms = reinterpret_cast<uint32_t*>(ws + wl.tok_atoms);
  ka.d = static_cast<__nv_bfloat16*>(g->d);
  ka.d_row_stride = g->d_row_stride;
  ka.d_rows = g->d_rows;
  ka.M = static_cast<int>(g->M);
  ka.N = static_cast<int>(g->N);
  ka.K = static_cast<int>(g->K);
  ka.E = static_cast<int>(g->E);
  ka.nblk = static_cast<int>(nblk);
  ka.tm = tm;
  ka.status = ctrl + kCtrlStatus;
  ka.zero_list = lists + kClassZero * nblk;
  const bool skip_ungrouped = (g->flags & CDG_FLAG_SKIP_UNGROUPED) != 0;
  ka.fill_rest = skip_ungrouped ? 0 : 1;

  if (t_prof_start && cudaEventRecord(t_prof_start, stream) != cudaSuccess) return CDG_ERR_CUDA;
  if (pair_path) {
    // CTA pairs (tcgen05 cta_group::2): two adjacent 128-column tiles per cluster; four MMA
    // issuers for tiny blocks, two for narrow; wide blocks in token tiles of the plane kernel
    // (cdg_gemm_planes_kernel), or, when their scales are powers of two, in
    // token tiles of cdg_gemm_direct_kernel on the raw rows (direct class).
    CUtensorMap p16, p32, tsf;
    st = make_pair_tmaps(g, hilo, nblk, sfw, &p16, &p32, &tsf);
    if (st != CDG_OK) return st;
    const unsigned grid = static_cast<unsigned>(sms / 2 * 2);
    // the planes kernel also writes the direct tiles' token scale atoms
    ka.direct_list = reinterpret_cast<const int4*>(ws + wl.direct_tiles);
    ka.list = lists + kClassTiny * nblk;
    ka.count_slot = kCtrlCount0 + kClassTiny;
    ka.do_zero_blocks = skip_ungrouped ? 0 : 1;
    if (launch_pdl(cdg_gemm_pair_kernel<16, 4>, grid, PairSmem<16, 4>::kThreads, PairSmem<16, 4>::kBytes, stream, tw,
                   p16, tsf, ka) != cudaSuccess)
      return CDG_ERR_CUDA;
    ka.do_zero_blocks = 0;
    ka.list = lists + kClassNarrow * nblk;
    ka.count_slot = kCtrlCount0 + kClassNarrow;
    if (launch_pdl(cdg_gemm_pair_kernel<32, 2>, grid, PairSmem<32, 2>::kThreads, PairSmem<32, 2>::kBytes, stream, tw,
                   p32, tsf, ka) != cudaSuccess)
      return CDG_ERR_CUDA;
    PlaneMaps planes;
    st = make_planes_tmap(g, hilo, nblk, &planes);
    if (st != CDG_OK) return st;
    ka.list = reinterpret_cast<const int4*>(ws + wl.plane_tiles);
    ka.count_slot = kCtrlPlaneTiles;
    if (launch_pdl(cdg_gemm_planes_kernel, grid, PlanesSmem::kThreads, PlanesSmem::kBytes, stream, tw, planes, tsf,
                   ka) != cudaSuccess)
      return CDG_ERR_CUDA;
    // Wide blocks whose activation scales are all powers of two: raw e4m3 rows.
    DirectMaps direct;
    CUtensorMap dtsf;
    st = make_direct_tmaps(g, ka.tok_atoms, nblk, &direct, &dtsf);
    if (st != CDG_OK) return st;
    ka.list = reinterpret_cast<const int4*>(ws + wl.direct_tiles);
    ka.count_slot = kCtrlDirectTiles;
    if (launch_pdl(cdg_gemm_direct_kernel, grid, DirectSmem::kThreads, DirectSmem::kBytes, stream, tw, direct, tsf,
                   dtsf, ka) != cudaSuccess)
      return CDG_ERR_CUDA;
  } else {
    // Tiny blocks (decode: at most 16 routed rows) and all-padding blocks.
    ka.list = lists + kClassTiny * nblk;
    ka.count_slot = kCtrlCount0 + kClassTiny;
    ka.do_zero_blocks = skip_ungrouped ? 0 : 1;
    if (launch_pdl(cdg_gemm_kernel<16>, sms, 256, GemmSmem<16>::kBytes, stream, tw, ta16, ka) != cudaSuccess)
      return CDG_ERR_CUDA;
    // Narrow blocks (17 to 32 routed rows).
    ka.do_zero_blocks = 0;
    ka.list = lists + kClassNarrow * nblk;
    ka.count_slot = kCtrlCount0 + kClassNarrow;
    if (launch_pdl(cdg_gemm_kernel<32>, sms, 256, GemmSmem<32>::kBytes, stream, tw, ta32, ka) != cudaSuccess)
      return CDG_ERR_CUDA;
    // Wide blocks (prefill-like).
    ka.list = lists + kClassWide * nblk;
    ka.count_slot = kCtrlCount0 + kClassWide;
    if (launch_pdl(cdg_gemm_kernel<128>, sms, 256, GemmSmem<128>::kBytes, stream, tw, ta128, ka) != cudaSuccess)
      return CDG_ERR_CUDA;
  }
  if (t_prof_stop && cudaEventRecord(t_prof_stop, stream) != cudaSuccess) return CDG_ERR_CUDA;
  // Blocks holding rows of several experts: exact SIMT path over the listed blocks.
  ga.ids = ids;
  ga.ids_is_64 = ids_dtype == CDG_DTYPE_I64;
  ga.list = lists + kClassIrregular * nblk;
  ga.count = ctrl + kCtrlCount0 + kClassIrregular;
  {
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(generic_units, int64_t(sms)));
    if (launch_pdl(cdg_generic_kernel, grid, 256, generic_smem, stream, ga) != cudaSuccess) return CDG_ERR_CUDA;
  }
  return CDG_OK;
}

}  // namespace
}  // namespace cdg

extern "C" {

int cdg_grouped_fp8_fp4_gemm_nt_contiguous(const cdg_gemm_args* args, void* workspace, size_t workspace_bytes,
                                           cdg_stream_t stream) {
  return cdg::run(args, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int cdg_grouped_fp8_fp4_gemm_nt_masked(const cdg_gemm_args* args, void* workspace, size_t workspace_bytes,
                                       cdg_stream_t stream) {
  if (!args || (args->index_form != CDG_INDEX_MASKED && args->index_form != CDG_INDEX_NONE))
    return CDG_ERR_INVALID_ARGUMENT;
  return cdg::run(args, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t cdg_grouped_fp8_fp4_workspace_bytes(const cdg_gemm_args* args) {
  if (cdg::validate(args) != CDG_OK) return 0;
  return cdg::layout_for(args).total;
}

int cdg_can_implement(const cdg_gemm_args* args) {
  if (cdg::validate(args) != CDG_OK) return -1;
  return cdg::fast_path(args) ? 1 : 0;
}

int cdg_transform_sf(const uint8_t* sf, int64_t stride_e, int64_t stride_n, int64_t E, int64_t N, int64_t KB,
                     uint8_t* out, cdg_stream_t stream) {
  if (!sf || !out || E <= 0 || N <= 0 || KB <= 0 || stride_n < KB || stride_e < stride_n * N)
    return CDG_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(out) % 4) return CDG_ERR_ALIGNMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= cdg::kMaxDevices) return CDG_ERR_CUDA;
  const cdg::DeviceInfo& di = cdg::device_info(dev);
  if (!di.ok) return CDG_ERR_CUDA;
  return cdg::launch_sf_atoms(sf, stride_e, stride_n, E, N, KB, reinterpret_cast<uint32_t*>(out),
                              reinterpret_cast<cudaStream_t>(stream), di.sm_count);
}

size_t cdg_sf_atoms_bytes(int64_t E, int64_t N, int64_t KB) {
  if (E <= 0 || N <= 0 || KB <= 0) return 0;
  return static_cast<size_t>(E) * ((N + 127) / 128) * ((KB + 3) / 4) * 512;
}

int cdg_read_device_status(const void* workspace, cdg_stream_t stream) {
  if (!workspace) return CDG_ERR_INVALID_ARGUMENT;
  int word = 0;
  const int* src = static_cast<const int*>(workspace) + cdg::kCtrlStatus;
  if (cudaMemcpyAsync(&word, src, sizeof(int), cudaMemcpyDeviceToHost, reinterpret_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return CDG_ERR_CUDA;
  if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return CDG_ERR_CUDA;
  return (word & cdg::kStatusTimeout) ? CDG_ERR_DEVICE_TIMEOUT : word ? CDG_ERR_DEVICE_INDEX : CDG_OK;
}

}  // extern "C"

namespace cdg {
int ep_sticky_status(int clear, int32_t* out);  // cdg_moe.cu: the exchange kernels' record
}  // namespace cdg

extern "C" {

int cdg_device_status(int32_t clear, int32_t* where) {
  int32_t gemm[2] = {0, 0}, ep[2] = {0, 0};
  if (cudaDeviceSynchronize() != cudaSuccess) return CDG_ERR_CUDA;
  if (cudaMemcpyFromSymbol(gemm, cdg::g_sticky_status, sizeof(gemm)) != cudaSuccess) return CDG_ERR_CUDA;
  if (clear) {
    const int32_t z[2] = {0, 0};
    if (cudaMemcpyToSymbol(cdg::g_sticky_status, z, sizeof(z)) != cudaSuccess) return CDG_ERR_CUDA;
  }
  const int st = cdg::ep_sticky_status(clear, ep);
  if (st != CDG_OK) return st;
  if (where) *where = gemm[1] ? gemm[1] : ep[1];
  const int bits = gemm[0] | ep[0];
  return (bits & cdg::kStatusTimeout) ? CDG_ERR_DEVICE_TIMEOUT : bits ? CDG_ERR_DEVICE_INDEX : CDG_OK;
}

int cdg_set_num_sms(int32_t num_sms) {
  if (num_sms < 0) return CDG_ERR_INVALID_ARGUMENT;
  cdg::g_num_sms.store(num_sms, std::memory_order_relaxed);
  return CDG_OK;
}

int cdg_set_pdl(int32_t enable) {
  cdg::g_pdl.store(enable ? 1 : 0, std::memory_order_relaxed);
  return CDG_OK;
}

int cdg_get_pdl(void) { return cdg::g_pdl.load(std::memory_order_relaxed); }

int cdg_get_num_sms(void) {
  const int n = cdg::g_num_sms.load(std::memory_order_relaxed);
  if (n > 0) return n;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                 cudaSuccess)
    return 0;
  return sms;
}

const char* cdg_build_info(void) {
  return "consumer-deepgemm-b200; arch=sm_100a; abi=1; kernels=tcgen05.mma.kind::mxf8f6f4.block_scale "
         "(TMA 16U4_ALIGN16B weights, e4m3 hi/lo activation planes), exact SIMT fallback";
}

int cdg_mk_alignment_for_contiguous_layout(void) { return 128; }

int cdg_set_profile_events(void* start_event, void* stop_event) {
  if ((start_event == nullptr) != (stop_event == nullptr)) return CDG_ERR_INVALID_ARGUMENT;
  cdg::t_prof_start = static_cast<cudaEvent_t>(start_event);
  cdg::t_prof_stop = static_cast<cudaEvent_t>(stop_event);
  return CDG_OK;
}

const char* cdg_status_string(int status) {
  switch (status) {
    case CDG_OK: return "ok";
    case CDG_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CDG_ERR_UNSUPPORTED: return "unsupported";
    case CDG_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case CDG_ERR_WORKSPACE: return "workspace missing or too small";
    case CDG_ERR_CUDA: return "CUDA runtime error";
    case CDG_ERR_DEVICE_TIMEOUT: return "device pipeline wait timed out";
    case CDG_ERR_NO_SM100: return "device is not compute capability 10.x (B200)";
    case CDG_ERR_SCRATCH_TOO_SMALL:
      return "problem needs more workspace than the 64 MiB static scratch of the no-allocation entry point";
    case CDG_ERR_DEVICE_INDEX: return "a kernel skipped an access outside its buffer or misaligned";
    default: return "unknown status";
  }
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// No-allocation entry point: the workspace is a file-scope device array instead of caller memory.
// ---------------------------------------------------------------------------------------------
namespace cdg {
namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[CDG_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on each device, looked up once with that device current.
// In host code the array's name only stands in for the symbol; kernels need this address.
struct NoallocScratch {
  uint8_t* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};

const NoallocScratch& noalloc_scratch(int dev) {
  static NoallocScratch slots[kMaxDevices];
  static std::once_flag flags[kMaxDevices];
  std::call_once(flags[dev], [dev] {
    void* p = nullptr;
    slots[dev].err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    slots[dev].ptr = static_cast<uint8_t*>(p);
    // a failed lookup is reported by every call through slots[dev].err; it must not stay
    // behind as the thread's last error, where the launch checks that follow would see it
    if (slots[dev].err != cudaSuccess) (void)cudaGetLastError();
  });
  return slots[dev];
}

}  // namespace
}  // namespace cdg

extern "C" int cdg_grouped_fp8_fp4_gemm_nt_contiguous_noalloc(const cdg_gemm_args* args, cdg_stream_t stream) {
  const int st = cdg::validate(args);
  if (st != CDG_OK) return st;
  // The shared workspace layout wants 1024-byte alignment; the array is 256-aligned.
  const size_t need = cdg::layout_for(args).total + 1024;
  if (need > CDG_NOALLOC_SCRATCH_BYTES) return CDG_ERR_SCRATCH_TOO_SMALL;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= cdg::kMaxDevices) return CDG_ERR_CUDA;
  // A device that is not a B200 is reported as such before the scratch is looked up there.
  const cdg::DeviceInfo& di = cdg::device_info(dev);
  if (!di.ok) return CDG_ERR_CUDA;
  if (di.cc_major != 10) return CDG_ERR_NO_SM100;
  const cdg::NoallocScratch& sc = cdg::noalloc_scratch(dev);
  if (sc.err != cudaSuccess || sc.ptr == nullptr) return CDG_ERR_CUDA;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(sc.ptr) + 1023) & ~uintptr_t(1023);
  const size_t usable = CDG_NOALLOC_SCRATCH_BYTES - (base - reinterpret_cast<uintptr_t>(sc.ptr));
  return cdg::run(args, reinterpret_cast<void*>(base), usable, reinterpret_cast<cudaStream_t>(stream));
}
