/*
 * cdg_b200.h -- C ABI of the B200 (sm_100a) grouped FP8 x MXFP4 MoE GEMM.
 *
 * One library, libcdg_b200.so, with plain pointers, sizes and a CUDA stream in
 * every signature (no torch types), so that any FFI (ctypes, cgo, JNI, a C++
 * host) can drive it.  The Python package consumer_deep_gemm binds it through
 * its torch extension; tests bind it through ctypes.
 *
 * Each entry point names the reference interface (lmxxf/Consumer-DeepGEMM) it
 * replaces.
 *
 * Conventions
 *   - All device pointers belong to the caller; nothing here allocates device
 *     memory.  Temporaries live in a caller-provided workspace whose size is
 *     given by cdg_grouped_fp8_fp4_workspace_bytes().
 *   - Work is enqueued on `stream` and nothing blocks the host; no device to host
 *     copy happens on the GEMM path.
 *   - Return values are cdg_status codes.  Input errors are detected on the host
 *     before anything is launched.  Errors seen on the device (a pipeline wait
 *     that timed out) are recorded in the workspace status word, readable with
 *     cdg_read_device_status(), and in a per-device record of the library,
 *     readable with cdg_device_status().
 */
#ifndef CDG_B200_H_
#define CDG_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* cdg_stream_t; /* == cudaStream_t */

#define CDG_ABI_VERSION 2

typedef enum cdg_status {
  CDG_OK = 0,
  CDG_ERR_INVALID_ARGUMENT = 1, /* shapes, strides or dtypes that the operation cannot mean */
  CDG_ERR_UNSUPPORTED = 2,      /* a well-formed request this build does not implement */
  CDG_ERR_ALIGNMENT = 3,        /* a pointer or stride breaks an alignment rule */
  CDG_ERR_WORKSPACE = 4,        /* workspace missing or smaller than required */
  CDG_ERR_CUDA = 5,             /* a CUDA runtime call failed (see cudaGetLastError) */
  CDG_ERR_DEVICE_TIMEOUT = 6,   /* a kernel gave up waiting on its pipeline */
  CDG_ERR_NO_SM100 = 7,         /* the current device is not compute capability 10.x */
  CDG_ERR_SCRATCH_TOO_SMALL = 8, /* the problem needs more than the static scratch of the no-allocation entry */
  CDG_ERR_DEVICE_INDEX = 9       /* a kernel met an index or address it cannot use (outside its buffer, or a
                                    D row address that is not 16-byte aligned) and skipped that access */
} cdg_status;

typedef enum cdg_dtype {
  CDG_DTYPE_E4M3 = 1,   /* float8 e4m3fn */
  CDG_DTYPE_BF16 = 2,   /* bfloat16 */
  CDG_DTYPE_F32 = 3,    /* float32 */
  CDG_DTYPE_UE8M0 = 4,  /* unsigned 8-bit power-of-two scale, value 2^(b-127) */
  CDG_DTYPE_I32 = 5,    /* int32 group ids */
  CDG_DTYPE_I64 = 6,    /* int64 group ids */
  CDG_DTYPE_UE8M0_X4 = 7, /* int32 words of four UE8M0 activation scales: the scale of 128-wide K
                            block kb is byte kb % 4 of word kb / 4 (the packed format of DeepGEMM's
                            UE8M0 recipe, e.g. vLLM's silu_mul_quant_fp8_packed) */
  CDG_DTYPE_E4M3_PLANES = 8 /* activations given as the two e4m3 planes the tensor cores read: `a` is
                               uint8 [2][M][K] (hi plane, then lo plane; a_row_stride = K, M a multiple
                               of 128), `sa` is int32 [M] row exponents E (sa_dtype = CDG_DTYPE_I32),
                               and row r stands for (hi + lo) * 2^E, the reference's BF16 dequant of an
                               e4m3 row with FP32 1x128 scales as cdg_ep_* producers split it (see
                               cdg_ep_quant_dispatch_local).  Per-row m_indices with 128-aligned groups
                               only; a block with rows of several experts is left out and reported
                               (CDG_ERR_DEVICE_INDEX from cdg_device_status).  Used by the MoE
                               layer, whose own quantising steps write the planes, so the GEMM skips its
                               plane split */
} cdg_dtype;

/* How the weight scales `sfb` are laid out. */
typedef enum cdg_sf_layout {
  CDG_SF_ROW_MAJOR = 0, /* [E, N, K/32] with the given strides (bytes or floats) */
  CDG_SF_ATOMS = 1      /* output of cdg_transform_sf(): 512-byte 128x4 atoms, dense */
} cdg_sf_layout;

/* What `m_indices` holds. */
typedef enum cdg_index_form {
  CDG_INDEX_PER_ROW = 0, /* one group id per row of A, -1 (any id outside [0,E)) = no group */
  CDG_INDEX_PSUM = 1,    /* E cumulative row ends: group g owns rows [end[g-1], end[g]) */
  CDG_INDEX_NONE = 2,    /* no ids: E must be 1 and every row belongs to group 0 */
  CDG_INDEX_MASKED = 3   /* E per-group row counts (masked_m): with S = M / E, group g owns rows
                            [g*S, g*S + count[g]); a count above S runs on into the following rows,
                            later groups winning; every other row of D is written as 0 */
} cdg_index_form;

/*
 * Arguments of D[r, :] = deq(A[r, :]) . deq(B[g(r)])^T for every row r whose
 * group g(r) is in [0, E); every other row of D is written as 0.
 *
 *   a          [M, K] activations, a_dtype E4M3 (with sa) or BF16/F32 (sa ignored)
 *   sa         [M, sa_cols] float32 activation scales, one per row and K block of
 *              K / sa_cols elements (1x128 blocks: sa_cols = K/128)
 *   b          [E, N, K/2] packed E2M1 weights, low nibble = even k
 *   sfb        weight scales, UE8M0 bytes or float32, per 32 K (see sfb_layout)
 *   m_indices  group ids, int32 or int64 (see index_form)
 *   d          [M, N] output, BF16 or F32
 * Strides are in elements of the tensor's own dtype (bytes for b).
 */
typedef struct cdg_gemm_args {
  const void* a;
  int32_t a_dtype;
  int64_t a_row_stride;
  const float* sa;
  int64_t sa_stride_m, sa_stride_k;
  int32_t sa_cols;
  const void* b;
  int64_t b_stride_e, b_stride_n;
  const void* sfb;
  int32_t sfb_dtype;
  int32_t sfb_layout;
  int64_t sfb_stride_e, sfb_stride_n;
  const void* m_indices;
  int32_t m_indices_dtype;
  int32_t index_form;
  int64_t m_indices_len;
  void* d;
  int32_t d_dtype;
  int64_t d_row_stride;
  int64_t M, N, K, E;
  int32_t flags; /* CDG_FLAG_* */
  int32_t sa_dtype; /* scales of an e4m3 `a`: CDG_DTYPE_F32 (0 reads as F32) or CDG_DTYPE_UE8M0_X4, whose
                       sa_cols counts int32 words and whose strides are in words */
  const uint64_t* d_rows; /* optional (ABI 2), device memory: M row addresses; when set, row r of D is
                             stored at d_rows[r] instead of d + r * d_row_stride (BF16 only; `d` may
                             be NULL).  A zero address leaves the row unwritten; an address that is
                             not 16-byte aligned is not written and raises the bad-index status.  The
                             addresses may lie in another GPU's memory (peer or IPC mappings): the
                             kernels end with a system-scope fence when the table is set.  This is
                             how an expert-parallel layer returns FC2 rows straight into each
                             source rank's window */
} cdg_gemm_args;

#define CDG_FLAG_FORCE_GENERIC 1 /* run the exact SIMT path even where the tensor-core path applies */
#define CDG_FLAG_SINGLE_CTA 2    /* tensor-core path: one CTA per 128-column tile even where N % 256 == 0
                                    would allow CTA pairs (for comparisons; same results) */
#define CDG_FLAG_SKIP_UNGROUPED 4 /* rows of D outside every group may be left unwritten instead of
                                     zeroed (for callers that never read them, e.g. a layer's own padded
                                     buffers); the reference always zeroes them */
#define CDG_FLAG_ROUND_SFB 8       /* float32 weight scales: round each to the nearest power of two (the
                                     reference's native path, _float_scale_to_e8m0 in
                                     consumer_deep_gemm/gemm.py:62-73, used at :130-144) and run the
                                     tensor cores.  Without it, float32 weight scales run the tensor
                                     cores when every one is a power of two (exact) and the exact SIMT
                                     kernel otherwise, the reference's dequant fallback; the device
                                     decides, per call */

/* Grouped FP8 x MXFP4 GEMM, contiguous layout.
 * Replaces m_grouped_fp8_fp4_gemm_nt_contiguous (consumer_deep_gemm/gemm.py:467-470),
 * its native stub (csrc/bindings.cpp:103-129) and launcher
 * (csrc/cutlass_mxfp8_mxfp4_probe.cu:444-614, exported at :660-673). */
int cdg_grouped_fp8_fp4_gemm_nt_contiguous(const cdg_gemm_args* args, void* workspace, size_t workspace_bytes,
                                           cdg_stream_t stream);

/* Grouped FP8 x MXFP4 GEMM, masked layout: args->index_form is CDG_INDEX_MASKED with
 * m_indices = masked_m [E] (int32/int64, on the device; read by the kernels, no host
 * synchronisation), or CDG_INDEX_NONE for one group over all rows.  A and D are the
 * [E * S, K] / [E * S, N] row-major views of the [E, S, ...] tensors.  Blocks of 128
 * rows never cross a group's block of S rows.  Workspace as for the contiguous entry
 * (cdg_grouped_fp8_fp4_workspace_bytes with the same args).
 * Replaces m_grouped_fp8_fp4_gemm_nt_masked (consumer_deep_gemm/gemm.py:529-551). */
int cdg_grouped_fp8_fp4_gemm_nt_masked(const cdg_gemm_args* args, void* workspace, size_t workspace_bytes,
                                       cdg_stream_t stream);

/* Workspace the call above needs for these arguments (0 on invalid arguments).
 * Replaces the launcher's process-global workspace and segment buffers
 * (csrc/cutlass_mxfp8_mxfp4_probe.cu:391-438). */
size_t cdg_grouped_fp8_fp4_workspace_bytes(const cdg_gemm_args* args);

/* 1 if the tensor-core kernel takes these arguments, 0 if the exact SIMT path
 * will run them, -1 if they are invalid.  For float32 weight scales 1 means: the tensor cores
 * run them when all are powers of two (or with CDG_FLAG_ROUND_SFB), which the device decides
 * during the call; otherwise the exact SIMT kernel does.
 * Replaces cutlass_mxfp8_mxfp4_can_implement_probe (csrc/cutlass_mxfp8_mxfp4_probe.cu:158-188,633-639). */
int cdg_can_implement(const cdg_gemm_args* args);

/* Weight scale factors [E, N, KB] (KB = K/32, UE8M0 bytes, strides in bytes) ->
 * dense 512-byte atoms [E][ceil(N/128)][ceil(KB/4)][128 rows x 4], padding 127.
 * Run once at weight-load time; pass the result with CDG_SF_ATOMS.
 * Replaces transform_sf_into_required_layout (consumer_deep_gemm/layout.py:6-19),
 * reorder_scale_kernel (csrc/cutlass_mxfp8_mxfp4_probe.cu:258-295) and the
 * lazily filled per-expert cache (:340-385). */
int cdg_transform_sf(const uint8_t* sf, int64_t stride_e, int64_t stride_n, int64_t E, int64_t N, int64_t KB,
                     uint8_t* out, cdg_stream_t stream);

/* Bytes cdg_transform_sf() writes.
 * Replaces cutlass_mxfp8_mxfp4_scale_layout_sizes (csrc/cutlass_mxfp8_mxfp4_probe.cu:641-657). */
size_t cdg_sf_atoms_bytes(int64_t E, int64_t N, int64_t KB);

/* Reads (synchronising `stream`) the device status word a GEMM call left in its
 * workspace; returns CDG_OK, CDG_ERR_DEVICE_TIMEOUT or CDG_ERR_DEVICE_INDEX (as
 * cdg_device_status).  No reference counterpart:
 * the reference reports device failures only as a launch result
 * (csrc/cutlass_mxfp8_mxfp4_probe.cu:598-613). */
int cdg_read_device_status(const void* workspace, cdg_stream_t stream);

/* Device-side errors of every call on the current device since the last clear, whatever
 * workspace (or exchange window) the call used: after synchronising the device, returns
 * CDG_OK, CDG_ERR_DEVICE_TIMEOUT (a bounded wait gave up: an mbarrier wait of a GEMM
 * kernel, or a wait on another rank's flag in the peer-memory exchange) or, when no wait
 * gave up, CDG_ERR_DEVICE_INDEX (a kernel skipped an access it could not make: a block the
 * planes form cannot run, exchange rows that do not match their header, a misaligned D row
 * address), stores the first recorded code in *where (may be NULL; 0 when none), and clears
 * the record when `clear` is nonzero.  A wait code holds the role (bits 28-31: 1 producer/empty, 2 issuer/tempty,
 * 3 issuer/full, 4 epilogue/tfull, 5 issuer/done, 6 scale copier, 7 scale producer,
 * 8 exchange dispatch flag, 9 exchange return flag, 10 exchange rows not matching their
 * header's counts (bit 2 of the status: such rows are dropped), 15 TMEM allocation not at column 0),
 * then the CTA rank, issuer or source rank, stage, phase and step.  Also covers the
 * no-allocation entry point, whose workspace is private.  No reference counterpart: the
 * reference reports device failures only as a launch result
 * (csrc/cutlass_mxfp8_mxfp4_probe.cu:598-613, csrc/bindings.cpp:113-127). */
int cdg_device_status(int32_t clear, int32_t* where);

/* SMs the persistent GEMM kernels may use (0 = all; values above the device's count mean
 * all), e.g. to leave SMs to kernels that overlap the GEMM on another stream.  Process-wide,
 * read at every launch.  Replaces set_num_sms / get_num_sms (consumer_deep_gemm/utils.py:12-22),
 * which the reference stores without using.  cdg_get_num_sms returns the setting, or the
 * current device's SM count when it is 0. */
int cdg_set_num_sms(int32_t num_sms);
int cdg_get_num_sms(void);

/* Whether the GEMM's kernels after the first are launched with programmatic stream
 * serialization (1, the default: each may be scheduled while its predecessor drains and
 * waits for it on the device) or as plain stream-ordered launches (0).  Process-wide.
 * Replaces set_pdl / get_pdl (consumer_deep_gemm/utils.py:44-50), stored there unused. */
int cdg_set_pdl(int32_t enable);
int cdg_get_pdl(void);

/* Static description of the build ("sm_100a; ...").
 * Replaces native.build_info (consumer_deep_gemm/native.py:26-39) and the SM120
 * probes (csrc/cutlass_sm120_probe.cu:6-22). */
const char* cdg_build_info(void);

/* Row alignment of each group in the contiguous layout (128).
 * Replaces get_mk_alignment_for_contiguous_layout (consumer_deep_gemm/layout.py:32-34). */
int cdg_mk_alignment_for_contiguous_layout(void);

/* Profiling hook: when both are non-NULL, every later GEMM call made from this
 * host thread records `start_event` on its stream just before the tensor-core
 * GEMM kernels and `stop_event` just after them (cudaEvent_t handles created
 * with timing enabled).  NULL, NULL switches it off.  Replaces the reference's
 * CDG_PROFILE wrappers (consumer_deep_gemm/__init__.py:62-114), which
 * synchronised the whole device around every call. */
int cdg_set_profile_events(void* start_event, void* stop_event);

/* Size of the static device scratch that the no-allocation entry point below uses (64 MiB). */
#define CDG_NOALLOC_SCRATCH_BYTES (64u << 20)

/* Grouped FP8 x MXFP4 GEMM that allocates nothing.  No counterpart in the
 * reference: it exists for callers that cannot hand this library a workspace,
 * because they cannot allocate device memory at call time -- for example a
 * service whose device memory is entirely reserved up front by another caching
 * allocator (a raw allocation then fails for lack of free memory), or a
 * foreign host (JNI, cgo, a plugin) with no path to the owning allocator.
 *
 * Same arguments and results as cdg_grouped_fp8_fp4_gemm_nt_contiguous, but the
 * temporaries live in a file-scope device array of CDG_NOALLOC_SCRATCH_BYTES,
 * which every GPU that loads the library keeps until the process exits.
 *   - Problems whose workspace (cdg_grouped_fp8_fp4_workspace_bytes + 1 KiB of
 *     alignment) exceeds that size are refused with CDG_ERR_SCRATCH_TOO_SMALL
 *     before anything is launched.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - All calls share one array, which keeps the previous call's contents (the
 *     call clears the words that must start at zero).  Calls that overlap on the
 *     GPU -- on different streams, or from several host threads -- race on it
 *     and must be serialised by the caller.
 *   - No cudaMalloc, cudaFree or allocating library routine is called. */
int cdg_grouped_fp8_fp4_gemm_nt_contiguous_noalloc(const cdg_gemm_args* args, cdg_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Mixture-of-experts layer around the grouped GEMM, and expert parallelism.
 * None of these exist in the reference (it ships the GEMM only); they are the
 * steps vLLM runs on either side of it, restated for this library:
 *   activation quantisation  deep_gemm/utils/math.py:21-37 (per_block_cast_to_fp8)
 *   SiLU-mul + requant       vLLM DeepGemmFP4Experts._act_mul_quant (experts/deep_gemm_moe.py:420-453),
 *                            gate = first half of FC1's output (consumer_deep_gemm/mega.py:19-22)
 *   permute / unpermute      vLLM deepgemm_moe_permute / deepgemm_unpermute_and_reduce
 *                            (fused_moe/deep_gemm_utils.py:347, 420)
 * Strides are in elements; e4m3 tensors are bytes.
 * ------------------------------------------------------------------------------------------- */

/* Activation scale recipes of the quantising steps (scale_fmt); amax = the largest |x| of the
 * 128-column block, clamped at 1e-12; FP32 arithmetic, e4m3 round to nearest even:
 *   CDG_SCALE_FP32  s = amax / 448, q = e4m3(x / amax * 448)   (per_block_cast_to_fp8)
 *   CDG_SCALE_POW2  s = amax / 448 rounded up to a power of two (exactly), q = e4m3(x / s)
 *                   (the UE8M0 recipe DeepGEMM's SM100 path uses; s is still stored as FP32,
 *                   and such scales put the GEMM's blocks in its direct class) */
#define CDG_SCALE_FP32 0
#define CDG_SCALE_POW2 1

/* q[r, :], s[r, kb] = 1x128 e4m3 quantisation of x (scale_fmt recipe); x is BF16 or F32
 * (x_dtype), K a multiple of 128. */
int cdg_quant_fp8_rows(const void* x, int32_t x_dtype, int64_t x_stride, int64_t M, int64_t K, uint8_t* q,
                       int64_t q_stride, float* s, int64_t s_stride_m, int64_t s_stride_k, int32_t scale_fmt,
                       cdg_stream_t stream);

/* in = [gate | up] BF16 [M, 2I]: q, s = 1x128 e4m3 quantisation of silu(gate) * up (FP32,
 * scale_fmt recipe).  Rows whose m_indices entry is negative are skipped (m_indices may be NULL). */
int cdg_silu_mul_quant_fp8(const void* in, int64_t in_stride, int64_t M, int64_t I, const int32_t* m_indices,
                           uint8_t* q, int64_t q_stride, float* s, int64_t s_stride_m, int64_t s_stride_k,
                           int32_t scale_fmt, cdg_stream_t stream);

/* counts[e] = number of entries of topk_ids (n of them, int32 or int64) equal to e, e in [0, E). */
int cdg_ep_count(const void* topk_ids, int32_t ids_dtype, int64_t n, int64_t E, int32_t* counts, cdg_stream_t stream);
/* The same counts, and expert_off[e] (int64) = the start row of expert e's group in the 128-aligned
 * contiguous layout (sum over e' < e of counts rounded up to 128), computed on the device: the offsets
 * cdg_ep_quant_dispatch_local takes, without a host round trip.  scratch: int32 [1]. */
int cdg_ep_count_offsets(const void* topk_ids, int32_t ids_dtype, int64_t n, int64_t E, int32_t* counts,
                         int64_t* expert_off, int32_t* scratch, cdg_stream_t stream);

/* Bytes of one dispatched row for hidden size H: [e4m3 data H][FP32 scales H/128]
 * [int32 local expert id], padded to 16 (0 for an invalid H). */
int64_t cdg_ep_row_bytes(int64_t H);

/* Send buffer of expert parallelism: every (token t, slot j) with expert e in [0, E) writes
 * token t's e4m3 row, its scales and the expert's local id e % (E / ranks) as one packed row
 * (cdg_ep_row_bytes) of destination rank e / (E / ranks), rows of a destination starting at
 * send_off[dest]; send_index[t*topk + j] is that row (-1 for skipped slots).
 * `fill` is [ranks] scratch. */
int cdg_ep_pack(const uint8_t* xq, int64_t xq_stride, const float* xs, int64_t xs_stride, const void* topk_ids,
                int32_t ids_dtype, int64_t T, int64_t topk, int64_t E, int64_t ranks, int64_t H,
                const int64_t* send_off, int32_t* fill, uint8_t* out_rows, int32_t* send_index, cdg_stream_t stream);

/* Received packed rows -> contiguous layout: row i of local expert e lands in
 * [expert_off[e], +count), expert_off being the 128-aligned offsets; m_indices[M_pad] is -1
 * except on placed rows; perm_pos[i] is row i's position.  `fill` is [E_local] scratch. */
int cdg_ep_permute(const uint8_t* recv_rows, int64_t R, int64_t H, int64_t E_local, const int64_t* expert_off,
                   int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices, int64_t M_pad, int32_t* perm_pos,
                   cdg_stream_t stream);

/* One rank, no exchange: quantise each token's row once (1x128 e4m3, scale_fmt recipe) and
 * write it straight into the contiguous layout, at row expert_off[e] + k of every slot (t, j)
 * whose expert e = topk_ids[t, j] is in [0, E) (k counts the expert's rows; expert_off are the
 * 128-aligned offsets from cdg_ep_count's counts).  m_indices[M_pad] is -1 except on placed
 * rows; perm_pos[t*topk + j] is the slot's row and send_index[t*topk + j] the slot itself (-1
 * for skipped slots): the arguments cdg_ep_unpermute_combine takes.  Replaces the
 * quantise / pack / permute sequence (one read of x, no intermediate rows).  `fill` is [E]
 * scratch; topk <= 32; row order within an expert depends on timing. */
int cdg_ep_quant_dispatch_local(const void* x, int32_t x_dtype, int64_t x_stride, const void* topk_ids,
                                int32_t ids_dtype, int64_t T, int64_t topk, int64_t E, int64_t H,
                                const int64_t* expert_off, int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices,
                                int64_t M_pad, int32_t* perm_pos, int32_t* send_index, int32_t scale_fmt,
                                cdg_stream_t stream);

/* Planes forms of the layer's quantising steps (FP32 1x128 recipe only): instead of e4m3 rows and
 * their scales they write the two e4m3 planes the grouped GEMM reads, planes uint8 [2][M_pad][H]
 * (plane stride M_pad * H; M_pad a multiple of 128), and int32 row exponents row_exp [M_pad], the split
 * the GEMM's prep kernel would make of those rows (hi = e4m3(x / 2^E), lo = e4m3(x / 2^E - hi) with
 * x = bf16(bf16(q) * bf16(s)) and E the frexp exponent of the row's largest |bf16(s)|).  Passed to the
 * GEMM as a_dtype CDG_DTYPE_E4M3_PLANES they spare it the plane split (a read of the rows and a write
 * of both planes).  Same row placement, m_indices, perm_pos / send_index and ret_slot as the row
 * forms; the rows' values equal theirs bit for bit.
 *   cdg_ep_quant_dispatch_local_planes  as cdg_ep_quant_dispatch_local
 *   cdg_silu_mul_quant_planes           as cdg_silu_mul_quant_fp8 (rows 16-byte aligned; rows with a
 *                                        negative m_indices entry are skipped)
 *   cdg_ep_permute_p2p_planes           as cdg_ep_permute_p2p */
int cdg_ep_quant_dispatch_local_planes(const void* x, int32_t x_dtype, int64_t x_stride, const void* topk_ids,
                                       int32_t ids_dtype, int64_t T, int64_t topk, int64_t E, int64_t H,
                                       const int64_t* expert_off, int32_t* fill, uint8_t* planes, int32_t* row_exp,
                                       int32_t* m_indices, int64_t M_pad, int32_t* perm_pos, int32_t* send_index,
                                       cdg_stream_t stream);
int cdg_silu_mul_quant_planes(const void* in, int64_t in_stride, int64_t M, int64_t I, const int32_t* m_indices,
                              uint8_t* planes, int32_t* row_exp, cdg_stream_t stream);
int cdg_ep_permute_p2p_planes(void* window, int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H,
                              int64_t E_local, int32_t* fill, uint8_t* planes, int32_t* row_exp, int32_t* m_indices,
                              int64_t M_pad, int32_t* ret_slot, const uint64_t* peers, uint64_t* ret_rows,
                              cdg_stream_t stream);

/* Fixed-capacity exchange (no host synchronisation).  The send (and receive) buffer holds
 * per destination (source) rank a region of 1 + cap packed rows of cdg_ep_row_bytes(H):
 * row 0 a header with the int32 number of rows routed to each of that rank's E/ranks local
 * experts, then the rows themselves.
 *
 * cdg_ep_quant_pack_fixed quantises token t's BF16/FP32 row (1x128 e4m3 + FP32 scales, the
 * scale_fmt recipe) into a packed row of the region of rank e / (E / ranks) for
 * every slot j with expert e = topk_ids[t, j] in [0, E); send_index[t*topk + j] is that row
 * (-1 for skipped slots and for slots beyond `cap`, which the caller should size to
 * T * topk to drop nothing).  `scratch` is int32 [cdg_ep_fixed_scratch_ints(ranks, E)],
 * zeroed by the call. */
int64_t cdg_ep_fixed_scratch_ints(int64_t ranks, int64_t E);
int cdg_ep_quant_pack_fixed(const void* x, int32_t x_dtype, int64_t x_stride, const void* topk_ids, int32_t ids_dtype,
                            int64_t T, int64_t topk, int64_t E, int64_t ranks, int64_t H, int64_t cap, int32_t* scratch,
                            uint8_t* out_rows, int32_t* send_index, int32_t scale_fmt, cdg_stream_t stream);

/* Fixed-capacity receive buffer -> contiguous layout (group offsets derived on the device
 * from the headers).  M_pad must be at least ranks*cap + 127*E_local (the worst case);
 * m_indices is -1 on every other row; perm_pos[i] is row i's position or -1 for headers and
 * unused rows.  E_local <= 1024, ranks <= 256, 4*E_local <= cdg_ep_row_bytes(H). */
int cdg_ep_permute_fixed(const uint8_t* recv_rows, int64_t ranks, int64_t cap, int64_t H, int64_t E_local,
                         int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices, int64_t M_pad, int32_t* perm_pos,
                         cdg_stream_t stream);

/* Row gathers of transform_weights_for_mega_moe (consumer_deep_gemm/mega.py:14-50):
 * dst[g, n, :] = src[g, f(n), :] for G groups of N rows of row_bytes bytes (source strides in
 * bytes, destination dense).  kind 1: interleave the gate half and the up half of the rows in
 * granules of 8 (N % 16 == 0); kind 2: transpose each 128-row block as [4 x 32] -> [32 x 4]
 * (N % 128 == 0); kind 3: both (the L1 scale transform).  The caller keeps tensors whose N is
 * not a multiple of 128 unchanged for kind 2, as the reference does. */
int cdg_mega_moe_transform_rows(const void* src, int64_t stride_g, int64_t stride_n, void* dst, int64_t G, int64_t N,
                                int64_t row_bytes, int32_t kind, cdg_stream_t stream);

/* Peer-memory exchange (expert parallelism over NVLink without a collective library).
 * Every rank owns an exchange window (cdg_ep_window_bytes) shared with the other ranks
 * through CUDA IPC: create it with cdg_ep_window_create, send the 64-byte handle to the
 * other ranks (any host channel), open theirs with cdg_ep_window_open, and pass the
 * ranks' window addresses as a device array `peers` (uint64 [ranks], this rank's own
 * window `window` at index `me`).  Windows are sized for at most `max_tokens` tokens per
 * rank with `topk` slots each.  Each rank runs, once per exchange step and in this order:
 *   cdg_ep_dispatch_p2p   quantise each token's row once (1x128 e4m3, scale_fmt recipe) and
 *                         store it, with the token index and the local expert of each of its
 *                         slots, into the window of every rank that owns one of its experts
 *                         (one row per token and destination rank), then raise this rank's
 *                         flag there; send_index[t*topk + j] = t*topk + j (-1: no expert);
 *   cdg_ep_permute_p2p    wait (bounded) for every source's flag, then lay the received rows
 *                         out per local expert (128-aligned groups, A / SA / m_indices as the
 *                         grouped GEMM reads them; a row with several slots here is written
 *                         to each slot's group); ret_slot[pos] says where GEMM row pos goes back;
 *                         with `peers` and `ret_rows` given (both or neither), ret_rows[pos]
 *                         (uint64 [M_pad], 0 on unplaced rows) is that place's address in the
 *                         source's window: the d_rows table of an FC2 GEMM that stores its rows
 *                         straight back (cdg_gemm_args.d_rows), making the return step part of FC2;
 *   cdg_ep_return_p2p     (when FC2 wrote into a local buffer) store each GEMM row into its
 *                         source's window at the source's slot index, raise flags;
 *   cdg_ep_combine_p2p    wait for every rank's rows, weighted top-k sum (as cdg_ep_combine),
 *                         and advance the window's step counter; with `peers` given, it first
 *                         raises this rank's return flags (for an FC2 that stored through
 *                         ret_rows; NULL after cdg_ep_return_p2p, which raised them).
 * The step number (flag value; the windows are double-buffered by its parity) lives in the
 * window, so the calls take no per-step argument and a whole step can be captured in a CUDA
 * graph; every rank must run the same number of steps.  Plain stores and loads over NVLink:
 * no multicast.  A wait that gives up after its bound (2 s, cdg_ep_set_wait_timeout_ns)
 * skips its CTA's work and sets the window's status word (cdg_ep_window_status and
 * cdg_device_status report it).  scratch: int32 [cdg_ep_fixed_scratch_ints(ranks, E)] for
 * dispatch, int32 [1] for return, int32 [2] for combine.  Limits: ranks <= 128, topk <= 32, E / ranks <=
 * 1024, H a multiple of 128, ranks * max_tokens * topk < 2^31; M_pad of the permute at least
 * ranks * max_tokens * topk + 127 * E_local (the worst case). */
size_t cdg_ep_window_bytes(int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H);
int cdg_ep_window_create(size_t bytes, void** window, void* ipc_handle /* 64 bytes out */);
int cdg_ep_window_open(const void* ipc_handle, void** window);
int cdg_ep_window_close(void* window, int32_t opened);
int cdg_ep_window_status(const void* window, cdg_stream_t stream);
int cdg_ep_dispatch_p2p(const void* x, int32_t x_dtype, int64_t x_stride, const void* topk_ids, int32_t ids_dtype,
                        int64_t T, int64_t topk, int64_t E, int64_t ranks, int64_t H, int64_t max_tokens,
                        const uint64_t* peers, void* window, int32_t me, int32_t* scratch, int32_t* send_index,
                        int32_t scale_fmt, cdg_stream_t stream);
int cdg_ep_permute_p2p(void* window, int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H, int64_t E_local,
                       int32_t* fill, uint8_t* A, float* SA, int32_t* m_indices, int64_t M_pad, int32_t* ret_slot,
                       const uint64_t* peers, uint64_t* ret_rows, cdg_stream_t stream);
int cdg_ep_return_p2p(const void* Y, int64_t y_stride, int64_t y_rows, const int32_t* ret_slot, int64_t M_pad,
                      int64_t ranks, int64_t max_tokens, int64_t topk, int64_t H, const uint64_t* peers, void* window,
                      int32_t me, int32_t* scratch, cdg_stream_t stream);
int cdg_ep_combine_p2p(void* window, const int32_t* send_index, const float* topk_w, int64_t T, int64_t topk,
                       int64_t H, int64_t ranks, int64_t max_tokens, const uint64_t* peers, int32_t me,
                       int32_t* scratch, void* y, cdg_stream_t stream);
/* Bound of the exchange's waits on other ranks' flags on the current device, in ns (0 = the
 * default 2 s; at most 60 s).  A wait that runs out sets the window's status word and the
 * record cdg_device_status() reads; the waiting step then places no rows (permute) or writes
 * zero rows (combine), so nothing downstream reads memory that was never written. */
int cdg_ep_set_wait_timeout_ns(uint64_t ns);

/* out[i, :] = Y[perm_pos[i], :] (BF16 rows of length H); rows with perm_pos[i] = -1 are not written. */
int cdg_ep_unpermute(const void* Y, int64_t y_stride, const int32_t* perm_pos, int64_t R, int64_t H, void* out,
                     cdg_stream_t stream);

/* y[t, :] = bf16(sum_j topk_w[t, j] * rows[send_index[t*topk + j], :]) in FP32, skipping -1 slots. */
int cdg_ep_combine(const void* rows, const int32_t* send_index, const float* topk_w, int64_t T, int64_t topk,
                   int64_t H, void* y, cdg_stream_t stream);

/* Fused unpermute + combine for a layer without an exchange (one rank): y[t, :] =
 * bf16(sum_j topk_w[t, j] * Y[perm_pos[send_index[t*topk + j]], :]) in FP32, skipping -1 slots; the
 * same values as cdg_ep_unpermute followed by cdg_ep_combine, without the intermediate rows.
 * Replaces vLLM deepgemm_unpermute_and_reduce (fused_moe/deep_gemm_utils.py:420) for this layout. */
int cdg_ep_unpermute_combine(const void* Y, int64_t y_stride, const int32_t* perm_pos, const int32_t* send_index,
                             const float* topk_w, int64_t T, int64_t topk, int64_t H, void* y, cdg_stream_t stream);

/* Human-readable name of a cdg_status value. */
const char* cdg_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* CDG_B200_H_ */
