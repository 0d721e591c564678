/*
 * mxfp4_b200 — C ABI of the B200 (sm_100a) MXFP4-weight x BF16-activation GEMM library.
 *
 * Plain pointers and sizes only.  Every device pointer must be 16-byte aligned and refer to
 * contiguous row-major memory on the current CUDA device; `stream` is a cudaStream_t
 * (NULL = legacy default stream).  All entry points are asynchronous on `stream`, allocate
 * nothing, keep no per-call host state and are safe to call from several host threads.
 * Return value: 0 on success, a cudaError_t value (1..999) for a CUDA error, or one of the
 * MXFP4_ERR_* codes below; mxfp4_error_string() turns either into text.
 *
 * Data formats (identical bytes to the reference package mxfp4_cdna3):
 *   E2M1 nibble = sign<<3 | magnitude index, magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6};
 *   two nibbles per byte along K, even k in the low nibble;
 *   one E8M0 scale byte per 32 K-elements, value 2**(byte - 127).
 * Weight layouts accepted by the GEMM and the prepack:
 *   MXFP4_LAYOUT_REF       B_packed uint8 [K/2, N], B_scales uint8 [K/32, N]
 *                          (reference: csrc/mxfp4_ext.cpp:21-24, python/mxfp4_cdna3/ref.py:14-47)
 *   MXFP4_LAYOUT_NK        W_packed uint8 [N, K/2], W_scales uint8 [N, K/32] (row-major weights)
 *   MXFP4_LAYOUT_G         the reference's strategy-G prepack, flattened
 *                          (python/mxfp4_cdna3/ref.py:85-101; needs N % 128 == 0)
 *   MXFP4_LAYOUT_PREPACKED this library's chunk layout from mxfp4_prepack(); B_scales unused
 */
#ifndef MXFP4_B200_H_
#define MXFP4_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MXFP4_B200_ABI_VERSION 1

enum mxfp4_layout {
  MXFP4_LAYOUT_REF = 0,
  MXFP4_LAYOUT_NK = 1,
  MXFP4_LAYOUT_G = 2,
  MXFP4_LAYOUT_PREPACKED = 3
};

enum mxfp4_dtype { MXFP4_DTYPE_F32 = 0, MXFP4_DTYPE_BF16 = 1 };

enum mxfp4_path {
  MXFP4_PATH_AUTO = 0,     /* cost model picks (mxfp4_select_path) */
  MXFP4_PATH_TC = 1,       /* large-M tcgen05 kernel, dequantised weights in tensor memory */
  MXFP4_PATH_TC_SMEM = 2,  /* large-M tcgen05 kernel, dequantised weights in shared memory */
  MXFP4_PATH_GEMV = 3      /* small-M (M <= 16) streaming kernel, cluster split-K */
};

enum mxfp4_quant_rule {
  MXFP4_RULE_REF = 0, /* reference rule: ceil(log2(amax/6)), ties to the lower magnitude */
  MXFP4_RULE_OCP = 1  /* OCP MX: floor(log2(amax)) - 2, round-nearest-even, saturate at 6 */
};

#define MXFP4_ERR_INVALID_ARGUMENT 1000 /* null pointer, negative size, bad enum */
#define MXFP4_ERR_UNSUPPORTED_SHAPE 1001 /* shape outside what the chosen path handles */
#define MXFP4_ERR_MISALIGNED 1002 /* pointer or row stride not 16-byte aligned */
#define MXFP4_ERR_WORKSPACE 1003 /* workspace missing or smaller than required */
#define MXFP4_ERR_DRIVER 1004 /* driver entry point (tensor-map encoder) unavailable */
#define MXFP4_ERR_DEVICE 1005 /* current device is not an sm_100 part */
#define MXFP4_ERR_NOALLOC_LIMIT 1006 /* weights too large for the fixed buffer of mxfp4_gemm_noalloc */

typedef struct mxfp4_device_info {
  char name[256];
  int major, minor;
  int multi_processor_count;
  int warp_size;
  long long total_global_mem;
  long long shared_mem_per_block;
  long long shared_mem_per_block_optin;
  long long l2_cache_size;
  int clock_rate_khz;
  int memory_clock_rate_khz;
  int memory_bus_width;
} mxfp4_device_info;

/* Library ABI version (MXFP4_B200_ABI_VERSION). */
int mxfp4_abi_version(void);

/* Device properties (replaces the reference's device_info, csrc/mxfp4_ext.cpp:156-168). */
int mxfp4_device_info_get(int device, mxfp4_device_info* out);

/* Reads the device error word that bounded waits inside the kernels set when they give up
 * (0 = none); clears it when `clear` is non-zero.  Synchronises the device. */
int mxfp4_device_error(int clear, unsigned int* code_out);

const char* mxfp4_error_string(int code);

/* Test hook (no counterpart in the reference, whose kernels have no bounded waits): sets, on
 * the current device, the limit of every bounded wait inside the kernels (wait_limit_ns; 0
 * restores the default of one second) and a switch that makes the weight producers of the
 * large-M and decode kernels issue no copies (withhold != 0).  With the switch on, the
 * consumers' waits run out after the limit, the kernel records a wait error readable with
 * mxfp4_device_error(), releases its tensor memory and returns: the abort path runs without any
 * fault.  Synchronous; for tests only -- turn the switch off again before real work. */
int mxfp4_test_hooks(int withhold, unsigned long long wait_limit_ns);

/* Quantise fp32 x[rows, cols] along `axis` (0: groups of 32 rows -> packed [rows/2, cols],
 * scales [rows/32, cols]; 1: groups of 32 columns -> [rows, cols/2], [rows, cols/32]).
 * Replaces quantize_mxfp4 (python/mxfp4_cdna3/ref.py:14-47) for rule MXFP4_RULE_REF. */
int mxfp4_quantize(const float* x, int rows, int cols, int axis, int rule, uint8_t* packed,
                   uint8_t* scales, void* stream);

/* Dequantise to fp32 or bf16.  layout MXFP4_LAYOUT_REF: [K/2,N]+[K/32,N] -> out [K,N];
 * MXFP4_LAYOUT_NK: [N,K/2]+[N,K/32] -> out [N,K].
 * Replaces dequantize_mxfp4 (python/mxfp4_cdna3/ref.py:50-72). */
int mxfp4_dequantize(const uint8_t* packed, const uint8_t* scales, int K, int N, int layout,
                     void* out, int out_dtype, void* stream);

/* Bytes of the prepacked form of an N x K weight (N padded to 128, K to 64). */
size_t mxfp4_prepacked_bytes(int N, int K);

/* Re-lay weights (src_layout REF, NK or G) into the chunk layout the GEMM kernels stream.
 * Replaces prepack_b_mxfp4 (python/mxfp4_cdna3/ref.py:85-101) as the B200 analogue of the
 * strategy-G layout.  dst must hold mxfp4_prepacked_bytes(N, K) bytes. */
int mxfp4_prepack(const uint8_t* packed, const uint8_t* scales, int N, int K, int src_layout,
                  uint8_t* dst, void* stream);

/* Dequantise prepacked weights to bf16 bit patterns out[N, K] with the exact table-lookup
 * routine the tensor-core kernel uses (for bit-exact verification of the GEMM's tile). */
int mxfp4_dequantize_prepacked(const uint8_t* wpack, int N, int K, uint16_t* out, void* stream);

/* Path the cost model picks for C[M,N] = A[M,K] * dequant(B) (an mxfp4_path value). */
int mxfp4_select_path(int M, int N, int K);

/* 1 if `path` (MXFP4_PATH_*) handles the shape, else 0.  Replaces shape_supported_{c,d,e,f,g}
 * (csrc/common.h:80-99): every path here needs K % 32 == 0 and N % 8 == 0. */
int mxfp4_shape_supported(int path, int M, int N, int K);

/* Workspace bytes mxfp4_gemm uses for a weight layout: the prepacked copy of B for layouts
 * other than PREPACKED (required), plus, for M <= 16 (shapes the decode path may serve), room for the
 * activations converted once per call (optional: with less workspace every decode CTA converts
 * its own slice, which is slower for M >= 4). */
size_t mxfp4_gemm_workspace_bytes(int M, int N, int K, int layout);

/* C[M,N] = A[M,K] (bf16) * dequant(B)[K,N], fp32 accumulation, C in c_dtype.
 * Replaces the launcher ABI launch_strategy_{a..m} (csrc/common.h:43-78) and the dispatch
 * in csrc/mxfp4_ext.cpp:36-48; the reference always writes fp32 C, this adds bf16.
 * For layouts other than PREPACKED the weights are first re-laid into `workspace`; any room
 * left after them (see mxfp4_gemm_workspace_bytes) serves the decode path's staged activations.
 * Calls sharing one workspace must not overlap on the GPU. */
int mxfp4_gemm(const void* A, const uint8_t* B, const uint8_t* B_scales, void* C, int c_dtype,
               int M, int N, int K, int layout, int path, void* workspace, size_t workspace_bytes,
               void* stream);

/* Column-parallel GEMM with the all-gather fused into the epilogue.  Replaces the reference
 * pair "gemm_X on this rank's weight columns" + a separate all-gather of the outputs (the
 * multi-GPU sharding the reference leaves to its callers; no single reference function).
 * B_prepacked: this GPU's column slice of the weights (N columns), PREPACKED layout.  The
 * [M, N] result is written, as the tiles are produced, into each of the n_dst (<= 8) buffers
 * C_dst[i] -- every GPU's full [M, ldc] output, this GPU's own and its peers' (opened with
 * mxfp4_ipc_open) -- at columns n_off .. n_off+N-1.  The stores are made visible system-wide
 * before the kernel ends; the caller still orders the peers' later reads after this kernel
 * (e.g. a stream-ordered collective on the same stream on every GPU).  Workspace as for
 * mxfp4_gemm with the PREPACKED layout. */
int mxfp4_gemm_allgather(const void* A, const uint8_t* B_prepacked, void* const* C_dst, int n_dst, int n_off,
                         int ldc, int c_dtype, int M, int N, int K, int path, void* workspace,
                         size_t workspace_bytes, void* stream);

/* CUDA IPC for the all-gather destinations (no reference counterpart: the reference runs on
 * one GPU).  mxfp4_ipc_export gives the handle (mxfp4_ipc_handle_bytes() bytes) of the
 * allocation holding dev_ptr and dev_ptr's offset in it; another process on the same node
 * maps it with mxfp4_ipc_open and unmaps it with mxfp4_ipc_close (same offset). */
size_t mxfp4_ipc_handle_bytes(void);
int mxfp4_ipc_export(const void* dev_ptr, void* handle_out, size_t* offset_out);
int mxfp4_ipc_open(const void* handle, size_t offset, void** dev_ptr_out);
int mxfp4_ipc_close(void* dev_ptr, size_t offset);

/* Copy-engine form of the column all-gather (no reference counterpart): copies `rows` rows of
 * width_bytes each from src (row pitch src_pitch) to dst (row pitch dst_pitch) as one pitched
 * device-to-device copy on `stream`.  With dst a peer's output buffer (mxfp4_ipc_open) at this
 * GPU's column offset, it pushes this GPU's output columns over NVLink without occupying any
 * SM, so it overlaps the next GEMM on another stream.  The caller orders the peers' reads (a
 * stream-ordered collective after the copies on every GPU). */
int mxfp4_copy_columns(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width_bytes,
                       int rows, void* stream);

/* Fixed size of the device buffer mxfp4_gemm_noalloc uses in place of a workspace. */
#define MXFP4_NOALLOC_SCRATCH_BYTES (32u << 20)

/* No counterpart in the reference.  Same as mxfp4_gemm for weights in the REF, NK or G layout,
 * but for callers that cannot allocate device memory -- code that must not call cudaMalloc
 * (a custom or pool allocator owns all device memory, an allocation would synchronise the
 * device mid-pipeline, or the caller is a plugin with no allocator handle) and so cannot
 * hand over the workspace mxfp4_gemm wants.  The re-laid weights go into a buffer that is
 * part of the library itself: a fixed MXFP4_NOALLOC_SCRATCH_BYTES (32 MiB) device array
 * that every GPU which loads the library holds until the process exits.  Weights needing
 * more than that (mxfp4_prepacked_bytes(N, K) > 32 MiB, e.g. beyond about N*K = 63M
 * elements) are rejected with MXFP4_ERR_NOALLOC_LIMIT.  The first call on a device looks up
 * the buffer's device address for that device; make that first call before any stream
 * capture.  All calls share the one buffer, so calls that may overlap on the GPU (different
 * streams, or several host threads) race on it and give wrong results; serialise them. */
int mxfp4_gemm_noalloc(const void* A, const uint8_t* B, const uint8_t* B_scales, void* C, int c_dtype,
                       int M, int N, int K, int layout, int path, void* stream);

/* ---- Block-scaled paths (no reference counterpart) ---------------------------------------
 * C[M,N] = A' * dequant(W) on the tensor cores' block-scaled MMA (kind::mxf8f6f4): the weights
 * stay E2M1 + E8M0 and the bf16 activations are coded as E4M3 pieces with one E8M0 scale per
 * 32 k of a row; the MMA applies both scales.  `mode`:
 *   MXFP4_MX_Q8      one piece, the OCP MX rule (exponent floor(log2(amax)) - 8, round to
 *                    nearest even, saturate at 448): activations keep 4 significant bits;
 *   MXFP4_MX_SPLIT2  two pieces, hi (exponent floor(log2(amax)) - 7) plus the exact residual
 *                    coded the same way: every element within 2**-8 of its group's max.
 * Reference: (sum of the dequantised pieces) @ dequant(W) in fp32.  M <= 16 runs a stream-K
 * decode kernel, larger M a persistent tile kernel.  Needs K % 32 == 0 and N % 8 == 0; the
 * re-laid weights and the workspace 32-byte aligned. */
#define MXFP4_MX_Q8 0
#define MXFP4_MX_SPLIT2 1

/* Bytes of the block-scaled weight layout: E2M1 nibbles [Np][Kp/2] (K contiguous) followed by
 * 512-byte scale blocks [Np/128][Kp/128]; Np = N rounded up to 128, Kp = K rounded up to 128. */
size_t mxfp4_mx_weight_bytes(int N, int K);
/* Re-lay REF or NK weights into that layout (dst: mxfp4_mx_weight_bytes(N, K) bytes). */
int mxfp4_prepack_mx(const uint8_t* packed, const uint8_t* scales, int N, int K, int src_layout, uint8_t* dst,
                     void* stream);
/* Workspace of mxfp4_gemm_mx: the coded activations (E4M3 code rows [rows][Kp], then at the
 * next 256-byte boundary their 512-byte scale blocks [Kp/128][rows rounded up to 128, /128]),
 * then for M <= 16 an fp32 [M][N] accumulation buffer.  Code row b holds piece p of activation
 * row m: M <= 16: b = 16p + m (32 rows); M > 16, Q8: b = m (M rounded up to 256 rows); M > 16,
 * SPLIT2: b = 256*(m/128) + 128p + m%128 (2 * (M rounded up to 128) rows). */
size_t mxfp4_mx_workspace_bytes(int M, int N, int K, int mode);
/* Code bf16 A[M,K] into dst in that layout (codes and scale blocks; exposed for verification). */
int mxfp4_quantize_act_mx8(const void* A, int M, int K, int mode, uint8_t* dst, void* stream);
/* The GEMM: codes A into `workspace`, then the block-scaled kernel (c_dtype MXFP4_DTYPE_F32 or
 * MXFP4_DTYPE_BF16, C [M, N] row-major). */
int mxfp4_gemm_mx(const void* A, const uint8_t* w_mx, void* C, int c_dtype, int M, int N, int K, int mode,
                  void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MXFP4_B200_H_ */
