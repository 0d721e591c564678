// C ABI of the library: argument checking, path selection, launches.
// Single translation unit: the kernels live in the included .cuh files.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/mxfp4_b200.h"
#include "common.cuh"
#include "gemm_large.cuh"
#include "gemm_mx.cuh"
#include "gemm_small.cuh"
#include "gemm_small_sk.cuh"
#include "gemm_small_tc.cuh"
#include "quant.cuh"

namespace mxb {
namespace {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int ret(cudaError_t e) { return e == cudaSuccess ? 0 : static_cast<int>(e); }

inline int launch_status() { return ret(cudaGetLastError()); }

// Per-device facts queried once.  `ready` is published after sm_count and major are written;
// the *_attr flags only skip repeating an idempotent cudaFuncSetAttribute, so concurrent
// first calls at worst repeat it.
struct DeviceState {
  std::atomic<bool> ready{false};
  int sm_count = 0;
  int major = 0;
  std::atomic<bool> tc_attr[4] = {false, false, false, false};
  std::atomic<bool> gv_attr[4] = {false, false, false, false};
  std::atomic<bool> gt_attr[2] = {false, false};
  std::atomic<bool> sk_attr[4] = {false, false, false, false};
  std::atomic<bool> mx_attr[4] = {false, false, false, false};
  std::atomic<bool> gm_attr{false};
};

constexpr int kMaxDevices = 64;
DeviceState g_dev[kMaxDevices];
std::mutex g_mu;

int current_device(DeviceState** st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ret(e);
  if (dev < 0 || dev >= kMaxDevices) return MXFP4_ERR_DEVICE;
  DeviceState& d = g_dev[dev];
  if (!d.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!d.ready.load(std::memory_order_relaxed)) {
      int sms = 0, major = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
      if (e != cudaSuccess) return ret(e);
      d.major = major;
      d.sm_count = sms;
      d.ready.store(true, std::memory_order_release);
    }
  }
  if (d.major != 10) return MXFP4_ERR_DEVICE;
  *st = &d;
  return 0;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t inner,
              uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXFP4_ERR_DRIVER;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : MXFP4_ERR_DRIVER;
}

// 2-D map over rows of `inner` elements spaced `row_bytes` apart (a column slice of a wider
// row-major matrix), no swizzle.
int encode_2d_strided(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t inner,
                      uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXFP4_ERR_DRIVER;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : MXFP4_ERR_DRIVER;
}

inline int k_blocks_of(int K) { return ceil_div(K, kChunkK); }
inline int n_blocks_of(int N) { return ceil_div(N, kChunkRows); }

// Where a GEMM's [M, N] result goes: dst[i] + (m * ldc + n_off + n) elements, i < count.
struct OutSpec {
  void* const* dst;
  int count, ldc, n_off, fence_sys;
};

// ------------------------------------------------------------------ large-M launch
// Split-K plan of the large-M kernel: with fewer tiles than half the SMs, K is split so that
// ~all SMs work (at most 8 slices, each at least 8 K-blocks).  1 = no split.
struct SplitPlan {
  int splits, kbps;
};
int env_knob(const char* name);
SplitPlan plan_splitk(int M, int N, int K, int sm_count) {
  // tuning knobs (sweeps only): the most slices and the fewest K-blocks per slice
  static const int max_knob = env_knob("MXFP4_TC_MAX_SPLITS"), kbps_knob = env_knob("MXFP4_TC_MIN_KBPS");
  const int max_s = max_knob >= 1 && max_knob <= 16 ? max_knob : 8;
  const int min_kbps = kbps_knob >= 1 && kbps_knob <= 64 ? kbps_knob : 8;
  const int tiles = ceil_div(M, kTcTileAct) * n_blocks_of(N);
  const int kb = k_blocks_of(K);
  SplitPlan p{1, kb};
  if (2 * tiles > sm_count || N % 4) return p;
  int s = std::min({max_s, sm_count / tiles, kb / min_kbps});
  if (s < 2) return p;
  p.kbps = ceil_div(kb, s);
  p.splits = ceil_div(kb, p.kbps);  // no empty slice
  return p;
}
size_t splitk_bytes(int M, int N, int K, int sm_count) {
  const SplitPlan p = plan_splitk(M, N, K, sm_count);
  return p.splits > 1 ? static_cast<size_t>(p.splits) * M * N * 4 : 0;
}

int encode_3d_f32(CUtensorMap* map, const float* base, uint64_t n, uint64_t m, uint64_t planes) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXFP4_ERR_DRIVER;
  cuuint64_t dims[3] = {n, m, planes};
  cuuint64_t strides[2] = {n * 4, n * m * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : MXFP4_ERR_DRIVER;
}

template <bool kTS, typename OutT>
int launch_tc(const void* A, const uint8_t* wpack, const OutSpec& o, int M, int N, int K, cudaStream_t stream,
              DeviceState* d, const SplitPlan& sp = SplitPlan{1, 0}, float* splitws = nullptr) {
  using Cfg = TcCfg<kTS, OutT>;
  const int slot = (kTS ? 0 : 2) + (sizeof(OutT) == 4 ? 0 : 1);
  if (!d->tc_attr[slot]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<kTS, OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmemBytes);
    if (e != cudaSuccess) return ret(e);
    d->tc_attr[slot] = true;
  }
  CUtensorMap tm_act;
  TcOut out;
  std::memset(&out, 0, sizeof(out));
  int rc = encode_2d(&tm_act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, A, K, M, kTcBK, kTcTileAct,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  for (int i = 0; i < (sp.splits > 1 ? 0 : o.count); ++i) {
    rc = encode_2d_strided(&out.map[i],
                           sizeof(OutT) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                           static_cast<int>(sizeof(OutT)), static_cast<OutT*>(o.dst[i]) + o.n_off, N, M,
                           static_cast<uint64_t>(o.ldc) * sizeof(OutT),
                           sizeof(OutT) == 2 && o.count > 1 ? 64 : 32, 32);  // paired bf16 slabs
    if (rc) return rc;
  }
  out.count = o.count;
  out.fence_sys = o.fence_sys;
  if (sp.splits > 1) {  // fp32 partials [splits][M][N] into the workspace (OutT is float here)
    rc = encode_3d_f32(&out.map[0], splitws, N, M, sp.splits);
    if (rc) return rc;
    out.count = 1;
    out.split3d = 1;
  }
  const int m_blocks = ceil_div(M, kTcTileAct);
  const int n_blocks = n_blocks_of(N);
  const int tiles = m_blocks * n_blocks * sp.splits;
  const int grid = std::min(tiles, d->sm_count);
  gemm_tc_kernel<kTS, OutT><<<grid, kTcThreads, Cfg::kSmemBytes, stream>>>(
      tm_act, out, wpack, M, k_blocks_of(K), m_blocks, n_blocks, sp.splits, sp.splits > 1 ? sp.kbps : k_blocks_of(K));
  return launch_status();
}

template <typename... KArgs, typename... Args>
int launch_pdl_grid(void (*kernel)(KArgs...), dim3 grid, int threads, int smem, cudaStream_t stream, Args... args);

// Large-M kernel with split-K: fp32 partials into `ws`, then one reduction into C (a
// programmatic dependent launch: it waits for the GEMM's partials with griddepcontrol.wait).
template <bool kTS>
int launch_tc_splitk(const void* A, const uint8_t* wpack, const OutSpec& o, int c_dtype, int M, int N, int K,
                     const SplitPlan& sp, float* ws, cudaStream_t stream, DeviceState* d) {
  int rc = launch_tc<kTS, float>(A, wpack, o, M, N, K, stream, d, sp, ws);
  if (rc) return rc;
  const size_t work = static_cast<size_t>(M) * (N / 4);
  const int blocks = static_cast<int>(std::min<size_t>(ceil_div(static_cast<int>(std::min<size_t>(work, 1u << 30)), 256),
                                                       static_cast<size_t>(d->sm_count) * 8));
  if (c_dtype == MXFP4_DTYPE_F32)
    return launch_pdl_grid(splitk_reduce_kernel<float>, dim3(blocks), 256, 0, stream, static_cast<const float*>(ws),
                           sp.splits, M, N, static_cast<float*>(o.dst[0]) + o.n_off, o.ldc);
  return launch_pdl_grid(splitk_reduce_kernel<__nv_bfloat16>, dim3(blocks), 256, 0, stream,
                         static_cast<const float*>(ws), sp.splits, M, N,
                         static_cast<__nv_bfloat16*>(o.dst[0]) + o.n_off, o.ldc);
}

// ------------------------------------------------------------------ small-M launch
struct GvPlan {
  int nt, ks, kbps, stages, smem;
};

int env_knob(const char* name) {
  const char* e = std::getenv(name);
  return e ? std::atoi(e) : 0;
}

// Programmatic dependent launch between our own chained kernels is on unless MXFP4_NO_PDL=1
// (read once per process): with it off every launch waits for the previous one in its stream,
// which separates a kernel's own faults from the ordering of the chain when bringing one up.
bool pdl_enabled() {
  static const bool on = env_knob("MXFP4_NO_PDL") != 1;
  return on;
}

// Decode plan: the K-split (cluster size) and ring depth.  Enough CTAs to fill every SM
// twice and each CTA's K range at most 2048 (32 chunks) so the staged activations stay
// small.  Two ring stages (35 KB): measured on B200, more resident CTAs (more compute warps
// per SM) beat a deeper ring at every decode shape.
GvPlan plan_gemv(int M, int N, int K, int sm_count) {
  GvPlan p;
  p.nt = M <= 8 ? 1 : 2;
  const int nb = n_blocks_of(N), kb = k_blocks_of(K);
  p.ks = 1;
  while (p.ks < 8 && (nb * p.ks < 2 * sm_count || ceil_div(kb, p.ks) > 32)) p.ks *= 2;
  p.stages = 2;
  // tuning knobs (sweeps only): force the K-split (1, 2, 4, 8) or the ring depth (2..8)
  static const int ks_knob = env_knob("MXFP4_GEMV_KS"), st_knob = env_knob("MXFP4_GEMV_STAGES");
  if (ks_knob == 1 || ks_knob == 2 || ks_knob == 4 || ks_knob == 8) p.ks = ks_knob;
  if (st_knob >= 2 && st_knob <= kGvMaxStages) p.stages = st_knob;
  p.kbps = ceil_div(kb, p.ks);
  p.smem = p.nt == 1 ? GvCfg<1>::smem_bytes(p.stages, p.kbps, M, false) : GvCfg<2>::smem_bytes(p.stages, p.kbps, M, false);
  return p;
}

template <int NT, typename OutT>
int launch_gemv_t(const void* A, const uint8_t* wpack, const OutSpec& o, int M, int N, int K, const GvPlan& p,
                  cudaStream_t stream, DeviceState* d, const uint8_t* xpre, const int* xpre_shift) {
  GvOut<OutT> out;
  std::memset(&out, 0, sizeof(out));
  for (int i = 0; i < o.count; ++i) out.p[i] = static_cast<OutT*>(o.dst[i]);
  out.count = o.count;
  out.ldc = o.ldc;
  out.n_off = o.n_off;
  out.fence_sys = o.fence_sys;
  const int slot = (NT == 1 ? 0 : 2) + (sizeof(OutT) == 4 ? 0 : 1);
  if (!d->gv_attr[slot]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<NT, OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         232448 - 1024);
    if (e != cudaSuccess) return ret(e);
    d->gv_attr[slot] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_blocks_of(N), p.ks, 1);
  cfg.blockDim = dim3(kGvThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = p.ks;
  attr[0].val.clusterDim.z = 1;
  // With prestaged activations the launch before this one is our own prestage kernel, which
  // writes nothing this kernel reads before griddep_wait(): let it start early.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = xpre && pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_kernel<NT, OutT>, static_cast<const __nv_bfloat16*>(A), M, K,
                                     wpack, k_blocks_of(K), p.kbps, p.stages, out, N,
                                     xpre, xpre_shift);
  return ret(e);
}

// Bytes of decode-kernel workspace for activations staged once per GEMM (0 when the decode
// kernel stages them itself): f16 [k_blocks*64] x M plus M row shifts.
size_t gemv_prestage_bytes(int M, int N, int K) {
  (void)N;
  if (M < 1 || M > 16) return 0;
  return static_cast<size_t>(k_blocks_of(K)) * kGtXChunkBytes + 256;  // covers both kernels' layouts
}

// Which decode kernel runs when the caller's workspace has room: the persistent stream-K
// gemv_sk_kernel by default; MXFP4_GEMV_KERNEL=1 selects the cluster split-K gemv_kernel and
// MXFP4_GEMV_KERNEL=2 the tcgen05 gemv_tc_kernel (measured slower on B200: 1.0-1.9 TB/s), kept
// as alternatives for comparison.
int gemv_kernel_knob() {
  static const int knob = env_knob("MXFP4_GEMV_KERNEL");
  return knob;
}
bool gemv_use_tc() { return gemv_kernel_knob() == 2; }

// Workspace of the stream-K decode path (0 when the shape is outside its range: M <= 16, and
// K <= 32768 so that one prestage thread holds its share of an activation row).
size_t gemv_sk_bytes(int M, int N, int K) {
  if (M < 1 || M > 16 || k_blocks_of(K) * 8 > kSkPreThreads * kSkPreVecs) return 0;
  return sk_workspace(M, n_blocks_of(N), k_blocks_of(K)).total;
}

// Launch with the programmatic-dependent-launch attribute (unless MXFP4_NO_PDL=1): the kernel
// may start while the launch before it in the stream (our own producer of its inputs) runs,
// and waits with griddepcontrol.wait before it reads what that launch writes.
template <typename... KArgs, typename... Args>
int launch_pdl_grid(void (*kernel)(KArgs...), dim3 grid, int threads, int smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return ret(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

template <typename OutT>
int launch_gemv_sk_finalize(const OutSpec& o, int M, int N, const SkWorkspace& w, uint8_t* ws, cudaStream_t stream,
                            DeviceState* d) {
  GvOut<OutT> out;
  std::memset(&out, 0, sizeof(out));
  for (int i = 0; i < o.count; ++i) out.p[i] = static_cast<OutT*>(o.dst[i]);
  out.count = o.count;
  out.ldc = o.ldc;
  out.n_off = o.n_off;
  out.fence_sys = o.fence_sys;
  const long long work = static_cast<long long>(M) * ((N + 1) / 2);
  const int blocks = static_cast<int>(std::min<long long>((work + 255) / 256, 4LL * d->sm_count));
  return launch_pdl_grid(gemv_sk_finalize_kernel<OutT>, dim3(blocks), 256, 0, stream,
                         reinterpret_cast<const float*>(ws + w.acc_off), reinterpret_cast<const int*>(ws + w.shift_off),
                         M, N, n_blocks_of(N) * kChunkRows, out);
}

// Warps per chunk of the stream-K decode kernel for 8 < M <= 16 (two n8 activation tiles).
#ifndef MXFP4_SK_WPC_WIDE
#define MXFP4_SK_WPC_WIDE 4
#endif
constexpr int kSkWpcWide = MXFP4_SK_WPC_WIDE;
// ... and for M <= 8 (one n8 activation tile).
#ifndef MXFP4_SK_WPC_NARROW
#define MXFP4_SK_WPC_NARROW 1
#endif
constexpr int kSkWpcNarrow = MXFP4_SK_WPC_NARROW;

// Stream-K decode: prestage (activations to f16, sums zeroed), the streaming kernel, then the
// conversion of the sums to the output -- three launches chained by programmatic dependent launch.
int launch_gemv_sk(const void* A, const uint8_t* wpack, const OutSpec& C, int c_dtype, int M, int N, int K,
                   uint8_t* ws, cudaStream_t stream, DeviceState* d) {
  const int nb = n_blocks_of(N), kb = k_blocks_of(K);
  const SkWorkspace w = sk_workspace(M, nb, kb);
  const long long zero_n4 = static_cast<long long>((w.total - w.acc_off) / 16);
  const int grid = std::max(M, d->sm_count);
  if (!(MXFP4_SK_DIAG & 32))
  gemv_sk_prestage_kernel<<<grid, kSkPreThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(A), M, K, kb,
                                                             ws + w.x_off, reinterpret_cast<int*>(ws + w.shift_off),
                                                             reinterpret_cast<float4*>(ws + w.acc_off), zero_n4);
  int rc = launch_status();
  if (rc) return rc;
  const int slot = M <= 8 ? 0 : 1;
  if (!d->sk_attr[slot]) {
    cudaError_t e = M <= 8 ? cudaFuncSetAttribute(gemv_sk_kernel<1, kSkWpcNarrow>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  std::max(sk_smem_bytes(1), sk_smem_bytes(8)))
                           : cudaFuncSetAttribute(gemv_sk_kernel<2, kSkWpcWide>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  std::max(sk_smem_bytes(9), sk_smem_bytes(16)));
    if (e != cudaSuccess) return ret(e);
    d->sk_attr[slot] = true;
  }
  const dim3 sk_grid(static_cast<unsigned>(std::min<long long>(d->sm_count, static_cast<long long>(nb) * kb)));
  const uint8_t* xpre = ws + w.x_off;
  float* acc = reinterpret_cast<float*>(ws + w.acc_off);
  rc = M <= 8 ? launch_pdl_grid(gemv_sk_kernel<1, kSkWpcNarrow>, sk_grid, kSkThreads, sk_smem_bytes(M), stream, wpack, M, kb, nb,
                                xpre, acc)
              : launch_pdl_grid(gemv_sk_kernel<2, kSkWpcWide>, sk_grid, kSkThreads, sk_smem_bytes(M), stream, wpack, M, kb, nb,
                                xpre, acc);
  if (rc) return rc;
  if (MXFP4_SK_DIAG & 16) return 0;
  return c_dtype == MXFP4_DTYPE_F32 ? launch_gemv_sk_finalize<float>(C, M, N, w, ws, stream, d)
                                    : launch_gemv_sk_finalize<__nv_bfloat16>(C, M, N, w, ws, stream, d);
}

template <typename OutT>
int launch_gemv_tc_t(const uint8_t* wpack, const OutSpec& o, int M, int N, int K, int sm_count,
                     cudaStream_t stream, DeviceState* d, const uint8_t* xpre, const int* xshift) {
  const int slot = sizeof(OutT) == 4 ? 0 : 1;
  if (!d->gt_attr[slot]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_tc_kernel<OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GtCfg::kSmemBytes);
    if (e != cudaSuccess) return ret(e);
    d->gt_attr[slot] = true;
  }
  const int nb = n_blocks_of(N), kb = k_blocks_of(K);
  int ks = 1;
  while (ks < 8 && nb * ks < 3 * sm_count && ceil_div(kb, ks * 2) >= kGtStageChunks) ks *= 2;
  static const int ks_knob = env_knob("MXFP4_GEMV_KS");
  if (ks_knob == 1 || ks_knob == 2 || ks_knob == 4 || ks_knob == 8) ks = ks_knob;
  const int kbps = ceil_div(kb, ks);
  GvOut<OutT> out;
  std::memset(&out, 0, sizeof(out));
  for (int i = 0; i < o.count; ++i) out.p[i] = static_cast<OutT*>(o.dst[i]);
  out.count = o.count;
  out.ldc = o.ldc;
  out.n_off = o.n_off;
  out.fence_sys = o.fence_sys;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nb, ks, 1);
  cfg.blockDim = dim3(kGtThreads, 1, 1);
  cfg.dynamicSmemBytes = GtCfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = ks;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // after our prestage kernel
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_tc_kernel<OutT>, wpack, M, kb, kbps, xpre, xshift, out, N);
  return ret(e);
}

int launch_gemv(const void* A, const uint8_t* wpack, const OutSpec& C, int c_dtype, int M, int N, int K,
                cudaStream_t stream, DeviceState* d, uint8_t* xws, size_t xws_bytes) {
  const size_t sk_need = gemv_sk_bytes(M, N, K);
  if (gemv_kernel_knob() == 0 && sk_need && xws && xws_bytes >= sk_need && (reinterpret_cast<uintptr_t>(xws) & 255) == 0)
    return launch_gemv_sk(A, wpack, C, c_dtype, M, N, K, xws, stream, d);
  GvPlan p = plan_gemv(M, N, K, d->sm_count);
  const size_t need = gemv_prestage_bytes(M, N, K);
  uint8_t* xpre = nullptr;
  int* xshift = nullptr;
  if (need && xws && xws_bytes >= need && aligned16(xws)) {
    xpre = xws;
    xshift = reinterpret_cast<int*>(xws + need - 256);
    if (gemv_use_tc()) {
      gemv_prestage_tc_kernel<<<16, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(A), M, K, k_blocks_of(K),
                                                      xpre, xshift);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return ret(e);
      return c_dtype == MXFP4_DTYPE_F32
                 ? launch_gemv_tc_t<float>(wpack, C, M, N, K, d->sm_count, stream, d, xpre, xshift)
                 : launch_gemv_tc_t<__nv_bfloat16>(wpack, C, M, N, K, d->sm_count, stream, d, xpre, xshift);
    }
    static const int min_m_knob = env_knob("MXFP4_GEMV_PRESTAGE_MIN_M");  // sweeps
    const int min_m = min_m_knob > 0 ? min_m_knob : 4;
    if (M >= min_m) {  // below it the mma.sync kernel stages the few rows itself
      gemv_prestage_kernel<<<M, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(A), M, K, k_blocks_of(K),
                                                  xpre, xshift);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return ret(e);
    } else {
      xpre = nullptr;
      xshift = nullptr;
    }
  }
  if (xpre) {  // activations travel in the weight ring: no staged-activation region
    // K-split for this case, measured on B200: each CTA's K range at most 64 chunks, and at least
    // 1.5 CTAs per SM (gate+up 57344 x 8192: 2 splits; 8192- and 10240-row shapes: 4).
    const int nb = n_blocks_of(N), kb = k_blocks_of(K);
    int ks = 1;
    while (ks < 8 && (ceil_div(kb, ks) > 64 || 2 * nb * ks < 3 * d->sm_count)) ks *= 2;
    static const int ks_knob = env_knob("MXFP4_GEMV_KS");
    if (ks_knob == 1 || ks_knob == 2 || ks_knob == 4 || ks_knob == 8) ks = ks_knob;
    p.ks = ks;
    p.kbps = ceil_div(kb, ks);
  }
  if (xpre)
    p.smem = p.nt == 1 ? GvCfg<1>::smem_bytes(p.stages, p.kbps, M, true) : GvCfg<2>::smem_bytes(p.stages, p.kbps, M, true);
  if (p.smem > 232448 - 1024) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (p.nt == 1)
    return c_dtype == MXFP4_DTYPE_F32 ? launch_gemv_t<1, float>(A, wpack, C, M, N, K, p, stream, d, xpre, xshift)
                                      : launch_gemv_t<1, __nv_bfloat16>(A, wpack, C, M, N, K, p, stream, d, xpre, xshift);
  return c_dtype == MXFP4_DTYPE_F32 ? launch_gemv_t<2, float>(A, wpack, C, M, N, K, p, stream, d, xpre, xshift)
                                    : launch_gemv_t<2, __nv_bfloat16>(A, wpack, C, M, N, K, p, stream, d, xpre, xshift);
}

size_t prepacked_bytes(int N, int K) {
  return static_cast<size_t>(n_blocks_of(N)) * k_blocks_of(K) * kChunkBytes;
}

int do_prepack(const uint8_t* packed, const uint8_t* scales, int N, int K, int layout, uint8_t* dst,
               cudaStream_t stream) {
  const int kb = k_blocks_of(K), nb = n_blocks_of(N);
  const long long total = static_cast<long long>(nb) * kb * 2 * kChunkRows;
  const int threads = 256;
  prepack_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0, stream>>>(
      packed, scales, N, K, layout, kb, nb, dst);
  return launch_status();
}

// ------------------------------------------------------------------ block-scaled path
inline int round_up(int x, int m) { return (x + m - 1) / m * m; }
inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Re-laid weights of the block-scaled path: nibbles [Np][Kp/2], then the scale blocks.
size_t mx_weight_data_bytes(int N, int K) {
  return static_cast<size_t>(round_up(N, kTcTileW)) * (round_up(K, kMxBK) / 2);
}
size_t mx_weight_bytes(int N, int K) {
  return mx_weight_data_bytes(N, K) + static_cast<size_t>(round_up(N, kTcTileW)) * (round_up(K, kMxBK) / kGroup);
}
// Coded activations (layout in gemm_mx.cuh): E4M3 code rows [rows][Kp], then (256-byte
// aligned) the scale blocks of rows_sf rows, then for the decode kernel (M <= 16) its fp32
// accumulation buffer [M][N].
struct MxActPlan {
  int G, rows, rows_sf, Kp;
  size_t codes_bytes, sf_bytes, acc_bytes;
  size_t sf_off() const { return codes_bytes; }
  size_t acc_off() const { return codes_bytes + align256(sf_bytes); }
  size_t total() const { return acc_off() + acc_bytes; }
};
MxActPlan mx_act_plan(int M, int N, int K, int mode) {
  MxActPlan p;
  p.Kp = round_up(K, kMxBK);
  if (M <= kMxDecodeM) {
    p.G = kMxDecodeM;
    p.rows = kGmRows;
  } else if (mode == kMxQ8) {
    p.G = 0;
    p.rows = round_up(M, kMxTileB);
  } else {
    p.G = kMxTileB / 2;
    p.rows = 2 * round_up(M, kMxTileB / 2);
  }
  p.rows_sf = round_up(p.rows, kChunkRows);
  p.codes_bytes = align256(static_cast<size_t>(p.rows) * p.Kp);
  p.sf_bytes = static_cast<size_t>(p.rows_sf) * (p.Kp / kGroup);
  p.acc_bytes = M <= kMxDecodeM ? static_cast<size_t>(M) * N * 4 : 0;
  return p;
}

int code_act_mx8(const void* A, int M, int N, int K, int mode, uint8_t* dst, bool zero_acc, cudaStream_t stream) {
  const MxActPlan p = mx_act_plan(M, N, K, mode);
  const long long work = static_cast<long long>(p.rows_sf) * (p.Kp / kGroup);
  const int threads = 256;
  float* acc = zero_acc && p.acc_bytes ? reinterpret_cast<float*>(dst + p.acc_off()) : nullptr;
  quant_act_mx8_kernel<<<static_cast<unsigned>((work + threads - 1) / threads), threads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(A), M, K, p.Kp, p.G, mode == kMxSplit2, p.rows, p.rows_sf, dst,
      dst + p.sf_off(), acc, acc ? static_cast<long long>(M) * N : 0);
  return launch_status();
}

// Launch with the programmatic-dependent-launch attribute: the kernel may start while the
// launch before it in the stream (our own producer of its inputs) runs, and waits for that
// launch with griddepcontrol.wait before it reads what the producer writes.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), int grid, int threads, int smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return ret(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

// 2-D map over 4-bit values [outer][inner] (rows of inner/2 bytes) that the TMA expands to
// 16-byte units holding 8 bytes of data, the shared-memory form of an E2M1 kind::mxf8f6f4
// operand.  inner is a multiple of 128 and the base 32-byte aligned.
int encode_2d_e2m1_expanded(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                            uint32_t box_outer) {
  auto enc = tensor_map_encoder();
  if (!enc) return MXFP4_ERR_DRIVER;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner / 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : MXFP4_ERR_DRIVER;
}

template <typename OutT, bool kSplit>
int launch_mx(const uint8_t* codes, const uint8_t* wmx, void* C, int M, int N, int K, cudaStream_t stream,
              DeviceState* d) {
  using Cfg = MxCfg<OutT>;
  const int slot = (sizeof(OutT) == 4 ? 0 : 1) + (kSplit ? 2 : 0);
  if (!d->mx_attr[slot]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_mx_kernel<OutT, kSplit>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmemBytes);
    if (e != cudaSuccess) return ret(e);
    d->mx_attr[slot] = true;
  }
  const MxActPlan p = mx_act_plan(M, N, K, kSplit ? kMxSplit2 : kMxQ8);
  const int Np = round_up(N, kTcTileW);
  CUtensorMap tm_act, tm_w, tm_out;
  int rc = encode_2d(&tm_act, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, codes, p.Kp, p.rows, kMxBK, kMxTileB,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d_e2m1_expanded(&tm_w, wmx, p.Kp, Np, kMxBK, kTcTileW);
  if (rc) return rc;
  rc = encode_2d_strided(&tm_out, sizeof(OutT) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         static_cast<int>(sizeof(OutT)), C, N, M, static_cast<uint64_t>(N) * sizeof(OutT), 32, 32);
  if (rc) return rc;
  const int m_blocks = p.rows / kMxTileB, n_blocks = Np / kTcTileW;
  return launch_pdl(gemm_mx_kernel<OutT, kSplit>, std::min(m_blocks * n_blocks, d->sm_count), kMxThreads,
                    Cfg::kSmemBytes, stream, tm_act, tm_w, tm_out, wmx + mx_weight_data_bytes(N, K),
                    codes + p.sf_off(), M, p.Kp / kMxBK, m_blocks, n_blocks);
}

// Decode (M <= 16): stream-K kernel into the zeroed fp32 buffer (C itself for fp32 output),
// then a conversion for bf16 output.
int launch_gemv_mx(const uint8_t* ws, const uint8_t* wmx, void* C, int c_dtype, int M, int N, int K,
                   cudaStream_t stream, DeviceState* d) {
  if (!d->gm_attr) {
    cudaError_t e =
        cudaFuncSetAttribute(gemv_mx_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GmCfg::kSmemBytes);
    if (e != cudaSuccess) return ret(e);
    d->gm_attr = true;
  }
  const MxActPlan p = mx_act_plan(M, N, K, kMxSplit2);
  const int Np = round_up(N, kTcTileW);
  CUtensorMap tm_w, tm_b;
  int rc = encode_2d_e2m1_expanded(&tm_w, wmx, p.Kp, Np, kMxBK, kTcTileW);
  if (rc) return rc;
  rc = encode_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws, p.Kp, kGmRows, kMxBK, kGmRows,
                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  float* acc = c_dtype == MXFP4_DTYPE_F32 ? static_cast<float*>(C)
                                          : reinterpret_cast<float*>(const_cast<uint8_t*>(ws) + p.acc_off());
  const int n_blocks = Np / kTcTileW, k_steps = p.Kp / kMxBK;
  const long long steps = static_cast<long long>(n_blocks) * k_steps;
  const int grid = static_cast<int>(std::min<long long>(d->sm_count, (steps + 3) / 4));  // >= 4 steps per CTA
  rc = launch_pdl(gemv_mx_kernel, grid, kGmThreads, GmCfg::kSmemBytes, stream, tm_w, tm_b,
                  wmx + mx_weight_data_bytes(N, K), ws + p.sf_off(), acc, M, N, n_blocks, k_steps);
  if (rc || c_dtype == MXFP4_DTYPE_F32) return rc;
  const long long n = static_cast<long long>(M) * N;
  const int blocks = static_cast<int>(std::min<long long>((n / 2 + 255) / 256, 4LL * d->sm_count));
  return launch_pdl(mx_finalize_kernel, blocks, 256, 0, stream, static_cast<const float*>(acc), n,
                    static_cast<__nv_bfloat16*>(C));
}

}  // namespace
}  // namespace mxb

using namespace mxb;

extern "C" {

int mxfp4_abi_version(void) { return MXFP4_B200_ABI_VERSION; }

int mxfp4_device_info_get(int device, mxfp4_device_info* out) {
  if (!out) return MXFP4_ERR_INVALID_ARGUMENT;
  cudaDeviceProp p;
  cudaError_t e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) return ret(e);
  std::memset(out, 0, sizeof(*out));
  std::strncpy(out->name, p.name, sizeof(out->name) - 1);
  out->major = p.major;
  out->minor = p.minor;
  out->multi_processor_count = p.multiProcessorCount;
  out->warp_size = p.warpSize;
  out->total_global_mem = static_cast<long long>(p.totalGlobalMem);
  out->shared_mem_per_block = static_cast<long long>(p.sharedMemPerBlock);
  out->shared_mem_per_block_optin = static_cast<long long>(p.sharedMemPerBlockOptin);
  out->l2_cache_size = p.l2CacheSize;
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrClockRate, device) == cudaSuccess) out->clock_rate_khz = v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMemoryClockRate, device) == cudaSuccess) out->memory_clock_rate_khz = v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrGlobalMemoryBusWidth, device) == cudaSuccess) out->memory_bus_width = v;
  return 0;
}

int mxfp4_device_error(int clear, unsigned int* code_out) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_mxfp4_error, sizeof(v));
  if (e != cudaSuccess) return ret(e);
  if (clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_mxfp4_error, &z, sizeof(z));
    if (e != cudaSuccess) return ret(e);
  }
  if (code_out) *code_out = v;
  return 0;
}

int mxfp4_test_hooks(int withhold, unsigned long long wait_limit_ns) {
  const int w = withhold ? 1 : 0;
  const unsigned long long lim = wait_limit_ns ? wait_limit_ns : kWaitLimitNs;
  cudaError_t e = cudaMemcpyToSymbol(g_mxfp4_test_withhold, &w, sizeof(w));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_mxfp4_wait_limit_ns, &lim, sizeof(lim));
  return ret(e);
}

const char* mxfp4_error_string(int code) {
  switch (code) {
    case 0: return "success";
    case MXFP4_ERR_INVALID_ARGUMENT: return "mxfp4: invalid argument";
    case MXFP4_ERR_UNSUPPORTED_SHAPE: return "mxfp4: shape not supported by the selected path";
    case MXFP4_ERR_MISALIGNED: return "mxfp4: pointer or row stride not 16-byte aligned";
    case MXFP4_ERR_WORKSPACE: return "mxfp4: workspace missing or too small";
    case MXFP4_ERR_DRIVER: return "mxfp4: tensor-map encoder unavailable or rejected the tensor";
    case MXFP4_ERR_DEVICE: return "mxfp4: current device is not an sm_100 GPU";
    case MXFP4_ERR_NOALLOC_LIMIT:
      return "mxfp4: weights need more than the 32 MiB buffer of mxfp4_gemm_noalloc (use mxfp4_gemm)";
    default: return cudaGetErrorString(static_cast<cudaError_t>(code));
  }
}

int mxfp4_quantize(const float* x, int rows, int cols, int axis, int rule, uint8_t* packed, uint8_t* scales,
                   void* stream) {
  if (!x || !packed || !scales || rows <= 0 || cols <= 0 || (axis != 0 && axis != 1) || (rule != 0 && rule != 1))
    return MXFP4_ERR_INVALID_ARGUMENT;
  const int qlen = axis == 0 ? rows : cols;
  if (qlen % kGroup) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (axis == 1 && !aligned16(x)) return MXFP4_ERR_MISALIGNED;
  if (axis == 1 && !aligned16(packed)) return MXFP4_ERR_MISALIGNED;
  auto s = static_cast<cudaStream_t>(stream);
  const long long work = static_cast<long long>(rows / (axis == 0 ? kGroup : 1)) * (cols / (axis == 0 ? 1 : kGroup));
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((work + threads - 1) / threads);
  if (axis == 0) {
    if (rule == 0) quantize_axis0_kernel<0><<<blocks, threads, 0, s>>>(x, rows, cols, packed, scales);
    else quantize_axis0_kernel<1><<<blocks, threads, 0, s>>>(x, rows, cols, packed, scales);
  } else {
    if (rule == 0) quantize_axis1_kernel<0><<<blocks, threads, 0, s>>>(x, rows, cols, packed, scales);
    else quantize_axis1_kernel<1><<<blocks, threads, 0, s>>>(x, rows, cols, packed, scales);
  }
  return launch_status();
}

int mxfp4_dequantize(const uint8_t* packed, const uint8_t* scales, int K, int N, int layout, void* out,
                     int out_dtype, void* stream) {
  if (!packed || !scales || !out || K <= 0 || N <= 0) return MXFP4_ERR_INVALID_ARGUMENT;
  if (K % kGroup) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if ((layout != MXFP4_LAYOUT_REF && layout != MXFP4_LAYOUT_NK) || (out_dtype != 0 && out_dtype != 1))
    return MXFP4_ERR_INVALID_ARGUMENT;
  auto s = static_cast<cudaStream_t>(stream);
  const long long work = static_cast<long long>(K / 2) * N;
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((work + threads - 1) / threads);
  if (layout == MXFP4_LAYOUT_REF) {
    if (out_dtype == MXFP4_DTYPE_F32)
      dequant_ref_kernel<float><<<blocks, threads, 0, s>>>(packed, scales, K, N, static_cast<float*>(out));
    else
      dequant_ref_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(packed, scales, K, N,
                                                                   static_cast<__nv_bfloat16*>(out));
  } else {
    if (out_dtype == MXFP4_DTYPE_F32)
      dequant_nk_kernel<float><<<blocks, threads, 0, s>>>(packed, scales, K, N, static_cast<float*>(out));
    else
      dequant_nk_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(packed, scales, K, N,
                                                                  static_cast<__nv_bfloat16*>(out));
  }
  return launch_status();
}

size_t mxfp4_prepacked_bytes(int N, int K) {
  if (N <= 0 || K <= 0) return 0;
  return prepacked_bytes(N, K);
}

int mxfp4_prepack(const uint8_t* packed, const uint8_t* scales, int N, int K, int src_layout, uint8_t* dst,
                  void* stream) {
  if (!packed || !scales || !dst || N <= 0 || K <= 0) return MXFP4_ERR_INVALID_ARGUMENT;
  if (src_layout != MXFP4_LAYOUT_REF && src_layout != MXFP4_LAYOUT_NK && src_layout != MXFP4_LAYOUT_G)
    return MXFP4_ERR_INVALID_ARGUMENT;
  if (K % kGroup) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (src_layout == MXFP4_LAYOUT_G && (N % 128 || K % 8)) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (!aligned16(dst)) return MXFP4_ERR_MISALIGNED;
  return do_prepack(packed, scales, N, K, src_layout, dst, static_cast<cudaStream_t>(stream));
}

int mxfp4_dequantize_prepacked(const uint8_t* wpack, int N, int K, uint16_t* out, void* stream) {
  if (!wpack || !out || N <= 0 || K <= 0) return MXFP4_ERR_INVALID_ARGUMENT;
  if (K % kGroup) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (!aligned16(wpack) || !aligned16(out)) return MXFP4_ERR_MISALIGNED;
  const int kb = k_blocks_of(K), nb = n_blocks_of(N);
  const long long total = static_cast<long long>(nb) * kb * 2 * kChunkRows;
  const int threads = 256;
  dequant_prepacked_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0,
                             static_cast<cudaStream_t>(stream)>>>(wpack, N, K, kb, nb, out);
  return launch_status();
}

int mxfp4_select_path(int M, int N, int K) {
  (void)N;
  (void)K;
  // Decode shapes are weight-streaming bound; the tcgen05 tile is 256 activation rows wide
  // and would waste >90% of its MMA work below 17 rows.
  return M <= 16 ? MXFP4_PATH_GEMV : MXFP4_PATH_TC;
}

int mxfp4_shape_supported(int path, int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || K % kGroup || N % 8) return 0;
  switch (path) {
    case MXFP4_PATH_AUTO: return 1;
    case MXFP4_PATH_TC:
    case MXFP4_PATH_TC_SMEM: return 1;
    case MXFP4_PATH_GEMV: return M <= 16 ? 1 : 0;
    default: return 0;
  }
}

size_t mxfp4_gemm_workspace_bytes(int M, int N, int K, int layout) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const size_t pre = layout == MXFP4_LAYOUT_PREPACKED ? 0 : (prepacked_bytes(N, K) + 255) / 256 * 256;
  // M <= 16: the decode path may serve the call (stream-K workspace, or the prestaged activations of
  // the other decode kernels)
  const size_t x = std::max(gemv_prestage_bytes(M, N, K), gemv_sk_bytes(M, N, K));
  DeviceState* d = nullptr;
  const size_t sk = M > 16 && current_device(&d) == 0 ? splitk_bytes(M, N, K, d->sm_count) : 0;
  return pre + std::max(x, sk);
}

// ------------------------------------------------------------------ block-scaled path
size_t mxfp4_mx_weight_bytes(int N, int K) {
  if (N <= 0 || K <= 0) return 0;
  return mx_weight_bytes(N, K);
}

int mxfp4_prepack_mx(const uint8_t* packed, const uint8_t* scales, int N, int K, int src_layout, uint8_t* dst,
                     void* stream) {
  if (!packed || !scales || !dst || N <= 0 || K <= 0) return MXFP4_ERR_INVALID_ARGUMENT;
  if (src_layout != MXFP4_LAYOUT_REF && src_layout != MXFP4_LAYOUT_NK) return MXFP4_ERR_INVALID_ARGUMENT;
  if (K % kGroup) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (reinterpret_cast<uintptr_t>(dst) & 31u) return MXFP4_ERR_MISALIGNED;
  auto s = static_cast<cudaStream_t>(stream);
  const int Np = round_up(N, kTcTileW), Kp = round_up(K, kMxBK);
  const int threads = 256;
  const long long dwork = static_cast<long long>(Np) * (Kp / 32), swork = static_cast<long long>(Np) * (Kp / kMxBK);
  const unsigned db = static_cast<unsigned>((dwork + threads - 1) / threads);
  const unsigned sb = static_cast<unsigned>((swork + threads - 1) / threads);
  uint8_t* sfa = dst + mx_weight_data_bytes(N, K);
  if (src_layout == MXFP4_LAYOUT_REF) {
    prepack_mx_data_kernel<true><<<db, threads, 0, s>>>(packed, N, K, Np, Kp, dst);
    prepack_mx_scale_kernel<true><<<sb, threads, 0, s>>>(scales, N, K, Np, Kp, sfa);
  } else {
    prepack_mx_data_kernel<false><<<db, threads, 0, s>>>(packed, N, K, Np, Kp, dst);
    prepack_mx_scale_kernel<false><<<sb, threads, 0, s>>>(scales, N, K, Np, Kp, sfa);
  }
  return launch_status();
}

size_t mxfp4_mx_workspace_bytes(int M, int N, int K, int mode) {
  if (M <= 0 || N <= 0 || K <= 0 || (mode != kMxQ8 && mode != kMxSplit2)) return 0;
  return mx_act_plan(M, N, K, mode).total();
}

int mxfp4_quantize_act_mx8(const void* A, int M, int K, int mode, uint8_t* dst, void* stream) {
  if (!A || !dst || M <= 0 || K <= 0 || (mode != kMxQ8 && mode != kMxSplit2)) return MXFP4_ERR_INVALID_ARGUMENT;
  if (K % kGroup) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (!aligned16(A) || !aligned16(dst)) return MXFP4_ERR_MISALIGNED;
  return code_act_mx8(A, M, 8, K, mode, dst, false, static_cast<cudaStream_t>(stream));
}

int mxfp4_gemm_mx(const void* A, const uint8_t* w_mx, void* C, int c_dtype, int M, int N, int K, int mode,
                  void* workspace, size_t workspace_bytes, void* stream) {
  if (!A || !w_mx || !C || M <= 0 || N <= 0 || K <= 0) return MXFP4_ERR_INVALID_ARGUMENT;
  if (c_dtype != MXFP4_DTYPE_F32 && c_dtype != MXFP4_DTYPE_BF16) return MXFP4_ERR_INVALID_ARGUMENT;
  if (mode != kMxQ8 && mode != kMxSplit2) return MXFP4_ERR_INVALID_ARGUMENT;
  if (K % kGroup || N % 8) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (!workspace || workspace_bytes < mx_act_plan(M, N, K, mode).total()) return MXFP4_ERR_WORKSPACE;
  if (!aligned16(A) || !aligned16(C) || (reinterpret_cast<uintptr_t>(w_mx) & 31u) ||
      (reinterpret_cast<uintptr_t>(workspace) & 31u))
    return MXFP4_ERR_MISALIGNED;
  DeviceState* d = nullptr;
  int rc = current_device(&d);
  if (rc) return rc;
  auto s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (M <= kMxDecodeM) {
    // the coder also zeroes the fp32 accumulation target (C itself for fp32 output)
    if (c_dtype == MXFP4_DTYPE_F32) {
      rc = ret(cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * 4, s));
      if (rc) return rc;
    }
    rc = code_act_mx8(A, M, N, K, mode, ws, c_dtype != MXFP4_DTYPE_F32, s);
    if (rc) return rc;
    return launch_gemv_mx(ws, w_mx, C, c_dtype, M, N, K, s, d);
  }
  rc = code_act_mx8(A, M, N, K, mode, ws, false, s);
  if (rc) return rc;
  if (mode == kMxSplit2)
    return c_dtype == MXFP4_DTYPE_F32 ? launch_mx<float, true>(ws, w_mx, C, M, N, K, s, d)
                                      : launch_mx<__nv_bfloat16, true>(ws, w_mx, C, M, N, K, s, d);
  return c_dtype == MXFP4_DTYPE_F32 ? launch_mx<float, false>(ws, w_mx, C, M, N, K, s, d)
                                    : launch_mx<__nv_bfloat16, false>(ws, w_mx, C, M, N, K, s, d);
}

}  // extern "C"

namespace {
int gemm_impl(const void* A, const uint8_t* B, const uint8_t* B_scales, const OutSpec& C, int c_dtype, int M, int N,
              int K, int layout, int path, void* workspace, size_t workspace_bytes, void* stream) {
  if (!A || !B || M <= 0 || N <= 0 || K <= 0) return MXFP4_ERR_INVALID_ARGUMENT;
  if (C.count < 1 || C.count > kMaxOutDst || C.n_off < 0 || C.ldc < C.n_off + N) return MXFP4_ERR_INVALID_ARGUMENT;
  const size_t esz = c_dtype == MXFP4_DTYPE_F32 ? 4 : 2;
  for (int i = 0; i < C.count; ++i) {
    if (!C.dst[i]) return MXFP4_ERR_INVALID_ARGUMENT;
    if (!aligned16(static_cast<const char*>(C.dst[i]) + C.n_off * esz) || (C.ldc * esz) % 16)
      return MXFP4_ERR_MISALIGNED;
  }
  if (c_dtype != MXFP4_DTYPE_F32 && c_dtype != MXFP4_DTYPE_BF16) return MXFP4_ERR_INVALID_ARGUMENT;
  if (layout < MXFP4_LAYOUT_REF || layout > MXFP4_LAYOUT_PREPACKED) return MXFP4_ERR_INVALID_ARGUMENT;
  if (path < MXFP4_PATH_AUTO || path > MXFP4_PATH_GEMV) return MXFP4_ERR_INVALID_ARGUMENT;
  if (layout != MXFP4_LAYOUT_PREPACKED && !B_scales) return MXFP4_ERR_INVALID_ARGUMENT;
  if (path == MXFP4_PATH_AUTO) path = mxfp4_select_path(M, N, K);
  if (!mxfp4_shape_supported(path, M, N, K)) return MXFP4_ERR_UNSUPPORTED_SHAPE;
  if (!aligned16(A) || !aligned16(B)) return MXFP4_ERR_MISALIGNED;
  DeviceState* d = nullptr;
  int rc = current_device(&d);
  if (rc) return rc;
  auto s = static_cast<cudaStream_t>(stream);
  const uint8_t* wpack = B;
  uint8_t* rest = static_cast<uint8_t*>(workspace);  // workspace left after the re-laid weights
  size_t rest_bytes = workspace ? workspace_bytes : 0;
  if (layout != MXFP4_LAYOUT_PREPACKED) {
    const size_t need = prepacked_bytes(N, K);
    if (!workspace || workspace_bytes < need) return MXFP4_ERR_WORKSPACE;
    if (!aligned16(workspace)) return MXFP4_ERR_MISALIGNED;
    if (layout == MXFP4_LAYOUT_G && N % 128) return MXFP4_ERR_UNSUPPORTED_SHAPE;
    rc = do_prepack(B, B_scales, N, K, layout, static_cast<uint8_t*>(workspace), s);
    if (rc) return rc;
    wpack = static_cast<const uint8_t*>(workspace);
    const size_t used = (need + 255) / 256 * 256;
    rest = workspace_bytes > used ? static_cast<uint8_t*>(workspace) + used : nullptr;
    rest_bytes = workspace_bytes > used ? workspace_bytes - used : 0;
  }
  switch (path) {
    case MXFP4_PATH_TC:
    case MXFP4_PATH_TC_SMEM: {
      const SplitPlan sp = plan_splitk(M, N, K, d->sm_count);
      const size_t need = static_cast<size_t>(sp.splits) * M * N * 4;
      if (sp.splits > 1 && C.count == 1 && C.n_off % 4 == 0 && C.ldc % 4 == 0 && rest && rest_bytes >= need &&
          aligned16(rest)) {
        float* ws = reinterpret_cast<float*>(rest);
        return path == MXFP4_PATH_TC ? launch_tc_splitk<true>(A, wpack, C, c_dtype, M, N, K, sp, ws, s, d)
                                     : launch_tc_splitk<false>(A, wpack, C, c_dtype, M, N, K, sp, ws, s, d);
      }
      break;
    }
    default:
      break;
  }
  switch (path) {
    case MXFP4_PATH_TC:
      return c_dtype == MXFP4_DTYPE_F32 ? launch_tc<true, float>(A, wpack, C, M, N, K, s, d)
                                        : launch_tc<true, __nv_bfloat16>(A, wpack, C, M, N, K, s, d);
    case MXFP4_PATH_TC_SMEM:
      return c_dtype == MXFP4_DTYPE_F32 ? launch_tc<false, float>(A, wpack, C, M, N, K, s, d)
                                        : launch_tc<false, __nv_bfloat16>(A, wpack, C, M, N, K, s, d);
    case MXFP4_PATH_GEMV: return launch_gemv(A, wpack, C, c_dtype, M, N, K, s, d, rest, rest_bytes);
    default: return MXFP4_ERR_INVALID_ARGUMENT;
  }
}
}  // namespace

extern "C" {

int mxfp4_gemm(const void* A, const uint8_t* B, const uint8_t* B_scales, void* C, int c_dtype, int M, int N,
               int K, int layout, int path, void* workspace, size_t workspace_bytes, void* stream) {
  if (!C) return MXFP4_ERR_INVALID_ARGUMENT;
  void* dst[1] = {C};
  const OutSpec o{dst, 1, N, 0, 0};
  return gemm_impl(A, B, B_scales, o, c_dtype, M, N, K, layout, path, workspace, workspace_bytes, stream);
}

int mxfp4_gemm_allgather(const void* A, const uint8_t* B_prepacked, void* const* C_dst, int n_dst, int n_off,
                         int ldc, int c_dtype, int M, int N, int K, int path, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (!C_dst || n_dst < 1 || n_dst > kMaxOutDst) return MXFP4_ERR_INVALID_ARGUMENT;
  const OutSpec o{C_dst, n_dst, ldc, n_off, 1};
  return gemm_impl(A, B_prepacked, nullptr, o, c_dtype, M, N, K, MXFP4_LAYOUT_PREPACKED, path, workspace,
                   workspace_bytes, stream);
}

size_t mxfp4_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int mxfp4_ipc_export(const void* dev_ptr, void* handle_out, size_t* offset_out) {
  if (!dev_ptr || !handle_out || !offset_out) return MXFP4_ERR_INVALID_ARGUMENT;
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  if (!range_fn) return MXFP4_ERR_DRIVER;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return MXFP4_ERR_DRIVER;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return ret(e);
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uintptr_t>(dev_ptr) - static_cast<uintptr_t>(base);
  return 0;
}

int mxfp4_ipc_open(const void* handle, size_t offset, void** dev_ptr_out) {
  if (!handle || !dev_ptr_out) return MXFP4_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return ret(e);
  *dev_ptr_out = static_cast<char*>(base) + offset;
  return 0;
}

int mxfp4_ipc_close(void* dev_ptr, size_t offset) {
  if (!dev_ptr) return MXFP4_ERR_INVALID_ARGUMENT;
  return ret(cudaIpcCloseMemHandle(static_cast<char*>(dev_ptr) - offset));
}

int mxfp4_copy_columns(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width_bytes,
                       int rows, void* stream) {
  if (!dst || !src || rows < 0 || width_bytes > dst_pitch || width_bytes > src_pitch)
    return MXFP4_ERR_INVALID_ARGUMENT;
  if (rows == 0 || width_bytes == 0) return 0;
  // One pitched copy on the stream: the copy engines move it (a peer's buffer goes over NVLink),
  // no SM takes part, so it runs beside the kernels of other streams.
  return ret(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width_bytes, static_cast<size_t>(rows),
                               cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)));
}


}  // extern "C"

// ---------------------------------------------------------------------------------------
// Allocation-free variant of mxfp4_gemm for callers that may not allocate device memory.
// The library carries its own buffer for the re-laid weights.  Host code only knows the
// array by its host-side symbol, so the device address is looked up once per device (with
// that device current) and cached; the kernels then get that address like any workspace.
// The prepack writes every byte of the region the GEMM reads, so nothing in the buffer has
// to be cleared between calls; concurrent calls share it and must not overlap on the GPU.
namespace mxb {
namespace {
static __device__ __align__(256) uint8_t g_noalloc_scratch[MXFP4_NOALLOC_SCRATCH_BYTES];
void* g_noalloc_ptr[kMaxDevices];
std::mutex g_noalloc_mu;

int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ret(e);
  if (dev < 0 || dev >= kMaxDevices) return MXFP4_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return ret(e);
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}
}  // namespace
}  // namespace mxb

extern "C" int mxfp4_gemm_noalloc(const void* A, const uint8_t* B, const uint8_t* B_scales, void* C, int c_dtype,
                                  int M, int N, int K, int layout, int path, void* stream) {
  if (layout != MXFP4_LAYOUT_REF && layout != MXFP4_LAYOUT_NK && layout != MXFP4_LAYOUT_G)
    return MXFP4_ERR_INVALID_ARGUMENT;  // prepacked weights need no buffer: call mxfp4_gemm
  if (N <= 0 || K <= 0) return MXFP4_ERR_INVALID_ARGUMENT;
  const size_t need = mxb::prepacked_bytes(N, K);
  if (need > MXFP4_NOALLOC_SCRATCH_BYTES) return MXFP4_ERR_NOALLOC_LIMIT;
  void* scratch = nullptr;
  const int rc = mxb::noalloc_scratch(&scratch);
  if (rc) return rc;
  return mxfp4_gemm(A, B, B_scales, C, c_dtype, M, N, K, layout, path, scratch, MXFP4_NOALLOC_SCRATCH_BYTES,
                    stream);
}
