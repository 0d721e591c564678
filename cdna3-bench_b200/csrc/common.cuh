// Shared device helpers for the MXFP4 x BF16 library (sm_100a only).
//
// * PTX wrappers: mbarrier, TMA / bulk copies, tcgen05 (TMEM alloc, MMA, ld/st).
// * Bounded waits: every spin on an mbarrier gives up after kWaitLimitNs,
//   records an error code in g_mxfp4_error and tells the caller to unwind.
// * Exact E2M1 x E8M0 -> BF16 dequantisation used by the GEMM kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library targets sm_100a only"
#endif

namespace mxb {

// ---- format constants --------------------------------------------------------------
constexpr int kGroup = 32;          // elements per E8M0 scale
constexpr int kChunkRows = 128;     // weight rows (output columns) per prepacked chunk
constexpr int kChunkK = 64;         // K elements per prepacked chunk
constexpr int kChunkData = kChunkRows * kChunkK / 2;                     // 4096 B of nibbles
constexpr int kChunkBytes = kChunkData + kChunkRows * (kChunkK / kGroup);  // + 256 B scales

// Chunk byte layout.  Word t (bytes b = 0..3 hold k-pairs t + 4b of the group) of row r's
// 32-group grp sits at word 2*grp + (r/8)%2 of 16-byte unit chunk_unit(r, t): one unit holds
// the four A-fragment words lane (g = r%8, t) of an m16n8k16 MMA needs for rows 16*(r/16) .. +15
// and both groups.  Inside each 32-unit block (rows 16a .. 16a+15) unit (k = r%8, t) sits at
// position 8t + ((k + 2t) mod 8), so that both access patterns are free of shared-memory bank
// conflicts: the decode kernel's 8-lane phases (k in {2p, 2p+1}, t = 0..3) and the large-M
// kernel's (k = 0..7, one t) each touch 8 different 16-byte bank groups.  The scales follow the
// data, four to a 4-byte unit 8*(r/16) + r%8.
__host__ __device__ constexpr int chunk_unit(int r, int t) {
  return 32 * (r >> 4) + 8 * t + (((r & 7) + 2 * t) & 7);
}
__host__ __device__ constexpr int chunk_word_off(int r, int grp, int t) {
  return chunk_unit(r, t) * 16 + (2 * grp + ((r >> 3) & 1)) * 4;
}
__host__ __device__ constexpr int chunk_scale_off(int r, int grp) {
  return kChunkData + 4 * (8 * (r >> 4) + (r & 7)) + 2 * grp + ((r >> 3) & 1);
}

// ---- device error word -------------------------------------------------------------
// First non-zero code wins; the host reads and clears it with mxfp4_device_error().
enum DeviceError : unsigned {
  kErrNone = 0,
  kErrWaitFull = 0x101,      // consumer gave up waiting for a stage to be filled
  kErrWaitEmpty = 0x102,     // producer gave up waiting for a stage to be released
  kErrWaitDequant = 0x103,   // MMA issuer gave up waiting for dequantised weights
  kErrWaitAccFull = 0x104,   // epilogue gave up waiting for the accumulator
  kErrWaitAccEmpty = 0x105,  // MMA issuer gave up waiting for the epilogue
  kErrWaitDrain = 0x106,     // unwinding after an abort took too long
};

__device__ unsigned int g_mxfp4_error;

__device__ __forceinline__ void record_error(unsigned code) { atomicCAS(&g_mxfp4_error, 0u, code); }

constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s, the default limit

// Limit of every bounded wait (kWaitLimitNs unless a test lowers it with mxfp4_test_hooks) and a
// test switch that makes the weight producers of gemm_tc_kernel and gemv_kernel issue no copies,
// so that their consumers' waits run out: the abort path is exercised without any fault.
__device__ unsigned long long g_mxfp4_wait_limit_ns = kWaitLimitNs;
__device__ int g_mxfp4_test_withhold;

__device__ __forceinline__ unsigned long long wait_limit_ns() {
  return *static_cast<volatile unsigned long long*>(&g_mxfp4_wait_limit_ns);
}
__device__ __forceinline__ bool test_withhold() { return *static_cast<volatile int*>(&g_mxfp4_test_withhold) != 0; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ----------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity of `bar` has completed.  Gives up after
// kWaitLimitNs, or as soon as another role of the CTA has raised *abort; on its own
// timeout it records `code` and raises *abort.  Returns false when the caller must unwind.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code,
                                          volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = globaltimer();
  const unsigned long long limit = wait_limit_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(a, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > limit) {
      record_error(code);
      *abort = 1;
      return false;
    }
  }
}

// Warp-uniform wait: every lane polls, and the warp proceeds only if all lanes saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, unsigned code, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, code, abort);
  return __all_sync(0xffffffffu, ok);
}

// Bounded wait used only while unwinding: no abort check, short limit.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const unsigned long long t0 = globaltimer();
  const unsigned long long limit = wait_limit_ns() / 4 + 1000000ull;
  while (!mbar_try_wait(a, parity)) {
    if (globaltimer() - t0 > limit) {
      record_error(kErrWaitDrain);
      return;
    }
  }
}

// ---- explicit shared-memory accesses (32-bit shared addresses) -----------------------
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts16(uint32_t a, uint32_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"(static_cast<unsigned short>(v)) : "memory");
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// ---- bulk / tensor copies ----------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// Programmatic dependent launch: a launch made with the programmatic-serialisation attribute
// may start before the previous launch in its stream has finished; griddep_wait() blocks
// until that launch has completed and its writes are visible.  griddep_launch_dependents()
// lets the next such launch start early.  Both are no-ops for ordinary launches.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Barrier over `nthreads` threads that also ANDs a predicate across them: every thread gets
// true only if all of them passed true.  Lets warps that share a later barrier agree on
// leaving a loop, so that none is left waiting at it.
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n"
      " .reg .pred p, q;\n"
      " setp.ne.u32 p, %1, 0;\n"
      " bar.red.and.pred q, %2, %3, p;\n"
      " selp.u32 %0, 1, 0, q;\n"
      "}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// ---- tcgen05 -----------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (bf16 inputs, f32 accumulate)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
        "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
        "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// UMMA shared-memory descriptor for a K-major operand laid out with the 128-byte swizzle
// (rows of 128 B, 8-row atoms of 1024 B; the tile base must be 1024-byte aligned).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // [0,14) start address >> 4
  d |= static_cast<uint64_t>(1) << 16;                       // [16,30) LBO (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;               // [32,46) SBO: 8-row atom stride
  d |= static_cast<uint64_t>(1) << 46;                       // [46,48) descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                       // [61,64) SWIZZLE_128B
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 x bf16 -> f32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4)                                   // D format f32
         | (1u << 7)                                 // A format bf16
         | (1u << 10)                                // B format bf16
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// ---- exact dequantisation -----------------------------------------------------------
// The reference decodes a nibble as (+-)E2M1[em] * 2**(scale-127) in fp32.  Every such
// product is exactly representable in bf16 (two significant bits, exponent range of fp32),
// so the bf16 value is exact.  We build, per (row, 32-element group), an 8-entry bf16 table
// of E2M1 magnitudes times the group scale (computed in fp32 with IEEE semantics: 2**-127 is
// a subnormal, scale byte 255 is +inf, 0*inf is NaN exactly like NumPy), split into a
// low-byte table and a high-byte table, and look nibbles up with byte permutes.

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// 2**(s-127) as fp32 (s == 0 is the subnormal 2**-127; s == 255 gives +inf).
__device__ __forceinline__ float e8m0_to_f32(uint32_t s) {
  return __uint_as_float(s == 0 ? 0x00400000u : (s << 23));
}

struct Bf16Lut {
  uint32_t lo0, lo1, hi0, hi1;  // byte tables: lo0 = low bytes of entries 0..3, etc.
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ Bf16Lut make_lut(uint32_t scale_byte) {
  const float sc = e8m0_to_f32(scale_byte);
  const uint32_t p0 = pack_bf16x2(0.0f * sc, 0.5f * sc);
  const uint32_t p1 = pack_bf16x2(sc, 1.5f * sc);
  const uint32_t p2 = pack_bf16x2(2.0f * sc, 3.0f * sc);
  const uint32_t p3 = pack_bf16x2(4.0f * sc, 6.0f * sc);
  Bf16Lut t;
  t.lo0 = prmt(p0, p1, 0x6420);
  t.hi0 = prmt(p0, p1, 0x7531);
  t.lo1 = prmt(p2, p3, 0x6420);
  t.hi1 = prmt(p2, p3, 0x7531);
  return t;
}

// 8 nibbles (one 32-bit word, nibble i at bits 4i..4i+3) -> 4 bf16x2 words; output word j
// holds the two values of byte j (low nibble in the low half).
__device__ __forceinline__ void dequant8(uint32_t p, const Bf16Lut& t, uint32_t (&o)[4]) {
  const uint32_t c0 = p & 0x7777u;          // magnitude indices of nibbles 0..3
  const uint32_t c1 = (p >> 16) & 0x7777u;  // ... of nibbles 4..7
  const uint32_t q = p << 4;
  const uint32_t sa = prmt(q, p, 0x5140);   // byte i: bit 7 = sign of nibble i (0..3)
  const uint32_t sb = prmt(q, p, 0x7362);   // ... nibbles 4..7
  const uint32_t lo_a = prmt(t.lo0, t.lo1, c0);
  const uint32_t lo_b = prmt(t.lo0, t.lo1, c1);
  const uint32_t hi_a = prmt(t.hi0, t.hi1, c0) | (sa & 0x80808080u);
  const uint32_t hi_b = prmt(t.hi0, t.hi1, c1) | (sb & 0x80808080u);
  o[0] = prmt(lo_a, hi_a, 0x5140);
  o[1] = prmt(lo_a, hi_a, 0x7362);
  o[2] = prmt(lo_b, hi_b, 0x5140);
  o[3] = prmt(lo_b, hi_b, 0x7362);
}

// One prepacked row-group (16 bytes = 32 elements, word w holds k-pairs w, w+4, w+8, w+12)
// -> 16 bf16x2 words in k-pair order.
__device__ __forceinline__ void dequant_rowgroup(const uint4 d, uint32_t scale_byte, uint32_t (&out)[16]) {
  const Bf16Lut t = make_lut(scale_byte);
  const uint32_t w[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t o[4];
    dequant8(w[i], t, o);
#pragma unroll
    for (int b = 0; b < 4; ++b) out[i + 4 * b] = o[b];
  }
}

// Eight E2M1 values (4 bytes, low nibble of each byte first) -> 4 f16x2 words, exact and
// unscaled; o[j] holds the two values of byte j.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace mxb
