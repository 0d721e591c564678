// Block-scaled GEMMs: MXFP4 weights x MXFP8-coded activations on tcgen05 kind::mxf8f6f4.
//
// C[M, N] = A' * W^T where W stays MXFP4 (E2M1 elements, one E8M0 scale per 32 k) and A' is
// the bf16 activations coded as E4M3 pieces with one E8M0 scale per 32 k of a row.  The tensor
// core applies both operands' scales itself (block_scale): nothing is dequantised in software
// and the MMA runs at the 8-bit rate.  Two codings (the `mode` of the entry points):
//   MX_Q8     one piece, the OCP MX rule: scale exponent floor(log2(amax)) - 8, elements
//             rounded to nearest even and saturated at 448.  The activations keep 4
//             significant bits.
//   MX_SPLIT2 two pieces A ~ hi + lo: hi with exponent floor(log2(amax)) - 7 (the group max
//             lands in [128, 256), nothing saturates), lo the same rule applied to the exact
//             residual A - hi.  Every element is then within 2**-8 of its group's max of A:
//             about bf16's own resolution, and the GEMM stays far inside the 1e-2 bar.  The
//             two pieces are stacked as extra B-operand rows, so one MMA computes both
//             products and the epilogue adds them.
// Both differ from the exact path of gemm_large.cuh, so these are separate entry points whose
// reference is (sum of the dequantised pieces) @ dequant(W) in fp32.
//
// HBM layouts (built by kernels in this file):
//   * weights (prepack_mx_*_kernel): nibbles [Np][Kp/2], K contiguous, low nibble = even k;
//     Np = N rounded up to 128, Kp = K rounded up to 128, zero padded.  Scales in 512-byte
//     blocks [Np/128][Kp/128]; inside a block, byte 16*(r%32) + 4*(r/32) + j holds row r's
//     scale for 32-k group j of the 128-k step (padding: 127).
//   * activation codes (quant_act_mx8_kernel): E4M3 [rows][Kp].  Row b holds piece p of
//     activation row m, b = (m / G) * 2G + p * G + m % G for a G-row stacking group, or b = m
//     (G = 0, one piece):  M <= 16 (decode kernel): G = 16, 32 rows (lo rows zero for MX_Q8);
//     M > 16 MX_Q8: G = 0, M rounded up to 256 rows; M > 16 MX_SPLIT2: G = 128,
//     2 * (M rounded up to 128) rows.  Scales in blocks [Kp/128][rows/128 rounded up], same
//     in-block order; padding rows and groups are all-zero groups (scale byte 0).
// The in-block order is what tcgen05.cp .32x128b.warpx4 expects: 16-byte row r%32 goes to
// TMEM lane r%32 (copied to all four lane quarters), its 4-byte word r/32 to a column, and
// byte j is the scale the MMA of k-step j selects (scale-factor id j).
//
// Large-M kernel (gemm_mx_kernel): persistent CTAs (one per SM), tile = 128 weight rows x 256
// code rows (256 activation rows, or 128 in both pieces), 128 k per pipeline stage (four MMAs
// of K = 32), accumulator 128 lanes x 256 f32 columns of TMEM.
//   warp 0    TMA producer: code tile (256 rows x 128 B, 128-byte swizzle), weight tile
//             (128 rows x 128 nibbles, expanded by the TMA to 16-byte units holding 8 bytes of
//             data each, the operand form kind::mxf8f6f4 reads for E2M1; 128-byte swizzle), and
//             the stage's two scale blocks by bulk copy;
//   warp 1    TMEM owner and MMA issuer: copies the stage's scales into TMEM, then issues the
//             four block-scaled MMAs; tcgen05 copies and MMAs of one thread run in issue order,
//             so the next stage's scale copy cannot overtake this stage's MMAs;
//   warps 2-9 epilogue: tcgen05.ld (MX_SPLIT2: both pieces' columns, added), release the
//             accumulator, 32 x 32 slabs stored by TMA.
// Decode kernel (gemv_mx_kernel, M <= 16): stream-K over (128-row weight block, 128-k step)
// pairs, one CTA per SM with an equal share; MMA N = 32 code rows; a CTA adds each finished
// weight block's partial sums into an fp32 buffer with global atomics.
// Every wait is bounded (common.cuh); every CTA loads its own tiles.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "gemm_large.cuh"
#include "quant.cuh"

namespace mxb {

constexpr int kMxBK = 128;                              // k per pipeline stage
constexpr int kMxThreads = 32 * (2 + kTcEpiWarps);      // 320
constexpr int kMxTileB = 256;                           // code rows per large-M tile (UMMA N)
constexpr uint32_t kMxSfaCol = 256;                     // 4 TMEM columns: weight scales
constexpr uint32_t kMxSfbCol = 264;                     // 8 TMEM columns: code-row scales
constexpr int kMxSfBlock = 512;                         // 128 rows x 4 groups of scale bytes
constexpr int kMxDecodeM = 16;                          // decode kernel: M <= 16
constexpr int kMxQ8 = 0, kMxSplit2 = 1;

template <typename OutT>
struct MxCfg {
  static constexpr int kStages = sizeof(OutT) == 2 ? 4 : 3;
  static constexpr int kActBytes = kMxTileB * kMxBK;        // 32 KiB of E4M3
  static constexpr int kWBytes = kTcTileW * kMxBK;          // 16 KiB: 128 nibbles per row, expanded
  static constexpr int kWTxBytes = kTcTileW * kMxBK / 2;    // bytes the weight load transfers
  static constexpr int kSfaBytes = kMxSfBlock;
  static constexpr int kSfbBytes = 2 * kMxSfBlock;
  static constexpr int kSlabBytes = 32 * 32 * static_cast<int>(sizeof(OutT));
  static constexpr int kOffW = kStages * kActBytes;
  static constexpr int kOffSfa = kOffW + kStages * kWBytes;
  static constexpr int kOffSfb = kOffSfa + kStages * kSfaBytes;
  static constexpr int kOffOut = kOffSfb + kStages * kSfbBytes;
  static constexpr int kOffBar = kOffOut + kTcEpiWarps * kSlabBytes;
  static constexpr int kNumBars = 2 * kStages + 2;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + slack for 1024-byte alignment
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kOffOut % 128 == 0, "TMA store sources are 128-byte aligned");
};

// Instruction descriptor of tcgen05.mma kind::mxf8f6f4.block_scale: A = E2M1 (weights),
// B = E4M3 (activation codes), both K-major, E8M0 scales, f32 accumulator.  The scale-factor
// ids (bits 4-5 for B, 29-30 for A) are or-ed in per k-step.
__host__ __device__ constexpr uint32_t umma_idesc_mx(int m, int n) {
  return (5u << 7)                                   // A format E2M1
         | (0u << 10)                                // B format E4M3
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (1u << 23)                                // scale format E8M0
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

__device__ __forceinline__ void mma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Shared-memory descriptor of a 512-byte scale block for tcgen05.cp .32x128b: 32 rows of 16
// bytes, no swizzle, 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t sf_block_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // [0,14) start address >> 4
  d |= static_cast<uint64_t>(128 >> 4) << 16;                // [16,30) LBO
  d |= static_cast<uint64_t>(128 >> 4) << 32;                // [32,46) SBO: next 8 rows
  d |= static_cast<uint64_t>(1) << 46;                       // [46,48) descriptor version (sm_100)
  return d;                                                  // [61,64) = 0: no swizzle
}

__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// The four block-scaled MMAs of one 128-k stage (k-step j: 32 k = 32 bytes of both operand
// rows; scale byte j of each TMEM scale word).
__device__ __forceinline__ void mma_mx_stage(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t sfa_tmem, uint32_t sfb_tmem, bool first) {
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j)
    mma_mx(d_tmem, adesc + 2 * j, bdesc + 2 * j, idesc | (j << 29) | (j << 4), sfa_tmem | (j << 30),
           sfb_tmem | (j << 30), !(first && j == 0));
}

// Byte offset of (row r of a 128-row block, 32-k group j of a 128-k step) inside a scale block.
__host__ __device__ constexpr int mx_sf_in_block(int r, int j) { return 16 * (r & 31) + 4 * ((r >> 5) & 3) + j; }

// Stores 32 rows x 32 columns (float values v[j] = row mc + j, this lane's column n0 + lane)
// through the warp's staging slab with one TMA store.
template <typename OutT>
__device__ __forceinline__ void mx_store_slab(const CUtensorMap* map, uint8_t* stage_ptr, const float (&v)[32],
                                              int n0, int mc, int lane) {
  const uint32_t stage = smem_u32(stage_ptr);
  if (lane == 0) bulk_wait_read<0>();  // the previous store has read the buffer
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if constexpr (sizeof(OutT) == 2)
      sts16(stage + (j * 32 + lane) * 2, pack_bf16x2(v[j], 0.0f) & 0xFFFFu);
    else
      sts32(stage + (j * 32 + lane) * 4, __float_as_uint(v[j]));
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, stage_ptr, n0, mc);
    bulk_commit();
  }
}

template <typename OutT, bool kSplit>
__global__ void __launch_bounds__(kMxThreads, 1)
    gemm_mx_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_out, const uint8_t* __restrict__ sfa,
                   const uint8_t* __restrict__ sfb, int M, int k_steps, int m_blocks, int n_blocks) {
  using Cfg = MxCfg<OutT>;
  constexpr int S = Cfg::kStages;
  constexpr int kActRows = kSplit ? kMxTileB / 2 : kMxTileB;  // activation rows per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total = m_blocks * n_blocks;
  const int sf_rows = 2 * m_blocks;  // 128-row scale blocks per k-step of the codes

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kTcEpiWarps);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_act);
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, pend = 0, pend_ph = 0;
      bool aborted = false, coded = false;
      for (int t = blockIdx.x; t < total && !aborted; t += gridDim.x) {
        int mb, nb;
        tc_tile_coords(t, m_blocks, n_blocks, mb, nb);
        for (int kt = 0; kt < k_steps; ++kt) {
          if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
            aborted = true;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kActBytes + Cfg::kWTxBytes + Cfg::kSfaBytes + Cfg::kSfbBytes);
          tma_load_2d(smem + Cfg::kOffW + s * Cfg::kWBytes, &tm_w, &full[s], kt * kMxBK, nb * kTcTileW);
          bulk_load(smem + Cfg::kOffSfa + s * Cfg::kSfaBytes,
                    sfa + (static_cast<size_t>(nb) * k_steps + kt) * kMxSfBlock, Cfg::kSfaBytes, &full[s]);
          if (!coded) {  // the codes come from the coder launched just before (PDL)
            griddep_wait();
            coded = true;
          }
          tma_load_2d(smem + s * Cfg::kActBytes, &tm_act, &full[s], kt * kMxBK, mb * kMxTileB);
          bulk_load(smem + Cfg::kOffSfb + s * Cfg::kSfbBytes,
                    sfb + (static_cast<size_t>(kt) * sf_rows + 2 * mb) * kMxSfBlock, Cfg::kSfbBytes, &full[s]);
          pend |= 1u << s;
          pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (aborted) {  // let every copy we started land before the CTA can exit
        for (int i = 0; i < S; ++i)
          if ((pend >> i) & 1) mbar_wait_drain(&full[i], (pend_ph >> i) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_mx(kTcTileW, kMxTileB);
      int s = 0;
      uint32_t ph = 0, aph = 0;
      bool aborted = false, issued = false;
      for (int t = blockIdx.x; t < total && !aborted; t += gridDim.x) {
        if (!mbar_wait(acc_empty, aph ^ 1, kErrWaitAccEmpty, abort_flag)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        for (int kt = 0; kt < k_steps; ++kt) {
          if (!mbar_wait(&full[s], ph, kErrWaitFull, abort_flag)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t sfa_s = smem_u32(smem + Cfg::kOffSfa + s * Cfg::kSfaBytes);
          const uint32_t sfb_s = smem_u32(smem + Cfg::kOffSfb + s * Cfg::kSfbBytes);
          tmem_cp_sf(tmem + kMxSfaCol, sf_block_desc(sfa_s));
          tmem_cp_sf(tmem + kMxSfbCol, sf_block_desc(sfb_s));
          tmem_cp_sf(tmem + kMxSfbCol + 4, sf_block_desc(sfb_s + kMxSfBlock));
          mma_mx_stage(tmem + kTmemAccCol, umma_desc_sw128(smem_u32(smem + Cfg::kOffW + s * Cfg::kWBytes)),
                       umma_desc_sw128(smem_u32(smem + s * Cfg::kActBytes)), idesc, tmem + kMxSfaCol,
                       tmem + kMxSfbCol, kt == 0);
          issued = true;
          tc_commit(&empty[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        if (aborted) break;
        tc_commit(acc_full);
        aph ^= 1;
      }
      if (aborted && issued) {  // wait for the MMAs already issued before TMEM is released
        tc_commit(acc_full);
        mbar_wait_drain(acc_full, aph);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp (q, hh): TMEM lane quarter q = output columns n0 .. n0+31; hh picks its half of the
    // tile's activation rows (MX_SPLIT2: 64 rows, read from the hi columns and the lo columns
    // 128 further; MX_Q8: 128 rows).
    const int q = warp & 3;
    const int ew = warp - 2;
    const int hh = ew >> 2;
    uint8_t* stage_ptr = smem + Cfg::kOffOut + ew * Cfg::kSlabBytes;
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int mb, nb;
      tc_tile_coords(t, m_blocks, n_blocks, mb, nb);
      if (!warp_wait(acc_full, aph, kErrWaitAccFull, abort_flag)) break;
      tc_fence_after();
      const int n0 = nb * kTcTileW + 32 * q;
      const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q) << 16) + kTmemAccCol;
      if constexpr (kSplit) {
        const int m0 = mb * kActRows + 64 * hh;
        float v[2][32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t a[32], b[32];
          tmem_ld32(tq + 64 * hh + 32 * c, a);
          tmem_ld32(tq + 128 + 64 * hh + 32 * c, b);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[c][j] = __uint_as_float(a[j]) + __uint_as_float(b[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);  // accumulator free: the next tile's MMAs start
#pragma unroll
        for (int c = 0; c < 2; ++c)
          if (m0 + 32 * c < M) mx_store_slab<OutT>(&tm_out, stage_ptr, v[c], n0, m0 + 32 * c, lane);
      } else if constexpr (sizeof(OutT) == 2) {
        // bf16: all 128 columns into registers as bf16 pairs, release, then store
        const int m0 = mb * kActRows + 128 * hh;
        uint32_t packed[64];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t a[16];
          tmem_ld16(tq + 128 * hh + 16 * c, a);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            packed[8 * c + j] = pack_bf16x2(__uint_as_float(a[2 * j]), __uint_as_float(a[2 * j + 1]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);
        const uint32_t stage = smem_u32(stage_ptr);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int mc = m0 + 32 * c;
          if (mc < M) {
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint32_t pk = packed[16 * c + j];
              sts16(stage + ((2 * j) * 32 + lane) * 2, pk & 0xFFFFu);
              sts16(stage + ((2 * j + 1) * 32 + lane) * 2, pk >> 16);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tm_out, stage_ptr, n0, mc);
              bulk_commit();
            }
          }
        }
      } else {
        // f32: 32-column chunks, the accumulator released after the last load
        const int m0 = mb * kActRows + 128 * hh;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t a[32];
          tmem_ld32(tq + 128 * hh + 32 * c, a);
          tmem_wait_ld();
          if (c == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
          }
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(a[j]);
          if (m0 + 32 * c < M) mx_store_slab<OutT>(&tm_out, stage_ptr, v, n0, m0 + 32 * c, lane);
        }
      }
      aph ^= 1;
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------
// Decode kernel, M <= 16.  Work = every (128-row weight block nb, 128-k step kt) pair in
// nb-major order; CTA c takes the contiguous share [c*T/G, (c+1)*T/G).  A run of steps with
// one nb is a segment: its MMAs accumulate into one of two TMEM buffers (N = 32 code rows:
// 16 hi + 16 lo), and at the segment's end the four epilogue warps add hi + lo of each row
// m < M into ws[m][n] (fp32, zeroed before the launch) with atomics, while the MMAs of the
// next segment run into the other buffer.
// Warps: 0 TMA producer, 1 MMA issuer (+TMEM owner), 2..5 epilogue (one per lane quarter).
// ------------------------------------------------------------------------------------
constexpr int kGmRows = 2 * kMxDecodeM;  // code rows of the decode operand
constexpr int kGmStages = 8;
constexpr int kGmThreads = 32 * 6;
constexpr uint32_t kGmTmemCols = 128;     // two 32-column accumulators, then the scales
constexpr uint32_t kGmSfaCol = 64, kGmSfbCol = 72;

struct GmCfg {
  static constexpr int kWBytes = kTcTileW * kMxBK;        // 16 KiB (expanded E2M1)
  static constexpr int kWTxBytes = kTcTileW * kMxBK / 2;  // 8 KiB transferred
  static constexpr int kBBytes = kGmRows * kMxBK;         // 4 KiB of E4M3
  static constexpr int kOffB = kGmStages * kWBytes;
  static constexpr int kOffSfa = kOffB + kGmStages * kBBytes;
  static constexpr int kOffSfb = kOffSfa + kGmStages * kMxSfBlock;
  static constexpr int kOffBar = kOffSfb + kGmStages * kMxSfBlock;
  static constexpr int kNumBars = 2 * kGmStages + 4;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kOffB % 1024 == 0 && kBBytes % 1024 == 0, "128-byte-swizzled tiles are 1024-byte aligned");
};

// Segment of the stream-K share that starts at step s: its weight block and end step.
__device__ __forceinline__ void gm_segment(long long s, long long s1, int k_steps, int& nb, long long& end) {
  nb = static_cast<int>(s / k_steps);
  end = min(s1, static_cast<long long>(nb + 1) * k_steps);
}

__global__ void __launch_bounds__(kGmThreads, 1)
    gemv_mx_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_b,
                   const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb, float* __restrict__ ws,
                   int M, int N, int n_blocks, int k_steps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GmCfg::kOffBar);
  uint64_t* empty = full + kGmStages;
  uint64_t* acc_full = empty + kGmStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + GmCfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + GmCfg::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  griddep_launch_dependents();  // the bf16 conversion launched after this waits for it anyway
  const long long total = static_cast<long long>(n_blocks) * k_steps;
  const long long s0 = total * blockIdx.x / gridDim.x;
  const long long s1 = total * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kGmTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0, pend = 0, pend_ph = 0;
      bool coded = false;
      for (long long s = s0; s < s1; ++s) {
        const int nb = static_cast<int>(s / k_steps), kt = static_cast<int>(s % k_steps);
        if (!mbar_wait(&empty[st], ph ^ 1, kErrWaitEmpty, abort_flag)) {
          for (int i = 0; i < kGmStages; ++i)  // let every copy we started land before exiting
            if ((pend >> i) & 1) mbar_wait_drain(&full[i], (pend_ph >> i) & 1);
          break;
        }
        mbar_arrive_expect_tx(&full[st], GmCfg::kWTxBytes + GmCfg::kBBytes + 2 * kMxSfBlock);
        tma_load_2d(smem + st * GmCfg::kWBytes, &tm_w, &full[st], kt * kMxBK, nb * kTcTileW);
        bulk_load(smem + GmCfg::kOffSfa + st * kMxSfBlock, sfa + (static_cast<size_t>(nb) * k_steps + kt) * kMxSfBlock,
                  kMxSfBlock, &full[st]);
        if (!coded) {  // the codes come from the coder launched just before (PDL)
          griddep_wait();
          coded = true;
        }
        tma_load_2d(smem + GmCfg::kOffB + st * GmCfg::kBBytes, &tm_b, &full[st], kt * kMxBK, 0);
        bulk_load(smem + GmCfg::kOffSfb + st * kMxSfBlock, sfb + static_cast<size_t>(kt) * kMxSfBlock, kMxSfBlock,
                  &full[st]);
        pend |= 1u << st;
        pend_ph = (pend_ph & ~(1u << st)) | (ph << st);
        if (++st == kGmStages) {
          st = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_mx(kTcTileW, kGmRows);
      int st = 0, buf = 0;
      uint32_t ph = 0, eph = 0, cph = 0;  // bit b: acc_empty wait / acc_full commit parity of buffer b
      bool aborted = false, issued = false;
      for (long long s = s0; s < s1 && !aborted;) {
        int nb;
        long long end;
        gm_segment(s, s1, k_steps, nb, end);
        if (!mbar_wait(&acc_empty[buf], ((eph >> buf) & 1) ^ 1, kErrWaitAccEmpty, abort_flag)) {
          aborted = true;
          break;
        }
        eph ^= 1u << buf;
        tc_fence_after();
        for (const long long first = s; s < end; ++s) {
          if (!mbar_wait(&full[st], ph, kErrWaitFull, abort_flag)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t sfa_s = smem_u32(smem + GmCfg::kOffSfa + st * kMxSfBlock);
          const uint32_t sfb_s = smem_u32(smem + GmCfg::kOffSfb + st * kMxSfBlock);
          tmem_cp_sf(tmem + kGmSfaCol, sf_block_desc(sfa_s));
          tmem_cp_sf(tmem + kGmSfbCol, sf_block_desc(sfb_s));
          mma_mx_stage(tmem + 32 * buf, umma_desc_sw128(smem_u32(smem + st * GmCfg::kWBytes)),
                       umma_desc_sw128(smem_u32(smem + GmCfg::kOffB + st * GmCfg::kBBytes)), idesc,
                       tmem + kGmSfaCol, tmem + kGmSfbCol, s == first);
          issued = true;
          tc_commit(&empty[st]);
          if (++st == kGmStages) {
            st = 0;
            ph ^= 1;
          }
        }
        if (aborted) break;
        tc_commit(&acc_full[buf]);
        cph ^= 1u << buf;
        buf ^= 1;
      }
      if (aborted && issued) {  // wait for the MMAs already issued before TMEM is released
        tc_commit(&acc_full[buf]);
        mbar_wait_drain(&acc_full[buf], (cph >> buf) & 1);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quarter: weight rows 32q .. 32q+31 of the block
    griddep_wait();          // the coder has zeroed ws before the first atomic
    int buf = 0;
    uint32_t fph = 0;  // bit b: acc_full parity of buffer b
    for (long long s = s0; s < s1;) {
      int nb;
      long long end;
      gm_segment(s, s1, k_steps, nb, end);
      s = end;
      if (!warp_wait(&acc_full[buf], (fph >> buf) & 1, kErrWaitAccFull, abort_flag)) break;
      fph ^= 1u << buf;
      tc_fence_after();
      uint32_t a[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + 32 * buf, a);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      const int n = nb * kTcTileW + 32 * q + lane;
      if (n < N) {
#pragma unroll
        for (int m = 0; m < kMxDecodeM; ++m)
          if (m < M) atomicAdd(ws + static_cast<size_t>(m) * N + n, __uint_as_float(a[m]) + __uint_as_float(a[kMxDecodeM + m]));
      }
      buf ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kGmTmemCols);
  }
}

// fp32 [M][N] -> OutT [M][N] (the decode kernel's atomically summed result).
__global__ void __launch_bounds__(256) mx_finalize_kernel(const float* __restrict__ ws, long long n,
                                                          __nv_bfloat16* __restrict__ C) {
  griddep_wait();  // launched with PDL after the decode kernel: its atomics are complete
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n / 2;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float2 v = reinterpret_cast<const float2*>(ws)[i];
    reinterpret_cast<uint32_t*>(C)[i] = pack_bf16x2(v.x, v.y);
  }
}

// ------------------------------------------------------------------------------------
// Activation coder: bf16 [M, K] -> E4M3 code rows [rows][Kp] + scale blocks (layout above).
// One thread per (code row, 32-k group) over rows_sf rows (a multiple of 128) and Kp / 32
// groups.  Group exponent e = floor(log2(amax)) - below_top clipped to [-127, 127] (all-zero
// group: -127, scale byte 0); codes = cvt.rn.satfinite.e4m3x2(x * 2**-e) (the scaling is
// exact).  below_top = 8 for MX_Q8, 7 for both MX_SPLIT2 pieces; a lo-piece thread recomputes
// the hi piece and codes the exact residual x - hi.  Optionally zeroes zero_n floats of
// zero_ws (the decode kernel's accumulation buffer) with a grid-stride loop.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float2 e4m3x2_value(uint32_t c) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(static_cast<uint16_t>(c)));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Codes one 32-element group: exponent (returned) and 16 code pairs, 2 per 16-bit half.
__device__ __forceinline__ int mx_code_group(const float (&v)[32], int below_top, uint32_t (&o)[8]) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  int e = -127;
  if (amax > 0.0f) {
    int E;
    frexpf(amax, &E);  // amax = f * 2**E, f in [0.5, 1): floor(log2(amax)) = E - 1
    e = E - 1 - below_top;
    e = e < -127 ? -127 : (e > 127 ? 127 : e);
  }
  const float inv = exp2_neg(e);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    o[i] = e4m3x2(v[4 * i] * inv, v[4 * i + 1] * inv) | (e4m3x2(v[4 * i + 2] * inv, v[4 * i + 3] * inv) << 16);
  return e;
}

__global__ void __launch_bounds__(256) quant_act_mx8_kernel(const __nv_bfloat16* __restrict__ A, int M, int K,
                                                            int Kp, int G, int split, int rows_codes, int rows_sf,
                                                            uint8_t* __restrict__ codes, uint8_t* __restrict__ sfb,
                                                            float* __restrict__ zero_ws, long long zero_n) {
  griddep_launch_dependents();  // the GEMM launched after this may start its weight loads
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (zero_ws)
    for (long long i = idx; i < zero_n / 4; i += static_cast<long long>(gridDim.x) * blockDim.x)
      reinterpret_cast<float4*>(zero_ws)[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const int groups = Kp / kGroup;
  if (idx >= static_cast<long long>(rows_sf) * groups) return;
  const int b = static_cast<int>(idx / groups), g = static_cast<int>(idx - static_cast<long long>(b) * groups);
  int m = b, p = 0;
  if (G > 0) {
    const int blk = b / (2 * G), w = b - blk * 2 * G;
    p = w >= G;
    m = blk * G + w - p * G;
  }
  const bool live = b < rows_codes && m < M && g * kGroup < K && (p == 0 || split);
  float v[32];
  if (live) {
    const uint4* src = reinterpret_cast<const uint4*>(A + static_cast<size_t>(m) * K + g * kGroup);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = src[i];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
        v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.0f;
  }
  const int below_top = split ? 7 : 8;
  uint32_t o[8];
  int e = mx_code_group(v, below_top, o);
  if (p == 1) {  // lo piece: code the exact residual of the hi piece
    const float sc = e > -127 ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23) : __uint_as_float(0x00400000u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 a = e4m3x2_value(o[i] & 0xFFFFu), c = e4m3x2_value(o[i] >> 16);
      v[4 * i] -= a.x * sc;
      v[4 * i + 1] -= a.y * sc;
      v[4 * i + 2] -= c.x * sc;
      v[4 * i + 3] -= c.y * sc;
    }
    e = mx_code_group(v, below_top, o);
  }
  if (b < rows_codes) {
    uint4* dst = reinterpret_cast<uint4*>(codes + static_cast<size_t>(b) * Kp + g * kGroup);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
  const size_t blk = static_cast<size_t>(g >> 2) * (rows_sf / kChunkRows) + (b >> 7);
  sfb[blk * kMxSfBlock + mx_sf_in_block(b & 127, g & 3)] = static_cast<uint8_t>(e + 127);
}

// ------------------------------------------------------------------------------------
// Weight prepack for the block-scaled kernels.  Sources: the reference layout (packed
// [K/2, N], scales [K/32, N]) or the N-major one (packed [N, K/2], scales [N, K/32]).
// Nibbles: one thread per (row n, 16-byte unit u of the row), n fastest, so that a warp reads
// 32 neighbouring columns of each source row of the reference layout.
// ------------------------------------------------------------------------------------
template <bool kRefLayout>
__global__ void __launch_bounds__(256) prepack_mx_data_kernel(const uint8_t* __restrict__ packed, int N, int K,
                                                              int Np, int Kp, uint8_t* __restrict__ wq) {
  const int units = Kp / 32;  // 16-byte units per row (32 k each)
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<long long>(Np) * units) return;
  const int n = static_cast<int>(idx % Np), u = static_cast<int>(idx / Np);
  const int kh = K / 2;
  uint32_t w[4] = {0, 0, 0, 0};
  if (n < N) {
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      const int j = 16 * u + b;  // byte j of the row = k-pair (2j, 2j+1)
      uint32_t x = 0;
      if (j < kh) x = kRefLayout ? packed[static_cast<size_t>(j) * N + n] : packed[static_cast<size_t>(n) * kh + j];
      w[b >> 2] |= x << (8 * (b & 3));
    }
  }
  *reinterpret_cast<uint4*>(wq + static_cast<size_t>(n) * (Kp / 2) + 16 * u) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Scales: one thread per (row n, 128-k step kt) writes the row's 4-byte word of the block.
template <bool kRefLayout>
__global__ void __launch_bounds__(256) prepack_mx_scale_kernel(const uint8_t* __restrict__ scales, int N, int K,
                                                               int Np, int Kp, uint8_t* __restrict__ sfa) {
  const int steps = Kp / kMxBK;
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<long long>(Np) * steps) return;
  const int n = static_cast<int>(idx % Np), kt = static_cast<int>(idx / Np);
  const int kg = K / kGroup;
  uint32_t word = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int g = 4 * kt + j;
    uint32_t x = 127;
    if (n < N && g < kg) x = kRefLayout ? scales[static_cast<size_t>(g) * N + n] : scales[static_cast<size_t>(n) * kg + g];
    word |= x << (8 * j);
  }
  const size_t blk = static_cast<size_t>(n >> 7) * steps + kt;
  *reinterpret_cast<uint32_t*>(sfa + blk * kMxSfBlock + mx_sf_in_block(n & 127, 0)) = word;
}

}  // namespace mxb
