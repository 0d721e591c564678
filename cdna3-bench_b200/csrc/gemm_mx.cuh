// Opt-in block-scaled GEMM: MXFP4 weights x MXFP8 activations on tcgen05 kind::mxf8f6f4.
//
// C[M, N] = Q8(A) * W^T.  Q8 quantises the bf16 activations to OCP MXFP8 (E4M3 elements, one
// E8M0 scale per 32 k of a row); W stays MXFP4 (E2M1 elements, E8M0 per 32 k).  The tensor
// core applies both scales itself (block_scale), so nothing is dequantised in software and the
// MMA runs at the 8-bit rate.  The activations lose mantissa bits on the way, so this is a
// separate entry point with its own oracle (dequant(Q8(A)) @ dequant(W) in fp32), not the
// exact drop-in path of gemm_large.cuh.
//
// HBM layouts (both built by kernels in this file):
//   * weights (prepack_mx_*_kernel): nibbles [Np][Kp/2], K contiguous, low nibble = even k;
//     Np = N rounded up to 128, Kp = K rounded up to 128, zero padded.  Scales in 512-byte
//     blocks [Np/128][Kp/128]; inside a block, byte 16*(r%32) + 4*(r/32) + j holds row r's
//     scale for 32-k group j of the 128-k step (padding: 127).
//   * activations (quant_act_mx8_kernel): E4M3 bytes [M][Kp]; scales in 512-byte blocks
//     [Kp/128][Ma/128], same in-block order, Ma = M rounded up to 256 (padding rows and
//     groups are all-zero blocks, scale byte 0).
// The in-block order is what tcgen05.cp .32x128b.warpx4 expects: 16-byte row r%32 goes to
// TMEM lane r%32 (copied to all four lane quarters), its 4-byte word r/32 to a column, and
// byte j is the scale the MMA of k-step j selects (scale-factor id j).
//
// Kernel: persistent CTAs (one per SM), tile = 128 weight rows x 256 activation rows, 128 k per
// pipeline stage (four MMAs of K = 32), accumulator 128 lanes x 256 f32 columns of TMEM.
//   warp 0    TMA producer: activation tile (256 rows x 128 B, 128-byte swizzle), weight tile
//             (128 rows x 128 nibbles, expanded by the TMA to 16-byte units holding 8 bytes of
//             data each, the operand form kind::mxf8f6f4 reads for E2M1; 128-byte swizzle), and
//             the stage's two scale blocks by bulk copy;
//   warp 1    TMEM owner and MMA issuer: copies the stage's scales into TMEM, then issues the
//             four block-scaled MMAs; tcgen05 copies and MMAs of one thread run in issue order,
//             so the next stage's scale copy cannot overtake this stage's MMAs;
//   warps 2-9 epilogue, as in gemm_tc_kernel: tcgen05.ld, release the accumulator, 32 x 32
//             slabs stored by TMA.
// Every wait is bounded (common.cuh); no TMA multicast.
#pragma once

#include "common.cuh"
#include "gemm_large.cuh"
#include "quant.cuh"

namespace mxb {

constexpr int kMxBK = 128;                              // k per pipeline stage
constexpr int kMxThreads = 32 * (2 + kTcEpiWarps);      // 320
constexpr uint32_t kMxSfaCol = 256;                     // 4 TMEM columns: weight scales
constexpr uint32_t kMxSfbCol = 264;                     // 8 TMEM columns: activation scales
constexpr int kMxSfBlock = 512;                         // 128 rows x 4 groups of scale bytes

template <typename OutT>
struct MxCfg {
  static constexpr int kStages = sizeof(OutT) == 2 ? 4 : 3;
  static constexpr int kActBytes = kTcTileAct * kMxBK;      // 32 KiB of E4M3
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
// B = E4M3 (activations), both K-major, E8M0 scales, f32 accumulator.  The scale-factor ids
// (bits 4-5 for B, 29-30 for A) are or-ed in per k-step.
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

// Byte offset of (row r of a 128-row block, 32-k group j of a 128-k step) inside a scale block.
__host__ __device__ constexpr int mx_sf_in_block(int r, int j) { return 16 * (r & 31) + 4 * ((r >> 5) & 3) + j; }

template <typename OutT>
__global__ void __launch_bounds__(kMxThreads, 1)
    gemm_mx_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_out, const uint8_t* __restrict__ sfa,
                   const uint8_t* __restrict__ sfb, int M, int k_steps, int m_blocks, int n_blocks) {
  using Cfg = MxCfg<OutT>;
  constexpr int S = Cfg::kStages;
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
  const int sf_rows = 2 * m_blocks;  // 128-row scale blocks per k-step of the activations

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
      bool aborted = false;
      for (int t = blockIdx.x; t < total && !aborted; t += gridDim.x) {
        int mb, nb;
        tc_tile_coords(t, m_blocks, n_blocks, mb, nb);
        for (int kt = 0; kt < k_steps; ++kt) {
          if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
            aborted = true;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kActBytes + Cfg::kWTxBytes + Cfg::kSfaBytes + Cfg::kSfbBytes);
          tma_load_2d(smem + s * Cfg::kActBytes, &tm_act, &full[s], kt * kMxBK, mb * kTcTileAct);
          tma_load_2d(smem + Cfg::kOffW + s * Cfg::kWBytes, &tm_w, &full[s], kt * kMxBK, nb * kTcTileW);
          bulk_load(smem + Cfg::kOffSfa + s * Cfg::kSfaBytes,
                    sfa + (static_cast<size_t>(nb) * k_steps + kt) * kMxSfBlock, Cfg::kSfaBytes, &full[s]);
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
      constexpr uint32_t idesc = umma_idesc_mx(kTcTileW, kTcTileAct);
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
          const uint64_t adesc = umma_desc_sw128(smem_u32(smem + Cfg::kOffW + s * Cfg::kWBytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(smem + s * Cfg::kActBytes));
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j) {  // k-step j: 32 k = 32 bytes of both operand rows
            const uint32_t id = idesc | (j << 29) | (j << 4);
            mma_mx(tmem + kTmemAccCol, adesc + 2 * j, bdesc + 2 * j, id, (tmem + kMxSfaCol) | (j << 30),
                   (tmem + kMxSfbCol) | (j << 30), (kt | j) != 0);
          }
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
    const int q = warp & 3;  // TMEM lane quarter = 32 output columns
    const int ew = warp - 2;
    const int hh = ew >> 2;  // 128-column half of the accumulator
    uint8_t* stage_ptr = smem + Cfg::kOffOut + ew * Cfg::kSlabBytes;
    const uint32_t stage = smem_u32(stage_ptr);
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int mb, nb;
      tc_tile_coords(t, m_blocks, n_blocks, mb, nb);
      if (!warp_wait(acc_full, aph, kErrWaitAccFull, abort_flag)) break;
      tc_fence_after();
      const int m0 = mb * kTcTileAct + 128 * hh;  // activation rows m0 .. m0+127 of this warp
      const int n0 = nb * kTcTileW + 32 * q;      // output columns n0 .. n0+31 (one per lane)
      const uint32_t tb = tmem + (static_cast<uint32_t>(32 * q) << 16) + kTmemAccCol + 128 * hh;
      if constexpr (sizeof(OutT) == 2) {
        uint32_t packed[64];  // bf16 pairs (m, m+1) of this lane's output column
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t v[16];
          tmem_ld16(tb + 16 * c, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            packed[8 * c + j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);  // accumulator free: the next tile's MMAs start
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // four 32-row slabs
          const int mc = m0 + 32 * c;
          if (mc < M) {
            if (lane == 0) bulk_wait_read<0>();  // the previous store has read the buffer
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
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // f32 output: 32-column chunks, release after the last load
          uint32_t v[32];
          tmem_ld32(tb + 32 * c, v);
          tmem_wait_ld();
          if (c == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
          }
          const int mc = m0 + 32 * c;
          if (mc < M) {
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 32; ++j) sts32(stage + (j * 32 + lane) * 4, v[j]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tm_out, stage_ptr, n0, mc);
              bulk_commit();
            }
          }
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
// Activation quantiser: bf16 [M, K] -> E4M3 [M, Kp] + scale blocks, OCP MX rule for E4M3:
// scale exponent e = floor(log2(amax)) - 8 (8 = exponent of E4M3's largest normal, 448)
// clipped to [-127, 127], an all-zero group gets e = -127; elements x * 2**-e rounded to
// nearest even E4M3 and saturated at +-448 (cvt.rn.satfinite).  One thread per (row, 32-k
// group) over Ma rows and Kp / 32 groups; rows >= M and groups past K are written as zero
// groups (scale byte 0; E4M3 bytes only for rows < M).
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(256) quant_act_mx8_kernel(const __nv_bfloat16* __restrict__ A, int M, int K,
                                                            int Kp, int Ma, uint8_t* __restrict__ a8,
                                                            uint8_t* __restrict__ sfb) {
  const int groups = Kp / kGroup;
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<long long>(Ma) * groups) return;
  const int m = static_cast<int>(idx / groups), g = static_cast<int>(idx - static_cast<long long>(m) * groups);
  float v[32];
  const bool live = m < M && g * kGroup < K;
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
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  int e = -127;
  if (amax > 0.0f) {
    int E;
    frexpf(amax, &E);  // amax = f * 2**E, f in [0.5, 1): floor(log2(amax)) = E - 1
    e = E - 1 - 8;
    e = e < -127 ? -127 : (e > 127 ? 127 : e);
  }
  const float inv = exp2_neg(e);
  if (m < M) {
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o[i] = e4m3x2(v[4 * i] * inv, v[4 * i + 1] * inv) | (e4m3x2(v[4 * i + 2] * inv, v[4 * i + 3] * inv) << 16);
    uint4* dst = reinterpret_cast<uint4*>(a8 + static_cast<size_t>(m) * Kp + g * kGroup);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
  const size_t blk = static_cast<size_t>(g >> 2) * (Ma / kChunkRows) + (m >> 7);
  sfb[blk * kMxSfBlock + mx_sf_in_block(m & 127, g & 3)] = static_cast<uint8_t>(e + 127);
}

// ------------------------------------------------------------------------------------
// Weight prepack for the block-scaled path.  Sources: the reference layout (packed [K/2, N],
// scales [K/32, N]) or the N-major one (packed [N, K/2], scales [N, K/32]).
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
