// Small-M (decode, M <= 16) MXFP4 x BF16 GEMM on the 5th-generation tensor cores.
//
// Same grid, cluster split-K and DSMEM reduction as gemv_kernel, with the per-weight work moved
// off the issue slots: each of 128 converter threads owns one weight row, turns its 64 nibbles of
// a chunk into f16 with the hardware E2M1 conversion and writes them to tensor memory; one
// thread issues tcgen05 MMAs (M = 128 weight rows, N = 16 activation rows, K = 16, A from
// TMEM, B = the prestaged f16 activations in shared memory) into one TMEM accumulator per
// 32-element group; the converters read each group's 16 partial sums back with tcgen05.ld and
// fold in the group's E8M0 scale in fp32.  kGtSlots operand / accumulator slots keep several
// chunks' MMAs in flight while the converters prepare the next.  Each ring stage carries the chunks' weights
// and their 2 KiB activation blocks; a stage is refilled once the converters have read its
// weights and the MMAs that read its activations have completed.
//
// Measured on B200 it is slower than gemv_kernel (each converter thread's per-chunk chain of
// E2M1 conversion, tcgen05.st and tcgen05.ld round trips leaves the SM mostly waiting with only
// 4-8 converter warps per SM), so the launcher selects it only with MXFP4_GEMV_KERNEL=2.
//
// Needs the activations prestaged by gemv_prestage_tc_kernel (f16, one power-of-two shift per
// row so that every bf16 value is exact, 16 rows, rows >= M zero) in the UMMA K-major
// 128-byte-swizzled layout, one 2 KiB block per 64-k chunk; the launcher falls back to
// gemv_kernel without that workspace.
#pragma once

#include "common.cuh"
#include "gemm_small.cuh"

namespace mxb {

constexpr int kGtThreads = 192;  // warp 0 weight producer, 1 MMA issuer, 2..5 converters
constexpr int kGtStageChunks = 4;
constexpr int kGtStages = 2;
constexpr int kGtXChunkBytes = 16 * 64 * 2;  // B operand per chunk: 16 rows x 64 k f16
constexpr int kGtStageWBytes = kGtStageChunks * kChunkBytes;  // 17408 = 17 KiB: x blocks stay 1 KiB aligned
constexpr int kGtStageBytes = kGtStageWBytes + kGtStageChunks * kGtXChunkBytes;
#ifndef MXFP4_GT_SLOTS
#define MXFP4_GT_SLOTS 4
#endif
constexpr int kGtSlots = MXFP4_GT_SLOTS;  // operand / accumulator slots (chunks in flight)
constexpr uint32_t kGtACol = 0;                        // A slot a at columns 32a .. 32a+31
constexpr uint32_t kGtDCol = 32 * kGtSlots;            // accumulator slot a after the A slots
constexpr uint32_t kGtTmemCols = 64 * kGtSlots;

struct GtCfg {
  static constexpr int kOffBar = kGtStages * kGtStageBytes;  // ring; reused for the partials
  static constexpr int kNumBars = 2 * kGtStages + 2 * kGtSlots;  // full, empty, afull, dfull
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;     // + slack for 1 KiB alignment
  static_assert(kOffBar >= kChunkRows * 16 * 4, "partials alias the ring");
  static_assert(kGtStageWBytes % 1024 == 0 && kGtStageBytes % 1024 == 0, "swizzled blocks need 1 KiB alignment");
};

__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4)                                // D format f32; A, B format f16 (0)
         | (static_cast<uint32_t>(n >> 3) << 17)  // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

template <typename OutT>
__global__ void __launch_bounds__(kGtThreads)
    gemv_tc_kernel(const uint8_t* __restrict__ wpack, int M, int k_blocks, int kb_per_split,
                   const uint8_t* __restrict__ xpre, const int* __restrict__ xpre_shift, const GvOut<OutT> out,
                   int N) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GtCfg::kOffBar);
  uint64_t* empty = full + kGtStages;
  uint64_t* afull = empty + kGtStages;
  uint64_t* dfull = afull + kGtSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + GtCfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + GtCfg::kOffMisc + 4);
  float* red = reinterpret_cast<float*>(smem);  // [128 rows][16], after the ring has drained

  const int nb = blockIdx.x;
  const int split = blockIdx.y;
  const int ks = gridDim.y;
  const int kb0 = split * kb_per_split;
  const int nkb = max(0, min(k_blocks, kb0 + kb_per_split) - kb0);
  const int nst = ceil_div(nkb, kGtStageChunks);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kGtStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 5);  // the four converter warps + the MMAs of the stage's last chunk
    }
    for (int i = 0; i < kGtSlots; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&dfull[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kGtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      const uint8_t* src = wpack + (static_cast<size_t>(nb) * k_blocks + kb0) * kChunkBytes;
      const uint8_t* xsrc = xpre + static_cast<size_t>(kb0) * kGtXChunkBytes;
      uint32_t pend = 0, pend_ph = 0;
      bool aborted = false, waited = false;
      for (int i = 0; i < nst; ++i) {
        const int s = i % kGtStages;
        const uint32_t ph = (i / kGtStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
          aborted = true;
          break;
        }
        const int nch = min(kGtStageChunks, nkb - i * kGtStageChunks);
        mbar_arrive_expect_tx(&full[s], nch * (kChunkBytes + kGtXChunkBytes));
        bulk_load(smem + s * kGtStageBytes, src + static_cast<size_t>(i) * kGtStageWBytes, nch * kChunkBytes,
                  &full[s]);
        if (!waited) {  // the activations come from the launch just before this one
          griddep_wait();
          waited = true;
        }
        bulk_load(smem + s * kGtStageBytes + kGtStageWBytes,
                  xsrc + static_cast<size_t>(i) * kGtStageChunks * kGtXChunkBytes, nch * kGtXChunkBytes, &full[s]);
        pend |= 1u << s;
        pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
      }
      if (aborted)
        for (int i = 0; i < kGtStages; ++i)
          if ((pend >> i) & 1) mbar_wait_drain(&full[i], (pend_ph >> i) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && nkb > 0) {
      constexpr uint32_t idesc = umma_idesc_f16(kChunkRows, 16);
      for (int j = 0; j < nkb; ++j) {
        const int a = j % kGtSlots;
        const int i = j / kGtStageChunks, c = j - i * kGtStageChunks, s = i % kGtStages;
        if (c == 0 && !mbar_wait(&full[s], (i / kGtStages) & 1, kErrWaitFull, abort_flag)) break;
        if (!mbar_wait(&afull[a], (j / kGtSlots) & 1, kErrWaitDequant, abort_flag)) break;
        tc_fence_after();
        const uint64_t xdesc =
            umma_desc_sw128(smem_u32(smem + s * kGtStageBytes + kGtStageWBytes + c * kGtXChunkBytes));
#pragma unroll
        for (int G = 0; G < 2; ++G)
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
            mma_ts(tmem + kGtDCol + a * 32 + 16 * G, tmem + kGtACol + a * 32 + 16 * G + 8 * kk,
                   xdesc + 2 * (2 * G + kk), idesc, kk);
        tc_commit(&dfull[a]);
        if (c == kGtStageChunks - 1 || j == nkb - 1) tc_commit(&empty[s]);  // stage free once these finish
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ converters (one weight row each)
    const int q = warp & 3;
    const int r = 32 * q + lane;  // weight row == TMEM lane
    const int odd = (r >> 3) & 1;
    const uint32_t lane_t = static_cast<uint32_t>(32 * q) << 16;
    float acc[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) acc[m] = 0.0f;
    // group scales of the chunks in flight, oldest first: hist[k] belongs to chunk j - kGtSlots + k
    float h0[kGtSlots], h1[kGtSlots];
#pragma unroll
    for (int k = 0; k < kGtSlots; ++k) h0[k] = h1[k] = 0.0f;
    bool ok = true;
    // fold the accumulators of chunk jj (slot jj % kGtSlots) into acc with scales g0, g1
    auto drain = [&](int jj, float g0, float g1) {
      const int a = jj % kGtSlots;
      if (!warp_wait(&dfull[a], (jj / kGtSlots) & 1, kErrWaitDequant, abort_flag)) {
        ok = false;
        return;
      }
      tc_fence_after();
      uint32_t d0[16], d1[16];
      tmem_ld16(tmem + lane_t + kGtDCol + a * 32, d0);
      tmem_ld16(tmem + lane_t + kGtDCol + a * 32 + 16, d1);
      tmem_wait_ld();
#pragma unroll
      for (int m = 0; m < 16; ++m)
        acc[m] = fmaf(__uint_as_float(d1[m]), g1, fmaf(__uint_as_float(d0[m]), g0, acc[m]));
    };
    for (int j = 0; j < nkb && ok; ++j) {
      const int i = j / kGtStageChunks, c = j - i * kGtStageChunks;
      const int s = i % kGtStages;
      if (c == 0 && !warp_wait(&full[s], (i / kGtStages) & 1, kErrWaitFull, abort_flag)) break;
      const uint32_t st = smem_u32(smem + s * kGtStageBytes + c * kChunkBytes);
      uint32_t w0[4], w1[4];
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        const uint4 u = lds128(st + chunk_unit(r, tt) * 16);
        w0[tt] = odd ? u.y : u.x;  // (row, group 0)
        w1[tt] = odd ? u.w : u.z;  // (row, group 1)
      }
      const uint32_t sw = lds32(st + kChunkData + 4 * (8 * (r >> 4) + (r & 7)));
      if (c == kGtStageChunks - 1 || j == nkb - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // A row in natural k order: column 16*G + p holds k-pair p of group G; word t of a group
      // holds k-pairs t, t+4, t+8, t+12 (byte b = pair t + 4b).
      uint32_t v0[16], v1[16];
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        uint32_t o[4];
        e2m1x8_to_f16x2(w0[tt], o);
#pragma unroll
        for (int b = 0; b < 4; ++b) v0[tt + 4 * b] = o[b];
        e2m1x8_to_f16x2(w1[tt], o);
#pragma unroll
        for (int b = 0; b < 4; ++b) v1[tt + 4 * b] = o[b];
      }
      const int a = j % kGtSlots;
      if (j >= kGtSlots) {
        drain(j - kGtSlots, h0[0], h1[0]);  // also frees operand slot a
        if (!ok) break;
      }
      // scale bytes (row, G0) at byte odd, (row, G1) at byte 2 + odd -> 2**(s-127) as f32
      // bits (s << 23); a zero byte (2**-127) decodes to 0, far below the error bound.
#pragma unroll
      for (int k = 0; k + 1 < kGtSlots; ++k) {
        h0[k] = h0[k + 1];
        h1[k] = h1[k + 1];
      }
      h0[kGtSlots - 1] = __uint_as_float(((sw >> (8 * odd)) & 0xFFu) << 23);
      h1[kGtSlots - 1] = __uint_as_float(((sw >> (16 + 8 * odd)) & 0xFFu) << 23);
      tmem_st16(tmem + lane_t + kGtACol + a * 32, v0);
      tmem_st16(tmem + lane_t + kGtACol + a * 32 + 16, v1);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[a]);
    }
#pragma unroll
    for (int k = 0; k < kGtSlots; ++k) {  // the last chunks still in flight
      const int jj = nkb - kGtSlots + k;
      if (ok && jj >= 0) drain(jj, h0[k], h1[k]);
    }
    named_bar_sync(1, 128);  // every converter is done with the ring before it holds the partials
    griddep_wait();
#pragma unroll
    for (int m = 0; m < 16; ++m) red[r * 16 + m] = m < M ? ldexpf(acc[m], -xpre_shift[m]) : 0.0f;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kGtTmemCols);
  }

  // ------------------------------------------------------------ cluster split-K reduction
  cluster_sync_all();
  const int rows_per = kChunkRows / ks;
  const int row_lo = split * rows_per;
  for (int e = threadIdx.x; e < rows_per * M; e += kGtThreads) {
    const int rl = e % rows_per, m = e / rows_per;
    const int row = row_lo + rl;
    float sum = 0.0f;
    for (int rr = 0; rr < ks; ++rr) sum += ld_dsmem_f32(red + row * 16 + m, static_cast<uint32_t>(rr));
    const int n = nb * kChunkRows + row;
    if (n < N) {
      const OutT v = gv_out<OutT>(sum);
#pragma unroll
      for (int d = 0; d < 8; ++d)  // fixed trip count: out.p stays in the parameter space
        if (d < out.count) out.p[d][static_cast<size_t>(m) * out.ldc + out.n_off + n] = v;
    }
  }
  if (out.fence_sys) __threadfence_system();
  cluster_sync_all();
}

// Activation staging for gemv_tc_kernel: one CTA per row m < 16.  Row m's max |x| over all of K
// gives a power-of-two shift that puts it in [2^14, 2^15); the row is written as f16 into
// 2 KiB blocks (one per 64-k chunk): 16 rows x 128 bytes, rows 0-7 and 8-15 in two 1 KiB
// atoms, 16-byte chunk c of row m at position c ^ (m & 7) (the UMMA 128-byte swizzle).  Rows
// m >= M and columns k >= K are zero.
__global__ void __launch_bounds__(256) gemv_prestage_tc_kernel(const __nv_bfloat16* __restrict__ A, int M, int K,
                                                               int k_blocks, uint8_t* __restrict__ xpre,
                                                               int* __restrict__ xpre_shift) {
  griddep_launch_dependents();
  __shared__ float wmax[8];
  const int m = blockIdx.x;
  const int nvec = k_blocks * 8;
  const bool live = m < M;
  const __nv_bfloat16* arow = A + static_cast<size_t>(live ? m : 0) * K;
  float amax = 0.0f;
  if (live)
    for (int v = threadIdx.x; v < nvec; v += 256)
      if (v * 8 < K) {
        const uint4 raw = *reinterpret_cast<const uint4*>(arow + v * 8);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          amax = fmaxf(amax, fabsf(__uint_as_float(w[i] << 16)));
          amax = fmaxf(amax, fabsf(__uint_as_float(w[i] & 0xFFFF0000u)));
        }
      }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, wmax[i]);
  int shift = 0;
  if (amax > 0.0f && amax <= 3.0e38f) {
    int E;
    frexpf(amax, &E);
    shift = 15 - E;
  }
  if (threadIdx.x == 0 && live) xpre_shift[m] = shift;
  const float f1 = exp2i(shift / 2), f2 = exp2i(shift - shift / 2);
  uint8_t* rowbase = xpre + (m >> 3) * 1024 + (m & 7) * 128;
  for (int v = threadIdx.x; v < nvec; v += 256) {
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (live && v * 8 < K) raw = *reinterpret_cast<const uint4*>(arow + v * 8);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t h[4];
#pragma unroll
    for (int tt = 0; tt < 4; ++tt)
      h[tt] = f16x2_from(__uint_as_float(w[tt] << 16) * f1 * f2, __uint_as_float(w[tt] & 0xFFFF0000u) * f1 * f2);
    const int kb = v >> 3, c = v & 7;
    *reinterpret_cast<uint4*>(rowbase + static_cast<size_t>(kb) * kGtXChunkBytes + ((c ^ (m & 7)) << 4)) =
        make_uint4(h[0], h[1], h[2], h[3]);
  }
}

}  // namespace mxb
