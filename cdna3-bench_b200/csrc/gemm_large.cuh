// Large-M MXFP4 x BF16 GEMM on the 5th-generation tensor cores (tcgen05).
//
// C[M, N] = A[M, K] (bf16) * dequant(W)^T with W the prepacked MXFP4 weights (N rows).
//
// The MMA computes the transposed product D = W_tile * A_tile^T so that the operand that
// must be dequantised (the weights) is the MMA's "A" operand:
//   * UMMA M = 128 weight rows (one prepacked chunk row block), UMMA N = 256 activation
//     rows, K = 64 per pipeline stage (4 MMAs of K = 16).
//   * Activations: TMA tiled load [256 rows x 64 k] bf16, 128-byte swizzle, K-major smem
//     operand (the UMMA "B" operand).
//   * Weights: one 4352-byte chunk per stage by a 1-D bulk copy; eight dequant warps expand
//     it to bf16 exactly (table lookup, see common.cuh) and write it either
//       kTS = true : into tensor memory with tcgen05.st (the MMA reads A from TMEM, which
//                    keeps the dequantised tile off the shared-memory bandwidth), or
//       kTS = false: into a 128B-swizzled K-major smem tile (classic SS MMA).
//   * Accumulator: 128 lanes x 256 f32 columns of TMEM.  Eight epilogue warps (two per TMEM
//     lane quarter, one per 128-column half) read their columns into registers (packed to
//     bf16) and hand the accumulator back to the MMA issuer BEFORE storing, so the next
//     tile's MMAs overlap the stores; each warp then writes 32 x 32 slabs through its own
//     smem staging buffer with TMA tensor stores.
//   * Persistent CTAs (one per SM) walk the tile list in a grouped raster order.  When there are
//     too few tiles to fill the GPU (small M x N), K is split too: each tile slice stores an
//     fp32 partial through a 3-D map into workspace and splitk_reduce_kernel sums them.
//
// Warp roles (576 threads): 0 = TMA producer, 1 = MMA issuer (+TMEM owner),
// 2..9 = epilogue, 10..17 = dequant (one per TMEM lane quarter in each of two groups that
// take alternate pipeline stages).  A warp may touch TMEM lanes 32*(warp%4) .. +31 only.
#pragma once

#include "common.cuh"

// Profiling switch, 0 in every product build.  -DMXFP4_TC_DIAG=<bit mask> removes pipeline
// stages so the remaining ones can be timed in isolation (results are then wrong):
//   1: dequant warps skip the table lookup (zeros go to TMEM),  2: ... skip the TMEM store,
//   4: the MMA issuer commits without issuing MMAs,  8: the epilogue skips staging and stores.
#ifndef MXFP4_TC_DIAG
#define MXFP4_TC_DIAG 0
#endif

namespace mxb {

constexpr int kTcEpiWarps = 8;
constexpr int kTcFirstEpiWarp = 2;
constexpr int kTcFirstDqWarp = kTcFirstEpiWarp + kTcEpiWarps;
constexpr int kTcThreads = 32 * (kTcFirstDqWarp + 8);  // 576
constexpr int kTcTileAct = 256;  // activation rows per tile (UMMA N)
constexpr int kTcTileW = 128;    // weight rows per tile (UMMA M)
constexpr int kTcBK = 64;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemAccCol = 0;
constexpr uint32_t kTmemARingCol = 256;

template <bool kTS, typename OutT>
struct TcCfg {
  static constexpr int kStages = kTS ? 5 : 3;
  static constexpr int kActBytes = kTcTileAct * kTcBK * 2;          // 32 KiB
  static constexpr int kATileBytes = kTS ? 0 : kTcTileW * kTcBK * 2;  // 16 KiB (SS only)
  static constexpr int kSlabBytes = 32 * 32 * static_cast<int>(sizeof(OutT));  // 32 m x 32 n
  static constexpr int kOffA = kStages * kActBytes;
  static constexpr int kOffOut = kOffA + kStages * kATileBytes;
  static constexpr int kOffW = kOffOut + kTcEpiWarps * kSlabBytes;
  static constexpr int kOffBar = kOffW + kStages * kChunkBytes;
  static constexpr int kNumBars = 3 * kStages + 2;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + slack for 1024-byte alignment
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

__device__ __forceinline__ void tc_tile_coords(int t, int m_blocks, int n_blocks, int& mb, int& nb) {
  constexpr int kGroupM = 8;  // raster: 8 activation blocks share the weight stream
  const int per_group = kGroupM * n_blocks;
  const int grp = t / per_group;
  const int first = grp * kGroupM;
  const int gm = min(m_blocks - first, kGroupM);
  const int local = t - grp * per_group;
  mb = first + local % gm;
  nb = local / gm;
}

// Tile t of the persistent schedule: split-K slice ks (outermost), then the grouped raster.
__device__ __forceinline__ void tc_tile(int t, int m_blocks, int n_blocks, int k_blocks, int kbps, int& mb,
                                        int& nb, int& kb_lo, int& kb_hi, int& ks) {
  const int mn = m_blocks * n_blocks;
  ks = t / mn;
  tc_tile_coords(t - ks * mn, m_blocks, n_blocks, mb, nb);
  kb_lo = ks * kbps;
  kb_hi = min(k_blocks, kb_lo + kbps);
}

// Output destinations: the epilogue stores every output slab through each of these maps.  One
// map is the plain GEMM; several give the all-gather form, where each map covers this GPU's
// column slice of one GPU's full output buffer (its own, or a peer's over NVLink).
constexpr int kMaxOutDst = 8;
struct TcOut {
  CUtensorMap map[kMaxOutDst];
  int count;
  int fence_sys;  // 1: make the stores visible system-wide before the kernel ends (peer buffers)
  int split3d;    // 1: map[0] is a 3-D fp32 map over split-K partials [splits][M][N]
};

template <bool kTS, typename OutT>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ TcOut out,
                   const uint8_t* __restrict__ wpack, int M, int k_blocks, int m_blocks, int n_blocks,
                   int k_splits, int kbps) {
  using Cfg = TcCfg<kTS, OutT>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* dqd = full + S;
  uint64_t* empty = dqd + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total = m_blocks * n_blocks * k_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&dqd[s], 4);  // four dequant warps per stage
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kTcEpiWarps);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_act);
    for (int d = 0; d < out.count; ++d) prefetch_tmap(&out.map[d]);
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
      bool aborted = test_withhold();  // test switch: issue nothing, the consumers' waits run out
      for (int t = blockIdx.x; t < total && !aborted; t += gridDim.x) {
        int mb, nb, kb_lo, kb_hi, ks;
        tc_tile(t, m_blocks, n_blocks, k_blocks, kbps, mb, nb, kb_lo, kb_hi, ks);
        const uint8_t* wsrc = wpack + static_cast<size_t>(nb) * k_blocks * kChunkBytes;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
            aborted = true;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kActBytes + kChunkBytes);
          tma_load_2d(smem + s * Cfg::kActBytes, &tm_act, &full[s], kb * kTcBK, mb * kTcTileAct);
          bulk_load(smem + Cfg::kOffW + s * kChunkBytes, wsrc + static_cast<size_t>(kb) * kChunkBytes,
                    kChunkBytes, &full[s]);
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
      constexpr uint32_t idesc = umma_idesc_bf16(kTcTileW, kTcTileAct);
      int s = 0;
      uint32_t ph = 0, aph = 0;
      bool aborted = false, issued = false;
      for (int t = blockIdx.x; t < total && !aborted; t += gridDim.x) {
        if (!mbar_wait(acc_empty, aph ^ 1, kErrWaitAccEmpty, abort_flag)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        int mb, nb, kb_lo, kb_hi, ks;
        tc_tile(t, m_blocks, n_blocks, k_blocks, kbps, mb, nb, kb_lo, kb_hi, ks);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[s], ph, kErrWaitFull, abort_flag) ||
              !mbar_wait(&dqd[s], ph, kErrWaitDequant, abort_flag)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = umma_desc_sw128(smem_u32(smem + s * Cfg::kActBytes));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (MXFP4_TC_DIAG & 4) break;
            const uint32_t acc = ((kb - kb_lo) | i) != 0;
            if constexpr (kTS) {
              mma_ts(tmem + kTmemAccCol, tmem + kTmemARingCol + s * 32 + i * 8, bdesc + 2 * i, idesc, acc);
            } else {
              const uint64_t adesc = umma_desc_sw128(smem_u32(smem + Cfg::kOffA + s * Cfg::kATileBytes));
              mma_ss(tmem + kTmemAccCol, adesc + 2 * i, bdesc + 2 * i, idesc, acc);
            }
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
  } else if (warp < kTcFirstDqWarp) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;   // TMEM lane quarter = 32 output columns
    const int ew = warp - kTcFirstEpiWarp;
    const int hh = ew >> 2;   // 128-column half of the accumulator
    uint8_t* stage_ptr = smem + Cfg::kOffOut + ew * Cfg::kSlabBytes;
    const uint32_t stage = smem_u32(stage_ptr);
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int mb, nb, kb_lo, kb_hi, ks;
      tc_tile(t, m_blocks, n_blocks, k_blocks, kbps, mb, nb, kb_lo, kb_hi, ks);
      bool ok = warp_wait(acc_full, aph, kErrWaitAccFull, abort_flag);
      // The two warps of a bf16 slab pair meet at a named barrier below: they leave the loop
      // together (if either gave up waiting), or neither does.
      if (sizeof(OutT) == 2 && out.count > 1) ok = named_bar_and(2 + (ew >> 1), 64, ok);
      if (!ok) break;
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
        if (out.count == 1) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {  // four 32-row slabs
            const int mc = m0 + 32 * c;
            if (!(MXFP4_TC_DIAG & 8) && mc < M) {
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
                tma_store_2d(&out.map[0], stage_ptr, n0, mc);
                bulk_commit();
              }
            }
          }
        } else {
          // bf16: the two warps of adjacent column quarters (ew, ew^1) fill one 32-row x 64-column
          // slab (128-byte rows, the unit that crosses NVLink efficiently when a destination is a
          // peer's buffer) and the even warp stores it.
          const int pair = ew >> 1, half = ew & 1;
          uint8_t* pair_ptr = smem + Cfg::kOffOut + pair * 2 * Cfg::kSlabBytes;
          const uint32_t pstage = smem_u32(pair_ptr);
          const int n_pair = n0 - 32 * half;
#pragma unroll
          for (int c = 0; c < 4; ++c) {  // four 32-row slabs
            const int mc = m0 + 32 * c;
            if (!(MXFP4_TC_DIAG & 8) && mc < M) {
              if (half == 0 && lane == 0) bulk_wait_read<0>();  // the previous store has read the buffer
              named_bar_sync(2 + pair, 64);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const uint32_t pk = packed[16 * c + j];
                sts16(pstage + ((2 * j) * 64 + 32 * half + lane) * 2, pk & 0xFFFFu);
                sts16(pstage + ((2 * j + 1) * 64 + 32 * half + lane) * 2, pk >> 16);
              }
              fence_proxy_async_smem();
              named_bar_sync(2 + pair, 64);
              if (half == 0 && lane == 0) {
                for (int d = 0; d < out.count; ++d) tma_store_2d(&out.map[d], pair_ptr, n_pair, mc);
                bulk_commit();
              }
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
          if (!(MXFP4_TC_DIAG & 8) && mc < M) {
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 32; ++j) sts32(stage + (j * 32 + lane) * 4, v[j]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (out.split3d)
                tma_store_3d(&out.map[0], stage_ptr, n0, mc, ks);
              else
                for (int d = 0; d < out.count; ++d) tma_store_2d(&out.map[d], stage_ptr, n0, mc);
              bulk_commit();
            }
          }
        }
      }
      aph ^= 1;
    }
    if (lane == 0) {
      bulk_wait_all();
      if (out.fence_sys) asm volatile("fence.acq_rel.sys;" ::: "memory");
    }
  } else {
    // ------------------------------------------------------------ dequant
    // Two groups of four warps take the pipeline steps in turn (group 0 the even ones, group 1
    // the odd ones); in its step a warp dequantises both 32-element groups of its 32 rows.  Lane
    // r reads the four 16-byte units chunk_unit(r, t), t = 0..3 (each holds word t of rows r and
    // r^8 in both groups; lanes r and r^8 share a unit and the unit placement puts each 8-lane
    // phase on distinct bank groups) and keeps the words of its own row.
    const int q = warp & 3;
    const int grp = (warp - kTcFirstDqWarp) >> 2;
    const int r = 32 * q + lane;  // weight row inside the tile == TMEM lane
    const int odd = (r >> 3) & 1;
    const uint32_t wbase = smem_u32(smem + Cfg::kOffW);
    int s = 0;
    uint32_t ph = 0, it = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < total && !aborted; t += gridDim.x) {
      int mb, nb, kb_lo, kb_hi, ks;
      tc_tile(t, m_blocks, n_blocks, k_blocks, kbps, mb, nb, kb_lo, kb_hi, ks);
      for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
        if ((it & 1) == static_cast<uint32_t>(grp)) {
          // With an odd stage count the two groups take turns on each stage, so a group waits on
          // every second phase of full[s], always with the same parity -- and a parity wait cannot
          // tell its own phase from the one two back while the other group's load of the phase
          // between is still in flight.  So first wait until the other group has finished that
          // phase (dqd[s] of iteration it - S: unambiguous, since its next phase needs this
          // group's own arrival); after it, the parity wait on full[s] names exactly one phase.
          if (it >= static_cast<uint32_t>(S) && !warp_wait(&dqd[s], ph ^ 1, kErrWaitDequant, abort_flag)) {
            aborted = true;
            break;
          }
          if (!warp_wait(&full[s], ph, kErrWaitFull, abort_flag)) {
            aborted = true;
            break;
          }
          const uint32_t wst = wbase + s * kChunkBytes;
          uint32_t v0[16], v1[16];
          if (MXFP4_TC_DIAG & 1) {
#pragma unroll
            for (int i = 0; i < 16; ++i) v0[i] = v1[i] = 0;
          } else {
            uint32_t w0[4], w1[4];
#pragma unroll
            for (int tt = 0; tt < 4; ++tt) {
              const uint4 u = lds128(wst + chunk_unit(r, tt) * 16);
              w0[tt] = odd ? u.y : u.x;  // (row, group 0)
              w1[tt] = odd ? u.w : u.z;  // (row, group 1)
            }
            const uint32_t sc = lds32(wst + kChunkData + 4 * (8 * (r >> 4) + (r & 7)));
            dequant_rowgroup(make_uint4(w0[0], w0[1], w0[2], w0[3]), (sc >> (8 * odd)) & 0xFF, v0);
            dequant_rowgroup(make_uint4(w1[0], w1[1], w1[2], w1[3]), (sc >> (16 + 8 * odd)) & 0xFF, v1);
          }
          if (MXFP4_TC_DIAG & 2) {
          } else if constexpr (kTS) {
            tc_fence_after();
            const uint32_t ta = tmem + (static_cast<uint32_t>(32 * q) << 16) + kTmemARingCol + s * 32;
            tmem_st16(ta, v0);
            tmem_st16(ta + 16, v1);
            tmem_wait_st();
            tc_fence_before();
          } else {
            const uint32_t at = smem_u32(smem + Cfg::kOffA + s * Cfg::kATileBytes) + r * 128;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              sts128(at + ((j ^ (r & 7)) << 4), make_uint4(v0[4 * j], v0[4 * j + 1], v0[4 * j + 2], v0[4 * j + 3]));
              sts128(at + (((4 + j) ^ (r & 7)) << 4),
                     make_uint4(v1[4 * j], v1[4 * j + 1], v1[4 * j + 2], v1[4 * j + 3]));
            }
            fence_proxy_async_smem();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&dqd[s]);
        }
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Sum of the split-K partials ws[splits][M][N] (fp32) into C (row stride ldc).  Four columns
// per thread; N is a multiple of 4 on this path.  Launched as a programmatic dependent of the
// GEMM that writes the partials, so its launch overlaps the GEMM's tail.
template <typename OutT>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N,
                                                            OutT* __restrict__ C, int ldc) {
  griddep_wait();  // launched as the GEMM's programmatic dependent: its partials are complete here
  const size_t n4 = static_cast<size_t>(N) / 4;
  const size_t total = static_cast<size_t>(M) * n4;
  const size_t plane = static_cast<size_t>(M) * N;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t m = i / n4, c = (i - m * n4) * 4;
    float4 acc = *reinterpret_cast<const float4*>(ws + m * N + c);
    for (int s = 1; s < splits; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(ws + s * plane + m * N + c);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    OutT* dst = C + m * ldc + c;
    if constexpr (sizeof(OutT) == 4) {
      *reinterpret_cast<float4*>(dst) = acc;
    } else {
      const uint32_t lo = pack_bf16x2(acc.x, acc.y), hi = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
    }
  }
}

}  // namespace mxb
