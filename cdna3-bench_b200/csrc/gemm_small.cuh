// Small-M (decode, M <= 16) MXFP4 x BF16 GEMM.  HBM-bound: the job is to stream the
// packed weights once at full bandwidth and keep the per-element instruction count low.
//
// * Grid (N/128 weight-row blocks, KS K-splits); the KS CTAs of a row block form one
//   thread-block cluster and reduce their partial sums through distributed shared memory,
//   so the kernel needs no global scratch and no second launch.
// * A producer warp streams the CTA's contiguous run of 4352-byte prepacked chunks into a
//   shared-memory ring with 1-D bulk copies of kGvStageChunks chunks each (mbarrier
//   complete_tx).  The bytes in flight then come from shared memory, not registers: a
//   register-prefetch design is limited by the registers each resident thread can spare
//   and measured at under half the HBM rate.  The first stages are issued before the
//   activations are staged.
// * Eight compute warps own 16 weight rows each.  The chunk layout (chunk_word_off in
//   common.cuh) puts every word lane (g, t) of an m16n8k16 MMA needs from a chunk into one
//   16-byte unit, so a lane reads a chunk with one conflict-free 128-bit shared load plus
//   one 32-bit load of its four scales.
// * Weights are converted in registers with the hardware E2M1->f16 conversion (exact,
//   unscaled) straight into mma.sync fragments; the activations are staged once per CTA in
//   f16, pre-scaled per row by a power of two so that every bf16 activation is represented
//   exactly (up to f16 subnormal range at the row's small end).  Each 32-element group's
//   fp32 partial is multiplied by its E8M0 scale 2**(s-127) and accumulated in fp32; the
//   per-row activation shift is undone before the cross-CTA reduction.
#pragma once

#include "common.cuh"

namespace mxb {

#ifndef MXFP4_GV_DIAG
#define MXFP4_GV_DIAG 0  // sweep-only bitmask: 1 = skip the E2M1 conversion, 2 = skip the scale decode,
                         // 4 = skip the MMAs, 8 = skip the activation staging
#endif
constexpr int kGvThreads = 288;     // 8 compute warps + 1 producer warp
constexpr int kGvMinBlocks = 4;     // register cap so that four CTAs fit on an SM
constexpr int kGvStageChunks = 4;   // chunks per bulk copy / ring stage
constexpr int kGvStageWBytes = kGvStageChunks * kChunkBytes;  // weights of one stage
constexpr int kGvMaxStages = 8;

template <int NT>
struct GvCfg {
  static constexpr int kMP = 8 * NT;  // padded activation rows
  // [ring: stages x stage_bytes; reused for the partial sums once drained][full/empty
  // barriers][xshift, abort, xmax][activations staged in-kernel: two 32-groups x M rows x 16 f16
  // pairs per chunk].  With prestaged activations each stage carries its chunks' activation
  // blocks after the weights and there is no separate activation region.
  __host__ __device__ static int stage_bytes(int M, bool prestaged) {
    return kGvStageChunks * (kChunkBytes + (prestaged ? 2 * M * 64 : 0));
  }
  __host__ __device__ static int off_bar(int stages, int sb) { return stages * sb; }
  __host__ __device__ static int off_shift(int stages, int sb) { return off_bar(stages, sb) + (2 * kGvMaxStages + 2) * 8; }
  __host__ __device__ static int off_x(int stages, int sb) { return (off_shift(stages, sb) + 8 * kMP + 16 + 127) & ~127; }
  __host__ __device__ static int smem_bytes(int stages, int kb_per_split, int M, bool prestaged) {
    const int sb = stage_bytes(M, prestaged);
    return off_x(stages, sb) + (prestaged ? 0 : kb_per_split * 2 * M * 64);
  }
};

// 2**e as an f32 for e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  // not volatile: the compiler may interleave independent MMAs with the conversions
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t f16x2_from(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename OutT>
__device__ __forceinline__ OutT gv_out(float v);
template <>
__device__ __forceinline__ float gv_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 gv_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Output destinations of the decode kernel: C[m, n] goes to p[d][m * ldc + n_off + n] for every
// d < count (one destination for the plain GEMM; one per GPU for the all-gather form).
template <typename OutT>
struct GvOut {
  OutT* p[8];
  int count, ldc, n_off, fence_sys;
};

template <int NT, typename OutT>
__global__ void __launch_bounds__(kGvThreads, kGvMinBlocks)
    gemv_kernel(const __nv_bfloat16* __restrict__ A, int M, int K, const uint8_t* __restrict__ wpack,
                int k_blocks, int kb_per_split, int stages, const GvOut<OutT> out, int N,
                const uint8_t* __restrict__ xpre, const int* __restrict__ xpre_shift) {
  using Cfg = GvCfg<NT>;
  constexpr int MP = Cfg::kMP;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  const bool pre = xpre != nullptr;
  const int sbytes = Cfg::stage_bytes(M, pre);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::off_bar(stages, sbytes));
  uint64_t* empty = full + kGvMaxStages;
  int* xshift = reinterpret_cast<int*>(smem + Cfg::off_shift(stages, sbytes));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(xshift + MP);
  unsigned* xmax = reinterpret_cast<unsigned*>(xshift + MP + 4);  // per-row max |x| (float bits)
  float* red = reinterpret_cast<float*>(smem);  // aliases the drained ring
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + Cfg::off_x(stages, sbytes));

  const int nb = blockIdx.x;
  const int split = blockIdx.y;
  const int ks = gridDim.y;  // == cluster size; rank of this CTA == split
  const int kb0 = split * kb_per_split;
  const int nkb = max(0, min(k_blocks, kb0 + kb_per_split) - kb0);
  const int nst = ceil_div(nkb, kGvStageChunks);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < MP) xmax[threadIdx.x] = 0u;
  __syncthreads();

  if (warp == 8) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      const uint8_t* src = wpack + (static_cast<size_t>(nb) * k_blocks + kb0) * kChunkBytes;
      uint32_t pend = 0, pend_ph = 0;
      bool aborted = false;
      // With prestaged activations (written by the launch just before this one) each stage also
      // carries its chunks' activation blocks; the first weight copy goes out before waiting
      // for that launch to finish.
      const uint32_t xblk = 2u * M * 64;
      bool waited = false;
      const int n_issue = test_withhold() ? 0 : nst;  // test switch: issue nothing
      for (int i = 0; i < n_issue; ++i) {
        const int s = i % stages;
        const uint32_t ph = (i / stages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
          aborted = true;
          break;
        }
        const uint32_t nch = min(kGvStageChunks, nkb - i * kGvStageChunks);
        mbar_arrive_expect_tx(&full[s], nch * (kChunkBytes + (pre ? xblk : 0u)));
        bulk_load(ring + s * sbytes, src + static_cast<size_t>(i) * kGvStageWBytes, nch * kChunkBytes, &full[s]);
        if (pre) {
          if (!waited) {
            griddep_wait();
            waited = true;
          }
          bulk_load(ring + s * sbytes + kGvStageWBytes,
                    xpre + (static_cast<size_t>(kb0) + static_cast<size_t>(i) * kGvStageChunks) * xblk, nch * xblk,
                    &full[s]);
        }
        pend |= 1u << s;
        pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
      }
      if (aborted)
        for (int i = 0; i < stages; ++i)
          if ((pend >> i) & 1) mbar_wait_drain(&full[i], (pend_ph >> i) & 1);
    }
    __syncwarp();
  } else {
    const int g = lane >> 2, t = lane & 3;
    // ------------------------------------------------------------ stage activations (f16)
    // The 256 compute threads split this CTA's K range; each handles all M rows of its
    // columns.  Pass 1: per-row max |x| (warp reduction, then one shared atomicMax on the
    // float bits, which orders like the values for non-negative floats).  Pass 2: re-read
    // (L1 hits), scale by 2**shift (two exact power-of-two products, so every shift in range
    // is exact) and convert to f16 pairs.  Layout: block (grp, m, t) of 16 bytes holds pairs
    // t, t+4, t+8, t+12 of group grp for row m, stored at block position
    // (grp*M + m)*4 + (t ^ (kg & 3)), kg = 2*kb0 + grp the group's index along all of K, so that
    // the word stores spread over the banks (the prestaged layout of gemv_prestage_kernel is the
    // same with kg in place of grp).  Only the M real rows are staged; the MMA lanes of padding
    // rows use zero registers.
    if (pre) {
      griddep_wait();
      if (threadIdx.x < MP) xshift[threadIdx.x] = threadIdx.x < M ? xpre_shift[threadIdx.x] : 0;
    } else if (!(MXFP4_GV_DIAG & 8)) {
      const int k_lo = kb0 * 64;
      const int nvec = nkb * 8;  // 16-byte vectors (8 bf16) per row in the staged range
      const __nv_bfloat16* a_lo = A + k_lo;
      float am[MP];
#pragma unroll
      for (int m = 0; m < MP; ++m) am[m] = 0.0f;
      for (int v = threadIdx.x; v < nvec; v += 256) {
        const bool kin = k_lo + v * 8 < K;
#pragma unroll
        for (int m = 0; m < MP; ++m)
          if (m < M && kin) {
            const uint4 raw = *reinterpret_cast<const uint4*>(a_lo + static_cast<size_t>(m) * K + v * 8);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              am[m] = fmaxf(am[m], fabsf(__uint_as_float(w[i] << 16)));
              am[m] = fmaxf(am[m], fabsf(__uint_as_float(w[i] & 0xFFFF0000u)));
            }
          }
      }
#pragma unroll
      for (int m = 0; m < MP; ++m)
        if (m < M) {
          float a = am[m];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
          if (lane == 0 && a > 0.0f) atomicMax(xmax + m, __float_as_uint(a));
        }
      named_bar_sync(1, 256);
      if (threadIdx.x < MP) {
        const float amax = __uint_as_float(xmax[threadIdx.x]);
        int shift = 0;
        if (threadIdx.x < M && amax > 0.0f && amax <= 3.0e38f) {
          int E;
          frexpf(amax, &E);
          shift = 15 - E;  // the row max lands in [2^14, 2^15)
        }
        xshift[threadIdx.x] = shift;
      }
      named_bar_sync(1, 256);
      float f1[MP], f2[MP];
#pragma unroll
      for (int m = 0; m < MP; ++m) {
        const int sh = xshift[m];
        f1[m] = exp2i(sh / 2);
        f2[m] = exp2i(sh - sh / 2);
      }
      for (int v = threadIdx.x; v < nvec; v += 256) {
        const bool kin = k_lo + v * 8 < K;
        const int grp = v >> 2, slot = v & 3;  // vector v = pairs 4*slot .. 4*slot+3 of group grp
#pragma unroll
        for (int m = 0; m < MP; ++m)
          if (m < M) {
            uint4 raw = make_uint4(0, 0, 0, 0);
            if (kin) raw = *reinterpret_cast<const uint4*>(a_lo + static_cast<size_t>(m) * K + v * 8);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
            const uint32_t blk = smem_u32(xs + (grp * M + m) * 16 + slot);
#pragma unroll
            for (int tt = 0; tt < 4; ++tt) {
              const float lo = __uint_as_float(w[tt] << 16) * f1[m] * f2[m];
              const float hi = __uint_as_float(w[tt] & 0xFFFF0000u) * f1[m] * f2[m];
              sts32(blk + (tt ^ ((grp + 2 * kb0) & 3)) * 16, f16x2_from(lo, hi));
            }
          }
      }
    }
    named_bar_sync(1, 256);

    // ------------------------------------------------------------ tensor-core GEMV
    const int row = 16 * warp + g;
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
    const uint32_t ring_a = smem_u32(ring);
    const uint32_t xs_a = smem_u32(xs);
    const uint32_t lane_d = chunk_unit(16 * warp + g, t) * 16;  // this lane's fragment unit
    const uint32_t lane_s = kChunkData + (8 * warp + g) * 4;
    // activation block of (local group xg, row 8*jt + g) for this lane: lane_x[xg & 3] + xg*M*64 + jt*512
    uint32_t lane_x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) lane_x[j] = g * 64 + (t ^ ((j + 2 * kb0) & 3)) * 16;
    const uint32_t m64 = static_cast<uint32_t>(M) * 64;
    bool row_live[NT];
#pragma unroll
    for (int jt = 0; jt < NT; ++jt) row_live[jt] = 8 * jt + g < M;
    for (int i = 0; i < nst; ++i) {
      const int s = i % stages;
      if (!warp_wait(&full[s], (i / stages) & 1, kErrWaitFull, abort_flag)) break;
      const uint32_t st = ring_a + s * sbytes;
      // activation blocks of this stage's chunks (2*M*64 bytes each): in the stage after the
      // weights when prestaged, else in the staged region
      const uint32_t xstage = pre ? st + kGvStageWBytes : xs_a + static_cast<uint32_t>(i) * (2 * kGvStageChunks) * m64;
#pragma unroll
      for (int c = 0; c < kGvStageChunks; ++c) {
        const int ci = i * kGvStageChunks + c;
        if (ci < nkb) {
          const uint4 d = lds128(st + c * kChunkBytes + lane_d);
          const uint32_t sw = lds32(st + c * kChunkBytes + lane_s);
          const uint32_t wv[4] = {d.x, d.y, d.z, d.w};  // (g,G0) (g+8,G0) (g,G1) (g+8,G1)
          // scale bytes (g,G0) (g+8,G0) (g,G1) (g+8,G1) -> 2**(s-127) as f32 bits (s << 23);
          // a zero byte (2**-127) decodes to 0, a difference far below the error bound.
          const float sc[4] = {__uint_as_float((sw << 23) & 0x7F800000u), __uint_as_float((sw << 15) & 0x7F800000u),
                               __uint_as_float((sw << 7) & 0x7F800000u), __uint_as_float((sw >> 1) & 0x7F800000u)};
#pragma unroll
          for (int G = 0; G < 2; ++G) {
#if MXFP4_GV_DIAG & 2
            const float sl = 1.0f, sh = __uint_as_float(sw);
#else
            const float sl = sc[2 * G], sh = sc[2 * G + 1];
#endif
            uint32_t fl[4], fh[4];
#if MXFP4_GV_DIAG & 1
            fl[0] = wv[2 * G]; fl[1] = wv[2 * G] >> 4; fl[2] = wv[2 * G] >> 8; fl[3] = wv[2 * G] >> 12;
            fh[0] = wv[2 * G + 1]; fh[1] = wv[2 * G + 1] >> 4; fh[2] = wv[2 * G + 1] >> 8; fh[3] = wv[2 * G + 1] >> 12;
#else
            e2m1x8_to_f16x2(wv[2 * G], fl);
            e2m1x8_to_f16x2(wv[2 * G + 1], fh);
#endif
            const int xl = 2 * c + G;  // group index within the stage; (2*ci + G) & 3 == xl & 3
#pragma unroll
            for (int jt = 0; jt < NT; ++jt) {
              uint4 xb = make_uint4(0, 0, 0, 0);
              if (row_live[jt]) xb = lds128(lane_x[xl & 3] + xstage + xl * m64 + jt * 512);
              float dd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#if MXFP4_GV_DIAG & 4
              dd[0] = __uint_as_float((fl[0] ^ fh[1] ^ fl[2] ^ fh[3] ^ xb.x ^ xb.w) & 0x3fffffff);
#else
              mma_f16_16816(dd, fl[0], fh[0], fl[1], fh[1], xb.x, xb.y);
              mma_f16_16816(dd, fl[2], fh[2], fl[3], fh[3], xb.z, xb.w);
#endif
              acc[jt][0] = fmaf(dd[0], sl, acc[jt][0]);
              acc[jt][1] = fmaf(dd[1], sl, acc[jt][1]);
              acc[jt][2] = fmaf(dd[2], sh, acc[jt][2]);
              acc[jt][3] = fmaf(dd[3], sh, acc[jt][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    named_bar_sync(1, 256);  // every warp is done reading the ring before it holds the partials
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int c0 = 8 * j + 2 * t;
      red[row * MP + c0] = ldexpf(acc[j][0], -xshift[c0]);
      red[row * MP + c0 + 1] = ldexpf(acc[j][1], -xshift[c0 + 1]);
      red[(row + 8) * MP + c0] = ldexpf(acc[j][2], -xshift[c0]);
      red[(row + 8) * MP + c0 + 1] = ldexpf(acc[j][3], -xshift[c0 + 1]);
    }
  }

  // ------------------------------------------------------------ cluster split-K reduction
  cluster_sync_all();
  const int rows_per = kChunkRows / ks;
  const int row_lo = split * rows_per;
  for (int e = threadIdx.x; e < rows_per * M; e += kGvThreads) {
    const int rl = e % rows_per, m = e / rows_per;
    const int row = row_lo + rl;
    float sum = 0.0f;
    for (int r = 0; r < ks; ++r) sum += ld_dsmem_f32(red + row * MP + m, static_cast<uint32_t>(r));
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

// Activation staging done once per GEMM for the decode kernel (used when the caller gives
// workspace for it): one CTA per activation row computes the row's max |x| over all of K, a
// power-of-two shift that puts it in [2^14, 2^15), and writes the row as f16 pairs in the
// layout gemv_kernel stages into shared memory, over all k_blocks*64 columns (zeros past K):
// 16-byte block (kg, m, t), kg the 32-group index along K, at block position
// (kg*M + m)*4 + (t ^ (kg & 3)), holding pairs t, t+4, t+8, t+12 of the group.  Each decode
// CTA then fetches its K range with one bulk copy instead of converting it again.  The
// dependent decode launch may start as soon as every CTA here has begun.
__global__ void __launch_bounds__(256) gemv_prestage_kernel(const __nv_bfloat16* __restrict__ A, int M, int K,
                                                            int k_blocks, uint8_t* __restrict__ xpre,
                                                            int* __restrict__ xpre_shift) {
  griddep_launch_dependents();
  __shared__ float wmax[8];
  const int m = blockIdx.x;
  const int nvec = k_blocks * 8;
  const __nv_bfloat16* arow = A + static_cast<size_t>(m) * K;
  float amax = 0.0f;
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
  if (threadIdx.x == 0) xpre_shift[m] = shift;
  const float f1 = exp2i(shift / 2), f2 = exp2i(shift - shift / 2);
  for (int v = threadIdx.x; v < nvec; v += 256) {
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (v * 8 < K) raw = *reinterpret_cast<const uint4*>(arow + v * 8);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    const int kg = v >> 2, slot = v & 3;
    uint32_t* blk = reinterpret_cast<uint32_t*>(xpre) + (static_cast<size_t>(kg) * M + m) * 16 + slot;
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {
      const float lo = __uint_as_float(w[tt] << 16) * f1 * f2;
      const float hi = __uint_as_float(w[tt] & 0xFFFF0000u) * f1 * f2;
      blk[(tt ^ (kg & 3)) * 4] = f16x2_from(lo, hi);
    }
  }
}

}  // namespace mxb
