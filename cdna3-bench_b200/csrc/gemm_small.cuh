// Small-M (decode, M <= 16) MXFP4 x BF16 GEMM.  HBM-bound: the job is to stream the
// packed weights once at full bandwidth and keep the per-element instruction count low.
//
// * Grid (N/128 weight-row blocks, KS K-splits); the KS CTAs of a row block form one
//   thread-block cluster and reduce their partial sums through distributed shared memory,
//   so the kernel needs no global scratch and no second launch.
// * A producer warp streams the CTA's contiguous run of 4352-byte prepacked chunks into an
//   8-slot smem ring with 1-D bulk copies (mbarrier complete_tx).
// * Eight compute warps own 16 weight rows each.  Weights are converted in registers with
//   the hardware E2M1->f16 conversion (exact, unscaled) straight into mma.sync fragments;
//   the activations are staged once per CTA in f16, pre-scaled per row by a power of two
//   so that every bf16 activation is represented exactly (up to f16 subnormal range at the
//   row's small end).  Each 32-element group's fp32 partial is multiplied by its E8M0
//   scale 2**(s-127) and accumulated in fp32; the per-row activation shift is undone
//   before the cross-CTA reduction.
//
// Fragment/layout contract with the prepack: in a 16-byte row-group, 4-byte word w holds
// k-pairs {w, w+4, w+8, w+12}; lane (g, t) of an m16n8k16 MMA needs exactly pairs t and
// t+4 (first MMA) and t+8, t+12 (second MMA) of rows g and g+8, i.e. one word per row.
#pragma once

#include "common.cuh"

namespace mxb {

constexpr int kGvThreads = 288;  // 8 compute warps + 1 producer warp
constexpr int kGvRing = 8;

template <int NT>
struct GvCfg {
  static constexpr int kMP = 8 * NT;  // padded activation rows
  static constexpr int kOffBar = kGvRing * kChunkBytes;
  static constexpr int kOffShift = kOffBar + 2 * kGvRing * 8;
  static constexpr int kOffMax = kOffShift + 4 * kMP + 16;
  static constexpr int kOffRed = (kOffMax + 4 * kMP + 127) & ~127;
  static constexpr int kOffX = kOffRed + kChunkRows * kMP * 4;
  static constexpr int kXBytesPerKb = 2 * kMP * 64;  // two 32-groups x MP rows x 16 f16 pairs
  static int smem_bytes(int kb_per_split) { return kOffX + kb_per_split * kXBytesPerKb; }
};

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
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

template <int NT, typename OutT>
__global__ void __launch_bounds__(kGvThreads)
    gemv_kernel(const __nv_bfloat16* __restrict__ A, int M, int K, const uint8_t* __restrict__ wpack,
                int k_blocks, int kb_per_split, OutT* __restrict__ C, int N) {
  using Cfg = GvCfg<NT>;
  constexpr int MP = Cfg::kMP;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* empty = full + kGvRing;
  int* xshift = reinterpret_cast<int*>(smem + Cfg::kOffShift);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(xshift + MP);
  float* xmax = reinterpret_cast<float*>(smem + Cfg::kOffMax);
  float* red = reinterpret_cast<float*>(smem + Cfg::kOffRed);
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + Cfg::kOffX);

  const int nb = blockIdx.x;
  const int split = blockIdx.y;
  const int ks = gridDim.y;  // == cluster size; rank of this CTA == split
  const int kb0 = split * kb_per_split;
  const int nkb = max(0, min(k_blocks, kb0 + kb_per_split) - kb0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kGvRing; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < MP) xmax[threadIdx.x] = 0.0f;
  __syncthreads();

  if (warp == 8) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      const uint8_t* src = wpack + (static_cast<size_t>(nb) * k_blocks + kb0) * kChunkBytes;
      uint32_t pend = 0, pend_ph = 0;
      bool aborted = false;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % kGvRing;
        const uint32_t ph = (i / kGvRing) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
          aborted = true;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kChunkBytes);
        bulk_load(ring + s * kChunkBytes, src + static_cast<size_t>(i) * kChunkBytes, kChunkBytes, &full[s]);
        pend |= 1u << s;
        pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
      }
      if (aborted)
        for (int i = 0; i < kGvRing; ++i)
          if ((pend >> i) & 1) mbar_wait_drain(&full[i], (pend_ph >> i) & 1);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ stage activations (f16)
    // All 256 compute threads split the staged K range.  Pass 1: per-row max |x| (warp
    // reduce + shared atomicMax on the float bits, valid for non-negative floats).  Pass 2:
    // scale by 2**shift and convert to f16 pairs.  Layout: block (grp, m, t) of 16 bytes holds
    // pairs t, t+4, t+8, t+12 of group grp for row m, stored at block position
    // (grp*MP + m)*4 + (t ^ (grp & 3)) so that the pass-2 word stores spread over the banks.
    const int k_lo = kb0 * 64;
    const int nvec = nkb * 8;  // 16-byte vectors (8 bf16) per row in the staged range
    const int tid = threadIdx.x;
    for (int m = 0; m < M; ++m) {
      float amax = 0.0f;
      for (int v = tid; v < nvec; v += 256) {
        const int k = k_lo + v * 8;
        if (k < K) {
          const uint4 raw = *reinterpret_cast<const uint4*>(A + static_cast<size_t>(m) * K + k);
          const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            amax = fmaxf(amax, fabsf(__uint_as_float(w[i] << 16)));
            amax = fmaxf(amax, fabsf(__uint_as_float(w[i] & 0xFFFF0000u)));
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (lane == 0 && amax > 0.0f) atomicMax(reinterpret_cast<unsigned*>(xmax) + m, __float_as_uint(amax));
    }
    named_bar_sync(1, 256);
    if (tid < MP) {
      const float amax = __uint_as_float(reinterpret_cast<unsigned*>(xmax)[tid]);
      int shift = 0;
      if (amax > 0.0f && amax <= 3.0e38f) {
        int E;
        frexpf(amax, &E);
        shift = 15 - E;  // the row max lands in [2^14, 2^15)
      }
      xshift[tid] = shift;
    }
    named_bar_sync(1, 256);
    for (int e = tid; e < MP * nvec; e += 256) {
      const int m = e / nvec, v = e - m * nvec;
      const int k = k_lo + v * 8;
      uint4 raw = make_uint4(0, 0, 0, 0);
      if (m < M && k < K) raw = *reinterpret_cast<const uint4*>(A + static_cast<size_t>(m) * K + k);
      const int shift = xshift[m];
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      const int grp = v >> 2, slot = v & 3;  // vector v = pairs 4*slot .. 4*slot+3 of group grp
      const uint32_t blk = smem_u32(xs + (grp * MP + m) * 16 + slot);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float lo = ldexpf(__uint_as_float(w[t] << 16), shift);
        const float hi = ldexpf(__uint_as_float(w[t] & 0xFFFF0000u), shift);
        sts32(blk + (t ^ (grp & 3)) * 16, f16x2_from(lo, hi));
      }
    }
    named_bar_sync(1, 256);

    // ------------------------------------------------------------ tensor-core GEMV
    const int g = lane >> 2, t = lane & 3;
    const int row = 16 * warp + g;
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
    const uint32_t ring_a = smem_u32(ring);
    const uint32_t xs_a = smem_u32(xs);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kGvRing;
      if (!warp_wait(&full[s], (i / kGvRing) & 1, kErrWaitFull, abort_flag)) break;
      const uint32_t ch = ring_a + s * kChunkBytes;
#pragma unroll
      for (int G = 0; G < 2; ++G) {
        const uint32_t wl = lds32(ch + G * 2048 + row * 16 + 4 * t);
        const uint32_t wh = lds32(ch + G * 2048 + (row + 8) * 16 + 4 * t);
        const float sl = e8m0_to_f32(lds_u8(ch + kChunkData + G * kChunkRows + row));
        const float sh = e8m0_to_f32(lds_u8(ch + kChunkData + G * kChunkRows + row + 8));
        uint32_t fl[4], fh[4];
        e2m1x8_to_f16x2(wl, fl);
        e2m1x8_to_f16x2(wh, fh);
        const int xg = 2 * i + G;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const uint4 xb = lds128(xs_a + (((xg * MP + 8 * j + g) * 4 + (t ^ (xg & 3))) * 4) * 4);
          float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          mma_f16_16816(d, fl[0], fh[0], fl[1], fh[1], xb.x, xb.y);
          mma_f16_16816(d, fl[2], fh[2], fl[3], fh[3], xb.z, xb.w);
          acc[j][0] = fmaf(d[0], sl, acc[j][0]);
          acc[j][1] = fmaf(d[1], sl, acc[j][1]);
          acc[j][2] = fmaf(d[2], sh, acc[j][2]);
          acc[j][3] = fmaf(d[3], sh, acc[j][3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
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
    if (n < N) C[static_cast<size_t>(m) * N + n] = gv_out<OutT>(sum);
  }
  cluster_sync_all();
}

}  // namespace mxb
