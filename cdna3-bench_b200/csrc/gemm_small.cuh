// Small-M (decode, M <= 16) MXFP4 x BF16 GEMM.  HBM-bound: the job is to stream the
// packed weights once at full bandwidth and keep the per-element instruction count low.
//
// * Grid (N/128 weight-row blocks, KS K-splits); the KS CTAs of a row block form one
//   thread-block cluster and reduce their partial sums through distributed shared memory,
//   so the kernel needs no global scratch and no second launch.
// * Eight warps own 16 weight rows each.  The chunk layout (chunk_word_off in common.cuh)
//   puts every word lane (g, t) of an m16n8k16 MMA needs from a chunk into one 16-byte unit,
//   so each lane streams the weights with coalesced 128-bit loads straight into registers
//   (a warp reads 512 contiguous bytes per chunk); no shared-memory staging of the weights.
//   Loads go out in batches of kGvBatch chunks into two register sets and a set is consumed
//   only as a whole: a rolling one-chunk refill makes each wait also cover younger loads
//   (outstanding loads share a handful of hardware counters) and measured at about a third
//   of the batched bandwidth.
// * Weights are converted in registers with the hardware E2M1->f16 conversion (exact,
//   unscaled) straight into mma.sync fragments; the activations are staged once per CTA in
//   f16, pre-scaled per row by a power of two so that every bf16 activation is represented
//   exactly (up to f16 subnormal range at the row's small end).  Each 32-element group's
//   fp32 partial is multiplied by its E8M0 scale 2**(s-127) and accumulated in fp32; the
//   per-row activation shift is undone before the cross-CTA reduction.
#pragma once

#include "common.cuh"

namespace mxb {

#ifndef MXFP4_GV_MINB
#define MXFP4_GV_MINB 1
#endif
#ifndef MXFP4_GV_DIAG
#define MXFP4_GV_DIAG 0
#endif
constexpr int kGvThreads = 256;  // 8 warps x 16 weight rows
constexpr int kGvBatch = 4;      // chunks per load batch; two batches in flight per lane

template <int NT>
struct GvCfg {
  static constexpr int kMP = 8 * NT;  // padded activation rows
  static constexpr int kOffShift = 0;
  static constexpr int kOffRed = (kOffShift + 4 * kMP + 127) & ~127;
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

// Streaming loads of data read exactly once (read-only path, no L1 allocation).
__device__ __forceinline__ uint4 ldg_stream128(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_stream32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
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
__global__ void __launch_bounds__(kGvThreads, MXFP4_GV_MINB)
    gemv_kernel(const __nv_bfloat16* __restrict__ A, int M, int K, const uint8_t* __restrict__ wpack,
                int k_blocks, int kb_per_split, OutT* __restrict__ C, int N) {
  using Cfg = GvCfg<NT>;
  constexpr int MP = Cfg::kMP;
  extern __shared__ __align__(128) uint8_t smem[];
  int* xshift = reinterpret_cast<int*>(smem + Cfg::kOffShift);
  float* red = reinterpret_cast<float*>(smem + Cfg::kOffRed);
  uint32_t* xs = reinterpret_cast<uint32_t*>(smem + Cfg::kOffX);

  const int nb = blockIdx.x;
  const int split = blockIdx.y;
  const int ks = gridDim.y;  // == cluster size; rank of this CTA == split
  const int kb0 = split * kb_per_split;
  const int nkb = max(0, min(k_blocks, kb0 + kb_per_split) - kb0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int g = lane >> 2, t = lane & 3;

  // Weight stream; the first batch goes out before the activations are staged.
  const uint8_t* wbase = wpack + (static_cast<size_t>(nb) * k_blocks + kb0) * kChunkBytes;
  const uint8_t* dptr = wbase + (32 * warp + lane) * 16;          // this lane's 16-byte unit
  const uint8_t* sptr = wbase + kChunkData + (8 * warp + g) * 4;  // its four scales
  uint4 da[kGvBatch], db[kGvBatch];
  uint32_t sa[kGvBatch], sb[kGvBatch];
  auto load_batch = [&](uint4(&d)[kGvBatch], uint32_t(&sc)[kGvBatch], int c0) {
#pragma unroll
    for (int j = 0; j < kGvBatch; ++j)
      if (c0 + j < nkb) {
        d[j] = ldg_stream128(dptr + static_cast<size_t>(c0 + j) * kChunkBytes);
        sc[j] = ldg_stream32(sptr + static_cast<size_t>(c0 + j) * kChunkBytes);
      }
  };
  load_batch(da, sa, 0);

  // ------------------------------------------------------------ stage activations (f16)
  // Warp w stages rows w, w+8, ... of this CTA's K range.  Pass 1: the row's max |x| (loads
  // unrolled, one warp reduction).  Pass 2: re-read (L1 hits), scale by 2**shift and convert to
  // f16 pairs.  Layout: block (grp, m, t) of 16 bytes holds pairs t, t+4, t+8, t+12 of group
  // grp for row m, stored at block position (grp*MP + m)*4 + (t ^ (grp & 3)) so that the
  // pass-2 word stores spread over the banks.  Rows m >= M are zero.
  {
    const int k_lo = kb0 * 64;
    const int nvec = nkb * 8;  // 16-byte vectors (8 bf16) per row in the staged range
    for (int m = warp; m < MP; m += kGvThreads / 32) {
      const __nv_bfloat16* arow = A + static_cast<size_t>(m) * K;
      int shift = 0;
      if (m < M) {
        float amax = 0.0f;
#pragma unroll 8
        for (int v = lane; v < nvec; v += 32) {
          const int k = k_lo + v * 8;
          if (k < K) {
            const uint4 raw = *reinterpret_cast<const uint4*>(arow + k);
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
        if (amax > 0.0f && amax <= 3.0e38f) {
          int E;
          frexpf(amax, &E);
          shift = 15 - E;  // the row max lands in [2^14, 2^15)
        }
      }
      if (lane == 0) xshift[m] = shift;
#pragma unroll 4
      for (int v = lane; v < nvec; v += 32) {
        const int k = k_lo + v * 8;
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (m < M && k < K) raw = *reinterpret_cast<const uint4*>(arow + k);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        const int grp = v >> 2, slot = v & 3;  // vector v = pairs 4*slot .. 4*slot+3 of group grp
        const uint32_t blk = smem_u32(xs + (grp * MP + m) * 16 + slot);
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
          const float lo = ldexpf(__uint_as_float(w[tt] << 16), shift);
          const float hi = ldexpf(__uint_as_float(w[tt] & 0xFFFF0000u), shift);
          sts32(blk + (tt ^ (grp & 3)) * 16, f16x2_from(lo, hi));
        }
      }
    }
  }
  __syncthreads();

  // ------------------------------------------------------------ tensor-core GEMV
  const int row = 16 * warp + g;
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  const uint32_t xs_a = smem_u32(xs);
  auto use_batch = [&](const uint4(&d)[kGvBatch], const uint32_t(&sc)[kGvBatch], int c0) {
#pragma unroll
    for (int j = 0; j < kGvBatch; ++j) {
      const int i = c0 + j;
      if (i < nkb) {
        const uint32_t wv[4] = {d[j].x, d[j].y, d[j].z, d[j].w};  // (g,G0) (g+8,G0) (g,G1) (g+8,G1)
        const uint32_t sw = sc[j];
#pragma unroll
        for (int G = 0; G < 2; ++G) {
          const float sl = e8m0_to_f32((sw >> (16 * G)) & 0xFF);
          const float sh = e8m0_to_f32((sw >> (16 * G + 8)) & 0xFF);
          uint32_t fl[4], fh[4];
          e2m1x8_to_f16x2(wv[2 * G], fl);
          e2m1x8_to_f16x2(wv[2 * G + 1], fh);
          const int xg = 2 * i + G;
#pragma unroll
          for (int jt = 0; jt < NT; ++jt) {
            const uint4 xb = lds128(xs_a + (((xg * MP + 8 * jt + g) * 4 + (t ^ (xg & 3))) * 4) * 4);
            float dd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#if MXFP4_GV_DIAG == 1
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
  };
  for (int c = 0; c < nkb; c += 2 * kGvBatch) {
    load_batch(db, sb, c + kGvBatch);
    use_batch(da, sa, c);
    load_batch(da, sa, c + 2 * kGvBatch);
    use_batch(db, sb, c + kGvBatch);
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int c0 = 8 * j + 2 * t;
    red[row * MP + c0] = ldexpf(acc[j][0], -xshift[c0]);
    red[row * MP + c0 + 1] = ldexpf(acc[j][1], -xshift[c0 + 1]);
    red[(row + 8) * MP + c0] = ldexpf(acc[j][2], -xshift[c0]);
    red[(row + 8) * MP + c0 + 1] = ldexpf(acc[j][3], -xshift[c0 + 1]);
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
