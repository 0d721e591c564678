// Small-M (decode, M <= 16) MXFP4 x BF16 GEMM, persistent stream-K form.
//
// Decode GEMMs are bound by streaming the packed weights from HBM once.  Two things keep a
// streaming kernel below the HBM rate: too few bytes in flight per SM (each SM must cover the
// DRAM latency with outstanding copies) and work that does not divide evenly into waves of CTAs
// (a short weight matrix leaves most SMs idle in its last wave).  This kernel addresses both:
//
// * One CTA per SM, each streaming an equal, contiguous share of the (128-row weight block,
//   64-k chunk) sequence in row-block-major order -- the shares differ by at most one chunk, so
//   all SMs finish together whatever the shape.
// * A producer warp keeps a ring of up to 64 one-chunk stages (~200 KB of shared memory) full
//   with 1-D bulk copies: the chunk's 4352 bytes of weights plus its 128*M bytes of activations
//   (f16, pre-scaled per row by a power of two so that every bf16 value is exact, staged once
//   per GEMM by gemv_sk_prestage_kernel), so the whole ring is in flight from the start.
// * 16 compute warps in 4 groups; group q takes the CTA's chunks i = q (mod 4) and each of its
//   warps owns 32 weight rows (two m16 tiles) of the chunk.  Weights go through the hardware
//   E2M1 -> f16 conversion (exact, unscaled) into mma.sync.m16n8k16 fragments with the
//   activation rows as the n8 operand; each 32-element group's fp32 partial is multiplied by
//   its E8M0 scale 2**(s-127) and accumulated in fp32 registers.
// * Where a CTA's share ends inside a row block, several CTAs hold partial sums of it: at the
//   end of each row-block segment every warp adds its partial sums into an fp32 buffer in
//   workspace (zeroed by the prestage kernel) with global reductions, fences, and adds the
//   number of chunks it covered to the row block's counter.  The warp whose addition completes
//   the count (4 warps x k_blocks chunks) converts the row block's 128 x M sums to the output
//   (undoing the activation row shifts) and writes it to every destination.  No warp waits
//   for another one: there is no inter-CTA barrier and no named barrier, so a wait that gives
//   up cannot strand anybody.
// * The launch carries the programmatic-dependent-launch attribute: it starts while the
//   prestage kernel runs, issues its first weight copies and waits (griddepcontrol.wait) only
//   before it touches the activations, the sums or the counters.
#pragma once

#include "common.cuh"
#include "gemm_small.cuh"

namespace mxb {

constexpr int kSkGroups = 4;                     // chunk groups (chunks i = q mod 4)
constexpr int kSkComputeWarps = 4 * kSkGroups;   // each group: 4 warps x 32 weight rows
constexpr int kSkThreads = 32 * (kSkComputeWarps + 1);  // + 1 producer warp = 544
constexpr int kSkMaxStages = 64;
constexpr int kSkRingBytes = 200 * 1024;

// Host and device agree on the ring from these.
__host__ __device__ constexpr int sk_stage_bytes(int M) { return kChunkBytes + 128 * M; }
__host__ __device__ constexpr int sk_stages(int M) {
  return (kSkRingBytes / sk_stage_bytes(M) < kSkMaxStages ? kSkRingBytes / sk_stage_bytes(M) : kSkMaxStages) & ~3;
}
__host__ __device__ constexpr int sk_off_bar(int M) { return sk_stages(M) * sk_stage_bytes(M); }
__host__ __device__ constexpr int sk_smem_bytes(int M) { return sk_off_bar(M) + 2 * kSkMaxStages * 8 + 16; }

// Workspace of the stream-K decode path, carved in this order (each part 256-byte aligned):
//   activations f16, k_blocks * 128 * M bytes (gemv_prestage_kernel's layout);
//   row shifts int[16];
//   fp32 sums [M][n_blocks * 128];
//   chunk counters int[n_blocks].
struct SkWorkspace {
  size_t x_off, shift_off, acc_off, cnt_off, total;
};
__host__ __device__ inline size_t sk_align(size_t x) { return (x + 255) / 256 * 256; }
__host__ __device__ inline SkWorkspace sk_workspace(int M, int n_blocks, int k_blocks) {
  SkWorkspace w;
  w.x_off = 0;
  w.shift_off = sk_align(static_cast<size_t>(k_blocks) * 128 * M);
  w.acc_off = w.shift_off + 256;
  w.cnt_off = w.acc_off + sk_align(static_cast<size_t>(M) * n_blocks * kChunkRows * 4);
  w.total = w.cnt_off + sk_align(static_cast<size_t>(n_blocks) * 4);
  return w;
}

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Activations to f16 for the stream-K kernel, and the zeroing of its sums and counters.
// Blocks b < M stage activation row b exactly as gemv_prestage_kernel does; every block also
// zeroes its share of the fp32 sums and chunk counters.  The dependent decode launch may start
// as soon as every block here has begun.
__global__ void __launch_bounds__(256) gemv_sk_prestage_kernel(const __nv_bfloat16* __restrict__ A, int M, int K,
                                                               int k_blocks, uint8_t* __restrict__ xpre,
                                                               int* __restrict__ xshift, float4* __restrict__ zero,
                                                               long long zero_n4) {
  griddep_launch_dependents();
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < zero_n4; i += static_cast<long long>(gridDim.x) * 256)
    zero[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const int m = blockIdx.x;
  if (m >= M) return;
  __shared__ float wmax[8];
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
    shift = 15 - E;  // the row max lands in [2^14, 2^15)
  }
  if (threadIdx.x == 0) xshift[m] = shift;
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

template <int NT, typename OutT>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemv_sk_kernel(const uint8_t* __restrict__ wpack, int M, int N, int k_blocks, int n_blocks,
                   const uint8_t* __restrict__ xpre, const int* __restrict__ xshift, float* __restrict__ acc,
                   int* __restrict__ cnt, const GvOut<OutT> out) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int stages = sk_stages(M);
  const int sbytes = sk_stage_bytes(M);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sk_off_bar(M));
  uint64_t* empty = full + kSkMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kSkMaxStages);

  const long long units = static_cast<long long>(n_blocks) * k_blocks;
  const long long u0 = units * blockIdx.x / gridDim.x;
  const int n_my = static_cast<int>(units * (blockIdx.x + 1) / gridDim.x - u0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t xbytes = 128u * M;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);  // the four warps of the stage's group
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kSkComputeWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint64_t pend = 0, pend_ph = 0;
      bool aborted = false, waited = false;
      const int n_issue = test_withhold() ? 0 : n_my;  // test switch: issue nothing
      for (int i = 0; i < n_issue; ++i) {
        const int s = i % stages;
        const uint32_t ph = (i / stages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
          aborted = true;
          break;
        }
        const long long u = u0 + i;
        const int kc = static_cast<int>(u % k_blocks);
        uint8_t* st = smem + s * sbytes;
        mbar_arrive_expect_tx(&full[s], kChunkBytes + xbytes);
        bulk_load(st, wpack + u * kChunkBytes, kChunkBytes, &full[s]);
        if (!waited) {  // the activations come from the prestage launch just before this one
          griddep_wait();
          waited = true;
        }
        bulk_load(st + kChunkBytes, xpre + static_cast<size_t>(kc) * xbytes, xbytes, &full[s]);
        pend |= 1ull << s;
        pend_ph = (pend_ph & ~(1ull << s)) | (static_cast<uint64_t>(ph) << s);
      }
      if (aborted)  // let every copy we started land before the CTA can exit
        for (int i = 0; i < stages; ++i)
          if ((pend >> i) & 1) mbar_wait_drain(&full[i], (pend_ph >> i) & 1);
    }
    return;
  }

  // -------------------------------------------------------------- compute warps
  griddep_wait();  // sums and counters zeroed, row shifts written
  const int q = warp >> 2;   // chunk group
  const int wq = warp & 3;   // rows 32*wq .. 32*wq+31 of every chunk
  const int g = lane >> 2, t = lane & 3;
  const int Np = n_blocks * kChunkRows;
  uint32_t lane_d[2], lane_s[2];
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    lane_d[a] = chunk_unit(32 * wq + 16 * a + g, t) * 16;
    lane_s[a] = kChunkData + (8 * (2 * wq + a) + g) * 4;
  }
  bool row_live[NT];
  uint32_t xrow[NT];  // this lane's activation block offset for group G = 0 (without the slot)
#pragma unroll
  for (int jt = 0; jt < NT; ++jt) {
    row_live[jt] = 8 * jt + g < M;
    xrow[jt] = (8 * jt + g) * 64;
  }
  const uint32_t x_g1 = static_cast<uint32_t>(M) * 64;  // group G = 1 starts M rows further
  float accr[2][NT][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int j = 0; j < NT; ++j) accr[a][j][0] = accr[a][j][1] = accr[a][j][2] = accr[a][j][3] = 0.0f;

  // Adds this warp's partial sums of row block rb (covering nch chunks) into the fp32 sums and
  // the row block's counter; the warp that completes the count writes the row block's output.
  auto flush = [&](int rb, int nch) {
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int jt = 0; jt < NT; ++jt) {
        const int n = rb * kChunkRows + 32 * wq + 16 * a + g;
        const int m = 8 * jt + 2 * t;
        if (m < M) {
          red_add_f32(acc + static_cast<size_t>(m) * Np + n, accr[a][jt][0]);
          red_add_f32(acc + static_cast<size_t>(m) * Np + n + 8, accr[a][jt][2]);
        }
        if (m + 1 < M) {
          red_add_f32(acc + static_cast<size_t>(m + 1) * Np + n, accr[a][jt][1]);
          red_add_f32(acc + static_cast<size_t>(m + 1) * Np + n + 8, accr[a][jt][3]);
        }
        accr[a][jt][0] = accr[a][jt][1] = accr[a][jt][2] = accr[a][jt][3] = 0.0f;
      }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(cnt + rb, nch) + nch == 4 * k_blocks;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    for (int m = 0; m < M; ++m) {
      const int sh = __ldcg(xshift + m);
#pragma unroll
      for (int r = lane; r < kChunkRows; r += 32) {
        const int n = rb * kChunkRows + r;
        if (n < N) {
          const OutT v = gv_out<OutT>(ldexpf(__ldcg(acc + static_cast<size_t>(m) * Np + n), -sh));
#pragma unroll
          for (int d = 0; d < 8; ++d)  // fixed trip count: out.p stays in the parameter space
            if (d < out.count) out.p[d][static_cast<size_t>(m) * out.ldc + out.n_off + n] = v;
        }
      }
    }
    if (out.fence_sys) __threadfence_system();
  };

  int seg_rb = -1, seg_n = 0;
  for (int i = q; i < n_my; i += kSkGroups) {
    const long long u = u0 + i;
    const int rb = static_cast<int>(u / k_blocks);
    const int kc = static_cast<int>(u - static_cast<long long>(rb) * k_blocks);
    if (rb != seg_rb) {
      if (seg_rb >= 0) flush(seg_rb, seg_n);
      seg_rb = rb;
      seg_n = 0;
    }
    const int s = i % stages;
    if (!warp_wait(&full[s], (i / stages) & 1, kErrWaitFull, abort_flag)) {
      seg_rb = -1;  // aborted: this segment's sums stay incomplete (the error word says so)
      break;
    }
    const uint32_t st = smem_u32(smem + s * sbytes);
    uint4 dw[2];
    uint32_t sw[2];
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      dw[a] = lds128(st + lane_d[a]);
      sw[a] = lds32(st + lane_s[a]);
    }
    const uint32_t xs = st + kChunkBytes;
#pragma unroll
    for (int G = 0; G < 2; ++G) {
      const uint32_t slot = static_cast<uint32_t>(t ^ ((2 * kc + G) & 3)) * 16;
      uint4 xb[NT];
#pragma unroll
      for (int jt = 0; jt < NT; ++jt) {
        xb[jt] = make_uint4(0, 0, 0, 0);
        if (row_live[jt]) xb[jt] = lds128(xs + G * x_g1 + xrow[jt] + slot);
      }
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const uint32_t wl = G ? dw[a].z : dw[a].x;  // row g, group G
        const uint32_t wh = G ? dw[a].w : dw[a].y;  // row g + 8, group G
        // scale bytes (g,G0) (g+8,G0) (g,G1) (g+8,G1) -> 2**(s-127) as f32 bits (s << 23); a
        // zero byte (2**-127) decodes to 0, a difference far below the error bound
        const float sl = __uint_as_float((sw[a] << (23 - 16 * G)) & 0x7F800000u);
        const float sh = __uint_as_float(G ? (sw[a] >> 1) & 0x7F800000u : (sw[a] << 15) & 0x7F800000u);
        uint32_t fl[4], fh[4];
        e2m1x8_to_f16x2(wl, fl);
        e2m1x8_to_f16x2(wh, fh);
#pragma unroll
        for (int jt = 0; jt < NT; ++jt) {
          float dd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          mma_f16_16816(dd, fl[0], fh[0], fl[1], fh[1], xb[jt].x, xb[jt].y);
          mma_f16_16816(dd, fl[2], fh[2], fl[3], fh[3], xb[jt].z, xb[jt].w);
          accr[a][jt][0] = fmaf(dd[0], sl, accr[a][jt][0]);
          accr[a][jt][1] = fmaf(dd[1], sl, accr[a][jt][1]);
          accr[a][jt][2] = fmaf(dd[2], sh, accr[a][jt][2]);
          accr[a][jt][3] = fmaf(dd[3], sh, accr[a][jt][3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    ++seg_n;
  }
  if (seg_rb >= 0) flush(seg_rb, seg_n);
}

}  // namespace mxb
