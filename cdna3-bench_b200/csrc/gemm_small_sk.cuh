// Small-M (decode, M <= 16) MXFP4 x BF16 GEMM, persistent stream-K form.
//
// Decode GEMMs are bound by streaming the packed weights from HBM once.  What keeps a streaming
// kernel below the HBM rate on B200: (1) the TMA engine of an SM handles a 1-D bulk copy at a
// fixed cost of ~460 cycles up to ~16 KB (measured: 4 KB copies stream at 2.6 TB/s, 16 KB ones
// at 6.9 TB/s, whatever the number in flight), so copies must be large; (2) work that does not
// divide into whole waves of CTAs (a short weight matrix leaves most SMs idle in its last wave).
//
// * One CTA per SM, each streaming an equal, contiguous share of the (128-row weight block,
//   64-k chunk) sequence in row-block-major order -- the shares differ by at most one chunk, so
//   all SMs finish together whatever the shape.
// * A producer warp keeps a ring of stages full, each stage kSkStageChunks consecutive chunks of
//   weights fetched with one bulk copy (consecutive chunks of the row-block-major sequence are
//   adjacent in memory: 17 KB per copy).  The activations do not travel through the copy engine
//   (a small copy costs it as much time as a large one): they are staged once per GEMM by
//   gemv_sk_prestage_kernel (f16, pre-scaled per row by a power of two so that every bf16 value
//   is exact; 128*M bytes per chunk, L2-resident) and each compute warp loads its fragments of
//   the next chunk it will process with plain 16-byte loads while it computes the current one.
// * 16 compute warps in groups of WPC (1 for M <= 8, 2 above); group q takes the CTA's chunks
//   i = q (mod 16/WPC) and each of its warps owns 128/WPC weight rows (8/WPC m16 tiles) of the
//   chunk, so the per-chunk work of waiting, indexing and loading activations is paid once per
//   128 or 64 rows.  Weights go through the hardware E2M1 -> f16 conversion (exact, unscaled)
//   into mma.sync.m16n8k16 fragments with the activation rows as the n8 operand; each
//   32-element group's fp32 partial is multiplied by its E8M0 scale 2**(s-127) and accumulated
//   in fp32 registers.  Ring positions and row-block and k indices advance incrementally: no
//   integer division in the streaming loops.
// * At the end of each row-block segment every warp adds its partial sums into an fp32 buffer
//   in workspace (zeroed by the prestage kernel) with global reductions: several CTAs (and
//   several groups of one CTA) hold parts of a row block.  No warp waits for another one: there is
//   no inter-CTA barrier and no named barrier, so a wait that gives up strands nobody.
// * gemv_sk_finalize_kernel turns the sums into the output (undoing the activation row shifts),
//   for every destination.
// * The three launches are chained with programmatic dependent launch: each starts while the one
//   before runs and waits (griddepcontrol.wait) only before it reads that one's results.
#pragma once

#include "common.cuh"
#include "gemm_small.cuh"

namespace mxb {

#ifndef MXFP4_SK_DIAG
#define MXFP4_SK_DIAG 0  // sweep-only: 1 = consumers skip the arithmetic, 2 = the producer issues nothing
                         // and the consumers do not wait for it (compute rate alone), 8 = no global
                         // reductions, 16 = no finalize launch, 32 = no prestage launch; results are
                         // wrong in these builds
#endif

constexpr int kSkComputeWarps = 16;  // consumers; a chunk is shared by WPC of them (template)
constexpr int kSkThreads = 32 * (kSkComputeWarps + 1);  // + 1 producer warp = 544
#ifndef MXFP4_SK_STAGE_CHUNKS
#define MXFP4_SK_STAGE_CHUNKS 4
#endif
constexpr int kSkStageChunks = MXFP4_SK_STAGE_CHUNKS;  // consecutive chunks per ring stage
constexpr int kSkMaxStages = 64;
constexpr int kSkRingBytes = 12 * kSkStageChunks * kChunkBytes;  // 204 KiB: twelve 4-chunk stages

// Host and device agree on the ring from these (the argument M is kept for the interface: the
// ring holds weights only).
__host__ __device__ constexpr int sk_stage_bytes(int M) { return (void)M, kSkStageChunks * kChunkBytes; }
__host__ __device__ constexpr int sk_stages(int M) {
  return kSkRingBytes / sk_stage_bytes(M) < kSkMaxStages ? kSkRingBytes / sk_stage_bytes(M) : kSkMaxStages;
}
__host__ __device__ constexpr int sk_off_bar(int M) { return sk_stages(M) * sk_stage_bytes(M); }
__host__ __device__ constexpr int sk_smem_bytes(int M) { return sk_off_bar(M) + 2 * kSkMaxStages * 8 + 16; }

// Workspace of the stream-K decode path, carved in this order (each part 256-byte aligned):
//   activations f16, k_blocks * 128 * M bytes (gemv_prestage_kernel's layout);
//   row shifts int[16];
//   fp32 sums [M][n_blocks * 128].
struct SkWorkspace {
  size_t x_off, shift_off, acc_off, total;
};
__host__ __device__ inline size_t sk_align(size_t x) { return (x + 255) / 256 * 256; }
__host__ __device__ inline SkWorkspace sk_workspace(int M, int n_blocks, int k_blocks) {
  SkWorkspace w;
  w.x_off = 0;
  w.shift_off = sk_align(static_cast<size_t>(k_blocks) * 128 * M);
  w.acc_off = w.shift_off + 256;
  w.total = w.acc_off + sk_align(static_cast<size_t>(M) * n_blocks * kChunkRows * 4);
  return w;
}

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

constexpr int kSkPreThreads = 1024;
constexpr int kSkPreVecs = 4;  // 16-byte vectors of a row each prestage thread holds (K <= 32768)

// Activations to f16 for the stream-K kernel, and the zeroing of its fp32 sums.  Blocks b < M
// stage activation row b in the layout gemv_prestage_kernel writes: each thread loads its
// (up to four) 16-byte vectors of the row once, the block reduces the row's max |x| to a power-
// of-two shift that puts it in [2^14, 2^15), and the same registers are converted and stored --
// two memory round trips per row.  Every block also zeroes a share of the sums.  The dependent
// decode launch may start as soon as every block here has begun.
__global__ void __launch_bounds__(kSkPreThreads) gemv_sk_prestage_kernel(const __nv_bfloat16* __restrict__ A, int M,
                                                                         int K, int k_blocks,
                                                                         uint8_t* __restrict__ xpre,
                                                                         int* __restrict__ xshift,
                                                                         float4* __restrict__ zero, long long zero_n4) {
  griddep_launch_dependents();
  for (long long i = blockIdx.x * static_cast<long long>(kSkPreThreads) + threadIdx.x; i < zero_n4;
       i += static_cast<long long>(gridDim.x) * kSkPreThreads)
    zero[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const int m = blockIdx.x;
  if (m >= M) return;
  __shared__ float wmax[kSkPreThreads / 32];
  const int nvec = k_blocks * 8;
  const __nv_bfloat16* arow = A + static_cast<size_t>(m) * K;
  uint4 raw[kSkPreVecs];
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < kSkPreVecs; ++j) {
    const int v = threadIdx.x + j * kSkPreThreads;
    raw[j] = make_uint4(0, 0, 0, 0);
    if (v < nvec && v * 8 < K) raw[j] = *reinterpret_cast<const uint4*>(arow + v * 8);
  }
#pragma unroll
  for (int j = 0; j < kSkPreVecs; ++j) {
    const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
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
  for (int i = 0; i < kSkPreThreads / 32; ++i) amax = fmaxf(amax, wmax[i]);
  int shift = 0;
  if (amax > 0.0f && amax <= 3.0e38f) {
    int E;
    frexpf(amax, &E);
    shift = 15 - E;  // the row max lands in [2^14, 2^15)
  }
  if (threadIdx.x == 0) xshift[m] = shift;
  const float f1 = exp2i(shift / 2), f2 = exp2i(shift - shift / 2);
#pragma unroll
  for (int j = 0; j < kSkPreVecs; ++j) {
    const int v = threadIdx.x + j * kSkPreThreads;
    if (v >= nvec) break;
    const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
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

template <int NT, int WPC>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemv_sk_kernel(const uint8_t* __restrict__ wpack, int M, int k_blocks, int n_blocks,
                   const uint8_t* __restrict__ xpre, float* __restrict__ acc) {
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
  const size_t xbytes = 128u * M;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], WPC * kSkStageChunks);  // each chunk's WPC warps
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch_dependents();  // the finalize launch waits for this grid anyway

  if (warp == kSkComputeWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint64_t pend = 0, pend_ph = 0;
      bool aborted = false;
      const int n_issue = (test_withhold() || (MXFP4_SK_DIAG & 2)) ? 0 : n_my;  // test switch: issue nothing
      // stage and its phase parity advance without divisions; the weights do not depend on the
      // prestage launch, so the producer never waits for it
      const int nst = (n_issue + kSkStageChunks - 1) / kSkStageChunks;
      const uint8_t* wsrc = wpack + u0 * kChunkBytes;
      int s = 0;
      uint32_t ph = 0;
      for (int j = 0; j < nst; ++j) {
        if (!mbar_wait(&empty[s], ph ^ 1, kErrWaitEmpty, abort_flag)) {
          aborted = true;
          break;
        }
        const int nch = min(kSkStageChunks, n_issue - j * kSkStageChunks);
        mbar_arrive_expect_tx(&full[s], nch * kChunkBytes);
        bulk_load(smem + s * sbytes, wsrc, nch * kChunkBytes, &full[s]);
        pend |= 1ull << s;
        pend_ph = (pend_ph & ~(1ull << s)) | (static_cast<uint64_t>(ph) << s);
        wsrc += nch * kChunkBytes;
        if (++s == stages) {
          s = 0;
          ph ^= 1;
        }
      }
      if (aborted)  // let every copy we started land before the CTA can exit
        for (int i = 0; i < stages; ++i)
          if ((pend >> i) & 1) mbar_wait_drain(&full[i], (pend_ph >> i) & 1);
    }
    return;
  }

  // -------------------------------------------------------------- compute warps
  constexpr int NG = kSkComputeWarps / WPC;  // chunk groups
  constexpr int RW = kChunkRows / WPC;       // weight rows per warp
  constexpr int MT = RW / 16;                // m16 tiles per warp
  static_assert(kSkComputeWarps % WPC == 0 && NG % kSkStageChunks == 0, "group layout");
  griddep_wait();  // the sums are zeroed and the activations staged
  const int q = warp / WPC;   // chunk group
  const int wq = warp % WPC;  // rows RW*wq .. RW*wq+RW-1 of every chunk
  const int g = lane >> 2, t = lane & 3;
  const int Np = n_blocks * kChunkRows;
  bool row_live[NT];
  uint32_t xrow[NT];  // this lane's activation block offset for group G = 0 (without the slot)
#pragma unroll
  for (int jt = 0; jt < NT; ++jt) {
    row_live[jt] = 8 * jt + g < M;
    xrow[jt] = (8 * jt + g) * 64;
  }
  const uint32_t x_g1 = static_cast<uint32_t>(M) * 64;  // group G = 1 starts M rows further
  // this lane's activation fragments of the chunk with k index kx: block (G, row 8jt+g, slot)
  auto load_x = [&](int kx, uint4 (&xb)[2][NT]) {
    const uint8_t* base = xpre + static_cast<size_t>(kx) * xbytes;
#pragma unroll
    for (int G = 0; G < 2; ++G) {
      const uint32_t slot = static_cast<uint32_t>(t ^ ((2 * kx + G) & 3)) * 16;
#pragma unroll
      for (int jt = 0; jt < NT; ++jt) {
        xb[G][jt] = make_uint4(0, 0, 0, 0);
        if (row_live[jt]) xb[G][jt] = __ldg(reinterpret_cast<const uint4*>(base + G * x_g1 + xrow[jt] + slot));
      }
    }
  };
  float accr[MT][NT][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int j = 0; j < NT; ++j) accr[a][j][0] = accr[a][j][1] = accr[a][j][2] = accr[a][j][3] = 0.0f;

  // Adds this warp's partial sums of row block rb into the fp32 sums and clears them.
  auto flush = [&](int rb) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int jt = 0; jt < NT; ++jt) {
        const int n = rb * kChunkRows + RW * wq + 16 * a + g;
        const int m = 8 * jt + 2 * t;
        if ((MXFP4_SK_DIAG & 8) == 0 && m < M) {
          red_add_f32(acc + static_cast<size_t>(m) * Np + n, accr[a][jt][0]);
          red_add_f32(acc + static_cast<size_t>(m) * Np + n + 8, accr[a][jt][2]);
        }
        if ((MXFP4_SK_DIAG & 8) == 0 && m + 1 < M) {
          red_add_f32(acc + static_cast<size_t>(m + 1) * Np + n, accr[a][jt][1]);
          red_add_f32(acc + static_cast<size_t>(m + 1) * Np + n + 8, accr[a][jt][3]);
        }
        accr[a][jt][0] = accr[a][jt][1] = accr[a][jt][2] = accr[a][jt][3] = 0.0f;
      }
  };

  // chunk i of this CTA: stage i / kSkStageChunks at ring slot s with phase parity ph, position
  // c in the stage, row block rb, k index kc -- advanced by NG chunks per iteration (NG is a
  // multiple of the stage size, so c stays and the slot moves by NG / kSkStageChunks)
  const int c = q % kSkStageChunks;
  int s = (q / kSkStageChunks) % stages;
  uint32_t ph = ((q / kSkStageChunks) / stages) & 1;
  const long long uq = u0 + q;
  int rb = static_cast<int>(uq / k_blocks);
  int kc = static_cast<int>(uq - static_cast<long long>(rb) * k_blocks);
  int seg_rb = -1;
  uint4 xcur[2][NT], xnext[2][NT];
  if (q < n_my) load_x(kc, xcur);
  // m16 tile a of this warp: rows 16 (MT wq + a) + g and + 8; its unit lies 32 units (512 bytes)
  // further per tile and its scale word 8 words further (chunk_unit / chunk_scale_off)
  const uint32_t lane_u = static_cast<uint32_t>(chunk_unit(RW * wq + g, t)) * 16;
  const uint32_t lane_s = kChunkData + (8 * (MT * wq) + g) * 4;
  for (int i = q; i < n_my; i += NG) {
    {  // prefetch the activations of this group's next chunk
      int kn = kc + NG;
      while (kn >= k_blocks) kn -= k_blocks;
      if (i + NG < n_my) load_x(kn, xnext);
    }
    if (rb != seg_rb) {
      if (seg_rb >= 0) flush(seg_rb);
      seg_rb = rb;
    }
    if (!(MXFP4_SK_DIAG & 2) && !warp_wait(&full[s], ph, kErrWaitFull, abort_flag)) {
      seg_rb = -1;  // aborted: this segment's sums stay incomplete (the error word says so)
      break;
    }
    const uint32_t st = smem_u32(smem + s * sbytes) + c * kChunkBytes;  // this chunk's weights
    if (!(MXFP4_SK_DIAG & 1)) {
#pragma unroll
      for (int a = 0; a < MT; ++a) {
        const uint4 dw = lds128(st + lane_u + a * 512);
        const uint32_t sw = lds32(st + lane_s + a * 32);
#pragma unroll
        for (int G = 0; G < 2; ++G) {
          const uint32_t wl = G ? dw.z : dw.x;  // row g, group G
          const uint32_t wh = G ? dw.w : dw.y;  // row g + 8, group G
          // scale bytes (g,G0) (g+8,G0) (g,G1) (g+8,G1) -> 2**(s-127) as f32 bits (s << 23); a
          // zero byte (2**-127) decodes to 0, a difference far below the error bound
          const float sl = __uint_as_float((sw << (23 - 16 * G)) & 0x7F800000u);
          const float sh = __uint_as_float(G ? (sw >> 1) & 0x7F800000u : (sw << 15) & 0x7F800000u);
          uint32_t fl[4], fh[4];
          e2m1x8_to_f16x2(wl, fl);
          e2m1x8_to_f16x2(wh, fh);
#pragma unroll
          for (int jt = 0; jt < NT; ++jt) {
            float dd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            mma_f16_16816(dd, fl[0], fh[0], fl[1], fh[1], xcur[G][jt].x, xcur[G][jt].y);
            mma_f16_16816(dd, fl[2], fh[2], fl[3], fh[3], xcur[G][jt].z, xcur[G][jt].w);
            accr[a][jt][0] = fmaf(dd[0], sl, accr[a][jt][0]);
            accr[a][jt][1] = fmaf(dd[1], sl, accr[a][jt][1]);
            accr[a][jt][2] = fmaf(dd[2], sh, accr[a][jt][2]);
            accr[a][jt][3] = fmaf(dd[3], sh, accr[a][jt][3]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    s += NG / kSkStageChunks;
    if (s >= stages) {
      s -= stages;
      ph ^= 1;
    }
    kc += NG;
    while (kc >= k_blocks) {
      kc -= k_blocks;
      ++rb;
    }
#pragma unroll
    for (int G = 0; G < 2; ++G)
#pragma unroll
      for (int jt = 0; jt < NT; ++jt) xcur[G][jt] = xnext[G][jt];
  }
  if (seg_rb >= 0) flush(seg_rb);
}

// fp32 sums [M][Np] -> C[m][n] = sums * 2**-shift[m] for n < N, to every destination.  Two
// outputs per thread and grid-stride iteration.
template <typename OutT>
__global__ void __launch_bounds__(256) gemv_sk_finalize_kernel(const float* __restrict__ acc,
                                                               const int* __restrict__ xshift, int M, int N, int Np,
                                                               const GvOut<OutT> out) {
  griddep_wait();  // the decode kernel's reductions are complete
  const int half = (N + 1) / 2;
  const long long total = static_cast<long long>(M) * half;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += static_cast<long long>(gridDim.x) * 256) {
    const int m = static_cast<int>(i / half);
    const int n = 2 * static_cast<int>(i - static_cast<long long>(m) * half);
    const int sh = xshift[m];
    const float2 v = *reinterpret_cast<const float2*>(acc + static_cast<size_t>(m) * Np + n);
    const OutT a = gv_out<OutT>(ldexpf(v.x, -sh)), b = gv_out<OutT>(ldexpf(v.y, -sh));
#pragma unroll
    for (int d = 0; d < 8; ++d)  // fixed trip count: out.p stays in the parameter space
      if (d < out.count) {
        OutT* row = out.p[d] + static_cast<size_t>(m) * out.ldc + out.n_off;
        row[n] = a;
        if (n + 1 < N) row[n + 1] = b;
      }
  }
  if (out.fence_sys) __threadfence_system();
}

}  // namespace mxb
