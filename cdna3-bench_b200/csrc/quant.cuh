// Format kernels: MXFP4 quantisers, dequantisers and the weight prepack.
//
// All of these are HBM-bound byte work: one thread per 32-element group (or per byte
// column for the reference layout), loads coalesced across neighbouring threads.
#pragma once

#include "common.cuh"

namespace mxb {

// ------------------------------------------------------------------------------------
// Quantisers.  Input fp32 [rows, cols] row-major, quantised along `axis`:
//   axis 0: packed [rows/2, cols], scales [rows/32, cols]  (the reference's weight layout)
//   axis 1: packed [rows, cols/2], scales [rows, cols/32]
// rule 0 = the reference rule (ref.py:14-47): e = ceil(log2(max(amax,1e-38)/6)) clipped to
//          [-127,127], nearest E2M1 magnitude with ties to the LOWER magnitude;
// rule 1 = OCP MX: e = floor(log2(amax)) - 2 (all-zero block: -127), round to nearest even
//          on the E2M1 grid, saturate at 6.
// ------------------------------------------------------------------------------------

// E2M1 magnitude index of |v| (v already divided by the block scale).
__device__ __forceinline__ uint32_t e2m1_index_ties_low(float m) {
  // number of midpoints strictly below m: midpoints 0.25 0.75 1.25 1.75 2.5 3.5 5
  return (m > 0.25f) + (m > 0.75f) + (m > 1.25f) + (m > 1.75f) + (m > 2.5f) + (m > 3.5f) + (m > 5.0f);
}
__device__ __forceinline__ uint32_t e2m1_index_rne(float m) {
  // a tie between codes c and c+1 goes to the even code
  uint32_t i = (m > 0.25f) + (m >= 0.75f) + (m > 1.25f) + (m >= 1.75f) + (m > 2.5f) + (m >= 3.5f) +
               (m > 5.0f);
  return i > 7 ? 7 : i;
}

// Exponent of the reference rule.  NumPy evaluates ceil(log2(y)) with a float32 log2; we
// round a double-precision log2 to float32 before the ceil, which agrees with a correctly
// rounded float32 log2 (the only place the two rules can differ is y one or two ulps above
// a power of two).
__device__ __forceinline__ int ref_rule_exponent(float amax) {
  const float y = fmaxf(amax, 1e-38f) / 6.0f;
  const float l = static_cast<float>(log2(static_cast<double>(y)));
  int e = static_cast<int>(ceilf(l));
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}

__device__ __forceinline__ int ocp_rule_exponent(float amax) {
  if (!(amax > 0.0f)) return -127;
  int E;
  frexpf(amax, &E);  // amax = m * 2**E, m in [0.5, 1)
  int e = (E - 1) - 2;
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}

// 2**(-e) for e in [-127, 127] as an exact fp32 (2**-127 is subnormal).
__device__ __forceinline__ float exp2_neg(int e) {
  const int b = 127 - e;  // biased exponent of 2**-e, in [0, 254]
  return b > 0 ? __uint_as_float(static_cast<uint32_t>(b) << 23) : __uint_as_float(0x00400000u);
}

template <int kRule>
__device__ __forceinline__ void quantize_group(const float (&v)[32], uint8_t (&packed)[16], uint8_t& scale) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int e = kRule == 0 ? ref_rule_exponent(amax) : ocp_rule_exponent(amax);
  scale = static_cast<uint8_t>(e + 127);
  const float inv = exp2_neg(e);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t nib[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float s = v[2 * i + h] * inv;
      const float m = fabsf(s);
      const uint32_t idx = kRule == 0 ? e2m1_index_ties_low(m) : e2m1_index_rne(m);
      nib[h] = idx | (s < 0.0f ? 8u : 0u);
    }
    packed[i] = static_cast<uint8_t>(nib[0] | (nib[1] << 4));
  }
}

// axis 0: one thread per (group g, column c); consecutive threads take consecutive columns.
template <int kRule>
__global__ void quantize_axis0_kernel(const float* __restrict__ x, int rows, int cols,
                                      uint8_t* __restrict__ packed, uint8_t* __restrict__ scales) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int groups = rows / kGroup;
  if (idx >= static_cast<long long>(groups) * cols) return;
  const int c = static_cast<int>(idx % cols);
  const int g = static_cast<int>(idx / cols);
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = x[static_cast<size_t>(g * kGroup + i) * cols + c];
  uint8_t p[16], s;
  quantize_group<kRule>(v, p, s);
#pragma unroll
  for (int i = 0; i < 16; ++i) packed[static_cast<size_t>(g * 16 + i) * cols + c] = p[i];
  scales[static_cast<size_t>(g) * cols + c] = s;
}

// axis 1: one thread per (row r, group g); the group's 32 floats are contiguous.
template <int kRule>
__global__ void quantize_axis1_kernel(const float* __restrict__ x, int rows, int cols,
                                      uint8_t* __restrict__ packed, uint8_t* __restrict__ scales) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int groups = cols / kGroup;
  if (idx >= static_cast<long long>(groups) * rows) return;
  const int g = static_cast<int>(idx % groups);
  const int r = static_cast<int>(idx / groups);
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * cols + g * kGroup);
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 q = src[i];
    v[4 * i] = q.x, v[4 * i + 1] = q.y, v[4 * i + 2] = q.z, v[4 * i + 3] = q.w;
  }
  uint8_t p[16], s;
  quantize_group<kRule>(v, p, s);
  uint4 out;
  out.x = p[0] | (p[1] << 8) | (p[2] << 16) | (static_cast<uint32_t>(p[3]) << 24);
  out.y = p[4] | (p[5] << 8) | (p[6] << 16) | (static_cast<uint32_t>(p[7]) << 24);
  out.z = p[8] | (p[9] << 8) | (p[10] << 16) | (static_cast<uint32_t>(p[11]) << 24);
  out.w = p[12] | (p[13] << 8) | (p[14] << 16) | (static_cast<uint32_t>(p[15]) << 24);
  *reinterpret_cast<uint4*>(packed + static_cast<size_t>(r) * (cols / 2) + g * 16) = out;
  scales[static_cast<size_t>(r) * groups + g] = s;
}

// ------------------------------------------------------------------------------------
// Plain dequantiser (the GPU counterpart of ref.py:50-72), written independently of the
// table-lookup dequant the GEMMs use so the two can be checked against each other.
//   layout 0 (reference): packed [K/2, N], scales [K/32, N] -> out [K, N]
//   layout 1 (row-major weights): packed [N, K/2], scales [N, K/32] -> out [N, K]
// out_dtype 0 = fp32, 1 = bf16.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ float e2m1_value(uint32_t nib) {
  // magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}: index >= 2 is (1 + m/2) * 2**(e-1) with e = idx>>1, m = idx&1
  const uint32_t em = nib & 7;
  const float m = em < 2 ? 0.5f * static_cast<float>(em)
                         : __uint_as_float(((126u + (em >> 1)) << 23) | ((em & 1u) << 22));
  return (nib & 8) ? -m : m;
}

template <typename OutT>
__device__ __forceinline__ OutT to_out(float v);
template <>
__device__ __forceinline__ float to_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename OutT>
__global__ void dequant_ref_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                                   int K, int N, OutT* __restrict__ out) {
  // one thread per byte: (k-pair kp, column n)
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(K / 2) * N) return;
  const int n = static_cast<int>(idx % N);
  const int kp = static_cast<int>(idx / N);
  const uint32_t b = packed[idx];
  const float sc = e8m0_to_f32(scales[static_cast<size_t>(kp / 16) * N + n]);
  out[static_cast<size_t>(2 * kp) * N + n] = to_out<OutT>(e2m1_value(b & 0xF) * sc);
  out[static_cast<size_t>(2 * kp + 1) * N + n] = to_out<OutT>(e2m1_value(b >> 4) * sc);
}

template <typename OutT>
__global__ void dequant_nk_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales,
                                  int K, int N, OutT* __restrict__ out) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(K / 2) * N) return;
  const int kp = static_cast<int>(idx % (K / 2));
  const int n = static_cast<int>(idx / (K / 2));
  const uint32_t b = packed[idx];
  const float sc = e8m0_to_f32(scales[static_cast<size_t>(n) * (K / 32) + kp / 16]);
  out[static_cast<size_t>(n) * K + 2 * kp] = to_out<OutT>(e2m1_value(b & 0xF) * sc);
  out[static_cast<size_t>(n) * K + 2 * kp + 1] = to_out<OutT>(e2m1_value(b >> 4) * sc);
}

// ------------------------------------------------------------------------------------
// Prepack into the B200 chunk layout (see the header for the byte-level description):
//   chunk (nb, kb) of 4352 bytes = data[g 0..1][r 0..127][16 B] + scales[g][r]
//   within a row-group, byte b of 4-byte word w is the k-pair w + 4*b.
// src_layout 0: reference [K/2, N] + [K/32, N]
// src_layout 1: row-major weights [N, K/2] + [N, K/32]
// src_layout 2: the reference's strategy-G prepack (ref.py:85-101; needs N % 128 == 0)
// Rows n >= N and k >= K are padded with zero nibbles and scale 127.
// One thread per (nb, kb, g, r) row-group.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t src_byte(const uint8_t* __restrict__ p, int layout, int kp, int n, int K,
                                             int N) {
  if (layout == 0) return p[static_cast<size_t>(kp) * N + n];
  if (layout == 1) return p[static_cast<size_t>(n) * (K / 2) + kp];
  // strategy G: [nb][K/8][128][4]; byte b of the word is K-byte 4*chunk + b
  const int nbg = n >> 7, ni = n & 127, chunk = kp >> 2, b = kp & 3;
  return p[((static_cast<size_t>(nbg) * (K / 8) + chunk) * 128 + ni) * 4 + b];
}
__device__ __forceinline__ uint32_t src_scale(const uint8_t* __restrict__ s, int layout, int kg, int n, int K,
                                              int N) {
  if (layout == 0) return s[static_cast<size_t>(kg) * N + n];
  if (layout == 1) return s[static_cast<size_t>(n) * (K / 32) + kg];
  const int nbg = n >> 7, ni = n & 127;
  return s[(static_cast<size_t>(nbg) * (K / 32) + kg) * 128 + ni];
}

__global__ void prepack_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales, int N,
                               int K, int layout, int k_blocks, int n_blocks, uint8_t* __restrict__ dst) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(n_blocks) * k_blocks * 2 * kChunkRows;
  if (idx >= total) return;
  const int r = static_cast<int>(idx % kChunkRows);
  const int g = static_cast<int>((idx / kChunkRows) % 2);
  const long long chunk = idx / (2 * kChunkRows);  // = nb * k_blocks + kb
  const int kb = static_cast<int>(chunk % k_blocks);
  const int nb = static_cast<int>(chunk / k_blocks);
  const int n = nb * kChunkRows + r;
  const int kg = kb * 2 + g;  // global 32-group index
  const bool live = (n < N) && (kg * kGroup < K);
  uint32_t w[4] = {0, 0, 0, 0};
  uint32_t sc = 127;
  if (live) {
#pragma unroll
    for (int wi = 0; wi < 4; ++wi)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int kp = kg * 16 + wi + 4 * b;
        w[wi] |= src_byte(packed, layout, kp, n, K, N) << (8 * b);
      }
    sc = src_scale(scales, layout, kg, n, K, N);
  }
  uint8_t* c = dst + chunk * kChunkBytes;
#pragma unroll
  for (int t = 0; t < 4; ++t) *reinterpret_cast<uint32_t*>(c + chunk_word_off(r, g, t)) = w[t];
  c[chunk_scale_off(r, g)] = static_cast<uint8_t>(sc);
}

// Dequantise prepacked chunks to bf16 [N, K] with the GEMM kernels' table-lookup routine
// (dequant_rowgroup), so that the exact bf16 tile the tensor cores consume can be compared
// bit for bit with the reference dequantiser.  One thread per row-group.
__global__ void dequant_prepacked_kernel(const uint8_t* __restrict__ wpack, int N, int K, int k_blocks,
                                         int n_blocks, uint16_t* __restrict__ out) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(n_blocks) * k_blocks * 2 * kChunkRows;
  if (idx >= total) return;
  const int r = static_cast<int>(idx % kChunkRows);
  const int g = static_cast<int>((idx / kChunkRows) % 2);
  const long long chunk = idx / (2 * kChunkRows);
  const int kb = static_cast<int>(chunk % k_blocks);
  const int nb = static_cast<int>(chunk / k_blocks);
  const int n = nb * kChunkRows + r;
  const int k0 = (kb * 2 + g) * kGroup;
  if (n >= N || k0 >= K) return;
  const uint8_t* c = wpack + chunk * kChunkBytes;
  const uint4 d = make_uint4(*reinterpret_cast<const uint32_t*>(c + chunk_word_off(r, g, 0)),
                             *reinterpret_cast<const uint32_t*>(c + chunk_word_off(r, g, 1)),
                             *reinterpret_cast<const uint32_t*>(c + chunk_word_off(r, g, 2)),
                             *reinterpret_cast<const uint32_t*>(c + chunk_word_off(r, g, 3)));
  uint32_t o[16];
  dequant_rowgroup(d, c[chunk_scale_off(r, g)], o);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(n) * K + k0);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
}

}  // namespace mxb
