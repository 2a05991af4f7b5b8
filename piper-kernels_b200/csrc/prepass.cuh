// Quantization prepass of Piper Attention (HBM-bound).
//
// Restates, for sm_100a, what the reference computes before its attention
// loop (Piper Kernels 0.2.1):
//   * K and V sequence means           attention/piper_attention/reference.py:46-52,
//                                      qk_quantization/int8/sage/reference.py:88-89
//                                      (Triton: _kv_mean_partial/_finalize, triton.py:68-173)
//   * Q codes, one scale per 32 rows   qk reference.py:61-77, 90-95 (quantize_per_group)
//   * centered K, one scale per 64 rows qk reference.py:96-100
//   * V per key row, centered when non-causal  reference.py:22-32, 59
// with the reference's fp32 semantics: scale = amax/127 + 1e-7 (IEEE divide
// then add), code = clamp(round_half_even(x/scale), -127, 127).
//
// Two launches:
//   kv_sum_kernel      grid (chunks, B*H, 2 or 1): one 512-row chunk of K
//                      (or of V, when non-causal) per CTA, 16-byte vector
//                      loads, exact fp64 column sums; the last of a (b,h)'s
//                      CTAs to finish turns the partial sums of both tensors
//                      into fp32 means (fixed order, so results are
//                      deterministic).  For a sequence shard it writes the
//                      shard's fp64 column totals instead; the caller sums
//                      them over the ranks and finalize_means_kernel divides
//                      by the total key count.
//   quantize_kernel    grid (ceil(max(Nq,Nk)/64), B*H, 3 at D = 128, 1 at
//                      D = 64): one 64-row tile of one tensor per CTA at
//                      D = 128, of all three at D = 64; group amax via warp
//                      shuffles + shared memory, scales computed once per
//                      group or row; V codes transposed to [D, keys] through
//                      shared memory so the attention kernel's PV operand is
//                      K-major.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "layout.h"
#include "sm100.cuh"

namespace piper {

constexpr int kPrepassThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// clamp(round_half_even(x / scale), -127, 127), bit-exact with the IEEE
// quotient, without a division or a float-to-int conversion per element.
// q = x * (1/scale) (reciprocal correctly rounded) is within
// |x/scale| * 2^-22 <= 127 * 2^-22 < 2^-14 of the true quotient
// (|x| <= amax < 127 * scale), so rounding q gives the same integer unless q
// lies within 2^-14 of a half-integer; only then is the exact quotient used.
// Rounding is the add of 1.5 * 2^23 (half-to-even in the FPU); the code is
// the low byte of the sum's bits.  The clamp never binds for the fast path:
// |x/scale| < 127 for finite inputs because scale = amax/127 + 1e-7 exceeds
// amax/127.
constexpr float kMagic = 12582912.0f;
constexpr float kNearTie = 0.5f - 1.0f / 16384.0f;

__device__ __forceinline__ uint32_t exact_code_bits(float x, float scale) {
  return __float_as_uint(__fadd_rn(fminf(fmaxf(__fdiv_rn(x, scale), -127.0f), 127.0f), kMagic));
}

__device__ __forceinline__ float group_scale(float amax) {
  return __fadd_rn(__fdiv_rn(amax, 127.0f), 1e-7f);
}

struct PrepassArgs {
  const void* q;
  const void* k;
  const void* v;
  int64_t qs[3], ks[3], vs[3];  // B, H, N strides in elements
  int64_t heads, nq, nk;
  int causal;
  int sums_only;       // kv_sum_kernel: write the shard's fp64 totals, not means
  int64_t total_keys;  // finalize_means_kernel: keys over all shards
  uint8_t* ws;         // workspace base
  piper_b200_workspace_layout_t L;
};

// ---------------------------------------------------------------------------
// Raw 16-byte load of 8 consecutive fp16/bf16 elements (element-wise when the
// address or strides are not 16-byte aligned) and its exact widening.
template <typename T, bool kVec16>
__device__ __forceinline__ uint4 load_raw8(const T* p) {
  if constexpr (kVec16) {
    return __ldg(reinterpret_cast<const uint4*>(p));
  } else {
    const uint16_t* e = reinterpret_cast<const uint16_t*>(p);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = static_cast<uint32_t>(e[2 * i]) | (static_cast<uint32_t>(e[2 * i + 1]) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& r, float (&out)[8]) {
  const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = to_f32<T>(e[i]);
}

// ---------------------------------------------------------------------------
// Column sums of K (and V when non-causal) over one chunk of rows, in fp64.
template <typename T, int D, bool kVec16>
// One tensor per CTA (K when blockIdx.z == 0, V when 1): eight rows per step,
// all eight 16-byte loads issued first, at four CTAs per SM (64 registers).
// Measured against one CTA summing both K and V (sixteen loads in flight per
// thread, two CTAs per SM): 10% faster on c4, 15% on c2, 25% on causal c3 (K
// only): twice the warps per SM to hide the loads and conversions.
__global__ void __launch_bounds__(kPrepassThreads, 4) kv_sum_kernel(PrepassArgs a) {
  constexpr int kVpr = D / 8;                      // 16-byte vectors per row
  constexpr int kRpp = kPrepassThreads / kVpr;     // rows per pass
  __shared__ double red[kRpp][D];
  __shared__ int is_last;

  const int chunk = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const bool is_v = blockIdx.z == 1;
  const int64_t b = bh / a.heads, h = bh % a.heads;
  const int tid = threadIdx.x;
  const int vec = tid % kVpr;
  const int ro = tid / kVpr;
  const bool with_v = !a.causal;

  const int64_t s0 = is_v ? a.vs[0] : a.ks[0], s1 = is_v ? a.vs[1] : a.ks[1], s2 = is_v ? a.vs[2] : a.ks[2];
  const T* base = static_cast<const T*>(is_v ? a.v : a.k) + b * s0 + h * s1 + vec * 8;
  double sum[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sum[i] = 0.0;

  const int64_t r0 = static_cast<int64_t>(chunk) * kSumChunkRows;
  const int64_t r1 = min(r0 + kSumChunkRows, a.nk);
  constexpr int kUnroll = 8;
  int64_t r = r0 + ro;
  // A row pointer advanced by a precomputed step (no 64-bit multiply per load).
  const int64_t step = kRpp * s2;
  const T* ptr = base + r * s2;
  for (; r + (kUnroll - 1) * kRpp < r1; r += kUnroll * kRpp) {
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) raw[u] = load_raw8<T, kVec16>(ptr + u * step);
    ptr += kUnroll * step;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float x[8];
      unpack8<T>(raw[u], x);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum[i] += static_cast<double>(x[i]);
    }
  }
  for (; r < r1; r += kRpp) {
    float x[8];
    unpack8<T>(load_raw8<T, kVec16>(base + r * s2), x);
#pragma unroll
    for (int i = 0; i < 8; ++i) sum[i] += static_cast<double>(x[i]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[ro][vec * 8 + i] = sum[i];
  __syncthreads();

  double* kpart = reinterpret_cast<double*>(a.ws + a.L.ksum);
  double* vpart = reinterpret_cast<double*>(a.ws + a.L.vsum);
  const int64_t chunks = a.L.chunks;
  if (tid < D) {
    double t = 0.0;
    for (int rr = 0; rr < kRpp; ++rr) t += red[rr][tid];
    (is_v ? vpart : kpart)[(bh * chunks + chunk) * D + tid] = t;
  }
  __threadfence();
  __syncthreads();
  // The last of the head's chunks x tensors CTAs to finish turns the partial
  // sums of both tensors into the means.
  if (tid == 0) {
    unsigned int* counter = reinterpret_cast<unsigned int*>(a.ws + a.L.counter) + bh;
    const unsigned int done = atomicAdd(counter, 1u);
    is_last = (done == static_cast<unsigned int>(chunks * gridDim.z - 1));
    if (is_last) *counter = 0u;  // leave the counter ready for the next call
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (tid < D) {
    double s = 0.0, t = 0.0;
    for (int64_t c = 0; c < chunks; ++c) {
      s += __ldcg(&kpart[(bh * chunks + c) * D + tid]);
      if (with_v) t += __ldcg(&vpart[(bh * chunks + c) * D + tid]);
    }
    if (a.sums_only) {
      // A sequence shard: its totals are summed over the ranks by the caller
      // and turned into means by finalize_means_kernel.
      double* totals = reinterpret_cast<double*>(a.ws + a.L.totals);
      const int64_t bh_all = static_cast<int64_t>(gridDim.y);
      totals[bh * D + tid] = s;
      totals[(bh_all + bh) * D + tid] = with_v ? t : 0.0;
    } else {
      float* kmean = reinterpret_cast<float*>(a.ws + a.L.kmean);
      float* vmean = reinterpret_cast<float*>(a.ws + a.L.vmean);
      kmean[bh * D + tid] = static_cast<float>(s / static_cast<double>(a.nk));
      vmean[bh * D + tid] = with_v ? static_cast<float>(t / static_cast<double>(a.nk)) : 0.0f;
    }
  }
}

// Means of a sequence-sharded problem from the K and V column totals summed
// over every shard: the same fp64 division and single rounding to fp32 as the
// one-GPU finalize above.  grid (B*H), D threads.
template <int D>
__global__ void __launch_bounds__(D) finalize_means_kernel(PrepassArgs a) {
  const int64_t bh = blockIdx.x;
  const int64_t bh_all = static_cast<int64_t>(gridDim.x);
  const int tid = threadIdx.x;
  const double* totals = reinterpret_cast<const double*>(a.ws + a.L.totals);
  float* kmean = reinterpret_cast<float*>(a.ws + a.L.kmean);
  float* vmean = reinterpret_cast<float*>(a.ws + a.L.vmean);
  const double n = static_cast<double>(a.total_keys);
  kmean[bh * D + tid] = static_cast<float>(totals[bh * D + tid] / n);
  vmean[bh * D + tid] = a.causal ? 0.0f : static_cast<float>(totals[(bh_all + bh) * D + tid] / n);
}

// Eight INT8 codes as the bits of q + 1.5*2^23 (the code is the low byte),
// computed in packed f32x2 arithmetic.  One near-tie test covers all eight,
// through their largest distance from the rounded value, and feeds one vote
// over the active lanes, so the exact-division fallback is a real branch
// that warps skip unless one of their lanes has a near-tie (it is never
// issued predicated off for every element).
__device__ __forceinline__ void round_codes(const float (&x)[8], float s, float rs, uint32_t (&y)[8]) {
  float dm = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const float2 q = __fmul2_rn(make_float2(x[i], x[i + 1]), make_float2(rs, rs));
    const float2 t = __fadd2_rn(q, make_float2(kMagic, kMagic));
    const float2 r = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
    const float2 d = __ffma2_rn(r, make_float2(-1.0f, -1.0f), q);
    dm = fmax3(dm, fabsf(d.x), fabsf(d.y));
    y[i] = __float_as_uint(t.x);
    y[i + 1] = __float_as_uint(t.y);
  }
  if (__any_sync(__activemask(), dm > kNearTie)) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float q = __fmul_rn(x[i], rs);
      if (fabsf(__fsub_rn(q, __fsub_rn(__fadd_rn(q, kMagic), kMagic))) > kNearTie) y[i] = exact_code_bits(x[i], s);
    }
  }
}

// Eight INT8 codes packed into two words.
__device__ __forceinline__ uint2 pack_codes(const float (&x)[8], float s, float rs) {
  uint32_t y[8];
  round_codes(x, s, rs, y);
  const uint32_t w0 = __byte_perm(__byte_perm(y[0], y[1], 0x0040), __byte_perm(y[2], y[3], 0x0040), 0x5410);
  const uint32_t w1 = __byte_perm(__byte_perm(y[4], y[5], 0x0040), __byte_perm(y[6], y[7], 0x0040), 0x5410);
  return make_uint2(w0, w1);
}

// Eight INT8 codes as fp16 values (exact: integers in [-127, 127]), packed
// in pairs: the V operand of the attention kernel's fp16 PV product.
__device__ __forceinline__ uint4 pack_codes_f16(const float (&x)[8], float s, float rs) {
  uint32_t y[8];
  round_codes(x, s, rs, y);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 c = __fadd2_rn(make_float2(__uint_as_float(y[2 * i]), __uint_as_float(y[2 * i + 1])),
                                make_float2(-kMagic, -kMagic));
    const __half2 h = __floats2half2_rn(c.x, c.y);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Largest |x| of eight raw fp16/bf16 values (one 16-byte vector) and `acc`,
// in packed 16-bit arithmetic: the maximum is exact in the input type, so it
// converts to the same float as the fp32 maximum of the widened values.
template <typename T>
struct PairOf;
template <>
struct PairOf<__half> {
  using type = __half2;
};
template <>
struct PairOf<__nv_bfloat16> {
  using type = __nv_bfloat162;
};

template <typename T>
__device__ __forceinline__ uint32_t absmax8(const uint4& r, uint32_t acc) {
  using P = typename PairOf<T>::type;
  P m = *reinterpret_cast<const P*>(&acc);
  const P* e = reinterpret_cast<const P*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) m = __hmax2(m, __habs2(e[i]));
  return *reinterpret_cast<const uint32_t*>(&m);
}

template <typename T>
__device__ __forceinline__ float absmax_pair_to_f32(uint32_t m) {
  const T* e = reinterpret_cast<const T*>(&m);
  return fmaxf(to_f32<T>(e[0]), to_f32<T>(e[1]));
}

// One 64-row tile of one tensor per CTA.  Each thread holds its raw 16-byte
// vectors of that tensor (rows past the sequence end hold zeros).  The
// functions below contain CTA-wide barriers, and every thread of the CTA calls
// one of them for the same tile.
template <int D>
struct QuantTile {
  static constexpr int kVpr = D / 8;                   // 16-byte vectors per row
  static constexpr int kRpp = kPrepassThreads / kVpr;  // rows per pass
  static constexpr int kPasses = kKeyBlock / kRpp;     // passes over the 64-row tile
  static constexpr int kRowWords = D / 2 + 1;          // padded fp16 V code row, in words
  static constexpr int kWarps = kPrepassThreads / 32;
};

// Largest value of `v` over the CTA, through the per-warp slots red[][c]
// (two barriers; the result is the same in every thread).
template <int D>
__device__ __forceinline__ float cta_max(float v, float (*red)[2], int c) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp][c] = v;
  __syncthreads();
  float m = 0.0f;
#pragma unroll
  for (int w = 0; w < QuantTile<D>::kWarps; ++w) m = fmaxf(m, red[w][c]);
  return m;
}

// Q codes of one tile: two 32-row groups, each scale from the packed 16-bit
// maxima of the raw values (exact in the input type, so equal to the fp32
// maximum; rows past the sequence end count as zero, as the reference's zero
// padding).
template <typename T, int D>
__device__ __forceinline__ void quantize_q_tile(const PrepassArgs& a, int64_t bh, int tile,
                                                const uint4 (&rq)[QuantTile<D>::kPasses], float (*red)[2],
                                                float* gsc) {
  using Q = QuantTile<D>;
  const int tid = threadIdx.x;
  const int vec = tid % Q::kVpr, ro = tid / Q::kVpr;
  const int64_t row0 = static_cast<int64_t>(tile) * kKeyBlock;
  const int nvq = static_cast<int>(min(int64_t(kKeyBlock), max(int64_t(0), a.nq - row0)));
  uint32_t qm[2] = {0u, 0u};
#pragma unroll
  for (int p = 0; p < Q::kPasses; ++p) {
    const int g = (p * Q::kRpp) / kQueryGroup;  // compile-time: kRpp divides or is divided by 32
    qm[g] = absmax8<T>(rq[p], qm[g]);
  }
  float m0 = absmax_pair_to_f32<T>(qm[0]), m1 = absmax_pair_to_f32<T>(qm[1]);
  const int lane = tid % 32, warp = tid / 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
  }
  if (lane == 0) {
    red[warp][0] = m0;
    red[warp][1] = m1;
  }
  __syncthreads();
  // The group scales, computed once (threads 0 and 1).
  if (tid < 2) {
    float m = 0.0f;
#pragma unroll
    for (int w = 0; w < Q::kWarps; ++w) m = fmaxf(m, red[w][tid]);
    const float sc = group_scale(m);
    gsc[tid] = sc;
    gsc[2 + tid] = __frcp_rn(sc);
    const int64_t g = row0 / kQueryGroup + tid;
    if (g < a.L.q_groups) reinterpret_cast<float*>(a.ws + a.L.qscale)[bh * a.L.q_groups + g] = sc;
  }
  __syncthreads();
  // This thread's first code row; later passes are kRpp rows further on.
  int8_t* q8 = reinterpret_cast<int8_t*>(a.ws + a.L.q8) + ((bh * a.nq + row0 + ro) * D + vec * 8);
#pragma unroll
  for (int p = 0; p < Q::kPasses; ++p) {
    if (ro + p * Q::kRpp < nvq) {
      const int g = (p * Q::kRpp) / kQueryGroup;
      float x[8];
      unpack8<T>(rq[p], x);
      *reinterpret_cast<uint2*>(q8 + p * Q::kRpp * D) = pack_codes(x, gsc[g], gsc[2 + g]);
    }
  }
}

// K codes of one tile, centered by the sequence mean: one 64-row group.
template <typename T, int D>
__device__ __forceinline__ void quantize_k_tile(const PrepassArgs& a, int64_t bh, int tile,
                                                const uint4 (&rk)[QuantTile<D>::kPasses], float (*red)[2],
                                                float* gsc) {
  using Q = QuantTile<D>;
  const int tid = threadIdx.x;
  const int vec = tid % Q::kVpr, ro = tid / Q::kVpr;
  const int64_t row0 = static_cast<int64_t>(tile) * kKeyBlock;
  const int nvk = static_cast<int>(min(int64_t(kKeyBlock), max(int64_t(0), a.nk - row0)));
  // Negated means in pairs: x - m is computed as x + (-m), the same IEEE result.
  float2 nkm[4];
  {
    const float* kmean = reinterpret_cast<const float*>(a.ws + a.L.kmean) + bh * D + vec * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) nkm[i] = make_float2(-kmean[2 * i], -kmean[2 * i + 1]);
  }
  float kmx = 0.0f;
#pragma unroll
  for (int p = 0; p < Q::kPasses; ++p) {
    if (ro + p * Q::kRpp < nvk) {
      float x[8];
      unpack8<T>(rk[p], x);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 c = __fadd2_rn(make_float2(x[2 * i], x[2 * i + 1]), nkm[i]);
        kmx = fmax3(kmx, fabsf(c.x), fabsf(c.y));
      }
    }
  }
  const float m = cta_max<D>(kmx, red, 0);
  if (tid == 0) {
    const float sc = group_scale(m);
    gsc[0] = sc;
    gsc[1] = __frcp_rn(sc);
    reinterpret_cast<float*>(a.ws + a.L.kscale)[bh * a.L.k_groups + tile] = sc;
  }
  __syncthreads();
  const float sk = gsc[0], rsk = gsc[1];
  int8_t* k8 = reinterpret_cast<int8_t*>(a.ws + a.L.k8) + ((bh * a.nk + row0 + ro) * D + vec * 8);
#pragma unroll
  for (int p = 0; p < Q::kPasses; ++p) {
    if (ro + p * Q::kRpp < nvk) {
      float x[8];
      unpack8<T>(rk[p], x);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 c = __fadd2_rn(make_float2(x[2 * i], x[2 * i + 1]), nkm[i]);
        x[2 * i] = c.x;
        x[2 * i + 1] = c.y;
      }
      *reinterpret_cast<uint2*>(k8 + p * Q::kRpp * D) = pack_codes(x, sk, rsk);
    }
  }
}

// V codes of one tile: one scale per key row (centered by the sequence mean
// when non-causal).  Each row's max is a shuffle among the threads of that
// row; its scale, reciprocal and log2 are computed once, by thread `row`.  V
// codes go row-major as fp16 into a padded shared tile (row stride D/2 + 1
// words, so rows fall on distinct banks), then are transposed 4 keys x 2
// features at a time with two permutes and written as [D, keys] with 8-byte
// stores.
template <typename T, int D>
__device__ __forceinline__ void quantize_v_tile(const PrepassArgs& a, int64_t bh, int tile,
                                                const uint4 (&rv)[QuantTile<D>::kPasses], uint32_t* vrow,
                                                float* vstat) {
  using Q = QuantTile<D>;
  const int tid = threadIdx.x;
  const int vec = tid % Q::kVpr, ro = tid / Q::kVpr;
  const int64_t row0 = static_cast<int64_t>(tile) * kKeyBlock;
  const auto& L = a.L;
  const int nvk = static_cast<int>(min(int64_t(kKeyBlock), max(int64_t(0), a.nk - row0)));
  float2 nvm[4];
  {
    const float* vmean = reinterpret_cast<const float*>(a.ws + L.vmean) + bh * D + vec * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      nvm[i] = a.causal ? make_float2(-0.0f, -0.0f) : make_float2(-vmean[2 * i], -vmean[2 * i + 1]);
  }
#pragma unroll
  for (int p = 0; p < Q::kPasses; ++p) {
    const int lr = ro + p * Q::kRpp;
    float x[8];
    unpack8<T>(rv[p], x);
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 c = __fadd2_rn(make_float2(x[2 * i], x[2 * i + 1]), nvm[i]);
      amax = fmax3(amax, fabsf(c.x), fabsf(c.y));
    }
    if (lr >= nvk) amax = 0.0f;
#pragma unroll
    for (int o = Q::kVpr / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (vec == 0) vstat[lr] = amax;
  }
  __syncthreads();
  if (tid < kKeyBlock) {
    const int64_t r = row0 + tid;
    const bool valid = tid < nvk;
    const float sv = group_scale(vstat[tid]);
    const float rsv = __frcp_rn(sv);
    vstat[tid] = sv;
    vstat[kKeyBlock + tid] = rsv;
    reinterpret_cast<float*>(a.ws + L.vscale)[bh * L.nk_pad + r] = valid ? sv : 0.0f;
    reinterpret_cast<float*>(a.ws + L.vlog2)[bh * L.nk_pad + r] = valid ? log2f(sv) : -INFINITY;
    reinterpret_cast<float*>(a.ws + L.vrcp)[bh * L.nk_pad + r] = valid ? rsv : 0.0f;
  }
  __syncthreads();
#pragma unroll
  for (int p = 0; p < Q::kPasses; ++p) {
    const int lr = ro + p * Q::kRpp;
    float x[8];
    unpack8<T>(rv[p], x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 c = __fadd2_rn(make_float2(x[2 * i], x[2 * i + 1]), nvm[i]);
      x[2 * i] = c.x;
      x[2 * i + 1] = c.y;
    }
    const uint4 codes = lr < nvk ? pack_codes_f16(x, vstat[lr], vstat[kKeyBlock + lr]) : make_uint4(0u, 0u, 0u, 0u);
    uint32_t* dst = vrow + lr * Q::kRowWords + 4 * vec;
    dst[0] = codes.x;
    dst[1] = codes.y;
    dst[2] = codes.z;
    dst[3] = codes.w;
  }
  __syncthreads();
  // Transpose to [D, keys]: each step moves 4 keys x 2 features (one word of
  // each of 4 rows); a warp covers 8 key quads x 4 feature pairs, so its
  // shared loads fall on 32 distinct banks.  8-byte index of (d, key) =
  // ((bh*D + d) * nk_pad + key) / 4; nk_pad and row0 are multiples of 64.
  uint2* v16t = reinterpret_cast<uint2*>(a.ws + L.v8t) + (bh * D * L.nk_pad + row0) / 4;
  const int64_t row_words = L.nk_pad / 4;  // one feature row, in 8-byte units
  constexpr int kPairs = D / 2;
  constexpr int kBlocks = kPairs * (kKeyBlock / 4);
#pragma unroll
  for (int blk = tid; blk < kBlocks; blk += kPrepassThreads) {
    const int kq = (blk % 8) + 8 * (blk / (8 * kPairs));
    const int dp = (blk / 8) % kPairs;
    const uint32_t w0 = vrow[(4 * kq + 0) * Q::kRowWords + dp];
    const uint32_t w1 = vrow[(4 * kq + 1) * Q::kRowWords + dp];
    const uint32_t w2 = vrow[(4 * kq + 2) * Q::kRowWords + dp];
    const uint32_t w3 = vrow[(4 * kq + 3) * Q::kRowWords + dp];
    uint2* out = v16t + (2 * dp) * row_words + kq;
    out[0] = make_uint2(__byte_perm(w0, w1, 0x5410), __byte_perm(w2, w3, 0x5410));
    out[row_words] = make_uint2(__byte_perm(w0, w1, 0x7632), __byte_perm(w2, w3, 0x7632));
  }
}

// This thread's raw 16-byte vectors of one tensor's 64-row tile (zeros past
// the sequence end): all loads issued up front.
template <typename T, int D, bool kVec16>
__device__ __forceinline__ void load_tile(const void* src, const int64_t (&st)[3], int64_t b, int64_t h, int64_t row0,
                                          int64_t rows, uint4 (&raw)[QuantTile<D>::kPasses]) {
  using Q = QuantTile<D>;
  const int vec = threadIdx.x % Q::kVpr, ro = threadIdx.x / Q::kVpr;
  // This thread's first row; pass p is p * kRpp rows further.
  const T* base = static_cast<const T*>(src) + b * st[0] + h * st[1] + (row0 + ro) * st[2] + vec * 8;
  const int64_t step = Q::kRpp * st[2];
  const int nv = static_cast<int>(min(int64_t(kKeyBlock), max(int64_t(0), rows - row0)));
#pragma unroll
  for (int p = 0; p < Q::kPasses; ++p)
    raw[p] = (ro + p * Q::kRpp < nv) ? load_raw8<T, kVec16>(base + p * step) : make_uint4(0u, 0u, 0u, 0u);
}

// At D = 128, grid (ceil(max(Nq,Nk)/64), B*H, 3): one 64-row tile of one
// tensor per CTA (blockIdx.z: 0 = Q, 1 = K, 2 = V), four CTAs per SM (62
// registers).  Measured against one CTA quantizing all three tensors of a tile
// (three CTAs per SM, 80 registers), over two runs: 3-6% faster on c4, 4-6% on
// c2, 6-9% on causal c3.  At D = 64, grid (..., B*H, 1): one CTA loads all
// three tensors' tile and quantizes Q, K, V in turn, four CTAs per SM; the
// split form is 9-15% slower there (half-size tiles: the per-CTA barriers and
// scale work weigh more), and this form is 3% slower than the former
// single-function kernel (more barriers).  A persistent form with the next tiles staged in shared memory by
// bulk copies, two CTAs per SM, was measured 36% slower on c4: the kernel is
// held by the latency of its arithmetic, which more resident warps hide.
template <typename T, int D, bool kVec16>
__global__ void __launch_bounds__(kPrepassThreads, 4) quantize_kernel(PrepassArgs a) {
  using Q = QuantTile<D>;
  __shared__ float red[Q::kWarps][2];
  __shared__ uint32_t vrow[kKeyBlock * Q::kRowWords];
  __shared__ float vstat[2 * kKeyBlock];  // V row maxima, then scales and reciprocals
  __shared__ float gsc[4];                // group scales and their reciprocals

  const int tile = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / a.heads, h = bh % a.heads;
  const int64_t row0 = static_cast<int64_t>(tile) * kKeyBlock;
  if constexpr (D == 128) {
    const int part = blockIdx.z;
    const int64_t rows = part == 0 ? a.nq : a.nk;
    if (row0 >= rows) return;  // the whole CTA: this tensor has no rows here
    uint4 raw[Q::kPasses];
    if (part == 0) {
      load_tile<T, D, kVec16>(a.q, a.qs, b, h, row0, a.nq, raw);
      quantize_q_tile<T, D>(a, bh, tile, raw, red, gsc);
    } else if (part == 1) {
      load_tile<T, D, kVec16>(a.k, a.ks, b, h, row0, a.nk, raw);
      quantize_k_tile<T, D>(a, bh, tile, raw, red, gsc);
    } else {
      load_tile<T, D, kVec16>(a.v, a.vs, b, h, row0, a.nk, raw);
      quantize_v_tile<T, D>(a, bh, tile, raw, vrow, vstat);
    }
  } else {
    // Q, K and V in turn.  Between the calls, every thread passes a barrier
    // of the next call before any thread writes `red` or `gsc` again.
    uint4 rq[Q::kPasses], rk[Q::kPasses], rv[Q::kPasses];
    load_tile<T, D, kVec16>(a.q, a.qs, b, h, row0, a.nq, rq);
    load_tile<T, D, kVec16>(a.k, a.ks, b, h, row0, a.nk, rk);
    load_tile<T, D, kVec16>(a.v, a.vs, b, h, row0, a.nk, rv);
    if (row0 < a.nq) quantize_q_tile<T, D>(a, bh, tile, rq, red, gsc);
    if (row0 < a.nk) {
      quantize_k_tile<T, D>(a, bh, tile, rk, red, gsc);
      quantize_v_tile<T, D>(a, bh, tile, rv, vrow, vstat);
    }
  }
}

}  // namespace piper
