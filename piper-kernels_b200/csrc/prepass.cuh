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
//   kv_sum_kernel      grid (chunks, B*H): 16-byte vector loads of K (and V),
//                      exact fp64 column sums per 512-row chunk; the last
//                      chunk of each (b,h) to finish turns the partial sums
//                      into fp32 means (fixed order, so results are
//                      deterministic).  For a sequence shard it writes
//                      the shard's fp64 column totals instead; the caller
//                      sums them over the ranks and finalize_means_kernel
//                      divides by the total key count.
//   quantize_kernel    grid (ceil(max(Nq,Nk)/64), B*H): one 64-row tile of Q,
//                      K and V per CTA; group amax via warp shuffles + shared
//                      memory; V codes transposed to [D, keys] through shared
//                      memory so the attention kernel's PV operand is K-major.
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

// The arithmetic of one 64-row tile of Q, K and V, given each thread's raw
// 16-byte vectors (rows past a sequence end hold zeros).  The two 32-row Q
// group maxima (packed 16-bit maxima of the raw values) and the 64-row K
// group max share one block-wide reduction; each V row's max is a shuffle
// among the threads of that row.  V codes go row-major as fp16 into a padded
// shared tile (row stride D/2 + 1 words, so rows fall on distinct banks), then
// are transposed 4 keys x 2 features at a time with two permutes and written
// as [D, keys] with 8-byte stores.  Contains CTA-wide barriers: every thread
// of the CTA calls it for the same tile.  `vrow` is the padded V code tile,
// `red` the per-warp maxima, `vstat` (2 x 64 floats) and `gsc` (6 floats) the
// V row and Q/K group scales with their reciprocals.
template <typename T, int D>
__device__ __forceinline__ void quantize_tile(const PrepassArgs& a, int64_t bh, int tile,
                                              const uint4 (&rq)[kKeyBlock / (kPrepassThreads / (D / 8))],
                                              const uint4 (&rk)[kKeyBlock / (kPrepassThreads / (D / 8))],
                                              const uint4 (&rv)[kKeyBlock / (kPrepassThreads / (D / 8))],
                                              uint32_t* vrow, float (*red)[3], float* vstat, float* gsc) {
  constexpr int kVpr = D / 8;                   // 16-byte vectors per row
  constexpr int kRpp = kPrepassThreads / kVpr;  // rows per pass
  constexpr int kPasses = kKeyBlock / kRpp;     // passes over the 64-row tile
  constexpr int kRowWords = D / 2 + 1;          // padded fp16 V code row, in words
  constexpr int kWarps = kPrepassThreads / 32;
  const int tid = threadIdx.x;
  const int lane = tid % 32, warp = tid / 32;
  const int vec = tid % kVpr;
  const int ro = tid / kVpr;
  const int64_t row0 = static_cast<int64_t>(tile) * kKeyBlock;
  const auto& L = a.L;
  const bool has_q = row0 < a.nq;
  const bool has_kv = row0 < a.nk;
  // Rows of this tile inside each sequence (0..64), for 32-bit row tests.
  const int nvq = static_cast<int>(min(int64_t(kKeyBlock), max(int64_t(0), a.nq - row0)));
  const int nvk = static_cast<int>(min(int64_t(kKeyBlock), max(int64_t(0), a.nk - row0)));
  float km[8], vm[8];
  {
    const float* kmean = reinterpret_cast<const float*>(a.ws + L.kmean) + bh * D + vec * 8;
    const float* vmean = reinterpret_cast<const float*>(a.ws + L.vmean) + bh * D + vec * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      km[i] = has_kv ? kmean[i] : 0.0f;
      vm[i] = (has_kv && !a.causal) ? vmean[i] : 0.0f;
    }
  }
  // Negated means in pairs: x - m is computed as x + (-m), the same IEEE result.
  float2 nkm[4], nvm[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    nkm[i] = make_float2(-km[2 * i], -km[2 * i + 1]);
    nvm[i] = make_float2(-vm[2 * i], -vm[2 * i + 1]);
  }

  // ---- group maxima: Q (two 32-row groups) and centered K (one 64-row group);
  // rows past the sequence end count as zero, as the reference's zero padding.
  float am[3];
  {
    uint32_t qm[2] = {0u, 0u};  // packed |q| maxima of the two Q groups
    float kmx = 0.0f;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int g = (p * kRpp) / kQueryGroup;  // compile-time: kRpp divides or is divided by 32
      qm[g] = absmax8<T>(rq[p], qm[g]);
      if (ro + p * kRpp < nvk) {
        float x[8];
        unpack8<T>(rk[p], x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 c = __fadd2_rn(make_float2(x[2 * i], x[2 * i + 1]), nkm[i]);
          kmx = fmax3(kmx, fabsf(c.x), fabsf(c.y));
        }
      }
    }
    am[0] = absmax_pair_to_f32<T>(qm[0]);
    am[1] = absmax_pair_to_f32<T>(qm[1]);
    am[2] = kmx;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int c = 0; c < 3; ++c) am[c] = fmaxf(am[c], __shfl_xor_sync(0xffffffffu, am[c], o));
  }
  if (lane == 0) {
#pragma unroll
    for (int c = 0; c < 3; ++c) red[warp][c] = am[c];
  }
  // Each V row's max (centered when non-causal; zero past the sequence end):
  // a shuffle among the kVpr consecutive lanes of that row.
  if (has_kv) {
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int lr = ro + p * kRpp;
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
      for (int o = kVpr / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (vec == 0) vstat[lr] = amax;
    }
  }
  __syncthreads();
  // Scales, computed once: the Q and K group scales and reciprocals by
  // threads 0-2, each V row's scale, reciprocal and log2 by thread `row`
  // (the same IEEE operations on the same maxima as every thread did before).
  if (tid < 3) {
    float m = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, red[w][tid]);
    const float sc = group_scale(m);
    gsc[tid] = sc;
    gsc[3 + tid] = __frcp_rn(sc);
  }
  if (has_kv && tid < kKeyBlock) {
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

  // ---- Q codes.
  if (has_q) {
    const float sq[2] = {gsc[0], gsc[1]};
    const float rq2[2] = {gsc[3], gsc[4]};
    // This thread's first code row; later passes are kRpp rows further on.
    int8_t* q8 = reinterpret_cast<int8_t*>(a.ws + L.q8) + ((bh * a.nq + row0 + ro) * D + vec * 8);
    if (tid < 2) {
      const int64_t g = row0 / kQueryGroup + tid;
      if (g < L.q_groups) reinterpret_cast<float*>(a.ws + L.qscale)[bh * L.q_groups + g] = sq[tid];
    }
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      if (ro + p * kRpp < nvq) {
        const int g = (p * kRpp) / kQueryGroup;
        float x[8];
        unpack8<T>(rq[p], x);
        *reinterpret_cast<uint2*>(q8 + p * kRpp * D) = pack_codes(x, sq[g], rq2[g]);
      }
    }
  }
  if (!has_kv) return;

  // ---- K codes (centered by the sequence mean).
  {
    const float sk = gsc[2];
    const float rsk = gsc[5];
    int8_t* k8 = reinterpret_cast<int8_t*>(a.ws + L.k8) + ((bh * a.nk + row0 + ro) * D + vec * 8);
    if (tid == 0) reinterpret_cast<float*>(a.ws + L.kscale)[bh * L.k_groups + tile] = sk;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      if (ro + p * kRpp < nvk) {
        float x[8];
        unpack8<T>(rk[p], x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 c = __fadd2_rn(make_float2(x[2 * i], x[2 * i + 1]), nkm[i]);
          x[2 * i] = c.x;
          x[2 * i + 1] = c.y;
        }
        *reinterpret_cast<uint2*>(k8 + p * kRpp * D) = pack_codes(x, sk, rsk);
      }
    }
  }

  // ---- V: per key row (centered when non-causal), fp16 codes into the
  // shared tile (row-major, rows of kRowWords words).
  {
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int lr = ro + p * kRpp;
      const bool valid = lr < nvk;
      float x[8];
      unpack8<T>(rv[p], x);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 c = __fadd2_rn(make_float2(x[2 * i], x[2 * i + 1]), nvm[i]);
        x[2 * i] = c.x;
        x[2 * i + 1] = c.y;
      }
      const uint4 codes = valid ? pack_codes_f16(x, vstat[lr], vstat[kKeyBlock + lr]) : make_uint4(0u, 0u, 0u, 0u);
      uint32_t* dst = vrow + lr * kRowWords + 4 * vec;
      dst[0] = codes.x;
      dst[1] = codes.y;
      dst[2] = codes.z;
      dst[3] = codes.w;
    }
  }
  __syncthreads();
  // ---- transpose to [D, keys]: each step moves 4 keys x 2 features (one
  // word of each of 4 rows); a warp covers 8 key quads x 4 feature pairs, so
  // its shared loads fall on 32 distinct banks (row stride D/2 + 1 words).
  {
    // 8-byte index of (d, key) = ((bh*D + d) * nk_pad + key) / 4; nk_pad and
    // row0 are multiples of 64.
    uint2* v16t = reinterpret_cast<uint2*>(a.ws + L.v8t) + (bh * D * L.nk_pad + row0) / 4;
    const int64_t row_words = L.nk_pad / 4;  // one feature row, in 8-byte units
    constexpr int kPairs = D / 2;
    constexpr int kBlocks = kPairs * (kKeyBlock / 4);
#pragma unroll
    for (int blk = tid; blk < kBlocks; blk += kPrepassThreads) {
      const int kq = (blk % 8) + 8 * (blk / (8 * kPairs));
      const int dp = (blk / 8) % kPairs;
      const uint32_t w0 = vrow[(4 * kq + 0) * kRowWords + dp];
      const uint32_t w1 = vrow[(4 * kq + 1) * kRowWords + dp];
      const uint32_t w2 = vrow[(4 * kq + 2) * kRowWords + dp];
      const uint32_t w3 = vrow[(4 * kq + 3) * kRowWords + dp];
      uint2* out = v16t + (2 * dp) * row_words + kq;
      out[0] = make_uint2(__byte_perm(w0, w1, 0x5410), __byte_perm(w2, w3, 0x5410));
      out[row_words] = make_uint2(__byte_perm(w0, w1, 0x7632), __byte_perm(w2, w3, 0x7632));
    }
  }
}

// One 64-row tile of Q, K and V per CTA, all raw 16-byte loads issued up
// front.  A persistent form with the next tiles staged in shared memory by
// bulk copies, two CTAs per SM, was measured 36% slower on c4: the kernel is
// held by the latency of its arithmetic, which more resident warps hide.
template <typename T, int D, bool kVec16>
// Resident CTAs per SM, measured: at D = 128 three (80 registers, a few
// spilled) beat two (114, no spills) by 3% and four (64, 212 bytes spilled) by
// 7%; at D = 64 four (64 registers) beat three by 6%.
__global__ void __launch_bounds__(kPrepassThreads, D == 64 ? 4 : 3) quantize_kernel(PrepassArgs a) {
  constexpr int kVpr = D / 8;
  constexpr int kRpp = kPrepassThreads / kVpr;
  constexpr int kPasses = kKeyBlock / kRpp;
  constexpr int kRowWords = D / 2 + 1;
  constexpr int kWarps = kPrepassThreads / 32;
  __shared__ float red[kWarps][3];
  __shared__ uint32_t vrow[kKeyBlock * kRowWords];
  __shared__ float vstat[2 * kKeyBlock];  // V row maxima, then scales and reciprocals
  __shared__ float gsc[6];                // Q, Q, K group scales, then their reciprocals

  const int tile = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / a.heads, h = bh % a.heads;
  const int tid = threadIdx.x;
  const int vec = tid % kVpr;
  const int ro = tid / kVpr;
  const int64_t row0 = static_cast<int64_t>(tile) * kKeyBlock;
  // This thread's first row of each tensor; pass p is p * kRpp rows further.
  const int64_t r = row0 + ro;
  const T* qb = static_cast<const T*>(a.q) + b * a.qs[0] + h * a.qs[1] + r * a.qs[2] + vec * 8;
  const T* kb = static_cast<const T*>(a.k) + b * a.ks[0] + h * a.ks[1] + r * a.ks[2] + vec * 8;
  const T* vb = static_cast<const T*>(a.v) + b * a.vs[0] + h * a.vs[1] + r * a.vs[2] + vec * 8;
  const int64_t qstep = kRpp * a.qs[2], kstep = kRpp * a.ks[2], vstep = kRpp * a.vs[2];
  const int nvq = static_cast<int>(min(int64_t(kKeyBlock), max(int64_t(0), a.nq - row0)));
  const int nvk = static_cast<int>(min(int64_t(kKeyBlock), max(int64_t(0), a.nk - row0)));
  uint4 rq[kPasses], rk[kPasses], rv[kPasses];
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const int lr = ro + p * kRpp;
    rq[p] = (lr < nvq) ? load_raw8<T, kVec16>(qb + p * qstep) : make_uint4(0u, 0u, 0u, 0u);
    const bool kv_ok = lr < nvk;
    rk[p] = kv_ok ? load_raw8<T, kVec16>(kb + p * kstep) : make_uint4(0u, 0u, 0u, 0u);
    rv[p] = kv_ok ? load_raw8<T, kVec16>(vb + p * vstep) : make_uint4(0u, 0u, 0u, 0u);
  }
  quantize_tile<T, D>(a, bh, tile, rq, rk, rv, vrow, red, vstat, gsc);
}

}  // namespace piper
