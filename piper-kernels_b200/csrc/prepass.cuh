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
// Three CTAs per SM keep more loads in flight (measured: the prepass is
// latency-bound at two).
__global__ void __launch_bounds__(kPrepassThreads, 3) kv_sum_kernel(PrepassArgs a) {
  constexpr int kVpr = D / 8;                      // 16-byte vectors per row
  constexpr int kRpp = kPrepassThreads / kVpr;     // rows per pass
  __shared__ double red[2][kRpp][D];
  __shared__ int is_last;

  const int chunk = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / a.heads, h = bh % a.heads;
  const int tid = threadIdx.x;
  const int vec = tid % kVpr;
  const int ro = tid / kVpr;
  const bool with_v = !a.causal;

  const T* kbase = static_cast<const T*>(a.k) + b * a.ks[0] + h * a.ks[1] + vec * 8;
  const T* vbase = static_cast<const T*>(a.v) + b * a.vs[0] + h * a.vs[1] + vec * 8;
  double ksum[8], vsum[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) ksum[i] = vsum[i] = 0.0;

  const int64_t r0 = static_cast<int64_t>(chunk) * kSumChunkRows;
  const int64_t r1 = min(r0 + kSumChunkRows, a.nk);
  // Four rows per step with all their loads issued first, so each thread
  // keeps 4 (K only) or 8 (K and V) 16-byte loads in flight.
  constexpr int kUnroll = 4;
  int64_t r = r0 + ro;
  for (; r + (kUnroll - 1) * kRpp < r1; r += kUnroll * kRpp) {
    uint4 rk[kUnroll], rv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) rk[u] = load_raw8<T, kVec16>(kbase + (r + u * kRpp) * a.ks[2]);
    if (with_v) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) rv[u] = load_raw8<T, kVec16>(vbase + (r + u * kRpp) * a.vs[2]);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float x[8];
      unpack8<T>(rk[u], x);
#pragma unroll
      for (int i = 0; i < 8; ++i) ksum[i] += static_cast<double>(x[i]);
      if (with_v) {
        unpack8<T>(rv[u], x);
#pragma unroll
        for (int i = 0; i < 8; ++i) vsum[i] += static_cast<double>(x[i]);
      }
    }
  }
  for (; r < r1; r += kRpp) {
    float x[8];
    unpack8<T>(load_raw8<T, kVec16>(kbase + r * a.ks[2]), x);
#pragma unroll
    for (int i = 0; i < 8; ++i) ksum[i] += static_cast<double>(x[i]);
    if (with_v) {
      unpack8<T>(load_raw8<T, kVec16>(vbase + r * a.vs[2]), x);
#pragma unroll
      for (int i = 0; i < 8; ++i) vsum[i] += static_cast<double>(x[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    red[0][ro][vec * 8 + i] = ksum[i];
    red[1][ro][vec * 8 + i] = vsum[i];
  }
  __syncthreads();

  double* kpart = reinterpret_cast<double*>(a.ws + a.L.ksum);
  double* vpart = reinterpret_cast<double*>(a.ws + a.L.vsum);
  const int64_t chunks = a.L.chunks;
  if (tid < D) {
    double s = 0.0;
    for (int r = 0; r < kRpp; ++r) s += red[0][r][tid];
    kpart[(bh * chunks + chunk) * D + tid] = s;
    if (with_v) {
      double t = 0.0;
      for (int r = 0; r < kRpp; ++r) t += red[1][r][tid];
      vpart[(bh * chunks + chunk) * D + tid] = t;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned int* counter = reinterpret_cast<unsigned int*>(a.ws + a.L.counter) + bh;
    const unsigned int done = atomicAdd(counter, 1u);
    is_last = (done == static_cast<unsigned int>(chunks - 1));
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

// Eight INT8 codes packed into two words, computed in packed f32x2
// arithmetic.  The near-tie test of all eight feeds one vote over the active
// lanes, so the exact-division fallback is a real branch that warps skip
// unless one of their lanes has a near-tie (it is never issued predicated
// off for every element).
__device__ __forceinline__ uint2 pack_codes(const float (&x)[8], float s, float rs) {
  uint32_t y[8];
  bool near = false;
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const float2 q = __fmul2_rn(make_float2(x[i], x[i + 1]), make_float2(rs, rs));
    const float2 t = __fadd2_rn(q, make_float2(kMagic, kMagic));
    const float2 r = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
    const float2 d = __ffma2_rn(r, make_float2(-1.0f, -1.0f), q);
    near |= (fabsf(d.x) > kNearTie) | (fabsf(d.y) > kNearTie);
    y[i] = __float_as_uint(t.x);
    y[i + 1] = __float_as_uint(t.y);
  }
  if (__any_sync(__activemask(), near)) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float q = __fmul_rn(x[i], rs);
      if (fabsf(__fsub_rn(q, __fsub_rn(__fadd_rn(q, kMagic), kMagic))) > kNearTie) y[i] = exact_code_bits(x[i], s);
    }
  }
  const uint32_t w0 = __byte_perm(__byte_perm(y[0], y[1], 0x0040), __byte_perm(y[2], y[3], 0x0040), 0x5410);
  const uint32_t w1 = __byte_perm(__byte_perm(y[4], y[5], 0x0040), __byte_perm(y[6], y[7], 0x0040), 0x5410);
  return make_uint2(w0, w1);
}

// One 64-row tile of Q, K and V per CTA.  All loads are issued up front; the
// two 32-row Q group maxima and the 64-row K group max share one block-wide
// reduction; each V row's max is a shuffle among the threads of that row.  V
// codes go row-major into a padded shared tile (row stride D/4+1 words, so
// rows fall on distinct banks), then are transposed 4x4 bytes at a time with
// byte permutes and written as [D, keys] with coalesced 4-byte stores.
// Four INT8 codes (one per byte) to four fp16 values, exactly: byte b holds
// c; (c + 128) placed under the fp16 exponent of 1024 reads as 1152 + c, and
// one packed subtraction leaves c.
__device__ __forceinline__ uint2 codes_to_f16x4(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;  // c + 128 in each byte
  const __half2 k = __halves2half2(__float2half_rn(1152.0f), __float2half_rn(1152.0f));
  uint32_t lo = __byte_perm(u, 0x64646464u, 0x5140);  // halves 0x64:(c0+128), 0x64:(c1+128)
  uint32_t hi = __byte_perm(u, 0x64646464u, 0x5342);
  __half2 a = __hsub2(*reinterpret_cast<__half2*>(&lo), k);
  __half2 b = __hsub2(*reinterpret_cast<__half2*>(&hi), k);
  return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

template <typename T, int D, bool kVec16>
// Three CTAs per SM (80 registers, a few spilled) beat two at 111 registers
// by about 10% on the whole prepass: more 16-byte loads in flight.
__global__ void __launch_bounds__(kPrepassThreads, 3) quantize_kernel(PrepassArgs a) {
  constexpr int kVpr = D / 8;                   // 16-byte vectors per row
  constexpr int kRpp = kPrepassThreads / kVpr;  // rows per pass
  constexpr int kPasses = kKeyBlock / kRpp;     // passes over the 64-row tile
  constexpr int kRowWords = D / 4 + 1;          // padded V code row, in words
  constexpr int kWarps = kPrepassThreads / 32;
  __shared__ float red[kWarps][3];
  __shared__ uint32_t vrow[kKeyBlock * kRowWords];

  const int tile = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / a.heads, h = bh % a.heads;
  const int tid = threadIdx.x;
  const int lane = tid % 32, warp = tid / 32;
  const int vec = tid % kVpr;
  const int ro = tid / kVpr;
  const int64_t row0 = static_cast<int64_t>(tile) * kKeyBlock;
  const auto& L = a.L;
  const bool has_q = row0 < a.nq;
  const bool has_kv = row0 < a.nk;

  const T* qb = static_cast<const T*>(a.q) + b * a.qs[0] + h * a.qs[1] + vec * 8;
  const T* kb = static_cast<const T*>(a.k) + b * a.ks[0] + h * a.ks[1] + vec * 8;
  const T* vb = static_cast<const T*>(a.v) + b * a.vs[0] + h * a.vs[1] + vec * 8;
  uint4 rq[kPasses], rk[kPasses], rv[kPasses];
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const int64_t r = row0 + ro + p * kRpp;
    rq[p] = (r < a.nq) ? load_raw8<T, kVec16>(qb + r * a.qs[2]) : make_uint4(0u, 0u, 0u, 0u);
    const bool kv_ok = r < a.nk;
    rk[p] = kv_ok ? load_raw8<T, kVec16>(kb + r * a.ks[2]) : make_uint4(0u, 0u, 0u, 0u);
    rv[p] = kv_ok ? load_raw8<T, kVec16>(vb + r * a.vs[2]) : make_uint4(0u, 0u, 0u, 0u);
  }
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

  // ---- group maxima: Q (two 32-row groups) and centered K (one 64-row group);
  // rows past the sequence end count as zero, as the reference's zero padding.
  float am[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const int64_t r = row0 + ro + p * kRpp;
    float x[8];
    unpack8<T>(rq[p], x);
    const int g = (p * kRpp) / kQueryGroup;  // compile-time: kRpp divides or is divided by 32
#pragma unroll
    for (int i = 0; i < 8; ++i) am[g] = fmaxf(am[g], fabsf(x[i]));
    if (r < a.nk) {
      unpack8<T>(rk[p], x);
#pragma unroll
      for (int i = 0; i < 8; ++i) am[2] = fmaxf(am[2], fabsf(__fsub_rn(x[i], km[i])));
    }
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
  __syncthreads();
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    float m = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, red[w][c]);
    am[c] = m;
  }

  // ---- Q codes.
  if (has_q) {
    const float sq[2] = {group_scale(am[0]), group_scale(am[1])};
    const float rq2[2] = {__frcp_rn(sq[0]), __frcp_rn(sq[1])};
    int8_t* q8 = reinterpret_cast<int8_t*>(a.ws + L.q8);
    if (tid < 2) {
      const int64_t g = row0 / kQueryGroup + tid;
      if (g < L.q_groups) reinterpret_cast<float*>(a.ws + L.qscale)[bh * L.q_groups + g] = sq[tid];
    }
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int64_t r = row0 + ro + p * kRpp;
      if (r < a.nq) {
        const int g = (p * kRpp) / kQueryGroup;
        float x[8];
        unpack8<T>(rq[p], x);
        *reinterpret_cast<uint2*>(q8 + (bh * a.nq + r) * D + vec * 8) = pack_codes(x, sq[g], rq2[g]);
      }
    }
  }
  if (!has_kv) return;

  // ---- K codes (centered by the sequence mean).
  {
    const float sk = group_scale(am[2]);
    const float rsk = __frcp_rn(sk);
    int8_t* k8 = reinterpret_cast<int8_t*>(a.ws + L.k8);
    if (tid == 0) reinterpret_cast<float*>(a.ws + L.kscale)[bh * L.k_groups + tile] = sk;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int64_t r = row0 + ro + p * kRpp;
      if (r < a.nk) {
        float x[8];
        unpack8<T>(rk[p], x);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = __fsub_rn(x[i], km[i]);
        *reinterpret_cast<uint2*>(k8 + (bh * a.nk + r) * D + vec * 8) = pack_codes(x, sk, rsk);
      }
    }
  }

  // ---- V: per key row (centered when non-causal), codes into the shared tile.
  {
    float* vscale = reinterpret_cast<float*>(a.ws + L.vscale) + bh * L.nk_pad;
    float* vlog2 = reinterpret_cast<float*>(a.ws + L.vlog2) + bh * L.nk_pad;
    float* vrcp = reinterpret_cast<float*>(a.ws + L.vrcp) + bh * L.nk_pad;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int lr = ro + p * kRpp;
      const int64_t r = row0 + lr;
      const bool valid = r < a.nk;
      float x[8];
      unpack8<T>(rv[p], x);
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[i] = __fsub_rn(x[i], vm[i]);
        amax = fmaxf(amax, fabsf(x[i]));
      }
      if (!valid) amax = 0.0f;
      // The kVpr threads of one row are consecutive lanes.
#pragma unroll
      for (int o = kVpr / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = group_scale(amax);
      const float rs = __frcp_rn(s);
      const uint2 codes = valid ? pack_codes(x, s, rs) : make_uint2(0u, 0u);
      vrow[lr * kRowWords + 2 * vec] = codes.x;
      vrow[lr * kRowWords + 2 * vec + 1] = codes.y;
      if (vec == 0) {
        vscale[r] = valid ? s : 0.0f;
        vlog2[r] = valid ? log2f(s) : -INFINITY;
        vrcp[r] = valid ? rs : 0.0f;
      }
    }
  }
  __syncthreads();
  // ---- transpose to [D, keys]: each step moves a 4-key x 4-feature block;
  // the codes are stored as fp16 (the attention kernel's PV operand).
  {
    uint2* v16t = reinterpret_cast<uint2*>(a.ws + L.v8t);
    constexpr int kBlocks = (D / 4) * (kKeyBlock / 4);
#pragma unroll
    for (int blk = tid; blk < kBlocks; blk += kPrepassThreads) {
      const int kq = blk % (kKeyBlock / 4);
      const int dq = blk / (kKeyBlock / 4);
      const uint32_t w0 = vrow[(4 * kq + 0) * kRowWords + dq];
      const uint32_t w1 = vrow[(4 * kq + 1) * kRowWords + dq];
      const uint32_t w2 = vrow[(4 * kq + 2) * kRowWords + dq];
      const uint32_t w3 = vrow[(4 * kq + 3) * kRowWords + dq];
      const uint32_t t0 = __byte_perm(w0, w1, 0x5140), t1 = __byte_perm(w2, w3, 0x5140);
      const uint32_t t2 = __byte_perm(w0, w1, 0x7362), t3 = __byte_perm(w2, w3, 0x7362);
      const uint32_t o[4] = {__byte_perm(t0, t1, 0x5410), __byte_perm(t0, t1, 0x7632), __byte_perm(t2, t3, 0x5410),
                             __byte_perm(t2, t3, 0x7632)};
      // 8-byte index of (d, key) = ((bh*D + d) * nk_pad + key) / 4; nk_pad and row0 are multiples of 64.
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v16t[((bh * D + 4 * dq + j) * L.nk_pad + row0) / 4 + kq] = codes_to_f16x4(o[j]);
    }
  }
}

}  // namespace piper
