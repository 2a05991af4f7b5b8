// Quantization prepass of SageAttention2++ (the 8+8 path) for sm_100a.
//
// Restates what the reference computes before its attention loop (Piper
// Kernels 0.2.1) with its default qk_quantization = "per_thread":
//   * K sequence mean (K smoothing)   qk_quantization/int8/sage/reference.py:88-89
//   * Q codes, one scale for each set of 4 rows {g, g+8, g+16, g+24} of a
//     32-row block                    qk reference.py:23-41
//   * centred K codes, one scale for each set of 16 rows {8a + 2g + c} of a
//     64-row block                    qk reference.py:44-60
//   * V codes in FP8 e4m3, one scale per channel over the whole sequence:
//     scale = max_N |v| / 2.25 + 1e-7  sage_attention_2pp/reference.py:21-24
// INT8 codes use the exact division-free rounding of prepass.cuh; V codes are
// v / scale (IEEE division) converted with round-to-nearest-even.  Scales are
// stored per query row and per key, so the attention kernel reads one per row
// and one vector per key block.
//
// Two launches:
//   sage_stats_kernel     grid (chunks, B*H): exact fp64 K column sums and
//                         fp32 V column |max| per 512-row chunk; the last
//                         chunk of each (b,h) writes the K mean and the V
//                         scales (fixed order, deterministic).
//   sage_quantize_kernel  grid (ceil(max(Nq,Nk)/64), B*H): one 64-row tile of
//                         Q, K and V per CTA; per-row maxima in shared memory
//                         give the interleaved group scales; V codes are
//                         transposed to [D, keys] through shared memory.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "prepass.cuh"

namespace piper {

constexpr float kSageVMax = 2.25f;       // V codes span [-2.25, 2.25] before FP8

// Workspace of one SageAttention2++ call (256-byte aligned regions):
//   q8      int8  [BH, Nq, D]        Q codes
//   qscale  f32   [BH, Nq]           per-row Q scale (its interleaved group's)
//   k8      int8  [BH, Nk, D]        centred K codes
//   v8t     e4m3  [BH, D, Nk_pad]    V codes transposed (keys contiguous)
//   kscale  f32   [BH, Nk_pad]       per-key K scale; 0 on padded keys
//   kmask   f32   [BH, Nk_pad]       0 on keys, -inf on padded keys
//   vscale  f32   [BH, D]            per-channel V scale
//   kmean   f32   [BH, D]            K sequence mean
//   ksum    f64   [BH, chunks, D]    partial K sums
//   vmax    f32   [BH, chunks, D]    partial V |max|
//   counter u32   [BH]
inline piper_b200_sage2pp_layout_t make_sage_layout(int64_t bh, int64_t nq, int64_t nk, int64_t d) {
  piper_b200_sage2pp_layout_t L{};
  L.nk_pad = (nk + kKeyBlock - 1) / kKeyBlock * kKeyBlock;
  L.chunks = (nk + kSumChunkRows - 1) / kSumChunkRows;
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    const uint64_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  L.q8 = take(static_cast<uint64_t>(bh * nq * d));
  L.qscale = take(static_cast<uint64_t>(bh * nq) * 4);
  L.k8 = take(static_cast<uint64_t>(bh * nk * d));
  L.v8t = take(static_cast<uint64_t>(bh * d * L.nk_pad));
  L.kscale = take(static_cast<uint64_t>(bh * L.nk_pad) * 4);
  L.kmask = take(static_cast<uint64_t>(bh * L.nk_pad) * 4);
  L.vscale = take(static_cast<uint64_t>(bh * d) * 4);
  L.kmean = take(static_cast<uint64_t>(bh * d) * 4);
  L.ksum = take(static_cast<uint64_t>(bh * L.chunks * d) * 8);
  L.vmax = take(static_cast<uint64_t>(bh * L.chunks * d) * 4);
  L.counter = take(static_cast<uint64_t>(bh) * 4);
  L.total_bytes = off;
  return L;
}

struct SagePrepassArgs {
  const void* q;
  const void* k;
  const void* v;
  int64_t qs[3], ks[3], vs[3];  // B, H, N strides in elements
  int64_t heads, nq, nk;
  uint8_t* ws;
  piper_b200_sage2pp_layout_t L;
};

// Two floats to two FP8 e4m3 bytes (round to nearest even, saturating at
// +-448): `lo` goes to the low byte.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// ---------------------------------------------------------------------------
template <typename T, int D, bool kVec16>
__global__ void __launch_bounds__(kPrepassThreads) sage_stats_kernel(SagePrepassArgs a) {
  constexpr int kVpr = D / 8;
  constexpr int kRpp = kPrepassThreads / kVpr;
  __shared__ double red_k[kRpp][D];
  __shared__ float red_v[kRpp][D];
  __shared__ int is_last;
  const int chunk = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / a.heads, h = bh % a.heads;
  const int tid = threadIdx.x;
  const int vec = tid % kVpr;
  const int ro = tid / kVpr;
  const T* kbase = static_cast<const T*>(a.k) + b * a.ks[0] + h * a.ks[1] + vec * 8;
  const T* vbase = static_cast<const T*>(a.v) + b * a.vs[0] + h * a.vs[1] + vec * 8;
  double ksum[8];
  float vmax[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ksum[i] = 0.0;
    vmax[i] = 0.0f;
  }
  const int64_t r0 = static_cast<int64_t>(chunk) * kSumChunkRows;
  const int64_t r1 = min(r0 + kSumChunkRows, a.nk);
  for (int64_t r = r0 + ro; r < r1; r += kRpp) {
    const uint4 rk = load_raw8<T, kVec16>(kbase + r * a.ks[2]);
    const uint4 rv = load_raw8<T, kVec16>(vbase + r * a.vs[2]);
    float x[8];
    unpack8<T>(rk, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) ksum[i] += static_cast<double>(x[i]);
    unpack8<T>(rv, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) vmax[i] = fmaxf(vmax[i], fabsf(x[i]));
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    red_k[ro][vec * 8 + i] = ksum[i];
    red_v[ro][vec * 8 + i] = vmax[i];
  }
  __syncthreads();
  const auto& L = a.L;
  double* kpart = reinterpret_cast<double*>(a.ws + L.ksum);
  float* vpart = reinterpret_cast<float*>(a.ws + L.vmax);
  const int64_t chunks = L.chunks;
  if (tid < D) {
    double s = 0.0;
    float m = 0.0f;
    for (int r = 0; r < kRpp; ++r) {
      s += red_k[r][tid];
      m = fmaxf(m, red_v[r][tid]);
    }
    kpart[(bh * chunks + chunk) * D + tid] = s;
    vpart[(bh * chunks + chunk) * D + tid] = m;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned int* counter = reinterpret_cast<unsigned int*>(a.ws + L.counter) + bh;
    const unsigned int done = atomicAdd(counter, 1u);
    is_last = (done == static_cast<unsigned int>(chunks - 1));
    if (is_last) *counter = 0u;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (tid < D) {
    double s = 0.0;
    float m = 0.0f;
    for (int64_t c = 0; c < chunks; ++c) {
      s += __ldcg(&kpart[(bh * chunks + c) * D + tid]);
      m = fmaxf(m, __ldcg(&vpart[(bh * chunks + c) * D + tid]));
    }
    reinterpret_cast<float*>(a.ws + L.kmean)[bh * D + tid] = static_cast<float>(s / static_cast<double>(a.nk));
    reinterpret_cast<float*>(a.ws + L.vscale)[bh * D + tid] = __fadd_rn(__fdiv_rn(m, kSageVMax), 1e-7f);
  }
}

// ---------------------------------------------------------------------------
template <typename T, int D, bool kVec16>
__global__ void __launch_bounds__(kPrepassThreads, 3) sage_quantize_kernel(SagePrepassArgs a) {
  constexpr int kVpr = D / 8;                   // threads per row (consecutive lanes)
  constexpr int kRpp = kPrepassThreads / kVpr;  // rows per pass
  constexpr int kPasses = kKeyBlock / kRpp;
  constexpr int kRowWords = D / 4 + 1;
  __shared__ float qrow[kKeyBlock], krow[kKeyBlock];
  __shared__ uint32_t vrow[kKeyBlock * kRowWords];
  const int tile = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / a.heads, h = bh % a.heads;
  const int tid = threadIdx.x;
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
  float km[8], vsc[8];
  {
    const float* kmean = reinterpret_cast<const float*>(a.ws + L.kmean) + bh * D + vec * 8;
    const float* vscale = reinterpret_cast<const float*>(a.ws + L.vscale) + bh * D + vec * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      km[i] = has_kv ? kmean[i] : 0.0f;
      vsc[i] = has_kv ? vscale[i] : 1.0f;
    }
  }
  // ---- per-row maxima of Q and of centred K (rows past the end are zero,
  // like the reference's zero padding).
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const int lr = ro + p * kRpp;
    const int64_t r = row0 + lr;
    float x[8];
    unpack8<T>(rq[p], x);
    float mq = 0.0f, mk = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mq = fmaxf(mq, fabsf(x[i]));
    if (r < a.nk) {
      unpack8<T>(rk[p], x);
#pragma unroll
      for (int i = 0; i < 8; ++i) mk = fmaxf(mk, fabsf(__fsub_rn(x[i], km[i])));
    }
#pragma unroll
    for (int o = kVpr / 2; o > 0; o >>= 1) {
      mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, o));
      mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o));
    }
    if (vec == 0) {
      qrow[lr] = mq;
      krow[lr] = mk;
    }
  }
  __syncthreads();

  // ---- Q codes: row lr's scale is that of rows {g, g+8, g+16, g+24} of its
  // 32-row block, g = lr % 8.
  if (has_q) {
    int8_t* q8 = reinterpret_cast<int8_t*>(a.ws + L.q8);
    float* qscale = reinterpret_cast<float*>(a.ws + L.qscale) + bh * a.nq;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int lr = ro + p * kRpp;
      const int64_t r = row0 + lr;
      if (r < a.nq) {
        const int base = (lr / kQueryGroup) * kQueryGroup + lr % 8;
        const float m = fmaxf(fmaxf(qrow[base], qrow[base + 8]), fmaxf(qrow[base + 16], qrow[base + 24]));
        const float s = group_scale(m);
        float x[8];
        unpack8<T>(rq[p], x);
        *reinterpret_cast<uint2*>(q8 + (bh * a.nq + r) * D + vec * 8) = pack_codes(x, s, __frcp_rn(s));
        if (vec == 0) qscale[r] = s;
      }
    }
  }
  if (!has_kv) return;

  // ---- K codes: key lr's scale is that of keys {8a + 2g + c} of the 64-row
  // block, g = (lr / 2) % 4.
  {
    int8_t* k8 = reinterpret_cast<int8_t*>(a.ws + L.k8);
    float* kscale = reinterpret_cast<float*>(a.ws + L.kscale) + bh * L.nk_pad;
    float* kmask = reinterpret_cast<float*>(a.ws + L.kmask) + bh * L.nk_pad;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int lr = ro + p * kRpp;
      const int64_t r = row0 + lr;
      const int g = (lr / 2) % 4;
      float m = 0.0f;
#pragma unroll
      for (int aa = 0; aa < 8; ++aa) m = fmaxf(m, fmaxf(krow[8 * aa + 2 * g], krow[8 * aa + 2 * g + 1]));
      const float s = group_scale(m);
      if (r < a.nk) {
        float x[8];
        unpack8<T>(rk[p], x);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = __fsub_rn(x[i], km[i]);
        *reinterpret_cast<uint2*>(k8 + (bh * a.nk + r) * D + vec * 8) = pack_codes(x, s, __frcp_rn(s));
      }
      if (vec == 0) {
        kscale[r] = r < a.nk ? s : 0.0f;
        kmask[r] = r < a.nk ? 0.0f : -INFINITY;
      }
    }
  }

  // ---- V codes: FP8 e4m3 of v / scale[channel], into the shared tile.
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const int lr = ro + p * kRpp;
    const bool valid = row0 + lr < a.nk;
    float x[8];
    unpack8<T>(rv[p], x);
    uint32_t w0 = 0u, w1 = 0u;
    if (valid) {
      w0 = e4m3x2(__fdiv_rn(x[0], vsc[0]), __fdiv_rn(x[1], vsc[1])) |
           (e4m3x2(__fdiv_rn(x[2], vsc[2]), __fdiv_rn(x[3], vsc[3])) << 16);
      w1 = e4m3x2(__fdiv_rn(x[4], vsc[4]), __fdiv_rn(x[5], vsc[5])) |
           (e4m3x2(__fdiv_rn(x[6], vsc[6]), __fdiv_rn(x[7], vsc[7])) << 16);
    }
    vrow[lr * kRowWords + 2 * vec] = w0;
    vrow[lr * kRowWords + 2 * vec + 1] = w1;
  }
  __syncthreads();
  // ---- transpose to [D, keys], 4 keys x 4 channels at a time.
  {
    uint32_t* v8t = reinterpret_cast<uint32_t*>(a.ws + L.v8t);
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
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v8t[((bh * D + 4 * dq + j) * L.nk_pad + row0) / 4 + kq] = o[j];
    }
  }
}

}  // namespace piper
