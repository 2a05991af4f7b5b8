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
//                      deterministic).
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

// Loads 8 consecutive elements (16 bytes when `kVec16`, else element-wise).
template <typename T, bool kVec16>
__device__ __forceinline__ void load8(const T* p, float (&out)[8]) {
  if constexpr (kVec16) {
    const int4 raw = __ldg(reinterpret_cast<const int4*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = to_f32<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = to_f32<T>(p[i]);
  }
}

__device__ __forceinline__ int8_t quantize_int8(float x, float scale) {
  float r = rintf(__fdiv_rn(x, scale));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
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
  uint8_t* ws;  // workspace base
  piper_b200_workspace_layout_t L;
};

// ---------------------------------------------------------------------------
// Column sums of K (and V when non-causal) over one chunk of rows, in fp64.
template <typename T, int D, bool kVec16>
__global__ void __launch_bounds__(kPrepassThreads) kv_sum_kernel(PrepassArgs a) {
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
  for (int64_t r = r0 + ro; r < r1; r += kRpp) {
    float x[8];
    load8<T, kVec16>(kbase + r * a.ks[2], x);
#pragma unroll
    for (int i = 0; i < 8; ++i) ksum[i] += static_cast<double>(x[i]);
    if (with_v) {
      load8<T, kVec16>(vbase + r * a.vs[2], x);
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
  float* kmean = reinterpret_cast<float*>(a.ws + a.L.kmean);
  float* vmean = reinterpret_cast<float*>(a.ws + a.L.vmean);
  if (tid < D) {
    double s = 0.0, t = 0.0;
    for (int64_t c = 0; c < chunks; ++c) {
      s += __ldcg(&kpart[(bh * chunks + c) * D + tid]);
      if (with_v) t += __ldcg(&vpart[(bh * chunks + c) * D + tid]);
    }
    kmean[bh * D + tid] = static_cast<float>(s / static_cast<double>(a.nk));
    vmean[bh * D + tid] = with_v ? static_cast<float>(t / static_cast<double>(a.nk)) : 0.0f;
  }
}

// ---------------------------------------------------------------------------
// Block-wide max of non-negative values; `scratch` holds one float per warp.
__device__ __forceinline__ float block_max_nonneg(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float m = 0.0f;
#pragma unroll
  for (int w = 0; w < kPrepassThreads / 32; ++w) m = fmaxf(m, scratch[w]);
  return m;
}

template <typename T, int D, bool kVec16>
__global__ void __launch_bounds__(kPrepassThreads) quantize_kernel(PrepassArgs a) {
  constexpr int kVpr = D / 8;
  constexpr int kRpp = kPrepassThreads / kVpr;
  constexpr int kPasses = kKeyBlock / kRpp;  // 64-row tile
  __shared__ float scratch[2][kPrepassThreads / 32];
  __shared__ __align__(16) int8_t vt[D][kKeyBlock];

  const int tile = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / a.heads, h = bh % a.heads;
  const int tid = threadIdx.x;
  const int vec = tid % kVpr;
  const int ro = tid / kVpr;
  const int64_t row0 = static_cast<int64_t>(tile) * kKeyBlock;
  const auto& L = a.L;

  // ---- Q: two 32-row groups per tile.
  if (row0 < a.nq) {
    const T* base = static_cast<const T*>(a.q) + b * a.qs[0] + h * a.qs[1] + vec * 8;
    float x[kPasses][8];
    float amax[2] = {0.0f, 0.0f};
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int lr = ro + p * kRpp;
      const int64_t r = row0 + lr;
      if (r < a.nq) {
        load8<T, kVec16>(base + r * a.qs[2], x[p]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[p][i] = 0.0f;
      }
      const int g = (p * kRpp) / kQueryGroup;  // compile-time: kRpp divides or is divided by 32
#pragma unroll
      for (int i = 0; i < 8; ++i) amax[g] = fmaxf(amax[g], fabsf(x[p][i]));
    }
    float scale[2];
    scale[0] = group_scale(block_max_nonneg(amax[0], scratch[0]));
    scale[1] = group_scale(block_max_nonneg(amax[1], scratch[1]));
    int8_t* q8 = reinterpret_cast<int8_t*>(a.ws + L.q8);
    float* qscale = reinterpret_cast<float*>(a.ws + L.qscale);
    if (tid < 2) {
      const int64_t g = row0 / kQueryGroup + tid;
      if (g < L.q_groups) qscale[bh * L.q_groups + g] = scale[tid];
    }
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int lr = ro + p * kRpp;
      const int64_t r = row0 + lr;
      if (r < a.nq) {
        const float s = scale[(p * kRpp) / kQueryGroup];
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int i = 0; i < 8; ++i)
          packed[i / 4] |= (static_cast<uint32_t>(static_cast<uint8_t>(quantize_int8(x[p][i], s))))
                           << (8 * (i % 4));
        *reinterpret_cast<uint2*>(q8 + (bh * a.nq + r) * D + vec * 8) = make_uint2(packed[0], packed[1]);
      }
    }
  }

  if (row0 >= a.nk) return;
  const float* kmean = reinterpret_cast<const float*>(a.ws + L.kmean) + bh * D + vec * 8;
  const float* vmean = reinterpret_cast<const float*>(a.ws + L.vmean) + bh * D + vec * 8;

  // ---- K: centered by the sequence mean, one 64-row group per tile.
  {
    const T* base = static_cast<const T*>(a.k) + b * a.ks[0] + h * a.ks[1] + vec * 8;
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = kmean[i];
    float x[kPasses][8];
    float amax = 0.0f;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int64_t r = row0 + ro + p * kRpp;
      if (r < a.nk) {
        load8<T, kVec16>(base + r * a.ks[2], x[p]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          x[p][i] = __fsub_rn(x[p][i], m[i]);
          amax = fmaxf(amax, fabsf(x[p][i]));
        }
      }
    }
    const float s = group_scale(block_max_nonneg(amax, scratch[0]));
    int8_t* k8 = reinterpret_cast<int8_t*>(a.ws + L.k8);
    float* kscale = reinterpret_cast<float*>(a.ws + L.kscale);
    if (tid == 0) kscale[bh * L.k_groups + tile] = s;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int64_t r = row0 + ro + p * kRpp;
      if (r < a.nk) {
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int i = 0; i < 8; ++i)
          packed[i / 4] |= (static_cast<uint32_t>(static_cast<uint8_t>(quantize_int8(x[p][i], s))))
                           << (8 * (i % 4));
        *reinterpret_cast<uint2*>(k8 + (bh * a.nk + r) * D + vec * 8) = make_uint2(packed[0], packed[1]);
      }
    }
  }

  // ---- V: per key row, centered when non-causal; codes transposed.
  {
    const T* base = static_cast<const T*>(a.v) + b * a.vs[0] + h * a.vs[1] + vec * 8;
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = a.causal ? 0.0f : vmean[i];
    float* vscale = reinterpret_cast<float*>(a.ws + L.vscale) + bh * L.nk_pad;
    float* vlog2 = reinterpret_cast<float*>(a.ws + L.vlog2) + bh * L.nk_pad;
    float* vrcp = reinterpret_cast<float*>(a.ws + L.vrcp) + bh * L.nk_pad;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int lr = ro + p * kRpp;
      const int64_t r = row0 + lr;
      const bool valid = r < a.nk;
      float x[8];
      float amax = 0.0f;
      if (valid) {
        load8<T, kVec16>(base + r * a.vs[2], x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          x[i] = __fsub_rn(x[i], m[i]);
          amax = fmaxf(amax, fabsf(x[i]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = 0.0f;
      }
      // The kVpr threads of one row are consecutive lanes.
#pragma unroll
      for (int o = kVpr / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = group_scale(amax);
#pragma unroll
      for (int i = 0; i < 8; ++i) vt[vec * 8 + i][lr] = valid ? quantize_int8(x[i], s) : int8_t(0);
      if (vec == 0) {
        vscale[r] = valid ? s : 0.0f;
        vlog2[r] = valid ? log2f(s) : -INFINITY;
        vrcp[r] = valid ? __frcp_rn(s) : 0.0f;
      }
    }
    __syncthreads();
    int8_t* v8t = reinterpret_cast<int8_t*>(a.ws + L.v8t);
    constexpr int kChunks = D * kKeyBlock / 16;  // 16-byte pieces of the [D][64] tile
    for (int c = tid; c < kChunks; c += kPrepassThreads) {
      const int d = c / (kKeyBlock / 16);
      const int part = c % (kKeyBlock / 16);
      *reinterpret_cast<int4*>(v8t + (bh * D + d) * L.nk_pad + row0 + part * 16) =
          *reinterpret_cast<const int4*>(&vt[d][part * 16]);
    }
  }
}

}  // namespace piper
