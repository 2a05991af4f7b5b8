// Fused Piper Attention forward for sm_100a (tensor-core + softmax bound).
//
// Restates the recurrence of the reference (Piper Kernels 0.2.1,
// src/piper_kernels/attention/piper_attention/reference.py:61-118; Triton
// kernel triton.py:303-635) on the prepass's INT8 operands:
//   for each 64-key block j:
//     S      = Q8 . K8^T                                  (INT32, tensor cores)
//     x      = S*qs*ks*scale*log2(e) + log2(vs_k)          (log2 domain)
//     mb     = max_k x ;  m' = max(m, mb)
//     e_k    = 2^(x_k - mb)  (= p_k * vs_k, in [0,1])
//     P8_k   = round_half_even(255 * e_k)                  (UINT8 codes)
//     l      = l*2^(m-m') + (sum_k e_k / vs_k) * 2^(mb-m')  (FP32 denominator on unquantized p)
//     O      = O*2^(m-m') + (P8 . V8) * 2^(mb-m')/255      (UINT8 x INT8 -> INT32, tensor cores)
//   out = O / max(l, 1e-30) + mean_V
// which is the reference's arithmetic with exp/log taken base 2 (identical
// maxima and weights; rounding differs at the last-ulp level only).
//
// CTA = 384 threads, one CTA per SM (TMEM: all 512 columns):
//   warpgroup 0 / 1  softmax + numerator for Q tile 0 / 1 (128 rows each;
//                    thread i owns row i = TMEM lane i; fp32 O in registers)
//   warp 8           TMA producer: Q tiles once, then K, V^T tiles and the
//                    per-key log2(vs), 1/vs vectors into a kStages ring
//   warp 9           TMEM allocator + single-thread tcgen05.mma issuer:
//                    QK^T of block j (both tiles) then PV of block j-1
// Shared-memory operands are in the canonical 128B/64B-swizzled K-major
// layouts TMA writes; P codes are written by the softmax threads into the
// same 64B-swizzled layout.  No multicast anywhere.
//
// Every mbarrier wait is bounded (sm100.cuh): on timeout the CTA raises an
// abort flag, all roles leave their loops, drain what they issued (bounded),
// free TMEM and exit; the host reads the status word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "layout.h"
#include "sm100.cuh"

namespace piper {

constexpr int kAttnThreads = 384;
constexpr int kTileM = 128;  // query rows per softmax warpgroup
constexpr int kTiles = 2;    // Q tiles per CTA
constexpr int kStages = 4;   // K/V ring depth
constexpr uint64_t kWaitBudgetNs = 2000000000ull;  // 2 s per wait

__device__ uint32_t g_piper_status = 0;

template <int D>
struct AttnSmem {
  static constexpr int kQBytes = kTileM * D;       // one Q tile (SW128 for D=128, SW64 for D=64)
  static constexpr int kKBytes = kKeyBlock * D;    // one K block
  static constexpr int kVBytes = D * kKeyBlock;    // one V^T block (D rows x 64 keys, SW64)
  static constexpr int kPBytes = kTileM * kKeyBlock;  // one P tile (128 rows x 64 keys, SW64)
  static constexpr int kVecBytes = 2 * kKeyBlock * 4;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTiles * kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKBytes;
  static constexpr int kOffP = kOffV + kStages * kVBytes;
  static constexpr int kOffVec = kOffP + kTiles * 2 * kPBytes;
  static constexpr int kOffBar = kOffVec + kStages * kVecBytes;
  static constexpr int kNumBars = 1 + 2 * kStages + 3 * kTiles * 2 + 2 * kTiles + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
};

struct AttnParams {
  const float* qscale;
  const float* kscale;
  const float* vlog2;
  const float* vrcp;
  const float* vmean;
  void* out;
  int64_t heads, nq, nk, nk_pad, q_groups, k_groups;
  float scale_log2e;
  int causal;
  int q_tiles;  // ceil(Nq / 256)
  uint64_t wait_budget_ns;
};

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Folds the INT32 PV partial of block jj (in TMEM) into the fp32 numerator
// held in registers: o = o * w_old + PV * w_cur/255 (reference.py:102, 113).
template <int D>
__device__ __forceinline__ bool fold_pv(float (&o)[D], uint64_t* full, uint64_t* free_bar, int jj,
                                        uint32_t tm_pv, float w_old, float w_pv, int lane,
                                        uint64_t budget, uint32_t* status, volatile int* abort_flag) {
  if (!mbar_wait_warp(full, jj & 1, budget, status, kStatusTimeoutMma, abort_flag)) return false;
  tc_fence_after();
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    uint32_t v[32];
    tmem_ld32(tm_pv + c * 32, v);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * w_old + exact_i2f(v[i]) * w_pv;
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(free_bar);
  return true;
}

template <typename T, int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    piper_attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                           const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using S = AttnSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;     // [tile][buf]
  uint64_t* s_free = s_full + kTiles * 2;    // [tile][buf]
  uint64_t* p_full = s_free + kTiles * 2;    // [tile][buf]
  uint64_t* pv_full = p_full + kTiles * 2;   // [tile]
  uint64_t* pv_free = pv_full + kTiles;      // [tile]
  uint64_t* mma_done = pv_free + kTiles;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::kOffMisc + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int64_t bh = blockIdx.y;
  // Causal work grows with the query position: hand out heavy tiles first.
  const int qt = p.causal ? (p.q_tiles - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int64_t q0 = static_cast<int64_t>(qt) * kTileM * kTiles;
  const int nblocks_all = static_cast<int>((p.nk + kKeyBlock - 1) / kKeyBlock);
  int nb[kTiles];
#pragma unroll
  for (int t = 0; t < kTiles; ++t) {
    const int64_t first = q0 + t * kTileM;
    if (first >= p.nq) {
      nb[t] = 0;
    } else if (p.causal) {
      const int64_t last = min(first + kTileM - 1, p.nq - 1);
      nb[t] = min(static_cast<int>(last / kKeyBlock) + 1, nblocks_all);
    } else {
      nb[t] = nblocks_all;
    }
  }
  const int nb_max = max(nb[0], nb[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < kTiles * 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&pv_full[t], 1);
      mbar_init(&pv_free[t], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint64_t budget = p.wait_budget_ns;
  uint32_t* status = &g_piper_status;

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 40;");
    if (warp == 8 && lane == 0) {
      // ------------------------------------------------ TMA producer
      uint32_t q_bytes = 0;
      for (int t = 0; t < kTiles; ++t)
        if (nb[t] > 0) q_bytes += S::kQBytes;
      mbar_arrive_expect_tx(q_full, q_bytes);
      for (int t = 0; t < kTiles; ++t)
        if (nb[t] > 0)
          tma_load_3d(smem + S::kOffQ + t * S::kQBytes, &tmQ, q_full, 0,
                      static_cast<int>(q0 + t * kTileM), static_cast<int>(bh));
      const float* vlog2 = p.vlog2 + bh * p.nk_pad;
      const float* vrcp = p.vrcp + bh * p.nk_pad;
      int issued = 0;
      for (int j = 0; j < nb_max; ++j) {
        const int s = j % kStages;
        if (!mbar_wait(&kv_empty[s], ((j / kStages) & 1) ^ 1, budget, status, kStatusTimeoutEmpty,
                       abort_flag))
          break;
        uint64_t* fb = &kv_full[s];
        mbar_arrive_expect_tx(fb, S::kKBytes + S::kVBytes + S::kVecBytes);
        tma_load_3d(smem + S::kOffK + s * S::kKBytes, &tmK, fb, 0, j * kKeyBlock, static_cast<int>(bh));
        tma_load_3d(smem + S::kOffV + s * S::kVBytes, &tmV, fb, j * kKeyBlock, 0, static_cast<int>(bh));
        uint8_t* vec = smem + S::kOffVec + s * S::kVecBytes;
        bulk_load(vec, vlog2 + j * kKeyBlock, kKeyBlock * 4, fb);
        bulk_load(vec + kKeyBlock * 4, vrcp + j * kKeyBlock, kKeyBlock * 4, fb);
        ++issued;
      }
      // Drain: every copy this thread issued must land before the CTA exits.
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, budget, status, kStatusTimeoutDrain, nullptr);
      mbar_wait(q_full, 0, budget, status, kStatusTimeoutDrain, nullptr);
    } else if (warp == 9 && lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t kIdescQK = umma_idesc_i8(true, true, kTileM, kKeyBlock);
      constexpr uint32_t kIdescPV = umma_idesc_i8(false, true, kTileM, D);
      bool ok = mbar_wait(q_full, 0, budget, status, kStatusTimeoutFull, abort_flag);
      tc_fence_after();
      uint64_t descQ[kTiles];
      for (int t = 0; t < kTiles; ++t)
        descQ[t] = umma_desc_kmajor(smem_u32(smem + S::kOffQ + t * S::kQBytes), D);
      for (int j = 0; ok && j <= nb_max; ++j) {
        if (j < nb_max) {
          const int s = j % kStages;
          if (!(ok = mbar_wait(&kv_full[s], (j / kStages) & 1, budget, status, kStatusTimeoutFull, abort_flag)))
            break;
          tc_fence_after();
          const uint64_t descK = umma_desc_kmajor(smem_u32(smem + S::kOffK + s * S::kKBytes), D);
          for (int t = 0; t < kTiles; ++t) {
            if (j >= nb[t]) continue;
            const int buf = j & 1;
            if (!(ok = mbar_wait(&s_free[t * 2 + buf], ((j >> 1) & 1) ^ 1, budget, status,
                                 kStatusTimeoutEmpty, abort_flag)))
              break;
            tc_fence_after();
            const uint32_t dcol = tmem_base + t * 256 + buf * kKeyBlock;
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk)
              umma_i8(dcol, descQ[t] + 2 * kk, descK + 2 * kk, kIdescQK, kk > 0 ? 1u : 0u);
            umma_commit(&s_full[t * 2 + buf]);
          }
          if (!ok) break;
        }
        if (j >= 1) {
          const int jp = j - 1;
          const int sp = jp % kStages;
          const int bufp = jp & 1;
          const uint64_t descV = umma_desc_kmajor(smem_u32(smem + S::kOffV + sp * S::kVBytes), kKeyBlock);
          for (int t = 0; t < kTiles; ++t) {
            if (jp >= nb[t]) continue;
            if (!(ok = mbar_wait(&p_full[t * 2 + bufp], (jp >> 1) & 1, budget, status, kStatusTimeoutFull,
                                 abort_flag)))
              break;
            if (!(ok = mbar_wait(&pv_free[t], (jp & 1) ^ 1, budget, status, kStatusTimeoutEmpty, abort_flag)))
              break;
            tc_fence_after();
            const uint64_t descP =
                umma_desc_kmajor(smem_u32(smem + S::kOffP + (t * 2 + bufp) * S::kPBytes), kKeyBlock);
            const uint32_t dcol = tmem_base + t * 256 + 128;
#pragma unroll
            for (int kk = 0; kk < kKeyBlock / 32; ++kk)
              umma_i8(dcol, descP + 2 * kk, descV + 2 * kk, kIdescPV, kk > 0 ? 1u : 0u);
            umma_commit(&pv_full[t]);
          }
          if (!ok) break;
          umma_commit(&kv_empty[sp]);
        }
      }
      // Everything issued must complete before TMEM is freed.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, budget, status, kStatusTimeoutMma, nullptr);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 232;");
    // -------------------------------------------------- softmax warpgroups
    const int t = warp / 4;
    const int r = threadIdx.x % kTileM;
    const int64_t row = q0 + t * kTileM + r;
    const bool valid_row = row < p.nq;
    const int nbt = nb[t];
    const uint32_t lane_base = static_cast<uint32_t>((warp % 4) * 32) << 16;
    const uint32_t tm_s = tmem_base + lane_base + t * 256;
    const uint32_t tm_pv = tm_s + 128;
    const float qs = valid_row ? __ldg(p.qscale + bh * p.q_groups + row / kQueryGroup) : 0.0f;
    const float c_row = qs * p.scale_log2e;
    const float* kscale = p.kscale + bh * p.k_groups;

    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    float pend_old = 0.0f, pend_w = 0.0f;  // weights of the PV block awaiting its fold
    bool ok = true;

    for (int j = 0; j < nbt; ++j) {
      const int s = j % kStages;
      const int buf = j & 1;
      if (!(ok = mbar_wait_warp(&kv_full[s], (j / kStages) & 1, budget, status, kStatusTimeoutFull, abort_flag)))
        break;
      if (!(ok = mbar_wait_warp(&s_full[t * 2 + buf], (j >> 1) & 1, budget, status, kStatusTimeoutMma, abort_flag)))
        break;
      tc_fence_after();
      float x[kKeyBlock];
      {
        uint32_t a[32], b[32];
        tmem_ld32(tm_s + buf * kKeyBlock, a);
        tmem_ld32(tm_s + buf * kKeyBlock + 32, b);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[t * 2 + buf]);
        const float c = c_row * __ldg(kscale + j);
        const float4* vl = reinterpret_cast<const float4*>(smem + S::kOffVec + s * S::kVecBytes);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 la = vl[i], lb = vl[8 + i];
          x[4 * i + 0] = fmaf(exact_i2f(a[4 * i + 0]), c, la.x);
          x[4 * i + 1] = fmaf(exact_i2f(a[4 * i + 1]), c, la.y);
          x[4 * i + 2] = fmaf(exact_i2f(a[4 * i + 2]), c, la.z);
          x[4 * i + 3] = fmaf(exact_i2f(a[4 * i + 3]), c, la.w);
          x[32 + 4 * i + 0] = fmaf(exact_i2f(b[4 * i + 0]), c, lb.x);
          x[32 + 4 * i + 1] = fmaf(exact_i2f(b[4 * i + 1]), c, lb.y);
          x[32 + 4 * i + 2] = fmaf(exact_i2f(b[4 * i + 2]), c, lb.z);
          x[32 + 4 * i + 3] = fmaf(exact_i2f(b[4 * i + 3]), c, lb.w);
        }
      }
      if (p.causal) {
        const int64_t key0 = static_cast<int64_t>(j) * kKeyBlock;
        if (key0 + kKeyBlock - 1 > row) {
#pragma unroll
          for (int i = 0; i < kKeyBlock; ++i)
            if (key0 + i > row) x[i] = -INFINITY;
        }
      }
      float mb = x[0];
#pragma unroll
      for (int i = 1; i < kKeyBlock; ++i) mb = fmaxf(mb, x[i]);
      const float m_new = fmaxf(m_run, mb);
      const float m_use = (mb == -INFINITY) ? 0.0f : mb;
      const float4* vr = reinterpret_cast<const float4*>(smem + S::kOffVec + s * S::kVecBytes) + kKeyBlock / 4;
      float psum = 0.0f;
      uint32_t words[kKeyBlock / 4];
#pragma unroll
      for (int w = 0; w < kKeyBlock / 4; ++w) {
        const float4 rv = vr[w];
        const float rr[4] = {rv.x, rv.y, rv.z, rv.w};
        uint32_t y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float e = ex2_approx(x[4 * w + i] - m_use);
          psum = fmaf(e, rr[i], psum);
          y[i] = __float_as_uint(fmaf(e, 255.0f, 12582912.0f));
        }
        words[w] = __byte_perm(__byte_perm(y[0], y[1], 0x0040), __byte_perm(y[2], y[3], 0x0040), 0x5410);
      }
      const float w_old = ex2_approx(m_run - m_new);
      const float w_cur = ex2_approx(mb - m_new);
      l_run = l_run * w_old + psum * w_cur;
      m_run = m_new;
      {
        uint8_t* prow = smem + S::kOffP + (t * 2 + buf) * S::kPBytes + r * kKeyBlock;
        const int sw = (r >> 1) & 3;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(prow + ((c ^ sw) << 4)) =
              make_uint4(words[4 * c], words[4 * c + 1], words[4 * c + 2], words[4 * c + 3]);
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t * 2 + buf]);
      }
      if (j >= 1 && !(ok = fold_pv<D>(o, &pv_full[t], &pv_free[t], j - 1, tm_pv, pend_old, pend_w, lane, budget, status, abort_flag))) break;
      pend_old = w_old;
      pend_w = w_cur * (1.0f / 255.0f);
    }
    if (ok && nbt > 0) ok = fold_pv<D>(o, &pv_full[t], &pv_free[t], nbt - 1, tm_pv, pend_old, pend_w, lane, budget, status, abort_flag);

    if (ok && valid_row && !*abort_flag) {
      const float inv = 1.0f / fmaxf(l_run, 1e-30f);
      const float* vm = p.vmean + bh * D;
      uint32_t* orow = reinterpret_cast<uint32_t*>(static_cast<T*>(p.out) + (bh * p.nq + row) * D);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        uint4 pk;
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = o[c * 8 + i] * inv + __ldg(vm + c * 8 + i);
        pk.x = pack2<T>(f[0], f[1]);
        pk.y = pack2<T>(f[2], f[3]);
        pk.z = pack2<T>(f[4], f[5]);
        pk.w = pack2<T>(f[6], f[7]);
        reinterpret_cast<uint4*>(orow)[c] = pk;
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------------------
// Diagnostic GEMM through the same TMA + tcgen05 kind::i8 path:
// C[128 x 64 tile] = A[128 x K] . B[64 x K]^T, K in 128-byte slabs.
template <bool kASigned>
__global__ void __launch_bounds__(128, 1)
    selftest_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         int32_t* c, int64_t n, int64_t k, uint64_t budget_ns) {
  __shared__ __align__(1024) uint8_t sa[128 * 128];
  __shared__ __align__(1024) uint8_t sb[64 * 128];
  __shared__ uint64_t full_bar, mma_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int ok_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    ok_flag = 1;
    mbar_init(&full_bar, 1);
    mbar_init(&mma_bar, 1);
    fence_mbarrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int m0 = blockIdx.x * 128, n0 = blockIdx.y * 64;
  constexpr uint32_t kIdesc = umma_idesc_i8(kASigned, true, 128, 64);
  const int slabs = static_cast<int>(k / 128);
  for (int kb = 0; kb < slabs; ++kb) {
    if (threadIdx.x == 0 && ok_flag) {
      bool ok;
      mbar_arrive_expect_tx(&full_bar, 128 * 128 + 64 * 128);
      tma_load_3d(sa, &tmA, &full_bar, kb * 128, m0, 0);
      tma_load_3d(sb, &tmB, &full_bar, kb * 128, n0, 0);
      ok = mbar_wait(&full_bar, kb & 1, budget_ns, &g_piper_status, kStatusTimeoutFull, nullptr);
      tc_fence_after();
      if (ok) {
        const uint64_t da = umma_desc_kmajor(smem_u32(sa), 128);
        const uint64_t db = umma_desc_kmajor(smem_u32(sb), 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_i8(tmem, da + 2 * kk, db + 2 * kk, kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&mma_bar);
        ok = mbar_wait(&mma_bar, kb & 1, budget_ns, &g_piper_status, kStatusTimeoutMma, nullptr);
      }
      if (!ok) ok_flag = 0;
    }
    __syncthreads();
  }
  __syncwarp();
  tc_fence_after();
  uint32_t v[32];
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  for (int cc = 0; cc < 2; ++cc) {
    tmem_ld32(tmem + lane_base + cc * 32, v);
    tmem_ld_wait();
    const int64_t row = m0 + warp * 32 + lane;
    for (int i = 0; i < 32; ++i) c[row * n + n0 + cc * 32 + i] = static_cast<int32_t>(v[i]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// Waits on an mbarrier that nothing ever arrives at, with a short budget,
// and reports whether the wait gave up (the failure-detection self-test).
__global__ void selftest_wait_kernel(uint64_t budget_ns, int* timed_out, uint32_t* probe_status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool arrived = mbar_wait(&bar, 0, budget_ns, probe_status, kStatusTimeoutProbe, nullptr);
    *timed_out = arrived ? 0 : 1;
  }
}

}  // namespace piper
