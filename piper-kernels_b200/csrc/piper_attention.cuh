// Fused Piper Attention forward for sm_100a: the production kernel.
//
// The recurrence is the one attention.cuh states (reference.py:61-118, Triton
// kernel triton.py:303-635): per 64-key reference block, INT8 QK^T, a base-2
// online softmax with the block's own maximum, UINT8 probability codes
// round(255 * 2^(x - max)) weighted by the block's factor, and a numerator
// accumulated by the tensor cores.  What differs from the 64-key-block kernel
// is the schedule, chosen from tcgen05 measurements on B200: an MMA costs the
// tensor pipe about 65-75 cycles whatever its size up to N = 128 (an
// M128 N64 K32 INT8 MMA, which needs 32 cycles of math, runs at 43% of the
// pipe's rate; N = 128 at 84-95%).  So each iteration covers 128 keys, two
// reference blocks, with one N = 128 QK^T MMA per 32-byte K step:
//
//   per Q tile t (128 rows) and iteration j (keys 128j .. 128j + 127):
//     QK(j)   S_t <- Q_t . K(j)^T            4 x kind::i8 M128 N128 K32 (D = 128)
//     softmax reads S_t (128 INT32 columns), takes the two block maxima,
//             applies the lazy rescale, writes the weighted fp16 codes of both
//             blocks into TMEM over S_t's first 64 columns, releases P(j)
//     PV(j)   O_t += P(j) . V(j)              8 x kind::f16 M128 N=D K16, A from TMEM
//     QK(j+1) issued by the same thread right after PV(j): the tensor pipe
//             runs one thread's MMAs in issue order, so S_t is overwritten
//             only after PV(j) has read P(j)
//
// TMEM (512 columns): tile t owns columns [256t, 256t + 128) for S / P and
// [256t + 128, 256t + 128 + D) for its F32 numerator.  One S buffer per tile:
// a single issuing thread serves the tiles in a fixed order, so tile 1's
// scores arrive one tensor phase after tile 0's and one tile's softmax runs
// while the other tile's PV and QK^T execute (measured with clock64 probes:
// the tiles settle half an iteration apart).  Measured on B200 against the
// 64-key-block kernel with two issuers (same box, prepared inputs): c4 +1%,
// c2 +1%, causal c3 +3%, D = 64 +8%.
//
// CTA = 384 threads, one CTA per SM:
//   warpgroup 0 / 1  softmax for Q tile 0 / 1 (thread i owns row i = lane i)
//   warp 8           TMA producer: Q tiles once, then per iteration two
//                    64-row K boxes, two 64-key V^T boxes (fp16 codes) and the
//                    per-key log2(vs), 1/vs vectors into a 3-stage ring
//                    (6 at D = 64)
//   warp 9           TMEM allocator and the MMA issuer (one thread): QK(0)
//                    of both tiles, then per iteration PV(j), QK(j+1) of
//                    tile 0, then of tile 1
// A stage returns to the producer when both tiles' PV(j) have completed.
// No TMA multicast.  Every wait is bounded (sm100.cuh).
#pragma once

#include "attention.cuh"

namespace piper {

constexpr int kPairKeys = 2 * kKeyBlock;  // keys per iteration (two reference blocks)

template <int D>
struct PairSmem {
  static constexpr int kStages = D == 128 ? 3 : 6;          // K/V ring depth (iterations)
  static constexpr int kQBytes = kTileM * D;                // one Q tile
  static constexpr int kKBytes = kPairKeys * D;             // 128 K rows (two 64-row boxes)
  static constexpr int kVBoxBytes = D * kKeyBlock * 2;      // one 64-key V^T box of fp16 codes
  static constexpr int kVBytes = 2 * kVBoxBytes;
  static constexpr int kVecBytes = 2 * kPairKeys * 4;       // log2(vs)[128] then 1/vs[128]
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTiles * kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKBytes;
  static constexpr int kOffVec = kOffV + kStages * kVBytes;
  static constexpr int kOffBar = kOffVec + kStages * kVecBytes;
  // q_full, kv_full[stages], kv_empty[stages], s_full[2], p_full[2][2], o_done[2], mma_done
  static constexpr int kNumBars = 1 + 2 * kStages + 4 * kTiles + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
};

static_assert(PairSmem<128>::kAlloc <= 232448 && PairSmem<64>::kAlloc <= 232448,
              "attention shared memory exceeds 227 KB");
static_assert(PairSmem<128>::kOffV % 1024 == 0 && PairSmem<64>::kOffV % 1024 == 0 &&
                  PairSmem<128>::kVBoxBytes % 1024 == 0 && PairSmem<64>::kVBoxBytes % 1024 == 0,
              "V^T boxes must start on 1024-byte swizzle atoms");

// Keys of one reference block after `lim` (the block's last visible key
// relative to its first, clamped to [-1, 64]) are masked.
__device__ __forceinline__ void mask_after(float2 (&x)[32], int lim) {
  if (lim < kKeyBlock - 1) {
#pragma unroll
    for (int i = 0; i < kKeyBlock / 2; ++i) {
      if (2 * i > lim) x[i].x = -INFINITY;
      if (2 * i + 1 > lim) x[i].y = -INFINITY;
    }
  }
}

// Maximum of one block's 64 values: four independent 3-input chains.
__device__ __forceinline__ float block_max(const float2 (&x)[32]) {
  float mx[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) mx[q] = fmaxf(x[q].x, x[q].y);
#pragma unroll
  for (int i = 4; i < kKeyBlock / 2; i += 4) {
#pragma unroll
    for (int q = 0; q < 4; ++q) mx[q] = fmax3(mx[q], x[i + q].x, x[i + q].y);
  }
  return fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]);
}

// UINT8 codes of one block, weighted: for each key e = 2^(x - mb) (= p*vs),
// code = round_half_even(255 e), written into TMEM at tm_p (32 columns, fp16
// pairs: column c holds keys 2c, 2c + 1) as the fp16 value code * w * kPScale
// / 255 with w = 2^(mb - m_ref).  Returns sum_k e_k / vs_k (the block's
// unweighted denominator); *w_out = w.
template <int D>
__device__ __forceinline__ float block_codes(const float2 (&x)[32], float mb, float m_ref, uint32_t vr, uint32_t tm_p,
                                             float* w_out) {
  const float m_use = (mb == -INFINITY) ? 0.0f : mb;
  const float2 mneg = make_float2(-m_use, -m_use);
  const float w = (mb == -INFINITY) ? 0.0f : ex2_approx(mb - m_ref);
  *w_out = w;
  const __half wh = __float2half_rn(w * (kPScale / 255.0f));
  const __half2 w512 = __half2half2(__hmul(wh, __float2half_rn(512.0f)));
  const __half2 w1024n = __half2half2(__hneg(__hmul(wh, __float2half_rn(1024.0f))));
  float2 ps[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                  make_float2(0.0f, 0.0f)};
  const float2 k255 = make_float2(255.0f, 255.0f);
  const float2 kb2 = make_float2(kBias, kBias);
  // All 64 exponentials first: independent MUFU (or FMA-pipe) operations
  // that one warp can issue back to back, then the code arithmetic.
  float2 e[kKeyBlock / 2];
#pragma unroll
  for (int i = 0; i < kKeyBlock / 2; ++i) {
    e[i] = __fadd2_rn(x[i], mneg);
    // At D = 64 one pair in eight goes to the FMA pipe (measured on the
    // 64-key kernel: +7% there, -2% at D = 128).
    if (D == 64 && (i & 7) == 0)
      e[i] = exp2_poly2(e[i]);
    else
      e[i] = make_float2(ex2_approx(e[i].x), ex2_approx(e[i].y));
  }
  uint32_t words[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {  // 8 keys per step
    const float4 ra = lds128(vr + 32 * c), rb = lds128(vr + 32 * c + 16);
    const float2 rv[4] = {make_float2(ra.x, ra.y), make_float2(ra.z, ra.w), make_float2(rb.x, rb.y),
                          make_float2(rb.z, rb.w)};
    uint32_t* wc = words + 4 * (c & 1);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      ps[q] = __ffma2_rn(e[4 * c + q], rv[q], ps[q]);
      const float2 y = __ffma2_rn(e[4 * c + q], k255, kb2);
      uint32_t h = __byte_perm(__float_as_uint(y.x), __float_as_uint(y.y), 0x6420);  // 2 + c/512, twice
      __half2 pw = __hfma2(*reinterpret_cast<__half2*>(&h), w512, w1024n);
      wc[q] = *reinterpret_cast<uint32_t*>(&pw);
    }
    if (c & 1) tmem_st8(tm_p + 4 * (c - 1), words);  // keys 8(c-1) .. 8c+7: columns 4(c-1) .. 4c+3
  }
  return ((ps[0].x + ps[0].y) + (ps[1].x + ps[1].y)) + ((ps[2].x + ps[2].y) + (ps[3].x + ps[3].y));
}

// Softmax warpgroup t: thread i owns query row i of tile t (TMEM lane i).
// nbt = 64-key blocks this tile sees; iteration j covers blocks 2j (A) and
// 2j + 1 (B, absent when 2j + 1 == nbt).
template <typename T, int D>
__device__ __forceinline__ void pair_softmax_role(const AttnParams& p, uint32_t sbase, uint32_t tmem_base,
                                                  uint32_t kv_full, uint32_t s_full, uint32_t p_full_a,
                                                  uint32_t p_full_b, uint32_t o_done, uint32_t abort_flag, int nbt,
                                                  int64_t q0,
                                                  int64_t bh, int split, int64_t key0, uint32_t* status,
                                                  uint64_t budget) {
  using S = PairSmem<D>;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int t = warp / 4;
  const int r = threadIdx.x % kTileM;
  const int row = static_cast<int>(q0) + t * kTileM + r;
  const bool valid_row = row < p.nq;
  const int64_t grow = p.q_row0 + row;  // row within the head's nq_all rows
  const uint32_t lane_base = static_cast<uint32_t>((warp % 4) * 32) << 16;
  const uint32_t tm_s = tmem_base + lane_base + t * 256;
  const uint32_t tm_o = tm_s + 128;
  const float qs = valid_row ? __ldg(p.qscale + bh * p.q_groups + grow / kQueryGroup) : 0.0f;
  const float c_row = qs * p.scale_log2e;
  const float* kscale = p.kscale + bh * p.k_groups + key0 / kKeyGroup;

  // m_ref trails the running max by less than kRescaleThreshold (lazy
  // rescale: an exact identity that skips almost every rescale).
  float m_ref = -INFINITY, l_run = 0.0f;
  bool ok = true;
  // In a split tile only key range 0 continues from the carried state.
  const bool load = (p.state_mode & kStateLoad) && split <= 0;
  if (load) {
    // The carried numerator goes into TMEM (x kPScale) before PV(0) adds to it.
    const float4* so = reinterpret_cast<const float4*>(p.state_o + (bh * p.nq_all + grow) * D);
#pragma unroll 4
    for (int c = 0; c < D / 8; ++c) {
      uint32_t v[8];
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (valid_row) {
        a = so[2 * c];
        b = so[2 * c + 1];
      }
      v[0] = __float_as_uint(a.x * kPScale);
      v[1] = __float_as_uint(a.y * kPScale);
      v[2] = __float_as_uint(a.z * kPScale);
      v[3] = __float_as_uint(a.w * kPScale);
      v[4] = __float_as_uint(b.x * kPScale);
      v[5] = __float_as_uint(b.y * kPScale);
      v[6] = __float_as_uint(b.z * kPScale);
      v[7] = __float_as_uint(b.w * kPScale);
      tmem_st8(tm_o + 8 * c, v);
    }
    tmem_st_wait();
    if (valid_row) {
      const float2 ml = reinterpret_cast<const float2*>(p.state_ml)[bh * p.nq_all + grow];
      m_ref = ml.x;
      l_run = ml.y;
    }
  }

  const int nit = (nbt + 1) / 2;
  for (int j = 0; j < nit; ++j) {
    const int s = j % S::kStages;
    const bool has_b = 2 * j + 1 < nbt;
    const float ksa = __ldg(kscale + 2 * j);
    const float ksb = has_b ? __ldg(kscale + 2 * j + 1) : 0.0f;
    if (!(ok = mbar_wait_warp(kv_full + 8 * s, (j / S::kStages) & 1, budget, status, kStatusTimeoutFull,
                              abort_flag)))
      break;
    if (!(ok = mbar_wait_sleep_warp(s_full, j & 1, budget, status, kStatusTimeoutMma, abort_flag))) break;
    tc_fence_after();
    const uint32_t vec = sbase + S::kOffVec + s * S::kVecBytes;
    float2 xa[kKeyBlock / 2], xb[kKeyBlock / 2];
    {
      uint32_t a0[32], a1[32], b0[32], b1[32];
      tmem_ld32(tm_s, a0);
      tmem_ld32(tm_s + 32, a1);
      tmem_ld32(tm_s + 64, b0);
      tmem_ld32(tm_s + 96, b1);
      tmem_ld_wait();
      scores_to_x<true>(a0, a1, xa, c_row * ksa, vec);
      scores_to_x<true>(b0, b1, xb, c_row * ksb, vec + kKeyBlock * 4);
    }
    if (!has_b) {
      // Block B lies past this tile's keys: its smem may hold stale data.
#pragma unroll
      for (int i = 0; i < kKeyBlock / 2; ++i) xb[i] = make_float2(-INFINITY, -INFINITY);
    }
    if (p.causal) {
      // Keys after this row are masked (reference.py:86-91); only diagonal
      // blocks need work.
      const int64_t rel = static_cast<int64_t>(row) + p.causal_shift - 2 * j * kKeyBlock;
      mask_after(xa, static_cast<int>(max(min(rel, int64_t(kKeyBlock)), int64_t(-1))));
      mask_after(xb, static_cast<int>(max(min(rel - kKeyBlock, int64_t(kKeyBlock)), int64_t(-1))));
    }
    const float mba = block_max(xa);
    const float mbb = block_max(xb);
    const float mb = fmaxf(mba, mbb);
    // Lazy rescale of numerator and denominator.  PV(j - 1) has completed:
    // the issuer committed s_full after QK(j), which it issued after PV(j - 1).
    const bool need = mb > m_ref + kRescaleThreshold;
    if (__any_sync(0xffffffffu, need)) {
      const float new_ref = need ? mb : m_ref;
      const float w_old = need ? ex2_approx(m_ref - new_ref) : 1.0f;
      if (j >= 1 || load) {
        const float2 w2 = make_float2(w_old, w_old);
#pragma unroll 2
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32_split(tm_o + 32 * c, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 y = __fmul2_rn(f2(v[2 * i], v[2 * i + 1]), w2);
            v[2 * i] = __float_as_uint(y.x);
            v[2 * i + 1] = __float_as_uint(y.y);
          }
          tmem_st8(tm_o + 32 * c, v);
          tmem_st8(tm_o + 32 * c + 8, v + 8);
          tmem_st8(tm_o + 32 * c + 16, v + 16);
          tmem_st8(tm_o + 32 * c + 24, v + 24);
        }
      }
      l_run *= w_old;
      m_ref = new_ref;
    }
    // Probabilities relative to each block's max (reference.py:99, 104-108),
    // written into TMEM over the spent scores: block A in columns 0-31,
    // block B in 32-63.
    // Block A's codes are released first, so that its PV MMAs run while
    // block B's are computed.
    const uint32_t vr = vec + kPairKeys * 4;
    float wa, wb = 0.0f;
    const float psa = block_codes<D>(xa, mba, m_ref, vr, tm_s, &wa);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_full_a);
    float psb = 0.0f;
    if (has_b) {
      psb = block_codes<D>(xb, mbb, m_ref, vr + kKeyBlock * 4, tm_s + kKeyBlock / 2, &wb);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full_b);
    }
    l_run = fmaf(psa, wa, l_run);
    l_run = fmaf(psb, wb, l_run);
  }
  if (ok && nbt > 0) {
    ok = mbar_wait_sleep_warp(o_done, 0, budget, status, kStatusTimeoutMma, abort_flag);
    tc_fence_after();
  }
  write_row_result<T, D>(p, tm_o, t, r, valid_row, grow, m_ref, l_run, ok && flag_get(abort_flag) == 0,
                         nbt > 0 || load);
}

template <typename T, int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    piper_attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using S = PairSmem<D>;
  constexpr int kStages = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t q_full = sbase + S::kOffBar;
  const uint32_t kv_full = q_full + 8;                // [stage]
  const uint32_t kv_empty = kv_full + 8 * kStages;    // [stage]
  const uint32_t s_full = kv_empty + 8 * kStages;     // [tile]
  const uint32_t p_full = s_full + 8 * kTiles;        // [tile][block A, block B]
  const uint32_t o_done = p_full + 16 * kTiles;       // [tile]
  const uint32_t mma_done = o_done + 8 * kTiles;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kOffMisc);
  const uint32_t abort_flag = sbase + S::kOffMisc + 4;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const WorkUnit wu = decode_unit(p);
  const int split = wu.split;  // >= 0: this CTA is key range `split` of a tail tile
  int64_t bh;
  int qt;
  tile_coords(p, wu.tile, bh, qt);
  const int64_t q0 = static_cast<int64_t>(qt) * kTileM * kTiles;
  int64_t key0 = p.k_key0;  // first key of this CTA's range
  int64_t nk_cta = p.nk;
  if (split >= 0) {
    const int64_t blocks = (p.nk + kKeyBlock - 1) / kKeyBlock;
    const int64_t b0 = blocks * split / p.splits, b1 = blocks * (split + 1) / p.splits;
    key0 = p.k_key0 + b0 * kKeyBlock;
    nk_cta = min(p.nk, b1 * kKeyBlock) - b0 * kKeyBlock;
  }
  const int nblocks_all = static_cast<int>((nk_cta + kKeyBlock - 1) / kKeyBlock);
  int nb[kTiles];
#pragma unroll
  for (int t = 0; t < kTiles; ++t) {
    const int64_t first = q0 + t * kTileM;
    if (first >= p.nq) {
      nb[t] = 0;
    } else if (p.causal) {
      // Last key any row of the tile sees; none when the whole shard of keys
      // lies after the tile.
      const int64_t last_key = min(first + kTileM - 1, p.nq - 1) + p.causal_shift;
      nb[t] = last_key < 0 ? 0 : static_cast<int>(min(last_key / kKeyBlock + 1, static_cast<int64_t>(nblocks_all)));
    } else {
      nb[t] = nblocks_all;
    }
  }
  const int nb_max = max(nb[0], nb[1]);
  const int nit_max = (nb_max + 1) / 2;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(kv_full + 8 * s, 1);
      mbar_init(kv_empty + 8 * s, 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(s_full + 8 * t, 1);
      mbar_init(p_full + 16 * t, 4);  // one arrival per softmax warp
      mbar_init(p_full + 16 * t + 8, 4);
      mbar_init(o_done + 8 * t, 1);
    }
    mbar_init(mma_done, 1);
    flag_set(abort_flag, 0u);
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
  if (warp < 8) {
    // The F32 numerator accumulates from zero (or from a carried state the
    // softmax writes before its first P release).
    const uint32_t lane_tm = tmem_base + (static_cast<uint32_t>((warp % 4) * 32) << 16) + (warp / 4) * 256;
#pragma unroll
    for (int c = 0; c < D; c += 4) tmem_st4_same(lane_tm + 128 + c, 0u);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    if (warp == 8 && lane == 0) {
      // ------------------------------------------------ TMA producer
      uint32_t q_bytes = 0;
      for (int t = 0; t < kTiles; ++t)
        if (nb[t] > 0) q_bytes += S::kQBytes;
      mbar_arrive_expect_tx(q_full, q_bytes);
      for (int t = 0; t < kTiles; ++t)
        if (nb[t] > 0)
          tma_load_3d(sbase + S::kOffQ + t * S::kQBytes, &tmQ, q_full, 0,
                      static_cast<int>(p.q_row0 + q0 + t * kTileM), static_cast<int>(bh));
      const float* vlog2 = p.vlog2 + bh * p.nk_pad + key0;
      const float* vrcp = p.vrcp + bh * p.nk_pad + key0;
      int issued = 0;
      for (int j = 0; j < nit_max; ++j) {
        const int s = j % kStages;
        if (!mbar_wait_sleep(kv_empty + 8 * s, ((j / kStages) & 1) ^ 1, budget, status, kStatusTimeoutEmpty,
                             abort_flag))
          break;
        // Block B of the last iteration may lie past every tile's keys: then
        // only block A is loaded (the issuer skips block B's PV MMAs and the
        // softmax masks its scores, so its stale K rows are harmless).
        const bool two = 2 * j + 1 < nb_max;
        const int nblk = two ? 2 : 1;
        const uint32_t fb = kv_full + 8 * s;
        mbar_arrive_expect_tx(fb, nblk * (S::kKBytes / 2 + S::kVBoxBytes + kKeyBlock * 8));
        const int k0 = static_cast<int>(key0) + j * kPairKeys;
        for (int b = 0; b < nblk; ++b) {
          tma_load_3d(sbase + S::kOffK + s * S::kKBytes + b * (S::kKBytes / 2), &tmK, fb, 0, k0 + b * kKeyBlock,
                      static_cast<int>(bh));
          tma_load_3d(sbase + S::kOffV + s * S::kVBytes + b * S::kVBoxBytes, &tmV, fb, k0 + b * kKeyBlock, 0,
                      static_cast<int>(bh));
        }
        const uint32_t vec = sbase + S::kOffVec + s * S::kVecBytes;
        bulk_load(vec, vlog2 + j * kPairKeys, nblk * kKeyBlock * 4, fb);
        bulk_load(vec + kPairKeys * 4, vrcp + j * kPairKeys, nblk * kKeyBlock * 4, fb);
        ++issued;
      }
      // Drain: every copy this thread issued must land before the CTA exits.
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait(kv_full + 8 * (j % kStages), (j / kStages) & 1, budget, status, kStatusTimeoutDrain, 0u);
      mbar_wait(q_full, 0, budget, status, kStatusTimeoutDrain, 0u);
    } else if (warp == 9 && lane == 0) {
      // ------------------------------------------------ MMA issuer (one thread)
      // Fixed order per iteration: tile 0's PV(j) then QK(j+1), then tile 1's.
      // The tensor pipe runs them in that order, so tile 1's scores arrive one
      // tensor phase after tile 0's and the two softmax warpgroups stay
      // staggered: one computes while the other's MMAs run.  (Two issuing
      // threads let the pipe interleave both tiles' MMAs, which put the tiles
      // in lockstep: measured 30% slower.)  Block A's PV MMAs go as soon as
      // its codes are released, block B's when its codes are.
      constexpr uint32_t kIdescQK = umma_idesc_i8(true, true, kTileM, kPairKeys);
      constexpr uint32_t kIdescPV = umma_idesc_f16(kTileM, D);
      const uint64_t descK0 = umma_desc_kmajor(sbase + S::kOffK, D);
      const uint64_t descV0 = umma_desc_kmajor(sbase + S::kOffV, kKeyBlock * 2);
      int nit[kTiles];
      for (int t = 0; t < kTiles; ++t) nit[t] = (nb[t] + 1) / 2;
      bool ok = nit_max == 0 || (mbar_wait(q_full, 0, budget, status, kStatusTimeoutFull, abort_flag) &&
                                 mbar_wait(kv_full, 0, budget, status, kStatusTimeoutFull, abort_flag));
      tc_fence_after();
      for (int t = 0; ok && t < kTiles; ++t) {
        if (nit[t] == 0) continue;
        const uint64_t descQ = umma_desc_kmajor(sbase + S::kOffQ + t * S::kQBytes, D);
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk)
          umma_i8(tmem_base + t * 256, descQ + 2 * kk, descK0 + 2 * kk, kIdescQK, kk > 0 ? 1u : 0u);
        umma_commit(s_full + 8 * t);
      }
      for (int j = 0; ok && j < nit_max; ++j) {
        const int s = j % kStages;
        const uint64_t descV = descV0 + static_cast<uint64_t>((s * S::kVBytes) >> 4);
        for (int t = 0; ok && t < kTiles; ++t) {
          if (j >= nit[t]) continue;
          const uint32_t tm_s = tmem_base + t * 256;
          const uint32_t tm_o = tm_s + 128;
          // PV(j): 16 keys per MMA, A (the weighted codes) from TMEM, 8
          // columns per MMA; V^T from the stage's two 64-key boxes.
          const int halves = 2 * j + 1 < nb[t] ? 2 : 1;
          for (int hb = 0; ok && hb < halves; ++hb) {
            if (!(ok = mbar_wait(p_full + 16 * t + 8 * hb, j & 1, budget, status, kStatusTimeoutFull, abort_flag)))
              break;
            tc_fence_after();
            const uint64_t descVb = descV + static_cast<uint64_t>((hb * S::kVBoxBytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < kKeyBlock / 16; ++kk)
              umma_f16_ts(tm_o, tm_s + 32 * hb + 8 * kk, descVb + 2 * kk, kIdescPV, 1u);
          }
          if (!ok) break;
          if (j + 1 < nit[t]) {
            const int s1 = (j + 1) % kStages;
            if (!(ok = mbar_wait(kv_full + 8 * s1, ((j + 1) / kStages) & 1, budget, status, kStatusTimeoutFull,
                                 abort_flag)))
              break;
            tc_fence_after();
            const uint64_t descQ = umma_desc_kmajor(sbase + S::kOffQ + t * S::kQBytes, D);
            const uint64_t descK = descK0 + static_cast<uint64_t>((s1 * S::kKBytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk)
              umma_i8(tm_s, descQ + 2 * kk, descK + 2 * kk, kIdescQK, kk > 0 ? 1u : 0u);
            umma_commit(s_full + 8 * t);
          } else {
            umma_commit(o_done + 8 * t);
          }
        }
        // Both tiles' PV(j) are issued: stage s returns to the producer when
        // they complete.
        if (ok) umma_commit(kv_empty + 8 * s);
      }
      // Everything issued must complete before TMEM is freed.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, budget, status, kStatusTimeoutMma, 0u);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int t = warp / 4;
    pair_softmax_role<T, D>(p, sbase, tmem_base, kv_full, s_full + 8 * t, p_full + 16 * t, p_full + 16 * t + 8,
                            o_done + 8 * t, abort_flag, nb[t], q0, bh, split, key0, status, budget);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace piper
