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
//     O      = O*2^(m-m') + (P8 . V8) * 2^(mb-m')/255      (the numerator)
//   out = O / max(l, 1e-30) + mean_V
// which is the reference's arithmetic with exp/log taken base 2 (identical
// maxima and weights; rounding differs at the last-ulp level only).
//
// The numerator is accumulated by the tensor cores in F32 in TMEM across all
// blocks: each UINT8 code is written as the fp16 value P8_k * 2^(mb-m')/255
// (times a constant; one fp16 rounding), V codes are fp16 (exact), and the
// PV product is one tcgen05 kind::f16 MMA per 16 keys.  The codes are the
// reference's; only the per-block weight is applied per code instead of per
// INT32 block sum.  The lazy rescale (m' moves by more than 2^8) scales O in
// TMEM.
//
// This file holds what the attention kernels share (parameters, work units,
// tile order, constants, the row epilogue) and the 64-key-block kernel,
// block64_attention_kernel, which runs SageAttention2++ and the re-arm form of
// Piper Attention.  The production Piper kernel, with 128 keys per iteration,
// is piper_attention.cuh.  block64_attention_kernel: CTA = 384 threads, one
// CTA per SM (TMEM: all 512 columns):
//   warpgroup 0 / 1  softmax for Q tile 0 / 1 (128 rows each; thread i owns
//                    row i = TMEM lane i)
//   warp 8           TMA producer: Q tiles once, then K, V^T tiles and the
//                    per-key vectors into a K/V ring
//   warp 9           TMEM allocator + the QK^T issuer (one thread)
//   warp 10          the PV issuer (one thread); both event driven: each MMA
//                    issued as soon as its operands are ready
// Shared-memory operands are in the canonical 128B/64B-swizzled K-major
// layouts TMA writes; P is written by the softmax threads into the same
// swizzled layout.  No multicast anywhere.

// Sequence shards (ring attention): the recurrence above is associative over
// key blocks, so a launch may cover one shard of the keys and carry each
// row's (O, m, l) in a state buffer to the launch over the next shard
// (state_mode); only the last launch writes the output.  causal_shift places
// the key shard relative to the query shard for the causal mask.
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
constexpr uint64_t kWaitBudgetNs = 2000000000ull;  // 2 s per wait
// Register split (setmaxnreg): launch = 168 x 384 = 64512 registers; control
// warpgroup 56, the two softmax warpgroups 224: 128*56 + 256*224 = 64512.
// At 40 for the control warps the MMA issuer and the producer spilled (about
// 150 bytes); at 56 neither kernel spills, and the production kernel is 1.5%
// faster on c4 (measured).  The host refuses to launch if the compiled
// kernel's launch register count differs from kLaunchRegs, since an increase
// could then never be granted.
constexpr int kLaunchRegs = 168;
constexpr int kRegsControl = 56;
constexpr int kRegsSoftmax = 224;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kLaunchRegs * kAttnThreads,
              "setmaxnreg split exceeds the launch register allocation");

__device__ uint32_t g_piper_status = 0;

// Shared memory of one CTA.  kWide: the PV operands are 16-bit (Piper: fp16
// V codes and weighted fp16 probabilities, rows of 128 B, SW128); otherwise
// 8-bit (SageAttention2++: e4m3, rows of 64 B, SW64).
template <int D, bool kWide = false>
struct AttnSmem {
  static constexpr int kStages = (kWide && D == 128) ? 5 : 6;  // K/V ring depth
  static constexpr int kPVElem = kWide ? 2 : 1;                 // bytes per V / P element
  static constexpr int kQBytes = kTileM * D;       // one Q tile (SW128 for D=128, SW64 for D=64)
  static constexpr int kKBytes = kKeyBlock * D;    // one K block
  static constexpr int kVBytes = D * kKeyBlock * kPVElem;    // one V^T block (D rows x 64 keys)
  static constexpr int kPBytes = kTileM * kKeyBlock * kPVElem;  // one P tile (128 rows x 64 keys)
  static constexpr int kPVRow = kKeyBlock * kPVElem;  // bytes per V^T / P row: the swizzle width
  static constexpr int kVecBytes = 2 * kKeyBlock * 4;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTiles * kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKBytes;
  static constexpr int kOffP = kOffV + kStages * kVBytes;
  static constexpr int kOffVec = kOffP + kTiles * 2 * kPBytes;
  static constexpr int kOffBar = kOffVec + kStages * kVecBytes;
  static constexpr int kNumBars = 1 + 2 * kStages + 3 * kTiles * 2 + kTiles + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
};

static_assert(AttnSmem<128, true>::kAlloc <= 232448 && AttnSmem<128>::kAlloc <= 232448,
              "attention shared memory exceeds 227 KB");

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
  int reverse_tiles;  // heaviest-first tile order (causal): see tile_coords
  int q_tiles;  // ceil(Nq / 256)
  int64_t bh_count;  // B*H of the launch
  uint64_t wait_budget_ns;
  // Sequence shards.  Causal visibility is key <= query + causal_shift in
  // shard-local indices (causal_shift = first query position - first key
  // position; 0 for one shard).  state_mode: kStateLoad starts every row from
  // the carried (numerator, reference max, denominator) instead of zero;
  // kStateStore writes that triple back instead of the output.
  int64_t causal_shift;
  int state_mode;
  float* state_o;   // f32 [B*H, nq_all, D]  numerator (bias-free)
  float* state_ml;  // f32 [B*H, nq_all, 2]  (reference max in log2 units, denominator)
  // Sub-ranges: this launch covers rows [q_row0, q_row0 + nq) of the nq_all
  // rows per head (Q codes and scales, output and state are indexed over
  // nq_all), and keys [k_key0, k_key0 + nk) of the K/V operands (K/V codes,
  // scales and per-key vectors are laid out for the full key count).
  // q_row0 and k_key0 are multiples of 64.  One launch over everything has
  // q_row0 = k_key0 = 0 and nq_all = nq.
  int64_t nq_all, q_row0, k_key0;
  // Split-KV tail (non-causal launches): CTA u < main_units
  // takes tile u whole; CTA main_units + i takes key range i % splits of tile
  // main_units + i / splits and writes its partial state (bias-free numerator
  // [split_units][256][D], then (reference max, denominator)
  // [split_units][256][2]) to split_state; merge_split_kernel combines them
  // (key range 0 starts from the carried state under kStateLoad) and writes
  // the output, or the state under kStateStore.
  // Without a tail, splits = 0 and main_units = every tile.
  int64_t main_units;
  int splits;
  int64_t split_units;
  float* split_state;
};

constexpr int kStateLoad = 1;
constexpr int kStateStore = 2;

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

// In the re-arm form the TMEM score accumulators are pre-loaded with the bit
// pattern of 1.5*2^23 before every QK^T chain (which accumulates onto it), so
// an INT32 result v with |v| < 2^22 reads back as the float 1.5*2^23 + v
// exactly: one packed subtraction converts two values.  The other kernels
// accumulate S from zero and convert with I2F.
constexpr uint32_t kBiasBits = 0x4B400000u;
constexpr float kBias = 12582912.0f;
constexpr float kLog2FP8Max = 8.807354922057604f;  // log2(448): SageAttention2++ P codes top out at 448
constexpr float kRescaleThreshold = 8.0f;  // log2 units: numerator rescaled only past 2^8 growth

// 2^x for a pair of x <= 0 on the FMA pipe, used for a share of the
// probabilities so the MUFU pipe (16 ex2 per clock per SM, shared by the two
// softmax warps of each SMSP) is not the only source (the offload
// FlashAttention-4 publishes).  Cody-Waite split x = n + f with
// n = round(x) (the 1.5*2^23 add) and f in [-0.5, 0.5]; 2^f by a degree-5
// polynomial whose coefficients were fitted here for relative error
// (iteratively reweighted least squares, 2.3e-7 worst case in fp32 Horner,
// on a par with ex2.approx); 2^n by adding n to the exponent field (one
// integer multiply-add).  x is clamped at -126.5: for x = -inf the result is
// a denormal near 1e-38 instead of 0, which rounds to a zero UINT8 code and
// is negligible in the denominator.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  x.x = fmaxf(x.x, -126.5f);
  x.y = fmaxf(x.y, -126.5f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.0f, 12582912.0f));
  const float2 u = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(u, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(make_float2(0.001327644451521337f, 0.001327644451521337f), f,
                        make_float2(0.00967553723603487f, 0.00967553723603487f));
  p = __ffma2_rn(p, f, make_float2(0.05550713464617729f, 0.05550713464617729f));
  p = __ffma2_rn(p, f, make_float2(0.24022120237350464f, 0.24022120237350464f));
  p = __ffma2_rn(p, f, make_float2(0.6931469440460205f, 0.6931469440460205f));
  p = __ffma2_rn(p, f, make_float2(1.0000001192092896f, 1.0000001192092896f));
  return make_float2(__uint_as_float(__float_as_uint(t.x) * 0x800000u + __float_as_uint(p.x)),
                     __uint_as_float(__float_as_uint(t.y) * 0x800000u + __float_as_uint(p.y)));
}

__device__ __forceinline__ float2 f2(uint32_t a, uint32_t b) {
  return make_float2(__uint_as_float(a), __uint_as_float(b));
}

// Two INT32 scores accumulated from zero as floats (exact: |S| < 2^22).
__device__ __forceinline__ float2 i2f_pair(uint32_t u0, uint32_t u1) {
  return make_float2(__int2float_rn(static_cast<int>(u0)), __int2float_rn(static_cast<int>(u1)));
}

// Writes the bias pattern into `cols` consecutive TMEM columns of this lane.
template <int kCols>
__device__ __forceinline__ void tmem_fill_bias(uint32_t taddr) {
#pragma unroll
  for (int c = 0; c < kCols; c += 4) tmem_st4_same(taddr + c, kBiasBits);
}

// Work unit of this CTA: the tile it takes and, for a CTA of the split tail,
// its key range (split >= 0).  Cheap enough to recompute where needed, so no
// register carries it across the main loop.
struct WorkUnit {
  int64_t unit, tile;
  int split;
};
__device__ __forceinline__ WorkUnit decode_unit(const AttnParams& p) {
  WorkUnit w;
  w.unit = static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(gridDim.x) * blockIdx.y;
  w.tile = w.unit;
  w.split = -1;
  if (w.unit >= p.main_units) {
    const int64_t u = w.unit - p.main_units;
    w.tile = p.main_units + u / p.splits;
    w.split = static_cast<int>(u % p.splits);
  }
  return w;
}

// Tile index -> (b*h, query tile).  In order, query tiles run fastest within a
// head.  With reverse_tiles (causal launches, where a query tile's work grows
// with its position), the query tile is the slow index, counted down: every
// head's last query tile comes first, then every head's second-to-last, and so
// on -- the longest-work-first order in which whole-grid scheduling balances
// best, also when the grid is only a few waves (a few heads per GPU).
__device__ __forceinline__ void tile_coords(const AttnParams& p, int64_t tile, int64_t& bh, int& qt) {
  if (p.reverse_tiles) {
    bh = tile % p.bh_count;
    qt = p.q_tiles - 1 - static_cast<int>(tile / p.bh_count);
  } else {
    bh = tile / p.q_tiles;
    qt = static_cast<int>(tile % p.q_tiles);
  }
}

// ---------------------------------------------------------------------------
// SageAttention2++ (8+8) softmax role, the counterpart of the Piper softmax
// warpgroups below (sage_attention_2pp/reference.py:63-104):
//   x      = S*qs_row*ks_key*scale*log2(e) (+ -inf on padded keys)
//   m'     = max(m, max_k x - log2(448))    running max, shifted so that the
//                                           block's largest probability is 448
//   p_k    = 2^(x_k - m')  in [0, 448]      P codes: FP8 e4m3 of p_k
//   l      = l*2^(m-m') + sum_k p_k
//   O      = O*2^(m-m') + (P8 . V8)         e4m3 x e4m3 -> F32 on the tensor core
//   out    = O * vscale / max(l, 1e-30)
// The numerator is accumulated in F32 in TMEM across the blocks; the
// reference rounds each 64-key partial to fp16 first (the FP16-accumulating
// MMA it emulates), a difference at the fp16 rounding level.  The per-key K
// scale and the padded-key mask arrive through the producer's two per-key
// vector slots.
struct SoftmaxBars {
  uint32_t kv_full, s_full, s_free, p_full, pv_full, abort_flag;
};

__device__ __forceinline__ uint32_t e4m3x4(float2 a, float2 b) {
  uint32_t lo, hi;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n\tcvt.u32.u16 %0, t;\n\t}"
      : "=r"(lo) : "f"(a.y), "f"(a.x));
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n\tcvt.u32.u16 %0, t;\n\t}"
      : "=r"(hi) : "f"(b.y), "f"(b.x));
  return __byte_perm(lo, hi, 0x5410);
}

// Scales this thread's numerator row in TMEM (D columns) by w, 32 at a time.
template <int D>
__device__ __forceinline__ void tmem_scale_row(uint32_t tm_o, float w) {
  const float2 w2 = make_float2(w, w);
#pragma unroll 1
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
  tmem_st_wait();
}

// The numerator accumulates in F32 in TMEM across all blocks (the PV MMAs of
// every block add onto it); when a row's running max rises, the warp scales
// its rows there once the PV MMAs issued so far have completed.  Each block
// consumes the previous block's PV completion before releasing its own P, so
// every pv_full parity wait is unambiguous and the P buffer a block writes
// (last read by PV(j - 2)) is free.
template <typename T, int D>
__device__ __forceinline__ void sage_softmax_role(const AttnParams& p, uint8_t* smem, uint32_t sbase,
                                                  uint32_t tmem_base, const SoftmaxBars& bars, int nbt, int64_t q0,
                                                  int64_t bh, uint32_t* status, uint64_t budget) {
  using S = AttnSmem<D>;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int t = warp / 4;
  const int r = threadIdx.x % kTileM;
  const int row = static_cast<int>(q0) + t * kTileM + r;
  const bool valid_row = row < p.nq;
  const uint32_t lane_base = static_cast<uint32_t>((warp % 4) * 32) << 16;
  const uint32_t tm_s = tmem_base + lane_base + t * 256;
  const uint32_t tm_o = tm_s + 128;
  const float qs = valid_row ? __ldg(p.qscale + bh * p.nq_all + p.q_row0 + row) : 0.0f;
  const float c_row = qs * p.scale_log2e;
  const float2 c2 = make_float2(c_row, c_row);
  float m_run = -INFINITY, l_run = 0.0f;
  bool ok = true;
  int pv_seen = 0;  // pv_full completions consumed (one per block)
  for (int j = 0; j < nbt; ++j) {
    const int s = j % S::kStages;
    const int buf = j & 1;
    if (!(ok = mbar_wait_warp(bars.kv_full + 8 * s, (j / S::kStages) & 1, budget, status, kStatusTimeoutFull,
                              bars.abort_flag)))
      break;
    if (!(ok = mbar_wait_warp(bars.s_full + 8 * (t * 2 + buf), (j >> 1) & 1, budget, status, kStatusTimeoutMma,
                              bars.abort_flag)))
      break;
    tc_fence_after();
    float2 x[kKeyBlock / 2];
    {
      uint32_t a[32], b[32];
      tmem_ld32_split(tm_s + buf * kKeyBlock, a);
      tmem_ld32_split(tm_s + buf * kKeyBlock + 32, b);
      tmem_ld_wait();
      const uint32_t vm = sbase + S::kOffVec + s * S::kVecBytes;  // padded-key mask
      const uint32_t vk = vm + kKeyBlock * 4;                     // per-key K scale
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 ma = lds128(vm + 16 * i), mb = lds128(vm + 16 * (8 + i));
        const float4 ka = lds128(vk + 16 * i), kb = lds128(vk + 16 * (8 + i));
        x[2 * i] = __ffma2_rn(i2f_pair(a[4 * i], a[4 * i + 1]), __fmul2_rn(c2, make_float2(ka.x, ka.y)),
                              make_float2(ma.x, ma.y));
        x[2 * i + 1] = __ffma2_rn(i2f_pair(a[4 * i + 2], a[4 * i + 3]), __fmul2_rn(c2, make_float2(ka.z, ka.w)),
                                  make_float2(ma.z, ma.w));
        x[16 + 2 * i] = __ffma2_rn(i2f_pair(b[4 * i], b[4 * i + 1]), __fmul2_rn(c2, make_float2(kb.x, kb.y)),
                                   make_float2(mb.x, mb.y));
        x[16 + 2 * i + 1] = __ffma2_rn(i2f_pair(b[4 * i + 2], b[4 * i + 3]), __fmul2_rn(c2, make_float2(kb.z, kb.w)),
                                       make_float2(mb.z, mb.w));
      }
    }
    if (p.causal) {
      const int lim = static_cast<int>(
          max(min(static_cast<int64_t>(row) + p.causal_shift - j * kKeyBlock, static_cast<int64_t>(kKeyBlock)),
              static_cast<int64_t>(-1)));
      if (lim < kKeyBlock - 1) {
#pragma unroll
        for (int i = 0; i < kKeyBlock / 2; ++i) {
          if (2 * i > lim) x[i].x = -INFINITY;
          if (2 * i + 1 > lim) x[i].y = -INFINITY;
        }
      }
    }
    float mx[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) mx[q] = fmaxf(x[q].x, x[q].y);
#pragma unroll
    for (int i = 4; i < kKeyBlock / 2; i += 4) {
#pragma unroll
      for (int q = 0; q < 4; ++q) mx[q] = fmax3(mx[q], x[i + q].x, x[i + q].y);
    }
    const float mb = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bars.s_free + 8 * (t * 2 + buf));
    // Running max, shifted by log2(448) (reference.py:83-86): rescale the
    // numerator (in TMEM, after the earlier PV MMAs) and the denominator.
    const float msh = mb - kLog2FP8Max;
    const bool need = msh > m_run;
    if (__any_sync(0xffffffffu, need)) {
      const float m_new = need ? msh : m_run;
      // Lanes that keep their maximum scale by exactly 1 (also when it is
      // still -inf, where the difference would be NaN).
      const float w_old = need ? ex2_approx(m_run - m_new) : 1.0f;
      if (j >= 1) {
        if (!(ok = mbar_wait_warp(bars.pv_full + 8 * t, (j - 1) & 1, budget, status, kStatusTimeoutMma,
                                  bars.abort_flag)))
          break;
        pv_seen = j;
        tc_fence_after();
        tmem_scale_row<D>(tm_o, w_old);
      }
      l_run *= w_old;
      m_run = m_new;
    }
    const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
    const float2 mneg = make_float2(-m_use, -m_use);
    float2 ps[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                    make_float2(0.0f, 0.0f)};
    uint8_t* prow = smem + S::kOffP + (t * 2 + buf) * S::kPBytes + r * kKeyBlock;
    const int sw = (r >> 1) & 3;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t words[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int w = 4 * c + q;
        float2 e0 = __fadd2_rn(x[2 * w], mneg);
        float2 e1 = __fadd2_rn(x[2 * w + 1], mneg);
        e0 = make_float2(ex2_approx(e0.x), ex2_approx(e0.y));
        if (q == 0)
          e1 = exp2_poly2(e1);
        else
          e1 = make_float2(ex2_approx(e1.x), ex2_approx(e1.y));
        ps[q] = __fadd2_rn(ps[q], __fadd2_rn(e0, e1));
        words[q] = e4m3x4(e0, e1);
      }
      *reinterpret_cast<uint4*>(prow + ((c ^ sw) << 4)) = make_uint4(words[0], words[1], words[2], words[3]);
    }
    fence_proxy_async_shared();
    // PV(j - 1) completes before P(j) is released (one pv_full phase per block).
    if (j >= 1 && pv_seen < j) {
      if (!(ok = mbar_wait_warp(bars.pv_full + 8 * t, (j - 1) & 1, budget, status, kStatusTimeoutMma,
                                bars.abort_flag)))
        break;
      pv_seen = j;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bars.p_full + 8 * (t * 2 + buf));
    l_run += ((ps[0].x + ps[0].y) + (ps[1].x + ps[1].y)) + ((ps[2].x + ps[2].y) + (ps[3].x + ps[3].y));
  }
  if (ok && nbt > 0) {
    ok = mbar_wait_warp(bars.pv_full + 8 * t, (nbt - 1) & 1, budget, status, kStatusTimeoutMma, bars.abort_flag);
    tc_fence_after();
  }
  if (ok && flag_get(bars.abort_flag) == 0 && nbt > 0) {
    const float inv = 1.0f / fmaxf(l_run, 1e-30f);
    const float* vs = p.vmean + bh * D;  // per-channel V scale
    uint4* orow = reinterpret_cast<uint4*>(static_cast<T*>(p.out) + (bh * p.nq_all + p.q_row0 + row) * D);
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t v[32];
      __syncwarp();
      tmem_ld32_split(tm_o + 32 * c, v);
      tmem_ld_wait();
      if (valid_row) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 s0 = __ldg(reinterpret_cast<const float4*>(vs + 32 * c) + 2 * i);
          const float4 s1 = __ldg(reinterpret_cast<const float4*>(vs + 32 * c) + 2 * i + 1);
          const float* o = reinterpret_cast<const float*>(v) + 8 * i;
          uint4 pk;
          pk.x = pack2<T>(o[0] * s0.x * inv, o[1] * s0.y * inv);
          pk.y = pack2<T>(o[2] * s0.z * inv, o[3] * s0.w * inv);
          pk.z = pack2<T>(o[4] * s1.x * inv, o[5] * s1.y * inv);
          pk.w = pack2<T>(o[6] * s1.z * inv, o[7] * s1.w * inv);
          orow[4 * c + i] = pk;
        }
      }
    }
  }
}

// x = S*c + log2(vs_k) for the 64 scores of a block (two packed f32 per
// pair of keys).  kFromZero false: the accumulator was pre-biased, so the
// INT32 scores read as floats 1.5*2^23 + S and one packed subtraction leaves
// S exactly.  kFromZero true: the scores were accumulated from zero and are
// converted with I2F, also exactly (|S| < 2^22); measured on the 128-key
// kernel against adding the bias bits as integers and subtracting: c4 +6.8%,
// c2 +5.5%, causal c3 +5.8%, D = 64 +9.4%, identical results.
template <bool kFromZero>
__device__ __forceinline__ void scores_to_x(const uint32_t (&a)[32], const uint32_t (&b)[32], float2 (&x)[32],
                                            float c, uint32_t vl) {
  const float2 c2 = make_float2(c, c);
  const float2 nb2 = make_float2(-kBias, -kBias);
  auto pair = [&](uint32_t u0, uint32_t u1) {
    if constexpr (kFromZero)
      return i2f_pair(u0, u1);
    else
      return __fadd2_rn(f2(u0, u1), nb2);
  };
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 la = lds128(vl + 16 * i), lb = lds128(vl + 16 * (8 + i));
    x[2 * i] = __ffma2_rn(pair(a[4 * i], a[4 * i + 1]), c2, make_float2(la.x, la.y));
    x[2 * i + 1] = __ffma2_rn(pair(a[4 * i + 2], a[4 * i + 3]), c2, make_float2(la.z, la.w));
    x[16 + 2 * i] = __ffma2_rn(pair(b[4 * i], b[4 * i + 1]), c2, make_float2(lb.x, lb.y));
    x[16 + 2 * i + 1] = __ffma2_rn(pair(b[4 * i + 2], b[4 * i + 3]), c2, make_float2(lb.z, lb.w));
  }
}

// Scale of the fp16 probabilities: the PV operand of block j is
// code * w_j * kPScale / 255 (w_j = 2^(max_j - m_ref) <= 2^8), so the numerator
// in TMEM carries a factor kPScale, removed in the epilogue.  32 keeps every
// operand and the constants below within fp16 range.
constexpr float kPScale = 32.0f;

// Writes one softmax thread's query row once its last PV MMA has completed:
// the output O / (kPScale * max(l, 1e-30)) + mean_V (reference.py:116-118),
// or, for a split-tail CTA or under kStateStore, the bias-free carried state
// (O / kPScale, reference max, denominator).  `run` is false after a failed
// wait or an abort (nothing is written); `any` is false when the row saw no
// key and carried no state (the empty recurrence: output = mean_V, state =
// zeros).  Every lane takes part in the TMEM loads (warp-collective); only
// valid rows write.
template <typename T, int D>
__device__ __forceinline__ void write_row_result(const AttnParams& p, uint32_t tm_o, int t, int r, bool valid_row,
                                                 int64_t grow, float m_ref, float l_run, bool run, bool any) {
  // Recomputed here rather than kept live through the main loop.
  const WorkUnit we = decode_unit(p);
  int64_t bh_e;
  int qt_e;
  tile_coords(p, we.tile, bh_e, qt_e);
  const bool store = we.split >= 0 || (p.state_mode & kStateStore);
  if (run && any) {
    const bool write = valid_row;
    float4* so = nullptr;
    uint4* orow = nullptr;
    const float* vm = p.vmean + bh_e * D;
    float inv = 0.0f;
    if (store) {
      if (we.split >= 0) {
        const int64_t slot = (we.unit - p.main_units) * (kTileM * kTiles) + t * kTileM + r;
        so = reinterpret_cast<float4*>(p.split_state + slot * D);
        if (write) reinterpret_cast<float2*>(p.split_state + p.split_units * (kTileM * kTiles) * D)[slot] =
            make_float2(m_ref, l_run);
      } else {
        so = reinterpret_cast<float4*>(p.state_o + (bh_e * p.nq_all + grow) * D);
        if (write) reinterpret_cast<float2*>(p.state_ml)[bh_e * p.nq_all + grow] = make_float2(m_ref, l_run);
      }
    } else {
      inv = (1.0f / kPScale) / fmaxf(l_run, 1e-30f);
      orow = reinterpret_cast<uint4*>(static_cast<T*>(p.out) + (bh_e * p.nq_all + grow) * D);
    }
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t v[32];
      __syncwarp();
      tmem_ld32_split(tm_o + 32 * c, v);
      tmem_ld_wait();
      if (!write) {
      } else if (store) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          so[8 * c + i] = make_float4(__uint_as_float(v[4 * i]) * (1.0f / kPScale),
                                      __uint_as_float(v[4 * i + 1]) * (1.0f / kPScale),
                                      __uint_as_float(v[4 * i + 2]) * (1.0f / kPScale),
                                      __uint_as_float(v[4 * i + 3]) * (1.0f / kPScale));
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 m0 = __ldg(reinterpret_cast<const float4*>(vm + 32 * c) + 2 * i);
          const float4 m1 = __ldg(reinterpret_cast<const float4*>(vm + 32 * c) + 2 * i + 1);
          const float* o = reinterpret_cast<const float*>(v) + 8 * i;
          uint4 pk;
          pk.x = pack2<T>(fmaf(o[0], inv, m0.x), fmaf(o[1], inv, m0.y));
          pk.y = pack2<T>(fmaf(o[2], inv, m0.z), fmaf(o[3], inv, m0.w));
          pk.z = pack2<T>(fmaf(o[4], inv, m1.x), fmaf(o[5], inv, m1.y));
          pk.w = pack2<T>(fmaf(o[6], inv, m1.z), fmaf(o[7], inv, m1.w));
          orow[4 * c + i] = pk;
        }
      }
    }
  } else if (run && valid_row) {
    // No visible key and no carried state: an empty recurrence.
    if (store) {
      float4* so;
      float2* sml;
      if (we.split >= 0) {
        const int64_t slot = (we.unit - p.main_units) * (kTileM * kTiles) + t * kTileM + r;
        so = reinterpret_cast<float4*>(p.split_state + slot * D);
        sml = reinterpret_cast<float2*>(p.split_state + p.split_units * (kTileM * kTiles) * D) + slot;
      } else {
        so = reinterpret_cast<float4*>(p.state_o + (bh_e * p.nq_all + grow) * D);
        sml = reinterpret_cast<float2*>(p.state_ml) + bh_e * p.nq_all + grow;
      }
      for (int i = 0; i < D / 4; ++i) so[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      *sml = make_float2(m_ref, l_run);
    } else {
      const float* vm = p.vmean + bh_e * D;
      uint4* orow = reinterpret_cast<uint4*>(static_cast<T*>(p.out) + (bh_e * p.nq_all + grow) * D);
      for (int c = 0; c < D / 8; ++c) {
        const float4 m0 = __ldg(reinterpret_cast<const float4*>(vm) + 2 * c);
        const float4 m1 = __ldg(reinterpret_cast<const float4*>(vm) + 2 * c + 1);
        orow[c] = make_uint4(pack2<T>(m0.x, m0.y), pack2<T>(m0.z, m0.w), pack2<T>(m1.x, m1.y), pack2<T>(m1.z, m1.w));
      }
    }
  }
}

// Piper softmax warpgroups (reference.py:61-118): thread i of warpgroup t owns
// query row i of tile t (TMEM lane i).  Per 64-key block it converts the
// INT32 scores, takes the block max, applies the lazy rescale, and writes the
// UINT8 codes round(255 * 2^(x - max)) -- each already multiplied by its
// block weight, as fp16 -- for an fp16 PV MMA that accumulates the numerator
// in F32 in TMEM across all blocks.  The weighting is exact up to one fp16
// rounding per probability: the code bits c from the +1.5*2^23 add are placed
// under an fp16 exponent (2 + c/512), and one HFMA2 with the power-of-two
// multiples 512*w and -1024*w of the fp16 weight w gives c*w.
// This is the re-arm form (the execution plan's `rearm = 1`): the S
// accumulators are re-armed with the bias pattern by the softmax (tcgen05.st)
// after each read, and the weighted codes go to a 128B-swizzled
// shared-memory tile that the PV MMA reads.  The production form, with 128
// keys per iteration and the probabilities in TMEM, is piper_attention.cuh.
template <typename T, int D>
__device__ __forceinline__ void piper_softmax_role(const AttnParams& p, uint8_t* smem, uint32_t sbase,
                                                   uint32_t tmem_base, const SoftmaxBars& bars, int nbt, int64_t q0,
                                                   int64_t bh, int split, int64_t key0, uint32_t* status,
                                                   uint64_t budget) {
  using S = AttnSmem<D, true>;
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

  // m_ref: reference max of the numerator and denominator (log2 units).  It
  // trails the true running max by less than kRescaleThreshold, which leaves
  // O/l unchanged and skips almost every rescale.
  float m_ref = -INFINITY, l_run = 0.0f;
  bool ok = true;
  int pv_seen = 0;  // pv_full completions consumed (one per block)
  // In a split tile only key range 0 continues from the carried state; the
  // merge combines the ranges.
  const bool load = (p.state_mode & kStateLoad) && split <= 0;
  if (load) {
    // Continue the recurrence of earlier key shards: the carried numerator
    // goes into TMEM (x kPScale) before the first PV MMA accumulates onto it.
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

  for (int j = 0; j < nbt; ++j) {
    const int s = j % S::kStages;
    const int buf = j & 1;
    const float ks = __ldg(kscale + j);
    if (!(ok = mbar_wait_warp(bars.kv_full + 8 * s, (j / S::kStages) & 1, budget, status, kStatusTimeoutFull,
                              bars.abort_flag)))
      break;
    if (!(ok = mbar_wait_warp(bars.s_full + 8 * (t * 2 + buf), (j >> 1) & 1, budget, status, kStatusTimeoutMma,
                              bars.abort_flag)))
      break;
    tc_fence_after();
    float2 x[kKeyBlock / 2];
    {
      uint32_t a[32], b[32];
      tmem_ld32_split(tm_s + buf * kKeyBlock, a);
      tmem_ld32_split(tm_s + buf * kKeyBlock + 32, b);
      tmem_ld_wait();
      const uint32_t vl = sbase + S::kOffVec + s * S::kVecBytes;
      // Re-arm the S buffer; s_free is signalled after the block max, by
      // which time this store has long completed.
      tmem_fill_bias<kKeyBlock>(tm_s + buf * kKeyBlock);
      scores_to_x<false>(a, b, x, c_row * ks, vl);
    }
    if (p.causal) {
      // Keys after this row are masked (reference.py:86-91); only the
      // diagonal block needs work: lim = last visible key - first key of
      // the block, clamped to [-1, 64].
      const int lim = static_cast<int>(
          max(min(static_cast<int64_t>(row) + p.causal_shift - j * kKeyBlock, static_cast<int64_t>(kKeyBlock)),
              static_cast<int64_t>(-1)));
      if (lim < kKeyBlock - 1) {
#pragma unroll
        for (int i = 0; i < kKeyBlock / 2; ++i) {
          if (2 * i > lim) x[i].x = -INFINITY;
          if (2 * i + 1 > lim) x[i].y = -INFINITY;
        }
      }
    }
    // Block max (reference.py:94-95), four independent 3-input chains.
    float mx[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) mx[q] = fmaxf(x[q].x, x[q].y);
#pragma unroll
    for (int i = 4; i < kKeyBlock / 2; i += 4) {
#pragma unroll
      for (int q = 0; q < 4; ++q) mx[q] = fmax3(mx[q], x[i + q].x, x[i + q].y);
    }
    const float mb = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bars.s_free + 8 * (t * 2 + buf));
    // Lazy rescale of numerator and denominator (exact identity).  The
    // numerator lives in TMEM: it is scaled there once the PV MMAs of the
    // earlier blocks have completed.
    const bool need = mb > m_ref + kRescaleThreshold;
    if (__any_sync(0xffffffffu, need)) {
      const float new_ref = need ? mb : m_ref;
      const float w_old = need ? ex2_approx(m_ref - new_ref) : 1.0f;
      if (j >= 1 || load) {
        if (j >= 1 && pv_seen < j) {
          // PV(j - 1) and, in issue order, every earlier PV have completed.
          if (!(ok = mbar_wait_warp(bars.pv_full + 8 * t, (j - 1) & 1, budget, status, kStatusTimeoutMma,
                                    bars.abort_flag)))
            break;
          pv_seen = j;
        }
        tc_fence_after();
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
        tmem_st_wait();
      }
      l_run *= w_old;
      m_ref = new_ref;
    }
    // Probabilities relative to the block max: e = p * vs in [0,1]
    // (reference.py:99, 104-108); UINT8 codes round(255 e) half-to-even,
    // stored as code * w_j * kPScale / 255 in fp16.
    const float m_use = (mb == -INFINITY) ? 0.0f : mb;
    const float2 mneg = make_float2(-m_use, -m_use);
    const float w_cur = (mb == -INFINITY) ? 0.0f : ex2_approx(mb - m_ref);
    const __half wh = __float2half_rn(w_cur * (kPScale / 255.0f));
    const __half2 w512 = __half2half2(__hmul(wh, __float2half_rn(512.0f)));
    const __half2 w1024n = __half2half2(__hneg(__hmul(wh, __float2half_rn(1024.0f))));
    const uint32_t vr = sbase + S::kOffVec + s * S::kVecBytes + kKeyBlock * 4;
    float2 ps[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                    make_float2(0.0f, 0.0f)};
    const float2 k255 = make_float2(255.0f, 255.0f);
    const float2 kb2 = make_float2(kBias, kBias);
    uint8_t* prow = smem + S::kOffP + (t * 2 + buf) * S::kPBytes + r * S::kPVRow;
    const int sw = r & 7;  // 128B swizzle: 16-byte chunk index ^ (row % 8)
    uint32_t words[4];
#pragma unroll
    for (int c = 0; c < 8; ++c) {  // 8 keys per 16-byte chunk
      const float4 ra = lds128(vr + 32 * c), rb = lds128(vr + 32 * c + 16);
      const float2 rv[4] = {make_float2(ra.x, ra.y), make_float2(ra.z, ra.w), make_float2(rb.x, rb.y),
                            make_float2(rb.z, rb.w)};
      uint32_t* wc = words;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 e = __fadd2_rn(x[4 * c + q], mneg);
        // At D=64 one pair in eight goes to the FMA pipe; at D=128 the PV
        // MMA's longer shadow leaves the MUFU enough time (measured: the
        // polynomial share costs 2% there and gains 7% at D=64).
        if (D == 64 && q == 0 && (c & 1) == 0)
          e = exp2_poly2(e);
        else
          e = make_float2(ex2_approx(e.x), ex2_approx(e.y));
        ps[q] = __ffma2_rn(e, rv[q], ps[q]);
        const float2 y = __ffma2_rn(e, k255, kb2);
        uint32_t h = __byte_perm(__float_as_uint(y.x), __float_as_uint(y.y), 0x6420);  // 2 + c/512, twice
        __half2 pw = __hfma2(*reinterpret_cast<__half2*>(&h), w512, w1024n);
        wc[q] = *reinterpret_cast<uint32_t*>(&pw);
      }
      *reinterpret_cast<uint4*>(prow + ((c ^ sw) << 4)) = make_uint4(wc[0], wc[1], wc[2], wc[3]);
    }
    fence_proxy_async_shared();
    // PV of the previous block must have completed before this block's P is
    // released, so each pv_full phase is consumed before the next can
    // complete (and the P buffer of block j + 1 is free).
    if (j >= 1 && pv_seen < j) {
      if (!(ok = mbar_wait_warp(bars.pv_full + 8 * t, (j - 1) & 1, budget, status, kStatusTimeoutMma,
                                bars.abort_flag)))
        break;
      pv_seen = j;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bars.p_full + 8 * (t * 2 + buf));
    const float psum = ((ps[0].x + ps[0].y) + (ps[1].x + ps[1].y)) + ((ps[2].x + ps[2].y) + (ps[3].x + ps[3].y));
    l_run = fmaf(psum, w_cur, l_run);
  }
  if (ok && nbt > 0) {
    ok = mbar_wait_warp(bars.pv_full + 8 * t, (nbt - 1) & 1, budget, status, kStatusTimeoutMma, bars.abort_flag);
    tc_fence_after();
  }

  write_row_result<T, D>(p, tm_o, t, r, valid_row, grow, m_ref, l_run,
                         ok && flag_get(bars.abort_flag) == 0, nbt > 0 || load);
}

// The 64-key-block kernel: SageAttention2++ (kSage) and the re-arm form of
// Piper Attention.
template <typename T, int D, bool kSage>
__global__ void __launch_bounds__(kAttnThreads, 1)
    block64_attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                           const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using S = AttnSmem<D, !kSage>;
  constexpr int kStages = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align to 1024 B (the 128B-swizzle atom) while keeping the pointer derived
  // from the shared array, so every access stays a 32-bit shared access.
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
  // Shared-window addresses of the barriers (8 bytes each) and flags.
  const uint32_t sbase = smem_u32(smem);
  const uint32_t q_full = sbase + S::kOffBar;
  const uint32_t kv_full = q_full + 8;                    // [stage]
  const uint32_t kv_empty = kv_full + 8 * kStages;        // [stage]
  const uint32_t s_full = kv_empty + 8 * kStages;         // [tile][buf]
  const uint32_t s_free = s_full + 8 * kTiles * 2;        // [tile][buf]
  const uint32_t p_full = s_free + 8 * kTiles * 2;        // [tile][buf]
  const uint32_t pv_full = p_full + 8 * kTiles * 2;       // [tile]
  const uint32_t mma_done = pv_full + 8 * kTiles;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kOffMisc);
  const uint32_t abort_flag = sbase + S::kOffMisc + 4;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  // Work unit -> (tile, key range).  Tiles run query-tile fastest.
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

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(kv_full + 8 * s, 1);
      mbar_init(kv_empty + 8 * s, 1);
    }
    for (int i = 0; i < kTiles * 2; ++i) {
      mbar_init(s_full + 8 * i, 1);
      mbar_init(s_free + 8 * i, 4);
      mbar_init(p_full + 8 * i, 4);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(pv_full + 8 * t, 1);
    }
    mbar_init(mma_done, 2);  // one commit per issuing thread
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
    // Re-arm form: every QK^T MMA accumulates onto the bias pattern, so both
    // S buffers of this thread's lane are armed before the first MMA
    // (SageAttention2++ accumulates S from zero).  The numerator is cleared.
    const uint32_t lane_tm = tmem_base + (static_cast<uint32_t>((warp % 4) * 32) << 16) + (warp / 4) * 256;
    if constexpr (!kSage) tmem_fill_bias<2 * kKeyBlock>(lane_tm);
    // The F32 numerator accumulates from zero.
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
      for (int j = 0; j < nb_max; ++j) {
        const int s = j % kStages;
        if (!mbar_wait(kv_empty + 8 * (s), ((j / kStages) & 1) ^ 1, budget, status, kStatusTimeoutEmpty,
                       abort_flag))
          break;
        const uint32_t fb = kv_full + 8 * (s);
        mbar_arrive_expect_tx(fb, S::kKBytes + S::kVBytes + S::kVecBytes);
        tma_load_3d(sbase + S::kOffK + s * S::kKBytes, &tmK, fb, 0, static_cast<int>(key0) + j * kKeyBlock,
                    static_cast<int>(bh));
        tma_load_3d(sbase + S::kOffV + s * S::kVBytes, &tmV, fb, static_cast<int>(key0) + j * kKeyBlock, 0,
                    static_cast<int>(bh));
        const uint32_t vec = sbase + S::kOffVec + s * S::kVecBytes;
        bulk_load(vec, vlog2 + j * kKeyBlock, kKeyBlock * 4, fb);
        bulk_load(vec + kKeyBlock * 4, vrcp + j * kKeyBlock, kKeyBlock * 4, fb);
        ++issued;
      }
      // Drain: every copy this thread issued must land before the CTA exits.
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait(kv_full + 8 * (j % kStages), (j / kStages) & 1, budget, status, kStatusTimeoutDrain, 0u);
      mbar_wait(q_full, 0, budget, status, kStatusTimeoutDrain, 0u);
    } else if ((warp == 9 || warp == 10) && lane == 0) {
      // ------------------------------------------------ MMA issuers
      // Two issuing threads: warp 9 issues every QK^T, warp 10 every PV.  One
      // thread issuing both was the kernel's bottleneck (measured: each
      // tcgen05.mma costs its issuing thread about 80-200 cycles, and a block
      // needs 16 of them), so the scores arrived late; split, each stream of
      // MMAs advances on its own (c4 929 -> 1049 TOPS).
      // Event driven: each tile advances on its own.  QK^T of block j needs
      // the K/V stage loaded and the S buffer released by the softmax; PV of
      // block j needs its P (it accumulates onto the numerator in TMEM).
      // A stage is released to the producer by the PV thread once every tile
      // has issued its PV for that block (QK(j) has completed before P(j)
      // exists, so the PV thread's commit covers both readers of the stage).
      const bool qk_role = warp == 9;
      constexpr uint32_t kIdescQK = umma_idesc_i8(true, true, kTileM, kKeyBlock);
      bool ok = mbar_wait(q_full, 0, budget, status, kStatusTimeoutFull, abort_flag);
      tc_fence_after();
      uint64_t descQ[kTiles];
      for (int t = 0; t < kTiles; ++t) descQ[t] = umma_desc_kmajor(sbase + S::kOffQ + t * S::kQBytes, D);
      const uint64_t descK0 = umma_desc_kmajor(sbase + S::kOffK, D);
      const uint64_t descV0 = umma_desc_kmajor(sbase + S::kOffV, S::kPVRow);
      const uint64_t descP0 = umma_desc_kmajor(sbase + S::kOffP, S::kPVRow);
      int qk_next[kTiles] = {0, 0}, pv_next[kTiles] = {0, 0};
      int released = 0;
      uint64_t idle_since = 0;
      while (ok) {
        bool progress = false;
#pragma unroll
        for (int t = 0; t < kTiles; ++t) {
          const int jq = qk_next[t];
          if (qk_role && jq < nb[t] &&
              mbar_test(kv_full + 8 * (jq % kStages), (jq / kStages) & 1) &&
              mbar_test(s_free + 8 * (t * 2 + (jq & 1)), ((jq >> 1) & 1) ^ 1)) {
            tc_fence_after();
            const uint64_t descK = descK0 + static_cast<uint64_t>(((jq % kStages) * S::kKBytes) >> 4);
            const uint32_t dcol = tmem_base + t * 256 + (jq & 1) * kKeyBlock;
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk)
              umma_i8(dcol, descQ[t] + 2 * kk, descK + 2 * kk, kIdescQK, (kSage && kk == 0) ? 0u : 1u);
            umma_commit(s_full + 8 * (t * 2 + (jq & 1)));
            qk_next[t] = jq + 1;
            progress = true;
          }
          const int jp = pv_next[t];
          // PV accumulates in TMEM across blocks: no accumulator to wait for.
          if (!qk_role && jp < nb[t] && mbar_test(p_full + 8 * (t * 2 + (jp & 1)), (jp >> 1) & 1)) {
            tc_fence_after();
            const uint64_t descV = descV0 + static_cast<uint64_t>(((jp % kStages) * S::kVBytes) >> 4);
            const uint64_t descP = descP0 + static_cast<uint64_t>(((t * 2 + (jp & 1)) * S::kPBytes) >> 4);
            const uint32_t dcol = tmem_base + t * 256 + 128;
            if constexpr (kSage) {
              constexpr uint32_t kIdescPVf8 = umma_idesc_e4m3(kTileM, D);
#pragma unroll
              for (int kk = 0; kk < kKeyBlock / 32; ++kk)
                umma_f8(dcol, descP + 2 * kk, descV + 2 * kk, kIdescPVf8, 1u);
            } else {
              // fp16 weighted probabilities x fp16 V codes, 16 keys (32 B) per
              // MMA, accumulated in F32 onto the numerator in TMEM.
              constexpr uint32_t kIdescPVf16 = umma_idesc_f16(kTileM, D);
#pragma unroll
              for (int kk = 0; kk < kKeyBlock / 16; ++kk)
                umma_f16(dcol, descP + 2 * kk, descV + 2 * kk, kIdescPVf16, 1u);
            }
            umma_commit(pv_full + 8 * t);
            pv_next[t] = jp + 1;
            progress = true;
          }
        }
        while (!qk_role && released < nb_max && (released >= nb[0] || pv_next[0] > released) &&
               (released >= nb[1] || pv_next[1] > released)) {
          umma_commit(kv_empty + 8 * (released % kStages));
          ++released;
        }
        if (qk_role ? (qk_next[0] >= nb[0] && qk_next[1] >= nb[1]) : released >= nb_max) break;
        if (progress) {
          idle_since = 0;
        } else {
          const uint64_t now = global_timer_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > budget) {
            atomicOr(status, kStatusTimeoutEmpty);
            flag_set(abort_flag, 1u);
            ok = false;
          } else if (flag_get(abort_flag) != 0) {
            ok = false;
          }
          __nanosleep(32);
        }
      }
      // Everything issued (by both threads: two arrivals) must complete
      // before TMEM is freed.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, budget, status, kStatusTimeoutMma, 0u);
    }
  } else if constexpr (kSage) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const SoftmaxBars bars{kv_full, s_full, s_free, p_full, pv_full, abort_flag};
    sage_softmax_role<T, D>(p, smem, sbase, tmem_base, bars, nb[warp / 4], q0, bh, status, budget);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const SoftmaxBars bars{kv_full, s_full, s_free, p_full, pv_full, abort_flag};
    piper_softmax_role<T, D>(p, smem, sbase, tmem_base, bars, nb[warp / 4], q0, bh, split, key0, status, budget);
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
// Combines the partial states of the split tail tiles: with M = max_i m_i,
// out = sum_i O_i 2^(m_i - M) / max(sum_i l_i 2^(m_i - M), 1e-30) + mean_V
// (the same identity as the lazy rescale), or under kStateStore the merged
// state (sum_i O_i 2^(m_i - M), M, sum_i l_i 2^(m_i - M)).  One thread per
// (query row, 8 columns): grid (tail tiles, D / 8), 256 threads = 256 / (D /
// 8) rows x D / 8 column chunks, so even a handful of tail tiles spreads over
// many SMs (one CTA per tile, a row per thread, kept 24 SMs busy for the 24
// tail tiles of a 5-head launch).
template <typename T, int D>
__global__ void __launch_bounds__(kTileM * kTiles) merge_split_kernel(const AttnParams p) {
  constexpr int kChunks = D / 8;                      // 8-column chunks per row
  constexpr int kRowsPerCta = kTileM * kTiles / kChunks;
  constexpr int kRows = kTileM * kTiles;
  const int64_t st = blockIdx.x;
  const int64_t tile = p.main_units + st;
  int64_t bh;
  int qt;
  tile_coords(p, tile, bh, qt);  // same tile order as the attention kernel
  const int r = static_cast<int>(blockIdx.y) * kRowsPerCta + static_cast<int>(threadIdx.x) / kChunks;  // row in the tile
  const int c = static_cast<int>(threadIdx.x) % kChunks;
  const int64_t row = static_cast<int64_t>(qt) * kRows + r;
  if (row >= p.nq) return;
  const float2* ml = reinterpret_cast<const float2*>(p.split_state + p.split_units * kRows * D);
  float mx = -INFINITY;
  for (int i = 0; i < p.splits; ++i) mx = fmaxf(mx, ml[(st * p.splits + i) * kRows + r].x);
  float l = 0.0f;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < p.splits; ++i) {
    const float2 v = ml[(st * p.splits + i) * kRows + r];
    const float w = ex2_approx(v.x - mx);
    l = fmaf(v.y, w, l);
    const float4* so = reinterpret_cast<const float4*>(p.split_state + ((st * p.splits + i) * kRows + r) * D) + 2 * c;
    const float4 a = so[0], b = so[1];
    acc[0] = fmaf(a.x, w, acc[0]);
    acc[1] = fmaf(a.y, w, acc[1]);
    acc[2] = fmaf(a.z, w, acc[2]);
    acc[3] = fmaf(a.w, w, acc[3]);
    acc[4] = fmaf(b.x, w, acc[4]);
    acc[5] = fmaf(b.y, w, acc[5]);
    acc[6] = fmaf(b.z, w, acc[6]);
    acc[7] = fmaf(b.w, w, acc[7]);
  }
  const int64_t grow = p.q_row0 + row;
  if (p.state_mode & kStateStore) {
    float4* srow = reinterpret_cast<float4*>(p.state_o + (bh * p.nq_all + grow) * D) + 2 * c;
    srow[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    srow[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    if (c == 0) reinterpret_cast<float2*>(p.state_ml)[bh * p.nq_all + grow] = make_float2(mx, l);
  } else {
    const float inv = 1.0f / fmaxf(l, 1e-30f);
    const float4* vm = reinterpret_cast<const float4*>(p.vmean + bh * D) + 2 * c;
    const float4 m0 = vm[0], m1 = vm[1];
    uint4 pk;
    pk.x = pack2<T>(fmaf(acc[0], inv, m0.x), fmaf(acc[1], inv, m0.y));
    pk.y = pack2<T>(fmaf(acc[2], inv, m0.z), fmaf(acc[3], inv, m0.w));
    pk.z = pack2<T>(fmaf(acc[4], inv, m1.x), fmaf(acc[5], inv, m1.y));
    pk.w = pack2<T>(fmaf(acc[6], inv, m1.z), fmaf(acc[7], inv, m1.w));
    reinterpret_cast<uint4*>(static_cast<T*>(p.out) + (bh * p.nq_all + grow) * D)[c] = pk;
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
    mbar_init(smem_u32(&full_bar), 1);
    mbar_init(smem_u32(&mma_bar), 1);
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
      mbar_arrive_expect_tx(smem_u32(&full_bar), 128 * 128 + 64 * 128);
      tma_load_3d(smem_u32(sa), &tmA, smem_u32(&full_bar), kb * 128, m0, 0);
      tma_load_3d(smem_u32(sb), &tmB, smem_u32(&full_bar), kb * 128, n0, 0);
      ok = mbar_wait(smem_u32(&full_bar), kb & 1, budget_ns, &g_piper_status, kStatusTimeoutFull, 0u);
      tc_fence_after();
      if (ok) {
        const uint64_t da = umma_desc_kmajor(smem_u32(sa), 128);
        const uint64_t db = umma_desc_kmajor(smem_u32(sb), 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_i8(tmem, da + 2 * kk, db + 2 * kk, kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(smem_u32(&mma_bar));
        ok = mbar_wait(smem_u32(&mma_bar), kb & 1, budget_ns, &g_piper_status, kStatusTimeoutMma, 0u);
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

// The software exp2 of the softmax, element by element (self-test).
__global__ void selftest_exp2_kernel(const float* x, float* y, float* ex2, int64_t n) {
  const int64_t i = 2 * (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float2 v = make_float2(x[i], i + 1 < n ? x[i + 1] : 0.0f);
  const float2 e = exp2_poly2(v);
  if (y != nullptr) {
    y[i] = e.x;
    if (i + 1 < n) y[i + 1] = e.y;
  }
  if (ex2 != nullptr) {
    ex2[i] = ex2_approx(v.x);
    if (i + 1 < n) ex2[i + 1] = ex2_approx(v.y);
  }
}

// Waits on an mbarrier that nothing ever arrives at, with a short budget,
// and reports whether the wait gave up (the failure-detection self-test).
__global__ void selftest_wait_kernel(uint64_t budget_ns, int* timed_out, uint32_t* probe_status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool arrived = mbar_wait(smem_u32(&bar), 0, budget_ns, probe_status, kStatusTimeoutProbe, 0u);
    *timed_out = arrived ? 0 : 1;
  }
}

}  // namespace piper
