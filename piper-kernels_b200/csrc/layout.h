// Workspace layout shared by the host launcher and the kernels.
//
// One contiguous caller-owned device buffer holds every intermediate of a
// piper_attention call.  Region offsets are 256-byte aligned.  Sizes for a
// problem (B,H,Nq,Nk,D) with BH = B*H, in address order:
//   q8      int8  [BH, Nq, D]                 Q codes (row-major, per-32-row scale)
//   qscale  f32   [BH, ceil(Nq/32)]           Q group scales   (reference: query_scale)
//   -- K/V pack: k8 .. vrcp are one contiguous span (kv_pack, kv_pack_bytes),
//      the unit a sequence-sharded ring passes from rank to rank --
//   k8      int8  [BH, Nk, D]                 centered-K codes (per-64-row scale)
//   v8t     f16   [BH, D, Nk_pad]             V codes (the INT8 values, exact in fp16)
//                                             transposed: keys contiguous
//   kscale  f32   [BH, ceil(Nk/64)]           K group scales   (reference: key_scale)
//   vscale  f32   [BH, Nk_pad]                V row scales     (reference: value_scale)
//   vlog2   f32   [BH, Nk_pad]                log2(vscale); -inf on padded keys
//   vrcp    f32   [BH, Nk_pad]                1/vscale; 0 on padded keys
//   -- end of the K/V pack --
//   kmean   f32   [BH, D]                     K sequence mean
//   vmean   f32   [BH, D]                     V sequence mean (zeros when causal)
//   totals  f64   [2, BH, D]                  K and V column sums of a sequence shard
//   ksum    f64   [BH, chunks, D]             per-chunk partial sums of K
//   vsum    f64   [BH, chunks, D]             per-chunk partial sums of V
//   counter u32   [BH]                        chunk-completion counters
//   split   f32   [U, 256, D] + [U, 256, 2]   partial states of the split-KV tail
// with Nk_pad = roundup(Nk, 64), chunks = ceil(Nk / kSumChunkRows) and
// U = split_units_max = min(kMaxSplitUnits, 8 * BH * ceil(Nq / 256)).
// Everything before `split` is required; the split region is optional (a
// workspace that stops at `split` runs without the split tail).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "piper_b200.h"

namespace piper {
constexpr int kQueryGroup = 32;     // rows per Q scale (per_warp granularity)
constexpr int kKeyGroup = 64;       // rows per K scale
constexpr int kKeyBlock = 64;       // keys per online-softmax block (PV block)
constexpr int kSumChunkRows = 512;  // rows per partial-sum chunk of the mean pass
constexpr int kMaxSplitUnits = 512;  // split-KV tail CTAs (a few waves of short units)
constexpr int kMaxSplits = 8;       // key ranges per tail tile

inline uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

inline piper_b200_workspace_layout_t make_layout(int64_t bh, int64_t nq, int64_t nk, int64_t d) {
  piper_b200_workspace_layout_t L{};
  L.q_groups = (nq + kQueryGroup - 1) / kQueryGroup;
  L.k_groups = (nk + kKeyGroup - 1) / kKeyGroup;
  L.nk_pad = (nk + kKeyBlock - 1) / kKeyBlock * kKeyBlock;
  L.chunks = (nk + kSumChunkRows - 1) / kSumChunkRows;
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    uint64_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  L.q8 = take(static_cast<uint64_t>(bh * nq * d));
  L.qscale = take(static_cast<uint64_t>(bh * L.q_groups) * 4);
  L.k8 = take(static_cast<uint64_t>(bh * nk * d));
  L.v8t = take(static_cast<uint64_t>(bh * d * L.nk_pad) * 2);
  L.kscale = take(static_cast<uint64_t>(bh * L.k_groups) * 4);
  L.vscale = take(static_cast<uint64_t>(bh * L.nk_pad) * 4);
  L.vlog2 = take(static_cast<uint64_t>(bh * L.nk_pad) * 4);
  L.vrcp = take(static_cast<uint64_t>(bh * L.nk_pad) * 4);
  L.kv_pack = L.k8;
  L.kv_pack_bytes = off - L.k8;
  L.kmean = take(static_cast<uint64_t>(bh * d) * 4);
  L.vmean = take(static_cast<uint64_t>(bh * d) * 4);
  L.totals = take(static_cast<uint64_t>(2 * bh * d) * 8);
  L.ksum = take(static_cast<uint64_t>(bh * L.chunks * d) * 8);
  L.vsum = take(static_cast<uint64_t>(bh * L.chunks * d) * 8);
  L.counter = take(static_cast<uint64_t>(bh) * 4);
  const int64_t tiles = bh * ((nq + 255) / 256);
  L.split_units_max = tiles > kMaxSplitUnits / kMaxSplits ? kMaxSplitUnits : tiles * kMaxSplits;
  L.split_state = take(static_cast<uint64_t>(L.split_units_max) * 256 * (d + 2) * 4);
  L.total_bytes = off;
  return L;
}
}  // namespace piper
