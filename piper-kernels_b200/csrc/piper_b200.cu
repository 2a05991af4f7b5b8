// C ABI of the B200 Piper Attention backend (declared in include/piper_b200.h).
//
// Host orchestration that replaces the reference's Triton launch sequence
// (Piper Kernels 0.2.1, attention/piper_attention/triton.py:772-981):
// argument checks, per-device one-time set-up, TMA tensor-map encoding and
// the three kernel launches, all on the caller's stream with no host sync.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "attention.cuh"
#include "piper_attention.cuh"
#include "layout.h"
#include "piper_b200.h"
#include "prepass.cuh"
#include "sage2pp.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(PIPER_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

#define PIPER_CUDA(call)                                   \
  do {                                                     \
    cudaError_t e_ = (call);                               \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);    \
  } while (0)

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

constexpr int kMaxDevices = 64;
std::mutex g_init_mutex;
bool g_device_ready[kMaxDevices] = {};
unsigned long long g_device_context[kMaxDevices] = {};  // context the set-up was done in
int g_device_sms[kMaxDevices] = {};
EncodeTiledFn g_encode = nullptr;
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

// Identity of the calling thread's current CUDA context (0 when none is
// current).  Per-device set-up lives in a context: after cudaDeviceReset, or
// once the primary context is destroyed and made again, kernel attributes and
// symbol addresses of the old context no longer apply, and the new context
// has a new id (cuCtxGetId ids are unique for the life of the process).
// Called with g_init_mutex held.
unsigned long long current_context_id() {
  if (g_ctx_get_current == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(fn);
    cudaGetLastError();
  }
  CUcontext ctx = nullptr;
  if (g_ctx_get_current == nullptr || g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (g_ctx_get_id != nullptr && g_ctx_get_id(ctx, &id) == CUDA_SUCCESS) return id + 1;
  return static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(ctx));
}

// Per-device set-up (thread safe), redone whenever the device's context
// changes: architecture check and the dynamic shared-memory opt-in of the
// attention kernels.
int ensure_device(int* device_out) {
  int device = 0;
  PIPER_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices) return fail(PIPER_B200_ERR_UNSUPPORTED_DEVICE, "device index out of range");
  *device_out = device;
  // Makes the device's primary context current (creating it after a reset),
  // so that its id can be compared with the one the set-up was done in.
  PIPER_CUDA(cudaSetDevice(device));
  std::lock_guard<std::mutex> lock(g_init_mutex);
  const unsigned long long context = current_context_id();
  if (g_device_ready[device] && context != 0 && g_device_context[device] == context) return PIPER_B200_OK;
  g_device_ready[device] = false;
  cudaDeviceProp prop;
  PIPER_CUDA(cudaGetDeviceProperties(&prop, device));
  g_device_sms[device] = prop.multiProcessorCount;
  if (prop.major != 10 || prop.minor != 0)
    return fail(PIPER_B200_ERR_UNSUPPORTED_DEVICE,
                "piper_b200 requires an sm_100 (B200-class) GPU, got sm_" + std::to_string(prop.major) +
                    std::to_string(prop.minor));
  if (g_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    PIPER_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || fn == nullptr)
      return fail(PIPER_B200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  // The attention kernels redistribute registers between warpgroups with
  // setmaxnreg, which is only safe at the launch register count the split was
  // computed for.
  // Piper: the production kernel (128 keys per iteration, P in TMEM) and
  // the re-arm form of the 64-key-block kernel; SageAttention2++: the
  // 64-key-block kernel with 8-bit PV operands.
  struct Instance {
    const void* fn;
    int smem;
  };
  const Instance kernels[] = {
      {reinterpret_cast<const void*>(piper::piper_attention_kernel<__half, 64>), piper::PairSmem<64>::kAlloc},
      {reinterpret_cast<const void*>(piper::piper_attention_kernel<__half, 128>), piper::PairSmem<128>::kAlloc},
      {reinterpret_cast<const void*>(piper::piper_attention_kernel<__nv_bfloat16, 64>), piper::PairSmem<64>::kAlloc},
      {reinterpret_cast<const void*>(piper::piper_attention_kernel<__nv_bfloat16, 128>), piper::PairSmem<128>::kAlloc},
      {reinterpret_cast<const void*>(piper::block64_attention_kernel<__half, 64, false>), piper::AttnSmem<64, true>::kAlloc},
      {reinterpret_cast<const void*>(piper::block64_attention_kernel<__half, 128, false>), piper::AttnSmem<128, true>::kAlloc},
      {reinterpret_cast<const void*>(piper::block64_attention_kernel<__nv_bfloat16, 64, false>), piper::AttnSmem<64, true>::kAlloc},
      {reinterpret_cast<const void*>(piper::block64_attention_kernel<__nv_bfloat16, 128, false>), piper::AttnSmem<128, true>::kAlloc},
      {reinterpret_cast<const void*>(piper::block64_attention_kernel<__half, 64, true>), piper::AttnSmem<64>::kAlloc},
      {reinterpret_cast<const void*>(piper::block64_attention_kernel<__half, 128, true>), piper::AttnSmem<128>::kAlloc},
      {reinterpret_cast<const void*>(piper::block64_attention_kernel<__nv_bfloat16, 64, true>), piper::AttnSmem<64>::kAlloc},
      {reinterpret_cast<const void*>(piper::block64_attention_kernel<__nv_bfloat16, 128, true>), piper::AttnSmem<128>::kAlloc},
  };
  for (const Instance& k : kernels) {
    const void* fn = k.fn;
    const int smem_bytes = k.smem;
    PIPER_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes));
    cudaFuncAttributes attr;
    PIPER_CUDA(cudaFuncGetAttributes(&attr, fn));
    if (attr.numRegs != piper::kLaunchRegs)
      return fail(PIPER_B200_ERR_CUDA, "attention kernel compiled with " + std::to_string(attr.numRegs) +
                                           " registers per thread; its warpgroup register split needs " +
                                           std::to_string(piper::kLaunchRegs));
    int resident = 0;
    PIPER_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, fn, piper::kAttnThreads, smem_bytes));
    if (resident < 1)
      return fail(PIPER_B200_ERR_UNSUPPORTED_DEVICE, "an attention CTA does not fit on one SM of this device");
  }
  g_device_ready[device] = true;
  g_device_context[device] = current_context_id();
  return PIPER_B200_OK;
}

// 3-D tensor map of 1- or 2-byte elements: dims {inner, mid, outer} in
// elements with byte strides {mid_stride, outer_stride}, a box {box_inner,
// box_mid, 1} and the swizzle matching the box's inner extent in bytes (64 or
// 128).
int encode_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t mid, uint64_t outer,
               uint64_t mid_stride, uint64_t outer_stride, uint32_t box_inner, uint32_t box_mid,
               int elem_bytes = 1) {
  const cuuint64_t dims[3] = {inner, mid, outer};
  const cuuint64_t strides[2] = {mid_stride, outer_stride};
  const cuuint32_t box[3] = {box_inner, box_mid, 1};
  const cuuint32_t elem[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw =
      box_inner * elem_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapDataType type = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUresult r = g_encode(map, type, 3, const_cast<void*>(base), dims, strides, box,
                              elem, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PIPER_B200_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return PIPER_B200_OK;
}

int check_shape(int dtype, int64_t b, int64_t h, int64_t nq, int64_t nk, int64_t d, int causal) {
  if (dtype != PIPER_B200_FLOAT16 && dtype != PIPER_B200_BFLOAT16)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "dtype must be PIPER_B200_FLOAT16 or PIPER_B200_BFLOAT16");
  if (d != 64 && d != 128)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "head_dim must be 64 or 128, got " + std::to_string(d));
  if (b <= 0 || h <= 0) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "batch and heads must be positive");
  if (nq <= 0 || nk <= 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "query and key lengths must be positive");
  if (causal && nq != nk)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "causal attention requires equal query and key lengths");
  if (b * h > 65535) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "batch*heads must be at most 65535");
  if (nq > (int64_t(1) << 30) || nk > (int64_t(1) << 30))
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "sequence lengths must be below 2^30");
  return PIPER_B200_OK;
}

bool aligned16(const void* p, const int64_t s[3]) {
  return (reinterpret_cast<uintptr_t>(p) % 16 == 0) && s[0] % 8 == 0 && s[1] % 8 == 0 && s[2] % 8 == 0;
}

// Which prepass kernels a call runs.
enum PrepassPart { kSums = 1, kFinalize = 2, kQuantize = 4 };

template <typename T, int D, bool V16>
void launch_prepass_t(const piper::PrepassArgs& a, int64_t bh, int parts, cudaStream_t stream) {
  if (parts & kSums) {
    // One CTA per (chunk, head, tensor): K, and V unless causal.
    const dim3 sum_grid(static_cast<unsigned>(a.L.chunks), static_cast<unsigned>(bh), a.causal ? 1u : 2u);
    piper::kv_sum_kernel<T, D, V16><<<sum_grid, piper::kPrepassThreads, 0, stream>>>(a);
  }
  if (parts & kFinalize) piper::finalize_means_kernel<D><<<static_cast<unsigned>(bh), D, 0, stream>>>(a);
  if (parts & kQuantize) {
    const int64_t tiles = (std::max(a.nq, a.nk) + piper::kKeyBlock - 1) / piper::kKeyBlock;
    // At D = 128 one CTA per (tile, head, tensor): Q, K, V; at D = 64 one per
    // (tile, head).
    const dim3 q_grid(static_cast<unsigned>(tiles), static_cast<unsigned>(bh), D == 128 ? 3u : 1u);
    piper::quantize_kernel<T, D, V16><<<q_grid, piper::kPrepassThreads, 0, stream>>>(a);
  }
}

template <typename T, int D>
void launch_prepass_d(const piper::PrepassArgs& a, int64_t bh, bool v16, int parts, cudaStream_t stream) {
  if (v16)
    launch_prepass_t<T, D, true>(a, bh, parts, stream);
  else
    launch_prepass_t<T, D, false>(a, bh, parts, stream);
}

// Shared argument checks and launches of the prepass entry points.
// `parts` selects the kernels; `sums_only` makes the mean pass write the
// shard's fp64 totals; `total_keys` is the mean's denominator for kFinalize.
int run_prepass(const void* query, const int64_t query_strides[3], const void* key, const int64_t key_strides[3],
                const void* value, const int64_t value_strides[3], int dtype, int64_t batch, int64_t heads,
                int64_t query_length, int64_t key_length, int64_t head_dim, int is_causal, void* workspace,
                size_t workspace_bytes, void* stream, int parts, int sums_only, int64_t total_keys) {
  int rc = check_shape(dtype, batch, heads, query_length, key_length, head_dim, is_causal);
  if (rc != PIPER_B200_OK) return rc;
  if (!key || !value || !workspace || !key_strides || !value_strides)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  if ((parts & kQuantize) && (!query || !query_strides))
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  int device = 0;
  if ((rc = ensure_device(&device)) != PIPER_B200_OK) return rc;
  const int64_t bh = batch * heads;
  const piper_b200_workspace_layout_t L = piper::make_layout(bh, query_length, key_length, head_dim);
  if (workspace_bytes < L.split_state)
    return fail(PIPER_B200_ERR_WORKSPACE_TOO_SMALL,
                "workspace needs " + std::to_string(L.split_state) + " bytes, got " + std::to_string(workspace_bytes));
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  piper::PrepassArgs a{};
  a.q = query;
  a.k = key;
  a.v = value;
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = query_strides ? query_strides[i] : 0;
    a.ks[i] = key_strides[i];
    a.vs[i] = value_strides[i];
  }
  a.heads = heads;
  a.nq = query_length;
  a.nk = key_length;
  a.causal = is_causal ? 1 : 0;
  a.sums_only = sums_only;
  a.total_keys = total_keys;
  a.ws = static_cast<uint8_t*>(workspace);
  a.L = L;
  bool v16 = aligned16(key, key_strides) && aligned16(value, value_strides);
  if (parts & kQuantize) v16 = v16 && aligned16(query, query_strides);
  if (parts & kSums) PIPER_CUDA(cudaMemsetAsync(a.ws + L.counter, 0, static_cast<size_t>(bh) * 4, s));
  if (dtype == PIPER_B200_FLOAT16) {
    if (head_dim == 64)
      launch_prepass_d<__half, 64>(a, bh, v16, parts, s);
    else
      launch_prepass_d<__half, 128>(a, bh, v16, parts, s);
  } else {
    if (head_dim == 64)
      launch_prepass_d<__nv_bfloat16, 64>(a, bh, v16, parts, s);
    else
      launch_prepass_d<__nv_bfloat16, 128>(a, bh, v16, parts, s);
  }
  PIPER_CUDA(cudaGetLastError());
  return PIPER_B200_OK;
}

// Production plan of one attention launch over `q_rows` query rows and `keys`
// keys per head (pure host logic).  The tile shape and ring depth are fixed by
// the compiled kernels; the rest are the measured choices:
//   - rearm = 0: the production kernel (128 keys per iteration, the
//     probabilities in TMEM) is faster than the 64-key re-arm kernel for
//     every launch kind.
//   - heavy_first: causal grids run longest-work-first across all heads.
//   - split-KV tail: when the tiles do not fill whole waves on the SMs, the
//     `tail` tiles of the last partial wave are cut into k key ranges, k in
//     [2, min(kMaxSplits, key blocks / 2)] chosen to minimise the tail's time
//     in tile units, ceil(tail * k / SMs) / k (the smaller k on ties); no
//     split when no k beats one whole wave (non-causal launches, and only
//     when the workspace has the split region for tail * k units).  For
//     example 44 tail tiles on 148 SMs take k = 3 (one wave of third
//     tiles), 96 take k = 3 (two waves of third tiles: 0.67 of a tile
//     instead of a whole one).
piper_b200_plan_t make_plan(int64_t bh, int64_t q_rows, int64_t keys, int64_t d, bool causal, int sms,
                            bool split_region, int64_t split_units_max) {
  piper_b200_plan_t P{};
  P.tile_rows = piper::kTileM * piper::kTiles;
  P.key_block = piper::kKeyBlock;
  P.stages = d == 128 ? piper::PairSmem<128>::kStages : piper::PairSmem<64>::kStages;
  P.rearm = 0;
  P.heavy_first = causal ? 1 : 0;
  P.sms = sms;
  P.tiles = (q_rows + P.tile_rows - 1) / P.tile_rows * bh;
  if (!causal && split_region && P.tiles < (int64_t(1) << 30)) {
    const int64_t tail = P.tiles % sms;
    const int64_t blocks = (keys + piper::kKeyBlock - 1) / piper::kKeyBlock;
    // Compare costs as fractions ceil(tail*k/sms)/k against best_num/best_den.
    int64_t best_k = 0, best_num = 1, best_den = 1;
    for (int64_t k = 2; tail > 0 && k <= piper::kMaxSplits && k <= blocks / 2 && tail * k <= split_units_max; ++k) {
      const int64_t waves = (tail * k + sms - 1) / sms;
      if (waves * best_den < best_num * k) {
        best_k = k;
        best_num = waves;
        best_den = k;
      }
    }
    if (best_k > 0) {
      P.split_k = static_cast<int32_t>(best_k);
      P.tail_tiles = tail;
    }
  }
  P.ctas = P.tiles - P.tail_tiles + P.tail_tiles * P.split_k;
  P.kernels = P.split_k > 0 ? 2 : 1;
  return P;
}

// Checks a caller-edited plan against what the kernels can run and fills in
// its derived fields.
int check_plan(piper_b200_plan_t* P, int64_t bh, int64_t q_rows, int64_t keys, int64_t d, bool causal,
               bool split_region, int64_t split_units_max) {
  const piper_b200_plan_t ref = make_plan(bh, q_rows, keys, d, causal, P->sms > 0 ? P->sms : 148, false, 0);
  if (P->tile_rows != ref.tile_rows || P->key_block != ref.key_block || P->stages != ref.stages)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "plan tile_rows, key_block and stages are fixed by the kernels (" +
                                                     std::to_string(ref.tile_rows) + ", " +
                                                     std::to_string(ref.key_block) + ", " +
                                                     std::to_string(ref.stages) + ")");
  if ((P->rearm != 0 && P->rearm != 1) || (P->heavy_first != 0 && P->heavy_first != 1))
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "plan rearm and heavy_first must be 0 or 1");
  P->tiles = ref.tiles;
  if (P->split_k == 0) {
    P->tail_tiles = 0;
  } else {
    const int64_t blocks = (keys + piper::kKeyBlock - 1) / piper::kKeyBlock;
    if (causal) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "the split-KV tail applies to non-causal launches only");
    if (!split_region)
      return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "plan splits keys but the workspace has no split region");
    if (P->tiles >= (int64_t(1) << 30))
      return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "too many tiles for a split-KV tail");
    if (P->split_k < 2 || P->split_k > piper::kMaxSplits || P->split_k > blocks)
      return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "plan split_k must be 0 or in [2, min(" +
                                                       std::to_string(piper::kMaxSplits) + ", key blocks)]");
    if (P->tail_tiles <= 0 || P->tail_tiles > P->tiles || P->tail_tiles * P->split_k > split_units_max)
      return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "plan tail_tiles must be in [1, tiles] with tail_tiles * split_k <= " +
                                                       std::to_string(split_units_max));
  }
  P->ctas = P->tiles - P->tail_tiles + P->tail_tiles * P->split_k;
  P->kernels = P->split_k > 0 ? 2 : 1;
  return PIPER_B200_OK;
}

// The attention kernel instance the plan names (S re-arm with P in shared
// memory, or no re-arm with P in TMEM), then the split-KV merge if any.
template <typename T, int D>
void launch_piper_kernels(const dim3& grid, const dim3& merge_grid, bool rearm, const CUtensorMap& tmQ,
                          const CUtensorMap& tmK, const CUtensorMap& tmV, const piper::AttnParams& p,
                          cudaStream_t s) {
  if (rearm)
    piper::block64_attention_kernel<T, D, false>
        <<<grid, piper::kAttnThreads, piper::AttnSmem<D, true>::kAlloc, s>>>(tmQ, tmK, tmV, p);
  else
    piper::piper_attention_kernel<T, D><<<grid, piper::kAttnThreads, piper::PairSmem<D>::kAlloc, s>>>(tmQ, tmK, tmV, p);
  if (p.split_units)
    piper::merge_split_kernel<T, D><<<merge_grid, piper::kTileM * piper::kTiles, 0, s>>>(p);
}

// The attention launch shared by the one-shot and the sharded entry points:
// Q side (codes, scales, V mean) from `workspace`, K/V side from `kv_pack`
// (a K/V pack laid out as in the workspace of the same shape).  The workspace
// and pack are for (batch, heads, nq_all, nk_all, head_dim); the launch covers
// rows [q_row0, q_row0 + q_rows) and keys [key0, key0 + keys).
int run_attention(void* out, int dtype, int64_t batch, int64_t heads, int64_t nq_all, int64_t q_row0, int64_t q_rows,
                  int64_t nk_all, int64_t key0, int64_t keys, int64_t head_dim, double scale, int is_causal,
                  const void* workspace, size_t workspace_bytes, const void* kv_pack, int64_t causal_shift,
                  float* state, int state_mode, void* stream, bool sharded = false,
                  const piper_b200_plan_t* plan_in = nullptr) {
  // Sharded causal attention pairs independent query and key shards: only the
  // one-shard form needs Nq == Nk.
  int rc = check_shape(dtype, batch, heads, nq_all, nk_all, head_dim, sharded ? 0 : is_causal);
  if (rc != PIPER_B200_OK) return rc;
  if (q_row0 < 0 || q_rows <= 0 || q_row0 + q_rows > nq_all || key0 < 0 || keys <= 0 || key0 + keys > nk_all)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "row or key range outside the problem");
  if (q_row0 % piper::kKeyBlock != 0 || key0 % piper::kKeyBlock != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "row and key ranges must start at multiples of 64");
  if (!workspace || !kv_pack) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  if (!(state_mode & piper::kStateStore) && !out) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL output");
  if (state_mode != 0 && !state) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL state");
  if (!(std::isfinite(scale) && scale > 0.0))
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "scale must be finite and positive");
  if (out && reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "output must be 16-byte aligned");
  if (state && reinterpret_cast<uintptr_t>(state) % 16 != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(kv_pack) % 256 != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "K/V pack must be 256-byte aligned");
  int device = 0;
  if ((rc = ensure_device(&device)) != PIPER_B200_OK) return rc;
  const int64_t bh = batch * heads;
  const piper_b200_workspace_layout_t L = piper::make_layout(bh, nq_all, nk_all, head_dim);
  if (workspace_bytes < L.split_state)
    return fail(PIPER_B200_ERR_WORKSPACE_TOO_SMALL, "workspace too small for this problem");
  const uint8_t* ws = static_cast<const uint8_t*>(workspace);
  const uint8_t* kv = static_cast<const uint8_t*>(kv_pack) - L.kv_pack;  // same offsets as the workspace
  const uint64_t d = static_cast<uint64_t>(head_dim);
  CUtensorMap tmQ, tmK, tmV;
  if ((rc = encode_map(&tmQ, ws + L.q8, d, nq_all, bh, d, nq_all * d, static_cast<uint32_t>(d), piper::kTileM)) !=
      PIPER_B200_OK)
    return rc;
  if ((rc = encode_map(&tmK, kv + L.k8, d, nk_all, bh, d, nk_all * d, static_cast<uint32_t>(d), piper::kKeyBlock)) !=
      PIPER_B200_OK)
    return rc;
  // V codes are fp16: rows of nk_pad elements (2 bytes each).
  if ((rc = encode_map(&tmV, kv + L.v8t, L.nk_pad, d, bh, L.nk_pad * 2, L.nk_pad * d * 2, piper::kKeyBlock,
                       static_cast<uint32_t>(d), 2)) != PIPER_B200_OK)
    return rc;
  piper::AttnParams p{};
  p.qscale = reinterpret_cast<const float*>(ws + L.qscale);
  p.kscale = reinterpret_cast<const float*>(kv + L.kscale);
  p.vlog2 = reinterpret_cast<const float*>(kv + L.vlog2);
  p.vrcp = reinterpret_cast<const float*>(kv + L.vrcp);
  p.vmean = reinterpret_cast<const float*>(ws + L.vmean);
  p.out = out;
  p.heads = heads;
  p.nq = q_rows;
  p.nk = keys;
  p.nk_pad = L.nk_pad;
  p.q_groups = L.q_groups;
  p.k_groups = L.k_groups;
  p.scale_log2e = static_cast<float>(scale * 1.4426950408889634);
  p.causal = is_causal ? 1 : 0;
  p.q_tiles = static_cast<int>((q_rows + piper::kTileM * piper::kTiles - 1) / (piper::kTileM * piper::kTiles));
  p.wait_budget_ns = piper::kWaitBudgetNs;
  p.causal_shift = causal_shift;
  p.state_mode = state_mode;
  p.state_o = state;
  p.state_ml = state ? state + bh * nq_all * head_dim : nullptr;
  p.nq_all = nq_all;
  p.q_row0 = q_row0;
  p.k_key0 = key0;
  // Work units: every tile whole, except that the plan may cut the trailing
  // tiles into key ranges (split-KV tail) whose partial states
  // merge_split_kernel then combines (key range 0 starts from any carried
  // state).
  const int sms = g_device_sms[device] > 0 ? g_device_sms[device] : 148;
  const bool split_region = workspace_bytes >= L.total_bytes;
  piper_b200_plan_t plan;
  if (plan_in != nullptr) {
    plan = *plan_in;
    if ((rc = check_plan(&plan, bh, q_rows, keys, head_dim, is_causal != 0, split_region, L.split_units_max)) !=
        PIPER_B200_OK)
      return rc;
  } else {
    plan = make_plan(bh, q_rows, keys, head_dim, is_causal != 0, sms, split_region, L.split_units_max);
  }
  p.reverse_tiles = plan.heavy_first;
  p.bh_count = bh;
  const int64_t tiles = static_cast<int64_t>(p.q_tiles) * bh;
  p.main_units = tiles - plan.tail_tiles;
  p.splits = plan.split_k;
  p.split_units = plan.tail_tiles * plan.split_k;
  p.split_state = reinterpret_cast<float*>(const_cast<uint8_t*>(ws) + L.split_state);
  const int64_t units = p.main_units + p.split_units;
  const dim3 grid = units < (int64_t(1) << 31) ? dim3(static_cast<unsigned>(units), 1)
                                                : dim3(static_cast<unsigned>(p.q_tiles), static_cast<unsigned>(bh));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 merge_grid(static_cast<unsigned>(p.split_units > 0 ? p.split_units / p.splits : 0),
                        static_cast<unsigned>(head_dim / 8));
  if (dtype == PIPER_B200_FLOAT16) {
    if (head_dim == 64)
      launch_piper_kernels<__half, 64>(grid, merge_grid, plan.rearm != 0, tmQ, tmK, tmV, p, s);
    else
      launch_piper_kernels<__half, 128>(grid, merge_grid, plan.rearm != 0, tmQ, tmK, tmV, p, s);
  } else {
    if (head_dim == 64)
      launch_piper_kernels<__nv_bfloat16, 64>(grid, merge_grid, plan.rearm != 0, tmQ, tmK, tmV, p, s);
    else
      launch_piper_kernels<__nv_bfloat16, 128>(grid, merge_grid, plan.rearm != 0, tmQ, tmK, tmV, p, s);
  }
  PIPER_CUDA(cudaGetLastError());
  return PIPER_B200_OK;
}

}  // namespace

extern "C" {

int piper_b200_abi_version(void) { return 104; }

const char* piper_b200_last_error(void) { return g_last_error.c_str(); }

int piper_b200_supports_device(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return (prop.major == 10 && prop.minor == 0) ? 1 : 0;
}

int piper_b200_workspace_layout(int64_t batch, int64_t heads, int64_t query_length, int64_t key_length,
                                int64_t head_dim, piper_b200_workspace_layout_t* layout) {
  if (layout == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "layout is NULL");
  if (batch <= 0 || heads <= 0 || query_length <= 0 || key_length <= 0 || head_dim <= 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "sizes must be positive");
  *layout = piper::make_layout(batch * heads, query_length, key_length, head_dim);
  return PIPER_B200_OK;
}

int piper_b200_workspace_bytes(int64_t batch, int64_t heads, int64_t query_length, int64_t key_length,
                               int64_t head_dim, size_t* bytes) {
  piper_b200_workspace_layout_t L;
  const int rc = piper_b200_workspace_layout(batch, heads, query_length, key_length, head_dim, &L);
  if (rc != PIPER_B200_OK) return rc;
  if (bytes == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "bytes is NULL");
  *bytes = static_cast<size_t>(L.total_bytes);
  return PIPER_B200_OK;
}

int piper_b200_prepass(const void* query, const int64_t query_strides[3], const void* key,
                       const int64_t key_strides[3], const void* value, const int64_t value_strides[3], int dtype,
                       int64_t batch, int64_t heads, int64_t query_length, int64_t key_length, int64_t head_dim,
                       int is_causal, void* workspace, size_t workspace_bytes, void* stream) {
  return run_prepass(query, query_strides, key, key_strides, value, value_strides, dtype, batch, heads, query_length,
                     key_length, head_dim, is_causal, workspace, workspace_bytes, stream, kSums | kQuantize, 0,
                     key_length);
}

int piper_b200_attention_prepared(void* out, int dtype, int64_t batch, int64_t heads, int64_t query_length,
                                  int64_t key_length, int64_t head_dim, double scale, int is_causal,
                                  const void* workspace, size_t workspace_bytes, void* stream) {
  if (!out || !workspace) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  int rc = check_shape(dtype, batch, heads, query_length, key_length, head_dim, is_causal);
  if (rc != PIPER_B200_OK) return rc;
  const piper_b200_workspace_layout_t L = piper::make_layout(batch * heads, query_length, key_length, head_dim);
  return run_attention(out, dtype, batch, heads, query_length, 0, query_length, key_length, 0, key_length, head_dim,
                       scale, is_causal, workspace, workspace_bytes, static_cast<const uint8_t*>(workspace) + L.kv_pack,
                       0, nullptr, 0, stream);
}

int piper_b200_select_plan(int64_t batch, int64_t heads, int64_t query_length, int64_t key_length,
                           int64_t head_dim, int is_causal, int sms, int split_region, piper_b200_plan_t* plan) {
  if (plan == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (batch <= 0 || heads <= 0 || query_length <= 0 || key_length <= 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "sizes must be positive");
  if (head_dim != 64 && head_dim != 128)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "head_dim must be 64 or 128, got " + std::to_string(head_dim));
  if (sms < 0) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "sms must be non-negative");
  if (sms == 0) {
    int device = 0;
    sms = 148;
    if (cudaGetDevice(&device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
      cudaGetLastError();
      sms = 148;
    }
  }
  const piper_b200_workspace_layout_t L = piper::make_layout(batch * heads, query_length, key_length, head_dim);
  *plan = make_plan(batch * heads, query_length, key_length, head_dim, is_causal != 0, sms, split_region != 0,
                    L.split_units_max);
  return PIPER_B200_OK;
}

int piper_b200_attention_prepared_plan(void* out, int dtype, int64_t batch, int64_t heads, int64_t query_length,
                                       int64_t key_length, int64_t head_dim, double scale, int is_causal,
                                       const void* workspace, size_t workspace_bytes, const piper_b200_plan_t* plan,
                                       void* stream) {
  if (!out || !workspace || !plan) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  int rc = check_shape(dtype, batch, heads, query_length, key_length, head_dim, is_causal);
  if (rc != PIPER_B200_OK) return rc;
  const piper_b200_workspace_layout_t L = piper::make_layout(batch * heads, query_length, key_length, head_dim);
  return run_attention(out, dtype, batch, heads, query_length, 0, query_length, key_length, 0, key_length, head_dim,
                       scale, is_causal, workspace, workspace_bytes, static_cast<const uint8_t*>(workspace) + L.kv_pack,
                       0, nullptr, 0, stream, false, plan);
}

int piper_b200_shard_column_sums(const void* key, const int64_t key_strides[3], const void* value,
                                 const int64_t value_strides[3], int dtype, int64_t batch, int64_t heads,
                                 int64_t query_length, int64_t key_length, int64_t head_dim, int is_causal,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  return run_prepass(nullptr, nullptr, key, key_strides, value, value_strides, dtype, batch, heads, query_length,
                     key_length, head_dim, is_causal, workspace, workspace_bytes, stream, kSums, 1, key_length);
}

int piper_b200_shard_prepass(const void* query, const int64_t query_strides[3], const void* key,
                             const int64_t key_strides[3], const void* value, const int64_t value_strides[3],
                             int dtype, int64_t batch, int64_t heads, int64_t query_length, int64_t key_length,
                             int64_t head_dim, int is_causal, int64_t total_keys, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (total_keys < key_length)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "total_keys must be at least this shard's key length");
  return run_prepass(query, query_strides, key, key_strides, value, value_strides, dtype, batch, heads,
                     query_length, key_length, head_dim, is_causal, workspace, workspace_bytes, stream,
                     kFinalize | kQuantize, 0, total_keys);
}

int piper_b200_attention_shard_range(void* out, int dtype, int64_t batch, int64_t heads, int64_t query_length,
                                     int64_t query_begin, int64_t query_count, int64_t key_length,
                                     int64_t key_begin, int64_t key_count, int64_t head_dim, double scale,
                                     int is_causal, int64_t causal_shift, const void* workspace,
                                     size_t workspace_bytes, const void* kv_pack, float* state, int state_mode,
                                     void* stream) {
  if (state_mode < 0 || state_mode > (PIPER_B200_STATE_LOAD | PIPER_B200_STATE_STORE))
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "state_mode must combine PIPER_B200_STATE_LOAD/STORE");
  if (!is_causal && causal_shift != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "causal_shift applies to causal attention only");
  if (is_causal && (causal_shift < -(int64_t(1) << 40) || causal_shift > (int64_t(1) << 40)))
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "causal_shift out of range");
  return run_attention(out, dtype, batch, heads, query_length, query_begin, query_count, key_length, key_begin,
                       key_count, head_dim, scale, is_causal, workspace, workspace_bytes, kv_pack, causal_shift, state,
                       state_mode, stream, true);
}

int piper_b200_attention_shard(void* out, int dtype, int64_t batch, int64_t heads, int64_t query_length,
                               int64_t key_length, int64_t head_dim, double scale, int is_causal,
                               int64_t causal_shift, const void* workspace, size_t workspace_bytes,
                               const void* kv_pack, float* state, int state_mode, void* stream) {
  return piper_b200_attention_shard_range(out, dtype, batch, heads, query_length, 0, query_length, key_length, 0,
                                          key_length, head_dim, scale, is_causal, causal_shift, workspace,
                                          workspace_bytes, kv_pack, state, state_mode, stream);
}

size_t piper_b200_state_bytes(int64_t batch, int64_t heads, int64_t query_length, int64_t head_dim) {
  if (batch <= 0 || heads <= 0 || query_length <= 0 || head_dim <= 0) return 0;
  return static_cast<size_t>(batch * heads * query_length * (head_dim + 2) * 4);
}

int piper_b200_attention_fwd(const void* query, const int64_t query_strides[3], const void* key,
                             const int64_t key_strides[3], const void* value, const int64_t value_strides[3],
                             void* out, int dtype, int64_t batch, int64_t heads, int64_t query_length,
                             int64_t key_length, int64_t head_dim, double scale, int is_causal, void* workspace,
                             size_t workspace_bytes, void* stream) {
  int rc = piper_b200_prepass(query, query_strides, key, key_strides, value, value_strides, dtype, batch, heads,
                              query_length, key_length, head_dim, is_causal, workspace, workspace_bytes, stream);
  if (rc != PIPER_B200_OK) return rc;
  return piper_b200_attention_prepared(out, dtype, batch, heads, query_length, key_length, head_dim, scale,
                                       is_causal, workspace, workspace_bytes, stream);
}

int piper_b200_device_status(int device, int clear, uint32_t* status) {
  if (status == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "status is NULL");
  int prev = 0;
  PIPER_CUDA(cudaGetDevice(&prev));
  PIPER_CUDA(cudaSetDevice(device));
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, piper::g_piper_status, sizeof(uint32_t));
  if (e == cudaSuccess && clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(piper::g_piper_status, &zero, sizeof(uint32_t));
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device status word");
  return PIPER_B200_OK;
}

int piper_b200_selftest_wait_timeout(uint64_t budget_ns, int* timed_out, void* stream) {
  if (timed_out == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "timed_out is NULL");
  if (budget_ns > 10ull * 1000 * 1000 * 1000) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "budget above 10 s");
  int device = 0;
  int rc = ensure_device(&device);
  if (rc != PIPER_B200_OK) return rc;
  int* d_flag = nullptr;
  uint32_t* d_status = nullptr;
  PIPER_CUDA(cudaMalloc(&d_flag, sizeof(int)));
  cudaError_t e = cudaMalloc(&d_status, sizeof(uint32_t));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d_flag, 0xff, sizeof(int), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(d_status, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess) {
    piper::selftest_wait_kernel<<<1, 32, 0, s>>>(budget_ns, d_flag, d_status);
    e = cudaGetLastError();
  }
  int host_flag = -1;
  uint32_t host_status = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host_flag, d_flag, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host_status, d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(d_flag);
  if (d_status) cudaFree(d_status);
  if (e != cudaSuccess) return cuda_fail(e, "wait-timeout self-test");
  *timed_out = (host_flag == 1 && (host_status & piper::kStatusTimeoutProbe)) ? 1 : 0;
  return PIPER_B200_OK;
}

int piper_b200_selftest_exp2(const float* x, float* y, float* ex2, int64_t n, void* stream) {
  if (n < 0 || n > (int64_t(1) << 31)) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "n must be in [0, 2^31]");
  if (n == 0) return PIPER_B200_OK;
  if (x == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "x is NULL");
  int device = 0;
  int rc = ensure_device(&device);
  if (rc != PIPER_B200_OK) return rc;
  const int64_t pairs = (n + 1) / 2;
  piper::selftest_exp2_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, y, ex2, n);
  PIPER_CUDA(cudaGetLastError());
  return PIPER_B200_OK;
}

int piper_b200_selftest_gemm_i8(const void* a, const void* b, int32_t* c, int64_t m, int64_t n, int64_t k,
                                int a_signed, void* stream) {
  if (!a || !b || !c) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  if (m <= 0 || n <= 0 || k <= 0 || m % 128 || n % 64 || k % 128)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "need M%128 == 0, N%64 == 0, K%128 == 0");
  int device = 0;
  int rc = ensure_device(&device);
  if (rc != PIPER_B200_OK) return rc;
  CUtensorMap tmA, tmB;
  if ((rc = encode_map(&tmA, a, k, m, 1, k, m * k, 128, 128)) != PIPER_B200_OK) return rc;
  if ((rc = encode_map(&tmB, b, k, n, 1, k, n * k, 128, 64)) != PIPER_B200_OK) return rc;
  const dim3 grid(static_cast<unsigned>(m / 128), static_cast<unsigned>(n / 64));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a_signed)
    piper::selftest_gemm_kernel<true><<<grid, 128, 0, s>>>(tmA, tmB, c, n, k, piper::kWaitBudgetNs);
  else
    piper::selftest_gemm_kernel<false><<<grid, 128, 0, s>>>(tmA, tmB, c, n, k, piper::kWaitBudgetNs);
  PIPER_CUDA(cudaGetLastError());
  return PIPER_B200_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Forward pass without any device allocation (piper_b200_attention_fwd_no_alloc).
//
// For callers that cannot allocate device memory: the scratch lives in this
// fixed file-scope array instead of a caller-provided workspace.  Host code
// must not hand the array's name to a kernel (on the host it is only a
// stand-in symbol); the device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, and passed down as an
// ordinary pointer.  The existing forward path then runs unchanged on it;
// that path already clears the only region that must start at zero (the
// mean-pass counters) on every call, so leftovers of an earlier call on the
// shared array do no harm.  Calls that overlap on the GPU share the array and
// race.
namespace {

static __device__ __align__(256) uint8_t g_no_alloc_workspace[PIPER_B200_NO_ALLOC_WORKSPACE_BYTES];

void* g_no_alloc_address[kMaxDevices] = {};
unsigned long long g_no_alloc_context[kMaxDevices] = {};  // context the address belongs to

// The array's device address in the current context of `device` (which
// ensure_device made current).  Looked up once per context: a reset device
// gets a new context, a new copy of the array and so a new address.
int no_alloc_workspace(int device, void** ptr) {
  std::lock_guard<std::mutex> lock(g_init_mutex);
  const unsigned long long context = current_context_id();
  if (g_no_alloc_address[device] == nullptr || context == 0 || g_no_alloc_context[device] != context) {
    void* address = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&address, g_no_alloc_workspace);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc workspace)");
    if (address == nullptr || reinterpret_cast<uintptr_t>(address) % 256 != 0)
      return fail(PIPER_B200_ERR_CUDA, "no-alloc workspace has no usable device address");
    g_no_alloc_address[device] = address;
    g_no_alloc_context[device] = context;
  }
  *ptr = g_no_alloc_address[device];
  return PIPER_B200_OK;
}

}  // namespace

extern "C" int piper_b200_attention_fwd_no_alloc(const void* query, const int64_t query_strides[3], const void* key,
                                                 const int64_t key_strides[3], const void* value,
                                                 const int64_t value_strides[3], void* out, int dtype, int64_t batch,
                                                 int64_t heads, int64_t query_length, int64_t key_length,
                                                 int64_t head_dim, double scale, int is_causal, void* stream) {
  int rc = check_shape(dtype, batch, heads, query_length, key_length, head_dim, is_causal);
  if (rc != PIPER_B200_OK) return rc;
  const piper_b200_workspace_layout_t L = piper::make_layout(batch * heads, query_length, key_length, head_dim);
  if (L.split_state > PIPER_B200_NO_ALLOC_WORKSPACE_BYTES)
    return fail(PIPER_B200_ERR_WORKSPACE_TOO_SMALL,
                "this problem needs " + std::to_string(L.split_state) +
                    " bytes of scratch; piper_b200_attention_fwd_no_alloc holds at most " +
                    std::to_string(PIPER_B200_NO_ALLOC_WORKSPACE_BYTES) +
                    " bytes (use piper_b200_attention_fwd with a caller-provided workspace)");
  int device = 0;
  if ((rc = ensure_device(&device)) != PIPER_B200_OK) return rc;
  void* workspace = nullptr;
  if ((rc = no_alloc_workspace(device, &workspace)) != PIPER_B200_OK) return rc;
  return piper_b200_attention_fwd(query, query_strides, key, key_strides, value, value_strides, out, dtype, batch,
                                  heads, query_length, key_length, head_dim, scale, is_causal, workspace,
                                  PIPER_B200_NO_ALLOC_WORKSPACE_BYTES, stream);
}

// ---------------------------------------------------------------------------
// Host-to-host forward pass (piper_b200_attention_fwd_host).
//
// The heads are split into chunks; each chunk goes through a ring of
// kHostSlots device slots: H2D copy of its Q/K/V on a copy stream, prepass +
// attention on one of two compute streams (the caller's and an internal one,
// alternating, so one chunk's kernels fill the SMs the other's wave tail
// leaves idle), D2H copy of its output on a second copy stream.  Copies in
// both directions overlap the kernels of other chunks, so the call takes
// about max(H2D, compute, D2H) instead of their sum.
namespace {

constexpr int kHostSlots = 4;

constexpr int kMaxHostChunks = 4096;

struct HostPlan {
  int64_t heads_per_slot = 0, chunks = 0;
  int64_t chunk_h0[kMaxHostChunks], chunk_heads[kMaxHostChunks];
  uint64_t q_bytes = 0, kv_bytes = 0, out_bytes = 0, ws_bytes = 0;  // per slot (heads_per_slot heads)
  uint64_t slot_bytes = 0, total_bytes = 0;
  uint64_t off_q = 0, off_k = 0, off_v = 0, off_out = 0, off_ws = 0;
};

// The heads are cut into chunks: a first chunk of at most one wave of CTAs
// (the kernels start as soon as it has landed), then chunks of `hc` heads,
// and the remainder in one-wave chunks (everything after the final
// host-to-device copy -- the last chunk's kernels and its copy back -- stays
// short).  `hc` holds about kHostChunkBytes of inputs, about a millisecond of
// PCIe traffic (measured best on B200 for B1 H40 N16384 and B4 H32 N8192),
// at most 16 heads and at most a third of them so that copies and kernels
// overlap.
constexpr double kHostChunkBytes = 52e6;

// At most kMaxTailChunks chunks carry the remainder after the bulk chunks.
constexpr int64_t kMaxTailChunks = 16;

void make_host_plan(int64_t bh, int64_t nq, int64_t nk, int64_t d, int sms, HostPlan* P) {
  const int64_t q_tiles = (nq + piper::kTileM * piper::kTiles - 1) / (piper::kTileM * piper::kTiles);
  const double head_bytes = static_cast<double>((nq + 2 * nk) * d * 2);
  const int64_t max_hc = std::max<int64_t>(1, std::min<int64_t>(16, bh / 3));
  int64_t hc = std::max<int64_t>(1, std::min<int64_t>(max_hc, std::llround(kHostChunkBytes / head_bytes)));
  // The chunk count is bounded: one first chunk, at most
  // kMaxHostChunks - 1 - kMaxTailChunks bulk chunks, at most kMaxTailChunks
  // remainder chunks.
  hc = std::max<int64_t>(hc, (bh + kMaxHostChunks - 2 - kMaxTailChunks) / (kMaxHostChunks - 1 - kMaxTailChunks));
  const int64_t per_wave = std::max<int64_t>(1, std::min<int64_t>(hc, sms / std::max<int64_t>(q_tiles, 1)));
  int64_t n = 0, h = 0;
  auto add = [&](int64_t heads) {
    if (n >= kMaxHostChunks) return;  // unreachable with the bounds above; never write past the arrays
    P->chunk_h0[n] = h;
    P->chunk_heads[n++] = heads;
    h += heads;
  };
  add(std::min<int64_t>(per_wave, bh));
  while (bh - h > hc) add(hc);
  // The remainder (at most hc heads) in one-wave chunks, or in
  // kMaxTailChunks equal chunks when one-wave chunks would be more.
  const int64_t tail_chunk = std::max<int64_t>(per_wave, (bh - h + kMaxTailChunks - 1) / kMaxTailChunks);
  while (h < bh && n < kMaxHostChunks) add(std::min<int64_t>(tail_chunk, bh - h));
  P->chunks = n;
  P->heads_per_slot = hc;
  P->q_bytes = static_cast<uint64_t>(hc * nq * d) * 2;
  P->kv_bytes = static_cast<uint64_t>(hc * nk * d) * 2;
  P->out_bytes = P->q_bytes;
  P->ws_bytes = piper::make_layout(hc, nq, nk, d).total_bytes;
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    const uint64_t at = off;
    off = piper::align_up(off + bytes, 256);
    return at;
  };
  P->off_q = take(P->q_bytes);
  P->off_k = take(P->kv_bytes);
  P->off_v = take(P->kv_bytes);
  P->off_out = take(P->out_bytes);
  P->off_ws = take(P->ws_bytes);
  P->slot_bytes = off;
  P->total_bytes = P->slot_bytes * kHostSlots;
}

struct HostStreams {
  bool ready = false;
  unsigned long long context = 0;  // the context the streams and events belong to
  cudaStream_t h2d = nullptr, d2h = nullptr, compute = nullptr;
  cudaEvent_t start = nullptr;
  cudaEvent_t loaded[kHostSlots] = {}, computed[kHostSlots] = {}, drained[kHostSlots] = {};
  std::mutex enqueue;  // one call at a time enqueues on the shared copy streams
};
HostStreams g_host[kMaxDevices];

int host_streams(int device, HostStreams** out) {
  std::lock_guard<std::mutex> lock(g_init_mutex);
  HostStreams& h = g_host[device];
  // Streams and events die with their context (a device reset): make new ones then.
  const unsigned long long context = current_context_id();
  if (!h.ready || context == 0 || h.context != context) {
    h.ready = false;
    PIPER_CUDA(cudaStreamCreateWithFlags(&h.h2d, cudaStreamNonBlocking));
    PIPER_CUDA(cudaStreamCreateWithFlags(&h.d2h, cudaStreamNonBlocking));
    PIPER_CUDA(cudaStreamCreateWithFlags(&h.compute, cudaStreamNonBlocking));
    PIPER_CUDA(cudaEventCreateWithFlags(&h.start, cudaEventDisableTiming));
    for (int i = 0; i < kHostSlots; ++i) {
      PIPER_CUDA(cudaEventCreateWithFlags(&h.loaded[i], cudaEventDisableTiming));
      PIPER_CUDA(cudaEventCreateWithFlags(&h.computed[i], cudaEventDisableTiming));
      PIPER_CUDA(cudaEventCreateWithFlags(&h.drained[i], cudaEventDisableTiming));
    }
    h.ready = true;
    h.context = context;
  }
  *out = &h;
  return PIPER_B200_OK;
}

int sm_count(int device, int* sms) {
  PIPER_CUDA(cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, device));
  return PIPER_B200_OK;
}

}  // namespace

extern "C" int piper_b200_host_scratch_bytes(int64_t batch, int64_t heads, int64_t query_length,
                                             int64_t key_length, int64_t head_dim, size_t* bytes) {
  if (bytes == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (batch <= 0 || heads <= 0 || query_length <= 0 || key_length <= 0 || head_dim <= 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "sizes must be positive");
  // The chunking depends on the SM count of the current device (148 on a
  // B200, also assumed when no device is visible).
  int device = 0, sms = 148;
  if (cudaGetDevice(&device) != cudaSuccess || sm_count(device, &sms) != PIPER_B200_OK) {
    cudaGetLastError();
    sms = 148;
  }
  HostPlan* plan = new HostPlan;
  make_host_plan(batch * heads, query_length, key_length, head_dim, sms, plan);
  *bytes = static_cast<size_t>(plan->total_bytes);
  delete plan;
  return PIPER_B200_OK;
}

extern "C" int piper_b200_attention_fwd_host(const void* query, const void* key, const void* value, void* out,
                                             int dtype, int64_t batch, int64_t heads, int64_t query_length,
                                             int64_t key_length, int64_t head_dim, double scale, int is_causal,
                                             void* scratch, size_t scratch_bytes, void* stream) {
  int rc = check_shape(dtype, batch, heads, query_length, key_length, head_dim, is_causal);
  if (rc != PIPER_B200_OK) return rc;
  if (!query || !key || !value || !out || !scratch) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  if (!(std::isfinite(scale) && scale > 0.0))
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "scale must be finite and positive");
  if (reinterpret_cast<uintptr_t>(scratch) % 256 != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "scratch must be 256-byte aligned");
  int device = 0;
  if ((rc = ensure_device(&device)) != PIPER_B200_OK) return rc;
  int sms = 148;
  if ((rc = sm_count(device, &sms)) != PIPER_B200_OK) return rc;
  const int64_t bh = batch * heads;
  static thread_local HostPlan plan_storage;  // ~64 KB: kept off the stack
  HostPlan& P = plan_storage;
  make_host_plan(bh, query_length, key_length, head_dim, sms, &P);
  if (scratch_bytes < P.total_bytes)
    return fail(PIPER_B200_ERR_WORKSPACE_TOO_SMALL, "scratch needs " + std::to_string(P.total_bytes) + " bytes, got " +
                                                         std::to_string(scratch_bytes));
  HostStreams* hs = nullptr;
  if ((rc = host_streams(device, &hs)) != PIPER_B200_OK) return rc;
  std::lock_guard<std::mutex> lock(hs->enqueue);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  const uint8_t* hq = static_cast<const uint8_t*>(query);
  const uint8_t* hk = static_cast<const uint8_t*>(key);
  const uint8_t* hv = static_cast<const uint8_t*>(value);
  uint8_t* ho = static_cast<uint8_t*>(out);
  const uint64_t q_head = static_cast<uint64_t>(query_length * head_dim) * 2;
  const uint64_t kv_head = static_cast<uint64_t>(key_length * head_dim) * 2;
  // Nothing of this call may start before the caller's earlier work.
  PIPER_CUDA(cudaEventRecord(hs->start, s));
  PIPER_CUDA(cudaStreamWaitEvent(hs->h2d, hs->start, 0));
  PIPER_CUDA(cudaStreamWaitEvent(hs->d2h, hs->start, 0));
  PIPER_CUDA(cudaStreamWaitEvent(hs->compute, hs->start, 0));
  for (int64_t c = 0; c < P.chunks; ++c) {
    const int slot = static_cast<int>(c % kHostSlots);
    const int64_t h0 = P.chunk_h0[c];
    const int64_t hc = P.chunk_heads[c];
    uint8_t* sb = base + slot * P.slot_bytes;
    // H2D into the slot once its previous chunk's output has been copied out.
    if (c >= kHostSlots) PIPER_CUDA(cudaStreamWaitEvent(hs->h2d, hs->drained[slot], 0));
    PIPER_CUDA(cudaMemcpyAsync(sb + P.off_q, hq + h0 * q_head, hc * q_head, cudaMemcpyHostToDevice, hs->h2d));
    PIPER_CUDA(cudaMemcpyAsync(sb + P.off_k, hk + h0 * kv_head, hc * kv_head, cudaMemcpyHostToDevice, hs->h2d));
    PIPER_CUDA(cudaMemcpyAsync(sb + P.off_v, hv + h0 * kv_head, hc * kv_head, cudaMemcpyHostToDevice, hs->h2d));
    PIPER_CUDA(cudaEventRecord(hs->loaded[slot], hs->h2d));
    // Kernels on the caller's stream or the internal compute stream (the
    // chunk is a [1, hc, N, D] problem).
    cudaStream_t cs = (c & 1) ? hs->compute : s;
    PIPER_CUDA(cudaStreamWaitEvent(cs, hs->loaded[slot], 0));
    const int64_t qs[3] = {hc * query_length * head_dim, query_length * head_dim, head_dim};
    const int64_t ks[3] = {hc * key_length * head_dim, key_length * head_dim, head_dim};
    const uint64_t ws_bytes = piper::make_layout(hc, query_length, key_length, head_dim).total_bytes;
    rc = piper_b200_attention_fwd(sb + P.off_q, qs, sb + P.off_k, ks, sb + P.off_v, ks, sb + P.off_out, dtype, 1, hc,
                                  query_length, key_length, head_dim, scale, is_causal, sb + P.off_ws, ws_bytes, cs);
    if (rc != PIPER_B200_OK) return rc;
    PIPER_CUDA(cudaEventRecord(hs->computed[slot], cs));
    // D2H of the chunk's output.
    PIPER_CUDA(cudaStreamWaitEvent(hs->d2h, hs->computed[slot], 0));
    PIPER_CUDA(cudaMemcpyAsync(ho + h0 * q_head, sb + P.off_out, hc * q_head, cudaMemcpyDeviceToHost, hs->d2h));
    PIPER_CUDA(cudaEventRecord(hs->drained[slot], hs->d2h));
  }
  // The caller's stream completes when the last output bytes have landed
  // (which follows every chunk's kernels, on either compute stream).
  const int last = static_cast<int>((P.chunks - 1) % kHostSlots);
  PIPER_CUDA(cudaStreamWaitEvent(s, hs->drained[last], 0));
  return PIPER_B200_OK;
}

// ---------------------------------------------------------------------------
// SageAttention2++ (8+8): prepass and attention launches.
namespace {

template <typename T, int D, bool V16>
void launch_sage_prepass_t(const piper::SagePrepassArgs& a, int64_t bh, cudaStream_t stream) {
  const dim3 stats_grid(static_cast<unsigned>(a.L.chunks), static_cast<unsigned>(bh));
  piper::sage_stats_kernel<T, D, V16><<<stats_grid, piper::kPrepassThreads, 0, stream>>>(a);
  const int64_t tiles = (std::max(a.nq, a.nk) + piper::kKeyBlock - 1) / piper::kKeyBlock;
  const dim3 q_grid(static_cast<unsigned>(tiles), static_cast<unsigned>(bh));
  piper::sage_quantize_kernel<T, D, V16><<<q_grid, piper::kPrepassThreads, 0, stream>>>(a);
}

template <typename T, int D>
void launch_sage_prepass_d(const piper::SagePrepassArgs& a, int64_t bh, bool v16, cudaStream_t stream) {
  if (v16)
    launch_sage_prepass_t<T, D, true>(a, bh, stream);
  else
    launch_sage_prepass_t<T, D, false>(a, bh, stream);
}

}  // namespace

extern "C" int piper_b200_sage2pp_layout(int64_t batch, int64_t heads, int64_t query_length, int64_t key_length,
                                         int64_t head_dim, piper_b200_sage2pp_layout_t* layout) {
  if (layout == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "layout is NULL");
  if (batch <= 0 || heads <= 0 || query_length <= 0 || key_length <= 0 || head_dim <= 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "sizes must be positive");
  *layout = piper::make_sage_layout(batch * heads, query_length, key_length, head_dim);
  return PIPER_B200_OK;
}

extern "C" int piper_b200_sage2pp_workspace_bytes(int64_t batch, int64_t heads, int64_t query_length,
                                                  int64_t key_length, int64_t head_dim, size_t* bytes) {
  piper_b200_sage2pp_layout_t L;
  const int rc = piper_b200_sage2pp_layout(batch, heads, query_length, key_length, head_dim, &L);
  if (rc != PIPER_B200_OK) return rc;
  if (bytes == nullptr) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "bytes is NULL");
  *bytes = static_cast<size_t>(L.total_bytes);
  return PIPER_B200_OK;
}

extern "C" int piper_b200_sage2pp_prepass(const void* query, const int64_t query_strides[3], const void* key,
                                          const int64_t key_strides[3], const void* value,
                                          const int64_t value_strides[3], int dtype, int64_t batch, int64_t heads,
                                          int64_t query_length, int64_t key_length, int64_t head_dim,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_shape(dtype, batch, heads, query_length, key_length, head_dim, 0);
  if (rc != PIPER_B200_OK) return rc;
  if (!query || !key || !value || !workspace || !query_strides || !key_strides || !value_strides)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  int device = 0;
  if ((rc = ensure_device(&device)) != PIPER_B200_OK) return rc;
  const int64_t bh = batch * heads;
  const piper_b200_sage2pp_layout_t L = piper::make_sage_layout(bh, query_length, key_length, head_dim);
  if (workspace_bytes < L.total_bytes)
    return fail(PIPER_B200_ERR_WORKSPACE_TOO_SMALL,
                "workspace needs " + std::to_string(L.total_bytes) + " bytes, got " + std::to_string(workspace_bytes));
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  piper::SagePrepassArgs a{};
  a.q = query;
  a.k = key;
  a.v = value;
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = query_strides[i];
    a.ks[i] = key_strides[i];
    a.vs[i] = value_strides[i];
  }
  a.heads = heads;
  a.nq = query_length;
  a.nk = key_length;
  a.ws = static_cast<uint8_t*>(workspace);
  a.L = L;
  const bool v16 = aligned16(query, query_strides) && aligned16(key, key_strides) && aligned16(value, value_strides);
  PIPER_CUDA(cudaMemsetAsync(a.ws + L.counter, 0, static_cast<size_t>(bh) * 4, s));
  if (dtype == PIPER_B200_FLOAT16) {
    if (head_dim == 64)
      launch_sage_prepass_d<__half, 64>(a, bh, v16, s);
    else
      launch_sage_prepass_d<__half, 128>(a, bh, v16, s);
  } else {
    if (head_dim == 64)
      launch_sage_prepass_d<__nv_bfloat16, 64>(a, bh, v16, s);
    else
      launch_sage_prepass_d<__nv_bfloat16, 128>(a, bh, v16, s);
  }
  PIPER_CUDA(cudaGetLastError());
  return PIPER_B200_OK;
}

extern "C" int piper_b200_sage2pp_attention_prepared(void* out, int dtype, int64_t batch, int64_t heads,
                                                     int64_t query_length, int64_t key_length, int64_t head_dim,
                                                     double scale, int is_causal, const void* workspace,
                                                     size_t workspace_bytes, void* stream) {
  int rc = check_shape(dtype, batch, heads, query_length, key_length, head_dim, is_causal);
  if (rc != PIPER_B200_OK) return rc;
  if (!out || !workspace) return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "NULL pointer argument");
  if (!(std::isfinite(scale) && scale > 0.0))
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "scale must be finite and positive");
  if (reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return fail(PIPER_B200_ERR_INVALID_ARGUMENT, "output must be 16-byte aligned");
  int device = 0;
  if ((rc = ensure_device(&device)) != PIPER_B200_OK) return rc;
  const int64_t bh = batch * heads;
  const piper_b200_sage2pp_layout_t L = piper::make_sage_layout(bh, query_length, key_length, head_dim);
  if (workspace_bytes < L.total_bytes) return fail(PIPER_B200_ERR_WORKSPACE_TOO_SMALL, "workspace too small");
  const uint8_t* ws = static_cast<const uint8_t*>(workspace);
  const uint64_t d = static_cast<uint64_t>(head_dim);
  CUtensorMap tmQ, tmK, tmV;
  if ((rc = encode_map(&tmQ, ws + L.q8, d, query_length, bh, d, query_length * d, static_cast<uint32_t>(d),
                       piper::kTileM)) != PIPER_B200_OK)
    return rc;
  if ((rc = encode_map(&tmK, ws + L.k8, d, key_length, bh, d, key_length * d, static_cast<uint32_t>(d),
                       piper::kKeyBlock)) != PIPER_B200_OK)
    return rc;
  if ((rc = encode_map(&tmV, ws + L.v8t, L.nk_pad, d, bh, L.nk_pad, L.nk_pad * d, piper::kKeyBlock,
                       static_cast<uint32_t>(d))) != PIPER_B200_OK)
    return rc;
  piper::AttnParams p{};
  p.qscale = reinterpret_cast<const float*>(ws + L.qscale);  // per query row
  p.vlog2 = reinterpret_cast<const float*>(ws + L.kmask);    // per-key vector slot 0: padded-key mask
  p.vrcp = reinterpret_cast<const float*>(ws + L.kscale);    // per-key vector slot 1: K scale
  p.vmean = reinterpret_cast<const float*>(ws + L.vscale);   // per-channel V scale
  p.out = out;
  p.heads = heads;
  p.nq = query_length;
  p.nk = key_length;
  p.nk_pad = L.nk_pad;
  p.scale_log2e = static_cast<float>(scale * 1.4426950408889634);
  p.causal = is_causal ? 1 : 0;
  p.reverse_tiles = p.causal;
  p.bh_count = bh;
  p.q_tiles = static_cast<int>((query_length + piper::kTileM * piper::kTiles - 1) / (piper::kTileM * piper::kTiles));
  p.wait_budget_ns = piper::kWaitBudgetNs;
  p.nq_all = query_length;
  p.main_units = static_cast<int64_t>(p.q_tiles) * bh;
  const int64_t units = p.main_units;
  const dim3 grid = units < (int64_t(1) << 31) ? dim3(static_cast<unsigned>(units), 1)
                                                : dim3(static_cast<unsigned>(p.q_tiles), static_cast<unsigned>(bh));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PIPER_B200_FLOAT16) {
    if (head_dim == 64)
      piper::block64_attention_kernel<__half, 64, true><<<grid, piper::kAttnThreads, piper::AttnSmem<64>::kAlloc, s>>>(tmQ, tmK, tmV, p);
    else
      piper::block64_attention_kernel<__half, 128, true><<<grid, piper::kAttnThreads, piper::AttnSmem<128>::kAlloc, s>>>(tmQ, tmK, tmV, p);
  } else {
    if (head_dim == 64)
      piper::block64_attention_kernel<__nv_bfloat16, 64, true><<<grid, piper::kAttnThreads, piper::AttnSmem<64>::kAlloc, s>>>(tmQ, tmK, tmV, p);
    else
      piper::block64_attention_kernel<__nv_bfloat16, 128, true><<<grid, piper::kAttnThreads, piper::AttnSmem<128>::kAlloc, s>>>(tmQ, tmK, tmV, p);
  }
  PIPER_CUDA(cudaGetLastError());
  return PIPER_B200_OK;
}

extern "C" int piper_b200_sage2pp_fwd(const void* query, const int64_t query_strides[3], const void* key,
                                      const int64_t key_strides[3], const void* value, const int64_t value_strides[3],
                                      void* out, int dtype, int64_t batch, int64_t heads, int64_t query_length,
                                      int64_t key_length, int64_t head_dim, double scale, int is_causal,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_shape(dtype, batch, heads, query_length, key_length, head_dim, is_causal);
  if (rc != PIPER_B200_OK) return rc;
  rc = piper_b200_sage2pp_prepass(query, query_strides, key, key_strides, value, value_strides, dtype, batch, heads,
                                  query_length, key_length, head_dim, workspace, workspace_bytes, stream);
  if (rc != PIPER_B200_OK) return rc;
  return piper_b200_sage2pp_attention_prepared(out, dtype, batch, heads, query_length, key_length, head_dim, scale,
                                               is_causal, workspace, workspace_bytes, stream);
}
