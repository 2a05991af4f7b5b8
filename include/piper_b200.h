/*
 * piper_b200 -- C ABI of the B200 (sm_100a) backend of Piper Attention.
 *
 * This is the boundary the Python operator binds (through ctypes) and that
 * any other host language can bind the same way.  Signatures use only plain
 * pointers, integers and sizes: no torch, no C++ types.  No C++ exception
 * crosses it; every entry point returns a piper_b200_status and, on failure,
 * records a message readable with piper_b200_last_error().
 *
 * Reference interfaces replaced (Piper Kernels 0.2.1, paths inside the
 * project):
 *   piper_b200_attention_fwd       <- torch.ops.piper_kernels.piper_attention
 *                                     src/piper_kernels/attention/piper_attention/triton.py:984-999
 *                                     (== _run_piper_attention, triton.py:954-981)
 *   piper_b200_prepass             <- _prepare_piper_attention, triton.py:772-890
 *                                     (_compute_kv_means 638-699, prepare_query/prepare_key
 *                                     qk_quantization/int8/sage/triton.py:238-356,
 *                                     _quantize_value_per_key_kernel triton.py:176-246)
 *   piper_b200_attention_prepared  <- _launch_piper_attention, triton.py:893-951
 *   piper_b200_workspace_bytes /
 *   piper_b200_workspace_layout    <- the per-call torch allocations of triton.py:814-838, 874
 *                                     (the caller owns the memory here)
 *   piper_b200_supports_device     <- AcceleratorTarget.supports_uint8_int8_mma,
 *                                     src/piper_kernels/_triton/targets.py:100-104
 *
 * Conventions:
 *   - q/k/v are [B, H, N, D] with the head dimension contiguous; strides[3]
 *     are the B, H and N strides in ELEMENTS (arbitrary, like the reference's
 *     strided-input contract, src/piper_kernels/attention/_validation.py:12-23).
 *   - out is a contiguous [B, H, Nq, D] tensor of the input dtype.
 *   - dtype: PIPER_B200_FLOAT16 or PIPER_B200_BFLOAT16; D in {64, 128};
 *     causal requires Nq == Nk (the Python layer validates first, with the
 *     reference's messages; these checks are the backstop).
 *   - stream is a cudaStream_t (NULL = legacy default stream).  Nothing here
 *     synchronises the host.
 *   - workspace: caller-owned device memory of at least
 *     piper_b200_workspace_bytes(...) bytes, 256-byte aligned.
 */
#ifndef PIPER_B200_H_
#define PIPER_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum piper_b200_status {
  PIPER_B200_OK = 0,
  PIPER_B200_ERR_INVALID_ARGUMENT = 1,
  PIPER_B200_ERR_UNSUPPORTED_DEVICE = 2,
  PIPER_B200_ERR_CUDA = 3,
  PIPER_B200_ERR_TIMEOUT = 4,
  PIPER_B200_ERR_WORKSPACE_TOO_SMALL = 5
} piper_b200_status;

enum { PIPER_B200_FLOAT16 = 0, PIPER_B200_BFLOAT16 = 1 };

/* Byte offsets of each intermediate inside the workspace (see layout.h in
 * the sources for shapes).  Exposed so tests can read the INT8 codes and
 * scales the prepass produced.  v8t holds the V codes as fp16 values (the
 * INT8 codes exactly), transposed to [B*H, D, nk_pad]: the operand of the
 * attention kernel's fp16 PV product. */
typedef struct piper_b200_workspace_layout_s {
  uint64_t q8, k8, v8t, qscale, kscale, vscale, vlog2, vrcp, kmean, vmean, ksum, vsum, counter;
  uint64_t total_bytes;
  int64_t q_groups, k_groups, nk_pad, chunks;
  /* k8 .. vrcp form one contiguous span: [kv_pack, kv_pack + kv_pack_bytes). */
  uint64_t kv_pack, kv_pack_bytes;
  /* fp64 [2, B*H, D]: K then V column sums of a sequence shard. */
  uint64_t totals;
  /* Optional tail of the workspace: partial states of the split-KV tail
   * (split_units_max CTAs).  A workspace of only `split_state` bytes is
   * accepted and runs without the split. */
  uint64_t split_state;
  int64_t split_units_max;
} piper_b200_workspace_layout_t;

/* Byte offsets of the intermediates of a SageAttention2++ call (see
 * sage2pp.cuh in the sources for shapes). */
typedef struct piper_b200_sage2pp_layout_s {
  uint64_t q8, qscale, k8, v8t, kscale, kmask, vscale, kmean, ksum, vmax, counter;
  uint64_t total_bytes;
  int64_t nk_pad, chunks;
} piper_b200_sage2pp_layout_t;

/* ABI version of this header (major*100 + minor). */
int piper_b200_abi_version(void);

/* Message of the most recent failure on the calling thread ("" if none). */
const char* piper_b200_last_error(void);

/* 1 when `device` is an sm_100 GPU this library was built for, else 0. */
int piper_b200_supports_device(int device);

int piper_b200_workspace_bytes(int64_t batch, int64_t heads, int64_t query_length,
                               int64_t key_length, int64_t head_dim, size_t* bytes);

int piper_b200_workspace_layout(int64_t batch, int64_t heads, int64_t query_length,
                                int64_t key_length, int64_t head_dim,
                                piper_b200_workspace_layout_t* layout);

/* Quantization prepass: K/V sequence means, K smoothing, per-32-row Q and
 * per-64-row K INT8 codes + scales, per-key-row V INT8 codes (centered by the
 * V mean when non-causal; stored as exact fp16 values) + scales, into the
 * workspace. */
int piper_b200_prepass(const void* query, const int64_t query_strides[3], const void* key,
                       const int64_t key_strides[3], const void* value,
                       const int64_t value_strides[3], int dtype, int64_t batch, int64_t heads,
                       int64_t query_length, int64_t key_length, int64_t head_dim, int is_causal,
                       void* workspace, size_t workspace_bytes, void* stream);

/* The fused INT8-QK / UINT8xINT8-PV attention on a prepared workspace. */
int piper_b200_attention_prepared(void* out, int dtype, int64_t batch, int64_t heads,
                                  int64_t query_length, int64_t key_length, int64_t head_dim,
                                  double scale, int is_causal, const void* workspace,
                                  size_t workspace_bytes, void* stream);

/* piper_b200_prepass followed by piper_b200_attention_prepared. */
int piper_b200_attention_fwd(const void* query, const int64_t query_strides[3], const void* key,
                             const int64_t key_strides[3], const void* value,
                             const int64_t value_strides[3], void* out, int dtype, int64_t batch,
                             int64_t heads, int64_t query_length, int64_t key_length,
                             int64_t head_dim, double scale, int is_causal, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ---- Execution plan ----------------------------------------------------
 * Host-side launch choices of one attention call, the counterpart of the
 * reference's PiperAttentionExecutionPlan / select_execution_plan
 * (src/piper_kernels/attention/piper_attention/_policy.py:14-96) and of its
 * offline tuner's candidate plans (benchmarks/tune_piper_attention.py:53-101).
 * The first three fields are fixed by the compiled kernels and only
 * reported; the others are run-time choices. */
typedef struct piper_b200_plan_s {
  int32_t tile_rows;   /* query rows per CTA (two 128-row tiles) */
  int32_t key_block;   /* keys per online-softmax block */
  int32_t stages;      /* depth of the production kernel's K/V shared-memory ring, in iterations
                          of 128 keys */
  int32_t rearm;       /* 0: the production kernel: 128 keys (two blocks) per iteration with
                          N = 128 QK^T MMAs, the scores converted with I2F and the probabilities
                          written into TMEM over the spent scores;
                          1: the 64-key-block kernel that re-arms the S accumulators with the
                          bias pattern after each read and passes the probabilities through
                          shared memory */
  int32_t heavy_first; /* causal: longest-work-first grid order across all heads (every head's
                          last query tile first, then every head's second-to-last, ...) */
  int32_t split_k;     /* key ranges per tile of the split-KV tail; 0 = no split */
  int64_t tiles;       /* query tiles of the launch: B*H*ceil(Nq / tile_rows) */
  int64_t tail_tiles;  /* trailing tiles cut into split_k key ranges (0 when split_k is 0) */
  int64_t ctas;        /* CTAs of the attention kernel: tiles - tail_tiles + tail_tiles*split_k */
  int32_t kernels;     /* kernel launches of one prepared call: 1, or 2 with the split merge */
  int32_t sms;         /* SM count the plan was made for */
} piper_b200_plan_t;

/* The production plan for a problem on a device with `sms` SMs (0 = the
 * current device's count, or 148 when no device is visible).  `split_region`
 * says whether the workspace includes the optional split-KV region (a
 * workspace of piper_b200_workspace_bytes bytes does).  Pure host logic: it
 * needs no GPU. */
int piper_b200_select_plan(int64_t batch, int64_t heads, int64_t query_length, int64_t key_length,
                           int64_t head_dim, int is_causal, int sms, int split_region,
                           piper_b200_plan_t* plan);

/* piper_b200_attention_prepared with an explicit plan (from
 * piper_b200_select_plan, possibly edited: rearm, heavy_first, split_k and
 * tail_tiles are honoured; tiles, ctas and kernels are recomputed).  Plans
 * that the kernels cannot run (a split for causal attention, more split CTAs
 * than the workspace's split region holds) are rejected with
 * PIPER_B200_ERR_INVALID_ARGUMENT. */
int piper_b200_attention_prepared_plan(void* out, int dtype, int64_t batch, int64_t heads,
                                       int64_t query_length, int64_t key_length, int64_t head_dim,
                                       double scale, int is_causal, const void* workspace,
                                       size_t workspace_bytes, const piper_b200_plan_t* plan,
                                       void* stream);

/* ---- Sequence-sharded (ring) attention --------------------------------
 * For a sequence split over ranks (rank r holds query/key/value rows of
 * shard r).  No counterpart in the reference, which runs on one GPU; these
 * three calls compose the same arithmetic as piper_b200_attention_fwd:
 *   1. piper_b200_shard_column_sums: the shard's fp64 K (and V) column sums
 *      into the workspace's `totals` region (fp64 [2, B*H, D]).
 *   2. The caller sums `totals` over the ranks (e.g. an NCCL all-reduce),
 *      then piper_b200_shard_prepass turns them into the sequence means
 *      (divided by total_keys) and quantizes this shard.  Shards must start at
 *      multiples of 64 rows so the per-64-row K groups match one GPU's.
 *   3. piper_b200_attention_shard once per key shard, the K/V operands taken
 *      from a K/V pack (the workspace's span [kv_pack, kv_pack+kv_pack_bytes)
 *      of the rank that owns the keys, copied here), carrying each query row's
 *      online-softmax state in `state` (piper_b200_state_bytes) between calls:
 *      state_mode PIPER_B200_STATE_LOAD continues from the state, and
 *      PIPER_B200_STATE_STORE writes the state instead of the output, so the
 *      last call omits STORE and writes `out`.  For causal attention,
 *      causal_shift = first query position - first key position of the two
 *      shards (keys with local index > query local index + shift are masked). */
#define PIPER_B200_STATE_LOAD 1
#define PIPER_B200_STATE_STORE 2

int piper_b200_shard_column_sums(const void* key, const int64_t key_strides[3], const void* value,
                                 const int64_t value_strides[3], int dtype, int64_t batch,
                                 int64_t heads, int64_t query_length, int64_t key_length,
                                 int64_t head_dim, int is_causal, void* workspace,
                                 size_t workspace_bytes, void* stream);

int piper_b200_shard_prepass(const void* query, const int64_t query_strides[3], const void* key,
                             const int64_t key_strides[3], const void* value,
                             const int64_t value_strides[3], int dtype, int64_t batch,
                             int64_t heads, int64_t query_length, int64_t key_length,
                             int64_t head_dim, int is_causal, int64_t total_keys, void* workspace,
                             size_t workspace_bytes, void* stream);

int piper_b200_attention_shard(void* out, int dtype, int64_t batch, int64_t heads,
                               int64_t query_length, int64_t key_length, int64_t head_dim,
                               double scale, int is_causal, int64_t causal_shift,
                               const void* workspace, size_t workspace_bytes, const void* kv_pack,
                               float* state, int state_mode, void* stream);

/* piper_b200_attention_shard over a sub-range: query rows
 * [query_begin, query_begin + query_count) of the query_length rows per head
 * and keys [key_begin, key_begin + key_count) of the key_length keys of the
 * K/V pack (both begins multiples of 64).  The workspace, pack, output and
 * state keep their full shapes; only the range's rows of `out` or of the
 * state are written.  For causal attention, causal_shift = global position of
 * query_begin - global position of key_begin.  Used for zig-zag causal rings
 * and for splitting a problem's keys over several CTAs. */
int piper_b200_attention_shard_range(void* out, int dtype, int64_t batch, int64_t heads,
                                     int64_t query_length, int64_t query_begin,
                                     int64_t query_count, int64_t key_length, int64_t key_begin,
                                     int64_t key_count, int64_t head_dim, double scale,
                                     int is_causal, int64_t causal_shift, const void* workspace,
                                     size_t workspace_bytes, const void* kv_pack, float* state,
                                     int state_mode, void* stream);

/* Bytes of the per-row state of piper_b200_attention_shard: fp32
 * [B*H, Nq, D] numerators followed by fp32 [B*H, Nq, 2] (max, denominator);
 * 0 for non-positive sizes. */
size_t piper_b200_state_bytes(int64_t batch, int64_t heads, int64_t query_length,
                              int64_t head_dim);

/* ---- Host-to-host forward pass -----------------------------------------
 * piper_b200_attention_fwd for inputs and output in HOST memory (contiguous
 * [B, H, N, D]; page-locked memory is needed for the copies to overlap).  No
 * counterpart in the reference, where the caller moves tensors to the GPU
 * first.  The heads are processed in chunks through a ring of device slots:
 * host-to-device copies, the kernels and device-to-host copies of different
 * chunks overlap, so the call costs about the slowest of the three rather
 * than their sum.  `scratch` is device memory of piper_b200_host_scratch_bytes
 * bytes (256-byte aligned).  Kernels run on `stream` and on an internal
 * stream, the copies on two more internal streams, all ordered after the work
 * already on `stream`; `stream` is made to wait for the last output copy, so
 * synchronising `stream` (or an event recorded on it) means `out` is
 * complete. */
int piper_b200_host_scratch_bytes(int64_t batch, int64_t heads, int64_t query_length,
                                  int64_t key_length, int64_t head_dim, size_t* bytes);

int piper_b200_attention_fwd_host(const void* query, const void* key, const void* value, void* out,
                                  int dtype, int64_t batch, int64_t heads, int64_t query_length,
                                  int64_t key_length, int64_t head_dim, double scale, int is_causal,
                                  void* scratch, size_t scratch_bytes, void* stream);

/* ---- SageAttention2++ (8+8) --------------------------------------------
 * The sibling operator of the reference's sage_attention_2pp
 * (src/piper_kernels/attention/sage_attention_2pp/dispatch.py:37-64, Triton
 * backend triton.py:1135-1155): INT8 Q/K with per_thread scales (K centred
 * by its sequence mean), FP8 e4m3 V with per-channel scales, FP8 e4m3
 * probabilities against the running max shifted by log2(448), and an e4m3 x
 * e4m3 PV product on the tensor cores (tcgen05 kind::f8f6f4, F32 accumulator).
 * Same argument conventions as piper_b200_attention_fwd. */
int piper_b200_sage2pp_layout(int64_t batch, int64_t heads, int64_t query_length,
                              int64_t key_length, int64_t head_dim,
                              piper_b200_sage2pp_layout_t* layout);

int piper_b200_sage2pp_workspace_bytes(int64_t batch, int64_t heads, int64_t query_length,
                                       int64_t key_length, int64_t head_dim, size_t* bytes);

int piper_b200_sage2pp_prepass(const void* query, const int64_t query_strides[3],
                               const void* key, const int64_t key_strides[3], const void* value,
                               const int64_t value_strides[3], int dtype, int64_t batch,
                               int64_t heads, int64_t query_length, int64_t key_length,
                               int64_t head_dim, void* workspace, size_t workspace_bytes,
                               void* stream);

int piper_b200_sage2pp_attention_prepared(void* out, int dtype, int64_t batch, int64_t heads,
                                          int64_t query_length, int64_t key_length,
                                          int64_t head_dim, double scale, int is_causal,
                                          const void* workspace, size_t workspace_bytes,
                                          void* stream);

int piper_b200_sage2pp_fwd(const void* query, const int64_t query_strides[3], const void* key,
                           const int64_t key_strides[3], const void* value,
                           const int64_t value_strides[3], void* out, int dtype, int64_t batch,
                           int64_t heads, int64_t query_length, int64_t key_length,
                           int64_t head_dim, double scale, int is_causal, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Scratch capacity of piper_b200_attention_fwd_no_alloc: 16 MiB per GPU. */
#define PIPER_B200_NO_ALLOC_WORKSPACE_BYTES (16u * 1024u * 1024u)

/* The same forward pass as piper_b200_attention_fwd, for callers that cannot
 * allocate device memory.  Examples: a plugin inside a host process that owns
 * the whole GPU memory budget and refuses outside allocations; a binding from
 * a language runtime that can hand over input and output pointers but has no
 * device allocator; a steady-state loop where a cudaMalloc, which may
 * synchronise the device, is not allowed.  It has no counterpart in the
 * reference, which always allocates through torch.
 *
 * The caller still passes inputs and output.  The scratch comes from a
 * fixed 16 MiB array (PIPER_B200_NO_ALLOC_WORKSPACE_BYTES) compiled into this
 * library: every GPU that loads the library holds that array until the
 * process exits.  The limit applies to the required part of the workspace,
 * the bytes before its optional split-KV region (the `split_state` offset of
 * piper_b200_workspace_layout): a problem whose required part exceeds 16 MiB
 * is rejected with PIPER_B200_ERR_WORKSPACE_TOO_SMALL.  When the whole
 * workspace (piper_b200_workspace_bytes, split region included) does not fit
 * but its required part does, the call runs without the split-KV tail (the
 * same output to fp32 rounding).  No cudaMalloc, cudaFree or other allocating
 * call is made.  The first call on a device (and the first after the device's
 * context is reset) looks up the array's device address for that context
 * (make that first call before any stream capture).  All calls on a device
 * share the one array, so two calls whose work overlaps on the GPU (different
 * streams, no ordering between them) race and corrupt each other; order such
 * calls on one stream. */
int piper_b200_attention_fwd_no_alloc(const void* query, const int64_t query_strides[3],
                                      const void* key, const int64_t key_strides[3],
                                      const void* value, const int64_t value_strides[3], void* out,
                                      int dtype, int64_t batch, int64_t heads,
                                      int64_t query_length, int64_t key_length, int64_t head_dim,
                                      double scale, int is_causal, void* stream);

/* Reads (and, if `clear`, resets) the device status word that kernels set when
 * a bounded wait gave up.  Synchronises the device.  *status == 0 means no
 * kernel of this library has timed out on `device`. */
int piper_b200_device_status(int device, int clear, uint32_t* status);

/* Self-test of the bounded-wait path: launches one CTA that waits on an
 * mbarrier nothing ever arrives at, with a `budget_ns` limit, and reports
 * whether it gave up cleanly (*timed_out = 1) while the context stays usable. */
int piper_b200_selftest_wait_timeout(uint64_t budget_ns, int* timed_out, void* stream);

/* Self-test of the kernels' software exp2 (the FMA-pipe polynomial that
 * takes a share of the probabilities off the MUFU unit): y[i] = 2^x[i] as the
 * attention kernel computes it, and ex2[i] = the hardware ex2.approx of the
 * same x (either output may be NULL).  x, y and ex2 are device float arrays of
 * n elements; tests compare both against exact 2^x. */
int piper_b200_selftest_exp2(const float* x, float* y, float* ex2, int64_t n, void* stream);

/* Diagnostic GEMM on the tensor cores: C[M,N] (int32) = A[M,K] * B[N,K]^T with
 * A u8 or s8 (a_signed), B s8, both K-major, through the same TMA + tcgen05
 * kind::i8 path the attention kernel uses.  M % 128 == 0, N % 64 == 0,
 * K % 128 == 0; all pointers are device memory. */
int piper_b200_selftest_gemm_i8(const void* a, const void* b, int32_t* c, int64_t m, int64_t n,
                                int64_t k, int a_signed, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PIPER_B200_H_ */
