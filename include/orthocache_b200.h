/*
 * orthocache_b200 — C ABI of the B200 (sm_100a) OrthoCache eviction +
 * attention hot path.
 *
 * Conventions (all entry points):
 *   - Plain device pointers and sizes; the caller owns every buffer.  Tensors
 *     are dense row-major.  Keys / values / queries are float32 (OC_F32) or
 *     bfloat16 (OC_BF16); all arithmetic is float32.
 *   - Layouts follow the reference's (seq, heads, dim) convention with an
 *     optional leading batch dimension: keys/values (B, S, Hkv, D), queries
 *     (B, Sq, Hq, D), per-block outputs (B, nb, Hkv[, D]) with nb = S / 512.
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *     stream) and is asynchronous.  Counts stay on the device.
 *   - Return 0 on success or a negative OC_ERR_* code.  Arguments are checked
 *     on the host before anything is launched; oc_last_error() returns a
 *     message for the calling thread's last failure.
 *   - Functions that need scratch memory take (workspace, workspace_bytes);
 *     the matching *_workspace_bytes() query gives the size.  No entry point
 *     allocates device memory.
 *
 * Reference interfaces cited as file:line of the reference project
 * (j-arndt/orthocache v0.3.0).
 */
#ifndef ORTHOCACHE_B200_H
#define ORTHOCACHE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* oc_stream_t; /* == cudaStream_t */

enum oc_dtype { OC_F32 = 0, OC_BF16 = 1 };

enum oc_status {
  OC_OK = 0,
  OC_ERR_NULL = -1,        /* a required pointer is NULL */
  OC_ERR_SHAPE = -2,       /* inconsistent or unsupported shape */
  OC_ERR_ALIGN = -3,       /* pointer not 16-byte aligned */
  OC_ERR_CAPACITY = -4,    /* workspace too small / size above a limit */
  OC_ERR_DTYPE = -5,       /* unsupported dtype */
  OC_ERR_CUDA = -6,        /* CUDA runtime error (message has details) */
  OC_ERR_UNSUPPORTED = -7, /* valid request this build does not implement */
  OC_ERR_COMM = -8         /* NCCL error (message has details) */
};

/* Library version (major*10000 + minor*100 + patch). */
int oc_version(void);
/* Static description of an OC_ERR_* code. */
const char* oc_status_string(int status);
/* Message of the calling thread's last failure ("" if none). */
const char* oc_last_error(void);

/* Device-side status of the pipelined kernels: nonzero if a bounded wait on
 * an asynchronous copy gave up (the kernel then skipped its remaining work
 * instead of hanging).  Bit 0: scorer / fused decode layer; bit 1: split-KV
 * attention; bit 2: chunked-prefill attention.  Synchronises the current device; reset != 0 clears it.
 * Returns the status (>= 0) or an OC_ERR_* code. */
int oc_device_status(int reset);

/* Limit of every bounded wait in the kernels of the current device (default
 * 2 s; 1 us .. 60 s): after it a wait gives up, the kernel records the status
 * above and returns.  Meant for tests and watchdogs that want a failure to
 * surface fast; no counterpart in the reference (JAX has no device waits). */
int oc_set_wait_limit_ns(uint64_t ns);

/* ---------------------------------------------------------------------------
 * fwht_512 — replaces `fwht_512(x)` (src/orthocache/fwht.py:4-65).
 * x: (512, ncols) row-major, dtype `x_dtype`; y: (512, ncols) float32.
 * Natural (Hadamard) order, 9 butterfly stages h = 1..256 in the reference's
 * order, then an IEEE float32 division by 22.627416997969522 (fwht.py:61):
 * bit-identical to the reference's float32 butterfly.
 */
int oc_fwht512(const void* x, int x_dtype, int64_t ncols, float* y, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused block scorer — replaces, in one pass over the keys,
 *   compute_spectral_bands        (src/orthocache/spectral_energy.py:69-106)
 *   compute_spectral_decay_ratio  (spectral_energy.py:109-138)
 *   compute_query_aware_bounds    (spectral_energy.py:141-177), max over rows
 *   compute_query_aware_mask      (spectral_energy.py:180-196)
 *   compute_multiband_mask        (spectral_energy.py:199-234)
 *
 * keys: (B, S, Hkv, D), S % 512 == 0, D in {64, 128, 256}.
 * q: (B, Sq, Hq, D) of the same dtype, Hq % Hkv == 0; may be NULL (then no
 *    bound is computed and the logit gate passes every block).
 * Bands are half-open coefficient-index ranges [lo, hi) of the natural-order
 * WHT (reference defaults (1,64), (64,256), (256,512)).  ζ = E_high /
 * (E_low + 1e-6).  bound_max[b,j,h] = max over the Sq*G query rows of KV
 * head h of  q·mean_j/√D + ‖q‖·√E_AC/√D  (GQA: query head hq reads KV head
 * hq / G, G = Hq / Hkv).  keep = (bound_max >= tau) && (zeta <= zeta_max).
 *
 * Outputs, each nullable: dc (B, nb, Hkv, D) = WHT coefficient 0;
 * e_low / e_mid / e_high / zeta / bound_max (B, nb, Hkv) float32;
 * bounds (B, Sq, nb, Hq) float32 = the bound of every query row before the
 * max (the (seq_len_q, num_blocks, num_heads) array of
 * compute_query_aware_bounds); keep (B, nb, Hkv) uint8 0/1.
 *
 * mode: 0 = automatic; 1 = the partial-transform scorer (band edges must be
 * 0, 1 or multiples of 64; bfloat16 keys stream through a bulk-tensor (TMA)
 * shared-memory pipeline); 2 = the full 9-stage butterfly scorer (any
 * bands); 3 = the partial-transform scorer with per-thread vector loads
 * (same results as 1, kept as a cross-check).
 */
int oc_score_blocks(const void* keys, const void* q, int dtype,
                    int batch, int seq_len, int kv_heads, int head_dim,
                    int q_len, int q_heads,
                    int band_low0, int band_low1, int band_mid0, int band_mid1,
                    int band_high0, int band_high1,
                    float tau, float zeta_max,
                    float* dc, float* e_low, float* e_mid, float* e_high,
                    float* zeta, float* bound_max, float* bounds, uint8_t* keep,
                    int mode, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Write-time spectral metadata.  ζ, the DC coefficients and E_AC of a block
 * do not depend on the query (docs/mathematical_framework.md:244-250 of the
 * reference: "computed once when the block is written to the KV cache"), so
 * a cache that keeps them needs to read only them at decode time instead of
 * every key.
 *
 * oc_block_metadata: for keys (B, S, Hkv, D) with the reference's default
 * bands, write dc (B, nb, Hkv, D) = WHT coefficient 0, e_ac (B, nb, Hkv) =
 * energy of coefficients 1..511 (spectral_energy.py:159-160) and zeta
 * (B, nb, Hkv) (spectral_energy.py:109-138); each output nullable.  Values
 * equal oc_score_blocks' for the same keys.  Run it on a slice of whole
 * blocks to refresh only the blocks that were (re)written.
 */
int oc_block_metadata(const void* keys, int dtype, int batch, int seq_len, int kv_heads, int head_dim,
                      float* dc, float* e_ac, float* zeta, oc_stream_t stream);

/* oc_score_from_metadata: the two gates of compute_multiband_mask
 * (spectral_energy.py:199-234) from that metadata and the queries alone:
 * bound = q·(dc/√512)/√D + ‖q‖·√E_AC/√D per query row (spectral_energy.py:
 * 150-177, GQA rows as in oc_score_blocks), bound_max (B, nb, Hkv) its max,
 * bounds (B, Sq, nb, Hq), keep = bound_max >= tau && zeta <= zeta_max; each
 * output nullable.  q (B, Sq, Hq, D) of q_dtype. */
int oc_score_from_metadata(const float* dc, const float* e_ac, const float* zeta, const void* q, int q_dtype,
                           int batch, int num_blocks, int kv_heads, int head_dim, int q_len, int q_heads,
                           float tau, float zeta_max, float* bound_max, float* bounds, uint8_t* keep,
                           oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Sum of squared keys per (block, head) — replaces compute_block_energy_jax
 * (spectral_energy.py:21-35).  energy: (B, nb, H) float32.  block_size any
 * divisor of S.
 */
int oc_block_energy(const void* keys, int dtype, int batch, int seq_len, int heads,
                    int head_dim, int block_size, float* energy, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Stream compaction — replaces the index part of
 *   compaction.stream_compact           (src/orthocache/compaction.py:28-100)
 *   alltoallv.stream_compact            (src/orthocache/alltoallv.py:44-75)
 *   distributed_attention.stream_compact (distributed_attention.py:31-46)
 *   adaptive_attention.stream_compact   (adaptive_attention.py:29-40)
 * keep: (B, nb, heads) uint8; a block is active if any head keeps it
 * (compaction.py:65).  perm: (B, nb) int32, the stable permutation with the
 * active blocks first in ascending order, then the inactive blocks ascending
 * (compaction.py:76-82).  count: (B) int32 number of active blocks.
 */
int oc_stream_compact(const uint8_t* keep, int batch, int num_blocks, int heads,
                      int32_t* perm, int32_t* count, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Block gather — replaces the K/V gather of compaction.stream_compact
 * (compaction.py:85-98), alltoallv.pack_active_blocks (alltoallv.py:150-212)
 * and distributed_attention._pack_active_blocks (distributed_attention.py:49-75).
 * src: (B, nb_src, block_elems) elements of `dtype`; dst: (B, nb_dst,
 * block_elems).  For i < min(count[b], nb_dst): dst[b,i] = src[b, perm[b*perm_stride+i]];
 * for i >= count[b]: zero if zero_tail, untouched otherwise.  count may be
 * NULL (= nb_dst).  block_elems * sizeof(dtype) must be a multiple of 16.
 */
int oc_gather_blocks(const void* src, int dtype, int batch, int nb_src, int64_t block_elems,
                     const int32_t* perm, int perm_stride, const int32_t* count,
                     void* dst, int nb_dst, int zero_tail, oc_stream_t stream);

/* Inverse of oc_gather_blocks — replaces compaction.stream_decompact
 * (compaction.py:103-154): dst is zeroed, then dst[b, perm[b*perm_stride+i]]
 * = src[b, i] for i < count[b] (count NULL = nb_src). */
int oc_scatter_blocks(const void* src, int dtype, int batch, int nb_src, int64_t block_elems,
                      const int32_t* perm, int perm_stride, const int32_t* count,
                      void* dst, int nb_dst, oc_stream_t stream);

/* Bucketed block count of indirect_attention (indirect_attention.py:20-26,
 * 150-157): out[i] = the smallest of 1, 2, 4, ..., 512 that is >= count[i]
 * (a count above 512 is kept; 0 stays 0), clamped to cap.  The reference's
 * Pallas kernel attends to exactly that many leading entries of the
 * permutation, i.e. to the active blocks plus the first inactive ones up to
 * the bucket. */
int oc_bucket_count(const int32_t* count, int n, int cap, int32_t* out, oc_stream_t stream);

/* The two gates on precomputed scores (spectral_energy.py:196, 231-234):
 * keep[i] = (bound_max[i] >= tau) && (zeta[i] <= zeta_max).  bound_max or
 * zeta may be NULL (that gate passes); tau_dev (nullable) is a device float
 * that overrides tau, so a threshold computed on the device needs no host
 * round trip. */
int oc_apply_gates(const float* bound_max, const float* zeta, int64_t cells, const float* tau_dev,
                   float tau, float zeta_max, uint8_t* keep, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Indirect block attention — replaces
 *   indirect_attention.indirect_attention (src/orthocache/indirect_attention.py:127-170)
 *   adaptive_attention._multihead_loop    (adaptive_attention.py:90-120)
 *   distributed_attention._online_softmax_indirect_attention
 *                                         (distributed_attention.py:78-128)
 * Every query head attends to the tokens of blocks idx[b*idx_stride + i],
 * i < count[b]; logits = q·k/√D in float32, softmax over all those tokens,
 * output o / l cast to out_dtype.  count[b] == 0 gives zeros
 * (indirect_attention.py:150-151).
 * q (B, Sq, Hq, D); k, v (B, S, Hkv, D); out (B, Sq, Hq, D).
 * block_size % 64 == 0 and S % block_size == 0; D in {64, 128, 256}
 * (float32 inputs: D <= 128).  max_blocks bounds count (the number of index
 * slots scanned).
 * Index addressing: the index list of (batch b, kv head h) starts at
 * idx[b*idx_stride + h*idx_head_stride] and its length is
 * count[b*count_stride + h*count_head_stride].  The union form of the
 * reference (one list per batch row shared by all heads) is
 * idx_head_stride = count_head_stride = 0, count_stride = 1; per-head lists
 * (the predicated per-head mask of sparse_attention.py:46-49) use nonzero
 * head strides.
 */
size_t oc_indirect_attention_workspace_bytes(int batch, int q_len, int q_heads, int kv_heads,
                                             int head_dim, int block_size, int max_blocks);
int oc_indirect_attention(const void* q, const void* k, const void* v, int dtype,
                          const int32_t* idx, int idx_stride, int idx_head_stride,
                          const int32_t* count, int count_stride, int count_head_stride,
                          int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                          int seq_len, int block_size, int max_blocks,
                          void* out, int out_dtype,
                          void* workspace, size_t workspace_bytes, oc_stream_t stream);

/* Predicated-attention semantics for a head with no kept block
 * (sparse_attention.py:49-57: every logit masked to -1e9, so the softmax is
 * uniform): for each (b, h) with count[b*count_stride + h*count_head_stride]
 * == 0, write the mean over all S value rows of head h to the G query heads
 * of that group in out (B, Sq, Hq, D).  Other rows are untouched; run it after
 * oc_indirect_attention with per-head lists. */
int oc_empty_heads_mean(const void* v, int dtype, const int32_t* count, int count_stride,
                        int count_head_stride, int batch, int q_len, int q_heads, int kv_heads,
                        int head_dim, int seq_len, void* out, int out_dtype, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * oc_indirect_attention without a workspace argument.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory when
 * they run the attention (an allocator-free FFI host, a serving loop whose
 * memory pool forbids allocations during a step, a process whose allocator
 * is exhausted).  Same inputs, outputs and results as oc_indirect_attention;
 * the scratch comes from a fixed 32 MiB device array that every GPU which
 * loads this library holds until the process exits.  It never calls
 * cudaMalloc or cudaFree.
 *   - Shapes whose scratch need (oc_indirect_attention_workspace_bytes) is
 *     above oc_indirect_attention_noalloc_max_scratch_bytes() are rejected
 *     with OC_ERR_CAPACITY.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.  The address is cached for the life of the
 *     process: a device reset (cudaDeviceReset) or a torn-down primary
 *     context is not supported afterwards.
 *   - All calls on a device share the one array: calls whose kernels overlap
 *     on the GPU (different streams, or other threads) race and corrupt each
 *     other's results.  Serialise them.  Nothing in the array needs to start
 *     at zero; it keeps the last call's contents.
 */
size_t oc_indirect_attention_noalloc_max_scratch_bytes(void);
int oc_indirect_attention_noalloc(const void* q, const void* k, const void* v, int dtype,
                                  const int32_t* idx, int idx_stride, int idx_head_stride,
                                  const int32_t* count, int count_stride, int count_head_stride,
                                  int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                                  int seq_len, int block_size, int max_blocks,
                                  void* out, int out_dtype, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Chunked-prefill indirect attention on the tensor cores (tcgen05 + tensor
 * memory) — replaces indirect_attention / _multihead_loop
 * (src/orthocache/indirect_attention.py:29-83, :127-170;
 * adaptive_attention.py:90-120) when the query chunk is long: every query row
 * attends to the tokens of blocks idx[0 .. count) (count clipped to
 * max_blocks), online softmax in float32, o / l; count == 0 gives zeros.
 * Same index / count conventions as oc_indirect_attention (per-row lists with
 * idx_head_stride = count_head_stride = 0, per-KV-head lists otherwise).
 *
 * bfloat16 q (B, Sq, Hq, D), k / v (B, S, Hkv, D) with head_dim 128;
 * block_size a multiple of 128 dividing seq_len; out (B, Sq, Hq, D) in
 * out_dtype (OC_BF16 or OC_F32).  Any q_len >= 1 (query rows are processed in
 * tiles of 128; the last tile of a chunk is partial).  P is rounded to
 * bfloat16 for the P.V product, as in FlashAttention-style kernels.  Needs no
 * workspace.  One persistent CTA per SM holding 224 KB of shared memory and
 * all 512 tensor-memory columns of its SM.
 */
int oc_prefill_attention(const void* q, const void* k, const void* v, int dtype,
                         const int32_t* idx, int idx_stride, int idx_head_stride,
                         const int32_t* count, int count_stride, int count_head_stride,
                         int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                         int seq_len, int block_size, int max_blocks,
                         void* out, int out_dtype, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * One decode step of the OrthoCache pipeline on the device: score (two-gate
 * keep mask), compact (perm, count) and attend over the retained blocks —
 * the path of pipeline.orthocache_forward(mode='compact')
 * (src/orthocache/pipeline.py:33-157) with compute_multiband_mask
 * (spectral_energy.py:199-234) feeding indirect attention instead of the K/V
 * copy of compact_and_attend (compaction.py:157-222).
 * Shapes as above; keep (B, nb, Hkv) uint8, perm (B, nb), count (B) are
 * outputs; out (B, Sq, Hq, D) in out_dtype.
 *
 * bfloat16 with head_dim 128, Sq * (Hq / Hkv) <= 8 query rows per KV head and
 * B * Hkv <= the number of SMs runs as ONE persistent kernel: the scorer
 * decides each block as soon as its Hkv tiles are scored, and the same CTAs
 * then stream K and V of the retained blocks and merge the attention in
 * log-sum-exp form.  Other shapes run the scorer, the compaction and the
 * split-KV attention as separate kernels.
 *
 * Workspace: oc_decode_step_workspace_bytes() bytes, 256-byte aligned, and
 * ZERO-FILLED before its first use (cudaMemset once).  Its leading region
 * holds an epoch and two counter sets that the one-kernel path keeps
 * consistent from call to call, so later calls need no clearing.  Calls that
 * share a workspace must not overlap on the GPU.  If oc_device_status()
 * reports a wait that gave up, zero the workspace again.
 */
size_t oc_decode_step_workspace_bytes(int batch, int q_len, int q_heads, int kv_heads,
                                      int head_dim, int seq_len);
int oc_decode_step(const void* q, const void* k, const void* v, int dtype,
                   int batch, int q_len, int q_heads, int kv_heads, int head_dim, int seq_len,
                   float tau, float zeta_max,
                   uint8_t* keep, int32_t* perm, int32_t* count,
                   void* out, int out_dtype,
                   void* workspace, size_t workspace_bytes, oc_stream_t stream);

/* The same decode step with the blocks' gates taken from write-time
 * spectral metadata (oc_block_metadata output: dc (B, nb, Hkv, D), e_ac and
 * zeta (B, nb, Hkv) float32) instead of a pass over the keys: the bound of
 * compute_query_aware_bounds (spectral_energy.py:141-177) from the DC
 * coefficients and E_AC, the zeta gate of compute_multiband_mask
 * (spectral_energy.py:199-234) from the stored zeta; the keys are read only
 * for the retained blocks.  Same shapes, outputs and workspace contract as
 * oc_decode_step (the one-kernel path under the same conditions; the
 * separate kernels oc_score_from_metadata, oc_stream_compact and
 * oc_indirect_attention otherwise). */
int oc_decode_step_from_metadata(const void* q, const void* k, const void* v, int dtype,
                                 const float* dc, const float* e_ac, const float* zeta,
                                 int batch, int q_len, int q_heads, int kv_heads, int head_dim, int seq_len,
                                 float tau, float zeta_max,
                                 uint8_t* keep, int32_t* perm, int32_t* count,
                                 void* out, int out_dtype,
                                 void* workspace, size_t workspace_bytes, oc_stream_t stream);

/* The decode step of one sequence shard, for the log-sum-exp merge across
 * shards (distributed_attention.py:95-128 applied across devices): as
 * oc_decode_step, but instead of out it writes the shard's unnormalised
 * partial per output row in the format of oc_partial_attention — m (rows),
 * l (rows), o (rows, D) float32, rows = B*Sq*Hq, m in log2 units of the
 * scaled logits (m = -inf, l = 0, o = 0 when the shard retains nothing).
 * Same workspace contract as oc_decode_step (zero-filled once). */
int oc_decode_step_partial(const void* q, const void* k, const void* v, int dtype,
                           int batch, int q_len, int q_heads, int kv_heads, int head_dim, int seq_len,
                           float tau, float zeta_max,
                           uint8_t* keep, int32_t* perm, int32_t* count,
                           float* m, float* l, float* o,
                           void* workspace, size_t workspace_bytes, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Sequence-parallel exchange helpers (the device-side index math of
 * distributed_attention.py:179-191, alltoallv.py:113-145 and
 * benchmarks/phase_e_stratified.py:182-197,242-265).
 *
 * oc_exchange_index: all_counts (P) int32 per-device active counts; slots =
 * blocks each device contributed to the gathered buffer.  order (P*slots)
 * int32 = slots j with j % slots < counts[j / slots] first (ascending), then
 * the rest; total (1) int32 = sum of counts; offsets (P) int32 (nullable) =
 * exclusive prefix sum of counts.
 */
int oc_exchange_index(const int32_t* all_counts, int num_devices, int slots,
                      int32_t* order, int32_t* total, int32_t* offsets, oc_stream_t stream);

/* Stratified capacity bucket of build_stratified (phase_e_stratified.py:182-197,
 * 262-265), computed on the host: the smallest of the four buckets
 * max(1,nb/4), max(1,nb/2), max(1,3nb/4), nb that is >= gmax. */
int oc_stratified_bucket(int nb_per_device, int gmax);

/* Merge of per-shard partial attention (m, l, o): the log-sum-exp combine of
 * the online softmax in distributed_attention.py:95-128 applied across
 * shards.  m, l: (P, rows), o: (P, rows, D) float32 as written by
 * oc_partial_attention; out (rows, D) in out_dtype; rows = B*Sq*Hq. */
int oc_merge_partials(const float* m, const float* l, const float* o, int parts, int rows,
                      int head_dim, void* out, int out_dtype, oc_stream_t stream);

/* oc_merge_partials on the packed layout that one all-gather of per-shard
 * partials produces: part p occupies rows * (D + 2) floats at
 * packed + p * rows * (D + 2), holding m (rows), then l (rows), then
 * o (rows, D). */
int oc_merge_partials_packed(const float* packed, int parts, int rows, int head_dim, void* out, int out_dtype,
                             oc_stream_t stream);

/* Partial (unnormalised) attention of one shard for the LSE merge: same
 * arguments as oc_indirect_attention but writes m (rows), l (rows) and
 * o (rows, D) float32, rows = B*Sq*Hq in output order; m is in log2 units of
 * the scaled logits.  A shard with count 0 writes m = -inf, l = 0, o = 0. */
int oc_partial_attention(const void* q, const void* k, const void* v, int dtype,
                         const int32_t* idx, int idx_stride, int idx_head_stride,
                         const int32_t* count, int count_stride, int count_head_stride,
                         int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                         int seq_len, int block_size, int max_blocks,
                         float* m, float* l, float* o,
                         void* workspace, size_t workspace_bytes, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Paged KV cache.  The reference's index table (indirect_attention.py:155-159:
 * the kernel reads keys and values only through block indices) doubles as a
 * page table: keys / values live in a pool of num_pages blocks of block_size
 * tokens, k_pool / v_pool (num_pages * block_size, kv_heads, head_dim), shared
 * by the batch; logical block j of batch row b is pool page
 * block_table[b * table_stride + j].  idx / count are the compaction of the
 * LOGICAL mask (oc_stream_compact), exactly as for the contiguous entry
 * points; a page outside [0, num_pages) is skipped.
 *
 * Attention (split-KV, any q_len; dtype / head_dim as oc_indirect_attention);
 * workspace = oc_indirect_attention_paged_workspace_bytes(). */
size_t oc_indirect_attention_paged_workspace_bytes(int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                                                   int block_size, int max_blocks);
int oc_indirect_attention_paged(const void* q, const void* k_pool, const void* v_pool, int dtype,
                                const int32_t* block_table, int table_stride, const int32_t* idx, int idx_stride,
                                const int32_t* count, int count_stride, int batch, int q_len, int q_heads,
                                int kv_heads, int head_dim, int num_pages, int block_size, int max_blocks, void* out,
                                int out_dtype, void* workspace, size_t workspace_bytes, oc_stream_t stream);
/* Chunked prefill on the tensor cores over a paged pool (conditions of
 * oc_prefill_attention); workspace = oc_prefill_attention_paged_workspace_bytes(). */
size_t oc_prefill_attention_paged_workspace_bytes(int batch, int max_blocks);
int oc_prefill_attention_paged(const void* q, const void* k_pool, const void* v_pool, int dtype,
                               const int32_t* block_table, int table_stride, const int32_t* idx, int idx_stride,
                               const int32_t* count, int count_stride, int batch, int q_len, int q_heads,
                               int kv_heads, int head_dim, int num_pages, int block_size, int max_blocks, void* out,
                               int out_dtype, void* workspace, size_t workspace_bytes, oc_stream_t stream);
/* The two gates from the write-time metadata of a paged pool: dc_pool
 * (num_pages, kv_heads, head_dim), e_ac_pool / zeta_pool (num_pages,
 * kv_heads) as oc_block_metadata writes them for the pool (batch 1, seq_len
 * num_pages * 512); outputs per LOGICAL (batch, block, head) as
 * oc_score_from_metadata. */
int oc_score_from_metadata_paged(const float* dc_pool, const float* e_ac_pool, const float* zeta_pool, int num_pages,
                                 const int32_t* block_table, int table_stride, const void* q, int q_dtype, int batch,
                                 int num_blocks, int kv_heads, int head_dim, int q_len, int q_heads, float tau,
                                 float zeta_max, float* bound_max, float* bounds, uint8_t* keep, oc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Sequence-parallel exchange over NCCL (one rank per GPU).  `comm` is an
 * ncclComm_t created by the caller (any NCCL 2.x: the library resolves NCCL
 * at run time, preferring the copy already loaded in the process, else
 * libnccl.so.2 or the path in the environment variable OC_NCCL_LIBRARY) or
 * by oc_comm_init.  The reference's pmap axis (axis_name) becomes this
 * communicator.  Calls are collective: every rank makes the same call in the
 * same order.
 */
/* NCCL_VERSION_CODE of the NCCL in use, or OC_ERR_UNSUPPORTED. */
int oc_nccl_version(void);
/* A 128-byte ncclUniqueId (rank 0), to be shared with the other ranks. */
int oc_comm_unique_id(void* id_out);
/* ncclCommInitRank on the current device. */
int oc_comm_init(void** comm_out, const void* id, int nranks, int rank);
int oc_comm_destroy(void* comm);
/* Host-side failure detection: OC_ERR_COMM (with NCCL's message) if the
 * communicator holds an asynchronous error (a peer failed or aborted), else 0.
 * A watchdog polls it and calls oc_comm_abort to release blocked ranks. */
int oc_comm_check(void* comm);
int oc_comm_abort(void* comm);

/* Workspace of oc_exchange_stratified / oc_alltoallv_heads: the packed K
 * and V send buffers of one shard of num_blocks blocks. */
size_t oc_exchange_workspace_bytes(int num_blocks, int kv_heads, int head_dim, int dtype, int block_size);

/* Stratified all-gather of the retained blocks — replaces build_stratified
 * (benchmarks/phase_e_stratified.py:164-273) and the exchange of
 * distributed_orthocache_attention (distributed_attention.py:156-191).
 * k, v: this shard (num_blocks * block_size, kv_heads, head_dim); idx, count:
 * its compaction (oc_stream_compact).  Gathers every rank's count into
 * all_counts (P, device), reads them on the host (the one synchronisation:
 * the bucket sizes the collective), picks bucket = oc_stratified_bucket(
 * num_blocks, max count), packs this rank's first `bucket` retained blocks
 * (zero tail) and all-gathers them: k_recv / v_recv (P * num_blocks *
 * block_size, kv_heads, head_dim) hold P chunks of `bucket` blocks in rank
 * order (capacity for the largest bucket, num_blocks).  order / total: the
 * valid-slot index of oc_exchange_index over the P * bucket gathered slots,
 * ready for oc_indirect_attention.  *bucket_out (nullable) = bucket.  Blocks
 * are bit-exact copies. */
int oc_exchange_stratified(void* comm, const void* k, const void* v, int dtype, const int32_t* idx,
                           const int32_t* count, int num_blocks, int kv_heads, int head_dim, int block_size,
                           void* k_recv, void* v_recv, int32_t* all_counts, int32_t* order, int32_t* total,
                           int* bucket_out, void* workspace, size_t workspace_bytes, oc_stream_t stream);

/* AllToAllv of the retained blocks by KV head — the exchange of
 * alltoallv_kv_exchange (alltoallv.py:217-259, 340-440) with each rank
 * receiving only the KV heads it owns (rank r: heads r*H/P .. (r+1)*H/P - 1;
 * kv_heads % P == 0) instead of every head: grouped ncclSend / ncclRecv with
 * per-peer sizes from the count all-gather (read on the host).  k_recv /
 * v_recv: (P * num_blocks * block_size, kv_heads / P, head_dim) capacity;
 * the first total blocks are every rank's retained blocks of this rank's
 * heads in rank order (the layout unpack_received_blocks leaves), so they
 * are attended to with idx = 0, 1, ..., total - 1.  *total_out (nullable) =
 * total.  Bit-exact copies. */
int oc_alltoallv_heads(void* comm, const void* k, const void* v, int dtype, const int32_t* idx,
                       const int32_t* count, int num_blocks, int kv_heads, int head_dim, int block_size,
                       void* k_recv, void* v_recv, int32_t* all_counts, int* total_out, void* workspace,
                       size_t workspace_bytes, oc_stream_t stream);

/* One decode layer of sequence-parallel attention through NCCL: the fused
 * layer of this rank's shard writes its (m, l, o) partial
 * (oc_decode_step_partial), the P packed partials are all-gathered, and the
 * log-sum-exp merge writes out on every rank — attention over the union of
 * all shards' retained blocks (distributed_attention.py:95-128 across
 * devices).  No KV block crosses NVLink.  Workspace: the size below,
 * zero-filled once (its leading region is oc_decode_step's).  Without
 * oc_sharded_connect the exchange is an NCCL all-gather of the packed
 * partials and a merge kernel; every rank must make the same calls. */
size_t oc_decode_step_sharded_workspace_bytes(int nranks, int batch, int q_len, int q_heads, int kv_heads,
                                              int head_dim, int seq_len);
/* Collective, once per workspace (after zero-filling it): map every rank's
 * exchange region (inside its workspace) into every other rank by CUDA IPC
 * (plain peer memory over NVLink; no multicast).  Afterwards
 * oc_decode_step_sharded on this workspace runs as ONE kernel per layer: the
 * fused layer's group merges store this shard's partial into every rank's
 * region, publish it with a release flag carrying the call number, wait
 * (bounded) for every rank's flag and merge the P partials — no NCCL kernel
 * and no host synchronisation in the step, so the step can be captured in
 * a CUDA graph.  All ranks agree on the outcome (a rank that cannot map the
 * regions makes every rank return an error and keep the NCCL path).  Needs
 * bf16, head_dim 128 and <= 8 query rows per KV head; the caller keeps the
 * workspace alive until oc_sharded_disconnect. */
int oc_sharded_connect(void* comm, void* workspace, size_t workspace_bytes, int batch, int q_len, int q_heads,
                       int kv_heads, int head_dim, int seq_len, oc_stream_t stream);
int oc_sharded_disconnect(void* workspace);
int oc_decode_step_sharded(void* comm, const void* q, const void* k, const void* v, int dtype, int batch,
                           int q_len, int q_heads, int kv_heads, int head_dim, int seq_len, float tau,
                           float zeta_max, uint8_t* keep, int32_t* perm, int32_t* count, void* out, int out_dtype,
                           void* workspace, size_t workspace_bytes, oc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ORTHOCACHE_B200_H */
