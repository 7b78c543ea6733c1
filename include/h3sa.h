/* h3sa — B200 (sm_100a) streaming audio-video attention: the C ABI.
 *
 * Plain pointers, sizes and a CUDA stream handle (cudaStream_t passed as void*); no
 * framework types. Every entry point validates its arguments on the host, enqueues work on
 * `stream` and returns without synchronising. Return value: H3SA_OK or an H3SA_ERR_* code;
 * h3sa_last_error() gives a message for the calling thread's most recent failure.
 *
 * Device-side failures (a page index outside its pool, a bounded wait that gave up) are
 * OR-ed into the optional `device_error` word (int32 in device memory) as H3SA_DEVERR_*
 * bits; the caller reads it when it next synchronises.
 *
 * Tensor layouts (row-major, contiguous, 16-byte aligned base pointers):
 *   packed rows  [rows, heads, head_dim]              the post-Ulysses q/k/v layout
 *   paged pool   [heads, pool_pages * 128, head_dim]  page p of head h = rows [128p, 128p+128)
 *   page table   int32 [table_blocks]: logical KV block b (rows [128b, 128b+128)) -> page
 * head_dim is 128 for the attention kernels.
 */
#ifndef H3SA_H_
#define H3SA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3SA_ABI_VERSION 1

#if defined(__GNUC__)
#define H3SA_API __attribute__((visibility("default")))
#else
#define H3SA_API
#endif

enum {
  H3SA_OK = 0,
  H3SA_ERR_INVALID = 1,     /* bad shape, size, pointer or alignment */
  H3SA_ERR_UNSUPPORTED = 2, /* valid request this build does not implement */
  H3SA_ERR_CUDA = 3         /* a CUDA runtime/driver call failed */
};

enum {
  H3SA_DEVERR_WAIT_TIMEOUT = 1, /* a pipeline wait gave up; outputs are invalid */
  H3SA_DEVERR_BAD_PAGE = 2,     /* page-table entry outside the pool */
  H3SA_DEVERR_BAD_INDEX = 4     /* row or block index outside its range */
};

/* One attention problem of a launch: queries [q_lo, q_hi) of the packed query tensor attend
 * to logical KV rows [kv_lo, kv_hi) of the page sequence; the result goes to the same rows
 * of the output. sparse != 0 restricts each 128-row query block to the KV blocks listed for
 * it (flex BlockMask layout, see h3sa_attention_fwd). */
typedef struct h3sa_problem {
  int32_t q_lo, q_hi;
  int32_t kv_lo, kv_hi;
  int32_t sparse;
  int32_t reserved[3];
} h3sa_problem;

/* A row space for the KV copy kernels: packed rows or a paged pool. */
typedef struct h3sa_rows {
  void* base;
  int32_t paged;              /* 0: packed [extent, heads, head_dim]; 1: paged pool */
  int32_t extent;             /* packed: rows; paged: pool_pages */
  const int32_t* page_table;  /* paged only */
  int32_t table_blocks;       /* paged only */
  int32_t reserved;
} h3sa_rows;

H3SA_API int h3sa_abi_version(void);
H3SA_API const char* h3sa_last_error(void);
H3SA_API size_t h3sa_attention_smem_bytes(int fp8);

/* Non-causal softmax(Q K^T * softmax_scale) V in bf16 with fp32 accumulation.
 * query/out: packed [rows, heads, 128] bf16. key_pool/value_pool: paged [heads, pool_pages*128,
 * 128] bf16. Up to 4 problems per launch. Block-sparse problems read kv_num_blocks
 * [heads, q_blocks] and kv_indices [heads, q_blocks, kv_index_stride] (int32, device; each
 * list sorted ascending, absolute logical block indices); q-block j of a problem covers query
 * rows [q_lo + 128j, q_lo + 128j + 128). Dense-only launches pass NULL lists.
 * Block-sparse problems spanning more than 64 KV blocks run split-KV: a query block with a
 * long list (launches with a block-sparse problem give every query block its own list) is
 * processed as up to 4 KV segments whose partial results are merged on the device. Their workspace belongs to the (device, stream) pair and is grown on demand;
 * growing it allocates device memory and waits for the device, so it must not happen during
 * stream capture (make one uncaptured call of the same size first). Launches on one stream
 * share it; launches on different streams get their own.
 *
 * Replaces: the FlashAttention-3 calls of the streaming hook and the K/V concatenation in
 * front of them (T/streaming/attention_hook.py:77-92; F/streaming/attention_hook.py:288-316,
 * 1068-1110), and the compiled flex_attention block-sparse call
 * (F/inference/dynamic_block_sparse.py:127-172). */
H3SA_API int h3sa_attention_fwd(const void* query, void* out, int32_t rows, int32_t heads,
                       int32_t head_dim, const void* key_pool, const void* value_pool,
                       int32_t pool_pages, const int32_t* page_table, int32_t table_blocks,
                       const h3sa_problem* problems, int32_t num_problems, float softmax_scale,
                       const int32_t* kv_num_blocks, const int32_t* kv_indices,
                       int32_t q_blocks, int32_t kv_index_stride, int32_t* device_error,
                       void* stream);

/* h3sa_attention_fwd with the Ulysses heads -> sequence exchange fused into the output store:
 * query row r (of `rows`, the all-rank sequence) is written, for local head h, to
 * out_peers[r / out_rows_per_rank] (a device array of out_ranks device addresses, this rank's
 * IPC mappings of every rank's [out_rows_per_rank, out_heads, 128] bf16 output) at row
 * r % out_rows_per_rank, head out_head0 + h. The stores go over NVLink to the other ranks;
 * the caller orders them with the readers (a barrier after the launch on every rank).
 * Replaces heads_to_sequence after the hook (T/distributed/ulysses.py:77-84): the O
 * all-to-all and its layout copies. */
H3SA_API int h3sa_attention_fwd_scatter(const void* query, int32_t rows, int32_t heads,
                               int32_t head_dim, const void* key_pool, const void* value_pool,
                               int32_t pool_pages, const int32_t* page_table,
                               int32_t table_blocks, const h3sa_problem* problems,
                               int32_t num_problems, float softmax_scale,
                               const int32_t* kv_num_blocks, const int32_t* kv_indices,
                               int32_t q_blocks, int32_t kv_index_stride,
                               const uint64_t* out_peers, int32_t out_ranks,
                               int32_t out_rows_per_rank, int32_t out_heads, int32_t out_head0,
                               int32_t* device_error, void* stream);

/* The same attention on e4m3 query and KV pools with per-head dequantisation scales
 * (q_scale, k_scale, v_scale: fp32 [heads], device), bf16 output: the FP8 FlashAttention-3
 * call with q/k/v_descale (F/streaming/attention_hook.py:1081-1107). */
H3SA_API int h3sa_attention_fwd_fp8(const void* query, void* out, int32_t rows, int32_t heads,
                           int32_t head_dim, const void* key_pool, const void* value_pool,
                           int32_t pool_pages, const int32_t* page_table, int32_t table_blocks,
                           const h3sa_problem* problems, int32_t num_problems,
                           float softmax_scale, const float* q_scale, const float* k_scale,
                           const float* v_scale, const int32_t* kv_num_blocks,
                           const int32_t* kv_indices, int32_t q_blocks, int32_t kv_index_stride,
                           int32_t* device_error, void* stream);

/* The e4m3 attention over a segmented KV sequence whose parts carry their own per-head
 * scales: the FP8 history the reference quantises once per committed block plus the current
 * parts quantised per call, all attended in one pass. block_part (int32 [table_blocks],
 * device) gives, for every logical KV block, its part index in the low 16 bits and its valid
 * rows (1..128) in the high 16 bits: every part starts on a 128-row block boundary and the
 * rows after it in its last block are masked (and should hold finite values, e.g. zeros).
 * part_k_scale / part_v_scale: fp32 [num_parts, heads]; q_scale fp32 [heads]. Scores use
 * q_scale * k_scale(part); P stays unscaled, O is accumulated in units of the current part's
 * V scale and rescaled by v_prev / v_new where the walk enters a part with another V scale,
 * so the result is attention over the dequantised parts.
 * Replaces the segmented FP8 FlashAttention-3 calls, one per part, and their LSE merge
 * (F/streaming/attention_hook.py:1015-1066, merge 319-334). */
H3SA_API int h3sa_attention_fwd_fp8_parts(
    const void* query, void* out, int32_t rows, int32_t heads, int32_t head_dim,
    const void* key_pool, const void* value_pool, int32_t pool_pages, const int32_t* page_table,
    int32_t table_blocks, const h3sa_problem* problems, int32_t num_problems, float softmax_scale,
    const float* q_scale, const int32_t* block_part, int32_t num_parts, const float* part_k_scale,
    const float* part_v_scale, const int32_t* kv_num_blocks, const int32_t* kv_indices,
    int32_t q_blocks, int32_t kv_index_stride, int32_t* device_error, void* stream);

/* Row copies between packed tensors and paged pools (num_tensors pairs, same indexing):
 * for i < count and every head, src row (src_index ? src_index[i] : src_start + i) goes to
 * dst row (dst_index ? dst_index[i] : dst_start + i). row_bytes = head_dim * element size
 * (a multiple of 16). Replaces the index_select / torch.cat traffic of the clean KV cache
 * (T/streaming/cache.py:156-171 stage, 188-199 commit, 246-284 retention). */
H3SA_API int h3sa_kv_copy_rows(const h3sa_rows* src, const h3sa_rows* dst, int32_t num_tensors,
                      const int32_t* src_index, int32_t src_start, const int32_t* dst_index,
                      int32_t dst_start, int32_t count, int32_t heads, int32_t row_bytes,
                      int32_t* device_error, void* stream);

/* Per-(batch, head) absmax e4m3 quantiser: x [batch, seq, heads, dim] bf16 -> y e4m3 of the
 * same shape and scale fp32 [batch, heads], scale = max(amax / 448, 1e-12),
 * y = RTNE(clamp(x / scale, -448, 448)). Uses a device scratch of
 * batch * heads * ceil(seq / 256) floats taken from the stream-ordered allocator.
 * Replaces quantize_fp8_e4m3_per_head (F/inference/fused_kernels.py:823-877). */
H3SA_API int h3sa_quantize_fp8_per_head(const void* x, void* y, float* scale, int32_t batch,
                               int32_t seq, int32_t heads, int32_t dim, void* stream);

/* The same quantiser, same arguments and results, but it allocates no device memory: its
 * scratch is a fixed 256 KiB device array inside the library, so
 * batch * heads * ceil(seq / 256) must be at most 65536 (H3SA_ERR_INVALID otherwise). It is
 * for callers that may not allocate while they run (a caller that owns all device memory
 * through its own pool, or one running where the stream-ordered allocator must not be
 * touched). The first call on each device looks up the array's device address with that
 * device current; make that first call before any stream capture. The array is shared by
 * every call on a device: calls whose device work can overlap (unordered streams, several
 * host threads) race on it and must be serialised by the caller. No counterpart in the
 * reference. */
H3SA_API int h3sa_quantize_fp8_per_head_noalloc(const void* x, void* y, float* scale,
                                                int32_t batch, int32_t seq, int32_t heads,
                                                int32_t dim, void* stream);

/* The same quantiser over logical KV rows [0, rows) of a paged bf16 pool, written to an e4m3
 * pool through the same page table: one scale per head over the whole logical sequence, as
 * the FP8 dynamic backend quantises the concatenated K (or V) parts
 * (F/streaming/attention_hook.py:1081-1098). */
H3SA_API int h3sa_quantize_fp8_pool(const void* pool, void* pool_fp8, float* scale, int32_t heads,
                           int32_t pool_pages, const int32_t* page_table, int32_t table_blocks,
                           int32_t rows, int32_t* device_error, void* stream);

/* The per-head e4m3 quantiser over one part of a row space, the form a segmented FP8 history
 * needs: rows [src_start, src_start + count) of num_tensors (1 or 2, e.g. K and V) bf16 row
 * spaces (packed or paged, 256-byte rows) are quantised, each tensor with its own per-head
 * scale max(amax / 448, 1e-12) over those rows (fp32 [heads] in scale0 / scale1), into e4m3
 * row spaces (128-byte rows) at [dst_start, dst_start + count). zero_tail != 0 writes zeros
 * into the destination rows after the part up to the end of its 128-row block (paged
 * destinations), so the block's unused rows hold finite values. amax_workspace: uint32
 * [num_tensors * heads] of device memory owned by the caller, cleared on `stream` first; calls
 * that share it must be ordered. Same arithmetic and results as h3sa_quantize_fp8_per_head on
 * those rows. Replaces the commit-time quantisation of a history block and the per-call
 * quantisation of the current parts (F/streaming/cache.py:835-855;
 * F/streaming/attention_hook.py:1029-1049). */
H3SA_API int h3sa_quantize_fp8_rows(const h3sa_rows* src, const h3sa_rows* dst,
                                    int32_t num_tensors, int32_t src_start, int32_t dst_start,
                                    int32_t count, int32_t heads, float* scale0, float* scale1,
                                    uint32_t* amax_workspace, int32_t zero_tail,
                                    int32_t* device_error, void* stream);

/* Column means of bf16 rows per segment, the summaries of commit-level top-k selection:
 * for segment i = (first logical row, rows) of segments (int32 [num_segments][2], device) and
 * every head, means[i][head][d] = fp32 mean over the segment's rows of src[row][head][d] (src
 * packed or paged, 256-byte rows; max_rows >= every segment's rows). Sums are fp64 in
 * `workspace` (double [num_segments * heads * 128], device, cleared on `stream` first); the
 * mean is their fp64 quotient rounded to fp32. Replaces key.float().mean(dim=0) of a committed
 * history block (F/streaming/cache.py:854, after retention :1031-1034) and
 * media_query.float().mean(dim=0) (F/streaming/attention_hook.py:1279). */
H3SA_API int h3sa_segment_row_means(const h3sa_rows* src, const int32_t* segments,
                                    int32_t num_segments, int32_t max_rows, int32_t heads,
                                    double* workspace, float* means, int32_t* device_error,
                                    void* stream);

/* Commit-level top-k scores: scores[i] (fp64, device) = mean over heads of the dot product of
 * summaries[i] (fp32 [num_parts][heads][128]) with query_mean (fp32 [heads][128]), products
 * and sums in fp64. Replaces history_summary.mul(query_summary).sum(-1).mean(-1)
 * (F/streaming/attention_hook.py:1281-1286); the top-k itself runs on the host, where the
 * reference reads the selection back (.tolist(), :1287-1290). */
H3SA_API int h3sa_commit_scores(const float* summaries, const float* query_mean,
                                int32_t num_parts, int32_t heads, double* scores, void* stream);

/* Rectangular SOL-Attn: query [query_tokens, heads, 128] bf16 against one packed K/V
 * sequence key / value [key_tokens, heads, 128] bf16, cut into 64-row blocks. The first
 * ceil(sink_tokens / 64) key blocks are exact for every query; the rest are routed per 64-row
 * query block and head: exact when the block's mean proxy score (query rows . key centroid,
 * times softmax_scale * log2(e)) exceeds mu + tau * sqrt(var + 1e-6), mu and var the proxy
 * score's mean and diagonal variance over the key centroids; every other block enters the
 * softmax through its centroid, weighted by its row count, with its V sum as value. Scratch
 * and side outputs, all device memory: key_centroids and value_sums bf16
 * [ceil(key_tokens / 64), heads, 128]; key_stats fp32 [heads, 2, 128]; exact_blocks uint32
 * [heads, ceil(query_tokens / 64), ceil(key_blocks / 32)] (bit b of a query block's words =
 * key block b is exact); telemetry int64 [4] or NULL, to which the launch adds the counts of
 * routed, exact, routable and candidate blocks. out bf16 [query_tokens, heads, 128]. Up to
 * 4096 key blocks (262144 key rows); every pointer 16-byte aligned. Replaces
 * sol_attn_rectangular without a static summary cache (F/inference/sol_attention.py:366-598),
 * the FL2AV hook's sol_attn backend call (F/streaming/attention_hook.py:909-991). */
H3SA_API int h3sa_sol_attention(const void* query, int32_t query_tokens, const void* key,
                                const void* value, int32_t key_tokens, int32_t heads,
                                int32_t head_dim, float softmax_scale, float tau,
                                int32_t sink_tokens, void* key_centroids, void* value_sums,
                                float* key_stats, uint32_t* exact_blocks, int64_t* telemetry,
                                void* out, int32_t* device_error, void* stream);

/* W8A8 projection GEMM (tcgen05 kind::i8, int32 accumulation in TMEM):
 * out[m, n] = bf16_rn(a_scale[m] * (b_scale[n] * float(sum_k a[m, k] * b[n, k])))
 * a: int8 [m, k] activations, b: int8 [n, k] weights (both row-major, K contiguous);
 * a_scale fp32 [m], b_scale fp32 [n]; out bf16 [m, ldo]. k a multiple of 16, n and ldo of 8,
 * every pointer 16-byte aligned. Replaces vLLM's cutlass_scaled_mm under the reference's W8A8
 * QKV / FC1 projection (T/inference/w8a8.py:190-221). */
H3SA_API int h3sa_w8a8_gemm(const void* a, const float* a_scale, const void* b,
                            const float* b_scale, void* out, int32_t m, int32_t n, int32_t k,
                            int32_t ldo, int32_t* device_error, void* stream);

/* bf16 GEMM on the same tcgen05 kernel (kind::f16, fp32 accumulation in TMEM):
 * out[m, n] = bf16_rn(sum_k a[m, k] * b[n, k]), a bf16 [m, k], b bf16 [n, k] (K contiguous,
 * k a multiple of 8, n and ldo of 8, 16-byte aligned). With partial_peers (device array of
 * `ranks` addresses, each rank's partial buffer [ranks][m][ldo] bf16 mapped here), the tile
 * is also stored into slot `slot` of every rank's buffer over NVLink: the row-parallel
 * out_proj's local product with its TP all-reduce exchange fused in (T/model/layers.py:441-443,
 * T/distributed/linear.py:186-191). out may be NULL then. */
H3SA_API int h3sa_gemm_bf16(const void* a, const void* b, void* out, int32_t m, int32_t n,
                            int32_t k, int32_t ldo, const uint64_t* partial_peers, int32_t ranks,
                            int32_t slot, int32_t* device_error, void* stream);

/* out[m, n] = bf16_rn(sum over t = 0 .. ranks-1 of slots[t][m][n]) (fp32 sum in rank order),
 * slots bf16 [ranks][m][ldo]: the reduction half of the TP all-reduce after h3sa_gemm_bf16
 * stored every rank's partial (T/distributed/collectives.py:51-55). */
H3SA_API int h3sa_tp_reduce(const void* slots, void* out, int32_t m, int32_t n, int32_t ldo,
                            int32_t ranks, void* stream);

/* Per-row int8 quantisation of bf16 rows x [rows, cols] into q int8 [rows, cols] and scale fp32
 * [rows] (cols a multiple of 8). mode 0 (activations, dynamic per token):
 * scale = amax / 127, q = clamp(rint(x * (127 / amax)), -128, 127), zero rows give zeros;
 * mode 1 (weights): scale = max(amax / 127, 1e-12), q = clamp(rint(x / scale), -127, 127).
 * Replaces scaled_int8_quant of the W8A8 input and _quantize_weight
 * (T/inference/w8a8.py:56-63, 190-221). */
H3SA_API int h3sa_quantize_int8_rows(const void* x, void* q, float* scale, int32_t rows,
                                     int32_t cols, int32_t mode, void* stream);

/* Generic layout permute of 16-byte-aligned records: for every index (i0, i1, i2, i3) of
 * the row-major space dims[4], copy row_bytes from src + sum(i_k * src_strides[k]) to
 * dst + sum(i_k * dst_strides[k]) (strides in bytes, multiples of 16). Serves the Ulysses
 * send/receive layouts: [T, 3, W, H/W, d] -> [W, 3, T, H/W, d] before the QKV all-to-all and
 * the inverse moves around the output all-to-all (T/distributed/ulysses.py:10-55, 103-132;
 * F/distributed/ulysses_layout.py:8-60). */
H3SA_API int h3sa_permute_rows(const void* src, void* dst, const int64_t* dims,
                               const int64_t* src_strides, const int64_t* dst_strides,
                               int32_t row_bytes, void* stream);

/* QK-RMSNorm + rotate-half RoPE in place on merged QKV [tokens, 3, heads, head_dim] bf16
 * (V untouched): inv = 1/sqrt(mean(v^2) + eps), n = bf16(v * inv * w), rope = bf16(bf16(n *
 * cos) + bf16(rot(n) * sin)) on dims [0, rotary). cos_sin: bf16 [cache_rows, rotary] (cos in
 * the first rotary/2 columns, sin in the rest); positions: int64 [tokens] rows of it.
 * Replaces fused_qkv_qk_norm_rope_ (T/inference/fused_kernels.py:805-855). */
H3SA_API int h3sa_qkv_norm_rope(void* qkv, const void* q_weight, const void* k_weight,
                                const void* cos_sin, int32_t cache_rows, int32_t rotary,
                                const int64_t* positions, int32_t tokens, int32_t heads,
                                int32_t head_dim, float eps, int32_t* device_error, void* stream);

/* The same prologue reading merged QKV and writing Q, K (normalised, rotated) and V into the
 * Ulysses send layout [world, 3, tokens, heads/world, head_dim] in one pass: the prologue
 * and the send-side permute of merged_qkv_sequence_to_heads (T/distributed/ulysses.py:
 * 103-132) fused. */
H3SA_API int h3sa_qkv_norm_rope_pack(const void* qkv, void* send, const void* q_weight,
                                     const void* k_weight, const void* cos_sin,
                                     int32_t cache_rows, int32_t rotary,
                                     const int64_t* positions, int32_t tokens, int32_t heads,
                                     int32_t head_dim, int32_t world, float eps,
                                     int32_t* device_error, void* stream);

/* The prologue fused with the sequence -> heads exchange and the cache append: this rank's
 * merged QKV shard [tokens, 3, heads, 128] bf16 (straight from the QKV projection, not
 * modified) is normalised and rotated, and every row is stored at the rank owning its head:
 * Q rows into peer_q[owner] (a [world * tokens, heads / world, 128] plane, row
 * rank * tokens + t), K and V rows into the owner's paged pools peer_key_pool[owner] /
 * peer_value_pool[owner] ([heads / world, pool_pages * 128, 128] bf16) at logical row
 * dst_start + rank * tokens + t through page_table (the same on every rank of the group).
 * world = 1 with this rank's own addresses writes the local plane and cache. A page-table
 * entry outside the pool sets H3SA_DEVERR_BAD_PAGE and the row is skipped. The caller orders
 * the stores with the readers (a barrier before attention).
 * Replaces, in one kernel: fused_qkv_qk_norm_rope_ (T/inference/fused_kernels.py:805-855),
 * merged_qkv_sequence_to_heads (T/distributed/ulysses.py:103-132) and the cache's copy of the
 * chunk's K/V (T/streaming/cache.py:133-171). */
H3SA_API int h3sa_qkv_norm_rope_scatter_paged(
    const void* qkv, const void* q_weight, const void* k_weight, const void* cos_sin,
    int32_t cache_rows, int32_t rotary, const int64_t* positions, int32_t tokens, int32_t heads,
    int32_t head_dim, int32_t world, int32_t rank, const uint64_t* peer_q,
    const uint64_t* peer_key_pool, const uint64_t* peer_value_pool, int32_t pool_pages,
    const int32_t* page_table, int32_t table_blocks, int32_t dst_start, float eps,
    int32_t* device_error, void* stream);

/* The e4m3 form of the fused prologue: RMSNorm + RoPE + per-head e4m3 quantisation, writing
 * Q and the chunk's K/V part straight into the owners' e4m3 planes and paged, head-major
 * caches. Two passes over this rank's merged QKV shard:
 * 1. h3sa_qkv_norm_rope_amax: amax (uint32 [3][heads], float bits, cleared first) receives
 *    the max |x| of every plane and head over the rotated rows whose amax_rows flag is set
 *    (uint8 [tokens], NULL: every row). With world > 1 the caller reduces the words with MAX
 *    over the Ulysses group: an NCCL all-reduce of 3 * heads int32, or h3sa_publish_words
 *    into every rank's [world][3 * heads] slots followed by a peer barrier, pass 2 then
 *    taking the maximum over amax_sets = world sets.
 * 2. h3sa_qkv_norm_rope_scatter_fp8: the rows again, quantised with scale = max(amax / 448,
 *    1e-12) (the arithmetic of h3sa_quantize_fp8_rows: same bytes), Q into peer_q8[owner]
 *    ([world * tokens, heads / world, 128] e4m3), K / V into the owners' e4m3 pools
 *    ([heads / world, pool8_pages * 128, 128]) at logical row dst8_start + rank * tokens + t of
 *    page_table8; this rank's heads' scales into q_scale / k_scale / v_scale (fp32 [heads /
 *    world]); with peer_q / peer_key_pool non-NULL the bf16 Q / K / V rows go to the bf16
 *    plane and pools as h3sa_qkv_norm_rope_scatter_paged stores them (with
 *    bf16_unflagged_only, only the rows whose amax_rows flag is 0). amax holds amax_sets
 *    consecutive [3][heads] sets whose maximum is used. */
/* Copies `count` words into slot `rank` of every rank's [world][count] slot array
 * (peer_slots: device array of the `world` arrays' addresses), visible to the other GPUs when
 * the kernel completes: the group maximum of the e4m3 prologue over peer memory. No reference
 * counterpart (it replaces a small all-reduce). */
H3SA_API int h3sa_publish_words(const uint32_t* words, const uint64_t* peer_slots, int32_t world,
                                int32_t rank, int32_t count, void* stream);
/* The two passes of the e4m3 prologue described above. Together they replace
 * fused_qkv_qk_norm_rope_ (T/inference/fused_kernels.py:805-855), the per-head
 * quantisation of Q and of the current K / V part (F/inference/fused_kernels.py:823-877 as
 * called at F/streaming/attention_hook.py:1026-1049), and the exchange and cache append. */
H3SA_API int h3sa_qkv_norm_rope_amax(const void* qkv, const void* q_weight, const void* k_weight,
                                     const void* cos_sin, int32_t cache_rows, int32_t rotary,
                                     const int64_t* positions, int32_t tokens, int32_t heads,
                                     int32_t head_dim, const uint8_t* amax_rows, uint32_t* amax,
                                     float eps, int32_t* device_error, void* stream);
H3SA_API int h3sa_qkv_norm_rope_scatter_fp8(
    const void* qkv, const void* q_weight, const void* k_weight, const void* cos_sin,
    int32_t cache_rows, int32_t rotary, const int64_t* positions, int32_t tokens, int32_t heads,
    int32_t head_dim, int32_t world, int32_t rank, const uint32_t* amax, int32_t amax_sets,
    const uint8_t* amax_rows, int32_t bf16_unflagged_only, const uint64_t* peer_q8,
    const uint64_t* peer_key_pool8, const uint64_t* peer_value_pool8, int32_t pool8_pages,
    const int32_t* page_table8, int32_t table8_blocks, int32_t dst8_start, float* q_scale,
    float* k_scale, float* v_scale, const uint64_t* peer_q, const uint64_t* peer_key_pool,
    const uint64_t* peer_value_pool, int32_t pool_pages, const int32_t* page_table,
    int32_t table_blocks, int32_t dst_start, float eps, int32_t* device_error, void* stream);

/* Block-sparse selection policy for h3sa_block_mask. */
typedef struct h3sa_mask_policy {
  int32_t mode;                   /* 0: history top-k, 1: composite */
  int32_t n_hist;                 /* history rows: logical KV rows [0, n_hist) */
  int32_t n_kv;                   /* logical KV rows of the attention */
  int32_t sinks;                  /* mode 1: leading KV blocks always kept */
  int32_t window;                 /* mode 1: +- band of KV blocks around a query block */
  int32_t reserved;
  double density;                 /* (0, 1] */
  const uint8_t* q_block_audio;   /* mode 1: [q blocks] 1 if the block holds an audio query */
  const uint8_t* kv_block_audio;  /* mode 1: [KV blocks] 1 if the block holds an audio key */
} h3sa_mask_policy;

/* Per (head, 128-row query block of rows [q_lo, q_hi)) KV block selection written as the
 * flex BlockMask inputs kv_num_blocks int32 [heads, q blocks] and kv_indices int32
 * [heads, q blocks, kv_index_stride] (ascending, zero padded). Scores are block-mean dot
 * products in fixed-order fp64; mode 0 restates _dynamic_history_mask
 * (F/inference/dynamic_block_sparse.py:50-124). Uses fp64 block-mean scratch from the
 * stream-ordered allocator. */
H3SA_API int h3sa_block_mask(const void* query, int32_t rows, int32_t heads, int32_t head_dim,
                             int32_t q_lo, int32_t q_hi, const void* key_pool,
                             int32_t pool_pages, const int32_t* page_table,
                             int32_t table_blocks, const h3sa_mask_policy* policy,
                             int32_t* kv_num_blocks, int32_t* kv_indices,
                             int32_t kv_index_stride, int32_t* device_error, void* stream);

/* Peer memory for the fused Ulysses exchanges (no counterpart in the reference, whose
 * exchange is torch.distributed.all_to_all_single over NCCL). h3sa_peer_alloc returns
 * cudaMalloc memory that h3sa_ipc_handle exports (a 64-byte cudaIpcMemHandle_t) and that
 * another process on the node maps with h3sa_ipc_open (close with h3sa_ipc_close). */
H3SA_API int h3sa_peer_alloc(size_t bytes, void** ptr);
H3SA_API int h3sa_peer_free(void* ptr);
H3SA_API int h3sa_ipc_handle(const void* ptr, void* handle);
H3SA_API int h3sa_ipc_open(const void* handle, void** ptr);
H3SA_API int h3sa_ipc_close(void* ptr);

/* Sequence -> heads exchange as one kernel: this rank's merged QKV shard
 * [tokens, 3, heads, 128] bf16 (post prologue) is stored straight into the attention-ready
 * q/k/v planes [3, world * tokens, heads / world, 128] of the rank owning each head, at rows
 * [rank * tokens, (rank + 1) * tokens). peer_qkv: device array of world device addresses (this
 * rank's IPC mappings of every rank's planes). Replaces merged_qkv_sequence_to_heads
 * (T/distributed/ulysses.py:103-132): the send permute, the all-to-all and the receive
 * permute. The caller orders the stores with the readers (a barrier before attention). */
/* Barrier of the ranks of one node over peer memory, ordered on `stream`: stores `epoch`
 * into slot `rank` of every rank's uint32 flag array (peer_flags: device array of world device
 * addresses, this rank's mappings of every rank's array, zero-initialised) and waits until its
 * own array holds at least `epoch` in every slot. Work enqueued after it on any rank starts
 * after every rank's work enqueued before it. `epoch` must grow by one per call (wrapping
 * compare); a wait that gives up after 2 s sets H3SA_DEVERR_WAIT_TIMEOUT in device_error. */
H3SA_API int h3sa_peer_barrier(const uint64_t* peer_flags, int32_t world, int32_t rank,
                               uint32_t epoch, int32_t* device_error, void* stream);

/* h3sa_peer_barrier with the caller's wait limit limit_ns in (0, 60 s] instead of 2 s: a rank
 * that has not arrived by then leaves this rank's wait with H3SA_DEVERR_WAIT_TIMEOUT set, so a
 * dead or late peer shows up as a device error word the host reads, never as a hung stream.
 * Counterpart of the reference's collective error path, which gathers every rank's failure
 * into one error for the caller (T/runtime/direct.py:227-237). */
H3SA_API int h3sa_peer_barrier_limit(const uint64_t* peer_flags, int32_t world, int32_t rank,
                                     uint32_t epoch, int64_t limit_ns, int32_t* device_error,
                                     void* stream);

H3SA_API int h3sa_scatter_qkv(const void* merged, int32_t tokens, int32_t heads,
                              int32_t head_dim, int32_t world, int32_t rank,
                              const uint64_t* peer_qkv, void* stream);

/* h3sa_scatter_qkv with the cache append folded in: Q rows go to peer_q[owner] (a
 * [world * tokens, heads / world, 128] plane, row rank * tokens + t), K and V rows straight into
 * the owner's paged pools peer_key_pool[owner] / peer_value_pool[owner] ([heads / world,
 * pool_pages * 128, 128] bf16) at logical row dst_start + rank * tokens + t through page_table,
 * which must be the same on every rank (the ranks of a Ulysses group commit the same rows).
 * A page-table entry outside the pool sets H3SA_DEVERR_BAD_PAGE and the row is skipped.
 * Replaces: merged_qkv_sequence_to_heads (T/distributed/ulysses.py:103-132) followed by the
 * cache's stage/commit copy of the current chunk's K/V (T/streaming/cache.py:133-171). */
H3SA_API int h3sa_scatter_qkv_paged(const void* merged, int32_t tokens, int32_t heads,
                                    int32_t head_dim, int32_t world, int32_t rank,
                                    const uint64_t* peer_q, const uint64_t* peer_key_pool,
                                    const uint64_t* peer_value_pool, int32_t pool_pages,
                                    const int32_t* page_table, int32_t table_blocks,
                                    int32_t dst_start, int32_t* device_error, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* H3SA_H_ */
