/*
 * C ABI of libaether_b200.so: sm_100a (B200) kernels for Aether-2B's CSA/HCA
 * decode path over a paged TurboQuant KV cache.
 *
 * Conventions
 *   - All pointers are device pointers unless stated; sizes are element counts.
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued, not waited.
 *   - Return 0 on success, 1 for an invalid argument, 2 for a CUDA error; the
 *     message is in aether_last_error() (thread-local).
 *   - `err` (optional, may be NULL) is a device int that kernels OR error bits
 *     into: 1 = a bounded wait expired, 2 = page id outside the pool,
 *     4 = a size exceeded a compiled limit.
 *   - dtype codes: 0 = float32, 1 = float16, 2 = bfloat16.
 *   - Cache pages: 64 entries per page stored as [64 code rows][64 fp32
 *     scales]; row bytes = dim * bits / 8 (4-bit codes: two's complement
 *     nibbles, even element in the low nibble).
 *
 * Reference citations are file:line inside itz-sayak/deepseek-v4-codebase.
 */
#ifndef AETHER_B200_H_
#define AETHER_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char* aether_last_error(void);
int aether_abi_version(void);
int aether_compiled_arch(void);

/* ---------------------------------------------------------------- TurboQuant
 * Replaces PolarQuant.encode (aether_2b/turbo_quant.py:127-166): codes are
 * bit-identical to the reference's fp32 path.  x [rows, d] (d = 64 or 128),
 * diag [d] the +-1 Rademacher diagonal (turbo_quant.py:111-121).
 * codes: int8 [rows, d] (bits 8) or uint8 [rows, d/2] (bits 4); scales [rows]. */
int aether_tq_encode(const void* x, int dtype, long long rows, int d, int bits, const float* diag,
                     uint8_t* codes, float* scales, int* err, void* stream);

/* Cache append (replaces aether_2b/serving.py:327-344 _quant_append): encodes
 * x [batch, rows_per_seq, d] and writes row i of sequence b at logical
 * position start_pos[b] + i of that sequence's pages in page_pool. */
int aether_tq_encode_into_pages(const void* x, int dtype, int batch, int rows_per_seq, int d, int bits,
                                const float* diag, const int32_t* page_table, int table_stride,
                                const int32_t* start_pos, int num_pages, uint8_t* page_pool, int* err,
                                void* stream);

/* Compress-on-emit for B finishing blocks, one call per stream (replaces
 * aether_2b/serving.py:495-505 _hca_emit and the main / index halves of
 * :540-575 _emit_csa_block; model form modeling.py:273-287, 437-482):
 *   out = RMSNorm(RoPE(sum_r softmax_r(z_r + bias_r) * c_r))   per channel,
 * softmax over the rows of segment 0 ([B, rows0, d] c0 / z0, bias0 [rows0, d]
 * or NULL) and, where has_seg1[b] != 0 (has_seg1 NULL = all), segment 1
 * (CSA's previous-block b half; rows1 = 0 for HCA).  RoPE (rope_dim = 0 to
 * skip) rotates the last rope_dim channels in interleaved pairs at
 * positions[b] with inv_freq [rope_dim/2] (modeling.py:122-155);
 * norm_weight [d] (NULL to skip) applies RMSNorm with norm_eps
 * (modeling.py:32-41).  The result is TurboQuant-encoded into the page slot
 * of logical position slot_pos[b] (page_table as aether_tq_encode_into_pages;
 * page_pool NULL to skip) and, if out is not NULL, stored as fp32 [B, d]. */
int aether_compress_emit(const void* c0, const void* z0, const float* bias0, int rows0, const void* c1,
                         const void* z1, const float* bias1, int rows1, const int32_t* has_seg1, int dtype, int B,
                         int d, const int32_t* positions, const float* inv_freq, int rope_dim,
                         const float* norm_weight, float norm_eps, int bits, const float* diag,
                         const int32_t* page_table, int table_stride, const int32_t* slot_pos, int num_pages,
                         uint8_t* page_pool, float* out, int* err, void* stream);

/* Replaces PolarQuant.decode (aether_2b/turbo_quant.py:168-211). */
int aether_tq_decode(const uint8_t* codes, const float* scales, long long rows, int d, int bits,
                     const float* diag, void* out, int out_dtype, void* stream);

/* Lloyd-Max level format (alternative to the uniform levels; no reference
 * counterpart).  Encode: y = WHT(diag * x), scale = max|y| / cmax, code =
 * number of the 2^bits - 1 ascending fp32 `thresholds` (level midpoints)
 * strictly below y / scale; codes uint8 [rows, d] (8-bit) or index nibbles
 * [rows, d/2] (4-bit, even element low).  Decode: x = diag * WHT(levels[code]
 * * scale).  The codebook is aether_kernels/codebook.py (Lloyd's algorithm for
 * N(0, 1)). */
int aether_tq_encode_lut(const void* x, int dtype, long long rows, int d, int bits, const float* diag,
                         const float* thresholds, float cmax, uint8_t* codes, float* scales, void* stream);
int aether_tq_decode_lut(const uint8_t* codes, const float* scales, long long rows, int d, int bits,
                         const float* diag, const float* levels, void* out, int out_dtype, void* stream);

/* Normalised Walsh-Hadamard transform, fp32 (aether_2b/turbo_quant.py:49-76). */
int aether_wht(const float* x, float* out, long long rows, int d, void* stream);

/* ------------------------------------------------ reference extension ops
 * Replaces sparse_sink_attention (aether_kernels/csrc/bindings.cpp:21-46,
 * sparse_sink_attention_cuda.cu:118-177).  q [B,T,H,D], kv [B,S,2,D],
 * topk_indices [B,T,K] int32 or int64 (entries outside [0,S) skipped),
 * sink scalar or [H], all in `dtype`; out [B,T,H,D]. */
int aether_sparse_sink_attention(const void* q, const void* kv, const void* topk_indices, int idx_is_int64,
                                 const void* sink, int sink_numel, void* out, int dtype, int B, int T, int H, int D,
                                 int S, int K, float softmax_scale, void* stream);

/* Replaces tiled_prefill_attention (bindings.cpp:58-77): every target token
 * attends to all S sources; the sink enters the denominator once. */
int aether_tiled_prefill_attention(const void* q, const void* kv, const void* sink, int sink_numel, void* out,
                                   int dtype, int B, int T, int H, int D, int S, float softmax_scale, int tile_size,
                                   void* stream);

/* Replaces csa_indexer_topk (bindings.cpp:88-101) with the canonical score
 * sum_h softplus(w_h) * relu(q_h . k_s) (aether_2b/modeling.py:609-611);
 * out [B,k] int64 ordered by (score desc, index asc).  `scratch` holds
 * aether_csa_indexer_topk_scratch_bytes(B, S) bytes. */
size_t aether_csa_indexer_topk_scratch_bytes(int B, int S);
int aether_csa_indexer_topk(const float* index_q, const float* index_kv, const float* index_weight, int B, int IH,
                            int IC, int S, int k, float* scratch, int64_t* out, void* stream);

/* Variant of aether_csa_indexer_topk that allocates nothing; it has no
 * counterpart in the reference.  For callers that cannot allocate device
 * memory where they call the indexer (host callbacks, allocator hooks, code
 * running while another stream is being captured, plugins handed only their
 * input and output buffers): the score buffer is a fixed array inside the
 * library, B * S <= aether_csa_indexer_topk_noalloc_max_scores() (1 Mi scores,
 * 4 MiB held on every GPU that loads the library until exit).  Larger sizes
 * return 1 with a message.  The first call on a device (that device current)
 * looks up the array's address; make it before any stream capture.  Calls
 * share the array: calls whose kernels overlap on the GPU race. */
long long aether_csa_indexer_topk_noalloc_max_scores(void);
int aether_csa_indexer_topk_noalloc(const float* index_q, const float* index_kv, const float* index_weight, int B,
                                    int IH, int IC, int S, int k, int64_t* out, void* stream);

/* Replaces hca_compress (bindings.cpp:110-119): softmax over the window of
 * buffer_z per channel, weighted sum of buffer_c; out [B,D]. */
int aether_hca_compress(const void* buffer_c, const void* buffer_z, void* out, int dtype, int B, int M, int D,
                        void* stream);

/* ------------------------------------------------- fused paged decode
 * One CSA decode step for B sequences (replaces the data flow of
 * aether_2b/serving.py:597-625 + the backend call at :450-467):
 *   q [B,H,128] bf16, index_q [B,4,64] fp32, index_w [B,4] fp32 raw head
 *   weights, sink [H] fp32, window [B,W,128] bf16 (window_len[b] valid rows,
 *   oldest first), idx_pages / kv_pages page pools, page_table [B,table_stride]
 *   int32, nblocks [B] visible compressed blocks (<= max_nblocks <= 262144;
 *   sequences over 8192 blocks are selected in two levels),
 *   diag_idx [64] / diag_kv [128] Rademacher diagonals.
 * out [B,H,128] bf16 (attention output before the inverse output RoPE),
 * sel_out [B,top_k] int32 selected block ids ascending, -1 padded (may be NULL).
 * workspace: aether_csa_decode_workspace_bytes(B, max_nblocks) bytes of device
 * memory for per-block score keys (cluster 0 only; contents need no clearing).
 * cluster: 0 = score kernel + select/attend kernel (default); 4 or 8 = one
 * thread-block cluster per sequence.
 * pdl: 1 = programmatic dependent launch; the kernel then reads page_table,
 * nblocks, window_len, cache pages and all window rows but the newest before
 * the previous kernel in the stream has completed. */
int aether_csa_decode_paged(const void* q, const float* index_q, const float* index_w, const float* sink,
                            const void* window, const int32_t* window_len, const uint8_t* idx_pages,
                            const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                            const int32_t* nblocks, int max_nblocks, const float* diag_idx, const float* diag_kv,
                            int B, int H, int W, int bits, int top_k, float softmax_scale, void* out,
                            int32_t* sel_out, uint32_t* workspace, int* err, int cluster, int pdl, void* stream);

/* As aether_csa_decode_paged (cluster 0) with the inverse output RoPE fused
 * into the final store (aether_2b/serving.py:469-472): the last rope_dim
 * channels (a multiple of 4) of every head's output are rotated in
 * interleaved pairs by -rope_pos[b] * rope_inv_freq[i] (rope_inv_freq
 * [rope_dim / 2], e.g. get_rope_freqs of modeling.py:60-99). */
int aether_csa_decode_paged_rope(const void* q, const float* index_q, const float* index_w, const float* sink,
                                 const void* window, const int32_t* window_len, const uint8_t* idx_pages,
                                 const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                                 const int32_t* nblocks, int max_nblocks, const float* diag_idx, const float* diag_kv,
                                 int B, int H, int W, int bits, int top_k, float softmax_scale, void* out,
                                 int32_t* sel_out, uint32_t* workspace, int* err, int pdl, const int32_t* rope_pos,
                                 const float* rope_inv_freq, int rope_dim, void* stream);

/* As aether_csa_decode_paged (cluster 0) for a cache in the Lloyd-Max level
 * format (PolarQuant(bits, codebook="lloyd-max")): codes are indices into
 * levels [2^bits] fp32 (4-bit: index nibbles, even element in the low
 * nibble), an entry is levels[code] * scale in the rotated domain.  The level
 * table is applied inside the kernels: the index scores in fp32 (the exact
 * integer limb MMAs need integer codes), the attention through its code LUT.
 * Not in the reference (its PolarQuant has uniform levels only,
 * aether_2b/turbo_quant.py:150-166). */
int aether_csa_decode_paged_levels(const void* q, const float* index_q, const float* index_w, const float* sink,
                                   const void* window, const int32_t* window_len, const uint8_t* idx_pages,
                                   const uint8_t* kv_pages, const int32_t* page_table, int table_stride,
                                   int num_pages, const int32_t* nblocks, int max_nblocks, const float* diag_idx,
                                   const float* diag_kv, int B, int H, int W, int bits, int top_k,
                                   float softmax_scale, const float* levels, void* out, int32_t* sel_out,
                                   uint32_t* workspace, int* err, int pdl, void* stream);

/* As aether_hca_decode_paged (cluster 0) for a cache in the Lloyd-Max level
 * format (see aether_csa_decode_paged_levels). */
int aether_hca_decode_paged_levels(const void* q, const float* sink, const void* window, const int32_t* window_len,
                                   const uint8_t* kv_pages, const int32_t* page_table, int table_stride,
                                   int num_pages, const int32_t* nblocks, int max_nblocks, const float* diag_kv,
                                   int B, int H, int W, int bits, float softmax_scale, const float* levels,
                                   void* out, int* err, int pdl, void* stream);

/* As aether_csa_decode_paged, also writing each visible block's index score
 * to score_out[b * score_stride + block]. */
int aether_csa_decode_paged_scores(const void* q, const float* index_q, const float* index_w, const float* sink,
                                   const void* window, const int32_t* window_len, const uint8_t* idx_pages,
                                   const uint8_t* kv_pages, const int32_t* page_table, int table_stride,
                                   int num_pages, const int32_t* nblocks, int max_nblocks, const float* diag_idx,
                                   const float* diag_kv, int B, int H, int W, int bits, int top_k,
                                   float softmax_scale, void* out, int32_t* sel_out, float* score_out,
                                   int score_stride, uint32_t* workspace, int* err, int cluster, int pdl,
                                   void* stream);

/* aether_csa_decode_paged with host buffers: one call enqueues the copy of
 * in_bytes of packed step inputs from pinned host_in to dev_in, the decode
 * (score + select/attend kernels), and the copy of out_bytes of packed
 * results from dev_out to pinned host_out.  q, index_q, index_w, window_len,
 * nblocks point into dev_in; out, sel_out into dev_out.  h2d_stream,
 * d2h_stream and the staging slot's events ev_h2d / ev_comp / ev_d2h
 * (cudaEvent_t) are optional (NULL: everything in order on `stream`); with
 * them the input copy waits for the slot's previous decode, the decode for the
 * input copy and the slot's previous output copy, and the output copy for the
 * decode, so callers alternating two slots overlap copies with kernels.
 * slot_flags (optional, with copy streams): two device u32 words per staging
 * slot, zero before its first step, and seq = 1, 2, 3, ... per slot.  The
 * copy streams then publish copy completion by writing seq into the words
 * (stream memory operations) and the kernels poll them with bounded waits, so
 * the decode stream carries no cross-stream wait and consecutive steps keep
 * their programmatic-launch overlap.  A poll that runs out sets bit 1 of *err. */
int aether_csa_decode_paged_host(const void* host_in, void* dev_in, size_t in_bytes, void* host_out,
                                 const void* dev_out, size_t out_bytes, const void* q, const float* index_q,
                                 const float* index_w, const float* sink, const void* window,
                                 const int32_t* window_len, const uint8_t* idx_pages, const uint8_t* kv_pages,
                                 const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                                 int max_nblocks, const float* diag_idx, const float* diag_kv, int B, int H, int W,
                                 int bits, int top_k, float softmax_scale, void* out, int32_t* sel_out,
                                 uint32_t* workspace, int* err, int pdl, void* stream, void* h2d_stream,
                                 void* d2h_stream, void* ev_h2d, void* ev_comp, void* ev_d2h, uint32_t* slot_flags,
                                 uint32_t seq);

/* A prepared host-buffer CSA decode.  create binds what stays fixed across
 * steps: two staging slots (dev_in0/1 and dev_out0/1, packed as
 * aether_csa_decode_paged_host expects, with the device offsets of
 * q / index_q / index_w / window_len / nblocks in in_offsets[5] and of
 * out / sel_out in out_offsets[2]), four zeroed device u32 copy-completion
 * words (slot_flags), the cache, the launch shape, the workspace (sized for
 * table_stride pages, the widest page table a step may pass) and the error
 * word.  The plan owns two copy streams and six events.  Each step
 * passes only its pinned host buffers, the layer's page table, sink and
 * window, the scale and the decode stream, and uses the next staging slot
 * (alternating), so a step's copies overlap its neighbours' kernels.  The
 * per-step host cost is one short call instead of the 45-argument entry.
 * destroy waits for the plan's copies.  After a failed step, destroy the
 * plan. */
int aether_csa_decode_host_plan_create(void* dev_in0, void* dev_in1, size_t in_bytes, const size_t* in_offsets,
                                       void* dev_out0, void* dev_out1, size_t out_bytes, const size_t* out_offsets,
                                       uint32_t* slot_flags, const uint8_t* idx_pages, const uint8_t* kv_pages,
                                       int table_stride, int num_pages, int max_nblocks, const float* diag_idx,
                                       const float* diag_kv, int B, int H, int W, int bits, int top_k,
                                       uint32_t* workspace, int* err, int pdl, void** plan_out);
int aether_csa_decode_host_plan_step(void* plan, const void* host_in, void* host_out, const int32_t* page_table,
                                     int table_stride, const float* sink, const void* window, float softmax_scale,
                                     void* stream);
/* Orders the plan's copy streams against `stream`: wait_for_copies 0 makes
 * later copies start after the work enqueued on `stream` so far, 1 makes later
 * work on `stream` start after every copy the plan has enqueued so far. */
int aether_csa_decode_host_plan_fence(void* plan, void* stream, int wait_for_copies);
void aether_csa_decode_host_plan_destroy(void* plan);

/* One HCA decode step (replaces aether_2b/serving.py:507-522): attention over
 * every visible compressed block plus the window; nblocks <= 1024.
 * cluster 0: a 4-CTA cluster per sequence that stages the pages, their fp16
 * expansion and all window rows but the newest before waiting on the previous
 * kernel when pdl is set (programmatic dependent launch: only when that
 * kernel writes none of them); 4 or 8: the older one-kernel cluster path
 * (pdl ignored). */
int aether_hca_decode_paged(const void* q, const float* sink, const void* window, const int32_t* window_len,
                            const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                            const int32_t* nblocks, int max_nblocks, const float* diag_kv, int B, int H, int W,
                            int bits, float softmax_scale, void* out, int* err, int cluster, int pdl,
                            void* stream);

/* ------------------------------------------ context-parallel decode
 * New design (the reference has no multi-GPU attention): a
 * sequence's compressed blocks are split into contiguous ranges, one per
 * device; this device holds blocks [id_base, id_base + nblocks[b]).
 *
 * Step 1: exact top_k of each 8192-block chunk of this device's range.
 * cand_keys / cand_ids [B][chunks * top_k] (chunks = ceil(max_nblocks/8192),
 * top_k a multiple of 4): order-preserving u32 score keys and global block
 * ids, ascending; padding has key 0 and id -1.  workspace: as for
 * aether_csa_decode_paged. */
int aether_csa_local_candidates(const float* index_q, const float* index_w, const uint8_t* idx_pages,
                                const int32_t* page_table, int table_stride, int num_pages, const int32_t* nblocks,
                                int max_nblocks, const float* diag_idx, int B, int bits, int top_k, int id_base,
                                uint32_t* cand_keys, int32_t* cand_ids, void* workspace, int* err, void* stream);

/* Step 2: exact top_k over the all-gathered candidate lists (cand_n entries
 * per row, ids ascending), attention over the winners held here plus this
 * device's window rows (window_len 0 where the window lives elsewhere).
 * part_o [B][H][128] and part_ml [B][H][2] (max logit, sum of exponentials)
 * receive the un-normalised partial result; with them NULL, out [B][H][128]
 * bf16 receives the final one.  sel_out [B][top_k] (optional): global winners. */
int aether_csa_attend_candidates(const void* q, const float* sink, const void* window, const int32_t* window_len,
                                 const uint8_t* kv_pages, const int32_t* page_table, int table_stride, int num_pages,
                                 const int32_t* nblocks, int max_nblocks, const float* diag_kv,
                                 const uint32_t* cand_keys, const int32_t* cand_ids, int cand_n, int cand_stride,
                                 int id_base, int B, int H, int W, int bits, int top_k, float softmax_scale, void* out,
                                 int32_t* sel_out, float* part_o, float* part_ml, int* err, void* stream);

/* Step 3: log-sum-exp merge of G partials [G][B][H][128] / [G][B][H][2] with
 * the sink counted once (aether_pipeline/serving.py:99-130 softmax over the
 * union of the source sets); out [B][H][128] bf16. */
int aether_lse_merge(const float* part_o, const float* part_ml, const float* sink, int G, int B, int H, void* out,
                     void* stream);

/* ------------------------------------------------ chunked prefill
 * Indexer top-k for the query tokens of prefill chunks against the paged
 * cache (the per-query-row indexer of aether_2b/modeling.py:605-615 with the
 * causal block mask s < t // compression of :612-614), on tcgen05 tensor
 * cores.  R requests: req_info [R][4] int32 = (first row of the request's
 * queries in index_q / index_w / the outputs, number of queries, absolute
 * position t of its first query, compressed blocks held in the cache, its
 * own chunk's blocks included); request r uses page_table row r.
 * tiles [ntiles][2] int32 = (request, first query within the request), one
 * per 32 consecutive queries.  index_q [Q][4][64], index_w [Q][4] fp32 raw.
 * cand_keys / cand_ids [Q][top_k]: order-preserving u32 score keys and block
 * ids of the exact top min(top_k, t // compression) blocks (score desc, lower
 * block first among equal scores), ids ascending, padding key 0 / id -1;
 * top_k <= 256.  The rows feed aether_csa_attend_candidates. */
int aether_csa_prefill_topk(const float* index_q, const float* index_w, const uint8_t* idx_pages,
                            const int32_t* page_table, int table_stride, int num_pages, const int32_t* req_info,
                            const int32_t* tiles, int ntiles, int compression, const float* diag_idx, int bits,
                            int top_k, uint32_t* cand_keys, int32_t* cand_ids, int* err, void* stream);

/* The optional low-precision indexer of the paper's CSA indexer path
 * (Aether.txt:765-769, 1087-1093; no counterpart kernel in the reference
 * code): as aether_csa_prefill_topk, with the scores computed on e4m3
 * operands on tcgen05 (kind::f8f6f4).  The rotated index query is quantised
 * to e4m3 per (query, head) with scale max|q| / 448; 4-bit codes are exact in
 * e4m3, 8-bit codes are rounded to it.  The rows are the exact top-k of those
 * scores: they match the exact indexer's only up to a recall below 1. */
int aether_csa_prefill_topk_fp8(const float* index_q, const float* index_w, const uint8_t* idx_pages,
                                const int32_t* page_table, int table_stride, int num_pages, const int32_t* req_info,
                                const int32_t* tiles, int ntiles, int compression, const float* diag_idx, int bits,
                                int top_k, uint32_t* cand_keys, int32_t* cand_ids, int* err, void* stream);

/* Chunked-prefill attention (aether_2b/modeling.py:616-640 per query row):
 * query b attends the blocks of its candidate row (cand_keys / cand_ids from
 * aether_csa_prefill_topk, cand_stride >= top_k) plus its window, with the
 * sink.  q [B][H][128] bf16; page-table row q_row[b]; visible blocks
 * nblocks[b] (<= max_nblocks); window rows win_row[b] .. win_row[b] +
 * window_len[b] - 1 (oldest first, window_len <= 128) of the flat bf16
 * buffer window [rows][128].  out [B][H][128] bf16 (before the inverse output
 * RoPE); sel_out [B][top_k] (optional) the attended block ids.  Runs as one
 * persistent CTA per SM on the tcgen05 tensor cores (top_k <= 256, H <= 16). */
int aether_csa_prefill_attend(const void* q, const float* sink, const void* window, const long long* win_row,
                              const int32_t* window_len, const uint8_t* kv_pages, const int32_t* page_table,
                              int table_stride, int num_pages, const int32_t* q_row, const int32_t* nblocks,
                              int max_nblocks, const float* diag_kv, const uint32_t* cand_keys,
                              const int32_t* cand_ids, int cand_stride, int B, int H, int bits, int top_k,
                              float softmax_scale, void* out, int32_t* sel_out, int* err, void* stream);

/* As aether_lse_merge with rank r's partials at part_o + r * stride_o and
 * part_ml + r * stride_ml (float elements; part_o rows 16-byte aligned), e.g.
 * the rows of one all-gathered buffer packing each rank's O and (max, sum). */
int aether_lse_merge_strided(const float* part_o, const float* part_ml, long long stride_o, long long stride_ml,
                             const float* sink, int G, int B, int H, void* out, void* stream);

/* Workspace bytes of aether_csa_decode_paged (cluster 0). */
size_t aether_csa_decode_workspace_bytes(int B, int max_nblocks);

/* Shared-memory bytes of the select/attend CSA decode kernel. */
int aether_csa_decode_smem_bytes(int bits);

/* ---- peer-memory exchange for context-parallel decode (no counterpart in
 * the reference, which has no multi-GPU decode; it replaces the two NCCL
 * all-gathers of a context-parallel step).  One process per GPU.  Each rank
 * creates one exchange buffer and shares its 64-byte CUDA IPC handle; the
 * others open it.  The first aether_cp_control_bytes() bytes of a buffer are
 * its control area (flag words and the step word).
 *
 * aether_peer_push: copy `rows` rows of `row_bytes` (row stride src_stride)
 * from local device memory into every buffer bases[0..G-1] at
 * dst_offset + dst_col + row * dst_stride, then raise this rank's flag of
 * `kind` (0..3) in every buffer to the step number.  bump = 1 starts a new
 * step (the local step word is incremented first).  Sizes, strides and
 * offsets are multiples of 16 bytes; dst_offset lies past the control area.
 * aether_peer_wait: stream-ordered wait until all G flags of `kind` in the
 * local buffer reach the local step number; bounded (0.2 s), a timeout sets
 * the wait-timeout bit of *err. */
long long aether_cp_control_bytes(void);
int aether_cp_buffer_create(long long bytes, void** ptr, void* ipc_handle);
int aether_cp_buffer_open(const void* ipc_handle, void** ptr);
int aether_cp_buffer_close(void* ptr);
int aether_cp_buffer_destroy(void* ptr);
int aether_peer_push(const void* src, long long rows, long long row_bytes, long long src_stride, void* const* bases,
                     int G, int rank, long long dst_offset, long long dst_stride, long long dst_col, int kind,
                     int bump, void* stream);
int aether_peer_wait(const void* local_base, int G, int kind, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AETHER_B200_H_ */
