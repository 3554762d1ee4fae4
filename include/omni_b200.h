/*
 * omni_b200 — C ABI of the B200-native talker decode step.
 *
 * Every entry point takes raw device pointers, element counts and strides
 * (in elements), and a CUDA stream (cudaStream_t passed as void*; NULL is the
 * legacy default stream).  Launches are asynchronous; no entry point
 * synchronises the device or reads device memory on the host, so each can be
 * captured in a CUDA graph.
 *
 * Dtypes are fixed per argument and named in the comment: bf16 = 16-bit
 * brain float (uint16_t storage), f32, i64, i32, u8.
 *
 * Return codes mirror the reference's error conventions
 * (sglang_omni/models/qwen3_tts/sampling_kernels.py:847-866 returns None for
 * an unsupported contract; shape violations raise ValueError, capacity
 * RuntimeError):
 */
#ifndef OMNI_B200_H_
#define OMNI_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OMNI_OK 0
#define OMNI_ERR_UNSUPPORTED 1 /* outside the kernel's contract: caller keeps its own path */
#define OMNI_ERR_INVALID 2     /* malformed arguments (ValueError)                       */
#define OMNI_ERR_CAPACITY 3    /* a fixed capacity would be exceeded (RuntimeError)      */
#define OMNI_ERR_CUDA 4        /* the CUDA launch itself failed                           */

#if defined(_WIN32)
#define OMNI_API __declspec(dllexport)
#else
#define OMNI_API __attribute__((visibility("default")))
#endif

/* Library version string and the last error message of the calling thread. */
OMNI_API const char* omni_version(void);
OMNI_API const char* omni_last_error(void);

/* Sticky device status written by bounded waits that gave up (0 = none).
 * reset != 0 clears it.  Synchronous: reads device memory. */
#define OMNI_DEV_TIMEOUT_TMA 0x100u  /* a wait for copies into shared memory gave up */
#define OMNI_DEV_TIMEOUT_MMA 0x200u  /* a wait for tensor-core work gave up */
#define OMNI_DEV_BAD_INDEX 0x300u    /* an index outside its table was skipped */
#define OMNI_DEV_TIMEOUT_FLAG 0x400u /* a wait on a flag in global memory gave up */
OMNI_API unsigned int omni_device_status(int reset);

/* ======================================================================== */
/* Sampling                                                                 */
/* ======================================================================== */

/* Seeded temperature / top-k / top-p sampling from raw bf16 logits.
 * Replaces sample_from_logits_with_seed_top_k_top_p
 * (sglang_omni/models/qwen3_tts/sampling_kernels.py:836-950; kernel :441-529).
 *   logits      bf16 [rows, vocab], row stride logits_stride (16-byte aligned rows)
 *   temperatures f32 [rows]; top_ks i64 [rows]; top_ps f32 [rows];
 *   seeds i64 [rows]; positions i64 [rows]
 *   max_top_k   graph-signature width, one of 4 8 16 32 50 64 128 256 512 1024
 *   has_top_p   0/1
 *   out         i64 [rows]
 * vocab in [block width, 4096], multiple of 8. */
OMNI_API int omni_sample_topk_topp(const void* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                   const float* temperatures, const int64_t* top_ks, const float* top_ps,
                                   const int64_t* seeds, const int64_t* positions, int32_t max_top_k,
                                   int32_t has_top_p, int64_t* out, void* stream);

/* One residual-codebook step of the code predictor, fused: sample (or argmax
 * for rows whose do_sample is 0) the codebook token from the lm_head logits,
 * write it to codes[row * codes_stride], and gather its embedding row:
 * gathered[row] = table[token] and summed[row] = bf16(summed[row] + table[token]).
 * Replaces the pair sample_subtalker_token (sglang_model.py:1918-1952) +
 * gather_codec_embedding_and_add (predictor_kernels.py:87-229) of
 * code_predictor_forward_incremental (sglang_model.py:1819-1878).
 * The seed position of a row is positions[row] * pos_mul + pos_add
 * (sub_seed_positions, sglang_model.py:1908-1916).
 *   do_sample  u8 [rows] or NULL (all rows sampled); argmax_all != 0 takes argmax on every row
 *   table      bf16 [vocab, hidden]; gathered, summed bf16 [rows, hidden] or NULL
 *   gathered_ss f32 [rows] or NULL: sum of squares of each gathered row (the
 *   next pass's folded RMSNorm input, see omni_linear_fused) */
OMNI_API int omni_predictor_sample_step(const void* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                        const float* temperatures, const int64_t* top_ks, const float* top_ps,
                                        const int64_t* seeds, const int64_t* positions, int64_t pos_mul,
                                        int64_t pos_add, const uint8_t* do_sample, int32_t argmax_all,
                                        int32_t max_top_k, int32_t has_top_p, int64_t* codes, int64_t codes_stride,
                                        const void* table, int64_t hidden, void* gathered, void* summed,
                                        float* gathered_ss, void* stream);

/* Seeded Gumbel-max over pre-sorted fp32 log-probabilities.
 * Replaces sample_from_sorted_logprobs_with_seed_small_k
 * (sampling_kernels.py:721-790; kernel :81-121).
 *   logprobs f32 [rows, cols]; sorted_idx i64 [rows, cols]; cols <= 1024 */
OMNI_API int omni_sample_sorted_seeded(const float* logprobs, const int64_t* sorted_idx, int64_t rows,
                                       int64_t cols, const int64_t* seeds, const int64_t* positions, int64_t* out,
                                       void* stream);

/* Greedy codebook step: code = argmax(logits) (first NaN, else first maximum),
 * codes[row * codes_stride] = code, gathered[row] = table[code] (nullable),
 * summed[row] += table[code] (bf16, nullable).
 * Replaces codebook_step (sglang_omni/utils/predictor_layers.py:963-993). */
OMNI_API int omni_codebook_step(const void* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                const void* table, int64_t hidden, int64_t* codes, int64_t codes_stride,
                                void* gathered, void* summed, void* stream);

/* gathered[row] = table[token_ids[row]]; accumulated[row] += gathered[row] (bf16);
 * with projected_table != NULL also projected[row] = projected_table[token].
 * token_ids are i64 (token_is_i32 = 0) or i32 (1).
 * Replaces gather_codec_embedding_and_add (predictor_kernels.py:87-229). */
OMNI_API int omni_gather_embedding_add(const void* token_ids, int32_t token_is_i32, int64_t rows,
                                       const void* table, int64_t hidden, void* gathered, void* accumulated,
                                       const void* projected_table, int64_t projected_size, void* projected,
                                       void* stream);

/* Layer-0 (talker codec head) sampling: repetition penalty on rep_mask
 * columns (l > 0 ? l / p : l * p), suppression to -inf, temperature, full
 * softmax, top-k / top-p / min-p, seeded Gumbel draw over the sorted ranks.
 * Replaces Qwen3OmniTalker.sample_decode_tokens
 * (sglang_omni/models/qwen3_omni/components/talker.py:1376-1412) and the
 * sglang sampler it hands off to.
 *   logits f32 [rows, vocab] row stride logits_stride; vocab % 4 == 0, <= 8192
 *   penalties f32 [rows]; rep_mask, suppress_mask u8 [rows, vocab] or NULL
 *   temperatures, top_ps, min_ps (nullable) f32 [rows]; top_ks, seeds, positions i64 [rows]
 *   max_top_k <= 1024: the widest top_k of the batch.
 *   rep_mask_update u8 [rows, vocab] or NULL: the drawn token is marked 1 (the
 *   next step's repetition mask: prepare_decode_buffers, talker.py:1065-1215). */
OMNI_API int omni_layer0_sample(const float* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                const float* penalties, const uint8_t* rep_mask, const uint8_t* suppress_mask,
                                const float* temperatures, const int64_t* top_ks, const float* top_ps,
                                const float* min_ps, const int64_t* seeds, const int64_t* positions,
                                int32_t max_top_k, int64_t* out, uint8_t* rep_mask_update, void* stream);

/* First pass of the code predictor for one frame (code_predictor_forward_incremental,
 * sglang_model.py:1784-1813) with the talker's final RMSNorm
 * (talker.py:482-491) applied on the way: hidden = bf16(h * rstd * final_norm)
 * where rstd comes from the per-row sums of squares ss_in of the talker's last
 * residual h (ss_parts parts, see omni_linear_fused); hidden goes to
 * hidden_out (nullable) and to pair row 2 r; e = table[layer0_codes[r]] goes
 * to pair row 2 r + 1 and to summed; codes[r * codes_stride] = layer0_codes[r];
 * pair_ss[2 r], pair_ss[2 r + 1] = the pair rows' sums of squares.
 *   talker_residual bf16 [rows, hidden]; table bf16 [vocab, hidden];
 *   pair bf16 [2 rows, hidden]; summed, hidden_out bf16 [rows, hidden].
 *   final_norm_weight NULL: talker_residual is already the normalized hidden state
 *   (the reference's code_predictor_forward input) and is copied unchanged; ss_in
 *   is then not read. */
OMNI_API int omni_predictor_pair_inputs(const int64_t* layer0_codes, const void* talker_residual,
                                        int64_t residual_stride, const void* final_norm_weight, const float* ss_in,
                                        int32_t ss_parts, int64_t ss_stride, float eps, void* hidden_out,
                                        const void* table, int64_t rows, int64_t hidden, void* pair, void* summed,
                                        float* pair_ss, int64_t* codes, int64_t codes_stride, void* stream);


/* ======================================================================== */
/* Projections (tcgen05 tensor cores)                                       */
/* ======================================================================== */

#define OMNI_EPI_STORE 0    /* y = bf16(x W^T)                                   */
#define OMNI_EPI_RESIDUAL 1 /* y = bf16(x W^T + residual) (residual may alias y) */
#define OMNI_EPI_SWIGLU 2   /* W = [gate; up] (2I x K): y[:, :I] = silu(g) * u   */
#define OMNI_EPI_F32 3      /* y = x W^T in f32 (logits)                          */

/* Bytes of global workspace omni_linear needs for this shape: always 0 (the
 * split-K partials go through a 24 MiB scratch array inside the library, reduced
 * by the owning CTA of each cluster; GEMM launches that overlap on the GPU, other
 * than consecutive launches on one stream under programmatic dependent launch,
 * must be serialised). */
OMNI_API int64_t omni_linear_workspace_bytes(int64_t rows, int64_t k, int64_t n, int32_t epilogue, int32_t splits);

/* y[rows, N] = epilogue(x[rows, K] . w[N, K]^T): the decode-step linears
 * (QKVParallelLinear / RowParallelLinear / MergedColumnParallelLinear +
 * SiluAndMul / codec_head / lm_head of thinker_model.py:152-402,
 * talker.py:216-247, sglang_model.py:1294-1302, 2101-2152).
 *   x, w, residual bf16; y bf16 (f32 for OMNI_EPI_F32); K % 64 == 0, N % 128 == 0.
 *   splits: K-splits per 128-feature tile (one thread-block cluster each),
 *   0 = chosen by the library so that one wave covers the GPU, else 1..16
 *   (narrowed when a wide row tile exceeds shared memory or the grid's split
 *   partials exceed the scratch array).  With 0, a batch of more than 256 rows
 *   with a (row tile, feature tile) pair for every SM runs a persistent
 *   tile-loop kernel without split (store, residual and SwiGLU epilogues; the
 *   same bits as one split).
 *   workspace / workspace_bytes: unused (may be NULL / 0). */
OMNI_API int omni_linear(const void* x, int64_t rows, int64_t k, int64_t x_stride, const void* w, int64_t n,
                         int32_t epilogue, const void* residual, int64_t residual_stride, void* y, int64_t y_stride,
                         void* workspace, int64_t workspace_bytes, int32_t splits, void* stream);

#define OMNI_EPI_QKV_ROPE 4 /* qkv projection + per-head RMSNorm + neox RoPE + KV store */
#define OMNI_EPI_ROUTER 5   /* MoE router: bf16 logits + softmax, top-k, renormalise   */

/* Arguments of omni_linear_fused (unused fields zero).  Replaces, in one launch,
 * the chain RMSNorm -> linear [-> residual add] of the decoder layers
 * (thinker_model.py:259-402, talker.py:216-247, predictor_forward_tokens
 * sglang_model.py:2036-2098) and, with OMNI_EPI_QKV_ROPE, also apply_qk_norm +
 * rotary_emb(FusedSetKVBufferArg) (thinker_model.py:272-345):
 *   - folded RMSNorm: w holds the layer's weight times the norm gain (column
 *     scaled); the accumulator of row r is scaled by
 *     rsqrt(sum_p ss_in[p * ss_in_stride + r] / norm_dim + norm_eps);
 *   - ss_out (store / residual epilogues): per-row sum of squares of the bf16
 *     output, one part per 128-feature tile (part t at ss_out + t * ss_out_stride),
 *     the next folded RMSNorm's ss_in;
 *   - OMNI_EPI_QKV_ROPE: y receives q [rows, Hq * head_dim]; k and v go to
 *     k_cache / v_cache [slots, Hkv, head_dim] at cache_loc (or the implicit
 *     predictor slots, as omni_qknorm_rope_store). */
typedef struct OmniLinearArgs {
  const void* x;
  int64_t rows, k, x_stride;
  const void* w;
  int64_t n;
  int32_t epilogue;
  int32_t splits;
  const float* ss_in;
  int32_t ss_in_parts;
  int64_t ss_in_stride;
  int32_t norm_dim;
  float norm_eps;
  const void* residual;
  int64_t residual_stride;
  void* y;
  int64_t y_stride;
  float* ss_out;
  int64_t ss_out_stride;
  int32_t num_q_heads, num_kv_heads, head_dim;
  const void* q_norm;
  const void* k_norm;
  float qk_eps;
  const float* cos_sin;
  int64_t max_position;
  const int64_t* positions;
  const int64_t* cache_loc;
  int32_t tokens_per_req, slot_stride, slot_base;
  void* k_cache;
  void* v_cache;
  /* OMNI_EPI_ROUTER (N = 128 experts): y receives the bf16 router logits;
   * topk_ids [rows, top_k] int32 and topk_weights [rows, top_k] f32 the
   * experts by (softmax prob desc, index asc) and their renormalised probs
   * (TopK with renormalize, thinker_model.py:428-433, fused_topk). */
  int32_t* topk_ids;
  float* topk_weights;
  int32_t top_k;
  /* Optional L2 prefetch (nullable): the launch's CTAs prefetch these bytes into
   * L2 at their start, for a later launch on the stream (the next projection's
   * weights); 16-byte aligned, no effect on this GEMM's results. */
  const void* l2_prefetch;
  int64_t l2_prefetch_bytes;
} OmniLinearArgs;

OMNI_API int omni_linear_fused(const OmniLinearArgs* args, void* stream);

/* ======================================================================== */
/* Norms and rotary embedding                                               */
/* ======================================================================== */

/* out = RMSNorm(s) * weight with s = x (addend == NULL) or s = bf16(x + addend)
 * (written to residual_out when given): sglang RMSNorm(x) / RMSNorm(x, residual)
 * (vendor/sglang/layers.py:57-98; add_rmsnorm_rounded, predictor_layers.py:603-622).
 * hidden = 256 * {1,2,4,8,16,32}; bf16 rows 16-byte aligned. */
OMNI_API int omni_rmsnorm(const void* x, int64_t x_stride, const void* addend, int64_t addend_stride,
                          void* residual_out, int64_t residual_stride, const void* weight, float eps, void* out,
                          int64_t out_stride, int64_t rows, int64_t hidden, void* stream);

/* sum = bf16(a + b) (b nullable: a copy of a) and ss_out[r] = sum of squares of
 * row r of sum: the decode input row (write_feedback_buffers,
 * talker_model_runner.py:564-606: feedback embedding + text row) ahead of a
 * folded first RMSNorm.  hidden = 256 * {1,2,4,8}. */
OMNI_API int omni_add_sumsq(const void* a, int64_t a_stride, const void* b, int64_t b_stride, void* sum,
                            int64_t sum_stride, float* ss_out, int64_t rows, int64_t hidden, void* stream);

/* Per-head q/k RMSNorm, neox rotary embedding and the KV store
 * (apply_qk_norm + rotary_emb with FusedSetKVBufferArg, thinker_model.py:272-345;
 * predictor_cached_self_attention, sglang_model.py:2168-2233).
 *   qkv bf16 [rows, (Hq + 2 Hkv) head_dim]; cos_sin_cache f32 [max_position, head_dim]
 *   (cos in the first half, sin in the second).
 *   positions / cache_loc i64 [rows], or both NULL for the predictor layout:
 *   row r = (request r / T, token r % T), position = slot_base + r % T,
 *   slot = (r / T) * slot_stride + position.
 *   q_out bf16 [rows, Hq head_dim]; k_cache, v_cache bf16 [slots, Hkv, head_dim]. */
OMNI_API int omni_qknorm_rope_store(const void* qkv, int64_t qkv_stride, int64_t rows, int32_t num_q_heads,
                                    int32_t num_kv_heads, int32_t head_dim, const void* q_norm_weight,
                                    const void* k_norm_weight, float eps, const float* cos_sin_cache,
                                    int64_t max_position, const int64_t* positions, const int64_t* cache_loc,
                                    int32_t tokens_per_req, int32_t slot_stride, int32_t slot_base, void* q_out,
                                    int64_t q_stride, void* k_cache, void* v_cache, void* stream);

/* ======================================================================== */
/* Attention                                                                */
/* ======================================================================== */

/* Workspace bytes of omni_paged_decode_attention; -1 for negative sizes or a
 * byte count beyond 2^60 (the entry points reject those with OMNI_ERR_INVALID). */
OMNI_API int64_t omni_paged_attention_workspace_bytes(int64_t rows, int32_t num_kv_heads, int64_t work_capacity);

/* Paged-KV GQA decode attention (RadixAttention decode, thinker_model.py:373-379).
 *   q bf16 [rows, Hq, 128]; k_cache, v_cache bf16 [slots, Hkv, 128], page size 16;
 *   page_indptr i32 [rows+1] / page_indices i32 (page ids); seq_lens i64 [rows];
 *   out bf16 [rows, Hq, 128].
 *   The flattened page list is split into grid_ctas equal ranges per KV head (0 = two
 *   CTAs per SM over all KV heads); a row spread over several ranges is merged by a
 *   second launch.  work_capacity = partial segments the workspace holds: at least
 *   rows + ranges - 1 (fewer ranges are used when it is smaller).  workspace:
 *   omni_paged_attention_workspace_bytes(rows, Hkv, work_capacity), 256-byte aligned.
 *   work_indptr and pages_per_chunk are unused: they belonged to a fixed-size chunk
 *   list that the range partition replaced; they stay in the signature so that
 *   existing bindings keep working (pass NULL and any positive value).
 *   Programmatic dependent launch: the page table, seq_lens and every KV slot except
 *   each row's newest token are read before the kernel waits on its predecessor, so
 *   they must have been written before the previous kernel on the stream started (the
 *   previous kernel may store the new tokens' K/V and the queries). */
OMNI_API int omni_paged_decode_attention(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                                         const int32_t* page_indptr, const int32_t* page_indices,
                                         const int64_t* seq_lens, const int32_t* work_indptr, int64_t rows,
                                         int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                         int32_t page_size, int32_t pages_per_chunk, int64_t work_capacity,
                                         float sm_scale, void* out, int64_t out_stride, void* workspace,
                                         int64_t workspace_bytes, int32_t grid_ctas, void* stream);

/* omni_paged_decode_attention without a caller workspace; this entry point has
 * no counterpart in the reference.  For callers that may not allocate device
 * memory (a host that owns and budgets all device memory, or a real-time
 * audio thread that must not block in cudaMalloc): the scratch comes from an
 * 8 MiB array built into the library, one per GPU that loads it, held until
 * process exit.  Calls needing more than 8 MiB of scratch
 * (omni_paged_attention_workspace_bytes) fail with OMNI_ERR_CAPACITY.  All
 * calls on a device share the array: calls that overlap on the GPU race.
 * Every call writes the partial outputs it reads in the same call, so the
 * array needs no clearing between calls (its counter region is reserved and
 * unused).  The first call on a device resolves the array's address
 * (cudaGetSymbolAddress) with that device current; make it before any stream
 * capture. */
OMNI_API int omni_paged_decode_attention_noalloc(const void* q, int64_t q_stride, const void* k_cache,
                                                 const void* v_cache, const int32_t* page_indptr,
                                                 const int32_t* page_indices, const int64_t* seq_lens,
                                                 const int32_t* work_indptr, int64_t rows, int32_t num_q_heads,
                                                 int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                                 int32_t pages_per_chunk, int64_t work_capacity, float sm_scale,
                                                 void* out, int64_t out_stride, int32_t grid_ctas, void* stream);

/* The code predictor's attention over its per-request cache slots
 * (predictor_gqa_attention / decode_attention_kernel, sglang_model.py:113-150,
 * predictor_layers.py:336-396).  Row r = (request r / T, token r % T) attends to
 * slots [0, slot_base + r % T] of its request (causal for the opening pair). */
OMNI_API int omni_predictor_attention(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                                      int64_t rows, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                      int32_t tokens_per_req, int32_t slot_stride, int32_t slot_base, float sm_scale,
                                      void* out, int64_t out_stride, void* stream);

/* ======================================================================== */
/* Batch packing                                                            */
/* ======================================================================== */

/* prepare_for_decode + ForwardBatch metadata (omni_scheduler.py:2000-2022,
 * model_runner/base.py:577-623, talker_scheduler.py:198-225): seq_lens += 1, one
 * KV slot per row (a new page from free_pages[*free_head...] when
 * (seq_len - 1) % page_size == 0, pages taken in row order), req_to_token written,
 * positions = seq_len - 1, kv_indptr / kv_indices (token level, nullable),
 * page_indptr / page_indices, work_indptr (attention chunks, nullable).
 * status (nullable) becomes 1 if the free list ran dry. */
OMNI_API int omni_decode_prepare(int64_t rows, int64_t* seq_lens, const int64_t* req_pool_indices,
                                 int32_t* req_to_token, int64_t max_ctx, int32_t page_size, const int32_t* free_pages,
                                 int64_t num_free, int64_t* free_head, int64_t* out_cache_loc, int64_t* positions,
                                 int32_t* kv_indptr, int32_t* kv_indices, int32_t* page_indptr,
                                 int32_t* page_indices, int32_t* work_indptr, int32_t pages_per_chunk,
                                 int32_t* status, void* stream);

/* rollback_decode_prep_after_skip (talker_scheduler.py:198-225): free the pages
 * this step opened (their slots listed in freed_slots, count in num_freed),
 * seq_lens -= 1, req_to_token cleared at the rolled-back position. */
OMNI_API int omni_decode_rollback(int64_t rows, int64_t* seq_lens, const int64_t* req_pool_indices,
                                  int32_t* req_to_token, int64_t max_ctx, int32_t page_size,
                                  const int64_t* out_cache_loc, int64_t* free_head, int64_t* freed_slots,
                                  int64_t* num_freed, void* stream);

/* Batch compaction of the continuous-batching runner (the row moves of an
 * omni_sched_plan, include/omni_sched.h): for every move m and tensor t, row
 * dst[m] of tensor t becomes a copy of its row src[m].  bases / row_bytes /
 * row_strides (bytes) describe up to 24 per-row state tensors; bases, src and
 * dst are HOST arrays (passed by value to the kernel).  Sources and
 * destinations must be disjoint row sets. */
OMNI_API int omni_move_rows(void* const* bases, const int64_t* row_bytes, const int64_t* row_strides,
                            int32_t num_tensors, const int32_t* src, const int32_t* dst, int32_t num_moves,
                            void* stream);

/* Admission of n streams planned by omni_sched_schedule (prepare_for_extend's
 * req_to_token writes): stream i's req_to_token row slots[i] gets the slots of
 * its first prompt_lens[i] tokens from its pages (page_indptr / pages, i32
 * CSR), seq_lens[rows[i]] = prompt_lens[i], req_pool_indices[rows[i]] = slots[i].
 * All arrays on the device.  status (nullable) becomes 2 on a stream whose
 * pages cannot hold its prompt. */
OMNI_API int omni_admit_streams(int64_t n, const int32_t* rows, const int32_t* slots, const int64_t* prompt_lens,
                                const int32_t* page_indptr, const int32_t* pages, int32_t* req_to_token,
                                int64_t max_ctx, int32_t page_size, int64_t* seq_lens, int64_t* req_pool_indices,
                                int32_t* status, void* stream);

/* ---------------------------------------------------------------------------
 * MoE block (a9): Qwen3OmniMoeTalkerSparseMoeBlock.forward (talker.py:325-351)
 * over Qwen3OmniMoeThinkerTextSparseMoeBlock (thinker_model.py:405-470) with
 * block-FP8 experts (quantization.py:124-167).  The router is omni_linear_fused
 * with OMNI_EPI_ROUTER (gate + TopK(renormalize), thinker_model.py:428-433).
 * ------------------------------------------------------------------------- */

/* post_attention_layernorm (decoder layer, thinker_model.py) followed by
 * per_token_group_quant_fp8 (group 128) of its output, as FusedMoE's block-FP8
 * path does on entry: x = bf16(h * rsqrt(sum_p ss[p][row] / hidden + eps) *
 * gain); xq e4m3 [rows, hidden]; xs [rows, hidden / 128] f32 with
 * scale = max(amax, 1e-10) / 448.  hidden % 1024 == 0. */
OMNI_API int omni_moe_rmsnorm_quant(const void* h, int64_t h_stride, const float* ss, int32_t ss_parts,
                                    int64_t ss_stride, const void* gain, float eps, int64_t rows, int32_t hidden,
                                    void* x, int64_t x_stride, void* xq, float* xs, void* stream);

/* Work-list capacity (chunks of <= 32 rows) for tokens x top_k pairs. */
OMNI_API int64_t omni_moe_chunk_capacity(int64_t tokens, int32_t top_k, int32_t experts);

/* moe_align_block_size + the activation permute of FusedMoE: pairs (t, k)
 * sorted by expert, stable by token; slot_of [tokens, top_k] = row of the pair
 * in the sorted order; expert_offsets [experts + 1]; chunks int4 {expert,
 * first row, rows, 0} [chunk_capacity] and *n_chunks; permuted_q / permuted_s
 * receive the pairs' e4m3 rows and scales.  tokens <= 4096, top_k <= 8,
 * experts <= 256. */
OMNI_API int omni_moe_align_gather(const int32_t* topk_ids, int64_t tokens, int32_t top_k, int32_t experts,
                                   const void* xq, const float* xs, int32_t hidden, void* permuted_q,
                                   float* permuted_s, int32_t* slot_of, int32_t* expert_offsets, void* chunks,
                                   int64_t chunk_capacity, int32_t* n_chunks, void* stream);

/* FusedMoE w13 GEMM + SiluAndMul + per_token_group_quant_fp8 of the
 * activation, per sorted row: w13 e4m3 [experts][2 inter][hidden] (gate rows
 * then up rows), w13_scale f32 [experts][2 inter / 128][hidden / 128];
 * act_q e4m3 [rows_cap, inter], act_s f32 [rows_cap, inter / 128].
 * hidden <= 1024, both multiples of 128. */
OMNI_API int omni_moe_gate_up_fp8(const void* permuted_q, const float* permuted_s, int64_t rows_cap, int32_t hidden,
                                  const void* w13, const float* w13_scale, int32_t experts, int32_t inter,
                                  const void* chunks, const int32_t* n_chunks, void* act_q, float* act_s,
                                  void* stream);

/* FusedMoE w2 GEMM per sorted row: w2 e4m3 [experts][hidden][inter],
 * w2_scale f32 [experts][hidden / 128][inter / 128]; y bf16 [rows_cap, hidden]. */
OMNI_API int omni_moe_down_fp8(const void* act_q, const float* act_s, int64_t rows_cap, int32_t inter,
                               const void* w2, const float* w2_scale, int32_t experts, int32_t hidden,
                               const void* chunks, const int32_t* n_chunks, void* y, int64_t y_stride,
                               void* stream);

/* moe_sum of the routed outputs + the gated shared expert (talker.py:341-350)
 * + the decoder layer's residual add: h = bf16(h + bf16(bf16(sum_k w_k y[slot])
 * + bf16(shared * sigmoid(bf16(x . shared_gate_weight))))); ss_out
 * [hidden / 128, rows] (stride ss_stride) the new rows' per-128-feature sums
 * of squares (nullable). */
OMNI_API int omni_moe_combine(const void* y, int64_t y_stride, const int32_t* slot_of, const float* topk_weights,
                              int32_t top_k, const void* x, int64_t x_stride, const void* shared_gate_weight,
                              const void* shared_out, int64_t shared_stride, void* h, int64_t h_stride,
                              float* ss_out, int64_t ss_stride, int64_t rows, int32_t hidden, void* stream);

/* omni_moe_align_gather over strided inputs (rows of a receive buffer that packs
 * each token's e4m3 row, scales and local expert ids): ids_stride in int32
 * elements, xq_stride in bytes, xs_stride in floats.  An expert id of -1 marks an
 * entry with no local expert: skipped, slot_of -1.  tokens <= 4096. */
OMNI_API int omni_moe_align_gather_strided(const int32_t* topk_ids, int64_t ids_stride, int64_t tokens,
                                           int32_t top_k, int32_t experts, const void* xq, int64_t xq_stride,
                                           const float* xs, int64_t xs_stride, int32_t hidden, void* permuted_q,
                                           float* permuted_s, int32_t* slot_of, int32_t* expert_offsets,
                                           void* chunks, int64_t chunk_capacity, int32_t* n_chunks, void* stream);

/* Expert-parallel dispatch packing (the all-to-all send side of the EP variant of
 * the reference's FusedMoE, talker.py:325-351 with experts sharded over the ranks).
 * Rank d holds experts [d e, (d + 1) e), e = experts_per_rank.  Every token goes once
 * to each rank holding at least one of its top_k experts, as one packed row of
 * row_bytes: its e4m3 codes (hidden bytes), group scales (hidden / 128 floats), the k
 * expert ids local to that rank (-1 for the others) and the k routing weights.  The
 * row lands at send[d cap + j], j = the count of earlier tokens going to d (token
 * order); the unused rows of every block get ids -1; part_index[t][d] = d cap + j or
 * -1, the row of token t's returned partial.  tokens <= cap, world <= 32. */
OMNI_API int omni_moe_ep_pack(const int32_t* topk_ids, const float* topk_weights, int64_t tokens, int32_t top_k,
                              const void* xq, int64_t xq_stride, const float* xs, int64_t xs_stride, int32_t hidden,
                              int32_t world, int32_t experts_per_rank, int64_t cap, void* send, int64_t row_bytes,
                              int32_t* part_index, void* stream);

/* Expert-parallel combine side: the partial routed sum of one received row over the
 * experts this rank holds,
 * out[r] = bf16(sum_k w[r][k] * y[slot_of[r][k]]) over slot_of >= 0 (k order),
 * zero when none. */
OMNI_API int omni_moe_partial_sum(const void* y, int64_t y_stride, const int32_t* slot_of, const float* weights,
                                  int64_t weights_stride, int32_t top_k, int64_t rows, int32_t hidden, void* out,
                                  int64_t out_stride, void* stream);

/* omni_moe_combine with the routed sum given as up to n_parts bf16 partial rows per
 * token (parts row part_index[t][p], -1 = none), summed in p order. */
OMNI_API int omni_moe_combine_parts(const void* parts, int64_t parts_stride, const int32_t* part_index,
                                    int32_t n_parts, const void* x, int64_t x_stride, const void* shared_gate_weight,
                                    const void* shared_out, int64_t shared_stride, void* h, int64_t h_stride,
                                    float* ss_out, int64_t ss_stride, int64_t rows, int32_t hidden, void* stream);

/* ---------------------------------------------------------------------------
 * Extend (prefill) of new streams in a mixed batch (config 2's fused forward:
 * ScheduleBatch.prepare_for_extend + ForwardBatch.init_new in extend mode,
 * model_runner/base.py:577-623; compose_prefill_embeds talker_model_runner.py:
 * 347-425 supplies the rows).  The scheduler has reserved the new tokens' slots
 * in req_to_token; this packs seq_lens = prefix + extend, qo_indptr (cu_seqlens),
 * each new token's out_cache_loc and position (prefix + j), the page lists and,
 * with tile_indptr, the q-tile list of omni_prefill_attention (q_tile rows). */
OMNI_API int omni_extend_prepare(int64_t rows, const int64_t* prefix_lens, const int64_t* extend_lens,
                                 const int64_t* req_pool_indices, const int32_t* req_to_token, int64_t max_ctx,
                                 int32_t page_size, int64_t* seq_lens, int32_t* qo_indptr, int64_t* out_cache_loc,
                                 int64_t* positions, int32_t* page_indptr, int32_t* page_indices, int32_t* tile_indptr,
                                 int32_t q_tile, int32_t* status, void* stream);

/* Causal extend attention (RadixAttention extend, thinker_model.py:373-379) over
 * the paged pool: the extend rows of stream s are q[qo_indptr[s] ..
 * qo_indptr[s+1]) (q_rows rows in all) and query j sees keys [0, prefix + j] of the
 * stream's pages; out has the rows of q.  Grid of max_tiles x Hq CTAs (tiles of 128
 * queries, tile_indptr from omni_extend_prepare with q_tile 128; the tiles past
 * tile_indptr[streams] exit).  head_dim 128, page 16; k_cache / v_cache hold
 * num_slots slots.  tcgen05 tensor cores: S and O accumulate in tensor memory. */
OMNI_API int omni_prefill_attention(const void* q, int64_t q_stride, int64_t q_rows, const void* k_cache,
                                   const void* v_cache, int64_t num_slots, const int32_t* qo_indptr,
                                   const int64_t* seq_lens, const int32_t* page_indptr, const int32_t* page_indices,
                                   const int32_t* tile_indptr, int64_t streams, int64_t max_tiles,
                                   int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                   float sm_scale, void* out, int64_t out_stride, void* stream);

/* ======================================================================== */
/* Streaming vocoder (code2wav) step                                        */
/* ======================================================================== */

/* dtype codes of the vocoder entry points */
#define OMNI_DTYPE_BF16 0
#define OMNI_DTYPE_F16 1
#define OMNI_DTYPE_F32 2

/* out = SnakeBeta(conv_output + bias [+ residual]) with every intermediate rounded to
 * the activations' dtype where the eager adds and SnakeBeta round; sum_out (nullable)
 * receives the pre-activation sum.  Replaces fused_bias_snake_beta
 * (sglang_omni/kernels/bias_snake_beta.py:100-151).
 *   conv_output, out: [batch, length, channels] bf16 / fp16, rows contiguous, batch
 *   strides given; residual, sum_out contiguous; bias, alpha_scale (exp(alpha)),
 *   inverse_beta (1 / (exp(beta) + eps)): [channels]; channels % 8 == 0, 16-byte
 *   aligned operands. */
OMNI_API int omni_bias_snake_beta(const void* conv_output, int64_t conv_batch_stride, const void* bias,
                                  const void* residual, void* sum_out, void* out, int64_t out_batch_stride,
                                  const void* alpha_scale, const void* inverse_beta, int64_t batch, int64_t length,
                                  int64_t channels, int32_t dtype, void* stream);

/* out[b, 0, t] = clamp(bias + sum_{tap, c} padded[b, t + tap, c] * weight[0, c, tap], -1, 1)
 * (NaN kept), accumulated in fp32 and rounded once; a position's bits do not depend on
 * how positions are split across calls.  Replaces clamped_single_output_conv
 * (sglang_omni/kernels/single_output_conv.py:68-102).
 *   padded [batch, length + taps - 1, channels] channels-last, rows contiguous;
 *   weight [1, channels, taps] with the given strides; out [batch, 1, length]. */
OMNI_API int omni_clamped_single_output_conv(const void* padded, int64_t padded_batch_stride, const void* weight,
                                             int64_t weight_channel_stride, int64_t weight_tap_stride,
                                             const void* bias, void* out, int64_t batch, int64_t length,
                                             int64_t channels, int32_t taps, int32_t dtype, void* stream);

/* The windows a causal conv reads, as the rows of its GEMM operand:
 * out[r * length + t, j * channels + c] = padded[r, t + j * dilation, c] for taps j.
 *   padded [rows, padded_samples, channels] channels-last (row stride padded_row_stride
 *   elements, samples contiguous), padded_samples >= length + (taps - 1) * dilation;
 *   out [rows * length, taps * channels] contiguous.  channels x element_bytes, the row
 *   stride in bytes and both pointers are 16-byte multiples.  No counterpart in the
 *   reference, whose convs run on cuDNN's channels-last convolution
 *   (sglang_omni/utils/channels_last_conv.py); here the code2wav's causal convs run as one
 *   cuBLAS GEMM over these windows. */
OMNI_API int omni_conv_window_gather(const void* padded, int64_t padded_row_stride, int64_t padded_samples,
                                     int64_t rows, int64_t length, int32_t taps, int32_t dilation, int32_t channels,
                                     int32_t element_bytes, void* out, void* stream);

/* Implicit-GEMM causal conv on tcgen05 (the code2wav's ungrouped convs,
 * qwen3_omni/components/code2wav.py:326-460, transformers' Qwen3OmniMoeCausalConvNet):
 *   out[r, t, n] = sum_{j < taps} sum_c padded[r, t + j dilation, c] weight[n, j * C_in + c]
 * for t < length, channels last.  padded bf16 [rows, padded_positions, C_in] contiguous
 * (padded_positions >= length + (taps - 1) dilation: the history in front); weight bf16
 * [C_out, taps * C_in] (conv.weight [C_out, C_in, taps] permuted to [C_out, taps, C_in]);
 * out rows r at out + r * out_batch_stride, positions C_out apart.  With taps = 1 it is the
 * GEMM of a 1x1 conv or of a transposed conv's taps.  C_in, C_out multiples of 32.
 * alpha_scale == NULL: out = bf16(conv).  Else, with bias, inverse_beta [C_out] and
 * optionally residual / sum_out (contiguous [rows, length, C_out]), the vocoder's next
 * SnakeBeta fused in: total = conv + bias (+ residual), sum_out = total, out = SnakeBeta
 * (total), with the rounding points of omni_bias_snake_beta. */
OMNI_API int omni_conv1d_gemm(const void* padded, int64_t rows, int64_t padded_positions, int32_t cin,
                              const void* weight, int32_t cout, int32_t taps, int32_t dilation, int64_t length,
                              void* out, int64_t out_batch_stride, const void* bias, const void* residual,
                              void* sum_out, const void* alpha_scale, const void* inverse_beta, void* stream);

/* Causal-conv state: padded [rows, history + new + tail, channels] gets each row's slot
 * history in front (zeros for a cold slot) and zeros after the new samples; the slot
 * keeps the last `history` samples of (history ++ new).  history <= 64.  Replaces
 * history_exchange (sglang_omni/kernels/codec_state.py:153-184). */
OMNI_API int omni_history_exchange(void* padded, int64_t padded_row_stride, int64_t padded_sample_stride,
                                   int64_t padded_channel_stride, void* history_pool, int64_t pool_slot_stride,
                                   int64_t pool_sample_stride, int64_t pool_channel_stride, const int64_t* slot_index,
                                   int64_t rows, int32_t history_samples, int32_t new_samples, int32_t tail_samples,
                                   int32_t channels, int32_t is_cold, int32_t element_bytes, void* stream);

/* Transposed-conv state: output [rows, emitted + overlap, channels]: the slot's overlap
 * is added into the first samples (not for a cold slot, rounded once) and the samples
 * past the emitted ones become the slot's overlap.  emitted >= overlap.  Replaces
 * overlap_exchange (sglang_omni/kernels/codec_state.py:187-210). */
OMNI_API int omni_overlap_exchange(void* output, int64_t output_row_stride, int64_t output_sample_stride,
                                   int64_t output_channel_stride, void* overlap_pool, int64_t pool_slot_stride,
                                   int64_t pool_sample_stride, int64_t pool_channel_stride, const int64_t* slot_index,
                                   int64_t rows, int32_t overlap_samples, int32_t emitted_samples, int32_t channels,
                                   int32_t is_cold, int32_t dtype, void* stream);

/* ======================================================================== */
/* Test hooks                                                               */
/* ======================================================================== */

/* No counterpart in the reference.  Launches the bf16 store GEMM (omni_linear,
 * epilogue 0, row-major x [rows, k], w [n, k]) with a producer that issues no
 * copies and every mbarrier wait bounded by wait_limit polls, so that the waits
 * run out.  The kernel records OMNI_DEV_TIMEOUT_TMA (or _MMA) in the status word
 * read by omni_device_status and returns with nothing in flight; y is not
 * written.  Exists so that tests can show a bounded device wait ending without
 * faulting the GPU. */
OMNI_API int omni_gemm_wait_probe(const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* y,
                                  int32_t splits, uint32_t wait_limit, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OMNI_B200_H_ */
