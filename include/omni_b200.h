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
 *   table      bf16 [vocab, hidden]; gathered, summed bf16 [rows, hidden] or NULL */
OMNI_API int omni_predictor_sample_step(const void* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                        const float* temperatures, const int64_t* top_ks, const float* top_ps,
                                        const int64_t* seeds, const int64_t* positions, int64_t pos_mul,
                                        int64_t pos_add, const uint8_t* do_sample, int32_t argmax_all,
                                        int32_t max_top_k, int32_t has_top_p, int64_t* codes, int64_t codes_stride,
                                        const void* table, int64_t hidden, void* gathered, void* summed,
                                        void* stream);

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
 *   max_top_k <= 1024: the widest top_k of the batch. */
OMNI_API int omni_layer0_sample(const float* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                const float* penalties, const uint8_t* rep_mask, const uint8_t* suppress_mask,
                                const float* temperatures, const int64_t* top_ks, const float* top_ps,
                                const float* min_ps, const int64_t* seeds, const int64_t* positions,
                                int32_t max_top_k, int64_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OMNI_B200_H_ */
