/*
 * omni_b200 — C ABI of the host-side continuous-batching scheduler.
 *
 * The scheduler owns the talker's request admission, the KV page allocator
 * (a free-page stack), the request slots (rows of req_to_token), retraction
 * when the pool runs dry, the rollback of a skipped decode step and the
 * compaction of batch rows.  It replaces, for the talker decode path, the
 * batch selection of the reference's OmniScheduler over the upstream sglang
 * Scheduler (sglang_omni/scheduling/omni_scheduler.py:2000-2160,
 * event_loop_normal :3616-3653) and the talker's rollback
 * (sglang_omni/models/qwen3_omni/talker_scheduler.py:190-225).
 *
 * Host code only: no call touches the GPU.  One step of the event loop is
 *   omni_sched_add_request* -> omni_sched_schedule -> (device step) ->
 *   omni_sched_commit (or omni_sched_rollback for a skipped decode step).
 * Rows: the running streams occupy batch rows [0, B) with no holes.  A step's
 * plan first lists row moves (compaction after finishes, aborts and
 * retractions: move_dst <- move_src for every per-row device state; every
 * source row is >= every destination row, so the moves are independent),
 * then the decode rows [0, decode_rows), then the admitted streams at rows
 * [decode_rows, decode_rows + new_rows).  Page 0 is never handed out.
 *
 * Return codes are the OMNI_* codes of omni_b200.h.
 */
#ifndef OMNI_SCHED_H_
#define OMNI_SCHED_H_

#include <stdint.h>

#include "omni_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

#define OMNI_SCHED_IDLE 0   /* nothing to run                                    */
#define OMNI_SCHED_DECODE 1 /* decode rows only                                   */
#define OMNI_SCHED_MIXED 2  /* decode rows and admitted prompts in one forward    */

typedef struct {
  int64_t num_pages;          /* pages in the KV pool; page 0 is reserved           */
  int32_t page_size;          /* tokens per page                                    */
  int32_t max_batch;          /* rows of a step (decode + admitted)                 */
  int64_t max_context;        /* tokens a stream may reach (req_to_token row)       */
  int64_t max_prefill_tokens; /* prompt tokens admitted in one step                 */
  int32_t coalesce_requests;  /* prefill gate: <= 1 turns it off                    */
  int32_t coalesce_when_idle; /* gate also while no stream decodes                  */
  int64_t coalesce_wait_us;   /* gate window from the oldest stamped request        */
  int32_t prefill_decode_interval; /* decode-only steps after a step that admitted */
  int32_t reserved0;
  double reserve_ratio;       /* share of the live streams' future pages kept free  */
  int64_t eos_token;          /* layer-0 code that ends a stream, -1 = none          */
  uint64_t page_seed;         /* 0: pages handed out 1, 2, 3, ...; else a seeded     */
                              /* permutation (splitmix64 + Fisher-Yates)             */
  int32_t emit_messages;      /* 1: committed frames go to the vocoder message queue */
  int32_t codec_coalesce_frames;       /* <= 1: one message per frame             */
  int32_t codec_coalesce_first_frames; /* size of the first coalesced chunk (0: same) */
  int32_t codec_coalesce_early_frames; /* frames sent one by one before coalescing  */
} omni_sched_config;

typedef struct {
  /* outputs */
  int32_t mode;             /* OMNI_SCHED_*                                          */
  int32_t decode_rows;      /* rows [0, decode_rows) take one decode token           */
  int32_t new_rows;         /* admitted streams at rows decode_rows + i              */
  int32_t num_moves;
  int32_t num_decode_pages; /* pages opened by decode rows, in row order             */
  int32_t num_retracted;
  int64_t new_tokens;       /* sum of the admitted prompt lengths                    */
  /* caller-provided arrays; capacities: max_batch unless noted */
  int32_t* move_src;
  int32_t* move_dst;
  int32_t* decode_pages;
  int64_t* new_rid;
  int32_t* new_slot;        /* req_to_token row of each admitted stream              */
  int64_t* new_prompt_len;  /* tokens its prefill writes                             */
  int32_t* new_page_indptr; /* capacity max_batch + 1                                */
  int32_t* new_pages;       /* capacity num_pages                                    */
  int64_t* retracted_rid;
} omni_sched_plan;

/* A scheduler for one GPU's stream set; NULL on a malformed config
 * (omni_last_error says why). */
OMNI_API void* omni_sched_create(const omni_sched_config* config);
OMNI_API void omni_sched_destroy(void* sched);

/* Queue a stream (arrival): prompt_len tokens to prefill, max_frames frames to
 * produce.  INVALID for a duplicate rid or a stream that can never fit
 * (prompt over max_prefill_tokens, context over max_context, pages over the pool). */
OMNI_API int omni_sched_add_request(void* sched, int64_t rid, int64_t prompt_len, int64_t max_frames);

/* Remove a waiting or running stream between steps (its pages and slot are freed). */
OMNI_API int omni_sched_abort(void* sched, int64_t rid);

/* Plan the next step at host time now_us (the prefill gate's clock). */
OMNI_API int omni_sched_schedule(void* sched, int64_t now_us, omni_sched_plan* plan);

/* Close the planned step: codes [rows, groups] are the step's frames of rows
 * [0, decode_rows + new_rows) (rows must equal that count; column 0 is the layer-0
 * code; groups = 1 passes layer-0 codes only).  Streams that reached max_frames or
 * drew eos_token finish; their rids are written to finished_rids (capacity
 * max_batch), the count to num_finished.  With emit_messages the frames enter the
 * vocoder message queue (post_process_outputs / emit_code_chunks_and_feedback,
 * qwen3_tts/model_runner.py:254-294, qwen3_omni/talker_model_runner.py:178-315). */
OMNI_API int omni_sched_commit(void* sched, const int64_t* codes, int64_t rows, int32_t groups,
                               int64_t* finished_rids, int64_t* num_finished);

/* Pop the oldest vocoder message: stream rid, its frames first_frame ..
 * first_frame + frames - 1 (1-based) as codes [frames, groups], final = 1 on the
 * stream's last message.  frames = 0 when the queue is empty.  CAPACITY (nothing
 * popped) when the message holds more than capacity codes. */
OMNI_API int omni_sched_pop_message(void* sched, int64_t* rid, int64_t* first_frame, int32_t* frames,
                                    int32_t* final, int64_t* codes, int64_t capacity);

/* rollback_decode_prep_after_skip: undo a planned DECODE step that did not run
 * (its opened pages go back on the free stack, seq_len -= 1).  Row moves and
 * retractions of the plan stay. */
OMNI_API int omni_sched_rollback(void* sched);

/* Counters: [waiting, running, free_pages, free_slots, steps, frames,
 * finished, retracted, queued messages, emitted frames]; n <= 10 of them are
 * written. */
OMNI_API int omni_sched_stats(void* sched, int64_t* out, int32_t n);

/* rids of rows [0, B) (written to *rows); -1 marks a row freed since the
 * last plan (the next omni_sched_schedule compacts it away). */
OMNI_API int omni_sched_row_rids(void* sched, int64_t* rids, int64_t capacity, int64_t* rows);

/* A live stream's slot, seq_len and page list (capacity entries at most). */
OMNI_API int omni_sched_request_state(void* sched, int64_t rid, int32_t* slot, int64_t* seq_len, int32_t* pages,
                                      int64_t capacity, int64_t* num_pages);

/* Consistency of the allocator and rows: every page other than 0 is free or
 * owned by one running stream, slots likewise, each running stream's page
 * count matches its seq_len. */
OMNI_API int omni_sched_check(void* sched);

#ifdef __cplusplus
}
#endif

#endif /* OMNI_SCHED_H_ */
