/*
 * omni_b200 — C ABI of the codec-frame relay between the talker stage and the
 * vocoder stage (host code only).
 *
 * The talker's vocoder messages (omni_sched_pop_message: a stream's frames as
 * codes [frames, groups]) cross to the vocoder process through one
 * single-producer / single-consumer ring in POSIX shared memory.  It replaces,
 * for code chunks, the reference's per-tensor stage relays
 * (sglang_omni/relay/shm.py, relay/cuda_ipc.py, relay/nccl.py), which move one
 * tensor per transfer with a control message each way: code chunks are a few KB
 * and already on the host after the step's one device-to-host copy, so a
 * persistent ring with two shared counters carries them without a handshake.
 *
 * Records keep their order.  Push never blocks: CAPACITY when the ring has no
 * room (nothing written; the caller retries after the consumer drains).  Pop
 * never blocks: frames = 0 when the ring is empty.
 */
#ifndef OMNI_RELAY_H_
#define OMNI_RELAY_H_

#include <stdint.h>

#include "omni_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Open the ring `name` (a POSIX shared-memory name, "/..." ): create = 1 makes it
 * with capacity_bytes of records (a power of two >= 4096; the producer side),
 * create = 0 attaches to an existing one (capacity_bytes ignored).  NULL on
 * failure (omni_last_error says why). */
OMNI_API void* omni_relay_open(const char* name, int64_t capacity_bytes, int32_t create);

/* Unmap; unlink != 0 also removes the name (the creator, once both sides are done). */
OMNI_API void omni_relay_close(void* relay, int32_t unlink);

/* Append one message: stream rid, frames first_frame .. first_frame + frames - 1,
 * codes [frames, groups] (int64), final = 1 on the stream's last message. */
OMNI_API int omni_relay_push(void* relay, int64_t rid, int64_t first_frame, int32_t frames, int32_t groups,
                             int32_t final, const int64_t* codes);

/* Take the oldest message; frames = 0 when empty.  CAPACITY (not consumed) when its
 * codes exceed capacity entries. */
OMNI_API int omni_relay_pop(void* relay, int64_t* rid, int64_t* first_frame, int32_t* frames, int32_t* groups,
                            int32_t* final, int64_t* codes, int64_t capacity);

/* Counters: [messages pushed, messages popped, bytes in the ring, ring capacity];
 * n <= 4 of them are written. */
OMNI_API int omni_relay_stats(void* relay, int64_t* out, int32_t n);

#ifdef __cplusplus
}
#endif

#endif /* OMNI_RELAY_H_ */
