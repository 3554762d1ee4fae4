// Codec-frame relay from the talker stage to the vocoder stage (C ABI:
// include/omni_relay.h): one single-producer / single-consumer ring of
// variable-size records in POSIX shared memory.
//
// Layout of the segment: a 256-byte header (magic, capacity, and on separate
// cache lines the producer's byte count `head`, the consumer's byte count
// `tail`, and message counters), then `capacity` bytes of records.  A record is
// a 40-byte header (bytes, kind, rid, first frame, frames, groups, final) and
// frames x groups int64 codes; records never straddle the end of the ring: a
// record that does not fit before the end leaves a skip marker and starts at 0.
// The producer publishes a record by storing `head` with release order after
// writing it; the consumer reads `head` with acquire order, copies the record
// out, then releases its bytes by storing `tail` (release), which the producer
// reads with acquire order before reusing them.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <new>
#include <string>

#include "capi_util.h"
#include "omni_relay.h"

namespace omni {
namespace {

constexpr uint64_t kMagic = 0x31594C52494E4D4FULL;  // "OMNIRLY1"
constexpr size_t kHeaderBytes = 256;
constexpr uint32_t kKindMessage = 1, kKindSkip = 2;

struct alignas(64) SegmentHeader {
  uint64_t magic;
  uint64_t capacity;
  alignas(64) std::atomic<uint64_t> head;
  alignas(64) std::atomic<uint64_t> tail;
  alignas(64) std::atomic<uint64_t> pushed;
  std::atomic<uint64_t> popped;
};
static_assert(sizeof(SegmentHeader) <= kHeaderBytes, "segment header exceeds its reserved bytes");

struct RecordHeader {
  uint32_t bytes;
  uint32_t kind;
  int64_t rid;
  int64_t first_frame;
  int32_t frames;
  int32_t groups;
  int32_t final;
  int32_t reserved;
};
static_assert(sizeof(RecordHeader) == 40, "record header layout");

struct Relay {
  std::string name;
  void* base = nullptr;
  size_t bytes = 0;
  SegmentHeader* hdr = nullptr;
  uint8_t* data = nullptr;
  uint64_t cap = 0;
};

Relay* as_relay(void* h) { return static_cast<Relay*>(h); }

}  // namespace
}  // namespace omni

using omni::Relay;
using omni::set_error;

extern "C" OMNI_API void* omni_relay_open(const char* name, int64_t capacity_bytes, int32_t create) {
  if (name == nullptr || name[0] != '/') {
    set_error(OMNI_ERR_INVALID, "relay name must start with '/'");
    return nullptr;
  }
  if (create && (capacity_bytes < 4096 || (capacity_bytes & (capacity_bytes - 1)) != 0)) {
    set_error(OMNI_ERR_INVALID, "relay capacity must be a power of two >= 4096");
    return nullptr;
  }
  const int fd = create ? shm_open(name, O_CREAT | O_EXCL | O_RDWR, 0600) : shm_open(name, O_RDWR, 0600);
  if (fd < 0) {
    set_error(OMNI_ERR_INVALID, create ? "shm_open failed (name in use?)" : "shm_open failed (no such relay)");
    return nullptr;
  }
  size_t bytes = 0;
  if (create) {
    bytes = omni::kHeaderBytes + (size_t)capacity_bytes;
    if (ftruncate(fd, (off_t)bytes) != 0) {
      close(fd);
      shm_unlink(name);
      set_error(OMNI_ERR_CAPACITY, "ftruncate of the relay segment failed");
      return nullptr;
    }
  } else {
    struct stat st {};
    if (fstat(fd, &st) != 0 || (size_t)st.st_size < omni::kHeaderBytes + 4096) {
      close(fd);
      set_error(OMNI_ERR_INVALID, "relay segment too small");
      return nullptr;
    }
    bytes = (size_t)st.st_size;
  }
  void* base = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (base == MAP_FAILED) {
    if (create) shm_unlink(name);
    set_error(OMNI_ERR_CAPACITY, "mmap of the relay segment failed");
    return nullptr;
  }
  auto* hdr = static_cast<omni::SegmentHeader*>(base);
  if (create) {
    std::memset(base, 0, omni::kHeaderBytes);
    new (hdr) omni::SegmentHeader();
    hdr->capacity = (uint64_t)capacity_bytes;
    hdr->head.store(0, std::memory_order_relaxed);
    hdr->tail.store(0, std::memory_order_relaxed);
    hdr->pushed.store(0, std::memory_order_relaxed);
    hdr->popped.store(0, std::memory_order_relaxed);
    std::atomic_thread_fence(std::memory_order_release);
    hdr->magic = omni::kMagic;
  } else if (hdr->magic != omni::kMagic || hdr->capacity + omni::kHeaderBytes > bytes) {
    munmap(base, bytes);
    set_error(OMNI_ERR_INVALID, "not a relay segment");
    return nullptr;
  }
  auto* r = new (std::nothrow) Relay();
  if (r == nullptr) {
    munmap(base, bytes);
    set_error(OMNI_ERR_CAPACITY, "out of host memory");
    return nullptr;
  }
  r->name = name;
  r->base = base;
  r->bytes = bytes;
  r->hdr = hdr;
  r->data = static_cast<uint8_t*>(base) + omni::kHeaderBytes;
  r->cap = hdr->capacity;
  return r;
}

extern "C" OMNI_API void omni_relay_close(void* relay, int32_t unlink) {
  Relay* r = omni::as_relay(relay);
  if (r == nullptr) return;
  munmap(r->base, r->bytes);
  if (unlink) shm_unlink(r->name.c_str());
  delete r;
}

extern "C" OMNI_API int omni_relay_push(void* relay, int64_t rid, int64_t first_frame, int32_t frames, int32_t groups,
                                        int32_t final, const int64_t* codes) {
  Relay* r = omni::as_relay(relay);
  if (r == nullptr || frames <= 0 || groups <= 0 || codes == nullptr)
    return set_error(OMNI_ERR_INVALID, "relay push: null relay or empty message");
  const uint64_t need = sizeof(omni::RecordHeader) + (uint64_t)frames * (uint64_t)groups * 8;
  if (need > r->cap / 2) return set_error(OMNI_ERR_INVALID, "message larger than half the ring");
  uint64_t h = r->hdr->head.load(std::memory_order_relaxed);
  const uint64_t t = r->hdr->tail.load(std::memory_order_acquire);
  uint64_t pos = h & (r->cap - 1);
  const uint64_t contiguous = r->cap - pos;
  const uint64_t skip = contiguous < need ? contiguous : 0;
  if (need + skip > r->cap - (h - t)) return set_error(OMNI_ERR_CAPACITY, "relay ring full");
  if (skip) {
    auto* mark = reinterpret_cast<omni::RecordHeader*>(r->data + pos);
    mark->bytes = (uint32_t)skip;
    mark->kind = omni::kKindSkip;
    h += skip;
    pos = 0;
  }
  auto* rec = reinterpret_cast<omni::RecordHeader*>(r->data + pos);
  rec->bytes = (uint32_t)need;
  rec->kind = omni::kKindMessage;
  rec->rid = rid;
  rec->first_frame = first_frame;
  rec->frames = frames;
  rec->groups = groups;
  rec->final = final;
  rec->reserved = 0;
  std::memcpy(rec + 1, codes, (size_t)frames * (size_t)groups * 8);
  r->hdr->head.store(h + need, std::memory_order_release);
  r->hdr->pushed.fetch_add(1, std::memory_order_relaxed);
  return OMNI_OK;
}

extern "C" OMNI_API int omni_relay_pop(void* relay, int64_t* rid, int64_t* first_frame, int32_t* frames,
                                       int32_t* groups, int32_t* final, int64_t* codes, int64_t capacity) {
  Relay* r = omni::as_relay(relay);
  if (r == nullptr || !rid || !first_frame || !frames || !groups || !final || (!codes && capacity > 0))
    return set_error(OMNI_ERR_INVALID, "relay pop: null relay or output");
  *frames = 0;
  uint64_t t = r->hdr->tail.load(std::memory_order_relaxed);
  for (;;) {
    const uint64_t h = r->hdr->head.load(std::memory_order_acquire);
    if (t == h) return OMNI_OK;
    const auto* rec = reinterpret_cast<const omni::RecordHeader*>(r->data + (t & (r->cap - 1)));
    if (rec->bytes == 0 || rec->bytes > h - t) return set_error(OMNI_ERR_INVALID, "relay ring corrupted");
    if (rec->kind == omni::kKindSkip) {
      t += rec->bytes;
      r->hdr->tail.store(t, std::memory_order_release);
      continue;
    }
    const int64_t n = (int64_t)rec->frames * rec->groups;
    if (n > capacity) return set_error(OMNI_ERR_CAPACITY, "message larger than the output buffer");
    *rid = rec->rid;
    *first_frame = rec->first_frame;
    *groups = rec->groups;
    *final = rec->final;
    std::memcpy(codes, rec + 1, (size_t)n * 8);
    *frames = rec->frames;
    r->hdr->tail.store(t + rec->bytes, std::memory_order_release);
    r->hdr->popped.fetch_add(1, std::memory_order_relaxed);
    return OMNI_OK;
  }
}

extern "C" OMNI_API int omni_relay_stats(void* relay, int64_t* out, int32_t n) {
  Relay* r = omni::as_relay(relay);
  if (r == nullptr || out == nullptr) return set_error(OMNI_ERR_INVALID, "null relay or output");
  const uint64_t h = r->hdr->head.load(std::memory_order_acquire);
  const uint64_t t = r->hdr->tail.load(std::memory_order_acquire);
  const int64_t v[4] = {(int64_t)r->hdr->pushed.load(), (int64_t)r->hdr->popped.load(), (int64_t)(h - t),
                        (int64_t)r->cap};
  for (int i = 0; i < n && i < 4; ++i) out[i] = v[i];
  return OMNI_OK;
}
