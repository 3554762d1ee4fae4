// Continuous batching of talker streams on the host (C ABI: include/omni_sched.h).
//
// The policy restates the batch selection the reference's talker stage runs:
//   - event loop (sglang_omni/scheduling/omni_scheduler.py:3616-3653): admit
//     arrivals, pick the next batch, run it, process its results;
//   - the prefill gate (omni_scheduler.py:2096-2160): with coalescing on, a
//     waiting queue shorter than coalesce_requests is held until its oldest
//     stamped request has waited coalesce_wait_us; requests are stamped the
//     first time the gate looks at them; an idle decode loop bypasses the gate
//     unless coalesce_when_idle;
//   - admission (upstream sglang's PrefillAdder, absent from the reference
//     tree, restated at page granularity): first come first served while rows,
//     the prefill token budget and the free pages allow, keeping reserve_ratio
//     of the live streams' future pages free; admitted prompts run in the same
//     forward as the decode rows (sglang's mixed-chunk mode);
//   - decode (upstream prepare_for_decode): a row whose next token starts a
//     page (seq_len % page_size == 0) takes a page off the free stack, in row
//     order; when the stack cannot cover the step, streams are retracted
//     (upstream retract_decode: the one with the fewest frames, then the
//     longest original prompt, first) and requeued at the front with their
//     whole context as the new prompt;
//   - rollback_decode_prep_after_skip (models/qwen3_omni/talker_scheduler.py:
//     198-225): a planned decode step that did not run returns the pages it
//     opened and takes seq_len back by one.
// Rows stay compact: after finishes, aborts and retractions the highest live
// rows fill the lowest holes, and the plan lists those moves.
// Committed frames go to the vocoder stage as messages, coalesced as the Qwen3-Omni
// talker's emit_code_chunks_and_feedback does (models/qwen3_omni/
// talker_model_runner.py:178-235, coalesce_threshold / flush_codec_rows :268-298,
// on_request_finished :300-315): with coalescing off every frame is a message; with it
// on, the first `early` frames go one by one, then frames are held and flushed in
// chunks once `coalesce` (the first chunk: `first`) are pending, the newest frame always
// held back; a finishing stream flushes its held frames and then its last frame alone.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <deque>
#include <new>
#include <unordered_map>
#include <vector>

#include "capi_util.h"
#include "omni_sched.h"

namespace omni {
namespace {

enum State { kWaiting = 0, kRunning = 1 };

struct Stream {
  int64_t rid = 0;
  int64_t prompt_len = 0;       // tokens the next prefill writes
  int64_t orig_prompt_len = 0;  // the prompt at arrival (retract order)
  int64_t max_frames = 0;
  int64_t frames_done = 0;
  int64_t seq_len = 0;          // tokens in the KV pool
  int64_t stamp_us = -1;        // prefill-gate stamp (-1: not yet seen)
  int32_t slot = -1;
  int32_t row = -1;
  State state = kWaiting;
  std::vector<int32_t> pages;
  // vocoder emission
  int64_t frames_seen = 0;
  bool first_flush_done = false;
  int64_t pending_first = 0;         // frame index (1-based) of the first held frame
  std::vector<int64_t> pending;      // held frames, groups codes each
};

struct Message {
  int64_t rid, first_frame;
  int32_t frames, final;
  std::vector<int64_t> codes;
};

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

uint64_t splitmix64(uint64_t& s) {
  // Steele, Lea, Flood, "Fast splittable pseudorandom number generators" (2014)
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

class Scheduler {
 public:
  explicit Scheduler(const omni_sched_config& c) : cfg_(c) {
    // pages 1 .. num_pages-1, handed out from the back of the stack
    std::vector<int32_t> order;
    order.reserve((size_t)(c.num_pages - 1));
    for (int64_t p = 1; p < c.num_pages; ++p) order.push_back((int32_t)p);
    if (c.page_seed != 0) {
      uint64_t s = c.page_seed;
      for (size_t i = order.size(); i > 1; --i) {
        const size_t j = (size_t)(splitmix64(s) % (uint64_t)i);
        std::swap(order[i - 1], order[j]);
      }
    }
    free_pages_.assign(order.rbegin(), order.rend());
    for (int32_t s = c.max_batch - 1; s >= 0; --s) free_slots_.push_back(s);
  }

  int add(int64_t rid, int64_t prompt_len, int64_t max_frames) {
    if (streams_.count(rid)) return set_error(OMNI_ERR_INVALID, "duplicate request id");
    if (prompt_len <= 0 || max_frames <= 0) return set_error(OMNI_ERR_INVALID, "prompt_len and max_frames must be > 0");
    if (prompt_len > cfg_.max_prefill_tokens)
      return set_error(OMNI_ERR_INVALID, "prompt longer than max_prefill_tokens (no chunked prefill)");
    const int64_t final_len = prompt_len + max_frames - 1;
    if (final_len > cfg_.max_context) return set_error(OMNI_ERR_INVALID, "stream exceeds max_context");
    if (ceil_div(final_len, cfg_.page_size) > cfg_.num_pages - 1)
      return set_error(OMNI_ERR_INVALID, "stream needs more pages than the pool holds");
    Stream s;
    s.rid = rid;
    s.prompt_len = s.orig_prompt_len = prompt_len;
    s.max_frames = max_frames;
    streams_.emplace(rid, std::move(s));
    waiting_.push_back(rid);
    return OMNI_OK;
  }

  int abort(int64_t rid) {
    if (!committed_) return set_error(OMNI_ERR_INVALID, "abort inside a planned step");
    auto it = streams_.find(rid);
    if (it == streams_.end()) return set_error(OMNI_ERR_INVALID, "unknown request id");
    Stream& s = it->second;
    if (s.state == kWaiting) {
      waiting_.erase(std::find(waiting_.begin(), waiting_.end(), rid));
    } else {
      rows_[(size_t)s.row] = -1;
      release(s);
    }
    streams_.erase(it);
    return OMNI_OK;
  }

  int schedule(int64_t now_us, omni_sched_plan* plan) {
    if (!committed_) return set_error(OMNI_ERR_INVALID, "the previous step was neither committed nor rolled back");
    // rows at the start of the step, for the move list
    std::unordered_map<int64_t, int32_t> row_before;
    for (size_t r = 0; r < rows_.size(); ++r)
      if (rows_[r] >= 0) row_before[rows_[r]] = (int32_t)r;
    compact();
    int64_t B = (int64_t)rows_.size();
    const int64_t P = cfg_.page_size;

    // ---- admission (prefill gate, then first come first served) ----
    std::vector<int64_t> admit;
    if (!waiting_.empty() && gate_open(now_us, B) && B < cfg_.max_batch && interval_left_ == 0) {
      const int64_t avail = (int64_t)free_pages_.size();
      int64_t used = 0;
      double future = 0.0;
      for (int64_t rid : rows_) {
        const Stream& s = streams_.at(rid);
        const int64_t opens = s.seq_len % P == 0 ? 1 : 0;
        used += opens;
        future += (double)(ceil_div(s.seq_len + (s.max_frames - s.frames_done), P) - (int64_t)s.pages.size() - opens);
      }
      if (used <= avail) {
        int64_t tokens = 0;
        for (int64_t rid : waiting_) {
          if (B + (int64_t)admit.size() >= cfg_.max_batch) break;
          const Stream& s = streams_.at(rid);
          if (tokens + s.prompt_len > cfg_.max_prefill_tokens) break;
          const int64_t need = ceil_div(s.prompt_len, P);
          const double fut =
              (double)(ceil_div(s.prompt_len + (s.max_frames - s.frames_done - 1), P) - need);
          const int64_t keep = (int64_t)std::ceil(cfg_.reserve_ratio * (future + fut));
          if (used + need + keep > avail) break;
          admit.push_back(rid);
          used += need;
          tokens += s.prompt_len;
          future += fut;
        }
      }
    }

    // ---- decode rows: retract while the free stack cannot cover the step ----
    std::vector<int64_t> retracted;
    if (admit.empty() && B > 0) {
      auto opening = [&]() {
        int64_t n = 0;
        for (int64_t rid : rows_) n += streams_.at(rid).seq_len % P == 0 ? 1 : 0;
        return n;
      };
      if (opening() > (int64_t)free_pages_.size()) {
        // fewest frames first, then the longest original prompt; ties: the later row
        std::vector<int64_t> order(rows_.begin(), rows_.end());
        std::stable_sort(order.begin(), order.end(), [&](int64_t a, int64_t b) {
          const Stream& x = streams_.at(a);
          const Stream& y = streams_.at(b);
          if (x.frames_done != y.frames_done) return x.frames_done > y.frames_done;
          return -x.orig_prompt_len > -y.orig_prompt_len;
        });
        while (!order.empty() && opening() > (int64_t)free_pages_.size()) {
          const int64_t rid = order.back();
          order.pop_back();
          Stream& s = streams_.at(rid);
          rows_[(size_t)s.row] = -1;
          compact();
          s.prompt_len = s.seq_len;
          release(s);  // frames_done is kept: the stream resumes at its next frame
          retracted.push_back(rid);
          ++retracted_total_;
        }
        waiting_.insert(waiting_.begin(), retracted.begin(), retracted.end());
        B = (int64_t)rows_.size();
      }
    }

    // ---- the plan ----
    plan->mode = B == 0 && admit.empty() ? OMNI_SCHED_IDLE : (admit.empty() ? OMNI_SCHED_DECODE : OMNI_SCHED_MIXED);
    plan->decode_rows = (int32_t)B;
    plan->new_rows = (int32_t)admit.size();
    plan->num_retracted = (int32_t)retracted.size();
    for (size_t i = 0; i < retracted.size(); ++i) plan->retracted_rid[i] = retracted[i];
    // moves: every surviving stream whose row changed
    int32_t nm = 0;
    for (size_t r = 0; r < rows_.size(); ++r) {
      auto it = row_before.find(rows_[r]);
      if (it != row_before.end() && it->second != (int32_t)r) {
        plan->move_src[nm] = it->second;
        plan->move_dst[nm] = (int32_t)r;
        ++nm;
      }
    }
    plan->num_moves = nm;
    // decode pages in row order
    opened_rows_.clear();
    int32_t nd = 0;
    for (size_t r = 0; r < rows_.size(); ++r) {
      Stream& s = streams_.at(rows_[r]);
      if (s.seq_len % P == 0) {
        const int32_t pg = free_pages_.back();
        free_pages_.pop_back();
        s.pages.push_back(pg);
        plan->decode_pages[nd++] = pg;
        opened_rows_.push_back((int32_t)r);
      }
      s.seq_len += 1;
    }
    plan->num_decode_pages = nd;
    // admitted streams: slot, prompt pages, rows after the decode rows
    int64_t tokens = 0;
    int32_t np = 0;
    plan->new_page_indptr[0] = 0;
    for (size_t i = 0; i < admit.size(); ++i) {
      Stream& s = streams_.at(admit[i]);
      waiting_.erase(std::find(waiting_.begin(), waiting_.end(), admit[i]));
      s.state = kRunning;
      s.slot = free_slots_.back();
      free_slots_.pop_back();
      s.row = (int32_t)rows_.size();
      rows_.push_back(s.rid);
      const int64_t need = ceil_div(s.prompt_len, P);
      for (int64_t k = 0; k < need; ++k) {
        const int32_t pg = free_pages_.back();
        free_pages_.pop_back();
        s.pages.push_back(pg);
        plan->new_pages[np++] = pg;
      }
      s.seq_len = s.prompt_len;
      s.stamp_us = -1;
      plan->new_rid[i] = s.rid;
      plan->new_slot[i] = s.slot;
      plan->new_prompt_len[i] = s.prompt_len;
      plan->new_page_indptr[i + 1] = np;
      tokens += s.prompt_len;
    }
    plan->new_tokens = tokens;
    last_mode_ = plan->mode;
    last_rows_ = (int64_t)rows_.size();
    interval_before_ = interval_left_;
    if (plan->mode == OMNI_SCHED_MIXED) {
      interval_left_ = cfg_.prefill_decode_interval;
    } else if (plan->mode == OMNI_SCHED_DECODE && interval_left_ > 0) {
      --interval_left_;
    }
    committed_ = plan->mode == OMNI_SCHED_IDLE;
    return OMNI_OK;
  }

  int commit(const int64_t* codes, int64_t n, int32_t groups, int64_t* finished, int64_t* num_finished) {
    if (committed_) return set_error(OMNI_ERR_INVALID, "no planned step to commit");
    if (n != last_rows_) return set_error(OMNI_ERR_INVALID, "commit rows differ from the planned step's rows");
    if (groups < 1 || (cfg_.emit_messages && codes == nullptr))
      return set_error(OMNI_ERR_INVALID, "commit needs codes (groups >= 1) when messages are emitted");
    int64_t nf = 0;
    for (int64_t r = 0; r < n; ++r) {
      Stream& s = streams_.at(rows_[(size_t)r]);
      s.frames_done += 1;
      ++frames_total_;
      const int64_t* frame = codes != nullptr ? codes + r * groups : nullptr;
      const bool eos = cfg_.eos_token >= 0 && frame != nullptr && frame[0] == cfg_.eos_token;
      const bool done = s.frames_done >= s.max_frames || eos;
      if (cfg_.emit_messages) emit(s, frame, groups, done);
      if (done) {
        if (finished) finished[nf] = s.rid;
        ++nf;
        rows_[(size_t)r] = -1;
        release(s);
        streams_.erase(s.rid);
        ++finished_total_;
      }
    }
    if (num_finished) *num_finished = nf;
    ++steps_;
    committed_ = true;
    return OMNI_OK;
  }

  int pop_message(int64_t* rid, int64_t* first_frame, int32_t* frames, int32_t* final, int64_t* codes,
                  int64_t capacity) {
    *frames = 0;
    if (messages_.empty()) return OMNI_OK;
    const Message& m = messages_.front();
    if ((int64_t)m.codes.size() > capacity) return set_error(OMNI_ERR_CAPACITY, "message larger than the buffer");
    *rid = m.rid;
    *first_frame = m.first_frame;
    *frames = m.frames;
    *final = m.final;
    std::copy(m.codes.begin(), m.codes.end(), codes);
    messages_.pop_front();
    return OMNI_OK;
  }

  int rollback() {
    if (committed_ || last_mode_ != OMNI_SCHED_DECODE)
      return set_error(OMNI_ERR_INVALID, "only a planned decode step can be rolled back");
    for (auto it = opened_rows_.rbegin(); it != opened_rows_.rend(); ++it) {
      Stream& s = streams_.at(rows_[(size_t)*it]);
      free_pages_.push_back(s.pages.back());
      s.pages.pop_back();
    }
    for (int64_t rid : rows_) streams_.at(rid).seq_len -= 1;
    opened_rows_.clear();
    interval_left_ = interval_before_;
    committed_ = true;
    return OMNI_OK;
  }

  void stats(int64_t* out, int n) const {
    const int64_t live = (int64_t)std::count_if(rows_.begin(), rows_.end(), [](int64_t r) { return r >= 0; });
    const int64_t v[10] = {(int64_t)waiting_.size(), live, (int64_t)free_pages_.size(),
                           (int64_t)free_slots_.size(), steps_, frames_total_, finished_total_, retracted_total_,
                           (int64_t)messages_.size(), frames_emitted_};
    for (int i = 0; i < n && i < 10; ++i) out[i] = v[i];
  }

  int row_rids(int64_t* rids, int64_t cap, int64_t* n) const {
    if (n) *n = (int64_t)rows_.size();
    if ((int64_t)rows_.size() > cap) return set_error(OMNI_ERR_CAPACITY, "row capacity");
    for (size_t r = 0; r < rows_.size(); ++r) rids[r] = rows_[r];
    return OMNI_OK;
  }

  int request_state(int64_t rid, int32_t* slot, int64_t* seq_len, int32_t* pages, int64_t cap, int64_t* n) const {
    auto it = streams_.find(rid);
    if (it == streams_.end()) return set_error(OMNI_ERR_INVALID, "unknown request id");
    const Stream& s = it->second;
    if (slot) *slot = s.slot;
    if (seq_len) *seq_len = s.seq_len;
    if (n) *n = (int64_t)s.pages.size();
    if (pages)
      for (size_t k = 0; k < s.pages.size() && (int64_t)k < cap; ++k) pages[k] = s.pages[k];
    return OMNI_OK;
  }

  int check() const {
    std::vector<int> owner((size_t)cfg_.num_pages, 0);
    for (int32_t p : free_pages_) {
      if (p <= 0 || p >= cfg_.num_pages) return set_error(OMNI_ERR_INVALID, "free page out of range");
      owner[(size_t)p] += 1;
    }
    std::vector<int> slot_use((size_t)cfg_.max_batch, 0);
    for (int32_t s : free_slots_) slot_use[(size_t)s] += 1;
    for (size_t r = 0; r < rows_.size(); ++r) {
      if (rows_[r] < 0) continue;  // freed since the last plan; compacted by the next
      const Stream& s = streams_.at(rows_[r]);
      if (s.row != (int32_t)r || s.state != kRunning) return set_error(OMNI_ERR_INVALID, "row bookkeeping");
      if ((int64_t)s.pages.size() != ceil_div(s.seq_len, cfg_.page_size))
        return set_error(OMNI_ERR_INVALID, "page count does not match seq_len");
      for (int32_t p : s.pages) owner[(size_t)p] += 1;
      slot_use[(size_t)s.slot] += 1;
    }
    for (int64_t p = 1; p < cfg_.num_pages; ++p)
      if (owner[(size_t)p] != 1) return set_error(OMNI_ERR_INVALID, "a page is lost or owned twice");
    if (owner[0] != 0) return set_error(OMNI_ERR_INVALID, "page 0 handed out");
    for (int v : slot_use)
      if (v != 1) return set_error(OMNI_ERR_INVALID, "a slot is lost or owned twice");
    for (int64_t rid : waiting_) {
      const Stream& s = streams_.at(rid);
      if (s.state != kWaiting || s.slot >= 0 || !s.pages.empty())
        return set_error(OMNI_ERR_INVALID, "waiting bookkeeping");
    }
    return OMNI_OK;
  }

 private:
  bool gate_open(int64_t now_us, int64_t running) {
    if (cfg_.coalesce_requests <= 1) return true;
    if (!cfg_.coalesce_when_idle && running == 0) return true;
    if ((int64_t)waiting_.size() >= cfg_.coalesce_requests) return true;
    int64_t oldest = now_us;
    for (int64_t rid : waiting_) {
      Stream& s = streams_.at(rid);
      if (s.stamp_us < 0) s.stamp_us = now_us;
      oldest = std::min(oldest, s.stamp_us);
    }
    return now_us - oldest >= cfg_.coalesce_wait_us;
  }

  void push_message(const Stream& s, int64_t first, const int64_t* codes, int64_t n_codes, int32_t frames,
                    bool final) {
    Message m{s.rid, first, frames, final ? 1 : 0, std::vector<int64_t>(codes, codes + n_codes)};
    messages_.push_back(std::move(m));
    frames_emitted_ += frames;
  }

  void flush(Stream& s, int32_t groups, bool final) {
    if (s.pending.empty()) return;
    s.first_flush_done = true;
    const int32_t k = (int32_t)(s.pending.size() / (size_t)groups);
    push_message(s, s.pending_first, s.pending.data(), (int64_t)s.pending.size(), k, final);
    s.pending.clear();
  }

  // One committed frame of stream s (frame index s.frames_done).
  void emit(Stream& s, const int64_t* frame, int32_t groups, bool done) {
    const int64_t idx = s.frames_done;
    const int32_t coalesce = cfg_.codec_coalesce_frames;
    if (coalesce <= 1) {
      push_message(s, idx, frame, groups, 1, done);
      return;
    }
    s.frames_seen += 1;
    if (s.frames_seen <= cfg_.codec_coalesce_early_frames) {
      push_message(s, idx, frame, groups, 1, done);
      return;
    }
    const int64_t held = (int64_t)(s.pending.size() / (size_t)groups);
    int64_t threshold = coalesce;
    if (cfg_.codec_coalesce_early_frames <= 0 && cfg_.codec_coalesce_first_frames > 0 && !s.first_flush_done)
      threshold = cfg_.codec_coalesce_first_frames;
    if (held >= threshold) flush(s, groups, false);
    if (s.pending.empty()) s.pending_first = idx;
    s.pending.insert(s.pending.end(), frame, frame + groups);
    if (done) {
      // the held frames, then the last frame alone
      std::vector<int64_t> last(s.pending.end() - groups, s.pending.end());
      s.pending.resize(s.pending.size() - (size_t)groups);
      flush(s, groups, false);
      push_message(s, idx, last.data(), groups, 1, true);
    }
  }

  // The highest live rows fill the lowest holes.
  void compact() {
    size_t lo = 0, hi = rows_.size();
    while (true) {
      while (hi > 0 && rows_[hi - 1] < 0) --hi;
      while (lo < hi && rows_[lo] >= 0) ++lo;
      if (lo >= hi) break;
      rows_[lo] = rows_[hi - 1];
      streams_.at(rows_[lo]).row = (int32_t)lo;
      rows_[hi - 1] = -1;
    }
    rows_.resize(hi);
  }

  // Frees a running stream's pages (in list order onto the stack) and slot.
  void release(Stream& s) {
    for (int32_t p : s.pages) free_pages_.push_back(p);
    s.pages.clear();
    if (s.slot >= 0) free_slots_.push_back(s.slot);
    s.slot = -1;
    s.row = -1;
    s.seq_len = 0;
    s.state = kWaiting;
  }

  omni_sched_config cfg_;
  std::vector<int32_t> free_pages_;
  std::vector<int32_t> free_slots_;
  std::deque<int64_t> waiting_;
  std::unordered_map<int64_t, Stream> streams_;
  std::vector<int64_t> rows_;
  std::vector<int32_t> opened_rows_;
  int64_t interval_left_ = 0, interval_before_ = 0;
  int last_mode_ = OMNI_SCHED_IDLE;
  int64_t last_rows_ = 0;
  bool committed_ = true;
  int64_t steps_ = 0, frames_total_ = 0, finished_total_ = 0, retracted_total_ = 0, frames_emitted_ = 0;
  std::deque<Message> messages_;
};

Scheduler* as_sched(void* h) { return static_cast<Scheduler*>(h); }

}  // namespace
}  // namespace omni

using omni::as_sched;
using omni::set_error;

extern "C" OMNI_API void* omni_sched_create(const omni_sched_config* c) {
  if (c == nullptr || c->num_pages < 2 || c->page_size <= 0 || c->max_batch <= 0 || c->max_context <= 0 ||
      c->max_prefill_tokens <= 0 || c->reserve_ratio < 0.0 || c->coalesce_wait_us < 0 ||
      c->prefill_decode_interval < 0 || c->num_pages > INT32_MAX || c->codec_coalesce_frames < 0 ||
      c->codec_coalesce_first_frames < 0 || c->codec_coalesce_early_frames < 0) {
    set_error(OMNI_ERR_INVALID, "malformed scheduler config");
    return nullptr;
  }
  return new (std::nothrow) omni::Scheduler(*c);
}

extern "C" OMNI_API void omni_sched_destroy(void* sched) { delete as_sched(sched); }

extern "C" OMNI_API int omni_sched_add_request(void* sched, int64_t rid, int64_t prompt_len, int64_t max_frames) {
  if (!sched) return set_error(OMNI_ERR_INVALID, "null scheduler");
  return as_sched(sched)->add(rid, prompt_len, max_frames);
}

extern "C" OMNI_API int omni_sched_abort(void* sched, int64_t rid) {
  if (!sched) return set_error(OMNI_ERR_INVALID, "null scheduler");
  return as_sched(sched)->abort(rid);
}

extern "C" OMNI_API int omni_sched_schedule(void* sched, int64_t now_us, omni_sched_plan* plan) {
  if (!sched || !plan || !plan->move_src || !plan->move_dst || !plan->decode_pages || !plan->new_rid ||
      !plan->new_slot || !plan->new_prompt_len || !plan->new_page_indptr || !plan->new_pages || !plan->retracted_rid)
    return set_error(OMNI_ERR_INVALID, "null scheduler or plan array");
  return as_sched(sched)->schedule(now_us, plan);
}

extern "C" OMNI_API int omni_sched_commit(void* sched, const int64_t* codes, int64_t rows, int32_t groups,
                                          int64_t* finished_rids, int64_t* num_finished) {
  if (!sched) return set_error(OMNI_ERR_INVALID, "null scheduler");
  return as_sched(sched)->commit(codes, rows, groups, finished_rids, num_finished);
}

extern "C" OMNI_API int omni_sched_pop_message(void* sched, int64_t* rid, int64_t* first_frame, int32_t* frames,
                                               int32_t* final, int64_t* codes, int64_t capacity) {
  if (!sched || !rid || !first_frame || !frames || !final || (!codes && capacity > 0))
    return set_error(OMNI_ERR_INVALID, "null scheduler or output");
  return as_sched(sched)->pop_message(rid, first_frame, frames, final, codes, capacity);
}

extern "C" OMNI_API int omni_sched_rollback(void* sched) {
  if (!sched) return set_error(OMNI_ERR_INVALID, "null scheduler");
  return as_sched(sched)->rollback();
}

extern "C" OMNI_API int omni_sched_stats(void* sched, int64_t* out, int32_t n) {
  if (!sched || !out || n < 0) return set_error(OMNI_ERR_INVALID, "null scheduler or output");
  as_sched(sched)->stats(out, n);
  return OMNI_OK;
}

extern "C" OMNI_API int omni_sched_row_rids(void* sched, int64_t* rids, int64_t capacity, int64_t* rows) {
  if (!sched || !rids) return set_error(OMNI_ERR_INVALID, "null scheduler or output");
  return as_sched(sched)->row_rids(rids, capacity, rows);
}

extern "C" OMNI_API int omni_sched_request_state(void* sched, int64_t rid, int32_t* slot, int64_t* seq_len,
                                                 int32_t* pages, int64_t capacity, int64_t* num_pages) {
  if (!sched) return set_error(OMNI_ERR_INVALID, "null scheduler");
  return as_sched(sched)->request_state(rid, slot, seq_len, pages, capacity, num_pages);
}

extern "C" OMNI_API int omni_sched_check(void* sched) {
  if (!sched) return set_error(OMNI_ERR_INVALID, "null scheduler");
  return as_sched(sched)->check();
}
