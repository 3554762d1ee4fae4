// Decode batch packing (prepare_for_decode + ForwardBatch metadata) on the GPU.
//
// One CTA of 1024 threads packs the whole batch in row blocks of 1024:
//   seq_len += 1; a row whose new token opens a page ((seq_len - 1) % P == 0)
//   takes the next free page in row order (block prefix sum), else the slot
//   after its last one; req_to_token[req, seq_len - 1] = slot; positions =
//   seq_len - 1 (talker_scheduler.py:198-225 is the same rule read backwards).
// Then the attention metadata of ForwardBatch.init_new (model_runner/base.py:
// 577-623): kv_indptr = cumsum(seq_lens) with kv_indices = the req_to_token
// rows (token level, optional), the page-level page_indptr / page_indices, and
// the attention work list work_indptr = cumsum(ceil(pages / pages_per_chunk)).
//
// extend_prepare_kernel packs an extend (prefill) batch whose slots the
// scheduler has already reserved in req_to_token (prepare_for_extend):
// seq_len = prefix + extend, qo_indptr = cumsum(extend) (cu_seqlens),
// out_cache_loc / positions of every new token (positions prefix + j), the
// page list of each stream and the q-tile list of the prefill attention.
//
// rollback_kernel undoes one prepare (rollback_decode_prep_after_skip): it
// returns the pages the step opened to the free list (the allocator is a
// stack, so restoring its head returns exactly those pages), lists their
// slots, decrements seq_lens and clears req_to_token at the old position.
#include <algorithm>

#include "capi_util.h"
#include "common.cuh"

namespace omni {
namespace {

constexpr int kPackThreads = 1024;

OMNI_DEVINL int block_excl_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int ws = warp_sums[lane];
    int wi = ws;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, wi, off);
      if (lane >= off) wi += n;
    }
    warp_sums[lane] = wi - ws;  // exclusive prefix of warps
    if (lane == 31) warp_sums[32] = wi;
  }
  __syncthreads();
  const int r = warp_sums[warp] + incl - v;
  total = warp_sums[32];
  __syncthreads();
  return r;
}

struct PackParams {
  int rows;
  int64_t* seq_lens;
  const int64_t* req_pool_indices;
  int32_t* req_to_token;
  int64_t max_ctx;
  int page_size;
  const int32_t* free_pages;
  int64_t num_free;
  int64_t* free_head;  // device counter
  int64_t* out_cache_loc;
  int64_t* positions;
  int32_t* kv_indptr;    // nullable
  int32_t* kv_indices;   // nullable
  int32_t* page_indptr;
  int32_t* page_indices;
  int32_t* work_indptr;  // nullable
  int pages_per_chunk;
  int* status;           // nullable: set to 1 if the free list ran dry
};

__global__ void __launch_bounds__(kPackThreads) decode_prepare_kernel(const __grid_constant__ PackParams p) {
  __shared__ int ws[33];
  __shared__ int64_t carry_need, carry_pages, carry_tokens, carry_work;
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0) {
    carry_need = 0;
    carry_pages = 0;
    carry_tokens = 0;
    carry_work = 0;
  }
  __syncthreads();
  const int64_t head0 = *p.free_head;
  for (int base = 0; base < p.rows; base += kPackThreads) {
    const int i = base + threadIdx.x;
    const bool in = i < p.rows;
    int64_t L = 0, req = 0;
    int need = 0;
    if (in) {
      L = p.seq_lens[i] + 1;
      req = p.req_pool_indices[i];
      need = ((L - 1) % p.page_size) == 0;
    }
    int tot_need;
    const int rank = block_excl_scan(need, ws, tot_need);
    if (in) {
      int64_t loc;
      if (need) {
        const int64_t slot = head0 + carry_need + rank;
        if (slot >= p.num_free) {
          if (p.status) atomicExch(p.status, 1);
          loc = 0;
        } else {
          loc = (int64_t)p.free_pages[slot] * p.page_size;
        }
      } else if (L - 2 < p.max_ctx) {
        loc = (int64_t)p.req_to_token[req * p.max_ctx + (L - 2)] + 1;
      } else {
        if (p.status) atomicExch(p.status, 2);
        loc = 0;
      }
      if (L <= p.max_ctx) p.req_to_token[req * p.max_ctx + (L - 1)] = (int32_t)loc;
      p.seq_lens[i] = L;
      p.out_cache_loc[i] = loc;
      p.positions[i] = L - 1;
    }
    const int npages = in ? (int)((L + p.page_size - 1) / p.page_size) : 0;
    const int nwork = (in && p.work_indptr) ? (npages + p.pages_per_chunk - 1) / p.pages_per_chunk : 0;
    int tot_pages, tot_tokens, tot_work;
    const int pg_off = block_excl_scan(npages, ws, tot_pages);
    const int tk_off = block_excl_scan(in ? (int)L : 0, ws, tot_tokens);
    const int wk_off = block_excl_scan(nwork, ws, tot_work);
    if (in) {
      p.page_indptr[i] = (int32_t)(carry_pages + pg_off);
      if (p.kv_indptr) p.kv_indptr[i] = (int32_t)(carry_tokens + tk_off);
      if (p.work_indptr) p.work_indptr[i] = (int32_t)(carry_work + wk_off);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      carry_need += tot_need;
      carry_pages += tot_pages;
      carry_tokens += tot_tokens;
      carry_work += tot_work;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    p.page_indptr[p.rows] = (int32_t)carry_pages;
    if (p.kv_indptr) p.kv_indptr[p.rows] = (int32_t)carry_tokens;
    if (p.work_indptr) p.work_indptr[p.rows] = (int32_t)carry_work;
    *p.free_head = head0 + carry_need;
  }
  __syncthreads();
  // page lists and token lists: one warp per row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < p.rows; i += kPackThreads / 32) {
    const int64_t req = p.req_pool_indices[i];
    const int64_t L = p.seq_lens[i];
    const int32_t* r2t = p.req_to_token + req * p.max_ctx;
    const int pbeg = p.page_indptr[i];
    const int64_t Lc = L < p.max_ctx ? L : p.max_ctx;
    const int np = (int)((Lc + p.page_size - 1) / p.page_size);
    for (int k = lane; k < np; k += 32) p.page_indices[pbeg + k] = r2t[(int64_t)k * p.page_size] / p.page_size;
    if (p.kv_indices) {
      const int tbeg = p.kv_indptr[i];
      for (int k = lane; k < Lc; k += 32) p.kv_indices[tbeg + k] = r2t[k];
    }
  }
}

__global__ void __launch_bounds__(kPackThreads) decode_rollback_kernel(int rows, int64_t* seq_lens,
                                                                       const int64_t* req_pool_indices,
                                                                       int32_t* req_to_token, int64_t max_ctx,
                                                                       int page_size, const int64_t* out_cache_loc,
                                                                       int64_t* free_head, int64_t* freed_slots,
                                                                       int64_t* num_freed) {
  __shared__ int ws[33];
  __shared__ int64_t carry;
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < rows; base += kPackThreads) {
    const int i = base + threadIdx.x;
    const bool in = i < rows;
    int64_t L = in ? seq_lens[i] : 0;
    const int opened = in && (page_size == 1 || ((L - 1) % page_size) == 0);
    int tot;
    const int rank = block_excl_scan(opened, ws, tot);
    if (opened && freed_slots) freed_slots[carry + rank] = out_cache_loc[i];
    if (in) {
      seq_lens[i] = L - 1;
      req_to_token[req_pool_indices[i] * max_ctx + (L - 1)] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *free_head -= carry;
    if (num_freed) *num_freed = carry;
  }
}

struct ExtendParams {
  int rows;
  const int64_t* prefix_lens;
  const int64_t* extend_lens;
  const int64_t* req_pool_indices;
  const int32_t* req_to_token;
  int64_t max_ctx;
  int page_size;
  int64_t* seq_lens;
  int32_t* qo_indptr;
  int64_t* out_cache_loc;
  int64_t* positions;
  int32_t* page_indptr;
  int32_t* page_indices;
  int32_t* tile_indptr;  // nullable
  int q_tile;
  int* status;
};

__global__ void __launch_bounds__(kPackThreads) extend_prepare_kernel(const __grid_constant__ ExtendParams p) {
  __shared__ int ws[33];
  __shared__ int64_t carry_q, carry_pages, carry_tiles;
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0) {
    carry_q = 0;
    carry_pages = 0;
    carry_tiles = 0;
  }
  __syncthreads();
  for (int base = 0; base < p.rows; base += kPackThreads) {
    const int i = base + threadIdx.x;
    const bool in = i < p.rows;
    int64_t E = 0, L = 0;
    if (in) {
      E = p.extend_lens[i];
      L = p.prefix_lens[i] + E;
      if (E < 0 || L > p.max_ctx) {
        if (p.status) atomicExch(p.status, 2);
        E = 0;
        L = 0;
      }
      p.seq_lens[i] = L;
    }
    const int npages = (int)((L + p.page_size - 1) / p.page_size);
    const int ntiles = p.tile_indptr ? (int)((E + p.q_tile - 1) / p.q_tile) : 0;
    int tot_q, tot_pages, tot_tiles;
    const int q_off = block_excl_scan((int)E, ws, tot_q);
    const int pg_off = block_excl_scan(npages, ws, tot_pages);
    const int t_off = block_excl_scan(ntiles, ws, tot_tiles);
    if (in) {
      p.qo_indptr[i] = (int32_t)(carry_q + q_off);
      p.page_indptr[i] = (int32_t)(carry_pages + pg_off);
      if (p.tile_indptr) p.tile_indptr[i] = (int32_t)(carry_tiles + t_off);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      carry_q += tot_q;
      carry_pages += tot_pages;
      carry_tiles += tot_tiles;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    p.qo_indptr[p.rows] = (int32_t)carry_q;
    p.page_indptr[p.rows] = (int32_t)carry_pages;
    if (p.tile_indptr) p.tile_indptr[p.rows] = (int32_t)carry_tiles;
  }
  __syncthreads();
  // one warp per stream: its new tokens' slots and positions, and its page list
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < p.rows; i += kPackThreads / 32) {
    const int64_t req = p.req_pool_indices[i];
    const int32_t* r2t = p.req_to_token + req * p.max_ctx;
    const int64_t L = p.seq_lens[i];
    const int q0 = p.qo_indptr[i], q1 = p.qo_indptr[i + 1];
    const int64_t prefix = L - (q1 - q0);
    for (int j = lane; j < q1 - q0; j += 32) {
      p.out_cache_loc[q0 + j] = r2t[prefix + j];
      p.positions[q0 + j] = prefix + j;
    }
    const int pbeg = p.page_indptr[i];
    const int np = (int)((L + p.page_size - 1) / p.page_size);
    for (int k = lane; k < np; k += 32) p.page_indices[pbeg + k] = r2t[(int64_t)k * p.page_size] / p.page_size;
  }
}

// Row moves of the per-row state tensors (batch compaction): every move copies
// row src to row dst of every tensor.  Sources and destinations are disjoint, so
// the moves run in parallel: one CTA per (move, tensor).
constexpr int kMoveThreads = 128;
constexpr int kMaxMoveTensors = 24;
constexpr int kMaxMovesPerLaunch = 384;

struct MoveParams {
  int num_tensors, num_moves;
  uint8_t* base[kMaxMoveTensors];
  int64_t row_bytes[kMaxMoveTensors];
  int64_t stride[kMaxMoveTensors];
  int32_t src[kMaxMovesPerLaunch];
  int32_t dst[kMaxMovesPerLaunch];
};

__global__ void __launch_bounds__(kMoveThreads) move_rows_kernel(const __grid_constant__ MoveParams p) {
  griddep_wait();
  griddep_launch();
  const int m = blockIdx.x, t = blockIdx.y;
  const uint8_t* from = p.base[t] + (int64_t)p.src[m] * p.stride[t];
  uint8_t* to = p.base[t] + (int64_t)p.dst[m] * p.stride[t];
  const int64_t n = p.row_bytes[t];
  const uintptr_t al = reinterpret_cast<uintptr_t>(from) | reinterpret_cast<uintptr_t>(to) | (uintptr_t)n;
  if ((al & 15) == 0) {
    for (int64_t i = threadIdx.x; i < n / 16; i += kMoveThreads)
      reinterpret_cast<uint4*>(to)[i] = reinterpret_cast<const uint4*>(from)[i];
  } else if ((al & 3) == 0) {
    for (int64_t i = threadIdx.x; i < n / 4; i += kMoveThreads)
      reinterpret_cast<uint32_t*>(to)[i] = reinterpret_cast<const uint32_t*>(from)[i];
  } else {
    for (int64_t i = threadIdx.x; i < n; i += kMoveThreads) to[i] = from[i];
  }
}

// Admission of new streams: req_to_token rows from their page lists (token t of
// stream i sits in slot pages[indptr[i] + t / P] * P + t % P), and the stream's
// batch row gets seq_len = prompt_len and its request slot.  One CTA per stream.
__global__ void __launch_bounds__(256) admit_streams_kernel(int n, const int32_t* rows, const int32_t* slots,
                                                            const int64_t* prompt_lens, const int32_t* page_indptr,
                                                            const int32_t* pages, int32_t* req_to_token,
                                                            int64_t max_ctx, int page_size, int64_t* seq_lens,
                                                            int64_t* req_pool_indices, int* status) {
  griddep_wait();
  griddep_launch();
  const int i = blockIdx.x;
  if (i >= n) return;
  const int64_t L = prompt_lens[i];
  const int64_t slot = slots[i];
  const int p0 = page_indptr[i], p1 = page_indptr[i + 1];
  if (L < 0 || L > max_ctx || (int64_t)(p1 - p0) * page_size < L) {
    if (threadIdx.x == 0 && status) atomicExch(status, 2);
    return;
  }
  int32_t* r2t = req_to_token + slot * max_ctx;
  for (int64_t t = threadIdx.x; t < L; t += blockDim.x)
    r2t[t] = pages[p0 + t / page_size] * page_size + (int32_t)(t % page_size);
  if (threadIdx.x == 0) {
    seq_lens[rows[i]] = L;
    req_pool_indices[rows[i]] = slot;
  }
}

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int omni_decode_prepare(int64_t rows, int64_t* seq_lens, const int64_t* req_pool_indices,
                                            int32_t* req_to_token, int64_t max_ctx, int32_t page_size,
                                            const int32_t* free_pages, int64_t num_free, int64_t* free_head,
                                            int64_t* out_cache_loc, int64_t* positions, int32_t* kv_indptr,
                                            int32_t* kv_indices, int32_t* page_indptr, int32_t* page_indices,
                                            int32_t* work_indptr, int32_t pages_per_chunk, int32_t* status,
                                            void* stream) {
  if (rows < 0 || max_ctx <= 0 || page_size <= 0) return set_error(OMNI_ERR_INVALID, "bad packing arguments");
  if ((kv_indptr == nullptr) != (kv_indices == nullptr))
    return set_error(OMNI_ERR_INVALID, "kv_indptr and kv_indices are given together");
  if (work_indptr && pages_per_chunk <= 0) return set_error(OMNI_ERR_INVALID, "pages_per_chunk must be > 0");
  if (rows == 0) return OMNI_OK;
  PackParams p{};
  p.rows = (int)rows;
  p.seq_lens = seq_lens;
  p.req_pool_indices = req_pool_indices;
  p.req_to_token = req_to_token;
  p.max_ctx = max_ctx;
  p.page_size = page_size;
  p.free_pages = free_pages;
  p.num_free = num_free;
  p.free_head = free_head;
  p.out_cache_loc = out_cache_loc;
  p.positions = positions;
  p.kv_indptr = kv_indptr;
  p.kv_indices = kv_indices;
  p.page_indptr = page_indptr;
  p.page_indices = page_indices;
  p.work_indptr = work_indptr;
  p.pages_per_chunk = pages_per_chunk;
  p.status = status;
  return check_launch(
      launch(decode_prepare_kernel, dim3(1), dim3(kPackThreads), 0, static_cast<cudaStream_t>(stream), p));
}

extern "C" OMNI_API int omni_decode_rollback(int64_t rows, int64_t* seq_lens, const int64_t* req_pool_indices,
                                             int32_t* req_to_token, int64_t max_ctx, int32_t page_size,
                                             const int64_t* out_cache_loc, int64_t* free_head,
                                             int64_t* freed_slots, int64_t* num_freed, void* stream) {
  if (rows < 0 || max_ctx <= 0 || page_size <= 0) return set_error(OMNI_ERR_INVALID, "bad rollback arguments");
  if (rows == 0) return OMNI_OK;
  return check_launch(launch(decode_rollback_kernel, dim3(1), dim3(kPackThreads), 0,
                             static_cast<cudaStream_t>(stream), (int)rows, seq_lens, req_pool_indices, req_to_token,
                             max_ctx, (int)page_size, out_cache_loc, free_head, freed_slots, num_freed));
}

extern "C" OMNI_API int omni_extend_prepare(int64_t rows, const int64_t* prefix_lens, const int64_t* extend_lens,
                                            const int64_t* req_pool_indices, const int32_t* req_to_token,
                                            int64_t max_ctx, int32_t page_size, int64_t* seq_lens,
                                            int32_t* qo_indptr, int64_t* out_cache_loc, int64_t* positions,
                                            int32_t* page_indptr, int32_t* page_indices, int32_t* tile_indptr,
                                            int32_t q_tile, int32_t* status, void* stream) {
  if (rows < 0 || max_ctx <= 0 || page_size <= 0) return set_error(OMNI_ERR_INVALID, "bad packing arguments");
  if (tile_indptr && q_tile <= 0) return set_error(OMNI_ERR_INVALID, "q_tile must be > 0");
  if (rows == 0) return OMNI_OK;
  ExtendParams p{};
  p.rows = (int)rows;
  p.prefix_lens = prefix_lens;
  p.extend_lens = extend_lens;
  p.req_pool_indices = req_pool_indices;
  p.req_to_token = req_to_token;
  p.max_ctx = max_ctx;
  p.page_size = page_size;
  p.seq_lens = seq_lens;
  p.qo_indptr = qo_indptr;
  p.out_cache_loc = out_cache_loc;
  p.positions = positions;
  p.page_indptr = page_indptr;
  p.page_indices = page_indices;
  p.tile_indptr = tile_indptr;
  p.q_tile = q_tile;
  p.status = status;
  return check_launch(
      launch(extend_prepare_kernel, dim3(1), dim3(kPackThreads), 0, static_cast<cudaStream_t>(stream), p));
}

extern "C" OMNI_API int omni_move_rows(void* const* bases, const int64_t* row_bytes, const int64_t* row_strides,
                                       int32_t num_tensors, const int32_t* src, const int32_t* dst,
                                       int32_t num_moves, void* stream) {
  if (num_tensors < 0 || num_tensors > kMaxMoveTensors || num_moves < 0)
    return set_error(OMNI_ERR_INVALID, "move_rows: at most 24 tensors");
  if (num_moves == 0 || num_tensors == 0) return OMNI_OK;
  if (!bases || !row_bytes || !row_strides || !src || !dst) return set_error(OMNI_ERR_INVALID, "move_rows: null array");
  MoveParams p{};
  p.num_tensors = num_tensors;
  for (int t = 0; t < num_tensors; ++t) {
    if (!bases[t] || row_bytes[t] < 0 || row_strides[t] < row_bytes[t])
      return set_error(OMNI_ERR_INVALID, "move_rows: bad tensor descriptor");
    p.base[t] = static_cast<uint8_t*>(bases[t]);
    p.row_bytes[t] = row_bytes[t];
    p.stride[t] = row_strides[t];
  }
  for (int m = 0; m < num_moves; ++m)
    if (src[m] < 0 || dst[m] < 0) return set_error(OMNI_ERR_INVALID, "move_rows: negative row");
  for (int m0 = 0; m0 < num_moves; m0 += kMaxMovesPerLaunch) {
    const int k = std::min(kMaxMovesPerLaunch, num_moves - m0);
    p.num_moves = k;
    for (int m = 0; m < k; ++m) {
      p.src[m] = src[m0 + m];
      p.dst[m] = dst[m0 + m];
    }
    const int rc = check_launch(launch(move_rows_kernel, dim3(k, num_tensors), dim3(kMoveThreads), 0,
                                       static_cast<cudaStream_t>(stream), p));
    if (rc != OMNI_OK) return rc;
  }
  return OMNI_OK;
}

extern "C" OMNI_API int omni_admit_streams(int64_t n, const int32_t* rows, const int32_t* slots,
                                           const int64_t* prompt_lens, const int32_t* page_indptr,
                                           const int32_t* pages, int32_t* req_to_token, int64_t max_ctx,
                                           int32_t page_size, int64_t* seq_lens, int64_t* req_pool_indices,
                                           int32_t* status, void* stream) {
  if (n < 0 || max_ctx <= 0 || page_size <= 0) return set_error(OMNI_ERR_INVALID, "bad admission arguments");
  if (n == 0) return OMNI_OK;
  return check_launch(launch(admit_streams_kernel, dim3((unsigned)n), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), (int)n, rows, slots, prompt_lens, page_indptr, pages,
                             req_to_token, max_ctx, (int)page_size, seq_lens, req_pool_indices, status));
}
