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
// rollback_kernel undoes one prepare (rollback_decode_prep_after_skip): it
// returns the pages the step opened to the free list (the allocator is a
// stack, so restoring its head returns exactly those pages), lists their
// slots, decrements seq_lens and clears req_to_token at the old position.
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
