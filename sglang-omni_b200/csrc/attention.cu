// Attention kernels of the decode step.
//
// paged_decode_attention_kernel — GQA decode over the paged KV pool (L1:
//   RadixAttention decode, thinker_model.py:373-379).  The batch's flattened page
//   list is cut into equal ranges (row pieces weighted by their fixed cost), two
//   CTAs per SM over the KV heads; the 4 warps of a CTA take a piece's pages in
//   turn, each streaming whole pages (16 tokens x head_dim, K and V) with 16-byte
//   cp.async into a swizzled ring, and run S = K Q^T and O^T += V^T P^T on mma.sync
//   m16n8k16 (the group's 8 query heads), with an online base-2 softmax.  Warps
//   combine in shared memory; rows spread over several ranges are merged by
//   paged_attention_merge_kernel in segment order (deterministic).
//
// The causal extend (prefill) attention is in prefill_attention.cu.
//
// predictor_attention_kernel — the code predictor's attention over its <= G+1
//   per-request cache slots (predictor_cached_self_attention,
//   sglang_model.py:2168-2233; decode_attention_kernel,
//   predictor_layers.py:336-396): one warp per (row, KV head) serving the
//   group's query heads, lanes = slots, causal for the opening pair; every K and V
//   load is issued up front (the earlier passes' slots before the PDL wait), V rows
//   into shared memory.
#include <mutex>

#include "capi_util.h"
#include "common.cuh"

namespace omni {
namespace {

constexpr int kPage = 16;
constexpr int kD = 128;       // head_dim of the talker
constexpr int kGroup = 8;     // query heads per KV head
constexpr int kPageBytes = kPage * kD * 2;  // one head's K (or V) page: 4 KB

OMNI_DEVINL void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
OMNI_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
OMNI_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
OMNI_DEVINL void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
OMNI_DEVINL void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
OMNI_DEVINL void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Swizzled offset of (token row, 16-byte chunk) inside a 16 x 256-byte page tile.
OMNI_DEVINL uint32_t swz(int row, int chunk) { return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4)); }

constexpr int kAttnWarps = 4;
constexpr int kWarpStages = 3;                // pages in flight per warp
constexpr int kCombStride = kD + 4;           // padded head stride of the combine area
constexpr int kStageBytes = 2 * kPageBytes;   // K + V of one head's page: 8 KB
constexpr int kMaxRowsInSmem = 512;
constexpr int kCombSlot = kWarpStages - 1;    // the ring stage that holds a warp's combine partial
static_assert((kGroup * kCombStride + 2 * kGroup) * 4 <= kStageBytes, "combine partial exceeds a ring stage");

struct PagedAttnParams {
  const uint16_t* q;  // [B, Hq, D] row stride q_stride
  int64_t q_stride;
  const uint16_t* k_cache;  // [slots, Hkv, D]
  const uint16_t* v_cache;
  const int32_t* page_indptr;  // [B + 1]
  const int32_t* page_indices;
  const int64_t* seq_lens;     // [B]
  int rows, hkv, ctas;         // ctas: CTAs per KV head (grid x)
  float scale_log2;  // softmax scale * log2(e)
  uint16_t* out;     // [B, Hq, D]
  int64_t out_stride;
  float* part_o;     // [segments][Hkv][8][D]
  float* part_lse;   // [segments][Hkv][8]
  int* counters;     // [B][Hkv]
};

// The flattened page list is cut in a virtual space where every row is preceded by
// w units (the fixed cost of a row piece: its queries, the warps' combine and the
// store), so that CTAs whose ranges hold many short rows get fewer pages: row b's
// pages sit at virtual positions [pptr[b] + (b + 1) w, pptr[b + 1] + (b + 1) w).
// w = kRowWeight once the batch has more pages than ranges; with fewer, every range is
// one page (w = 0) and a row's split does not depend on the other rows.
#ifndef OMNI_ATTN_ROW_WEIGHT
#define OMNI_ATTN_ROW_WEIGHT 4
#endif
constexpr int kRowWeight = OMNI_ATTN_ROW_WEIGHT;
// First virtual position of CTA c's range: [bound(c), bound(c + 1)).
OMNI_DEVINL int range_bound(int c, int total, int ctas) { return (int)(((int64_t)total * c) / ctas); }
// CTA whose range holds flattened page `pos` (ranges are non-empty: ctas <= total).
OMNI_DEVINL int cta_of(int pos, int total, int ctas) {
  int c = (int)(((int64_t)pos * ctas) / total);
  while (c + 1 < ctas && range_bound(c + 1, total, ctas) <= pos) ++c;
  while (c > 0 && range_bound(c, total, ctas) > pos) --c;
  return c;
}

// Split-KV decode attention with a balanced split: the flattened page list of the batch
// is cut into `ctas` equal ranges per KV head (two CTAs per SM over both heads); CTA c
// walks the row pieces of its range in order.  The 4 warps take the pages of a piece in
// turn, each keeping kWarpStages pages in flight (16-byte cp.async into a swizzled
// per-warp ring).  Per page a warp computes S^T = K Q^T (16 tokens x the group's 8
// query heads, mma.sync m16n8k16 with K as the A operand, so no padding rows), an online
// base-2 softmax per head, and O^T += V^T P^T (V^T by transposed ldmatrix, P^T moved
// into the B-operand layout by four shuffles).  The warps combine in shared memory, each
// warp's partial in the last stage of its ring, while the next piece's first pages
// already stream into the other stages (no memory-latency bubble at row boundaries); a
// piece that is the whole row stores it, otherwise the piece's (o, lse) goes to segment
// c + b and paged_attention_merge_kernel (the next launch) merges the row's segments in
// order (deterministic).
__global__ void __launch_bounds__(kAttnWarps * 32, 2) paged_decode_attention_kernel(
    const __grid_constant__ PagedAttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_ptr[kMaxRowsInSmem + 1];  // page_indptr, when the batch fits
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int h = blockIdx.y, c = blockIdx.x;
  // The page table and sequence lengths are step metadata written before the previous
  // kernel started, and so is every KV slot but each row's newest token: the tables and
  // the first pages are read before griddepcontrol.wait, overlapping the previous
  // kernel's tail.  The queries and each row's last page are read after it.
  const bool ptr_in_smem = p.rows <= kMaxRowsInSmem;
  if (ptr_in_smem)
    for (int i = threadIdx.x; i <= p.rows; i += blockDim.x) s_ptr[i] = p.page_indptr[i];
  __syncthreads();
  const int* pptr = ptr_in_smem ? s_ptr : p.page_indptr;
  const int total = pptr[p.rows];
  // at most one CTA per page (ctas <= total <= the virtual length): every range is non-empty
  const int ctas = min(p.ctas, total);
  if (c >= ctas) {
    griddep_wait();
    griddep_launch();
    return;
  }
  const int rw = total > p.ctas ? kRowWeight : 0;
  const int tv = total + p.rows * rw;  // virtual length
  const int a0 = range_bound(c, tv, ctas), a1 = range_bound(c + 1, tv, ctas);
  int lo = 0, hi = p.rows - 1;  // first row of the range: first b whose virtual end passes a0
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (pptr[mid + 1] + (mid + 1) * rw > a0) hi = mid;
    else lo = mid + 1;
  }
  uint8_t* wring = smem + warp * (kWarpStages * kStageBytes);
  // combine area of warp w: the last stage of its ring ([8][kCombStride] o, then m[8],
  // l[8]); at a piece boundary the next piece's first pages already stream into the
  // other stages while the warps combine
  auto comb = [&](int w) { return reinterpret_cast<float*>(smem + (w * kWarpStages + kCombSlot) * kStageBytes); };

  // the next row piece of the range from row bb on: (b, r0, r1) with r0 < r1
  auto find_piece = [&](int bb, int& b, int& r0, int& r1) -> bool {
    for (b = bb; b < p.rows && pptr[b] + (b + 1) * rw < a1; ++b) {
      const int off = (b + 1) * rw;  // virtual - page position in row b
      r0 = max(a0 - off, pptr[b]);
      r1 = min(a1 - off, pptr[b + 1]);
      if (r0 < r1) return true;
    }
    return false;
  };
  // this warp's pages of a piece: r0 + warp + 4 i, i < nmine; ids one per lane
  int pid_lane = 0, nmine = 0, cur_r0 = 0;
  auto issue = [&](int i) {  // i-th page of this warp into stage i % kWarpStages
    const int64_t page = i < 32 ? __shfl_sync(0xFFFFFFFFu, pid_lane, i)
                                : p.page_indices[cur_r0 + warp + kAttnWarps * i];
    const uint16_t* kbase = p.k_cache + (page * kPage * p.hkv + h) * kD;
    const uint16_t* vbase = p.v_cache + (page * kPage * p.hkv + h) * kD;
    uint8_t* kd = wring + (i % kWarpStages) * kStageBytes;
    uint8_t* vd = kd + kPageBytes;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int id = u * 32 + lane;
      const int row = id >> 4, ch = id & 15;
      const int64_t goff = (int64_t)row * p.hkv * kD + ch * 8;
      cp_async16(kd + swz(row, ch), kbase + goff);
      cp_async16(vd + swz(row, ch), vbase + goff);
    }
    cp_async_commit();
  };
  auto piece_ids = [&](int r0, int r1) {
    cur_r0 = r0;
    const int npg = r1 - r0;
    nmine = npg > warp ? (npg - warp + kAttnWarps - 1) / kAttnWarps : 0;
    pid_lane = lane < nmine ? p.page_indices[r0 + warp + kAttnWarps * lane] : 0;
  };
  int b, r0, r1;
  bool have = find_piece(lo, b, r0, r1);
  // The first piece's pages stream in before the wait, up to its row's last page: only
  // that page holds a token the previous kernel may have stored (the step's new KV).
  int early = 0;
  if (have) {
    piece_ids(r0, r1);
    const int first = nmine < kWarpStages ? nmine : kWarpStages;
    const int last_pos = pptr[b + 1] - 1;
    while (early < first && r0 + warp + kAttnWarps * early != last_pos) issue(early++);
  }
  griddep_wait();
  griddep_launch();
  if (have) {
    const int first = nmine < kWarpStages ? nmine : kWarpStages;
    for (int i = early; i < first; ++i) issue(i);
  }
  // Q^T as the B operand: head g, dims 16 ks + 2t (+1) and + 8; the next piece's row
  // is loaded at the piece boundary, during the combine
  uint32_t qb[8][2];
  auto load_q = [&](int row) {
    const uint16_t* qrow = p.q + (int64_t)row * p.q_stride + (int64_t)(h * kGroup + g) * kD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qb[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 2 * t);
      qb[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8 + 2 * t);
    }
  };
  int seq_len = 0;
  if (have) {
    load_q(b);
    seq_len = (int)p.seq_lens[b];
  }
  while (have) {
    const int rp0 = pptr[b], rp1 = pptr[b + 1];
    // O^T accumulators: m-tile mt holds dims 16 mt + g (+ 8) for heads 2t, 2t + 1
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // heads 2t, 2t + 1
    const int src_a = 8 * t + (g >> 1), src_b = src_a + 4;       // lanes holding P[g][2t], P[g][2t + 1]

    for (int i = 0; i < nmine; ++i) {
      // page i is complete once at most (issued - i - 1) later groups are pending
      const int pending = min(nmine, i + kWarpStages) - i - 1;
      if (pending >= 2) cp_async_wait<2>();
      else if (pending == 1) cp_async_wait<1>();
      else cp_async_wait<0>();
      __syncwarp();
      uint8_t* kd = wring + (i % kWarpStages) * kStageBytes;
      const int tok_base = (r0 - rp0 + warp + kAttnWarps * i) * kPage;
      if (seq_len - tok_base < kPage) {
        // slots past the sequence end hold stale values: zero their V rows so
        // that P = 0 never meets a non-finite value in P V
        uint8_t* vd = kd + kPageBytes;
        const int f0 = max(seq_len - tok_base, 0);
        for (int id = f0 * 16 + lane; id < kPage * 16; id += 32)
          *reinterpret_cast<uint4*>(vd + swz(id >> 4, id & 15)) = make_uint4(0, 0, 0, 0);
        __syncwarp();
      }
      const uint32_t kb = smem_u32(kd);
      const uint32_t vb = kb + kPageBytes;
      // S^T = K Q^T: 16 tokens x 8 heads
      float sacc[4] = {0, 0, 0, 0};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int tok = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = 2 * ks + (lane >> 4);
        uint32_t x0, x1, x2, x3;
        ldsm_x4(kb + swz(tok, ch), x0, x1, x2, x3);
        mma_bf16_16816(sacc, x0, x1, x2, x3, qb[ks][0], qb[ks][1]);
      }
      // sacc: [0] token g head 2t, [1] token g head 2t+1, [2] token g+8 head 2t, [3] token g+8 head 2t+1
      const bool v_lo = tok_base + g < seq_len, v_hi = tok_base + g + 8 < seq_len;
      const float s0 = v_lo ? sacc[0] * p.scale_log2 : -INFINITY;
      const float s1 = v_lo ? sacc[1] * p.scale_log2 : -INFINITY;
      const float s2 = v_hi ? sacc[2] * p.scale_log2 : -INFINITY;
      const float s3 = v_hi ? sacc[3] * p.scale_log2 : -INFINITY;
      float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float al0 = (m0 == -INFINITY) ? 0.0f : exp2f(m0 - mn0);
      const float al1 = (m1 == -INFINITY) ? 0.0f : exp2f(m1 - mn1);
      const float p0 = s0 == -INFINITY ? 0.0f : exp2f(s0 - mn0);
      const float p1 = s1 == -INFINITY ? 0.0f : exp2f(s1 - mn1);
      const float p2 = s2 == -INFINITY ? 0.0f : exp2f(s2 - mn0);
      const float p3 = s3 == -INFINITY ? 0.0f : exp2f(s3 - mn1);
      float rs0 = p0 + p2, rs1 = p1 + p3;
#pragma unroll
      for (int off = 4; off <= 16; off <<= 1) {
        rs0 += __shfl_xor_sync(0xFFFFFFFFu, rs0, off);
        rs1 += __shfl_xor_sync(0xFFFFFFFFu, rs1, off);
      }
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
      }
      // P^T as the B operand: this lane needs P[head g][tokens 2t, 2t+1, 2t+8, 2t+9];
      // lane 8t' + j holds tokens (2t' + (j >> 2)) of the pair-packed heads 2 (j & 3), + 1
      const uint32_t x01 = pack_bf2(p0, p1), x23 = pack_bf2(p2, p3);
      const uint32_t a01 = __shfl_sync(0xFFFFFFFFu, x01, src_a), b01 = __shfl_sync(0xFFFFFFFFu, x01, src_b);
      const uint32_t a23 = __shfl_sync(0xFFFFFFFFu, x23, src_a), b23 = __shfl_sync(0xFFFFFFFFu, x23, src_b);
      // head g is the low half of the pair when g is even
      const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
      const uint32_t pb0 = __byte_perm(a01, b01, sel), pb1 = __byte_perm(a23, b23, sel);
      // O^T += V^T P^T, 8 m-tiles of 16 dims
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int tok = (lane & 7) + ((lane >> 4) << 3);
        const int ch = 2 * mt + ((lane >> 3) & 1);
        uint32_t x0, x1, x2, x3;
        ldsm_x4_t(vb + swz(tok, ch), x0, x1, x2, x3);
        mma_bf16_16816(o[mt], x0, x1, x2, x3, pb0, pb1);
      }
      __syncwarp();
      if (i + kWarpStages < nmine) issue(i + kWarpStages);
    }

    // ---- the next piece's first pages stream in during the combine ----
    // (this warp's stages are all consumed; the combine slot is left out)
    const bool whole = r0 == rp0 && r1 == rp1;
    const int seg = c + b;
    int nb = 0, nr0 = 0, nr1 = 0;
    const bool nhave = find_piece(b + 1, nb, nr0, nr1);
    if (nhave) {
      piece_ids(nr0, nr1);
      const int pre = nmine < kCombSlot ? nmine : kCombSlot;
      for (int i = 0; i < pre; ++i) issue(i);
      load_q(nb);
    }
    const int seq_next = nhave ? (int)p.seq_lens[nb] : 0;
    // ---- combine the warps ----
    {
      float* wo = comb(warp);
      float* wm = wo + kGroup * kCombStride;
      if (g == 0) {
        wm[2 * t] = m0;
        wm[2 * t + 1] = m1;
        wm[kGroup + 2 * t] = l0;
        wm[kGroup + 2 * t + 1] = l1;
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        float* w0 = wo + (2 * t) * kCombStride + 16 * mt + g;
        float* w1 = w0 + kCombStride;
        w0[0] = o[mt][0];
        w1[0] = o[mt][1];
        w0[8] = o[mt][2];
        w1[8] = o[mt][3];
      }
    }
    __syncthreads();
    const int hg = threadIdx.x >> 4;          // head within group
    const int d0 = (threadIdx.x & 15) * 8;    // 8 dims
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float M = -INFINITY, L = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, comb(w)[kGroup * kCombStride + hg]);
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float* wo = comb(w);
      const float lw = wo[kGroup * kCombStride + kGroup + hg];
      if (lw == 0.0f) continue;
      const float sc = exp2f(wo[kGroup * kCombStride + hg] - M);
      L += lw * sc;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += wo[hg * kCombStride + d0 + e] * sc;
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    if (whole) {
      uint16_t* dst = p.out + (int64_t)b * p.out_stride + (int64_t)(h * kGroup + hg) * kD + d0;
      *reinterpret_cast<uint4*>(dst) =
          make_uint4(pack_bf2(acc[0] * inv, acc[1] * inv), pack_bf2(acc[2] * inv, acc[3] * inv),
                     pack_bf2(acc[4] * inv, acc[5] * inv), pack_bf2(acc[6] * inv, acc[7] * inv));
    } else {
      float* po = p.part_o + (((int64_t)seg * p.hkv + h) * kGroup + hg) * kD + d0;
      *reinterpret_cast<float4*>(po) = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
      *reinterpret_cast<float4*>(po + 4) = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
      if ((threadIdx.x & 15) == 0)
        p.part_lse[((int64_t)seg * p.hkv + h) * kGroup + hg] = L > 0.0f ? M + log2f(L) : -INFINITY;
    }
    __syncthreads();  // the combine slots are free for the next piece
    if (nhave)
      for (int i = kCombSlot; i < (nmine < kWarpStages ? nmine : kWarpStages); ++i) issue(i);
    have = nhave;
    seq_len = seq_next;
    b = nb;
    r0 = nr0;
    r1 = nr1;
  }
}

// Rows whose pages span several CTA ranges: row b's segments are c_lo + b .. c_hi + b
// (the ranges holding its first and last pages), merged in segment order with their
// log-sum-exp weights.  Rows held by one range were stored by the attention kernel.
__global__ void __launch_bounds__(kGroup * 16) paged_attention_merge_kernel(const __grid_constant__ PagedAttnParams p) {
  const int b = blockIdx.x, h = blockIdx.y;
  // step metadata, read before the wait (as in the attention kernel)
  const int total = p.page_indptr[p.rows];
  const int rp0 = p.page_indptr[b], rp1 = p.page_indptr[b + 1];
  griddep_wait();
  griddep_launch();
  if (rp0 >= rp1) return;
  const int ctas = min(p.ctas, total);
  const int rw = total > p.ctas ? kRowWeight : 0;
  const int tv = total + p.rows * rw, off = (b + 1) * rw;
  const int c_lo = cta_of(rp0 + off, tv, ctas), c_hi = cta_of(rp1 - 1 + off, tv, ctas);
  const int nseg = c_hi - c_lo + 1;
  if (nseg == 1) return;
  const int hg = threadIdx.x >> 4;        // head within group
  const int d0 = (threadIdx.x & 15) * 8;  // 8 dims
  const int w0 = c_lo + b;
  float M = -INFINITY;
  for (int cc = 0; cc < nseg; ++cc) M = fmaxf(M, p.part_lse[((int64_t)(w0 + cc) * p.hkv + h) * kGroup + hg]);
  float W = 0.0f, sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  // segments in batches of 8 with every load of a batch in flight before the sums,
  // summed in segment order
  for (int s0 = 0; s0 < nseg; s0 += 8) {
    float lse[8];
    float4 lo4[8], hi4[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (s0 + u < nseg) {
        const int64_t base = ((int64_t)(w0 + s0 + u) * p.hkv + h) * kGroup + hg;
        lse[u] = p.part_lse[base];
        const float4* pp = reinterpret_cast<const float4*>(p.part_o + base * kD + d0);
        lo4[u] = pp[0];
        hi4[u] = pp[1];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (s0 + u < nseg) {
        const float wgt = lse[u] == -INFINITY ? 0.0f : exp2f(lse[u] - M);
        W += wgt;
        sum[0] += lo4[u].x * wgt;
        sum[1] += lo4[u].y * wgt;
        sum[2] += lo4[u].z * wgt;
        sum[3] += lo4[u].w * wgt;
        sum[4] += hi4[u].x * wgt;
        sum[5] += hi4[u].y * wgt;
        sum[6] += hi4[u].z * wgt;
        sum[7] += hi4[u].w * wgt;
      }
    }
  }
  const float iw = W > 0.0f ? 1.0f / W : 0.0f;
  uint16_t* dst = p.out + (int64_t)b * p.out_stride + (int64_t)(h * kGroup + hg) * kD + d0;
  *reinterpret_cast<uint4*>(dst) =
      make_uint4(pack_bf2(sum[0] * iw, sum[1] * iw), pack_bf2(sum[2] * iw, sum[3] * iw),
                 pack_bf2(sum[4] * iw, sum[5] * iw), pack_bf2(sum[6] * iw, sum[7] * iw));
}


// ---------------------------------------------------------------------------
// Predictor attention: rows laid out (request, token); a row attends to the
// request's slots [0, base + t] (t = the row's token index within the request).
// One warp per (row, KV head) serves the G query heads of the group: lane s
// scores slot s (<= 32 slots) against every query head of the group, the
// softmax runs across lanes, then lane l accumulates dimensions
// [l*D/32, (l+1)*D/32) of P V over the slots.
// ---------------------------------------------------------------------------
template <int E, int G>  // head_dim = 32 * E, G query heads per KV head
__global__ void __launch_bounds__(128) predictor_attention_kernel(const uint16_t* __restrict__ q, int64_t q_stride,
                                                                  const uint16_t* __restrict__ k_cache,
                                                                  const uint16_t* __restrict__ v_cache, int rows,
                                                                  int hq, int hkv, int tokens_per_req,
                                                                  int slot_stride, int slot_base, float scale,
                                                                  uint16_t* __restrict__ out, int64_t out_stride) {
  constexpr int D = 32 * E;
  constexpr int CH = D / 8;  // 16-byte chunks of a K or V row
  __shared__ float qs[4][G][D];
  __shared__ __align__(16) uint16_t vs[4][32][D];  // this warp's V rows, slot-major
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int item = blockIdx.x * 4 + warp;
  const bool live = item < rows * hkv;
  const int row = live ? item / hkv : 0, kvh = live ? item % hkv : 0;
  const int req = row / tokens_per_req, tk = row % tokens_per_req;
  const int last = slot_base + tk;  // inclusive
  const int64_t slot0 = (int64_t)req * slot_stride;
  const uint16_t* kbase = k_cache + (slot0 * hkv + kvh) * D;
  const uint16_t* vbase = v_cache + (slot0 * hkv + kvh) * D;
  // The slots before slot_base were stored by earlier passes: their K row (lane = slot)
  // and V rows load before griddepcontrol.wait; the step's own slots (and q) after it.
  uint4 kreg[CH];
  if (live && lane < slot_base) {
#pragma unroll
    for (int c = 0; c < CH; ++c) kreg[c] = reinterpret_cast<const uint4*>(kbase + (int64_t)lane * hkv * D)[c];
  }
  if (live)
    for (int idx = lane; idx < slot_base * CH; idx += 32)
      cp_async16(&vs[warp][idx / CH][(idx % CH) * 8], vbase + (int64_t)(idx / CH) * hkv * D + (idx % CH) * 8);
  griddep_wait();
  griddep_launch();
  if (!live) return;
  if (lane >= slot_base && lane <= last) {
#pragma unroll
    for (int c = 0; c < CH; ++c) kreg[c] = reinterpret_cast<const uint4*>(kbase + (int64_t)lane * hkv * D)[c];
  }
  for (int idx = slot_base * CH + lane; idx < (last + 1) * CH; idx += 32)
    cp_async16(&vs[warp][idx / CH][(idx % CH) * 8], vbase + (int64_t)(idx / CH) * hkv * D + (idx % CH) * 8);
  cp_async_commit();
  // the group's query heads, scaled, into this warp's shared slice
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < E; ++j)
      qs[warp][g][E * lane + j] = bf2f(q[row * q_stride + (kvh * G + g) * D + E * lane + j]) * scale;
  __syncwarp();
  // scores: lane = slot
  float sc[G];
  const bool valid = lane <= last;
  if (valid) {
#pragma unroll
    for (int g = 0; g < G; ++g) sc[g] = 0.0f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const uint32_t w[4] = {kreg[c].x, kreg[c].y, kreg[c].z, kreg[c].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float k0 = bf_lo(w[e]), k1 = bf_hi(w[e]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          sc[g] = __fmaf_rn(qs[warp][g][8 * c + 2 * e], k0, sc[g]);
          sc[g] = __fmaf_rn(qs[warp][g][8 * c + 2 * e + 1], k1, sc[g]);
        }
      }
    }
  } else {
#pragma unroll
    for (int g = 0; g < G; ++g) sc[g] = -INFINITY;
  }
  float pr[G], inv[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float m = warp_max_xor(sc[g]);
    pr[g] = valid ? expf(sc[g] - m) : 0.0f;
    inv[g] = 1.0f / warp_sum_xor(pr[g]);
  }
  cp_async_wait<0>();
  __syncwarp();
  // P V: lane l owns dimensions E*l .. E*l+E-1
  float acc[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < E; ++j) acc[g][j] = 0.0f;
  for (int sl = 0; sl <= last; ++sl) {
    const uint16_t* vrow = &vs[warp][sl][E * lane];
    float v[E];
    if constexpr (E == 2) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(vrow);
      v[0] = bf_lo(w);
      v[1] = bf_hi(w);
    } else {
      const uint2 w = *reinterpret_cast<const uint2*>(vrow);
      v[0] = bf_lo(w.x);
      v[1] = bf_hi(w.x);
      v[2] = bf_lo(w.y);
      v[3] = bf_hi(w.y);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float ps = __shfl_sync(0xFFFFFFFFu, pr[g], sl);
#pragma unroll
      for (int j = 0; j < E; ++j) acc[g][j] = __fmaf_rn(ps, v[j], acc[g][j]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < E; ++j)
      out[row * out_stride + (kvh * G + g) * D + E * lane + j] = f2bf(acc[g][j] * inv[g]);
}

}  // namespace
}  // namespace omni

using namespace omni;

// -1 for a negative size or one whose byte count would not fit in 2^60.
extern "C" OMNI_API int64_t omni_paged_attention_workspace_bytes(int64_t rows, int32_t num_kv_heads,
                                                                 int64_t work_capacity) {
  constexpr int64_t kLimit = int64_t(1) << 60;
  if (rows < 0 || num_kv_heads <= 0 || work_capacity < 0) return -1;
  if (rows > kLimit / (4 * (int64_t)num_kv_heads) ||
      work_capacity > kLimit / ((int64_t)num_kv_heads * kGroup * (kD + 1) * 4 + 256))
    return -1;
  const int64_t ctr = (rows * num_kv_heads * 4 + 255) / 256 * 256;
  const int64_t lse = (work_capacity * num_kv_heads * kGroup * 4 + 255) / 256 * 256;
  return ctr + lse + work_capacity * num_kv_heads * kGroup * kD * 4;
}

extern "C" OMNI_API int omni_paged_decode_attention(const void* q, int64_t q_stride, const void* k_cache,
                                                    const void* v_cache, const int32_t* page_indptr,
                                                    const int32_t* page_indices, const int64_t* seq_lens,
                                                    const int32_t* work_indptr, int64_t rows, int32_t num_q_heads,
                                                    int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                                    int32_t pages_per_chunk, int64_t work_capacity, float sm_scale,
                                                    void* out, int64_t out_stride, void* workspace,
                                                    int64_t workspace_bytes, int32_t grid_ctas, void* stream) {
  if (rows < 0 || num_kv_heads <= 0 || pages_per_chunk <= 0) return set_error(OMNI_ERR_INVALID, "bad attention shape");
  if (head_dim != kD || page_size != kPage || num_q_heads != num_kv_heads * kGroup)
    return set_error(OMNI_ERR_UNSUPPORTED, "paged attention supports head_dim 128, page 16, 8 query heads per KV head");
  if ((reinterpret_cast<uintptr_t>(out) & 15) || out_stride % 8 || (reinterpret_cast<uintptr_t>(q) & 3) ||
      q_stride % 2 || (reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
    return set_error(OMNI_ERR_UNSUPPORTED, "misaligned attention operands");
  const int64_t need = omni_paged_attention_workspace_bytes(rows, num_kv_heads, work_capacity);
  if (need < 0) return set_error(OMNI_ERR_INVALID, "attention workspace size out of range");
  if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(OMNI_ERR_CAPACITY, "attention workspace too small or misaligned");
  if (rows == 0) return OMNI_OK;
  // one partial segment per (row, CTA page range) piece: at most ctas + rows - 1 of them
  const int sms = device_sm_count();
  // two CTAs per SM over all KV heads
  int64_t ctas = grid_ctas > 0 ? grid_ctas : (2 * sms) / num_kv_heads;
  if (ctas > work_capacity - rows + 1) ctas = work_capacity - rows + 1;
  if (ctas < 1) return set_error(OMNI_ERR_CAPACITY, "attention work capacity below the row count");
  PagedAttnParams p{};
  p.q = static_cast<const uint16_t*>(q);
  p.q_stride = q_stride;
  p.k_cache = static_cast<const uint16_t*>(k_cache);
  p.v_cache = static_cast<const uint16_t*>(v_cache);
  p.page_indptr = page_indptr;
  p.page_indices = page_indices;
  p.seq_lens = seq_lens;
  p.rows = (int)rows;
  p.hkv = num_kv_heads;
  p.ctas = (int)ctas;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.out = static_cast<uint16_t*>(out);
  p.out_stride = out_stride;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t ctr = (rows * num_kv_heads * 4 + 255) / 256 * 256;
  const int64_t lse = (work_capacity * num_kv_heads * kGroup * 4 + 255) / 256 * 256;
  p.counters = reinterpret_cast<int*>(ws);
  p.part_lse = reinterpret_cast<float*>(ws + ctr);
  p.part_o = reinterpret_cast<float*>(ws + ctr + lse);
  const size_t smem = (size_t)kAttnWarps * kWarpStages * kStageBytes;  // 96 KB of rings (+ combine area)
  // the attribute belongs to the device that is current when it is set
  const cudaError_t e = once_per_device(reinterpret_cast<const void*>(paged_decode_attention_kernel), kAttrSmem, [smem] {
    return cudaFuncSetAttribute(paged_decode_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (e != cudaSuccess) return check_launch(e);
  (void)work_indptr;
  (void)pages_per_chunk;
  const int rc = check_launch(launch(paged_decode_attention_kernel, dim3((unsigned)ctas, (unsigned)num_kv_heads),
                                     dim3(kAttnWarps * 32), smem, static_cast<cudaStream_t>(stream), p));
  if (rc != OMNI_OK) return rc;
  return check_launch(launch(paged_attention_merge_kernel, dim3((unsigned)rows, (unsigned)num_kv_heads),
                             dim3(kGroup * 16), 0, static_cast<cudaStream_t>(stream), p));
}

extern "C" OMNI_API int omni_predictor_attention(const void* q, int64_t q_stride, const void* k_cache,
                                                 const void* v_cache, int64_t rows, int32_t num_q_heads,
                                                 int32_t num_kv_heads, int32_t head_dim, int32_t tokens_per_req,
                                                 int32_t slot_stride, int32_t slot_base, float sm_scale, void* out,
                                                 int64_t out_stride, void* stream) {
  if (rows < 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 || tokens_per_req <= 0 ||
      slot_base < 0 || slot_base + tokens_per_req > slot_stride)
    return set_error(OMNI_ERR_INVALID, "bad predictor attention shape");
  if (rows % tokens_per_req != 0) return set_error(OMNI_ERR_INVALID, "rows must be whole requests");
  if (head_dim != 64 && head_dim != 128) return set_error(OMNI_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (slot_base + tokens_per_req > 32) return set_error(OMNI_ERR_UNSUPPORTED, "at most 32 cache slots");
  const int G = num_q_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4) return set_error(OMNI_ERR_UNSUPPORTED, "1, 2 or 4 query heads per KV head");
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
    return set_error(OMNI_ERR_UNSUPPORTED, "misaligned caches");
  if (rows == 0) return OMNI_OK;
  dim3 g((unsigned)((rows * num_kv_heads + 3) / 4)), b(128);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto Q = static_cast<const uint16_t*>(q);
  auto K = static_cast<const uint16_t*>(k_cache);
  auto V = static_cast<const uint16_t*>(v_cache);
  auto O = static_cast<uint16_t*>(out);
#define OMNI_PA(EE, GG)                                                                                        \
  return check_launch(launch(predictor_attention_kernel<EE, GG>, g, b, 0, st, Q, q_stride, K, V, (int)rows,     \
                             num_q_heads, num_kv_heads, tokens_per_req, slot_stride, slot_base, sm_scale, O,    \
                             out_stride))
  if (head_dim == 64) {
    if (G == 1) OMNI_PA(2, 1);
    if (G == 2) OMNI_PA(2, 2);
    OMNI_PA(2, 4);
  }
  if (G == 1) OMNI_PA(4, 1);
  if (G == 2) OMNI_PA(4, 2);
  OMNI_PA(4, 4);
#undef OMNI_PA
}

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory: a host process that owns and
// budgets every byte of device memory (a serving runtime with its own pool),
// or a thread on the real-time audio path that must not call cudaMalloc,
// whose implicit device-wide synchronisation would stall the streams of the
// other live speakers.  For them, this variant takes its scratch (the
// per-chunk partial outputs, their log-sum-exps and the per-row merge
// counters) from a fixed array compiled into the library instead of a
// caller-provided workspace.
//
// Limits and sharing:
//   - the array holds kNoAllocScratchBytes (8 MiB); a call whose scratch need
//     (omni_paged_attention_workspace_bytes(rows, num_kv_heads, work_capacity))
//     exceeds it is rejected with OMNI_ERR_CAPACITY before any launch;
//   - every GPU that loads the library keeps its own copy of the array until
//     the process exits;
//   - all calls on a device share the array, so calls whose kernels overlap on
//     the GPU (different streams without ordering) race on it; serialise them;
//   - the scratch layout is omni_paged_attention_workspace_bytes's: a per-row
//     counter region that the current kernels neither read nor write, then the
//     log-sum-exps and partial outputs, which every call rewrites before it
//     reads them, so nothing needs clearing between calls.
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current and caches it; make that
// first call before any stream capture on the device.
// ---------------------------------------------------------------------------
namespace omni {
namespace {
constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) unsigned char g_noalloc_attn_scratch[kNoAllocScratchBytes];
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};
}  // namespace
}  // namespace omni

extern "C" OMNI_API int omni_paged_decode_attention_noalloc(
    const void* q, int64_t q_stride, const void* k_cache, const void* v_cache, const int32_t* page_indptr,
    const int32_t* page_indices, const int64_t* seq_lens, const int32_t* work_indptr, int64_t rows,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t page_size, int32_t pages_per_chunk,
    int64_t work_capacity, float sm_scale, void* out, int64_t out_stride, int32_t grid_ctas, void* stream) {
  if (rows < 0 || num_kv_heads <= 0 || work_capacity < 0) return set_error(OMNI_ERR_INVALID, "bad attention shape");
  const int64_t need = omni_paged_attention_workspace_bytes(rows, num_kv_heads, work_capacity);
  if (need < 0) return set_error(OMNI_ERR_INVALID, "attention scratch size out of range");
  if (need > (int64_t)kNoAllocScratchBytes)
    return set_error(OMNI_ERR_CAPACITY,
                     "scratch need exceeds the 8 MiB built-in array of the allocation-free attention entry point");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_launch(e);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return set_error(OMNI_ERR_UNSUPPORTED, "device ordinal out of range");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_attn_scratch);
      if (e != cudaSuccess || p == nullptr) {
        set_error(OMNI_ERR_CUDA, "cudaGetSymbolAddress of the built-in attention scratch failed");
        return OMNI_ERR_CUDA;
      }
      g_noalloc_ptr[dev] = p;
    }
    scratch = g_noalloc_ptr[dev];
  }
  return omni_paged_decode_attention(q, q_stride, k_cache, v_cache, page_indptr, page_indices, seq_lens, work_indptr,
                                     rows, num_q_heads, num_kv_heads, head_dim, page_size, pages_per_chunk,
                                     work_capacity, sm_scale, out, out_stride, scratch, need, grid_ctas, stream);
}

