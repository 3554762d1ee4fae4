// MoE block of the talker decode step (a9): block-FP8 routed experts.
//
// The reference's sparse MoE block (Qwen3OmniMoeTalkerSparseMoeBlock.forward,
// talker.py:325-351; Qwen3OmniMoeThinkerTextSparseMoeBlock, thinker_model.py:
// 405-470) runs: router gate -> TopK(renormalize) -> FusedMoE over FP8 e4m3
// experts with per-128x128 weight block scales and per-token 128-group
// activation scales (quantization.py:124-167) -> sum, plus a shared expert
// gated by sigmoid(shared_expert_gate(x)).  Here the step is:
//
//   rmsnorm_quant   x = RMSNorm(h) in bf16, and its e4m3 codes + group scales
//   router GEMM     (gemm.cu, OMNI_EPI_ROUTER) logits, top-k ids, weights
//   align_gather    expert-sorted order of the (token, k) pairs (stable by
//                   token), the work list of row chunks, and the e4m3 rows
//                   gathered into that order
//   grouped GEMMs   persistent tcgen05 kind::f8f6f4 kernels over the work
//                   list: gate/up (two accumulators, SwiGLU, e4m3 re-quant of
//                   the activation) and down (bf16 rows per pair), over
//                   work items of <= 32 rows of one expert
//   combine         h += bf16(bf16(sum_k w_k y_k) + bf16(shared * sigmoid(g)))
//                   and the residual stream's per-128-feature sums of squares
//
// Block scales are applied per K-block of 128: each K-block's four MMAs
// (K = 32 e4m3 each) accumulate into a fresh TMEM slot; the epilogue warps
// read the slot and fold it into register accumulators with the product of
// the weight block scale and the per-row activation scale.  A ring of TMEM
// slots lets the MMAs of the next K-blocks run while a slot is drained.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_util.h"
#include "common.cuh"

namespace omni {
namespace {
OMNI_DEFINE_STATUS(moe)

constexpr int kBlk = 128;       // quantisation group = K-block = feature tile
constexpr int kChunk = 32;      // activation rows per work item (MMA N <= 32)
constexpr int kMaxKBlocks = 8;  // K <= 1024 for the gate/up GEMM
constexpr int kGroupedThreads = 320;
constexpr int kMaxStagesG = 8;
constexpr int kMaxExperts = 256;
constexpr int kMaxTokens = 4096;

// Two fp32 values to two e4m3 codes (round to nearest even, saturating to
// +-448): lo in the low byte.
OMNI_DEVINL uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f8f6f4 (e4m3 inputs, fp32 accumulate).
OMNI_DEVINL void tc_mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
// Bounded mbarrier wait that also gives up as soon as another role of the CTA
// has raised the abort flag.
OMNI_DEVINL bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && *abort_flag) return false;
  }
  return false;
}

// kind::f8f6f4 instruction descriptor: A = B = e4m3 (format 0), D = f32, K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// x = bf16(h * rstd * gain) with rstd from the residual stream's per-128-feature
// sums of squares (RMSNorm of the post-attention layernorm, thinker_model.py
// decoder layer), and the per-row 128-group e4m3 quantisation of x
// (per_token_group_quant_fp8: amax = max(max|x|, 1e-10), scale = amax / 448,
// q = e4m3(x / scale)).  One CTA of 128 threads per row, 8 features a thread.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) rmsnorm_quant_kernel(const uint16_t* __restrict__ h, int64_t h_stride,
                                                            const float* __restrict__ ss, int ss_parts,
                                                            int64_t ss_stride, const uint16_t* __restrict__ gain,
                                                            float eps, int hidden, uint16_t* __restrict__ x,
                                                            int64_t x_stride, uint8_t* __restrict__ xq,
                                                            float* __restrict__ xs) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  float ssum = 0.0f;
  for (int q = 0; q < ss_parts; ++q) ssum += ss[q * ss_stride + row];
  const float rstd = rsqrtf(ssum / (float)hidden + eps);
  const int groups = hidden / kBlk;
  for (int c0 = threadIdx.x * 8; c0 < hidden; c0 += 128 * 8) {
    const uint4 hv = *reinterpret_cast<const uint4*>(h + row * h_stride + c0);
    const uint4 gv = *reinterpret_cast<const uint4*>(gain + c0);
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t xw[4];
    float v[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float a = bf_lo(hw[q]) * rstd * bf_lo(gw[q]);
      const float b = bf_hi(hw[q]) * rstd * bf_hi(gw[q]);
      xw[q] = pack_bf2(a, b);
      v[2 * q] = bf_lo(xw[q]);
      v[2 * q + 1] = bf_hi(xw[q]);
    }
    *reinterpret_cast<uint4*>(x + row * x_stride + c0) = make_uint4(xw[0], xw[1], xw[2], xw[3]);
    // the 16 threads of a 128-group are 16 consecutive lanes
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
    const float sc = __fdiv_rn(fmaxf(amax, 1e-10f), 448.0f);
    uint32_t qw[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint32_t lo = e4m3x2(__fdiv_rn(v[4 * q], sc), __fdiv_rn(v[4 * q + 1], sc));
      const uint32_t hi = e4m3x2(__fdiv_rn(v[4 * q + 2], sc), __fdiv_rn(v[4 * q + 3], sc));
      qw[q] = lo | (hi << 16);
    }
    *reinterpret_cast<uint2*>(xq + (int64_t)row * hidden + c0) = make_uint2(qw[0], qw[1]);
    if ((threadIdx.x & 15) == 0) xs[(int64_t)row * groups + c0 / kBlk] = sc;
  }
}

// ---------------------------------------------------------------------------
// Expert-sorted order of the (token, k) pairs, stable by token (the order of a
// stable counting sort by expert id, as moe_align_block_size's sorted ids):
// pair (t, k) with expert e lands in row off[e] + #{t' < t choosing e}.  Every
// CTA rebuilds the expert membership bitmaps from topk_ids in shared memory
// (tokens x experts bits) and gathers the e4m3 rows and scales of its own
// tokens into their rows; CTA 0 also writes the expert offsets and the work
// list of row chunks (expert, first row, rows <= 32).  An expert id of -1 marks a
// (token, k) entry with no local expert (expert-parallel receive buffers): it is
// skipped and its slot_of entry is -1.
// ---------------------------------------------------------------------------
struct AlignParams {
  const int32_t* topk_ids;
  int64_t ids_stride;  // int32 elements between rows of topk_ids
  int tokens, top_k, experts;
  const uint8_t* xq;
  int64_t xq_stride;   // bytes between e4m3 rows
  const float* xs;
  int64_t xs_stride;   // floats between scale rows
  int hidden, groups;
  uint8_t* pq;
  float* ps;
  int32_t* slot_of;
  int32_t* expert_off;
  int4* chunks;
  int32_t* n_chunks;
  int chunk_cap;
};

__global__ void __launch_bounds__(1024) moe_align_gather_kernel(const __grid_constant__ AlignParams p) {
  extern __shared__ uint32_t mask[];  // [experts][W]
  __shared__ int cnt[kMaxExperts], off[kMaxExperts + 1], coff[kMaxExperts + 1];
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = (p.tokens + 31) / 32;
  for (int i = tid; i < p.experts * W; i += blockDim.x) mask[i] = 0u;
  __syncthreads();
  for (int i = tid; i < p.tokens * p.top_k; i += blockDim.x) {
    const int t = i / p.top_k;
    const int e = p.topk_ids[t * p.ids_stride + i % p.top_k];
    if (e == -1) continue;
    if (e < 0 || e >= p.experts) {
      report_status(kDevBadIndex);
      continue;
    }
    atomicOr(&mask[e * W + (t >> 5)], 1u << (t & 31));
  }
  __syncthreads();
  for (int e = tid; e < p.experts; e += blockDim.x) {
    int c = 0;
    for (int w = 0; w < W; ++w) c += __popc(mask[e * W + w]);
    cnt[e] = c;
  }
  __syncthreads();
  if (warp == 0) {
    // lane l scans experts [l * per, (l + 1) * per)
    const int per = (p.experts + 31) / 32;
    int rows = 0, chs = 0;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < p.experts) {
        rows += cnt[e];
        chs += (cnt[e] + kChunk - 1) / kChunk;
      }
    }
    int ir = rows, ic = chs;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xFFFFFFFFu, ir, o), b = __shfl_up_sync(0xFFFFFFFFu, ic, o);
      if (lane >= o) {
        ir += a;
        ic += b;
      }
    }
    int r = ir - rows, c = ic - chs;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < p.experts) {
        off[e] = r;
        coff[e] = c;
        r += cnt[e];
        c += (cnt[e] + kChunk - 1) / kChunk;
      }
    }
    if (lane == 31) {
      off[p.experts] = r;
      coff[p.experts] = c;
    }
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = tid; e <= p.experts; e += blockDim.x) p.expert_off[e] = off[e];
    const bool fits = coff[p.experts] <= p.chunk_cap;
    if (tid == 0) {
      *p.n_chunks = fits ? coff[p.experts] : 0;
      if (!fits) report_status(kDevBadIndex);
    }
    if (fits)
      for (int e = tid; e < p.experts; e += blockDim.x)
        for (int c = 0; c * kChunk < cnt[e]; ++c)
          p.chunks[coff[e] + c] = make_int4(e, off[e] + c * kChunk, min(kChunk, cnt[e] - c * kChunk), 0);
  }
  // gather: one warp per token of this CTA
  const int per_cta = (p.tokens + gridDim.x - 1) / gridDim.x;
  const int t_end = min(p.tokens, (int)(blockIdx.x + 1) * per_cta);
  for (int t = blockIdx.x * per_cta + warp; t < t_end; t += blockDim.x / 32) {
    for (int kk = 0; kk < p.top_k; ++kk) {
      const int e = p.topk_ids[t * p.ids_stride + kk];
      if (e < 0 || e >= p.experts) {
        if (lane == 0) p.slot_of[t * p.top_k + kk] = -1;
        continue;
      }
      // rank of t among the tokens choosing e: whole mask words below t's word
      // (lane-strided, summed across the warp) plus the lower bits of its word
      int part = 0;
      for (int w = lane; w < (t >> 5); w += 32) part += __popc(mask[e * W + w]);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xFFFFFFFFu, part, o);
      const int slot = off[e] + __popc(mask[e * W + (t >> 5)] & ((1u << (t & 31)) - 1u)) + part;
      if (lane == 0) p.slot_of[t * p.top_k + kk] = slot;
      const uint4* src = reinterpret_cast<const uint4*>(p.xq + (int64_t)t * p.xq_stride);
      uint4* dst = reinterpret_cast<uint4*>(p.pq + (int64_t)slot * p.hidden);
      for (int v = lane; v < p.hidden / 16; v += 32) dst[v] = src[v];
      for (int g = lane; g < p.groups; g += 32) p.ps[(int64_t)slot * p.groups + g] = p.xs[(int64_t)t * p.xs_stride + g];
    }
  }
}

// ---------------------------------------------------------------------------
// Grouped block-FP8 GEMM over the work list (persistent, one CTA per SM).
//
//   mode 0 (gate/up):  W = w13 [E][2I][K] (gate rows, then up rows); work item =
//     (chunk, tile t < I/128): gate rows 128t.., up rows I + 128t..; output
//     act = bf16(silu(bf16(g)) * bf16(u)) re-quantised per 128-group (the tile)
//     into out_q [rows][I] e4m3 and out_s [rows][I/128].
//   mode 1 (down):     W = w2 [E][N][K]; work item = (chunk, tile < N/128);
//     output y [rows][N] bf16.
//
// Roles (320 threads): warp 0 lane 0 = TMA producer, warp 1 lane 0 = MMA
// issuer, warps 2-5 and 6-9 = two epilogue groups (TMEM lane quarter = warp %
// 4) taking the CTA's work items alternately, so that one group's closing
// epilogue (SwiGLU, re-quantisation, stores) overlaps the other group's
// accumulation of the next item.  Only the chunk's row columns are read.
// ---------------------------------------------------------------------------
struct GroupedParams {
  int mode;
  int kblocks;      // K / 128
  int tiles;        // feature tiles per expert
  int w_rows;       // rows of one expert's weight matrix
  int half;         // mode 0: I (first up row)
  int stages;
  int slots;        // TMEM ring slots
  int slot_cols;    // columns per slot (mode 0: 128 = gate 64 + up 64; mode 1: 64)
  int tmem_cols;
  const float* w_scale;  // [E][w_rows / 128][kblocks]
  const float* a_scale;  // [rows_cap][kblocks]
  const int4* chunks;
  const int32_t* n_chunks;
  uint8_t* out_q;
  float* out_s;
  int out_cols;          // mode 0: I
  uint16_t* y;
  int64_t y_stride;
};

template <int MODE>
__global__ void __launch_bounds__(kGroupedThreads, 1)
    moe_grouped_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ GroupedParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr uint32_t kWTile = kBlk * kBlk;                   // 16 KB of e4m3
  constexpr uint32_t kWBytes = MODE == 0 ? 2 * kWTile : kWTile;
  constexpr uint32_t kABytes = kChunk * kBlk;                // 8 KB
  constexpr uint32_t kStageBytes = kWBytes + kABytes;
  const int ST = p.stages;
  const int NS = p.slots;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* stage_base = smem;
  // per epilogue group: act [64][128] bf16 (mode 0) and the chunk's activation scales [kb][64]
  uint16_t* act_all = reinterpret_cast<uint16_t*>(smem + ST * kStageBytes);
  float* sa_all = reinterpret_cast<float*>(smem + ST * kStageBytes + 2 * kChunk * kBlk * 2);
  // barriers: smem stages full/empty; TMEM slots full (one set per epilogue group, so
  // that each group waits on every phase of its own barriers) and empty; per group
  // "scales ready", "activation staged" and "item done" (128 arrivals each)
  uint64_t* full = reinterpret_cast<uint64_t*>(sa_all + 2 * kMaxKBlocks * kChunk);
  uint64_t* empty = full + kMaxStagesG;
  uint64_t* tfull = empty + kMaxStagesG;  // [2][8]
  uint64_t* tempty = tfull + 16;          // [8]
  uint64_t* gbar = tempty + 8;            // [2][3]: sa ready, act staged, item done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbar + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tfull[8 + s], 1);
      mbar_init(&tempty[s], 4);  // one arrive per warp of the consuming group
    }
    for (int b = 0; b < 6; ++b) mbar_init(&gbar[b], 128);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_a);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch();
  const int n_items = *p.n_chunks * p.tiles;
  const int KB = p.kblocks;
  const int wtile_rows = p.w_rows / kBlk;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int w = blockIdx.x; w < n_items && !*abort_flag; w += gridDim.x) {
        const int4 c = p.chunks[w / p.tiles];
        const int tile = w % p.tiles;
        const int wrow = c.x * p.w_rows + tile * kBlk;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % ST;
          if (it >= ST && !mbar_wait_or_abort(&empty[s], ((it / ST) - 1) & 1, abort_flag)) {
            report_status(kDevTimeoutMma);
            *abort_flag = 1;
            break;
          }
          uint8_t* st = stage_base + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_2d(st, &tmap_w, &full[s], kb * kBlk, wrow);
          if (MODE == 0) tma_load_2d(st + kWTile, &tmap_w, &full[s], kb * kBlk, wrow + p.half);
          tma_load_2d(st + kWBytes, &tmap_a, &full[s], kb * kBlk, c.y);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, bt = 0, li = 0;
      for (int w = blockIdx.x; w < n_items && !*abort_flag; w += gridDim.x, ++li) {
        const int4 c = p.chunks[w / p.tiles];
        const int N = (c.z + 15) & ~15;
        const uint32_t idesc = idesc_e4m3_f32(kBlk, N);
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++it, ++bt) {
          const int s = it % ST, ts = bt % NS;
          if (!mbar_wait_or_abort(&full[s], (it / ST) & 1, abort_flag) ||
              (bt >= NS && !mbar_wait_or_abort(&tempty[ts], ((bt / NS) - 1) & 1, abort_flag))) {
            report_status(kDevTimeoutTma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = stage_base + s * kStageBytes;
          const uint64_t bd = smem_desc_sw128(st + kWBytes);
          const uint32_t d0 = tmem + (uint32_t)(ts * p.slot_cols);
          const uint64_t ag = smem_desc_sw128(st);
#pragma unroll
          for (int kk = 0; kk < kBlk / 32; ++kk) tc_mma_f8(d0, ag + 2 * kk, bd + 2 * kk, idesc, kk > 0 ? 1u : 0u);
          if (MODE == 0) {
            const uint64_t au = smem_desc_sw128(st + kWTile);
#pragma unroll
            for (int kk = 0; kk < kBlk / 32; ++kk)
              tc_mma_f8(d0 + kChunk, au + 2 * kk, bd + 2 * kk, idesc, kk > 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          tc_commit(&tfull[(li & 1) * 8 + ts]);
        }
        if (!ok) break;
      }
    }
  } else {
    // epilogue group gi takes the CTA's items gi, gi + 2, ...; TMEM lane quarter q =
    // warp % 4, feature f = 32 q + lane of the tile
    const int gi = (warp - 2) >> 2;
    const int q = warp & 3;
    const int f = q * 32 + lane;
    const int et = ((warp - 2) & 3) * 32 + lane;  // 0..127 within the group
    uint16_t* act = act_all + gi * kChunk * kBlk;
    float* sa = sa_all + gi * kMaxKBlocks * kChunk;
    uint64_t* g_sa = &gbar[3 * gi];
    uint64_t* g_act = &gbar[3 * gi + 1];
    uint64_t* g_done = &gbar[3 * gi + 2];
    uint64_t* my_tfull = &tfull[8 * gi];
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    // bounded group-wide wait; on timeout every later wait of this thread is skipped
    auto gwait = [&](uint64_t* bar, uint32_t parity) -> bool {
      if (*abort_flag) return false;
      if (mbar_wait_or_abort(bar, parity, abort_flag)) return true;
      report_status(kDevTimeoutFlag);
      *abort_flag = 1;
      return false;
    };
    // completed phases of this group's TMEM-full barriers, one bit per slot: the slot
    // of a block depends on the CTA-wide block index, so a group's uses of a slot are
    // counted here rather than derived from its own item count
    uint32_t tphase = 0;
    for (int li = gi; blockIdx.x + li * gridDim.x < n_items; li += 2) {
      const int w = blockIdx.x + li * gridDim.x;
      const int k = li >> 1;  // this group's item count so far
      // the group's previous item has finished reading sa and act
      if (k > 0 && !gwait(g_done, (k - 1) & 1)) break;
      const int4 c = p.chunks[w / p.tiles];
      const int tile = w % p.tiles;
      const int e = c.x, r0 = c.y, nr = c.z;
      const int N = (nr + 15) & ~15;
      // per-row activation scales of the chunk, [kb][row]
      for (int i = et; i < KB * kChunk; i += 128) {
        const int kb = i / kChunk, jr = i % kChunk;
        sa[kb * kChunk + jr] = jr < nr ? p.a_scale[(int64_t)(r0 + jr) * KB + kb] : 0.0f;
      }
      const float* swg = p.w_scale + ((int64_t)e * wtile_rows + tile) * KB;
      const float* swu = p.w_scale + ((int64_t)e * wtile_rows + p.half / kBlk + tile) * KB;
      mbar_arrive(g_sa);
      if (!gwait(g_sa, k & 1)) break;
      float accg[kChunk], accu[MODE == 0 ? kChunk : 1];
#pragma unroll
      for (int jj = 0; jj < kChunk; ++jj) accg[jj] = 0.0f;
#pragma unroll
      for (int jj = 0; jj < (MODE == 0 ? kChunk : 1); ++jj) accu[jj] = 0.0f;
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb) {
        const int bt = li * KB + kb, ts = bt % NS;
        const float wg = swg[kb], wu = MODE == 0 ? swu[kb] : 0.0f;
        // the group's blocks in slot ts complete my_tfull[ts] once each, in order: the
        // MMA refills a slot only after its previous block has been drained
        if (!gwait(&my_tfull[ts], (tphase >> ts) & 1u)) {
          ok = false;
          break;
        }
        tphase ^= 1u << ts;
        tc_fence_after();
        const uint32_t base = tmem + lane_off + (uint32_t)(ts * p.slot_cols);
        uint32_t r[32];
#pragma unroll
        for (int h = 0; h < kChunk / 32; ++h) {
          if (32 * h < N) {
            tmem_ld_32x32b_x32(base + (uint32_t)(32 * h), r);
            tc_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              accg[32 * h + jj] = __fmaf_rn(__uint_as_float(r[jj]), wg * sa[kb * kChunk + 32 * h + jj],
                                            accg[32 * h + jj]);
          }
        }
        if (MODE == 0) {
#pragma unroll
          for (int h = 0; h < kChunk / 32; ++h) {
            if (32 * h < N) {
              tmem_ld_32x32b_x32(base + (uint32_t)(kChunk + 32 * h), r);
              tc_wait_ld();
#pragma unroll
              for (int jj = 0; jj < 32; ++jj)
                accu[32 * h + jj] = __fmaf_rn(__uint_as_float(r[jj]), wu * sa[kb * kChunk + 32 * h + jj],
                                              accu[32 * h + jj]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[ts]);
      }
      if (!ok) break;
      if (MODE == 0) {
        // act = bf16(silu(bf16(g)) * bf16(u)), staged [row][feature] for the per-row quantisation
#pragma unroll
        for (int jj = 0; jj < kChunk; ++jj) {
          if (jj < nr) {
            const float g = bf2f(f2bf(accg[jj])), u = bf2f(f2bf(accu[jj]));
            act[jj * kBlk + f] = f2bf(__fdividef(g, 1.0f + __expf(-g)) * u);
          }
        }
        mbar_arrive(g_act);
        if (!gwait(g_act, k & 1)) break;
        // warp et / 32 of the group quantises rows et / 32, + 4, ...: lane l holds features 4l..4l+3
        for (int jr = et >> 5; jr < nr; jr += 4) {
          const uint2 a2 = *reinterpret_cast<const uint2*>(act + jr * kBlk + 4 * lane);
          const float v[4] = {bf_lo(a2.x), bf_hi(a2.x), bf_lo(a2.y), bf_hi(a2.y)};
          float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
          const float sc = __fdiv_rn(fmaxf(amax, 1e-10f), 448.0f);
          const uint32_t lo = e4m3x2(__fdiv_rn(v[0], sc), __fdiv_rn(v[1], sc));
          const uint32_t hi = e4m3x2(__fdiv_rn(v[2], sc), __fdiv_rn(v[3], sc));
          *reinterpret_cast<uint32_t*>(p.out_q + (int64_t)(r0 + jr) * p.out_cols + tile * kBlk + 4 * lane) =
              lo | (hi << 16);
          if (lane == 0) p.out_s[(int64_t)(r0 + jr) * (p.out_cols / kBlk) + tile] = sc;
        }
        mbar_arrive(g_done);  // act and sa are rewritten by this group's next item
      } else {
#pragma unroll
        for (int jj = 0; jj < kChunk; ++jj)
          if (jj < nr) p.y[(int64_t)(r0 + jj) * p.y_stride + tile * kBlk + f] = f2bf(accg[jj]);
        mbar_arrive(g_done);  // sa is rewritten by this group's next item
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
}

// ---------------------------------------------------------------------------
// Combine (the routed sum + gated shared expert + residual add):
//   routed = bf16(sum_k w_k * y[slot(t, k)])            (fp32, k order)
//   g      = bf16(x . w_sg)                              (shared_expert_gate)
//   shared = bf16(s * sigmoid(g))
//   h      = bf16(h + bf16(routed + shared))
// and ss_out[part][t] = sum over the part's 128 features of h^2.
// One CTA of 128 threads per token, 8 features a thread.
// ---------------------------------------------------------------------------
// parts != nullptr: the routed sum arrives as up to top_k bf16 partial rows per token
// (expert-parallel: one per rank that holds some of the token's experts), parts rows
// slot_of[t][k] (or -1), summed in k order; topk_w is unused.
__global__ void __launch_bounds__(128) moe_combine_kernel(
    const uint16_t* __restrict__ y, int64_t y_stride, const int32_t* __restrict__ slot_of,
    const float* __restrict__ topk_w, int top_k, const uint16_t* __restrict__ x, int64_t x_stride,
    const uint16_t* __restrict__ w_sg, const uint16_t* __restrict__ shared, int64_t sh_stride,
    uint16_t* __restrict__ h, int64_t h_stride, float* __restrict__ ss_out, int64_t ss_stride, int hidden,
    int parts_mode) {
  __shared__ float red[4];
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // shared-expert gate: per-thread products in feature order, warp butterfly, warps in order
  float dot = 0.0f;
  for (int c0 = threadIdx.x * 8; c0 < hidden; c0 += 1024) {
    const uint4 xv = *reinterpret_cast<const uint4*>(x + t * x_stride + c0);
    const uint4 wv = *reinterpret_cast<const uint4*>(w_sg + c0);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      dot = __fmaf_rn(bf_lo(xw[q]), bf_lo(ww[q]), dot);
      dot = __fmaf_rn(bf_hi(xw[q]), bf_hi(ww[q]), dot);
    }
  }
  dot = warp_sum_xor(dot);
  if (lane == 0) red[warp] = dot;
  __syncthreads();
  const float g = bf2f(f2bf(((red[0] + red[1]) + red[2]) + red[3]));
  const float gate = 1.0f / (1.0f + expf(-g));
  int slot[8];
  float wk[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    slot[k] = k < top_k ? slot_of[t * top_k + k] : -1;
    wk[k] = (k < top_k && !parts_mode) ? topk_w[t * top_k + k] : 1.0f;
  }
  for (int c0 = threadIdx.x * 8; c0 < hidden; c0 += 1024) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < top_k && slot[k] >= 0) {
        const uint4 yv = *reinterpret_cast<const uint4*>(y + (int64_t)slot[k] * y_stride + c0);
        const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] = __fmaf_rn(wk[k], bf_lo(yw[q]), acc[2 * q]);
          acc[2 * q + 1] = __fmaf_rn(wk[k], bf_hi(yw[q]), acc[2 * q + 1]);
        }
      }
    }
    const uint4 sv = *reinterpret_cast<const uint4*>(shared + t * sh_stride + c0);
    const uint4 hv = *reinterpret_cast<const uint4*>(h + t * h_stride + c0);
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w}, hw[4] = {hv.x, hv.y, hv.z, hv.w};
    uint32_t ow[4];
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float o2[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float routed = bf2f(f2bf(acc[2 * q + u]));
        const float sh = bf2f(f2bf((u ? bf_hi(sw[q]) : bf_lo(sw[q])) * gate));
        const float moe = bf2f(f2bf(routed + sh));
        o2[u] = bf2f(f2bf((u ? bf_hi(hw[q]) : bf_lo(hw[q])) + moe));
        ss = __fmaf_rn(o2[u], o2[u], ss);
      }
      ow[q] = pack_bf2(o2[0], o2[1]);
    }
    *reinterpret_cast<uint4*>(h + t * h_stride + c0) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
    if (ss_out && (lane & 15) == 0) ss_out[(int64_t)(c0 / kBlk) * ss_stride + t] = ss;
  }
}

// ---------------------------------------------------------------------------
// Expert-parallel partial routed sum of one received row: out[r] = bf16(sum over
// its k entries with slot >= 0 of w[r][k] * y[slot]) in k order (fp32), zero when
// none.  One CTA of 128 threads per row, 8 features a thread.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) moe_partial_sum_kernel(const uint16_t* __restrict__ y, int64_t y_stride,
                                                              const int32_t* __restrict__ slot_of,
                                                              const float* __restrict__ w, int64_t w_stride,
                                                              int top_k, int hidden, uint16_t* __restrict__ out,
                                                              int64_t out_stride) {
  griddep_wait();
  griddep_launch();
  const int r = blockIdx.x;
  int slot[8];
  float wk[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    slot[k] = k < top_k ? slot_of[(int64_t)r * top_k + k] : -1;
    wk[k] = k < top_k ? w[(int64_t)r * w_stride + k] : 0.0f;
  }
  for (int c0 = threadIdx.x * 8; c0 < hidden; c0 += 1024) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (slot[k] >= 0) {
        const uint4 yv = *reinterpret_cast<const uint4*>(y + (int64_t)slot[k] * y_stride + c0);
        const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] = __fmaf_rn(wk[k], bf_lo(yw[q]), acc[2 * q]);
          acc[2 * q + 1] = __fmaf_rn(wk[k], bf_hi(yw[q]), acc[2 * q + 1]);
        }
      }
    }
    *reinterpret_cast<uint4*>(out + (int64_t)r * out_stride + c0) =
        make_uint4(pack_bf2(acc[0], acc[1]), pack_bf2(acc[2], acc[3]), pack_bf2(acc[4], acc[5]),
                   pack_bf2(acc[6], acc[7]));
  }
}


// ---------------------------------------------------------------------------
// Expert-parallel dispatch packing.  CTA t < tokens: the token's destination ranks
// (a rank holds experts [d e, (d + 1) e)), its row in each destination's block (the
// count of earlier tokens going there: every CTA re-counts the tokens before it, at
// most a few thousand ids), the packed row (e4m3 codes, group scales, the k ids local
// to that rank or -1, the k weights) and part_index[t][d] = d cap + row or -1.  CTA
// tokens + d: clears the expert ids of block d's unused rows to -1.
// ---------------------------------------------------------------------------
constexpr int kEpMaxWorld = 32;

__global__ void __launch_bounds__(256) moe_ep_pack_kernel(const int32_t* __restrict__ ids, const float* __restrict__ tw,
                                                         int tokens, int top_k, const uint8_t* __restrict__ xq,
                                                         int64_t xq_stride, const float* __restrict__ xs,
                                                         int64_t xs_stride, int hidden, int world, int e_per_rank,
                                                         int cap, uint8_t* __restrict__ send, int64_t row_bytes,
                                                         int32_t* __restrict__ part_index) {
  __shared__ int counts[kEpMaxWorld];
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.x;
  const int groups = hidden / 128;
  const int64_t off_ids = hidden + 4 * groups, off_w = off_ids + 4 * top_k;
  if (threadIdx.x < kEpMaxWorld) counts[threadIdx.x] = 0;
  __syncthreads();
  // destinations of token u as a bit mask (ids outside [0, world e) are dropped)
  auto dests = [&](int u) {
    uint32_t m = 0u;
    for (int k = 0; k < top_k; ++k) {
      const int e = ids[(int64_t)u * top_k + k];
      if (e >= 0 && e < world * e_per_rank) m |= 1u << (e / e_per_rank);
    }
    return m;
  };
  const int upto = b < tokens ? b : tokens;  // tokens counted: those before b (all for a clearing CTA)
  for (int u = threadIdx.x; u < upto; u += blockDim.x) {
    uint32_t m = dests(u);
    while (m) {
      const int d = __ffs(m) - 1;
      m &= m - 1u;
      atomicAdd(&counts[d], 1);
    }
  }
  __syncthreads();
  if (b >= tokens) {
    // clear block d's rows past its count
    const int d = b - tokens;
    for (int r = counts[d] + threadIdx.x; r < cap; r += blockDim.x) {
      int32_t* rid = reinterpret_cast<int32_t*>(send + ((int64_t)d * cap + r) * row_bytes + off_ids);
      for (int k = 0; k < top_k; ++k) rid[k] = -1;
    }
    return;
  }
  const uint32_t mine = dests(b);
  for (int d = 0; d < world; ++d) {
    const bool go = (mine >> d) & 1u;
    if (threadIdx.x == 0) part_index[(int64_t)b * world + d] = go ? d * cap + counts[d] : -1;
    if (!go || counts[d] >= cap) continue;
    uint8_t* row = send + ((int64_t)d * cap + counts[d]) * row_bytes;
    const uint4* src = reinterpret_cast<const uint4*>(xq + (int64_t)b * xq_stride);
    for (int v = threadIdx.x; v < hidden / 16; v += blockDim.x) reinterpret_cast<uint4*>(row)[v] = src[v];
    float* rs = reinterpret_cast<float*>(row + hidden);
    for (int gq = threadIdx.x; gq < groups; gq += blockDim.x) rs[gq] = xs[(int64_t)b * xs_stride + gq];
    if (threadIdx.x < top_k) {
      const int k = threadIdx.x;
      const int e = ids[(int64_t)b * top_k + k];
      const bool local = e >= d * e_per_rank && e < (d + 1) * e_per_rank;
      reinterpret_cast<int32_t*>(row + off_ids)[k] = local ? e - d * e_per_rank : -1;
      reinterpret_cast<float*>(row + off_w)[k] = tw[(int64_t)b * top_k + k];
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn_moe() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(q);
  });
  return fn;
}

// 2D uint8 [rows, cols] row-major, box {128, box_rows}, 128-byte swizzle.
bool make_tmap_u8(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  auto fn = encode_fn_moe();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)kBlk, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms_moe() { return device_sm_count(); }

template <int MODE>
int launch_grouped(const void* a_q, int64_t rows_cap, int64_t k, const void* w, int64_t experts, int64_t w_rows,
                   GroupedParams gp, void* stream) {
  CUtensorMap tw, ta;
  if (!make_tmap_u8(&tw, w, experts * w_rows, k, kBlk) || !make_tmap_u8(&ta, a_q, rows_cap, k, kChunk))
    return set_error(OMNI_ERR_UNSUPPORTED, "tensor map encoding failed");
  const size_t stage_bytes = (MODE == 0 ? 2 : 1) * kBlk * kBlk + kChunk * kBlk;
  const size_t fixed =
      1024 + 2 * ((size_t)kChunk * kBlk * 2 + kMaxKBlocks * kChunk * 4) + (2 * kMaxStagesG + 16 + 8 + 6) * 8 + 16;
  int st = kMaxStagesG;
  while (st > 2 && fixed + st * stage_bytes > 227 * 1024) --st;
  gp.stages = st;
  gp.slot_cols = MODE == 0 ? 2 * kChunk : kChunk;
  gp.tmem_cols = MODE == 0 ? 512 : 256;
  gp.slots = gp.tmem_cols / gp.slot_cols;
  if (gp.slots > 8) gp.slots = 8;
  const size_t smem = fixed + st * stage_bytes;
  const cudaError_t ae = once_per_device(reinterpret_cast<const void*>(moe_grouped_kernel<MODE>), kAttrSmem, [] {
    return cudaFuncSetAttribute(moe_grouped_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (ae != cudaSuccess) return check_launch(ae);
  return check_launch(launch(moe_grouped_kernel<MODE>, dim3((unsigned)num_sms_moe()), dim3(kGroupedThreads), smem,
                             static_cast<cudaStream_t>(stream), tw, ta, gp));
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int omni_moe_rmsnorm_quant(const void* h, int64_t h_stride, const float* ss, int32_t ss_parts,
                                               int64_t ss_stride, const void* gain, float eps, int64_t rows,
                                               int32_t hidden, void* x, int64_t x_stride, void* xq, float* xs,
                                               void* stream) {
  if (rows < 0 || hidden <= 0 || hidden % 1024 != 0 || ss_parts <= 0 || ss == nullptr)
    return set_error(OMNI_ERR_UNSUPPORTED, "rmsnorm_quant: hidden a multiple of 1024 and ss partials required");
  if (!al16(h) || !al16(x) || !al16(gain) || !al16(xq) || h_stride % 8 || x_stride % 8)
    return set_error(OMNI_ERR_UNSUPPORTED, "rmsnorm_quant: 16-byte aligned rows required");
  if (rows == 0) return OMNI_OK;
  return check_launch(launch(rmsnorm_quant_kernel, dim3((unsigned)rows), dim3(128), 0,
                             static_cast<cudaStream_t>(stream), static_cast<const uint16_t*>(h), h_stride, ss,
                             (int)ss_parts, ss_stride, static_cast<const uint16_t*>(gain), eps, (int)hidden,
                             static_cast<uint16_t*>(x), x_stride, static_cast<uint8_t*>(xq), xs));
}

extern "C" OMNI_API int64_t omni_moe_chunk_capacity(int64_t tokens, int32_t top_k, int32_t experts) {
  return experts + (tokens * top_k + kChunk - 1) / kChunk;
}

extern "C" OMNI_API int omni_moe_align_gather_strided(
    const int32_t* topk_ids, int64_t ids_stride, int64_t tokens, int32_t top_k, int32_t experts, const void* xq,
    int64_t xq_stride, const float* xs, int64_t xs_stride, int32_t hidden, void* permuted_q, float* permuted_s,
    int32_t* slot_of, int32_t* expert_offsets, void* chunks, int64_t chunk_capacity, int32_t* n_chunks,
    void* stream) {
  if (tokens < 0 || tokens > kMaxTokens || top_k < 1 || top_k > 8 || experts < 1 || experts > kMaxExperts ||
      top_k > experts || ids_stride < top_k)
    return set_error(OMNI_ERR_UNSUPPORTED, "align: tokens <= 4096, 1 <= top_k <= 8, experts <= 256");
  if (hidden % kBlk != 0 || !al16(xq) || xq_stride % 16 || xq_stride < hidden || xs_stride < hidden / kBlk ||
      !al16(permuted_q) || !al16(chunks))
    return set_error(OMNI_ERR_UNSUPPORTED, "align: hidden a multiple of 128, 16-byte aligned rows");
  if (chunk_capacity < omni_moe_chunk_capacity(tokens, top_k, experts))
    return set_error(OMNI_ERR_CAPACITY, "align: chunk capacity too small");
  AlignParams p{};
  p.topk_ids = topk_ids;
  p.ids_stride = ids_stride;
  p.tokens = (int)tokens;
  p.top_k = top_k;
  p.experts = experts;
  p.xq = static_cast<const uint8_t*>(xq);
  p.xq_stride = xq_stride;
  p.xs = xs;
  p.xs_stride = xs_stride;
  p.hidden = hidden;
  p.groups = hidden / kBlk;
  p.pq = static_cast<uint8_t*>(permuted_q);
  p.ps = permuted_s;
  p.slot_of = slot_of;
  p.expert_off = expert_offsets;
  p.chunks = static_cast<int4*>(chunks);
  p.n_chunks = n_chunks;
  p.chunk_cap = (int)chunk_capacity;
  const int W = (int)((tokens + 31) / 32);
  const size_t smem = (size_t)experts * (W > 0 ? W : 1) * 4;
  if (smem > 48 * 1024) {
    const cudaError_t ae = once_per_device(reinterpret_cast<const void*>(moe_align_gather_kernel), kAttrSmem, [] {
      return cudaFuncSetAttribute(moe_align_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    });
    if (ae != cudaSuccess) return check_launch(ae);
  }
  const int grid = tokens > 0 ? (int)((tokens + 31) / 32) : 1;
  return check_launch(launch(moe_align_gather_kernel, dim3((unsigned)grid), dim3(1024), smem,
                             static_cast<cudaStream_t>(stream), p));
}

extern "C" OMNI_API int omni_moe_align_gather(const int32_t* topk_ids, int64_t tokens, int32_t top_k,
                                              int32_t experts, const void* xq, const float* xs, int32_t hidden,
                                              void* permuted_q, float* permuted_s, int32_t* slot_of,
                                              int32_t* expert_offsets, void* chunks, int64_t chunk_capacity,
                                              int32_t* n_chunks, void* stream) {
  return omni_moe_align_gather_strided(topk_ids, top_k, tokens, top_k, experts, xq, hidden, xs, hidden / kBlk,
                                       hidden, permuted_q, permuted_s, slot_of, expert_offsets, chunks,
                                       chunk_capacity, n_chunks, stream);
}

extern "C" OMNI_API int omni_moe_gate_up_fp8(const void* permuted_q, const float* permuted_s, int64_t rows_cap,
                                             int32_t hidden, const void* w13, const float* w13_scale,
                                             int32_t experts, int32_t inter, const void* chunks,
                                             const int32_t* n_chunks, void* act_q, float* act_s, void* stream) {
  if (hidden % kBlk || hidden / kBlk > kMaxKBlocks || inter % kBlk || experts < 1)
    return set_error(OMNI_ERR_UNSUPPORTED, "gate_up: hidden and inter multiples of 128, hidden <= 1024");
  if (!al16(permuted_q) || !al16(w13) || !al16(act_q))
    return set_error(OMNI_ERR_UNSUPPORTED, "gate_up: 16-byte aligned operands");
  GroupedParams gp{};
  gp.mode = 0;
  gp.kblocks = hidden / kBlk;
  gp.tiles = inter / kBlk;
  gp.w_rows = 2 * inter;
  gp.half = inter;
  gp.w_scale = w13_scale;
  gp.a_scale = permuted_s;
  gp.chunks = static_cast<const int4*>(chunks);
  gp.n_chunks = n_chunks;
  gp.out_q = static_cast<uint8_t*>(act_q);
  gp.out_s = act_s;
  gp.out_cols = inter;
  return launch_grouped<0>(permuted_q, rows_cap, hidden, w13, experts, 2 * inter, gp, stream);
}

extern "C" OMNI_API int omni_moe_down_fp8(const void* act_q, const float* act_s, int64_t rows_cap, int32_t inter,
                                          const void* w2, const float* w2_scale, int32_t experts, int32_t hidden,
                                          const void* chunks, const int32_t* n_chunks, void* y, int64_t y_stride,
                                          void* stream) {
  if (inter % kBlk || inter / kBlk > kMaxKBlocks || hidden % kBlk || experts < 1)
    return set_error(OMNI_ERR_UNSUPPORTED, "down: inter and hidden multiples of 128, inter <= 1024");
  if (!al16(act_q) || !al16(w2)) return set_error(OMNI_ERR_UNSUPPORTED, "down: 16-byte aligned operands");
  GroupedParams gp{};
  gp.mode = 1;
  gp.kblocks = inter / kBlk;
  gp.tiles = hidden / kBlk;
  gp.w_rows = hidden;
  gp.w_scale = w2_scale;
  gp.a_scale = act_s;
  gp.chunks = static_cast<const int4*>(chunks);
  gp.n_chunks = n_chunks;
  gp.y = static_cast<uint16_t*>(y);
  gp.y_stride = y_stride;
  return launch_grouped<1>(act_q, rows_cap, inter, w2, experts, hidden, gp, stream);
}

extern "C" OMNI_API int omni_moe_combine(const void* y, int64_t y_stride, const int32_t* slot_of,
                                         const float* topk_weights, int32_t top_k, const void* x, int64_t x_stride,
                                         const void* shared_gate_weight, const void* shared_out, int64_t shared_stride,
                                         void* h, int64_t h_stride, float* ss_out, int64_t ss_stride, int64_t rows,
                                         int32_t hidden, void* stream) {
  if (top_k < 1 || top_k > 8 || hidden % 1024 != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "combine: 1 <= top_k <= 8, hidden a multiple of 1024");
  if (!al16(y) || !al16(x) || !al16(shared_gate_weight) || !al16(shared_out) || !al16(h) || y_stride % 8 ||
      x_stride % 8 || shared_stride % 8 || h_stride % 8)
    return set_error(OMNI_ERR_UNSUPPORTED, "combine: 16-byte aligned rows required");
  if (rows == 0) return OMNI_OK;
  return check_launch(launch(moe_combine_kernel, dim3((unsigned)rows), dim3(128), 0, static_cast<cudaStream_t>(stream),
                             static_cast<const uint16_t*>(y), y_stride, slot_of, topk_weights, (int)top_k,
                             static_cast<const uint16_t*>(x), x_stride,
                             static_cast<const uint16_t*>(shared_gate_weight),
                             static_cast<const uint16_t*>(shared_out), shared_stride, static_cast<uint16_t*>(h),
                             h_stride, ss_out, ss_stride, (int)hidden, 0));
}

extern "C" OMNI_API int omni_moe_combine_parts(const void* parts, int64_t parts_stride, const int32_t* part_index,
                                               int32_t n_parts, const void* x, int64_t x_stride,
                                               const void* shared_gate_weight, const void* shared_out,
                                               int64_t shared_stride, void* h, int64_t h_stride, float* ss_out,
                                               int64_t ss_stride, int64_t rows, int32_t hidden, void* stream) {
  if (n_parts < 1 || n_parts > 8 || hidden % 1024 != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "combine_parts: 1 <= parts <= 8, hidden a multiple of 1024");
  if (!al16(parts) || !al16(x) || !al16(shared_gate_weight) || !al16(shared_out) || !al16(h) || parts_stride % 8 ||
      x_stride % 8 || shared_stride % 8 || h_stride % 8)
    return set_error(OMNI_ERR_UNSUPPORTED, "combine_parts: 16-byte aligned rows required");
  if (rows == 0) return OMNI_OK;
  return check_launch(launch(moe_combine_kernel, dim3((unsigned)rows), dim3(128), 0, static_cast<cudaStream_t>(stream),
                             static_cast<const uint16_t*>(parts), parts_stride, part_index,
                             static_cast<const float*>(nullptr), (int)n_parts, static_cast<const uint16_t*>(x),
                             x_stride, static_cast<const uint16_t*>(shared_gate_weight),
                             static_cast<const uint16_t*>(shared_out), shared_stride, static_cast<uint16_t*>(h),
                             h_stride, ss_out, ss_stride, (int)hidden, 1));
}

extern "C" OMNI_API int omni_moe_partial_sum(const void* y, int64_t y_stride, const int32_t* slot_of,
                                             const float* weights, int64_t weights_stride, int32_t top_k,
                                             int64_t rows, int32_t hidden, void* out, int64_t out_stride,
                                             void* stream) {
  if (top_k < 1 || top_k > 8 || hidden % 1024 != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "partial_sum: 1 <= top_k <= 8, hidden a multiple of 1024");
  if (!al16(y) || !al16(out) || y_stride % 8 || out_stride % 8)
    return set_error(OMNI_ERR_UNSUPPORTED, "partial_sum: 16-byte aligned rows required");
  if (rows == 0) return OMNI_OK;
  return check_launch(launch(moe_partial_sum_kernel, dim3((unsigned)rows), dim3(128), 0,
                             static_cast<cudaStream_t>(stream), static_cast<const uint16_t*>(y), y_stride, slot_of,
                             weights, weights_stride, (int)top_k, (int)hidden, static_cast<uint16_t*>(out),
                             out_stride));
}

extern "C" OMNI_API int omni_moe_ep_pack(const int32_t* topk_ids, const float* topk_weights, int64_t tokens,
                                         int32_t top_k, const void* xq, int64_t xq_stride, const float* xs,
                                         int64_t xs_stride, int32_t hidden, int32_t world, int32_t experts_per_rank,
                                         int64_t cap, void* send, int64_t row_bytes, int32_t* part_index,
                                         void* stream) {
  if (tokens < 0 || top_k < 1 || top_k > 32 || world < 1 || world > kEpMaxWorld || experts_per_rank < 1 ||
      cap < tokens || hidden % 128 != 0 || hidden <= 0)
    return set_error(OMNI_ERR_INVALID, "ep_pack: 1 <= top_k <= 32, 1 <= world <= 32, tokens <= cap, hidden % 128 == 0");
  if (row_bytes < hidden + 4 * (hidden / 128) + 8 * top_k || row_bytes % 16)
    return set_error(OMNI_ERR_INVALID, "ep_pack: row_bytes below the packed row or not a multiple of 16");
  if (!al16(xq) || !al16(send) || xq_stride % 16 || tokens > 65535)
    return set_error(OMNI_ERR_UNSUPPORTED, "ep_pack: 16-byte aligned rows, at most 65535 tokens");
  const unsigned grid = (unsigned)(tokens + world);
  return check_launch(launch(moe_ep_pack_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream),
                             topk_ids, topk_weights, (int)tokens, (int)top_k, static_cast<const uint8_t*>(xq),
                             xq_stride, xs, xs_stride, (int)hidden, (int)world, (int)experts_per_rank, (int)cap,
                             static_cast<uint8_t*>(send), row_bytes, part_index));
}
