// Weight-streaming GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   Y[rows, N] = epilogue( X[rows, K] . W[N, K]^T )        (nn.Linear layout)
//
// Decode-step projections have few activation rows (8-512) and many output
// features, so the kernel is "swap-AB": a CTA owns 128 output features, which
// sit on the MMA's M axis (TMEM lanes), and up to 256 activation rows, which
// sit on its N axis (TMEM columns).  W tiles (128 x 64, bf16, 128-byte
// swizzle) stream from HBM through a TMA pipeline; X tiles come from L2.
//
// Split-K: the S CTAs that share a feature tile form one thread-block cluster
// (S <= 16, chosen so that every cluster of the grid is co-resident).  CTA c
// owns the c-th contiguous block of the tile's rows.  Each CTA writes its fp32
// partial tile from TMEM into an L2-resident scratch slab ([rows][128], each
// warp store one coalesced 128-byte row segment); after one cluster barrier
// (release / acquire) each owner reads the S slabs' rows of its block in split
// order (deterministic), applies the epilogue and stores.  The slabs live in a
// static device array of the library, so GEMM launches that overlap on the GPU
// (other than through programmatic dependent launch on one stream, where a
// launch writes its slabs only after its predecessor has completed) must be
// serialised.  A CTA without split (S = 1) keeps its partial in shared memory.
// (Distributed shared memory moves about 12-16 bytes a cycle per SM here,
// which made a shared-memory exchange of 32 KB per CTA cost about 1.5 us.)
// The epilogue operands of the owned rows (RMSNorm scale, rotary position, KV
// slot, residual) are fetched while the MMAs run.  The only global scratch is
// the slab array above; the entry points take no workspace.
//
// Programmatic dependent launch: weights never depend on the previous kernel,
// so the producer issues the first stages' weight loads before
// griddepcontrol.wait, overlapping them with the predecessor's tail.
//
// Roles (256 threads): warp 0 = TMA producer, warp 1 = MMA issuer (each warp
// walks its loop together, one elected lane issues), warps 2-7 = epilogue
// operands during the main loop; all eight warps
// drain TMEM (warp w reads lanes 32 (w % 4) .. + 31, column half w / 4) and run
// the epilogue.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>
#include <map>
#include <mutex>
#include <utility>

#include "capi_util.h"
#include "common.cuh"
#include "detmath.cuh"

namespace omni {
namespace {
OMNI_DEFINE_STATUS(gemm)

constexpr int kBK = 64;        // K elements per stage (one 128-byte swizzle row)
constexpr int kTileN = 128;    // output features per CTA (MMA M)
constexpr int kMaxRows = 256;  // activation rows per CTA (MMA N)
constexpr int kMaxStages = 6;
constexpr int kThreadsG = 256;
constexpr int kMaxSplits = 16;
constexpr int kPrefillRows = 128;  // row tile cap beyond 256 rows

enum Epilogue : int { kEpiStore = 0, kEpiResidual = 1, kEpiSwiGLU = 2, kEpiF32 = 3, kEpiQKV = 4, kEpiRouter = 5 };

struct GemmParams {
  int rows;         // total activation rows
  int K;            // reduction length (multiple of 64)
  int N;            // output features of W (for SwiGLU: 2 * I)
  int row_tile;     // rows per CTA (multiple of 16, <= 256)
  int num_kb;       // K / 64
  int splits;       // CTAs per (feature tile, row tile)
  int stages;       // pipeline depth
  int tmem_cols;    // power of two >= row_tile
  int region;       // bytes of the pipeline / partial-tile region (1024-aligned)
  int swiglu_half;  // I for SwiGLU (gate rows [0, I), up rows [I, 2I))
  const uint16_t* residual;
  int64_t res_stride;
  void* y;
  int64_t y_stride;
  // folded RMSNorm: acc *= rsqrt(sum_p ss_in[p * ss_in_stride + row] / norm_dim + eps)
  const float* ss_in;
  int ss_in_parts;
  int64_t ss_in_stride;
  int norm_dim;
  float norm_eps;
  // per-row sum of squares of the bf16 output, one part per 128-feature tile
  float* ss_out;
  int64_t ss_out_stride;
  // qkv epilogue: per-head RMSNorm, neox rotary, q to y, k and v to their cache slot
  int hq, hkv, head_dim;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  float qk_eps;
  const float* cos_sin;
  int64_t max_pos;
  const int64_t* positions;
  const int64_t* cache_loc;
  int tokens_per_req, slot_stride, slot_base;
  uint16_t* k_cache;
  uint16_t* v_cache;
  // router epilogue: top_k experts per row by (prob desc, index asc), renormalised
  int32_t* topk_ids;
  float* topk_w;
  int top_k;
  // bytes to prefetch into L2 for a later launch (e.g. the next GEMM's weights), each
  // CTA its slice, issued at the start ahead of griddepcontrol.wait
  const uint8_t* l2_prefetch;
  int64_t l2_prefetch_bytes;
  // test hook (omni_gemm_wait_probe): polls per bounded wait (0 = kWaitLimit) and
  // a producer that issues no copies, so that the waits run out
  uint32_t wait_limit;
  int withhold_loads;
};

OMNI_DEVINL uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
OMNI_DEVINL void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
OMNI_DEVINL void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Shared-memory load by shared-window address.
OMNI_DEVINL float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
// Global load cached in L2 only (another SM wrote the line during this launch).
OMNI_DEVINL float4 ld_cg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Split-K partial slabs: [tile][row tile][split][row_tile][128] fp32.
constexpr size_t kScratchFloats = size_t(6) << 20;  // 24 MiB
__device__ __align__(16) float g_partials[kScratchFloats];

// SiLU by the fast exponential and division intrinsics: a few fp32 ulps from the exact
// form, far inside the bf16 rounding that follows (at 38.7 k rows the exact form held
// the SwiGLU epilogue back: gate_up 539 -> 415 us)
OMNI_DEVINL float silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Rows of the tile owned (reduced and stored) by cluster rank q: a contiguous block.
struct RowBlock {
  int per, begin, count;
};
OMNI_DEVINL RowBlock row_block(int rows_here, int S, int q) {
  RowBlock b;
  b.per = (rows_here + S - 1) / S;
  b.begin = q * b.per;
  b.count = max(0, min(b.per, rows_here - b.begin));
  return b;
}

// ---------------------------------------------------------------------------
// Epilogue of four consecutive output features of one row (lane ln of the row's warp
// holds features tile * 128 + 4 ln .. + 3, already scaled by the row's folded-norm
// factor): the fp32, router, qkv, store and residual epilogues.  Shared by the
// split-K kernel and the tile-loop kernel below; the whole warp calls it for one row.
// ---------------------------------------------------------------------------
// The global operands of one lane's four features, fetched ahead of the arithmetic so
// that a warp can have several rows' loads in flight: the residual, or for the qkv
// epilogue the rotary cos / sin of the features' pair dimensions and the head-norm gain.
struct QuadIn {
  uint2 rv;
  float4 c4, s4;
  uint2 gw;
};
template <int EPI>
OMNI_DEVINL QuadIn quad_fetch(const GemmParams& p, int64_t grow, int tile, int ln, int64_t pos) {
  QuadIn in;
  in.rv = make_uint2(0u, 0u);
  in.gw = make_uint2(0u, 0u);
  in.c4 = in.s4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const int64_t col = (int64_t)tile * kTileN + ln * 4;
  if (EPI == kEpiResidual) in.rv = *reinterpret_cast<const uint2*>(p.residual + grow * p.res_stride + col);
  if (EPI == kEpiQKV) {
    const int D = p.head_dim, half = D / 2;
    const int gh = (int)(col / D), d = (int)(col % D), ii = d % half;
    const float* cs = p.cos_sin + pos * D;
    in.c4 = *reinterpret_cast<const float4*>(cs + ii);
    in.s4 = *reinterpret_cast<const float4*>(cs + half + ii);
    if (gh < p.hq + p.hkv) in.gw = *reinterpret_cast<const uint2*>((gh < p.hq ? p.q_norm : p.k_norm) + d);
  }
  return in;
}

template <int EPI>
OMNI_DEVINL void quad_epilogue(const GemmParams& p, int64_t grow, int tile, int ln, float (&o)[4], const QuadIn& in,
                               int64_t loc) {
  const int f = ln * 4;
  const int64_t col = (int64_t)tile * kTileN + f;
  const uint2 rv = in.rv;
  if (EPI == kEpiF32) {
    float* Y = static_cast<float*>(p.y);
    *reinterpret_cast<float4*>(Y + grow * p.y_stride + col) = make_float4(o[0], o[1], o[2], o[3]);
  } else if (EPI == kEpiRouter) {
    // bf16 router logits (the gate projection's output), then the fp32 softmax over
    // the 128 experts of the row: lane l holds experts 4l..4l+3, partial sums in index
    // order, xor butterfly 16..1; top-k by (prob desc, index asc); weights renormalised
    // by their sum in selection order
    const uint2 packed = make_uint2(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]));
    uint16_t* Y = static_cast<uint16_t*>(p.y);
    *reinterpret_cast<uint2*>(Y + grow * p.y_stride + col) = packed;
    const float lg[4] = {bf_lo(packed.x), bf_hi(packed.x), bf_lo(packed.y), bf_hi(packed.y)};
    float mx = fmaxf(fmaxf(lg[0], lg[1]), fmaxf(lg[2], lg[3]));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
    float ex[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) ex[j] = det_expf(__fsub_rn(lg[j], mx));
    float z = __fadd_rn(__fadd_rn(__fadd_rn(ex[0], ex[1]), ex[2]), ex[3]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) z = __fadd_rn(z, __shfl_xor_sync(0xFFFFFFFFu, z, off));
    unsigned long long key[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t pb = __float_as_uint(__fdiv_rn(ex[j], z));
      const uint32_t ord = (pb >> 31) ? ~pb : (pb | 0x80000000u);
      key[j] = ((unsigned long long)ord << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)(f + j));
    }
    float wsum = 0.0f, wsel = 0.0f;
    int idsel = 0;
    for (int kk = 0; kk < p.top_k; ++kk) {
      unsigned long long best = 0ull;
#pragma unroll
      for (int j = 0; j < 4; ++j) best = key[j] > best ? key[j] : best;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const unsigned long long o2 = __shfl_xor_sync(0xFFFFFFFFu, best, off);
        best = o2 > best ? o2 : best;
      }
      const int e = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu));
      const uint32_t ob = (uint32_t)(best >> 32);
      const float pe = __uint_as_float((ob >> 31) ? (ob & 0x7FFFFFFFu) : ~ob);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (f + j == e) key[j] = 0ull;
      wsum = kk == 0 ? pe : __fadd_rn(wsum, pe);
      if (ln == kk) {
        wsel = pe;
        idsel = e;
      }
    }
    if (ln < p.top_k) {
      p.topk_ids[grow * p.top_k + ln] = idsel;
      p.topk_w[grow * p.top_k + ln] = __fdiv_rn(wsel, wsum);
    }
  } else if (EPI == kEpiQKV) {
    const int D = p.head_dim;
    const int gh = (int)(col / D);  // global head of these 4 features
    const int d = (int)(col % D);   // first dimension within the head
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = bf2f(f2bf(o[j]));  // the qkv projection's bf16 output
    const bool is_q = gh < p.hq, is_k = !is_q && gh < p.hq + p.hkv;
    // lanes sharing a head: D/4 consecutive lanes (the whole warp for D = 128)
    const int head_lanes = D / 4;
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) ss = __fmaf_rn(o[j], o[j], ss);
    for (int off = 1; off < head_lanes; off <<= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
    if (is_q || is_k) {
      // D is 64 or 128: scaling by the exact reciprocal is the same rounding as the division
      const float hr = rsqrtf(ss * (D == 128 ? 0.0078125f : 0.015625f) + p.qk_eps);
      const uint2 wv = in.gw;
      const float gw4[4] = {bf_lo(wv.x), bf_hi(wv.x), bf_lo(wv.y), bf_hi(wv.y)};
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = bf2f(f2bf(o[j] * hr * gw4[j]));
    }
    // neox rotation pairs d with d + D/2, held by lane ^ (D/8); every lane joins the shuffle
    const int half = D / 2;
    const float c4[4] = {in.c4.x, in.c4.y, in.c4.z, in.c4.w}, s4[4] = {in.s4.x, in.s4.y, in.s4.z, in.s4.w};
    float y4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float other = __shfl_xor_sync(0xFFFFFFFFu, o[j], D / 8);
      const int dd = d + j;
      const float c = c4[j], sn = s4[j];
      y4[j] = dd < half ? o[j] * c - other * sn : o[j] * c + other * sn;
    }
    const uint2 packed_rot = make_uint2(pack_bf2(y4[0], y4[1]), pack_bf2(y4[2], y4[3]));
    if (is_q) {
      uint16_t* Y = static_cast<uint16_t*>(p.y);
      *reinterpret_cast<uint2*>(Y + grow * p.y_stride + col) = packed_rot;
    } else if (is_k) {
      const int kh = gh - p.hq;
      *reinterpret_cast<uint2*>(p.k_cache + (loc * p.hkv + kh) * D + d) = packed_rot;
    } else {
      const int vh = gh - p.hq - p.hkv;
      *reinterpret_cast<uint2*>(p.v_cache + (loc * p.hkv + vh) * D + d) =
          make_uint2(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]));
    }
  } else {
    if (EPI == kEpiResidual) {
      o[0] += bf_lo(rv.x);
      o[1] += bf_hi(rv.x);
      o[2] += bf_lo(rv.y);
      o[3] += bf_hi(rv.y);
    }
    uint16_t* Y = static_cast<uint16_t*>(p.y);
    const uint2 packed = make_uint2(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]));
    *reinterpret_cast<uint2*>(Y + grow * p.y_stride + col) = packed;
    if (p.ss_out) {
      float ss = 0.0f;
      const float q4[4] = {bf_lo(packed.x), bf_hi(packed.x), bf_lo(packed.y), bf_hi(packed.y)};
#pragma unroll
      for (int j = 0; j < 4; ++j) ss = __fmaf_rn(q4[j], q4[j], ss);
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
      if (ln == 0) p.ss_out[tile * p.ss_out_stride + grow] = ss;
    }
  }
}

// SwiGLU of four outputs (out_col .. + 3) of one row from the gate and up sums.
OMNI_DEVINL void swiglu_quad(const GemmParams& p, int64_t grow, int64_t out_col, float4 gt, float4 up, float sc) {
  const float gg[4] = {gt.x, gt.y, gt.z, gt.w}, uu[4] = {up.x, up.y, up.z, up.w};
  float o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = silu(bf2f(f2bf(gg[j] * sc))) * bf2f(f2bf(uu[j] * sc));
  uint16_t* Y = static_cast<uint16_t*>(p.y);
  *reinterpret_cast<uint2*>(Y + grow * p.y_stride + out_col) = make_uint2(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]));
}

// Two CTAs fit on an SM (<= 128 registers a thread) for every epilogue but the fp32
// one (the codec head, once a step), so that with programmatic dependent launch the
// next GEMM's CTAs can start, and stream their weights, beside the CTAs of the
// current one.
template <int EPI>
__global__ void __launch_bounds__(kThreadsG, (EPI == kEpiF32) ? 1 : 2)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = p.stages;
  const int Rt = p.row_tile;
  const int S = p.splits;
  const uint32_t a_bytes = kTileN * kBK * 2;
  const uint32_t b_bytes = (uint32_t)Rt * kBK * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, rtile = blockIdx.y, split = blockIdx.z;
  const int row0 = rtile * Rt;
  const int rows_here = min(Rt, p.rows - row0);
  const uint32_t crank = S > 1 ? cluster_ctarank() : 0u;
  const RowBlock mine = row_block(rows_here, S, (int)crank);
  // shared memory: region [stages A][stages B], then [row info][barriers].  After
  // the main loop the region holds the S splits' fp32 partials of the owned rows,
  // receive slots [S][per][128] (slot q written by cluster rank q).
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + ST * a_bytes;
  float* row_info = reinterpret_cast<float*>(smem + p.region);  // [per] rstd, [per] position, [per] slot
  uint64_t* full = reinterpret_cast<uint64_t*>(row_info + 3 * ((mine.per + 1) & ~1));
  uint64_t* empty = full + kMaxStages;
  uint64_t* mma_done = empty + kMaxStages;
  uint64_t* pre_bar = mma_done + 1;  // the stages resident before the main loop, as one group
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 2);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] abort
  float* recv = reinterpret_cast<float*>(smem);

  const int kb_begin = (int)(((int64_t)p.num_kb * split) / S);
  const int kb_end = (int)(((int64_t)p.num_kb * (split + 1)) / S);
  const int nk = kb_end - kb_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(mma_done, 1);
    mbar_init(pre_bar, 1);
    flags[0] = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto load_w = [&](int s, int kb, uint64_t* bar) {
    uint8_t* dst = a_smem + s * a_bytes;
    const int kx = kb * kBK;
    if (EPI == kEpiSwiGLU) {
      const int g0 = tile * (kTileN / 2);
      tma_load_2d(dst, &tmap_w, bar, kx, g0);
      tma_load_2d(dst + (kTileN / 2) * kBK * 2, &tmap_w, bar, kx, p.swiglu_half + g0);
    } else {
      tma_load_2d(dst, &tmap_w, bar, kx, tile * kTileN);
    }
  };

  // Stages 0 .. pre-1 fill before the main loop and complete together on pre_bar
  // (one wait for the MMA warp); later stages cycle through the ring on full /
  // empty, starting at phase 0.
  const int pre = nk < ST ? nk : ST;
  const uint32_t lim = p.wait_limit ? p.wait_limit : kWaitLimit;
  if (warp == 0 && lane == 0 && !p.withhold_loads) {
    mbar_arrive_expect_tx(pre_bar, (uint32_t)pre * (a_bytes + b_bytes));
    for (int i = 0; i < pre; ++i) load_w(i, kb_begin + i, pre_bar);
  }
  if (p.l2_prefetch != nullptr && warp == 2 && lane == 0) {
    // this CTA's 16-byte aligned slice of the range, in pieces of at most 64 KB
    const int64_t ctas = (int64_t)gridDim.x * gridDim.y * gridDim.z;
    const int64_t cid = ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    const int64_t per = ((p.l2_prefetch_bytes + ctas - 1) / ctas + 15) & ~(int64_t)15;
    const int64_t b0 = cid * per;
    const int64_t b1 = min(p.l2_prefetch_bytes & ~(int64_t)15, b0 + per);
    for (int64_t b = b0; b < b1; b += 65536) bulk_prefetch_l2(p.l2_prefetch + b, (uint32_t)min((int64_t)65536, b1 - b));
  }
  griddep_wait();
  griddep_launch();

  if (warp == 0) {
    // producer: the whole warp walks the stages (warp-uniform addresses and
    // phases), one elected lane issues the copies
    const bool leader = elect_one();
    if (leader && !p.withhold_loads)
      for (int i = 0; i < pre; ++i) tma_load_2d(b_smem + i * b_bytes, &tmap_x, pre_bar, (kb_begin + i) * kBK, row0);
    int s = 0;
    uint32_t ph = 0;
    for (int i = pre; i < nk; ++i) {
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&empty[s], ph, lim))) {
        if (leader) {
          report_status(kDevTimeoutMma);
          flags[0] = 1;
        }
        break;
      }
      if (leader && !p.withhold_loads) {
        mbar_arrive_expect_tx(&full[s], a_bytes + b_bytes);
        load_w(s, kb_begin + i, &full[s]);
        tma_load_2d(b_smem + s * b_bytes, &tmap_x, &full[s], (kb_begin + i) * kBK, row0);
      }
      __syncwarp();
      if (++s == ST) {
        s = 0;
        ph ^= 1u;
      }
    }
  } else if (warp == 1) {
    // MMA issuer: the whole warp waits, one elected lane issues
    const bool leader = elect_one();
    // A = W (128 features on M), B = X (the tile's rows on N)
    const uint32_t idesc = idesc_bf16_f32(kTileN, Rt);
    const uint64_t wd0 = smem_desc_sw128(a_smem), xd0 = smem_desc_sw128(b_smem);
    bool ok = nk == 0 || __all_sync(0xFFFFFFFFu, mbar_wait(pre_bar, 0, lim));
    if (!ok && leader) {
      report_status(kDevTimeoutTma);
      flags[0] = 1;
    }
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; ok && i < nk; ++i) {
      if (i >= pre && !__all_sync(0xFFFFFFFFu, mbar_wait(&full[s], ph, lim))) {
        if (leader) {
          report_status(kDevTimeoutTma);
          flags[0] = 1;
        }
        ok = false;
        break;
      }
      tc_fence_after();
      // descriptor start addresses advance by 16-byte units: a stage, then 32 bytes per K step
      const uint64_t wd = wd0 + (uint64_t)(s * (a_bytes >> 4)), xd = xd0 + (uint64_t)(s * (b_bytes >> 4));
      if (leader) {
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          tc_mma_bf16(tmem, wd + 2 * kk, xd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        // the stage is refilled only when a later K block reuses it
        if (i + ST < nk) tc_commit(&empty[s]);
      }
      __syncwarp();
      if (++s == ST) {
        s = 0;
        if (i >= pre) ph ^= 1u;
      }
    }
    if (leader) {
      if (ok) tc_commit(mma_done);
      else mbar_arrive(mma_done);
    }
  } else if (warp >= 2) {
    // while the MMAs run: per-row epilogue operands of the rows this CTA owns
    for (int i = threadIdx.x - 64; i < mine.count; i += kThreadsG - 64) {
      const int64_t grow = row0 + mine.begin + i;
      float rs = 1.0f;
      if (p.ss_in != nullptr) {
        float ssum = 0.0f;
        for (int q = 0; q < p.ss_in_parts; ++q) ssum += p.ss_in[q * p.ss_in_stride + grow];
        rs = rsqrtf(ssum / (float)p.norm_dim + p.norm_eps);
      }
      row_info[i] = rs;
      if (EPI == kEpiQKV) {
        int64_t pos, loc;
        if (p.positions) {
          pos = p.positions[grow];
          loc = p.cache_loc[grow];
        } else {
          const int t = (int)(grow % p.tokens_per_req);
          pos = p.slot_base + t;
          loc = (grow / p.tokens_per_req) * p.slot_stride + p.slot_base + t;
        }
        if (pos < 0 || pos >= p.max_pos) pos = 0;
        reinterpret_cast<int*>(row_info)[mine.per + i] = (int)pos;
        reinterpret_cast<int*>(row_info)[2 * mine.per + i] = (int)loc;
      }
    }
  }
  __syncwarp();

  // ---- accumulators: TMEM -> this split's slab (S > 1) or shared memory (S = 1) ----
  const bool have_acc = nk > 0;
  if (have_acc) {
    if (!mbar_wait(mma_done, 0, lim)) {
      report_status(kDevTimeoutMma);
      flags[0] = 1;
    }
  }
  tc_fence_after();
  __syncthreads();
  bool aborted = flags[0] != 0;
  // the residual rows this thread will add, fetched ahead of the reduction
  constexpr int kPre = 4;
  uint2 res_pre[kPre];
  if (EPI == kEpiResidual && !aborted) {
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      const int idx = threadIdx.x + u * kThreadsG;
      if (idx < mine.count * 32)
        res_pre[u] = *reinterpret_cast<const uint2*>(p.residual + (int64_t)(row0 + mine.begin + (idx >> 5)) *
                                                                         p.res_stride +
                                                     (int64_t)tile * kTileN + (idx & 31) * 4);
    }
  }
  // this launch's slabs: split q of the tile at slab + q * Rt * 128
  float* slab = g_partials + ((size_t)(tile * gridDim.y + rtile) * S) * (size_t)Rt * kTileN;
  if (!aborted) {
    // warp w: TMEM lanes (features) 32 (w % 4) .., 32-column chunks w / 4, w / 4 + 2, ...
    const int f = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    // S > 1: each warp store writes one coalesced 128-byte row segment of the slab
    float* gdst = slab + (size_t)split * Rt * kTileN + f;
    float* sdst = recv + f;
    auto put_rows = [&](int cb, const uint32_t(&r)[32]) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (cb + j < rows_here) {
          if (S > 1) gdst[(cb + j) * kTileN] = __uint_as_float(r[j]);
          else sdst[(cb + j) * kTileN] = __uint_as_float(r[j]);
        }
    };
    for (int c0 = (warp >> 2) * 32; c0 < rows_here; c0 += 128) {
      // two 32-column loads in flight per wait
      uint32_t r0[32], r1[32];
      if (have_acc) {
        tmem_ld_32x32b_x32(lane_base + (uint32_t)c0, r0);
        if (c0 + 64 < rows_here) tmem_ld_32x32b_x32(lane_base + (uint32_t)(c0 + 64), r1);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r0[j] = r1[j] = 0u;
      }
      put_rows(c0, r0);
      if (c0 + 64 < rows_here) put_rows(c0 + 64, r1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  // every split's slab is written (the release orders the global stores for the
  // cluster's readers)
  if (S > 1) {
    cluster_arrive_release();
    cluster_wait();
  }

  // ---- sum the owned rows' partials in split order and apply the epilogue ----
  const uint32_t recv_u32 = smem_u32(recv);
  const size_t slab_floats = (size_t)Rt * kTileN;
  auto acc4 = [&](int i, int f) -> float4 {
    float4 v[kMaxSplits];
    const int r = mine.begin + i;
    if (S == 1) {
      v[0] = ld_shared_f4(recv_u32 + (uint32_t)((r * kTileN + f) * 4));
    } else {
      const float* a0 = slab + r * kTileN + f;
#pragma unroll
      for (int q = 0; q < kMaxSplits; ++q)
        if (q < S) v[q] = ld_cg_f4(a0 + q * slab_floats);
    }
    float4 a = v[0];
#pragma unroll
    for (int q = 1; q < kMaxSplits; ++q)
      if (q < S) {
        a.x += v[q].x;
        a.y += v[q].y;
        a.z += v[q].z;
        a.w += v[q].w;
      }
    return a;
  };
  const int items = aborted ? 0 : mine.count;
  if (EPI == kEpiSwiGLU) {
    // features 0..63: gate, 64..127: up, for outputs tile*64 .. tile*64+63
    for (int idx = threadIdx.x; idx < items * 16; idx += kThreadsG) {
      const int i = idx >> 4;
      const int g = (idx & 15) * 4;
      // gate and up summed side by side in split order (two CTAs per SM leave no
      // registers for all S slots of both in flight)
      const int r = mine.begin + i;
      float4 gt, up;
      const float* sg = slab + r * kTileN + g;
      if (S == 1) {
        gt = ld_shared_f4(recv_u32 + (uint32_t)((r * kTileN + g) * 4));
        up = ld_shared_f4(recv_u32 + (uint32_t)((r * kTileN + g + 64) * 4));
      } else {
        gt = ld_cg_f4(sg);
        up = ld_cg_f4(sg + 64);
      }
      for (int q = 1; q < S; ++q) {
        const float4 a = ld_cg_f4(sg + q * slab_floats);
        const float4 b = ld_cg_f4(sg + q * slab_floats + 64);
        gt.x += a.x;
        gt.y += a.y;
        gt.z += a.z;
        gt.w += a.w;
        up.x += b.x;
        up.y += b.y;
        up.z += b.z;
        up.w += b.w;
      }
      swiglu_quad(p, row0 + mine.begin + i, tile * 64 + g, gt, up, row_info[i]);
    }
    return;
  }
  // one warp per owned row, lane l holds features 4l..4l+3; kPre rows per thread per
  // round, their residuals loaded together (the first round's ahead of the reduction)
  for (int base = 0; base < items * 32; base += kThreadsG * kPre) {
  uint2 rv[kPre];
  if (EPI == kEpiResidual) {
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      const int idx = base + threadIdx.x + u * kThreadsG;
      if (idx < items * 32)
        rv[u] = base == 0 ? res_pre[u]
                          : *reinterpret_cast<const uint2*>(p.residual + (int64_t)(row0 + mine.begin + (idx >> 5)) *
                                                                             p.res_stride +
                                                            (int64_t)tile * kTileN + (idx & 31) * 4);
    }
  }
#pragma unroll
  for (int u = 0; u < kPre; ++u) {
    const int idx = base + threadIdx.x + u * kThreadsG;
    if (idx >= items * 32) break;  // warp-uniform: items * 32 is a multiple of 32
    const int i = idx >> 5;
    const int ln = idx & 31;
    const float sc = row_info[i];
    const float4 a = acc4(i, ln * 4);
    float o[4] = {a.x * sc, a.y * sc, a.z * sc, a.w * sc};
    int64_t pos = 0, loc = 0;
    if (EPI == kEpiQKV) {
      pos = reinterpret_cast<const int*>(row_info)[mine.per + i];
      loc = reinterpret_cast<const int*>(row_info)[2 * mine.per + i];
    }
    QuadIn in;
    if (EPI == kEpiResidual) {
      in.rv = rv[u];
    } else {
      in = quad_fetch<EPI>(p, row0 + mine.begin + i, tile, ln, pos);
    }
    quad_epilogue<EPI>(p, row0 + mine.begin + i, tile, ln, o, in, loc);
  }
  }
}

// ---------------------------------------------------------------------------
// Prefill-sized batches: a persistent tile loop, one CTA per SM.  The CTA walks the
// (row tile of 128, feature tile of 128) pairs c, c + grid, ... (feature tile fastest,
// so neighbouring CTAs share an activation block in L2).  Warp 0 streams W and X
// k-steps through a five-stage ring across tile boundaries; warp 1 issues each tile's
// MMAs into one of two TMEM accumulators; two epilogue groups of four warps take the
// tiles in turn (group g the accumulator g), so that a tile's epilogue runs while the
// next tile's MMAs do.  An epilogue group drains its accumulator 32 rows at a time
// into a 16 KB staging buffer (lane = feature as TMEM holds it, row-contiguous in
// shared memory), then a warp per row applies the same fused epilogue as the split-K
// kernel.  No split: every tile sums its whole K in TMEM.
// ---------------------------------------------------------------------------
constexpr int kLoopThreads = 320;
constexpr int kLoopWBytes = kTileN * kBK * 2;  // 16 KB
// Row tile RT (the MMA's N): 128 rows with five 32 KB stages, drained 32 rows at a time;
// or 256 rows with four 48 KB stages (twice the multiply-adds per staged byte), drained
// 16 rows at a time so that the staging fits beside them.
template <int RT>
struct LoopCfg {
  static constexpr int kStages = RT == 256 ? 4 : 5;
  static constexpr int kChunk = RT == 256 ? 16 : 32;
  static constexpr int kStageBytes = kLoopWBytes + RT * kBK * 2;
  static constexpr int kStagingBytes = kChunk * kTileN * 4;
  static constexpr int kStagingOff = kStages * kStageBytes;
  static constexpr int kInfoOff = kStagingOff + 2 * kStagingBytes;
  static constexpr int kBarOff = kInfoOff + 2 * 3 * RT * 4;
  static constexpr size_t kSmem = (size_t)kBarOff + 256 + 1024;
};

struct LoopBars {
  uint64_t full[5], empty[5], acc_full[2], acc_empty[2];
  uint32_t tmem;
};

OMNI_DEVINL void group_sync(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }
// Barrier of the group's 128 threads that also ANDs a predicate over them (so that the
// group leaves a wait that ran out together).
OMNI_DEVINL bool group_all(int id, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id)
      : "memory");
  return r != 0;
}

template <int EPI, int RT>
__global__ void __launch_bounds__(kLoopThreads, 1)
    gemm_loop_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                     const __grid_constant__ GemmParams p) {
  using C = LoopCfg<RT>;
  constexpr int kLoopRows = RT, kLoopStages = C::kStages, kChunk = C::kChunk;
  constexpr int kLoopStageBytes = C::kStageBytes, kLoopStagingBytes = C::kStagingBytes;
  constexpr int kLoopStagingOff = C::kStagingOff, kLoopInfoOff = C::kInfoOff, kLoopBarOff = C::kBarOff;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  LoopBars* bars = reinterpret_cast<LoopBars*>(smem + kLoopBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = EPI == kEpiSwiGLU ? p.swiglu_half / (kTileN / 2) : p.N / kTileN;
  const int total = tiles_n * ((p.rows + kLoopRows - 1) / kLoopRows);
  const int nk = p.num_kb;
  const uint32_t lim = kWaitLimit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kLoopStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 128);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem, 2 * kLoopRows);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  griddep_wait();

  if (warp == 0) {
    // ---------------- producer ----------------
    const bool leader = elect_one();
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      const int t = tile % tiles_n, row0 = (tile / tiles_n) * kLoopRows;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % kLoopStages;
        if (it >= kLoopStages &&
            !__all_sync(0xFFFFFFFFu, mbar_wait(&bars->empty[s], ((it / kLoopStages) - 1) & 1, lim))) {
          if (leader) report_status(kDevTimeoutMma);
          tile = total;
          break;
        }
        if (leader) {
          uint8_t* st = smem + s * kLoopStageBytes;
          mbar_arrive_expect_tx(&bars->full[s], kLoopStageBytes);
          if (EPI == kEpiSwiGLU) {
            tma_load_2d(st, &tmap_w, &bars->full[s], kb * kBK, t * (kTileN / 2));
            tma_load_2d(st + (kTileN / 2) * kBK * 2, &tmap_w, &bars->full[s], kb * kBK, p.swiglu_half + t * (kTileN / 2));
          } else {
            tma_load_2d(st, &tmap_w, &bars->full[s], kb * kBK, t * kTileN);
          }
          tma_load_2d(st + kLoopWBytes, &tmap_x, &bars->full[s], kb * kBK, row0);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const bool leader = elect_one();
    const uint32_t idesc = idesc_bf16_f32(kTileN, kLoopRows);
    int it = 0, i = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++i) {
      const int b = i & 1;
      if (i >= 2 && !__all_sync(0xFFFFFFFFu, mbar_wait(&bars->acc_empty[b], ((i >> 1) - 1) & 1, lim))) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % kLoopStages;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars->full[s], (it / kLoopStages) & 1, lim))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* st = smem + s * kLoopStageBytes;
        const uint64_t wd = smem_desc_sw128(st), xd = smem_desc_sw128(st + kLoopWBytes);
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc_mma_bf16(tmem + b * kLoopRows, wd + 2 * kk, xd + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&bars->empty[s]);
        }
        __syncwarp();
      }
      if (ok && leader) tc_commit(&bars->acc_full[b]);
      __syncwarp();
    }
    if (!ok && leader) report_status(kDevTimeoutTma);
  } else {
    // ---------------- epilogue groups ----------------
    const int g = (warp - 2) >> 2;           // group: accumulator g, tiles i = g (mod 2)
    const int wl = (warp - 2) & 3;           // warp within the group
    const int q = warp & 3;                  // TMEM lane quarter: features 32 q .. 32 q + 31
    const int gt = wl * 32 + lane;           // thread within the group
    float* staging = reinterpret_cast<float*>(smem + kLoopStagingOff + g * kLoopStagingBytes);
    float* info = reinterpret_cast<float*>(smem + kLoopInfoOff) + g * 3 * kLoopRows;
    int* ipos = reinterpret_cast<int*>(info + kLoopRows);
    int* iloc = reinterpret_cast<int*>(info + 2 * kLoopRows);
    int i = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++i) {
      if ((i & 1) != g) continue;
      const int t = tile % tiles_n, row0 = (tile / tiles_n) * kLoopRows;
      const int rows_here = min(kLoopRows, p.rows - row0);
      // the tile's per-row operands while its MMAs run
      for (int r = gt; r < rows_here; r += 128) {
        const int64_t grow = row0 + r;
        float rs = 1.0f;
        if (p.ss_in != nullptr) {
          float ssum = 0.0f;
          for (int pp = 0; pp < p.ss_in_parts; ++pp) ssum += p.ss_in[pp * p.ss_in_stride + grow];
          rs = rsqrtf(ssum / (float)p.norm_dim + p.norm_eps);
        }
        info[r] = rs;
        if (EPI == kEpiQKV) {
          int64_t pos, loc;
          if (p.positions) {
            pos = p.positions[grow];
            loc = p.cache_loc[grow];
          } else {
            const int tt = (int)(grow % p.tokens_per_req);
            pos = p.slot_base + tt;
            loc = (grow / p.tokens_per_req) * p.slot_stride + p.slot_base + tt;
          }
          if (pos < 0 || pos >= p.max_pos) pos = 0;
          ipos[r] = (int)pos;
          iloc[r] = (int)loc;
        }
      }
      if (!group_all(1 + g, mbar_wait(&bars->acc_full[g], (i >> 1) & 1, lim))) {
        if (gt == 0) report_status(kDevTimeoutMma);
        break;
      }
      tc_fence_after();
      const int nchunks = (rows_here + kChunk - 1) / kChunk;
      for (int c = 0; c < nchunks; ++c) {
        uint32_t v[kChunk];
        const uint32_t ta = tmem + g * kLoopRows + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * kChunk);
        if constexpr (kChunk == 32) tmem_ld_32x32b_x32(ta, v);
        else tmem_ld_32x32b_x16(ta, v);
        tc_wait_ld();
        if (c == nchunks - 1) {
          // every read of this accumulator is done: the MMA warp may refill it
          tc_fence_before();
          mbar_arrive(&bars->acc_empty[g]);
        }
        group_sync(1 + g);  // the previous chunk's rows are done with the staging buffer
#pragma unroll
        for (int j = 0; j < kChunk; ++j) staging[j * kTileN + q * 32 + lane] = __uint_as_float(v[j]);
        group_sync(1 + g);
        const int rmax = min(kChunk, rows_here - c * kChunk);
        if (EPI == kEpiSwiGLU) {
          // two rows a warp: lanes 0-15 and 16-31, four outputs a lane
          for (int rr = 2 * wl + (lane >> 4); rr < rmax; rr += 8) {
            const int gq = (lane & 15) * 4;
            const float4 gv = *reinterpret_cast<const float4*>(staging + rr * kTileN + gq);
            const float4 uv = *reinterpret_cast<const float4*>(staging + rr * kTileN + 64 + gq);
            swiglu_quad(p, row0 + c * kChunk + rr, (int64_t)t * 64 + gq, gv, uv, info[c * kChunk + rr]);
          }
        } else {
          // rows wl, wl + 4, ... of the chunk, four at a time: their global operands
          // first (four rows' loads in flight), then the arithmetic and the stores
          for (int r0 = wl; r0 < rmax; r0 += 16) {
            QuadIn in[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int rr = r0 + 4 * u;
              if (rr < rmax) {
                const int r = c * kChunk + rr;
                in[u] = quad_fetch<EPI>(p, row0 + r, t, lane, EPI == kEpiQKV ? ipos[r] : 0);
              }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int rr = r0 + 4 * u;
              if (rr < rmax) {
                const int r = c * kChunk + rr;
                const float4 a = *reinterpret_cast<const float4*>(staging + rr * kTileN + lane * 4);
                const float sc = info[r];
                float o[4] = {a.x * sc, a.y * sc, a.z * sc, a.w * sc};
                quad_epilogue<EPI>(p, row0 + r, t, lane, o, in[u], EPI == kEpiQKV ? iloc[r] : 0);
              }
            }
          }
        }
      }
      group_sync(1 + g);  // the group's row info and staging are free for its next tile
    }
  }
  griddep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 2 * kLoopRows);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2D bf16 row-major [rows, cols] with row stride (elements), box {64, box_rows}, 128B swizzle.
bool make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t stride, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct Plan {
  int row_tile, num_rt, tiles, num_kb, splits, stages, tmem_cols, region;
  size_t smem;
};

int num_sms() { return device_sm_count(); }

// Kernel attributes belong to the device that is current when they are set.
template <int EPI>
void set_kernel_attrs() {
  const void* k = reinterpret_cast<const void*>(gemm_kernel<EPI>);
  if (once_per_device(k, kAttrSmem, [] {
        return cudaFuncSetAttribute(gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      }) != cudaSuccess)
    cudaGetLastError();
  if (once_per_device(k, kAttrCluster, [] {
        return cudaFuncSetAttribute(gemm_kernel<EPI>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      }) != cudaSuccess)
    cudaGetLastError();
  prefer_max_shared(k);
}

// Co-resident clusters of S CTAs with this much shared memory (cached).
template <int EPI>
int max_active_clusters(int S, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;  // (device, S * 64 + smem KB / 4)
  std::lock_guard<std::mutex> g(mu);
  const int key = (int)((smem + 4095) / 4096);
  if (key >= 64) return 0;
  int& slot = cache.emplace(std::make_pair(current_device(), S * 64 + key), -1).first->second;
  if (slot >= 0) return slot;
  set_kernel_attrs<EPI>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, (unsigned)S);
  cfg.blockDim = dim3(kThreadsG);
  cfg.dynamicSmemBytes = (size_t)key * 4096;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)S;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel<EPI>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  // The cluster query counts one CTA per SM here, while two of these CTAs fit on an SM
  // (and are placed so, measured): for cluster sizes that fit in any GPC (<= 8) count
  // the per-SM occupancy instead.
  int per_sm = 0;
  if (S <= 8 && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_kernel<EPI>, kThreadsG,
                                                              (size_t)key * 4096) == cudaSuccess) {
    const int by_sm = per_sm * num_sms() / S;
    if (by_sm > n) n = by_sm;
  } else {
    cudaGetLastError();
  }
  slot = n;
  return n;
}

// Bytes of the region that holds the pipeline stages during the main loop and,
// after it, without split, the partial tile [row_tile][128] fp32.
size_t plan_region(int row_tile, int stages, int splits) {
  const size_t stage_bytes = (size_t)kTileN * kBK * 2 + (size_t)row_tile * kBK * 2;
  // without split the partial tile [row_tile][128] fp32 stays here
  const size_t partials = splits == 1 ? (size_t)row_tile * kTileN * 4 : 0;
  const size_t pipe = (size_t)stages * stage_bytes;
  const size_t r = pipe > partials ? pipe : partials;
  return (r + 1023) & ~(size_t)1023;
}

size_t plan_smem(int row_tile, int stages, int splits) {
  const int per = (row_tile + splits - 1) / splits;
  const size_t info = (size_t)3 * ((per + 1) & ~1) * 4;
  return 1024 + plan_region(row_tile, stages, splits) + info + (2 * kMaxStages + 2) * 8 + 16;
}

int plan_stages(int row_tile, int kb_per, int splits) {
  int st = kb_per < 4 ? kb_per : 4;
  if (st < 1) st = 1;
  while (st > 1 && plan_smem(row_tile, st, splits) > 227 * 1024) --st;
  return st;
}

// Rows per CTA.  Splitting the rows into several tiles re-reads the weights
// from L2 once per tile but shrinks each CTA's partial tile and epilogue;
// split-K instead shrinks each CTA's weight stream.  Measured on B200 over the
// decode-step shapes (K 1024 / 3072, 8..48 feature tiles, every split): 32-row
// tiles up to 64 rows, 64-row tiles up to 256 rows; beyond that (prefill-sized
// batches) about 48 (feature tile, row tile) pairs when K <= 1024 and 32 beyond,
// with power-of-two row tiles of at least 32 rows (64 when K > 1024) and at most
// 128: at 38.7k rows (the mixed prefill step's projections) 128-row tiles with
// three stages, two CTAs an SM, ran 666 / 753 / 761 / 889 TFLOP/s (qkv, o,
// gate_up, down) against 543 / 612 / 596 / 769 with 256-row tiles (one CTA an SM).
int plan_row_tile(int64_t rows, int64_t k, int tiles) {
  const int min_rt = k > 1024 ? 64 : 32;
  const int target = k > 1024 ? 32 : 48;
  int64_t rt;
  if (rows <= 32) {
    rt = rows;
  } else if (rows <= 64) {
    rt = 32;
  } else if (rows <= 256) {
    rt = 64;
  } else {
    const int nrt = (target + tiles - 1) / tiles;
    const int64_t want = (rows + nrt - 1) / nrt;
    rt = min_rt;
    while (rt * 2 <= want && rt * 2 <= kPrefillRows) rt *= 2;
  }
  rt = (rt + 15) / 16 * 16;
  if (rt < 16) rt = 16;
  if (rt > kMaxRows) rt = kMaxRows;
  return (int)rt;
}

template <int EPI>
Plan make_plan(int64_t rows, int64_t k, int64_t n, int splits_req) {
  Plan pl{};
  pl.tiles = (int)(EPI == kEpiSwiGLU ? (n / 2) / (kTileN / 2) : n / kTileN);
  pl.row_tile = plan_row_tile(rows, k, pl.tiles);
  // every row tile starts inside the activation rows
  pl.num_rt = (int)((rows + pl.row_tile - 1) / pl.row_tile);
  if (pl.num_rt < 1) pl.num_rt = 1;
  pl.num_kb = (int)(k / kBK);
  const int clusters = pl.tiles * pl.num_rt;
  // split partial slabs of the whole grid fit in the scratch array
  auto slabs_fit = [&](int S) {
    return S == 1 || (size_t)clusters * S * pl.row_tile * kTileN <= kScratchFloats;
  };
  int best = 1;
  if (splits_req > 0) {
    // the requested split, narrowed until the tile fits in shared memory and the
    // slabs in the scratch array
    best = splits_req;
    while (best > 1 && (plan_smem(pl.row_tile, plan_stages(pl.row_tile, (pl.num_kb + best - 1) / best, best), best) >
                            227 * 1024 ||
                        !slabs_fit(best)))
      --best;
  } else {
    // the widest split whose clusters all fit in one wave, preferring more busy SMs; at
    // decode row counts (<= 64) instead the widest split of at most 8 with at most 160
    // CTAs (192 for SwiGLU), about one CTA per SM, which a B200 sweep of the decode
    // projections measured faster than filling both CTA slots of every SM (the exchange
    // then waits on fewer, fuller CTAs): predictor gate_up 7.8 -> 6.7 us, talker qkv
    // 5.7 -> 5.2 us, the others within 0.15 us
    const bool decode = rows <= 64;
    const long cap = decode ? (EPI == kEpiSwiGLU ? 192 : 160) : LONG_MAX;
    const int max_s = decode ? 8 : kMaxSplits;
    long best_busy = 0;
    for (int S = 1; S <= max_s && S <= pl.num_kb; ++S) {
      const int st = plan_stages(pl.row_tile, (pl.num_kb + S - 1) / S, S);
      const size_t sm = plan_smem(pl.row_tile, st, S);
      if (sm > 227 * 1024 || !slabs_fit(S)) continue;
      const long busy = (long)clusters * S;
      if (decode) {
        // clusters never wait on one another, so a grid above one wave only costs time
        if (busy > cap && S > 1) continue;
      } else {
        const int fit = S == 1 ? num_sms() : max_active_clusters<EPI>(S, sm);
        if (clusters > fit) continue;
      }
      if (busy > best_busy) {
        best_busy = busy;
        best = S;
      }
    }
  }
  if (best > pl.num_kb) best = pl.num_kb;
  if (best < 1) best = 1;
  pl.splits = best;
  pl.stages = plan_stages(pl.row_tile, (pl.num_kb + best - 1) / best, best);
  // prefill-sized batches: as many stages as leave room for a second CTA on the SM
  // (its main loop overlaps this one's epilogue), at least two
  if (rows > 256)
    while (pl.stages > 2 && 2 * (plan_smem(pl.row_tile, pl.stages, best) + 1024) > 228 * 1024) --pl.stages;
  int tc = 32;
  while (tc < pl.row_tile) tc <<= 1;
  pl.tmem_cols = tc;
  pl.smem = plan_smem(pl.row_tile, pl.stages, best);
  pl.region = (int)plan_region(pl.row_tile, pl.stages, best);
  return pl;
}

// Prefill-sized batches with enough (row tile, feature tile) pairs for every SM take the
// tile loop; a call that asks for a split count (1 included) keeps the split-K kernel.
template <int EPI, int RT>
int launch_loop(const void* x, int64_t rows, int64_t k, int64_t x_stride, const void* w, int64_t n, GemmParams gp,
                int tiles, cudaStream_t st) {
  constexpr int kLoopRows = RT;
  constexpr size_t kLoopSmem = LoopCfg<RT>::kSmem;
  CUtensorMap tw, tx;
  const int wbox = EPI == kEpiSwiGLU ? kTileN / 2 : kTileN;
  if (!make_tmap(&tw, w, n, k, k, wbox) || !make_tmap(&tx, x, rows, k, x_stride, kLoopRows))
    return set_error(OMNI_ERR_UNSUPPORTED, "tensor map encoding failed");
  gp.rows = (int)rows;
  gp.K = (int)k;
  gp.N = (int)n;
  gp.row_tile = kLoopRows;
  gp.num_kb = (int)(k / kBK);
  gp.splits = 1;
  gp.swiglu_half = (int)(n / 2);
  const void* kern = reinterpret_cast<const void*>(gemm_loop_kernel<EPI, RT>);
  if (once_per_device(kern, kAttrSmem, [] {
        return cudaFuncSetAttribute(gemm_loop_kernel<EPI, RT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)LoopCfg<RT>::kSmem);
      }) != cudaSuccess)
    return check_launch(cudaGetLastError());
  const int64_t total = (int64_t)tiles * ((rows + kLoopRows - 1) / kLoopRows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(total < num_sms() ? total : num_sms()));
  cfg.blockDim = dim3(kLoopThreads);
  cfg.dynamicSmemBytes = kLoopSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return check_launch(cudaLaunchKernelEx(&cfg, gemm_loop_kernel<EPI, RT>, tw, tx, gp));
}

template <int EPI>
int launch_gemm(const void* x, int64_t rows, int64_t k, int64_t x_stride, const void* w, int64_t n, GemmParams gp,
                int splits_req, cudaStream_t st) {
  // the tile loop's two four-warp epilogue groups keep up with the store, residual and
  // SwiGLU epilogues; the qkv one (head norms, rotary, K/V scatter) measured faster on
  // the split-K kernel's sixteen epilogue warps an SM (38.7 k rows: 504 against 669 us),
  // and the router and fp32 ones stay there too
  if (EPI == kEpiStore || EPI == kEpiResidual || EPI == kEpiSwiGLU) {
    const int tiles = (int)(EPI == kEpiSwiGLU ? (n / 2) / (kTileN / 2) : n / kTileN);
    // 256-row tiles once they give every SM a tile (38.7 k rows: down 1 023 -> 1 215,
    // qkv (store epilogue) 1 002 -> 1 160, o 973 -> 1 034, gate_up 904 -> 1 174 TFLOP/s),
    // else 128-row tiles
    if (rows > 256 && splits_req == 0) {
      if ((int64_t)tiles * ((rows + 255) / 256) >= num_sms())
        return launch_loop<EPI, 256>(x, rows, k, x_stride, w, n, gp, tiles, st);
      if ((int64_t)tiles * ((rows + 127) / 128) >= num_sms())
        return launch_loop<EPI, 128>(x, rows, k, x_stride, w, n, gp, tiles, st);
    }
  }
  const Plan pl = make_plan<EPI>(rows, k, n, splits_req);
  if (pl.splits > kMaxSplits) return set_error(OMNI_ERR_UNSUPPORTED, "at most 16 K-splits");
  if (pl.smem > 227 * 1024) return set_error(OMNI_ERR_UNSUPPORTED, "GEMM tile does not fit in shared memory");
  CUtensorMap tw, tx;
  const int wbox = EPI == kEpiSwiGLU ? kTileN / 2 : kTileN;
  if (!make_tmap(&tw, w, n, k, k, wbox) || !make_tmap(&tx, x, rows, k, x_stride, pl.row_tile))
    return set_error(OMNI_ERR_UNSUPPORTED, "tensor map encoding failed");
  gp.rows = (int)rows;
  gp.K = (int)k;
  gp.N = (int)n;
  gp.row_tile = pl.row_tile;
  gp.num_kb = pl.num_kb;
  gp.splits = pl.splits;
  gp.stages = pl.stages;
  gp.tmem_cols = pl.tmem_cols;
  gp.region = pl.region;
  gp.swiglu_half = (int)(n / 2);
  set_kernel_attrs<EPI>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.tiles, (unsigned)pl.num_rt, (unsigned)pl.splits);
  cfg.blockDim = dim3(kThreadsG);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pl.splits > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = (unsigned)pl.splits;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return check_launch(cudaLaunchKernelEx(&cfg, gemm_kernel<EPI>, tw, tx, gp));
}

int run_linear(const void* x, int64_t rows, int64_t k, int64_t x_stride, const void* w, int64_t n, int epilogue,
               const GemmParams& gp, int splits, cudaStream_t st) {
  if (rows < 0 || k <= 0 || n <= 0) return set_error(OMNI_ERR_INVALID, "bad GEMM shape");
  if (epilogue < 0 || epilogue > 5) return set_error(OMNI_ERR_INVALID, "unknown epilogue");
  if (splits < 0 || splits > kMaxSplits) return set_error(OMNI_ERR_INVALID, "splits must be in [0, 16]");
  if (k % kBK != 0) return set_error(OMNI_ERR_UNSUPPORTED, "K must be a multiple of 64");
  if (n % kTileN != 0) return set_error(OMNI_ERR_UNSUPPORTED, "N must be a multiple of 128");
  auto mis16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (mis16(x) || mis16(w) || (x_stride % 8) != 0 || mis16(gp.y) || (gp.y_stride % 4) != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "operands must be 16-byte aligned with 16-byte row strides");
  if (epilogue == kEpiResidual && (gp.residual == nullptr || (gp.res_stride % 4) != 0 ||
                                   (reinterpret_cast<uintptr_t>(gp.residual) & 7) != 0))
    return set_error(OMNI_ERR_INVALID, "residual epilogue needs an 8-byte aligned residual");
  if (gp.ss_in && (gp.ss_in_parts <= 0 || gp.ss_in_parts > 64 || gp.norm_dim <= 0))
    return set_error(OMNI_ERR_INVALID, "ss_in needs 1..64 parts and norm_dim > 0");
  if (gp.ss_out && (epilogue == kEpiSwiGLU || epilogue == kEpiF32 || epilogue == kEpiQKV || epilogue == kEpiRouter))
    return set_error(OMNI_ERR_UNSUPPORTED, "ss_out is produced by the store and residual epilogues only");
  if (epilogue == kEpiQKV) {
    if (gp.head_dim != 64 && gp.head_dim != 128)
      return set_error(OMNI_ERR_UNSUPPORTED, "qkv epilogue supports head_dim 64 or 128");
    if (gp.hq <= 0 || gp.hkv <= 0 || (int64_t)(gp.hq + 2 * gp.hkv) * gp.head_dim != n)
      return set_error(OMNI_ERR_INVALID, "qkv epilogue: N must be (Hq + 2 Hkv) * head_dim");
    if ((gp.positions == nullptr) != (gp.cache_loc == nullptr))
      return set_error(OMNI_ERR_INVALID, "positions and cache_loc are given together");
    if (gp.positions == nullptr && (gp.tokens_per_req <= 0 || gp.slot_stride <= 0 || gp.slot_base < 0 ||
                                    gp.slot_base + gp.tokens_per_req > gp.max_pos))
      return set_error(OMNI_ERR_INVALID, "implicit slots need tokens_per_req, slot_stride > 0 within the rotary table");
    if (!gp.q_norm || !gp.k_norm || !gp.cos_sin || !gp.k_cache || !gp.v_cache)
      return set_error(OMNI_ERR_INVALID, "qkv epilogue needs norms, cos/sin table and caches");
  }
  if (epilogue == kEpiRouter &&
      (n != kTileN || gp.top_k < 1 || gp.top_k > 32 || gp.topk_ids == nullptr || gp.topk_w == nullptr))
    return set_error(OMNI_ERR_UNSUPPORTED, "router epilogue: 128 experts, 1 <= top_k <= 32, top-k outputs given");
  if (rows == 0) return OMNI_OK;
  if (splits > k / kBK) splits = (int)(k / kBK);
  switch (epilogue) {
    case kEpiStore: return launch_gemm<kEpiStore>(x, rows, k, x_stride, w, n, gp, splits, st);
    case kEpiResidual: return launch_gemm<kEpiResidual>(x, rows, k, x_stride, w, n, gp, splits, st);
    case kEpiSwiGLU: return launch_gemm<kEpiSwiGLU>(x, rows, k, x_stride, w, n, gp, splits, st);
    case kEpiQKV: return launch_gemm<kEpiQKV>(x, rows, k, x_stride, w, n, gp, splits, st);
    case kEpiRouter: return launch_gemm<kEpiRouter>(x, rows, k, x_stride, w, n, gp, splits, st);
    default: return launch_gemm<kEpiF32>(x, rows, k, x_stride, w, n, gp, splits, st);
  }
}

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int64_t omni_linear_workspace_bytes(int64_t rows, int64_t k, int64_t n, int32_t epilogue,
                                                        int32_t splits) {
  (void)rows, (void)k, (void)n, (void)epilogue, (void)splits;
  return 0;  // split-K partials go through the library's own L2-resident slab array
}

extern "C" OMNI_API int omni_linear(const void* x, int64_t rows, int64_t k, int64_t x_stride, const void* w,
                                    int64_t n, int32_t epilogue, const void* residual, int64_t residual_stride,
                                    void* y, int64_t y_stride, void* workspace, int64_t workspace_bytes_avail,
                                    int32_t splits, void* stream) {
  (void)workspace, (void)workspace_bytes_avail;
  if (epilogue == kEpiQKV || epilogue == kEpiRouter)
    return set_error(OMNI_ERR_INVALID, "the qkv and router epilogues are reached through omni_linear_fused");
  GemmParams gp{};
  gp.residual = static_cast<const uint16_t*>(residual);
  gp.res_stride = residual_stride;
  gp.y = y;
  gp.y_stride = y_stride;
  return run_linear(x, rows, k, x_stride, w, n, epilogue, gp, splits, static_cast<cudaStream_t>(stream));
}

extern "C" OMNI_API int omni_linear_fused(const OmniLinearArgs* a, void* stream) {
  if (a == nullptr) return set_error(OMNI_ERR_INVALID, "null arguments");
  GemmParams gp{};
  gp.residual = static_cast<const uint16_t*>(a->residual);
  gp.res_stride = a->residual_stride;
  gp.y = a->y;
  gp.y_stride = a->y_stride;
  gp.ss_in = a->ss_in;
  gp.ss_in_parts = a->ss_in_parts;
  gp.ss_in_stride = a->ss_in_stride;
  gp.norm_dim = a->norm_dim;
  gp.norm_eps = a->norm_eps;
  gp.ss_out = a->ss_out;
  gp.ss_out_stride = a->ss_out_stride;
  gp.hq = a->num_q_heads;
  gp.hkv = a->num_kv_heads;
  gp.head_dim = a->head_dim;
  gp.q_norm = static_cast<const uint16_t*>(a->q_norm);
  gp.k_norm = static_cast<const uint16_t*>(a->k_norm);
  gp.qk_eps = a->qk_eps;
  gp.cos_sin = a->cos_sin;
  gp.max_pos = a->max_position;
  gp.positions = a->positions;
  gp.cache_loc = a->cache_loc;
  gp.tokens_per_req = a->tokens_per_req;
  gp.slot_stride = a->slot_stride;
  gp.slot_base = a->slot_base;
  gp.k_cache = static_cast<uint16_t*>(a->k_cache);
  gp.v_cache = static_cast<uint16_t*>(a->v_cache);
  gp.topk_ids = a->topk_ids;
  gp.topk_w = a->topk_weights;
  gp.top_k = a->top_k;
  if (a->l2_prefetch != nullptr) {
    if ((reinterpret_cast<uintptr_t>(a->l2_prefetch) & 15) != 0 || a->l2_prefetch_bytes < 0)
      return set_error(OMNI_ERR_INVALID, "l2_prefetch must be 16-byte aligned with a non-negative size");
    gp.l2_prefetch = static_cast<const uint8_t*>(a->l2_prefetch);
    gp.l2_prefetch_bytes = a->l2_prefetch_bytes;
  }
  return run_linear(a->x, a->rows, a->k, a->x_stride, a->w, a->n, a->epilogue, gp, a->splits,
                    static_cast<cudaStream_t>(stream));
}

// Test hook: the store GEMM with a producer that issues no copies and waits
// bounded by wait_limit polls, so that every wait runs out.  The kernel must
// record kDevTimeoutTma (or kDevTimeoutMma) in the status word and return with
// nothing in flight; `y` is left unwritten.
extern "C" OMNI_API int omni_gemm_wait_probe(const void* x, int64_t rows, int64_t k, const void* w, int64_t n,
                                             void* y, int32_t splits, uint32_t wait_limit, void* stream) {
  if (wait_limit == 0) return set_error(OMNI_ERR_INVALID, "the probe needs a positive wait limit");
  GemmParams gp{};
  gp.y = y;
  gp.y_stride = n;
  gp.wait_limit = wait_limit;
  gp.withhold_loads = 1;
  return run_linear(x, rows, k, k, w, n, kEpiStore, gp, splits, static_cast<cudaStream_t>(stream));
}
