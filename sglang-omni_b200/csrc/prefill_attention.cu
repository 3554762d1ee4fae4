// Causal extend (prefill) attention over the paged KV pool on the 5th-generation
// tensor cores (RadixAttention extend, thinker_model.py:373-379; the extend rows of a
// mixed batch attend causally over their stream's pages, which the qkv epilogue has
// just written).
//
// Two kernels: prefill_attention_pair_kernel (below) when the query heads of a KV head
// come in pairs (a CTA serves two of them, each K / V tile loaded once for both), and
// prefill_attention_tc_kernel for an odd group size: CTA = 128 queries of one stream x
// one query head; the stream's keys go by in tiles of 128 (8 pages).  Ten warps:
//   warp 0    TMA producer: the Q tile once (two 64-column halves, 128B swizzle), then
//             per key tile the 8 pages of K and of V, one 16-row x 64-column box per
//             lane (32 lanes, 32 boxes), into a two-stage ring; pages past the stream
//             are loaded from beyond the pool (zero fill);
//   warp 1    MMA issuer (one elected lane), whichever is ready first: S_j = Q K_j^T
//             into one of two TMEM buffers (M 128 queries x N 128 keys, fp32), or
//             O += P_{j-1} V_{j-1} (issued as soon as P is written, so that the K/V
//             stage frees for the next load without waiting for the next tile's K)
//             (A = P from shared memory, K-major; B = V, MN-major: the key rows as they
//             sit in the pool are the K dimension, the head dimension the N one) --
//             the QK^T of a tile runs while the softmax works on the previous one;
//   warps 2-9 softmax, two threads per query row (TMEM lane; 64 columns each, the row
//             max and sum swapped through spare TMEM columns): P = exp2(s * scale *
//             log2 e - m) against the running max m in one pass over the tile (masking
//             only the tiles that cross the causal diagonal), written as bf16 into a
//             swizzled P buffer; the first tile, and a tile whose max passes m by more
//             than 2^8, rescale O and the running sum and write P again; at the end
//             O / sum goes to the output row.
// Every barrier wait is bounded; a wait that gives up records a status and ends the
// role's loop.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_util.h"
#include "common.cuh"

namespace omni {
namespace {

OMNI_DEFINE_STATUS(prefill_tc)

constexpr int kD = 128;
constexpr int kPage = 16;
constexpr int kRows = 128;                 // queries per CTA = TMEM lanes
constexpr int kKeys = 128;                 // keys per tile
constexpr int kHalfBytes = 128 * 128;      // [128 rows][64 bf16]
constexpr int kTileBytes = 2 * kHalfBytes;  // 32 KB
constexpr int kThreads = 320;  // TMA warp, MMA warp, 8 softmax warps
constexpr int kQOff = 0;
constexpr int kKVOff = kTileBytes;                       // stage s: K at + s*64K, V at + s*64K + 32K
constexpr int kPOff = kKVOff + 4 * kTileBytes;           // P buffer b at + b*32K
constexpr int kBarOff = kPOff + 2 * kTileBytes;          // 224 KB
constexpr size_t kSmemBytes = (size_t)kBarOff + 256 + 1024;  // + barriers + alignment slack
constexpr float kRescaleLog2 = 8.0f;

struct PrefillTcParams {
  const int32_t* qo_indptr;
  const int64_t* seq_lens;
  const int32_t* page_indptr;
  const int32_t* page_indices;
  const int32_t* tile_indptr;
  int streams, hq, hkv;
  int64_t num_slots;
  float scale_log2;
  uint16_t* out;
  int64_t out_stride;
};

struct Bars {
  uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], s_free[2], p_full[2], pv_done[2], drain, pair[4];
  uint32_t tmem;
};

// K-major / MN-major 128B-swizzle operand descriptors.  MN-major (the V operand):
// 64-element rows along N, 8-row groups along K 1024 B apart (SBO), the second
// 64 columns of N 16 KB away (LBO).
OMNI_DEVINL uint64_t desc_mn_sw128(const void* p) {
  uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= (uint64_t)(kHalfBytes >> 4) << 16;  // LBO: the next 64 elements of N
  d |= (uint64_t)(1024 >> 4) << 32;        // SBO: the next 8 rows of K
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

OMNI_DEVINL void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
OMNI_DEVINL void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
OMNI_DEVINL void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 2^x by the PTX ex2.approx instruction (flush-to-zero; 2^-inf = +0).
OMNI_DEVINL float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// (query tile, head slot) of this CTA; false when the grid holds more CTAs than
// tiles.  CTAs start in grid order (x fastest), and a causal tile's key count
// grows toward its stream's end, so the walk goes from the last tile back with
// all head slots of a tile side by side: the long tiles start first and the
// last wave holds short ones (on the 16 prompts of 64..4096 rows this takes the
// modelled makespan from 8.6% over the even split to 1.9%).
OMNI_DEVINL bool block_work(const PrefillTcParams& p, int& tile, int& head) {
  const int total = p.tile_indptr[p.streams];
  const int heads = (int)gridDim.y;
  const int w = (int)(blockIdx.y * gridDim.x + blockIdx.x);
  if (w >= total * heads) return false;
  tile = total - 1 - w / heads;
  head = w % heads;
  return true;
}

__global__ void __launch_bounds__(kThreads, 1) prefill_attention_tc_kernel(
    const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
    const __grid_constant__ CUtensorMap tv, const __grid_constant__ PrefillTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();
  griddep_launch();
  int tile, hh;
  if (!block_work(p, tile, hh)) return;
  int lo = 0, hi = p.streams - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.tile_indptr[mid] <= tile) lo = mid;
    else hi = mid - 1;
  }
  const int st = lo;
  const int qs0 = p.qo_indptr[st], ext = p.qo_indptr[st + 1] - qs0;
  const int64_t seq_len = p.seq_lens[st];
  const int prefix = (int)(seq_len - ext);
  const int q0 = (tile - p.tile_indptr[st]) * kRows;  // first query of the tile (within the extend)
  const int nq = min(kRows, ext - q0);
  const int kvh = hh / (p.hq / p.hkv);
  const int pg0 = p.page_indptr[st], npages = p.page_indptr[st + 1] - pg0;
  const int nt = (prefix + q0 + nq + kKeys - 1) / kKeys;  // key tiles the tile needs

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->kv_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 8 * 32);
      mbar_init(&bars->p_full[i], 8 * 32);
      mbar_init(&bars->pv_done[i], 1);
    }
    mbar_init(&bars->drain, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&bars->pair[i], 64);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem;
  const uint32_t tO = tbase + 256;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_arrive_expect_tx(&bars->q_full, kTileBytes);
    }
    __syncwarp();
    if (lane < 2) tma_load_2d(smem + kQOff + lane * kHalfBytes, &tq, &bars->q_full, hh * kD + lane * 64, qs0 + q0);
    for (int j = 0; j < nt; ++j) {
      const int s = j & 1;
      if (j >= 2 && !mbar_wait(&bars->kv_empty[s], ((j - 2) >> 1) & 1)) {
        report_status(kDevTimeoutTma);
        break;
      }
      if (lane == 0) mbar_arrive_expect_tx(&bars->kv_full[s], 2 * kTileBytes);
      __syncwarp();
      const int idx = lane & 15, pg = idx >> 1, half = idx & 1;
      const int pgl = j * (kKeys / kPage) + pg;
      const int64_t y = pgl < npages ? (int64_t)p.page_indices[pg0 + pgl] * kPage : p.num_slots;
      uint8_t* dst = smem + kKVOff + s * 2 * kTileBytes + (lane < 16 ? 0 : kTileBytes) + half * kHalfBytes +
                     pg * kPage * 128;
      tma_load_2d(dst, lane < 16 ? (const void*)&tk : (const void*)&tv, &bars->kv_full[s], kvh * kD + half * 64,
                  (int)y);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const bool leader = elect_one();
    const uint32_t idesc_qk = idesc_bf16_f32(kRows, kKeys);
    const uint32_t idesc_pv = idesc_bf16_f32(kRows, kD) | (1u << 16);  // B MN-major
    bool ok = mbar_wait(&bars->q_full, 0);
    // Issue whichever MMA is ready: the P V of tile ip as soon as its P is written
    // (its completion frees the K/V stage for the next load), the QK^T of tile jq as
    // soon as its K has landed and its S buffer is free.  Lane 0 polls, the warp
    // follows its decision.
    auto ready = [&](uint64_t* bar, uint32_t parity) -> bool {
      uint32_t r = lane == 0 ? (mbar_test_wait(bar, parity) ? 1u : 0u) : 0u;
      return __shfl_sync(0xFFFFFFFFu, r, 0) != 0;
    };
    int jq = 0, ip = 0;
    uint32_t idle = 0;
    while (ok && ip < nt) {
      bool progressed = false;
      if (ip < jq && ready(&bars->p_full[ip & 1], (ip >> 1) & 1)) {
        const int s = ip & 1;
        tc_fence_after();
        if (leader) {
          const uint8_t* pt = smem + kPOff + s * kTileBytes;
          const uint8_t* vt = smem + kKVOff + s * 2 * kTileBytes + kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint64_t ad = smem_desc_sw128(pt + (k >> 2) * kHalfBytes) + 2 * (k & 3);
            const uint64_t bd = desc_mn_sw128(vt + k * 16 * 128);
            tc_mma_bf16(tO, ad, bd, idesc_pv, (ip > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&bars->pv_done[s]);
          tc_commit(&bars->kv_empty[s]);
        }
        __syncwarp();
        ++ip;
        progressed = true;
      }
      if (jq < nt && jq <= ip + 1 && ready(&bars->kv_full[jq & 1], (jq >> 1) & 1) &&
          (jq < 2 || ready(&bars->s_free[jq & 1], ((jq - 2) >> 1) & 1))) {
        const int s = jq & 1;
        tc_fence_after();
        if (leader) {
          const uint8_t* kt = smem + kKVOff + s * 2 * kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint64_t ad = smem_desc_sw128(smem + kQOff + (k >> 2) * kHalfBytes) + 2 * (k & 3);
            const uint64_t bd = smem_desc_sw128(kt + (k >> 2) * kHalfBytes) + 2 * (k & 3);
            tc_mma_bf16(tbase + s * 128, ad, bd, idesc_qk, k > 0 ? 1u : 0u);
          }
          tc_commit(&bars->s_full[s]);
        }
        __syncwarp();
        ++jq;
        progressed = true;
      }
      if (progressed) idle = 0;
      else if (++idle > 4 * kWaitLimit) ok = false;
    }
    if (!ok) report_status(kDevTimeoutMma);
    // every MMA of this warp has completed before the TMEM is freed
    if (leader) tc_commit(&bars->drain);
    __syncwarp();
    mbar_wait(&bars->drain, 0);
  } else {
    // ---------------- softmax: two threads per query row ----------------
    // warps 2-5 take columns 0-63 of S, O and P, warps 6-9 columns 64-127, of the
    // rows of their TMEM lane quarter; the two threads of a row swap their maxima
    // (and at the end their sums) through two spare TMEM columns of the row.
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int hc = (warp - 2) >> 2;         // column half
    const int r = q * 32 + lane;            // query row of the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t txch = tbase + lane_off + 384;  // exchange columns 384 .. 389
    const int lim = prefix + q0 + r;        // last key this query sees
    const float sl = p.scale_log2;
    float m_use = -INFINITY, l = 0.0f;
    bool ok = true;
    uint32_t pair_phase = 0;
    // this thread's value and its partner's, through the row's TMEM exchange columns
    auto swap = [&](float mine, int slot) -> float {
      uint32_t v1[1] = {__float_as_uint(mine)};
      asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(txch + slot * 2 + hc), "r"(v1[0])
                   : "memory");
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&bars->pair[q]);
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars->pair[q], pair_phase & 1))) ok = false;
      ++pair_phase;
      tc_fence_after();
      uint32_t o1;
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(o1) : "r"(txch + slot * 2 + (hc ^ 1))
                   : "memory");
      tc_wait_ld();
      return __uint_as_float(o1);
    };
    // P = exp2(s * scale - m_use) for this thread's 64 keys of tile j into its half of
    // the swizzled P buffer (masked keys 0); returns their sum and raw max score
    // (key pairs by the packed fp32x2 forms, as in the pair kernel)
    auto write_p = [&](uint32_t ts, uint8_t* phalf, int j, bool masked, float& mx) -> float {
      const uint64_t sl2 = f2_make(sl, sl), nm2 = f2_make(-m_use, -m_use);
      uint64_t rs2 = f2_make(0.0f, 0.0f);
      mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(ts + c * 32, v);
        tc_wait_ld();
        const int k0 = j * kKeys + hc * 64 + c * 32;
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float a = __uint_as_float(v[e]), b = __uint_as_float(v[e + 1]);
          if (masked) {
            a = k0 + e <= lim ? a : -INFINITY;
            b = k0 + e + 1 <= lim ? b : -INFINITY;
          }
          mx = fmax3(mx, a, b);
          float ta, tb;
          f2_split(f2_fma(f2_make(a, b), sl2, nm2), ta, tb);
          const uint64_t pp = f2_make(ex2_approx(ta), ex2_approx(tb));
          rs2 = f2_add(rs2, pp);
          pk[e >> 1] = f2_to_bf2(pp);
        }
        // keys hc*64 + c*32 .. + 31: 16-byte chunks c*4 .. c*4+3 of the row in half hc
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int chunk = c * 4 + u;
          uint8_t* dst = phalf + ((chunk ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      float ra, rb;
      f2_split(rs2, ra, rb);
      return ra + rb;
    };
    for (int j = 0; j < nt && ok; ++j) {
      const int s = j & 1;
      // (every branch of this loop is warp-uniform: the tcgen05.ld / st are
      // warp-collective)
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars->s_full[s], (j >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ts = tbase + lane_off + s * 128 + hc * 64;
      // the P buffer of tile j - 2 is free once its P V has completed
      if (j >= 2 && !__all_sync(0xFFFFFFFFu, mbar_wait(&bars->pv_done[s], ((j - 2) >> 1) & 1))) {
        ok = false;
        break;
      }
      uint8_t* phalf = smem + kPOff + s * kTileBytes + hc * kHalfBytes + r * 128;
      // every key of the tile is visible to every query of the CTA: no mask
      const bool masked = j * kKeys + kKeys - 1 > prefix + q0;
      float mx;
      // one pass against the running max; the rare tile whose max passes it by more
      // than 2^8 (and the first tile) rescales O and the sum and writes P again
      float rs = 0.0f;
      if (j == 0) {  // m_use is -inf on every row until tile 0 (key 0 is visible to all rows)
        mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(ts + c * 32, v);
          tc_wait_ld();
          const int k0 = j * kKeys + hc * 64 + c * 32;
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (!masked || k0 + e <= lim) mx = fmaxf(mx, __uint_as_float(v[e]));
        }
      } else {
        rs = write_p(ts, phalf, j, masked, mx);
      }
      mx = fmaxf(mx, swap(mx, j & 1));  // the row's max over both halves
      if (!ok) break;
      const float m_tile = mx == -INFINITY ? -INFINITY : mx * sl;
      const bool resc = m_tile != -INFINITY && (m_use == -INFINITY || m_tile > m_use + kRescaleLog2);
      // the warp rescales if any of its rows must (the others with alpha = 1 and their
      // running max kept, which rewrites the same P); both threads of a row scale their
      // O columns, whatever their own half of the sum
      if (__any_sync(0xFFFFFFFFu, resc)) {
        const float alpha = !resc ? 1.0f : m_use == -INFINITY ? 0.0f : ex2_approx(m_use - m_tile);
        if (j > 0) {
          // O holds tiles < j once the previous P V has completed
          if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars->pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tO + lane_off + hc * 64 + c * 32, v);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            tmem_st_32x32b_x32(tO + lane_off + hc * 64 + c * 32, v);
          }
          tc_wait_st();
        }
        l *= alpha;
        if (resc) m_use = m_tile;
        float unused;
        rs = write_p(ts, phalf, j, masked, unused);
      }
      l += rs;
      tc_fence_before();
      mbar_arrive(&bars->s_free[s]);
      fence_proxy_async();  // the P stores, visible to the tensor core
      mbar_arrive(&bars->p_full[s]);
    }
    const float l_row = ok ? l + swap(l, 2) : 0.0f;
    if (ok && nt > 0 && __all_sync(0xFFFFFFFFu, mbar_wait(&bars->pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1))) {
      tc_fence_after();
      const float inv = l_row > 0.0f ? 1.0f / l_row : 0.0f;
      uint16_t* orow = p.out + (int64_t)(qs0 + q0 + r) * p.out_stride + (int64_t)hh * kD + hc * 64;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tO + lane_off + hc * 64 + c * 32, v);
        tc_wait_ld();
        if (r < nq) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            pk[e >> 1] = pack_bf2(__uint_as_float(v[e]) * inv, __uint_as_float(v[e + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int u = 0; u < 4; ++u) dst[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
    } else if (nt > 0) {
      report_status(kDevTimeoutMma);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ---------------------------------------------------------------------------
// GQA pair kernel: CTA = 128 queries of one stream x two query heads of one KV
// head, so each K / V tile is loaded once for both heads; keys go by in tiles of 64
// (4 pages).  TMEM (512 columns): each head's Q (64 columns, bf16 pairs), its S
// buffer (64), its O accumulator (128).  Q sits in TMEM as the A operand of S, so an S
// k-step reads only K from shared memory: with Q from shared memory as well, the
// operands of an N = 64 S k-step wanted about 192 B/cycle and the MMAs, not the
// softmax, set the pace (an MMA warp blocked in issue for most of each round).  With
// one S buffer a head the heads take turns on the tensor core: the head-1 softmax runs
// on S_1(j) while the tensor core does P_0 V(j) and S_0(j + 1), and the other way round.
// Ten warps:
//   warp 0    TMA producer: both heads' Q tiles once; per key tile the 4 pages of K
//             and of V (one 16-row x 64-column box per lane) into three-slot K and V
//             rings;
//   warp 1    MMA issuer, in a fixed order: S_0(0), S_1(0), then per tile i
//             P_0 V(i), S_0(i + 1), P_1 V(i), S_1(i + 1); each half of a P V once the
//             head's softmax has written that half of P(i), after V(i) and K(i + 1)
//             have landed;
//             P_h(i) sits over the first 32 of the head's S columns, and S_h(i + 1) is
//             issued after P_h V(i), which reads it first (MMAs execute in order);
//   warps 2-5 softmax of head 0, warps 6-9 of head 1: first copy their row of Q from
//             the swizzled shared tile into TMEM; then per tile one thread per query
//             row (TMEM lane) over the 64 columns, so a row's max and sum stay in one
//             thread: the tile's max first; the first tile and a tile whose max passes
//             the running max m by more than 2^8 rescale O and the running sum (the
//             whole warp when any of its rows must: the tcgen05.ld / st are
//             warp-collective; the other rows keep their max, alpha = 1); then P =
//             exp2(s * scale * log2 e - m) 32 keys at a time, each half written over
//             the S columns just read and handed to the MMA warp at once, so that its
//             two P V k-steps run under the next half (13 % on the kernel against one
//             hand-off a tile).  The completion of S_h(j) covers every MMA issued
//             before it, P_h V(j - 1) included, so the softmax never waits for P V
//             inside the loop.  One barrier arrival a warp.
// Shared memory: Q 2 x 32 KB (read once into TMEM), K and V rings 3 x 16 KB each
// (160 KB).  History at config 2 (TFLOP/s of causal QK^T + PV): one head a CTA with
// 128-key tiles 409; two heads with 128-key tiles (one S buffer a head, softmax and MMAs
// not overlapped) 495; 64-key tiles with two S buffers a head and Q in shared memory
// 507; the MMA warp polling eight barriers in one ballot and sleeping between idle
// rounds 559; P in TMEM 573; the softmax's key pairs on the packed fp32x2 forms with a
// 3-input max and the bf16 pack by Veltkamp splitting 596; CTAs walking the tiles
// heaviest-first (block_work) 623-642; the second head's P V interleaved with the first
// head's S and one arrival a warp 633-672; Q in TMEM with the heads taking turns
// (this layout) 697-702; P handed over in halves 851.  Measured slower: a polynomial exp2 on the FMA pipe for 4 to 16 of
// every 32 keys (933-1 049 against 882 us; again with the packed forms, on the MMA
// warp's sub-partition only: 10-13 % slower), twelve warps with setmaxnreg, lane 0
// waiting for its warp (14 % slower than every thread polling), the page table read
// one tile ahead (no change), the MMA warp testing four barriers with one lane instead
// of eight with eight (no change).
// ---------------------------------------------------------------------------
constexpr int kPKeys = 64;                              // keys per tile
constexpr int kPHalf = kPKeys * 128;                    // [64 keys][64 bf16]: 8 KB
constexpr int kPTile = 2 * kPHalf;                      // a K or V tile: 16 KB
constexpr int kPSlots = 3;
constexpr int kPairQOff = 0;                            // head h: + h * 32 KB
constexpr int kPairKOff = 2 * kTileBytes;               // slot s: + s * 16 KB
constexpr int kPairVOff = kPairKOff + kPSlots * kPTile;
constexpr int kPairBarOff = kPairVOff + kPSlots * kPTile;  // 160 KB
constexpr size_t kPairSmemBytes = (size_t)kPairBarOff + 512 + 1024;

// D[tmem] (+)= A[tmem] * B[smem], kind::f16: the A operand (here P, bf16 packed two
// to a 32-bit column, M rows on the TMEM lanes) read from tensor memory.
OMNI_DEVINL void tc_mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}

struct PairBars {
  uint64_t q_full, q_tmem, k_full[kPSlots], k_empty[kPSlots], v_full[kPSlots], v_empty[kPSlots];
  uint64_t s_full[2], p_full[2][2], pv_done[2], drain;
  uint32_t tmem;
};

// MN-major 128B-swizzle descriptor of a V tile of 64 keys: 64-element rows along N
// (the head dimension), 8-row groups along K 1024 B apart, the second 64 columns of N
// one 8 KB half away.
OMNI_DEVINL uint64_t desc_mn_sw128_64(const void* p) {
  uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= (uint64_t)(kPHalf >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__global__ void __launch_bounds__(kThreads, 1) prefill_attention_pair_kernel(
    const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
    const __grid_constant__ CUtensorMap tv, const __grid_constant__ PrefillTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + kPairBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();
  griddep_launch();
  int tile, pair;
  if (!block_work(p, tile, pair)) return;
  const int h0 = 2 * pair;  // query heads h0, h0 + 1
  int lo = 0, hi = p.streams - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.tile_indptr[mid] <= tile) lo = mid;
    else hi = mid - 1;
  }
  const int st = lo;
  const int qs0 = p.qo_indptr[st], ext = p.qo_indptr[st + 1] - qs0;
  const int64_t seq_len = p.seq_lens[st];
  const int prefix = (int)(seq_len - ext);
  const int q0 = (tile - p.tile_indptr[st]) * kRows;
  const int nq = min(kRows, ext - q0);
  const int kvh = h0 / (p.hq / p.hkv);
  const int pg0 = p.page_indptr[st], npages = p.page_indptr[st + 1] - pg0;
  const int nt = (prefix + q0 + nq + kPKeys - 1) / kPKeys;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_tmem, 8);  // one arrival per softmax warp
    for (int i = 0; i < kPSlots; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&bars->s_full[h], 1);
      mbar_init(&bars->p_full[h][0], 4);  // one arrival per softmax warp of the head
      mbar_init(&bars->p_full[h][1], 4);
      mbar_init(&bars->pv_done[h], 1);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_arrive_expect_tx(&bars->q_full, 2 * kTileBytes);
    }
    __syncwarp();
    if (lane < 4)
      tma_load_2d(smem + kPairQOff + (lane >> 1) * kTileBytes + (lane & 1) * kHalfBytes, &tq, &bars->q_full,
                  (h0 + (lane >> 1)) * kD + (lane & 1) * 64, qs0 + q0);
    const int pg = lane >> 1, half = lane & 1;  // lanes 0-7: page pg of the tile, head-dim half
    auto load_tile = [&](const void* map, uint8_t* base, uint64_t* bar, int j) {
      if (lane == 0) mbar_arrive_expect_tx(bar, kPTile);
      __syncwarp();
      if (lane < 8) {
        const int pgl = j * (kPKeys / kPage) + pg;
        const int64_t y = pgl < npages ? (int64_t)p.page_indices[pg0 + pgl] * kPage : p.num_slots;
        tma_load_2d(base + half * kPHalf + pg * kPage * 128, map, bar, kvh * kD + half * 64, (int)y);
      }
    };
    for (int j = 0; j < nt; ++j) {
      const int s = j % kPSlots;
      const uint32_t par = ((j / kPSlots) - 1) & 1;
      if (j >= kPSlots && !mbar_wait(&bars->k_empty[s], par)) {
        report_status(kDevTimeoutTma);
        break;
      }
      load_tile(&tk, smem + kPairKOff + s * kPTile, &bars->k_full[s], j);
      if (j >= kPSlots && !mbar_wait(&bars->v_empty[s], par)) {
        report_status(kDevTimeoutTma);
        break;
      }
      load_tile(&tv, smem + kPairVOff + s * kPTile, &bars->v_full[s], j);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: P_0 V(i), S_0(i + 1), P_1 V(i), S_1(i + 1), ... ----------------
    const bool leader = elect_one();
    const uint32_t idesc_qk = idesc_bf16_f32(kRows, kPKeys);
    const uint32_t idesc_pv = idesc_bf16_f32(kRows, kD) | (1u << 16);  // B MN-major
    // S_h(j) = Q_h K_j^T: A = head h's Q from TMEM (columns h * 64, 8 a k-step of 16
    // dimensions), B = K_j from shared memory, into head h's S columns 128 + h * 64
    // (descriptors from one base a tile plus constant offsets, computed by the whole
    // warp: the elected lane only issues)
    auto issue_s = [&](int h, int j) {
      const int s = j % kPSlots;
      const uint64_t kd = smem_desc_sw128(smem + kPairKOff + s * kPTile);
      const uint32_t ta = tbase + h * 64, td = tbase + 128 + h * 64;
      if (leader) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          tc_mma_bf16_ts(td, ta + k * 8, kd + (uint64_t)(((k >> 2) * kPHalf) >> 4) + 2 * (k & 3), idesc_qk,
                         k > 0 ? 1u : 0u);
        tc_commit(&bars->s_full[h]);
        if (h == 1) tc_commit(&bars->k_empty[s]);  // both heads' S of tile j
      }
      __syncwarp();
    };
    // O_h += P_h(i) V_i, keys 32 * half .. + 31 (k-steps 2 * half, 2 * half + 1): A = P_h(i)
    // over the first 32 of the head's S columns, 16 keys a k-step
    auto issue_pv = [&](int h, int i, int half) {
      const int s = i % kPSlots;
      const uint64_t vd = desc_mn_sw128_64(smem + kPairVOff + s * kPTile);
      const uint32_t ta = tbase + 128 + h * 64, td = tbase + 256 + h * 128;
      if (leader) {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int k = 2 * half + kk;  // 16 rows of V, 2 KB on
          tc_mma_bf16_ts(td, ta + k * 8, vd + (uint64_t)((k * 16 * 128) >> 4), idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
        }
        if (half == 1 && i == nt - 1) tc_commit(&bars->pv_done[h]);
        if (half == 1 && h == 1) tc_commit(&bars->v_empty[s]);  // both heads' P V of tile i
      }
      __syncwarp();
    };
    bool ok = mbar_wait(&bars->q_tmem, 0) && (nt == 0 || mbar_wait(&bars->k_full[0], 0));
    if (ok && nt > 0) {
      tc_fence_after();
      issue_s(0, 0);
      issue_s(1, 0);
    }
    for (int i = 0; i < nt && ok; ++i) {
      // V(i) and K(i + 1) land long before the softmax has written P(i) (their loads
      // wait only for MMAs issued rounds ago): wait for them first, so that P V and
      // S go out the moment P is in
      if (!mbar_wait(&bars->v_full[i % kPSlots], (i / kPSlots) & 1) ||
          (i + 1 < nt && !mbar_wait(&bars->k_full[(i + 1) % kPSlots], ((i + 1) / kPSlots) & 1))) {
        ok = false;
        break;
      }
      for (int h = 0; h < 2 && ok; ++h) {
        // each half of P_h(i) once the head's four softmax warps have written it (the
        // first half after S_h(i) has been read)
        for (int half = 0; half < 2; ++half) {
          if (!mbar_wait(&bars->p_full[h][half], i & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(h, i, half);
        }
        // after P_h V(i) in issue order, so P_h(i) is read before S_h(i + 1) overwrites it
        if (ok && i + 1 < nt) issue_s(h, i + 1);
      }
    }
    if (!ok) report_status(kDevTimeoutMma);
    if (leader) tc_commit(&bars->drain);
    __syncwarp();
    mbar_wait(&bars->drain, 0);
  } else {
    // ---------------- softmax: one thread per query row of one head ----------------
    const int h = (warp - 2) >> 2;          // head of this warpgroup
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int r = q * 32 + lane;            // query row of the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t tQ = tbase + lane_off + h * 64;
    const uint32_t tS = tbase + lane_off + 128 + h * 64;
    const uint32_t tO = tbase + lane_off + 256 + h * 128;
    const int lim = prefix + q0 + r;        // last key this query sees
    const float sl = p.scale_log2;
    float m_use = -INFINITY, l = 0.0f;
    // this row's Q (bf16 pairs, the dimensions in order) from the swizzled shared tile
    // into the head's Q columns of TMEM, the A operand of every S
    bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&bars->q_full, 0));
    if (ok) {
      const uint8_t* qrow = smem + kPairQOff + h * kTileBytes + r * 128;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t v[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 x = *reinterpret_cast<const uint4*>(qrow + hf * kHalfBytes + ((c ^ (r & 7)) << 4));
          v[4 * c] = x.x;
          v[4 * c + 1] = x.y;
          v[4 * c + 2] = x.z;
          v[4 * c + 3] = x.w;
        }
        tmem_st_32x32b_x32(tQ + hf * 32, v);
      }
      tc_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->q_tmem);
    for (int j = 0; j < nt && ok; ++j) {
      // (every branch of this loop is warp-uniform: the tcgen05.ld / st below are
      // warp-collective)
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&bars->s_full[h], j & 1))) {
        ok = false;
        break;
      }
      // S_h(j) has completed, and with it every MMA issued before it: the head's
      // P V(j - 1) too, so O holds tiles < j and P(j - 1) has been read
      tc_fence_after();
      const bool masked = j * kPKeys + kPKeys - 1 > prefix + q0;
      // the row's 64 scores (keys past the diagonal -inf), and their max first
      uint32_t vv[2][32];
      tmem_ld_32x32b_x32(tS, vv[0]);
      tmem_ld_32x32b_x32(tS + 32, vv[1]);
      tc_wait_ld();
      if (masked) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (j * kPKeys + c * 32 + e > lim) vv[c][e] = __float_as_uint(-INFINITY);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 2) mx = fmax3(mx, __uint_as_float(vv[c][e]), __uint_as_float(vv[c][e + 1]));
      const float m_tile = mx == -INFINITY ? -INFINITY : mx * sl;
      const bool resc = m_tile != -INFINITY && (m_use == -INFINITY || m_tile > m_use + kRescaleLog2);
      // the warp rescales if any of its rows must (the others with alpha = 1 and their
      // running max kept)
      if (__any_sync(0xFFFFFFFFu, resc)) {
        const float alpha = !resc ? 1.0f : m_use == -INFINITY ? 0.0f : ex2_approx(m_use - m_tile);
        if (__any_sync(0xFFFFFFFFu, resc && j > 0 && l > 0.0f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tO + c * 32, v);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            tmem_st_32x32b_x32(tO + c * 32, v);
          }
          tc_wait_st();
        }
        l *= alpha;
        if (resc) m_use = m_tile;
      }
      // P = exp2(s * scale - m_use), 32 keys at a time over the S columns just read
      // (bf16 pairs: 16 columns a half), each half handed to the MMA warp as soon as
      // it is written so that its P V k-steps run under the next half.  Key pairs go
      // through the packed fp32x2 forms: one FMA for both arguments, one add into a
      // two-lane row sum and a 4-instruction bf16 pack.
      const uint64_t sl2 = f2_make(sl, sl), nm2 = f2_make(-m_use, -m_use);
      uint64_t rs2 = f2_make(0.0f, 0.0f);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float ta, tb;
          f2_split(f2_fma(f2_make(__uint_as_float(vv[c][e]), __uint_as_float(vv[c][e + 1])), sl2, nm2), ta, tb);
          const uint64_t pp = f2_make(ex2_approx(ta), ex2_approx(tb));
          rs2 = f2_add(rs2, pp);
          pk[e >> 1] = f2_to_bf2(pp);
        }
        tmem_st_32x32b_x16(tS + c * 16, pk);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[h][c]);  // one arrival a warp
      }
      float ra, rb;
      f2_split(rs2, ra, rb);
      l += ra + rb;
    }
    if (ok && nt > 0 && __all_sync(0xFFFFFFFFu, mbar_wait(&bars->pv_done[h], 0))) {
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      uint16_t* orow = p.out + (int64_t)(qs0 + q0 + r) * p.out_stride + (int64_t)(h0 + h) * kD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tO + c * 32, v);
        tc_wait_ld();
        if (r < nq) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            pk[e >> 1] = pack_bf2(__uint_as_float(v[e]) * inv, __uint_as_float(v[e + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int u = 0; u < 4; ++u) dst[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
    } else if (nt > 0) {
      report_status(kDevTimeoutMma);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// bf16 [rows, cols] with row stride (elements), box {64, box_rows}, 128B swizzle.
bool tmap_2d(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t stride, int box_rows) {
  auto fn = encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int omni_prefill_attention(const void* q, int64_t q_stride, int64_t q_rows, const void* k_cache,
                                              const void* v_cache, int64_t num_slots, const int32_t* qo_indptr,
                                              const int64_t* seq_lens, const int32_t* page_indptr,
                                              const int32_t* page_indices, const int32_t* tile_indptr,
                                              int64_t streams, int64_t max_tiles, int32_t num_q_heads,
                                              int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                              float sm_scale, void* out, int64_t out_stride, void* stream) {
  if (streams < 0 || max_tiles < 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || q_rows < 0 ||
      num_slots <= 0)
    return set_error(OMNI_ERR_INVALID, "bad prefill attention shape");
  if (head_dim != kD || page_size != kPage)
    return set_error(OMNI_ERR_UNSUPPORTED, "prefill attention supports head_dim 128 and pages of 16");
  if ((reinterpret_cast<uintptr_t>(q) & 15) || q_stride % 8 || (reinterpret_cast<uintptr_t>(out) & 15) ||
      out_stride % 8 || (reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
    return set_error(OMNI_ERR_UNSUPPORTED, "misaligned prefill attention operands");
  if (streams == 0 || max_tiles == 0 || q_rows == 0) return OMNI_OK;
  CUtensorMap tq, tk, tv;
  const int64_t kv_cols = (int64_t)num_kv_heads * kD;
  if (!tmap_2d(&tq, q, q_rows, (int64_t)num_q_heads * kD, q_stride, kRows) ||
      !tmap_2d(&tk, k_cache, num_slots, kv_cols, kv_cols, kPage) ||
      !tmap_2d(&tv, v_cache, num_slots, kv_cols, kv_cols, kPage))
    return set_error(OMNI_ERR_UNSUPPORTED, "tensor map encoding failed");
  PrefillTcParams p{};
  p.qo_indptr = qo_indptr;
  p.seq_lens = seq_lens;
  p.page_indptr = page_indptr;
  p.page_indices = page_indices;
  p.tile_indptr = tile_indptr;
  p.streams = (int)streams;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.num_slots = num_slots;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.out = static_cast<uint16_t*>(out);
  p.out_stride = out_stride;
  if ((num_q_heads / num_kv_heads) % 2 == 0) {
    // two query heads of one KV head a CTA
    const cudaError_t ae =
        once_per_device(reinterpret_cast<const void*>(prefill_attention_pair_kernel), kAttrSmem, [] {
          return cudaFuncSetAttribute(prefill_attention_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kPairSmemBytes);
        });
    if (ae != cudaSuccess) return check_launch(ae);
    return check_launch(launch(prefill_attention_pair_kernel,
                               dim3((unsigned)max_tiles, (unsigned)(num_q_heads / 2)), dim3(kThreads), kPairSmemBytes,
                               static_cast<cudaStream_t>(stream), tq, tk, tv, p));
  }
  const cudaError_t ae = once_per_device(reinterpret_cast<const void*>(prefill_attention_tc_kernel), kAttrSmem, [] {
    return cudaFuncSetAttribute(prefill_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kSmemBytes);
  });
  if (ae != cudaSuccess) return check_launch(ae);
  return check_launch(launch(prefill_attention_tc_kernel, dim3((unsigned)max_tiles, (unsigned)num_q_heads),
                             dim3(kThreads), kSmemBytes, static_cast<cudaStream_t>(stream), tq, tk, tv, p));
}
