// Sampling kernels of the talker decode step: the residual-codebook sampler
// fused with its embedding gather (K6/K7/K9/K10) and the layer-0 codec sampler
// (a11).  One CTA of 256 threads per row; the row's logits are read once with
// 16-byte vector loads, the top-k set is found by an MSB-first radix select on
// order-preserving 32-bit keys, and the post-selection softmax / top-p /
// Gumbel-max runs in one warp.
//
// Floating-point specification shared with the CPU oracle (bit-exact parity):
// exp/log are this file's own functions (Cody–Waite + Taylor for exp, the
// atanh series for log, f32 and f64), every multiply-add is an explicit
// round-to-nearest intrinsic, and every reduction has the fixed order stated
// at its definition.
#include "common.cuh"
#include "capi_util.h"
#include "detmath.cuh"

namespace omni {
namespace {
OMNI_DEFINE_STATUS(sampling)

// ---------------------------------------------------------------------------
// Deterministic elementary functions (det_expf in detmath.cuh).
// ---------------------------------------------------------------------------
OMNI_DEVINL float det_logf(float x) {
  if (x != x) return x;
  if (x < 0.0f) return __uint_as_float(0x7FC00000u);
  if (x == 0.0f) return __uint_as_float(0xFF800000u);
  if (x == __uint_as_float(0x7F800000u)) return x;
  uint32_t u = __float_as_uint(x);
  int e = 0;
  if ((u & 0x7F800000u) == 0) {
    x = __fmul_rn(x, 8388608.0f);
    u = __float_as_uint(x);
    e = -23;
  }
  e += (int)((u >> 23) & 0xFF) - 127;
  float m = __uint_as_float((u & 0x007FFFFFu) | 0x3F800000u);
  if (m > 0x1.6a09e6p+0f) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  float s2 = __fmul_rn(s, s);
  float q = 0x1.c71c72p-3f;
  q = __fmaf_rn(q, s2, 0x1.24924ap-2f);
  q = __fmaf_rn(q, s2, 0x1.99999ap-2f);
  q = __fmaf_rn(q, s2, 0x1.555556p-1f);
  float lm = __fmaf_rn(__fmul_rn(s, s2), q, __fmul_rn(2.0f, s));
  float fe = (float)e;
  return __fmaf_rn(fe, 0x1.62e4p-1f, __fmaf_rn(fe, 0x1.7f7d1cp-20f, lm));
}

OMNI_DEVINL double det_log(double x) {
  if (x != x) return x;
  if (x < 0.0) return __longlong_as_double(0x7FF8000000000000ll);
  if (x == 0.0) return __longlong_as_double((long long)0xFFF0000000000000ull);
  if (x == __longlong_as_double(0x7FF0000000000000ll)) return x;
  uint64_t u = (uint64_t)__double_as_longlong(x);
  int e = 0;
  if ((u & 0x7FF0000000000000ull) == 0) {
    x = __dmul_rn(x, 18014398509481984.0);
    u = (uint64_t)__double_as_longlong(x);
    e = -54;
  }
  e += (int)((u >> 52) & 0x7FF) - 1023;
  double m = __longlong_as_double((long long)((u & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull));
  if (m > 0x1.6a09e667f3bcdp+0) {
    m = __dmul_rn(m, 0.5);
    e += 1;
  }
  double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
  double s2 = __dmul_rn(s, s);
  double q = 0x1.47ae147ae147bp-4;
  q = __fma_rn(q, s2, 0x1.642c8590b2164p-4);
  q = __fma_rn(q, s2, 0x1.8618618618618p-4);
  q = __fma_rn(q, s2, 0x1.af286bca1af28p-4);
  q = __fma_rn(q, s2, 0x1.e1e1e1e1e1e1ep-4);
  q = __fma_rn(q, s2, 0x1.1111111111111p-3);
  q = __fma_rn(q, s2, 0x1.3b13b13b13b14p-3);
  q = __fma_rn(q, s2, 0x1.745d1745d1746p-3);
  q = __fma_rn(q, s2, 0x1.c71c71c71c71cp-3);
  q = __fma_rn(q, s2, 0x1.2492492492492p-2);
  q = __fma_rn(q, s2, 0x1.999999999999ap-2);
  q = __fma_rn(q, s2, 0x1.5555555555555p-1);
  double lm = __fma_rn(__dmul_rn(s, s2), q, __dmul_rn(2.0, s));
  double de = (double)e;
  return __fma_rn(de, 0x1.62e42feep-1, __fma_rn(de, 0x1.a39ef35793c76p-33, lm));
}

// MurmurHash3 x86_32 mixing (Appleby, public domain) of (seed lo, seed hi,
// position, column), length 16 (sampling_kernels.py:43-65, 633-677).
OMNI_DEVINL uint32_t mm3_mix(uint32_t h, uint32_t k) {
  k *= 0xCC9E2D51u;
  k = __funnelshift_l(k, k, 15);
  k *= 0x1B873593u;
  h ^= k;
  h = __funnelshift_l(h, h, 13);
  return h * 5u + 0xE6546B64u;
}
OMNI_DEVINL uint32_t mm3_prefix(int64_t seed, int64_t position) {
  uint64_t s = (uint64_t)seed;
  uint32_t h = mm3_mix(0u, (uint32_t)(s & 0xFFFFFFFFu));
  h = mm3_mix(h, (uint32_t)(s >> 32));
  return mm3_mix(h, (uint32_t)((uint64_t)position & 0xFFFFFFFFu));
}
OMNI_DEVINL uint32_t mm3_finish(uint32_t prefix, uint32_t column) {
  uint32_t h = mm3_mix(prefix, column) ^ 16u;
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}
// Gumbel noise with sglang multinomial_with_seed's endpoint clamp
// (sampling_kernels.py:67-78).
OMNI_DEVINL double gumbel_of(uint32_t h) {
  double u = __ddiv_rn((double)h, 4294967295.0);
  double lu = det_log(u);
  lu = lu < -1.7976931348623157e308 ? -1.7976931348623157e308 : lu;
  lu = lu > -2.3283064365386963e-10 ? -2.3283064365386963e-10 : lu;
  return -det_log(-lu);
}

// Order-preserving 32-bit key of a float (+0 above -0; positive NaN on top).
OMNI_DEVINL uint32_t ordered_bits(float f) {
  uint32_t b = __float_as_uint(f);
  return (b >> 31) ? ~b : (b | 0x80000000u);
}
OMNI_DEVINL float unordered_float(uint32_t o) { return __uint_as_float((o >> 31) ? (o & 0x7FFFFFFFu) : ~o); }

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBlockK = 1024;

struct SelectSmem {
  int hist[256];
  unsigned long long warp_tot[kWarps];
  unsigned long long keys[kMaxBlockK];
  int digit;
  int krem;
  float fred[kWarps];
  int ired[kWarps];
  int64_t token;
};

// ---------------------------------------------------------------------------
// Block radix select: the ordered score T of the K-th largest valid element
// (counted with multiplicity) and the number krem of T-valued elements among
// the top K.  Every thread passes its EPT keys and validity flags.
// ---------------------------------------------------------------------------
template <int EPT>
OMNI_DEVINL void block_radix_select(const uint32_t (&o)[EPT], const bool (&valid)[EPT], int K, SelectSmem& sm,
                                    uint32_t& T, int& krem_out) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, pmask = 0;
  int krem = K;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    sm.hist[tid] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < EPT; ++j)
      if (valid[j] && (o[j] & pmask) == prefix) atomicAdd(&sm.hist[(o[j] >> shift) & 255], 1);
    __syncthreads();
    if (warp == 0) {
      // lane l owns digits 255-8l down to 248-8l (descending)
      int c[8], tot = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = sm.hist[255 - 8 * lane - i];
        tot += c[i];
      }
      int incl = tot;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        int n = __shfl_up_sync(0xFFFFFFFFu, incl, off);
        if (lane >= off) incl += n;
      }
      int excl = incl - tot;
      if (excl < krem && krem <= incl) {
        int running = excl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (running + c[i] >= krem) {
            sm.digit = 255 - 8 * lane - i;
            sm.krem = krem - running;
            break;
          }
          running += c[i];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sm.digit << shift;
    pmask |= 0xFFu << shift;
    krem = sm.krem;
  }
  T = prefix;
  krem_out = krem;
}

// Block exclusive scan of a packed triple of 21-bit counts.
OMNI_DEVINL unsigned long long block_excl_scan_u64(unsigned long long v, SelectSmem& sm,
                                                   unsigned long long& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    unsigned long long n = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) sm.warp_tot[warp] = incl;
  __syncthreads();
  unsigned long long before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    if (w < warp) before += sm.warp_tot[w];
    all += sm.warp_tot[w];
  }
  total = all;
  return before + incl - v;
}

// Descending bitonic sort of n (power of two, <= 1024) keys in shared memory.
OMNI_DEVINL void smem_bitonic_desc(unsigned long long* keys, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < (n >> 1); i += kThreads) {
        int lo = 2 * stride * (i / stride) + (i % stride);
        int hi = lo + stride;
        bool desc = (lo & size) == 0;
        unsigned long long a = keys[lo], b = keys[hi];
        if ((a < b) == desc) {
          keys[lo] = b;
          keys[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

// Descending bitonic sort of 64 keys held two per lane (element 2 lane + j),
// entirely in registers; lane l ends with ranks 2l and 2l + 1.
OMNI_DEVINL void warp_sort64_desc(unsigned long long& a0, unsigned long long& a1) {
  const int lane = threadIdx.x & 31;
  const int i0 = 2 * lane;
#pragma unroll
  for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const bool desc = (i0 & size) == 0;
      if (stride == 1) {
        if ((a0 < a1) == desc) {
          const unsigned long long t = a0;
          a0 = a1;
          a1 = t;
        }
      } else {
        const unsigned long long o0 = __shfl_xor_sync(0xFFFFFFFFu, a0, stride >> 1);
        const unsigned long long o1 = __shfl_xor_sync(0xFFFFFFFFu, a1, stride >> 1);
        const bool take_max = ((i0 & stride) == 0) == desc;
        a0 = take_max ? (a0 > o0 ? a0 : o0) : (a0 < o0 ? a0 : o0);
        a1 = take_max ? (a1 > o1 ? a1 : o1) : (a1 < o1 ? a1 : o1);
      }
    }
  }
}

// torch.topk's 32-entry descending bitonic network over the gathered
// candidates, one entry per lane (sampling_kernels.py:123-312).
OMNI_DEVINL void warp_bitonic32_torch(float& sc, uint32_t& id, int max_top_k) {
  const int lane = threadIdx.x & 31;
  int valid = lane < max_top_k;
  const int rounds[15][3] = {{1, 2, 0}, {2, 4, 0}, {1, 4, 0}, {4, 8, 0},  {2, 8, 0},
                             {1, 8, 0}, {8, 16, 0}, {4, 16, 0}, {2, 16, 0}, {1, 16, 0},
                             {16, 32, 1}, {8, 32, 1}, {4, 32, 1}, {2, 32, 1}, {1, 32, 1}};
#pragma unroll
  for (int r = 0; r < 15; ++r) {
    const int stride = rounds[r][0], net = rounds[r][1], fin = rounds[r][2];
    float psc = __shfl_xor_sync(0xFFFFFFFFu, sc, stride);
    uint32_t pid = __shfl_xor_sync(0xFFFFFFFFu, id, stride);
    int pvalid = __shfl_xor_sync(0xFFFFFFFFu, valid, stride);
    bool is_right = (lane & stride) != 0;
    float left_s = is_right ? psc : sc, right_s = is_right ? sc : psc;
    int left_v = is_right ? pvalid : valid, right_v = is_right ? valid : pvalid;
    bool direction;
    if (fin) {
      direction = false;
    } else {
      int left_off = lane - (is_right ? stride : 0);
      int thread_id = (left_off / (2 * stride)) * stride + (left_off % stride);
      direction = (thread_id & (net / 2)) != 0;
    }
    bool should_swap = ((left_s > right_s) && left_v) || (right_v == 0);
    if (should_swap == direction) {
      sc = psc;
      id = pid;
      valid = pvalid;
    }
  }
}

// Hillis–Steele inclusive scan over lanes, offsets 1..16.
OMNI_DEVINL float warp_scan_incl(float v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    float n = __shfl_up_sync(0xFFFFFFFFu, v, off);
    if (lane >= off) v = v + n;
  }
  return v;
}

// Softmax over ranks < top_k, top-p removal, log-probabilities and the seeded
// Gumbel-max, one warp.  Lane l holds ranks [l*C, l*C+C).  Returns the
// winning token (valid in every lane).  Follows sample_sorted_top_k
// (sampling_kernels.py:385-438) and the torch fallback (sglang_model.py:1987-2034).
template <int C>
OMNI_DEVINL int64_t warp_sample_sorted_g(const float (&sc)[C], const uint32_t (&id)[C], int64_t top_k, float top_p,
                                         bool has_top_p, const double (&gum)[C]);
// Gumbel noise of ranks lane * C + j (depends only on the seed and the position).
template <int C>
OMNI_DEVINL void rank_gumbels(uint32_t hash_prefix, double (&gum)[C]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < C; ++j) gum[j] = gumbel_of(mm3_finish(hash_prefix, (uint32_t)(lane * C + j)));
}
template <int C>
OMNI_DEVINL int64_t warp_sample_sorted(const float (&sc)[C], const uint32_t (&id)[C], int64_t top_k, float top_p,
                                       bool has_top_p, uint32_t hash_prefix) {
  double gum[C];
  rank_gumbels<C>(hash_prefix, gum);
  return warp_sample_sorted_g<C>(sc, id, top_k, top_p, has_top_p, gum);
}
template <int C>
OMNI_DEVINL int64_t warp_sample_sorted_g(const float (&sc)[C], const uint32_t (&id)[C], int64_t top_k, float top_p,
                                         bool has_top_p, const double (&gum)[C]) {
  const int lane = threadIdx.x & 31;
  float masked[C], e[C], p[C];
  float mx = __uint_as_float(0xFF800000u);
#pragma unroll
  for (int j = 0; j < C; ++j) {
    const int r = lane * C + j;
    masked[j] = ((int64_t)r < top_k) ? sc[j] : __uint_as_float(0xFF800000u);
    mx = fmaxf(mx, masked[j]);
  }
  mx = warp_max_xor(mx);
  float part = 0.0f;
#pragma unroll
  for (int j = 0; j < C; ++j) {
    e[j] = det_expf(__fsub_rn(masked[j], mx));
    part = (j == 0) ? e[j] : __fadd_rn(part, e[j]);
  }
  float total = __shfl_sync(0xFFFFFFFFu, warp_scan_incl(part), 31);
#pragma unroll
  for (int j = 0; j < C; ++j) p[j] = __fdiv_rn(e[j], total);
  bool keep[C];
#pragma unroll
  for (int j = 0; j < C; ++j) keep[j] = (int64_t)(lane * C + j) < top_k;
  if (has_top_p) {
    float q[C], acc = 0.0f;
#pragma unroll
    for (int j = 0; j < C; ++j) {
      acc = (j == 0) ? p[j] : __fadd_rn(acc, p[j]);
      q[j] = acc;
    }
    float incl = warp_scan_incl(acc);
    float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
    if (lane == 0) excl = 0.0f;
    const bool active = (top_p > 0.0f) && (top_p < 1.0f);
#pragma unroll
    for (int j = 0; j < C; ++j) {
      const int r = lane * C + j;
      float cdf = __fadd_rn(excl, q[j]);
      if (r != 0 && active && (__fsub_rn(cdf, p[j]) >= top_p)) keep[j] = false;
    }
  }
  double best = 0.0;
  int best_rank = 0x7FFFFFFF;
  uint32_t best_id = 0;
#pragma unroll
  for (int j = 0; j < C; ++j) {
    const int r = lane * C + j;
    float lp = keep[j] ? det_logf(p[j]) : __uint_as_float(0xFF800000u);
    double v = __dadd_rn((double)lp, gum[j]);
    if (j == 0 || v > best) {
      best = v;
      best_rank = r;
      best_id = id[j];
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    double ov = __shfl_xor_sync(0xFFFFFFFFu, best, off);
    int orank = __shfl_xor_sync(0xFFFFFFFFu, best_rank, off);
    uint32_t oid = __shfl_xor_sync(0xFFFFFFFFu, best_id, off);
    if (ov > best || (ov == best && orank < best_rank)) {
      best = ov;
      best_rank = orank;
      best_id = oid;
    }
  }
  return (int64_t)best_id;
}

// torch.argmax order: the first NaN, else the first maximum.
OMNI_DEVINL bool argmax_better(float a, int ia, float b, int ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return (an && bn) ? ia < ib : an;
  if (a != b) return a > b;
  return ia < ib;
}

template <int EPT>
OMNI_DEVINL int block_argmax(const float (&v)[EPT], const bool (&valid)[EPT], int base, SelectSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float bv = 0.0f;
  int bi = 0x7FFFFFFF;
#pragma unroll
  for (int j = 0; j < EPT; ++j)
    if (valid[j] && (bi == 0x7FFFFFFF || argmax_better(v[j], base + j, bv, bi))) {
      bv = v[j];
      bi = base + j;
    }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
    int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
    if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || argmax_better(ov, oi, bv, bi))) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sm.fred[warp] = bv;
    sm.ired[warp] = bi;
  }
  __syncthreads();
  bv = sm.fred[0];
  bi = sm.ired[0];
  for (int w = 1; w < kWarps; ++w)
    if (sm.ired[w] != 0x7FFFFFFF && (bi == 0x7FFFFFFF || argmax_better(sm.fred[w], sm.ired[w], bv, bi))) {
      bv = sm.fred[w];
      bi = sm.ired[w];
    }
  return bi;
}

// Fused embedding epilogue: gathered[row] = table[token]; summed[row] += it;
// returns this thread's part of the gathered row's sum of squares.
OMNI_DEVINL float gather_add_row(const uint16_t* __restrict__ table, int hidden, int64_t token,
                                 uint16_t* __restrict__ gathered, uint16_t* __restrict__ summed,
                                 const uint4* summed_pre = nullptr) {
  const uint4* src = reinterpret_cast<const uint4*>(table + token * (int64_t)hidden);
  float ss = 0.0f;
  for (int v = threadIdx.x; v < hidden / 8; v += kThreads) {
    uint4 w = src[v];
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      ss = __fmaf_rn(bf_lo(ws[q]), bf_lo(ws[q]), ss);
      ss = __fmaf_rn(bf_hi(ws[q]), bf_hi(ws[q]), ss);
    }
    if (gathered) reinterpret_cast<uint4*>(gathered)[v] = w;
    if (summed) {
      uint4 s = (summed_pre && v == (int)threadIdx.x) ? *summed_pre : reinterpret_cast<uint4*>(summed)[v];
      s.x = pack_bf2(__fadd_rn(bf_lo(s.x), bf_lo(w.x)), __fadd_rn(bf_hi(s.x), bf_hi(w.x)));
      s.y = pack_bf2(__fadd_rn(bf_lo(s.y), bf_lo(w.y)), __fadd_rn(bf_hi(s.y), bf_hi(w.y)));
      s.z = pack_bf2(__fadd_rn(bf_lo(s.z), bf_lo(w.z)), __fadd_rn(bf_hi(s.z), bf_hi(w.z)));
      s.w = pack_bf2(__fadd_rn(bf_lo(s.w), bf_lo(w.w)), __fadd_rn(bf_hi(s.w), bf_hi(w.w)));
      reinterpret_cast<uint4*>(summed)[v] = s;
    }
  }
  return ss;
}

struct ResidualParams {
  const uint16_t* logits;
  int64_t stride;
  int vocab;
  const float* temps;
  const int64_t* top_ks;
  const float* top_ps;
  const int64_t* seeds;
  const int64_t* positions;
  int64_t pos_mul, pos_add;
  const uint8_t* do_sample;
  int argmax_all;
  int max_top_k, block_k, has_top_p;
  int64_t* out;
  int64_t out_stride;
  const uint16_t* table;
  int hidden;
  uint16_t* gathered;
  uint16_t* summed;
  float* gathered_ss;  // nullable: sum of squares of each gathered row
};

// Loads EPT consecutive bf16 logits of a row: thread t holds [t*EPT, t*EPT+EPT).
template <int EPT>
OMNI_DEVINL void load_bf16_row(const uint16_t* row, int vocab, float (&v)[EPT], bool (&valid)[EPT]) {
  const int base = threadIdx.x * EPT;
  if (base + EPT <= vocab) {
    static_assert(EPT % 4 == 0, "EPT");
#pragma unroll
    for (int c = 0; c < EPT / 4; ++c) {
      uint2 w = *reinterpret_cast<const uint2*>(row + base + 4 * c);
      v[4 * c + 0] = bf_lo(w.x);
      v[4 * c + 1] = bf_hi(w.x);
      v[4 * c + 2] = bf_lo(w.y);
      v[4 * c + 3] = bf_hi(w.y);
    }
#pragma unroll
    for (int j = 0; j < EPT; ++j) valid[j] = true;
  } else {
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      valid[j] = base + j < vocab;
      v[j] = valid[j] ? bf2f(row[base + j]) : 0.0f;
    }
  }
}

template <int EPT, int C>
__global__ void __launch_bounds__(kThreads) residual_sample_kernel(const __grid_constant__ ResidualParams p) {
  __shared__ SelectSmem sm;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Step metadata (the row's sampling parameters, seed and position) and the running sum
  // of the frame's codec embeddings come from kernels before the previous one: they load,
  // and the rank Gumbel noise is computed, before griddepcontrol.wait.  The logits (the
  // previous kernel's output) are read after it.
  const bool sample = !p.argmax_all && (p.do_sample == nullptr || p.do_sample[row] != 0);
  float t_row = 1.0f, top_p_row = 1.0f;
  int64_t top_k_row = 0;
  double gum[C];
  if (sample) {
    t_row = p.temps[row];
    top_k_row = p.top_ks[row];
    top_p_row = p.top_ps[row];
    if (warp == 0) rank_gumbels<C>(mm3_prefix(p.seeds[row], p.positions[row] * p.pos_mul + p.pos_add), gum);
  }
  uint4 summed_pre = make_uint4(0, 0, 0, 0);
  const bool has_pre = p.table != nullptr && p.summed != nullptr && tid < p.hidden / 8;
  if (has_pre) summed_pre = reinterpret_cast<const uint4*>(p.summed + (int64_t)row * p.hidden)[tid];
  griddep_wait();
  griddep_launch();
  float v[EPT];
  bool valid[EPT];
  load_bf16_row<EPT>(p.logits + row * p.stride, p.vocab, v, valid);

  int64_t token;
  if (!sample) {
    int idx = block_argmax<EPT>(v, valid, tid * EPT, sm);
    token = idx;
  } else {
    float t = t_row;
    if (!(t >= 1e-5f)) t = (t != t) ? t : 1e-5f;
    uint32_t o[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      v[j] = __fdiv_rn(v[j], t);
      o[j] = ordered_bits(v[j]);
    }
    const bool small = p.max_top_k <= 32;
    const int K = small ? p.max_top_k : p.block_k;
    uint32_t T;
    int krem;
    block_radix_select<EPT>(o, valid, K, sm, T, krem);
    const int G = K - krem;
    // class counts: 0 above T, 1 equal to T, 2 below T
    unsigned long long cnt = 0;
#pragma unroll
    for (int j = 0; j < EPT; ++j)
      if (valid[j]) cnt += o[j] > T ? 1ull : (o[j] == T ? (1ull << 21) : (1ull << 42));
    unsigned long long tot;
    unsigned long long ex = block_excl_scan_u64(cnt, sm, tot);
    const int E = (int)((tot >> 21) & 0x1FFFFF);
    int e0 = (int)(ex & 0x1FFFFF), e1 = (int)((ex >> 21) & 0x1FFFFF), e2 = (int)(ex >> 42);
    const int limit = small ? 32 : p.block_k;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      if (!valid[j]) continue;
      const uint32_t idx = (uint32_t)(tid * EPT + j);
      const unsigned long long key = ((unsigned long long)o[j] << 32) | (0xFFFFFFFFu - idx);
      int pos = -1;
      if (o[j] > T) pos = e0++;
      else if (o[j] == T) pos = G + e1++;
      else if (small) pos = G + E + e2++;
      if (pos >= 0 && pos < limit) sm.keys[pos] = key;
    }
    __syncthreads();
    if (!small && C != 2) smem_bitonic_desc(sm.keys, p.block_k);
    if (warp == 0) {
      float sc[C];
      uint32_t id[C];
      unsigned long long kk[C];
#pragma unroll
      for (int j = 0; j < C; ++j) kk[j] = sm.keys[lane * C + j];
      if constexpr (C == 2) warp_sort64_desc(kk[0], kk[1]);
#pragma unroll
      for (int j = 0; j < C; ++j) {
        const unsigned long long key = kk[j];
        sc[j] = unordered_float((uint32_t)(key >> 32));
        id[j] = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
      }
      if (small) {
        if constexpr (C == 1) warp_bitonic32_torch(sc[0], id[0], p.max_top_k);
      }
      int64_t tok = warp_sample_sorted_g<C>(sc, id, top_k_row, top_p_row, p.has_top_p != 0, gum);
      if (lane == 0) sm.token = tok;
    }
    __syncthreads();
    token = sm.token;
  }
  if (tid == 0) p.out[row * p.out_stride] = token;
  if (p.table != nullptr) {
    float ss = gather_add_row(p.table, p.hidden, token, p.gathered ? p.gathered + (int64_t)row * p.hidden : nullptr,
                              p.summed ? p.summed + (int64_t)row * p.hidden : nullptr,
                              has_pre ? &summed_pre : nullptr);
    if (p.gathered_ss) {
      ss = warp_sum_xor(ss);
      __syncthreads();
      if (lane == 0) sm.fred[warp] = ss;
      __syncthreads();
      if (tid == 0) {
        float t = sm.fred[0];
        for (int w = 1; w < kWarps; ++w) t += sm.fred[w];
        p.gathered_ss[row] = t;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Gumbel-max over pre-sorted log-probabilities (one warp per row).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) sorted_sample_kernel(const float* __restrict__ logprobs,
                                                            const int64_t* __restrict__ sorted_idx, int64_t rows,
                                                            int cols, const int64_t* __restrict__ seeds,
                                                            const int64_t* __restrict__ positions,
                                                            int64_t* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint32_t hp = mm3_prefix(seeds[row], positions[row]);
  double best = 0.0;
  int best_c = 0x7FFFFFFF;
  for (int c = lane; c < cols; c += 32) {
    double v = __dadd_rn((double)logprobs[row * cols + c], gumbel_of(mm3_finish(hp, (uint32_t)c)));
    if (best_c == 0x7FFFFFFF || v > best) {
      best = v;
      best_c = c;
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    double ov = __shfl_xor_sync(0xFFFFFFFFu, best, off);
    int oc = __shfl_xor_sync(0xFFFFFFFFu, best_c, off);
    if (oc != 0x7FFFFFFF && (best_c == 0x7FFFFFFF || ov > best || (ov == best && oc < best_c))) {
      best = ov;
      best_c = oc;
    }
  }
  if (lane == 0) out[row] = sorted_idx[row * cols + best_c];
}

// ---------------------------------------------------------------------------
// Embedding gather + accumulate (K10).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) gather_add_kernel(const void* __restrict__ tokens, int tok_i32,
                                                              const uint16_t* __restrict__ table, int hidden,
                                                              uint16_t* __restrict__ gathered,
                                                              uint16_t* __restrict__ acc,
                                                              const uint16_t* __restrict__ ptable, int psize,
                                                              uint16_t* __restrict__ projected) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  const int64_t tok = tok_i32 ? (int64_t)reinterpret_cast<const int32_t*>(tokens)[row]
                              : reinterpret_cast<const int64_t*>(tokens)[row];
  gather_add_row(table, hidden, tok, gathered + (int64_t)row * hidden, acc + (int64_t)row * hidden);
  if (ptable) {
    const uint4* src = reinterpret_cast<const uint4*>(ptable + tok * (int64_t)psize);
    uint4* dst = reinterpret_cast<uint4*>(projected + (int64_t)row * psize);
    for (int c = threadIdx.x; c < psize / 8; c += kThreads) dst[c] = src[c];
  }
}

// ---------------------------------------------------------------------------
// Layer-0 sampler over fp32 logits (vocab % 4 == 0, <= 8192).
// Thread t holds elements 4t + 1024 j (j < J), folded in (j, element) order;
// block sums: xor butterfly 16..1 per warp, warp totals folded in order.
// ---------------------------------------------------------------------------
struct Layer0Params {
  const float* logits;
  int64_t stride;
  int vocab;
  const float* penalties;
  const uint8_t* rep_mask;
  const uint8_t* suppress_mask;
  const float* temps;
  const int64_t* top_ks;
  const float* top_ps;
  const float* min_ps;
  const int64_t* seeds;
  const int64_t* positions;
  int block_k;
  int64_t* out;
  uint8_t* rep_mask_update;  // nullable: marks the drawn token as seen
};

template <int J, int C>
__global__ void __launch_bounds__(kThreads) layer0_sample_kernel(const __grid_constant__ Layer0Params p) {
  __shared__ SelectSmem sm;
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int EPT = 4 * J;
  float s[EPT];
  bool valid[EPT];
  uint32_t o[EPT];
  float t = p.temps[row];
  if (!(t >= 1e-5f)) t = (t != t) ? t : 1e-5f;
  const float pen = p.penalties ? p.penalties[row] : 1.0f;
  float mx = __uint_as_float(0xFF800000u);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int base = 4 * tid + 1024 * j;
    const bool in = base < p.vocab;
    float4 x = in ? *reinterpret_cast<const float4*>(p.logits + row * p.stride + base) : make_float4(0, 0, 0, 0);
    uint32_t rm = 0, sp = 0;
    if (in && p.rep_mask) rm = *reinterpret_cast<const uint32_t*>(p.rep_mask + row * (int64_t)p.vocab + base);
    if (in && p.suppress_mask)
      sp = *reinterpret_cast<const uint32_t*>(p.suppress_mask + row * (int64_t)p.vocab + base);
    float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float l = xs[e];
      if ((rm >> (8 * e)) & 0xFF) l = l > 0.0f ? __fdiv_rn(l, pen) : __fmul_rn(l, pen);
      if ((sp >> (8 * e)) & 0xFF) l = __uint_as_float(0xFF800000u);
      const int k = 4 * j + e;
      valid[k] = in;
      s[k] = __fdiv_rn(l, t);
      o[k] = ordered_bits(s[k]);
      if (in) mx = fmaxf(mx, s[k]);
    }
  }
  // block max (exact in any order)
  mx = warp_max_xor(mx);
  if (lane == 0) sm.fred[warp] = mx;
  __syncthreads();
  mx = sm.fred[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, sm.fred[w]);
  __syncthreads();
  float part = 0.0f;
  bool first = true;
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    if (!valid[k]) continue;
    float e = det_expf(__fsub_rn(s[k], mx));
    part = first ? e : __fadd_rn(part, e);
    first = false;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xFFFFFFFFu, part, off));
  if (lane == 0) sm.fred[warp] = part;
  __syncthreads();
  float z = sm.fred[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) z = __fadd_rn(z, sm.fred[w]);

  // top block_k by (score desc, index asc)
  uint32_t T;
  int krem;
  block_radix_select<EPT>(o, valid, p.block_k, sm, T, krem);
  const int G = p.block_k - krem;
  unsigned long long cnt = 0;
#pragma unroll
  for (int k = 0; k < EPT; ++k)
    if (valid[k]) cnt += o[k] > T ? 1ull : (o[k] == T ? (1ull << 21) : 0ull);
  unsigned long long tot;
  unsigned long long ex = block_excl_scan_u64(cnt, sm, tot);
  int e0 = (int)(ex & 0x1FFFFF), e1 = (int)((ex >> 21) & 0x1FFFFF);
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    if (!valid[k]) continue;
    const uint32_t idx = (uint32_t)(4 * tid + 1024 * (k / 4) + (k % 4));
    const unsigned long long key = ((unsigned long long)o[k] << 32) | (0xFFFFFFFFu - idx);
    int pos = -1;
    if (o[k] > T) pos = e0++;
    else if (o[k] == T) pos = G + e1++;
    if (pos >= 0 && pos < p.block_k) sm.keys[pos] = key;
  }
  __syncthreads();
  if (C != 2) smem_bitonic_desc(sm.keys, p.block_k);
  if (warp == 0) {
    float pr[C], q[C];
    uint32_t id[C];
    float acc = 0.0f;
    unsigned long long kk[C];
#pragma unroll
    for (int j = 0; j < C; ++j) kk[j] = sm.keys[lane * C + j];
    if constexpr (C == 2) warp_sort64_desc(kk[0], kk[1]);
#pragma unroll
    for (int j = 0; j < C; ++j) {
      const unsigned long long key = kk[j];
      const float sc = unordered_float((uint32_t)(key >> 32));
      id[j] = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu);
      pr[j] = __fdiv_rn(det_expf(__fsub_rn(sc, mx)), z);
      acc = (j == 0) ? pr[j] : __fadd_rn(acc, pr[j]);
      q[j] = acc;
    }
    float incl = warp_scan_incl(acc);
    float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
    if (lane == 0) excl = 0.0f;
    const float p0 = __shfl_sync(0xFFFFFFFFu, pr[0], 0);
    const float top_p = p.top_ps[row];
    const float min_p = p.min_ps ? p.min_ps[row] : 0.0f;
    const float min_thr = __fmul_rn(p0, min_p);
    const int64_t top_k = p.top_ks[row];
    const uint32_t hp = mm3_prefix(p.seeds[row], p.positions[row]);
    double best = 0.0;
    int best_rank = 0x7FFFFFFF;
    uint32_t best_id = 0;
#pragma unroll
    for (int j = 0; j < C; ++j) {
      const int r = lane * C + j;
      bool keep = (int64_t)r < top_k;
      if (__fsub_rn(__fadd_rn(excl, q[j]), pr[j]) > top_p) keep = false;
      if (min_p > 0.0f && pr[j] < min_thr) keep = false;
      float lp = (keep && pr[j] > 0.0f) ? det_logf(pr[j]) : __uint_as_float(0xFF800000u);
      double v = __dadd_rn((double)lp, gumbel_of(mm3_finish(hp, (uint32_t)r)));
      if (j == 0 || v > best) {
        best = v;
        best_rank = r;
        best_id = id[j];
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      double ov = __shfl_xor_sync(0xFFFFFFFFu, best, off);
      int orank = __shfl_xor_sync(0xFFFFFFFFu, best_rank, off);
      uint32_t oid = __shfl_xor_sync(0xFFFFFFFFu, best_id, off);
      if (ov > best || (ov == best && orank < best_rank)) {
        best = ov;
        best_rank = orank;
        best_id = oid;
      }
    }
    if (lane == 0) {
      p.out[row] = (int64_t)best_id;
      if (p.rep_mask_update) p.rep_mask_update[row * (int64_t)p.vocab + best_id] = 1;
    }
  }
}

int block_k_of(int max_top_k) {
  if (max_top_k <= 32) return 32;
  int b = 1;
  while (b < max_top_k) b <<= 1;
  return b;
}

bool ladder_ok(int k) {
  switch (k) {
    case 4: case 8: case 16: case 32: case 50: case 64: case 128: case 256: case 512: case 1024:
      return true;
    default:
      return false;
  }
}

template <int EPT>
cudaError_t launch_residual(const ResidualParams& p, int64_t rows, cudaStream_t st) {
  switch (p.block_k) {
    case 32: return launch(residual_sample_kernel<EPT, 1>, dim3((unsigned)rows), dim3(kThreads), 0, st, p);
    case 64: return launch(residual_sample_kernel<EPT, 2>, dim3((unsigned)rows), dim3(kThreads), 0, st, p);
    case 128: return launch(residual_sample_kernel<EPT, 4>, dim3((unsigned)rows), dim3(kThreads), 0, st, p);
    case 256: return launch(residual_sample_kernel<EPT, 8>, dim3((unsigned)rows), dim3(kThreads), 0, st, p);
    case 512: return launch(residual_sample_kernel<EPT, 16>, dim3((unsigned)rows), dim3(kThreads), 0, st, p);
    case 1024: return launch(residual_sample_kernel<EPT, 32>, dim3((unsigned)rows), dim3(kThreads), 0, st, p);
  }
  return cudaErrorInvalidValue;
}

int run_residual(ResidualParams& p, int64_t rows, int vocab, int max_top_k, bool need_block, cudaStream_t st) {
  if (rows < 0) return set_error(OMNI_ERR_INVALID, "rows must be >= 0");
  if (vocab < 1 || vocab > 4096 || vocab % 8 != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "vocab must be a multiple of 8 in [8, 4096]");
  if ((p.stride % 8) != 0 || (reinterpret_cast<uintptr_t>(p.logits) & 15) != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "logits rows must be 16-byte aligned");
  if (p.table && (p.hidden % 8 != 0 || (reinterpret_cast<uintptr_t>(p.table) & 15) != 0 ||
                  (p.gathered && (reinterpret_cast<uintptr_t>(p.gathered) & 15) != 0) ||
                  (p.summed && (reinterpret_cast<uintptr_t>(p.summed) & 15) != 0)))
    return set_error(OMNI_ERR_UNSUPPORTED, "embedding rows must be 16-byte aligned, hidden % 8 == 0");
  if (need_block) {
    if (!ladder_ok(max_top_k)) return set_error(OMNI_ERR_UNSUPPORTED, "max_top_k is not on the width ladder");
    p.block_k = block_k_of(max_top_k);
    if (p.block_k > vocab) return set_error(OMNI_ERR_UNSUPPORTED, "max_top_k exceeds the vocabulary");
  } else {
    p.block_k = 32;
  }
  p.max_top_k = max_top_k;
  if (rows == 0) return OMNI_OK;
  cudaError_t e;
  if (vocab <= 1024) e = launch_residual<4>(p, rows, st);
  else if (vocab <= 2048) e = launch_residual<8>(p, rows, st);
  else e = launch_residual<16>(p, rows, st);
  return check_launch(e);
}

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int omni_sample_topk_topp(const void* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                              const float* temperatures, const int64_t* top_ks, const float* top_ps,
                                              const int64_t* seeds, const int64_t* positions, int32_t max_top_k,
                                              int32_t has_top_p, int64_t* out, void* stream) {
  ResidualParams p = {};
  p.logits = static_cast<const uint16_t*>(logits);
  p.stride = logits_stride;
  p.vocab = (int)vocab;
  p.temps = temperatures;
  p.top_ks = top_ks;
  p.top_ps = top_ps;
  p.seeds = seeds;
  p.positions = positions;
  p.pos_mul = 1;
  p.pos_add = 0;
  p.has_top_p = has_top_p;
  p.out = out;
  p.out_stride = 1;
  return run_residual(p, rows, (int)vocab, max_top_k, true, static_cast<cudaStream_t>(stream));
}

extern "C" OMNI_API int omni_predictor_sample_step(const void* logits, int64_t rows, int64_t vocab,
                                                   int64_t logits_stride, const float* temperatures,
                                                   const int64_t* top_ks, const float* top_ps, const int64_t* seeds,
                                                   const int64_t* positions, int64_t pos_mul, int64_t pos_add,
                                                   const uint8_t* do_sample, int32_t argmax_all, int32_t max_top_k,
                                                   int32_t has_top_p, int64_t* codes, int64_t codes_stride,
                                                   const void* table, int64_t hidden, void* gathered, void* summed,
                                                   float* gathered_ss, void* stream) {
  ResidualParams p = {};
  p.logits = static_cast<const uint16_t*>(logits);
  p.stride = logits_stride;
  p.vocab = (int)vocab;
  p.temps = temperatures;
  p.top_ks = top_ks;
  p.top_ps = top_ps;
  p.seeds = seeds;
  p.positions = positions;
  p.pos_mul = pos_mul;
  p.pos_add = pos_add;
  p.do_sample = do_sample;
  p.argmax_all = argmax_all;
  p.has_top_p = has_top_p;
  p.out = codes;
  p.out_stride = codes_stride;
  p.table = static_cast<const uint16_t*>(table);
  p.hidden = (int)hidden;
  p.gathered = static_cast<uint16_t*>(gathered);
  p.summed = static_cast<uint16_t*>(summed);
  p.gathered_ss = gathered_ss;
  return run_residual(p, rows, (int)vocab, argmax_all ? 32 : max_top_k, !argmax_all,
                      static_cast<cudaStream_t>(stream));
}

extern "C" OMNI_API int omni_codebook_step(const void* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                           const void* table, int64_t hidden, int64_t* codes, int64_t codes_stride,
                                           void* gathered, void* summed, void* stream) {
  ResidualParams p = {};
  p.logits = static_cast<const uint16_t*>(logits);
  p.stride = logits_stride;
  p.vocab = (int)vocab;
  p.argmax_all = 1;
  p.out = codes;
  p.out_stride = codes_stride;
  p.table = static_cast<const uint16_t*>(table);
  p.hidden = (int)hidden;
  p.gathered = static_cast<uint16_t*>(gathered);
  p.summed = static_cast<uint16_t*>(summed);
  return run_residual(p, rows, (int)vocab, 32, false, static_cast<cudaStream_t>(stream));
}

extern "C" OMNI_API int omni_sample_sorted_seeded(const float* logprobs, const int64_t* sorted_idx, int64_t rows,
                                                  int64_t cols, const int64_t* seeds, const int64_t* positions,
                                                  int64_t* out, void* stream) {
  if (rows < 0 || cols < 0) return set_error(OMNI_ERR_INVALID, "negative shape");
  if (cols == 0 || cols > 1024) return set_error(OMNI_ERR_UNSUPPORTED, "cols must be in [1, 1024]");
  if (rows == 0) return OMNI_OK;
  return check_launch(launch(sorted_sample_kernel, dim3((unsigned)((rows + 3) / 4)), dim3(128), 0,
                             static_cast<cudaStream_t>(stream), logprobs, sorted_idx, rows, (int)cols, seeds,
                             positions, out));
}

extern "C" OMNI_API int omni_gather_embedding_add(const void* token_ids, int32_t token_is_i32, int64_t rows,
                                                  const void* table, int64_t hidden, void* gathered,
                                                  void* accumulated, const void* projected_table,
                                                  int64_t projected_size, void* projected, void* stream) {
  if (rows < 0 || hidden < 0) return set_error(OMNI_ERR_INVALID, "negative shape");
  if (hidden % 8 != 0 || (projected_table && (projected_size % 8 != 0 || projected_size > hidden)))
    return set_error(OMNI_ERR_UNSUPPORTED, "hidden and projected sizes must be multiples of 8");
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (mis(table) || mis(gathered) || mis(accumulated) || (projected_table && (mis(projected_table) || mis(projected))))
    return set_error(OMNI_ERR_UNSUPPORTED, "rows must be 16-byte aligned");
  if (rows == 0 || hidden == 0) return OMNI_OK;
  return check_launch(launch(gather_add_kernel, dim3((unsigned)rows), dim3(kThreads), 0,
                             static_cast<cudaStream_t>(stream), token_ids, (int)token_is_i32,
                             static_cast<const uint16_t*>(table), (int)hidden, static_cast<uint16_t*>(gathered),
                             static_cast<uint16_t*>(accumulated), static_cast<const uint16_t*>(projected_table),
                             (int)projected_size, static_cast<uint16_t*>(projected)));
}

extern "C" OMNI_API int omni_layer0_sample(const float* logits, int64_t rows, int64_t vocab, int64_t logits_stride,
                                           const float* penalties, const uint8_t* rep_mask,
                                           const uint8_t* suppress_mask, const float* temperatures,
                                           const int64_t* top_ks, const float* top_ps, const float* min_ps,
                                           const int64_t* seeds, const int64_t* positions, int32_t max_top_k,
                                           int64_t* out, uint8_t* rep_mask_update, void* stream) {
  if (rows < 0) return set_error(OMNI_ERR_INVALID, "rows must be >= 0");
  if (vocab < 32 || vocab > 8192 || vocab % 4 != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "vocab must be a multiple of 4 in [32, 8192]");
  if (max_top_k < 1 || max_top_k > 1024) return set_error(OMNI_ERR_UNSUPPORTED, "max_top_k must be in [1, 1024]");
  const int bk = block_k_of(max_top_k);
  if (bk > vocab) return set_error(OMNI_ERR_UNSUPPORTED, "max_top_k exceeds the vocabulary");
  if ((logits_stride % 4) != 0 || (reinterpret_cast<uintptr_t>(logits) & 15) != 0 ||
      (rep_mask && (reinterpret_cast<uintptr_t>(rep_mask) & 3) != 0) ||
      (suppress_mask && (reinterpret_cast<uintptr_t>(suppress_mask) & 3) != 0))
    return set_error(OMNI_ERR_UNSUPPORTED, "logits rows must be 16-byte aligned");
  if (rows == 0) return OMNI_OK;
  Layer0Params p = {logits, logits_stride, (int)vocab, penalties, rep_mask, suppress_mask, temperatures, top_ks,
                    top_ps, min_ps, seeds, positions, bk, out, rep_mask_update};
  const int J = (int)((vocab + 1023) / 1024);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 g((unsigned)rows), b(kThreads);
#define OMNI_L0(JJ)                                                               \
  case JJ:                                                                        \
    switch (bk) {                                                                 \
      case 32: return check_launch(launch(layer0_sample_kernel<JJ, 1>, g, b, 0, st, p));   \
      case 64: return check_launch(launch(layer0_sample_kernel<JJ, 2>, g, b, 0, st, p));   \
      case 128: return check_launch(launch(layer0_sample_kernel<JJ, 4>, g, b, 0, st, p));  \
      case 256: return check_launch(launch(layer0_sample_kernel<JJ, 8>, g, b, 0, st, p));  \
      case 512: return check_launch(launch(layer0_sample_kernel<JJ, 16>, g, b, 0, st, p)); \
      case 1024: return check_launch(launch(layer0_sample_kernel<JJ, 32>, g, b, 0, st, p)); \
    }                                                                             \
    break;
  switch (J) {
    OMNI_L0(1)
    OMNI_L0(2)
    OMNI_L0(3)
    OMNI_L0(4)
    OMNI_L0(8)
    default:
      break;
  }
#undef OMNI_L0
  if (J > 4 && J < 8) {
    // widths 5-7 pages run the 8-page variant (tails masked)
    switch (bk) {
      case 32: return check_launch(launch(layer0_sample_kernel<8, 1>, g, b, 0, st, p));
      case 64: return check_launch(launch(layer0_sample_kernel<8, 2>, g, b, 0, st, p));
      case 128: return check_launch(launch(layer0_sample_kernel<8, 4>, g, b, 0, st, p));
      case 256: return check_launch(launch(layer0_sample_kernel<8, 8>, g, b, 0, st, p));
      case 512: return check_launch(launch(layer0_sample_kernel<8, 16>, g, b, 0, st, p));
      case 1024: return check_launch(launch(layer0_sample_kernel<8, 32>, g, b, 0, st, p));
    }
  }
  return set_error(OMNI_ERR_UNSUPPORTED, "unsupported layer-0 vocab");
}

// ---------------------------------------------------------------------------
// Opening inputs of the code predictor for one frame.  The talker's final
// RMSNorm is applied here (its gain and the per-row sums of squares of the
// talker's last residual): hidden = bf16(h * rstd * gain) is written to the
// caller's hidden rows and to pair row 2r; the layer-0 code's embedding goes
// to pair row 2r + 1 and to summed; both pair rows' sums of squares are written.
// ---------------------------------------------------------------------------
namespace omni {
namespace {
__global__ void __launch_bounds__(128) predictor_pair_inputs_kernel(
    const int64_t* __restrict__ c0, const uint16_t* __restrict__ h, int64_t h_stride,
    const uint16_t* __restrict__ final_norm, const float* __restrict__ ss_in, int ss_parts, int64_t ss_stride,
    float eps, uint16_t* __restrict__ hidden_out, const uint16_t* __restrict__ table, int H,
    uint16_t* __restrict__ pair, uint16_t* __restrict__ summed, float* __restrict__ pair_ss,
    int64_t* __restrict__ codes, int64_t codes_stride) {
  __shared__ float red[2][4];
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t code = c0[row];
  if (threadIdx.x == 0) codes[row * codes_stride] = code;
  // final_norm == nullptr: h is already the normalized hidden state (copied unchanged)
  const bool norm = final_norm != nullptr;
  float rstd = 1.0f;
  if (norm) {
    float tot = 0.0f;
    for (int q = 0; q < ss_parts; ++q) tot += ss_in[q * ss_stride + row];
    rstd = rsqrtf(tot / (float)H + eps);
  }
  const uint4* e = reinterpret_cast<const uint4*>(table + code * H);
  const uint4* hs = reinterpret_cast<const uint4*>(h + row * h_stride);
  const uint4* gw = reinterpret_cast<const uint4*>(final_norm);
  uint4* p0 = reinterpret_cast<uint4*>(pair + (int64_t)(2 * row) * H);
  uint4* p1 = reinterpret_cast<uint4*>(pair + (int64_t)(2 * row + 1) * H);
  uint4* sm = reinterpret_cast<uint4*>(summed + (int64_t)row * H);
  uint4* ho = hidden_out ? reinterpret_cast<uint4*>(hidden_out + (int64_t)row * H) : nullptr;
  float ss0 = 0.0f, ss1 = 0.0f;
  for (int v = threadIdx.x; v < H / 8; v += 128) {
    const uint4 hv = hs[v], gv = norm ? gw[v] : make_uint4(0u, 0u, 0u, 0u), w = e[v];
    const uint32_t hx[4] = {hv.x, hv.y, hv.z, hv.w}, gx[4] = {gv.x, gv.y, gv.z, gv.w}, wx[4] = {w.x, w.y, w.z, w.w};
    uint32_t nx[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      nx[q] = norm ? pack_bf2(bf_lo(hx[q]) * rstd * bf_lo(gx[q]), bf_hi(hx[q]) * rstd * bf_hi(gx[q])) : hx[q];
      ss0 = __fmaf_rn(bf_lo(nx[q]), bf_lo(nx[q]), ss0);
      ss0 = __fmaf_rn(bf_hi(nx[q]), bf_hi(nx[q]), ss0);
      ss1 = __fmaf_rn(bf_lo(wx[q]), bf_lo(wx[q]), ss1);
      ss1 = __fmaf_rn(bf_hi(wx[q]), bf_hi(wx[q]), ss1);
    }
    const uint4 n = make_uint4(nx[0], nx[1], nx[2], nx[3]);
    p0[v] = n;
    if (ho) ho[v] = n;
    p1[v] = w;
    sm[v] = w;
  }
  ss0 = warp_sum_xor(ss0);
  ss1 = warp_sum_xor(ss1);
  if (lane == 0) {
    red[0][warp] = ss0;
    red[1][warp] = ss1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    pair_ss[2 * row] = red[0][0] + red[0][1] + red[0][2] + red[0][3];
    pair_ss[2 * row + 1] = red[1][0] + red[1][1] + red[1][2] + red[1][3];
  }
}
}  // namespace
}  // namespace omni

extern "C" OMNI_API int omni_predictor_pair_inputs(const int64_t* layer0_codes, const void* talker_residual,
                                                   int64_t residual_stride, const void* final_norm_weight,
                                                   const float* ss_in, int32_t ss_parts, int64_t ss_stride,
                                                   float eps, void* hidden_out, const void* table, int64_t rows,
                                                   int64_t hidden, void* pair, void* summed, float* pair_ss,
                                                   int64_t* codes, int64_t codes_stride, void* stream) {
  if (rows < 0 || hidden <= 0 || !pair_ss || (final_norm_weight && (ss_parts <= 0 || !ss_in)))
    return omni::set_error(OMNI_ERR_INVALID, "bad shape");
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (hidden % 8 || residual_stride % 8 || mis(talker_residual) || mis(table) || mis(pair) || mis(summed) ||
      mis(final_norm_weight) || (hidden_out && mis(hidden_out)))
    return omni::set_error(OMNI_ERR_UNSUPPORTED, "rows must be 16-byte aligned");
  if (rows == 0) return OMNI_OK;
  return omni::check_launch(omni::launch(
      omni::predictor_pair_inputs_kernel, dim3((unsigned)rows), dim3(128), 0, static_cast<cudaStream_t>(stream),
      layer0_codes, static_cast<const uint16_t*>(talker_residual), residual_stride,
      static_cast<const uint16_t*>(final_norm_weight), ss_in, (int)ss_parts, ss_stride, eps,
      static_cast<uint16_t*>(hidden_out), static_cast<const uint16_t*>(table), (int)hidden,
      static_cast<uint16_t*>(pair), static_cast<uint16_t*>(summed), pair_ss, codes, codes_stride));
}
