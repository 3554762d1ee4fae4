/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of the integer/byte and sampling arithmetic of the
 * SGLang-Omni talker decode step.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load this library; the product path
 * (sglang-omni_b200/) never links or calls it.
 *
 * Parity pins: the hash and the Gumbel endpoints are checked against the
 * reference's own golden vectors (tests/golden/, produced by executing the
 * reference's pure-torch functions); the residual sampler against the
 * reference's torch fallback executed on CPU; the argmax, penalty and
 * rollback known answers against the reference's unit tests.
 *
 * Floating-point conventions (so that a GPU implementation of the same
 * specification can be compared bit for bit):
 *   - compiled with -ffp-contract=off: no implicit FMA; fmaf/fma only where
 *     written;
 *   - exp/log are this file's own functions (Cody–Waite reduction + Taylor
 *     series for exp, the atanh series for log), not libm;
 *   - every reduction uses the fixed order documented at its definition.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#include <float.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* bf16 <-> f32                                                              */
/* ------------------------------------------------------------------------ */
static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    /* round to nearest even; NaN kept quiet */
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint64_t d2u(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }
static inline double u2d(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }

/* ------------------------------------------------------------------------ */
/* MurmurHash3 x86_32 mixing (Austin Appleby, public domain), fed            */
/* (seed lo, seed hi, position, column) and finalised with length 16.        */
/* Follows sglang_omni/models/qwen3_tts/sampling_kernels.py:633-677.         */
/* ------------------------------------------------------------------------ */
static inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

static inline uint32_t mm3_mix(uint32_t h, uint32_t k) {
    k *= 0xCC9E2D51u;
    k = rotl32(k, 15);
    k *= 0x1B873593u;
    h ^= k;
    h = rotl32(h, 13);
    return h * 5u + 0xE6546B64u;
}

static inline uint32_t mm3_fmix(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85EBCA6Bu;
    h ^= h >> 13;
    h *= 0xC2B2AE35u;
    h ^= h >> 16;
    return h;
}

ORC_API uint32_t orc_hash(int64_t seed, int64_t position, uint32_t column) {
    uint64_t s = (uint64_t)seed;
    uint32_t h = 0;
    h = mm3_mix(h, (uint32_t)(s & 0xFFFFFFFFu));
    h = mm3_mix(h, (uint32_t)(s >> 32));
    h = mm3_mix(h, (uint32_t)((uint64_t)position & 0xFFFFFFFFu));
    h = mm3_mix(h, column);
    h ^= 16u;
    return mm3_fmix(h);
}

/* ------------------------------------------------------------------------ */
/* exp / log.                                                                */
/* expf: x = n ln2 + r, |r| <= ln2/2 (Cody & Waite two-constant reduction),  */
/*       e^r by its Taylor series to degree 7 in Horner form with fmaf,      */
/*       scaled by 2^n through the exponent field.                           */
/* logf/log: x = 2^e m, m in [sqrt(1/2), sqrt(2)), s = (m-1)/(m+1),          */
/*       log m = 2 atanh(s) = 2(s + s^3/3 + s^5/5 + ...), + e ln2.           */
/* ------------------------------------------------------------------------ */
static const float ORC_LOG2E_F = 0x1.715476p+0f;
static const float ORC_LN2_HI_F = 0x1.62e4p-1f;   /* 13 significant bits */
static const float ORC_LN2_LO_F = 0x1.7f7d1cp-20f; /* ln2 - hi, rounded */

static inline float scale_pow2_f(float p, int n) {
    /* p in [0.7, 1.5]; returns p * 2^n with one rounding at most */
    if (n > 127) { p = p * u2f(0x7F000000u); n -= 127; if (n > 127) n = 127; }
    if (n < -126) {
        p = p * u2f(0x00800000u); /* 2^-126 */
        n += 126;
        if (n < -126) n = -126;
    }
    return p * u2f((uint32_t)(n + 127) << 23);
}

ORC_API float orc_expf(float x) {
    if (x != x) return x;
    if (x > 88.7228394f) return INFINITY;
    if (x < -103.972084f) return 0.0f;
    float t = x * ORC_LOG2E_F;
    float n = floorf(t + 0.5f);
    float r = fmaf(-n, ORC_LN2_HI_F, x);
    r = fmaf(-n, ORC_LN2_LO_F, r);
    float p = 0x1.a01a02p-13f; /* 1/7! */
    p = fmaf(p, r, 0x1.6c16c2p-10f); /* 1/6! */
    p = fmaf(p, r, 0x1.111112p-7f); /* 1/5! */
    p = fmaf(p, r, 0x1.555556p-5f); /* 1/4! */
    p = fmaf(p, r, 0x1.555556p-3f); /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return scale_pow2_f(p, (int)n);
}

ORC_API float orc_logf(float x) {
    if (x != x) return x;
    if (x < 0.0f) return NAN;
    if (x == 0.0f) return -INFINITY;
    if (x == INFINITY) return INFINITY;
    uint32_t u = f2u(x);
    int e = 0;
    if ((u & 0x7F800000u) == 0) { /* subnormal */
        x = x * 8388608.0f;      /* 2^23 */
        u = f2u(x);
        e = -23;
    }
    e += (int)((u >> 23) & 0xFF) - 127;
    float m = u2f((u & 0x007FFFFFu) | 0x3F800000u); /* [1, 2) */
    if (m > 0x1.6a09e6p+0f) { m = m * 0.5f; e += 1; } /* sqrt 2 */
    float s = (m - 1.0f) / (m + 1.0f);
    float s2 = s * s;
    float q = 0x1.c71c72p-3f; /* 2/9 */
    q = fmaf(q, s2, 0x1.24924ap-2f); /* 2/7 */
    q = fmaf(q, s2, 0x1.99999ap-2f); /* 2/5 */
    q = fmaf(q, s2, 0x1.555556p-1f); /* 2/3 */
    float lm = fmaf(s * s2, q, 2.0f * s);
    float fe = (float)e;
    return fmaf(fe, ORC_LN2_HI_F, fmaf(fe, ORC_LN2_LO_F, lm));
}

static const double ORC_LN2_HI_D = 0x1.62e42feep-1; /* ln2, leading 33 bits */
static const double ORC_LN2_LO_D = 0x1.a39ef35793c76p-33; /* ln2 - hi */

ORC_API double orc_log(double x) {
    if (x != x) return x;
    if (x < 0.0) return NAN;
    if (x == 0.0) return -INFINITY;
    if (x == INFINITY) return INFINITY;
    uint64_t u = d2u(x);
    int e = 0;
    if ((u & 0x7FF0000000000000ull) == 0) {
        x = x * 18014398509481984.0; /* 2^54 */
        u = d2u(x);
        e = -54;
    }
    e += (int)((u >> 52) & 0x7FF) - 1023;
    double m = u2d((u & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull);
    if (m > 0x1.6a09e667f3bcdp+0) { m = m * 0.5; e += 1; } /* sqrt 2 */
    double s = (m - 1.0) / (m + 1.0);
    double s2 = s * s;
    double q = 0x1.47ae147ae147bp-4; /* 2/25 */
    q = fma(q, s2, 0x1.642c8590b2164p-4); /* 2/23 */
    q = fma(q, s2, 0x1.8618618618618p-4); /* 2/21 */
    q = fma(q, s2, 0x1.af286bca1af28p-4); /* 2/19 */
    q = fma(q, s2, 0x1.e1e1e1e1e1e1ep-4); /* 2/17 */
    q = fma(q, s2, 0x1.1111111111111p-3); /* 2/15 */
    q = fma(q, s2, 0x1.3b13b13b13b14p-3); /* 2/13 */
    q = fma(q, s2, 0x1.745d1745d1746p-3); /* 2/11 */
    q = fma(q, s2, 0x1.c71c71c71c71cp-3); /* 2/9 */
    q = fma(q, s2, 0x1.2492492492492p-2); /* 2/7 */
    q = fma(q, s2, 0x1.999999999999ap-2); /* 2/5 */
    q = fma(q, s2, 0x1.5555555555555p-1); /* 2/3 */
    double lm = fma(s * s2, q, 2.0 * s);
    double de = (double)e;
    return fma(de, ORC_LN2_HI_D, fma(de, ORC_LN2_LO_D, lm));
}

/* Gumbel noise of one hash value, float64, with sglang multinomial_with_seed's
 * endpoint handling: log u clamped to [-DBL_MAX, -2^-32] before the second log
 * (sampling_kernels.py:67-78). */
ORC_API double orc_gumbel(uint32_t h) {
    double u = (double)h / 4294967295.0;
    double lu = orc_log(u);
    if (lu < -DBL_MAX) lu = -DBL_MAX;
    if (lu > -2.3283064365386963e-10) lu = -2.3283064365386963e-10;
    return -orc_log(-lu);
}

/* ------------------------------------------------------------------------ */
/* Ordered keys: float bits mapped so that unsigned order == float order     */
/* (+0 above -0, positive NaN above +inf); sampling_kernels.py:314-338.      */
/* ------------------------------------------------------------------------ */
static inline uint32_t ordered_bits(float f) {
    uint32_t b = f2u(f);
    return (b >> 31) ? ~b : (b | 0x80000000u);
}
static inline float unordered_float(uint32_t o) {
    uint32_t b = (o >> 31) ? (o & 0x7FFFFFFFu) : ~o;
    return u2f(b);
}

static int cmp_u64_desc(const void* a, const void* b) {
    uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return (x < y) - (x > y);
}

/* The 32-lane reductions used after selection.  C = n/32 consecutive ranks
 * per lane; lane partials are sequential left folds; lanes are combined by a
 * Hillis–Steele inclusive scan with offsets 1, 2, 4, 8, 16. */
static void lane_scan_incl(const float* lane_vals, float* out) {
    float v[32], t[32];
    for (int l = 0; l < 32; ++l) v[l] = lane_vals[l];
    for (int off = 1; off < 32; off <<= 1) {
        for (int l = 0; l < 32; ++l) t[l] = (l >= off) ? v[l] + v[l - off] : v[l];
        for (int l = 0; l < 32; ++l) v[l] = t[l];
    }
    for (int l = 0; l < 32; ++l) out[l] = v[l];
}

/* Sample one row from candidates sorted by rank (sampling_kernels.py:385-438;
 * sglang_model.py:1987-2034).  n is a multiple of 32, <= 1024. */
static int64_t sample_sorted_candidates(const float* sorted_scores, const int64_t* sorted_ids, int n,
                                        int64_t top_k, float top_p, int has_top_p, int64_t seed,
                                        int64_t position) {
    float masked[1024], e[1024], p[1024], cdf[1024];
    int keep[1024];
    float mx = -INFINITY;
    for (int r = 0; r < n; ++r) {
        keep[r] = (int64_t)r < top_k;
        masked[r] = keep[r] ? sorted_scores[r] : -INFINITY;
        if (masked[r] > mx) mx = masked[r];
    }
    const int C = n / 32;
    float lane_part[32], lane_incl[32];
    for (int r = 0; r < n; ++r) e[r] = orc_expf(masked[r] - mx);
    for (int l = 0; l < 32; ++l) {
        float acc = e[l * C];
        for (int j = 1; j < C; ++j) acc = acc + e[l * C + j];
        lane_part[l] = acc;
    }
    lane_scan_incl(lane_part, lane_incl);
    float total = lane_incl[31];
    for (int r = 0; r < n; ++r) p[r] = e[r] / total;
    if (has_top_p) {
        float q[1024];
        for (int l = 0; l < 32; ++l) {
            float acc = p[l * C];
            q[l * C] = acc;
            for (int j = 1; j < C; ++j) { acc = acc + p[l * C + j]; q[l * C + j] = acc; }
            lane_part[l] = acc;
        }
        lane_scan_incl(lane_part, lane_incl);
        for (int l = 0; l < 32; ++l) {
            float excl = l == 0 ? 0.0f : lane_incl[l - 1];
            for (int j = 0; j < C; ++j) cdf[l * C + j] = excl + q[l * C + j];
        }
        int active = (top_p > 0.0f) && (top_p < 1.0f);
        for (int r = 1; r < n; ++r)
            if (active && (cdf[r] - p[r] >= top_p)) keep[r] = 0;
    }
    int best_rank = 0;
    double best = 0.0;
    for (int r = 0; r < n; ++r) {
        float lp = keep[r] ? orc_logf(p[r]) : -INFINITY;
        double v = (double)lp + orc_gumbel(orc_hash(seed, position, (uint32_t)r));
        if (r == 0 || v > best) { best = v; best_rank = r; }
    }
    return sorted_ids[best_rank];
}

/* One compare-exchange round of torch.topk's 32-entry descending bitonic
 * network (sampling_kernels.py:123-167). */
static void bitonic32_round(float* sc, int64_t* id, int* valid, int stride, int network_size, int final_round) {
    float nsc[32];
    int64_t nid[32];
    int nvalid[32];
    for (int o = 0; o < 32; ++o) {
        int partner = o ^ stride;
        int is_right = (o & stride) != 0;
        float left_s = is_right ? sc[partner] : sc[o];
        float right_s = is_right ? sc[o] : sc[partner];
        int left_v = is_right ? valid[partner] : valid[o];
        int right_v = is_right ? valid[o] : valid[partner];
        int direction;
        if (final_round) {
            direction = 0;
        } else {
            int left_off = o - (is_right ? stride : 0);
            int thread_id = (left_off / (2 * stride)) * stride + (left_off % stride);
            direction = (thread_id & (network_size / 2)) != 0;
        }
        int should_swap = ((left_s > right_s) && left_v) || (right_v == 0);
        int take_partner = (should_swap == direction);
        nsc[o] = take_partner ? sc[partner] : sc[o];
        nid[o] = take_partner ? id[partner] : id[o];
        nvalid[o] = take_partner ? valid[partner] : valid[o];
    }
    memcpy(sc, nsc, sizeof(nsc));
    memcpy(id, nid, sizeof(nid));
    memcpy(valid, nvalid, sizeof(nvalid));
}

static void bitonic32_sort(float* sc, int64_t* id, int max_top_k) {
    static const int rounds[15][3] = {
        {1, 2, 0}, {2, 4, 0}, {1, 4, 0}, {4, 8, 0}, {2, 8, 0}, {1, 8, 0}, {8, 16, 0}, {4, 16, 0},
        {2, 16, 0}, {1, 16, 0}, {16, 32, 1}, {8, 32, 1}, {4, 32, 1}, {2, 32, 1}, {1, 32, 1}};
    int valid[32];
    for (int o = 0; o < 32; ++o) valid[o] = o < max_top_k;
    for (int i = 0; i < 15; ++i) bitonic32_round(sc, id, valid, rounds[i][0], rounds[i][1], rounds[i][2]);
}

/* Smallest power of two >= max_top_k, with 32 for every width <= 32
 * (sampling_kernels.py:792-804). */
static int block_k_of(int max_top_k) {
    if (max_top_k <= 32) return 32;
    int b = 1;
    while (b < max_top_k) b <<= 1;
    return b;
}

/* Residual-codebook sampler: sample_from_logits_with_seed_top_k_top_p
 * (sampling_kernels.py:836-950; math of its torch fallback
 * sglang_model.py:1987-2034 and kernel :441-529).
 * logits: bf16 [rows, stride]; out: int64 [rows]. */
ORC_API int orc_sample_topk_topp(const uint16_t* logits, int64_t rows, int64_t vocab, int64_t stride,
                                 const float* temperatures, const int64_t* top_ks, const float* top_ps,
                                 const int64_t* seeds, const int64_t* positions, int max_top_k,
                                 int has_top_p, int64_t* out) {
    if (max_top_k < 1 || max_top_k > 1024 || vocab < 32 || vocab > 65536) return 1;
    int bk = block_k_of(max_top_k);
    if (bk > vocab) return 1;
    float* scores = (float*)malloc(sizeof(float) * vocab);
    uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * vocab);
    for (int64_t row = 0; row < rows; ++row) {
        const uint16_t* lg = logits + row * stride;
        float t = temperatures[row];
        if (!(t >= 1e-5f)) t = (t != t) ? t : 1e-5f;
        for (int64_t v = 0; v < vocab; ++v) {
            scores[v] = bf16_to_f32(lg[v]) / t;
            keys[v] = ((uint64_t)ordered_bits(scores[v]) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)v);
        }
        qsort(keys, (size_t)vocab, sizeof(uint64_t), cmp_u64_desc);
        float sorted_sc[1024];
        int64_t sorted_id[1024];
        if (max_top_k <= 32) {
            uint32_t thr = (uint32_t)(keys[max_top_k - 1] >> 32);
            int n = 0;
            for (int cls = 0; cls < 3 && n < 32; ++cls) {
                for (int64_t v = 0; v < vocab && n < 32; ++v) {
                    uint32_t o = ordered_bits(scores[v]);
                    int c = o > thr ? 0 : (o == thr ? 1 : 2);
                    if (c == cls) { sorted_sc[n] = scores[v]; sorted_id[n] = v; ++n; }
                }
            }
            bitonic32_sort(sorted_sc, sorted_id, max_top_k);
        } else {
            for (int r = 0; r < bk; ++r) {
                sorted_sc[r] = unordered_float((uint32_t)(keys[r] >> 32));
                sorted_id[r] = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[r] & 0xFFFFFFFFu));
            }
        }
        out[row] = sample_sorted_candidates(sorted_sc, sorted_id, bk, top_ks[row], top_ps[row], has_top_p,
                                            seeds[row], positions[row]);
    }
    free(scores);
    free(keys);
    return 0;
}

/* sample_from_sorted_logprobs_with_seed_small_k (sampling_kernels.py:81-121,
 * :721-790): Gumbel-max over given fp32 log-probabilities, columns = ranks. */
ORC_API int orc_sample_sorted(const float* logprobs, const int64_t* sorted_idx, int64_t rows, int64_t cols,
                              const int64_t* seeds, const int64_t* positions, int64_t* out) {
    if (cols <= 0 || cols > 1024) return 1;
    for (int64_t row = 0; row < rows; ++row) {
        int64_t best_rank = 0;
        double best = 0.0;
        for (int64_t c = 0; c < cols; ++c) {
            double v = (double)logprobs[row * cols + c] +
                       orc_gumbel(orc_hash(seeds[row], positions[row], (uint32_t)c));
            if (c == 0 || v > best) { best = v; best_rank = c; }
        }
        out[row] = sorted_idx[row * cols + best_rank];
    }
    return 0;
}

/* argmax with torch semantics: the first NaN, else the first maximum
 * (predictor_layers.py:548-584; known answer test_predictor_kernels.py:622-646). */
static int64_t argmax_first(const float* v, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 0; i < n; ++i) {
        if (v[i] != v[i]) return i;
        if (v[i] > v[best]) best = i;
    }
    return best;
}

/* codebook_step (predictor_layers.py:963-993): code = argmax(logits);
 * gathered = table[code]; summed = bf16(f32(summed) + f32(row)). */
ORC_API int orc_codebook_step(const uint16_t* logits, int64_t rows, int64_t vocab, const uint16_t* table,
                              int64_t hidden, int64_t* codes, int64_t codes_stride, uint16_t* gathered,
                              uint16_t* summed) {
    float* tmp = (float*)malloc(sizeof(float) * vocab);
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t v = 0; v < vocab; ++v) tmp[v] = bf16_to_f32(logits[r * vocab + v]);
        int64_t c = argmax_first(tmp, vocab);
        codes[r * codes_stride] = c;
        for (int64_t h = 0; h < hidden; ++h) {
            uint16_t w = table[c * hidden + h];
            if (gathered) gathered[r * hidden + h] = w;
            if (summed) summed[r * hidden + h] = f32_to_bf16(bf16_to_f32(summed[r * hidden + h]) + bf16_to_f32(w));
        }
    }
    free(tmp);
    return 0;
}

/* gather_codec_embedding_and_add (predictor_kernels.py:29-71). */
ORC_API int orc_gather_add(const int64_t* tokens, int64_t rows, const uint16_t* table, int64_t hidden,
                           uint16_t* gathered, uint16_t* summed) {
    for (int64_t r = 0; r < rows; ++r) {
        int64_t c = tokens[r];
        for (int64_t h = 0; h < hidden; ++h) {
            uint16_t w = table[c * hidden + h];
            gathered[r * hidden + h] = w;
            summed[r * hidden + h] = f32_to_bf16(bf16_to_f32(summed[r * hidden + h]) + bf16_to_f32(w));
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Layer-0 codec sampler (a11).  Repetition penalty and suppression as        */
/* talker.py:1376-1390; then temperature, a full-vocabulary softmax, top-k    */
/* by (score desc, index asc), top-p on the cumulative sorted probabilities   */
/* (drop where cdf - p > top_p), min-p, and the seeded Gumbel draw over the   */
/* ranks.  The third-party sglang sampler is not in the reference tree; this  */
/* restatement defines the semantics (parity unpinned for the draw).          */
/* Full-vocabulary reductions: 256 "threads", thread t folds elements         */
/* 4t..4t+3 + 1024 j in (j, element) order; 8 warps reduce by an xor          */
/* butterfly over offsets 16, 8, 4, 2, 1; the 8 warp sums fold in order.     */
/* ------------------------------------------------------------------------ */
static float block_sum_3072(const float* x, int64_t n) {
    float thread_part[256];
    for (int t = 0; t < 256; ++t) {
        float acc = 0.0f;
        int first = 1;
        for (int64_t base = 4 * t; base < n; base += 1024) {
            for (int j = 0; j < 4; ++j) {
                if (first) { acc = x[base + j]; first = 0; }
                else acc = acc + x[base + j];
            }
        }
        thread_part[t] = acc;
    }
    float warp_tot[8];
    for (int w = 0; w < 8; ++w) {
        float v[32], nv[32];
        for (int l = 0; l < 32; ++l) v[l] = thread_part[w * 32 + l];
        for (int off = 16; off >= 1; off >>= 1) {
            for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
            memcpy(v, nv, sizeof(v));
        }
        warp_tot[w] = v[0];
    }
    float s = warp_tot[0];
    for (int w = 1; w < 8; ++w) s = s + warp_tot[w];
    return s;
}

ORC_API int orc_layer0_sample(const float* logits, int64_t rows, int64_t vocab, const float* penalties,
                              const uint8_t* rep_mask, const uint8_t* suppress_mask, const float* temperatures,
                              const int64_t* top_ks, const float* top_ps, const float* min_ps,
                              const int64_t* seeds, const int64_t* positions, int max_top_k, int64_t* out,
                              float* processed /* optional [rows, vocab] penalised+suppressed logits */) {
    if (vocab % 4 != 0 || vocab > 8192 || max_top_k < 1 || max_top_k > 1024) return 1;
    int bk = block_k_of(max_top_k);
    if (bk > vocab) return 1;
    float* s = (float*)malloc(sizeof(float) * vocab);
    float* e = (float*)malloc(sizeof(float) * vocab);
    uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * vocab);
    for (int64_t r = 0; r < rows; ++r) {
        float t = temperatures[r];
        if (!(t >= 1e-5f)) t = (t != t) ? t : 1e-5f;
        float pen = penalties[r];
        float mx = -INFINITY;
        for (int64_t v = 0; v < vocab; ++v) {
            float l = logits[r * vocab + v];
            if (rep_mask && rep_mask[r * vocab + v]) l = l > 0.0f ? l / pen : l * pen;
            if (suppress_mask && suppress_mask[r * vocab + v]) l = -INFINITY;
            if (processed) processed[r * vocab + v] = l;
            s[v] = l / t;
            if (s[v] > mx) mx = s[v];
            keys[v] = ((uint64_t)ordered_bits(s[v]) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)v);
        }
        for (int64_t v = 0; v < vocab; ++v) e[v] = orc_expf(s[v] - mx);
        float z = block_sum_3072(e, vocab);
        qsort(keys, (size_t)vocab, sizeof(uint64_t), cmp_u64_desc);
        float p[1024], q[1024], cdf[1024], lane_part[32], lane_incl[32];
        int64_t ids[1024];
        for (int k = 0; k < bk; ++k) {
            float sc = unordered_float((uint32_t)(keys[k] >> 32));
            ids[k] = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[k] & 0xFFFFFFFFu));
            p[k] = orc_expf(sc - mx) / z;
        }
        const int C = bk / 32;
        for (int l = 0; l < 32; ++l) {
            float acc = p[l * C];
            q[l * C] = acc;
            for (int j = 1; j < C; ++j) { acc = acc + p[l * C + j]; q[l * C + j] = acc; }
            lane_part[l] = acc;
        }
        lane_scan_incl(lane_part, lane_incl);
        for (int l = 0; l < 32; ++l) {
            float excl = l == 0 ? 0.0f : lane_incl[l - 1];
            for (int j = 0; j < C; ++j) cdf[l * C + j] = excl + q[l * C + j];
        }
        float top_p = top_ps[r];
        float min_p = min_ps ? min_ps[r] : 0.0f;
        float min_thr = p[0] * min_p;
        int best_rank = 0;
        double best = 0.0;
        for (int k = 0; k < bk; ++k) {
            int keep = (int64_t)k < top_ks[r];
            if (cdf[k] - p[k] > top_p) keep = 0;
            if (min_p > 0.0f && p[k] < min_thr) keep = 0;
            float lp = (keep && p[k] > 0.0f) ? orc_logf(p[k]) : -INFINITY;
            double v = (double)lp + orc_gumbel(orc_hash(seeds[r], positions[r], (uint32_t)k));
            if (k == 0 || v > best) { best = v; best_rank = k; }
        }
        out[r] = ids[best_rank];
    }
    free(s);
    free(e);
    free(keys);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Decode batch packing (a1, a2).                                            */
/* prepare_for_decode: seq_len += 1; a row whose new token opens a page      */
/* ((seq_len-1) % P == 0) takes the next free page, in row order; the new    */
/* slot is page*P + (seq_len-1) % P, else last slot + 1; req_to_token is     */
/* written; positions = seq_len - 1 (talker_scheduler.py:198-225 states the  */
/* page rule in reverse).  Then the attention metadata: kv_indptr =          */
/* cumsum(seq_lens), kv_indices = req_to_token rows, and the page-level       */
/* view page_indptr / page_indices.                                          */
/* ------------------------------------------------------------------------ */
ORC_API int orc_decode_prepare(int64_t rows, int64_t* seq_lens, const int64_t* req_pool_indices,
                               int32_t* req_to_token, int64_t max_ctx, int64_t page_size,
                               const int32_t* free_pages, int64_t num_free, int64_t* free_head,
                               int64_t* out_cache_loc, int64_t* positions, int32_t* kv_indptr,
                               int32_t* kv_indices, int32_t* page_indptr, int32_t* page_indices) {
    for (int64_t i = 0; i < rows; ++i) {
        int64_t L = seq_lens[i] + 1;
        if (L > max_ctx) return 3;
        int64_t req = req_pool_indices[i];
        int64_t loc;
        if ((L - 1) % page_size == 0) {
            if (*free_head >= num_free) return 3;
            loc = (int64_t)free_pages[(*free_head)++] * page_size;
        } else {
            loc = (int64_t)req_to_token[req * max_ctx + (L - 2)] + 1;
        }
        req_to_token[req * max_ctx + (L - 1)] = (int32_t)loc;
        seq_lens[i] = L;
        out_cache_loc[i] = loc;
        positions[i] = L - 1;
    }
    int64_t acc = 0, pacc = 0;
    kv_indptr[0] = 0;
    page_indptr[0] = 0;
    for (int64_t i = 0; i < rows; ++i) {
        int64_t req = req_pool_indices[i];
        int64_t L = seq_lens[i];
        for (int64_t t = 0; t < L; ++t) kv_indices[acc + t] = req_to_token[req * max_ctx + t];
        int64_t np = (L + page_size - 1) / page_size;
        for (int64_t p = 0; p < np; ++p)
            page_indices[pacc + p] = req_to_token[req * max_ctx + p * page_size] / (int32_t)page_size;
        acc += L;
        pacc += np;
        kv_indptr[i + 1] = (int32_t)acc;
        page_indptr[i + 1] = (int32_t)pacc;
    }
    return 0;
}

/* rollback_decode_prep_after_skip (talker_scheduler.py:198-225): return the
 * pages this step opened to the free list (row order), decrement seq_lens
 * and clear req_to_token at the rolled-back position.  Returns the number of
 * freed pages written to freed_pages. */
ORC_API int64_t orc_decode_rollback(int64_t rows, int64_t* seq_lens, const int64_t* req_pool_indices,
                                    int32_t* req_to_token, int64_t max_ctx, int64_t page_size,
                                    const int64_t* out_cache_loc, int64_t* freed_slots) {
    int64_t nfree = 0;
    for (int64_t i = 0; i < rows; ++i) {
        int64_t L = seq_lens[i];
        if (page_size > 1) {
            if ((L - 1) % page_size == 0) freed_slots[nfree++] = out_cache_loc[i];
        } else {
            freed_slots[nfree++] = out_cache_loc[i];
        }
    }
    for (int64_t i = 0; i < rows; ++i) {
        seq_lens[i] -= 1;
        req_to_token[req_pool_indices[i] * max_ctx + seq_lens[i]] = 0;
    }
    return nfree;
}

/* ------------------------------------------------------------------------ */
/* MoE routing (a9): softmax over experts (fp32), top-k by (prob desc, index */
/* asc), renormalised (norm_topk_prob).  thinker_model.py:428-433;           */
/* hf_config.py:299-304.  Reductions: 32 lanes, lane l holds the contiguous  */
/* experts [l*E/32, (l+1)*E/32) folded in index order; xor butterfly 16..1;  */
/* the top-k weights are summed in selection order.                          */
/* ------------------------------------------------------------------------ */
ORC_API int orc_moe_route(const float* router_logits, int64_t tokens, int64_t experts, int64_t top_k,
                          int renormalize, int32_t* topk_ids, float* topk_weights) {
    if (experts % 32 != 0 || experts > 1024 || top_k < 1 || top_k > 32 || top_k > experts) return 1;
    float p[1024];
    int taken[1024];
    for (int64_t t = 0; t < tokens; ++t) {
        const float* lg = router_logits + t * experts;
        float mx = -INFINITY;
        for (int64_t e = 0; e < experts; ++e) if (lg[e] > mx) mx = lg[e];
        int per = (int)(experts / 32);
        float v[32], nv[32];
        for (int l = 0; l < 32; ++l) {
            float acc = orc_expf(lg[l * per] - mx);
            for (int j = 1; j < per; ++j) acc = acc + orc_expf(lg[l * per + j] - mx);
            v[l] = acc;
        }
        for (int off = 16; off >= 1; off >>= 1) {
            for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
            memcpy(v, nv, sizeof(v));
        }
        float z = v[0];
        for (int64_t e = 0; e < experts; ++e) { p[e] = orc_expf(lg[e] - mx) / z; taken[e] = 0; }
        float wsum = 0.0f;
        for (int64_t k = 0; k < top_k; ++k) {
            int64_t best = -1;
            for (int64_t e = 0; e < experts; ++e) {
                if (taken[e]) continue;
                if (best < 0 || ordered_bits(p[e]) > ordered_bits(p[best])) best = e;
            }
            taken[best] = 1;
            topk_ids[t * top_k + k] = (int32_t)best;
            topk_weights[t * top_k + k] = p[best];
            wsum = (k == 0) ? p[best] : wsum + p[best];
        }
        if (renormalize)
            for (int64_t k = 0; k < top_k; ++k) topk_weights[t * top_k + k] = topk_weights[t * top_k + k] / wsum;
    }
    return 0;
}

/* Expert permutation: a stable counting sort of the (token, slot) pairs by
 * expert id.  expert_offsets[E+1]; sorted_pairs[T*k] = token*k + slot. */
ORC_API int orc_moe_permute(const int32_t* topk_ids, int64_t tokens, int64_t top_k, int64_t experts,
                            int32_t* expert_offsets, int32_t* sorted_pairs) {
    for (int64_t e = 0; e <= experts; ++e) expert_offsets[e] = 0;
    for (int64_t i = 0; i < tokens * top_k; ++i) expert_offsets[topk_ids[i] + 1]++;
    for (int64_t e = 0; e < experts; ++e) expert_offsets[e + 1] += expert_offsets[e];
    int32_t* fill = (int32_t*)malloc(sizeof(int32_t) * experts);
    for (int64_t e = 0; e < experts; ++e) fill[e] = expert_offsets[e];
    for (int64_t i = 0; i < tokens * top_k; ++i) sorted_pairs[fill[topk_ids[i]]++] = (int32_t)i;
    free(fill);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* FP8 e4m3 (OCP "e4m3fn": bias 7, no infinities, max 448) and the per-token */
/* 128-group activation quantisation of the block-FP8 MoE path               */
/* (sglang per_token_group_quant_fp8, called from FusedMoE with              */
/* quantization.py:124-167's block config):                                  */
/*   amax = max(max|x_g|, 1e-10); scale = amax / 448;                        */
/*   q = e4m3(clamp(x / scale, -448, 448)), round to nearest even.           */
/* ------------------------------------------------------------------------ */
ORC_API uint8_t orc_e4m3_from_f32(float x) {
    uint32_t u = f2u(x);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80);
    if (x != x) return (uint8_t)(sign | 0x7F);
    float a = fabsf(x);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7E); /* saturate */
    if (a < 0.015625f) {                             /* below 2^-6: subnormal, quantum 2^-9 */
        float q = a * 512.0f;                        /* exact (power-of-two scale) */
        float r = rintf(q);                          /* nearest even */
        int m = (int)r;                              /* 0..8; 8 is the smallest normal */
        return (uint8_t)(sign | (uint8_t)m);
    }
    int e;
    frexpf(a, &e);                                   /* a = f * 2^e, f in [0.5, 1) */
    int E = e - 1;                                   /* a in [2^E, 2^(E+1)) */
    float q = ldexpf(a, 3 - E);                      /* [8, 16): exact */
    float r = rintf(q);
    int m = (int)r;
    if (m == 16) { m = 8; E += 1; }
    if (E > 8) return (uint8_t)(sign | 0x7E);
    uint8_t bits = (uint8_t)(((E + 7) << 3) | (m - 8));
    if (bits > 0x7E) bits = 0x7E;
    return (uint8_t)(sign | bits);
}

ORC_API float orc_e4m3_to_f32(uint8_t b) {
    float s = (b & 0x80) ? -1.0f : 1.0f;
    int E = (b >> 3) & 0xF, m = b & 7;
    if (E == 15 && m == 7) return NAN;
    if (E == 0) return s * ldexpf((float)m, -9);
    return s * ldexpf((float)(8 + m), E - 10);
}

/* x: rows x cols fp32 (bf16 values); group divides cols.  q: rows x cols
 * e4m3 bytes; scales: rows x (cols / group) fp32. */
ORC_API int orc_quant_fp8_group(const float* x, int64_t rows, int64_t cols, int64_t group, uint8_t* q,
                                float* scales) {
    if (group <= 0 || cols % group != 0) return 1;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t g = 0; g < cols / group; ++g) {
            const float* xs = x + r * cols + g * group;
            float amax = 0.0f;
            for (int64_t i = 0; i < group; ++i) { float a = fabsf(xs[i]); if (a > amax) amax = a; }
            if (amax < 1e-10f) amax = 1e-10f;
            const float sc = amax / 448.0f;
            scales[r * (cols / group) + g] = sc;
            for (int64_t i = 0; i < group; ++i) {
                float v = xs[i] / sc;
                if (v > 448.0f) v = 448.0f;
                if (v < -448.0f) v = -448.0f;
                q[r * cols + g * group + i] = orc_e4m3_from_f32(v);
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Extend packing (prepare_for_extend + ForwardBatch.init_new in extend mode, */
/* model_runner/base.py:577-623) for slots the scheduler reserved in         */
/* req_to_token: seq_len = prefix + extend; qo_indptr = cumsum(extend);      */
/* token j of row i: out_cache_loc = req_to_token[req, prefix + j],          */
/* position = prefix + j; page list = req_to_token[req, k P] / P; q tiles of */
/* q_tile rows: tile_indptr = cumsum(ceil(extend / q_tile)).                 */
/* ------------------------------------------------------------------------ */
ORC_API int orc_extend_prepare(int64_t rows, const int64_t* prefix_lens, const int64_t* extend_lens,
                               const int64_t* req_pool_indices, const int32_t* req_to_token, int64_t max_ctx,
                               int64_t page_size, int64_t q_tile, int64_t* seq_lens, int32_t* qo_indptr,
                               int64_t* out_cache_loc, int64_t* positions, int32_t* page_indptr,
                               int32_t* page_indices, int32_t* tile_indptr) {
    int64_t q = 0, pg = 0, tl = 0;
    for (int64_t i = 0; i < rows; ++i) {
        const int64_t E = extend_lens[i], L = prefix_lens[i] + E;
        if (E < 0 || L > max_ctx) return 1;
        seq_lens[i] = L;
        qo_indptr[i] = (int32_t)q;
        page_indptr[i] = (int32_t)pg;
        tile_indptr[i] = (int32_t)tl;
        const int32_t* r2t = req_to_token + req_pool_indices[i] * max_ctx;
        for (int64_t j = 0; j < E; ++j) {
            out_cache_loc[q + j] = r2t[prefix_lens[i] + j];
            positions[q + j] = prefix_lens[i] + j;
        }
        const int64_t np = (L + page_size - 1) / page_size;
        for (int64_t k = 0; k < np; ++k) page_indices[pg + k] = r2t[k * page_size] / (int32_t)page_size;
        q += E;
        pg += np;
        tl += (E + q_tile - 1) / q_tile;
    }
    qo_indptr[rows] = (int32_t)q;
    page_indptr[rows] = (int32_t)pg;
    tile_indptr[rows] = (int32_t)tl;
    return 0;
}
