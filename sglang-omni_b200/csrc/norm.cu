// Normalisation and rotary kernels of the decode step.
//
// rmsnorm_kernel: one warp per row; lane t holds columns 8t + 256b + j (16-byte
//   vectors), its squares (each rounded, then added: no fused multiply-add) are
//   folded in (b, j) order and combined by an xor butterfly 1, 2, 4, 8, 16 — the
//   reduction tree and rounding of the reference's add_rmsnorm_rounded
//   (sglang_omni/utils/predictor_layers.py:104-142, compiled without fp fusion).
//   Optionally adds a second operand first (bf16 sum, written back to the
//   residual stream): the fused add + RMSNorm of sglang's RMSNorm(x, residual).
//
// qknorm_rope_store_kernel: per (row, head) warp: RMSNorm over head_dim with
//   q_norm / k_norm weights (apply_qk_norm), neox rotary embedding from an fp32
//   cos/sin cache, q written to its own buffer, k and v stored into the KV
//   cache at the row's slot (rope with FusedSetKVBufferArg,
//   thinker_model.py:272-345; predictor_cached_self_attention,
//   sglang_model.py:2168-2233).
#include "capi_util.h"
#include "common.cuh"

namespace omni {
namespace {

// ---------------------------------------------------------------------------
template <int CHUNKS>  // hidden = 256 * CHUNKS
__global__ void __launch_bounds__(128) rmsnorm_kernel(const uint16_t* __restrict__ a, int64_t a_stride,
                                                      const uint16_t* __restrict__ b, int64_t b_stride,
                                                      uint16_t* __restrict__ residual_out, int64_t r_stride,
                                                      const uint16_t* __restrict__ weight, float eps,
                                                      uint16_t* __restrict__ out, int64_t out_stride, int rows) {
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  if (row >= rows) return;
  constexpr int H = 256 * CHUNKS;
  float v[CHUNKS][8];
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int col = 256 * c + 8 * lane;
    uint4 x = *reinterpret_cast<const uint4*>(a + row * a_stride + col);
    uint32_t xs[4] = {x.x, x.y, x.z, x.w};
    if (b) {
      uint4 y = *reinterpret_cast<const uint4*>(b + row * b_stride + col);
      uint32_t ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) xs[q] = pack_bf2(bf_lo(xs[q]) + bf_lo(ys[q]), bf_hi(xs[q]) + bf_hi(ys[q]));
      if (residual_out)
        *reinterpret_cast<uint4*>(residual_out + row * r_stride + col) = make_uint4(xs[0], xs[1], xs[2], xs[3]);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[c][2 * q] = bf_lo(xs[q]);
      v[c][2 * q + 1] = bf_hi(xs[q]);
    }
  }
  float acc = 0.0f;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn(v[c][j], v[c][j]));
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
  const float rstd = rsqrtf(acc / (float)H + eps);
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int col = 256 * c + 8 * lane;
    uint4 w = *reinterpret_cast<const uint4*>(weight + col);
    uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      o[q] = pack_bf2(v[c][2 * q] * rstd * bf_lo(ws[q]), v[c][2 * q + 1] * rstd * bf_hi(ws[q]));
    *reinterpret_cast<uint4*>(out + row * out_stride + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------
struct QkRopeParams {
  const uint16_t* qkv;
  int64_t qkv_stride;
  int rows, hq, hkv, head_dim;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  float eps;
  const float* cos_sin;  // [max_pos, head_dim]: cos (head_dim/2) then sin (head_dim/2)
  int64_t max_pos;
  const int64_t* positions;  // nullable: implicit positions
  const int64_t* cache_loc;  // nullable: implicit slots
  int tokens_per_req, slot_stride, slot_base;
  uint16_t* q_out;
  int64_t q_stride;
  uint16_t* k_cache;
  uint16_t* v_cache;
};

template <int E>  // head_dim = 32 * E
__global__ void __launch_bounds__(128) qknorm_rope_store_kernel(const __grid_constant__ QkRopeParams p) {
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = p.hq + p.hkv;
  const int item = blockIdx.x * 4 + warp;
  if (item >= p.rows * units) return;
  const int row = item / units, u = item % units;
  constexpr int D = 32 * E;
  constexpr int HALF = D / 2;
  int64_t pos, loc;
  if (p.positions) {
    pos = p.positions[row];
    loc = p.cache_loc[row];
  } else {
    const int t = row % p.tokens_per_req;
    pos = p.slot_base + t;
    loc = (int64_t)(row / p.tokens_per_req) * p.slot_stride + p.slot_base + t;
  }
  if (pos < 0 || pos >= p.max_pos) pos = 0;  // out-of-table positions rotate by angle 0 (host validates)
  const bool is_q = u < p.hq;
  const int head = is_q ? u : u - p.hq;
  const uint16_t* src = p.qkv + row * p.qkv_stride + (is_q ? head * D : (p.hq + head) * D);
  const uint16_t* nw = is_q ? p.q_norm : p.k_norm;
  float x[E];
  if constexpr (E == 4) {
    uint2 w = *reinterpret_cast<const uint2*>(src + 4 * lane);
    x[0] = bf_lo(w.x); x[1] = bf_hi(w.x); x[2] = bf_lo(w.y); x[3] = bf_hi(w.y);
  } else if constexpr (E == 2) {
    uint32_t w = *reinterpret_cast<const uint32_t*>(src + 2 * lane);
    x[0] = bf_lo(w); x[1] = bf_hi(w);
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) x[j] = bf2f(src[E * lane + j]);
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < E; ++j) ss = __fmaf_rn(x[j], x[j], ss);
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
  const float rstd = rsqrtf(ss / (float)D + p.eps);
#pragma unroll
  for (int j = 0; j < E; ++j) x[j] = bf2f(f2bf(x[j] * rstd * bf2f(nw[E * lane + j])));
  // neox rotation: element d pairs with d + D/2, held by lane ^ 16
  const float* cs = p.cos_sin + pos * D;
  float y[E];
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const int d = E * lane + j;
    const int i = d % HALF;
    const float c = cs[i], s = cs[HALF + i];
    const float other = __shfl_xor_sync(0xFFFFFFFFu, x[j], 16);
    y[j] = d < HALF ? x[j] * c - other * s : x[j] * c + other * s;
  }
  uint16_t* dst = is_q ? p.q_out + row * p.q_stride + head * D : p.k_cache + (loc * p.hkv + head) * D;
#pragma unroll
  for (int j = 0; j < E; ++j) dst[E * lane + j] = f2bf(y[j]);
  if (!is_q) {
    const uint16_t* vsrc = p.qkv + row * p.qkv_stride + (p.hq + p.hkv + head) * D;
    uint16_t* vdst = p.v_cache + (loc * p.hkv + head) * D;
#pragma unroll
    for (int j = 0; j < E; ++j) vdst[E * lane + j] = vsrc[E * lane + j];
  }
}

// ---------------------------------------------------------------------------
// sum = bf16(a + b) (or a copy of a) and its per-row sum of squares: the input
// row of a decoder stack whose first RMSNorm is folded into the next GEMM.
// ---------------------------------------------------------------------------
template <int CHUNKS>
__global__ void __launch_bounds__(128) add_sumsq_kernel(const uint16_t* __restrict__ a, int64_t a_stride,
                                                        const uint16_t* __restrict__ b, int64_t b_stride,
                                                        uint16_t* __restrict__ sum, int64_t s_stride,
                                                        float* __restrict__ ss_out, int rows) {
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  if (row >= rows) return;
  float acc = 0.0f;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int col = 256 * c + 8 * lane;
    uint4 x = *reinterpret_cast<const uint4*>(a + row * a_stride + col);
    uint32_t xs[4] = {x.x, x.y, x.z, x.w};
    if (b) {
      uint4 y = *reinterpret_cast<const uint4*>(b + row * b_stride + col);
      uint32_t ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) xs[q] = pack_bf2(bf_lo(xs[q]) + bf_lo(ys[q]), bf_hi(xs[q]) + bf_hi(ys[q]));
    }
    *reinterpret_cast<uint4*>(sum + row * s_stride + col) = make_uint4(xs[0], xs[1], xs[2], xs[3]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc = __fmaf_rn(bf_lo(xs[q]), bf_lo(xs[q]), acc);
      acc = __fmaf_rn(bf_hi(xs[q]), bf_hi(xs[q]), acc);
    }
  }
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
  if (lane == 0) ss_out[row] = acc;
}

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int omni_add_sumsq(const void* a, int64_t a_stride, const void* b, int64_t b_stride, void* sum,
                                       int64_t sum_stride, float* ss_out, int64_t rows, int64_t hidden,
                                       void* stream) {
  if (rows < 0 || hidden <= 0 || sum == nullptr || ss_out == nullptr) return set_error(OMNI_ERR_INVALID, "bad shape");
  if (hidden % 256 != 0 || hidden > 8192) return set_error(OMNI_ERR_UNSUPPORTED, "hidden must be 256k, <= 8192");
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (mis(a) || mis(sum) || (b && mis(b)) || a_stride % 8 || sum_stride % 8 || (b && b_stride % 8))
    return set_error(OMNI_ERR_UNSUPPORTED, "rows must be 16-byte aligned");
  if (rows == 0) return OMNI_OK;
  dim3 g((unsigned)((rows + 3) / 4)), bl(128);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto A = static_cast<const uint16_t*>(a);
  auto B = static_cast<const uint16_t*>(b);
  auto S = static_cast<uint16_t*>(sum);
  switch (hidden / 256) {
    case 1: return check_launch(launch(add_sumsq_kernel<1>, g, bl, 0, st, A, a_stride, B, b_stride, S, sum_stride, ss_out, (int)rows));
    case 2: return check_launch(launch(add_sumsq_kernel<2>, g, bl, 0, st, A, a_stride, B, b_stride, S, sum_stride, ss_out, (int)rows));
    case 4: return check_launch(launch(add_sumsq_kernel<4>, g, bl, 0, st, A, a_stride, B, b_stride, S, sum_stride, ss_out, (int)rows));
    case 8: return check_launch(launch(add_sumsq_kernel<8>, g, bl, 0, st, A, a_stride, B, b_stride, S, sum_stride, ss_out, (int)rows));
  }
  return set_error(OMNI_ERR_UNSUPPORTED, "hidden must be 256 x {1,2,4,8}");
}

extern "C" OMNI_API int omni_rmsnorm(const void* x, int64_t x_stride, const void* addend, int64_t addend_stride,
                                     void* residual_out, int64_t residual_stride, const void* weight, float eps,
                                     void* out, int64_t out_stride, int64_t rows, int64_t hidden, void* stream) {
  if (rows < 0 || hidden <= 0) return set_error(OMNI_ERR_INVALID, "bad norm shape");
  if (hidden % 256 != 0 || hidden > 8192) return set_error(OMNI_ERR_UNSUPPORTED, "hidden must be 256k, <= 8192");
  auto mis = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (mis(x) || mis(weight) || mis(out) || (addend && mis(addend)) || (residual_out && mis(residual_out)) ||
      x_stride % 8 || out_stride % 8 || (addend && addend_stride % 8) || (residual_out && residual_stride % 8))
    return set_error(OMNI_ERR_UNSUPPORTED, "rows must be 16-byte aligned");
  if (rows == 0) return OMNI_OK;
  dim3 g((unsigned)((rows + 3) / 4)), b(128);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto A = static_cast<const uint16_t*>(x);
  auto B = static_cast<const uint16_t*>(addend);
  auto R = static_cast<uint16_t*>(residual_out);
  auto W = static_cast<const uint16_t*>(weight);
  auto O = static_cast<uint16_t*>(out);
  switch (hidden / 256) {
    case 1: return check_launch(launch(rmsnorm_kernel<1>, g, b, 0, st, A, x_stride, B, addend_stride, R, residual_stride, W, eps, O, out_stride, (int)rows));
    case 2: return check_launch(launch(rmsnorm_kernel<2>, g, b, 0, st, A, x_stride, B, addend_stride, R, residual_stride, W, eps, O, out_stride, (int)rows));
    case 4: return check_launch(launch(rmsnorm_kernel<4>, g, b, 0, st, A, x_stride, B, addend_stride, R, residual_stride, W, eps, O, out_stride, (int)rows));
    case 8: return check_launch(launch(rmsnorm_kernel<8>, g, b, 0, st, A, x_stride, B, addend_stride, R, residual_stride, W, eps, O, out_stride, (int)rows));
    case 16: return check_launch(launch(rmsnorm_kernel<16>, g, b, 0, st, A, x_stride, B, addend_stride, R, residual_stride, W, eps, O, out_stride, (int)rows));
    case 32: return check_launch(launch(rmsnorm_kernel<32>, g, b, 0, st, A, x_stride, B, addend_stride, R, residual_stride, W, eps, O, out_stride, (int)rows));
  }
  return set_error(OMNI_ERR_UNSUPPORTED, "hidden must be 256 x {1,2,4,8,16,32}");
}

extern "C" OMNI_API int omni_qknorm_rope_store(const void* qkv, int64_t qkv_stride, int64_t rows, int32_t num_q_heads,
                                               int32_t num_kv_heads, int32_t head_dim, const void* q_norm_weight,
                                               const void* k_norm_weight, float eps, const float* cos_sin_cache,
                                               int64_t max_position, const int64_t* positions,
                                               const int64_t* cache_loc, int32_t tokens_per_req, int32_t slot_stride,
                                               int32_t slot_base, void* q_out, int64_t q_stride, void* k_cache,
                                               void* v_cache, void* stream) {
  if (rows < 0 || num_q_heads <= 0 || num_kv_heads <= 0) return set_error(OMNI_ERR_INVALID, "bad head counts");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return set_error(OMNI_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256");
  if ((positions == nullptr) != (cache_loc == nullptr))
    return set_error(OMNI_ERR_INVALID, "positions and cache_loc are given together");
  if (positions == nullptr && (tokens_per_req <= 0 || slot_stride <= 0 || slot_base < 0))
    return set_error(OMNI_ERR_INVALID, "implicit slots need tokens_per_req, slot_stride > 0");
  if (positions == nullptr && slot_base + tokens_per_req > max_position)
    return set_error(OMNI_ERR_INVALID, "implicit positions exceed the rotary table");
  if ((reinterpret_cast<uintptr_t>(qkv) & 7) || qkv_stride % 4)
    return set_error(OMNI_ERR_UNSUPPORTED, "qkv rows must be 8-byte aligned");
  if (rows == 0) return OMNI_OK;
  QkRopeParams p{};
  p.qkv = static_cast<const uint16_t*>(qkv);
  p.qkv_stride = qkv_stride;
  p.rows = (int)rows;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.head_dim = head_dim;
  p.q_norm = static_cast<const uint16_t*>(q_norm_weight);
  p.k_norm = static_cast<const uint16_t*>(k_norm_weight);
  p.eps = eps;
  p.cos_sin = cos_sin_cache;
  p.max_pos = max_position;
  p.positions = positions;
  p.cache_loc = cache_loc;
  p.tokens_per_req = tokens_per_req;
  p.slot_stride = slot_stride;
  p.slot_base = slot_base;
  p.q_out = static_cast<uint16_t*>(q_out);
  p.q_stride = q_stride;
  p.k_cache = static_cast<uint16_t*>(k_cache);
  p.v_cache = static_cast<uint16_t*>(v_cache);
  const int64_t items = rows * (num_q_heads + num_kv_heads);
  dim3 g((unsigned)((items + 3) / 4)), b(128);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 64: return check_launch(launch(qknorm_rope_store_kernel<2>, g, b, 0, st, p));
    case 128: return check_launch(launch(qknorm_rope_store_kernel<4>, g, b, 0, st, p));
    default: return check_launch(launch(qknorm_rope_store_kernel<8>, g, b, 0, st, p));
  }
}
