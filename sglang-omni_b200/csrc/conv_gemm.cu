// Implicit-GEMM causal convolution on the 5th-generation tensor cores (tcgen05 +
// TMEM), channels last:
//
//   out[r, t, n] = sum_{j < taps} sum_c padded[r, t + j * dil, c] * W[n, j, c]     (t < L)
//
// the code2wav's dilated causal convs (and, with taps = 1, its 1x1 convs and the
// GEMMs of its transposed convs).  The windows are never written to memory: a CTA
// owns 128 output positions of one row (the MMA's M axis, TMEM lanes) and a tile of
// output channels (N <= 256, TMEM columns); its K loop walks (tap j, channel block),
// and the A tile of each step is the 128 x KB window of the channels-last input that
// starts at position t0 + j * dil in the 2D view [rows * Lp, C_in].  When 128 +
// (taps - 1) dil <= 256 one TMA box of that many positions per channel block serves
// every tap (the MMA's descriptor starts j dil rows into it), which cuts the input's
// reads from L2 by the tap count; otherwise each step loads its own 128-row box.
// Positions past a row's L read the next row's samples or the fill value and are
// never stored.  B tiles (KB x N of the [C_out, taps * C_in] weight matrix) come by
// TMA in the same stage.  KB = 64 channels (128-byte swizzle) when C_in is a multiple
// of 64, else 32 (64-byte swizzle).
//
// Roles (320 threads, two CTAs an SM so that one CTA's epilogue runs while the other
// feeds the tensor cores): warp 0 = TMA producer, warp 1 = MMA issuer (one elected
// lane), warps 2..9 drain TMEM (warp w reads lanes 32 (w % 4) .., half of the column
// chunks each) and run the epilogue: the bf16 conv output, or fused with the vocoder's next step
// SnakeBeta(conv + bias [+ residual]) with the same rounding points as
// bias_snake_beta_kernel (vocoder.cu), the pre-activation sum optionally stored.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_util.h"
#include "common.cuh"

namespace omni {
namespace {
OMNI_DEFINE_STATUS(conv_gemm)

constexpr int kConvM = 128;       // output positions per CTA
constexpr int kConvThreads = 320;  // producer, MMA, 8 epilogue warps
constexpr int kConvMaxStages = 8;
constexpr int kConvMaxN = 256;

struct ConvGemmParams {
  int rows, length;        // batch rows, output positions per row
  int64_t lp;              // input positions per row (history + length)
  int cin, cout, taps, dil;
  int kb, num_k;           // channels per K block; K steps = (C_in / kb) x taps, taps inner
  int n_tile, tmem_cols;
  int a_union;             // 1: one A box of 128 + (taps - 1) dil positions per channel block
  int a_stages, b_stages;  // ring depths of the A and B tiles
  uint32_t a_bytes, a_tx, b_bytes;  // A stage bytes (1024-aligned), A box bytes, B stage bytes
  int snake;               // 0: out = bf16(conv); 1: SnakeBeta(conv + bias [+ residual])
  const uint16_t* bias;
  const uint16_t* residual;  // contiguous [rows, length, cout] or null
  uint16_t* sum_out;         // contiguous [rows, length, cout] or null
  const uint16_t* alpha_scale;
  const uint16_t* inverse_beta;
  uint16_t* out;             // out + r * out_batch_stride + t * cout + n
  int64_t out_batch_stride;
};

// K-major smem descriptor for a 64-byte swizzled operand (rows of 64 bytes, 8-row
// groups 512 bytes apart): the 32-channel blocks of C_in % 64 != 0.
OMNI_DEVINL uint64_t smem_desc_sw64(const void* smem_ptr) {
  uint64_t addr = smem_u32(smem_ptr);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;  // SWIZZLE_64B
  return d;
}

OMNI_DEVINL float rbf(float f) { return bf2f(f2bf(f)); }

__global__ void __launch_bounds__(kConvThreads, 2)
    conv_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ ConvGemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kConvM, row = blockIdx.y, n0 = blockIdx.z * p.n_tile;
  const int SA = p.a_stages, SB = p.b_stages;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + SA * p.a_bytes;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(b_smem + SB * p.b_bytes);
  uint64_t* empty_a = full_a + kConvMaxStages;
  uint64_t* full_b = empty_a + kConvMaxStages;
  uint64_t* empty_b = full_b + kConvMaxStages;
  uint64_t* done = empty_b + kConvMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kConvMaxStages; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&empty_a[s], 1);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_b[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
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

  const int64_t a_row0 = (int64_t)row * p.lp + t0;
  // K step i = (channel block cb, tap): cb = i / taps, tap = i % taps.  A tiles: one per
  // step, or with a_union one per channel block (the box covers every tap's window; the
  // MMA of tap j starts j x dil rows into it).  A step's A slot is its A index ka mod SA,
  // its B slot i mod SB; a slot is refilled at round k once the MMAs of round k - 1 have
  // released it.
  if (warp == 0) {
    const bool leader = elect_one();
    bool ok = true;
    for (int i = 0; i < p.num_k && ok; ++i) {
      const int cb = i / p.taps, tap = i - cb * p.taps;
      if (!p.a_union || tap == 0) {
        const int ka = p.a_union ? cb : i, sa = ka % SA;
        if (ka >= SA && !__all_sync(0xFFFFFFFFu, mbar_wait(&empty_a[sa], (uint32_t)((ka / SA - 1) & 1)))) {
          ok = false;
          break;
        }
        if (leader) {
          mbar_arrive_expect_tx(&full_a[sa], p.a_tx);
          tma_load_2d(a_smem + sa * p.a_bytes, &tmap_a, &full_a[sa], cb * p.kb,
                      (int)(a_row0 + (p.a_union ? 0 : (int64_t)tap * p.dil)));
        }
      }
      const int sb = i % SB;
      if (i >= SB && !__all_sync(0xFFFFFFFFu, mbar_wait(&empty_b[sb], (uint32_t)((i / SB - 1) & 1)))) {
        ok = false;
        break;
      }
      if (leader) {
        mbar_arrive_expect_tx(&full_b[sb], p.b_bytes);
        tma_load_2d(b_smem + sb * p.b_bytes, &tmap_b, &full_b[sb], tap * p.cin + cb * p.kb, n0);
      }
      __syncwarp();
    }
    if (!ok && leader) {
      report_status(kDevTimeoutMma);
      *abort_flag = 1;
    }
  } else if (warp == 1) {
    const bool leader = elect_one();
    const uint32_t idesc = idesc_bf16_f32(kConvM, p.n_tile);
    const bool sw128 = p.kb == 64;
    const uint32_t row_bytes = (uint32_t)p.kb * 2;
    bool ok = true;
    for (int i = 0; i < p.num_k; ++i) {
      const int cb = i / p.taps, tap = i - cb * p.taps;
      const int ka = p.a_union ? cb : i, sa = ka % SA, sb = i % SB;
      if ((!p.a_union || tap == 0) && !__all_sync(0xFFFFFFFFu, mbar_wait(&full_a[sa], (uint32_t)((ka / SA) & 1)))) {
        ok = false;
        break;
      }
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&full_b[sb], (uint32_t)((i / SB) & 1)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (leader) {
        // tap j's window starts j x dil rows into the union box: the swizzle is a function
        // of the absolute shared-memory address (TMA wrote the box the same way), so a
        // start inside a swizzle atom needs no base offset (measured: with the base-offset
        // field set to the row phase the products were wrong, with 0 they match fp32)
        const uint8_t* as = a_smem + sa * p.a_bytes + (p.a_union ? (uint32_t)(tap * p.dil) * row_bytes : 0u);
        const uint8_t* bs = b_smem + sb * p.b_bytes;
        const uint64_t ad = sw128 ? smem_desc_sw128(as) : smem_desc_sw64(as);
        const uint64_t bd = sw128 ? smem_desc_sw128(bs) : smem_desc_sw64(bs);
        // 16 channels (32 bytes) per MMA: the start address advances by 2 16-byte units
        for (int kk = 0; kk < p.kb / 16; ++kk)
          tc_mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&empty_b[sb]);
        if (!p.a_union || tap == p.taps - 1) tc_commit(&empty_a[sa]);
      }
      __syncwarp();
    }
    if (!ok && leader) {
      report_status(kDevTimeoutTma);
      *abort_flag = 1;
    }
    if (leader) {
      if (ok) tc_commit(done);
      else mbar_arrive(done);
    }
  } else {
    // epilogue: warp w drains TMEM lanes 32 (w % 4) .. + 31 = positions t0 + that, the
    // 32-column chunks 32 h, 32 h + 64, ... with h = (w - 2) / 4 (two warps a lane quarter)
    if (!mbar_wait(done, 0)) {
      report_status(kDevTimeoutMma);
      *abort_flag = 1;
    }
    tc_fence_after();
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int t = t0 + q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const bool aborted = *reinterpret_cast<volatile int*>(abort_flag) != 0;
    for (int c = half * 32; c < p.n_tile && !aborted; c += 64) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(lane_base + (uint32_t)c, r);
      tc_wait_ld();
      const int nb = n0 + c;
      if (t >= p.length || nb >= p.cout) continue;
      const int64_t pos = (int64_t)row * p.length + t;  // contiguous [rows, length, cout]
      uint16_t* dst = p.out + (int64_t)row * p.out_batch_stride + (int64_t)t * p.cout + nb;
      const int cnt = min(32, p.cout - nb);  // a multiple of 8 (cout % 8 == 0)
      for (int v = 0; v < cnt; v += 8) {
        uint32_t o[4], sv[4];
        uint4 rv = make_uint4(0, 0, 0, 0), bv = make_uint4(0, 0, 0, 0), av = bv, iv = bv;
        if (p.snake) {
          bv = *reinterpret_cast<const uint4*>(p.bias + nb + v);
          av = *reinterpret_cast<const uint4*>(p.alpha_scale + nb + v);
          iv = *reinterpret_cast<const uint4*>(p.inverse_beta + nb + v);
          if (p.residual) rv = *reinterpret_cast<const uint4*>(p.residual + pos * p.cout + nb + v);
        }
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w}, aw[4] = {av.x, av.y, av.z, av.w};
        const uint32_t iw[4] = {iv.x, iv.y, iv.z, iv.w}, rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float y2[2], s2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float conv = rbf(__uint_as_float(r[v + 2 * h + e]));  // the conv's bf16 output
            if (!p.snake) {
              y2[e] = conv;
              s2[e] = 0.0f;
              continue;
            }
            const uint32_t pick = e ? 16u : 0u;
            const float b = bf2f((uint16_t)(bw[h] >> pick)), a = bf2f((uint16_t)(aw[h] >> pick));
            const float ib = bf2f((uint16_t)(iw[h] >> pick));
            float total = rbf(conv + b);
            if (p.residual) total = rbf(total + bf2f((uint16_t)(rw[h] >> pick)));
            s2[e] = total;
            const float phase = rbf(total * a);
            const float sine = rbf(sinf(phase));
            const float sq = rbf(sine * sine);
            const float scaled = rbf(ib * sq);
            y2[e] = total + scaled;
          }
          o[h] = pack_bf2(y2[0], y2[1]);
          sv[h] = pack_bf2(s2[0], s2[1]);
        }
        *reinterpret_cast<uint4*>(dst + v) = make_uint4(o[0], o[1], o[2], o[3]);
        if (p.snake && p.sum_out)
          *reinterpret_cast<uint4*>(p.sum_out + pos * p.cout + nb + v) = make_uint4(sv[0], sv[1], sv[2], sv[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_conv() {
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

// 2D bf16 [rows, cols] (row stride in elements), box {kb, box_rows}, swizzle by kb.
bool conv_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t stride, int kb, int box_rows) {
  auto fn = encode_fn_conv();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)kb, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, kb == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int omni_conv1d_gemm(const void* padded, int64_t rows, int64_t padded_positions, int32_t cin,
                                         const void* weight, int32_t cout, int32_t taps, int32_t dilation,
                                         int64_t length, void* out, int64_t out_batch_stride, const void* bias,
                                         const void* residual, void* sum_out, const void* alpha_scale,
                                         const void* inverse_beta, void* stream) {
  if (rows < 0 || length < 0 || taps < 1 || dilation < 1 || cin < 1 || cout < 1)
    return set_error(OMNI_ERR_INVALID, "conv1d_gemm: bad shape");
  if (padded_positions < length + (int64_t)(taps - 1) * dilation)
    return set_error(OMNI_ERR_INVALID, "conv1d_gemm: the padded input is shorter than length + (taps - 1) x dilation");
  if (cin % 32 != 0 || cout % 32 != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "conv1d_gemm: C_in and C_out must be multiples of 32");
  auto mis16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (mis16(padded) || mis16(weight) || mis16(out) || out_batch_stride % 8 ||
      (bias && mis16(bias)) || (residual && mis16(residual)) || (sum_out && mis16(sum_out)) ||
      (alpha_scale && mis16(alpha_scale)) || (inverse_beta && mis16(inverse_beta)))
    return set_error(OMNI_ERR_UNSUPPORTED, "conv1d_gemm: 16-byte aligned operands required");
  const bool snake = alpha_scale != nullptr;
  if (snake && (!bias || !inverse_beta)) return set_error(OMNI_ERR_INVALID, "conv1d_gemm: SnakeBeta needs bias and 1/beta");
  if (!snake && (residual || sum_out)) return set_error(OMNI_ERR_INVALID, "conv1d_gemm: residual / sum_out need SnakeBeta");
  if (rows * padded_positions >= (int64_t(1) << 31) || rows > 65535)
    return set_error(OMNI_ERR_UNSUPPORTED, "conv1d_gemm: input too large for one call");
  if (rows == 0 || length == 0) return OMNI_OK;
  ConvGemmParams p{};
  p.rows = (int)rows;
  p.length = (int)length;
  p.lp = padded_positions;
  p.cin = cin;
  p.cout = cout;
  p.taps = taps;
  p.dil = dilation;
  p.kb = cin % 64 == 0 ? 64 : 32;
  p.num_k = taps * (cin / p.kb);
  // the output-channel tile: all of C_out when <= 256 (a multiple of 32), else the
  // widest multiple of 32 <= 256 that divides it
  int nt = cout;
  if (nt > kConvMaxN) {
    nt = kConvMaxN;
    while (nt > 32 && cout % nt) nt -= 32;
  }
  p.n_tile = nt;
  int tc = 32;
  while (tc < nt) tc <<= 1;
  p.tmem_cols = tc;
  p.b_bytes = (uint32_t)nt * p.kb * 2;
  // two CTAs an SM (one's epilogue runs under the other's main loop): at most ~110 KB each
  const size_t fixed = 1024 + (4 * kConvMaxStages + 1) * 8 + 16, budget = 110 * 1024;
  const int union_rows = kConvM + (taps - 1) * dilation;
  const uint32_t union_bytes = ((uint32_t)union_rows * p.kb * 2 + 1023u) & ~1023u;
  // the union box when it fits a TMA box (<= 256 rows) and two A + two B slots fit
  p.a_union = taps > 1 && union_rows <= 256 && fixed + 2 * (size_t)union_bytes + 2 * p.b_bytes <= budget;
  if (p.a_union) {
    p.a_bytes = union_bytes;
    p.a_tx = (uint32_t)union_rows * p.kb * 2;
    p.a_stages = 2;
    int sb = kConvMaxStages;
    while (sb > 2 && fixed + 2 * (size_t)union_bytes + (size_t)sb * p.b_bytes > budget) --sb;
    p.b_stages = sb;
  } else {
    p.a_bytes = p.a_tx = (uint32_t)kConvM * p.kb * 2;
    int st = kConvMaxStages;
    while (st > 2 && fixed + (size_t)st * (p.a_bytes + p.b_bytes) > budget) --st;
    p.a_stages = p.b_stages = st;
  }
  p.snake = snake ? 1 : 0;
  p.bias = static_cast<const uint16_t*>(bias);
  p.residual = static_cast<const uint16_t*>(residual);
  p.sum_out = static_cast<uint16_t*>(sum_out);
  p.alpha_scale = static_cast<const uint16_t*>(alpha_scale);
  p.inverse_beta = static_cast<const uint16_t*>(inverse_beta);
  p.out = static_cast<uint16_t*>(out);
  p.out_batch_stride = out_batch_stride;
  CUtensorMap ta, tb;
  if (!conv_tmap(&ta, padded, rows * padded_positions, cin, cin, p.kb, p.a_union ? union_rows : kConvM) ||
      !conv_tmap(&tb, weight, cout, (int64_t)taps * cin, (int64_t)taps * cin, p.kb, nt))
    return set_error(OMNI_ERR_UNSUPPORTED, "conv1d_gemm: tensor map encoding failed");
  const size_t smem = fixed + (size_t)p.a_stages * p.a_bytes + (size_t)p.b_stages * p.b_bytes;
  const cudaError_t ae = once_per_device(reinterpret_cast<const void*>(conv_gemm_kernel), kAttrSmem, [] {
    return cudaFuncSetAttribute(conv_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024);
  });
  if (ae != cudaSuccess) return check_launch(ae);
  const dim3 grid((unsigned)((length + kConvM - 1) / kConvM), (unsigned)rows, (unsigned)(cout / nt));
  return check_launch(launch(conv_gemm_kernel, grid, dim3(kConvThreads), smem, static_cast<cudaStream_t>(stream),
                             ta, tb, p));
}
