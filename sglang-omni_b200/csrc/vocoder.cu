// Kernels of the streaming vocoder (code2wav) step that consumes the decode step's codes:
//
// bias_snake_beta_kernel — SnakeBeta(conv + bias [+ residual]) over channels-last rows
//   (fused_bias_snake_beta, sglang_omni/kernels/bias_snake_beta.py:100-151): every
//   intermediate rounds to the activations' dtype where the eager adds and SnakeBeta
//   round (conv + bias, + residual, x * exp(alpha), sin, its square, the 1 / beta
//   scale, the final add), 16-byte vectors, parameters read at the vector's channel.
// single_output_conv_kernel — a stride-one, undilated conv from channels-last rows to
//   one output channel, + bias, clamped to [-1, 1] (NaN kept), accumulated in fp32 and
//   rounded once (clamped_single_output_conv, sglang_omni/kernels/single_output_conv.py:
//   68-102): a CTA stages 256 positions' input rows in shared memory and each thread
//   sums one position in a fixed order, so a position's bits do not depend on how the
//   positions are split into calls.
// history_exchange_kernel / overlap_exchange_kernel — the per-slot codec state of a
//   causal conv (its history in front of the new samples, zeros after) and of a
//   transposed conv (its overlap added into the next output) (history_exchange /
//   overlap_exchange, sglang_omni/kernels/codec_state.py:153-210): one CTA per (row,
//   channel block); every read of a slot's old state precedes every write of its new one.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "capi_util.h"
#include "common.cuh"

namespace omni {
namespace {

// dtype codes of these entry points
constexpr int kBF16 = 0, kF16 = 1, kF32 = 2;

template <int DT>
struct Elem;
template <>
struct Elem<kBF16> {
  using T = uint16_t;
  static OMNI_DEVINL float load(T v) { return bf2f(v); }
  static OMNI_DEVINL T store(float f) { return f2bf(f); }
};
template <>
struct Elem<kF16> {
  using T = uint16_t;
  static OMNI_DEVINL float load(T v) {
    __half h;
    *reinterpret_cast<uint16_t*>(&h) = v;
    return __half2float(h);
  }
  static OMNI_DEVINL T store(float f) {
    __half h = __float2half_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
  }
};
template <>
struct Elem<kF32> {
  using T = float;
  static OMNI_DEVINL float load(T v) { return v; }
  static OMNI_DEVINL T store(float f) { return f; }
};

// rounds through the activations' dtype
template <int DT>
OMNI_DEVINL float rnd(float f) {
  return Elem<DT>::load(Elem<DT>::store(f));
}

struct SnakeParams {
  const void* conv;
  int64_t conv_batch_stride;  // elements
  const void* bias;
  const void* residual;  // contiguous [B, L, C] or null
  void* sum_out;         // contiguous [B, L, C] or null
  void* out;
  int64_t out_batch_stride;
  const void* alpha_scale;   // [C]
  const void* inverse_beta;  // [C]
  int64_t row_vectors;       // L * C / vector elements
  int channel_vectors;       // C / vector elements
};

template <int DT>
__global__ void __launch_bounds__(256) bias_snake_beta_kernel(const __grid_constant__ SnakeParams p) {
  using T = typename Elem<DT>::T;
  constexpr int E = 16 / (int)sizeof(T);
  const int64_t batch = blockIdx.y;
  const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  griddep_wait();
  griddep_launch();
  if (v >= p.row_vectors) return;
  const int64_t ch0 = (v % p.channel_vectors) * E;
  const int64_t off = v * E;
  const uint4 cv = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.conv) + batch * p.conv_batch_stride + off);
  const uint4 bv = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.bias) + ch0);
  const uint4 av = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.alpha_scale) + ch0);
  const uint4 iv = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.inverse_beta) + ch0);
  const int64_t cbase = batch * p.row_vectors * E + off;  // contiguous [B, L, C]
  uint4 rv = make_uint4(0, 0, 0, 0);
  if (p.residual) rv = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.residual) + cbase);
  const T* c = reinterpret_cast<const T*>(&cv);
  const T* bb = reinterpret_cast<const T*>(&bv);
  const T* a = reinterpret_cast<const T*>(&av);
  const T* ib = reinterpret_cast<const T*>(&iv);
  const T* r = reinterpret_cast<const T*>(&rv);
  uint4 sv, ov;
  T* s = reinterpret_cast<T*>(&sv);
  T* o = reinterpret_cast<T*>(&ov);
#pragma unroll
  for (int j = 0; j < E; ++j) {
    float total = rnd<DT>(Elem<DT>::load(c[j]) + Elem<DT>::load(bb[j]));
    if (p.residual) total = rnd<DT>(total + Elem<DT>::load(r[j]));
    s[j] = Elem<DT>::store(total);
    const float phase = rnd<DT>(total * Elem<DT>::load(a[j]));
    const float sine = rnd<DT>(sinf(phase));
    const float sq = rnd<DT>(sine * sine);
    const float scaled = rnd<DT>(Elem<DT>::load(ib[j]) * sq);
    o[j] = Elem<DT>::store(total + scaled);
  }
  if (p.sum_out) *reinterpret_cast<uint4*>(static_cast<T*>(p.sum_out) + cbase) = sv;
  *reinterpret_cast<uint4*>(static_cast<T*>(p.out) + batch * p.out_batch_stride + off) = ov;
}

struct ConvParams {
  const void* padded;  // [B, L + taps - 1, C] rows contiguous
  int64_t padded_batch_stride;
  const void* weight;  // [1, C, taps] with the given strides
  int64_t w_channel_stride, w_tap_stride;
  const void* bias;    // [1]
  void* out;           // [B, 1, L] contiguous
  int64_t length;
  int channels, taps;
};

constexpr int kConvPositions = 256;  // output positions per CTA (one per thread)
constexpr int kConvMaxSmem = 200 * 1024;

// Padded row stride of the staged tile, in 16-byte vectors: odd, so that the 8 threads of
// a 16-byte access phase (consecutive rows) hit distinct bank groups.
__host__ __device__ __forceinline__ int conv_row_vectors(int vecs) { return vecs + ((vecs & 1) ? 2 : 1); }

// CTA: 256 consecutive output positions of one row.  Their input rows (256 + taps - 1,
// channels-last) are staged in shared memory with 16-byte vectors at an odd padded
// stride; the weights sit in shared memory too.  Thread p sums tap by tap over the
// channels in a fixed order, so a position's bits do not depend on the split of the
// positions into calls.
template <int DT>
__global__ void __launch_bounds__(kConvPositions) single_output_conv_kernel(const __grid_constant__ ConvParams p) {
  using T = typename Elem<DT>::T;
  constexpr int E = 16 / (int)sizeof(T);
  extern __shared__ __align__(16) uint8_t smem[];
  const int C = p.channels, taps = p.taps;
  const int rs = conv_row_vectors(C / E) * E;  // padded row stride (elements)
  const int nrows = kConvPositions + taps - 1;
  T* tile = reinterpret_cast<T*>(smem);
  float* wsm = reinterpret_cast<float*>(smem + (size_t)nrows * rs * sizeof(T));  // [taps][C]
  const int64_t batch = blockIdx.y;
  const int64_t pos0 = (int64_t)blockIdx.x * kConvPositions;
  const T* w = static_cast<const T*>(p.weight);
  // weights do not depend on the previous kernel
  for (int i = threadIdx.x; i < taps * C; i += blockDim.x) {
    const int tap = i / C, c = i % C;
    wsm[i] = Elem<DT>::load(w[(int64_t)c * p.w_channel_stride + (int64_t)tap * p.w_tap_stride]);
  }
  griddep_wait();
  griddep_launch();
  const T* src = static_cast<const T*>(p.padded) + batch * p.padded_batch_stride;
  const int64_t avail = p.length + taps - 1 - pos0;  // input rows left in this batch row
  const int vecs = C / E;
  for (int i = threadIdx.x; i < nrows * vecs; i += blockDim.x) {
    const int r = i / vecs, v = i % vecs;
    uint4 x = make_uint4(0, 0, 0, 0);
    if (r < avail) x = *reinterpret_cast<const uint4*>(src + (pos0 + r) * C + v * E);
    *reinterpret_cast<uint4*>(tile + r * rs + v * E) = x;
  }
  __syncthreads();
  const int64_t pos = pos0 + threadIdx.x;
  if (pos >= p.length) return;
  float acc = 0.0f;
  for (int tap = 0; tap < taps; ++tap) {
    const T* row = tile + (threadIdx.x + tap) * rs;
    const float* wt = wsm + tap * C;
    for (int v = 0; v < vecs; ++v) {
      const uint4 xv = *reinterpret_cast<const uint4*>(row + v * E);
      const T* x = reinterpret_cast<const T*>(&xv);
#pragma unroll
      for (int j = 0; j < E; ++j) acc = fmaf(Elem<DT>::load(x[j]), wt[v * E + j], acc);
    }
  }
  float y = acc + Elem<DT>::load(static_cast<const T*>(p.bias)[0]);
  if (y == y) y = fminf(fmaxf(y, -1.0f), 1.0f);  // NaN passes through
  static_cast<T*>(p.out)[batch * p.length + pos] = Elem<DT>::store(y);
}

constexpr int kChannelBlock = 64;
constexpr int kMaxStateSamples = 64;  // history / overlap samples held per CTA

struct HistoryParams {
  void* padded;
  int64_t pr, ps, pc;  // padded strides: row, sample, channel (elements)
  void* pool;
  int64_t qs_slot, qs_sample, qs_channel;  // pool strides
  const int64_t* slot_index;
  int history, new_samples, tail, channels, cold;
};

template <typename T>
__global__ void __launch_bounds__(kChannelBlock * 4) history_exchange_kernel(const __grid_constant__ HistoryParams p) {
  __shared__ T s_old[kMaxStateSamples][kChannelBlock];
  __shared__ T s_new[kMaxStateSamples][kChannelBlock];
  const int64_t row = blockIdx.x;
  const int c = blockIdx.y * kChannelBlock + (threadIdx.x % kChannelBlock);
  const int s0 = threadIdx.x / kChannelBlock, sstep = blockDim.x / kChannelBlock;
  griddep_wait();
  griddep_launch();
  const int64_t slot = p.slot_index[row];
  T* padded = static_cast<T*>(p.padded) + row * p.pr + (int64_t)c * p.pc;
  T* pool = static_cast<T*>(p.pool) + slot * p.qs_slot + (int64_t)c * p.qs_channel;
  const bool on = c < p.channels;
  // reads: the slot's old history, and the new history (the last `history` samples of
  // history + new samples)
  for (int s = s0; s < p.history; s += sstep) {
    T old = T(0), nh = T(0);
    if (on) {
      const int src = s + p.new_samples;  // position in (old history ++ new samples)
      if (!p.cold) old = pool[(int64_t)s * p.qs_sample];
      if (src >= p.history) nh = padded[(int64_t)src * p.ps];
      else if (!p.cold) nh = pool[(int64_t)src * p.qs_sample];
    }
    s_old[s][threadIdx.x % kChannelBlock] = old;
    s_new[s][threadIdx.x % kChannelBlock] = nh;
  }
  __syncthreads();
  if (!on) return;
  for (int s = s0; s < p.history; s += sstep) {
    padded[(int64_t)s * p.ps] = s_old[s][threadIdx.x % kChannelBlock];
    pool[(int64_t)s * p.qs_sample] = s_new[s][threadIdx.x % kChannelBlock];
  }
  for (int s = s0; s < p.tail; s += sstep) padded[(int64_t)(p.history + p.new_samples + s) * p.ps] = T(0);
}

struct OverlapParams {
  void* output;
  int64_t orow, osample, ochannel;
  void* pool;
  int64_t qs_slot, qs_sample, qs_channel;
  const int64_t* slot_index;
  int overlap, emitted, channels, cold;
};

template <int DT>
__global__ void __launch_bounds__(kChannelBlock * 4) overlap_exchange_kernel(const __grid_constant__ OverlapParams p) {
  using T = typename Elem<DT>::T;
  const int64_t row = blockIdx.x;
  const int c = blockIdx.y * kChannelBlock + (threadIdx.x % kChannelBlock);
  const int s0 = threadIdx.x / kChannelBlock, sstep = blockDim.x / kChannelBlock;
  griddep_wait();
  griddep_launch();
  if (c >= p.channels) return;
  const int64_t slot = p.slot_index[row];
  T* out = static_cast<T*>(p.output) + row * p.orow + (int64_t)c * p.ochannel;
  T* pool = static_cast<T*>(p.pool) + slot * p.qs_slot + (int64_t)c * p.qs_channel;
  // the ranges [0, overlap) and [emitted, emitted + overlap) are disjoint (emitted >= overlap)
  for (int s = s0; s < p.overlap; s += sstep) {
    const T tail = out[(int64_t)(p.emitted + s) * p.osample];
    if (!p.cold) {
      const T prev = pool[(int64_t)s * p.qs_sample];
      T* h = out + (int64_t)s * p.osample;
      *h = Elem<DT>::store(Elem<DT>::load(*h) + Elem<DT>::load(prev));
    }
    pool[(int64_t)s * p.qs_sample] = tail;
  }
}

bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

// The taps-wide windows of a causal conv's channels-last input, laid out as the rows of
// the conv's GEMM operand: out[r * length + t, j * C + c] = padded[r, t + j * dilation, c].
// One 16-byte vector a thread (grid-stride); a window's reads of neighbouring outputs hit
// L2, so the traffic is one read of the input and one write of the taps-times-larger output.
struct WindowParams {
  const uint8_t* padded;
  uint8_t* out;
  int64_t row_bytes;       // padded row stride in bytes
  uint32_t total;          // vectors in out
  uint32_t seg;            // vectors per sample (channels x element bytes / 16)
  uint32_t taps, length, dil_bytes_vec;  // dil_bytes_vec: dilation x seg
};

__global__ void __launch_bounds__(256) conv_window_gather_kernel(const __grid_constant__ WindowParams p) {
  griddep_wait();
  griddep_launch();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < p.total; i += gridDim.x * blockDim.x) {
    const uint32_t v = i % p.seg;
    uint32_t rest = i / p.seg;
    const uint32_t j = rest % p.taps;
    rest /= p.taps;
    const uint32_t t = rest % p.length;
    const uint32_t r = rest / p.length;
    const uint4* src = reinterpret_cast<const uint4*>(p.padded + (int64_t)r * p.row_bytes) +
                       ((size_t)t * p.seg + (size_t)j * p.dil_bytes_vec + v);
    reinterpret_cast<uint4*>(p.out)[i] = *src;
  }
}

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int omni_bias_snake_beta(const void* conv_output, int64_t conv_batch_stride, const void* bias,
                                             const void* residual, void* sum_out, void* out,
                                             int64_t out_batch_stride, const void* alpha_scale,
                                             const void* inverse_beta, int64_t batch, int64_t length,
                                             int64_t channels, int32_t dtype, void* stream) {
  if (batch < 0 || length < 0 || channels <= 0) return set_error(OMNI_ERR_INVALID, "bad SnakeBeta shape");
  if (dtype != kBF16 && dtype != kF16) return set_error(OMNI_ERR_UNSUPPORTED, "SnakeBeta runs on bf16 or fp16");
  const int E = 8;
  if (channels % E) return set_error(OMNI_ERR_UNSUPPORTED, "channels must split into 16-byte vectors");
  if (!aligned16(conv_output) || !aligned16(out) || !aligned16(bias) || !aligned16(alpha_scale) ||
      !aligned16(inverse_beta) || (residual && !aligned16(residual)) || (sum_out && !aligned16(sum_out)) ||
      conv_batch_stride % E || out_batch_stride % E)
    return set_error(OMNI_ERR_UNSUPPORTED, "SnakeBeta operands must be 16-byte aligned");
  if (batch == 0 || length == 0) return OMNI_OK;
  SnakeParams p{};
  p.conv = conv_output;
  p.conv_batch_stride = conv_batch_stride;
  p.bias = bias;
  p.residual = residual;
  p.sum_out = sum_out;
  p.out = out;
  p.out_batch_stride = out_batch_stride;
  p.alpha_scale = alpha_scale;
  p.inverse_beta = inverse_beta;
  p.row_vectors = length * channels / E;
  p.channel_vectors = (int)(channels / E);
  const dim3 grid((unsigned)((p.row_vectors + 255) / 256), (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return check_launch(dtype == kBF16 ? launch(bias_snake_beta_kernel<kBF16>, grid, dim3(256), 0, st, p)
                                     : launch(bias_snake_beta_kernel<kF16>, grid, dim3(256), 0, st, p));
}

extern "C" OMNI_API int omni_clamped_single_output_conv(const void* padded, int64_t padded_batch_stride,
                                                        const void* weight, int64_t weight_channel_stride,
                                                        int64_t weight_tap_stride, const void* bias, void* out,
                                                        int64_t batch, int64_t length, int64_t channels,
                                                        int32_t taps, int32_t dtype, void* stream) {
  if (batch < 0 || length < 0 || channels <= 0 || taps <= 0) return set_error(OMNI_ERR_INVALID, "bad conv shape");
  if (dtype != kBF16 && dtype != kF16 && dtype != kF32) return set_error(OMNI_ERR_UNSUPPORTED, "unsupported dtype");
  const int E = dtype == kF32 ? 4 : 8;
  if (channels % E || padded_batch_stride % E || !aligned16(padded))
    return set_error(OMNI_ERR_UNSUPPORTED, "channels-last rows must split into 16-byte vectors");
  if (batch == 0 || length == 0) return OMNI_OK;
  ConvParams p{};
  p.padded = padded;
  p.padded_batch_stride = padded_batch_stride;
  p.weight = weight;
  p.w_channel_stride = weight_channel_stride;
  p.w_tap_stride = weight_tap_stride;
  p.bias = bias;
  p.out = out;
  p.length = length;
  p.channels = (int)channels;
  p.taps = taps;
  const size_t smem = (size_t)(kConvPositions + taps - 1) * conv_row_vectors((int)(channels / E)) * 16 +
                      (size_t)taps * channels * 4;
  if (smem > (size_t)kConvMaxSmem) return set_error(OMNI_ERR_UNSUPPORTED, "conv tile exceeds shared memory");
  const dim3 grid((unsigned)((length + kConvPositions - 1) / kConvPositions), (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto go = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kConvMaxSmem);
    return check_launch(launch(kernel, grid, dim3(kConvPositions), smem, st, p));
  };
  if (dtype == kBF16) return go(single_output_conv_kernel<kBF16>);
  if (dtype == kF16) return go(single_output_conv_kernel<kF16>);
  return go(single_output_conv_kernel<kF32>);
}

extern "C" OMNI_API int omni_conv_window_gather(const void* padded, int64_t padded_row_stride,
                                                int64_t padded_samples, int64_t rows, int64_t length, int32_t taps,
                                                int32_t dilation, int32_t channels, int32_t element_bytes, void* out,
                                                void* stream) {
  if (rows < 0 || length < 0 || taps <= 0 || dilation <= 0 || channels <= 0)
    return set_error(OMNI_ERR_INVALID, "bad conv window shape");
  if (element_bytes != 2 && element_bytes != 4) return set_error(OMNI_ERR_UNSUPPORTED, "2- or 4-byte elements");
  if (length + (int64_t)(taps - 1) * dilation > padded_samples || padded_row_stride < padded_samples * channels)
    return set_error(OMNI_ERR_INVALID, "padded rows must hold length + (taps - 1) x dilation samples");
  const int64_t seg_bytes = (int64_t)channels * element_bytes;
  if (seg_bytes % 16 != 0 || (padded_row_stride * element_bytes) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(padded) % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "channels, row stride and pointers must be 16-byte multiples");
  const int64_t total = rows * length * taps * (seg_bytes / 16);
  if (total >= ((int64_t)1 << 31)) return set_error(OMNI_ERR_UNSUPPORTED, "output above 32 GiB");
  if (total == 0) return OMNI_OK;
  WindowParams p{};
  p.padded = static_cast<const uint8_t*>(padded);
  p.out = static_cast<uint8_t*>(out);
  p.row_bytes = padded_row_stride * element_bytes;
  p.total = (uint32_t)total;
  p.seg = (uint32_t)(seg_bytes / 16);
  p.taps = (uint32_t)taps;
  p.length = (uint32_t)length;
  p.dil_bytes_vec = (uint32_t)dilation * p.seg;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 8);
  return check_launch(launch(conv_window_gather_kernel, dim3((unsigned)blocks), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), p));
}

extern "C" OMNI_API int omni_history_exchange(void* padded, int64_t padded_row_stride, int64_t padded_sample_stride,
                                              int64_t padded_channel_stride, void* history_pool,
                                              int64_t pool_slot_stride, int64_t pool_sample_stride,
                                              int64_t pool_channel_stride, const int64_t* slot_index, int64_t rows,
                                              int32_t history_samples, int32_t new_samples, int32_t tail_samples,
                                              int32_t channels, int32_t is_cold, int32_t element_bytes,
                                              void* stream) {
  if (rows < 0 || history_samples < 0 || new_samples < 0 || tail_samples < 0 || channels <= 0)
    return set_error(OMNI_ERR_INVALID, "bad history exchange shape");
  if (history_samples > kMaxStateSamples || tail_samples > (1 << 20))
    return set_error(OMNI_ERR_UNSUPPORTED, "history longer than 64 samples");
  if (element_bytes != 2 && element_bytes != 4) return set_error(OMNI_ERR_UNSUPPORTED, "2- or 4-byte elements");
  if (rows == 0) return OMNI_OK;
  HistoryParams p{};
  p.padded = padded;
  p.pr = padded_row_stride;
  p.ps = padded_sample_stride;
  p.pc = padded_channel_stride;
  p.pool = history_pool;
  p.qs_slot = pool_slot_stride;
  p.qs_sample = pool_sample_stride;
  p.qs_channel = pool_channel_stride;
  p.slot_index = slot_index;
  p.history = history_samples;
  p.new_samples = new_samples;
  p.tail = tail_samples;
  p.channels = channels;
  p.cold = is_cold;
  const dim3 grid((unsigned)rows, (unsigned)((channels + kChannelBlock - 1) / kChannelBlock));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (element_bytes == 2)
    return check_launch(launch(history_exchange_kernel<uint16_t>, grid, dim3(kChannelBlock * 4), 0, st, p));
  return check_launch(launch(history_exchange_kernel<uint32_t>, grid, dim3(kChannelBlock * 4), 0, st, p));
}

extern "C" OMNI_API int omni_overlap_exchange(void* output, int64_t output_row_stride, int64_t output_sample_stride,
                                              int64_t output_channel_stride, void* overlap_pool,
                                              int64_t pool_slot_stride, int64_t pool_sample_stride,
                                              int64_t pool_channel_stride, const int64_t* slot_index, int64_t rows,
                                              int32_t overlap_samples, int32_t emitted_samples, int32_t channels,
                                              int32_t is_cold, int32_t dtype, void* stream) {
  if (rows < 0 || overlap_samples < 0 || emitted_samples < 0 || channels <= 0)
    return set_error(OMNI_ERR_INVALID, "bad overlap exchange shape");
  if (emitted_samples < overlap_samples)
    return set_error(OMNI_ERR_INVALID, "emitted samples must cover the overlap");
  if (dtype != kBF16 && dtype != kF16 && dtype != kF32) return set_error(OMNI_ERR_UNSUPPORTED, "unsupported dtype");
  if (rows == 0 || overlap_samples == 0) return OMNI_OK;
  OverlapParams p{};
  p.output = output;
  p.orow = output_row_stride;
  p.osample = output_sample_stride;
  p.ochannel = output_channel_stride;
  p.pool = overlap_pool;
  p.qs_slot = pool_slot_stride;
  p.qs_sample = pool_sample_stride;
  p.qs_channel = pool_channel_stride;
  p.slot_index = slot_index;
  p.overlap = overlap_samples;
  p.emitted = emitted_samples;
  p.channels = channels;
  p.cold = is_cold;
  const dim3 grid((unsigned)rows, (unsigned)((channels + kChannelBlock - 1) / kChannelBlock));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == kBF16) return check_launch(launch(overlap_exchange_kernel<kBF16>, grid, dim3(kChannelBlock * 4), 0, st, p));
  if (dtype == kF16) return check_launch(launch(overlap_exchange_kernel<kF16>, grid, dim3(kChannelBlock * 4), 0, st, p));
  return check_launch(launch(overlap_exchange_kernel<kF32>, grid, dim3(kChannelBlock * 4), 0, st, p));
}
