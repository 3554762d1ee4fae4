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
// (S <= 16, chosen so that every cluster of the grid is co-resident).  Each
// CTA stages its fp32 partial tile in its own shared memory; after a hardware
// cluster barrier, CTA c reduces rows c, c + S, ... of the tile by reading all
// S partials over distributed shared memory in split order (deterministic),
// applies the epilogue and stores the result.  No global scratch memory.
//
// Programmatic dependent launch: weights never depend on the previous kernel,
// so the producer issues the first stages' weight loads before
// griddepcontrol.wait, overlapping them with the predecessor's tail.
//
// Roles (128 threads): warp 0 lane 0 = TMA producer, warp 1 lane 0 = MMA
// issuer, all four warps = epilogue (warp w reads TMEM lanes 32w..32w+31).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_util.h"
#include "common.cuh"

namespace omni {
namespace {
OMNI_DEFINE_STATUS(gemm)

constexpr int kBK = 64;        // K elements per stage (one 128-byte swizzle row)
constexpr int kTileN = 128;    // output features per CTA (MMA M)
constexpr int kMaxRows = 256;  // activation rows per CTA (MMA N)
constexpr int kMaxStages = 6;
constexpr int kThreadsG = 128;

enum Epilogue : int { kEpiStore = 0, kEpiResidual = 1, kEpiSwiGLU = 2, kEpiF32 = 3 };

struct GemmParams {
  int rows;         // total activation rows
  int K;            // reduction length (multiple of 64)
  int N;            // output features of W (for SwiGLU: 2 * I)
  int row_tile;     // rows per CTA (multiple of 16, <= 256)
  int num_kb;       // K / 64
  int splits;       // CTAs per (feature tile, row tile)
  int stages;       // pipeline depth
  int tmem_cols;    // power of two >= row_tile
  int swiglu_half;  // I for SwiGLU (gate rows [0, I), up rows [I, 2I))
  const uint16_t* residual;
  int64_t res_stride;
  void* y;
  int64_t y_stride;
};

OMNI_DEVINL uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
OMNI_DEVINL void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
OMNI_DEVINL uint32_t map_cluster(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
OMNI_DEVINL float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

OMNI_DEVINL float silu(float g) { return g / (1.0f + expf(-g)); }

template <int EPI>
__global__ void __launch_bounds__(kThreadsG, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = p.stages;
  const int Rt = p.row_tile;
  const uint32_t a_bytes = kTileN * kBK * 2;
  const uint32_t b_bytes = (uint32_t)Rt * kBK * 2;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + ST * a_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_smem + ST * b_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* mma_done = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, rtile = blockIdx.y, split = blockIdx.z;
  const int kb_begin = (int)(((int64_t)p.num_kb * split) / p.splits);
  const int kb_end = (int)(((int64_t)p.num_kb * (split + 1)) / p.splits);
  const int nk = kb_end - kb_begin;
  const int row0 = rtile * Rt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(mma_done, 1);
    flags[0] = 0;
    flags[1] = 0;
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

  // Weight tile coordinates of k-block kb into stage s.
  auto load_w = [&](int s, int kb) {
    uint8_t* dst = a_smem + s * a_bytes;
    const int kx = kb * kBK;
    if (EPI == kEpiSwiGLU) {
      const int g0 = tile * (kTileN / 2);
      tma_load_2d(dst, &tmap_w, &full[s], kx, g0);
      tma_load_2d(dst + (kTileN / 2) * kBK * 2, &tmap_w, &full[s], kx, p.swiglu_half + g0);
    } else {
      tma_load_2d(dst, &tmap_w, &full[s], kx, tile * kTileN);
    }
  };

  const int pre = nk < ST ? nk : ST;
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], a_bytes + b_bytes);
      load_w(i, kb_begin + i);
    }
  }
  griddep_wait();
  griddep_launch();

  if (warp == 0 && lane == 0) {
    // producer
    for (int i = 0; i < pre; ++i) tma_load_2d(b_smem + i * b_bytes, &tmap_x, &full[i], (kb_begin + i) * kBK, row0);
    for (int i = pre; i < nk; ++i) {
      const int s = i % ST;
      if (!mbar_wait(&empty[s], ((i / ST) - 1) & 1)) {
        report_status(kDevTimeoutMma);
        flags[0] = 1;
        break;
      }
      mbar_arrive_expect_tx(&full[s], a_bytes + b_bytes);
      load_w(s, kb_begin + i);
      tma_load_2d(b_smem + s * b_bytes, &tmap_x, &full[s], (kb_begin + i) * kBK, row0);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer
    const uint32_t idesc = idesc_bf16_f32(kTileN, Rt);
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % ST;
      if (!mbar_wait(&full[s], (i / ST) & 1)) {
        report_status(kDevTimeoutTma);
        flags[0] = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t ad = smem_desc_sw128(a_smem + s * a_bytes);
      const uint64_t bd = smem_desc_sw128(b_smem + s * b_bytes);
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk)
        tc_mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      tc_commit(&empty[s]);
    }
    if (ok) tc_commit(mma_done);
    else mbar_arrive(mma_done);
  }
  __syncwarp();

  // ---- epilogue: TMEM -> smem staging [Rt][128] fp32 ----
  float* stage = reinterpret_cast<float*>(smem);  // reuses the drained pipeline buffers
  const bool have_acc = nk > 0;
  if (have_acc) {
    if (!mbar_wait(mma_done, 0)) {
      report_status(kDevTimeoutMma);
      flags[0] = 1;
    }
  }
  tc_fence_after();
  __syncthreads();
  const bool aborted = flags[0] != 0;
  if (!aborted) {
    const int f = warp * 32 + lane;
    for (int c0 = 0; c0 < Rt; c0 += 32) {
      uint32_t r[32];
      if (have_acc) {
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < Rt) stage[(c0 + j) * kTileN + f] = __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, (uint32_t)p.tmem_cols);

  // ---- split-K reduction over the cluster's shared memory ----
  // Every CTA takes part in both cluster barriers, aborted or not.
  const int S = p.splits;
  if (S > 1) cluster_sync();  // all partial tiles staged and visible cluster-wide
  const uint32_t crank = S > 1 ? cluster_ctarank() : 0u;
  const uint32_t stage_local = smem_u32(stage);
  const bool any_abort = aborted;
  const int rows_here = min(Rt, p.rows - row0);
  // partial of split s, row r, features f..f+3 (s in split order)
  auto acc4 = [&](int r, int f) -> float4 {
    const uint32_t off = (uint32_t)((r * kTileN + f) * 4);
    if (S == 1) return *reinterpret_cast<const float4*>(stage + r * kTileN + f);
    float4 a = ld_cluster_f4(map_cluster(stage_local + off, 0));
    for (int q = 1; q < S; ++q) {
      const float4 b = ld_cluster_f4(map_cluster(stage_local + off, (uint32_t)q));
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    return a;
  };
  if (!any_abort) {
    if (EPI == kEpiSwiGLU) {
      // features 0..63: gate, 64..127: up, for outputs tile*64 .. tile*64+63
      uint16_t* Y = static_cast<uint16_t*>(p.y);
      const int nr = (rows_here - (int)crank + S - 1) / S;
      for (int idx = threadIdx.x; idx < nr * 16; idx += kThreadsG) {
        const int r = (int)crank + (idx >> 4) * S;
        const int g = (idx & 15) * 4;
        const float4 gt = acc4(r, g), up = acc4(r, 64 + g);
        const float gg[4] = {gt.x, gt.y, gt.z, gt.w}, uu[4] = {up.x, up.y, up.z, up.w};
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = silu(bf2f(f2bf(gg[j]))) * bf2f(f2bf(uu[j]));
        *reinterpret_cast<uint2*>(Y + (int64_t)(row0 + r) * p.y_stride + tile * 64 + g) =
            make_uint2(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]));
      }
    } else {
      // rows crank, crank + S, ...: 32 threads per row, 4 features each
      const int nr = (rows_here - (int)crank + S - 1) / S;
      for (int idx = threadIdx.x; idx < nr * 32; idx += kThreadsG) {
        const int r = (int)crank + (idx >> 5) * S;
        const int f = (idx & 31) * 4;
        const int64_t col = (int64_t)tile * kTileN + f;
        const float4 a = acc4(r, f);
        float o[4] = {a.x, a.y, a.z, a.w};
        if (EPI == kEpiF32) {
          float* Y = static_cast<float*>(p.y);
          *reinterpret_cast<float4*>(Y + (int64_t)(row0 + r) * p.y_stride + col) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
          if (EPI == kEpiResidual) {
            const uint2 rv = *reinterpret_cast<const uint2*>(p.residual + (int64_t)(row0 + r) * p.res_stride + col);
            o[0] += bf_lo(rv.x);
            o[1] += bf_hi(rv.x);
            o[2] += bf_lo(rv.y);
            o[3] += bf_hi(rv.y);
          }
          uint16_t* Y = static_cast<uint16_t*>(p.y);
          *reinterpret_cast<uint2*>(Y + (int64_t)(row0 + r) * p.y_stride + col) =
              make_uint2(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]));
        }
      }
    }
  }
  if (S > 1) cluster_sync();  // no CTA leaves while a peer still reads its partial
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
  int row_tile, num_rt, tiles, num_kb, splits, stages, tmem_cols;
  size_t smem;
};

int num_sms() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

constexpr int kMaxSplits = 16;

template <int EPI>
void set_kernel_attrs() {
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(gemm_kernel<EPI>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  });
}

// Co-resident clusters of S CTAs with this much shared memory (cached).
template <int EPI>
int max_active_clusters(int S, size_t smem) {
  static std::mutex mu;
  static int cache[kMaxSplits + 1][64];  // [S][smem KB / 4]
  static bool init = false;
  std::lock_guard<std::mutex> g(mu);
  if (!init) {
    for (auto& row : cache)
      for (int& v : row) v = -1;
    init = true;
  }
  const int key = (int)((smem + 4095) / 4096);
  if (key >= 64) return 0;
  int& slot = cache[S][key];
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
  slot = n;
  return n;
}

size_t plan_smem(int row_tile, int stages) {
  const size_t stage_bytes = (size_t)kTileN * kBK * 2 + (size_t)row_tile * kBK * 2;
  return 1024 + (size_t)stages * stage_bytes + 2 * kMaxStages * 8 + 8 + 16;
}

int plan_stages(int row_tile, int kb_per) {
  const size_t stage_bytes = (size_t)kTileN * kBK * 2 + (size_t)row_tile * kBK * 2;
  int st = kb_per < 4 ? kb_per : 4;
  if (st < 1) st = 1;
  // the epilogue staging [row_tile][128] fp32 reuses the stage buffers
  const size_t staging = (size_t)row_tile * kTileN * 4;
  while ((size_t)st * stage_bytes < staging && st < kMaxStages) ++st;
  return st;
}

template <int EPI>
Plan make_plan(int64_t rows, int64_t k, int64_t n, int splits_req) {
  Plan pl{};
  int nrt = (int)((rows + kMaxRows - 1) / kMaxRows);
  if (nrt < 1) nrt = 1;
  int64_t per = (rows + nrt - 1) / nrt;
  pl.row_tile = (int)((per + 15) / 16 * 16);
  if (pl.row_tile < 16) pl.row_tile = 16;
  if (pl.row_tile > kMaxRows) pl.row_tile = kMaxRows;
  // every row tile starts inside the activation rows
  pl.num_rt = (int)((rows + pl.row_tile - 1) / pl.row_tile);
  if (pl.num_rt < 1) pl.num_rt = 1;
  pl.tiles = (int)(EPI == kEpiSwiGLU ? (n / 2) / (kTileN / 2) : n / kTileN);
  pl.num_kb = (int)(k / kBK);
  const int clusters = pl.tiles * pl.num_rt;
  int best = 1;
  if (splits_req > 0) {
    best = splits_req;
  } else {
    // the widest split whose clusters all fit in one wave, preferring more busy SMs
    long best_busy = 0;
    for (int S = 1; S <= kMaxSplits && S <= pl.num_kb; ++S) {
      const int st = plan_stages(pl.row_tile, (pl.num_kb + S - 1) / S);
      const int fit = S == 1 ? num_sms() : max_active_clusters<EPI>(S, plan_smem(pl.row_tile, st));
      if (clusters > fit) continue;
      const long busy = (long)clusters * S;
      if (busy > best_busy) {
        best_busy = busy;
        best = S;
      }
    }
  }
  if (best > pl.num_kb) best = pl.num_kb;
  if (best < 1) best = 1;
  pl.splits = best;
  pl.stages = plan_stages(pl.row_tile, (pl.num_kb + best - 1) / best);
  int tc = 32;
  while (tc < pl.row_tile) tc <<= 1;
  pl.tmem_cols = tc;
  pl.smem = plan_smem(pl.row_tile, pl.stages);
  return pl;
}

template <int EPI>
int launch_gemm(const void* x, int64_t rows, int64_t k, int64_t x_stride, const void* w, int64_t n,
                const void* residual, int64_t residual_stride, void* y, int64_t y_stride, int splits_req,
                cudaStream_t st) {
  const Plan pl = make_plan<EPI>(rows, k, n, splits_req);
  if (pl.splits > kMaxSplits) return set_error(OMNI_ERR_UNSUPPORTED, "at most 16 K-splits");
  CUtensorMap tw, tx;
  const int wbox = EPI == kEpiSwiGLU ? kTileN / 2 : kTileN;
  if (!make_tmap(&tw, w, n, k, k, wbox) || !make_tmap(&tx, x, rows, k, x_stride, pl.row_tile))
    return set_error(OMNI_ERR_UNSUPPORTED, "tensor map encoding failed");
  GemmParams gp{};
  gp.rows = (int)rows;
  gp.K = (int)k;
  gp.N = (int)n;
  gp.row_tile = pl.row_tile;
  gp.num_kb = pl.num_kb;
  gp.splits = pl.splits;
  gp.stages = pl.stages;
  gp.tmem_cols = pl.tmem_cols;
  gp.swiglu_half = (int)(n / 2);
  gp.residual = static_cast<const uint16_t*>(residual);
  gp.res_stride = residual_stride;
  gp.y = y;
  gp.y_stride = y_stride;
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

}  // namespace
}  // namespace omni

using namespace omni;

extern "C" OMNI_API int64_t omni_linear_workspace_bytes(int64_t rows, int64_t k, int64_t n, int32_t epilogue,
                                                        int32_t splits) {
  (void)rows, (void)k, (void)n, (void)epilogue, (void)splits;
  return 0;  // split-K partials are reduced in distributed shared memory
}

extern "C" OMNI_API int omni_linear(const void* x, int64_t rows, int64_t k, int64_t x_stride, const void* w,
                                    int64_t n, int32_t epilogue, const void* residual, int64_t residual_stride,
                                    void* y, int64_t y_stride, void* workspace, int64_t workspace_bytes_avail,
                                    int32_t splits, void* stream) {
  (void)workspace, (void)workspace_bytes_avail;
  if (rows < 0 || k <= 0 || n <= 0) return set_error(OMNI_ERR_INVALID, "bad GEMM shape");
  if (epilogue < 0 || epilogue > 3) return set_error(OMNI_ERR_INVALID, "unknown epilogue");
  if (splits < 0 || splits > kMaxSplits) return set_error(OMNI_ERR_INVALID, "splits must be in [0, 16]");
  if (k % kBK != 0) return set_error(OMNI_ERR_UNSUPPORTED, "K must be a multiple of 64");
  if (n % kTileN != 0) return set_error(OMNI_ERR_UNSUPPORTED, "N must be a multiple of 128");
  auto mis16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  if (mis16(x) || mis16(w) || (x_stride % 8) != 0 || mis16(y) || (y_stride % 4) != 0)
    return set_error(OMNI_ERR_UNSUPPORTED, "operands must be 16-byte aligned with 16-byte row strides");
  if (epilogue == kEpiResidual && (residual == nullptr || (residual_stride % 4) != 0 ||
                                   (reinterpret_cast<uintptr_t>(residual) & 7) != 0))
    return set_error(OMNI_ERR_INVALID, "residual epilogue needs an 8-byte aligned residual");
  if (rows == 0) return OMNI_OK;
  if (splits > k / kBK) splits = (int32_t)(k / kBK);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (epilogue) {
    case kEpiStore: return launch_gemm<kEpiStore>(x, rows, k, x_stride, w, n, residual, residual_stride, y, y_stride, splits, st);
    case kEpiResidual: return launch_gemm<kEpiResidual>(x, rows, k, x_stride, w, n, residual, residual_stride, y, y_stride, splits, st);
    case kEpiSwiGLU: return launch_gemm<kEpiSwiGLU>(x, rows, k, x_stride, w, n, residual, residual_stride, y, y_stride, splits, st);
    default: return launch_gemm<kEpiF32>(x, rows, k, x_stride, w, n, residual, residual_stride, y, y_stride, splits, st);
  }
}
