// Shared device/host helpers for the omni_b200 sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

#include "../../include/omni_b200.h"

#define OMNI_DEVINL __device__ __forceinline__

namespace omni {

// ---------------------------------------------------------------------------
// Device status.  Every bounded wait that gives up records a code here and the
// kernel returns; the host reads it with omni_device_status().  One word per
// translation unit, registered by OMNI_DEFINE_STATUS.
// ---------------------------------------------------------------------------
enum DevStatus : unsigned int {
  kDevOk = 0,
  kDevTimeoutTma = 0x100,
  kDevTimeoutMma = 0x200,
  kDevBadIndex = 0x300,
  kDevTimeoutFlag = 0x400,
};

// Registration of one TU's status word with the host-side aggregator.
typedef unsigned int (*StatusReader)(int reset);
int register_status_reader(StatusReader r);

#define OMNI_DEFINE_STATUS(tu)                                                     \
  static __device__ unsigned int g_status_##tu;                                    \
  static unsigned int read_status_##tu(int reset) {                                \
    unsigned int v = 0;                                                            \
    if (cudaMemcpyFromSymbol(&v, g_status_##tu, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu; \
    if (reset && v) { unsigned int z = 0; cudaMemcpyToSymbol(g_status_##tu, &z, sizeof(z)); } \
    return v;                                                                      \
  }                                                                                \
  static int reg_status_##tu = omni::register_status_reader(read_status_##tu);     \
  static OMNI_DEVINL void report_status(unsigned int code) { atomicCAS(&g_status_##tu, 0u, code); }

// ---------------------------------------------------------------------------
// Programmatic dependent launch.
// ---------------------------------------------------------------------------
OMNI_DEVINL void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
OMNI_DEVINL void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

bool pdl_enabled();
void prefer_max_shared(const void* fn);

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  prefer_max_shared(reinterpret_cast<const void*>(kernel));
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// bf16 helpers
// ---------------------------------------------------------------------------
OMNI_DEVINL float bf2f(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
OMNI_DEVINL uint16_t f2bf(float f) {
  __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&b);
}
OMNI_DEVINL float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
OMNI_DEVINL float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
OMNI_DEVINL uint32_t pack_bf2(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

// Packed fp32 pairs (the .f32x2 forms of sm_100): one instruction works on two
// values held as one 64-bit register pair, lo in the low word.
OMNI_DEVINL uint64_t f2_make(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
OMNI_DEVINL void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
OMNI_DEVINL uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
OMNI_DEVINL uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
OMNI_DEVINL uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
OMNI_DEVINL uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
OMNI_DEVINL float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// bf16 pair of a packed pair of NORMAL or zero values by Veltkamp splitting
// (Dekker 1971): with g = v * (2^16 + 1), hi = g + (v - g) is v rounded to
// the 8 significant bits of bf16, nearest-even, so the result is bit-identical
// to pack_bf2 (checked over every float32 of whole binades from 2^-126 to 2^9).
// Three packed instructions and one byte permute for two values; subnormal
// inputs are outside its domain (the softmax's ex2.approx.ftz makes none).
OMNI_DEVINL uint32_t f2_to_bf2(uint64_t v) {
  const uint64_t sigma = f2_make(65537.0f, 65537.0f);
  const uint64_t g = f2_mul(v, sigma);
  const uint64_t h = f2_add(g, f2_sub(v, g));
  float lo, hi;
  f2_split(h, lo, hi);
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
}

// ---------------------------------------------------------------------------
// Shared-memory / async-proxy primitives (PTX ISA 8.6+, sm_100a).
// ---------------------------------------------------------------------------
OMNI_DEVINL uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// True in exactly one lane of the converged warp.
OMNI_DEVINL bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

OMNI_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
OMNI_DEVINL void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
OMNI_DEVINL void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

OMNI_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
OMNI_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
OMNI_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking test of a phase (for a warp that polls several barriers: try_wait
// may suspend the thread on one barrier while another is already complete).
OMNI_DEVINL bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: about a second of polling at most (try_wait itself suspends
// for a hardware-defined interval).  Returns false on timeout.
constexpr uint32_t kWaitLimit = 1u << 22;
OMNI_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit = kWaitLimit) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// Bounded wait with cluster-scope acquire: for barriers completed by peer CTAs'
// remote stores (st.async), whose data must be visible after the wait.
OMNI_DEVINL bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
OMNI_DEVINL bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
  }
  return false;
}

// TMA: 2D tiled load global -> shared, completion on an mbarrier.
OMNI_DEVINL void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// Bulk prefetch of [src, src + bytes) into L2 (bytes a multiple of 16, src 16-byte aligned).
OMNI_DEVINL void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
OMNI_DEVINL void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core) primitives.
// ---------------------------------------------------------------------------
OMNI_DEVINL void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
OMNI_DEVINL void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::); }
OMNI_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
OMNI_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
OMNI_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
OMNI_DEVINL void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
OMNI_DEVINL void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
OMNI_DEVINL void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit accumulators: thread t of the warp receives
// lane (base_lane + t), columns [col, col + 32).
OMNI_DEVINL void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
OMNI_DEVINL void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// layout that a TMA box of 64 bf16 x rows (SWIZZLE_128B) produces: rows of 128
// bytes, 8-row groups 1024 bytes apart.
OMNI_DEVINL uint64_t smem_desc_sw128(const void* smem_ptr) {
  uint64_t addr = smem_u32(smem_ptr);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;             // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                   // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A bf16
         | (1u << 10)                   // B bf16
         | ((uint32_t)(N >> 3) << 17)   // N
         | ((uint32_t)(M >> 4) << 24);  // M
}

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------
OMNI_DEVINL float warp_sum_xor(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  return v;
}
OMNI_DEVINL float warp_max_xor(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
  return v;
}

}  // namespace omni
