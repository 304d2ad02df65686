// Shared device helpers for the sm_100a kernels: mbarrier, TMA (cp.async.bulk[.tensor]), tcgen05 / TMEM,
// programmatic dependent launch, bounded waits and error reporting.
//
// Every spin-wait in these kernels is bounded by the global timer (GR_WAIT_NS); a wait that runs out records an
// error code in the caller's status word and the kernel tears down instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gravity_b200.h"

#ifndef GR_WAIT_NS
#define GR_WAIT_NS 2000000000ull  // 2 s
#endif
// Tuning knobs of the projection kernel (compile-time; the defaults are the measured best).
#ifndef GR_W_EVICT_FIRST
#define GR_W_EVICT_FIRST 1  // weight tiles loaded with an L2 evict-first hint
#endif
#ifndef GR_MAX_STAGES
#define GR_MAX_STAGES 8     // deepest TMA ring
#endif
#ifndef GR_MAX_NT
#define GR_MAX_NT 256       // widest token tile (MMA N)
#endif

namespace gr {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------------ launch timeline (timeline build only)
// Built with -DGR_TIMELINE (python -m gravityocr_b200.build --timeline): thread 0 of every CTA of every round kernel
// appends (kind, block, entry, exit) globaltimer stamps to its translation unit's record array, and a (0, block, t, t)
// record when griddepcontrol.wait returns; the host reads them with gr_timeline_read_<unit>.  This shows each
// launch's dependency release and its CTAs' critical path as the graphs replay, which a serialising profiler does
// not.  The product build compiles all of it out.
#ifdef GR_TIMELINE
struct TimelineRec {
  uint32_t kind, block;
  uint64_t t0, t1;
};
constexpr uint32_t kTimelineCap = 1u << 19;
static __device__ TimelineRec g_timeline[kTimelineCap];
static __device__ uint32_t g_timeline_n;
__device__ __forceinline__ void timeline_put(uint32_t kind, uint64_t t0, uint64_t t1) {
  const uint32_t i = atomicAdd(&g_timeline_n, 1u);
  if (i < kTimelineCap) {
    TimelineRec r;
    r.kind = kind;
    r.block = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    r.t0 = t0;
    r.t1 = t1;
    g_timeline[i] = r;
  }
}
#define GR_TL_BEGIN const uint64_t gr_tl_t0 = globaltimer();
#define GR_TL_END(kind) \
  if (threadIdx.x == 0) timeline_put((kind), gr_tl_t0, globaltimer());
#define GR_TL_DEP                        \
  if (threadIdx.x == 0) {                \
    const uint64_t gr_tl_t = globaltimer(); \
    timeline_put(0, gr_tl_t, gr_tl_t);   \
  }
#define GR_TIMELINE_EXPORTS(unit)                                                                              \
  extern "C" int gr_timeline_read_##unit(void* host, uint32_t* n) {                                           \
    if (cudaMemcpyFromSymbol(n, gr::g_timeline_n, sizeof(uint32_t)) != cudaSuccess) return 1;                \
    const uint32_t m = *n < gr::kTimelineCap ? *n : gr::kTimelineCap;                                          \
    return cudaMemcpyFromSymbol(host, gr::g_timeline, m * sizeof(gr::TimelineRec)) == cudaSuccess ? 0 : 1;    \
  }                                                                                                            \
  extern "C" int gr_timeline_clear_##unit(void) {                                                              \
    const uint32_t z = 0;                                                                                      \
    return cudaMemcpyToSymbol(gr::g_timeline_n, &z, sizeof(uint32_t)) == cudaSuccess ? 0 : 1;                  \
  }
#else
#define GR_TL_BEGIN
#define GR_TL_END(kind)
#define GR_TL_DEP
#define GR_TIMELINE_EXPORTS(unit)
#endif
// kinds of the timeline records (linear kernels: kTlLinear + epilogue mode)
enum : uint32_t {
  kTlAttentionMma = 1,
  kTlAttentionTc = 2,
  kTlArgmaxReduce = 3,
  kTlResidualNorm = 4,
  kTlEmbed = 6,
  kTlCommit = 7,
  kTlLogitsProcess = 8,
  kTlSampleRows = 9,
  kTlPenaltyCumulate = 5,
  kTlLinear = 10
};

// ------------------------------------------------------------------ programmatic dependent launch
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  GR_TL_DEP
}
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
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
// Non-blocking probe (test_wait: returns at once), for a thread that polls several barriers.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity) {
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
// Bounded wait for the phase with the given parity to complete.  Returns false (and records `code`) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if (globaltimer() - t0 > GR_WAIT_NS) {
      report(status, code);
      return false;
    }
  }
}

// ------------------------------------------------------------------ TMA / bulk copies
__device__ __forceinline__ void tma_prefetch_desc(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled tensor load into shared memory; x is the innermost (contiguous) coordinate in elements.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// 2-D tiled load with an L2 eviction-priority hint (weights are read once per forward: evict first).
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// L2 prefetch of a contiguous global range (16-byte aligned address and size).
__device__ __forceinline__ void l2_prefetch(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
               : "memory");
}
// Make generic-proxy shared-memory writes visible to the async proxy (TMA / tensor core reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate), issued by one thread.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Split form for software pipelining: issue a 16-column load, later wait for it.  The wait names the destination
// registers as operands so that no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns per thread: issue (wait with tmem_wait_ld) and store (wait with
// tmem_wait_st).
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld32_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major operand in the 128-byte-swizzle canonical layout (8 rows x 128 B atoms,
// 1024 B between 8-row groups), sm100 descriptor version 1.  `addr` is the shared-space byte address.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;             // leading byte offset (unused for swizzled K-major), 16 B
  d |= static_cast<uint64_t>(1024 >> 4) << 32;     // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1) << 46;             // descriptor version (sm100)
  d |= static_cast<uint64_t>(2) << 61;             // SWIZZLE_128B
  return d;
}
// MN-major operand in the 128-byte-swizzle canonical layout: each K index (reduction row) is a 128-byte line of 64
// consecutive MN elements, 8 such lines form a 1024-byte swizzle group (stride byte offset: the next 8 K rows), and
// the next 64 MN elements start `mn_block_bytes` further on (leading byte offset).
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t addr, uint32_t mn_block_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((mn_block_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// Instruction descriptor: bf16 x bf16 -> fp32, both operands K-major, M x N tile.  (Bit 16 set: B is MN-major.)
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// ------------------------------------------------------------------ warp-level mma.sync (attention)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled tile whose base is 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ------------------------------------------------------------------ RoPE angles
// sin and cos of an fp32 angle, |x| < 2^22, to about 1 ulp absolute, in registers (no table, no local memory):
// Cody-Waite reduction by pi/2 with a three-part split of pi/2 (each product subtracted by one fma), then the Taylor
// series of sin (to r^9) and cos (to r^10) on |r| <= pi/4, whose truncation error is below 2e-9.
__device__ __forceinline__ void rope_sincos(float x, float* s_out, float* c_out) {
  const float q = rintf(x * 0.636619747f);  // x * 2/pi
  float r = fmaf(q, -1.57079637f, x);       // pi/2 = 1.57079637f - 4.37113883e-8f - 1.71512451e-15f
  r = fmaf(q, 4.37113883e-8f, r);
  r = fmaf(q, 1.71512451e-15f, r);
  const float r2 = r * r;
  float ps = fmaf(r2, 2.75573188e-6f, -1.98412701e-4f);  // 1/9!, -1/7!
  ps = fmaf(r2, ps, 8.33333377e-3f);                        // 1/5!
  ps = fmaf(r2, ps, -0.166666672f);                         // -1/3!
  const float sn = fmaf(r2 * r, ps, r);
  float pc = fmaf(r2, -2.75573200e-7f, 2.48015876e-5f);   // -1/10!, 1/8!
  pc = fmaf(r2, pc, -1.38888892e-3f);                       // -1/6!
  pc = fmaf(r2, pc, 4.16666679e-2f);                        // 1/4!
  pc = fmaf(r2, pc, -0.5f);                                 // -1/2!
  const float cs = fmaf(r2, pc, 1.0f);
  const int qi = static_cast<int>(q) & 3;
  const float s1 = (qi & 1) ? cs : sn;
  const float c1 = (qi & 1) ? sn : cs;
  *s_out = (qi & 2) ? -s1 : s1;
  *c_out = ((qi + 1) & 2) ? -c1 : c1;
}

// ------------------------------------------------------------------ misc
// 2^x (PTX ex2.approx.ftz: relative error ~2^-22, subnormal results flushed to zero; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace gr
