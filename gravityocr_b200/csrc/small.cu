// Persistent forward for small batches (M = bs * K <= 64 rows), sm_100a.
//
// At batch 1 a forward is ~115 dependent launches of a few µs each, and most of each launch is pipeline fill, split-K
// reduction and the hand-off to the next launch, not the weight stream.  This kernel runs the same phases inside one
// cooperative launch (one CTA per SM), with a grid barrier between phases:
//   per layer  QKV + RoPE + K/V write | attention | o_proj partials | residual norm | gate_up + SwiGLU | down partials
//              | residual norm,  then lm_head records | argmax reduction.
// Every phase runs the same device code, on the same parameters, as the per-launch kernels (linear_dev.cuh,
// attention_dev.cuh, rowwise_dev.cuh), so its results are those of the per-launch forward.
//
// Roles per CTA (320 threads):
//   warp 0     projection producer: walks this CTA's (unit, K chunk) sequence of every projection phase through one
//              S-stage TMA ring.  Weights do not depend on the activations, so at the start of a projection phase it
//              issues the weight tiles of up to S stages at once and issues their activation tiles only after the
//              grid barrier of the phase before: the weight stream runs ahead of the barrier, under the attention and
//              norm phases.
//   warp 1     TMEM (double-buffered accumulators) and the tcgen05.mma issue loop.
//   warps 2-9  workers: projection epilogues, attention units (two warp groups, 2-stage ring, own TMA producer warp),
//              residual norms and the argmax reduction; they arrive on and wait for the grid barriers.
// Grid barrier p: each CTA's workers finish phase p, fence, add 1 to done[p]; phase p + 1 starts when done[p] equals
// the grid size.  The last CTA to leave re-arms the counters for the next launch.  Every wait is bounded; a wait that
// runs out records GR_ERR_TIMEOUT and raises the plan's abort flag, which every loop checks.
#include "attention_dev.cuh"
#include "linear_dev.cuh"
#include "rowwise_dev.cuh"

namespace gr {

constexpr int kSmallThreads = 320;
constexpr int kSmallWorkers = 256;  // warps 2-9
constexpr int kSmallAttnStages = 2;
constexpr int kBarWorkers = 1;      // named barrier: all workers (also the epilogue barrier of linear_dev.cuh)
constexpr int kBarAttnCompute = 4;  // named barrier: the attention compute warps
constexpr int kBarResNorm = 5;      // named barrier: the residual-norm threads
constexpr int kResNormThreads = 192;

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// The launch unwinds after any recorded error (a bounded wait that ran out anywhere, including inside a phase body).
__device__ __forceinline__ bool aborted(const SmallArgs& a) {
  return *reinterpret_cast<volatile int*>(a.abort) != 0 ||
         (a.status && *reinterpret_cast<volatile int*>(a.status) != 0);
}
__device__ __forceinline__ void raise_abort(const SmallArgs& a, int code) {
  report(a.status, code);
  atomicExch(a.abort, 1);
}
// Bounded wait until phase p is done on every CTA (p < 0: nothing to wait for).
__device__ bool wait_phase(const SmallArgs& a, int p) {
  if (p < 0) return true;
  const int n = static_cast<int>(gridDim.x);
  if (ld_acquire(a.done + p) >= n) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (ld_acquire(a.done + p) >= n) return true;
    if (aborted(a)) return false;
    if (globaltimer() - t0 > GR_WAIT_NS) {
      raise_abort(a, GR_ERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ void decode_unit(const LinearParams& p, int u, int& m_tile, int& split, int& n_tile) {
  m_tile = u % p.m_tiles;
  u /= p.m_tiles;
  split = u % p.splits;
  n_tile = u / p.splits;
}
__device__ __forceinline__ int n_units(const LinearParams& p) { return p.n_tiles * p.m_tiles * p.splits; }

// Phase bodies are separate (not inlined) functions: each gets its own register allocation instead of one kernel-wide
// allocation for every path.
template <int EPI>
__device__ __noinline__ void epilogue_dispatch_t(const LinearParams& p, uint32_t t_lane, int n_tile, int m_tile,
                                                    int split, bool run, float* scratch, int* flag_last,
                                                    uint64_t* acc_empty) {
  unit_epilogue<EPI>(p, t_lane, n_tile, m_tile, split, run, scratch, flag_last, acc_empty);
}
__device__ void epilogue_dispatch(int epi, const LinearParams& p, uint32_t t_lane, int n_tile, int m_tile, int split,
                                  bool run, float* scratch, int* flag_last, uint64_t* acc_empty) {
  switch (epi) {
    case GR_EPI_STORE_F32:
      epilogue_dispatch_t<GR_EPI_STORE_F32>(p, t_lane, n_tile, m_tile, split, run, scratch, flag_last, acc_empty);
      break;
    case GR_EPI_STORE_BF16:
      epilogue_dispatch_t<GR_EPI_STORE_BF16>(p, t_lane, n_tile, m_tile, split, run, scratch, flag_last, acc_empty);
      break;
    case GR_EPI_SWIGLU:
      epilogue_dispatch_t<GR_EPI_SWIGLU>(p, t_lane, n_tile, m_tile, split, run, scratch, flag_last, acc_empty);
      break;
    case GR_EPI_QKV_ROPE:
      epilogue_dispatch_t<GR_EPI_QKV_ROPE>(p, t_lane, n_tile, m_tile, split, run, scratch, flag_last, acc_empty);
      break;
    case GR_EPI_ARGMAX:
      epilogue_dispatch_t<GR_EPI_ARGMAX>(p, t_lane, n_tile, m_tile, split, run, scratch, flag_last, acc_empty);
      break;
    default:
      epilogue_dispatch_t<GR_EPI_PARTIAL_F32>(p, t_lane, n_tile, m_tile, split, run, scratch, flag_last, acc_empty);
      break;
  }
}

__device__ __forceinline__ void attention_call(const CUtensorMap* tmk, const CUtensorMap* tmv, const AttnParams& p,
                                            int split, int kvh, int b, int wt, AttnCta& ac) {
  attention_unit<kSmallAttnStages>(tmk, tmv, p, split, kvh, b, wt, kSmallWorkers, kBarWorkers, kBarAttnCompute, ac);
}
__device__ __noinline__ void resnorm_call(const ResNormParams& p, int row, int wt, float* red) {
  resnorm_row(p, row, wt, kResNormThreads, kBarResNorm, red);
}

// ------------------------------------------------------------------ warp 0: projection producer
__device__ void small_producer(const SmallArgs& a, uint8_t* w_smem, uint8_t* x_smem, uint64_t* full, uint64_t* empty) {
  const int S = a.stages;
  const uint32_t x_stage_bytes = static_cast<uint32_t>(a.nt) * 128u;
  const uint64_t pol = policy_evict_first();
  int st = 0;             // next stage
  uint32_t round = 0;     // passes over the ring so far (the stage's previous use is round - 1)
  long long issued = 0;   // k-blocks issued into the ring
  int pend_st[GR_MAX_STAGES], pend_xk[GR_MAX_STAGES], pend_row[GR_MAX_STAGES];
  bool stop = false;
  for (int ph = 0; ph < a.n_phases && !stop && !aborted(a); ++ph) {
    const SmallPhase& P = a.phases[ph];
    if (P.type != SP_LINEAR) continue;
    const LinearParams& p = P.lin;
    const CUtensorMap* tmw = a.maps + P.map_a;
    const CUtensorMap* tmx = a.maps + P.map_b;
    const int kc = p.kc_per_split;
    int n_pend = 0;
    bool ready = ph == 0;  // the first phase reads rows written before the launch
    auto release = [&]() {  // the phase's inputs are complete on every CTA: send the held activation tiles
      if (n_pend > 0) {
        wait_phase(a, ph - 1);  // on abort the held stages are released all the same, so that the ring drains
        fence_proxy_async_global();
        for (int i = 0; i < n_pend; ++i)
          tma_load_2d(x_smem + pend_st[i] * x_stage_bytes, tmx, full + pend_st[i], pend_xk[i], pend_row[i]);
      }
      n_pend = 0;
      ready = true;
    };
    for (int u = blockIdx.x; u < n_units(p) && !stop; u += gridDim.x) {
      int m_tile, split, n_tile;
      decode_unit(p, u, m_tile, split, n_tile);
      int xk = split * kc * 64;
      for (int c = 0; c < kc; ++c, xk += 64) {
        if (!ready && n_pend == S) release();  // the ring is full of held stages: only the barrier frees it
        if (issued >= S && !mbar_wait(empty + st, (round - 1) & 1, a.status, GR_ERR_TIMEOUT)) {
          raise_abort(a, GR_ERR_TIMEOUT);
          stop = true;
          break;
        }
        mbar_arrive_expect_tx(full + st, kWStageBytes + x_stage_bytes);
        if (GR_W_EVICT_FIRST)
          tma_load_2d_hint(w_smem + st * kWStageBytes, tmw, full + st, xk, n_tile * 128, pol);
        else
          tma_load_2d(w_smem + st * kWStageBytes, tmw, full + st, xk, n_tile * 128);
        if (ready) {
          tma_load_2d(x_smem + st * x_stage_bytes, tmx, full + st, xk, m_tile * p.nt);
        } else {
          pend_st[n_pend] = st;
          pend_xk[n_pend] = xk;
          pend_row[n_pend] = m_tile * p.nt;
          ++n_pend;
        }
        ++issued;
        if (++st == S) {
          st = 0;
          ++round;
        }
      }
    }
    if (!ready) release();
  }
  // no copy may still be landing in shared memory when the CTA exits: the last stages' full phases
  const long long first = issued > S ? issued - S : 0;
  for (long long g = first; g < issued; ++g)
    if (!mbar_wait(full + (g % S), (g / S) & 1, a.status, GR_ERR_TIMEOUT)) break;
}

// ------------------------------------------------------------------ warp 1: MMA issue
__device__ void small_mma(const SmallArgs& a, uint32_t tmem, uint32_t acc_cols, uint8_t* w_smem, uint8_t* x_smem,
                          uint64_t* full, uint64_t* empty, uint64_t* acc_full, uint64_t* acc_empty) {
  const int S = a.stages;
  const uint32_t x_stage_bytes = static_cast<uint32_t>(a.nt) * 128u;
  const uint32_t idesc = idesc_bf16_f32(128, a.nt);
  const uint64_t a0 = smem_desc_sw128(smem_u32(w_smem)), b0 = smem_desc_sw128(smem_u32(x_smem));
  int st = 0;
  uint32_t par = 0;
  int ku = 0;  // projection units of this CTA so far (accumulator buffer ku & 1)
  for (int ph = 0; ph < a.n_phases; ++ph) {
    const SmallPhase& P = a.phases[ph];
    if (P.type != SP_LINEAR) continue;
    const LinearParams& p = P.lin;
    const int kc = p.kc_per_split;
    for (int u = blockIdx.x; u < n_units(p); u += gridDim.x, ++ku) {
      if (aborted(a)) return;
      const int b = ku & 1;
      if (ku >= 2 && !mbar_wait(acc_empty + b, ((ku >> 1) - 1) & 1, a.status, GR_ERR_TIMEOUT)) {
        raise_abort(a, GR_ERR_TIMEOUT);
        return;
      }
      tc_fence_after();
      const uint32_t acc = tmem + b * acc_cols;
      for (int c = 0; c < kc; ++c) {
        if (!mbar_wait(full + st, par, a.status, GR_ERR_TIMEOUT)) {
          raise_abort(a, GR_ERR_TIMEOUT);
          return;
        }
        tc_fence_after();
        const uint64_t ad = a0 + ((static_cast<uint32_t>(st) * kWStageBytes) >> 4);
        const uint64_t bd = b0 + ((static_cast<uint32_t>(st) * x_stage_bytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tc_mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc, (c | kk) != 0);
        tc_commit(empty + st);
        if (++st == S) {
          st = 0;
          par ^= 1u;
        }
      }
      tc_commit(acc_full + b);
    }
  }
}

// ------------------------------------------------------------------ warps 2-9: workers
__device__ void small_workers(const SmallArgs& a, uint32_t tmem, uint32_t acc_cols, float* scratch, int* flags,
                              uint64_t* acc_full, uint64_t* acc_empty, AttnCta& ac, float* red) {
  const int wt = threadIdx.x - 64;
  const int warp = threadIdx.x >> 5;
  const int quad = warp & 3;
  int ku = 0;
  for (int ph = 0; ph < a.n_phases; ++ph) {
    const SmallPhase& P = a.phases[ph];
    const bool live = !aborted(a);
    if (P.type == SP_LINEAR) {
      const LinearParams& p = P.lin;
      for (int u = blockIdx.x; u < n_units(p); u += gridDim.x, ++ku) {
        int m_tile, split, n_tile;
        decode_unit(p, u, m_tile, split, n_tile);
        const int b = ku & 1;
        bool ok = !aborted(a) && mbar_wait(acc_full + b, (ku >> 1) & 1, a.status, GR_ERR_TIMEOUT);
        tc_fence_after();
        const uint32_t t_lane = tmem + b * acc_cols + (static_cast<uint32_t>(quad * 32) << 16);
        epi_bar();
        ok = ok && !aborted(a);
        epilogue_dispatch(P.epi, p, t_lane, n_tile, m_tile, split, ok, scratch, &flags[1], acc_empty + b);
        epi_bar();
      }
    } else if (P.type == SP_ATTENTION && live) {
      const AttnParams& p = P.att;
      const int units = p.bs * p.n_kv_heads * p.max_splits;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int split = u % p.max_splits, kvh = (u / p.max_splits) % p.n_kv_heads;
        const int zb = u / (p.max_splits * p.n_kv_heads);
        const int b = p.order ? p.order[zb] : zb;
        attention_call(a.maps + P.map_a, a.maps + P.map_b, p, split, kvh, b, wt, ac);
        named_bar(kBarWorkers, kSmallWorkers);  // the next unit restages the query rows
      }
    } else if (P.type == SP_RESNORM && live) {
      // the per-launch kernel's 192 threads per row, so that the sums run in the same order
      if (wt < kResNormThreads)
        for (int row = blockIdx.x; row < P.rn.m; row += gridDim.x)
          resnorm_call(P.rn, row, wt, red);
    } else if (P.type == SP_ARGREDUCE && live) {
      for (int t = blockIdx.x * 8 + (wt >> 5); t < P.lin.m; t += gridDim.x * 8) argmax_reduce_token(P.lin, t);
    }
    // grid barrier after phase ph
    named_bar(kBarWorkers, kSmallWorkers);
    if (wt == 0) {
      __threadfence();
      atomicAdd(a.done + ph, 1);
      wait_phase(a, ph);
      __threadfence();
    }
    named_bar(kBarWorkers, kSmallWorkers);
    fence_proxy_async_global();  // the next phase's TMA loads read what other CTAs stored in this one
  }
}

__global__ void __launch_bounds__(kSmallThreads, 1) small_forward_kernel(const SmallArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const uint32_t x_stage_bytes = static_cast<uint32_t>(a.nt) * 128u;
  uint8_t* w_smem = smem;
  uint8_t* x_smem = w_smem + S * kWStageBytes;
  float* scratch = reinterpret_cast<float*>(x_smem + S * x_stage_bytes);  // 16 KB (argmax transpose)
  uint8_t* attn_region = reinterpret_cast<uint8_t*>(scratch) + 16384;       // 1024-aligned
  AttnCta ac = attn_cta_layout<kSmallAttnStages>(attn_region, a.attn_rows_pad);
  uint64_t* bars = reinterpret_cast<uint64_t*>(attn_region + attn_region_bytes(a.attn_rows_pad, kSmallAttnStages));
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [1] last split
  float* red = reinterpret_cast<float*>(flags + 4);    // 32 floats
  const uint32_t acc_cols = a.nt <= 32 ? 32u : 64u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 8);  // one arrival per epilogue warp
    }
    for (int s = 0; s < kSmallAttnStages; ++s) {
      mbar_init(ac.full + s, 1);
      mbar_init(ac.empty + s, a.attn_row_tiles);
    }
    *ac.flag = 0;
    flags[0] = flags[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * acc_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) small_producer(a, w_smem, x_smem, full, empty);
  } else if (warp == 1) {
    if (lane == 0) small_mma(a, tmem, acc_cols, w_smem, x_smem, full, empty, acc_full, acc_empty);
  } else {
    small_workers(a, tmem, acc_cols, scratch, flags, acc_full, acc_empty, ac, red);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * acc_cols);
  }
  // the last CTA out re-arms the grid barriers (and clears an abort) for the next launch
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.exited, 1) == static_cast<int>(gridDim.x) - 1) {
      for (int p = 0; p < a.n_phases; ++p) a.done[p] = 0;
      *a.abort = 0;
      __threadfence();
      *a.exited = 0;
    }
  }
}

size_t small_smem_bytes(int nt, int stages, int attn_rows_pad) {
  return 1024 + static_cast<size_t>(stages) * (kWStageBytes + static_cast<size_t>(nt) * 128) + 16384 +
         attn_region_bytes(attn_rows_pad, kSmallAttnStages) + (2 * stages + 4) * 8 + 8 + 16 + 128;
}

cudaError_t launch_small_forward(const SmallArgs& a, int grid, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(small_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(small_forward_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kSmallThreads);
  cfg.dynamicSmemBytes = small_smem_bytes(a.nt, a.stages, a.attn_rows_pad);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers rely on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, small_forward_kernel, a);
}

}  // namespace gr
