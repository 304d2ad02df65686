// Weight-streaming GEMM for the decoder's projections and lm_head, sm_100a (tcgen05 + TMA + TMEM).
//
//   out[t, f] = sum_k X[t, k] * W[f, k]        X: [M, K] bf16 activations, W: [N, K] bf16 weights (nn.Linear layout)
//
// Swap-AB mapping: a CTA owns a 128-feature slab of W (the MMA's M = 128 rows) and NT tokens (the MMA's N, 16..256),
// so M = bs*(B+1) tokens as small as 5 still drive a full-height tensor-core tile and every weight byte is read once
// per token tile.  One unit of work = (feature tile, token tile, K split).  Per CTA:
//   warp 0      TMA producer: W tile 128x64 and X tile NTx64 per stage (128-byte swizzle), S-stage mbarrier ring.
//               Weight tiles do not depend on the previous kernel, so the first S stages are issued before
//               griddepcontrol.wait (programmatic dependent launch): the weight stream starts while the previous
//               kernel drains.
//   warp 1      allocates TMEM (NT fp32 columns), one thread issues tcgen05.mma (M=128, N=NT, K=16) x 4 per stage,
//               tcgen05.commit frees the stage and finally signals the accumulator.
//   warps 2-9   epilogue: tcgen05.ld of their TMEM lane quadrant (lane = output feature, column = token); the two
//               warps of a quadrant take alternate 16-token chunks.
// Split-K: each split writes an fp32 partial tile to the workspace; the last CTA of a tile to arrive (atomic ticket)
// sums the partials in split order (deterministic) and runs the epilogue, then re-arms the ticket for the next launch.
// Epilogues: fp32 / bf16 store, SwiGLU (gate and up rows interleaved per 64 features by the host), Q/K/V with
// interleaved-pair partial RoPE and the paged K/V cache write, and lm_head's vocab-wide argmax (top-1 index, top-1
// value and top-2 gap; logits are never written): each feature tile leaves one top-2 record per token and
// argmax_reduce_kernel, launched right after, reduces a token's records with one warp.
#include "linear_dev.cuh"

namespace gr {

constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue (two per TMEM lane quadrant)
// lm_head, second step: one warp per token (argmax_reduce_token).
constexpr int kReduceWarps = 8;
__global__ void __launch_bounds__(kReduceWarps * 32) argmax_reduce_kernel(const LinearParams p) {
  GR_TL_BEGIN
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * kReduceWarps + (threadIdx.x >> 5);
  if (t < p.m) argmax_reduce_token(p, t);
  GR_TL_END(kTlArgmaxReduce)
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                  const LinearParams p) {
  GR_TL_BEGIN
  // Persistent: CTA c processes one unit per wave k, unit k * grid + c.  With tail_last (chosen by the host's
  // schedule model) the units of full token tiles are numbered before those of a shorter last tile and odd waves run
  // in reverse (unit k * grid + grid - 1 - c), so the short units land on the CTAs whose earlier units were short.
  // The producer and the MMA issuer walk the same sequence of (unit, K chunk) through one S-stage ring, so the next
  // unit's weights stream while the current unit's epilogue runs; the accumulator is double-buffered in TMEM
  // (acc_full / acc_empty per buffer).
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  const uint32_t x_stage_bytes = static_cast<uint32_t>(p.nt) * 128u;
  uint8_t* w_smem = smem;
  uint8_t* x_smem = smem + S * kWStageBytes;
  float* scratch = reinterpret_cast<float*>(x_smem + S * x_stage_bytes);  // epilogue exchange
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(scratch) + epi_scratch_bytes(EPI));
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] abort, [1] last split

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kc = p.kc_per_split;
  const int n_units = p.n_tiles * p.m_tiles * p.splits;
  const int G = gridDim.x, waves = n_units / G, rem = n_units % G;
  const int n_my = waves + ((rem > 0 && ((p.tail_last && (waves & 1)) ? (int)blockIdx.x >= G - rem
                                                                        : (int)blockIdx.x < rem)) ? 1 : 0);
  auto unit_of = [&](int k) { return k * G + ((p.tail_last && (k & 1)) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x); };
  // token tiles 0 .. full_m - 1 hold nt rows; a shorter last tile runs its MMAs at N = its rows (rounded to 16)
  const int full_m = (p.m % p.nt == 0 || !p.tail_last) ? p.m_tiles : p.m_tiles - 1;
  const int full_units = full_m * p.splits * p.n_tiles;
  const uint32_t acc_cols = p.nt <= 32 ? 32u : (p.nt <= 64 ? 64u : (p.nt <= 128 ? 128u : 256u));
  const uint32_t tmem_cols = 2 * acc_cols;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 8);  // one arrival per epilogue warp
    }
    flags[0] = flags[1] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmw);
    tma_prefetch_desc(&tmx);
  }
  if (warp == 1) tmem_alloc(tmem_slot, tmem_cols);
  if (p.prefetch_bytes && warp == 2 && lane == 0) {
    // warm L2 with this CTA's share of the next kernel's weights
    const unsigned long long per = ((p.prefetch_bytes / gridDim.x) + 4095ull) & ~4095ull;
    const unsigned long long b0 = per * blockIdx.x;
    const unsigned long long b1 = min(b0 + per, p.prefetch_bytes & ~15ull);
    for (unsigned long long b = b0; b < b1; b += 32768ull)
      l2_prefetch(p.prefetch + b, static_cast<uint32_t>(min(32768ull, b1 - b)));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  // unit u -> (m_tile fastest, then split, then n_tile): the token tiles of one weight slab run side by side (L2
  // reuse); with tail_last the units of a shorter last token tile come after all full ones
  auto decode = [&](int u, int& m_tile, int& split, int& n_tile) {
    if (u < full_units) {
      m_tile = u % full_m;
      u /= full_m;
    } else {
      u -= full_units;
      m_tile = p.m_tiles - 1;
    }
    split = u % p.splits;
    n_tile = u / p.splits;
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const int total = n_my * kc;
      // (unit, K chunk) cursor, advanced without divisions: the producer thread's per-stage latency is part of the
      // ring's round trip
      int k = 0, c = 0, m_tile = 0, split = 0, n_tile = 0, xk = 0;
      auto start_unit = [&]() {
        decode(unit_of(k), m_tile, split, n_tile);
        xk = split * kc * 64;
      };
      auto advance = [&]() {
        if (++c == kc) {
          c = 0;
          if (++k < n_my) start_unit();
        } else {
          xk += 64;
        }
      };
      auto load_w = [&](int st) {
        if (GR_W_EVICT_FIRST)
          tma_load_2d_hint(w_smem + st * kWStageBytes, &tmw, full + st, xk, n_tile * 128, pol);
        else
          tma_load_2d(w_smem + st * kWStageBytes, &tmw, full + st, xk, n_tile * 128);
      };
      if (n_my > 0) start_unit();
      // weights do not depend on the previous kernel: the first S stages' weight tiles go out before the wait
      const int pre = min(S, total);
      int pre_xk[GR_MAX_STAGES], pre_row[GR_MAX_STAGES];
      for (int g = 0; g < pre; ++g) {
        mbar_arrive_expect_tx(full + g, kWStageBytes + x_stage_bytes);
        load_w(g);
        pre_xk[g] = xk;
        pre_row[g] = m_tile * p.nt;
        advance();
      }
      pdl_wait();
      for (int g = 0; g < pre; ++g) tma_load_2d(x_smem + g * x_stage_bytes, &tmx, full + g, pre_xk[g], pre_row[g]);
      int issued = pre;
      int st = 0;
      uint32_t par = 0;  // parity of the empty phase that frees stage st
      for (int g = pre; g < total; ++g) {
        if (!mbar_wait(empty + st, par, p.status, GR_ERR_TIMEOUT)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(full + st, kWStageBytes + x_stage_bytes);
        load_w(st);
        tma_load_2d(x_smem + st * x_stage_bytes, &tmx, full + st, xk, m_tile * p.nt);
        advance();
        issued = g + 1;
        if (++st == S) {
          st = 0;
          par ^= 1u;
        }
      }
      // no copy may still be landing in shared memory when the CTA exits
      for (int g = max(0, issued - S); g < issued; ++g) mbar_wait(full + (g % S), (g / S) & 1, p.status, GR_ERR_TIMEOUT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_full = idesc_bf16_f32(128, p.nt);
      const int n_last = min(p.nt, ((p.m - (p.m_tiles - 1) * p.nt) + 15) & ~15);
      const uint32_t idesc_last = idesc_bf16_f32(128, n_last);
      // descriptors of stage 0; a stage / K step moves the 16-byte start-address field (shared memory < 256 KB)
      const uint64_t a0 = smem_desc_sw128(smem_u32(w_smem)), b0 = smem_desc_sw128(smem_u32(x_smem));
      int st = 0;
      uint32_t par = 0;
      bool ok = true;
      for (int k = 0; k < n_my && ok; ++k) {
        const int b = k & 1;
        if (k >= 2 && !mbar_wait(acc_empty + b, ((k >> 1) - 1) & 1, p.status, GR_ERR_TIMEOUT)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + b * acc_cols;
        int m_tile, split, n_tile;
        decode(unit_of(k), m_tile, split, n_tile);
        const uint32_t idesc = m_tile == p.m_tiles - 1 ? idesc_last : idesc_full;
        for (int c = 0; c < kc; ++c) {
          if (!mbar_wait(full + st, par, p.status, GR_ERR_TIMEOUT)) {
            flags[0] = 1;
            ok = false;
            break;
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
  } else {
    // ---------------------------------------------------------------- epilogue warps 2..9
    // warp w reads TMEM lanes 32*(w%4).. (its quadrant); the two warps of a quadrant take alternate 16-token chunks
    pdl_wait();
    const int quad = warp & 3;
    for (int k = 0; k < n_my; ++k) {
      const int b = k & 1;
      int m_tile, split, n_tile;
      decode(unit_of(k), m_tile, split, n_tile);
      const bool ok = mbar_wait(acc_full + b, (k >> 1) & 1, p.status, GR_ERR_TIMEOUT);
      tc_fence_after();
      const uint32_t t_lane = tmem + b * acc_cols + (static_cast<uint32_t>(quad * 32) << 16);
      const bool run = epi_bar_and(ok && !flags[0]);
      unit_epilogue<EPI>(p, t_lane, n_tile, m_tile, split, run, scratch, &flags[1], acc_empty + b);
      epi_bar();  // flags / scratch are reused by the next unit
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
  GR_TL_END(kTlLinear + EPI)
}

// ------------------------------------------------------------------ host side
size_t linear_smem_bytes(int nt, int stages, int epi) {
  return 1024 + static_cast<size_t>(stages) * (kWStageBytes + static_cast<size_t>(nt) * 128) + epi_scratch_bytes(epi) +
         (2 * stages + 4) * 8 + 32;
}

template <int EPI>
cudaError_t launch_linear_t(const CUtensorMap& tmw, const CUtensorMap& tmx, const LinearParams& p, int grid,
                            size_t smem, cudaStream_t stream, bool pdl) {
  auto kern = linear_kernel<EPI>;
  static PerDeviceOnce configured;
  cudaError_t e = once_per_device(configured, [&] {
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (r != cudaSuccess) return r;
    return cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  });
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tmw, tmx, p);
}

cudaError_t launch_argmax_reduce(const LinearParams& p, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.m + kReduceWarps - 1) / kReduceWarps);
  cfg.blockDim = dim3(kReduceWarps * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, argmax_reduce_kernel, p);
}

cudaError_t launch_linear(int epi, const CUtensorMap& tmw, const CUtensorMap& tmx, const LinearParams& p, int grid,
                          size_t smem, cudaStream_t stream, bool pdl) {
  switch (epi) {
    case GR_EPI_STORE_F32: return launch_linear_t<GR_EPI_STORE_F32>(tmw, tmx, p, grid, smem, stream, pdl);
    case GR_EPI_STORE_BF16: return launch_linear_t<GR_EPI_STORE_BF16>(tmw, tmx, p, grid, smem, stream, pdl);
    case GR_EPI_SWIGLU: return launch_linear_t<GR_EPI_SWIGLU>(tmw, tmx, p, grid, smem, stream, pdl);
    case GR_EPI_QKV_ROPE: return launch_linear_t<GR_EPI_QKV_ROPE>(tmw, tmx, p, grid, smem, stream, pdl);
    case GR_EPI_ARGMAX: return launch_linear_t<GR_EPI_ARGMAX>(tmw, tmx, p, grid, smem, stream, pdl);
    case GR_EPI_PARTIAL_F32: return launch_linear_t<GR_EPI_PARTIAL_F32>(tmw, tmx, p, grid, smem, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gr

GR_TIMELINE_EXPORTS(linear)
