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
#include "params.cuh"

namespace gr {

constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue (two per TMEM lane quadrant)
constexpr uint32_t kWStageBytes = 128 * 128;  // 128 rows x 64 bf16
// Epilogue shared memory: the argmax transpose (two halves x [16 tokens][128 rows] fp32); the bf16 epilogues stage
// each warp's 16 tokens x 32 rows (1 KB per warp) so that global stores go out as 16-byte vectors per lane.
__host__ __device__ constexpr uint32_t epi_scratch_bytes(int epi) {
  return epi == GR_EPI_ARGMAX ? 16384u
                              : ((epi == GR_EPI_SWIGLU || epi == GR_EPI_QKV_ROPE || epi == GR_EPI_STORE_BF16) ? 8192u : 0u);
}

// all 8 epilogue warps
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// the 4 epilogue warps of one column half (one warp per TMEM lane quadrant)
__device__ __forceinline__ void half_bar(int half) { asm volatile("bar.sync %0, 128;" ::"r"(2 + half) : "memory"); }

struct Top2 {
  float v1;
  int i1;
  float v2;
};
__device__ __forceinline__ Top2 top2_merge(Top2 a, Top2 b) {
  const bool bw = (b.v1 > a.v1) || (b.v1 == a.v1 && b.i1 < a.i1);
  Top2 r;
  if (bw) {
    r.v1 = b.v1;
    r.i1 = b.i1;
    r.v2 = fmaxf(a.v1, b.v2);
  } else {
    r.v1 = a.v1;
    r.i1 = a.i1;
    r.v2 = fmaxf(a.v2, b.v1);
  }
  return r;
}
__device__ __forceinline__ Top2 top2_warp(Top2 x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Top2 y;
    y.v1 = __shfl_xor_sync(0xffffffffu, x.v1, o);
    y.i1 = __shfl_xor_sync(0xffffffffu, x.i1, o);
    y.v2 = __shfl_xor_sync(0xffffffffu, x.v2, o);
    x = top2_merge(x, y);
  }
  return x;
}

// Apply the epilogue to 16 consecutive tokens [t0, t0+16) of feature row f_local of this tile.  Called by the 128
// epilogue threads of one column half together (it may use warp shuffles, the half's barrier and the CTA's
// epilogue shared memory `scratch`).
template <int EPI>
__device__ __forceinline__ void epilogue16(const LinearParams& p, int n_tile, int m_tile, int f_local, int t0,
                                           const float* v, float* scratch, int split) {
  const int lane = threadIdx.x & 31;
  const int t_end = min(p.m, (m_tile + 1) * p.nt);
  // bf16 staging area of this warp: [16 tokens][32 rows]
  __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(scratch) + (((threadIdx.x >> 5) - 2) << 9);
  if constexpr (EPI == GR_EPI_STORE_F32 || EPI == GR_EPI_PARTIAL_F32) {
    const int f = n_tile * 128 + f_local;
    const size_t base = EPI == GR_EPI_PARTIAL_F32 ? (size_t)split * p.m * p.ld_out : 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int t = t0 + i;
      if (t < t_end) static_cast<float*>(p.out)[base + (size_t)t * p.ld_out + f] = v[i];
    }
  } else if constexpr (EPI == GR_EPI_STORE_BF16) {
    // stage [token][32 rows], then lane l writes 16 rows (32 B) of token l / 2
#pragma unroll
    for (int i = 0; i < 16; ++i) stage[i * 32 + lane] = __float2bfloat16_rn(v[i]);
    __syncwarp();
    const int tok = lane >> 1, hh = lane & 1;
    const uint4 a = *reinterpret_cast<const uint4*>(stage + tok * 32 + hh * 16);
    const uint4 c = *reinterpret_cast<const uint4*>(stage + tok * 32 + hh * 16 + 8);
    if (t0 + tok < t_end) {
      __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + (size_t)(t0 + tok) * p.ld_out + n_tile * 128 +
                           (f_local & ~31) + hh * 16;
      reinterpret_cast<uint4*>(dst)[0] = a;
      reinterpret_cast<uint4*>(dst)[1] = c;
    }
    __syncwarp();
  } else if constexpr (EPI == GR_EPI_SWIGLU) {
    // rows 2j / 2j+1 of the tile are gate / up of feature 64*n_tile + j (gr_pack_gate_up): the pair sits in adjacent
    // lanes, so one shuffle brings the up value to the gate lane.  The warp's 16 features x 16 tokens are staged
    // [token][16 features] and written as one 16-byte vector per lane (token lane / 2, features 8 * (lane & 1) + 0..7).
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float u = __shfl_xor_sync(0xffffffffu, v[i], 1);
      if (!(lane & 1)) {
        const float g = v[i];
        stage[i * 16 + (lane >> 1)] = __float2bfloat16_rn(u * __fdividef(g, 1.0f + __expf(-g)));
      }
    }
    __syncwarp();
    const int tok = lane >> 1, hh = lane & 1;
    const uint4 a = *reinterpret_cast<const uint4*>(stage + tok * 16 + hh * 8);
    if (t0 + tok < t_end)
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + (size_t)(t0 + tok) * p.ld_out + n_tile * 64 +
                                ((f_local >> 1) & ~15) + hh * 8) = a;
    __syncwarp();
  } else if constexpr (EPI == GR_EPI_QKV_ROPE) {
    // tile = one head: [0, nq) query heads, [nq, nq+nkv) key heads, then value heads; f_local = head dim
    const int head = n_tile;
    const int d = f_local;
    const bool is_q = head < p.n_q_heads;
    const bool is_v = head >= p.n_q_heads + p.n_kv_heads;
    const bool rot = !is_v && (d & ~31) < p.rotary_dim;  // warp-uniform: rotary_dim is a multiple of 32
    // The chunk's 16 positions / cache slots take one coalesced load per warp (lanes l and l + 16 fetch token l) and
    // reach every lane by shuffles; cos / sin are computed in registers.  Per-token loads here would share the SM's
    // L1 / shared-memory bandwidth with the tensor core's operand reads of the next unit.
    const int tl = min(t0 + (lane & 15), t_end - 1);
    const long long slot_l = is_q ? 0ll : p.row_slot[tl];
    float o[16];
    if (rot) {
      const int pos_l = p.row_pos[tl];
      const float fr = p.inv_freq[d >> 1];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[i], 1);
        const int pos = __shfl_sync(0xffffffffu, pos_l, i);
        float sn, cs;
        rope_sincos(__fmul_rn(static_cast<float>(pos), fr), &sn, &cs);  // the reference's fp32 pos * inv_freq
        o[i] = (d & 1) ? (v[i] * cs + partner * sn) : (v[i] * cs - partner * sn);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = v[i];
    }
    // stage [token][32 dims]; lane l then writes 16 dims (32 B) of token l / 2
#pragma unroll
    for (int i = 0; i < 16; ++i) stage[i * 32 + lane] = __float2bfloat16_rn(o[i]);
    __syncwarp();
    const int tok = lane >> 1, hh = lane & 1;
    const uint4 a = *reinterpret_cast<const uint4*>(stage + tok * 32 + hh * 16);
    const uint4 c = *reinterpret_cast<const uint4*>(stage + tok * 32 + hh * 16 + 8);
    const int d0 = (d & ~31) + hh * 16;
    __nv_bfloat16* dst;
    if (is_q) {
      dst = p.q_out + (size_t)(t0 + tok) * (p.n_q_heads * 128) + head * 128 + d0;
    } else {
      // page size 16 (the host checks): page = slot >> 4, offset = slot & 15
      const int kvh = is_v ? head - p.n_q_heads - p.n_kv_heads : head - p.n_q_heads;
      const uint64_t slot = static_cast<uint64_t>(__shfl_sync(0xffffffffu, slot_l, tok));
      dst = (is_v ? p.v_cache : p.k_cache) + ((((slot >> 4) * p.n_kv_heads + kvh) << 4) + (slot & 15)) * 128 + d0;
    }
    if (t0 + tok < t_end) {
      reinterpret_cast<uint4*>(dst)[0] = a;
      reinterpret_cast<uint4*>(dst)[1] = c;
    }
    __syncwarp();
  } else if constexpr (EPI == GR_EPI_ARGMAX) {
    // transpose through shared memory: [16 tokens][128 vocab rows]; then 8 threads per token scan 16 rows each and
    // merge with 3 shuffle rounds (ties: lowest vocab index)
    const int half = (((threadIdx.x >> 5) - 2) >> 2);
    const int tid = threadIdx.x & 127;
    float* xs = scratch + half * 2048;
#pragma unroll
    for (int i = 0; i < 16; ++i) xs[i * 128 + f_local] = v[i];
    half_bar(half);
    const int tok = tid >> 3, part = tid & 7;
    const float* row = xs + tok * 128 + part * 16;
    Top2 x{-INFINITY, 0x7fffffff, -INFINITY};
#pragma unroll
    for (int j = 0; j < 16; ++j) x = top2_merge(x, Top2{row[j], n_tile * 128 + part * 16 + j, -INFINITY});
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      Top2 y;
      y.v1 = __shfl_xor_sync(0xffffffffu, x.v1, o);
      y.i1 = __shfl_xor_sync(0xffffffffu, x.i1, o);
      y.v2 = __shfl_xor_sync(0xffffffffu, x.v2, o);
      x = top2_merge(x, y);
    }
    const int t = t0 + tok;
    if (part == 0 && t < t_end)
      p.ws_arg[(size_t)t * p.n_tiles + n_tile] = make_float4(x.v1, __int_as_float(x.i1), x.v2, 0.f);
    half_bar(half);
  }
}

// lm_head, second step: one warp per token merges the token's n_tiles top-2 records (ties: lowest vocab index).  The
// records of a token are contiguous; every lane issues all its loads before merging (up to 16 x 16 B in flight).
constexpr int kReduceWarps = 8;
__global__ void __launch_bounds__(kReduceWarps * 32) argmax_reduce_kernel(const LinearParams p) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * kReduceWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= p.m) return;
  const float4* rec = p.ws_arg + (size_t)t * p.n_tiles;
  Top2 x{-INFINITY, 0x7fffffff, -INFINITY};
  for (int n0 = 0; n0 < p.n_tiles; n0 += 32 * 16) {
    float4 r[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int n = n0 + j * 32 + lane;
      r[j] = n < p.n_tiles ? __ldcg(rec + n) : make_float4(-INFINITY, __int_as_float(0x7fffffff), -INFINITY, 0.f);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) x = top2_merge(x, Top2{r[j].x, __float_as_int(r[j].y), r[j].z});
  }
  x = top2_warp(x);
  if (lane == 0) {
    p.out_idx[t] = x.i1;
    if (p.out_top1) p.out_top1[t] = x.v1;
    if (p.out_gap) p.out_gap[t] = x.v1 - x.v2;
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                  const LinearParams p) {
  // Persistent: CTA c processes units c, c + gridDim.x, ...  The producer and the MMA issuer walk the same global
  // sequence of (unit, K chunk) through one S-stage ring, so the next unit's weights stream while the current unit's
  // epilogue runs; the accumulator is double-buffered in TMEM (acc_full / acc_empty per buffer).
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
  const int n_my = blockIdx.x < n_units ? (n_units - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
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

  // unit u -> (m_tile fastest, then split, then n_tile): the token tiles of one weight slab run side by side (L2 reuse)
  auto decode = [&](int u, int& m_tile, int& split, int& n_tile) {
    m_tile = u % p.m_tiles;
    u /= p.m_tiles;
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
        decode(blockIdx.x + k * gridDim.x, m_tile, split, n_tile);
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
      const uint32_t idesc = idesc_bf16_f32(128, p.nt);
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
    const int half = (warp - 2) >> 2;
    const int f_local = quad * 32 + lane;
    for (int k = 0; k < n_my; ++k) {
      const int b = k & 1;
      int m_tile, split, n_tile;
      decode(blockIdx.x + k * gridDim.x, m_tile, split, n_tile);
      const bool ok = mbar_wait(acc_full + b, (k >> 1) & 1, p.status, GR_ERR_TIMEOUT);
      tc_fence_after();
      const uint32_t t_lane = tmem + b * acc_cols + (static_cast<uint32_t>(quad * 32) << 16);
      const int t_beg = m_tile * p.nt;
      const int rows = min(p.nt, p.m - t_beg);
      epi_bar();
      const bool run = ok && !flags[0];
      if (p.splits == 1 || EPI == GR_EPI_PARTIAL_F32) {
        if (run) {
          // the next chunk's TMEM load is in flight while this chunk's epilogue runs
          uint32_t ra[16], rb[16];
          int c0 = half * 16;
          if (c0 < p.nt) tmem_ld16_issue(t_lane + c0, ra);
          while (c0 < p.nt) {
            float v[16];
            tmem_ld16_wait(ra);
            const int c1 = c0 + 32;
            if (c1 < p.nt) tmem_ld16_issue(t_lane + c1, rb);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(ra[i]);
            epilogue16<EPI>(p, n_tile, m_tile, f_local, t_beg + c0, v, scratch, split);
            if (c1 >= p.nt) break;
            tmem_ld16_wait(rb);
            c0 = c1 + 32;
            if (c0 < p.nt) tmem_ld16_issue(t_lane + c0, ra);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(rb[i]);
            epilogue16<EPI>(p, n_tile, m_tile, f_local, t_beg + c1, v, scratch, split);
          }
        }
        tc_fence_before();
        if (lane == 0) mbar_arrive(acc_empty + b);
      } else {
        const int tile = n_tile * p.m_tiles + m_tile;
        float* part = p.ws_partial + ((size_t)tile * p.splits + split) * p.nt * 128;
        if (run) {
          for (int c0 = half * 16; c0 < p.nt; c0 += 32) {
            float v[16];
            tmem_ld16(t_lane + c0, v);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c0 + i < rows) part[(c0 + i) * 128 + f_local] = v[i];
          }
        }
        tc_fence_before();
        if (lane == 0) mbar_arrive(acc_empty + b);  // the accumulator is free again; the rest reads global memory
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          const int prev = atomicAdd(&p.ws_ticket[tile], 1);
          flags[1] = (prev == p.splits - 1);
        }
        epi_bar();
        if (flags[1]) {
          __threadfence();
          const float* base = p.ws_partial + (size_t)tile * p.splits * p.nt * 128;
          for (int c0 = half * 16; c0 < p.nt; c0 += 32) {
            // split order is fixed (deterministic sums); the 16 rows' loads of one split are independent
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
            for (int s = 0; s < p.splits; ++s) {
              const float* src = base + ((size_t)s * p.nt + c0) * 128 + f_local;
              float x[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) x[i] = (c0 + i < rows) ? __ldcg(src + i * 128) : 0.f;
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] += x[i];
            }
            epilogue16<EPI>(p, n_tile, m_tile, f_local, t_beg + c0, v, scratch, split);
          }
          if (threadIdx.x == 64) p.ws_ticket[tile] = 0;
        }
      }
      epi_bar();  // flags / scratch are reused by the next unit
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
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
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    configured = true;
  }
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
