// Device code of the projection kernel (linear.cu): shared-memory sizes, the epilogues and the argmax reduction.
#pragma once

#include "params.cuh"

namespace gr {

constexpr uint32_t kWStageBytes = 128 * 128;  // 128 rows x 64 bf16
// Epilogue shared memory: the argmax transpose (two halves x [16 tokens][128 rows] fp32); the bf16 epilogues stage
// each warp's 16 tokens x 32 rows (1 KB per warp) so that global stores go out as 16-byte vectors per lane.
__host__ __device__ constexpr uint32_t epi_scratch_bytes(int epi) {
  return epi == GR_EPI_ARGMAX ? 16384u
                              : ((epi == GR_EPI_SWIGLU || epi == GR_EPI_QKV_ROPE || epi == GR_EPI_STORE_BF16) ? 8192u : 0u);
}

// all 8 epilogue warps
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// the same barrier, returning the AND of v over the 8 warps: a decision every epilogue thread takes alike (the argmax
// epilogue meets at the column halves' named barriers inside a unit, so no warp may run a unit that another skips)
__device__ __forceinline__ bool epi_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pv, pr;\n\tsetp.ne.u32 pv, %1, 0;\n\tbar.red.and.pred pr, 1, 256, pv;\n\t"
      "selp.u32 %0, 1, 0, pr;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}
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
// Per-row inputs of the QKV epilogue for one 16-token chunk as lane l holds them (token t0 + (l & 15), clamped to the
// tile's rows): RoPE position(s) and cache slot.  Loaded one chunk ahead, so their L2 round trip overlaps the
// previous chunk's work instead of opening every chunk.
struct RowIn {
  int pos_l, pos_h, pos_w;
  long long slot;
};
__device__ __forceinline__ RowIn qkv_row_inputs(const LinearParams& p, int t0, int t_end) {
  const int tl = min(t0 + (static_cast<int>(threadIdx.x) & 15), t_end - 1);
  RowIn r;
  if (p.row_pos3) {
    r.pos_l = p.row_pos3[tl * 3];
    r.pos_h = p.row_pos3[tl * 3 + 1];
    r.pos_w = p.row_pos3[tl * 3 + 2];
  } else {
    r.pos_l = p.row_pos[tl];
    r.pos_h = r.pos_w = 0;
  }
  r.slot = p.row_slot[tl];
  return r;
}

template <int EPI>
__device__ __forceinline__ void epilogue16(const LinearParams& p, int n_tile, int m_tile, int f_local, int t0,
                                           const float* v, float* scratch, int split, const RowIn& ri) {
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
    // lanes.  The gate lane computes tokens 0-7 and the up lane tokens 8-15 of the chunk: one shuffle per token pair
    // swaps the gate lane's gates 8-15 for the up lane's ups 0-7, so both lanes do half the math.  The warp's
    // 16 features x 16 tokens are staged [token][16 features] and written as one 16-byte vector per lane (token
    // lane / 2, features 8 * (lane & 1) + 0..7).
    const bool up_lane = lane & 1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, up_lane ? v[i] : v[8 + i], 1);
      const float g = up_lane ? other : v[i];     // gate of token (up_lane ? 8 + i : i)
      const float u = up_lane ? v[8 + i] : other;  // up of the same token
      stage[(up_lane ? 8 + i : i) * 16 + (lane >> 1)] = __float2bfloat16_rn(u * __fdividef(g, 1.0f + __expf(-g)));
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
    // The chunk's 16 positions / cache slots came with one coalesced load per warp (lanes l and l + 16 hold token l,
    // qkv_row_inputs) and reach every lane by shuffles; cos / sin are computed in registers.  Per-token loads here
    // would share the SM's L1 / shared-memory bandwidth with the tensor core's operand reads of the next unit.
    const long long slot_l = is_q ? 0ll : ri.slot;
    float o[16];
    if (rot) {
      // Lanes d and d ^ 1 rotate the same pair and need the same angles: the even lane computes cos / sin for
      // tokens 0-7 and the odd lane for tokens 8-15, and they swap the results.
      const float fr = p.inv_freq[d >> 1];
      const bool odd = d & 1;
      // multimodal positions: every lane fetches its token's three axes and picks, after the shuffle, the axis of
      // its own rotary pair (pairs of one warp can straddle a section boundary)
      const bool mm = p.row_pos3 != nullptr;
      const int pair = d >> 1;
      const int axis = pair < p.mrope_s0 ? 0 : (pair < p.mrope_s0 + p.mrope_s1 ? 1 : 2);
      const int pos_l = ri.pos_l, pos_h = ri.pos_h, pos_w = ri.pos_w;
      // In phases, each an independent unrolled loop: with one or two epilogue warps per scheduler there is nothing
      // else to hide latency behind, and the eight tokens' shuffle -> angle -> exchange chains interleave only when
      // no shuffle sits between one token's steps and the next token's.
      int pos[8];
      float pa[16], sn[8], cs[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        pos[i] = __shfl_sync(0xffffffffu, pos_l, odd ? 8 + i : i);
        if (mm) {
          const int ph = __shfl_sync(0xffffffffu, pos_h, odd ? 8 + i : i);
          const int pw = __shfl_sync(0xffffffffu, pos_w, odd ? 8 + i : i);
          pos[i] = axis == 0 ? pos[i] : (axis == 1 ? ph : pw);
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) pa[i] = __shfl_xor_sync(0xffffffffu, v[i], 1);  // the pair partner's values
#pragma unroll
      for (int i = 0; i < 8; ++i)
        rope_sincos(__fmul_rn(static_cast<float>(pos[i]), fr), &sn[i], &cs[i]);  // the reference's fp32 pos * inv_freq
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float cs_o = __shfl_xor_sync(0xffffffffu, cs[i], 1);
        const float sn_o = __shfl_xor_sync(0xffffffffu, sn[i], 1);
        const float ca = odd ? cs_o : cs[i], sa = odd ? sn_o : sn[i];  // token i
        const float cb = odd ? cs[i] : cs_o, sb = odd ? sn[i] : sn_o;  // token 8 + i
        o[i] = odd ? (v[i] * ca + pa[i] * sa) : (v[i] * ca - pa[i] * sa);
        o[8 + i] = odd ? (v[8 + i] * cb + pa[8 + i] * sb) : (v[8 + i] * cb - pa[8 + i] * sb);
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


// One unit's epilogue, run by the 8 epilogue warps (warps 2-9, 256 threads) of the CTA that owns the unit: the TMEM
// accumulator (this warp's lane quadrant at t_lane) -> epilogue16, or, for a split-K unit, a partial tile -> ticket ->
// the last split sums the partials in split order and runs the epilogue.  Arrives once per warp on `acc_empty` as
// soon as the accumulator has been read.  `flag_last` is a shared int.
template <int EPI>
__device__ __forceinline__ void unit_epilogue(const LinearParams& p, uint32_t t_lane, int n_tile, int m_tile, int split,
                                              bool run, float* scratch, int* flag_last, uint64_t* acc_empty) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = (warp - 2) >> 2;
  const int f_local = (warp & 3) * 32 + lane;
  const bool leader = warp == 2 && lane == 0;
  const int t_beg = m_tile * p.nt;
  const int rows = min(p.nt, p.m - t_beg);
  if (p.splits == 1 || EPI == GR_EPI_PARTIAL_F32) {
    if (run) {
      // the next chunk's TMEM load is in flight while this chunk's epilogue runs
      // (chunks past the tile's rows hold no tokens: a short last tile is computed at N = its rows)
      // (and, for QKV, the next chunk's row inputs)
      const int t_end = t_beg + rows;
      uint32_t ra[16], rb[16];
      RowIn ia{}, ib{};
      int c0 = half * 16;
      if (c0 < rows) {
        tmem_ld16_issue(t_lane + c0, ra);
        if constexpr (EPI == GR_EPI_QKV_ROPE) ia = qkv_row_inputs(p, t_beg + c0, t_end);
      }
      while (c0 < rows) {
        float v[16];
        tmem_ld16_wait(ra);
        const int c1 = c0 + 32;
        if (c1 < rows) {
          tmem_ld16_issue(t_lane + c1, rb);
          if constexpr (EPI == GR_EPI_QKV_ROPE) ib = qkv_row_inputs(p, t_beg + c1, t_end);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(ra[i]);
        epilogue16<EPI>(p, n_tile, m_tile, f_local, t_beg + c0, v, scratch, split, ia);
        if (c1 >= rows) break;
        tmem_ld16_wait(rb);
        c0 = c1 + 32;
        if (c0 < rows) {
          tmem_ld16_issue(t_lane + c0, ra);
          if constexpr (EPI == GR_EPI_QKV_ROPE) ia = qkv_row_inputs(p, t_beg + c0, t_end);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(rb[i]);
        epilogue16<EPI>(p, n_tile, m_tile, f_local, t_beg + c1, v, scratch, split, ib);
      }
    }
    tc_fence_before();
    if (lane == 0) mbar_arrive(acc_empty);
  } else {
    const int tile = n_tile * p.m_tiles + m_tile;
    float* part = p.ws_partial + ((size_t)tile * p.splits + split) * p.nt * 128;
    if (run) {
      for (int c0 = half * 16; c0 < rows; c0 += 32) {
        float v[16];
        tmem_ld16(t_lane + c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (c0 + i < rows) part[(c0 + i) * 128 + f_local] = v[i];
      }
    }
    tc_fence_before();
    if (lane == 0) mbar_arrive(acc_empty);  // the accumulator is free again; the rest reads global memory
    __threadfence();
    epi_bar();
    if (leader) {
      const int prev = atomicAdd(&p.ws_ticket[tile], 1);
      *flag_last = (prev == p.splits - 1);
    }
    epi_bar();
    if (*flag_last) {
      __threadfence();
      const float* base = p.ws_partial + (size_t)tile * p.splits * p.nt * 128;
      for (int c0 = half * 16; c0 < rows; c0 += 32) {
        RowIn ri{};  // issued with the partials' loads: one round trip
        if constexpr (EPI == GR_EPI_QKV_ROPE) ri = qkv_row_inputs(p, t_beg + c0, t_beg + rows);
        // split order is fixed (deterministic sums); four splits' 16 rows each in flight at a time (one L2 round
        // trip per four splits)
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        int s = 0;
        for (; s + 4 <= p.splits; s += 4) {
          float x[4][16];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float* src = base + ((size_t)(s + u) * p.nt + c0) * 128 + f_local;
#pragma unroll
            for (int i = 0; i < 16; ++i) x[u][i] = (c0 + i < rows) ? __ldcg(src + i * 128) : 0.f;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] += x[u][i];
        }
        for (; s < p.splits; ++s) {
          const float* src = base + ((size_t)s * p.nt + c0) * 128 + f_local;
          float x[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) x[i] = (c0 + i < rows) ? __ldcg(src + i * 128) : 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] += x[i];
        }
        epilogue16<EPI>(p, n_tile, m_tile, f_local, t_beg + c0, v, scratch, split, ri);
      }
      if (leader) p.ws_ticket[tile] = 0;
    }
  }
}

// lm_head, second step: one warp per token merges the token's n_tiles top-2 records (ties: lowest vocab index).  The
// records of a token are contiguous; every lane issues all its loads before merging (up to 16 x 16 B in flight).
__device__ __forceinline__ void argmax_reduce_token(const LinearParams& p, int t) {
  const int lane = threadIdx.x & 31;
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


}  // namespace gr
