// Attention device code of the mma.sync kernel (attention.cu), shared in part with the tcgen05 kernel
// (attention_tc.cu): one (split, kv head, request) unit, run by the CTA's participating warps.
#pragma once

#include "params.cuh"

namespace gr {

constexpr int kTile = 64;                       // tokens per pipeline stage
constexpr int kHalfBytes = kTile * 128;         // 64 rows x 64 dims bf16
constexpr int kStageBytes = 4 * kHalfBytes;     // K lo, K hi, V lo, V hi
constexpr int kMaxChunkPages = 4096 / 16;  // chunk <= 4096 tokens
constexpr int kMaxMergeSplits = 16;        // splits per (request, kv head); the host enforces it

// Cache positions [0, row_limit) that window row j sees: draft 1 (the served round) keeps row 0, the boundary token,
// causal and lets the mask rows see the whole block; draft 2 (the in-process round's first block, which has no
// boundary token) lets every row see the whole block; draft 0 is causal.
__device__ __forceinline__ int row_limit(const AttnParams& p, int j, int base) {
  if (p.draft) return (j == 0 && p.draft == 1) ? base + 1 : base + p.K;
  return base + j + 1;
}
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// All threads of every CTA of the cluster (release / acquire: shared-memory writes before it are visible to the
// cluster's DSMEM reads after it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float2 ld_dsmem_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}

// Shared-memory state of a CTA's attention ring, kept across the units it runs: ST stages of kStageBytes, the query
// staging area, the stage barriers (full: one arrival + bytes; empty: one per consuming warp), a flag word and the
// page ids of the current split.  tile_base counts the tiles streamed through the ring so far (stage g % ST, phase
// g / ST for the ring's g-th tile).
struct AttnCta {
  uint8_t* kv_smem;
  uint8_t* q_smem;
  uint64_t* full;
  uint64_t* empty;
  int* flag;
  int* pages;
  int tile_base;
};
__host__ __device__ constexpr int attn_rows_pad(int G, int K) { return ((G * K + 15) / 16) * 16; }
// bytes of the attention region (1024-aligned start assumed): stages, query staging, barriers, flag, page ids
__host__ __device__ constexpr size_t attn_region_bytes(int R_pad, int stages) {
  return static_cast<size_t>(stages) * kStageBytes + 2 * R_pad * 128 + 2 * stages * 8 + 16 + kMaxChunkPages * 4;
}
template <int ST>
__device__ __forceinline__ AttnCta attn_cta_layout(uint8_t* region, int R_pad) {
  AttnCta c;
  c.kv_smem = region;
  c.q_smem = region + ST * kStageBytes;
  c.full = reinterpret_cast<uint64_t*>(c.q_smem + 2 * R_pad * 128);
  c.empty = c.full + ST;
  c.flag = reinterpret_cast<int*>(c.empty + ST);
  c.pages = c.flag + 4;
  c.tile_base = 0;
  return c;
}

// Page ids of split `split`'s whole chunk of request b, by the 32 lanes of one warp, before the kernel waits for its
// predecessor: the page table and the launch order are written before a round starts, the lengths are not, so the
// clamp to the request's last page is applied when a tile is issued (attn_page).  pages[] holds chunk / page_size
// entries (<= kMaxChunkPages).
__device__ __forceinline__ void attn_preload_pages(const AttnParams& p, int b, int split, int lane, int* pages) {
  const int* pt = p.page_table + (size_t)b * p.pt_stride;
  const int pg_beg = split * p.chunk / p.page_size;
  const int n = p.chunk / p.page_size;
  for (int i = lane; i < n; i += 32) pages[i] = pt[min(pg_beg + i, p.pt_stride - 1)];
}
// Page of the split's k-th page slot: pages past the request's last page hold no visible token and are replaced by
// its last page, whose contents are finite.  pre: pages[] from attn_preload_pages (unclamped) or already clamped.
__device__ __forceinline__ int attn_page(const int* pages, int k, int last_slot, bool pre) {
  return pages[pre ? min(k, last_slot) : k];
}

// Split merge through global memory: every split of (request b, kv head kvh) has written its (O, m, l) partial to
// ws_o / ws_ml; the last split to arrive merges them in split order.  Called by all nthr participating threads of
// each split's CTA (named barrier bar_all); `flag` is a shared int, `wgt` shared scratch of R * kMaxMergeSplits
// floats.
__device__ inline void attention_merge_global(const AttnParams& p, int b, int kvh, int n_active, int wt, int nthr,
                                              int bar_all, int* flag, float* wgt) {
  const int G = p.n_q_heads / p.n_kv_heads;
  const int R = G * p.K;
  const int R_pad = attn_rows_pad(G, p.K);
  const size_t q_row_stride = (size_t)p.n_q_heads * 128;
  __threadfence();
  named_bar(bar_all, nthr);
  if (wt == 0) {
    int* tk = p.ws_ticket + (size_t)b * p.n_kv_heads + kvh;
    const int prev = atomicAdd(tk, 1);
    *flag = (prev == n_active - 1) ? 2 : 0;
    if (*flag) *tk = 0;
  }
  named_bar(bar_all, nthr);
  if (*flag != 2) return;
  __threadfence();
  const size_t slot0 = ((size_t)b * p.n_kv_heads + kvh) * p.max_splits;
  // phase A: per (row, split) weights exp2(m_s - M) / L into shared memory (the stage ring is idle now)
  for (int r = wt; r < R; r += nthr) {
    float M = -INFINITY;
    float ms[kMaxMergeSplits], ls[kMaxMergeSplits];
#pragma unroll
    for (int s = 0; s < kMaxMergeSplits; ++s) {
      if (s < n_active) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.ws_ml + ((slot0 + s) * R_pad + r) * 2));
        ms[s] = ml.x;
        ls[s] = ml.y;
        M = fmaxf(M, ml.x);
      }
    }
    const float Ms = (M == -INFINITY) ? 0.f : M;
    float Lsum = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxMergeSplits; ++s) {
      if (s < n_active) {
        const float w = (ms[s] == -INFINITY) ? 0.f : exp2f(ms[s] - Ms);
        ms[s] = w;
        Lsum += ls[s] * w;
      }
    }
    const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
#pragma unroll
    for (int s = 0; s < kMaxMergeSplits; ++s)
      if (s < n_active) wgt[r * kMaxMergeSplits + s] = ms[s] * inv;
  }
  named_bar(bar_all, nthr);
  // phase B: (row, 4 dims) items; every split's loads of an item are issued together, summed in split order.  With
  // at most 4 splits, four items' loads go out together.
  auto store4 = [&](int it, float4 acc) {
    const int r = it >> 5, q4 = it & 31;
    const int g = r / p.K, j = r % p.K;
    __nv_bfloat16* dst = p.out + ((size_t)b * p.K + j) * q_row_stride + (kvh * G + g) * 128 + q4 * 4;
    uint2 pk;
    pk.x = pack_bf16(acc.x, acc.y);
    pk.y = pack_bf16(acc.z, acc.w);
    *reinterpret_cast<uint2*>(dst) = pk;
  };
  if (n_active <= 4) {
    for (int it0 = wt; it0 < R * 32; it0 += 4 * nthr) {
      float4 os[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int it = it0 + u * nthr;
#pragma unroll
        for (int sp = 0; sp < 4; ++sp)
          if (it < R * 32 && sp < n_active)
            os[u][sp] = __ldcg(reinterpret_cast<const float4*>(p.ws_o + ((slot0 + sp) * R_pad + (it >> 5)) * 128) +
                               (it & 31));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int it = it0 + u * nthr;
        if (it >= R * 32) break;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < 4; ++sp) {
          if (sp < n_active) {
            const float w = wgt[(it >> 5) * kMaxMergeSplits + sp];
            acc.x += os[u][sp].x * w;
            acc.y += os[u][sp].y * w;
            acc.z += os[u][sp].z * w;
            acc.w += os[u][sp].w * w;
          }
        }
        store4(it, acc);
      }
    }
    return;
  }
  for (int it = wt; it < R * 32; it += nthr) {
    const int r = it >> 5, q4 = it & 31;
    float4 os[kMaxMergeSplits];
#pragma unroll
    for (int s = 0; s < kMaxMergeSplits; ++s)
      if (s < n_active) os[s] = __ldcg(reinterpret_cast<const float4*>(p.ws_o + ((slot0 + s) * R_pad + r) * 128) + q4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < kMaxMergeSplits; ++s) {
      if (s < n_active) {
        const float w = wgt[r * kMaxMergeSplits + s];
        acc.x += os[s].x * w;
        acc.y += os[s].y * w;
        acc.z += os[s].z * w;
        acc.w += os[s].w * w;
      }
    }
    store4(it, acc);
  }
}

// Split merge through distributed shared memory: the max_splits CTAs of (request b, kv head kvh) form one cluster
// (rank = split) and each holds its (O, m, l) partial in its own shared memory (part_o [R_pad][128], part_ml
// [R_pad][2], the same offsets in every CTA).  Called after a cluster barrier by every warp of every CTA; CTA `split`
// merges rows split*n_warps + warp (stride max_splits*n_warps) in split order with the arithmetic of the global
// merge.  The caller's second cluster barrier keeps the partials alive until read.
__device__ inline void attention_merge_cluster(const AttnParams& p, int b, int kvh, int split, int n_active, int warp,
                                               int lane, int n_warps, const float* part_o, const float* part_ml) {
  const int G = p.n_q_heads / p.n_kv_heads;
  const int R = G * p.K;
  const size_t q_row_stride = (size_t)p.n_q_heads * 128;
  if (n_active > 1) {
    const int cs = p.max_splits;
    for (int r = split * n_warps + warp; r < R; r += cs * n_warps) {
      float M = -INFINITY;
      float ms[kMaxMergeSplits], ls[kMaxMergeSplits];
#pragma unroll
      for (int s2 = 0; s2 < kMaxMergeSplits; ++s2) {
        if (s2 < n_active) {
          const float2 ml = ld_dsmem_f2(dsmem_addr(part_ml + r * 2, s2));
          ms[s2] = ml.x;
          ls[s2] = ml.y;
          M = fmaxf(M, ml.x);
        }
      }
      const float Ms = (M == -INFINITY) ? 0.f : M;
      float Lsum = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < kMaxMergeSplits; ++s2) {
        if (s2 < n_active) {
          const float w = (ms[s2] == -INFINITY) ? 0.f : exp2f(ms[s2] - Ms);
          ms[s2] = w;
          Lsum += ls[s2] * w;
        }
      }
      const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int s2 = 0; s2 < kMaxMergeSplits; ++s2) {
        if (s2 < n_active) {
          const float w = ms[s2] * inv;
          const float4 ov = ld_dsmem_f4(dsmem_addr(part_o + r * 128 + lane * 4, s2));
          acc.x += ov.x * w;
          acc.y += ov.y * w;
          acc.z += ov.z * w;
          acc.w += ov.w * w;
        }
      }
      const int g = r / p.K, j = r % p.K;
      __nv_bfloat16* dst = p.out + ((size_t)b * p.K + j) * q_row_stride + (kvh * G + g) * 128 + lane * 4;
      uint2 pk;
      pk.x = pack_bf16(acc.x, acc.y);
      pk.y = pack_bf16(acc.z, acc.w);
      *reinterpret_cast<uint2*>(dst) = pk;
    }
  }
}

// One unit.  Participating threads: wt in [0, nthr), warp aw = wt / 32; warps aw < groups * n_mt compute, warp
// aw == groups * n_mt is the TMA producer, the rest only help the split merge.  bar_all / bar_cw are named barrier
// ids for all participants / the compute warps.  Every participant calls with the same arguments.  PRE: the
// producer warp already holds the split's page ids (attn_preload_pages).
template <int ST, bool PRE = false>
__device__ void attention_unit(const CUtensorMap* tmk_p, const CUtensorMap* tmv_p, const AttnParams& p, int split,
                               int kvh, int b, int wt, int nthr, int bar_all, int bar_cw, AttnCta& c) {
  const CUtensorMap& tmk = *tmk_p;
  const CUtensorMap& tmv = *tmv_p;
  const int G = p.n_q_heads / p.n_kv_heads;
  const int R = G * p.K;
  const int n_mt = (R + 15) / 16;
  const int R_pad = n_mt * 16;
  const int NG = p.groups;  // warp groups taking alternate KV tiles
  const int n_cw = NG * n_mt;
  uint8_t* kv_smem = c.kv_smem;
  uint8_t* q_smem = c.q_smem;
  uint64_t* full = c.full;
  uint64_t* empty = c.empty;
  int* flag = c.flag;
  int* pages = c.pages;
  const int warp = wt >> 5, lane = wt & 31;
  const int64_t seq = p.seq_lens[b];
  const int base = static_cast<int>(seq) + p.base_add;
  const int L = base + p.K;  // the last row's limit
  const int n_active = (L + p.chunk - 1) / p.chunk;
  const bool active = split < n_active;
  if (!active && !p.cluster) return;  // a cluster's idle splits still join its barriers (and the merge)
  const int kv_beg = split * p.chunk;
  const int kv_end = min(L, kv_beg + p.chunk);
  const int n_tiles = active ? (kv_end - kv_beg + kTile - 1) / kTile : 0;
  // cluster merge: each split's (O, m, l) partial in its own shared memory, past the group exchange area
  float* part_o = reinterpret_cast<float*>(kv_smem + 32768);  // [R_pad][128]
  float* part_ml = part_o + R_pad * 128;                      // [R_pad][2]
  const int tb = c.tile_base;  // this unit streams the ring's tiles tb .. tb + n_tiles - 1
  c.tile_base += n_tiles;

  const int* pt = p.page_table + (size_t)b * p.pt_stride;
  const size_t q_row_stride = (size_t)p.n_q_heads * 128;
  if (!active) {
    // idle split of a cluster: no tiles, no partial
  } else if (warp == n_cw) {
    // ------------------------------------------------------------ producer
    // the whole split's page ids in one coalesced pass (pages past the request's last page hold no visible token:
    // they are replaced by its last page, whose contents are finite)
    const int last_page = (L - 1) / p.page_size;
    const int pg_beg = kv_beg / p.page_size;
    const int n_pg = n_tiles * (kTile / 16);
    if constexpr (!PRE)
      for (int i = lane; i < n_pg; i += 32) pages[i] = pt[min(pg_beg + i, last_page)];
    __syncwarp();
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < n_tiles; ++i) {
        const int g = tb + i;
        const int s = g % ST;
        if (g >= ST && !mbar_wait(empty + s, ((g / ST) - 1) & 1, p.status, GR_ERR_TIMEOUT)) break;
        mbar_arrive_expect_tx(full + s, kStageBytes);
        uint8_t* st = kv_smem + s * kStageBytes;
#pragma unroll
        for (int pg = 0; pg < 4; ++pg) {
          const int phys = attn_page(pages, i * 4 + pg, last_page - pg_beg, PRE);
          const int y = (phys * p.n_kv_heads + kvh) * p.page_size;
          tma_load_2d(st + 0 * kHalfBytes + pg * 2048, &tmk, full + s, 0, y);
          tma_load_2d(st + 1 * kHalfBytes + pg * 2048, &tmk, full + s, 64, y);
          tma_load_2d(st + 2 * kHalfBytes + pg * 2048, &tmv, full + s, 0, y);
          tma_load_2d(st + 3 * kHalfBytes + pg * 2048, &tmv, full + s, 64, y);
        }
        issued = i + 1;
      }
      for (int i = max(0, issued - ST); i < issued; ++i)
        mbar_wait(full + ((tb + i) % ST), ((tb + i) / ST) & 1, p.status, GR_ERR_TIMEOUT);
    }
  } else if (warp < n_cw) {
    // ------------------------------------------------------------ compute warps
    const int mt = warp % n_mt, grp = warp / n_mt;
    // group 0 stages the query rows into shared memory (128-byte swizzle, two 64-dim halves)
    if (grp == 0) {
      // all eight 16-byte loads of a lane in flight together
      uint4 val[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int e = lane + 32 * k;
        const int r = mt * 16 + (e >> 4), chunk = e & 15;
        val[k] = make_uint4(0, 0, 0, 0);
        if (r < R) {
          const int g = r / p.K, j = r % p.K;
          val[k] = *reinterpret_cast<const uint4*>(p.q + ((size_t)b * p.K + j) * q_row_stride + (kvh * G + g) * 128 +
                                                   chunk * 8);
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int e = lane + 32 * k;
        const int r = mt * 16 + (e >> 4), chunk = e & 15;
        *reinterpret_cast<uint4*>(q_smem + (chunk >> 3) * (R_pad * 128) + sw128(r, chunk & 7)) = val[k];
      }
    }
    named_bar(bar_cw, n_cw * 32);
    const int g4 = lane >> 2, t4 = lane & 3;
    int lim[2];
    bool live[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + g4 + 8 * h;
      live[h] = r < R;
      lim[h] = live[h] ? min(row_limit(p, r % p.K, base), kv_end) : 0;
    }
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    for (int i = grp; i < n_tiles; i += NG) {
      const int s = (tb + i) % ST;
      if (!mbar_wait(full + s, ((tb + i) / ST) & 1, p.status, GR_ERR_TIMEOUT)) {
        *flag = 1;
        break;
      }
      const uint8_t* st = kv_smem + s * kStageBytes;
      const int tok0 = kv_beg + i * kTile;
      // S = Q K^T for 16 rows x 64 tokens (query fragments re-read from shared memory: fewer live registers)
      float sc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t qf[4];
        ldsm_x4(smem_u32(q_smem + (ks >> 2) * (R_pad * 128) + sw128(mt * 16 + (lane & 15), 2 * (ks & 3) + (lane >> 4))),
                qf[0], qf[1], qf[2], qf[3]);
        const uint8_t* kh = st + (ks >> 2) * kHalfBytes;
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int trow = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int ch = 2 * (ks & 3) + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(smem_u32(kh + sw128(trow, ch)), b0, b1, b2, b3);
          mma_16816(sc[2 * np], qf, b0, b1);
          mma_16816(sc[2 * np + 1], qf, b2, b3);
        }
      }
      // mask + online softmax (rows g4 and g4+8 of this warp's tile)
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e >> 1;
          const int tok = tok0 + n * 8 + 2 * t4 + (e & 1);
          const float x = (tok < lim[h]) ? sc[n][e] * p.scale_log2 : -INFINITY;
          sc[n][e] = x;
          mx[h] = fmaxf(mx[h], x);
        }
      }
      float alpha[2], msafe[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        const float mn = fmaxf(m_run[h], mx[h]);
        msafe[h] = (mn == -INFINITY) ? 0.f : mn;
        alpha[h] = (m_run[h] == -INFINITY) ? 0.f : exp2f(m_run[h] - msafe[h]);
        m_run[h] = mn;
      }
      float rs[2] = {0.f, 0.f};
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e >> 1;
          const float pe = exp2f(sc[n][e] - msafe[h]);
          sc[n][e] = pe;
          rs[h] += pe;
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
        rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
        l_run[h] = l_run[h] * alpha[h] + rs[h];
      }
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= alpha[0];
        o[n][1] *= alpha[0];
        o[n][2] *= alpha[1];
        o[n][3] *= alpha[1];
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_bf16(sc[2 * kk][0], sc[2 * kk][1]);
        pa[1] = pack_bf16(sc[2 * kk][2], sc[2 * kk][3]);
        pa[2] = pack_bf16(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
        pa[3] = pack_bf16(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
        const int trow = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
          const uint8_t* vh = st + (2 + (dp >> 2)) * kHalfBytes;
          const int ch = 2 * (dp & 3) + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(vh + sw128(trow, ch)), b0, b1, b2, b3);
          mma_16816(o[2 * dp], pa, b0, b1);
          mma_16816(o[2 * dp + 1], pa, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);
    }

    // ------------------------------------------------------------ combine the warp groups (group 1 -> group 0)
    if (NG > 1) {
      float* xch = reinterpret_cast<float*>(kv_smem) + (size_t)(mt * 32 + lane) * 68;  // every tile is consumed
      named_bar(bar_cw, n_cw * 32);
      if (grp == 1) {
        xch[0] = m_run[0]; xch[1] = m_run[1]; xch[2] = l_run[0]; xch[3] = l_run[1];
#pragma unroll
        for (int n = 0; n < 16; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) xch[4 + n * 4 + e] = o[n][e];
        }
      }
      named_bar(bar_cw, n_cw * 32);
      if (grp == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float m1 = xch[h], l1 = xch[2 + h];
          const float mn = fmaxf(m_run[h], m1);
          const float ms = (mn == -INFINITY) ? 0.f : mn;
          const float a0 = (m_run[h] == -INFINITY) ? 0.f : exp2f(m_run[h] - ms);
          const float a1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - ms);
          m_run[h] = mn;
          l_run[h] = l_run[h] * a0 + l1 * a1;
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            o[n][2 * h] = o[n][2 * h] * a0 + xch[4 + n * 4 + 2 * h] * a1;
            o[n][2 * h + 1] = o[n][2 * h + 1] * a0 + xch[4 + n * 4 + 2 * h + 1] * a1;
          }
        }
      }
    }

    // ------------------------------------------------------------ write / merge (group 0)
    // the cluster partials overwrite the stage ring: every compute warp must be done with its last tile
    if (p.cluster && n_active > 1) named_bar(bar_cw, n_cw * 32);
    if (grp == 0) {
      if (n_active == 1) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!live[h]) continue;
          const int r = mt * 16 + g4 + 8 * h;
          const int g = r / p.K, j = r % p.K;
          const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
          __nv_bfloat16* dst = p.out + ((size_t)b * p.K + j) * q_row_stride + (kvh * G + g) * 128;
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            const int d = n * 8 + 2 * t4;
            *reinterpret_cast<uint32_t*>(dst + d) = pack_bf16(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
          }
        }
      } else if (p.cluster) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = mt * 16 + g4 + 8 * h;
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            const int d = n * 8 + 2 * t4;
            *reinterpret_cast<float2*>(part_o + r * 128 + d) = make_float2(o[n][2 * h], o[n][2 * h + 1]);
          }
          if (t4 == 0) *reinterpret_cast<float2*>(part_ml + r * 2) = make_float2(m_run[h], l_run[h]);
        }
      } else {
        const size_t slot = ((size_t)b * p.n_kv_heads + kvh) * p.max_splits + split;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = mt * 16 + g4 + 8 * h;
          float* dst = p.ws_o + (slot * R_pad + r) * 128;
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            const int d = n * 8 + 2 * t4;
            *reinterpret_cast<float2*>(dst + d) = make_float2(o[n][2 * h], o[n][2 * h + 1]);
          }
          if (t4 == 0) {
            float* ml = p.ws_ml + (slot * R_pad + r) * 2;
            ml[0] = m_run[h];
            ml[1] = l_run[h];
          }
        }
      }
    }
  }
  if (p.cluster) {
    // Every split of the (request, kv head) is a CTA of this cluster (rank = split).  After the barrier each CTA
    // merges a share of the rows, reading the splits' partials from their shared memory in split order with the
    // same arithmetic as the global-memory merge below; the second barrier keeps the partials alive until read.
    cluster_sync_all();
    attention_merge_cluster(p, b, kvh, split, n_active, warp, lane, nthr >> 5, part_o, part_ml);
    cluster_sync_all();
    return;
  }
  if (n_active == 1) return;
  attention_merge_global(p, b, kvh, n_active, wt, nthr, bar_all, flag, reinterpret_cast<float*>(kv_smem));
}

}  // namespace gr
