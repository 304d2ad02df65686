// Verify / draft attention on the 5th-generation tensor cores (tcgen05, TMEM accumulators), sm_100a: the default
// kernel of the paged attention (attention.cu keeps the mma.sync kernel for rows that do not fit, and as the body of
// the persistent small-batch forward), with the same unit (split, kv head, request), the same row limits (draft: x0
// causal, the block bidirectional; verify: causal), the same split-KV partials and the same merges.
//
// Rows of a unit: r = g*K + j (query head g of the GQA group, window row j), R = G*K <= 128, row r = TMEM lane r.
// One CTA per unit; with W = ceil(R / 32) lane quadrants in use and H column parts (1 on large grids, where two
// CTAs per SM hide the softmax; 2 on grids of at most one CTA per SM, where its latency is the launch's):
//   softmax warps q + 4h (q < W, h < H): quadrant q (TMEM lanes 32q..32q+31, one thread per row), score columns
//                 h*64/H.. of each tile; with H = 2 the two warps of a quadrant exchange their row maxima through
//                 shared memory and each keeps the sum of its own columns;
//   producer      TMA: 64-token tiles (4 pages, K and V, both 64-dim halves, 128-byte swizzle) into the ring;
//   MMA           allocates TMEM and issues the MMAs from one thread.
// Per 64-token tile i (M = 128: rows R..127 are padding whose TMEM lanes no thread reads):
//   S_i = Q K_i^T   tcgen05.mma, A = Q (K-major, shared memory), B = K tile (K-major), N = 64, D = TMEM S[i % 2];
//   softmax         each thread loads its part of its row of S_i (64/H columns), masks, and exponentiates against
//                   its row's reference max m: m moves (and the warps rescale their O columns in TMEM: ld, multiply,
//                   st) only when the tile's max exceeds m by more than 2^8, so P <= 256; the sums are kept in fp32
//                   against the same m.  P_i (bf16) is written as a K-major operand over the tile's consumed K (dims
//                   0..63);
//   O += P_i V_i    tcgen05.mma, A = P (K-major), B = V tile (MN-major: 64 dims per 128-byte line, the two dim halves
//                   8 KB apart), N = 128, D = TMEM O.  Its commit frees the stage.
// The MMA thread issues whichever of S_{i+1} (its K/V landed, S buffer free) and O += P_i V_i (P_i written) is ready,
// so the next tile's QK^T runs under this tile's softmax and a stage is freed as soon as its PV completes.
// The result is O / l with O and l taken against the same m: the same quantity as the running-max formulation, up
// to fp32 / bf16 rounding.
// Split partials go to the workspace (global merge by the last split) or, when the splits of a (request, kv head)
// form one thread-block cluster, to each CTA's idle ring (merge through distributed shared memory).
#include "attention_dev.cuh"

namespace gr {

constexpr int kTcStages = 3;       // large grids: two CTAs per SM
constexpr int kTcStagesSmall = 5;  // grids of at most one CTA per SM: a deeper ring (fits 128 rows in 227 KB)
constexpr uint32_t kTcTmemCols = 256;  // S[0] 0..63, S[1] 64..127, O 128..255
constexpr float kTcRescaleLog2 = 8.0f;  // the reference max moves when a row's max exceeds it by more than this

__host__ __device__ constexpr int tc_rows(int G, int K) { return G * K; }
__host__ __device__ constexpr int tc_quadrants(int R) { return (R + 31) / 32; }
// warps: softmax q + 4h, then the producer and the MMA warp (H = 2: in slots 2, 3 when W <= 2)
__host__ __device__ constexpr int tc_prod_warp(int W, int H) { return H == 1 ? W : (W <= 2 ? 2 : 4 + W); }
__host__ __device__ constexpr int tc_warps(int W, int H) {
  return tc_prod_warp(W, H) + 2 > 4 * (H - 1) + W ? tc_prod_warp(W, H) + 2 : 4 * (H - 1) + W;
}
// one 64-dim atom of the query operand: the rows rounded up to 8-row (1024-byte) swizzle groups
__host__ __device__ constexpr uint32_t tc_q_atom_bytes(int R) { return static_cast<uint32_t>((R + 7) / 8) * 1024; }
constexpr int kTcXchgBytes = (2 * 2 * 128 + 2 * 128) * 4;  // row maxima [tile parity][half][row], sums [half][row]

// Shared memory (1024-aligned): Q (two atoms), the ring, barriers, TMEM slot, flag, page ids, the halves' exchange.
// An M = 128 operand read from Q or from a stage's P runs past the rows written (rows that only feed padding lanes);
// everything it reads stays inside the allocation.
size_t attention_tc_smem_bytes(int G, int K, int stages) {
  return 1024 + 2 * static_cast<size_t>(tc_q_atom_bytes(tc_rows(G, K))) + static_cast<size_t>(stages) * kStageBytes +
         (3 * stages + 4) * 8 + 16 + kMaxChunkPages * 4 + kTcXchgBytes;
}

template <int ST, int H>
__global__ void __launch_bounds__(320) attention_tc_kernel(const __grid_constant__ CUtensorMap tmk,
                                                           const __grid_constant__ CUtensorMap tmv,
                                                           const AttnParams p) {
  GR_TL_BEGIN
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int G = p.n_q_heads / p.n_kv_heads;
  const int R = tc_rows(G, p.K);
  const int W = tc_quadrants(R);
  constexpr int CW = kTile / H;  // score columns per softmax thread
  const int w_prod = tc_prod_warp(W, H), w_mma = w_prod + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool is_sm = warp < 4 * H && (warp & 3) < W;
  const int q = warp & 3, h = warp >> 2;  // softmax warps: quadrant, column part
  const uint32_t qa = tc_q_atom_bytes(R);
  uint8_t* q_smem = smem;
  uint8_t* ring = smem + 2 * qa;
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(ring + ST * kStageBytes);
  uint64_t* kv_empty = kv_full + ST;  // PV of the stage's tile complete: stage free, O up to date
  uint64_t* s_full = kv_empty + ST;   // [2] by tile parity
  uint64_t* p_full = s_full + 2;      // [2] by tile parity
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_full + 2);
  int* flag = reinterpret_cast<int*>(tmem_slot + 2);
  int* pages = flag + 2;
  float* xm = reinterpret_cast<float*>(pages + kMaxChunkPages);  // [2][2][128]
  float* xl = xm + 2 * 2 * 128;                                  // [2][128]
  // cluster merge: this split's (O, m, l) partial in the idle ring once its last PV has completed
  float* part_o = reinterpret_cast<float*>(ring);         // [R_pad][128]
  float* part_ml = part_o + attn_rows_pad(G, p.K) * 128;  // [R_pad][2]

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(s_full + k, 1);
      mbar_init(p_full + k, H * W);  // one arrival per softmax warp
    }
    *flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }
  // TMEM is taken before the dependent launch is released: a CTA of a later kernel (which may wait for this grid)
  // can then never hold the columns this CTA is waiting for
  if (warp == w_mma) tmem_alloc(tmem_slot, kTcTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) pdl_trigger();
  // Blocks launch x fastest: grids are (split, kv head, request), or (kv head, request, split) with split_outer.
  // Requests in `order` (longest first) shorten the tail of a mixed-length batch.
  const int split = p.split_outer ? blockIdx.z : blockIdx.x, kvh = p.split_outer ? blockIdx.x : blockIdx.y;
  const int zr = p.split_outer ? blockIdx.y : blockIdx.z;
  const int b = p.order ? p.order[zr] : zr;
  // the producer warp reads the split's page ids while the previous kernel finishes
  if (warp == w_prod) attn_preload_pages(p, b, split, lane, pages);
  pdl_wait();

  const int base = static_cast<int>(p.seq_lens[b]) + p.base_add;
  const int L = base + p.K;  // the last row's limit
  const int n_active = (L + p.chunk - 1) / p.chunk;
  const bool active = split < n_active;  // uniform over the CTA
  const int kv_beg = split * p.chunk;
  const int kv_end = min(L, kv_beg + p.chunk);
  const int n_tiles = active ? (kv_end - kv_beg + kTile - 1) / kTile : 0;
  const size_t q_row_stride = static_cast<size_t>(p.n_q_heads) * 128;
  const int r = q * 32 + lane;  // softmax warps: this thread's row
  const bool valid = is_sm && r < R;
  const int g = valid ? r / p.K : 0, j = valid ? r % p.K : 0;

  if (active && is_sm) {
    // ------------------------------------------------------------ query rows -> shared memory (part h: dims
    // h*128/H.., the 64-dim atoms h*2/H..)
    constexpr int QC = 16 / H;  // 16-byte chunks of the row per thread
    const uint4* src = reinterpret_cast<const uint4*>(p.q + ((size_t)b * p.K + j) * q_row_stride +
                                                      (kvh * G + g) * 128 + h * (128 / H));
    uint4 val[QC];
#pragma unroll
    for (int c = 0; c < QC; ++c) val[c] = valid ? src[c] : make_uint4(0, 0, 0, 0);
    if (r < (R + 7) / 8 * 8) {
#pragma unroll
      for (int c = 0; c < QC; ++c) {
        const int cc = h * QC + c;  // chunk of the 128-dim row
        *reinterpret_cast<uint4*>(q_smem + (cc >> 3) * qa + sw128(r, cc & 7)) = val[c];
      }
    }
    fence_proxy_async_smem();
  }
  if (active && (is_sm || warp == w_mma)) named_bar(2, (H * W + 1) * 32);  // Q staged before the first MMA

  if (!active) {
    // no tiles: straight to the teardown
  } else if (warp == w_prod) {
    // ------------------------------------------------------------ producer (page ids preloaded above)
    const int last_slot = (L - 1) / p.page_size - kv_beg / p.page_size;
    __syncwarp();
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < n_tiles; ++i) {
        const int s = i % ST;
        if (i >= ST && !mbar_wait(kv_empty + s, ((i / ST) - 1) & 1, p.status, GR_ERR_TIMEOUT)) break;
        mbar_arrive_expect_tx(kv_full + s, kStageBytes);
        uint8_t* st = ring + s * kStageBytes;
#pragma unroll
        for (int pg = 0; pg < 4; ++pg) {
          const int y = (attn_page(pages, i * 4 + pg, last_slot, true) * p.n_kv_heads + kvh) * p.page_size;
          tma_load_2d(st + 0 * kHalfBytes + pg * 2048, &tmk, kv_full + s, 0, y);
          tma_load_2d(st + 1 * kHalfBytes + pg * 2048, &tmk, kv_full + s, 64, y);
          tma_load_2d(st + 2 * kHalfBytes + pg * 2048, &tmv, kv_full + s, 0, y);
          tma_load_2d(st + 3 * kHalfBytes + pg * 2048, &tmv, kv_full + s, 64, y);
        }
        issued = i + 1;
      }
      // no copy may still be landing in shared memory when the CTA moves on
      for (int i = max(0, issued - ST); i < issued; ++i)
        mbar_wait(kv_full + (i % ST), (i / ST) & 1, p.status, GR_ERR_TIMEOUT);
    }
  } else if (warp == w_mma) {
    // ------------------------------------------------------------ MMA issue (one thread)
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16_f32(128, kTile);
      const uint32_t id_pv = idesc_bf16_f32(128, 128) | (1u << 16);  // B (V) MN-major
      const uint64_t qd0 = smem_desc_sw128(smem_u32(q_smem));
      const uint64_t qd1 = smem_desc_sw128(smem_u32(q_smem + qa));
      const uint64_t kd = smem_desc_sw128(smem_u32(ring));  // stage 0: K dims 0..63, later P
      const uint64_t vd = smem_desc_sw128_mn(smem_u32(ring + 2 * kHalfBytes), kHalfBytes);  // stage 0: V dims 0..63
      int s_next = 0, pv_next = 0;
      uint64_t t0 = globaltimer();
      while (pv_next < n_tiles) {
        bool progress = false;
        // O += P_k V_k as soon as P_k is written (frees the stage)
        if (pv_next < s_next && mbar_poll(p_full + (pv_next & 1), (pv_next >> 1) & 1)) {
          tc_fence_after();
          const int s = pv_next % ST;
          const uint32_t so = (static_cast<uint32_t>(s) * kStageBytes) >> 4;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // 16 tokens per MMA: 32 bytes of a P row, 2 KB of V lines
            tc_mma_bf16(tmem + 128, kd + so + 2 * kk, vd + so + 128 * kk, id_pv, (pv_next | kk) != 0);
          tc_commit(kv_empty + s);
          ++pv_next;
          progress = true;
        }
        // S_i = Q K_i^T once its tile landed and its S buffer is free (the softmax is done with S_{i-2})
        if (s_next < n_tiles && s_next <= pv_next + 1 && mbar_poll(kv_full + s_next % ST, (s_next / ST) & 1)) {
          tc_fence_after();
          const uint32_t so = (static_cast<uint32_t>(s_next % ST) * kStageBytes) >> 4;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // 16 dims per MMA
            tc_mma_bf16(tmem + (s_next & 1) * kTile, (kk < 4 ? qd0 : qd1) + 2 * (kk & 3),
                        kd + so + (kk >> 2) * (kHalfBytes >> 4) + 2 * (kk & 3), id_s, kk != 0);
          tc_commit(s_full + (s_next & 1));
          ++s_next;
          progress = true;
        }
        if (progress) {
          t0 = globaltimer();
        } else if (globaltimer() - t0 > GR_WAIT_NS) {
          report(p.status, GR_ERR_TIMEOUT);
          break;
        }
      }
    }
  } else if (is_sm) {
    // ------------------------------------------------------------ softmax warps
    // Padding lanes (rows >= R) take the unmasked path on whatever their S holds: their P rows only feed O rows that
    // nobody reads, and they never ask for a rescale.  After a timed-out wait a warp stops working but keeps taking
    // its quadrant's exchange barriers, so that its partner never waits for it.
    const int lim = valid ? min(row_limit(p, j, base), kv_end) : 0x7fffffff;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const float sc = p.scale_log2;
    const int bar_q = 3 + q;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(s_full + (i & 1), (i >> 1) & 1, p.status, GR_ERR_TIMEOUT));
      uint32_t sr[CW];
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < CW / 32; ++c)
          tmem_ld32_issue(t_lane + (i & 1) * kTile + h * CW + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sr + 32 * c));
#pragma unroll
        for (int c = 0; c < CW / 32; ++c) tmem_ld32_wait(*reinterpret_cast<uint32_t(*)[32]>(sr + 32 * c));
      } else {
#pragma unroll
        for (int c = 0; c < CW; ++c) sr[c] = 0u;
      }
      const int tok0 = kv_beg + i * kTile + h * CW;
      // raw scores; masked positions become -inf (scale_log2 > 0, so the max of the raw scores scales)
      if (tok0 + CW > lim) {
#pragma unroll
        for (int c = 0; c < CW; ++c)
          if (tok0 + c >= lim) sr[c] = __float_as_uint(-INFINITY);
      }
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < CW; ++c) m4[c & 3] = fmaxf(m4[c & 3], __uint_as_float(sr[c]));
      float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      if constexpr (H == 2) {
        xm[((i & 1) * 2 + h) * 128 + r] = mx;
        named_bar(bar_q, 64);
        const float mo = xm[((i & 1) * 2 + (h ^ 1)) * 128 + r];
        mx = h == 0 ? fmaxf(mx, mo) : fmaxf(mo, mx);
      }
      mx *= sc;
      // the reference max moves only when the tile's max exceeds it by more than 2^8 (always for the first visible
      // token); O needs rescaling only if it already holds visible tokens
      float m_new = m_run;
      bool resc = false;
      if (mx > m_run + kTcRescaleLog2) {
        resc = valid && m_run != -INFINITY;
        m_new = mx;
      }
      const float alpha = resc ? ex2_approx(m_run - m_new) : 1.f;
      const float nm = (m_new == -INFINITY) ? 0.f : -m_new;
      float r4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[CW / 2];
#pragma unroll
      for (int c = 0; c < CW / 2; ++c) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(sr[2 * c]), sc, nm));
        const float p1 = ex2_approx(fmaf(__uint_as_float(sr[2 * c + 1]), sc, nm));
        r4[(2 * c) & 3] += p0;
        r4[(2 * c + 1) & 3] += p1;
        pk[c] = pack_bf16(p0, p1);
      }
      l_run = l_run * alpha + ((r4[0] + r4[1]) + (r4[2] + r4[3]));
      m_run = m_new;
      if (ok && __any_sync(0xffffffffu, resc)) {
        // O holds tiles 0..i-1 once the previous tile's PV completed (resc implies i > 0); this warp rescales its
        // part of the O columns
        const int k = i - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(kv_empty + k % ST, (k / ST) & 1, p.status, GR_ERR_TIMEOUT));
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (int c4 = 0; c4 < 4 / H; ++c4) {
            uint32_t o[32];
            const uint32_t ta = t_lane + 128 + h * (128 / H) + c4 * 32;
            tmem_ld32_issue(ta, o);
            tmem_ld32_wait(o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(ta, o);
          }
          tmem_wait_st();
        }
      }
      if (ok) {
        // this part of the P_i row over the stage's consumed K dims 0..63 (S_i, its only reader, has completed)
        uint8_t* p_smem = ring + (i % ST) * kStageBytes;
#pragma unroll
        for (int c = 0; c < CW / 8; ++c)
          *reinterpret_cast<uint4*>(p_smem + sw128(r, (CW / 8) * h + c)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + (i & 1));
      }
    }
    // ------------------------------------------------------------ output rows / split partials
    if (ok) {
      const int k = n_tiles - 1;  // the last PV
      ok = __all_sync(0xffffffffu, mbar_wait(kv_empty + k % ST, (k / ST) & 1, p.status, GR_ERR_TIMEOUT));
    }
    float l_tot = l_run;
    if constexpr (H == 2) {
      xl[h * 128 + r] = l_run;
      named_bar(bar_q, 64);
      l_tot = xl[r] + xl[128 + r];
    }
    if (ok) {
      tc_fence_after();
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
      const int R_pad = attn_rows_pad(G, p.K);
      const size_t slot = ((size_t)b * p.n_kv_heads + kvh) * p.max_splits + split;
      __nv_bfloat16* dst_o = p.out + ((size_t)b * p.K + j) * q_row_stride + (kvh * G + g) * 128 + h * (128 / H);
      // split partials: this CTA's shared memory (cluster merge) or the workspace (global merge)
      float* dst_w = (p.cluster ? part_o : p.ws_o + slot * R_pad * 128) + (valid ? r : 0) * 128 + h * (128 / H);
#pragma unroll 1
      for (int c4 = 0; c4 < 4 / H; ++c4) {
        uint32_t o[32];
        tmem_ld32_issue(t_lane + 128 + h * (128 / H) + c4 * 32, o);
        tmem_ld32_wait(o);
        if (!valid) continue;
        if (n_active == 1) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(o[8 * e + 0]) * inv, __uint_as_float(o[8 * e + 1]) * inv);
            v.y = pack_bf16(__uint_as_float(o[8 * e + 2]) * inv, __uint_as_float(o[8 * e + 3]) * inv);
            v.z = pack_bf16(__uint_as_float(o[8 * e + 4]) * inv, __uint_as_float(o[8 * e + 5]) * inv);
            v.w = pack_bf16(__uint_as_float(o[8 * e + 6]) * inv, __uint_as_float(o[8 * e + 7]) * inv);
            *reinterpret_cast<uint4*>(dst_o + c4 * 32 + e * 8) = v;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            *reinterpret_cast<float4*>(dst_w + c4 * 32 + e * 4) =
                make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]), __uint_as_float(o[4 * e + 2]),
                            __uint_as_float(o[4 * e + 3]));
        }
      }
      if (valid && h == 0 && n_active > 1) {
        float* ml = (p.cluster ? part_ml : p.ws_ml + slot * R_pad * 2) + r * 2;
        ml[0] = m_run;
        ml[1] = l_tot;
      }
    }
  }

  // every TMEM read done and every MMA complete (the softmax warps waited for the last PV)
  tc_fence_before();
  __syncthreads();
  if (warp == w_mma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  }
  if (p.cluster) {
    // every split of the (request, kv head) is a CTA of this cluster, idle ones included: after the barrier each
    // merges a share of the rows from the partials in the CTAs' shared memory; the second barrier keeps them alive
    cluster_sync_all();
    attention_merge_cluster(p, b, kvh, split, n_active, warp, lane, blockDim.x >> 5, part_o, part_ml);
    cluster_sync_all();
  } else if (active && n_active > 1) {  // the ring is idle: the merge's weights go there
    attention_merge_global(p, b, kvh, n_active, threadIdx.x, blockDim.x, 1, flag, reinterpret_cast<float*>(ring));
  }
  GR_TL_END(kTlAttentionTc)
}

template <int ST, int H>
static cudaError_t configure_attention_tc() {
  static PerDeviceOnce configured;
  return once_per_device(configured, [] {
    auto kern = attention_tc_kernel<ST, H>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  });
}

// Whether clusters of `size` CTAs of the small-grid configuration fit on the current device (cached per device, size,
// threads and shared memory).
static bool attention_tc_cluster_ok(int size, int threads, size_t smem) {
  static ClusterFitCache cache;
  return cluster_fit_cached(cache, size, threads, smem, [&] {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const bool ok =
        cudaOccupancyMaxActiveClusters(&n, attention_tc_kernel<kTcStagesSmall, 2>, &cfg) == cudaSuccess && n >= 1;
    cudaGetLastError();  // a refused query leaves no sticky error
    return ok;
  });
}

bool attention_tc_fits(const AttnParams& p) {
  const int G = p.n_q_heads / p.n_kv_heads;
  return G >= 1 && p.K >= 1 && G * p.K <= 128 && p.page_size == 16;
}

// small: grids of at most one CTA per SM (deeper ring, two column parts; the splits of a (request, kv head) form one
// cluster where the device holds such clusters, else the global merge).
cudaError_t launch_attention_tc(const CUtensorMap& tmk, const CUtensorMap& tmv, const AttnParams& p, bool small,
                                cudaStream_t stream, bool pdl) {
  if (!attention_tc_fits(p)) return cudaErrorInvalidValue;
  const int G = p.n_q_heads / p.n_kv_heads;
  const int warps = tc_warps(tc_quadrants(tc_rows(G, p.K)), small ? 2 : 1);
  const int stages = small ? kTcStagesSmall : kTcStages;
  cudaError_t e = small ? configure_attention_tc<kTcStagesSmall, 2>() : configure_attention_tc<kTcStages, 1>();
  if (e != cudaSuccess) return e;
  AttnParams q = p;
  q.groups = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(32 * warps);
  cfg.dynamicSmemBytes = attention_tc_smem_bytes(G, p.K, stages);
  cfg.stream = stream;
  q.cluster = (small && p.max_splits >= 2 && p.max_splits <= kMaxMergeSplits &&
               attention_tc_cluster_ok(p.max_splits, 32 * warps, cfg.dynamicSmemBytes)) ? 1 : 0;
  // With the widest chunk a second split holds only what a request has beyond 4,096 tokens, and most second splits
  // are idle (they exit at once).  Splits outermost: every request's first split launches before any second one, so
  // the idle CTAs come after all working ones instead of taking slots between them (config 3, 64 requests: 102.8 ->
  // 99.8 us).  With narrower chunks the second halves of long requests would launch last and lengthen the tail
  // (32 requests at 2,048: 55.7 -> 58.5 us), so they keep the request-major order.  A cluster spans x.
  q.split_outer = (!q.cluster && p.chunk >= kMaxChunkPages * p.page_size) ? 1 : 0;
  cfg.gridDim = q.split_outer ? dim3(p.n_kv_heads, p.bs, p.max_splits) : dim3(p.max_splits, p.n_kv_heads, p.bs);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (q.cluster) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = p.max_splits;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return small ? cudaLaunchKernelEx(&cfg, attention_tc_kernel<kTcStagesSmall, 2>, tmk, tmv, q)
               : cudaLaunchKernelEx(&cfg, attention_tc_kernel<kTcStages, 1>, tmk, tmv, q);
}

}  // namespace gr

GR_TIMELINE_EXPORTS(attention_tc)
