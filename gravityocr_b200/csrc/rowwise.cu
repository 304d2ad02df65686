// Row-wise kernels of the round: window planning + embedding + input norm, the sandwich residual norm, the
// accept-and-commit step and the forced-accept draft override.  All HBM-bound on a few KB per row; one CTA per row
// (192 threads x 8 bf16 lanes = one 1536-wide row per pass).
#include "rowwise_dev.cuh"

namespace gr {

constexpr int kRowThreads = 192;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// ------------------------------------------------------------------ embedding rows + window plan + input norm
__global__ void __launch_bounds__(kRowThreads) embed_rows_kernel(const EmbedParams p) {
  GR_TL_BEGIN
  __shared__ float red[32];
  __shared__ int64_t s_id;
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int b = t / p.K, j = t % p.K;
  if (threadIdx.x == 0) {
    const int64_t seq = p.seq_lens[b];
    int64_t id;
    int64_t pos;
    if (p.mode == GR_ROWS_DRAFT) {
      id = (j == 0) ? p.seeds[p.rpi[b]] : p.mask_id;
      pos = seq + j;
    } else if (p.mode == GR_ROWS_VERIFY) {
      id = p.ids32[t];
      pos = seq + 1 + j;
    } else {
      id = p.ids64[t];
      pos = seq + j;
    }
    if (id >= p.vocab || (id < 0 && (p.mode != GR_ROWS_EXPLICIT || p.row_embeds == nullptr))) {
      report(p.status, GR_ERR_BAD_ID);
      id = 0;
    }
    int64_t lp = pos / p.page_size;
    if (lp >= p.pages_per_req) {
      report(p.status, GR_ERR_BAD_PAGE);
      lp = p.pages_per_req - 1;
    }
    const int64_t phys = p.page_table[(size_t)b * p.pt_stride + lp];
    p.row_pos[t] = static_cast<int32_t>(pos + (p.rope_delta ? p.rope_delta[b] : 0));
    p.row_slot[t] = phys * p.page_size + (pos % p.page_size);
    if (p.row_ids) p.row_ids[t] = static_cast<int32_t>(id);
    s_id = id;
  }
  __syncthreads();
  const int64_t id = s_id;
  float v[8];
  float ss = 0.f;
  const int H = p.hidden;
  float* hrow = p.h_out + (size_t)t * H;
  __nv_bfloat16* xrow = p.x_out + (size_t)t * H;
  // one pass when H <= 8 * blockDim (the baseline's 1536); generic loop otherwise
  for (int c = threadIdx.x * 8; c < H; c += kRowThreads * 8) {
    if (id >= 0) {
      const uint4 raw = *reinterpret_cast<const uint4*>(p.embed + (size_t)id * H + c);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(e[i]);
    } else {
      const float4 a = *reinterpret_cast<const float4*>(p.row_embeds + (size_t)t * H + c);
      const float4 bb = *reinterpret_cast<const float4*>(p.row_embeds + (size_t)t * H + c + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = bb.x; v[5] = bb.y; v[6] = bb.z; v[7] = bb.w;
    }
    *reinterpret_cast<float4*>(hrow + c) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(hrow + c + 4) = make_float4(v[4], v[5], v[6], v[7]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  }
  const float r = rsqrtf(block_sum(ss, red) / H + p.eps);
  for (int c = threadIdx.x * 8; c < H; c += kRowThreads * 8) {
    const float4 a = *reinterpret_cast<const float4*>(hrow + c);
    const float4 bb = *reinterpret_cast<const float4*>(hrow + c + 4);
    const float hv[8] = {a.x, a.y, a.z, a.w, bb.x, bb.y, bb.z, bb.w};
    const uint4 wraw = *reinterpret_cast<const uint4*>(p.norm_w + c);
    const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(&wraw);
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = pack_bf16(__bfloat162float(w[2 * i]) * (hv[2 * i] * r), __bfloat162float(w[2 * i + 1]) * (hv[2 * i + 1] * r));
    *reinterpret_cast<uint4*>(xrow + c) = out;
  }
  GR_TL_END(kTlEmbed)
}

// ------------------------------------------------------------------ residual + sandwich norm
// One CTA per row; each thread owns up to kMaxChunks groups of 8 features, kept in registers between the passes.
// MC = 1 when the row fits one 8-feature chunk per thread (hidden <= 1536); four split partials in flight per thread.
// Many rows: the default register budget (62 registers at MC = 1, five CTAs resident per SM).  Few rows
// (<= kNormFewRows): an explicit one-block minimum, under which the compiler keeps more loads in flight (112 registers;
// batch-1 forward 0.825 -> 0.799 ms).  A cap of 40 registers for eight CTAs per SM spilled and was slower at 1,088
// rows.
constexpr int kNormFewRows = 512;
template <int MC>
__global__ void __launch_bounds__(kRowThreads) residual_norm_kernel(const ResNormParams p) {
  GR_TL_BEGIN
  __shared__ float red[32];
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  resnorm_row<MC>(p, blockIdx.x, threadIdx.x, blockDim.x, 1, red);
  GR_TL_END(kTlResidualNorm)
}
template <int MC>
__global__ void __launch_bounds__(kRowThreads, 1) residual_norm_few_rows_kernel(const ResNormParams p) {
  GR_TL_BEGIN
  __shared__ float red[32];
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  resnorm_row<MC>(p, blockIdx.x, threadIdx.x, blockDim.x, 1, red);
  GR_TL_END(kTlResidualNorm)
}

// Many rows (> kNormFewRows, hidden == 8 * kRowThreads, NP split-K partials): kNormCtasPerSm CTAs per SM walk the rows
// (row t, t + grid, ...).  A thread issues the next row's loads (its 8 features of every partial and of h) before the
// current row's two reductions, so each row's L2 round trip overlaps the previous row's reductions and stores
// instead of opening every CTA; the norm weights are loaded once, before the wait for the previous kernel.  Same
// arithmetic in the same order as resnorm_row (partials summed in split order, the same block reductions): the
// outputs are bit-identical.  One CTA per row measured 7.5 us at 1,088 rows inside the forward.  Up to two partials
// four CTAs per SM fit without spills (76 registers), three or four partials three CTAs per SM.
__host__ __device__ constexpr int norm_ctas_per_sm(int np) { return np <= 2 ? 4 : 3; }
template <int NP>
__global__ void __launch_bounds__(kRowThreads, norm_ctas_per_sm(NP)) residual_norm_rows_kernel(const ResNormParams p) {
  GR_TL_BEGIN
  __shared__ float red[32];
  if (threadIdx.x == 0) pdl_trigger();
  const int H = p.hidden;
  const int c = threadIdx.x * 8;
  const size_t part = (size_t)p.m * H;
  const uint4 wa = *reinterpret_cast<const uint4*>(p.w_a + c);
  const uint4 wb = *reinterpret_cast<const uint4*>(p.w_b + c);
  const __nv_bfloat16* wav = reinterpret_cast<const __nv_bfloat16*>(&wa);
  const __nv_bfloat16* wbv = reinterpret_cast<const __nv_bfloat16*>(&wb);
  float ny[NP][8], nh[8];
  auto load = [&](int t) {
    const float* yrow = p.y + (size_t)t * H + c;
#pragma unroll
    for (int s = 0; s < NP; ++s) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(yrow + s * part));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(yrow + s * part + 4));
      ny[s][0] = a.x; ny[s][1] = a.y; ny[s][2] = a.z; ny[s][3] = a.w;
      ny[s][4] = b.x; ny[s][5] = b.y; ny[s][6] = b.z; ny[s][7] = b.w;
    }
    const float4 ha = *reinterpret_cast<const float4*>(p.h_in + (size_t)t * H + c);
    const float4 hb = *reinterpret_cast<const float4*>(p.h_in + (size_t)t * H + c + 4);
    nh[0] = ha.x; nh[1] = ha.y; nh[2] = ha.z; nh[3] = ha.w;
    nh[4] = hb.x; nh[5] = hb.y; nh[6] = hb.z; nh[7] = hb.w;
  };
  pdl_wait();
  int t = blockIdx.x;
  if (t < p.m) load(t);
  for (; t < p.m; t += gridDim.x) {
    float yv[8], hv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int s = 0; s < NP; ++s) acc += ny[s][i];  // split order
      yv[i] = acc;
      hv[i] = nh[i];
    }
    if (t + gridDim.x < p.m) load(t + gridDim.x);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += yv[i] * yv[i];
    const float ra = rsqrtf(block_sum_bar(ss, red, threadIdx.x, kRowThreads, 1) / H + p.eps);
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      yv[i] = hv[i] + __bfloat162float(wav[i]) * (yv[i] * ra);  // the new residual
      s2 += yv[i] * yv[i];
    }
    float* hout = p.h_out + (size_t)t * H + c;
    *reinterpret_cast<float4*>(hout) = make_float4(yv[0], yv[1], yv[2], yv[3]);
    *reinterpret_cast<float4*>(hout + 4) = make_float4(yv[4], yv[5], yv[6], yv[7]);
    const float rb = rsqrtf(block_sum_bar(s2, red, threadIdx.x, kRowThreads, 1) / H + p.eps);
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = pack_bf16(__bfloat162float(wbv[2 * i]) * (yv[2 * i] * rb), __bfloat162float(wbv[2 * i + 1]) * (yv[2 * i + 1] * rb));
    *reinterpret_cast<uint4*>(p.x_out + (size_t)t * H + c) = out;
  }
  GR_TL_END(kTlResidualNorm)
}

// ------------------------------------------------------------------ accept and commit
constexpr int kCommitThreads = 256;

__global__ void __launch_bounds__(kCommitThreads) accept_commit_kernel(const CommitParams p) {
  GR_TL_BEGIN
  __shared__ int warp_tot[kCommitThreads / 32];
  __shared__ int carry;
  if (threadIdx.x == 0) {
    carry = 0;
    pdl_trigger();
  }
  pdl_wait();
  __syncthreads();
  const int K = p.K;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int b0 = 0; b0 < p.bs; b0 += kCommitThreads) {
    const int b = b0 + threadIdx.x;
    const bool act = b < p.bs;
    int acc = 0;
    if (act) {
      if (p.accept) {  // sampled verify: row j's bit says whether d_{j+1} was accepted
        const int32_t* a = p.accept + (size_t)b * K;
        while (acc + 1 < K && a[acc] != 0) ++acc;
      } else {  // greedy verify: d_{j+1} equals the argmax of row j
        const int32_t* d = p.am + (size_t)b * K;
        const int32_t* v = p.v + (size_t)b * K;
        while (acc + 1 < K && d[acc + 1] == v[acc]) ++acc;
      }
    }
    const int rej = act ? (K - 1 - acc) : 0;
    // block-wide exclusive scan of the rejected counts
    int x = rej;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[w] = x;
    __syncthreads();
    int before = carry;
    for (int i = 0; i < w; ++i) before += warp_tot[i];
    const int excl = before + x - rej;
    if (act) {
      const int32_t* d = p.am + (size_t)b * K;
      // verified token j: the verify argmax, or for a sampled verify the accepted draft / the final draw
      auto vtok = [&](int j) -> int32_t {
        if (!p.accept) return p.v[(size_t)b * K + j];
        return j < acc ? d[j + 1] : p.sample[(size_t)b * K + acc];
      };
      int32_t* row = p.packed + (size_t)b * (K + 2);
      row[0] = d[0];
      row[1] = acc;
      for (int j = 0; j < K; ++j) {
        const int32_t t = (j <= acc) ? vtok(j) : 0;
        row[2 + j] = t;
        if (p.predict) p.predict[(size_t)b * K + j] = t;
      }
      const int64_t seed = vtok(acc);
      p.seeds[p.rpi[b]] = seed;
      p.out_next[b] = seed;
      const int64_t s = p.seq_lens[b];
      const int64_t s_x0 = p.x0_committed ? s : s + 1;  // KV length with x0; verify row j sits at s_x0 + j
      p.seq_lens[b] = s_x0 + acc + 1;
      for (int j = acc + 1; j < K; ++j)
        p.released[excl + (j - acc - 1)] = p.loc ? p.loc[(size_t)b * K + j] : s_x0 + j;
      if (p.n_committed) p.n_committed[b] += acc + 2;
      if (p.rounds) p.rounds[b] += 1;
      if (p.accept_len) p.accept_len[b] = acc;
    }
    __syncthreads();
    if (threadIdx.x == kCommitThreads - 1) carry = excl + rej;
    __syncthreads();
  }
  if (threadIdx.x == 0 && p.n_released) p.n_released[0] = carry;
  if (threadIdx.x == 0 && p.rng) p.rng[1] += 1;  // the next round draws fresh coins
  GR_TL_END(kTlCommit)
}

// ------------------------------------------------------------------ forced-accept replay
__global__ void draft_override_kernel(const OverrideParams p) {
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= p.bs) return;
  const int c = p.n_committed[b];
  const int A = p.plan[(size_t)b * p.plan_stride + p.rounds[b]];
  int32_t* d = p.am + (size_t)b * p.K;
  const int32_t* g = p.g + (size_t)b * p.g_stride;
  for (int j = 1; j <= A && j < p.K; ++j) d[j] = g[c + j];
  if (A + 1 < p.K) {
    int t = (g[c + A + 1] + 1) % p.vocab;
    if (t == p.mask_id) t = (t + 1) % p.vocab;
    d[A + 1] = t;
  }
}

// ------------------------------------------------------------------ gate/up interleave (load time)
// destination row 2j = gate row j, 2j + 1 = up row j (the SwiGLU epilogue pairs adjacent TMEM lanes)
__global__ void pack_gate_up_kernel(const __nv_bfloat16* src, __nv_bfloat16* dst, int I, int H) {
  const int r = blockIdx.x;
  const int srow = (r & 1) ? I + (r >> 1) : (r >> 1);
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
    *reinterpret_cast<uint4*>(dst + (size_t)r * H + c) = *reinterpret_cast<const uint4*>(src + (size_t)srow * H + c);
}

// ------------------------------------------------------------------ launchers
template <typename Kern, typename P>
static cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, const P& p, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_embed_rows(const EmbedParams& p, cudaStream_t s, bool pdl) {
  return launch_pdl(embed_rows_kernel, dim3(p.bs * p.K), dim3(kRowThreads), p, s, pdl);
}
cudaError_t launch_residual_norm(const ResNormParams& p, cudaStream_t s, bool pdl) {
  if (p.hidden <= 8 * kRowThreads) {
    if (p.m <= kNormFewRows)
      return launch_pdl(residual_norm_few_rows_kernel<1>, dim3(p.m), dim3(kRowThreads), p, s, pdl);
    if (p.hidden == 8 * kRowThreads && p.y_parts <= 4) {
      const int sms = p.sms > 0 ? p.sms : 148;
      const dim3 grid(min(p.m, sms * norm_ctas_per_sm(p.y_parts)));
      switch (p.y_parts) {
        case 1: return launch_pdl(residual_norm_rows_kernel<1>, grid, dim3(kRowThreads), p, s, pdl);
        case 2: return launch_pdl(residual_norm_rows_kernel<2>, grid, dim3(kRowThreads), p, s, pdl);
        case 3: return launch_pdl(residual_norm_rows_kernel<3>, grid, dim3(kRowThreads), p, s, pdl);
        default: return launch_pdl(residual_norm_rows_kernel<4>, grid, dim3(kRowThreads), p, s, pdl);
      }
    }
    return launch_pdl(residual_norm_kernel<1>, dim3(p.m), dim3(kRowThreads), p, s, pdl);
  }
  return launch_pdl(residual_norm_kernel<kMaxChunks>, dim3(p.m), dim3(kRowThreads), p, s, pdl);
}
cudaError_t launch_accept_commit(const CommitParams& p, cudaStream_t s, bool pdl) {
  return launch_pdl(accept_commit_kernel, dim3(1), dim3(kCommitThreads), p, s, pdl);
}
cudaError_t launch_draft_override(const OverrideParams& p, cudaStream_t s, bool pdl) {
  return launch_pdl(draft_override_kernel, dim3((p.bs + 127) / 128), dim3(128), p, s, pdl);
}
cudaError_t launch_pack_gate_up(const __nv_bfloat16* src, __nv_bfloat16* dst, int I, int H, cudaStream_t s) {
  pack_gate_up_kernel<<<2 * I, 128, 0, s>>>(src, dst, I, H);
  return cudaGetLastError();
}

}  // namespace gr

GR_TIMELINE_EXPORTS(rowwise)
