// Non-greedy rounds on sm_100a: the logits processing AR decode applies to every row (penalizers, grammar mask, logit
// bias), AR's target distribution (softmax at the request's temperature, then top-k / top-p / min-p), the speculative
// accept test of each verify row and the draws, and the penalizer cumulation of committed tokens.  There is no
// contraction here: every kernel streams fp32 logits rows (237 KB at the baseline vocabulary) from HBM / L2.
//
// Arithmetic that decides tokens is exact and order-independent: probability mass is summed in 2^-40 fixed point
// (uint64; e = exp(x - max) <= 1, so a row's total stays below 2^56), the keep threshold of the filters is found by a
// four-pass 8-bit radix select over the IEEE bits of e (non-negative floats order like their bits), and draws invert
// the fixed-point CDF in vocabulary order.  Coins come from Philox-4x32-10 keyed by the round's seed.
#include "params.cuh"

namespace gr {

constexpr int kProcChunk = 2048;   // logits_process: vocabulary entries per CTA
constexpr int kProcThreads = 256;
// sample_rows: one CTA per row.  512 threads, two CTAs per SM, when the launch has at least as many rows as SMs (one
// row's barrier waits overlap the other's loads); 1,024 threads, one CTA per SM, below that, where a row's latency
// is the launch's (the a0 and prefill draws of one row per request).
constexpr int kSampThreadsMany = 512;
constexpr int kSampThreadsFew = 1024;
// A warp's bucket words are 32-bit and take under 2^20 + 1 per entry (count 1, mass halves of a weight <= 2^40).
static_assert(32 * ((kSampleMaxVocab + kSampThreadsMany - 1) / kSampThreadsMany) <= 4095, "bucket words could wrap");
// Row loops load kRowBatch entries per thread before using any: a row pass is bound by L2 latency, and one load in
// flight per thread (a dependent load per iteration) left 0.9 ms per 1,088-row launch in long-scoreboard stalls.
// The entries a thread visits, and their order, are unchanged.
constexpr int kRowBatch = 8;

// ---------------------------------------------------------------- Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11)
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}
// uniform in (0, 1]: ((x >> 8) + 1) * 2^-24, exact in fp32
__device__ __forceinline__ float coin(const uint64_t* rng, int b, int j, int kind) {
  const uint64_t seed = rng[0];
  const uint4 x = philox4x32_10(make_uint4(static_cast<uint32_t>(rng[1]), static_cast<uint32_t>(b),
                                           (static_cast<uint32_t>(j) & 0xFFFFFFu) | (static_cast<uint32_t>(kind) << 24), 0u),
                                make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32)));
  return static_cast<float>((x.x >> 8) + 1u) * 5.9604644775390625e-08f;
}

__device__ __forceinline__ uint64_t fixed40(float e) { return __float2ull_rn(e * 1099511627776.0f); }

__device__ __forceinline__ void set_status(int32_t* st, int code) {
  if (st) atomicCAS(st, 0, code);
}

// ---------------------------------------------------------------- logits processing
// Grid (chunks, requests).  Row r = b * K + j sees the request's penalizer state plus the verify ids cand[b, 1..j];
// the ops run in the orchestrator's order with the same IEEE operations as SGLang's penalizers (repetition: l < 0 ?
// l * S : l / S; presence / frequency: l - S; min_new_tokens: stop ids -> -inf), then the grammar mask and the bias.
// A CTA takes one vocabulary chunk of all K rows of a request: the request's penalizer state is read once for its K
// rows (one CTA per row read it K times), and a thread's K logits of an entry are loaded together.
constexpr int kProcMaxK = 128;
__global__ void __launch_bounds__(kProcThreads) logits_process_kernel(const SampleParams p) {
  GR_TL_BEGIN
  __shared__ int cand_s[kProcMaxK];
  __shared__ uint32_t cand_map[kProcChunk / 32];  // bit v - v0: v is one of cand[b, 1..K-1]
  const gr_sampling& s = p.s;
  const int V = s.vocab;
  const int K = p.K;
  const int b = blockIdx.y;
  const int v0 = blockIdx.x * kProcChunk;
  const int v1 = min(V, v0 + kProcChunk);
  for (int i = threadIdx.x; i < kProcChunk / 32; i += blockDim.x) cand_map[i] = 0u;
  for (int i = threadIdx.x; i < K; i += blockDim.x) cand_s[i] = p.cand ? p.cand[(size_t)b * K + i] : -1;
  __syncthreads();
  for (int i = 1 + threadIdx.x; i < K; i += blockDim.x) {
    const int c = cand_s[i];
    if (c >= v0 && c < v1) atomicOr(&cand_map[(c - v0) >> 5], 1u << ((c - v0) & 31));
  }
  __syncthreads();
  const int64_t slot = s.req_pool_idx[b];
  const float rep = s.repetition ? s.repetition[b] : 1.f;
  const float freq = s.frequency ? s.frequency[b] : 0.f;
  const float pres = s.presence ? s.presence[b] : 0.f;
  bool has_stop = false;
  for (int o = 0; o < s.n_order; ++o) has_stop |= s.order[o] == GR_PEN_MIN_NEW_TOKENS;
  const long long stop_len = has_stop ? static_cast<long long>(s.st_len[slot]) : 0;
  const int min_new = has_stop ? s.min_new_tokens[b] : 0;
  const int words = (V + 31) >> 5;
  // the op order, decoded once: each op then runs over 8 rows' values at a time
  int ops[4];
#pragma unroll
  for (int o = 0; o < 4; ++o) ops[o] = o < s.n_order ? s.order[o] : -1;
  const int n_stop = s.n_stop;
  const int* stop_ids = s.stop_ids + (size_t)b * n_stop;
  for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const size_t sv = (size_t)slot * V + v;
    const float srep = (rep != 1.f) ? s.st_rep[sv] : 1.f;
    const float spres = (pres != 0.f) ? s.st_pres[sv] : 0.f;
    const float sfreq = (freq != 0.f) ? s.st_freq[sv] : 0.f;
    const float bias = s.logit_bias ? s.logit_bias[(size_t)b * V + v] : 0.f;
    bool stop_v = false;  // v is one of the request's stop ids
    if (has_stop)
      for (int i = 0; i < n_stop; ++i) stop_v |= stop_ids[i] == v;
    // An entry that no op changes in any row is neither read nor written: never generated (repetition state 1,
    // presence and frequency state 0), not a draft id of the block, no stop mask, and no grammar mask or bias.  The
    // ops are then x * 1, x / 1 and x - 0, which return x exactly.
    const bool is_cand = (cand_map[(v - v0) >> 5] >> ((v - v0) & 31)) & 1u;
    if (!s.allowed && !s.logit_bias && !is_cand && srep == 1.f && spres == 0.f && sfreq == 0.f &&
        !(stop_v && stop_len < min_new))
      continue;
    float* col = p.logits + (size_t)b * K * V + v;  // row j of entry v at col[j * V]
    int c = 0;  // occurrences of v among cand[b, 1..j] for the current row j
    for (int j0 = 0; j0 < K; j0 += 8) {
      float lv[8];
      int cn[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) lv[u] = (j0 + u < K) ? col[(size_t)(j0 + u) * V] : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        if (j >= 1 && j < K && cand_s[j] == v) ++c;
        cn[u] = c;
      }
#pragma unroll
      for (int o = 0; o < 4; ++o) {
        const int op = ops[o];
        if (op == GR_PEN_REPETITION) {
          if (rep != 1.f) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const float S = cn[u] ? rep : srep;
              if (S != 1.f) lv[u] = lv[u] < 0.f ? lv[u] * S : lv[u] / S;  // x * 1 = x / 1 = x exactly
            }
          }
        } else if (op == GR_PEN_PRESENCE) {
          if (pres != 0.f) {
#pragma unroll
            for (int u = 0; u < 8; ++u) lv[u] = lv[u] - (cn[u] ? pres : spres);
          }
        } else if (op == GR_PEN_FREQUENCY) {
          if (freq != 0.f) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              float S = sfreq;
              for (int i = 0; i < cn[u]; ++i) S = S + freq;
              lv[u] = lv[u] - S;
            }
          }
        } else if (op == GR_PEN_MIN_NEW_TOKENS) {
          if (stop_v) {
#pragma unroll
            for (int u = 0; u < 8; ++u)
              if (stop_len + j0 + u < min_new) lv[u] = -INFINITY;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        if (j >= K) break;
        const size_t r = (size_t)b * K + j;
        float l = lv[u];
        if (s.allowed && !((s.allowed[r * words + (v >> 5)] >> (v & 31)) & 1u)) l = -INFINITY;
        if (s.logit_bias) l = l + bias;
        col[(size_t)j * V] = l;
      }
    }
  }
  GR_TL_END(kTlLogitsProcess)
}

// ---------------------------------------------------------------- block reductions (W warps)
template <int W>
__device__ __forceinline__ float block_max(float v, float* sh) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < W ? sh[l] : -INFINITY;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  v = sh[0];
  __syncthreads();
  return v;
}
__device__ __forceinline__ unsigned long long warp_sum64(unsigned long long v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <int W>
__device__ __forceinline__ unsigned long long block_sum64(unsigned long long v, unsigned long long* sh) {
  v = warp_sum64(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < W ? sh[l] : 0ull;
    v = warp_sum64(v);
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  v = sh[0];
  __syncthreads();
  return v;
}

// ---------------------------------------------------------------- keep threshold (radix select)
// Keep set of the filters: {x : #{y > x} < k and sum{y > x} < lim} (strict) or "<= lim" (non-strict), a prefix of the
// descending order.  Returns the smallest bit pattern tau such that "bits(e) >= tau" is exactly that set.  Four passes
// of 8 bits over the row: each warp builds a private histogram of count and fixed-point mass per bucket with 32-bit
// shared atomics (contention stays inside one warp even when a flat distribution puts every entry in one bucket), the
// warps' histograms are summed per bucket, and warp 0 scans the 256 buckets from the top.
// Once the bucket a level picked holds at most kCompactCap entries, the next level's pass over the row also copies
// those entries' bits into shared memory, and the levels after it read only that copy.
constexpr int kCompactCap = 4096;
template <int W>
struct SelectSmem {
  uint32_t wc[W][256];  // per-warp counts
  uint32_t wl[W][256];  // per-warp mass, low 20 bits of each entry's fixed-point value
  uint32_t wh[W][256];  // per-warp mass, the high bits (<= 2^20 per entry, at most 4,095 entries a warp)
  uint32_t hc[256];
  unsigned long long hs[256];
  uint32_t comp[kCompactCap];    // bits of the entries in the picked bucket (any order)
  uint32_t prefix, tau, done;
  uint32_t n_comp;               // entries copied to comp
  uint32_t c_bucket;             // entries in the bucket the last level picked
  unsigned long long c_above, s_above;
};
// One pass of the select: every positive entry whose higher bits equal `prefix` adds its count and fixed-point mass to
// bucket (bits >> shift) & 255 of this warp's histogram.  AGG keeps two buckets' sums in registers and adds them to the
// histogram only when a third bucket shows up or the pass ends.  On a flat row the first pass puts most entries in one
// or two buckets of the exponent, and every lane's atomic on the same word serialised; on a peaked row the entries
// spread over many buckets and the register cache only adds divergent branches.  The sums are integers, so both
// forms build the same histogram.
// comp (when given): every counted entry's bits are also appended there, n_comp counting them; the caller guarantees
// room (the count of the bucket this pass filters on is known from the previous level).  A warp's lanes run the same
// iterations, so the appends take one ballot and one shared atomic per warp.
template <bool AGG>
__device__ __forceinline__ void histogram_pass(const float* row, int V, int level, uint32_t prefix, bool need_c,
                                               bool need_m, uint32_t* wc, uint32_t* wl, uint32_t* wh,
                                               uint32_t* comp = nullptr, uint32_t* n_comp = nullptr) {
  const int lane = threadIdx.x & 31;
  const int shift = 24 - 8 * level;
  uint32_t bin_a = 0xFFFFFFFFu, bin_b = 0xFFFFFFFFu, cnt_a = 0, cnt_b = 0;
  uint64_t mass_a = 0, mass_b = 0;
  auto add = [&](uint32_t bin, uint32_t cnt, uint64_t mass) {
    if (cnt == 0) return;
    if (need_c) atomicAdd(&wc[bin], cnt);
    if (need_m) {  // two 32-bit halves: 64-bit shared atomics measured slower
      atomicAdd(&wl[bin], static_cast<uint32_t>(mass & 0xFFFFFu));
      atomicAdd(&wh[bin], static_cast<uint32_t>(mass >> 20));
    }
  };
  for (int w0 = threadIdx.x - lane; w0 < V; w0 += kRowBatch * blockDim.x) {  // uniform across the warp
    const int v0 = w0 + lane;
    float ev[kRowBatch];
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) {
      const int v = v0 + u * blockDim.x;
      ev[u] = v < V ? row[v] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) {
      const float e = ev[u];
      const uint32_t ub = __float_as_uint(e);
      const bool counted = e > 0.f && (level == 0 || (ub >> (shift + 8)) == prefix);
      if (comp) {
        const unsigned bal = __ballot_sync(0xffffffffu, counted);
        if (bal) {
          uint32_t base = 0;
          if (lane == 0) base = atomicAdd(n_comp, static_cast<uint32_t>(__popc(bal)));
          base = __shfl_sync(0xffffffffu, base, 0);
          const uint32_t at = base + static_cast<uint32_t>(__popc(bal & ((1u << lane) - 1u)));
          if (counted && at < kCompactCap) comp[at] = ub;
        }
      }
      if (counted) {
        const uint32_t bin = (ub >> shift) & 255u;
        const uint64_t w = need_m ? fixed40(e) : 0ull;
        if (!AGG) {
          add(bin, 1u, w);
        } else if (bin == bin_a) {
          ++cnt_a;
          mass_a += w;
        } else if (bin == bin_b) {
          ++cnt_b;
          mass_b += w;
        } else {
          add(bin_b, cnt_b, mass_b);
          bin_b = bin_a;
          cnt_b = cnt_a;
          mass_b = mass_a;
          bin_a = bin;
          cnt_a = 1;
          mass_a = w;
        }
      }
    }
  }
  if (AGG) {
    add(bin_a, cnt_a, mass_a);
    add(bin_b, cnt_b, mass_b);
  }
}

template <int W>
__device__ uint32_t select_threshold(const float* row, int V, long long k, double lim, bool strict, bool flat,
                                     SelectSmem<W>& sm) {
  // Counts are always taken (an off count criterion has k = 2^62): the picked bucket's count decides the copy.
  // The mass histogram is skipped when top-p is off.
  const bool need_m = lim < 1e300;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    sm.prefix = 0;
    sm.tau = 0;
    sm.done = 0;
    sm.c_above = 0;
    sm.s_above = 0;
    sm.n_comp = 0;
    sm.c_bucket = 0xFFFFFFFFu;
  }
  __syncthreads();
  const float* src = row;  // the row, or the shared copy of the picked bucket's entries once made
  int n_src = V;
  bool from_copy = false;
  for (int level = 0; level < 4; ++level) {
    const int shift = 24 - 8 * level;
    for (int i = lane; i < 256; i += 32) {
      sm.wc[warp][i] = 0;
      sm.wl[warp][i] = 0;
      sm.wh[warp][i] = 0;
    }
    __syncwarp();
    const uint32_t prefix = sm.prefix;
    const bool copy =
        !from_copy && (level == 1 || level == 2) && sm.c_bucket <= static_cast<uint32_t>(kCompactCap);
    if (flat && level == 0)
      histogram_pass<true>(row, V, 0, prefix, true, need_m, sm.wc[warp], sm.wl[warp], sm.wh[warp]);
    else
      histogram_pass<false>(src, n_src, level, prefix, true, need_m, sm.wc[warp], sm.wl[warp], sm.wh[warp],
                            copy ? sm.comp : nullptr, &sm.n_comp);
    __syncthreads();
    if (copy) {
      src = reinterpret_cast<const float*>(sm.comp);
      n_src = static_cast<int>(min(sm.n_comp, static_cast<uint32_t>(kCompactCap)));
      from_copy = true;
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      uint32_t c = 0;
      unsigned long long lo = 0, hi = 0;
#pragma unroll 8
      for (int q = 0; q < W; ++q) {
        c += sm.wc[q][i];
        lo += sm.wl[q][i];
        hi += sm.wh[q][i];
      }
      sm.hc[i] = c;
      sm.hs[i] = (hi << 20) + lo;
    }
    __syncthreads();
    if (warp == 0) {
      // lane t holds buckets 255 - 8t .. 248 - 8t (descending); inclusive scans from the top
      uint32_t c[8];
      unsigned long long sm8[8];
      uint32_t ct = 0;
      unsigned long long st = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = 255 - 8 * lane - i;
        ct += sm.hc[d];
        st += sm.hs[d];
        c[i] = ct;
        sm8[i] = st;
      }
      uint32_t cx = ct;
      unsigned long long sx = st;
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t cy = __shfl_up_sync(0xffffffffu, cx, o);
        const unsigned long long sy = __shfl_up_sync(0xffffffffu, sx, o);
        if (lane >= o) {
          cx += cy;
          sx += sy;
        }
      }
      const uint32_t c_before = cx - ct;            // buckets above this lane's eight
      const unsigned long long s_before = sx - st;
      const unsigned long long CA = sm.c_above, SA = sm.s_above;
      // first bucket (from the top) whose inclusion breaks the criterion for the entries below it
      int fail = -1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const long long cc = static_cast<long long>(CA + c_before + c[i]);
        const double ss = static_cast<double>(SA + s_before + sm8[i]);
        const bool ok = cc < k && (strict ? ss < lim : ss <= lim);
        if (!ok && fail < 0) fail = i;
      }
      const unsigned ball = __ballot_sync(0xffffffffu, fail >= 0);
      if (ball == 0u) {
        // every bucket of this level is kept entirely: the set reaches below the prefix range
        if (lane == 0) {
          sm.tau = level == 0 ? 0u : (prefix << (shift + 8));
          sm.done = 1;
        }
      } else {
        const int src = __ffs(ball) - 1;
        if (lane == src) {
          const int d = 255 - 8 * lane - fail;
          const uint32_t c_ex = c_before + (fail ? c[fail - 1] : 0u);
          const unsigned long long s_ex = s_before + (fail ? sm8[fail - 1] : 0ull);
          const unsigned long long c_top = CA + c_ex, s_top = SA + s_ex;
          const bool top_kept = static_cast<long long>(c_top) < k &&
                                (strict ? static_cast<double>(s_top) < lim : static_cast<double>(s_top) <= lim);
          const uint32_t here = (prefix << 8) | static_cast<uint32_t>(d);
          if (!top_kept) {
            // nothing of bucket d is kept: the set ends just above it
            sm.tau = (here + 1u) << shift;
            sm.done = 1;
          } else if (level == 3) {
            sm.tau = here;  // one value (tied entries): kept together
            sm.done = 1;
          } else {
            sm.prefix = here;
            sm.c_above = c_top;
            sm.s_above = s_top;
            sm.c_bucket = sm.hc[d];
            sm.n_comp = 0;
          }
        }
      }
    }
    __syncthreads();
    if (sm.done) break;
  }
  const uint32_t t = sm.tau;
  __syncthreads();
  return t;
}

// ---------------------------------------------------------------- target distribution, accept test, draws
template <int NT>
__global__ void __launch_bounds__(NT, NT == kSampThreadsMany ? 2 : 1) sample_rows_kernel(const SampleParams p) {
  constexpr int NW = NT / 32;  // warps
  GR_TL_BEGIN
  __shared__ float shf[NW];
  __shared__ unsigned long long shu[NW];
  extern __shared__ __align__(16) uint8_t dyn_smem[];
  SelectSmem<NW>& sel = *reinterpret_cast<SelectSmem<NW>*>(dyn_smem);
  __shared__ unsigned long long scan[NW];
  __shared__ int found;
  const gr_sampling& s = p.s;
  const int V = s.vocab;
  const int r = blockIdx.x;
  const int b = r / p.K, j = r % p.K;
  float* row = p.logits + (size_t)r * V;
  const float T = s.temperature[b];
  const long long k = s.top_k[b];
  const float P = s.top_p[b];
  const float mp = s.min_p[b];
  // pass 1: the maximum of x = l / T.  Rounding a division by T > 0 is monotone, so max(l / T) = max(l) / T exactly:
  // the pass takes the logits' maximum and divides once.
  float mx = -INFINITY;
  for (int v0 = threadIdx.x; v0 < V; v0 += kRowBatch * blockDim.x) {
    float lv[kRowBatch];
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) {
      const int v = v0 + u * blockDim.x;
      lv[u] = v < V ? row[v] : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) mx = fmaxf(mx, lv[u]);
  }
  const float m = block_max<NW>(mx, shf) / T;
  const int d = (p.K > 1 && j + 1 < p.K) ? p.cand[(size_t)b * p.K + j + 1] : -1;
  if (!(m > -INFINITY)) {  // every token masked
    if (threadIdx.x == 0) {
      set_status(p.status, GR_ERR_NO_TOKEN);
      p.sample[r] = 0;
      if (p.accept) p.accept[r] = 0;
      if (p.p_next) p.p_next[r] = 0.f;
      if (p.first_out) p.first_out[(size_t)b * p.first_stride] = 0;
    }
    return;
  }
  // pass 2: x = l / T, e = exp(x - max) (the maximum maps to exactly 1) and the fixed-point total
  uint64_t z = 0;
  for (int v0 = threadIdx.x; v0 < V; v0 += kRowBatch * blockDim.x) {
    float lv[kRowBatch];
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) {
      const int v = v0 + u * blockDim.x;
      lv[u] = v < V ? row[v] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) {
      const int v = v0 + u * blockDim.x;
      if (v < V) {
        const float e = expf(lv[u] / T - m);
        row[v] = e;
        z += fixed40(e);
      }
    }
  }
  const uint64_t Z = block_sum64<NW>(z, shu);
  // a mean weight of at least 1/32 (the maximum is 1) marks a flat row, whose first select pass aggregates in registers
  const bool flat = Z >= (static_cast<uint64_t>(V) << 35);
  // keep threshold of the filters
  uint32_t tau = 0;
  const bool want_k = k < V, want_p = P < 1.f;
  if (k <= 1) {
    tau = __float_as_uint(1.0f);  // the maximum's tie group
  } else if (s.filter == GR_FILTER_JOINT) {
    if (want_k || want_p)
      tau = select_threshold(row, V, want_k ? k : (1ll << 62), want_p ? static_cast<double>(P) * Z : 1e300, true, flat,
                             sel);
  } else if (s.filter == GR_FILTER_TORCH) {
    if (want_k || want_p)
      tau = select_threshold(row, V, want_k ? k : (1ll << 62), want_p ? static_cast<double>(P) * Z : 1e300, false, flat,
                             sel);
    if (mp > 0.f) tau = max(tau, __float_as_uint(mp));
  } else {  // sequential: top-k renorm, then top-p on the renormalised mass, then min-p
    uint32_t t1 = 0;
    if (want_k) t1 = select_threshold(row, V, k, 1e300, true, flat, sel);
    if (want_p) {
      uint64_t zk = 0;
      for (int v0 = threadIdx.x; v0 < V; v0 += kRowBatch * blockDim.x) {
        float ev[kRowBatch];
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) {
          const int v = v0 + u * blockDim.x;
          ev[u] = v < V ? row[v] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u)
          if (__float_as_uint(ev[u]) >= t1 && ev[u] > 0.f) zk += fixed40(ev[u]);
      }
      const uint64_t Zk = block_sum64<NW>(zk, shu);
      const uint32_t t2 = select_threshold(row, V, 1ll << 62, static_cast<double>(P) * Zk, true, flat, sel);
      t1 = max(t1, t2);
    }
    tau = t1;
    if (mp > 0.f) tau = max(tau, __float_as_uint(mp));
  }
  // draw pass: warp w owns the contiguous vocabulary segment [w * seg, (w + 1) * seg), read 32 entries at a time
  // (coalesced); the block scans the warps' kept mass in vocabulary order, and the warp holding the target walks its
  // segment again with a warp-wide inclusive scan per 32 entries
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = ((V + NW - 1) / NW + 31) & ~31;
  const int lo = warp * seg, hi = min(V, lo + seg);
  auto kept_w = [&](int v) -> uint64_t {
    const float e = row[v];
    return (e > 0.f && __float_as_uint(e) >= tau) ? fixed40(e) : 0ull;
  };
  auto kept_e = [&](float e) -> uint64_t { return (e > 0.f && __float_as_uint(e) >= tau) ? fixed40(e) : 0ull; };
  unsigned long long loc = 0;
  for (int v0 = lo + lane; v0 < hi; v0 += 32 * kRowBatch) {
    float ev[kRowBatch];
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) {
      const int v = v0 + 32 * u;
      ev[u] = v < hi ? row[v] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kRowBatch; ++u) loc += kept_e(ev[u]);
  }
  loc = warp_sum64(loc);
  const uint64_t wd = (d >= 0) ? kept_w(d) : 0ull;  // the same value every thread reads
  if (lane == 0) scan[warp] = loc;
  if (threadIdx.x == 0) found = -1;
  __syncthreads();
  uint64_t W = 0, before = 0;
  for (int i = 0; i < NW; ++i) {
    if (i == warp) before = W;
    W += scan[i];
  }
  const bool exclude = d >= 0;
  const uint64_t mine = loc - ((exclude && d >= lo && d < hi) ? wd : 0ull);
  const uint64_t before_x = before - ((exclude && d < lo) ? wd : 0ull);
  const uint64_t Wx = W - (exclude ? wd : 0ull);
  const float cf = p.K == 1 ? coin(s.rng, b, 0, p.first_kind) : coin(s.rng, b, 0, GR_COIN_FINAL);
  uint64_t target = static_cast<uint64_t>(static_cast<double>(cf) * static_cast<double>(Wx));
  if (Wx > 0 && target >= Wx) target = Wx - 1;
  if (Wx > 0 && mine > 0 && target >= before_x && target < before_x + mine) {
    uint64_t c = before_x;
    bool hit_any = false;
    for (int g0 = lo; g0 < hi && !hit_any; g0 += 32 * kRowBatch) {
      float ev[kRowBatch];  // kRowBatch groups of 32 entries loaded together, then scanned in order
#pragma unroll
      for (int u = 0; u < kRowBatch; ++u) {
        const int v = g0 + 32 * u + lane;
        ev[u] = v < hi ? row[v] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kRowBatch; ++u) {
        const int v = g0 + 32 * u + lane;
        if (g0 + 32 * u >= hi) break;
        uint64_t x = (v < hi && v != (exclude ? d : -1)) ? kept_e(ev[u]) : 0ull;
        for (int o = 1; o < 32; o <<= 1) {
          const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
          if (lane >= o) x += y;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, c + x > target);
        if (hit) {
          if (lane == __ffs(hit) - 1) found = v;
          hit_any = true;
          break;
        }
        c += __shfl_sync(0xffffffffu, x, 31);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int smp = found;
    if (smp < 0) smp = d >= 0 ? d : 0;  // no mass outside d (d held everything kept): never used, d is accepted
    p.sample[r] = smp;
    if (p.first_out) p.first_out[(size_t)b * p.first_stride] = smp;
    if (p.K > 1) {
      const float ca = coin(s.rng, b, j, GR_COIN_ACCEPT);
      const bool acc = d >= 0 && W > 0 && static_cast<double>(ca) * static_cast<double>(W) <= static_cast<double>(wd);
      p.accept[r] = acc ? 1 : 0;
    }
    if (p.p_next) p.p_next[r] = (d >= 0 && W > 0) ? static_cast<float>(static_cast<double>(wd) / static_cast<double>(W)) : 0.f;
  }
  GR_TL_END(kTlSampleRows)
}

// ---------------------------------------------------------------- penalizer cumulation
__global__ void penalty_cumulate_kernel(const SampleParams p) {
  GR_TL_BEGIN
  const gr_sampling& s = p.s;
  const int b = blockIdx.x;
  const int n = (p.counts ? p.counts[b] : 0) + p.add;
  const int64_t slot = s.req_pool_idx[b];
  const int V = s.vocab;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int t = p.tokens[(size_t)b * p.tok_stride + i];
    if (t < 0 || t >= V) continue;
    const size_t sv = (size_t)slot * V + t;
    for (int o = 0; o < s.n_order; ++o) {
      const int op = s.order[o];
      if (op == GR_PEN_REPETITION) s.st_rep[sv] = s.repetition[b];
      else if (op == GR_PEN_PRESENCE) s.st_pres[sv] = s.presence[b];
      else if (op == GR_PEN_FREQUENCY) atomicAdd(&s.st_freq[sv], s.frequency[b]);  // one addend value: order-free
    }
  }
  if (threadIdx.x == 0 && s.st_len) s.st_len[slot] += n;
  GR_TL_END(kTlPenaltyCumulate)
}

__global__ void gather_rows_kernel(const uint4* src, int words, int stride_rows, uint4* dst) {
  const int i = blockIdx.x;
  for (int w = threadIdx.x; w < words; w += blockDim.x)
    dst[(size_t)i * words + w] = src[(size_t)i * stride_rows * words + w];
}

// ---------------------------------------------------------------- launchers
cudaError_t launch_gather_rows(const void* src, int row_bytes, int n, int src_stride_rows, void* dst, cudaStream_t s) {
  gather_rows_kernel<<<n, 128, 0, s>>>(static_cast<const uint4*>(src), row_bytes / 16, src_stride_rows,
                                       static_cast<uint4*>(dst));
  return cudaGetLastError();
}
cudaError_t launch_logits_process(const SampleParams& p, cudaStream_t s) {
  if (p.K > kProcMaxK) return cudaErrorInvalidValue;
  const dim3 grid((p.s.vocab + kProcChunk - 1) / kProcChunk, p.bs);
  logits_process_kernel<<<grid, kProcThreads, 0, s>>>(p);
  return cudaGetLastError();
}
template <int NT>
static cudaError_t launch_sample_rows_t(const SampleParams& p, cudaStream_t s) {
  using Smem = SelectSmem<NT / 32>;
  static PerDeviceOnce configured;
  cudaError_t e = once_per_device(configured, [] {
    return cudaFuncSetAttribute(sample_rows_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(sizeof(Smem)));
  });
  if (e != cudaSuccess) return e;
  sample_rows_kernel<NT><<<p.bs * p.K, NT, sizeof(Smem), s>>>(p);
  return cudaGetLastError();
}
cudaError_t launch_sample_rows(const SampleParams& p, cudaStream_t s) {
  return p.bs * p.K < p.sms ? launch_sample_rows_t<kSampThreadsFew>(p, s)
                             : launch_sample_rows_t<kSampThreadsMany>(p, s);
}
cudaError_t launch_penalty_cumulate(const SampleParams& p, cudaStream_t s) {
  penalty_cumulate_kernel<<<p.bs, 64, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace gr

GR_TIMELINE_EXPORTS(sampling)
