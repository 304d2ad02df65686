// extern "C" entry points of libgravity_b200.so (declared in include/gravity_b200.h): argument checks, tile and
// split heuristics, TMA tensor-map encoding (cached per buffer) and the launches.
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "params.cuh"

namespace gr {

// ------------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

using MapKey = std::tuple<uintptr_t, uint64_t, uint64_t, uint32_t, uint32_t>;
static std::mutex g_map_mu;
static std::map<MapKey, CUtensorMap> g_maps;

// 2-D bf16 tensor [rows, cols] (cols contiguous, row stride = cols), box [box_rows, box_cols], 128-byte swizzle.
static int tensor_map_2d(const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows, uint32_t box_cols,
                         CUtensorMap* out) {
  const MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, box_rows, box_cols};
  {
    std::lock_guard<std::mutex> g(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return GR_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return GR_ERR_TMA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((cols * 2) & 15)) return GR_ERR_ARG;
  CUtensorMap m;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return GR_ERR_TMA;
  std::lock_guard<std::mutex> g(g_map_mu);
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps[key] = m;
  *out = m;
  return GR_OK;
}

static bool g_pdl = true;
static std::mutex g_sms_mu;
static int g_sms[kMaxDevices] = {};

// SM count of the current device (the persistent grids and split heuristics are sized by it); 148 without a device.
static int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return 148;
  }
  std::lock_guard<std::mutex> g(g_sms_mu);
  if (!g_sms[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return 148;
    }
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

struct LinearShape {
  int nt, m_tiles, n_tiles, kc;
  bool tail_last;  // a shorter last token tile's units run after all full tiles' (snake assignment)
};
static int round16(int x) { return ((x + 15) / 16) * 16; }

static int acc_cols_for(int nt) { return nt <= 32 ? 32 : (nt <= 64 ? 64 : (nt <= 128 ? 128 : 256)); }

// Pipeline depth and resident CTAs of the persistent projection kernel for a token tile of nt rows.
static void linear_launch_shape(int nt, int kc, int epi, int* stages, int* ctas_per_sm) {
  const size_t cap = 220 * 1024;
  int st = GR_MAX_STAGES;
  while (st > 2 && linear_smem_bytes(nt, st, epi) > cap) --st;
  if (st > kc) st = kc < 2 ? 2 : kc;
  while (st > 1 && linear_smem_bytes(nt, st, epi) > cap) --st;
  const int by_smem = static_cast<int>(233472 / (linear_smem_bytes(nt, st, epi) + 1024));
  const int by_tmem = 512 / (2 * acc_cols_for(nt));
  *stages = st;
  *ctas_per_sm = by_smem < by_tmem ? (by_smem < 1 ? 1 : by_smem) : by_tmem;
}

// Candidate token tilings of m rows, widest tile first within each kind:
//  * balanced: mt tiles of round16(m / mt) rows, from the fewest tiles whose tile fits one MMA (nt <= GR_MAX_NT) up
//    to 4x that; tiles narrower than 128 tokens only where the rows need no more (small batches stream weights: a
//    second token tile would read every weight tile twice);
//  * ragged: tiles of nt >= 128 rows and a shorter last tile, whose units run at MMA N = its rows.
// At most kMaxTiles (feature tile, token tile) pairs.  Calls f(m_tiles, nt) for each.
constexpr size_t kMaxTiles = 16384;  // feature tiles x token tiles of one call (lm_head at 8192 rows)
template <class F>
static void for_token_tilings(int m, int n_tiles, F f) {
  const int min_tiles = (m + GR_MAX_NT - 1) / GR_MAX_NT;
  int bal_nt[4 * 64 + 8];
  int n_bal = 0;
  for (int mt = min_tiles; mt <= min_tiles * 4 && mt <= m; ++mt) {
    int nt = round16((m + mt - 1) / mt);
    if (mt > min_tiles && nt < 128) break;
    if (nt < 16) nt = 16;
    if (static_cast<size_t>(mt) * n_tiles > kMaxTiles) continue;
    if (n_bal < static_cast<int>(sizeof(bal_nt) / sizeof(int))) bal_nt[n_bal++] = mt * 1024 + nt;
    f(mt, nt);
  }
  for (int nt = GR_MAX_NT; nt >= 128; nt -= 16) {
    const int mt = (m + nt - 1) / nt;
    if (mt == 1 || mt > 4 * min_tiles || static_cast<size_t>(mt) * n_tiles > kMaxTiles) continue;
    bool seen = false;
    for (int i = 0; i < n_bal; ++i) seen |= bal_nt[i] == mt * 1024 + nt;
    if (!seen) f(mt, nt);
  }
}

// Whether a call may number a shorter last token tile's units after all full tiles': only where the weights stay in
// L2 (otherwise that tile's pass would stream every weight tile from DRAM a second time).
static bool tail_last_allowed(int n_out, int k_in) {
  return static_cast<size_t>(n_out) * k_in * 2 <= (48u << 20);
}

// Output bytes per (row, feature) of an epilogue, for the cost model.
static int epi_out_bytes(int epi) {
  switch (epi) {
    case GR_EPI_STORE_F32: case GR_EPI_PARTIAL_F32: return 4;
    case GR_EPI_SWIGLU: return 1;
    default: return 2;
  }
}

// Critical path of the persistent schedule, in shared-memory cycles (~128 bytes each), as the kernel walks it: CTA c
// takes unit k * grid + c in wave k (with tail_last: grid - 1 - c in odd waves, and the short tile's units last).
// A unit costs a fixed kUnitCost (pipeline turn-around, accumulator hand-off) plus its main loop, (K chunks) x
// (128 + N) -- the 128-row weight tile and the N-row token tile both pass through shared memory, N = nt or the
// rounded rows of a shorter last tile; its epilogue the bytes it stores at ~64 bytes per cycle, plus, for a
// split-K unit that finishes its tile, its own fp32 partial and the reads of all splits' partials.  An epilogue
// overlaps the CTA's next main loop (double-buffered accumulators); the last one does not.  The maximum over CTAs.
// kUnitCost and the epilogue rate were fitted to B200 timings of the decoder's projections at 17-4,224 rows.
constexpr long long kUnitCost = 1024;
static long long schedule_cost(int n_tiles, int mt, int nt, int m, int sp, int kc, long long cap, int epi,
                               bool tail_last) {
  const int full_m = (m % nt == 0) ? mt : mt - 1;
  const long long full_units = static_cast<long long>(full_m) * sp * n_tiles;
  const long long units = static_cast<long long>(mt) * sp * n_tiles;
  const int last_rows = m - (mt - 1) * nt;
  const bool split_epi = sp > 1 && epi != GR_EPI_PARTIAL_F32;
  auto main_cost = [&](bool last) {
    return kUnitCost + static_cast<long long>(kc) * (128 + (last ? round16(last_rows) : nt));
  };
  auto epi_cost = [&](bool last) {
    const long long rows = last ? last_rows : nt;
    long long c = rows * 128 * epi_out_bytes(epi) / 64;
    if (split_epi) c += rows * 128 * 4 * (1 + sp) / 64;
    return c;
  };
  const long long G = units < cap ? units : cap;
  const long long waves = (units + G - 1) / G;
  long long worst = 0;
  for (long long c = 0; c < G; ++c) {
    long long t = 0, prev_epi = 0;
    for (long long w = 0; w < waves; ++w) {
      const long long u = w * G + ((tail_last && (w & 1)) ? G - 1 - c : c);
      if (u >= units) continue;
      const bool last = tail_last ? u >= full_units : (full_m < mt && u % mt == mt - 1);
      const long long mc = main_cost(last);
      t += mc > prev_epi ? mc : prev_epi;
      prev_epi = epi_cost(last);
    }
    t += prev_epi;
    if (t > worst) worst = t;
  }
  return worst;
}

// Token tiling for a split-K count `sp`: the candidate with the shortest critical path (ties: the first candidate).
// Memoised per shape: the schedule walk is O(units).  The cost goes to *cost_out.
static LinearShape linear_shape(int n_out, int k_in, int m, int sp = 1, int epi = GR_EPI_STORE_F32,
                                long long* cost_out = nullptr) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int>, std::pair<LinearShape, long long>> memo;
  const auto key = std::make_tuple(n_out, k_in, m, sp, epi, num_sms());
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = memo.find(key);
    if (it != memo.end()) {
      if (cost_out) *cost_out = it->second.second;
      return it->second.first;
    }
  }
  LinearShape s;
  s.n_tiles = n_out / 128;
  s.kc = k_in / 64;
  s.m_tiles = 1;
  s.nt = round16(m < GR_MAX_NT ? m : GR_MAX_NT);
  s.tail_last = false;
  const int kc = s.kc / sp;
  const bool tail_ok = tail_last_allowed(n_out, k_in);
  long long best = -1;
  for_token_tilings(m, s.n_tiles, [&](int mt, int nt) {
    // resident CTAs as for the full K depth (the deep ring): shallow split rings admit more CTAs per SM, which the
    // measurements do not reward
    int stages, per_sm;
    linear_launch_shape(nt, s.kc, epi, &stages, &per_sm);
    const long long cap = static_cast<long long>(num_sms()) * per_sm;
    long long cost = schedule_cost(s.n_tiles, mt, nt, m, sp, kc, cap, epi, false);
    bool tl = false;
    if (tail_ok && m % nt) {  // the short tile last, only where that shortens the critical path
      const long long c2 = schedule_cost(s.n_tiles, mt, nt, m, sp, kc, cap, epi, true);
      if (c2 < cost) {
        cost = c2;
        tl = true;
      }
    }
    if (best < 0 || cost < best) {
      best = cost;
      s.m_tiles = mt;
      s.nt = nt;
      s.tail_last = tl;
    }
  });
  {
    std::lock_guard<std::mutex> g(mu);
    memo.emplace(key, std::make_pair(s, best));
  }
  if (cost_out) *cost_out = best;
  return s;
}

// Split-K count, chosen together with the token tiling: the cost above minimised over the split counts that divide
// the K chunks (at most half of them) and whose fp32 partials stay a small, L2-resident fraction of the traffic;
// ties go to fewer splits (less partial traffic).  The argmax epilogue runs unsplit.
// Split-K count, chosen together with the token tiling: the cost above minimised over the split counts that divide
// the K chunks (at most half of them) and whose fp32 partials stay a small, L2-resident fraction of the traffic;
// ties go to fewer splits (less partial traffic).  The argmax epilogue runs unsplit.
static int default_splits(int n_out, int k_in, int m, int epi) {
  if (epi == GR_EPI_ARGMAX) return 1;
  const int kc = k_in / 64;
  long long best_cost = -1;
  int best = 1;
  for (int sp = 1; sp <= (kc / 2 > 1 ? kc / 2 : 1); ++sp) {
    if (kc % sp) continue;
    if (sp > 1 && static_cast<double>(sp) * m * (n_out / 128) * 128 * 4 > 32.0 * (1 << 20)) break;
    long long cost = 0;
    linear_shape(n_out, k_in, m, sp, epi, &cost);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

struct LinearWs {
  int* ticket;
  float* partial;
  float4* arg;
  size_t bytes;
};
static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
// Every call shares one scratch buffer, whatever its shape: the tickets live in a fixed region at its head (so a
// later call of another shape never finds another call's partial sums where its tickets are), then the fp32
// split-K partials, then the per-(token, feature tile) argmax records.
constexpr size_t kTicketBytes = kMaxTiles * sizeof(int);
static LinearWs linear_ws_layout(void* base, const LinearShape& s, int m, int splits) {
  LinearWs w;
  uint8_t* p = static_cast<uint8_t*>(base);
  const size_t tiles = static_cast<size_t>(s.n_tiles) * s.m_tiles;
  w.ticket = reinterpret_cast<int*>(p);
  size_t off = kTicketBytes;
  w.partial = reinterpret_cast<float*>(p + off);
  off += splits > 1 ? align256(tiles * splits * s.nt * 128 * sizeof(float)) : 0;
  w.arg = reinterpret_cast<float4*>(p + off);
  off += align256(static_cast<size_t>(s.n_tiles) * m * sizeof(float4));
  w.bytes = off;
  return w;
}

// attention scratch: tickets of (request, kv head) at the head, then the split partials
constexpr size_t kAttnTicketBytes = 65536;  // 16384 (request, kv head) pairs

}  // namespace gr

using namespace gr;

extern "C" {

int gr_version(void) { return 100; }

const char* gr_status_string(int code) {
  switch (code) {
    case GR_OK: return "ok";
    case GR_ERR_ARG: return "invalid argument";
    case GR_ERR_CUDA: return "CUDA runtime error";
    case GR_ERR_TMA: return "tensor map encoding failed";
    case GR_ERR_TIMEOUT: return "device wait timed out";
    case GR_ERR_BAD_ID: return "token id out of range";
    case GR_ERR_BAD_PAGE: return "position beyond page-table capacity";
    case GR_ERR_UNSUPPORTED: return "unsupported configuration";
    case GR_ERR_SCRATCH_LIMIT: return "needs more scratch than the 8 MiB no-alloc array (use gr_bd_attention with a workspace)";
    case GR_ERR_NO_TOKEN: return "a sampled row allowed no token";
    default: return "unknown status";
  }
}

void gr_set_pdl(int enable) { g_pdl = enable != 0; }
void gr_set_attention_tc(int mode) { g_attention_tc = mode < 0 ? 0 : (mode > 2 ? 2 : mode); }
int gr_num_sms(void) { return num_sms(); }

int gr_linear_default_splits(int n_out, int k_in, int m, int mode) {
  if (mode < GR_EPI_STORE_F32 || mode > GR_EPI_PARTIAL_F32) return 0;
  if (n_out <= 0 || (n_out % 128) || k_in <= 0 || (k_in % 64) || m <= 0) return 1;
  return default_splits(n_out, k_in, m, mode);
}

int gr_linear_plan(int n_out, int k_in, int m, int mode, int splits, int32_t* out) {
  if (!out || mode < GR_EPI_STORE_F32 || mode > GR_EPI_PARTIAL_F32 || n_out <= 0 || (n_out % 128) || k_in <= 0 ||
      (k_in % 64) || m <= 0)
    return GR_ERR_ARG;
  if (splits <= 0) splits = default_splits(n_out, k_in, m, mode);
  if ((k_in / 64) % splits) return GR_ERR_ARG;
  const LinearShape s = linear_shape(n_out, k_in, m, splits, mode);
  int stages, per_sm;
  linear_launch_shape(s.nt, s.kc / splits, mode, &stages, &per_sm);
  const long long units = static_cast<long long>(s.n_tiles) * s.m_tiles * splits;
  const long long cap = static_cast<long long>(num_sms()) * per_sm;
  out[0] = splits;
  out[1] = s.nt;
  out[2] = s.m_tiles;
  out[3] = s.tail_last ? 1 : 0;
  out[4] = static_cast<int32_t>(units < cap ? units : cap);
  return GR_OK;
}

size_t gr_linear_workspace_bytes(int n_out, int m, int splits) {
  if (n_out <= 0 || m <= 0) return 0;
  if (splits < 1) splits = 1;
  // the largest layout over every token tiling a call of this shape may use (the tiling also depends on K)
  size_t bytes = 0;
  for_token_tilings(m, n_out / 128, [&](int mt, int nt) {
    LinearShape s;
    s.n_tiles = n_out / 128;
    s.kc = 1;
    s.m_tiles = mt;
    s.nt = nt;
    const size_t b = linear_ws_layout(nullptr, s, m, splits).bytes;
    if (b > bytes) bytes = b;
  });
  return bytes;
}

// Checks, tiling, tensor maps and kernel parameters of one projection.
struct LinearLaunch {
  LinearParams p;
  CUtensorMap tmw, tmx;
  int grid, stages;
  size_t smem;
};
static int build_linear(const void* w, int n_out, int k_in, const void* x, int m, const gr_epilogue* epi, int splits,
                        void* workspace, size_t workspace_bytes, const void* prefetch, size_t prefetch_bytes,
                        int32_t* status, LinearLaunch* out) {
  if (!w || !x || !epi || m <= 0 || n_out <= 0 || (n_out % 128) || k_in <= 0 || (k_in % 64)) return GR_ERR_ARG;
  if (epi->mode < GR_EPI_STORE_F32 || epi->mode > GR_EPI_PARTIAL_F32) return GR_ERR_ARG;
  if (splits <= 0) splits = default_splits(n_out, k_in, m, epi->mode);
  if ((k_in / 64) % splits) return GR_ERR_ARG;
  LinearShape s = linear_shape(n_out, k_in, m, splits, epi->mode);
  const size_t ws_splits = epi->mode == GR_EPI_PARTIAL_F32 ? 1 : static_cast<size_t>(splits);
  const int kc = s.kc / splits;
  LinearWs ws = linear_ws_layout(workspace, s, m, static_cast<int>(ws_splits));
  if (!workspace || workspace_bytes < ws.bytes) return GR_ERR_ARG;
  if (static_cast<size_t>(s.n_tiles) * s.m_tiles > kMaxTiles) return GR_ERR_UNSUPPORTED;
  if (epi->mode == GR_EPI_QKV_ROPE) {
    if (!epi->q_out || !epi->k_cache || !epi->v_cache || !epi->row_pos || !epi->row_slot || !epi->inv_freq ||
        epi->rotary_dim % 32 || epi->rotary_dim > 128 || n_out != (epi->n_q_heads + 2 * epi->n_kv_heads) * 128 ||
        epi->page_size != 16)
      return GR_ERR_ARG;
    if (epi->row_pos3 && (epi->mrope_section[0] < 0 || epi->mrope_section[1] < 0 || epi->mrope_section[2] < 0 ||
                          epi->mrope_section[0] + epi->mrope_section[1] + epi->mrope_section[2] != epi->rotary_dim / 2))
      return GR_ERR_ARG;
  } else if (epi->mode == GR_EPI_ARGMAX) {
    if (!epi->out_idx) return GR_ERR_ARG;
  } else if (!epi->out || epi->ld_out <= 0) {
    return GR_ERR_ARG;
  }
  // the bf16 epilogues store 16-byte vectors
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if ((epi->mode == GR_EPI_SWIGLU || epi->mode == GR_EPI_STORE_BF16) && (!a16(epi->out) || epi->ld_out % 8))
    return GR_ERR_ARG;
  if (epi->mode == GR_EPI_QKV_ROPE && (!a16(epi->q_out) || !a16(epi->k_cache) || !a16(epi->v_cache))) return GR_ERR_ARG;
  // persistent grid: every resident CTA walks units c, c + grid, ...
  const int units = s.n_tiles * s.m_tiles * splits;
  int stages, per_sm;
  linear_launch_shape(s.nt, kc, epi->mode, &stages, &per_sm);
  const int cap = num_sms() * per_sm;
  const int grid = units < cap ? units : cap;
  CUtensorMap& tmw = out->tmw;
  CUtensorMap& tmx = out->tmx;
  int rc = tensor_map_2d(w, static_cast<uint64_t>(n_out), static_cast<uint64_t>(k_in), 128, 64, &tmw);
  if (rc) return rc;
  rc = tensor_map_2d(x, static_cast<uint64_t>(m), static_cast<uint64_t>(k_in), static_cast<uint32_t>(s.nt), 64, &tmx);
  if (rc) return rc;
  LinearParams& p = out->p;
  std::memset(&p, 0, sizeof(p));
  p.n_out = n_out;
  p.k_in = k_in;
  p.m = m;
  p.nt = s.nt;
  p.m_tiles = s.m_tiles;
  p.tail_last = s.tail_last ? 1 : 0;
  p.n_tiles = s.n_tiles;
  p.splits = splits;
  p.kc_per_split = kc;
  p.stages = stages;
  p.out = epi->out;
  p.ld_out = epi->ld_out;
  p.q_out = static_cast<__nv_bfloat16*>(epi->q_out);
  p.k_cache = static_cast<__nv_bfloat16*>(epi->k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(epi->v_cache);
  p.row_pos = epi->row_pos;
  p.row_pos3 = epi->row_pos3;
  p.mrope_s0 = epi->mrope_section[0];
  p.mrope_s1 = epi->mrope_section[1];
  p.row_slot = epi->row_slot;
  p.inv_freq = epi->inv_freq;
  p.rotary_dim = epi->rotary_dim;
  p.n_q_heads = epi->n_q_heads;
  p.n_kv_heads = epi->n_kv_heads;
  p.page_size = epi->page_size;
  p.out_idx = epi->out_idx;
  p.out_top1 = epi->out_top1;
  p.out_gap = epi->out_gap;
  p.ws_partial = ws.partial;
  p.ws_ticket = ws.ticket;
  p.ws_arg = ws.arg;
  p.prefetch = static_cast<const uint8_t*>(prefetch);
  p.prefetch_bytes = prefetch ? prefetch_bytes : 0;
  p.status = status;
  out->grid = grid;
  out->stages = stages;
  out->smem = linear_smem_bytes(s.nt, stages, epi->mode);
  return GR_OK;
}

int gr_linear(const void* w, int n_out, int k_in, const void* x, int m, const gr_epilogue* epi, int splits,
              void* workspace, size_t workspace_bytes, const void* prefetch, size_t prefetch_bytes, int32_t* status,
              void* stream) {
  LinearLaunch ll;
  const int rc = build_linear(w, n_out, k_in, x, m, epi, splits, workspace, workspace_bytes, prefetch, prefetch_bytes,
                              status, &ll);
  if (rc) return rc;
  cudaError_t e = launch_linear(epi->mode, ll.tmw, ll.tmx, ll.p, ll.grid, ll.smem, static_cast<cudaStream_t>(stream),
                                g_pdl);
  if (e == cudaSuccess && epi->mode == GR_EPI_ARGMAX)
    e = launch_argmax_reduce(ll.p, static_cast<cudaStream_t>(stream), g_pdl);
  return e == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

size_t gr_attention_workspace_bytes(int bs, int K, int n_q_heads, int n_kv_heads, int max_splits) {
  if (bs <= 0 || K <= 0 || n_kv_heads <= 0 || max_splits <= 0) return 0;
  const int G = n_q_heads / n_kv_heads;
  const size_t R_pad = ((G * K + 15) / 16) * 16;
  const size_t slots = static_cast<size_t>(bs) * n_kv_heads * max_splits;
  return kAttnTicketBytes + align256(slots * R_pad * 128 * sizeof(float)) + align256(slots * R_pad * 2 * sizeof(float));
}

// Checks, tensor maps and kernel parameters of one attention call; shared by the entry points.
struct AttnLaunch {
  AttnParams p;
  CUtensorMap tmk, tmv;
};
static int build_attention(const void* q, const void* k_cache, const void* v_cache, int64_t n_pages,
                           const int32_t* page_table, int pt_stride, const int64_t* seq_lens, const int32_t* req_order,
                           int bs, int K, int draft, int base_add, int n_q_heads, int n_kv_heads, int page_size,
                           int chunk, int max_splits, void* out, void* workspace, size_t workspace_bytes,
                           int32_t* status, AttnLaunch* al) {
  if (!q || !k_cache || !v_cache || !page_table || !seq_lens || !out || bs <= 0 || K <= 0 || n_pages <= 0)
    return GR_ERR_ARG;
  if (n_kv_heads <= 0 || n_q_heads % n_kv_heads || page_size != 16 || chunk <= 0 || chunk % 64 || chunk > 4096 ||
      max_splits <= 0 || draft < 0 || draft > 2)
    return GR_ERR_ARG;
  const int G = n_q_heads / n_kv_heads;
  if (G * K > 128 || static_cast<size_t>(bs) * n_kv_heads * sizeof(int) > kAttnTicketBytes) return GR_ERR_UNSUPPORTED;
  if (max_splits > 16) return GR_ERR_ARG;  // the split merge handles up to 16 splits per (request, kv head)
  const size_t need = gr_attention_workspace_bytes(bs, K, n_q_heads, n_kv_heads, max_splits);
  if (max_splits > 1 && (!workspace || workspace_bytes < need)) return GR_ERR_ARG;
  const uint64_t rows = static_cast<uint64_t>(n_pages) * n_kv_heads * page_size;
  CUtensorMap& tmk = al->tmk;
  CUtensorMap& tmv = al->tmv;
  int rc = tensor_map_2d(k_cache, rows, 128, static_cast<uint32_t>(page_size), 64, &tmk);
  if (rc) return rc;
  rc = tensor_map_2d(v_cache, rows, 128, static_cast<uint32_t>(page_size), 64, &tmv);
  if (rc) return rc;
  AttnParams& p = al->p;
  std::memset(&p, 0, sizeof(p));
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.page_table = page_table;
  p.pt_stride = pt_stride;
  p.seq_lens = seq_lens;
  p.bs = bs;
  p.K = K;
  p.draft = draft;
  p.base_add = base_add;
  p.n_q_heads = n_q_heads;
  p.n_kv_heads = n_kv_heads;
  p.page_size = page_size;
  p.chunk = chunk;
  p.max_splits = max_splits;
  p.scale_log2 = (1.0f / sqrtf(128.0f)) * 1.4426950408889634f;
  if (workspace) {
    uint8_t* b = static_cast<uint8_t*>(workspace);
    const size_t R_pad = ((G * K + 15) / 16) * 16;
    const size_t slots = static_cast<size_t>(bs) * n_kv_heads * max_splits;
    p.ws_ticket = reinterpret_cast<int*>(b);
    b += kAttnTicketBytes;
    p.ws_o = reinterpret_cast<float*>(b);
    b += align256(slots * R_pad * 128 * sizeof(float));
    p.ws_ml = reinterpret_cast<float*>(b);
  }
  p.status = status;
  p.order = req_order;
  return GR_OK;
}

int gr_bd_attention_ordered(const void* q, const void* k_cache, const void* v_cache, int64_t n_pages,
                            const int32_t* page_table, int pt_stride, const int64_t* seq_lens, const int32_t* req_order,
                            int bs, int K, int draft, int base_add, int n_q_heads, int n_kv_heads, int page_size,
                            int chunk, int max_splits, void* out, void* workspace, size_t workspace_bytes,
                            int32_t* status, void* stream) {
  AttnLaunch al;
  const int rc = build_attention(q, k_cache, v_cache, n_pages, page_table, pt_stride, seq_lens, req_order, bs, K, draft,
                                 base_add, n_q_heads, n_kv_heads, page_size, chunk, max_splits, out, workspace,
                                 workspace_bytes, status, &al);
  if (rc) return rc;
  cudaError_t e = launch_attention(al.tmk, al.tmv, al.p, static_cast<cudaStream_t>(stream), g_pdl);
  return e == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

int gr_bd_attention(const void* q, const void* k_cache, const void* v_cache, int64_t n_pages, const int32_t* page_table,
                    int pt_stride, const int64_t* seq_lens, int bs, int K, int draft, int base_add, int n_q_heads,
                    int n_kv_heads, int page_size, int chunk, int max_splits, void* out, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream) {
  return gr_bd_attention_ordered(q, k_cache, v_cache, n_pages, page_table, pt_stride, seq_lens, nullptr, bs, K, draft,
                                 base_add, n_q_heads, n_kv_heads, page_size, chunk, max_splits, out, workspace,
                                 workspace_bytes, status, stream);
}

int gr_embed_rows(int mode, int bs, int K, const int64_t* seeds, const int64_t* req_pool_idx, const int32_t* ids32,
                  const int64_t* ids64, const float* row_embeds, const int64_t* seq_lens, const int32_t* page_table,
                  int pt_stride, int page_size, int pages_per_req, const void* embed, int vocab, int mask_id,
                  const void* norm_w, float eps, int hidden, float* h_out, void* x_out, int32_t* row_pos,
                  int64_t* row_slot, int32_t* row_ids, const int32_t* rope_delta, int32_t* status, void* stream) {
  if (bs <= 0 || K <= 0 || !seq_lens || !page_table || !embed || !norm_w || !h_out || !x_out || !row_pos || !row_slot)
    return GR_ERR_ARG;
  if (hidden <= 0 || hidden % 8 || page_size <= 0 || pages_per_req <= 0) return GR_ERR_ARG;
  if (mode == GR_ROWS_DRAFT && (!seeds || !req_pool_idx)) return GR_ERR_ARG;
  if (mode == GR_ROWS_VERIFY && !ids32) return GR_ERR_ARG;
  if (mode == GR_ROWS_EXPLICIT && !ids64) return GR_ERR_ARG;
  if (mode < GR_ROWS_DRAFT || mode > GR_ROWS_EXPLICIT) return GR_ERR_ARG;
  EmbedParams p;
  std::memset(&p, 0, sizeof(p));
  p.mode = mode;
  p.bs = bs;
  p.K = K;
  p.hidden = hidden;
  p.vocab = vocab;
  p.mask_id = mask_id;
  p.page_size = page_size;
  p.pt_stride = pt_stride;
  p.pages_per_req = pages_per_req;
  p.seeds = seeds;
  p.rpi = req_pool_idx;
  p.ids32 = ids32;
  p.ids64 = ids64;
  p.row_embeds = row_embeds;
  p.seq_lens = seq_lens;
  p.page_table = page_table;
  p.rope_delta = rope_delta;
  p.embed = static_cast<const __nv_bfloat16*>(embed);
  p.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  p.eps = eps;
  p.h_out = h_out;
  p.x_out = static_cast<__nv_bfloat16*>(x_out);
  p.row_pos = row_pos;
  p.row_slot = row_slot;
  p.row_ids = row_ids;
  p.status = status;
  return launch_embed_rows(p, static_cast<cudaStream_t>(stream), g_pdl) == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

int gr_residual_norm(int m, int hidden, const float* h_in, const float* y, int y_parts, const void* w_a,
                     const void* w_b, float eps, float* h_out, void* x_out, void* stream) {
  if (m <= 0 || hidden <= 0 || hidden % 8 || !h_in || !y || !w_a || !w_b || !h_out || !x_out) return GR_ERR_ARG;
  if (h_in == h_out || y_parts < 1 || hidden > 8 * 192 * 4) return GR_ERR_ARG;
  ResNormParams p;
  p.m = m;
  p.hidden = hidden;
  p.y_parts = y_parts;
  p.h_in = h_in;
  p.y = y;
  p.w_a = static_cast<const __nv_bfloat16*>(w_a);
  p.w_b = static_cast<const __nv_bfloat16*>(w_b);
  p.eps = eps;
  p.h_out = h_out;
  p.x_out = static_cast<__nv_bfloat16*>(x_out);
  p.sms = num_sms();
  return launch_residual_norm(p, static_cast<cudaStream_t>(stream), g_pdl) == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

int gr_accept_commit(int bs, int K, const int32_t* am, const int32_t* v, int64_t* seeds, const int64_t* req_pool_idx,
                     int64_t* seq_lens, int x0_committed, const int64_t* loc, int32_t* packed, int64_t* released,
                     int32_t* n_released, int64_t* out_next, int32_t* n_committed, int32_t* rounds,
                     int32_t* accept_len, void* stream) {
  if (bs <= 0 || K < 2 || !am || !v || !seeds || !req_pool_idx || !seq_lens || !packed || !released || !out_next)
    return GR_ERR_ARG;
  CommitParams p;
  p.bs = bs;
  p.K = K;
  p.x0_committed = x0_committed ? 1 : 0;
  p.am = am;
  p.v = v;
  p.seeds = seeds;
  p.rpi = req_pool_idx;
  p.seq_lens = seq_lens;
  p.loc = loc;
  p.packed = packed;
  p.released = released;
  p.n_released = n_released;
  p.out_next = out_next;
  p.n_committed = n_committed;
  p.rounds = rounds;
  p.accept_len = accept_len;
  p.accept = nullptr;
  p.sample = nullptr;
  p.predict = nullptr;
  p.rng = nullptr;
  return launch_accept_commit(p, static_cast<cudaStream_t>(stream), g_pdl) == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

int gr_commit_sampled(int bs, int K, const int32_t* am, const int32_t* accept, const int32_t* sample, int64_t* seeds,
                      const int64_t* req_pool_idx, int64_t* seq_lens, int32_t* predict, int32_t* packed,
                      int64_t* released, int32_t* n_released, int64_t* out_next, int32_t* n_committed,
                      int32_t* rounds, int32_t* accept_len, uint64_t* rng, void* stream) {
  if (bs <= 0 || K < 2 || !am || !accept || !sample || !seeds || !req_pool_idx || !seq_lens || !predict || !packed ||
      !released || !out_next)
    return GR_ERR_ARG;
  CommitParams p;
  std::memset(&p, 0, sizeof(p));
  p.bs = bs;
  p.K = K;
  p.x0_committed = 0;
  p.am = am;
  p.v = predict;
  p.seeds = seeds;
  p.rpi = req_pool_idx;
  p.seq_lens = seq_lens;
  p.packed = packed;
  p.released = released;
  p.n_released = n_released;
  p.out_next = out_next;
  p.n_committed = n_committed;
  p.rounds = rounds;
  p.accept_len = accept_len;
  p.accept = accept;
  p.sample = sample;
  p.predict = predict;
  p.rng = rng;
  return launch_accept_commit(p, static_cast<cudaStream_t>(stream), g_pdl) == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

static int check_sampling(const gr_sampling* s) {
  if (!s || s->vocab <= 0 || s->vocab > kSampleMaxVocab || s->filter < GR_FILTER_JOINT ||
      s->filter > GR_FILTER_TORCH || s->n_order < 0 || s->n_order > 4 || !s->req_pool_idx || !s->rng)
    return GR_ERR_ARG;
  for (int i = 0; i < s->n_order; ++i) {
    const int op = s->order[i];
    if (op < GR_PEN_REPETITION || op > GR_PEN_MIN_NEW_TOKENS) return GR_ERR_ARG;
    if ((op == GR_PEN_REPETITION && (!s->repetition || !s->st_rep)) ||
        (op == GR_PEN_FREQUENCY && (!s->frequency || !s->st_freq)) ||
        (op == GR_PEN_PRESENCE && (!s->presence || !s->st_pres)) ||
        (op == GR_PEN_MIN_NEW_TOKENS && (!s->min_new_tokens || !s->st_len || (s->n_stop > 0 && !s->stop_ids))))
      return GR_ERR_ARG;
  }
  return GR_OK;
}

int gr_gather_rows(const void* src, int row_bytes, int n, int src_stride_rows, void* dst, void* stream) {
  if (!src || !dst || n <= 0 || row_bytes <= 0 || row_bytes % 16 || src_stride_rows < 1) return GR_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) return GR_ERR_ARG;
  return launch_gather_rows(src, row_bytes, n, src_stride_rows, dst, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? GR_OK
             : GR_ERR_CUDA;
}

int gr_logits_process(float* logits, int bs, int K, const int32_t* cand, const gr_sampling* s, void* stream) {
  int rc = check_sampling(s);
  if (rc) return rc;
  if (!logits || bs <= 0 || K <= 0 || (K > 1 && !cand) || K > 64) return GR_ERR_ARG;
  SampleParams p;
  std::memset(&p, 0, sizeof(p));
  p.s = *s;
  p.logits = logits;
  p.bs = bs;
  p.K = K;
  p.cand = cand;
  return launch_logits_process(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

int gr_sample_rows(float* logits, int bs, int K, const int32_t* cand, const gr_sampling* s, int first_kind,
                   int32_t* accept, int32_t* sample, float* p_next, int32_t* first_out, int first_stride,
                   int32_t* status, void* stream) {
  int rc = check_sampling(s);
  if (rc) return rc;
  if (!logits || bs <= 0 || K <= 0 || !sample || (K > 1 && (!cand || !accept)) || K > 64) return GR_ERR_ARG;
  if (first_kind != GR_COIN_FIRST && first_kind != GR_COIN_PREFILL) return GR_ERR_ARG;
  if (!s->temperature || !s->top_k || !s->top_p || !s->min_p) return GR_ERR_ARG;
  SampleParams p;
  std::memset(&p, 0, sizeof(p));
  p.s = *s;
  p.logits = logits;
  p.bs = bs;
  p.K = K;
  p.cand = cand;
  p.first_kind = first_kind;
  p.accept = accept;
  p.sample = sample;
  p.p_next = p_next;
  p.first_out = first_out;
  p.first_stride = first_stride;
  p.status = status;
  p.sms = num_sms();
  return launch_sample_rows(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

int gr_penalty_cumulate(int bs, const int32_t* tokens, int stride, const int32_t* counts, int add,
                        const gr_sampling* s, void* stream) {
  int rc = check_sampling(s);
  if (rc) return rc;
  if (bs <= 0 || !tokens || stride <= 0) return GR_ERR_ARG;
  SampleParams p;
  std::memset(&p, 0, sizeof(p));
  p.s = *s;
  p.bs = bs;
  p.tokens = tokens;
  p.tok_stride = stride;
  p.counts = counts;
  p.add = add;
  return launch_penalty_cumulate(p, static_cast<cudaStream_t>(stream)) == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

int gr_draft_override(int bs, int K, int32_t* am, const int32_t* g, int g_stride, const int32_t* n_committed,
                      const int32_t* accept_plan, int plan_stride, const int32_t* rounds, int vocab, int mask_id,
                      void* stream) {
  if (bs <= 0 || K < 2 || !am || !g || !n_committed || !accept_plan || !rounds || vocab <= 0) return GR_ERR_ARG;
  OverrideParams p;
  p.bs = bs;
  p.K = K;
  p.g_stride = g_stride;
  p.plan_stride = plan_stride;
  p.vocab = vocab;
  p.mask_id = mask_id;
  p.am = am;
  p.g = g;
  p.n_committed = n_committed;
  p.plan = accept_plan;
  p.rounds = rounds;
  return launch_draft_override(p, static_cast<cudaStream_t>(stream), g_pdl) == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}

int gr_pack_gate_up(const void* src, void* dst, int intermediate, int hidden, void* stream) {
  if (!src || !dst || intermediate % 64 || hidden % 8) return GR_ERR_ARG;
  return launch_pack_gate_up(static_cast<const __nv_bfloat16*>(src), static_cast<__nv_bfloat16*>(dst), intermediate,
                             hidden, static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? GR_OK
             : GR_ERR_CUDA;
}

}  // extern "C"

// ------------------------------------------------------------------ attention without a caller workspace
// The split scratch of gr_bd_attention_noalloc: one array per loaded device, zero at module load.  Host code may not use
// the name as a device address; it asks the runtime for the address once per device (below).
static __device__ __align__(256) uint8_t g_noalloc_attn_scratch[GR_NOALLOC_SCRATCH_BYTES];

namespace gr {
static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[kMaxDevices] = {};

// Device address of this device's scratch array; looked up on the device's first call (with that device current).
static int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return GR_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return GR_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_attn_scratch) != cudaSuccess || !p) return GR_ERR_CUDA;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return GR_OK;
}
}  // namespace gr

extern "C" int gr_bd_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, int64_t n_pages,
                                       const int32_t* page_table, int pt_stride, const int64_t* seq_lens, int bs, int K,
                                       int draft, int base_add, int n_q_heads, int n_kv_heads, int page_size, int chunk,
                                       int max_splits, void* out, int32_t* status, void* stream) {
  if (bs <= 0 || K <= 0 || n_kv_heads <= 0 || max_splits <= 0) return GR_ERR_ARG;
  const size_t need = gr_attention_workspace_bytes(bs, K, n_q_heads, n_kv_heads, max_splits);
  if (need > GR_NOALLOC_SCRATCH_BYTES) return GR_ERR_SCRATCH_LIMIT;
  void* ws = nullptr;
  int rc = gr::noalloc_scratch(&ws);
  if (rc) return rc;
  // every argument check runs before anything is queued: a refused call leaves nothing on the stream
  AttnLaunch al;
  rc = build_attention(q, k_cache, v_cache, n_pages, page_table, pt_stride, seq_lens, nullptr, bs, K, draft,
                           base_add, n_q_heads, n_kv_heads, page_size, chunk, max_splits, out, ws,
                           GR_NOALLOC_SCRATCH_BYTES, status, &al);
  if (rc) return rc;
  // the array keeps whatever the last call left; the tickets this call counts on must start at zero
  if (max_splits > 1 &&
      cudaMemsetAsync(ws, 0, static_cast<size_t>(bs) * n_kv_heads * sizeof(int), static_cast<cudaStream_t>(stream)) !=
          cudaSuccess)
    return GR_ERR_CUDA;
  const cudaError_t e = gr::launch_attention(al.tmk, al.tmv, al.p, static_cast<cudaStream_t>(stream), gr::g_pdl);
  return e == cudaSuccess ? GR_OK : GR_ERR_CUDA;
}
