// Parameter blocks of the kernels and their launchers, shared by the kernel files and the C-ABI layer.
#pragma once

#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"

namespace gr {
struct LinearParams {
  int n_out, k_in, m;
  int nt, m_tiles, n_tiles, splits, kc_per_split, stages;
  int tail_last;  // 1: the units of a shorter last token tile are numbered after all full tiles' units
  void* out;
  int ld_out;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  const int* row_pos;
  const int* row_pos3;  // [M][3] (t, h, w) positions, or NULL: every pair uses row_pos
  int mrope_s0, mrope_s1;  // pairs [0, s0) rotate by axis 0, [s0, s0 + s1) by axis 1, the rest by axis 2
  const int64_t* row_slot;
  const float* inv_freq;
  int rotary_dim, n_q_heads, n_kv_heads, page_size;
  int* out_idx;
  float* out_top1;
  float* out_gap;
  float* ws_partial;
  int* ws_ticket;
  float4* ws_arg;  // lm_head: per (token, feature tile) top-2 record {v1, i1 bits, v2, 0}, token-major
  const uint8_t* prefetch;
  unsigned long long prefetch_bytes;
  int* status;
};
struct AttnParams {
  const __nv_bfloat16* q;
  __nv_bfloat16* out;
  const int* page_table;
  int pt_stride;
  const int64_t* seq_lens;
  int bs, K, draft, base_add;
  int n_q_heads, n_kv_heads, page_size;
  int chunk, max_splits, groups;
  int cluster;           // 1: the max_splits CTAs of a (request, kv head) form one cluster and merge through DSMEM
  int split_outer;       // 1: grid (kv head, request, split) instead of (split, kv head, request); tcgen05 kernel only
  const int32_t* order;  // optional: grid z -> request (longest first), NULL = identity
  float scale_log2;
  float* ws_o;
  float* ws_ml;
  int* ws_ticket;
  int* status;
};
struct EmbedParams {
  int mode, bs, K, hidden, vocab, mask_id, page_size, pt_stride, pages_per_req;
  const int64_t* seeds;
  const int64_t* rpi;
  const int32_t* ids32;
  const int64_t* ids64;
  const float* row_embeds;
  const int64_t* seq_lens;
  const int32_t* page_table;
  const int32_t* rope_delta;
  const __nv_bfloat16* embed;
  const __nv_bfloat16* norm_w;
  float eps;
  float* h_out;
  __nv_bfloat16* x_out;
  int32_t* row_pos;
  int64_t* row_slot;
  int32_t* row_ids;
  int32_t* status;
};
struct ResNormParams {
  int m, hidden, y_parts;
  int sms;  // SMs of the device: the many-rows kernel runs a fixed number of CTAs per SM
  const float* h_in;
  const float* y;
  const __nv_bfloat16* w_a;
  const __nv_bfloat16* w_b;
  float eps;
  float* h_out;
  __nv_bfloat16* x_out;
};
struct CommitParams {
  int bs, K, x0_committed;
  const int32_t* am;
  const int32_t* v;
  int64_t* seeds;
  const int64_t* rpi;
  int64_t* seq_lens;
  const int64_t* loc;
  int32_t* packed;
  int64_t* released;
  int32_t* n_released;
  int64_t* out_next;
  int32_t* n_committed;
  int32_t* rounds;
  int32_t* accept_len;
  // sampled verify (accept != NULL): acc from the per-row accept bits, v[acc] = sample[acc], written to predict
  const int32_t* accept;
  const int32_t* sample;
  int32_t* predict;
  uint64_t* rng;
};
struct SampleParams {
  gr_sampling s;
  float* logits;
  int bs, K;
  const int32_t* cand;
  int first_kind;
  int32_t* accept;
  int32_t* sample;
  float* p_next;
  int32_t* first_out;
  int first_stride;
  int32_t* status;
  const int32_t* tokens;   // penalty cumulation
  int tok_stride;
  const int32_t* counts;
  int add;
  int sms;                 // SMs of the device (sample_rows picks its CTA size by the rows per SM)
};
struct OverrideParams {
  int bs, K, g_stride, plan_stride, vocab, mask_id;
  int32_t* am;
  const int32_t* g;
  const int32_t* n_committed;
  const int32_t* plan;
  const int32_t* rounds;
};

// Host-side set-up that belongs to one device context (function attributes, occupancy answers): done once per device,
// under a lock, by the first launch that runs with that device current.
constexpr int kMaxDevices = 64;
struct PerDeviceOnce {
  std::mutex mu;
  bool done[kMaxDevices] = {};
};
template <class F>
inline cudaError_t once_per_device(PerDeviceOnce& o, F f) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> g(o.mu);
  if (o.done[dev]) return cudaSuccess;
  e = f();
  if (e == cudaSuccess) o.done[dev] = true;
  return e;
}
// Cached yes/no answers keyed by (device, cluster size, threads, dynamic shared memory).
struct ClusterFitCache {
  std::mutex mu;
  std::map<std::tuple<int, int, int, size_t>, bool> known;
};
template <class F>
inline bool cluster_fit_cached(ClusterFitCache& c, int size, int threads, size_t smem, F query) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const auto key = std::make_tuple(dev, size, threads, smem);
  std::lock_guard<std::mutex> g(c.mu);
  auto it = c.known.find(key);
  if (it != c.known.end()) return it->second;
  const bool ok = query();
  c.known[key] = ok;
  return ok;
}

size_t linear_smem_bytes(int nt, int stages, int epi);
cudaError_t launch_linear(int epi, const CUtensorMap& tmw, const CUtensorMap& tmx, const LinearParams& p, int grid,
                          size_t smem, cudaStream_t stream, bool pdl);
cudaError_t launch_argmax_reduce(const LinearParams& p, cudaStream_t stream, bool pdl);

size_t attention_smem_bytes(int K, int G, int stages);
size_t attention_tc_smem_bytes(int G, int K, int stages);
bool attention_tc_fits(const AttnParams& p);
cudaError_t launch_attention_tc(const CUtensorMap& tmk, const CUtensorMap& tmv, const AttnParams& p, bool small,
                                cudaStream_t stream, bool pdl);
extern int g_attention_tc;
cudaError_t launch_attention(const CUtensorMap& tmk, const CUtensorMap& tmv, const AttnParams& p, cudaStream_t stream,
                             bool pdl);
cudaError_t launch_embed_rows(const EmbedParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_residual_norm(const ResNormParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_accept_commit(const CommitParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_draft_override(const OverrideParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_gather_rows(const void* src, int row_bytes, int n, int src_stride_rows, void* dst, cudaStream_t s);
cudaError_t launch_logits_process(const SampleParams& p, cudaStream_t s);
cudaError_t launch_sample_rows(const SampleParams& p, cudaStream_t s);
// Largest vocabulary sample_rows takes: a warp adds at most 4,095 entries per pass to its 32-bit bucket words.
constexpr int kSampleMaxVocab = 65024;
cudaError_t launch_penalty_cumulate(const SampleParams& p, cudaStream_t s);
cudaError_t launch_pack_gate_up(const __nv_bfloat16* src, __nv_bfloat16* dst, int I, int H, cudaStream_t s);

}  // namespace gr
