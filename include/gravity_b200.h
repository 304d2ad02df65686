/* C ABI of the B200-native self-speculative decode round (libgravity_b200.so).
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer owned by the caller, every call takes the
 * CUDA stream to launch on (as a void*, NULL = legacy default stream), returns GR_OK or an error code, allocates
 * nothing and never synchronises.  Kernels record run-time faults (a bounded wait that ran out, an out-of-range id
 * or page) in the caller's device `status` word (first error wins); the host reads it with the round's readback.
 *
 * Each entry cites the reference interface it replaces (trillion-labs/GravityOCR; paths inside that project).
 * Shapes use B = bd_size, K = B + 1 rows per request, M = bs * K rows per forward, H = hidden.
 */
#ifndef GRAVITY_B200_H
#define GRAVITY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum gr_status_code {
  GR_OK = 0,
  GR_ERR_ARG = 1,         /* invalid argument (shape, alignment, unsupported size) */
  GR_ERR_CUDA = 2,        /* a CUDA runtime call failed (launch, attribute) */
  GR_ERR_TMA = 3,         /* cuTensorMapEncodeTiled rejected a tensor map */
  GR_ERR_TIMEOUT = 4,     /* device: a bounded wait ran out (written to the status word) */
  GR_ERR_BAD_ID = 5,      /* device: a token id outside [0, vocab) */
  GR_ERR_BAD_PAGE = 6,    /* device: a position beyond the request's page-table capacity */
  GR_ERR_UNSUPPORTED = 7, /* the build does not support this configuration */
  GR_ERR_SCRATCH_LIMIT = 8, /* the call needs more scratch than gr_bd_attention_noalloc's fixed array holds */
  GR_ERR_NO_TOKEN = 9       /* device: a sampled row allowed no token (every logit -inf after masks and penalties) */
};

/* Epilogues of gr_linear. */
enum gr_epilogue_mode {
  GR_EPI_STORE_F32 = 0,  /* out[t, f] fp32 */
  GR_EPI_STORE_BF16 = 1, /* out[t, f] bf16 */
  GR_EPI_SWIGLU = 2,     /* out[t, j] = up * silu(gate), bf16; weight rows 2j / 2j+1 = gate j / up j (gr_pack_gate_up) */
  GR_EPI_QKV_ROPE = 3,   /* q -> q_out, k/v -> paged cache with partial interleaved RoPE */
  GR_EPI_ARGMAX = 4,     /* vocab-wide argmax per row: out_idx, out_top1, out_gap; no logits written */
  GR_EPI_PARTIAL_F32 = 5 /* split-K partials, out[split][t][f] fp32 (split stride m * ld_out); the consumer sums
                            them (gr_residual_norm with y_parts = splits) */
};

/* Row sources of gr_embed_rows. */
enum gr_rows_mode {
  GR_ROWS_DRAFT = 0,    /* row (b, j): id = j == 0 ? seeds[rpi[b]] : mask_id, position seq_lens[b] + j */
  GR_ROWS_VERIFY = 1,   /* row (b, j): id = ids32[b*K + j] (the draft argmax), position seq_lens[b] + 1 + j */
  GR_ROWS_EXPLICIT = 2  /* row t: id = ids64[t] (id < 0: take row_embeds[t]), position seq_lens[b] + j */
};

typedef struct gr_epilogue {
  int mode;               /* gr_epilogue_mode */
  void* out;              /* STORE_*, SWIGLU: [M, ld_out]; bf16 outputs 16-byte aligned with ld_out % 8 == 0 */
  int ld_out;
  /* QKV_ROPE: weight rows are [q heads | k heads | v heads] x head_dim 128; q_out and the caches 16-byte aligned */
  void* q_out;            /* bf16 [M, n_q_heads*128] */
  void* k_cache;          /* bf16 [pages, n_kv_heads, page_size, 128] of this layer */
  void* v_cache;
  const int32_t* row_pos;  /* [M] RoPE position of each row */
  const int64_t* row_slot; /* [M] cache slot (page * page_size + offset) of each row */
  const float* inv_freq;   /* [rotary_dim / 2] */
  int rotary_dim, n_q_heads, n_kv_heads, page_size;
  /* ARGMAX */
  int32_t* out_idx;       /* [M] */
  float* out_top1;        /* [M] or NULL */
  float* out_gap;         /* [M] top-1 minus top-2 logit, or NULL */
  /* QKV_ROPE with multimodal (3-axis) positions: row_pos3 [M][3] = (t, h, w) position of each row, or NULL for 1-D
   * row_pos.  Rotary pair i uses axis 0 for i < mrope_section[0], axis 1 for the next mrope_section[1] pairs, axis 2
   * after (transformers GlmOcrTextRotaryEmbedding.apply_mrope, sections [8, 12, 12]). */
  const int32_t* row_pos3;
  int mrope_section[3];
} gr_epilogue;

/* Library identity / diagnostics. */
int gr_version(void);
const char* gr_status_string(int code);
/* Programmatic dependent launch on (1, default) / off (0) for every later launch. */
void gr_set_pdl(int enable);
/* Which attention kernel runs: 0 the mma.sync kernel for every grid; 1 (default) the tcgen05 / TMEM kernel for
 * grids of more than one CTA per SM and the mma.sync kernel below that; 2 the tcgen05 kernel for every grid (small
 * grids as thread-block clusters).  All compute the same rows; the switch exists to compare them. */
void gr_set_attention_tc(int mode);
/* Number of SMs the split heuristics assume (queried for the current device on first use). */
int gr_num_sms(void);

/* Workspace (scratch) sizes in bytes for the calls below; the caller allocates them once, zero-filled, and passes
 * them on every call (the kernels leave their tickets re-armed at zero). */
size_t gr_linear_workspace_bytes(int n_out, int m, int splits);
size_t gr_attention_workspace_bytes(int bs, int K, int n_q_heads, int n_kv_heads, int max_splits);

/* Split-K count gr_linear uses by default (0 in `splits` below) for this shape and epilogue mode (gr_epilogue_mode):
 * the token tiling and the split count are planned together, and the plan depends on what the epilogue stores (a
 * split-K tile's last split reads every split's partial before it runs the epilogue; GR_EPI_PARTIAL_F32 leaves the
 * sum to its consumer). */
int gr_linear_default_splits(int n_out, int k_in, int m, int mode);
/* The plan gr_linear runs for this call shape (splits = 0: the default): out[0] split-K count, out[1] token-tile
 * height nt, out[2] token tiles, out[3] 1 when a shorter last tile's units run after the full tiles' (odd waves in
 * reverse), out[4] persistent grid.  Diagnostics: no reference counterpart. */
int gr_linear_plan(int n_out, int k_in, int m, int mode, int splits, int32_t* out);

/* Weight-streaming projection with a fused epilogue:  y[t, f] = sum_k x[t, k] * w[f, k].
 * w: bf16 [n_out, k_in] row-major (nn.Linear); x: bf16 [m, k_in] row-major; n_out % 128 == 0, k_in % 64 == 0,
 * k_in * 2 and the row strides 16-byte aligned.  splits = 0 picks gr_linear_default_splits.  prefetch /
 * prefetch_bytes: optional global range (the next kernel's weights) warmed into L2 while this one streams.
 * Replaces the cuBLAS GEMMs behind transformers' GlmOcrTextAttention q/k/v/o_proj and GlmOcrTextMLP
 * gate_up/down_proj (models/glm_ocr/modeling_glm_ocr.py:188-191, 242-243) plus, for GR_EPI_QKV_ROPE, RoPE (:121-165)
 * and the SGLang KV-cache write; for GR_EPI_ARGMAX the lm_head + logits.argmax of
 * patches/sglang/python/sglang/srt/speculative/selfspec_diffusion_worker.py:739-742 and src/fast_sampling.py:571-575. */
int gr_linear(const void* w, int n_out, int k_in, const void* x, int m, const gr_epilogue* epi, int splits,
              void* workspace, size_t workspace_bytes, const void* prefetch, size_t prefetch_bytes, int32_t* status,
              void* stream);

/* Layer-0 input rows of a forward and the window plan: for each row its token id, RoPE position and cache slot;
 * h_out[t] = embedding row (fp32), x_out[t] = RMSNorm(h_out[t]) * norm_w (bf16).  The RoPE position is the cache
 * position plus rope_delta[b] (int32 [bs], or NULL for 0): the multimodal position offset of a request whose image
 * tokens take fewer position values than cache slots (the M-RoPE delta, sglang_0.5.10_selfspec.patch:1371-1380).
 * Replaces the draft window build of selfspec_diffusion_worker.py:689-706 (_draft_block: [seed | mask x (K-1)],
 * positions seq_lens + j), the verify ids/positions of :849-884 (_fulldraft_verify: am[:, :K], seq_lens + 1 + j),
 * the embedding lookup with image-embedding injection of src/fast_sampling.py:483-488, and the first
 * input_layernorm (modeling_glm_ocr.py:50-64). */
int gr_embed_rows(int mode, int bs, int K, const int64_t* seeds, const int64_t* req_pool_idx, const int32_t* ids32,
                  const int64_t* ids64, const float* row_embeds, const int64_t* seq_lens, const int32_t* page_table,
                  int pt_stride, int page_size, int pages_per_req, const void* embed, int vocab, int mask_id,
                  const void* norm_w, float eps, int hidden, float* h_out, void* x_out, int32_t* row_pos,
                  int64_t* row_slot, int32_t* row_ids, const int32_t* rope_delta, int32_t* status, void* stream);

/* Sandwich-norm step: h_out = h_in + w_a * RMSNorm(y); x_out = w_b * RMSNorm(h_out) (bf16).  y may arrive as
 * y_parts split-K partials (y[p * m * hidden + t * hidden + f], summed in order p = 0, 1, ...).  The decoder layer's
 * post_self_attn / post_attention and post_mlp / next input_layernorm pairs (modeling_glm_ocr.py:281-302), and the
 * final model norm before lm_head. */
int gr_residual_norm(int m, int hidden, const float* h_in, const float* y, int y_parts, const void* w_a,
                     const void* w_b, float eps, float* h_out, void* x_out, void* stream);

/* Block-diffusion draft attention (draft = 1: row 0 causal, mask rows see the whole window; draft = 2: every row sees
 * the whole window, the first block of the in-process round of src/fast_sampling.py:508-510 with no pending token) or
 * causal verify / prefill attention (draft = 0) over the paged cache.  q/out: bf16 [bs*K, n_q_heads, 128]; k_cache/v_cache: bf16
 * [n_pages, n_kv_heads, page_size = 16, 128] of one layer; page_table int32 [bs, pt_stride]; window row j of request b
 * sits at position seq_lens[b] + base_add + j.  chunk: cache tokens per split (multiple of 64); max_splits: grid
 * extent (splits past a request's length exit at once).
 * Replaces flashinfer BatchPrefillWithPagedKVCacheWrapper in the draft (NON_CAUSAL + CAUSAL re-run of row 0) and
 * verify (CAUSAL) roles planned by patches/sglang/python/sglang/srt/speculative/selfspec_fast_attn.py:168-440 and
 * the flex_attention masks of src/fast_sampling.py:508-514. */
int gr_bd_attention(const void* q, const void* k_cache, const void* v_cache, int64_t n_pages, const int32_t* page_table,
                    int pt_stride, const int64_t* seq_lens, int bs, int K, int draft, int base_add, int n_q_heads,
                    int n_kv_heads, int page_size, int chunk, int max_splits, void* out, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream);

/* gr_bd_attention with a scheduling order: req_order (int32 [bs], a permutation of 0..bs-1, e.g. longest committed
 * length first) is the order in which requests' blocks are launched; results do not depend on it. */
int gr_bd_attention_ordered(const void* q, const void* k_cache, const void* v_cache, int64_t n_pages,
                            const int32_t* page_table, int pt_stride, const int64_t* seq_lens, const int32_t* req_order,
                            int bs, int K, int draft, int base_add, int n_q_heads, int n_kv_heads, int page_size,
                            int chunk, int max_splits, void* out, void* workspace, size_t workspace_bytes,
                            int32_t* status, void* stream);

/* gr_bd_attention without a caller-provided workspace.  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory -- a host that owns the whole device-memory budget (a serving framework whose
 * allocator accounts for every byte, so a private cudaMalloc would break its bookkeeping or fail under pressure), or
 * code that issues the call while a CUDA stream is being captured, where cudaMalloc is not permitted.
 * The split scratch lives in one file-scope __device__ array of GR_NOALLOC_SCRATCH_BYTES (8 MiB) that every GPU which
 * loads the library keeps until the process exits.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call before any stream capture.  Calls whose
 * scratch (gr_attention_workspace_bytes of the same arguments) exceeds the array return GR_ERR_SCRATCH_LIMIT.  The call
 * allocates nothing: it clears the tickets it uses with cudaMemsetAsync on `stream`, then runs the same kernel.  All
 * calls share the array, so two calls that can overlap on the GPU (different streams, no ordering) race. */
#define GR_NOALLOC_SCRATCH_BYTES (8u << 20)
int gr_bd_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, int64_t n_pages,
                            const int32_t* page_table, int pt_stride, const int64_t* seq_lens, int bs, int K, int draft,
                            int base_add, int n_q_heads, int n_kv_heads, int page_size, int chunk, int max_splits,
                            void* out, int32_t* status, void* stream);

/* Accept and commit (one CTA): acc = leading d_j == v[j-1] matches (linear-chain greedy verify); packed[b] =
 * (a0, acc, v[0..acc], zeros); seeds[rpi[b]] = out_next[b] = v[acc]; seq_lens[b] += acc + 1 (+1 more when
 * x0_committed == 0, i.e. x0 is committed here); released = the verify rows acc+1..K-1 compacted in row order, as
 * loc[b*K + j] when loc != NULL (physical slots, the reference free list) else as logical positions;
 * n_committed[b] += acc + 2 and rounds[b] += 1 when given.
 * Replaces sgl_kernel verify_tree_greedy on the linear chain (selfspec_diffusion_worker.py:530-548) and the Triton
 * _ss_commit_kernel (patches/sglang/python/sglang/srt/speculative/selfspec_fast_commit.py:108-147). */
int gr_accept_commit(int bs, int K, const int32_t* am, const int32_t* v, int64_t* seeds, const int64_t* req_pool_idx,
                     int64_t* seq_lens, int x0_committed, const int64_t* loc, int32_t* packed, int64_t* released,
                     int32_t* n_released, int64_t* out_next, int32_t* n_committed, int32_t* rounds,
                     int32_t* accept_len, void* stream);

/* Forced-accept replay (no reference counterpart; the baseline's config-2 replay mode): overwrite the draft so that
 * exactly A = accept_plan[b, rounds[b]] drafts match the known stream g: am[b, j] = g[b, c + j] for 1 <= j <= A and
 * am[b, A+1] = (g[b, c + A + 1] + 1) mod vocab (skipping mask_id), c = n_committed[b]. */
int gr_draft_override(int bs, int K, int32_t* am, const int32_t* g, int g_stride, const int32_t* n_committed,
                      const int32_t* accept_plan, int plan_stride, const int32_t* rounds, int vocab, int mask_id,
                      void* stream);

/* Load-time helper: reorder gate_up rows [gate(I) | up(I)] so that row 2j is gate j and row 2j+1 is up j (the layout
 * GR_EPI_SWIGLU expects).  src/dst: bf16 [2*I, H] device buffers. */
int gr_pack_gate_up(const void* src, void* dst, int intermediate, int hidden, void* stream);

/* ------------------------------------------------------------------ non-greedy rounds (sampling, penalties, grammar)
 * A batch with any sampled request, penalty, logit bias or grammar takes this path instead of the argmax epilogue:
 * lm_head writes fp32 logits (gr_linear with GR_EPI_STORE_F32), gr_logits_process applies what AR decode applies to
 * each row, gr_sample_rows draws / tests against AR's target distribution, and gr_commit_sampled commits.  The
 * reference's counterparts: selfspec_sampling.py (penalize_rows, verify_target_probs, cumulate_block) and
 * selfspec_fast_commit.py:150-230 (process_verify_logits, sampling_verify with sgl_kernel's
 * tree_speculative_sampling_target_only), and the worker's a0 draw (selfspec_diffusion_worker.py:504-528). */
enum gr_filter_mode {
  GR_FILTER_JOINT = 0,      /* flashinfer backend without min-p: keep q iff #{p > p_q} < k and sum{p > p_q} < top_p */
  GR_FILTER_SEQUENTIAL = 1, /* flashinfer backend with min-p: top-k renorm, then top-p renorm, then p >= min_p * max */
  GR_FILTER_TORCH = 2       /* "pytorch" backend: #{p > p_q} < k, sum{p > p_q} <= top_p, p >= min_p * max */
};
enum gr_penalty_op { GR_PEN_REPETITION = 0, GR_PEN_FREQUENCY = 1, GR_PEN_PRESENCE = 2, GR_PEN_MIN_NEW_TOKENS = 3 };
enum gr_coin_kind { GR_COIN_ACCEPT = 0, GR_COIN_FINAL = 1, GR_COIN_FIRST = 2, GR_COIN_PREFILL = 3 };

/* Sampling parameters of a batch.  Per-request arrays are [bs] device arrays; NULL means the neutral value for every
 * request.  The penalizer state is indexed by the request's pool slot, like the seed pool. */
typedef struct gr_sampling {
  int vocab;                    /* 1 .. 65,024; larger is GR_ERR_ARG */
  int filter;                   /* gr_filter_mode */
  const float* temperature;     /* > 0 (a greedy request has top_k = 1) */
  const int32_t* top_k;         /* >= 1; >= vocab keeps every token */
  const float* top_p;           /* (0, 1] */
  const float* min_p;           /* [0, 1) */
  int n_order;                  /* penalizers the batch uses, in the orchestrator's order (gr_penalty_op) */
  int order[4];
  const float* repetition;      /* 1 = off */
  const float* frequency;       /* 0 = off */
  const float* presence;        /* 0 = off */
  const int32_t* min_new_tokens;
  const int32_t* stop_ids;      /* [bs, n_stop] (-1 pads): masked while the output is shorter than min_new_tokens */
  int n_stop;
  float* st_rep;                /* [pool, vocab]: 1 where unseen, the repetition penalty where seen */
  float* st_freq;               /* [pool, vocab]: the frequency penalty added once per occurrence */
  float* st_pres;               /* [pool, vocab]: the presence penalty where seen */
  int32_t* st_len;              /* [pool]: output tokens so far */
  const int64_t* req_pool_idx;  /* [bs] */
  const uint32_t* allowed;      /* grammar: [rows, ceil(vocab / 32)] allowed-token bits, or NULL */
  const float* logit_bias;      /* [bs, vocab] or NULL */
  uint64_t* rng;                /* [2] = seed, round; gr_commit_sampled advances the round */
} gr_sampling;

/* rows[i] = src[i * src_stride_rows] (row_bytes each, 16-byte multiples): the draft's boundary-token rows for their
 * lm_head pass. */
int gr_gather_rows(const void* src, int row_bytes, int n, int src_stride_rows, void* dst, void* stream);

/* In place on logits [bs*K, vocab] fp32, row (b, j): the penalizers in s->order with the request's penalizer state
 * plus the verify ids cand[b, 1..j] (cand [bs, K]; NULL with K = 1, the first-token rows), the min_new_tokens stop-id
 * mask while st_len + j < min_new_tokens, the grammar mask (disallowed -> -inf), then logit_bias.
 * Replaces selfspec_sampling.py penalize_rows (:120-170) and process_verify_logits (selfspec_fast_commit.py:170-195). */
int gr_logits_process(float* logits, int bs, int K, const int32_t* cand, const gr_sampling* s, void* stream);

/* AR's target distribution of each row (softmax(logits / T) filtered by s->filter; the row is overwritten with
 * exp(x - max), except a row whose every token is masked: it keeps its logits and sets GR_ERR_NO_TOKEN), then:
 * K = 1 (first-token rows): sample[b] = a draw with coin `first_kind` (GR_COIN_FIRST for a0,
 * GR_COIN_PREFILL for the prefill's token), also written to first_out[b * first_stride] when given; K > 1 (verify
 * rows, cand [bs, K] = [a0, d1..]): accept[r] = coin(ACCEPT, b, j) <= p_j(d_{j+1}) (0 on the last row),
 * sample[r] = a draw from p_j without d_{j+1} with coin(FINAL, b), p_next[r] = p_j(d_{j+1}).  Coins are
 * Philox-4x32-10 of (seed; round, b, j | kind << 24).
 * Replaces verify_target_probs (selfspec_sampling.py:245-275), the sampler's a0 draw and the per-row half of
 * tree_speculative_sampling_target_only (selfspec_fast_commit.py:197-230). */
int gr_sample_rows(float* logits, int bs, int K, const int32_t* cand, const gr_sampling* s, int first_kind,
                   int32_t* accept, int32_t* sample, float* p_next, int32_t* first_out, int first_stride,
                   int32_t* status, void* stream);

/* gr_accept_commit for a sampled verify: acc = the first row j < K-1 with accept == 0 (else K-1); the verified tokens
 * are v[j] = am[j+1] for j < acc and v[acc] = sample[acc], written to predict [bs*K] (zeros past acc); then the same
 * packed row, seed, seq_lens, released positions and counters as gr_accept_commit, and the round counter s->rng[1]
 * advances.  The chain half of tree_speculative_sampling_target_only plus _ss_commit_kernel. */
int gr_commit_sampled(int bs, int K, const int32_t* am, const int32_t* accept, const int32_t* sample, int64_t* seeds,
                      const int64_t* req_pool_idx, int64_t* seq_lens, int32_t* predict, int32_t* packed,
                      int64_t* released, int32_t* n_released, int64_t* out_next, int32_t* n_committed,
                      int32_t* rounds, int32_t* accept_len, uint64_t* rng, void* stream);

/* Penalizer cumulation of committed tokens: for request b the tokens[b * stride + i], i < (counts ? counts[b] + add
 * : add); repetition / presence state set, frequency state increased by the penalty per occurrence, st_len advanced.
 * Replaces selfspec_sampling.py cumulate_block (:60-100) and the worker's a0 cumulation (:523-527). */
int gr_penalty_cumulate(int bs, const int32_t* tokens, int stride, const int32_t* counts, int add,
                        const gr_sampling* s, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GRAVITY_B200_H */
