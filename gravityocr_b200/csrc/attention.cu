// Block-diffusion draft attention and causal verify attention over the paged bf16 K/V cache, sm_100a.
//
// Rows of one request and one KV head: the GQA group's G query heads x K window rows (row r = g*K + j), packed into
// m16 tiles, one compute warp per tile.  Window row j sits at position base + j, base = seq_len (+1 for verify, whose
// window starts after the committed x0).  Row j sees cache positions [0, lim(j)):
//   draft  (reference selfspec_diffusion_worker.py:702-704, fast_sampling.py:508-510): lim(0) = base + 1 (x0 is
//          causal), lim(j >= 1) = base + K (the B mask rows see the whole block, bidirectionally);
//   causal (verify, fast_sampling.py:512-514; also chunked prefill): lim(j) = base + j + 1.
// Cache layout [page][kv_head][page_size = 16][128] per layer (bf16), K and V separate.  A producer warp streams
// 64-token tiles (4 pages, both 64-dim halves of K and V) with 2-D TMA loads in the 128-byte swizzle; compute warps
// run S = Q K^T and O += P V on mma.sync m16n8k16 with an fp32 online softmax (quad shuffles).
// Split-KV: CTA (split, kv_head, request) covers cache positions [split*chunk, (split+1)*chunk); when a request needs
// more than one split, each writes (m, l, O) partials and the last split to arrive merges them in split order.
// launch_attention is the entry of both attention kernels: grids of more than one CTA per SM go to the tcgen05 kernel
// (attention_tc.cu) when its rows fit (G*K <= 128), smaller grids stay on this one (g_attention_tc selects).
#include "attention_dev.cuh"

namespace gr {

constexpr int kMinWarps = 8;  // extra warps idle in the main loop and help the split merge

// tcgen05 kernel (attention_tc.cu) where it fits: 0 never, 1 large grids (default: on grids of at most one CTA per
// SM the mma.sync kernel's shorter per-CTA latency wins), 2 every grid
int g_attention_tc = 1;

// Two instantiations (ST = pipeline stages):
//   <288, 1, 3>  one warp group (the row tiles of a request's GQA group) + producer; large batches, two CTAs per SM;
//   <288, 1, 4>  two warp groups on alternate 64-token tiles + producer; small batches, where a CTA's latency is the
//                forward's.  Tile i uses stage i % 4 and group i % 2, so each stage has one consuming group and its
//                phases stay in order.
template <int MAXT, int MINB, int ST>
__global__ void __launch_bounds__(MAXT, MINB) attention_kernel(const __grid_constant__ CUtensorMap tmk,
                                                               const __grid_constant__ CUtensorMap tmv,
                                                               const AttnParams p) {
  GR_TL_BEGIN
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int G = p.n_q_heads / p.n_kv_heads;
  const int n_mt = (G * p.K + 15) / 16;
  AttnCta c = attn_cta_layout<ST>(smem, n_mt * 16);
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(c.full + s, 1);
      mbar_init(c.empty + s, n_mt);  // one warp group consumes each tile
    }
    *c.flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }
  __syncthreads();
  if (threadIdx.x == 0) pdl_trigger();
  // blocks launch in z-major order: a longest-first request order shortens the tail of a mixed-length batch
  const int b = p.order ? p.order[blockIdx.z] : blockIdx.z;
  // the producer warp reads the split's page ids while the previous kernel finishes
  if ((threadIdx.x >> 5) == p.groups * n_mt) attn_preload_pages(p, b, blockIdx.x, threadIdx.x & 31, c.pages);
  pdl_wait();
  attention_unit<ST, true>(&tmk, &tmv, p, blockIdx.x, blockIdx.y, b, threadIdx.x, blockDim.x, 1, 2, c);
  GR_TL_END(kTlAttentionMma)
}

size_t attention_smem_bytes(int K, int G, int stages) { return 1024 + attn_region_bytes(attn_rows_pad(G, K), stages); }

template <int MAXT, int MINB, int ST>
static cudaError_t configure_attention() {
  static PerDeviceOnce configured;
  return once_per_device(configured, [] {
    auto kern = attention_kernel<MAXT, MINB, ST>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  });
}

// Whether clusters of `size` CTAs of the small-batch configuration fit on the current device (cached per device,
// size, threads and shared memory).
static bool attention_cluster_ok(int size, int threads, size_t smem) {
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
    const bool ok = cudaOccupancyMaxActiveClusters(&n, attention_kernel<288, 1, 4>, &cfg) == cudaSuccess && n >= 1;
    cudaGetLastError();  // a refused query leaves no sticky error
    return ok;
  });
}

cudaError_t launch_attention(const CUtensorMap& tmk, const CUtensorMap& tmv, const AttnParams& p,
                             cudaStream_t stream, bool pdl) {
  const int G = p.n_q_heads / p.n_kv_heads;
  const int n_mt = (G * p.K + 15) / 16;
  // Large grids: one warp group, 3 stages, small CTAs (two per SM).  Grids of at most one CTA per SM: two groups on
  // alternate tiles over 4 stages (a CTA's latency is the launch's), and at least kMinWarps warps for the merge.
  AttnParams q = p;
  const bool small = p.bs * p.n_kv_heads * p.max_splits <= 148;
  if (g_attention_tc > (small ? 1 : 0) && attention_tc_fits(p))
    return launch_attention_tc(tmk, tmv, p, small, stream, pdl);
  q.groups = (small && 2 * n_mt + 1 <= 9) ? 2 : 1;  // up to 288 threads
  int warps = q.groups * n_mt + 1;
  if (small && p.max_splits > 1 && warps < kMinWarps) warps = kMinWarps;
  if (warps * 32 > 288) return cudaErrorInvalidValue;  // more than 8 row tiles: the host rejects G*K > 128
  const int stages = small ? 4 : 3;
  cudaError_t e = small ? configure_attention<288, 1, 4>() : configure_attention<288, 1, 3>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.max_splits, p.n_kv_heads, p.bs);
  cfg.blockDim = dim3(32 * warps);
  cfg.dynamicSmemBytes = attention_smem_bytes(p.K, G, stages);
  cfg.stream = stream;
  // Small batches with split KV: the splits of a (request, kv head) form one thread-block cluster and merge their
  // partials through distributed shared memory (no global round trip, no ticket), where the device can hold such
  // clusters.
  q.cluster = (small && p.max_splits >= 2 && p.max_splits <= 16 &&
               attention_cluster_ok(p.max_splits, 32 * warps, cfg.dynamicSmemBytes)) ? 1 : 0;
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
  return small ? cudaLaunchKernelEx(&cfg, attention_kernel<288, 1, 4>, tmk, tmv, q)
               : cudaLaunchKernelEx(&cfg, attention_kernel<288, 1, 3>, tmk, tmv, q);
}

}  // namespace gr

GR_TIMELINE_EXPORTS(attention)
