// Row-wise device code of the per-launch kernels (rowwise.cu).
#pragma once

#include "params.cuh"

namespace gr {

constexpr int kMaxChunks = 4;  // groups of 8 features per thread kept in registers between the norm passes

// Sum over the nthr participating threads (thread index wt; named barrier bar_id); `red` holds 32 floats.
__device__ __forceinline__ float block_sum_bar(float v, float* red, int wt, int nthr, int bar_id) {
  v = warp_sum(v);
  const int w = wt >> 5, l = wt & 31;
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthr) : "memory");
  if (l == 0) red[w] = v;
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthr) : "memory");
  float s = 0.f;
  const int nw = nthr >> 5;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// Residual + sandwich norm of row t by nthr threads: y = sum of the y_parts split-K partials (in split order),
// h_out = h_in + w_a * rms(y), x_out = w_b * rms(h_out) (bf16).  Every load of the row (partials, h_in, both norm
// vectors) is issued before the first reduction, the partials four at a time.
// MC: 8-feature chunks per thread held in registers (hidden <= 8 * MC * nthr).
template <int MC = kMaxChunks>
__device__ __forceinline__ void resnorm_row(const ResNormParams& p, int t, int wt, int nthr, int bar_id, float* red) {
  const int H = p.hidden;
  const size_t part = (size_t)p.m * H;
  const float* yrow = p.y + (size_t)t * H;
  const float* hin = p.h_in + (size_t)t * H;
  float* hout = p.h_out + (size_t)t * H;
  __nv_bfloat16* xrow = p.x_out + (size_t)t * H;
  float yv[MC][8];
  float hv[MC][8];
  uint4 wa[MC], wb[MC];
#pragma unroll
  for (int k = 0; k < MC; ++k) {
    const int c = (wt + k * nthr) * 8;
    if (c >= H) break;
    const float4 ha = *reinterpret_cast<const float4*>(hin + c);
    const float4 hb = *reinterpret_cast<const float4*>(hin + c + 4);
    hv[k][0] = ha.x; hv[k][1] = ha.y; hv[k][2] = ha.z; hv[k][3] = ha.w;
    hv[k][4] = hb.x; hv[k][5] = hb.y; hv[k][6] = hb.z; hv[k][7] = hb.w;
    wa[k] = *reinterpret_cast<const uint4*>(p.w_a + c);
    wb[k] = *reinterpret_cast<const uint4*>(p.w_b + c);
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < MC; ++k) {
    const int c = (wt + k * nthr) * 8;
    if (c >= H) break;
#pragma unroll
    for (int i = 0; i < 8; ++i) yv[k][i] = 0.f;
    // split-K partials summed in split order, four partials' loads in flight at a time
    int s = 0;
    for (; s + 4 <= p.y_parts; s += 4) {
      float4 a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a[u] = __ldcg(reinterpret_cast<const float4*>(yrow + (s + u) * part + c));
        b[u] = __ldcg(reinterpret_cast<const float4*>(yrow + (s + u) * part + c + 4));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        yv[k][0] += a[u].x; yv[k][1] += a[u].y; yv[k][2] += a[u].z; yv[k][3] += a[u].w;
        yv[k][4] += b[u].x; yv[k][5] += b[u].y; yv[k][6] += b[u].z; yv[k][7] += b[u].w;
      }
    }
    for (; s < p.y_parts; ++s) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(yrow + s * part + c));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(yrow + s * part + c + 4));
      yv[k][0] += a.x; yv[k][1] += a.y; yv[k][2] += a.z; yv[k][3] += a.w;
      yv[k][4] += b.x; yv[k][5] += b.y; yv[k][6] += b.z; yv[k][7] += b.w;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += yv[k][i] * yv[k][i];
  }
  const float ra = rsqrtf(block_sum_bar(ss, red, wt, nthr, bar_id) / H + p.eps);
  float s2 = 0.f;
#pragma unroll
  for (int k = 0; k < MC; ++k) {
    const int c = (wt + k * nthr) * 8;
    if (c >= H) break;
    const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(&wa[k]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      yv[k][i] = hv[k][i] + __bfloat162float(w[i]) * (yv[k][i] * ra);  // now the new residual
      s2 += yv[k][i] * yv[k][i];
    }
    *reinterpret_cast<float4*>(hout + c) = make_float4(yv[k][0], yv[k][1], yv[k][2], yv[k][3]);
    *reinterpret_cast<float4*>(hout + c + 4) = make_float4(yv[k][4], yv[k][5], yv[k][6], yv[k][7]);
  }
  const float rb = rsqrtf(block_sum_bar(s2, red, wt, nthr, bar_id) / H + p.eps);
#pragma unroll
  for (int k = 0; k < MC; ++k) {
    const int c = (wt + k * nthr) * 8;
    if (c >= H) break;
    const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(&wb[k]);
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = pack_bf16(__bfloat162float(w[2 * i]) * (yv[k][2 * i] * rb),
                       __bfloat162float(w[2 * i + 1]) * (yv[k][2 * i + 1] * rb));
    *reinterpret_cast<uint4*>(xrow + c) = out;
  }
}

}  // namespace gr
