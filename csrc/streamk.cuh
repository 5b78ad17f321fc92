// Stream-K decomposition shared by the GEMM and by the kernels that consume its partial sums.
//
// A stream-K GEMM over T output tiles with K/64 = kb k-blocks per tile splits the U = T*kb
// (tile, k-block) units evenly over G CTAs: CTA c owns units [c*U/G, (c+1)*U/G).  Each CTA
// writes one fp32 partial per tile segment it touched into ws[slot][M][N], where slot = c minus
// the first CTA that touched the tile.  A consumer sums slots 0..slots(tile)-1 of an element.
#pragma once

#include "common.cuh"

namespace vlm {

struct SkMeta {
  int M, N;
  int tiles_m, tiles_n;
  int kb_count;
  int grid;
  int bm, bn;
};

// Linear tile index of (tm, tn) under the GEMM's grouped raster (groups of 16 M-tiles).
__host__ __device__ inline long long sk_tile_index(const SkMeta& m, int tm, int tn) {
  const int G = 16;
  const int gid = tm / G, first = gid * G;
  const int gsz = (m.tiles_m - first) < G ? (m.tiles_m - first) : G;
  return static_cast<long long>(gid) * G * m.tiles_n + static_cast<long long>(tn) * gsz + (tm - first);
}

__host__ __device__ inline int sk_slots(const SkMeta& m, long long tile) {
  const long long U = static_cast<long long>(m.tiles_m) * m.tiles_n * m.kb_count;
  const long long first = tile * m.kb_count, last = first + m.kb_count - 1;
  const long long c0 = ((first + 1) * m.grid - 1) / U, c1 = ((last + 1) * m.grid - 1) / U;
  return static_cast<int>(c1 - c0 + 1);
}

// Sum of the partials of 8 consecutive columns (col % 8 == 0, inside one tile) of row `row`.
VLM_DEV void sk_sum8(const float* __restrict__ ws, const SkMeta& m, int row, int col, float (&out)[8]) {
  const long long tile = sk_tile_index(m, row / m.bm, col / m.bn);
  const int ns = sk_slots(m, tile);
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = 0.f;
  const long long stride = static_cast<long long>(m.M) * m.N;
  const float* p = ws + static_cast<long long>(row) * m.N + col;
  float4 a[4], b[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    if (s < ns) {
      a[s] = __ldcg(reinterpret_cast<const float4*>(p + s * stride));
      b[s] = __ldcg(reinterpret_cast<const float4*>(p + s * stride) + 1);
    }
  }
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    if (s < ns) {
      out[0] += a[s].x; out[1] += a[s].y; out[2] += a[s].z; out[3] += a[s].w;
      out[4] += b[s].x; out[5] += b[s].y; out[6] += b[s].z; out[7] += b[s].w;
    }
  }
  for (int s = 4; s < ns; ++s) {
    const float4 x = __ldcg(reinterpret_cast<const float4*>(p + s * stride));
    const float4 y = __ldcg(reinterpret_cast<const float4*>(p + s * stride) + 1);
    out[0] += x.x; out[1] += x.y; out[2] += x.z; out[3] += x.w;
    out[4] += y.x; out[5] += y.y; out[6] += y.z; out[7] += y.w;
  }
}

}  // namespace vlm
