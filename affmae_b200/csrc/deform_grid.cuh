// Uniform-grid spatial index of 2-D point sets (one grid per batch element)
// and an exact 4-nearest-neighbour query on it.
//
// The fused deformable attention of the reference
// (src/layers/kernels/fused_deform_attn.py:1085-1125, :1273-1290) finds the
// 4 nearest kv positions of every sample point by scanning all Nkv points
// (O(Nq*Nkv*H*4)).  Here the kv points are bucketed once per call into a
// G x G grid over their bounding box (counting sort: count, scan, scatter),
// and each sample visits grid rings around its cell until the distance to
// the unvisited region exceeds its current 4th-best distance.  Candidates are
// ranked by (fp32 squared distance, index) lexicographically, which is
// exactly the order produced by the reference's ascending-index scan with a
// strict '<' insertion, so the selected neighbours and their order match the
// brute-force result bit for bit.
#pragma once

#include "common.cuh"

namespace affb {

struct GridView {
  const float* params;   // [B][8]: minx, miny, cw, ch, inv_cw, inv_ch, -, -
  const int32_t* start;  // [B][G*G+1]
  const float4* pts;     // [B][Nkv]: x, y, index bits, 0
  int G;
  int64_t Nkv;
};

// Grid side: about AFFB_GRID_PPC points per cell.
#ifndef AFFB_GRID_PPC
#define AFFB_GRID_PPC 4
#endif
__host__ __device__ inline int grid_side(int64_t nkv) {
  int64_t g = 1;
  while (g * g * AFFB_GRID_PPC < nkv && g < 4096) ++g;
  return (int)g;
}

__host__ __device__ inline int64_t align256(int64_t x) { return (x + 255) & ~(int64_t)255; }

struct GridLayout {
  int G;
  int64_t off_params, off_start, off_cursor, off_pts, total;
};

// Byte layout of the grid inside a caller-provided workspace.
__host__ __device__ inline GridLayout grid_layout(int64_t B, int64_t nkv) {
  GridLayout L;
  L.G = grid_side(nkv);
  const int64_t ncell = (int64_t)L.G * L.G;
  L.off_params = 0;
  L.off_start = align256(B * 8 * 4);
  L.off_cursor = L.off_start + align256(B * (ncell + 1) * 4);
  L.off_pts = L.off_cursor + align256(B * ncell * 4);
  L.total = L.off_pts + align256(B * nkv * 16);
  return L;
}

__device__ __forceinline__ float sqdist2(float sx, float sy, float px, float py) {
  const float dx = __fsub_rn(sx, px), dy = __fsub_rn(sy, py);
  return __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy));
}

// Top-4 under the (distance, index) order; d[0] <= d[1] <= d[2] <= d[3].
// Empty slots hold (1e38, 0) like the reference's initial state.
struct Top4 {
  float d[4];
  int i[4];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int k = 0; k < 4; ++k) { d[k] = 1e38f; i[k] = 0; }
  }
  __device__ __forceinline__ static bool before(float da, int ia, float db, int ib) {
    return da < db || (da == db && ia < ib);
  }
  // Sorted insertion of (dd, ii) when it ranks before the 4th entry: one
  // guard compare, then selects only (no nested branches, so lanes of a warp
  // that insert at different depths do not serialise).
  __device__ __forceinline__ void offer(float dd, int ii) {
    if (!before(dd, ii, d[3], i[3])) return;
    const bool b0 = before(dd, ii, d[0], i[0]), b1 = before(dd, ii, d[1], i[1]),
               b2 = before(dd, ii, d[2], i[2]);
    d[3] = b2 ? d[2] : dd;
    i[3] = b2 ? i[2] : ii;
    d[2] = b1 ? d[1] : (b2 ? dd : d[2]);
    i[2] = b1 ? i[1] : (b2 ? ii : i[2]);
    d[1] = b0 ? d[0] : (b1 ? dd : d[1]);
    i[1] = b0 ? i[0] : (b1 ? ii : i[1]);
    d[0] = b0 ? dd : d[0];
    i[0] = b0 ? ii : i[0];
  }
};

__device__ __forceinline__ int cell_coord(float f, int G) {
  return (f >= 0.f) ? (f < (float)G ? (int)f : G - 1) : 0;
}

// Builds the grid of `nkv` points per batch element ([B, nkv, 2] fp32) in a
// workspace of grid_layout(B, nkv).total bytes (deform_knn.cu).
int build_grid(const float* pts, int64_t B, int64_t nkv, void* ws, GridView& gv, cudaStream_t st);

// Lower bound of the distance from (sx, sy) to any point outside the cells
// [x0, x1] x [y0, y1] (already visited), minus `slack`; `open` is false when
// those cells cover the whole grid.
__device__ __forceinline__ float outside_bound(const float* P, int G, int x0, int x1, int y0, int y1, float sx,
                                               float sy, float slack, bool& open) {
  const float minx = P[0], miny = P[1], cw = P[2], ch = P[3];
  float lb = 3.4e38f;
  open = false;
  if (x0 > 0) { lb = fminf(lb, sx - (minx + x0 * cw)); open = true; }
  if (x1 < G - 1) { lb = fminf(lb, (minx + (x1 + 1) * cw) - sx); open = true; }
  if (y0 > 0) { lb = fminf(lb, sy - (miny + y0 * ch)); open = true; }
  if (y1 < G - 1) { lb = fminf(lb, (miny + (y1 + 1) * ch) - sy); open = true; }
  return lb - slack;
}

// Slack for the rounding of cell assignment and of boundary positions.
__device__ __forceinline__ float grid_slack(const float* P, int G, float sx, float sy) {
  const float cw = P[2], ch = P[3];
  return 1e-4f * fmaxf(cw, ch) + 2e-6f * (fabsf(sx) + fabsf(sy) + fabsf(P[0]) + fabsf(P[1]) + G * fmaxf(cw, ch));
}

// Exact 4-NN of (sx, sy) among the points of batch element b.
//
// Square rings of cells around the sample's cell are visited until the
// distance to the unvisited region exceeds the current 4th-best distance.
// Rings 0 and 1 (the 3 x 3 block) are scanned first as three row runs: cells
// are stored row-major, so the points of three adjacent cells of a row are one
// contiguous range.  The result does not depend on the visiting order
// (candidates are ranked by (d2, index)).
#ifndef AFFB_KNN4_UNROLL
#define AFFB_KNN4_UNROLL 2
#endif
__device__ inline void grid_knn4(const GridView& g, int64_t b, float sx, float sy, Top4& top) {
  top.init();
  const float* P = g.params + b * 8;
  const float minx = P[0], miny = P[1], cw = P[2], ch = P[3], icw = P[4], ich = P[5];
  const int G = g.G;
  const int32_t* st = g.start + b * ((int64_t)G * G + 1);
  const float4* pts = g.pts + b * g.Nkv;
  int cx = cell_coord((sx - minx) * icw, G);
  int cy = cell_coord((sy - miny) * ich, G);
  if (!(sx == sx) || !(sy == sy)) { cx = 0; cy = 0; }
  // slack for the rounding of cell assignment and of boundary positions
  const float slack = 1e-4f * fmaxf(cw, ch) +
                      2e-6f * (fabsf(sx) + fabsf(sy) + fabsf(minx) + fabsf(miny) + G * fmaxf(cw, ch));
  // points t0 .. e-1: AFFB_KNN4_UNROLL loads in flight per step (2 measured best:
  // 4 raises the forward's spills at its 48-register budget)
  auto scan_range = [&](int t, int e) {
    constexpr int UR = AFFB_KNN4_UNROLL;
    for (; t + UR <= e; t += UR) {
      float4 q[UR];
#pragma unroll
      for (int u = 0; u < UR; ++u) q[u] = pts[t + u];
#pragma unroll
      for (int u = 0; u < UR; ++u) top.offer(sqdist2(sx, sy, q[u].x, q[u].y), __float_as_int(q[u].z));
    }
    for (; t < e; ++t) {
      const float4 q = pts[t];
      top.offer(sqdist2(sx, sy, q.x, q.y), __float_as_int(q.z));
    }
  };
  auto scan_run = [&](int c0, int c1) { scan_range(st[c0], st[c1 + 1]); };  // cells c0 .. c1 of one row
  {
    // the 3 x 3 block: the bounds of its three row runs are loaded together
    const int xlo = max(cx - 1, 0), xhi = min(cx + 1, G - 1);
    const int ylo = max(cy - 1, 0), yhi = min(cy + 1, G - 1);
    int rb[3], re[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int yy = min(ylo + k, yhi);
      rb[k] = st[yy * G + xlo];
      re[k] = ylo + k <= yhi ? st[yy * G + xhi + 1] : rb[k];
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) scan_range(rb[k], re[k]);
  }
  for (int r = 1; r <= G; ++r) {
    const int x0 = cx - r, x1 = cx + r, y0 = cy - r, y1 = cy + r;
    if (r >= 2) {
      const int ylo = max(y0, 0), yhi = min(y1, G - 1);
      const int xlo = max(x0, 0), xhi = min(x1, G - 1);
      for (int yy = ylo; yy <= yhi; ++yy) {
        if (yy == y0 || yy == y1) {
          scan_run(yy * G + xlo, yy * G + xhi);  // full edge row of the ring
        } else {
          if (x0 >= 0) scan_run(yy * G + x0, yy * G + x0);
          if (x1 < G) scan_run(yy * G + x1, yy * G + x1);
        }
      }
    }
    // lower bound of the distance to any point outside the visited square
    float lb = 3.4e38f;
    bool open = false;
    if (x0 > 0) { lb = fminf(lb, sx - (minx + x0 * cw)); open = true; }
    if (x1 < G - 1) { lb = fminf(lb, (minx + (x1 + 1) * cw) - sx); open = true; }
    if (y0 > 0) { lb = fminf(lb, sy - (miny + y0 * ch)); open = true; }
    if (y1 < G - 1) { lb = fminf(lb, (miny + (y1 + 1) * ch) - sy); open = true; }
    if (!open) break;
    lb -= slack;
    if (lb > 0.f && lb * lb * (1.f - 1e-5f) > top.d[3]) break;
  }
}

}  // namespace affb
