// Exact brute-force K-nearest-neighbour selection over 2/3/4-D points.
//
// Semantics follow the streaming top-K of the reference Triton kernels
// (src/layers/kernels/knn.py:258-338, :422-471): squared distance
// dx*dx + dy*dy (+ dz*dz ...) in fp32, evaluated left to right with every
// product and sum rounded separately, candidates streamed in ascending index
// order and inserted when strictly closer than the current K-th best, so that
// ties keep the lower index.  The reference only has kernels for K <= 8 and
// hands larger K to cdist + topk (knn.py:1312), whose tie order is undefined;
// here the same exact rule covers every K up to 256.
//
// Design: one warp per query.  The query's sorted top-K list is distributed
// across the warp (slot s = j*32 + lane, KPL = ceil(K/32) slots per lane), so
// an insertion is a warp-wide shift by one slot done with two shuffles per
// register.  Reference points are staged per block in shared memory in tiles;
// every lane evaluates one reference point per step and a ballot selects the
// few that beat the current K-th entry, which are then inserted.  The list is
// ordered by (distance, index), which selects exactly the same K points in
// the same order as the reference's ascending-index scan with strict '<'.
#include "common.cuh"
#include "deform_grid.cuh"

namespace affb {

constexpr int KNN_WARPS = 16;
constexpr int KNN_TILE = 2048;

template <int D>
__device__ __forceinline__ float sqdist(const float* q, const float* r) {
  float acc = 0.f;
#pragma unroll
  for (int d = 0; d < D; ++d) {
    const float df = __fsub_rn(q[d], r[d]);
    const float p = __fmul_rn(df, df);
    acc = (d == 0) ? p : __fadd_rn(acc, p);
  }
  return acc;
}

template <typename T, int D, int KPL>
__global__ void __launch_bounds__(KNN_WARPS * 32)
knn_kernel(const T* __restrict__ query, const T* __restrict__ ref, int64_t M, int64_t N, int K,
           int64_t* __restrict__ out) {
  __shared__ float sref[D][KNN_TILE];  // tile position r stored at slot (r % S) * 32 + r / S
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t qi = (int64_t)blockIdx.x * KNN_WARPS + warp;
  const bool active = qi < M;

  float qp[D];
#pragma unroll
  for (int d = 0; d < D; ++d) qp[d] = active ? ldf(query + (b * M + qi) * D + d) : 0.f;

  float ld[KPL];
  int li[KPL];
#pragma unroll
  for (int j = 0; j < KPL; ++j) { ld[j] = 1e38f; li[j] = 0; }
  float kth = 1e38f;
  int kth_i = 0;  // empty slots hold (1e38, 0), as in the reference's initial state
  const int kj = (K - 1) >> 5, kl = (K - 1) & 31;

  const T* rb = ref + b * N * D;
  for (int64_t t0 = 0; t0 < N; t0 += KNN_TILE) {
    const int tn = (N - t0) < KNN_TILE ? (int)(N - t0) : KNN_TILE;
    const int S = (tn + 31) >> 5;
    __syncthreads();
    for (int i = threadIdx.x; i < tn; i += blockDim.x) {
      const int slot = (i % S) * 32 + i / S;
#pragma unroll
      for (int d = 0; d < D; ++d) sref[d][slot] = ldf(rb + (t0 + i) * D + d);
    }
    __syncthreads();
    if (!active) continue;
    // Lane l scans tile positions l*S .. l*S + S - 1, so the 32 candidates of
    // a step are spread over the tile; spatially ordered inputs then shrink
    // the K-th distance quickly and few candidates are inserted.  Insertion
    // compares (distance, index) lexicographically, so the scan order does
    // not change the result.
    for (int step = 0; step < S; ++step) {
      const int r = lane * S + step;
      float dist = 0.f;
      bool cand = false;
      if (r < tn) {
        float rp[D];
#pragma unroll
        for (int d = 0; d < D; ++d) rp[d] = sref[d][step * 32 + lane];
        dist = sqdist<D>(qp, rp);
        cand = dist < kth || (dist == kth && (int)(t0 + r) < kth_i);
      }
      unsigned bal = __ballot_sync(0xffffffffu, cand);
      while (bal) {
        const int src = __ffs(bal) - 1;
        bal &= bal - 1;
        const float cd = __shfl_sync(0xffffffffu, dist, src);
        const int ci = (int)t0 + src * S + step;
        if (!(cd < kth || (cd == kth && ci < kth_i))) continue;  // threshold moved since the ballot
        int cnt = 0;
#pragma unroll
        for (int j = 0; j < KPL; ++j) cnt += (ld[j] < cd) || (ld[j] == cd && li[j] < ci);
        const int pos = __reduce_add_sync(0xffffffffu, cnt);
        float nd[KPL];
        int ni[KPL];
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
          float up_d = __shfl_up_sync(0xffffffffu, ld[j], 1);
          int up_i = __shfl_up_sync(0xffffffffu, li[j], 1);
          if (j > 0) {
            const float wd = __shfl_sync(0xffffffffu, ld[j - 1], 31);
            const int wi = __shfl_sync(0xffffffffu, li[j - 1], 31);
            if (lane == 0) { up_d = wd; up_i = wi; }
          }
          const int s2 = j * 32 + lane;
          nd[j] = s2 < pos ? ld[j] : (s2 == pos ? cd : up_d);
          ni[j] = s2 < pos ? li[j] : (s2 == pos ? ci : up_i);
        }
        float kv = 0.f;
        int ki = 0;
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
          ld[j] = nd[j];
          li[j] = ni[j];
          if (j == kj) { kv = nd[j]; ki = ni[j]; }
        }
        kth = __shfl_sync(0xffffffffu, kv, kl);
        kth_i = __shfl_sync(0xffffffffu, ki, kl);
      }
    }
  }
  if (!active) return;
  int64_t* o = out + (b * M + qi) * K;
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    const int s = j * 32 + lane;
    if (s < K) o[s] = li[j];
  }
}

// Offers the warp's 32 candidates (dist, idx, cand per lane) to the query's
// top-K list, distributed over the warp as in knn_kernel, in lane order.
template <int KPL>
__device__ __forceinline__ void warp_offer(float dist, int idx, bool cand, float (&ld)[KPL], int (&li)[KPL],
                                           float& kth, int& kth_i, int kj, int kl) {
  const int lane = threadIdx.x & 31;
  unsigned bal = __ballot_sync(0xffffffffu, cand);
  while (bal) {
    const int src = __ffs(bal) - 1;
    bal &= bal - 1;
    const float cd = __shfl_sync(0xffffffffu, dist, src);
    const int ci = __shfl_sync(0xffffffffu, idx, src);
    if (!(cd < kth || (cd == kth && ci < kth_i))) continue;
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < KPL; ++j) cnt += (ld[j] < cd) || (ld[j] == cd && li[j] < ci);
    const int pos = __reduce_add_sync(0xffffffffu, cnt);
    float nd[KPL];
    int ni[KPL];
#pragma unroll
    for (int j = 0; j < KPL; ++j) {
      float up_d = __shfl_up_sync(0xffffffffu, ld[j], 1);
      int up_i = __shfl_up_sync(0xffffffffu, li[j], 1);
      if (j > 0) {
        const float wd = __shfl_sync(0xffffffffu, ld[j - 1], 31);
        const int wi = __shfl_sync(0xffffffffu, li[j - 1], 31);
        if (lane == 0) { up_d = wd; up_i = wi; }
      }
      const int s2 = j * 32 + lane;
      nd[j] = s2 < pos ? ld[j] : (s2 == pos ? cd : up_d);
      ni[j] = s2 < pos ? li[j] : (s2 == pos ? ci : up_i);
    }
    float kv = 0.f;
    int ki = 0;
#pragma unroll
    for (int j = 0; j < KPL; ++j) {
      ld[j] = nd[j];
      li[j] = ni[j];
      if (j == kj) { kv = nd[j]; ki = ni[j]; }
    }
    kth = __shfl_sync(0xffffffffu, kv, kl);
    kth_i = __shfl_sync(0xffffffffu, ki, kl);
  }
}

// 2-D KNN through the uniform grid of the reference points (deform_grid.cuh):
// one warp per query visits rings of cells around the query's cell; a ring is
// at most 4r runs of consecutive cells, i.e. contiguous point segments, which
// the warp scans 32 points at a time with the same (distance, index) top-K
// insertion as knn_kernel.  The walk stops once the distance to the unvisited
// region exceeds the K-th best, so the result equals the brute-force scan.
template <int KPL>
__global__ void __launch_bounds__(KNN_WARPS * 32)
knn2d_grid_kernel(const float* __restrict__ query, GridView gv, int64_t M, int K, int64_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int64_t qi = (int64_t)blockIdx.x * KNN_WARPS + (threadIdx.x >> 5);
  if (qi >= M) return;
  const float qx = query[(b * M + qi) * 2], qy = query[(b * M + qi) * 2 + 1];
  float ld[KPL];
  int li[KPL];
#pragma unroll
  for (int j = 0; j < KPL; ++j) { ld[j] = 1e38f; li[j] = 0; }
  float kth = 1e38f;
  int kth_i = 0;
  const int kj = (K - 1) >> 5, kl = (K - 1) & 31;
  const float* P = gv.params + b * 8;
  const int G = gv.G;
  const int32_t* st = gv.start + b * ((int64_t)G * G + 1);
  const float4* pts = gv.pts + b * gv.Nkv;
  int cx = cell_coord((qx - P[0]) * P[4], G), cy = cell_coord((qy - P[1]) * P[5], G);
  if (!(qx == qx) || !(qy == qy)) { cx = 0; cy = 0; }
  const float slack = grid_slack(P, G, qx, qy);
  auto scan = [&](int s0, int s1) {
    for (int base = s0; base < s1; base += 32) {
      const int t = base + lane;
      const bool valid = t < s1;
      float dist = 0.f;
      int idx = 0;
      if (valid) {
        const float4 p = pts[t];
        dist = sqdist2(qx, qy, p.x, p.y);
        idx = __float_as_int(p.z);
      }
      const bool cand = valid && (dist < kth || (dist == kth && idx < kth_i));
      warp_offer<KPL>(dist, idx, cand, ld, li, kth, kth_i, kj, kl);
    }
  };
  for (int r = 0; r <= G; ++r) {
    const int x0 = cx - r, x1 = cx + r, y0 = cy - r, y1 = cy + r;
    const int ylo = max(y0, 0), yhi = min(y1, G - 1), xlo = max(x0, 0), xhi = min(x1, G - 1);
    for (int yy = ylo; yy <= yhi; ++yy) {
      const int32_t* rs = st + (int64_t)yy * G;
      if (yy == y0 || yy == y1) {
        scan(rs[xlo], rs[xhi + 1]);
      } else {
        if (x0 >= 0) scan(rs[x0], rs[x0 + 1]);
        if (x1 < G) scan(rs[x1], rs[x1 + 1]);
      }
    }
    bool open;
    const float lb = outside_bound(P, G, x0, x1, y0, y1, qx, qy, slack, open);
    if (!open) break;
    if (kth < 1e38f && lb > 0.f && lb * lb * (1.f - 1e-5f) > kth) break;
  }
  int64_t* o = out + (b * M + qi) * K;
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    const int s2 = j * 32 + lane;
    if (s2 < K) o[s2] = li[j];
  }
}

template <typename T, int D>
static void launch_knn_d(const T* q, const T* r, int64_t B, int64_t M, int64_t N, int K,
                         int64_t* out, cudaStream_t st) {
  dim3 grid((unsigned)((M + KNN_WARPS - 1) / KNN_WARPS), (unsigned)B);
  dim3 block(KNN_WARPS * 32);
  if (K <= 32) knn_kernel<T, D, 1><<<grid, block, 0, st>>>(q, r, M, N, K, out);
  else if (K <= 64) knn_kernel<T, D, 2><<<grid, block, 0, st>>>(q, r, M, N, K, out);
  else if (K <= 128) knn_kernel<T, D, 4><<<grid, block, 0, st>>>(q, r, M, N, K, out);
  else knn_kernel<T, D, 8><<<grid, block, 0, st>>>(q, r, M, N, K, out);
}

}  // namespace affb

using namespace affb;

extern "C" int affb_knn(const void* query, const void* ref, int dtype, int64_t B, int64_t M,
                        int64_t N, int D, int K, int64_t* out_idx, void* stream) {
  AFFB_REQUIRE(D >= 2 && D <= 4, "knn: D must be 2, 3 or 4 (got %d)", D);
  AFFB_REQUIRE(K >= 1 && K <= 256, "knn: K must be in [1, 256] (got %d)", K);
  AFFB_REQUIRE((int64_t)K <= N, "knn: k=%d exceeds number of reference points N=%lld", K,
               (long long)N);
  AFFB_REQUIRE(B >= 0 && M >= 0, "knn: negative size");
  AFFB_REQUIRE(N < (1ll << 31), "knn: N too large for int32 indices");
  AFFB_REQUIRE(B < 65536, "knn: batch too large");
  if (B == 0 || M == 0) return AFFB_OK;
  cudaStream_t st = as_stream(stream);
  AFFB_DISPATCH(dtype, T, {
    const T* q = (const T*)query;
    const T* r = (const T*)ref;
    if (D == 2) launch_knn_d<T, 2>(q, r, B, M, N, K, out_idx, st);
    else if (D == 3) launch_knn_d<T, 3>(q, r, B, M, N, K, out_idx, st);
    else launch_knn_d<T, 4>(q, r, B, M, N, K, out_idx, st);
  });
  AFFB_LAUNCH_CHECK("affb_knn");
  return AFFB_OK;
}

extern "C" int64_t affb_knn2d_workspace_bytes(int64_t B, int64_t N) {
  if (B < 0 || N < 0) return -1;
  return grid_layout(B, N).total;
}

extern "C" int affb_knn2d(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int K,
                          int64_t* out_idx, void* workspace, int64_t workspace_bytes, void* stream) {
  AFFB_REQUIRE(K >= 1 && K <= 256, "knn2d: K must be in [1, 256] (got %d)", K);
  AFFB_REQUIRE((int64_t)K <= N, "knn2d: k=%d exceeds number of reference points N=%lld", K, (long long)N);
  AFFB_REQUIRE(B >= 0 && M >= 0, "knn2d: negative size");
  AFFB_REQUIRE(N < (1ll << 31) && B < 65536, "knn2d: size too large");
  AFFB_REQUIRE(workspace_bytes >= grid_layout(B, N).total && ((uintptr_t)workspace & 255) == 0,
               "knn2d: workspace of at least affb_knn2d_workspace_bytes(B, N) bytes, 256-byte aligned");
  if (B == 0 || M == 0) return AFFB_OK;
  cudaStream_t st = as_stream(stream);
  GridView gv;
  if (int e = build_grid(ref, B, N, workspace, gv, st)) return e;
  dim3 grid((unsigned)((M + KNN_WARPS - 1) / KNN_WARPS), (unsigned)B);
  if (K <= 32) knn2d_grid_kernel<1><<<grid, KNN_WARPS * 32, 0, st>>>(query, gv, M, K, out_idx);
  else if (K <= 64) knn2d_grid_kernel<2><<<grid, KNN_WARPS * 32, 0, st>>>(query, gv, M, K, out_idx);
  else if (K <= 128) knn2d_grid_kernel<4><<<grid, KNN_WARPS * 32, 0, st>>>(query, gv, M, K, out_idx);
  else knn2d_grid_kernel<8><<<grid, KNN_WARPS * 32, 0, st>>>(query, gv, M, K, out_idx);
  AFFB_LAUNCH_CHECK("affb_knn2d");
  return AFFB_OK;
}
