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
