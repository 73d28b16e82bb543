// Neighbourhood attention on the tensor cores for cluster-block neighbour
// lists (bf16 / fp16, head_dim 32).
//
// In AFFMAE the neighbour list of a token is the concatenation of the 8
// members of its nearest clusters, and tokens are ordered so that cluster c
// is tokens [8c, 8c+8) (BasicLayer.forward, src/layers/aff.py:445-453;
// space_filling_cluster, src/utils/geometry.py:314-317).  Each list is then
// M/8 runs idx[8j .. 8j+7] = 8c_j + (0..7).  This kernel exploits that:
//   * per tile of 16 queries the union is a set of at most 16 * M/8
//     clusters, found by hashing the M/8 cluster ids of each row (not M keys);
//   * one mma n-tile (8 columns) is exactly one cluster, so the attended
//     pattern is a [16 x clusters] table of list positions j (or absent),
//     shared by all heads; bias[q, 8j + r] is read straight from the staged
//     bias rows (no per-head scatter), and dbias is stored straight from the
//     accumulator fragments;
//   * K/V rows of a cluster are 512 contiguous bytes per head.
// Semantics are those of the CUDA-core path (nbhd_row.cuh; reference
// local_attn.py:224-553).  A tile that is not of this form (or that lists a
// cluster twice in one row) runs the CUDA-core row
// code instead, so any neighbour list stays exact.
//
// Per warp and head the work is a flash-attention loop over 16-key chunks
// (two clusters): S = Q K^T on mma.sync in registers, online softmax in the
// accumulator layout, O += P V.  The backward recomputes S and dP = dO V^T,
// keeps dQ in registers and writes dbias; dK and dV come from the key-major
// pass of nbhd_attn_kv.cu, unless the call's lists are not all cluster runs,
// in which case dK = dS^T Q and dV = P^T dO are scatter-added per chunk.
#include "nbhd_tc.cuh"
#include "nbhd_mma.cuh"

namespace affb {

constexpr int CHS = 256;         // cluster hash slots
constexpr int BPT = 24;          // 16-bit row stride of the per-warp 16x16 P / dS tiles

// Tile structures for lists of at most MM neighbours (the call's M rounded up
// to 16, 32, 48 or 64), so that shared memory follows M.  The staged bias /
// dS tile of a warp is [16][M] (row stride M) followed, at offset 16 MM, by an
// 8-element block that absent clusters point at (-inf for bias, zeros for dS).
template <int MM>
struct BlkSetup {
  static constexpr int UCL = TQ * MM / 8;  // clusters per tile: every row's list, all distinct
  int uclu[UCL];                   // cluster ids of the union (key rows 8c .. 8c+7)
  int16_t boff[TQ][UCL];           // row q, cluster slot u: offset q*M + 8j of its bias run in the
                                   // staged tile (list position j), 16 MM when q does not list it
  int hkey[CHS], hval[CHS];
  int warp_tot[NW];
  int fail;
};

template <typename T, int MM>
struct BlkWarpFwd {
  alignas(16) T Q[TQ * TD];
  alignas(16) T bias[TQ * MM + 8];
  alignas(16) T KV[2][2][16 * TD];
};
template <typename T, int MM>
struct BlkWarpBwd {
  alignas(16) T Q[TQ * TD];
  alignas(16) T dO[TQ * TD];
  alignas(16) T bias[TQ * MM + 8];
  alignas(16) T KV[2][2][16 * TD];
  alignas(16) T P[TQ * BPT];
  alignas(16) T dS[TQ * BPT];
};
template <typename T, int MM>
struct BlkWarpDq {
  alignas(16) T dS[TQ * MM + 8];
  alignas(16) T K[2][16 * TD];
};
// A tile's cluster union as the forward built it, kept for the dQ kernel of
// the backward (same neighbour lists and mask): nclu (-1 for a tile that is
// not of cluster-run form), the cluster ids and the run-offset table.
template <int MM>
struct TilePlan {
  int nclu;
  int pad[3];
  int uclu[BlkSetup<MM>::UCL];
  int16_t boff[TQ][BlkSetup<MM>::UCL];
};

template <int MM>
__device__ __forceinline__ void tile_plan_store(TilePlan<MM>* tp, const BlkSetup<MM>& s, int nclu) {
  const int t = threadIdx.x;
  if (t == 0) tp->nclu = nclu;
  if (nclu <= 0) return;
  for (int i = t; i < nclu; i += TC_THREADS) tp->uclu[i] = s.uclu[i];
  for (int i = t; i < TQ * nclu; i += TC_THREADS) {
    const int r = i / nclu, u = i - r * nclu;
    tp->boff[r][u] = s.boff[r][u];
  }
}

// Returns the tile's nclu; its tables are in s after the block barrier.  The
// chunk loops read cluster slots in pairs, so with an odd count the slot
// after the last one is set to the absent-cluster offset, as blk_setup
// leaves it.
template <int MM>
__device__ __forceinline__ int tile_plan_load(const TilePlan<MM>* tp, BlkSetup<MM>& s) {
  const int t = threadIdx.x;
  const int nclu = tp->nclu;
  if (nclu > 0) {
    const int ncol = min(nclu + (nclu & 1), BlkSetup<MM>::UCL);
    for (int i = t; i < nclu; i += TC_THREADS) s.uclu[i] = tp->uclu[i];
    for (int i = t; i < TQ * ncol; i += TC_THREADS) {
      const int r = i / ncol, u = i - r * ncol;
      s.boff[r][u] = u < nclu ? tp->boff[r][u] : (int16_t)(TQ * MM);
    }
  }
  __syncthreads();
  return nclu;
}

// The staged neighbour rows are read only by the setup, before any warp
// buffer is written, so they share storage with the warps' buffers.
template <int MM, typename W>
struct BlkSmem {
  BlkSetup<MM> setup;
  union U {
    int idx[TQ * MM];
    W w[NW];
  } u;
};
template <typename T, int MM> using BlkFwdSmem = BlkSmem<MM, BlkWarpFwd<T, MM>>;
template <typename T, int MM> using BlkBwdSmem = BlkSmem<MM, BlkWarpBwd<T, MM>>;
template <typename T, int MM> using BlkDqSmem = BlkSmem<MM, BlkWarpDq<T, MM>>;

// True when list column `col` of query n is masked (mask == 0) in every mask
// head: the only form in which a run may extend past the last token.
__device__ __forceinline__ bool run_slot_masked(const NbhdArgs& a, int b, int n, int col) {
  if (!a.mask) return false;
  for (int hm = 0; hm < a.mask_heads; ++hm)
    if (a.mask[(((int64_t)b * a.mask_heads + hm) * a.N + n) * a.M + col] != 0) return false;
  return true;
}

__device__ __forceinline__ uint32_t clu_slot(int key) { return ((uint32_t)key * 2654435761u) >> 24; }

// Checks the cluster-block form of the tile and builds its cluster union.
// Returns the number of clusters, or -1 when the tile needs the general path.
template <int MM>
__device__ int blk_setup(BlkSetup<MM>& s, int* sidx, const NbhdArgs& a, int b, int n0, int nq) {
  const int N = a.N, M = a.M;
  const int32_t* __restrict__ midx = a.midx;
  const int t = threadIdx.x;
  const int J = M >> 3;  // clusters per list
  {
    const int32_t* src = midx + ((int64_t)b * N + n0) * M;
    const int nch = TQ * M / 4;  // 16-byte chunks of int32
    for (int i = t; i < nch; i += TC_THREADS) {
      const bool ok = (i * 4) / M < nq;
      cp_async16(sidx + i * 4, src + (ok ? i * 4 : 0), ok);
    }
    cp_commit();
  }
  for (int i = t; i < CHS; i += TC_THREADS) s.hkey[i] = -1;
  for (int i = t; i < TQ * BlkSetup<MM>::UCL / 2; i += TC_THREADS)
    reinterpret_cast<int*>(&s.boff[0][0])[i] = (TQ * MM) | ((TQ * MM) << 16);
  if (t == 0) s.fail = 0;
  cp_wait<0>();
  __syncthreads();
  // item (q, j) per thread: verify the run, insert its cluster id
  int cid = -1;
  const int q = t / 8, j = t % 8;  // TQ * 8 = 128 items cover J <= 8
  if (q < nq && j < J) {
    const int* run = sidx + q * M + 8 * j;
    const int c0 = run[0];
    bool ok = c0 >= 0 && (c0 & 7) == 0 && c0 < N;
#pragma unroll
    for (int r = 1; r < 8; ++r)  // past the last token: a masked padding slot of a partial last cluster
      ok = ok && (c0 + r < N ? run[r] == c0 + r : run_slot_masked(a, b, n0 + q, 8 * j + r));
    for (int jj = 0; jj < j; ++jj) ok = ok && sidx[q * M + 8 * jj] != c0;  // listed twice in one row
    if (ok) {
      cid = c0 >> 3;
      uint32_t h = clu_slot(cid);
      while (true) {
        const int old = atomicCAS(&s.hkey[h], -1, cid);
        if (old == -1 || old == cid) break;
        h = (h + 1) & (CHS - 1);
      }
    } else {
      s.fail = 1;
    }
  }
  __syncthreads();
  if (s.fail) return -1;
  // compact occupied slots (2 per thread) with a block scan
  const int lane = t & 31, w = t >> 5;
  const int c = (s.hkey[2 * t] >= 0) + (s.hkey[2 * t + 1] >= 0);
  int x = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s.warp_tot[w] = x;
  __syncthreads();
  int base = 0, total = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    if (i < w) base += s.warp_tot[i];
    total += s.warp_tot[i];
  }
  int pos = base + x - c;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int key = s.hkey[2 * t + i];
    if (key >= 0) {
      s.hval[2 * t + i] = pos;
      s.uclu[pos] = key;
      ++pos;
    }
  }
  __syncthreads();
  if (cid >= 0) {
    uint32_t h = clu_slot(cid);
    while (s.hkey[h] != cid) h = (h + 1) & (CHS - 1);
    s.boff[q][s.hval[h]] = (int16_t)(q * M + 8 * j);  // one writer per slot: duplicates rejected above
  }
  __syncthreads();
  return total;
}

// Staged bias tile of one warp: rows [16][M] of bias (zeros without bias),
// -inf where the mask is 0, and the -inf block at offset 16 MM for absent clusters.
// Called once the bias cp.async group has completed.
template <typename T, int MM>
__device__ __forceinline__ void warp_finish_bias(T* sb, const NbhdArgs& a, const uint8_t* mrow, int nq) {
  const int lane = threadIdx.x & 31, M = a.M;
  const T ninf = neg_inf<T>();
  if (!a.bias) {
    const T zero = pos_zero<T>();
    for (int i = lane; i < TQ * M; i += 32) sb[i] = zero;
  }
  if (mrow)
    for (int i = lane; i < nq * M; i += 32)
      if (mrow[i] == 0) sb[i] = ninf;
  if (lane < 8) sb[TQ * MM + lane] = ninf;
  __syncwarp();
}

// Bias pair at tile offset bo (columns 2tq, 2tq+1 of the run).
template <typename T>
__device__ __forceinline__ void bias_at(const T* sb, int bo, int tq, float& b0, float& b1) {
  const uint32_t u = *reinterpret_cast<const uint32_t*>(sb + bo + 2 * tq);
  const T* hp = reinterpret_cast<const T*>(&u);
  b0 = io<T>::ld(hp);
  b1 = io<T>::ld(hp + 1);
}

// cp.async of the K rows of cluster slots 2c, 2c+1 (16 keys), zeros past nclu.
template <typename T>
__device__ __forceinline__ void warp_load_k(T* dk, const T* __restrict__ kb, const int* uclu, int c, int nclu,
                                            int N) {
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, piece = lane & 3;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int u = 2 * c + hh;
    const int key = u < nclu ? uclu[u] * 8 + r : N;
    const bool ok = key < N;  // rows past the last token (partial last cluster) read as zeros
    const int64_t src = (int64_t)(ok ? key : 0) * TD + piece * 8;
    cp_async16(dk + swz(hh * 8 + r, piece), kb + src, ok);
  }
}

// cp.async of the K and V rows of cluster slots 2c, 2c+1 (16 keys), zeros past nclu.
template <typename T>
__device__ __forceinline__ void warp_load_kv(T* dk, T* dv, const T* __restrict__ kb, const T* __restrict__ vb,
                                             const int* uclu, int c, int nclu, int N) {
  const int lane = threadIdx.x & 31;
  const int r = lane >> 2, piece = lane & 3;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int u = 2 * c + hh;
    const int key = u < nclu ? uclu[u] * 8 + r : N;
    const bool ok = key < N;  // rows past the last token (partial last cluster) read as zeros
    const int64_t src = (int64_t)(ok ? key : 0) * TD + piece * 8;
    const int dst = swz(hh * 8 + r, piece);
    cp_async16(dk + dst, kb + src, ok);
    cp_async16(dv + dst, vb + src, ok);
  }
}

template <typename T, int MM>
__device__ void blk_fwd_head(const NbhdArgs& a, const BlkSetup<MM>& s, BlkWarpFwd<T, MM>& w, int b, int h, int n0,
                             int nq, int nclu) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int N = a.N, M = a.M;
  const int nchunk = (nclu + 1) / 2;
  const int64_t bh = (int64_t)b * a.H + h;
  const T* kb = (const T*)a.k + bh * N * TD;
  const T* vb = (const T*)a.v + bh * N * TD;
  const int* uclu = s.uclu;
  warp_load16(w.Q, (const T*)a.q + (bh * N + n0) * TD, [=](int i) -> int64_t { return i < nq ? i : -1; });
  if (a.bias) warp_stage_bias(w.bias, a, b, h, n0, nq);
  cp_commit();
  warp_load_kv(w.KV[0][0], w.KV[0][1], kb, vb, uclu, 0, nclu, N);
  cp_commit();
  const uint8_t* mrow = a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0) * M : nullptr;
  int ex[2] = {0, 0};
  if (mrow) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int row = g + hf * 8;
      int cnt = 0;
      if (row < nq)
        for (int e = tq; e < M; e += 4) cnt += mrow[row * M + e] == 0;
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
      ex[hf] = cnt;
    }
  }
  cp_wait<1>();
  __syncwarp();
  warp_finish_bias<T, MM>(w.bias, a, mrow, nq);
  uint32_t aq[2][4];
  load_a_frags(aq, w.Q);
  float sbv[2] = {-INFINITY, -INFINITY};
  if (a.blank_k) {
    rows_dot(w.Q, (const T*)a.blank_k + (int64_t)h * TD, sbv[0], sbv[1]);
    sbv[0] *= a.scale;
    sbv[1] *= a.scale;
  }
  // running max m per row (natural units) and m * log2(e), the offset of the
  // base-2 exponentials p = 2^(s * log2(e) - m * log2(e))
  float m[2] = {-1e11f, -1e11f}, m2[2] = {-1e11f * kLog2e, -1e11f * kLog2e}, l[2] = {0.f, 0.f};
  float o[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  for (int c = 0; c < nchunk; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunk) warp_load_kv(w.KV[buf ^ 1][0], w.KV[buf ^ 1][1], kb, vb, uclu, c + 1, nclu, N);
    cp_commit();
    cp_wait<1>();
    __syncwarp();
    float x[2][4];
    mma_chunk_nt<T>(x, aq, w.KV[buf][0], 0);
    float cm[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = g + hf * 8;
        float b0, b1;
        bias_at(w.bias, s.boff[row][2 * c + nt], tq, b0, b1);
        x[nt][2 * hf] = fmaf(x[nt][2 * hf], a.scale, b0);
        x[nt][2 * hf + 1] = fmaf(x[nt][2 * hf + 1], a.scale, b1);
        cm[hf] = fmaxf(cm[hf], fmaxf(x[nt][2 * hf], x[nt][2 * hf + 1]));
      }
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      cm[hf] = fmaxf(cm[hf], __shfl_xor_sync(0xffffffffu, cm[hf], 1));
      cm[hf] = fmaxf(cm[hf], __shfl_xor_sync(0xffffffffu, cm[hf], 2));
    }
    // rescale O and l only when some row of the warp has a new maximum
    if (__any_sync(0xffffffffu, cm[0] > m[0] || cm[1] > m[1])) {
      float al[2];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const float nm = fmaxf(m[hf], cm[hf]);
        al[hf] = ex2_approx((m[hf] - nm) * kLog2e);
        m[hf] = nm;
        m2[hf] = nm * kLog2e;
        l[hf] *= al[hf];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) { o[i][0] *= al[0]; o[i][1] *= al[0]; o[i][2] *= al[1]; o[i][3] *= al[1]; }
    }
    float p[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p[nt][e] = ex2_approx(fmaf(x[nt][e], kLog2e, -m2[e >> 1]));
        l[e >> 1] += p[nt][e];
      }
    const uint32_t pa[4] = {pack2<T>(p[0][0], p[0][1]), pack2<T>(p[0][2], p[0][3]),
                            pack2<T>(p[1][0], p[1][1]), pack2<T>(p[1][2], p[1][3])};
    mma_chunk_pv<T>(o, pa, w.KV[buf][1], 0);
    __syncwarp();
  }
  const int pad = padded_neighbours(M) - M;
  const T* bvp = a.blank_v ? (const T*)a.blank_v + (int64_t)h * TD : nullptr;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    float lf = l[hf];
    lf += __shfl_xor_sync(0xffffffffu, lf, 1);
    lf += __shfl_xor_sync(0xffffffffu, lf, 2);
    const float mm = a.blank_k ? fmaxf(m[hf], sbv[hf]) : m[hf];
    const float alf = expf(m[hf] - mm);
    const float pb = a.blank_k ? expf(sbv[hf] - mm) : 0.f;
    lf = lf * alf + pb + (float)(ex[hf] + pad) * expf(-1e11f - mm);
    const int row = g + hf * 8;
    if (row >= nq) continue;
    const float lse = mm + logf(lf + 1e-12f);
    const float inv = expf(mm - lse);
    T* orow = (T*)a.out + (bh * N + n0 + row) * TD;
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) {
      const int col = dt * 8 + 2 * tq;
      float v0 = o[dt][2 * hf] * alf, v1 = o[dt][2 * hf + 1] * alf;
      if (bvp) { v0 += pb * ldf(bvp + col); v1 += pb * ldf(bvp + col + 1); }
      *reinterpret_cast<uint32_t*>(orow + col) = pack2<T>(v0 * inv, v1 * inv);
    }
    if (tq == 0) a.lse[bh * N + n0 + row] = lse;
  }
}

template <typename T, int MM>
__global__ void __launch_bounds__(TC_THREADS, AFFB_FWD_MINB) nbhd_blk_fwd_kernel(NbhdArgs a) {
  dependent_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BlkFwdSmem<T, MM>& s = *reinterpret_cast<BlkFwdSmem<T, MM>*>(smem_raw);
  const int N = a.N;
  const int tiles = (N + TQ - 1) / TQ;
  const int b = blockIdx.x / tiles;
  const int n0 = (blockIdx.x % tiles) * TQ;
  const int nq = min(TQ, N - n0);
  const int nclu = blk_setup<MM>(s.setup, s.u.idx, a, b, n0, nq);
  if (a.tile_plan) tile_plan_store<MM>(reinterpret_cast<TilePlan<MM>*>(a.tile_plan) + blockIdx.x, s.setup, nclu);
  const int warp = threadIdx.x >> 5;
  if (nclu < 0) {  // not cluster-block lists: CUDA-core rows
    for (int w = warp; w < a.H * nq; w += NW) nbhd_fwd_row<T, 4>(a, b, w / nq, n0 + w % nq);
    return;
  }
  for (int h = warp; h < a.H; h += NW) blk_fwd_head<T, MM>(a, s.setup, s.u.w[warp], b, h, n0, nq, nclu);
}

// Full backward of one head for calls whose lists are not all cluster runs:
// dQ, dbias and the blank-token gradients, with dK / dV scatter-added into
// the fp32 sums a.dk / a.dv.
template <typename T, int MM>
__device__ void blk_bwd_head(const NbhdArgs& a, const BlkSetup<MM>& s, BlkWarpBwd<T, MM>& w, int b, int h, int n0,
                             int nq, int nclu) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int N = a.N, M = a.M;
  const int U = nclu * 8, nchunk = (nclu + 1) / 2;
  const int64_t bh = (int64_t)b * a.H + h;
  const T* kb = (const T*)a.k + bh * N * TD;
  const T* vb = (const T*)a.v + bh * N * TD;
  const int* uclu = s.uclu;
  auto rows_q = [=](int i) -> int64_t { return i < nq ? i : -1; };
  warp_load16(w.Q, (const T*)a.q + (bh * N + n0) * TD, rows_q);
  warp_load16(w.dO, (const T*)a.dout + (bh * N + n0) * TD, rows_q);
  if (a.bias) warp_stage_bias(w.bias, a, b, h, n0, nq);
  cp_commit();
  warp_load_kv(w.KV[0][0], w.KV[0][1], kb, vb, uclu, 0, nclu, N);
  cp_commit();
  const uint8_t* mrow = a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0) * M : nullptr;
  float dl[2], ls[2];
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int row = g + hf * 8;
    float p = 0.f;
    ls[hf] = 0.f;
    if (row < nq) {
      float ov[8], dv[8];
      ld8((const T*)a.o + (bh * N + n0 + row) * TD + tq * 8, ov);
      ld8((const T*)a.dout + (bh * N + n0 + row) * TD + tq * 8, dv);
#pragma unroll
      for (int e = 0; e < 8; ++e) p = fmaf(ov[e], dv[e], p);
      ls[hf] = a.lse[bh * N + n0 + row];
    }
    p += __shfl_xor_sync(0xffffffffu, p, 1);
    p += __shfl_xor_sync(0xffffffffu, p, 2);
    dl[hf] = p;
  }
  cp_wait<1>();
  __syncwarp();
  warp_finish_bias<T, MM>(w.bias, a, mrow, nq);
  uint32_t aq[2][4], ado[2][4];
  load_a_frags(aq, w.Q);
  load_a_frags(ado, w.dO);
  float dsb[2] = {0.f, 0.f};
  if (a.blank_k) {
    float sb[2], dpb[2], pbv[2];
    rows_dot(w.Q, (const T*)a.blank_k + (int64_t)h * TD, sb[0], sb[1]);
    rows_dot(w.dO, (const T*)a.blank_v + (int64_t)h * TD, dpb[0], dpb[1]);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      pbv[hf] = (g + hf * 8) < nq ? expf(sb[hf] * a.scale - ls[hf]) : 0.f;
      dsb[hf] = pbv[hf] * (dpb[hf] - dl[hf]);
    }
    float gk = 0.f, gv = 0.f;
#pragma unroll
    for (int row = 0; row < TQ; ++row) {
      const int src = (row & 7) * 4;
      const float ds_r = __shfl_sync(0xffffffffu, row < 8 ? dsb[0] : dsb[1], src);
      const float pb_r = __shfl_sync(0xffffffffu, row < 8 ? pbv[0] : pbv[1], src);
      gk = fmaf(ds_r, io<T>::ld(w.Q + swz(row, lane >> 3) + (lane & 7)), gk);
      gv = fmaf(pb_r, io<T>::ld(w.dO + swz(row, lane >> 3) + (lane & 7)), gv);
    }
    if (a.dbk) {  // null: the blank gradients are summed by the prologue kernel
      red_add(a.dbk + (int64_t)h * TD + lane, gk * a.scale);
      red_add(a.dbv + (int64_t)h * TD + lane, gv);
    }
  }
  T* dbase = a.dbias ? (T*)a.dbias + (bh * N + n0) * M : nullptr;
  float qacc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qacc[i][0] = qacc[i][1] = qacc[i][2] = qacc[i][3] = 0.f;
  for (int c = 0; c < nchunk; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunk) warp_load_kv(w.KV[buf ^ 1][0], w.KV[buf ^ 1][1], kb, vb, uclu, c + 1, nclu, N);
    cp_commit();
    cp_wait<1>();
    __syncwarp();
    float sx[2][4], dp[2][4];
    mma_chunk_nt<T>(sx, aq, w.KV[buf][0], 0);
    mma_chunk_nt<T>(dp, ado, w.KV[buf][1], 0);
    float p[2][4], ds[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int lc = nt * 8 + 2 * tq;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = g + hf * 8;
        const int bo = s.boff[row][2 * c + nt];
        float b0, b1;
        bias_at(w.bias, bo, tq, b0, b1);
        p[nt][2 * hf] = __expf(sx[nt][2 * hf] * a.scale + b0 - ls[hf]);
        p[nt][2 * hf + 1] = __expf(sx[nt][2 * hf + 1] * a.scale + b1 - ls[hf]);
        ds[nt][2 * hf] = p[nt][2 * hf] * (dp[nt][2 * hf] - dl[hf]);
        ds[nt][2 * hf + 1] = p[nt][2 * hf + 1] * (dp[nt][2 * hf + 1] - dl[hf]);
        const uint32_t dpk = pack2<T>(ds[nt][2 * hf], ds[nt][2 * hf + 1]);
        if (dbase && bo != TQ * MM && row < nq) *reinterpret_cast<uint32_t*>(dbase + bo + 2 * tq) = dpk;
        *reinterpret_cast<uint32_t*>(w.dS + row * BPT + lc) = dpk;
        *reinterpret_cast<uint32_t*>(w.P + row * BPT + lc) = pack2<T>(p[nt][2 * hf], p[nt][2 * hf + 1]);
      }
    }
    const uint32_t da[4] = {pack2<T>(ds[0][0], ds[0][1]), pack2<T>(ds[0][2], ds[0][3]),
                            pack2<T>(ds[1][0], ds[1][1]), pack2<T>(ds[1][2], ds[1][3])};
    mma_chunk_pv<T>(qacc, da, w.KV[buf][0], 0);
    __syncwarp();
    mma_chunk_scatter<T>(w.dS, BPT, w.Q, uclu, U, c * 16, a.scale, a.dk + bh * N * TD, N);
    mma_chunk_scatter<T>(w.P, BPT, w.dO, uclu, U, c * 16, 1.f, a.dv + bh * N * TD, N);
    __syncwarp();
  }
  const T* bkp = a.blank_k ? (const T*)a.blank_k + (int64_t)h * TD : nullptr;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int row = g + hf * 8;
    if (row >= nq) continue;
    T* qrow = (T*)a.dq + (bh * N + n0 + row) * TD;
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) {
      const int col = dt * 8 + 2 * tq;
      float v0 = qacc[dt][2 * hf], v1 = qacc[dt][2 * hf + 1];
      if (bkp) { v0 += dsb[hf] * ldf(bkp + col); v1 += dsb[hf] * ldf(bkp + col + 1); }
      *reinterpret_cast<uint32_t*>(qrow + col) = pack2<T>(v0 * a.scale, v1 * a.scale);
    }
  }
}

// Only for calls whose lists are not all cluster runs (flag set by the list
// builder); otherwise the key-side and dQ kernels do the backward.
template <typename T, int MM>
__global__ void __launch_bounds__(TC_THREADS, AFFB_BWD_MINB) nbhd_blk_bwd_kernel(NbhdArgs a) {
  dependent_wait();
  if (!*a.general) return;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BlkBwdSmem<T, MM>& s = *reinterpret_cast<BlkBwdSmem<T, MM>*>(smem_raw);
  const int N = a.N;
  const int tiles = (N + TQ - 1) / TQ;
  const int warp = threadIdx.x >> 5;
  // grid-stride over tiles: the launch is small so that the common case (flag
  // clear) costs one wave of blocks that return at once
  for (int64_t tile = blockIdx.x; tile < (int64_t)tiles * a.B; tile += gridDim.x) {
    const int b = (int)(tile / tiles);
    const int n0 = (int)(tile % tiles) * TQ;
    const int nq = min(TQ, N - n0);
    __syncthreads();  // the previous tile's warps are done with shared memory
    const int nclu = blk_setup<MM>(s.setup, s.u.idx, a, b, n0, nq);
    if (nclu < 0) {  // not cluster-block lists: CUDA-core rows, blank-token grads straight to global
      for (int w = warp; w < a.H * nq; w += NW) {
        const int h = w / nq;
        nbhd_bwd_row<T, 4>(a, b, h, n0 + w % nq, a.dbk ? a.dbk + (int64_t)h * TD : nullptr,
                           a.dbk ? a.dbv + (int64_t)h * TD : nullptr);
      }
      continue;
    }
    for (int h = warp; h < a.H; h += NW) blk_bwd_head<T, MM>(a, s.setup, s.u.w[warp], b, h, n0, nq, nclu);
  }
}

// dQ of one head and tile from dS, which the key-side kernel has written in
// bias layout ([B,H,N,M], a.ds):  dQ = scale * (sum_j dS[q, 8j+r] K[key] +
// ds_blank[q] blank_k).  The A fragments of each 16-key chunk are read from
// the staged dS rows through the bias-run offset table (absent clusters hit a
// zero block), so a chunk is two 32-bit loads per fragment half and four mma.
template <typename T, int MM>
__device__ void blk_dq_head(const NbhdArgs& a, const BlkSetup<MM>& s, BlkWarpDq<T, MM>& w, int b, int h, int n0,
                            int nq, int nclu) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int N = a.N, M = a.M;
  const int nchunk = (nclu + 1) / 2;
  const int64_t bh = (int64_t)b * a.H + h;
  const T* kb = (const T*)a.k + bh * N * TD;
  {
    const T* src = (const T*)a.ds + (bh * N + n0) * M;
    const int nch = TQ * M / 8;
    for (int i = lane; i < nch; i += 32) {
      const bool ok = (i * 8) / M < nq;
      cp_async16(w.dS + i * 8, src + (ok ? i * 8 : 0), ok);
    }
  }
  cp_commit();
  warp_load_k(w.K[0], kb, s.uclu, 0, nclu, N);
  cp_commit();
  if (lane < 8) w.dS[TQ * MM + lane] = pos_zero<T>();
  float qacc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qacc[i][0] = qacc[i][1] = qacc[i][2] = qacc[i][3] = 0.f;
  for (int c = 0; c < nchunk; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunk) warp_load_k(w.K[buf ^ 1], kb, s.uclu, c + 1, nclu, N);
    cp_commit();
    cp_wait<1>();
    __syncwarp();
    uint32_t da[4];
#pragma unroll
    for (int kh = 0; kh < 2; ++kh)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int bo = s.boff[g + 8 * hf][2 * c + kh];
        da[kh * 2 + hf] = *reinterpret_cast<const uint32_t*>(w.dS + bo + 2 * tq);
      }
    mma_chunk_pv<T>(qacc, da, w.K[buf], 0);
    __syncwarp();
  }
  const T* bkp = a.blank_k ? (const T*)a.blank_k + (int64_t)h * TD : nullptr;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int row = g + hf * 8;
    if (row >= nq) continue;
    const float dsb = bkp ? a.dsb[bh * N + n0 + row] : 0.f;
    T* qrow = (T*)a.dq + (bh * N + n0 + row) * TD;
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) {
      const int col = dt * 8 + 2 * tq;
      float v0 = qacc[dt][2 * hf], v1 = qacc[dt][2 * hf + 1];
      if (bkp) { v0 += dsb * ldf(bkp + col); v1 += dsb * ldf(bkp + col + 1); }
      *reinterpret_cast<uint32_t*>(qrow + col) = pack2<T>(v0 * a.scale, v1 * a.scale);
    }
  }
}

template <typename T, int MM>
__global__ void __launch_bounds__(TC_THREADS, AFFB_DQ_MINB) nbhd_blk_dq_kernel(NbhdArgs a) {
  dependent_wait();
  if (*a.general) return;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BlkDqSmem<T, MM>& s = *reinterpret_cast<BlkDqSmem<T, MM>*>(smem_raw);
  const int N = a.N;
  const int tiles = (N + TQ - 1) / TQ;
  const int b = blockIdx.x / tiles;
  const int n0 = (blockIdx.x % tiles) * TQ;
  const int nq = min(TQ, N - n0);
  const int nclu = a.tile_plan ? tile_plan_load<MM>(reinterpret_cast<const TilePlan<MM>*>(a.tile_plan) + blockIdx.x,
                                                   s.setup)
                               : blk_setup<MM>(s.setup, s.u.idx, a, b, n0, nq);
  if (nclu < 0) return;  // excluded by the list check that cleared the flag
  const int warp = threadIdx.x >> 5;
  for (int h = warp; h < a.H; h += NW) blk_dq_head<T, MM>(a, s.setup, s.u.w[warp], b, h, n0, nq, nclu);
}

template <typename K>
static int launch_blk(K kernel, size_t smem, const NbhdArgs& a, int B, cudaStream_t st, int64_t max_blocks = 0) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
      cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
    set_error("nbhd_attn: cannot reserve %zu bytes of shared memory", smem);
    return AFFB_ERR_CUDA;
  }
  int64_t tiles = (int64_t)((a.N + TQ - 1) / TQ) * B;
  if (max_blocks > 0 && tiles > max_blocks) tiles = max_blocks;
  if (launch_dependent(kernel, dim3((unsigned)tiles), dim3(TC_THREADS), smem, st, a) != cudaSuccess) {
    set_error("nbhd_attn: kernel failed to launch");
    return AFFB_ERR_CUDA;
  }
  return AFFB_OK;
}

// Neighbour capacity of the tile structures for M (a multiple of 8, <= 64).
static int blk_mm(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 48 ? 48 : 64; }

#define AFFB_BLK_LAUNCH(KERNEL, SMEM, MAXB)                                                                   \
  do {                                                                                                    \
    switch (blk_mm(a.M)) {                                                                                \
      case 16: return dtype == AFFB_BF16 ? launch_blk(KERNEL<__nv_bfloat16, 16>, sizeof(SMEM<__nv_bfloat16, 16>), a, B, st, MAXB) \
                                         : launch_blk(KERNEL<__half, 16>, sizeof(SMEM<__half, 16>), a, B, st, MAXB);             \
      case 32: return dtype == AFFB_BF16 ? launch_blk(KERNEL<__nv_bfloat16, 32>, sizeof(SMEM<__nv_bfloat16, 32>), a, B, st, MAXB) \
                                         : launch_blk(KERNEL<__half, 32>, sizeof(SMEM<__half, 32>), a, B, st, MAXB);             \
      case 48: return dtype == AFFB_BF16 ? launch_blk(KERNEL<__nv_bfloat16, 48>, sizeof(SMEM<__nv_bfloat16, 48>), a, B, st, MAXB) \
                                         : launch_blk(KERNEL<__half, 48>, sizeof(SMEM<__half, 48>), a, B, st, MAXB);             \
      default: return dtype == AFFB_BF16 ? launch_blk(KERNEL<__nv_bfloat16, 64>, sizeof(SMEM<__nv_bfloat16, 64>), a, B, st, MAXB) \
                                         : launch_blk(KERNEL<__half, 64>, sizeof(SMEM<__half, 64>), a, B, st, MAXB);             \
    }                                                                                                     \
  } while (0)

int64_t nbhd_tile_plan_bytes(int64_t B, int64_t N, int64_t M) {
  const int64_t tiles = B * ((N + TQ - 1) / TQ);
  switch (blk_mm((int)M)) {
    case 16: return tiles * (int64_t)sizeof(TilePlan<16>);
    case 32: return tiles * (int64_t)sizeof(TilePlan<32>);
    case 48: return tiles * (int64_t)sizeof(TilePlan<48>);
    default: return tiles * (int64_t)sizeof(TilePlan<64>);
  }
}

int nbhd_blk_fwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st) { AFFB_BLK_LAUNCH(nbhd_blk_fwd_kernel, BlkFwdSmem, 0); }
int nbhd_blk_bwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st) {
  AFFB_BLK_LAUNCH(nbhd_blk_bwd_kernel, BlkBwdSmem, 2 * sm_count());
}
int nbhd_blk_dq(const NbhdArgs& a, int dtype, int B, cudaStream_t st) { AFFB_BLK_LAUNCH(nbhd_blk_dq_kernel, BlkDqSmem, 0); }

}  // namespace affb
