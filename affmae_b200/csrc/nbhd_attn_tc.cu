// Neighbourhood attention on the tensor cores (bf16 / fp16, head_dim 32).
//
// Same semantics as the CUDA-core path (nbhd_row.cuh, reference
// local_attn.py:224-553).  The work unit is a tile of TQ = 16 consecutive
// queries of one batch element, all heads:
//   1. the tile's TQ x M neighbour indices are loaded once (not once per
//      head) and deduplicated in shared memory (open-addressing hash + block
//      scan) into the union U of key rows the tile touches; each (query,
//      neighbour) entry keeps its slot in U.  Queries of one cluster share
//      most neighbours, so |U| is ~120 instead of 16 x 48 = 768;
//   2. per head, the U rows of K and V are gathered into shared memory with
//      cp.async, and a [16 x U] table holds bias[q, m] at the slot of every
//      attended entry (-inf elsewhere), i.e. the block-sparse pattern;
//   3. flash-attention style on mma.sync m16n8k16 (fp32 accumulation): each
//      warp owns 16-slot chunks of U; S = Q K_U^T stays in registers, the
//      softmax is applied in the accumulator layout, which is reused as the
//      A operand of O = P V_U; the four warps' partial row max / sum / O are
//      merged through shared memory.
// Backward per head: S and dP = dO V_U^T in registers, p = exp(s - lse),
// ds = p (dp - Delta); dQ = dS K_U in registers (merged across warps);
// dK_U = dS^T Q and dV_U = P^T dO from the warp's own chunks, scattered once
// per (tile, key row) into fp32 accumulators; dbias is read back per entry.
// Tiles whose union exceeds UCAP rows, or whose neighbour lists repeat an
// index, run the CUDA-core row code instead (any input stays exact).
//
// Roofline: HBM-bound (about 16 flop per interface byte at B=32, N=4608,
// H=4, d=32, M=48), so mma.sync is sufficient for the contractions; the
// design goal is reading each interface byte once (neighbour indices once
// per tile instead of once per head, K/V rows once per tile instead of once
// per (query, neighbour)).
#include "nbhd_tc.cuh"
#include "nbhd_mma.cuh"

#include <stdlib.h>

namespace affb {

// ------------------------------------------------------------ tile setup --
struct TileSetup {
  short uof[TQ * MMAX];      // union slot per (row, neighbour) entry, -1 outside N
  int ukey[UCAP];            // key row of each union slot
  unsigned rowbits[TQ][UCAP / 32];
  int warp_tot[NW];
  int U;
  int dup;                   // some row lists one key twice
};

// Hash tables of the setup phase; they share storage with the per-head tables.
struct HashTables {
  int hkey[HS];
  int hval[HS];
};

__device__ __forceinline__ uint32_t hash_slot(int key) {
  return ((uint32_t)key * 2654435761u) >> (32 - 10);  // HS = 1024
}

// Builds the union of key rows of the tile's neighbour lists.  Thread t works
// on row t/8 and its entries [sub*EPT, sub*EPT + EPT).  Returns |U| (the
// tensor-core path needs |U| <= UCAP and no repeated key within a row).
__device__ int tile_union(TileSetup& s, HashTables& hs, const int32_t* __restrict__ midx, int b,
                          int n0, int nq, int N, int M) {
  const int t = threadIdx.x, r = t >> 3, sub = t & 7;
  const int EPT = (M + 7) >> 3;
  for (int i = t; i < HS; i += TC_THREADS) hs.hkey[i] = -1;
  for (int i = t; i < TQ * (UCAP / 32); i += TC_THREADS) (&s.rowbits[0][0])[i] = 0u;
  if (t == 0) s.dup = 0;
  int keys[MMAX / 8];
  const int32_t* ir = midx + ((int64_t)b * N + n0 + r) * M;
#pragma unroll
  for (int i = 0; i < MMAX / 8; ++i) {
    const int e = sub * EPT + i;
    keys[i] = (i < EPT && e < M && r < nq) ? ir[e] : -1;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < MMAX / 8; ++i) {
    const int key = keys[i];
    if (key < 0) continue;
    uint32_t h = hash_slot(key);
    while (true) {
      const int old = atomicCAS(&hs.hkey[h], -1, key);
      if (old == -1 || old == key) break;
      h = (h + 1) & (HS - 1);
    }
  }
  __syncthreads();
  // compact occupied slots in slot order: block exclusive scan of per-thread counts
  constexpr int PER = HS / TC_THREADS;
  int c = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) c += hs.hkey[t * PER + i] >= 0;
  const int lane = t & 31, w = t >> 5;
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
  for (int i = 0; i < PER; ++i) {
    const int key = hs.hkey[t * PER + i];
    if (key >= 0) {
      hs.hval[t * PER + i] = pos;
      if (pos < UCAP) s.ukey[pos] = key;
      ++pos;
    }
  }
  if (t == 0) s.U = total;
  __syncthreads();
  int dup = 0;
#pragma unroll
  for (int i = 0; i < MMAX / 8; ++i) {
    const int e = sub * EPT + i;
    if (i >= EPT || e >= M) continue;
    const int key = keys[i];
    short u = -1;
    if (key >= 0) {
      uint32_t h = hash_slot(key);
      while (hs.hkey[h] != key) h = (h + 1) & (HS - 1);
      u = (short)hs.hval[h];
      if (u < UCAP) {
        const unsigned bit = 1u << (u & 31);
        if (atomicOr(&s.rowbits[r][u >> 5], bit) & bit) dup = 1;
      }
    }
    s.uof[r * M + e] = u;
  }
  if (dup) s.dup = 1;
  __syncthreads();
  return total;
}

}  // namespace affb


namespace affb {

constexpr int TST = UCAP + 8;   // 16-bit row stride of the per-warp slot table
constexpr int PTS = 24;         // 16-bit row stride of the per-warp 16x16 P tile
#ifndef AFFB_NSTAGE
#define AFFB_NSTAGE 2
#endif
constexpr int NST = AFFB_NSTAGE;  // K/V chunk pipeline depth per warp

// Per-warp staging of one head of one tile.
template <typename T>
struct WarpFwd {
  alignas(16) T tab[TQ * TST];   // bias at attended (q, slot), -inf elsewhere
  alignas(16) T KV[NST][2][16 * KST];  // ring of 16-slot chunks of K_U ([s][0]) and V_U ([s][1])
  alignas(16) T Q[TQ * KST];
};
template <typename T>
struct WarpBwd {
  alignas(16) T tab[TQ * TST];   // bias, then dS in place
  alignas(16) T KV[NST][2][16 * KST];
  alignas(16) T Q[TQ * KST];
  alignas(16) T dO[TQ * KST];
  alignas(16) T P[TQ * PTS];
};

// Fills the per-warp slot table: tab[q][u] = bias (raw copy of the staged
// rows; 0 without bias) at attended entries, -inf elsewhere.  Returns the masked-entry count of rows
// g and g + 8 of the calling lane.
template <typename T>
__device__ __forceinline__ void warp_slot_table(T* tab, const TileSetup& s, const T* sbias, const uint8_t* gmask,
                                                int M, int nq, int Upad, int& ex0, int& ex1) {
  const int lane = threadIdx.x & 31, g = lane >> 2;
  const T ninf = neg_inf<T>();
  uint4 fill;
  {
    T f8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) f8[e] = ninf;
    fill = *reinterpret_cast<uint4*>(f8);
  }
#pragma unroll 4
  for (int row = 0; row < TQ; ++row)
    if (lane < Upad / 8) *reinterpret_cast<uint4*>(tab + row * TST + lane * 8) = fill;
  __syncwarp();
  ex0 = ex1 = 0;
#pragma unroll 4
  for (int r = 0; r < TQ; ++r) {
    if (r >= nq) break;
    int cnt = 0;
    for (int e = lane; e < M; e += 32) {
      const bool valid = gmask == nullptr || gmask[r * M + e] != 0;
      if (valid) tab[r * TST + s.uof[r * M + e]] = sbias ? sbias[r * M + e] : T(0.f);
      cnt += !valid;
    }
    if (gmask) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
      if (r == g) ex0 = cnt;
      if (r == g + 8) ex1 = cnt;
    }
  }
  __syncwarp();
}

}  // namespace affb

namespace affb {

template <typename T>
struct FwdSmem {
  TileSetup setup;
  union alignas(16) {
    HashTables hash;
    WarpFwd<T> w[NW];
  } x;
};
template <typename T>
struct BwdSmem {
  TileSetup setup;
  union alignas(16) {
    HashTables hash;
    WarpBwd<T> w[NW];
  } x;
};

// One warp, one head: streamed flash attention over the tile's union chunks.
template <typename T>
__device__ void fwd_head_warp(const NbhdArgs& a, const TileSetup& s, WarpFwd<T>& w, int b, int h, int n0,
                              int nq, int U) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int N = a.N;
  const int Upad = (U + 15) & ~15, nchunk = Upad / 16;
  const int64_t bh = (int64_t)b * a.H + h;
  const T* kb = (const T*)a.k + bh * N * TD;
  const T* vb = (const T*)a.v + bh * N * TD;
  const int* ukey = s.ukey;
  auto rows_u = [&](int u0) { return [=](int i) -> int64_t { return u0 + i < U ? ukey[u0 + i] : -1; }; };
  warp_load16(w.Q, (const T*)a.q + (bh * N + n0) * TD, [=](int i) -> int64_t { return i < nq ? i : -1; });
  static_assert(2 * 16 * KST >= TQ * MMAX, "bias staging does not fit");
  T* sbias = &w.KV[NST - 1][0][0];  // ring slot NST-1 is free until the slot table is built
  if (a.bias) warp_stage_bias(sbias, a, b, h, n0, nq);
  cp_commit();
#pragma unroll
  for (int c = 0; c < NST - 1; ++c) {
    if (c < nchunk) {
      warp_load16(w.KV[c][0], kb, rows_u(c * 16));
      warp_load16(w.KV[c][1], vb, rows_u(c * 16));
    }
    cp_commit();
  }
  cp_wait<NST - 1>();
  __syncwarp();
  int ex0, ex1;
  warp_slot_table<T>(w.tab, s, a.bias ? sbias : nullptr, a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0) * a.M : nullptr, a.M, nq, Upad, ex0, ex1);
  uint32_t aq[2][4];
  load_a_frags(aq, w.Q);
  float sb0 = -INFINITY, sb1 = -INFINITY;
  if (a.blank_k) {
    rows_dot(w.Q, (const T*)a.blank_k + (int64_t)h * TD, sb0, sb1);
    sb0 *= a.scale;
    sb1 *= a.scale;
  }
  float m0 = -1e11f, m1 = -1e11f, l0 = 0.f, l1 = 0.f;
  float o[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  for (int c = 0; c < nchunk; ++c) {
    const int buf = c % NST;
    {
      const int cn = c + NST - 1;  // refill the slot freed by chunk c - 1
      if (cn < nchunk) {
        warp_load16(w.KV[cn % NST][0], kb, rows_u(cn * 16));
        warp_load16(w.KV[cn % NST][1], vb, rows_u(cn * 16));
      }
      cp_commit();
      cp_wait<NST - 1>();
    }
    __syncwarp();
    float x[2][4];
    mma_chunk_nt<T>(x, aq, w.KV[buf][0], 0);
    float c0 = -INFINITY, c1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int col = c * 16 + j * 8 + 2 * tq;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = g + (e >> 1) * 8;
        x[j][e] = x[j][e] * a.scale + io<T>::ld(w.tab + row * TST + col + (e & 1));
        if (e < 2) c0 = fmaxf(c0, x[j][e]); else c1 = fmaxf(c1, x[j][e]);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      c0 = fmaxf(c0, __shfl_xor_sync(0xffffffffu, c0, off));
      c1 = fmaxf(c1, __shfl_xor_sync(0xffffffffu, c1, off));
    }
    const float n0m = fmaxf(m0, c0), n1m = fmaxf(m1, c1);
    const float al0 = __expf(m0 - n0m), al1 = __expf(m1 - n1m);
    m0 = n0m;
    m1 = n1m;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int i = 0; i < 4; ++i) { o[i][0] *= al0; o[i][1] *= al0; o[i][2] *= al1; o[i][3] *= al1; }
    float p[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p[j][e] = __expf(x[j][e] - (e < 2 ? m0 : m1));
        if (e < 2) l0 += p[j][e]; else l1 += p[j][e];
      }
    const uint32_t pa[4] = {pack2<T>(p[0][0], p[0][1]), pack2<T>(p[0][2], p[0][3]),
                            pack2<T>(p[1][0], p[1][1]), pack2<T>(p[1][2], p[1][3])};
    mma_chunk_pv<T>(o, pa, w.KV[buf][1], 0);
    __syncwarp();
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const int pad = padded_neighbours(a.M) - a.M;
  float mf[2] = {m0, m1}, lf[2] = {l0, l1}, pb[2] = {0.f, 0.f}, al[2] = {1.f, 1.f};
  const float sbs[2] = {sb0, sb1};
  const int exs[2] = {ex0, ex1};
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const float mm = a.blank_k ? fmaxf(mf[hf], sbs[hf]) : mf[hf];
    al[hf] = expf(mf[hf] - mm);
    if (a.blank_k) pb[hf] = expf(sbs[hf] - mm);
    lf[hf] = lf[hf] * al[hf] + pb[hf] + (float)(exs[hf] + pad) * expf(-1e11f - mm);
    mf[hf] = mm;
  }
  const T* bvp = a.blank_v ? (const T*)a.blank_v + (int64_t)h * TD : nullptr;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int row = g + hf * 8;
    if (row >= nq) continue;
    const float lse = mf[hf] + logf(lf[hf] + 1e-12f);
    const float inv = expf(mf[hf] - lse);
    T* orow = (T*)a.out + (bh * N + n0 + row) * TD;
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) {
      const int col = dt * 8 + 2 * tq;
      float v0 = o[dt][2 * hf] * al[hf], v1 = o[dt][2 * hf + 1] * al[hf];
      if (bvp) { v0 += pb[hf] * ldf(bvp + col); v1 += pb[hf] * ldf(bvp + col + 1); }
      *reinterpret_cast<uint32_t*>(orow + col) = pack2<T>(v0 * inv, v1 * inv);
    }
    if (tq == 0) a.lse[bh * N + n0 + row] = lse;
  }
}

// Tiles whose neighbour lists are not cluster blocks (listed by the block
// kernels) are processed here, persistent CTAs walking the list.
template <typename T>
__global__ void __launch_bounds__(TC_THREADS) nbhd_tc_fwd_list_kernel(NbhdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FwdSmem<T>& s = *reinterpret_cast<FwdSmem<T>*>(smem_raw);
  const int N = a.N, H = a.H;
  const int tiles = (N + TQ - 1) / TQ;
  const int count = *a.fb_count;
  const int warp = threadIdx.x >> 5;
  for (int i = blockIdx.x; i < count; i += gridDim.x) {
    const int tile = a.fb_list[i];
    const int b = tile / tiles;
    const int n0 = (tile % tiles) * TQ;
    const int nq = min(TQ, N - n0);
    __syncthreads();  // previous tile done with shared memory
    const int U = tile_union(s.setup, s.x.hash, a.midx, b, n0, nq, N, a.M);
    if (U > UCAP || s.setup.dup) {  // CUDA-core rows
      for (int w = warp; w < H * nq; w += NW) nbhd_fwd_row<T, 4>(a, b, w / nq, n0 + w % nq);
      continue;
    }
    for (int h = warp; h < H; h += NW) fwd_head_warp<T>(a, s.setup, s.x.w[warp], b, h, n0, nq, U);
  }
}

// One warp, one head of the backward.
template <typename T>
__device__ void bwd_head_warp(const NbhdArgs& a, const TileSetup& s, WarpBwd<T>& w, int b, int h, int n0,
                              int nq, int U) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int N = a.N, M = a.M;
  const int Upad = (U + 15) & ~15, nchunk = Upad / 16;
  const int64_t bh = (int64_t)b * a.H + h;
  const T* kb = (const T*)a.k + bh * N * TD;
  const T* vb = (const T*)a.v + bh * N * TD;
  const int* ukey = s.ukey;
  auto rows_u = [&](int u0) { return [=](int i) -> int64_t { return u0 + i < U ? ukey[u0 + i] : -1; }; };
  auto rows_q = [=](int i) -> int64_t { return i < nq ? i : -1; };
  warp_load16(w.Q, (const T*)a.q + (bh * N + n0) * TD, rows_q);
  warp_load16(w.dO, (const T*)a.dout + (bh * N + n0) * TD, rows_q);
  static_assert(2 * 16 * KST >= TQ * MMAX, "bias staging does not fit");
  T* sbias = &w.KV[NST - 1][0][0];  // ring slot NST-1 is free until the slot table is built
  if (a.bias) warp_stage_bias(sbias, a, b, h, n0, nq);
  cp_commit();
#pragma unroll
  for (int c = 0; c < NST - 1; ++c) {
    if (c < nchunk) {
      warp_load16(w.KV[c][0], kb, rows_u(c * 16));
      warp_load16(w.KV[c][1], vb, rows_u(c * 16));
    }
    cp_commit();
  }
  // Delta = rowsum(O * dO), lse for rows g and g + 8
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
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) p += __shfl_xor_sync(0xffffffffu, p, off);
    dl[hf] = p;
  }
  cp_wait<NST - 1>();
  __syncwarp();
  int ex0, ex1;
  warp_slot_table<T>(w.tab, s, a.bias ? sbias : nullptr, a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0) * a.M : nullptr, M, nq, Upad, ex0, ex1);
  uint32_t aq[2][4], ado[2][4];
  load_a_frags(aq, w.Q);
  load_a_frags(ado, w.dO);
  // blank token
  float dsb[2] = {0.f, 0.f};
  if (a.blank_k) {
    float sb[2], dpb[2];
    rows_dot(w.Q, (const T*)a.blank_k + (int64_t)h * TD, sb[0], sb[1]);
    rows_dot(w.dO, (const T*)a.blank_v + (int64_t)h * TD, dpb[0], dpb[1]);
    float pbv[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      pbv[hf] = (g + hf * 8) < nq ? expf(sb[hf] * a.scale - ls[hf]) : 0.f;
      dsb[hf] = pbv[hf] * (dpb[hf] - dl[hf]);
    }
    // lane d accumulates dims d over the 16 rows: dbk += scale*dsb*q, dbv += pb*dO
    float gk = 0.f, gv = 0.f;
#pragma unroll
    for (int row = 0; row < TQ; ++row) {
      const int src = (row & 7) * 4;
      const float ds_r = __shfl_sync(0xffffffffu, row < 8 ? dsb[0] : dsb[1], src);
      const float pb_r = __shfl_sync(0xffffffffu, row < 8 ? pbv[0] : pbv[1], src);
      gk = fmaf(ds_r, io<T>::ld(w.Q + row * KST + lane), gk);
      gv = fmaf(pb_r, io<T>::ld(w.dO + row * KST + lane), gv);
    }
    red_add(a.dbk + (int64_t)h * TD + lane, gk * a.scale);
    red_add(a.dbv + (int64_t)h * TD + lane, gv);
  }
  float qacc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qacc[i][0] = qacc[i][1] = qacc[i][2] = qacc[i][3] = 0.f;
  for (int c = 0; c < nchunk; ++c) {
    const int buf = c % NST;
    {
      const int cn = c + NST - 1;  // refill the slot freed by chunk c - 1
      if (cn < nchunk) {
        warp_load16(w.KV[cn % NST][0], kb, rows_u(cn * 16));
        warp_load16(w.KV[cn % NST][1], vb, rows_u(cn * 16));
      }
      cp_commit();
      cp_wait<NST - 1>();
    }
    __syncwarp();
    float sx[2][4], dp[2][4];
    mma_chunk_nt<T>(sx, aq, w.KV[buf][0], 0);
    mma_chunk_nt<T>(dp, ado, w.KV[buf][1], 0);
    float p[2][4], ds[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int lc = j * 8 + 2 * tq;
      const int col = c * 16 + lc;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hf = e >> 1, row = g + hf * 8;
        const float v = sx[j][e] * a.scale + io<T>::ld(w.tab + row * TST + col + (e & 1));
        p[j][e] = __expf(v - ls[hf]);
        ds[j][e] = p[j][e] * (dp[j][e] - dl[hf]);
      }
      *reinterpret_cast<uint32_t*>(w.tab + g * TST + col) = pack2<T>(ds[j][0], ds[j][1]);
      *reinterpret_cast<uint32_t*>(w.tab + (g + 8) * TST + col) = pack2<T>(ds[j][2], ds[j][3]);
      *reinterpret_cast<uint32_t*>(w.P + g * PTS + lc) = pack2<T>(p[j][0], p[j][1]);
      *reinterpret_cast<uint32_t*>(w.P + (g + 8) * PTS + lc) = pack2<T>(p[j][2], p[j][3]);
    }
    const uint32_t da[4] = {pack2<T>(ds[0][0], ds[0][1]), pack2<T>(ds[0][2], ds[0][3]),
                            pack2<T>(ds[1][0], ds[1][1]), pack2<T>(ds[1][2], ds[1][3])};
    mma_chunk_pv<T>(qacc, da, w.KV[buf][0], 0);
    __syncwarp();
    {
      mma_chunk_scatter<T>(w.tab + c * 16, TST, w.Q, ukey, U, c * 16, a.scale, a.dk + bh * N * TD);
      mma_chunk_scatter<T>(w.P, PTS, w.dO, ukey, U, c * 16, 1.f, a.dv + bh * N * TD);
    }
    __syncwarp();
  }
  // dQ
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
  // dbias per entry (masked entries: 0)
  if (a.dbias) {
    T* dbase = (T*)a.dbias + (bh * N + n0) * M;
#pragma unroll 1
    for (int r = 0; r < nq; ++r) {
      for (int e = lane; e < M; e += 32) {
        const bool valid = a.mask == nullptr ||
                           a.mask[(((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0 + r) * M + e] != 0;
        dbase[r * M + e] = valid ? w.tab[r * TST + s.uof[r * M + e]] : T(0.f);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(TC_THREADS) nbhd_tc_bwd_list_kernel(NbhdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BwdSmem<T>& s = *reinterpret_cast<BwdSmem<T>*>(smem_raw);
  const int N = a.N, H = a.H;
  const int tiles = (N + TQ - 1) / TQ;
  const int count = *a.fb_count;
  const int warp = threadIdx.x >> 5;
  for (int i = blockIdx.x; i < count; i += gridDim.x) {
    const int tile = a.fb_list[i];
    const int b = tile / tiles;
    const int n0 = (tile % tiles) * TQ;
    const int nq = min(TQ, N - n0);
    __syncthreads();
    const int U = tile_union(s.setup, s.x.hash, a.midx, b, n0, nq, N, a.M);
    if (U > UCAP || s.setup.dup) {  // CUDA-core rows; blank-token grads go straight to global
      for (int w = warp; w < H * nq; w += NW) {
        const int h = w / nq;
        nbhd_bwd_row<T, 4>(a, b, h, n0 + w % nq, a.dbk + (int64_t)h * TD, a.dbv + (int64_t)h * TD);
      }
      continue;
    }
    for (int h = warp; h < H; h += NW) bwd_head_warp<T>(a, s.setup, s.x.w[warp], b, h, n0, nq, U);
  }
}

template <typename K>
static int launch_list(K kernel, size_t smem, const NbhdArgs& a, int B, cudaStream_t st) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    set_error("nbhd_attn: cannot reserve %zu bytes of shared memory", smem);
    return AFFB_ERR_CUDA;
  }
  const int64_t tiles = (int64_t)((a.N + TQ - 1) / TQ) * B;
  const int grid = (int)imin64(tiles, (int64_t)sm_count() * 2);
  kernel<<<grid, TC_THREADS, smem, st>>>(a);
  return AFFB_OK;
}

int nbhd_tc_fwd_list(const NbhdArgs& a, int dtype, int B, cudaStream_t st) {
  if (dtype == AFFB_BF16) return launch_list(nbhd_tc_fwd_list_kernel<__nv_bfloat16>, sizeof(FwdSmem<__nv_bfloat16>), a, B, st);
  return launch_list(nbhd_tc_fwd_list_kernel<__half>, sizeof(FwdSmem<__half>), a, B, st);
}

int nbhd_tc_bwd_list(const NbhdArgs& a, int dtype, int B, cudaStream_t st) {
  if (dtype == AFFB_BF16) return launch_list(nbhd_tc_bwd_list_kernel<__nv_bfloat16>, sizeof(BwdSmem<__nv_bfloat16>), a, B, st);
  return launch_list(nbhd_tc_bwd_list_kernel<__half>, sizeof(BwdSmem<__half>), a, B, st);
}

}  // namespace affb
