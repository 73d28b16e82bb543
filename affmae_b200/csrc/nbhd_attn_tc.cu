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

namespace affb {

constexpr int TQ = 16;          // queries per tile
constexpr int TD = 32;          // head dim
constexpr int MMAX = 64;        // neighbours per query
constexpr int UCAP = 192;       // max union rows per tile on the tensor-core path
constexpr int HS = 1024;        // hash slots (>= TQ * MMAX)
constexpr int TC_THREADS = 128;
constexpr int KST = TD + 8;     // smem row stride (elements) of Q/K/V/dO tiles: 80 B
constexpr int BST = UCAP + 4;   // fp32 row stride of the bias/slot table
constexpr int PST = UCAP + 8;   // 16-bit row stride of P / dS tiles
constexpr int OST = TD + 4;     // fp32 row stride of the cross-warp O / dQ partials
constexpr int NW = TC_THREADS / 32;

template <typename T> struct MmaType;
template <> struct MmaType<__nv_bfloat16> {
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
};
template <> struct MmaType<__half> {
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void red_add_v2(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

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

// cp.async gather of key rows ukey[u] (u < U) of a [N, 32] head slice into a
// [Upad][KST] smem tile; rows U..Upad-1 are zero-filled.
template <typename T>
__device__ __forceinline__ void gather_rows(T* dst, const T* __restrict__ src, const int* ukey, int U,
                                            int Upad) {
  for (int r = threadIdx.x; r < Upad * 4; r += TC_THREADS) {
    const int row = r >> 2, c = r & 3;
    const bool ok = row < U;
    cp_async16(dst + row * KST + c * 8, src + (int64_t)(ok ? ukey[row] : 0) * TD + c * 8, ok);
  }
}
// cp.async of the tile's TQ query rows (rows >= nq zero-filled).
template <typename T>
__device__ __forceinline__ void load_qtile(T* dst, const T* __restrict__ src, int nq) {
  for (int r = threadIdx.x; r < TQ * 4; r += TC_THREADS) {
    const int row = r >> 2, c = r & 3;
    const bool ok = row < nq;
    cp_async16(dst + row * KST + c * 8, src + (int64_t)(ok ? row : 0) * TD + c * 8, ok);
  }
}

// The per-head slot table: tab[q][u] = bias[q, m] (0 without bias) where
// entry (q, m) is attended and sits in slot u, -inf elsewhere.  Returns via
// `excl` the number of masked entries of row t/8 (same value in its 8 threads).
template <typename T>
__device__ __forceinline__ void build_slot_table(float* tab, const TileSetup& s, const NbhdArgs& a, int b,
                                                 int h, int n0, int nq, int Upad, int& excl) {
  const int t = threadIdx.x, r = t >> 3, sub = t & 7;
  const int M = a.M, N = a.N;
  const int EPT = (M + 7) >> 3;
  for (int i = t; i < TQ * (Upad / 4); i += TC_THREADS) {
    const int row = i / (Upad / 4), c4 = i % (Upad / 4);
    *reinterpret_cast<float4*>(tab + row * BST + c4 * 4) = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  }
  __syncthreads();
  int cnt = 0;
  if (r < nq) {
    const int64_t rowg = ((int64_t)b * a.H + h) * N + n0 + r;
    const uint8_t* mr = a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0 + r) * M : nullptr;
    const T* br = a.bias ? (const T*)a.bias + rowg * M : nullptr;
    for (int i = 0; i < EPT; ++i) {
      const int e = sub * EPT + i;
      if (e >= M) break;
      if (mr && mr[e] == 0) { ++cnt; continue; }
      tab[r * BST + s.uof[r * M + e]] = br ? ldf(br + e) : 0.f;
    }
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  excl = cnt;
}

// Per-row dot of a smem tile row (KST stride, 32 dims) with a global vector,
// computed by the 8 threads of a row group (4 dims each).
template <typename T>
__device__ __forceinline__ float row_dot8(const T* rowp, const T* __restrict__ vec, int sub) {
  float p = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) p = fmaf(io<T>::ld(rowp + sub * 4 + e), ldf(vec + sub * 4 + e), p);
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
  return p;
}

// Fragments of S = A B^T for one 16-slot chunk: acc[j] covers slots
// u0 + 8j .. u0 + 8j + 7.  `a` holds the A fragments (16 x 32) of both k-steps.
template <typename T>
__device__ __forceinline__ void mma_chunk_nt(float (*acc)[4], const uint32_t (*a)[4], const T* Bm, int u0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint32_t bb[4];
    ldsm_x4(bb, Bm + (u0 + j * 8 + (lane & 7)) * KST + (lane >> 3) * 8);
    acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    MmaType<T>::mma(acc[j], a[0], bb);
    MmaType<T>::mma(acc[j], a[1], bb + 2);
  }
}

// out[4 d-tiles][4] += A(16 x 16 chunk, fragments) * X[u0..u0+15][0..31].
template <typename T>
__device__ __forceinline__ void mma_chunk_pv(float (*out)[4], const uint32_t* a, const T* X, int u0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int dp = 0; dp < 2; ++dp) {
    uint32_t bb[4];
    // matrices (u0-7, d), (u8-15, d), (u0-7, d+8), (u8-15, d+8)
    const int j = lane >> 3;
    ldsm_x4_t(bb, X + (u0 + (j & 1) * 8 + (lane & 7)) * KST + dp * 16 + (j >> 1) * 8);
    MmaType<T>::mma(out[dp * 2], a, bb);
    MmaType<T>::mma(out[dp * 2 + 1], a, bb + 2);
  }
}

// Scatter-add of R[16 x 32] = Pt[q][u0..u0+15]^T (16 x 16) * Y[16 x 32] (times
// `mul`) into rows ukey[u] of dst (fp32, row stride TD), u < U.
template <typename T>
__device__ __forceinline__ void mma_chunk_scatter(const T* Pt, const T* Y, const int* ukey, int U, int u0,
                                                  float mul, float* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  uint32_t a[4];
  const int j = lane >> 3, rr = lane & 7;
  ldsm_x4_t(a, Pt + ((j >> 1) * 8 + rr) * PST + u0 + (j & 1) * 8);
  const int ua = u0 + g, ub = ua + 8;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    uint32_t yb[2];
    ldsm_x2_t(yb, Y + (lane & 15) * KST + nt * 8);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    MmaType<T>::mma(acc, a, yb);
    const int col = nt * 8 + 2 * tq;
    if (ua < U) red_add_v2(dst + (int64_t)ukey[ua] * TD + col, acc[0] * mul, acc[1] * mul);
    if (ub < U) red_add_v2(dst + (int64_t)ukey[ub] * TD + col, acc[2] * mul, acc[3] * mul);
  }
}

template <typename T>
__device__ __forceinline__ void load_a_frags(uint32_t (*a)[4], const T* A) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks)
    ldsm_x4(a[ks], A + ((lane & 7) + ((lane >> 3) & 1) * 8) * KST + ks * 16 + (lane >> 4) * 8);
}

}  // namespace affb

namespace affb {

constexpr int CPW = (UCAP / 16 + NW - 1) / NW;  // max 16-slot chunks per warp

template <typename T>
struct FwdSmem {
  TileSetup setup;
  union alignas(16) {
    HashTables hash;
    struct {
      float tab[TQ * BST];
      float opart[NW][TQ * OST];
    } h;
  } x;
  alignas(16) T K[UCAP * KST];
  alignas(16) T V[UCAP * KST];
  alignas(16) T Q[TQ * KST];
  float pmax[NW][TQ], psum[NW][TQ];
  float sb[TQ];
  int excl[TQ];
};

template <typename T>
__global__ void __launch_bounds__(TC_THREADS) nbhd_tc_fwd_kernel(NbhdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FwdSmem<T>& s = *reinterpret_cast<FwdSmem<T>*>(smem_raw);
  const int N = a.N, H = a.H;
  const int tiles = (N + TQ - 1) / TQ;
  const int b = blockIdx.x / tiles;
  const int n0 = (blockIdx.x % tiles) * TQ;
  const int nq = min(TQ, N - n0);
  const int U = tile_union(s.setup, s.x.hash, a.midx, b, n0, nq, N, a.M);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int r = t >> 3, sub = t & 7;
  const int g = lane >> 2, tq = lane & 3;

  if (U > UCAP || s.setup.dup) {  // CUDA-core rows
    for (int w = warp; w < H * nq; w += NW) nbhd_fwd_row<T, 4>(a, b, w / nq, n0 + w % nq);
    return;
  }
  const int Upad = (U + 15) & ~15;
  const int nchunk = Upad / 16;
  const int pad_cols = padded_neighbours(a.M) - a.M;
  for (int h = 0; h < H; ++h) {
    const int64_t bh = (int64_t)b * H + h;
    __syncthreads();  // previous head done with K/V/Q/tables
    gather_rows(s.K, (const T*)a.k + bh * N * TD, s.setup.ukey, U, Upad);
    gather_rows(s.V, (const T*)a.v + bh * N * TD, s.setup.ukey, U, Upad);
    load_qtile(s.Q, (const T*)a.q + (bh * N + n0) * TD, nq);
    asm volatile("cp.async.commit_group;" ::: "memory");
    int excl;
    build_slot_table<T>(s.x.h.tab, s.setup, a, b, h, n0, nq, Upad, excl);
    if (sub == 0) s.excl[r] = excl;
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (a.blank_k) {
      const float sb = row_dot8(s.Q + r * KST, (const T*)a.blank_k + (int64_t)h * TD, sub) * a.scale;
      if (sub == 0) s.sb[r] = sb;
    }
    // ---- S chunks in registers, masked by the slot table
    uint32_t aq[2][4];
    load_a_frags(aq, s.Q);
    float lg[CPW][2][4];
    float mx0 = -1e11f, mx1 = -1e11f;  // rows g, g+8
#pragma unroll
    for (int ci = 0; ci < CPW; ++ci) {
      const int c = warp + ci * NW;
      if (c < nchunk) {
        mma_chunk_nt<T>(lg[ci], aq, s.K, c * 16);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int col = c * 16 + j * 8 + 2 * tq;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = g + (e >> 1) * 8;
            const float v = lg[ci][j][e] * a.scale + s.x.h.tab[row * BST + col + (e & 1)];
            lg[ci][j][e] = v;
            if (e < 2) mx0 = fmaxf(mx0, v); else mx1 = fmaxf(mx1, v);
          }
        }
      }
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    if (tq == 0) { s.pmax[warp][g] = mx0; s.pmax[warp][g + 8] = mx1; }
    __syncthreads();
    float m0 = a.blank_k ? s.sb[g] : -1e11f, m1 = a.blank_k ? s.sb[g + 8] : -1e11f;
    m0 = fmaxf(m0, -1e11f);
    m1 = fmaxf(m1, -1e11f);
#pragma unroll
    for (int w = 0; w < NW; ++w) { m0 = fmaxf(m0, s.pmax[w][g]); m1 = fmaxf(m1, s.pmax[w][g + 8]); }
    // ---- P = exp(S - m), partial row sums, partial O = P V_U
    float oacc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
    float l0 = 0.f, l1 = 0.f;
#pragma unroll
    for (int ci = 0; ci < CPW; ++ci) {
      const int c = warp + ci * NW;
      if (c < nchunk) {
        float p[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            p[j][e] = expf(lg[ci][j][e] - (e < 2 ? m0 : m1));
            if (e < 2) l0 += p[j][e]; else l1 += p[j][e];
          }
        uint32_t pa[4] = {pack2<T>(p[0][0], p[0][1]), pack2<T>(p[0][2], p[0][3]),
                          pack2<T>(p[1][0], p[1][1]), pack2<T>(p[1][2], p[1][3])};
        mma_chunk_pv<T>(oacc, pa, s.V, c * 16);
      }
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    if (tq == 0) { s.psum[warp][g] = l0; s.psum[warp][g + 8] = l1; }
    float* op = s.x.h.opart[warp];
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) {
      const int col = dt * 8 + 2 * tq;
      op[g * OST + col] = oacc[dt][0];
      op[g * OST + col + 1] = oacc[dt][1];
      op[(g + 8) * OST + col] = oacc[dt][2];
      op[(g + 8) * OST + col + 1] = oacc[dt][3];
    }
    __syncthreads();
    // ---- merge: thread -> (row r, dims 4*sub .. 4*sub+3)
    if (r < nq) {
      float m = a.blank_k ? fmaxf(s.sb[r], -1e11f) : -1e11f;
#pragma unroll
      for (int w = 0; w < NW; ++w) m = fmaxf(m, s.pmax[w][r]);
      float l = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) l += s.psum[w][r];
      const float pb = a.blank_k ? expf(s.sb[r] - m) : 0.f;
      l += pb + (float)(s.excl[r] + pad_cols) * expf(-1e11f - m);
      const float lse = m + logf(l + 1e-12f);
      const float inv = expf(m - lse);
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = sub * 4 + e;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) acc += s.x.h.opart[w][r * OST + d];
        if (a.blank_v) acc += pb * ldf((const T*)a.blank_v + (int64_t)h * TD + d);
        o[e] = acc * inv;
      }
      uint2 pk = make_uint2(pack2<T>(o[0], o[1]), pack2<T>(o[2], o[3]));
      *reinterpret_cast<uint2*>((T*)a.out + (bh * N + n0 + r) * TD + sub * 4) = pk;
      if (sub == 0) a.lse[bh * N + n0 + r] = lse;
    }
  }
}

}  // namespace affb

namespace affb {

template <typename T>
struct BwdSmem {
  TileSetup setup;
  union alignas(16) {
    HashTables hash;
    struct {
      float tab[TQ * BST];
      float qpart[NW][TQ * OST];
    } h;
  } x;
  alignas(16) T K[UCAP * KST];
  alignas(16) T V[UCAP * KST];
  alignas(16) T Q[TQ * KST];
  alignas(16) T dO[TQ * KST];
  alignas(16) T P16[TQ * PST];
  alignas(16) T dS16[TQ * PST];
  float delta[TQ], lse[TQ], dsb[TQ];
  float dbk[TD], dbv[TD];
};

template <typename T>
__global__ void __launch_bounds__(TC_THREADS) nbhd_tc_bwd_kernel(NbhdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BwdSmem<T>& s = *reinterpret_cast<BwdSmem<T>*>(smem_raw);
  const int N = a.N, H = a.H, M = a.M;
  const int tiles = (N + TQ - 1) / TQ;
  const int b = blockIdx.x / tiles;
  const int n0 = (blockIdx.x % tiles) * TQ;
  const int nq = min(TQ, N - n0);
  const int U = tile_union(s.setup, s.x.hash, a.midx, b, n0, nq, N, M);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int r = t >> 3, sub = t & 7;
  const int g = lane >> 2, tq = lane & 3;

  if (U > UCAP || s.setup.dup) {  // CUDA-core rows; blank-token grads go straight to global
    for (int w = warp; w < H * nq; w += NW) {
      const int h = w / nq;
      nbhd_bwd_row<T, 4>(a, b, h, n0 + w % nq, a.dbk + (int64_t)h * TD, a.dbv + (int64_t)h * TD);
    }
    return;
  }
  const int Upad = (U + 15) & ~15;
  const int nchunk = Upad / 16;
  const int EPT = (M + 7) >> 3;
  for (int h = 0; h < H; ++h) {
    const int64_t bh = (int64_t)b * H + h;
    __syncthreads();
    gather_rows(s.K, (const T*)a.k + bh * N * TD, s.setup.ukey, U, Upad);
    gather_rows(s.V, (const T*)a.v + bh * N * TD, s.setup.ukey, U, Upad);
    load_qtile(s.Q, (const T*)a.q + (bh * N + n0) * TD, nq);
    load_qtile(s.dO, (const T*)a.dout + (bh * N + n0) * TD, nq);
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (t < TD) { s.dbk[t] = 0.f; s.dbv[t] = 0.f; }
    int excl;
    build_slot_table<T>(s.x.h.tab, s.setup, a, b, h, n0, nq, Upad, excl);
    {  // Delta = rowsum(O * dO) from global (4 dims per thread), lse
      float p = 0.f;
      if (r < nq) {
        const T* orow = (const T*)a.o + (bh * N + n0 + r) * TD + sub * 4;
        const T* drow = (const T*)a.dout + (bh * N + n0 + r) * TD + sub * 4;
#pragma unroll
        for (int e = 0; e < 4; ++e) p = fmaf(ldf(orow + e), ldf(drow + e), p);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
      if (sub == 0) {
        s.delta[r] = p;
        s.lse[r] = r < nq ? a.lse[bh * N + n0 + r] : 0.f;
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // ---- blank token: dsb per row, dbk / dbv partial sums
    if (a.blank_k) {
      const float lse = s.lse[r], delta = s.delta[r];
      const float sb = row_dot8(s.Q + r * KST, (const T*)a.blank_k + (int64_t)h * TD, sub) * a.scale;
      const float dpb = row_dot8(s.dO + r * KST, (const T*)a.blank_v + (int64_t)h * TD, sub);
      const float pb = r < nq ? expf(sb - lse) : 0.f;
      const float dsb = pb * (dpb - delta);
      if (sub == 0) s.dsb[r] = dsb;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = sub * 4 + e;
        float gk = a.scale * dsb * io<T>::ld(s.Q + r * KST + d);
        float gv = pb * io<T>::ld(s.dO + r * KST + d);
        gk += __shfl_xor_sync(0xffffffffu, gk, 8);
        gk += __shfl_xor_sync(0xffffffffu, gk, 16);
        gv += __shfl_xor_sync(0xffffffffu, gv, 8);
        gv += __shfl_xor_sync(0xffffffffu, gv, 16);
        if (lane < 8) { atomicAdd(&s.dbk[d], gk); atomicAdd(&s.dbv[d], gv); }
      }
    }
    // ---- per warp chunks: S, dP -> P, dS; partial dQ; dK_U / dV_U scatter
    uint32_t aq[2][4], ado[2][4];
    load_a_frags(aq, s.Q);
    load_a_frags(ado, s.dO);
    const float lse0 = s.lse[g], lse1 = s.lse[g + 8];
    const float dl0 = s.delta[g], dl1 = s.delta[g + 8];
    float qacc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) qacc[i][0] = qacc[i][1] = qacc[i][2] = qacc[i][3] = 0.f;
    for (int c = warp; c < nchunk; c += NW) {
      float sacc[2][4], pacc[2][4];
      mma_chunk_nt<T>(sacc, aq, s.K, c * 16);
      mma_chunk_nt<T>(pacc, ado, s.V, c * 16);
      float p[2][4], ds[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int col = c * 16 + j * 8 + 2 * tq;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = g + (e >> 1) * 8;
          const float v = sacc[j][e] * a.scale + s.x.h.tab[row * BST + col + (e & 1)];
          p[j][e] = expf(v - (e < 2 ? lse0 : lse1));
          ds[j][e] = p[j][e] * (pacc[j][e] - (e < 2 ? dl0 : dl1));
        }
        *reinterpret_cast<uint32_t*>(&s.P16[g * PST + col]) = pack2<T>(p[j][0], p[j][1]);
        *reinterpret_cast<uint32_t*>(&s.P16[(g + 8) * PST + col]) = pack2<T>(p[j][2], p[j][3]);
        *reinterpret_cast<uint32_t*>(&s.dS16[g * PST + col]) = pack2<T>(ds[j][0], ds[j][1]);
        *reinterpret_cast<uint32_t*>(&s.dS16[(g + 8) * PST + col]) = pack2<T>(ds[j][2], ds[j][3]);
      }
      uint32_t da[4] = {pack2<T>(ds[0][0], ds[0][1]), pack2<T>(ds[0][2], ds[0][3]),
                        pack2<T>(ds[1][0], ds[1][1]), pack2<T>(ds[1][2], ds[1][3])};
      mma_chunk_pv<T>(qacc, da, s.K, c * 16);
      __syncwarp();
      mma_chunk_scatter<T>(s.dS16, s.Q, s.setup.ukey, U, c * 16, a.scale, a.dk + bh * N * TD);
      mma_chunk_scatter<T>(s.P16, s.dO, s.setup.ukey, U, c * 16, 1.f, a.dv + bh * N * TD);
    }
    float* qp = s.x.h.qpart[warp];
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) {
      const int col = dt * 8 + 2 * tq;
      qp[g * OST + col] = qacc[dt][0];
      qp[g * OST + col + 1] = qacc[dt][1];
      qp[(g + 8) * OST + col] = qacc[dt][2];
      qp[(g + 8) * OST + col + 1] = qacc[dt][3];
    }
    __syncthreads();
    // ---- dbias per entry from dS (masked entries: 0); dQ merge; blank grads
    if (r < nq) {
      const uint8_t* mr = a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0 + r) * M : nullptr;
      if (a.dbias) {
        T* dbr = (T*)a.dbias + (bh * N + n0 + r) * M;
        for (int i = 0; i < EPT; ++i) {
          const int e = sub * EPT + i;
          if (e >= M) break;
          const bool valid = mr == nullptr || mr[e] != 0;
          if (valid) dbr[e] = s.dS16[r * PST + s.setup.uof[r * M + e]];
          else stf(dbr + e, 0.f);
        }
      }
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = sub * 4 + e;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) acc += s.x.h.qpart[w][r * OST + d];
        if (a.blank_k) acc += s.dsb[r] * ldf((const T*)a.blank_k + (int64_t)h * TD + d);
        o[e] = acc * a.scale;
      }
      uint2 pk = make_uint2(pack2<T>(o[0], o[1]), pack2<T>(o[2], o[3]));
      *reinterpret_cast<uint2*>((T*)a.dq + (bh * N + n0 + r) * TD + sub * 4) = pk;
    }
    if (a.blank_k && t < TD) {
      red_add(a.dbk + (int64_t)h * TD + t, s.dbk[t]);
      red_add(a.dbv + (int64_t)h * TD + t, s.dbv[t]);
    }
  }
}

template <typename K>
static int launch_tc(K kernel, size_t smem, const NbhdArgs& a, int B, cudaStream_t st) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    set_error("nbhd_attn: cannot reserve %zu bytes of shared memory", smem);
    return AFFB_ERR_CUDA;
  }
  const int tiles = (a.N + TQ - 1) / TQ;
  kernel<<<(unsigned)((int64_t)tiles * B), TC_THREADS, smem, st>>>(a);
  return AFFB_OK;
}

int nbhd_tc_fwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st) {
  if (dtype == AFFB_BF16) return launch_tc(nbhd_tc_fwd_kernel<__nv_bfloat16>, sizeof(FwdSmem<__nv_bfloat16>), a, B, st);
  return launch_tc(nbhd_tc_fwd_kernel<__half>, sizeof(FwdSmem<__half>), a, B, st);
}

int nbhd_tc_bwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st) {
  if (dtype == AFFB_BF16) return launch_tc(nbhd_tc_bwd_kernel<__nv_bfloat16>, sizeof(BwdSmem<__nv_bfloat16>), a, B, st);
  return launch_tc(nbhd_tc_bwd_kernel<__half>, sizeof(BwdSmem<__half>), a, B, st);
}

}  // namespace affb
