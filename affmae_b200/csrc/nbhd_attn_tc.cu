// Neighbourhood attention on the tensor cores (bf16 / fp16, head_dim 32).
//
// Same semantics as the CUDA-core path (nbhd_row.cuh, reference
// local_attn.py:224-553).  The work unit is a tile of TQ = 16 consecutive
// queries of one batch element, all heads:
//   1. the tile's TQ x M neighbour indices are loaded once (not once per
//      head) and deduplicated in shared memory (open-addressing hash +
//      block scan) into the union U of key rows the tile touches; each
//      (query, neighbour) entry keeps its slot in U.  Queries of one cluster
//      share most neighbours, so |U| is ~120 instead of 16 x 48 = 768;
//   2. per head, the U rows of K and V are gathered into shared memory
//      with cp.async (zero-filled up to a multiple of 16 rows);
//   3. S = Q K_U^T (16 x U) on mma.sync m16n8k16 with fp32 accumulation;
//   4. the softmax runs per entry on CUDA cores (8 threads per query row):
//      logit = scale * S[q][u(q,m)] + bias[q,m] (masked -> excluded but
//      counted), plus the blank token; probabilities are summed per (q, u)
//      into P (duplicated neighbours add up) and rounded to the input dtype;
//   5. O = P V_U on mma.sync, normalised with lse = m + log(l + 1e-12).
// Backward per head: S and dP = dO V_U^T on mma; per entry p = exp(s - lse),
// ds = p (dp - Delta), dbias written directly; dQ = dS K_U, and
// dK_U = dS^T Q, dV_U = P^T dO on mma, scattered once per (tile, key row)
// with red.global.add.v2.f32 into fp32 accumulators.
// A tile whose union exceeds UCAP rows runs the CUDA-core row code instead.
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
constexpr int SST = UCAP + 4;   // fp32 row stride of S / P tiles
constexpr int PST = UCAP + 8;   // 16-bit row stride of P / dS tiles

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
  int idx[TQ * MMAX];        // neighbour index per entry (-1: row outside N)
  short uof[TQ * MMAX];      // union slot per entry
  int ukey[UCAP];            // key row of each union slot
  int hkey[HS];
  int hval[HS];
  int warp_tot[TC_THREADS / 32];
  int U;
};

__device__ __forceinline__ uint32_t hash_slot(int key) {
  return ((uint32_t)key * 2654435761u) >> (32 - 10);  // HS = 1024
}

// Loads the tile's neighbour indices and builds the union of key rows.
// Returns the union size (may exceed UCAP: then ukey is incomplete).
__device__ int tile_union(TileSetup& s, const int32_t* __restrict__ midx, int b, int n0, int nq,
                          int N, int M) {
  const int t = threadIdx.x;
  for (int i = t; i < HS; i += TC_THREADS) s.hkey[i] = -1;
  for (int e = t; e < TQ * M; e += TC_THREADS) {
    const int q = e / M;
    s.idx[e] = q < nq ? midx[((int64_t)b * N + n0 + q) * M + (e - q * M)] : -1;
  }
  __syncthreads();
  for (int e = t; e < TQ * M; e += TC_THREADS) {
    const int key = s.idx[e];
    if (key < 0) continue;
    uint32_t h = hash_slot(key);
    while (true) {
      const int old = atomicCAS(&s.hkey[h], -1, key);
      if (old == -1 || old == key) break;
      h = (h + 1) & (HS - 1);
    }
  }
  __syncthreads();
  // compact occupied slots in slot order: block exclusive scan of per-thread counts
  constexpr int PER = HS / TC_THREADS;
  int c = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) c += s.hkey[t * PER + i] >= 0;
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
  for (int i = 0; i < TC_THREADS / 32; ++i) {
    if (i < w) base += s.warp_tot[i];
    total += s.warp_tot[i];
  }
  int pos = base + x - c;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int key = s.hkey[t * PER + i];
    if (key >= 0) {
      s.hval[t * PER + i] = pos;
      if (pos < UCAP) s.ukey[pos] = key;
      ++pos;
    }
  }
  if (t == 0) s.U = total;
  __syncthreads();
  for (int e = t; e < TQ * M; e += TC_THREADS) {
    const int key = s.idx[e];
    short u = -1;
    if (key >= 0) {
      uint32_t h = hash_slot(key);
      while (s.hkey[h] != key) h = (h + 1) & (HS - 1);
      u = (short)s.hval[h];
    }
    s.uof[e] = u;
  }
  __syncthreads();
  return total;
}

// Gathers rows [ukey[u]] of a [N, 32] head slice into a [Upad][KST] smem tile
// (rows >= U zero-filled), and optionally TQ query-tile rows.
template <typename T>
__device__ __forceinline__ void gather_rows(T* dst, const T* __restrict__ src, const int* ukey, int U,
                                            int Upad) {
  for (int r = threadIdx.x; r < Upad * 4; r += TC_THREADS) {
    const int row = r >> 2, c = r & 3;
    const bool ok = row < U;
    cp_async16(dst + row * KST + c * 8, src + (int64_t)(ok ? ukey[row] : 0) * TD + c * 8, ok);
  }
}
template <typename T>
__device__ __forceinline__ void load_qtile(T* dst, const T* __restrict__ src, int nq) {
  for (int r = threadIdx.x; r < TQ * 4; r += TC_THREADS) {
    const int row = r >> 2, c = r & 3;
    const bool ok = row < nq;
    cp_async16(dst + row * KST + c * 8, src + (int64_t)(ok ? row : 0) * TD + c * 8, ok);
  }
}

// C[16 x Upad] (fp32, row stride SST) = A[16 x 32] * B[Upad x 32]^T, A/B in smem.
template <typename T>
__device__ __forceinline__ void mma_rows_by_union(float* C, const T* A, const T* Bm, int Upad) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t a[2][4];
#pragma unroll
  for (int ks = 0; ks < 2; ++ks)
    ldsm_x4(a[ks], A + ((lane & 7) + ((lane >> 3) & 1) * 8) * KST + ks * 16 + (lane >> 4) * 8);
  const int g = lane >> 2, tq = lane & 3;
  for (int nt = warp; nt < Upad / 8; nt += TC_THREADS / 32) {
    uint32_t bb[4];
    ldsm_x4(bb, Bm + (nt * 8 + (lane & 7)) * KST + (lane >> 3) * 8);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    MmaType<T>::mma(acc, a[0], bb);
    MmaType<T>::mma(acc, a[1], bb + 2);
    float* c0 = C + g * SST + nt * 8 + 2 * tq;
    c0[0] = acc[0];
    c0[1] = acc[1];
    c0[8 * SST] = acc[2];
    c0[8 * SST + 1] = acc[3];
  }
}

// acc[4] for output columns d0..d0+7 of R[16 x 32] = P[16 x Upad] * X[Upad x 32].
template <typename T>
__device__ __forceinline__ void mma_p_by_rows(float* acc, const T* P, const T* X, int Upad, int d0) {
  const int lane = threadIdx.x & 31;
  for (int ks = 0; ks < Upad / 16; ++ks) {
    uint32_t a[4], bb[2];
    ldsm_x4(a, P + ((lane & 7) + ((lane >> 3) & 1) * 8) * PST + ks * 16 + (lane >> 4) * 8);
    ldsm_x2_t(bb, X + (ks * 16 + (lane & 15)) * KST + d0);
    MmaType<T>::mma(acc, a, bb);
  }
}

// Scatter-add of R[Upad x 32] = Pt^T[Upad x 16] * Y[16 x 32] (times `mul`)
// into dst rows ukey[u] (fp32, row stride TD) for u < U.
template <typename T>
__device__ __forceinline__ void mma_scatter_union(const T* Pt, const T* Y, const int* ukey, int U, int Upad,
                                                  float mul, float* __restrict__ dst) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3;
  uint32_t yb[4][2];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) ldsm_x2_t(yb[nt], Y + (lane & 15) * KST + nt * 8);
  for (int mt = warp; mt < Upad / 16; mt += TC_THREADS / 32) {
    uint32_t a[4];
    // A[m = u][k = q] = Pt[q][u]: matrices (q0-7,u0-7), (q0-7,u8-15), (q8-15,u0-7), (q8-15,u8-15)
    const int j = lane >> 3, r = lane & 7;
    ldsm_x4_t(a, Pt + ((j >> 1) * 8 + r) * PST + mt * 16 + (j & 1) * 8);
    const int u0 = mt * 16 + g, u1 = u0 + 8;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      MmaType<T>::mma(acc, a, yb[nt]);
      const int col = nt * 8 + 2 * tq;
      if (u0 < U) red_add_v2(dst + (int64_t)ukey[u0] * TD + col, acc[0] * mul, acc[1] * mul);
      if (u1 < U) red_add_v2(dst + (int64_t)ukey[u1] * TD + col, acc[2] * mul, acc[3] * mul);
    }
  }
}

}  // namespace affb

namespace affb {

template <typename T>
struct FwdSmem {
  TileSetup setup;
  float S[TQ * SST];
  float P32[TQ * SST];
  alignas(16) T K[UCAP * KST];
  alignas(16) T V[UCAP * KST];
  alignas(16) T Q[TQ * KST];
  alignas(16) T P16[TQ * PST];
  float rowm[TQ], rowl[TQ], rowpb[TQ];
};

template <typename T>
struct BwdSmem {
  TileSetup setup;
  float S[TQ * SST];
  float dP[TQ * SST];
  float P32[TQ * SST];
  float dS32[TQ * SST];
  alignas(16) T K[UCAP * KST];
  alignas(16) T V[UCAP * KST];
  alignas(16) T Q[TQ * KST];
  alignas(16) T dO[TQ * KST];
  alignas(16) T P16[TQ * PST];
  alignas(16) T dS16[TQ * PST];
  float delta[TQ], lse[TQ], dsb[TQ];
  float dbk[TD], dbv[TD];
};

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

template <typename T>
__global__ void __launch_bounds__(TC_THREADS) nbhd_tc_fwd_kernel(NbhdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FwdSmem<T>& s = *reinterpret_cast<FwdSmem<T>*>(smem_raw);
  const int N = a.N, M = a.M, H = a.H;
  const int tiles = (N + TQ - 1) / TQ;
  const int b = blockIdx.x / tiles;
  const int n0 = (blockIdx.x % tiles) * TQ;
  const int nq = min(TQ, N - n0);
  const int U = tile_union(s.setup, a.midx, b, n0, nq, N, M);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;

  if (U > UCAP) {  // union too large for the tensor-core tile: CUDA-core rows
    for (int w = warp; w < H * nq; w += TC_THREADS / 32)
      nbhd_fwd_row<T, 4>(a, b, w / nq, n0 + w % nq);
    return;
  }
  const int Upad = (U + 15) & ~15;
  const int r = t >> 3, sub = t & 7;  // softmax: 8 threads per query row
  const int pad_cols = padded_neighbours(M) - M;
  for (int h = 0; h < H; ++h) {
    const int64_t bh = (int64_t)b * H + h;
    const T* kb = (const T*)a.k + bh * N * TD;
    const T* vb = (const T*)a.v + bh * N * TD;
    gather_rows(s.K, kb, s.setup.ukey, U, Upad);
    gather_rows(s.V, vb, s.setup.ukey, U, Upad);
    load_qtile(s.Q, (const T*)a.q + (bh * N + n0) * TD, nq);
    for (int i = t; i < TQ * SST; i += TC_THREADS) s.P32[i] = 0.f;
    cp_async_wait_all();
    __syncthreads();
    mma_rows_by_union(s.S, s.Q, s.K, Upad);
    __syncthreads();
    // ---- per-entry softmax (8 threads per row)
    {
      const bool rowok = r < nq;
      const uint8_t* mr = a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0 + r) * M : nullptr;
      const T* br = a.bias ? (const T*)a.bias + (bh * N + n0 + r) * M : nullptr;
      float lg[MMAX / 8];
      float m = -1e11f;
      int excluded = 0;
#pragma unroll
      for (int i = 0; i < MMAX / 8; ++i) {
        const int e = sub + i * 8;
        lg[i] = -INFINITY;
        if (rowok && e < M) {
          const bool valid = mr == nullptr || mr[e] != 0;
          if (valid) {
            float v = s.S[r * SST + s.setup.uof[r * M + e]] * a.scale;
            if (br) v += ldf(br + e);
            lg[i] = v;
            m = fmaxf(m, v);
          } else {
            ++excluded;
          }
        }
      }
      float sb = -INFINITY;
      if (a.blank_k) {
        sb = row_dot8(s.Q + r * KST, (const T*)a.blank_k + (int64_t)h * TD, sub) * a.scale;
        if (rowok) m = fmaxf(m, sb);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        excluded += __shfl_xor_sync(0xffffffffu, excluded, o);
      }
      float l = 0.f;
#pragma unroll
      for (int i = 0; i < MMAX / 8; ++i) {
        const int e = sub + i * 8;
        if (lg[i] != -INFINITY) {
          const float p = expf(lg[i] - m);
          l += p;
          atomicAdd(&s.P32[r * SST + s.setup.uof[r * M + e]], p);
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (sub == 0) {
        const float pb = a.blank_k ? expf(sb - m) : 0.f;
        l += pb + (float)(excluded + pad_cols) * expf(-1e11f - m);
        s.rowm[r] = m;
        s.rowl[r] = l;
        s.rowpb[r] = pb;
      }
    }
    __syncthreads();
    for (int i = t; i < TQ * (Upad / 2); i += TC_THREADS) {
      const int row = i / (Upad / 2), c = (i % (Upad / 2)) * 2;
      *reinterpret_cast<uint32_t*>(&s.P16[row * PST + c]) = pack2<T>(s.P32[row * SST + c], s.P32[row * SST + c + 1]);
    }
    __syncthreads();
    // ---- O = P V_U (warp w: output dims 8w..8w+7)
    {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int d0 = warp * 8;
      mma_p_by_rows(acc, s.P16, s.V, Upad, d0);
      const int g = lane >> 2, tq = lane & 3;
      const int col = d0 + 2 * tq;
      float bv0 = 0.f, bv1 = 0.f;
      if (a.blank_v) {
        bv0 = ldf((const T*)a.blank_v + (int64_t)h * TD + col);
        bv1 = ldf((const T*)a.blank_v + (int64_t)h * TD + col + 1);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int row = g + half * 8;
        if (row < nq) {
          const float m = s.rowm[row], l = s.rowl[row], pb = s.rowpb[row];
          const float lse = m + logf(l + 1e-12f);
          const float inv = expf(m - lse);
          const float o0 = (acc[2 * half] + pb * bv0) * inv;
          const float o1 = (acc[2 * half + 1] + pb * bv1) * inv;
          *reinterpret_cast<uint32_t*>((T*)a.out + (bh * N + n0 + row) * TD + col) = pack2<T>(o0, o1);
          if (warp == 0 && tq == 0) a.lse[bh * N + n0 + row] = lse;
        }
      }
    }
    __syncthreads();
  }
}

template <typename T>
__global__ void __launch_bounds__(TC_THREADS) nbhd_tc_bwd_kernel(NbhdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BwdSmem<T>& s = *reinterpret_cast<BwdSmem<T>*>(smem_raw);
  const int N = a.N, M = a.M, H = a.H;
  const int tiles = (N + TQ - 1) / TQ;
  const int b = blockIdx.x / tiles;
  const int n0 = (blockIdx.x % tiles) * TQ;
  const int nq = min(TQ, N - n0);
  const int U = tile_union(s.setup, a.midx, b, n0, nq, N, M);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;

  if (U > UCAP) {  // CUDA-core rows; blank-token grads go straight to global
    for (int w = warp; w < H * nq; w += TC_THREADS / 32) {
      const int h = w / nq;
      nbhd_bwd_row<T, 4>(a, b, h, n0 + w % nq, a.dbk + (int64_t)h * TD, a.dbv + (int64_t)h * TD);
    }
    return;
  }
  const int Upad = (U + 15) & ~15;
  const int r = t >> 3, sub = t & 7;
  for (int h = 0; h < H; ++h) {
    const int64_t bh = (int64_t)b * H + h;
    gather_rows(s.K, (const T*)a.k + bh * N * TD, s.setup.ukey, U, Upad);
    gather_rows(s.V, (const T*)a.v + bh * N * TD, s.setup.ukey, U, Upad);
    load_qtile(s.Q, (const T*)a.q + (bh * N + n0) * TD, nq);
    load_qtile(s.dO, (const T*)a.dout + (bh * N + n0) * TD, nq);
    for (int i = t; i < TQ * SST; i += TC_THREADS) { s.P32[i] = 0.f; s.dS32[i] = 0.f; }
    if (t < TD) { s.dbk[t] = 0.f; s.dbv[t] = 0.f; }
    cp_async_wait_all();
    __syncthreads();
    // Delta = rowsum(O * dO) and lse, 8 threads per row
    {
      float p = 0.f;
      if (r < nq) {
        const T* orow = (const T*)a.o + (bh * N + n0 + r) * TD + sub * 4;
#pragma unroll
        for (int e = 0; e < 4; ++e) p = fmaf(ldf(orow + e), io<T>::ld(s.dO + r * KST + sub * 4 + e), p);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
      if (sub == 0) {
        s.delta[r] = p;
        s.lse[r] = r < nq ? a.lse[bh * N + n0 + r] : 0.f;
      }
    }
    mma_rows_by_union(s.S, s.Q, s.K, Upad);
    mma_rows_by_union(s.dP, s.dO, s.V, Upad);
    __syncthreads();
    // ---- per-entry p, ds, dbias
    {
      const bool rowok = r < nq;
      const uint8_t* mr = a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n0 + r) * M : nullptr;
      const T* br = a.bias ? (const T*)a.bias + (bh * N + n0 + r) * M : nullptr;
      T* dbr = a.dbias ? (T*)a.dbias + (bh * N + n0 + r) * M : nullptr;
      const float lse = s.lse[r], delta = s.delta[r];
      for (int e = sub; e < M && rowok; e += 8) {
        const bool valid = mr == nullptr || mr[e] != 0;
        float ds = 0.f;
        if (valid) {
          const int u = s.setup.uof[r * M + e];
          float v = s.S[r * SST + u] * a.scale;
          if (br) v += ldf(br + e);
          const float p = expf(v - lse);
          ds = p * (s.dP[r * SST + u] - delta);
          atomicAdd(&s.P32[r * SST + u], p);
          atomicAdd(&s.dS32[r * SST + u], ds);
        }
        if (dbr) stf(dbr + e, ds);
      }
      if (a.blank_k) {
        const float sb = row_dot8(s.Q + r * KST, (const T*)a.blank_k + (int64_t)h * TD, sub) * a.scale;
        const float dpb = row_dot8(s.dO + r * KST, (const T*)a.blank_v + (int64_t)h * TD, sub);
        const float pb = rowok ? expf(sb - lse) : 0.f;
        const float dsb = pb * (dpb - delta);
        if (sub == 0) s.dsb[r] = dsb;
        // blank-token grads: dbk += scale*dsb*q, dbv += pb*dO (4 dims per thread)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = sub * 4 + e;
          float gk = a.scale * dsb * io<T>::ld(s.Q + r * KST + d);
          float gv = pb * io<T>::ld(s.dO + r * KST + d);
          // reduce over the 4 rows held by this warp (lanes 8 apart)
          gk += __shfl_xor_sync(0xffffffffu, gk, 8);
          gk += __shfl_xor_sync(0xffffffffu, gk, 16);
          gv += __shfl_xor_sync(0xffffffffu, gv, 8);
          gv += __shfl_xor_sync(0xffffffffu, gv, 16);
          if (lane < 8) { atomicAdd(&s.dbk[d], gk); atomicAdd(&s.dbv[d], gv); }
        }
      } else if (sub == 0) {
        s.dsb[r] = 0.f;
      }
    }
    __syncthreads();
    for (int i = t; i < TQ * (Upad / 2); i += TC_THREADS) {
      const int row = i / (Upad / 2), c = (i % (Upad / 2)) * 2;
      *reinterpret_cast<uint32_t*>(&s.P16[row * PST + c]) = pack2<T>(s.P32[row * SST + c], s.P32[row * SST + c + 1]);
      *reinterpret_cast<uint32_t*>(&s.dS16[row * PST + c]) = pack2<T>(s.dS32[row * SST + c], s.dS32[row * SST + c + 1]);
    }
    if (a.blank_k && t < TD) {
      red_add(a.dbk + (int64_t)h * TD + t, s.dbk[t]);
      red_add(a.dbv + (int64_t)h * TD + t, s.dbv[t]);
    }
    __syncthreads();
    // ---- dQ = scale * (dS K_U + dsb bk)
    {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int d0 = warp * 8;
      mma_p_by_rows(acc, s.dS16, s.K, Upad, d0);
      const int g = lane >> 2, tq = lane & 3;
      const int col = d0 + 2 * tq;
      float bk0 = 0.f, bk1 = 0.f;
      if (a.blank_k) {
        bk0 = ldf((const T*)a.blank_k + (int64_t)h * TD + col);
        bk1 = ldf((const T*)a.blank_k + (int64_t)h * TD + col + 1);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int row = g + half * 8;
        if (row < nq) {
          const float dsb = s.dsb[row];
          *reinterpret_cast<uint32_t*>((T*)a.dq + (bh * N + n0 + row) * TD + col) =
              pack2<T>((acc[2 * half] + dsb * bk0) * a.scale, (acc[2 * half + 1] + dsb * bk1) * a.scale);
        }
      }
    }
    // ---- dK_U = scale * dS^T Q, dV_U = P^T dO, scattered once per key row
    mma_scatter_union(s.dS16, s.Q, s.setup.ukey, U, Upad, a.scale, a.dk + bh * N * TD);
    mma_scatter_union(s.P16, s.dO, s.setup.ukey, U, Upad, 1.f, a.dv + bh * N * TD);
    __syncthreads();
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
