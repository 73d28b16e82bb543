// Shared building blocks of the tensor-core neighbourhood-attention kernels:
// mma.sync m16n8k16 (bf16 / fp16 in, fp32 accumulate), ldmatrix fragment
// loads, cp.async staging and the chunk-level contractions of the
// cluster-block kernels (nbhd_attn_blk.cu).
#pragma once

#include "nbhd_row.cuh"

namespace affb {

constexpr int TQ = 16;          // queries per tile
constexpr int TD = 32;          // head dim
constexpr int MMAX = 64;        // neighbours per query
constexpr int TC_THREADS = 128;
// Q/K/V/dO tiles in shared memory: rows of TD elements (64 B, unpadded) with
// the 16-byte chunks of row r stored in XOR order ch ^ ((r >> 1) & 3), so the
// eight rows one ldmatrix reads fall in eight distinct bank groups.
__device__ __forceinline__ int swz(int row, int ch) { return row * TD + ((ch ^ ((row >> 1) & 3)) << 3); }
constexpr int NW = TC_THREADS / 32;

// Minimum resident blocks per SM requested from the register allocator.
#ifndef AFFB_FWD_MINB
#define AFFB_FWD_MINB 7  // 72 registers: 7 forward tiles per SM
#endif
#ifndef AFFB_BWD_MINB
#define AFFB_BWD_MINB 1
#endif
#ifndef AFFB_DQ_MINB
#define AFFB_DQ_MINB 12  // 40 registers: 12 dQ tiles per SM (a few bytes spilled; 3.4 us faster at config 3 than 10 tiles at 48)
#endif
#ifndef AFFB_KV_MINB
#define AFFB_KV_MINB 7  // 72 registers: 7 blocks of the key-side kernel per SM (8 blocks at 64 spill and run slower)
#endif
#ifndef AFFB_PRE_MINB
#define AFFB_PRE_MINB 4  // 64 registers: 4 blocks of 256 threads of the backward prologue per SM
#endif

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

// Fragments of S = A B^T for one 16-slot chunk: acc[j] covers slots
// u0 + 8j .. u0 + 8j + 7.  `a` holds the A fragments (16 x 32) of both k-steps.
template <typename T>
__device__ __forceinline__ void mma_chunk_nt(float (*acc)[4], const uint32_t (*a)[4], const T* Bm, int u0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint32_t bb[4];
    ldsm_x4(bb, Bm + swz(u0 + j * 8 + (lane & 7), lane >> 3));
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
    ldsm_x4_t(bb, X + swz(u0 + (j & 1) * 8 + (lane & 7), dp * 2 + (j >> 1)));
    MmaType<T>::mma(out[dp * 2], a, bb);
    MmaType<T>::mma(out[dp * 2 + 1], a, bb + 2);
  }
}

// Scatter-add of R[16 x 32] = Pt[0..15][0..15]^T (16 x 16, row stride pst) *
// Y[16 x 32] (times `mul`) into key rows 8 * uclu[u >> 3] + (u & 7), u = u0 + i,
// of dst (fp32, row stride TD) for u < U and key rows below N (the partial
// last cluster has no rows past the last token).
template <typename T>
__device__ __forceinline__ void mma_chunk_scatter(const T* Pt, int pst, const T* Y, const int* uclu, int U,
                                                  int u0, float mul, float* __restrict__ dst, int N) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  uint32_t a[4];
  // A[m = u][k = q] = Pt[q][u]: matrices (q0-7,u0-7), (q0-7,u8-15), (q8-15,u0-7), (q8-15,u8-15)
  const int j = lane >> 3, rr = lane & 7;
  ldsm_x4_t(a, Pt + ((j >> 1) * 8 + rr) * pst + (j & 1) * 8);
  const int ua = u0 + g, ub = ua + 8;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    uint32_t yb[2];
    ldsm_x2_t(yb, Y + swz(lane & 15, nt));
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    MmaType<T>::mma(acc, a, yb);
    const int col = nt * 8 + 2 * tq;
    const int ka = ua < U ? uclu[ua >> 3] * 8 + (ua & 7) : N;
    const int kb = ub < U ? uclu[ub >> 3] * 8 + (ub & 7) : N;
    if (ka < N) red_add_v2(dst + (int64_t)ka * TD + col, acc[0] * mul, acc[1] * mul);
    if (kb < N) red_add_v2(dst + (int64_t)kb * TD + col, acc[2] * mul, acc[3] * mul);
  }
}

template <typename T>
__device__ __forceinline__ void load_a_frags(uint32_t (*a)[4], const T* A) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks)
    ldsm_x4(a[ks], A + swz((lane & 7) + ((lane >> 3) & 1) * 8, ks * 2 + (lane >> 4)));
}

constexpr float kLog2e = 1.4426950408889634f;

// 2^x by the ex2.approx instruction (the base-2 exponential of the softmaxes).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> __device__ __forceinline__ T neg_inf();
template <> __device__ __forceinline__ __nv_bfloat16 neg_inf<__nv_bfloat16>() { return __ushort_as_bfloat16(0xFF80); }
template <> __device__ __forceinline__ __half neg_inf<__half>() { return __ushort_as_half(0xFC00); }
template <typename T> __device__ __forceinline__ T pos_zero();
template <> __device__ __forceinline__ __nv_bfloat16 pos_zero<__nv_bfloat16>() { return __ushort_as_bfloat16(0); }
template <> __device__ __forceinline__ __half pos_zero<__half>() { return __ushort_as_half(0); }

// cp.async of 16 rows (64 B each): rows src + rowidx(i) * TD for valid i, zeros otherwise.
template <typename T, typename RowOf>
__device__ __forceinline__ void warp_load16(T* dst, const T* __restrict__ src, RowOf rowof) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = lane; i < 64; i += 32) {
    const int row = i >> 2, c = i & 3;
    const int64_t gr = rowof(row);
    cp_async16(dst + swz(row, c), src + (gr < 0 ? 0 : gr) * TD + c * 8, gr >= 0);
  }
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 8 : 0));
}

// cp.async of the tile's bias rows ([TQ][M] of T, contiguous in global) into a
// per-warp staging buffer (rows >= nq zero-filled).
template <typename T>
__device__ __forceinline__ void warp_stage_bias(T* sbias, const NbhdArgs& a, int b, int h, int n0, int nq) {
  const int lane = threadIdx.x & 31;
  const int M = a.M, N = a.N;
  const T* src = (const T*)a.bias + (((int64_t)b * a.H + h) * N + n0) * M;
  const int nch = TQ * M / 8;  // 16-byte chunks
  for (int i = lane; i < nch; i += 32) {
    const bool ok = (i * 8) / M < nq;
    cp_async16(sbias + i * 8, src + (ok ? i * 8 : 0), ok);
  }
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N_>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N_) : "memory"); }

// Partial dot of rows g and g+8 of a smem tile with a global 32-vector over
// dims 8*tq .. 8*tq+7, reduced over the 4 lanes of the row.
template <typename T>
__device__ __forceinline__ void rows_dot(const T* tile, const T* __restrict__ vec, float& d0, float& d1) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  float v[8], x0[8], x1[8];
  ld8(vec + tq * 8, v);
  ld8_shared(tile + swz(g, tq), x0);
  ld8_shared(tile + swz(g + 8, tq), x1);
  d0 = 0.f; d1 = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) { d0 = fmaf(x0[e], v[e], d0); d1 = fmaf(x1[e], v[e], d1); }
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    d0 += __shfl_xor_sync(0xffffffffu, d0, o);
    d1 += __shfl_xor_sync(0xffffffffu, d1, o);
  }
}

}  // namespace affb
