// Per-(b, h, query) neighbourhood attention on CUDA cores: the building block
// of the CUDA-core kernels (every dtype, any head_dim multiple of 8) and the
// fallback of the tensor-core kernels for query tiles whose neighbour union
// does not fit their shared-memory tile.
//
// Semantics of _nbhood_attn_fwd / _nbhood_attn_bwd_internal
// (src/layers/kernels/local_attn.py:224-340, :387-553):
//   s_j = scale * q . k[idx_j] + bias_j           (valid neighbour j)
//   s_j = -1e11, k = v = 0, bias ignored          (masked neighbour j)
//   s_b = scale * q . blank_k[h]                  (optional blank token)
//   p = softmax over {s_j} U {s_b};  o = sum_j p_j v[idx_j] + p_b blank_v[h]
//   lse = m + log(l + 1e-12)  with the running max m starting at -1e11
// The reference pads the neighbour loop to a multiple of its block width
// (smallest_valid_power_2(M), local_attn.py:46-57); padded columns behave
// like masked ones and only matter when every neighbour of a row is masked
// and there is no blank token.  That count is reproduced here.
//
// Layout: one warp per row; LPN lanes share one neighbour (each lane owns 8
// head dims), so a warp works on 32/LPN neighbours at a time.  Each neighbour
// group keeps its own online-softmax state, merged with shuffles at the end.
#pragma once

#include "common.cuh"

namespace affb {

template <int LPN>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = 1; o < LPN; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ void load8_or_zero(const T* p, bool ok, float* o) {
  if (ok) {
    ld8(p, o);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
  }
}

__host__ __device__ __forceinline__ int padded_neighbours(int M) {
  const int bn = M >= 32 ? 32 : M >= 16 ? 16 : M >= 8 ? 8 : M >= 4 ? 4 : 1;
  return ((M + bn - 1) / bn) * bn;
}

struct NbhdArgs {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* midx;
  const void* bias;
  const uint8_t* mask;
  int mask_heads;
  const void* blank_k;
  const void* blank_v;
  int B, H, N, D, M;
  float scale;
  // forward outputs
  void* out;
  float* lse;
  // backward inputs / outputs
  const void* o;
  const void* dout;
  void* dq;
  float* dk;
  float* dv;
  void* dbias;
  float* dbk;
  float* dbv;
  // cluster-block backward: list-form flag (nonzero: the query-side kernel
  // does the whole backward, scatter-adding dK / dV into dk / dv), dS in bias
  // layout [B,H,N,M] and the blank token's dS per (b, h, n)
  const int* general;
  // optional per-tile cluster unions (nbhd_attn_blk.cu TilePlan): written by
  // the forward, read by the dQ kernel instead of rebuilding them
  void* tile_plan;
  const void* ds;
  const float* dsb;
};

// Forward of one (b, h, n) row by one warp.
template <typename T, int LPN>
__device__ void nbhd_fwd_row(const NbhdArgs& a, int b, int h, int n) {
  constexpr int NPP = 32 / LPN;
  const int lane = threadIdx.x & 31;
  const int ch = lane % LPN, g = lane / LPN;
  const int D = a.D, M = a.M, N = a.N;
  const bool dvalid = ch * 8 < D;
  const int bh = b * a.H + h;
  const int64_t row = (int64_t)bh * N + n;
  const T* q = (const T*)a.q;
  float qv[8];
  load8_or_zero(q + row * D + ch * 8, dvalid, qv);
  const int32_t* ir = a.midx + ((int64_t)b * N + n) * M;
  const uint8_t* mr = a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n) * M : nullptr;
  const T* br = a.bias ? (const T*)a.bias + row * M : nullptr;
  const T* kb = (const T*)a.k + (int64_t)bh * N * D + ch * 8;
  const T* vb = (const T*)a.v + (int64_t)bh * N * D + ch * 8;

  float m_run = -1e11f, l = 0.f, acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int j0 = 0; j0 < M; j0 += NPP) {
    const int j = j0 + g;
    const bool inb = j < M;
    const bool valid = inb && (mr == nullptr || mr[j] != 0);
    const int kid = inb ? ir[j] : 0;
    float kc[8], vc[8];
    load8_or_zero(kb + (int64_t)kid * D, valid && dvalid, kc);
    load8_or_zero(vb + (int64_t)kid * D, valid && dvalid, vc);
    float part = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) part = fmaf(qv[e], kc[e], part);
    float s = group_sum<LPN>(part) * a.scale;
    if (!valid) s = -1e11f;
    else if (br) s += ldf(br + j);
    if (inb) {
      const float mn = fmaxf(m_run, s);
      const float alpha = expf(m_run - mn);
      const float p = expf(s - mn);
      l = l * alpha + p;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(p, vc[e], acc[e] * alpha);
      m_run = mn;
    }
  }
#pragma unroll
  for (int off = LPN; off < 32; off <<= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m_run, off);
    const float ol = __shfl_xor_sync(0xffffffffu, l, off);
    const float mn = fmaxf(m_run, om);
    const float a1 = expf(m_run - mn), a2 = expf(om - mn);
    l = l * a1 + ol * a2;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float oa = __shfl_xor_sync(0xffffffffu, acc[e], off);
      acc[e] = acc[e] * a1 + oa * a2;
    }
    m_run = mn;
  }
  const int pad = padded_neighbours(M) - M;
  if (pad > 0) l += (float)pad * expf(-1e11f - m_run);
  if (a.blank_k) {
    float bk[8], bv[8];
    load8_or_zero((const T*)a.blank_k + (int64_t)h * D + ch * 8, dvalid, bk);
    load8_or_zero((const T*)a.blank_v + (int64_t)h * D + ch * 8, dvalid, bv);
    float part = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) part = fmaf(qv[e], bk[e], part);
    const float sb = group_sum<LPN>(part) * a.scale;
    const float mn = fmaxf(m_run, sb);
    const float alpha = expf(m_run - mn), pb = expf(sb - mn);
    l = l * alpha + pb;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = fmaf(pb, bv[e], acc[e] * alpha);
    m_run = mn;
  }
  const float lrow = m_run + logf(l + 1e-12f);
  const float inv = expf(m_run - lrow);
  if (g == 0 && dvalid) {
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = acc[e] * inv;
    st8((T*)a.out + row * D + ch * 8, o);
  }
  if (lane == 0) a.lse[row] = lrow;
}

// Backward of one (b, h, n) row by one warp.  Blank-token gradients are
// added into dbk_acc / dbv_acc (shared or global memory) with atomics.
template <typename T, int LPN>
__device__ void nbhd_bwd_row(const NbhdArgs& a, int b, int h, int n, float* dbk_acc, float* dbv_acc) {
  constexpr int NPP = 32 / LPN;
  const int lane = threadIdx.x & 31;
  const int ch = lane % LPN, g = lane / LPN;
  const int D = a.D, M = a.M, N = a.N;
  const bool dvalid = ch * 8 < D;
  const int bh = b * a.H + h;
  const int64_t row = (int64_t)bh * N + n;
  float qv[8], dov[8], ov[8];
  load8_or_zero((const T*)a.q + row * D + ch * 8, dvalid, qv);
  load8_or_zero((const T*)a.dout + row * D + ch * 8, dvalid, dov);
  load8_or_zero((const T*)a.o + row * D + ch * 8, dvalid, ov);
  float part = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) part = fmaf(ov[e], dov[e], part);
  const float delta = group_sum<LPN>(part);
  const float lrow = a.lse[row];
  const int32_t* ir = a.midx + ((int64_t)b * N + n) * M;
  const uint8_t* mr = a.mask ? a.mask + (((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N + n) * M : nullptr;
  const T* br = a.bias ? (const T*)a.bias + row * M : nullptr;
  const int64_t base = (int64_t)bh * N * D + ch * 8;
  const T* k = (const T*)a.k;
  const T* v = (const T*)a.v;
  float dqa[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) dqa[e] = 0.f;
  for (int j0 = 0; j0 < M; j0 += NPP) {
    const int j = j0 + g;
    const bool inb = j < M;
    const bool valid = inb && (mr == nullptr || mr[j] != 0);
    const int kid = inb ? ir[j] : 0;
    float kc[8], vc[8];
    load8_or_zero(k + base + (int64_t)kid * D, valid && dvalid, kc);
    load8_or_zero(v + base + (int64_t)kid * D, valid && dvalid, vc);
    float pk = 0.f, pv = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      pk = fmaf(qv[e], kc[e], pk);
      pv = fmaf(dov[e], vc[e], pv);
    }
    float s = group_sum<LPN>(pk) * a.scale;
    const float dp = group_sum<LPN>(pv);
    if (!valid) s = -1e11f;
    else if (br) s += ldf(br + j);
    const float p = expf(s - lrow);
    const float ds = p * (dp - delta);
    if (valid) {
#pragma unroll
      for (int e = 0; e < 8; ++e) dqa[e] = fmaf(ds, kc[e], dqa[e]);
      if (dvalid) {
        float* dkp = a.dk + base + (int64_t)kid * D;
        float* dvp = a.dv + base + (int64_t)kid * D;
        const float sd = a.scale * ds;
        red_add_v4(dkp, sd * qv[0], sd * qv[1], sd * qv[2], sd * qv[3]);
        red_add_v4(dkp + 4, sd * qv[4], sd * qv[5], sd * qv[6], sd * qv[7]);
        red_add_v4(dvp, p * dov[0], p * dov[1], p * dov[2], p * dov[3]);
        red_add_v4(dvp + 4, p * dov[4], p * dov[5], p * dov[6], p * dov[7]);
      }
    }
    if (inb && a.dbias && ch == 0) stf((T*)a.dbias + row * M + j, valid ? ds : 0.f);
  }
#pragma unroll
  for (int off = LPN; off < 32; off <<= 1)
#pragma unroll
    for (int e = 0; e < 8; ++e) dqa[e] += __shfl_xor_sync(0xffffffffu, dqa[e], off);
  if (a.blank_k) {
    float bk[8], bv[8];
    load8_or_zero((const T*)a.blank_k + (int64_t)h * D + ch * 8, dvalid, bk);
    load8_or_zero((const T*)a.blank_v + (int64_t)h * D + ch * 8, dvalid, bv);
    float pk = 0.f, pv = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      pk = fmaf(qv[e], bk[e], pk);
      pv = fmaf(dov[e], bv[e], pv);
    }
    const float sb = group_sum<LPN>(pk) * a.scale;
    const float dpb = group_sum<LPN>(pv);
    const float pb = expf(sb - lrow);
    const float dsb = pb * (dpb - delta);
#pragma unroll
    for (int e = 0; e < 8; ++e) dqa[e] = fmaf(dsb, bk[e], dqa[e]);
    if (g == 0 && dvalid && dbk_acc) {  // null: the blank gradients are summed elsewhere
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        atomicAdd(&dbk_acc[ch * 8 + e], a.scale * dsb * qv[e]);
        atomicAdd(&dbv_acc[ch * 8 + e], pb * dov[e]);
      }
    }
  }
  if (g == 0 && dvalid) {
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = dqa[e] * a.scale;
    st8((T*)a.dq + row * D + ch * 8, r);
  }
}

}  // namespace affb
