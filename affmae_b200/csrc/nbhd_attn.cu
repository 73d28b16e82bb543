// Neighbourhood (cluster) softmax attention, forward and backward, CUDA-core
// path for every storage type.
//
// Semantics of _nbhood_attn_fwd / _nbhood_attn_bwd_internal
// (src/layers/kernels/local_attn.py:224-340, :387-553):
//   s_j = scale * q . k[idx_j] + bias_j           (valid neighbour j)
//   s_j = -1e11, k = v = 0, bias ignored          (masked neighbour j)
//   s_b = scale * q . blank_k[h]                  (optional blank token)
//   p = softmax over {s_j} U {s_b};  o = sum_j p_j v[idx_j] + p_b blank_v[h]
//   lse = m + log(l + 1e-12)
// The reference pads the neighbour loop to a multiple of its block width
// (smallest_valid_power_2(M), local_attn.py:46-57); padded columns behave
// like masked ones and only matter when every neighbour of a row is masked
// and there is no blank token.  That count is reproduced here.
// Unlike the reference, O is stored directly in the input dtype (the
// reference rounds it through fp16 even for fp32 inputs, local_attn.py:340).
//
// Layout: one warp per (b, h, query); LPN lanes share one neighbour (each
// lane owns 8 head dims), so a warp works on 32/LPN neighbours at a time.
// Each neighbour group keeps its own online-softmax state, merged across the
// groups with shuffles at the end (split-K softmax inside a warp).
// Backward: dq is reduced in registers; dk/dv go to fp32 accumulators with
// vector reductions (red.global.add.v4.f32); dbias is written directly (each
// (row, neighbour) is owned by one lane group); blank-token gradients are
// reduced per block in shared memory before one global reduction per block.
#include "common.cuh"

#include <type_traits>

namespace affb {

constexpr int NA_WARPS = 8;

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

template <typename T, int LPN>
__global__ void __launch_bounds__(NA_WARPS * 32)
nbhd_attn_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                     const int32_t* __restrict__ midx, const T* __restrict__ bias,
                     const uint8_t* __restrict__ mask, int mask_heads,
                     const T* __restrict__ blank_k, const T* __restrict__ blank_v, int H, int N,
                     int D, int M, float scale, T* __restrict__ out, float* __restrict__ lse) {
  constexpr int NPP = 32 / LPN;
  const int lane = threadIdx.x & 31;
  const int nblk = (N + NA_WARPS - 1) / NA_WARPS;
  const int bh = blockIdx.x / nblk;
  const int n = (blockIdx.x % nblk) * NA_WARPS + (threadIdx.x >> 5);
  if (n >= N) return;
  const int b = bh / H, h = bh % H;
  const int ch = lane % LPN, g = lane / LPN;
  const bool dvalid = ch * 8 < D;
  const int64_t row = (int64_t)bh * N + n;

  float qv[8];
  load8_or_zero(q + row * D + ch * 8, dvalid, qv);

  const int32_t* ir = midx + ((int64_t)b * N + n) * M;
  const uint8_t* mr = mask ? mask + (((int64_t)b * mask_heads + (mask_heads == 1 ? 0 : h)) * N + n) * M : nullptr;
  const T* br = bias ? bias + row * M : nullptr;
  const T* kb = k + (int64_t)bh * N * D + ch * 8;
  const T* vb = v + (int64_t)bh * N * D + ch * 8;

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
    float s = group_sum<LPN>(part) * scale;
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
  // merge the neighbour groups of the warp
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
  // padded (always-masked) columns of the reference's neighbour loop
  const int pad = padded_neighbours(M) - M;
  if (pad > 0) l += (float)pad * expf(-1e11f - m_run);

  if (blank_k) {
    float bk[8], bv[8];
    load8_or_zero(blank_k + (int64_t)h * D + ch * 8, dvalid, bk);
    load8_or_zero(blank_v + (int64_t)h * D + ch * 8, dvalid, bv);
    float part = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) part = fmaf(qv[e], bk[e], part);
    const float sb = group_sum<LPN>(part) * scale;
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
    st8(out + row * D + ch * 8, o);
  }
  if (lane == 0) lse[row] = lrow;
}

template <typename T, int LPN>
__global__ void __launch_bounds__(NA_WARPS * 32)
nbhd_attn_bwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                     const T* __restrict__ o, const T* __restrict__ dout,
                     const float* __restrict__ lse, const int32_t* __restrict__ midx,
                     const T* __restrict__ bias, const uint8_t* __restrict__ mask,
                     int mask_heads, const T* __restrict__ blank_k,
                     const T* __restrict__ blank_v, int H, int N, int D, int M, float scale,
                     T* __restrict__ dq, float* __restrict__ dk, float* __restrict__ dv,
                     T* __restrict__ dbias, float* __restrict__ dbk, float* __restrict__ dbv) {
  constexpr int NPP = 32 / LPN;
  __shared__ float s_dbk[256], s_dbv[256];
  const int lane = threadIdx.x & 31;
  const int nblk = (N + NA_WARPS - 1) / NA_WARPS;
  const int bh = blockIdx.x / nblk;
  const int n = (blockIdx.x % nblk) * NA_WARPS + (threadIdx.x >> 5);
  const bool active = n < N;
  const int b = bh / H, h = bh % H;
  const int ch = lane % LPN, g = lane / LPN;
  const bool dvalid = ch * 8 < D;
  const int64_t row = (int64_t)bh * N + n;

  if (blank_k) {
    for (int i = threadIdx.x; i < D; i += blockDim.x) { s_dbk[i] = 0.f; s_dbv[i] = 0.f; }
    __syncthreads();
  }

  if (active) {
    float qv[8], dov[8], ov[8];
    load8_or_zero(q + row * D + ch * 8, dvalid, qv);
    load8_or_zero(dout + row * D + ch * 8, dvalid, dov);
    load8_or_zero(o + row * D + ch * 8, dvalid, ov);
    float part = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) part = fmaf(ov[e], dov[e], part);
    const float delta = group_sum<LPN>(part);
    const float lrow = lse[row];

    const int32_t* ir = midx + ((int64_t)b * N + n) * M;
    const uint8_t* mr = mask ? mask + (((int64_t)b * mask_heads + (mask_heads == 1 ? 0 : h)) * N + n) * M : nullptr;
    const T* br = bias ? bias + row * M : nullptr;
    const int64_t base = (int64_t)bh * N * D + ch * 8;

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
      float s = group_sum<LPN>(pk) * scale;
      const float dp = group_sum<LPN>(pv);
      if (!valid) s = -1e11f;
      else if (br) s += ldf(br + j);
      const float p = expf(s - lrow);
      const float ds = p * (dp - delta);
      if (valid) {
#pragma unroll
        for (int e = 0; e < 8; ++e) dqa[e] = fmaf(ds, kc[e], dqa[e]);
        if (dvalid) {
          float* dkp = dk + base + (int64_t)kid * D;
          float* dvp = dv + base + (int64_t)kid * D;
          const float sd = scale * ds;
          red_add_v4(dkp, sd * qv[0], sd * qv[1], sd * qv[2], sd * qv[3]);
          red_add_v4(dkp + 4, sd * qv[4], sd * qv[5], sd * qv[6], sd * qv[7]);
          red_add_v4(dvp, p * dov[0], p * dov[1], p * dov[2], p * dov[3]);
          red_add_v4(dvp + 4, p * dov[4], p * dov[5], p * dov[6], p * dov[7]);
        }
      }
      if (inb && dbias && ch == 0) stf(dbias + row * M + j, valid ? ds : 0.f);
    }
#pragma unroll
    for (int off = LPN; off < 32; off <<= 1)
#pragma unroll
      for (int e = 0; e < 8; ++e) dqa[e] += __shfl_xor_sync(0xffffffffu, dqa[e], off);

    if (blank_k) {
      float bk[8], bv[8];
      load8_or_zero(blank_k + (int64_t)h * D + ch * 8, dvalid, bk);
      load8_or_zero(blank_v + (int64_t)h * D + ch * 8, dvalid, bv);
      float pk = 0.f, pv = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        pk = fmaf(qv[e], bk[e], pk);
        pv = fmaf(dov[e], bv[e], pv);
      }
      const float sb = group_sum<LPN>(pk) * scale;
      const float dpb = group_sum<LPN>(pv);
      const float pb = expf(sb - lrow);
      const float dsb = pb * (dpb - delta);
#pragma unroll
      for (int e = 0; e < 8; ++e) dqa[e] = fmaf(dsb, bk[e], dqa[e]);
      if (g == 0 && dvalid) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          atomicAdd(&s_dbk[ch * 8 + e], scale * dsb * qv[e]);
          atomicAdd(&s_dbv[ch * 8 + e], pb * dov[e]);
        }
      }
    }
    if (g == 0 && dvalid) {
      float r[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = dqa[e] * scale;
      st8(dq + row * D + ch * 8, r);
    }
  }
  if (blank_k) {
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      red_add(dbk + (int64_t)h * D + i, s_dbk[i]);
      red_add(dbv + (int64_t)h * D + i, s_dbv[i]);
    }
  }
}

static int check_na(int64_t B, int64_t H, int64_t N, int64_t D, int64_t M, int mask_heads,
                    const void* bk, const void* bv, const void* q, const void* k, const void* v) {
  AFFB_REQUIRE(B >= 0 && H >= 1 && N >= 0 && M >= 0, "nbhd_attn: invalid sizes");
  AFFB_REQUIRE(D % 8 == 0 && D >= 8 && D <= 256,
               "nbhd_attn: head_dim must be a multiple of 8 in [8, 256] (got %lld)", (long long)D);
  AFFB_REQUIRE(M % 8 == 0, "nbhd_attn: neighbor_size must be a multiple of 8 (got %lld)", (long long)M);
  AFFB_REQUIRE(mask_heads == 1 || mask_heads == H, "nbhd_attn: mask heads must be 1 or H");
  AFFB_REQUIRE((bk == nullptr) == (bv == nullptr),
               "nbhd_attn: blank_k and blank_v must both be given or both be NULL");
  AFFB_REQUIRE(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0,
               "nbhd_attn: q/k/v must be 16-byte aligned");
  AFFB_REQUIRE(((N + NA_WARPS - 1) / NA_WARPS) * B * H < (1ll << 31) && N < (1ll << 30),
               "nbhd_attn: size too large");
  return AFFB_OK;
}

template <typename F>
static void dispatch_lpn(int64_t D, F&& f) {
  const int c = (int)((D + 7) / 8);
  if (c <= 1) f(std::integral_constant<int, 1>{});
  else if (c <= 2) f(std::integral_constant<int, 2>{});
  else if (c <= 4) f(std::integral_constant<int, 4>{});
  else if (c <= 8) f(std::integral_constant<int, 8>{});
  else if (c <= 16) f(std::integral_constant<int, 16>{});
  else f(std::integral_constant<int, 32>{});
}

}  // namespace affb

using namespace affb;

extern "C" int affb_nbhd_attn_fwd(const void* q, const void* k, const void* v,
                                  const int32_t* member_idx, const void* bias,
                                  const uint8_t* mask, int mask_heads, const void* blank_k,
                                  const void* blank_v, int dtype, int64_t B, int64_t H,
                                  int64_t N, int64_t D, int64_t M, float scale, void* out,
                                  float* lse, void* stream) {
  if (int e = check_na(B, H, N, D, M, mask ? mask_heads : 1, blank_k, blank_v, q, k, v)) return e;
  if (B == 0 || N == 0) return AFFB_OK;
  dim3 grid((unsigned)(((N + NA_WARPS - 1) / NA_WARPS) * B * H));
  cudaStream_t st = as_stream(stream);
  AFFB_DISPATCH(dtype, T, dispatch_lpn(D, [&](auto L) {
    nbhd_attn_fwd_kernel<T, decltype(L)::value><<<grid, NA_WARPS * 32, 0, st>>>(
        (const T*)q, (const T*)k, (const T*)v, member_idx, (const T*)bias, mask, mask_heads,
        (const T*)blank_k, (const T*)blank_v, (int)H, (int)N, (int)D, (int)M, scale, (T*)out, lse);
  }));
  AFFB_LAUNCH_CHECK("affb_nbhd_attn_fwd");
  return AFFB_OK;
}

extern "C" int affb_nbhd_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                                  const void* dout, const float* lse,
                                  const int32_t* member_idx, const void* bias,
                                  const uint8_t* mask, int mask_heads, const void* blank_k,
                                  const void* blank_v, int dtype, int64_t B, int64_t H,
                                  int64_t N, int64_t D, int64_t M, float scale, void* dq,
                                  float* dk_acc, float* dv_acc, void* dbias, float* dbk_acc,
                                  float* dbv_acc, void* stream) {
  if (int e = check_na(B, H, N, D, M, mask ? mask_heads : 1, blank_k, blank_v, q, k, v)) return e;
  AFFB_REQUIRE(!blank_k || (dbk_acc && dbv_acc), "nbhd_attn_bwd: blank gradients need dbk/dbv buffers");
  AFFB_REQUIRE(!bias || dbias, "nbhd_attn_bwd: bias given without a dbias buffer");
  AFFB_REQUIRE(((uintptr_t)dk_acc | (uintptr_t)dv_acc) % 16 == 0,
               "nbhd_attn_bwd: dk/dv accumulators must be 16-byte aligned");
  if (B == 0 || N == 0) return AFFB_OK;
  dim3 grid((unsigned)(((N + NA_WARPS - 1) / NA_WARPS) * B * H));
  cudaStream_t st = as_stream(stream);
  AFFB_DISPATCH(dtype, T, dispatch_lpn(D, [&](auto L) {
    nbhd_attn_bwd_kernel<T, decltype(L)::value><<<grid, NA_WARPS * 32, 0, st>>>(
        (const T*)q, (const T*)k, (const T*)v, (const T*)o, (const T*)dout, lse, member_idx,
        (const T*)bias, mask, mask_heads, (const T*)blank_k, (const T*)blank_v, (int)H, (int)N,
        (int)D, (int)M, scale, (T*)dq, dk_acc, dv_acc, bias ? (T*)dbias : nullptr, dbk_acc,
        dbv_acc);
  }));
  AFFB_LAUNCH_CHECK("affb_nbhd_attn_bwd");
  return AFFB_OK;
}
