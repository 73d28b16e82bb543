// Importance-weighted neighbour gather and its scatter-add backward.
//
//   out[b,i,ic,c] = sum_m w[b,i,m,ic] * feat[b, idx[b,i,m], c]
//
// Forward of WeightedFeaturesFunction (src/layers/kernels/weighted_features.py:30-111)
// and, with IC == 1, WeightedGatherFunction (weighted_gather.py:21-102).
// Backward (weighted_features.py:164-345, weighted_gather.py:127-276):
//   dw[b,i,m,ic]          = sum_c feat[b,idx,c] * dout[b,i,ic,c]
//   dfeat[b,idx[b,i,m],c] += sum_ic w[b,i,m,ic] * dout[b,i,ic,c]
// computed in a single pass over the rows (the reference uses two kernels,
// re-gathering the features in each).
//
// Layout: one warp per output row (b,i).  Lanes cover the channel axis in
// chunks of EPL elements (8 => one 16-byte load per lane for 16-bit types);
// neighbour indices and weights are loaded once per 32 neighbours, one per
// lane, and broadcast with shuffles.  The op is gather-bound: the feature
// rows are the only large traffic, read once per (row, neighbour).
#include <type_traits>

#include "common.cuh"

namespace affb {

constexpr int WF_WARPS = 8;

template <typename T, int EPL>
__device__ __forceinline__ void ld_chunk(const T* p, float* o, int valid) {
  if constexpr (EPL == 8) {
    ld8(p, o);
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = e < valid ? ldf(p + e) : 0.f;
  }
}

template <typename T, int ICT, int EPL>
__global__ void __launch_bounds__(WF_WARPS * 32)
wf_fwd_kernel(const T* __restrict__ w, const T* __restrict__ feat, const int32_t* __restrict__ idx,
              int64_t No, int M, int IC, int ic0, int64_t N, int C, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WF_WARPS + (threadIdx.x >> 5);
  if (row >= No) return;
  const int64_t b = blockIdx.y;
  const int64_t r = b * No + row;
  const int32_t* ir = idx + r * M;
  const T* wr = w + r * (int64_t)M * IC;
  const T* fb = feat + b * N * C;
  // the channel loop is warp-uniform (shuffles inside); lanes past C idle
  for (int cb = 0; cb < C; cb += 32 * EPL) {
    const int c0 = cb + lane * EPL;
    const bool act = c0 < C;
    float acc[ICT][EPL];
#pragma unroll
    for (int i = 0; i < ICT; ++i)
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[i][e] = 0.f;
    for (int m0 = 0; m0 < M; m0 += 32) {
      const int m = m0 + lane;
      int my_idx = 0;
      float my_w[ICT];
#pragma unroll
      for (int i = 0; i < ICT; ++i) my_w[i] = 0.f;
      if (m < M) {
        my_idx = ir[m];
#pragma unroll
        for (int i = 0; i < ICT; ++i)
          if (ic0 + i < IC) my_w[i] = ldf(wr + (int64_t)m * IC + ic0 + i);
      }
      const int cnt = min(32, M - m0);
      for (int t = 0; t < cnt; ++t) {
        const int id = __shfl_sync(0xffffffffu, my_idx, t);
        float wv[ICT];
#pragma unroll
        for (int i = 0; i < ICT; ++i) wv[i] = __shfl_sync(0xffffffffu, my_w[i], t);
        if (!act) continue;
        float f[EPL];
        ld_chunk<T, EPL>(fb + (int64_t)id * C + c0, f, C - c0);
#pragma unroll
        for (int i = 0; i < ICT; ++i)
#pragma unroll
          for (int e = 0; e < EPL; ++e) acc[i][e] = fmaf(wv[i], f[e], acc[i][e]);
      }
    }
    if (!act) continue;
#pragma unroll
    for (int i = 0; i < ICT; ++i) {
      if (ic0 + i >= IC) break;
      T* o = out + (r * IC + ic0 + i) * C + c0;
      if constexpr (EPL == 8) {
        st8(o, acc[i]);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e)
          if (c0 + e < C) stf(o + e, acc[i][e]);
      }
    }
  }
}

template <typename T, int ICT, int EPL>
__global__ void __launch_bounds__(WF_WARPS * 32)
wf_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ w, const T* __restrict__ feat,
              const int32_t* __restrict__ idx, int64_t No, int M, int IC, int ic0, int64_t N,
              int C, T* __restrict__ dw, float* __restrict__ dfeat) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WF_WARPS + (threadIdx.x >> 5);
  if (row >= No) return;
  const int64_t b = blockIdx.y;
  const int64_t r = b * No + row;
  const int32_t* ir = idx + r * M;
  const T* wr = w + r * (int64_t)M * IC;
  const T* dor = dout + r * (int64_t)IC * C;
  const T* fb = feat + b * N * C;
  float* dfb = dfeat + b * N * C;
  for (int m0 = 0; m0 < M; m0 += 32) {
    const int m = m0 + lane;
    int my_idx = 0;
    float my_w[ICT];
#pragma unroll
    for (int i = 0; i < ICT; ++i) my_w[i] = 0.f;
    if (m < M) {
      my_idx = ir[m];
#pragma unroll
      for (int i = 0; i < ICT; ++i)
        if (ic0 + i < IC) my_w[i] = ldf(wr + (int64_t)m * IC + ic0 + i);
    }
    float my_dw[ICT];
#pragma unroll
    for (int i = 0; i < ICT; ++i) my_dw[i] = 0.f;
    const int cnt = min(32, M - m0);
    for (int t = 0; t < cnt; ++t) {
      const int id = __shfl_sync(0xffffffffu, my_idx, t);
      float wv[ICT], part[ICT];
#pragma unroll
      for (int i = 0; i < ICT; ++i) { wv[i] = __shfl_sync(0xffffffffu, my_w[i], t); part[i] = 0.f; }
      for (int c0 = lane * EPL; c0 < C; c0 += 32 * EPL) {
        float f[EPL], g[EPL];
        ld_chunk<T, EPL>(fb + (int64_t)id * C + c0, f, C - c0);
#pragma unroll
        for (int e = 0; e < EPL; ++e) g[e] = 0.f;
#pragma unroll
        for (int i = 0; i < ICT; ++i) {
          if (ic0 + i >= IC) break;
          float d[EPL];
          ld_chunk<T, EPL>(dor + (int64_t)(ic0 + i) * C + c0, d, C - c0);
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            part[i] = fmaf(f[e], d[e], part[i]);
            g[e] = fmaf(wv[i], d[e], g[e]);
          }
        }
        float* dst = dfb + (int64_t)id * C + c0;
        if constexpr (EPL == 8) {
          red_add_v4(dst, g[0], g[1], g[2], g[3]);
          red_add_v4(dst + 4, g[4], g[5], g[6], g[7]);
        } else {
#pragma unroll
          for (int e = 0; e < EPL; ++e)
            if (c0 + e < C) red_add(dst + e, g[e]);
        }
      }
#pragma unroll
      for (int i = 0; i < ICT; ++i) {
        const float s = warp_sum(part[i]);
        if (lane == t) my_dw[i] = s;
      }
    }
    if (m < M) {
#pragma unroll
      for (int i = 0; i < ICT; ++i)
        if (ic0 + i < IC) stf(dw + (r * M + m) * IC + ic0 + i, my_dw[i]);
    }
  }
}


// Vectorised path (C % 8 == 0): lane = slot * GL + chunk, chunk covering 8
// channels; the 32/GL lane groups work on different neighbours at once and
// are summed at the end, so narrow rows (C = 96, 128) keep every lane busy.
template <typename T, int ICT, int GL>
__global__ void __launch_bounds__(WF_WARPS * 32)
wf_fwd_grp_kernel(const T* __restrict__ w, const T* __restrict__ feat, const int32_t* __restrict__ idx,
                  int64_t No, int M, int IC, int ic0, int64_t N, int C, T* __restrict__ out) {
  constexpr int NS = 32 / GL;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WF_WARPS + (threadIdx.x >> 5);
  if (row >= No) return;
  const int slot = lane / GL, ch = lane % GL;
  const int64_t b = blockIdx.y;
  const int64_t r = b * No + row;
  const int32_t* ir = idx + r * M;
  const T* wr = w + r * (int64_t)M * IC;
  const T* fb = feat + b * N * C;
  for (int cb = 0; cb < C; cb += GL * 8) {
    const int c0 = cb + ch * 8;
    const bool act = c0 < C;
    float acc[ICT][8];
#pragma unroll
    for (int i = 0; i < ICT; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
    for (int m0 = 0; m0 < M; m0 += 32) {
      const int m = m0 + lane;
      int my_idx = 0;
      float my_w[ICT];
#pragma unroll
      for (int i = 0; i < ICT; ++i) my_w[i] = 0.f;
      if (m < M) {
        my_idx = ir[m];
#pragma unroll
        for (int i = 0; i < ICT; ++i)
          if (ic0 + i < IC) my_w[i] = ldf(wr + (int64_t)m * IC + ic0 + i);
      }
      const int cnt = min(32, M - m0);
#pragma unroll 2
      for (int t0 = 0; t0 < cnt; t0 += NS) {
        const int t = t0 + slot;
        const int id = __shfl_sync(0xffffffffu, my_idx, t & 31);
        float wv[ICT];
#pragma unroll
        for (int i = 0; i < ICT; ++i) wv[i] = __shfl_sync(0xffffffffu, my_w[i], t & 31);
        if (!act || t >= cnt) continue;
        float f[8];
        ld8(fb + (int64_t)id * C + c0, f);
#pragma unroll
        for (int i = 0; i < ICT; ++i)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[i][e] = fmaf(wv[i], f[e], acc[i][e]);
      }
    }
#pragma unroll
    for (int off = GL; off < 32; off <<= 1)
#pragma unroll
      for (int i = 0; i < ICT; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][e] += __shfl_xor_sync(0xffffffffu, acc[i][e], off);
    if (!act || slot != 0) continue;
#pragma unroll
    for (int i = 0; i < ICT; ++i) {
      if (ic0 + i >= IC) break;
      st8(out + (r * IC + ic0 + i) * C + c0, acc[i]);
    }
  }
}

template <typename T, int ICT, int GL>
__global__ void __launch_bounds__(WF_WARPS * 32)
wf_bwd_grp_kernel(const T* __restrict__ dout, const T* __restrict__ w, const T* __restrict__ feat,
                  const int32_t* __restrict__ idx, int64_t No, int M, int IC, int ic0, int64_t N, int C,
                  T* __restrict__ dw, float* __restrict__ dfeat) {
  constexpr int NS = 32 / GL;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WF_WARPS + (threadIdx.x >> 5);
  if (row >= No) return;
  const int slot = lane / GL, ch = lane % GL;
  const int64_t b = blockIdx.y;
  const int64_t r = b * No + row;
  const int32_t* ir = idx + r * M;
  const T* wr = w + r * (int64_t)M * IC;
  const T* dor = dout + r * (int64_t)IC * C;
  const T* fb = feat + b * N * C;
  float* dfb = dfeat + b * N * C;
  for (int m0 = 0; m0 < M; m0 += 32) {
    const int m = m0 + lane;
    int my_idx = 0;
    float my_w[ICT];
#pragma unroll
    for (int i = 0; i < ICT; ++i) my_w[i] = 0.f;
    if (m < M) {
      my_idx = ir[m];
#pragma unroll
      for (int i = 0; i < ICT; ++i)
        if (ic0 + i < IC) my_w[i] = ldf(wr + (int64_t)m * IC + ic0 + i);
    }
    float my_dw[ICT];
#pragma unroll
    for (int i = 0; i < ICT; ++i) my_dw[i] = 0.f;
    const int cnt = min(32, M - m0);
    for (int t0 = 0; t0 < cnt; t0 += NS) {
      const int t = t0 + slot;
      const bool tv = t < cnt;
      const int id = __shfl_sync(0xffffffffu, my_idx, t & 31);
      float wv[ICT], part[ICT];
#pragma unroll
      for (int i = 0; i < ICT; ++i) { wv[i] = __shfl_sync(0xffffffffu, my_w[i], t & 31); part[i] = 0.f; }
      for (int c0 = ch * 8; c0 < C; c0 += GL * 8) {
        if (!tv) break;
        float f[8], g[8];
        ld8(fb + (int64_t)id * C + c0, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = 0.f;
#pragma unroll
        for (int i = 0; i < ICT; ++i) {
          if (ic0 + i >= IC) break;
          float d[8];
          ld8(dor + (int64_t)(ic0 + i) * C + c0, d);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            part[i] = fmaf(f[e], d[e], part[i]);
            g[e] = fmaf(wv[i], d[e], g[e]);
          }
        }
        float* dst = dfb + (int64_t)id * C + c0;
        red_add_v4(dst, g[0], g[1], g[2], g[3]);
        red_add_v4(dst + 4, g[4], g[5], g[6], g[7]);
      }
#pragma unroll
      for (int i = 0; i < ICT; ++i) {
        float sm = part[i];
#pragma unroll
        for (int off = 1; off < GL; off <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
        // lane (t & 31) keeps the dot of neighbour t (held by group `slot`)
        const float got = __shfl_sync(0xffffffffu, sm, ((lane - t0) & (NS - 1)) * GL);
        if (lane >= t0 && lane < t0 + NS && lane < cnt) my_dw[i] = got;
      }
    }
    if (m < M) {
#pragma unroll
      for (int i = 0; i < ICT; ++i)
        if (ic0 + i < IC) stf(dw + (r * M + m) * IC + ic0 + i, my_dw[i]);
    }
  }
}

template <typename T, int ICT, int GL>
static void launch_grp(bool bwd, const T* dout, const T* w, const T* feat, const int32_t* idx, int64_t B,
                       int64_t No, int M, int IC, int ic0, int64_t N, int C, T* out, T* dw, float* dfeat,
                       cudaStream_t st) {
  dim3 grid((unsigned)((No + WF_WARPS - 1) / WF_WARPS), (unsigned)B);
  if (!bwd) wf_fwd_grp_kernel<T, ICT, GL><<<grid, WF_WARPS * 32, 0, st>>>(w, feat, idx, No, M, IC, ic0, N, C, out);
  else wf_bwd_grp_kernel<T, ICT, GL><<<grid, WF_WARPS * 32, 0, st>>>(dout, w, feat, idx, No, M, IC, ic0, N, C, dw, dfeat);
}

template <typename T, int ICT>
static void launch_wf(bool bwd, const T* dout, const T* w, const T* feat, const int32_t* idx,
                      int64_t B, int64_t No, int M, int IC, int ic0, int64_t N, int C, bool vec,
                      T* out, T* dw, float* dfeat, cudaStream_t st) {
  if (vec) {
    const int cpl = C / 8;  // 8-channel chunks per row
    if (cpl <= 4) launch_grp<T, ICT, 4>(bwd, dout, w, feat, idx, B, No, M, IC, ic0, N, C, out, dw, dfeat, st);
    else if (cpl <= 8) launch_grp<T, ICT, 8>(bwd, dout, w, feat, idx, B, No, M, IC, ic0, N, C, out, dw, dfeat, st);
    else if (cpl <= 16) launch_grp<T, ICT, 16>(bwd, dout, w, feat, idx, B, No, M, IC, ic0, N, C, out, dw, dfeat, st);
    else launch_grp<T, ICT, 32>(bwd, dout, w, feat, idx, B, No, M, IC, ic0, N, C, out, dw, dfeat, st);
    return;
  }
  dim3 grid((unsigned)((No + WF_WARPS - 1) / WF_WARPS), (unsigned)B);
  dim3 block(WF_WARPS * 32);
  if (!bwd) wf_fwd_kernel<T, ICT, 1><<<grid, block, 0, st>>>(w, feat, idx, No, M, IC, ic0, N, C, out);
  else wf_bwd_kernel<T, ICT, 1><<<grid, block, 0, st>>>(dout, w, feat, idx, No, M, IC, ic0, N, C, dw, dfeat);
}

template <typename T>
bool wf_fwd_tc(const T* w, const T* feat, const int32_t* idx, int64_t B, int64_t No, int M, int IC, int64_t N,
               int C, T* out, cudaStream_t st, int* err);

template <typename T>
bool wf_bwd_tc(const T* dout, const T* w, const T* feat, const int32_t* idx, int64_t B, int64_t No, int M, int IC,
               int64_t N, int C, T* dw, float* dfeat, cudaStream_t st, int* err);

// Returns AFFB_OK, or the error of a tensor-core launch that was chosen but
// could not be configured (its message is already set; nothing was launched).
template <typename T>
static int run_wf(bool bwd, const T* dout, const T* w, const T* feat, const int32_t* idx,
                  int64_t B, int64_t No, int M, int IC, int64_t N, int C, T* out, T* dw,
                  float* dfeat, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value) {
    // 16-bit features run on the tensor cores (wf_tc.cu)
    int err = AFFB_OK;
    if (!bwd && wf_fwd_tc<T>(w, feat, idx, B, No, M, IC, N, C, out, st, &err)) return err;
    if (bwd && wf_bwd_tc<T>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st, &err)) return err;
  }
  const bool vec = (C % 8 == 0) && ((uintptr_t)feat % 16 == 0) &&
                   (bwd ? ((uintptr_t)dout % 16 == 0 && (uintptr_t)dfeat % 16 == 0)
                        : ((uintptr_t)out % 16 == 0));
  if (IC == 1) launch_wf<T, 1>(bwd, dout, w, feat, idx, B, No, M, IC, 0, N, C, vec, out, dw, dfeat, st);
  else if (IC == 2) launch_wf<T, 2>(bwd, dout, w, feat, idx, B, No, M, IC, 0, N, C, vec, out, dw, dfeat, st);
  else if (IC <= 4) launch_wf<T, 4>(bwd, dout, w, feat, idx, B, No, M, IC, 0, N, C, vec, out, dw, dfeat, st);
  else
    for (int ic0 = 0; ic0 < IC; ic0 += 8)
      launch_wf<T, 8>(bwd, dout, w, feat, idx, B, No, M, IC, ic0, N, C, vec, out, dw, dfeat, st);
  return AFFB_OK;
}

static int check_wf(int64_t B, int64_t No, int64_t M, int64_t IC, int64_t N, int64_t C) {
  AFFB_REQUIRE(B >= 0 && No >= 0 && M >= 0 && IC >= 1 && N >= 0 && C >= 0,
               "weighted_features: invalid sizes");
  AFFB_REQUIRE(M < (1 << 30) && C < (1 << 30) && IC < (1 << 20) && B < 65536,
               "weighted_features: size too large");
  return AFFB_OK;
}

}  // namespace affb

using namespace affb;

extern "C" int affb_weighted_features_fwd(const void* w, const void* feat, const int32_t* idx,
                                          int dtype, int64_t B, int64_t No, int64_t M,
                                          int64_t IC, int64_t N, int64_t C, void* out,
                                          void* stream) {
  if (int e = check_wf(B, No, M, IC, N, C)) return e;
  if (B == 0 || No == 0 || C == 0) return AFFB_OK;
  int err = AFFB_OK;
  AFFB_DISPATCH(dtype, T,
                err = run_wf<T>(false, nullptr, (const T*)w, (const T*)feat, idx, B, No, (int)M,
                          (int)IC, N, (int)C, (T*)out, nullptr, nullptr, as_stream(stream)));
  if (err != AFFB_OK) return err;
  AFFB_LAUNCH_CHECK("affb_weighted_features_fwd");
  return AFFB_OK;
}

extern "C" int affb_weighted_features_bwd(const void* dout, const void* w, const void* feat,
                                          const int32_t* idx, int dtype, int64_t B,
                                          int64_t No, int64_t M, int64_t IC, int64_t N,
                                          int64_t C, void* dw, float* dfeat_acc,
                                          void* stream) {
  if (int e = check_wf(B, No, M, IC, N, C)) return e;
  if (B == 0 || No == 0 || M == 0) return AFFB_OK;
  int err = AFFB_OK;
  AFFB_DISPATCH(dtype, T,
                err = run_wf<T>(true, (const T*)dout, (const T*)w, (const T*)feat, idx, B, No,
                          (int)M, (int)IC, N, (int)C, nullptr, (T*)dw, dfeat_acc,
                          as_stream(stream)));
  if (err != AFFB_OK) return err;
  AFFB_LAUNCH_CHECK("affb_weighted_features_bwd");
  return AFFB_OK;
}
