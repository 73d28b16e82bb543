// Relative-position attention bias evaluated in the kernel.
//
// The reference builds the bias of ClusterAttention as
//   pe_table = Linear(5 -> H)(pre_table)          (attention.py:111-113)
//   bias[b,h,n,m] = pe_table[pe_idx[b,n,m], h]    (attention.py:120-124)
// where pre_table row i = (dx, dy, r, dy/r, dx/r) of the relative offset
// dx = i % 255 - 127, dy = i / 255 - 127, r = |(dx, dy)|, the last three zero
// at r = 0 (src/utils/pos_embed.py:8-22).  Here each element evaluates
// W[h] . f(pe) + b[h] directly, so the [65025, H] table is never formed, and
// the backward is a reduction into dW [H,5] and db [H] instead of a
// scatter-add of every bias gradient into table rows (most of which hit the
// same few hundred near-zero offsets).
#include "common.cuh"

namespace affb {

constexpr int RB_THREADS = 256;
constexpr int RB_EPT = 8;       // elements per thread in the backward
constexpr int RB_HMAX = 32;

__device__ __forceinline__ void rel_features(int64_t pe, float* f) {
  const int i = (int)pe;
  const float dx = (float)(i % 255 - 127), dy = (float)(i / 255 - 127);
  const float r = sqrtf(dx * dx + dy * dy);
  f[0] = dx;
  f[1] = dy;
  f[2] = r;
  f[3] = r > 0.f ? dy / r : 0.f;
  f[4] = r > 0.f ? dx / r : 0.f;
}

template <typename T>
__global__ void __launch_bounds__(RB_THREADS) rel_bias_fwd_kernel(const float* __restrict__ W,
                                                                  const float* __restrict__ bias,
                                                                  const int64_t* __restrict__ pe, int H,
                                                                  int64_t NM, int64_t total, T* __restrict__ out) {
  __shared__ float sw[RB_HMAX * 6];
  for (int i = threadIdx.x; i < H * 6; i += blockDim.x) sw[i] = i < H * 5 ? W[i] : bias[i - H * 5];
  __syncthreads();
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    float f[5];
    rel_features(__ldg(pe + e), f);
    const int64_t b = e / NM, nm = e - b * NM;
    T* o = out + b * H * NM + nm;
    for (int h = 0; h < H; ++h) {
      float v = sw[H * 5 + h];
#pragma unroll
      for (int k = 0; k < 5; ++k) v = fmaf(sw[h * 5 + k], f[k], v);
      stf(o + h * NM, v);
    }
  }
}

// Each block reduces RB_THREADS * RB_EPT elements for every head: per head, six
// sums (five weight columns and the bias) reduced through shuffles and shared
// memory, then one atomic add per value and block.
template <typename T>
__global__ void __launch_bounds__(RB_THREADS) rel_bias_bwd_kernel(const T* __restrict__ dbias,
                                                                  const int64_t* __restrict__ pe, int H,
                                                                  int64_t NM, int64_t total, float* __restrict__ dW,
                                                                  float* __restrict__ db) {
  __shared__ float part[RB_THREADS / 32][6];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t e0 = (int64_t)blockIdx.x * RB_THREADS * RB_EPT;
  float f[RB_EPT][5];
  int64_t off[RB_EPT];
  bool ok[RB_EPT];
#pragma unroll
  for (int i = 0; i < RB_EPT; ++i) {
    const int64_t e = e0 + i * RB_THREADS + threadIdx.x;
    ok[i] = e < total;
    rel_features(ok[i] ? __ldg(pe + e) : 0, f[i]);
    const int64_t b = ok[i] ? e / NM : 0;
    off[i] = ok[i] ? b * H * NM + (e - b * NM) : 0;
  }
  for (int h = 0; h < H; ++h) {
    float acc[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < RB_EPT; ++i) {
      const float g = ok[i] ? ldf(dbias + off[i] + h * NM) : 0.f;
#pragma unroll
      for (int k = 0; k < 5; ++k) acc[k] = fmaf(g, f[i][k], acc[k]);
      acc[5] += g;
    }
#pragma unroll
    for (int k = 0; k < 6; ++k) acc[k] = warp_sum(acc[k]);
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < 6; ++k) part[warp][k] = acc[k];
    }
    __syncthreads();
    if (threadIdx.x < 6) {
      float s = 0.f;
      for (int w = 0; w < RB_THREADS / 32; ++w) s += part[w][threadIdx.x];
      if (threadIdx.x < 5) red_add(dW + h * 5 + threadIdx.x, s);
      else red_add(db + h, s);
    }
    __syncthreads();
  }
}

}  // namespace affb

using namespace affb;

extern "C" int affb_rel_bias_fwd(const float* weight, const float* bias, const int64_t* pe_idx, int dtype,
                                 int64_t H, int64_t B, int64_t N, int64_t M, void* out, void* stream) {
  AFFB_REQUIRE(H >= 1 && H <= RB_HMAX, "rel_bias: heads must be in [1, %d]", RB_HMAX);
  AFFB_REQUIRE(B >= 0 && N >= 0 && M >= 0, "rel_bias: negative size");
  const int64_t total = B * N * M;
  if (total == 0) return AFFB_OK;
  const int64_t want = (total + RB_THREADS - 1) / RB_THREADS;
  const int blocks = (int)(want < 16LL * sm_count() ? want : 16LL * sm_count());
  AFFB_DISPATCH(dtype, T, rel_bias_fwd_kernel<T><<<blocks, RB_THREADS, 0, as_stream(stream)>>>(
                              weight, bias, pe_idx, (int)H, N * M, total, (T*)out));
  AFFB_LAUNCH_CHECK("affb_rel_bias_fwd");
  return AFFB_OK;
}

extern "C" int affb_rel_bias_bwd(const void* dbias, const int64_t* pe_idx, int dtype, int64_t H, int64_t B,
                                 int64_t N, int64_t M, float* dweight, float* dbias_vec, void* stream) {
  AFFB_REQUIRE(H >= 1 && H <= RB_HMAX, "rel_bias: heads must be in [1, %d]", RB_HMAX);
  AFFB_REQUIRE(B >= 0 && N >= 0 && M >= 0, "rel_bias: negative size");
  const int64_t total = B * N * M;
  if (total == 0) return AFFB_OK;
  const int64_t blocks = (total + RB_THREADS * RB_EPT - 1) / (RB_THREADS * RB_EPT);
  AFFB_REQUIRE(blocks < (1ll << 31), "rel_bias: size too large");
  AFFB_DISPATCH(dtype, T, rel_bias_bwd_kernel<T><<<(unsigned)blocks, RB_THREADS, 0, as_stream(stream)>>>(
                              (const T*)dbias, pe_idx, (int)H, N * M, total, dweight, dbias_vec));
  AFFB_LAUNCH_CHECK("affb_rel_bias_bwd");
  return AFFB_OK;
}
