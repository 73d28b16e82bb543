// ReLU followed by dropout in one pass, and its gradient in one pass.
//
// The decoder's feed-forward network (reference src/layers/decoder.py:138-141)
// computes linear2(dropout(relu(linear1(x)))).  PyTorch runs the ReLU, then a
// dropout that writes its output and a byte mask, and in the backward a
// dropout gradient and a ReLU gradient: four passes over the [rows, 2C]
// hidden activations (the largest tensors of the decoder).  Here
//   forward:  y = (x > 0 and keep(e)) ? x / (1 - p) : 0
//   backward: dx = (y > 0) ? dy / (1 - p) : 0
// keep(e) is the counter-based dropout bit of element e (Philox-4x32-10, the
// same stream as the fused LayerNorm's dropout).  The backward needs no mask:
// y > 0 exactly when the element was kept and x > 0, and y is saved anyway as
// the input of linear2's weight gradient.  Products are formed in fp32 and
// rounded once, as PyTorch's kernels do.
#include "common.cuh"
#include "philox.cuh"

namespace affb {

template <typename T, int VEC>
__global__ void __launch_bounds__(256) relu_drop_fwd_kernel(const T* __restrict__ x, int64_t n, uint32_t thr,
                                                            float scale, uint32_t seed, T* __restrict__ y) {
  const int64_t nv = n / VEC;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * VEC;
    T v[VEC];
    if constexpr (VEC == 1) {
      v[0] = x[e];
    } else {
      *reinterpret_cast<uint4*>(v) = reinterpret_cast<const uint4*>(x)[i];
    }
    uint32_t w[VEC];
    if (thr != 0u) {
      if constexpr (VEC % 4 == 0) {
#pragma unroll
        for (int k = 0; k < VEC; k += 4) drop_words<4>(seed, (uint64_t)(e + k), w + k);
      } else {
        drop_words<VEC>(seed, (uint64_t)e, w);
      }
    }
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      const float f = ldf(&v[k]);
      const bool keep = thr == 0u || w[k] >= thr;
      stf(&v[k], (f > 0.f && keep) ? f * scale : 0.f);
    }
    if constexpr (VEC == 1) {
      y[e] = v[0];
    } else {
      reinterpret_cast<uint4*>(y)[i] = *reinterpret_cast<const uint4*>(v);
    }
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(256) relu_drop_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ y,
                                                            int64_t n, float scale, T* __restrict__ dx) {
  const int64_t nv = n / VEC;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    T g[VEC], o[VEC];
    if constexpr (VEC == 1) {
      g[0] = dy[i];
      o[0] = y[i];
    } else {
      *reinterpret_cast<uint4*>(g) = reinterpret_cast<const uint4*>(dy)[i];
      *reinterpret_cast<uint4*>(o) = reinterpret_cast<const uint4*>(y)[i];
    }
#pragma unroll
    for (int k = 0; k < VEC; ++k) stf(&g[k], ldf(&o[k]) > 0.f ? ldf(&g[k]) * scale : 0.f);
    if constexpr (VEC == 1) {
      dx[i] = g[0];
    } else {
      reinterpret_cast<uint4*>(dx)[i] = *reinterpret_cast<const uint4*>(g);
    }
  }
}

static bool aligned16(const void* a, const void* b, const void* c) {
  return (((uintptr_t)a | (uintptr_t)b | (uintptr_t)c) & 15) == 0;
}

}  // namespace affb

using namespace affb;

extern "C" int affb_relu_dropout_fwd(const void* x, int dtype, int64_t n, float p, uint32_t seed, void* y,
                                     void* stream) {
  AFFB_REQUIRE(n >= 0, "relu_dropout: negative size");
  AFFB_REQUIRE(p >= 0.f && p < 1.f, "relu_dropout: dropout probability must be in [0, 1)");
  if (n == 0) return AFFB_OK;
  const uint32_t thr = drop_threshold(p);
  const float scale = 1.f / (1.f - p);
  cudaStream_t st = as_stream(stream);
  AFFB_DISPATCH(dtype, T, {
    constexpr int V = 16 / (int)sizeof(T);
    const bool vec = n % V == 0 && aligned16(x, y, y);
    const int64_t units = vec ? n / V : n;
    const unsigned blocks = (unsigned)imin64((units + 255) / 256, (int64_t)sm_count() * 8);
    if (vec) relu_drop_fwd_kernel<T, V><<<blocks, 256, 0, st>>>((const T*)x, n, thr, scale, seed, (T*)y);
    else relu_drop_fwd_kernel<T, 1><<<blocks, 256, 0, st>>>((const T*)x, n, thr, scale, seed, (T*)y);
  });
  AFFB_LAUNCH_CHECK("affb_relu_dropout_fwd");
  return AFFB_OK;
}

extern "C" int affb_relu_dropout_bwd(const void* dy, const void* y, int dtype, int64_t n, float p, void* dx,
                                     void* stream) {
  AFFB_REQUIRE(n >= 0, "relu_dropout: negative size");
  AFFB_REQUIRE(p >= 0.f && p < 1.f, "relu_dropout: dropout probability must be in [0, 1)");
  if (n == 0) return AFFB_OK;
  const float scale = 1.f / (1.f - p);
  cudaStream_t st = as_stream(stream);
  AFFB_DISPATCH(dtype, T, {
    constexpr int V = 16 / (int)sizeof(T);
    const bool vec = n % V == 0 && aligned16(dy, y, dx);
    const int64_t units = vec ? n / V : n;
    const unsigned blocks = (unsigned)imin64((units + 255) / 256, (int64_t)sm_count() * 8);
    if (vec) relu_drop_bwd_kernel<T, V><<<blocks, 256, 0, st>>>((const T*)dy, (const T*)y, n, scale, (T*)dx);
    else relu_drop_bwd_kernel<T, 1><<<blocks, 256, 0, st>>>((const T*)dy, (const T*)y, n, scale, (T*)dx);
  });
  AFFB_LAUNCH_CHECK("affb_relu_dropout_bwd");
  return AFFB_OK;
}
