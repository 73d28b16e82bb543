// Shared helpers for the affmae_b200 CUDA library (sm_100a).
//
// Element types crossing the C ABI are identified by an integer code
// (AFFB_F32 / AFFB_F16 / AFFB_BF16, declared in include/affmae_b200.h).
// Kernels compute in fp32 whatever the storage type; loads widen and
// stores narrow with round-to-nearest-even.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/affmae_b200.h"

// Size of the fixed device scratch of affb_deform_knn_fwd_noalloc.
#define AFFB_NOALLOC_SCRATCH_BYTES (16u << 20)

namespace affb {

// ---------------------------------------------------------------- errors --
// Thread-local last-error text, returned by affb_last_error().
void set_error(const char* fmt, ...);

#define AFFB_REQUIRE(cond, ...)                         \
  do {                                                  \
    if (!(cond)) {                                      \
      ::affb::set_error(__VA_ARGS__);                   \
      return AFFB_ERR_INVALID;                          \
    }                                                   \
  } while (0)

#define AFFB_LAUNCH_CHECK(name)                                            \
  do {                                                                     \
    cudaError_t e_ = cudaGetLastError();                                   \
    if (e_ != cudaSuccess) {                                               \
      ::affb::set_error("%s: launch failed: %s", name, cudaGetErrorString(e_)); \
      return AFFB_ERR_CUDA;                                                \
    }                                                                      \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch.  A kernel launched by launch_dependent() may
// be scheduled while its predecessor on the stream is still finishing; its
// first statement must be dependent_wait(), which returns once the
// predecessor grid has completed and its memory operations are visible (and
// is a no-op for a kernel launched the ordinary way).  What this saves is the
// launch gap between the kernels of one chain.
__device__ __forceinline__ void dependent_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                    Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------ conversions --
template <typename T> struct io;
template <> struct io<float> {
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ void st(float* p, float v) { *p = v; }
};
template <> struct io<__half> {
  static __device__ __forceinline__ float ld(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void st(__half* p, float v) { *p = __float2half_rn(v); }
};
template <> struct io<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

template <typename T> __device__ __forceinline__ float ldf(const T* p) { return io<T>::ld(p); }
template <typename T> __device__ __forceinline__ void stf(T* p, float v) { io<T>::st(p, v); }

// Load 8 consecutive elements into fp32.  Pointer aligned to 16 bytes.
__device__ __forceinline__ void ld8(const float* p, float* o) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p));
  float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* o) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = __uint_as_float(w[i] << 16);
    o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void ld8(const __half* p, float* o) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}

// Same loads through generic addressing (shared or global), without the
// read-only cache path.
__device__ __forceinline__ void ld8_shared(const float* p, float* o) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
__device__ __forceinline__ void ld8_shared(const __nv_bfloat16* p, float* o) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = __uint_as_float(w[i] << 16);
    o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void ld8_shared(const __half* p, float* o) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}

// Store 8 fp32 values as 8 consecutive elements of T.
__device__ __forceinline__ void st8(float* p, const float* v) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void st8(__half* p, const float* v) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// fp32 reductions into global memory (vector form needs sm_90+, 16-byte alignment).
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
__device__ __forceinline__ void red_add(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__host__ __device__ inline int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// Number of SMs of the current device (cached per process).
int sm_count();

// Dispatch on the storage dtype code.
#define AFFB_DISPATCH(dtype, T, ...)                                      \
  switch (dtype) {                                                        \
    case AFFB_F32: { using T = float; __VA_ARGS__; break; }               \
    case AFFB_F16: { using T = __half; __VA_ARGS__; break; }              \
    case AFFB_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }      \
    default: ::affb::set_error("unsupported dtype code %d", (int)(dtype)); \
      return AFFB_ERR_INVALID;                                            \
  }

}  // namespace affb
