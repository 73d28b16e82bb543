// Error reporting, device queries and the fp32 -> storage cast.
#include "common.cuh"

namespace affb {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

template <typename T>
__global__ void cast_f32_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) io<T>::st(dst + i, src[i]);
}

}  // namespace affb

using namespace affb;

extern "C" const char* affb_last_error(void) { return g_err; }
extern "C" int affb_abi_version(void) { return 1; }

extern "C" int affb_cast_f32(const float* src, void* dst, int dtype, int64_t n, void* stream) {
  AFFB_REQUIRE(n >= 0, "affb_cast_f32: negative size");
  if (n == 0) return AFFB_OK;
  const int64_t blocks = imin64((n + 255) / 256, (int64_t)sm_count() * 8);
  AFFB_DISPATCH(dtype, T,
                cast_f32_kernel<T><<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(src, (T*)dst, n));
  AFFB_LAUNCH_CHECK("affb_cast_f32");
  return AFFB_OK;
}
