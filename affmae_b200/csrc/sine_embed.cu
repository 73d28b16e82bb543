// Normalised sine position embedding of 2-D token positions.
//
// The decoder embeds query and key positions with PositionEmbeddingSine
// (reference src/layers/decoder.py:16-62, normalize=True, scale 2*pi):
//   t = coord / (max(coord) + 1e-6) * 2*pi,  u_i = t / freq[i]
//   out = [sin(u_x[0::2]), cos(u_x[1::2]), sin(u_y[0::2]), cos(u_y[1::2])]
// PyTorch evaluates it as a dozen passes (divisions, strided slices, sin, cos,
// three concatenations, a cast) over [rows, D]; here one pass writes each
// output element once from the two coordinates of its row, with the same
// fp32 operations in the same order (the maxima and the frequency table come
// from the caller), so the values equal the PyTorch sequence's.
#include "common.cuh"

namespace affb {

constexpr float TWO_PI_F = 6.283185307179586f;

// One thread per (row, frequency pair j < D/4): the four outputs of that
// frequency (sin and cos of x and of y) at channels j, D/4 + j, D/2 + j,
// 3D/4 + j; consecutive threads write consecutive channels of each quarter.
template <typename T>
__global__ void __launch_bounds__(256) sine_embed_kernel(const float* __restrict__ pos, int64_t R, int D,
                                                         const float* __restrict__ maxes,
                                                         const float* __restrict__ freq, T* __restrict__ out) {
  const int quarter = D / 4, half = D / 2;
  const float nx = maxes[0] + 1e-6f, ny = maxes[1] + 1e-6f;
  const int64_t total = R * (int64_t)quarter;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / quarter;
    const int j = (int)(t - r * quarter);
    const float2 p = reinterpret_cast<const float2*>(pos)[r];
    const float tx = __fmul_rn(__fdiv_rn(p.x, nx), TWO_PI_F);
    const float ty = __fmul_rn(__fdiv_rn(p.y, ny), TWO_PI_F);
    const float fs = freq[2 * j], fc = freq[2 * j + 1];
    T* o = out + r * D;
    stf(o + j, sinf(__fdiv_rn(tx, fs)));
    stf(o + quarter + j, cosf(__fdiv_rn(tx, fc)));
    stf(o + half + j, sinf(__fdiv_rn(ty, fs)));
    stf(o + half + quarter + j, cosf(__fdiv_rn(ty, fc)));
  }
}

}  // namespace affb

using namespace affb;

extern "C" int affb_sine_embed(const float* pos, int64_t R, int64_t D, const float* maxes, const float* freq,
                               void* out, int dtype, void* stream) {
  AFFB_REQUIRE(R >= 0 && D >= 4 && D % 4 == 0 && D < (1 << 30), "sine_embed: D must be a positive multiple of 4");
  AFFB_REQUIRE(((uintptr_t)pos & 7) == 0, "sine_embed: positions must be 8-byte aligned");
  if (R == 0) return AFFB_OK;
  cudaStream_t st = as_stream(stream);
  const int64_t total = R * (D / 4);
  const unsigned blocks = (unsigned)imin64((total + 255) / 256, (int64_t)sm_count() * 16);
  AFFB_DISPATCH(dtype, T, {
    sine_embed_kernel<T><<<blocks, 256, 0, st>>>(pos, R, (int)D, maxes, freq, (T*)out);
  });
  AFFB_LAUNCH_CHECK("affb_sine_embed");
  return AFFB_OK;
}
