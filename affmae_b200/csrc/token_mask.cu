// Token-mask multiply of the masked-autoencoder patch stem.
//
// The reference's AFFPatchEmbed (src/layers/aff.py:591-639) re-applies the
// patch mask after every stride-2 convolution: the [B, H/p, W/p] token mask
// is upsampled by repeat_interleave to the convolution's resolution and
// multiplied into the feature map (and, before the stem, into the image,
// src/models/aff_mae.py), so masked patches never leak into visible tokens.
// PyTorch materialises the upsampled mask at every resolution and runs a
// broadcast multiply over it; here one pass reads each feature element once
// and looks the mask up at (y / s, x / s) in the small token mask:
//   out[b, y, x, c] = x[b, y, x, c] * token_mask[b, y / s, x / s]
// for a channels-last map [B, h, w, C] (C = 1 covers a single-channel image)
// with h = s * th, w = s * tw.  The gradient is the same product.  The
// multiply is exact (the mask is 0 or 1), so the result equals the PyTorch
// sequence bit for bit.
#include "common.cuh"

namespace affb {

template <typename T, int VEC>
__global__ void __launch_bounds__(256) token_mask_kernel(const T* __restrict__ x, const uint8_t* __restrict__ tm,
                                                         int64_t rows, int C, int h, int w, int s, int th, int tw,
                                                         T* __restrict__ out) {
  const int cv = C / VEC;
  const int64_t total = rows * cv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cv;
    const int xx = (int)(r % w);
    const int64_t by = r / w;
    const int yy = (int)(by % h);
    const int64_t b = by / h;
    const bool keep = tm[(b * th + yy / s) * tw + xx / s] != 0;
    if constexpr (VEC == 1) {
      out[i] = keep ? x[i] : T(0.f);
    } else {
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      reinterpret_cast<uint4*>(out)[i] = keep ? reinterpret_cast<const uint4*>(x)[i] : z;
    }
  }
}

}  // namespace affb

using namespace affb;

extern "C" int affb_token_mask_apply(const void* x, int dtype, int64_t B, int64_t h, int64_t w, int64_t C,
                                     const uint8_t* token_mask, int64_t th, int64_t tw, void* out, void* stream) {
  AFFB_REQUIRE(B >= 0 && h >= 0 && w >= 0 && C >= 1 && th >= 1 && tw >= 1, "token_mask: invalid sizes");
  AFFB_REQUIRE(h % th == 0 && w % tw == 0 && h / th == w / tw,
               "token_mask: the map (%lld x %lld) must be an integer upsampling of the mask (%lld x %lld)",
               (long long)h, (long long)w, (long long)th, (long long)tw);
  AFFB_REQUIRE(h < (1ll << 31) && w < (1ll << 31) && C < (1ll << 31), "token_mask: size too large");
  const int64_t rows = B * h * w;
  if (rows == 0) return AFFB_OK;
  const int s = (int)(h / th);
  cudaStream_t st = as_stream(stream);
  const int esz = dtype == AFFB_F32 ? 4 : 2;
  const int vec = 16 / esz;
  const bool v = (C * esz) % 16 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0;
  const int64_t total = rows * (v ? C / vec : C);
  const unsigned blocks = (unsigned)imin64((total + 255) / 256, (int64_t)sm_count() * 16);
  AFFB_DISPATCH(dtype, T, {
    if (v) {
      if (esz == 4) token_mask_kernel<T, 4><<<blocks, 256, 0, st>>>((const T*)x, token_mask, rows, (int)C, (int)h,
                                                                     (int)w, s, (int)th, (int)tw, (T*)out);
      else token_mask_kernel<T, 8><<<blocks, 256, 0, st>>>((const T*)x, token_mask, rows, (int)C, (int)h, (int)w,
                                                            s, (int)th, (int)tw, (T*)out);
    } else {
      token_mask_kernel<T, 1><<<blocks, 256, 0, st>>>((const T*)x, token_mask, rows, (int)C, (int)h, (int)w, s,
                                                       (int)th, (int)tw, (T*)out);
    }
  });
  AFFB_LAUNCH_CHECK("affb_token_mask_apply");
  return AFFB_OK;
}
