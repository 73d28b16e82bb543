// Head-layout copies around the neighbourhood attention.
//
// ClusterAttention (src/layers/attention.py:126-207) projects tokens to
// [B, N, H*d] rows (q) and [B, N, H*2d] rows (k | v per head), while the
// attention operator takes [B, H, N, d]; its output goes back to [B, N, H*d]
// for the projection.  Every one of these moves (and their gradients) is
//   dst[b, n, h, j] = src[b, n, h, j],  j < d,
// with each side addressed by its own (batch, token, head) strides and d
// contiguous.  One thread moves one 16-byte piece; threads run over
// (b, n, h, piece) in that order, so the token-major side is read or written
// in whole rows and the head-major side in runs of d elements.
#include "common.cuh"

namespace affb {

struct Strides3 {
  int64_t b, n, h;
};

__global__ void __launch_bounds__(256) head_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                        int64_t N, int H, int P, Strides3 s, Strides3 t,
                                                        int64_t total) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(i % P);
    const int64_t r = i / P;
    const int h = (int)(r % H);
    const int64_t bn = r / H;
    const int64_t n = bn % N, b = bn / N;
    dst[b * t.b + n * t.n + h * t.h + p] = src[b * s.b + n * s.n + h * s.h + p];
  }
}

}  // namespace affb

using namespace affb;

extern "C" int affb_head_copy(const void* src, int64_t src_sb, int64_t src_sn, int64_t src_sh, void* dst,
                              int64_t dst_sb, int64_t dst_sn, int64_t dst_sh, int64_t elem_bytes, int64_t B,
                              int64_t N, int64_t H, int64_t d, void* stream) {
  AFFB_REQUIRE(B >= 0 && N >= 0 && H >= 1 && d >= 1, "head_copy: invalid sizes");
  AFFB_REQUIRE(elem_bytes == 2 || elem_bytes == 4, "head_copy: element size must be 2 or 4 bytes");
  AFFB_REQUIRE((d * elem_bytes) % 16 == 0, "head_copy: d * element size must be a multiple of 16 bytes");
  AFFB_REQUIRE(((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0, "head_copy: buffers must be 16-byte aligned");
  const int64_t v = 16 / elem_bytes;  // elements per piece
  AFFB_REQUIRE(src_sb % v == 0 && src_sn % v == 0 && src_sh % v == 0 && dst_sb % v == 0 && dst_sn % v == 0 &&
                   dst_sh % v == 0,
               "head_copy: strides must be multiples of 16 bytes");
  const int64_t P = d / v, total = B * N * H * P;
  if (total == 0) return AFFB_OK;
  const Strides3 s{src_sb / v, src_sn / v, src_sh / v}, t{dst_sb / v, dst_sn / v, dst_sh / v};
  const int64_t want = (total + 255) / 256;
  const unsigned blocks = (unsigned)imin64(want, (int64_t)sm_count() * 16);
  head_copy_kernel<<<blocks, 256, 0, as_stream(stream)>>>((const uint4*)src, (uint4*)dst, N, (int)H, (int)P, s, t,
                                                          total);
  AFFB_LAUNCH_CHECK("affb_head_copy");
  return AFFB_OK;
}
