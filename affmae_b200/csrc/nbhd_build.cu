// Neighbour lists of an AFF encoder stage from the nearest-cluster search.
//
// BasicLayer.forward (src/layers/aff.py:426-465) turns, for every token q
// (tokens in cluster order, clusters of 8 consecutive tokens), the ids c_j of
// its nnc nearest clusters into
//   member_idx[q, 8j + r] = 8 c_j + r            (0 where 8 c_j + r >= n: the
//                                                  padding of a partial last cluster)
//   mask[q, 8j + r]       = 8 c_j + r < n        (only when n % 8 != 0)
//   pe_idx[q, 8j + r]     = y * 255 + x, (x, y) = clamp(pos[member] - pos[q] + 127, 0, 254)
// PyTorch builds these with an expand, a where, a gather of 48 positions per
// token, a clamp and two index products over [B, n, 48] int64 tensors; here
// one thread per (token, run) reads the run's 8 positions (64 contiguous
// bytes) and writes its 8 entries of each output, and member_idx comes out
// as int32, the type the attention kernels read (no per-layer conversion).
// Every step is the fp32 arithmetic of the PyTorch sequence, separately
// rounded, so pe_idx is identical for any positions.
#include "common.cuh"

namespace affb {

__global__ void __launch_bounds__(256) nbhd_build_kernel(const float* __restrict__ pos, const int64_t* __restrict__ nearest,
                                                         int64_t B, int64_t n, int nnc, int32_t* __restrict__ member,
                                                         uint8_t* __restrict__ mask, int64_t* __restrict__ pe_idx) {
  const int64_t total = B * n * nnc;
  const int M = nnc * 8;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(t % nnc);
    const int64_t bq = t / nnc;
    const int64_t b = bq / n;
    const float* pb = pos + b * n * 2;
    const float qx = pos[2 * bq], qy = pos[2 * bq + 1];
    const float tx = __fsub_rn(qx, 127.f), ty = __fsub_rn(qy, 127.f);
    const int64_t c = nearest[t];
    int32_t mi[8];
    uint8_t mk[8];
    int64_t pe[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int64_t raw = c * 8 + r;
      const bool valid = raw < n;
      const int64_t id = valid ? raw : 0;
      mi[r] = (int32_t)id;
      mk[r] = valid ? 1 : 0;
      const float rx = fminf(fmaxf(__fsub_rn(pb[2 * id], tx), 0.f), 254.f);
      const float ry = fminf(fmaxf(__fsub_rn(pb[2 * id + 1], ty), 0.f), 254.f);
      pe[r] = (int64_t)__fadd_rn(__fmul_rn(ry, 255.f), rx);
    }
    const int64_t o = bq * M + 8 * j;
    int4* mo = reinterpret_cast<int4*>(member + o);
    mo[0] = make_int4(mi[0], mi[1], mi[2], mi[3]);
    mo[1] = make_int4(mi[4], mi[5], mi[6], mi[7]);
    if (mask) {
      uint2 u;
      u.x = mk[0] | (mk[1] << 8) | (mk[2] << 16) | ((uint32_t)mk[3] << 24);
      u.y = mk[4] | (mk[5] << 8) | (mk[6] << 16) | ((uint32_t)mk[7] << 24);
      *reinterpret_cast<uint2*>(mask + o) = u;
    }
    longlong2* po = reinterpret_cast<longlong2*>(pe_idx + o);
#pragma unroll
    for (int r = 0; r < 4; ++r) po[r] = make_longlong2(pe[2 * r], pe[2 * r + 1]);
  }
}

}  // namespace affb

using namespace affb;

extern "C" int affb_nbhd_build(const float* pos, const int64_t* nearest, int64_t B, int64_t n, int64_t nnc,
                               int32_t* member_idx, uint8_t* mask, int64_t* pe_idx, void* stream) {
  AFFB_REQUIRE(B >= 0 && n >= 0 && nnc >= 1 && nnc <= 64, "nbhd_build: invalid sizes");
  AFFB_REQUIRE(n < (1ll << 31), "nbhd_build: too many tokens");
  AFFB_REQUIRE(((uintptr_t)member_idx & 15) == 0 && ((uintptr_t)pe_idx & 15) == 0 && ((uintptr_t)mask & 7) == 0,
               "nbhd_build: member_idx / pe_idx must be 16-byte aligned, mask 8-byte aligned");
  const int64_t total = B * n * nnc;
  if (total == 0) return AFFB_OK;
  const unsigned blocks = (unsigned)imin64((total + 255) / 256, (int64_t)sm_count() * 16);
  nbhd_build_kernel<<<blocks, 256, 0, as_stream(stream)>>>(pos, nearest, B, n, (int)nnc, member_idx, mask, pe_idx);
  AFFB_LAUNCH_CHECK("affb_nbhd_build");
  return AFFB_OK;
}
