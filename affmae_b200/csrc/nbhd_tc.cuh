// Tensor-core neighbourhood attention (see nbhd_attn_tc.cu).
#pragma once

#include "nbhd_row.cuh"

namespace affb {

// 16-bit storage, head_dim 32 and at most 64 neighbours per query.
inline bool nbhd_tc_supported(int dtype, int64_t D, int64_t M) {
  return (dtype == AFFB_BF16 || dtype == AFFB_F16) && D == 32 && M <= 64 && M >= 1;
}

// Cluster-block kernels (nbhd_attn_blk.cu).
int nbhd_blk_fwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st);
int nbhd_blk_bwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st);

}  // namespace affb
