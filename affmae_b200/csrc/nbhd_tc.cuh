// Tensor-core neighbourhood attention (see nbhd_attn_tc.cu).
#pragma once

#include "nbhd_row.cuh"

namespace affb {

// 16-bit storage, head_dim 32 and at most 64 neighbours per query.
inline bool nbhd_tc_supported(int dtype, int64_t D, int64_t M) {
  return (dtype == AFFB_BF16 || dtype == AFFB_F16) && D == 32 && M <= 64 && M >= 1;
}

// Workspace of the tensor-core path: a tile counter and the list of tiles
// that need the neighbour-union kernels.
inline int64_t nbhd_tc_workspace_bytes(int64_t B, int64_t N) { return 16 + 4 * B * ((N + 15) / 16); }

// Cluster-block kernels (nbhd_attn_blk.cu): every tile whose neighbour lists
// are runs of 8 consecutive keys starting at multiples of 8; other tiles are
// appended to a.fb_list.
int nbhd_blk_fwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st);
int nbhd_blk_bwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st);
// Neighbour-union kernels (nbhd_attn_tc.cu) over the listed tiles.
int nbhd_tc_fwd_list(const NbhdArgs& a, int dtype, int B, cudaStream_t st);
int nbhd_tc_bwd_list(const NbhdArgs& a, int dtype, int B, cudaStream_t st);

}  // namespace affb
