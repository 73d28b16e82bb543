// Tensor-core neighbourhood attention: dispatch test, backward workspace
// layout and the kernels of nbhd_attn_blk.cu (query side) and
// nbhd_attn_kv.cu (key side).
#pragma once

#include "nbhd_row.cuh"

namespace affb {

// 16-bit storage, head_dim 32 and at most 64 neighbours per query.
inline bool nbhd_tc_supported(int dtype, int64_t D, int64_t M) {
  return (dtype == AFFB_BF16 || dtype == AFFB_F16) && D == 32 && M <= 64 && M >= 1;
}

// Backward workspace.  Tensor-core path: list-form flag, per-cluster counts
// and list offsets, per-entry cluster and rank, the inverse lists,
// D = rowsum(O * dO) per (b, h, n), and fp32 dK / dV sums used only when the
// lists are not all cluster runs.  CUDA-core path: the fp32 dK / dV sums.
struct NbhdBwdLayout {
  int* flag;
  int* counts;
  int* offs;
  int* ecl;
  int* erk;
  int* entries;
  float* di;
  float* dsb;
  void* ds;
  float* acc_k;
  float* acc_v;
  size_t zero_bytes;  // flag + counts, cleared at the start of every call
  size_t total;
};

inline size_t nbhd_align256(size_t x) { return (x + 255) & ~size_t(255); }

inline NbhdBwdLayout nbhd_bwd_layout(bool tc, bool acc_sums, int64_t B, int64_t H, int64_t N, int64_t D, int64_t M,
                                     unsigned char* base) {
  NbhdBwdLayout ly{};
  size_t off = 0;
  auto take = [&](size_t bytes) -> unsigned char* {
    unsigned char* p = base ? base + off : nullptr;
    off += nbhd_align256(bytes);
    return p;
  };
  const size_t acc = (size_t)(B * H * N * D) * sizeof(float);
  if (tc) {
    const int64_t Cc = (N + 7) / 8, J = M / 8;
    ly.flag = (int*)take(256);
    ly.counts = (int*)take((size_t)(B * Cc) * 4);
    ly.zero_bytes = off;
    ly.offs = (int*)take((size_t)(B * Cc) * 4);
    ly.ecl = (int*)take((size_t)(B * N * J) * 4);
    ly.erk = (int*)take((size_t)(B * N * J) * 4);
    ly.entries = (int*)take((size_t)(B * N * J) * 4);
    ly.di = (float*)take((size_t)(B * H * N) * 4);
    ly.dsb = (float*)take((size_t)(B * H * N) * 4);
    ly.ds = take((size_t)(B * H * N * M) * 2);  // 16-bit dS when the call has no dbias output
  }
  if (acc_sums) {
    ly.acc_k = (float*)take(acc);
    ly.acc_v = (float*)take(acc);
  }
  ly.total = off;
  return ly;
}

// Arguments of the key-side kernels.
struct KvArgs {
  const int* flag;
  const int* counts;
  const int* offs;
  const int* entries;
  float* di;         // D = rowsum(O * dO) per (b, h, n)
  float* dsb;        // blank token's dS per (b, h, n)
  void* ds;          // dS in bias layout [B,H,N,M] (the dbias output when there is a bias)
  const float* acc_k;
  const float* acc_v;
  void* dk;
  void* dv;
  int Cc;  // key clusters per image, ceil(N / 8)
};

// Query side (nbhd_attn_blk.cu).  A forward given a.tile_plan (of
// nbhd_tile_plan_bytes) stores its tiles' cluster unions there; a backward
// given the same plan skips rebuilding them in the dQ kernel.
int64_t nbhd_tile_plan_bytes(int64_t B, int64_t N, int64_t M);
int nbhd_blk_fwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st);
int nbhd_blk_bwd(const NbhdArgs& a, int dtype, int B, cudaStream_t st);
int nbhd_blk_dq(const NbhdArgs& a, int dtype, int B, cudaStream_t st);
// Key side (nbhd_attn_kv.cu).
// flag + counts cleared, list count and prologue (one launch), scan, fill
int nbhd_bwd_prepare(const NbhdArgs& a, const KvArgs& k, const NbhdBwdLayout& ly, int dtype, int B,
                     cudaStream_t st);
int nbhd_kv_bwd(const NbhdArgs& a, const KvArgs& k, int dtype, int B, cudaStream_t st);

}  // namespace affb
