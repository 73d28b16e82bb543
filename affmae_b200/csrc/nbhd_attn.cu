// Neighbourhood (cluster) attention entry points.
//
// Dispatch: 16-bit inputs with head_dim 32 and at most 64 neighbours run on
// the tensor-core cluster-block kernels (nbhd_attn_blk.cu), which take every
// 16-query tile whose neighbour lists are runs of 8 consecutive keys (the
// AFFMAE layout) and fall back to CUDA-core rows for other tiles.  Everything
// else (fp32, other head dims) runs on the CUDA-core row kernels below (one
// warp per (b, h, query), see nbhd_row.cuh).
#include "nbhd_row.cuh"
#include "nbhd_tc.cuh"

#include <type_traits>

namespace affb {

constexpr int NA_WARPS = 8;

template <typename T, int LPN>
__global__ void __launch_bounds__(NA_WARPS * 32) nbhd_attn_fwd_kernel(NbhdArgs a) {
  const int nblk = (a.N + NA_WARPS - 1) / NA_WARPS;
  const int bh = blockIdx.x / nblk;
  const int n = (blockIdx.x % nblk) * NA_WARPS + (threadIdx.x >> 5);
  if (n >= a.N) return;
  nbhd_fwd_row<T, LPN>(a, bh / a.H, bh % a.H, n);
}

template <typename T, int LPN>
__global__ void __launch_bounds__(NA_WARPS * 32) nbhd_attn_bwd_kernel(NbhdArgs a) {
  __shared__ float s_dbk[256], s_dbv[256];
  const int nblk = (a.N + NA_WARPS - 1) / NA_WARPS;
  const int bh = blockIdx.x / nblk;
  const int h = bh % a.H;
  const int n = (blockIdx.x % nblk) * NA_WARPS + (threadIdx.x >> 5);
  if (a.blank_k) {
    for (int i = threadIdx.x; i < a.D; i += blockDim.x) { s_dbk[i] = 0.f; s_dbv[i] = 0.f; }
    __syncthreads();
  }
  if (n < a.N) nbhd_bwd_row<T, LPN>(a, bh / a.H, h, n, s_dbk, s_dbv);
  if (a.blank_k) {
    __syncthreads();
    for (int i = threadIdx.x; i < a.D; i += blockDim.x) {
      red_add(a.dbk + (int64_t)h * a.D + i, s_dbk[i]);
      red_add(a.dbv + (int64_t)h * a.D + i, s_dbv[i]);
    }
  }
}

static int check_na(int64_t B, int64_t H, int64_t N, int64_t D, int64_t M, int mask_heads,
                    const void* bk, const void* bv, const void* q, const void* k, const void* v) {
  AFFB_REQUIRE(B >= 0 && H >= 1 && N >= 0 && M >= 0, "nbhd_attn: invalid sizes");
  AFFB_REQUIRE(D % 8 == 0 && D >= 8 && D <= 256,
               "nbhd_attn: head_dim must be a multiple of 8 in [8, 256] (got %lld)", (long long)D);
  AFFB_REQUIRE(M % 8 == 0, "nbhd_attn: neighbor_size must be a multiple of 8 (got %lld)", (long long)M);
  AFFB_REQUIRE(mask_heads == 1 || mask_heads == H, "nbhd_attn: mask heads must be 1 or H");
  AFFB_REQUIRE((bk == nullptr) == (bv == nullptr),
               "nbhd_attn: blank_k and blank_v must both be given or both be NULL");
  AFFB_REQUIRE(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0,
               "nbhd_attn: q/k/v must be 16-byte aligned");
  AFFB_REQUIRE(((N + NA_WARPS - 1) / NA_WARPS) * B * H < (1ll << 31) && N < (1ll << 30),
               "nbhd_attn: size too large");
  return AFFB_OK;
}

template <typename F>
static void dispatch_lpn(int64_t D, F&& f) {
  const int c = (int)((D + 7) / 8);
  if (c <= 1) f(std::integral_constant<int, 1>{});
  else if (c <= 2) f(std::integral_constant<int, 2>{});
  else if (c <= 4) f(std::integral_constant<int, 4>{});
  else if (c <= 8) f(std::integral_constant<int, 8>{});
  else if (c <= 16) f(std::integral_constant<int, 16>{});
  else f(std::integral_constant<int, 32>{});
}

static NbhdArgs make_args(const void* q, const void* k, const void* v, const int32_t* mi,
                          const void* bias, const uint8_t* mask, int mask_heads, const void* bk,
                          const void* bv, int64_t B, int64_t H, int64_t N, int64_t D, int64_t M, float scale) {
  NbhdArgs a{};
  a.q = q; a.k = k; a.v = v; a.midx = mi; a.bias = bias; a.mask = mask;
  a.mask_heads = mask ? mask_heads : 1;
  a.blank_k = bk; a.blank_v = bv;
  a.B = (int)B; a.H = (int)H; a.N = (int)N; a.D = (int)D; a.M = (int)M; a.scale = scale;
  return a;
}

}  // namespace affb

using namespace affb;

static int nbhd_fwd_impl(const void* q, const void* k, const void* v, const int32_t* member_idx, const void* bias,
                         const uint8_t* mask, int mask_heads, const void* blank_k, const void* blank_v, int dtype,
                         int64_t B, int64_t H, int64_t N, int64_t D, int64_t M, float scale, void* out, float* lse,
                         void* tile_plan, int64_t tile_plan_bytes, void* stream) {
  if (int e = check_na(B, H, N, D, M, mask ? mask_heads : 1, blank_k, blank_v, q, k, v)) return e;
  if (tile_plan) {
    AFFB_REQUIRE(nbhd_tc_supported(dtype, D, M), "nbhd_attn_fwd: a tile plan needs the tensor-core path "
                 "(bf16 / fp16, head_dim 32, at most 64 neighbours)");
    AFFB_REQUIRE(tile_plan_bytes >= nbhd_tile_plan_bytes(B, N, M) && ((uintptr_t)tile_plan & 15) == 0,
                 "nbhd_attn_fwd: tile plan of %lld bytes, %lld needed (16-byte aligned)", (long long)tile_plan_bytes,
                 (long long)nbhd_tile_plan_bytes(B, N, M));
  }
  if (B == 0 || N == 0) return AFFB_OK;
  NbhdArgs a = make_args(q, k, v, member_idx, bias, mask, mask_heads, blank_k, blank_v, B, H, N, D, M, scale);
  a.out = out;
  a.lse = lse;
  a.tile_plan = tile_plan;
  cudaStream_t st = as_stream(stream);
  if (nbhd_tc_supported(dtype, D, M)) {
    if (int e = nbhd_blk_fwd(a, dtype, (int)B, st)) return e;
  } else {
    dim3 grid((unsigned)(((N + NA_WARPS - 1) / NA_WARPS) * B * H));
    AFFB_DISPATCH(dtype, T, dispatch_lpn(D, [&](auto L) {
      nbhd_attn_fwd_kernel<T, decltype(L)::value><<<grid, NA_WARPS * 32, 0, st>>>(a);
    }));
  }
  AFFB_LAUNCH_CHECK("affb_nbhd_attn_fwd");
  return AFFB_OK;
}

extern "C" int affb_nbhd_attn_fwd(const void* q, const void* k, const void* v,
                                  const int32_t* member_idx, const void* bias,
                                  const uint8_t* mask, int mask_heads, const void* blank_k,
                                  const void* blank_v, int dtype, int64_t B, int64_t H,
                                  int64_t N, int64_t D, int64_t M, float scale, void* out,
                                  float* lse, void* stream) {
  return nbhd_fwd_impl(q, k, v, member_idx, bias, mask, mask_heads, blank_k, blank_v, dtype, B, H, N, D, M, scale,
                       out, lse, nullptr, 0, stream);
}

extern "C" int64_t affb_nbhd_tile_plan_bytes(int dtype, int64_t B, int64_t N, int64_t D, int64_t M) {
  if (B < 0 || N < 0 || M < 0) return -1;
  return nbhd_tc_supported(dtype, D, M) ? nbhd_tile_plan_bytes(B, N, M) : 0;
}

extern "C" int affb_nbhd_attn_fwd_plan(const void* q, const void* k, const void* v, const int32_t* member_idx,
                                       const void* bias, const uint8_t* mask, int mask_heads, const void* blank_k,
                                       const void* blank_v, int dtype, int64_t B, int64_t H, int64_t N, int64_t D,
                                       int64_t M, float scale, void* out, float* lse, void* tile_plan,
                                       int64_t tile_plan_bytes, void* stream) {
  return nbhd_fwd_impl(q, k, v, member_idx, bias, mask, mask_heads, blank_k, blank_v, dtype, B, H, N, D, M, scale,
                       out, lse, tile_plan, tile_plan_bytes, stream);
}

// fp32 runs the CUDA-core kernels straight into dk / dv; everything else
// needs fp32 sums (and the tensor-core path its inverse lists).
static NbhdBwdLayout bwd_layout(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, int64_t M,
                                unsigned char* base) {
  const bool tc = nbhd_tc_supported(dtype, D, M);
  return nbhd_bwd_layout(tc, tc || dtype != AFFB_F32, B, H, N, D, M, base);
}

extern "C" int64_t affb_nbhd_attn_bwd_workspace_bytes(int dtype, int64_t B, int64_t H, int64_t N,
                                                       int64_t D, int64_t M) {
  if (B < 0 || H < 0 || N < 0 || D < 0 || M < 0) return -1;
  return (int64_t)bwd_layout(dtype, B, H, N, D, M, nullptr).total;
}

static int nbhd_bwd_impl(const void* q, const void* k, const void* v, const void* o, const void* dout,
                         const float* lse, const int32_t* member_idx, const void* bias, const uint8_t* mask,
                         int mask_heads, const void* blank_k, const void* blank_v, int dtype, int64_t B, int64_t H,
                         int64_t N, int64_t D, int64_t M, float scale, void* dq, void* dk, void* dv, void* dbias,
                         float* dbk_acc, float* dbv_acc, const void* tile_plan, int64_t tile_plan_bytes,
                         void* workspace, int64_t workspace_bytes, void* stream) {
  if (int e = check_na(B, H, N, D, M, mask ? mask_heads : 1, blank_k, blank_v, q, k, v)) return e;
  AFFB_REQUIRE(!blank_k || (dbk_acc && dbv_acc), "nbhd_attn_bwd: blank gradients need dbk/dbv buffers");
  AFFB_REQUIRE(!bias || dbias, "nbhd_attn_bwd: bias given without a dbias buffer");
  AFFB_REQUIRE(((uintptr_t)dk | (uintptr_t)dv | (uintptr_t)o | (uintptr_t)dout | (uintptr_t)dq |
                (uintptr_t)member_idx) % 16 == 0,
               "nbhd_attn_bwd: o/dout/dq/dk/dv/member_idx buffers must be 16-byte aligned");
  AFFB_REQUIRE((uintptr_t)workspace % 256 == 0, "nbhd_attn_bwd: workspace must be 256-byte aligned");
  const NbhdBwdLayout ly = bwd_layout(dtype, B, H, N, D, M, (unsigned char*)workspace);
  AFFB_REQUIRE(workspace_bytes >= (int64_t)ly.total,
               "nbhd_attn_bwd: workspace of %lld bytes, %lld needed (affb_nbhd_attn_bwd_workspace_bytes)",
               (long long)workspace_bytes, (long long)ly.total);
  AFFB_REQUIRE(ly.total == 0 || workspace, "nbhd_attn_bwd: workspace is NULL");
  if (tile_plan)
    AFFB_REQUIRE(nbhd_tc_supported(dtype, D, M) && tile_plan_bytes >= nbhd_tile_plan_bytes(B, N, M) &&
                     ((uintptr_t)tile_plan & 15) == 0,
                 "nbhd_attn_bwd: the tile plan must come from the tensor-core forward of the same sizes");
  if (B == 0 || N == 0) return AFFB_OK;
  AFFB_REQUIRE(B * N * (M / 8) < (1ll << 31), "nbhd_attn_bwd: too many list entries");
  NbhdArgs a = make_args(q, k, v, member_idx, bias, mask, mask_heads, blank_k, blank_v, B, H, N, D, M, scale);
  a.o = o; a.dout = dout; a.lse = const_cast<float*>(lse);
  a.dq = dq; a.dbias = bias ? dbias : nullptr;
  a.dbk = dbk_acc; a.dbv = dbv_acc;
  cudaStream_t st = as_stream(stream);
  const int64_t nel = B * H * N * D;
  if (nbhd_tc_supported(dtype, D, M)) {
    // list count + prologue (D, blank terms) -> scan -> fill -> [query side,
    // only for lists that are not all cluster runs] -> key side (dK, dV, dS)
    // -> dQ from dS
    AFFB_REQUIRE(N * M < (1ll << 31), "nbhd_attn_bwd: N * M must be below 2^31 on the tensor-core path");
    a.dk = ly.acc_k; a.dv = ly.acc_v;
    a.general = ly.flag;
    KvArgs kv{};
    kv.flag = ly.flag; kv.counts = ly.counts; kv.offs = ly.offs; kv.entries = ly.entries;
    kv.di = ly.di; kv.dsb = ly.dsb; kv.ds = bias ? dbias : ly.ds;
    kv.acc_k = ly.acc_k; kv.acc_v = ly.acc_v;
    kv.dk = dk; kv.dv = dv;
    kv.Cc = (int)((N + 7) / 8);
    a.ds = kv.ds; a.dsb = ly.dsb;
    if (int e = nbhd_bwd_prepare(a, kv, ly, dtype, (int)B, st)) return e;
    NbhdArgs ag = a;  // the query-side kernel leaves the blank gradients to the prologue
    ag.dbk = nullptr;
    ag.dbv = nullptr;
    if (int e = nbhd_blk_bwd(ag, dtype, (int)B, st)) return e;
    if (int e = nbhd_kv_bwd(a, kv, dtype, (int)B, st)) return e;
    NbhdArgs aq = a;
    aq.tile_plan = const_cast<void*>(tile_plan);
    if (int e = nbhd_blk_dq(aq, dtype, (int)B, st)) return e;
  } else {
    float* sk = dtype == AFFB_F32 ? (float*)dk : ly.acc_k;
    float* sv = dtype == AFFB_F32 ? (float*)dv : ly.acc_v;
    if (cudaMemsetAsync(sk, 0, nel * sizeof(float), st) != cudaSuccess ||
        cudaMemsetAsync(sv, 0, nel * sizeof(float), st) != cudaSuccess) {
      set_error("nbhd_attn_bwd: cudaMemsetAsync failed");
      return AFFB_ERR_CUDA;
    }
    a.dk = sk; a.dv = sv;
    dim3 grid((unsigned)(((N + NA_WARPS - 1) / NA_WARPS) * B * H));
    AFFB_DISPATCH(dtype, T, dispatch_lpn(D, [&](auto L) {
      nbhd_attn_bwd_kernel<T, decltype(L)::value><<<grid, NA_WARPS * 32, 0, st>>>(a);
    }));
    if (dtype != AFFB_F32) {
      if (int e = affb_cast_f32(sk, dk, dtype, nel, stream)) return e;
      if (int e = affb_cast_f32(sv, dv, dtype, nel, stream)) return e;
    }
  }
  AFFB_LAUNCH_CHECK("affb_nbhd_attn_bwd");
  return AFFB_OK;
}

extern "C" int affb_nbhd_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                                  const void* dout, const float* lse,
                                  const int32_t* member_idx, const void* bias,
                                  const uint8_t* mask, int mask_heads, const void* blank_k,
                                  const void* blank_v, int dtype, int64_t B, int64_t H,
                                  int64_t N, int64_t D, int64_t M, float scale, void* dq,
                                  void* dk, void* dv, void* dbias, float* dbk_acc,
                                  float* dbv_acc, void* workspace, int64_t workspace_bytes,
                                  void* stream) {
  return nbhd_bwd_impl(q, k, v, o, dout, lse, member_idx, bias, mask, mask_heads, blank_k, blank_v, dtype, B, H, N,
                       D, M, scale, dq, dk, dv, dbias, dbk_acc, dbv_acc, nullptr, 0, workspace, workspace_bytes,
                       stream);
}

extern "C" int affb_nbhd_attn_bwd_plan(const void* q, const void* k, const void* v, const void* o,
                                       const void* dout, const float* lse, const int32_t* member_idx,
                                       const void* bias, const uint8_t* mask, int mask_heads, const void* blank_k,
                                       const void* blank_v, int dtype, int64_t B, int64_t H, int64_t N, int64_t D,
                                       int64_t M, float scale, void* dq, void* dk, void* dv, void* dbias,
                                       float* dbk_acc, float* dbv_acc, const void* tile_plan,
                                       int64_t tile_plan_bytes, void* workspace, int64_t workspace_bytes,
                                       void* stream) {
  AFFB_REQUIRE(tile_plan != nullptr, "nbhd_attn_bwd_plan: tile plan is NULL (use affb_nbhd_attn_bwd)");
  return nbhd_bwd_impl(q, k, v, o, dout, lse, member_idx, bias, mask, mask_heads, blank_k, blank_v, dtype, B, H, N,
                       D, M, scale, dq, dk, dv, dbias, dbk_acc, dbv_acc, tile_plan, tile_plan_bytes, workspace,
                       workspace_bytes, stream);
}
