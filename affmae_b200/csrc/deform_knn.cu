// Fused KNN + Shepard-weighted deformable attention (2-D, 4 points per head,
// 4 nearest neighbours per point), forward and backward.
//
// Forward semantics (src/layers/kernels/fused_deform_attn.py:1342-1509, the
// cross-attention kernel that saves its KNN; self-attention :1018-1181 is the
// same with kv_pos = pos):
//   s      = query_pos[n] + offsets[n,h,p]                    (fp32)
//   {j}    = 4 nearest kv positions of s, (d2, index) order
//   dist_j = sqrt(d2_j) + 1e-6 ;  P = max(power, 1e-6)
//   w_j    = exp(-P dist_j - max) / (sum + 1e-8)
//   out[n,h,:] = sum_p attn_w[n,h,p] * (w0 v_j0 + w1 v_j1 + w2 v_j2 + w3 v_j3)
// Backward (cross :1982-2381, self :1520-1975):
//   d_attn_w = dout . sum_j w_j v_j
//   dp_j     = v_j . (attn_w dout);  ds_j = w_j (dp_j - sum_k w_k dp_k)
//   d_power += sum_j ds_j * (-dist_j)
//   d_d2_j   = (-P ds_j) / (2 dist_j)          (dist_j includes the 1e-6)
//   d_off    = d_qpos contribution = 2 sum_j (s - kv_j) d_d2_j
//   d_kvpos[j] += -2 (s - kv_j) d_d2_j ;  d_values[j,h] += attn_w w_j dout
//
// Layout: one warp per query.  Lane l owns sample l (= h*4 + p) for the
// neighbour search and all per-sample scalar math; for the value gather and
// scatter the lanes are re-assigned to 8-channel chunks of the query's
// H*C output row, and per-sample scalars travel through shared memory.
// The neighbour search uses the grid index of deform_grid.cuh, built into a
// caller-provided workspace by four small kernels (bbox, count, scan, scatter).
#include "deform_grid.cuh"

#include <mutex>

namespace affb {

constexpr int DK_WARPS = 8;
// Block shapes: warps per block and the minimum resident blocks asked of the
// register allocator.  The forward's grid search is latency bound (waits on
// cell ranges and points in L1/L2), so residency is what hides it: at 5 blocks
// of 8 warps (48 registers, a few bytes spilled) config 4's forward + backward
// take 2.21 ms against 2.36 at 64 registers (4 blocks) and 3.57 at 100 (2).
#ifndef AFFB_DKF_WARPS
#define AFFB_DKF_WARPS 8
#endif
#ifndef AFFB_DKF_MINB
#define AFFB_DKF_MINB 5
#endif
#ifndef AFFB_DKB_MINB
#define AFFB_DKB_MINB 4
#endif
constexpr int DKF_WARPS = AFFB_DKF_WARPS;
constexpr int DK_SMAX = 64;
// backward shared memory per warp, in ints per sample slot: s_idx, s_first,
// s_w, s_cf, s_dot, s_ulist (4 each), s_aw (1), s_ucnt (1, a quarter used)
constexpr int DKB_SMEM_INTS = 26;  // samples per query (H * 4) handled per warp
constexpr int DK_FWD_SLOTS = 128;  // forward: samples of the queries a warp handles together

// Queries per warp in the forward: with H * 4 samples per query not a
// multiple of 32 (6 heads: 24) one query leaves lanes idle in both the search
// (one sample per lane) and the gather (one 8-channel chunk per lane), so a
// warp takes several consecutive queries and deals their samples and chunks
// out over its lanes (6 heads: 4 queries, 96 samples and 192 chunks, every
// lane busy).
static int deform_fwd_queries_per_warp(int S) {
  int q = 1;
  while (q < 4 && (q * S) % 32 != 0 && 2 * q * S <= DK_FWD_SLOTS) q *= 2;
  return q;
}

// ---------------------------------------------------------------- grid build
__global__ void grid_bbox_kernel(const float* __restrict__ pos, int64_t nkv, int G,
                                 float* __restrict__ params) {
  const int64_t b = blockIdx.x;
  const float* p = pos + b * nkv * 2;
  float mnx = 3.4e38f, mny = 3.4e38f, mxx = -3.4e38f, mxy = -3.4e38f;
  for (int64_t i = threadIdx.x; i < nkv; i += blockDim.x) {
    const float x = p[2 * i], y = p[2 * i + 1];
    if (x == x) { mnx = fminf(mnx, x); mxx = fmaxf(mxx, x); }
    if (y == y) { mny = fminf(mny, y); mxy = fmaxf(mxy, y); }
  }
  __shared__ float red[4][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mnx = fminf(mnx, __shfl_xor_sync(0xffffffffu, mnx, o));
    mny = fminf(mny, __shfl_xor_sync(0xffffffffu, mny, o));
    mxx = fmaxf(mxx, __shfl_xor_sync(0xffffffffu, mxx, o));
    mxy = fmaxf(mxy, __shfl_xor_sync(0xffffffffu, mxy, o));
  }
  if (lane == 0) { red[0][w] = mnx; red[1][w] = mny; red[2][w] = mxx; red[3][w] = mxy; }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nw = blockDim.x / 32;
    for (int i = 1; i < nw; ++i) {
      mnx = fminf(mnx, red[0][i]); mny = fminf(mny, red[1][i]);
      mxx = fmaxf(mxx, red[2][i]); mxy = fmaxf(mxy, red[3][i]);
    }
    if (!(mnx <= mxx)) { mnx = 0.f; mxx = 1.f; }
    if (!(mny <= mxy)) { mny = 0.f; mxy = 1.f; }
    float cw = (mxx - mnx) / G, ch = (mxy - mny) / G;
    if (!(cw > 0.f)) cw = 1.f;
    if (!(ch > 0.f)) ch = 1.f;
    float* P = params + b * 8;
    P[0] = mnx; P[1] = mny; P[2] = cw; P[3] = ch; P[4] = 1.f / cw; P[5] = 1.f / ch;
    P[6] = 0.f; P[7] = 0.f;
  }
}

__device__ __forceinline__ int cell_of(const float* P, int G, float x, float y) {
  int cx = cell_coord((x - P[0]) * P[4], G);
  int cy = cell_coord((y - P[1]) * P[5], G);
  if (!(x == x) || !(y == y)) { cx = 0; cy = 0; }
  return cy * G + cx;
}

__global__ void grid_count_kernel(const float* __restrict__ pos, int64_t B, int64_t nkv, int G,
                                  const float* __restrict__ params, int32_t* __restrict__ cnt) {
  const int64_t ncell = (int64_t)G * G;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < B * nkv;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / nkv;
    const int c = cell_of(params + b * 8, G, pos[2 * t], pos[2 * t + 1]);
    atomicAdd(cnt + b * ncell + c, 1);
  }
}

// Exclusive scan of the per-cell counts of one batch element (one block of
// 1024 threads).  Writes start[] and turns the counts into scatter cursors.
__global__ void grid_scan_kernel(int G, int32_t* __restrict__ cnt_cursor, int32_t* __restrict__ start) {
  const int64_t b = blockIdx.x;
  const int64_t ncell = (int64_t)G * G;
  int32_t* c = cnt_cursor + b * ncell;
  int32_t* s = start + b * (ncell + 1);
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int64_t base = 0; base < ncell; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const int32_t v = i < ncell ? c[i] : 0;
    int32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[w] = x;
    __syncthreads();
    if (w == 0) {
      int32_t t = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      if (lane < nw) warp_tot[lane] = t;
    }
    __syncthreads();
    const int32_t excl = carry + (w > 0 ? warp_tot[w - 1] : 0) + x - v;
    if (i < ncell) { s[i] = excl; c[i] = excl; }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) s[ncell] = carry;
}

__global__ void grid_scatter_kernel(const float* __restrict__ pos, int64_t B, int64_t nkv, int G,
                                    const float* __restrict__ params, int32_t* __restrict__ cursor,
                                    float4* __restrict__ pts) {
  const int64_t ncell = (int64_t)G * G;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < B * nkv;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / nkv;
    const float x = pos[2 * t], y = pos[2 * t + 1];
    const int c = cell_of(params + b * 8, G, x, y);
    const int slot = atomicAdd(cursor + b * ncell + c, 1);
    pts[b * nkv + slot] = make_float4(x, y, __int_as_float((int)(t - b * nkv)), 0.f);
  }
}

int build_grid(const float* kv_pos, int64_t B, int64_t nkv, void* ws, GridView& gv, cudaStream_t st) {
  const GridLayout L = grid_layout(B, nkv);
  char* base = (char*)ws;
  float* params = (float*)(base + L.off_params);
  int32_t* start = (int32_t*)(base + L.off_start);
  int32_t* cursor = (int32_t*)(base + L.off_cursor);
  float4* pts = (float4*)(base + L.off_pts);
  const int64_t ncell = (int64_t)L.G * L.G;
  if (cudaMemsetAsync(cursor, 0, B * ncell * 4, st) != cudaSuccess) {
    set_error("deform grid: memset failed");
    return AFFB_ERR_CUDA;
  }
  grid_bbox_kernel<<<(unsigned)B, 512, 0, st>>>(kv_pos, nkv, L.G, params);
  const int64_t tot = B * nkv;
  unsigned nb = (unsigned)imin64((tot + 255) / 256, (int64_t)sm_count() * 16);
  if (nb == 0) nb = 1;
  grid_count_kernel<<<nb, 256, 0, st>>>(kv_pos, B, nkv, L.G, params, cursor);
  grid_scan_kernel<<<(unsigned)B, 1024, 0, st>>>(L.G, cursor, start);
  grid_scatter_kernel<<<nb, 256, 0, st>>>(kv_pos, B, nkv, L.G, params, cursor, pts);
  gv.params = params;
  gv.start = start;
  gv.pts = pts;
  gv.G = L.G;
  gv.Nkv = nkv;
  return AFFB_OK;
}

// ------------------------------------------------------------ attention
__device__ __forceinline__ void shepard4(const float* d2, float P, float* w, float* dist) {
#pragma unroll
  for (int j = 0; j < 4; ++j) dist[j] = sqrtf(d2[j]) + 1e-6f;
  float lg[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) lg[j] = -P * dist[j];
  const float mx = fmaxf(fmaxf(lg[0], lg[1]), fmaxf(lg[2], lg[3]));
  float e[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) e[j] = expf(lg[j] - mx);
  const float sum = e[0] + e[1] + e[2] + e[3] + 1e-8f;
#pragma unroll
  for (int j = 0; j < 4; ++j) w[j] = e[j] / sum;
}

template <typename T>
__global__ void __launch_bounds__(DKF_WARPS * 32, AFFB_DKF_MINB)
deform_knn_fwd_kernel(const float* __restrict__ qpos, const float* __restrict__ offsets,
                      const float* __restrict__ attn_w, const T* __restrict__ values,
                      const float* __restrict__ power, int64_t B, int64_t Nq, int64_t Nkv, int H,
                      int C, int qpw, GridView gv, T* __restrict__ out, int32_t* __restrict__ knn_idx,
                      float* __restrict__ knn_d2) {
  // per warp: slots = qpw * H * 4 samples of (4 indices, 4 weights, 1 attention weight);
  // sized to the launch so the rest of the SM's shared/L1 storage caches the grid
  extern __shared__ int dk_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slots = qpw * H * 4;
  int* s_idx = dk_smem + warp * slots * 9;
  float* s_w = reinterpret_cast<float*>(s_idx + slots * 4);
  float* s_aw = s_w + slots * 4;
  const int64_t gq0 = ((int64_t)blockIdx.x * DKF_WARPS + warp) * qpw;   // first query of this warp
  if (gq0 >= B * Nq) return;
  const int nq = (int)(B * Nq - gq0 < qpw ? B * Nq - gq0 : qpw);
  const float P = fmaxf(power[0], 1e-6f);
  const int S = H * 4;
  // search: lane t takes sample t % S of query t / S
  for (int t = lane; t < nq * S; t += 32) {
    const int qi = t / S;
    const int64_t gq = gq0 + qi;
    const int64_t b = gq / Nq;
    const int64_t gs = gq0 * S + t;
    const float sx = __fadd_rn(qpos[2 * gq], offsets[2 * gs]);
    const float sy = __fadd_rn(qpos[2 * gq + 1], offsets[2 * gs + 1]);
    Top4 top;
    grid_knn4(gv, b, sx, sy, top);
    reinterpret_cast<int4*>(knn_idx)[gs] = make_int4(top.i[0], top.i[1], top.i[2], top.i[3]);
    if (knn_d2) reinterpret_cast<float4*>(knn_d2)[gs] = make_float4(top.d[0], top.d[1], top.d[2], top.d[3]);
    float w[4], dist[4];
    shepard4(top.d, P, w, dist);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s_idx[t * 4 + j] = top.i[j];
      s_w[t * 4 + j] = w[j];
    }
    s_aw[t] = attn_w[gs];
  }
  __syncwarp();
  // gather: lane t takes 8-channel chunk t % (H*C/8) of query t / (H*C/8)
  const int row = H * C;
  const int nc8 = row / 8;
  for (int t = lane; t < nq * nc8; t += 32) {
    const int qi = t / nc8, c8 = t - qi * nc8;
    const int64_t gq = gq0 + qi;
    const T* vb = values + (gq / Nq) * Nkv * row;
    const int h = (c8 * 8) / C;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int si = qi * S + h * 4 + p;
      float wv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) wv[e] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int id = s_idx[si * 4 + j];
        const float w = s_w[si * 4 + j];
        float v[8];
        ld8(vb + (int64_t)id * row + c8 * 8, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) wv[e] = fmaf(w, v[e], wv[e]);
      }
      const float aw = s_aw[si];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(aw, wv[e], acc[e]);
    }
    st8(out + gq * row + c8 * 8, acc);
  }
}

// Squared distances of sample gs to its 4 neighbours: the saved ones, or
// (knn_d2 == NULL) recomputed from the positions with the forward's rounding
// (sample = q + offset, then sqdist2), which reproduces them bit for bit.
__device__ __forceinline__ void load_d2(const float* __restrict__ knn_d2, int64_t gs, int4 ii,
                                        const float* __restrict__ kvb, float qx, float qy,
                                        const float* __restrict__ offsets, float* d2) {
  if (knn_d2) {
    const float4 dd = reinterpret_cast<const float4*>(knn_d2)[gs];
    d2[0] = dd.x; d2[1] = dd.y; d2[2] = dd.z; d2[3] = dd.w;
    return;
  }
  const float sx = __fadd_rn(qx, offsets[2 * gs]);
  const float sy = __fadd_rn(qy, offsets[2 * gs + 1]);
  const int id[4] = {ii.x, ii.y, ii.z, ii.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    d2[j] = sqdist2(sx, sy, kvb[2 * (int64_t)id[j]], kvb[2 * (int64_t)id[j] + 1]);
  }
}

// Backward, qpw consecutive queries per warp (several when one query's
// 8-channel chunks, H * C / 8, do not fill whole passes of 32 lanes: 6 heads
// of 64 channels give 48 chunks, so 2 queries give 3 full passes instead of
// 2 passes at 75 %).  Per head the 4 points x 4 neighbours give 16
// (kv row, coefficient aw * w) entries; entries naming the same kv row are
// merged first (neighbouring sampling points share neighbours), so each
// distinct row is gathered once for the dot products and receives one
// scatter-add of d_values.  The per-entry dot products v[row] . dout[head]
// are reduced over the head's lanes with shuffles when a head's 8-channel
// chunks form an aligned lane group (C/8 divides 32), else with shared-memory
// atomics.
template <typename T, int QPW>
__global__ void __launch_bounds__(DK_WARPS * 32, AFFB_DKB_MINB)
deform_knn_bwd_kernel(const float* __restrict__ qpos, const float* __restrict__ kvpos,
                      const float* __restrict__ offsets, const float* __restrict__ attn_w,
                      const T* __restrict__ values, const float* __restrict__ power,
                      const int32_t* __restrict__ knn_idx, const float* __restrict__ knn_d2,
                      const T* __restrict__ dout, int64_t B, int64_t Nq, int64_t Nkv, int H, int C,
                      float* __restrict__ d_off, float* __restrict__ d_aw,
                      float* __restrict__ d_qpos, float* __restrict__ d_kvpos,
                      float* __restrict__ d_val, float* __restrict__ d_power) {
  // per warp, for the slots = qpw * H * 4 samples of its queries (sized to the
  // launch so the rest of the SM's shared/L1 storage caches values and
  // positions): s_idx, s_first (first entry of the head with the same kv row),
  // s_w, s_cf (merged aw * w of a first entry), s_dot (v[row] . dout[head] of
  // a first entry), s_ulist (the first entries of each head, compacted):
  // slots * 4 each; s_aw: slots; s_ucnt (first entries per head): slots / 4
  __shared__ float s_pow[DK_WARPS];
  extern __shared__ int dkb_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float P = fmaxf(power[0], 1e-6f);
  const int S = H * 4;
  constexpr int qpw = QPW;
  const int slots = qpw * S;
  int* s_idx = dkb_smem + warp * slots * DKB_SMEM_INTS;
  int* s_first = s_idx + slots * 4;
  float* s_w = reinterpret_cast<float*>(s_first + slots * 4);
  float* s_cf = s_w + slots * 4;
  float* s_dot = s_cf + slots * 4;
  float* s_aw = s_dot + slots * 4;
  int* s_ulist = reinterpret_cast<int*>(s_aw + slots);
  int* s_ucnt = s_ulist + slots * 4;
  const int row = H * C;
  const int nc8 = row / 8;
  const int G = C / 8;  // lanes (8-channel chunks) per head
  const bool shfl = G <= 32 && (32 % G) == 0;
  float dpow = 0.f;
  const int64_t nqtot = B * Nq;
  for (int64_t gq0 = ((int64_t)blockIdx.x * DK_WARPS + warp) * qpw; gq0 < nqtot;
       gq0 += (int64_t)gridDim.x * DK_WARPS * qpw) {
    const int nq = (int)(nqtot - gq0 < qpw ? nqtot - gq0 : qpw);
    // sample slot t = qi * S + h * 4 + p of query gq0 + qi
    for (int t = lane; t < nq * S; t += 32) {
      const int64_t gq = gq0 + (QPW == 1 ? 0 : t / S);
      const float* kvb = kvpos + (gq / Nq) * Nkv * 2;
      const int64_t gs = gq0 * S + t;
      const int4 ii = reinterpret_cast<const int4*>(knn_idx)[gs];
      float d2[4];
      load_d2(knn_d2, gs, ii, kvb, qpos[2 * gq], qpos[2 * gq + 1], offsets, d2);
      float w[4], dist[4];
      shepard4(d2, P, w, dist);
      s_idx[t * 4 + 0] = ii.x; s_idx[t * 4 + 1] = ii.y;
      s_idx[t * 4 + 2] = ii.z; s_idx[t * 4 + 3] = ii.w;
#pragma unroll
      for (int j = 0; j < 4; ++j) { s_w[t * 4 + j] = w[j]; s_cf[t * 4 + j] = 0.f; s_dot[t * 4 + j] = 0.f; }
      s_aw[t] = attn_w[gs];
    }
    __syncwarp();
    // merge entries of a head that name the same kv row (entry e = slot * 4 + j;
    // the 16 entries of one head of one query are e >> 4)
    // The first entries of each head are also listed compactly (s_ulist, count
    // in s_ucnt): 32 lanes cover two heads' 16 entries.
    for (int t0 = 0; t0 < nq * S * 4; t0 += 32) {
      const int t = t0 + lane;
      const bool in = t < nq * S * 4;
      int f = t;
      if (in) {
        const int h0 = (t >> 4) << 4, id = s_idx[t];
        for (int u = h0; u < t; ++u)
          if (s_idx[u] == id) { f = u; break; }
        s_first[t] = f;
        atomicAdd(&s_cf[f], s_aw[t >> 2] * s_w[t]);
      }
      const unsigned firsts = __ballot_sync(0xffffffffu, in && f == t);
      const unsigned half = (firsts >> (lane & 16)) & 0xffffu;
      if (in && f == t) s_ulist[t & ~15 | __popc(half & ((1u << (lane & 15)) - 1u))] = t;
      if (in && (lane & 15) == 0) s_ucnt[t >> 4] = __popc(half);
    }
    __syncwarp();
    // chunk u = qi * nc8 + c8; a head's G chunks stay in one aligned lane group
    for (int base = 0; base < nq * nc8; base += 32) {
      const int u = base + lane;
      const bool act = u < nq * nc8;
      const int qi = (QPW == 1 || !act) ? 0 : u / nc8;
      const int c8 = act ? u - qi * nc8 : 0;
      const int h = (c8 * 8) / C;
      const int64_t gq = gq0 + qi;
      const int64_t b = gq / Nq;
      const T* vb = values + b * Nkv * row;
      float* dvb = d_val + b * Nkv * row;
      float g[8];
      if (act) ld8(dout + gq * row + c8 * 8, g);
      else {
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = 0.f;
      }
      // the head's distinct rows only, two per step: the two dot products are
      // reduced over the head's G lanes together (the first exchange swaps
      // halves, so one shuffle serves both)
      const int hs = (qi * H + h) * 16;
      const int cnt = act ? s_ucnt[hs >> 4] : 0;
      const int kmax = __reduce_max_sync(0xffffffffu, cnt);
      for (int k = 0; k < kmax; k += 2) {
        float dd[2];
        int tt[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const bool on = k + j < cnt;
          tt[j] = on ? s_ulist[hs + k + j] : -1;
          dd[j] = 0.f;
          if (on) {
            const int id = s_idx[tt[j]];
            float v[8];
            ld8(vb + (int64_t)id * row + c8 * 8, v);
#pragma unroll
            for (int e = 0; e < 8; ++e) dd[j] = fmaf(v[e], g[e], dd[j]);
            const float cf = s_cf[tt[j]];
            float* dst = dvb + (int64_t)id * row + c8 * 8;
            red_add_v4(dst, cf * g[0], cf * g[1], cf * g[2], cf * g[3]);
            red_add_v4(dst + 4, cf * g[4], cf * g[5], cf * g[6], cf * g[7]);
          }
        }
        if (shfl && G >= 2) {
          const int o = G >> 1;
          const bool hi = (lane & o) != 0;
          float mine = hi ? dd[1] : dd[0];
          mine += __shfl_xor_sync(0xffffffffu, hi ? dd[0] : dd[1], o);
          for (int oo = o >> 1; oo > 0; oo >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, oo);
          const int r = lane & (G - 1);
          if (r == 0 && tt[0] >= 0) s_dot[tt[0]] = mine;
          if (r == o && tt[1] >= 0) s_dot[tt[1]] = mine;
        } else if (shfl) {  // G == 1: a lane holds the whole row of the head
          if (tt[0] >= 0) s_dot[tt[0]] = dd[0];
          if (tt[1] >= 0) s_dot[tt[1]] = dd[1];
        } else {
          if (tt[0] >= 0) atomicAdd(&s_dot[tt[0]], dd[0]);
          if (tt[1] >= 0) atomicAdd(&s_dot[tt[1]], dd[1]);
        }
      }
    }
    __syncwarp();
    // d_kv_pos is summed per distinct kv row of a head in shared memory (in
    // s_ulist / s_cf, no longer read) and scattered once per row below; s_w
    // still holds the Shepard weights of the first pass
    float* s_gx = reinterpret_cast<float*>(s_ulist);
    for (int t = lane; t < nq * S * 4; t += 32) { s_gx[t] = 0.f; s_cf[t] = 0.f; }
    __syncwarp();
    float gqx[QPW], gqy[QPW];   // this lane's share of d_query_pos per query
#pragma unroll
    for (int i = 0; i < QPW; ++i) { gqx[i] = 0.f; gqy[i] = 0.f; }
    for (int t = lane; t < nq * S; t += 32) {
      const int qi = QPW == 1 ? 0 : t / S;
      const int64_t gq = gq0 + qi;
      const float* kvb = kvpos + (gq / Nq) * Nkv * 2;
      const float qx = qpos[2 * gq], qy = qpos[2 * gq + 1];
      const int64_t gs = gq0 * S + t;
      const float sx = __fadd_rn(qx, offsets[2 * gs]);
      const float sy = __fadd_rn(qy, offsets[2 * gs + 1]);
      // sample-to-neighbour vectors; the squared distances from them carry
      // the forward's rounding (sqdist2), unless the saved ones are given
      float exv[4], eyv[4], d2[4], w[4], dist[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int id = s_idx[t * 4 + j];
        const float px = kvb[2 * id], py = kvb[2 * id + 1];
        exv[j] = sx - px;
        eyv[j] = sy - py;
        d2[j] = sqdist2(sx, sy, px, py);
        w[j] = s_w[t * 4 + j];
      }
      if (knn_d2) {
        const float4 dd = reinterpret_cast<const float4*>(knn_d2)[gs];
        d2[0] = dd.x; d2[1] = dd.y; d2[2] = dd.z; d2[3] = dd.w;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) dist[j] = sqrtf(d2[j]) + 1e-6f;  // as in shepard4
      const float aw = s_aw[t];
      float dot[4], datt = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dot[j] = s_dot[s_first[t * 4 + j]];
        datt = fmaf(w[j], dot[j], datt);
      }
      d_aw[gs] = datt;
      float dp[4], wdp = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) { dp[j] = aw * dot[j]; wdp = fmaf(w[j], dp[j], wdp); }
      float dsx = 0.f, dsy = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float ds = w[j] * (dp[j] - wdp);
        dpow += ds * (-dist[j]);
        const float dd2 = (ds * (-P)) / (2.f * dist[j]);
        const float ex = exv[j], ey = eyv[j];
        dsx = fmaf(ex, dd2, dsx);
        dsy = fmaf(ey, dd2, dsy);
        const int f = s_first[t * 4 + j];
        atomicAdd(&s_gx[f], -2.f * ex * dd2);
        atomicAdd(&s_cf[f], -2.f * ey * dd2);
      }
      dsx *= 2.f;
      dsy *= 2.f;
      d_off[2 * gs] = dsx;
      d_off[2 * gs + 1] = dsy;
#pragma unroll
      for (int i = 0; i < QPW; ++i)
        if (i == qi) { gqx[i] += dsx; gqy[i] += dsy; }
    }
    __syncwarp();
    for (int t = lane; t < nq * S * 4; t += 32) {
      if (s_first[t] != t) continue;
      const int id = s_idx[t];
      float* dkvb = d_kvpos + ((gq0 + (QPW == 1 ? 0 : t / (S * 4))) / Nq) * Nkv * 2;
      red_add(dkvb + 2 * id, s_gx[t]);
      red_add(dkvb + 2 * id + 1, s_cf[t]);
    }
#pragma unroll
    for (int i = 0; i < QPW; ++i) {
      const float sx = warp_sum(gqx[i]), sy = warp_sum(gqy[i]);
      if (lane == 0 && i < nq) {
        red_add(d_qpos + 2 * (gq0 + i), sx);
        red_add(d_qpos + 2 * (gq0 + i) + 1, sy);
      }
    }
    __syncwarp();
  }
  dpow = warp_sum(dpow);
  if (lane == 0) s_pow[warp] = dpow;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < DK_WARPS; ++i) t += s_pow[i];
    atomicAdd(d_power, t);
  }
}

// Queries per warp in the backward: enough for whole passes of 32 chunks
// when the shared-memory slots allow (6 heads of 64 channels: 2).
static int deform_bwd_queries_per_warp(int S, int nc8) {
  int q = 1;
  while (q < 4 && (q * nc8) % 32 != 0 && 2 * q * S <= DK_SMAX) q *= 2;
  return q;
}

static int check_deform(int64_t B, int64_t Nq, int64_t Nkv, int64_t H, int64_t C) {
  AFFB_REQUIRE(B >= 0 && Nq >= 0 && Nkv >= 1 && H >= 1 && C >= 1, "deform_knn: invalid sizes");
  AFFB_REQUIRE(H * 4 <= DK_SMAX, "deform_knn: at most %d heads supported (got %lld)", DK_SMAX / 4,
               (long long)H);
  AFFB_REQUIRE(C % 8 == 0, "deform_knn: channels per head must be a multiple of 8 (got %lld)",
               (long long)C);
  AFFB_REQUIRE(Nkv < (1ll << 31) && B < 65536, "deform_knn: size too large");
  return AFFB_OK;
}

}  // namespace affb

using namespace affb;

extern "C" int64_t affb_deform_workspace_bytes(int64_t B, int64_t Nkv) {
  return grid_layout(B, Nkv).total;
}

extern "C" int affb_deform_knn_fwd(const float* query_pos, const float* kv_pos,
                                   const float* offsets, const float* attn_w, const void* values,
                                   const float* power, int dtype, int64_t B, int64_t Nq,
                                   int64_t Nkv, int64_t H, int64_t C, void* out,
                                   int32_t* knn_idx, float* knn_d2, void* workspace,
                                   void* stream) {
  if (int e = check_deform(B, Nq, Nkv, H, C)) return e;
  AFFB_REQUIRE(((uintptr_t)workspace & 255) == 0, "deform_knn: workspace must be 256-byte aligned");
  AFFB_REQUIRE(((uintptr_t)values & 15) == 0 && ((uintptr_t)out & 15) == 0 &&
                   ((uintptr_t)knn_idx & 15) == 0 && ((uintptr_t)knn_d2 & 15) == 0,
               "deform_knn: values/out/knn buffers must be 16-byte aligned");
  if (B == 0 || Nq == 0) return AFFB_OK;
  cudaStream_t st = as_stream(stream);
  GridView gv;
  if (int e = build_grid(kv_pos, B, Nkv, workspace, gv, st)) return e;
  const int qpw = deform_fwd_queries_per_warp((int)H * 4);
  const unsigned nb = (unsigned)((B * Nq + DKF_WARPS * qpw - 1) / (DKF_WARPS * qpw));
  const size_t smem = (size_t)DKF_WARPS * qpw * H * 4 * 9 * sizeof(int);
  AFFB_DISPATCH(dtype, T,
                deform_knn_fwd_kernel<T><<<nb, DKF_WARPS * 32, smem, st>>>(
                    query_pos, offsets, attn_w, (const T*)values, power, B, Nq, Nkv, (int)H,
                    (int)C, qpw, gv, (T*)out, knn_idx, knn_d2));
  AFFB_LAUNCH_CHECK("affb_deform_knn_fwd");
  return AFFB_OK;
}

extern "C" int affb_deform_knn_bwd(const float* query_pos, const float* kv_pos,
                                   const float* offsets, const float* attn_w, const void* values,
                                   const float* power, const int32_t* knn_idx,
                                   const float* knn_d2, const void* dout, int dtype, int64_t B,
                                   int64_t Nq, int64_t Nkv, int64_t H, int64_t C,
                                   float* d_offsets, float* d_attn_w, float* d_qpos,
                                   float* d_kvpos, float* d_values_acc, float* d_power,
                                   void* stream) {
  if (int e = check_deform(B, Nq, Nkv, H, C)) return e;
  AFFB_REQUIRE(((uintptr_t)values & 15) == 0 && ((uintptr_t)dout & 15) == 0 &&
                   ((uintptr_t)d_values_acc & 15) == 0,
               "deform_knn_bwd: values/dout/d_values must be 16-byte aligned");
  if (B == 0 || Nq == 0) return AFFB_OK;
  cudaStream_t st = as_stream(stream);
  const int qpw = deform_bwd_queries_per_warp((int)H * 4, (int)(H * C / 8));
  const int64_t need = (B * Nq + DK_WARPS * qpw - 1) / (DK_WARPS * qpw);
  const unsigned nb = (unsigned)imin64(need, (int64_t)sm_count() * 8);
  const size_t smem = (size_t)DK_WARPS * qpw * H * 4 * DKB_SMEM_INTS * sizeof(int);
#define AFFB_DKB_LAUNCH(Q)                                                                          \
  deform_knn_bwd_kernel<T, Q><<<nb, DK_WARPS * 32, smem, st>>>(                                      \
      query_pos, kv_pos, offsets, attn_w, (const T*)values, power, knn_idx, knn_d2, (const T*)dout, B, \
      Nq, Nkv, (int)H, (int)C, d_offsets, d_attn_w, d_qpos, d_kvpos, d_values_acc, d_power)
  AFFB_DISPATCH(dtype, T, {
    if (qpw == 1) AFFB_DKB_LAUNCH(1);
    else if (qpw == 2) AFFB_DKB_LAUNCH(2);
    else AFFB_DKB_LAUNCH(4);
  });
#undef AFFB_DKB_LAUNCH
  AFFB_LAUNCH_CHECK("affb_deform_knn_bwd");
  return AFFB_OK;
}

// ----------------------------------------------------------------------------
// Allocation-free variant of affb_deform_knn_fwd.
//
// The spatial grid lives in a fixed, file-scope device array instead of a
// caller-provided workspace.  Every GPU that loads this library reserves the
// array (AFFB_NOALLOC_SCRATCH_BYTES) for the life of the process.  Host code
// must not hand the array's name to a kernel: on the host it only stands for
// the symbol, so its device address is fetched once per device with
// cudaGetSymbolAddress (with that device current) and cached.
namespace affb {

static __device__ __align__(256) unsigned char g_noalloc_scratch[AFFB_NOALLOC_SCRATCH_BYTES];

static void* noalloc_scratch_address(int dev, int* err) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  *err = AFFB_OK;
  if (dev < 0 || dev >= 64) { *err = AFFB_ERR_INVALID; return nullptr; }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (rc != cudaSuccess || p == nullptr) {
      set_error("deform_knn_fwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(rc));
      *err = AFFB_ERR_CUDA;
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace affb

extern "C" int64_t affb_deform_noalloc_max_scratch_bytes(void) { return AFFB_NOALLOC_SCRATCH_BYTES; }

extern "C" int affb_deform_knn_fwd_noalloc(const float* query_pos, const float* kv_pos,
                                           const float* offsets, const float* attn_w,
                                           const void* values, const float* power, int dtype,
                                           int64_t B, int64_t Nq, int64_t Nkv, int64_t H, int64_t C,
                                           void* out, int32_t* knn_idx, float* knn_d2,
                                           void* stream) {
  if (int e = check_deform(B, Nq, Nkv, H, C)) return e;
  const int64_t need = grid_layout(B, Nkv).total;
  AFFB_REQUIRE(need <= (int64_t)AFFB_NOALLOC_SCRATCH_BYTES,
               "deform_knn_fwd_noalloc: B=%lld x Nkv=%lld needs %lld bytes of grid scratch; the fixed "
               "scratch holds %lld bytes (use affb_deform_knn_fwd with a workspace instead)",
               (long long)B, (long long)Nkv, (long long)need, (long long)AFFB_NOALLOC_SCRATCH_BYTES);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error("deform_knn_fwd_noalloc: no current CUDA device");
    return AFFB_ERR_CUDA;
  }
  int err = AFFB_OK;
  void* scratch = noalloc_scratch_address(dev, &err);
  if (err != AFFB_OK) return err;
  // The grid build clears its cell counters on every call, so the scratch
  // keeps no state that a later call depends on.
  return affb_deform_knn_fwd(query_pos, kv_pos, offsets, attn_w, values, power, dtype, B, Nq, Nkv, H,
                             C, out, knn_idx, knn_d2, scratch, stream);
}
