// Backward of the cluster-block neighbourhood attention, key side: dK and dV
// computed key-major from inverse neighbour lists, with no atomics and no
// fp32 accumulators.
//
// The reference accumulates dK / dV by atomically adding each query's
// contribution into fp32 buffers (local_attn.py:518-519, tl.atomic_add on
// DK / DV).  Here the lists are inverted once per call instead:
//   inv_count  one thread per query (sharing one launch with the prologue): checks that its list is M/8 runs of 8
//              consecutive keys starting at a multiple of 8 with no cluster
//              listed twice, where a run of the partial last cluster may end
//              in padding slots masked in every mask head (the same test as
//              the query-side tile setup),
//              counts the queries that list each key cluster and remembers
//              the rank of every (query, run) entry;
//   inv_scan   one block per image: exclusive scan of the counts;
//   inv_fill   writes entry q * 8 + j (query q lists the cluster as run j)
//              at its slot of the cluster's list.
// A call whose lists are not all of that form sets a flag instead; the
// query-side kernel then scatter-adds dK / dV into fp32 buffers as before
// (inv_fill zeroes them) and nbhd_kv_kernel converts them to the output type.
//
// nbhd_kv_kernel: one block per key cluster (8 keys), one warp per head.
// The cluster's list is sorted by query in shared memory (so the summation
// order, and the result, is deterministic); the warp walks it in chunks of 16
// queries, gathering their Q / dO rows, lse, D = rowsum(O * dO), bias run and
// mask run with cp.async, and computes on the tensor cores
//   S  = Q_c K^T,  dP = dO_c V^T            (16 queries x 8 keys)
//   P  = exp(S * scale + bias - lse),  dS = P (dP - D)
//   dV^T += dO_c^T P,  dK^T += Q_c^T dS      (32 dims x 8 keys)
// P and dS become the B operands of the last two products with one
// movmatrix.trans per 8x8 block.  Every computed (query, key) pair is a
// listed one, so no work is spent on masked pairs.
#include "nbhd_tc.cuh"
#include "nbhd_mma.cuh"

#include <type_traits>

namespace affb {

constexpr int KV_LCAP = 256;  // list segment held in shared memory; shorter lists are sorted

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0));
}

// ---------------------------------------------------------------- lists --

__device__ __forceinline__ void inv_count_block(const int32_t* __restrict__ midx, const uint8_t* __restrict__ mask,
                                                int mask_heads, int B, int N, int M, int Cc,
                                                int* __restrict__ flag, int* __restrict__ counts,
                                                int* __restrict__ ecl, int* __restrict__ erk, int64_t bid) {
  const int64_t t = bid * blockDim.x + threadIdx.x;
  const bool valid = t < (int64_t)B * N;
  const int b = valid ? (int)(t / N) : 0;
  const int64_t qn = valid ? t - (int64_t)b * N : 0;  // query index within its image
  const int J = M >> 3;
  const int4* row = reinterpret_cast<const int4*>(midx + (valid ? t : 0) * M);
  // one run at a time (two 16-byte loads): the launch shares its register
  // budget with the prologue
  int cs[8];
  bool ok = true;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    cs[j] = 0;
    if (j < J) {
      const int4 x = __ldg(row + 2 * j), y = __ldg(row + 2 * j + 1);
      const int c0 = x.x;
      const int v[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
      ok &= (c0 >= 0) & ((c0 & 7) == 0) & (c0 < N);
#pragma unroll
      for (int r = 1; r < 8; ++r) {
        if (c0 + r < N) {
          ok &= v[r] == c0 + r;
        } else {  // past the last token: must be a padding slot masked in every mask head
          bool masked = mask != nullptr;
          for (int hm = 0; hm < mask_heads && masked; ++hm)
            masked = mask[(((int64_t)b * mask_heads + hm) * N + qn) * M + 8 * j + r] == 0;
          ok &= masked;
        }
      }
      cs[j] = c0 >> 3;
#pragma unroll
      for (int jj = 0; jj < j; ++jj) ok &= cs[jj] != cs[j];
    }
  }
  if (valid && !ok) *reinterpret_cast<volatile int*>(flag) = 1;
  // Queries of one warp are neighbours and list mostly the same clusters: one
  // atomic per distinct cluster and warp, ranks in lane order.
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j < J) {  // J is uniform: every lane takes part in the match
      const bool use = valid && ok;
      const int key = use ? b * Cc + cs[j] : -1 - lane;
      const unsigned peers = __match_any_sync(0xffffffffu, key);
      const int leader = __ffs(peers) - 1;
      int base = 0;
      if (use && lane == leader) base = atomicAdd(counts + key, __popc(peers));
      base = __shfl_sync(0xffffffffu, base, leader);
      if (use) {
        ecl[t * J + j] = cs[j];
        erk[t * J + j] = base + __popc(peers & ((1u << lane) - 1u));
      }
    }
  }
}

// Exclusive scan of one image's cluster counts; slots of image b start at
// b * N * J (every query has exactly J entries).
__global__ void __launch_bounds__(1024) nbhd_inv_scan_kernel(const int* __restrict__ counts, int N, int J,
                                                             int Cc, const int* __restrict__ flag,
                                                             int* __restrict__ offs) {
  __shared__ int wsum[32];
  __shared__ int carry_s;
  dependent_wait();
  if (*flag) return;
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int* cnt = counts + (int64_t)b * Cc;
  int* off = offs + (int64_t)b * Cc;
  if (t == 0) carry_s = 0;
  __syncthreads();
  for (int base = 0; base < Cc; base += 1024) {
    const int v = base + t < Cc ? cnt[base + t] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int s = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      wsum[lane] = s;  // inclusive over warps
    }
    __syncthreads();
    const int carry = carry_s;
    const int excl = carry + (w ? wsum[w - 1] : 0) + x - v;
    if (base + t < Cc) off[base + t] = (int)((int64_t)b * N * J) + excl;
    __syncthreads();
    if (t == 0) carry_s = carry + wsum[31];
    __syncthreads();
  }
}

__global__ void nbhd_inv_fill_kernel(int B, int N, int M, int Cc, int H, const int* __restrict__ flag,
                                     const int* __restrict__ offs, const int* __restrict__ ecl,
                                     const int* __restrict__ erk, int* __restrict__ entries,
                                     float* __restrict__ acc_k, float* __restrict__ acc_v) {
  dependent_wait();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (int64_t)B * N) return;
  const int b = (int)(t / N), q = (int)(t % N);
  if (*flag) {  // general lists: the query side scatter-adds into zeroed fp32 buffers
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int h = 0; h < H; ++h) {
      float4* pk = reinterpret_cast<float4*>(acc_k + (((int64_t)b * H + h) * N + q) * TD);
      float4* pv = reinterpret_cast<float4*>(acc_v + (((int64_t)b * H + h) * N + q) * TD);
#pragma unroll
      for (int i = 0; i < TD / 4; ++i) { pk[i] = z; pv[i] = z; }
    }
    return;
  }
  const int J = M >> 3;
  for (int j = 0; j < J; ++j) {
    const int c = ecl[t * J + j];
    entries[offs[(int64_t)b * Cc + c] + erk[t * J + j]] = q * 8 + j;
  }
}

// Clears n 16-byte words (the list flag and counters of one call).
__global__ void nbhd_zero_kernel(uint4* __restrict__ p, int64_t n) {
  dependent_wait();
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = z;
}

// ------------------------------------------------------ query prologue --

// Per (b, h, n): D = rowsum(O * dO) and, with a blank token, its probability
// pb = exp(q . blank_k * scale - lse), dS_blank = pb (dO . blank_v - D), and
// the blank gradients dblank_k += dS_blank q scale, dblank_v += pb dO
// (reference local_attn.py:526-550).  One block per PRO_ROWS rows of one
// (b, h); four lanes per row, eight dims per lane; every row load of the
// block's four passes is issued before the first is used (the kernel is a
// stream bounded by loads in flight); the blank gradients are summed in
// registers over the block's rows and reduced once.
constexpr int PRO_ROWS = 256;
constexpr int PRO_PASSES = PRO_ROWS / 64;
#ifndef AFFB_PRE_GROUP
#define AFFB_PRE_GROUP 1  // passes whose loads are in flight together
#endif
constexpr int PRO_GROUP = AFFB_PRE_GROUP;

template <typename T>
__device__ __forceinline__ void cvt8(const uint4& u, float* o) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = __uint_as_float(w[i] << 16);
      o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void q_prologue_block(const NbhdArgs& a, const KvArgs& k, int64_t bid) {
  __shared__ float s_dbk[TD], s_dbv[TD];
  __shared__ alignas(16) float s_bk[TD], s_bv[TD];
  const int N = a.N;
  const int nblk = (N + PRO_ROWS - 1) / PRO_ROWS;
  const int64_t bh = bid / nblk;
  const int h = (int)(bh % a.H);
  const int t = threadIdx.x, lane = t & 31, sub = lane & 3;
  const int nbase = (int)(bid % nblk) * PRO_ROWS;
  const bool blank = a.blank_k != nullptr;
  float gk[8], gv[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) { gk[e] = 0.f; gv[e] = 0.f; }
  // the blank token's k / v rows are read from shared memory where they are
  // used, which keeps the register count within four blocks per SM
  if (blank && t < TD) {
    s_bk[t] = ldf((const T*)a.blank_k + (int64_t)h * TD + t);
    s_bv[t] = ldf((const T*)a.blank_v + (int64_t)h * TD + t);
    s_dbk[t] = 0.f;
    s_dbv[t] = 0.f;
  }
  __syncthreads();
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  // rows in groups of PRO_GROUP passes: every load of a group is issued
  // before the first is used
#pragma unroll 1
  for (int g0 = 0; g0 < PRO_PASSES; g0 += PRO_GROUP) {
    uint4 ro[PRO_GROUP], rd[PRO_GROUP], rq[PRO_GROUP];
    float ls[PRO_GROUP];
#pragma unroll
    for (int it = 0; it < PRO_GROUP; ++it) {
      const int n = nbase + (g0 + it) * 64 + (t >> 2);
      const int64_t row = bh * N + (n < N ? n : 0);
      const bool valid = n < N;
      ro[it] = valid ? __ldg(reinterpret_cast<const uint4*>((const T*)a.o + row * TD + sub * 8)) : z4;
      rd[it] = valid ? __ldg(reinterpret_cast<const uint4*>((const T*)a.dout + row * TD + sub * 8)) : z4;
      rq[it] = valid && blank ? __ldg(reinterpret_cast<const uint4*>((const T*)a.q + row * TD + sub * 8)) : z4;
      ls[it] = valid && blank ? __ldg(a.lse + row) : 0.f;
    }
#pragma unroll
    for (int it = 0; it < PRO_GROUP; ++it) {
      const int n = nbase + (g0 + it) * 64 + (t >> 2);
      const bool valid = n < N;
      const int64_t row = bh * N + n;
      float ov[8], dv[8], di = 0.f;
      cvt8<T>(ro[it], ov);
      cvt8<T>(rd[it], dv);
#pragma unroll
      for (int e = 0; e < 8; ++e) di = fmaf(ov[e], dv[e], di);
      di += __shfl_xor_sync(0xffffffffu, di, 1);
      di += __shfl_xor_sync(0xffffffffu, di, 2);
      if (valid && sub == 0) k.di[row] = di;
      if (blank) {
        float qv[8];
        cvt8<T>(rq[it], qv);
        const float4* bk4 = reinterpret_cast<const float4*>(s_bk + sub * 8);
        const float4* bv4 = reinterpret_cast<const float4*>(s_bv + sub * 8);
        const float4 k0 = bk4[0], k1 = bk4[1], v0 = bv4[0], v1 = bv4[1];
        const float bkv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
        const float bvv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        float sb = 0.f, dpb = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) { sb = fmaf(qv[e], bkv[e], sb); dpb = fmaf(dv[e], bvv[e], dpb); }
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
          sb += __shfl_xor_sync(0xffffffffu, sb, o);
          dpb += __shfl_xor_sync(0xffffffffu, dpb, o);
        }
        if (valid) {
          const float pb = expf(sb * a.scale - ls[it]);
          const float dsb = pb * (dpb - di);
          if (sub == 0) k.dsb[row] = dsb;
#pragma unroll
          for (int e = 0; e < 8; ++e) { gk[e] = fmaf(dsb, qv[e], gk[e]); gv[e] = fmaf(pb, dv[e], gv[e]); }
        }
      }
    }
  }
  if (!blank) return;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      gk[e] += __shfl_xor_sync(0xffffffffu, gk[e], o);
      gv[e] += __shfl_xor_sync(0xffffffffu, gv[e], o);
    }
  }
  if (lane < 4) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      atomicAdd(&s_dbk[sub * 8 + e], gk[e]);
      atomicAdd(&s_dbv[sub * 8 + e], gv[e]);
    }
  }
  __syncthreads();
  if (t < TD) {
    red_add(a.dbk + (int64_t)h * TD + t, s_dbk[t] * a.scale);
    red_add(a.dbv + (int64_t)h * TD + t, s_dbv[t]);
  }
}

// The list count (one thread per query) and the prologue (rows of one (b, h))
// share one launch: blocks [0, count_blocks) count, the rest run the prologue.
// The prologue does not wait for the list check: D, the blank dS and the
// blank-token gradients are the same whichever kernels do the rest.
template <typename T>
__global__ void __launch_bounds__(256, AFFB_PRE_MINB) nbhd_bwd_pre_kernel(NbhdArgs a, KvArgs k, NbhdBwdLayout ly,
                                                          int count_blocks, int B, int Cc) {
  dependent_wait();
  if (blockIdx.x < count_blocks) {
    inv_count_block(a.midx, a.mask, a.mask_heads, B, a.N, a.M, Cc, ly.flag, ly.counts, ly.ecl, ly.erk,
                    blockIdx.x);
    return;
  }
  q_prologue_block<T>(a, k, blockIdx.x - count_blocks);
}


// ------------------------------------------------------ key-major pass --

template <typename T>
struct KvWarp {
  alignas(16) T K[8 * TD];
  alignas(16) T V[8 * TD];
  alignas(16) T Q[2][16 * TD];
  alignas(16) T dO[2][16 * TD];
  alignas(16) T bias[2][16 * 8];
  alignas(16) uint8_t mask[2][16 * 8];
  alignas(16) float lse[2][16];
  alignas(16) float di[2][16];
  alignas(16) T ost[8 * TD];
};
// The block's list (or a segment of it) as per-entry offsets shared by the
// heads: qoff = q * D (Q / dO rows), roff = q * M + 8 j (bias / mask / dS runs).
template <typename T>
struct KvSmem {
  int qoff[KV_LCAP];
  int roff[KV_LCAP];
  KvWarp<T> w[NW];
};
static_assert(sizeof(((KvWarp<__half>*)0)->Q) >= KV_LCAP * sizeof(int), "sort buffer aliases a Q stage");

// Per-head base pointers of the key-side kernel.
template <typename T>
struct KvHead {
  const T* q;
  const T* dout;
  const T* bias;
  const uint8_t* mask;
  const float* lse;
  const float* di;
  T* ds;
};

// Gathers chunk rows base .. base+15 (of ns entries) into stage `buf`.
template <typename T>
__device__ __forceinline__ void kv_stage(const KvHead<T>& p, const KvSmem<T>& s, KvWarp<T>& w, int ns, int base,
                                         int buf) {
  const int lane = threadIdx.x & 31;
  const int nr = ns - base;
#pragma unroll
  for (int i = lane; i < 64; i += 32) {
    const int row = i >> 2, piece = i & 3;
    const bool valid = row < nr;
    const int qo = (valid ? s.qoff[base + row] : 0) + piece * 8;
    cp_async16(w.Q[buf] + swz(row, piece), p.q + qo, valid);
    cp_async16(w.dO[buf] + swz(row, piece), p.dout + qo, valid);
  }
  const int row = lane & 15;
  const bool valid = row < nr;
  const int q = valid ? s.qoff[base + row] / TD : 0;
  const int ro = valid ? s.roff[base + row] : 0;
  if (lane < 16) {
    if (p.bias) cp_async16(w.bias[buf] + row * 8, p.bias + ro, valid);
    cp_async4(&w.lse[buf][row], p.lse + q, valid);
  } else {
    if (p.mask) cp_async8(w.mask[buf] + row * 8, p.mask + ro, valid);
    cp_async4(&w.di[buf][row], p.di + q, valid);
  }
}

// Chunks of one list segment (ns entries in s) for one head: accumulates
// dK^T, dV^T and writes dS.
template <typename T>
__device__ __forceinline__ void kv_segment(const NbhdArgs& a, const KvHead<T>& p, const KvSmem<T>& s, KvWarp<T>& w,
                                           int ns, uint32_t* bk, uint32_t* bv, bool& frags, float (*dkt)[4],
                                           float (*dvt)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int nch = (ns + 15) >> 4;
  kv_stage<T>(p, s, w, ns, 0, 0);
  cp_commit();
  for (int ch = 0; ch < nch; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < nch) kv_stage<T>(p, s, w, ns, (ch + 1) * 16, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncwarp();
    if (!frags) {  // K / V rows of the cluster arrived with the first stage
      ldsm_x4(bk, w.K + swz(lane & 7, lane >> 3));
      ldsm_x4(bv, w.V + swz(lane & 7, lane >> 3));
      frags = true;
    }
    uint32_t aq[2][4], ado[2][4];
    load_a_frags(aq, w.Q[buf]);
    load_a_frags(ado, w.dO[buf]);
    float sc[4] = {0.f, 0.f, 0.f, 0.f}, dp[4] = {0.f, 0.f, 0.f, 0.f};
    MmaType<T>::mma(sc, aq[0], bk);
    MmaType<T>::mma(sc, aq[1], bk + 2);
    MmaType<T>::mma(dp, ado[0], bv);
    MmaType<T>::mma(dp, ado[1], bv + 2);
    const int nr = ns - ch * 16;
    uint32_t pp[2], pd[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int row = g + 8 * hf;
      const float ls = w.lse[buf][row], dd = w.di[buf][row];
      float b0 = 0.f, b1 = 0.f;
      if (p.bias) {
        const uint32_t u = *reinterpret_cast<const uint32_t*>(w.bias[buf] + row * 8 + 2 * tq);
        const T* hp = reinterpret_cast<const T*>(&u);
        b0 = io<T>::ld(hp);
        b1 = io<T>::ld(hp + 1);
      }
      bool v0 = row < nr, v1 = v0;
      if (p.mask) {
        v0 = v0 && w.mask[buf][row * 8 + 2 * tq] != 0;
        v1 = v1 && w.mask[buf][row * 8 + 2 * tq + 1] != 0;
      }
      const float p0 = v0 ? __expf(sc[2 * hf] * a.scale + b0 - ls) : 0.f;
      const float p1 = v1 ? __expf(sc[2 * hf + 1] * a.scale + b1 - ls) : 0.f;
      pp[hf] = pack2<T>(p0, p1);
      pd[hf] = pack2<T>(p0 * (dp[2 * hf] - dd), p1 * (dp[2 * hf + 1] - dd));
      // dS of the chunk staged as 16 runs of 8 (16 bytes each) for one vector store per run
      reinterpret_cast<uint32_t*>(w.ost)[row * 4 + tq] = pd[hf];
    }
    __syncwarp();
    // dS in bias layout: the run of query q's list position j (16-byte aligned: offset q*M + 8j)
    if (lane < 16 && lane < nr)
      *reinterpret_cast<uint4*>(p.ds + s.roff[ch * 16 + lane]) = reinterpret_cast<const uint4*>(w.ost)[lane];
    const uint32_t bp[2] = {movmatrix_t(pp[0]), movmatrix_t(pp[1])};
    const uint32_t bd[2] = {movmatrix_t(pd[0]), movmatrix_t(pd[1])};
    const int mi = lane >> 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      // A[m = dim][k = query] = X[query][dim]: matrices (d 0-7, q 0-7), (d 8-15, q 0-7), (d 0-7, q 8-15), (d 8-15, q 8-15)
      const int off = swz((mi >> 1) * 8 + (lane & 7), mt * 2 + (mi & 1));
      uint32_t ad[4], aqt[4];
      ldsm_x4_t(ad, w.dO[buf] + off);
      ldsm_x4_t(aqt, w.Q[buf] + off);
      MmaType<T>::mma(dvt[mt], ad, bp);
      MmaType<T>::mma(dkt[mt], aqt, bd);
    }
    __syncwarp();
  }
}

// Loads entries [seg0, seg0 + ns) of the list into the offset tables, sorted
// by query when `sort` (the whole list is one segment).
template <typename T>
__device__ __forceinline__ void kv_load_segment(KvSmem<T>& s, const int* src, int ns, int M, bool sort) {
  const int t = threadIdx.x;
  __syncthreads();  // previous segment no longer read
  if (!sort) {
    for (int i = t; i < ns; i += TC_THREADS) {
      const int e = src[i];
      s.qoff[i] = (e >> 3) * TD;
      s.roff[i] = (e >> 3) * M + 8 * (e & 7);
    }
  } else {  // rank sort (entries are distinct); before any staging, so a Q stage holds the copy
    int* tmp = reinterpret_cast<int*>(s.w[0].Q);
    const int n4 = (ns + 3) >> 2;  // padded with INT_MAX, which no entry exceeds
    for (int i = t; i < 4 * n4; i += TC_THREADS) tmp[i] = i < ns ? src[i] : 0x7fffffff;
    __syncthreads();
    const int4* t4 = reinterpret_cast<const int4*>(tmp);
    for (int i = t; i < ns; i += TC_THREADS) {
      const int e = tmp[i];
      int r = 0;
#pragma unroll 4
      for (int m = 0; m < n4; ++m) {
        const int4 v = t4[m];
        r += (v.x < e) + (v.y < e) + (v.z < e) + (v.w < e);
      }
      s.qoff[r] = (e >> 3) * TD;
      s.roff[r] = (e >> 3) * M + 8 * (e & 7);
    }
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(TC_THREADS, AFFB_KV_MINB) nbhd_kv_kernel(NbhdArgs a, KvArgs k) {
  dependent_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  KvSmem<T>& s = *reinterpret_cast<KvSmem<T>*>(smem_raw);
  const int N = a.N, M = a.M, Cc = k.Cc;
  const int b = blockIdx.x / Cc, c = blockIdx.x % Cc;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, g = lane >> 2, tq = lane & 3;
  const int kr0 = 8 * c, nkeys = min(8, N - kr0);
  if (*k.flag) {  // general lists: convert the fp32 sums of the query side
    const int per_head = nkeys * TD;
    for (int i = t; i < a.H * per_head; i += TC_THREADS) {
      const int h = i / per_head, r = i % per_head;
      const int64_t o = (((int64_t)b * a.H + h) * N + kr0) * TD + r;
      io<T>::st((T*)k.dk + o, k.acc_k[o]);
      io<T>::st((T*)k.dv + o, k.acc_v[o]);
    }
    return;
  }
  const int64_t cell = (int64_t)b * Cc + c;
  const int n = k.counts[cell];
  const int* src = k.entries + k.offs[cell];
  const bool one = n <= KV_LCAP;
  if (one) kv_load_segment(s, src, n, M, true);
  KvWarp<T>& w = s.w[warp];
  for (int hg = 0; hg < a.H; hg += NW) {
    const int h = hg + warp;
    const bool act = h < a.H;
    const int64_t bh = (int64_t)b * a.H + h;
    KvHead<T> p;
    p.q = (const T*)a.q + bh * N * TD;
    p.dout = (const T*)a.dout + bh * N * TD;
    p.bias = a.bias ? (const T*)a.bias + bh * N * M : nullptr;
    p.mask = a.mask ? a.mask + ((int64_t)b * a.mask_heads + (a.mask_heads == 1 ? 0 : h)) * N * M : nullptr;
    p.lse = a.lse + bh * N;
    p.di = k.di + bh * N;
    p.ds = (T*)k.ds + bh * N * M;
    float dkt[2][4], dvt[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) dkt[i][e] = dvt[i][e] = 0.f;
    uint32_t bk[4], bv[4];
    bool frags = false;
    if (act && n > 0) {  // completes with the first stage of kv_segment
      const int row = lane >> 2, piece = lane & 3;
      const bool valid = row < nkeys;
      const int64_t off = (bh * N + kr0 + (valid ? row : 0)) * TD + piece * 8;
      cp_async16(w.K + swz(row, piece), (const T*)a.k + off, valid);
      cp_async16(w.V + swz(row, piece), (const T*)a.v + off, valid);
    }
    for (int seg0 = 0; seg0 < n; seg0 += KV_LCAP) {
      const int ns = min(KV_LCAP, n - seg0);
      if (!one) kv_load_segment(s, src + seg0, ns, M, false);
      if (act) kv_segment<T>(a, p, s, w, ns, bk, bv, frags, dkt, dvt);
    }
    if (!act) continue;
    // transpose through shared memory and store 16-byte pieces of the key rows
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      const float(*acc)[4] = pass == 0 ? dkt : dvt;
      const float mul = pass == 0 ? a.scale : 1.f;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = mt * 16 + g + (e >> 1) * 8, key = 2 * tq + (e & 1);
          io<T>::st(w.ost + swz(key, d >> 3) + (d & 7), acc[mt][e] * mul);
        }
      __syncwarp();
      const int row = lane >> 2, piece = lane & 3;
      if (row < nkeys) {
        T* dst = (T*)(pass == 0 ? k.dk : k.dv) + (bh * N + kr0 + row) * TD + piece * 8;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(w.ost + swz(row, piece));
      }
      __syncwarp();
    }
  }
}

int nbhd_kv_bwd(const NbhdArgs& a, const KvArgs& k, int dtype, int B, cudaStream_t st) {
  const int64_t blocks = (int64_t)B * k.Cc;
  if (blocks == 0) return AFFB_OK;
  AFFB_REQUIRE(blocks < (1ll << 31), "nbhd_attn_bwd: too many key clusters");
  auto go = [&](auto kernel, size_t smem) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
      set_error("nbhd_attn_bwd: cannot reserve %zu bytes of shared memory", smem);
      return AFFB_ERR_CUDA;
    }
    if (launch_dependent(kernel, dim3((unsigned)blocks), dim3(TC_THREADS), smem, st, a, k) != cudaSuccess) {
      set_error("nbhd_attn_bwd: key-side kernel failed to launch");
      return AFFB_ERR_CUDA;
    }
    return AFFB_OK;
  };
  if (dtype == AFFB_BF16) return go(nbhd_kv_kernel<__nv_bfloat16>, sizeof(KvSmem<__nv_bfloat16>));
  return go(nbhd_kv_kernel<__half>, sizeof(KvSmem<__half>));
}

int nbhd_bwd_prepare(const NbhdArgs& a, const KvArgs& k, const NbhdBwdLayout& ly, int dtype, int B,
                     cudaStream_t st) {
  const int N = a.N, M = a.M, Cc = k.Cc;
  const int64_t rows = (int64_t)B * N;
  // the list flag and counters are cleared by a kernel (not a memset) so the
  // whole chain, from the forward on, runs under programmatic dependent launch
  const int64_t z16 = (int64_t)(ly.zero_bytes / 16);
  if (launch_dependent(nbhd_zero_kernel, dim3((unsigned)imin64((z16 + 255) / 256, (int64_t)sm_count() * 4)),
                       dim3(256), 0, st, reinterpret_cast<uint4*>(ly.flag), z16) != cudaSuccess) {
    set_error("nbhd_attn_bwd: list counter clear failed to launch");
    return AFFB_ERR_CUDA;
  }
  const int64_t cnt = (rows + 255) / 256;
  const int64_t pro = (int64_t)B * a.H * ((N + PRO_ROWS - 1) / PRO_ROWS);
  AFFB_REQUIRE(cnt + pro < (1ll << 31), "nbhd_attn_bwd: too many rows");
  const unsigned g = (unsigned)(cnt + pro);
  const cudaError_t le = dtype == AFFB_BF16
      ? launch_dependent(nbhd_bwd_pre_kernel<__nv_bfloat16>, dim3(g), dim3(256), 0, st, a, k, ly, (int)cnt, B, Cc)
      : launch_dependent(nbhd_bwd_pre_kernel<__half>, dim3(g), dim3(256), 0, st, a, k, ly, (int)cnt, B, Cc);
  if (le != cudaSuccess) {
    set_error("nbhd_attn_bwd: list count / prologue kernel failed to launch");
    return AFFB_ERR_CUDA;
  }
  if (launch_dependent(nbhd_inv_scan_kernel, dim3(B), dim3(1024), 0, st, ly.counts, N, M >> 3, Cc, ly.flag,
                       ly.offs) != cudaSuccess ||
      launch_dependent(nbhd_inv_fill_kernel, dim3((unsigned)cnt), dim3(256), 0, st, B, N, M, Cc, a.H, ly.flag,
                       ly.offs, ly.ecl, ly.erk, ly.entries, ly.acc_k, ly.acc_v) != cudaSuccess) {
    set_error("nbhd_attn_bwd: list kernels failed to launch");
    return AFFB_ERR_CUDA;
  }
  return AFFB_OK;
}

}  // namespace affb
