// Weighted features forward on the tensor cores (16-bit storage, C % 16 == 0,
// IC <= 8):
//
//   out[b,i,ic,c] = sum_m w[b,i,m,ic] * feat[b, idx[b,i,m], c]
//
// is, per output token, the product out^T [C x IC] = F^T [C x M] . W [M x IC]
// of its gathered neighbour rows F and its weights W.  One warp streams tasks
// (token, channel slice of at most 128 channels); each task is ceil(M/16)
// steps of 16 neighbour rows, gathered with cp.async into a 4-stage ring of
// shared-memory tiles (row stride CW + 8 elements, so ldmatrix.trans reads
// them without bank conflicts) while earlier stages are multiplied:
// mma.m16n8k16 with A = 16 channels x 16 neighbours (ldmatrix.trans of the
// rows) and B = 16 neighbours x 8 weight columns (IC of them non-zero).  The
// CUDA-core kernels of weighted_features.cu spend 4 x 96 x 48 multiply-adds
// per token of config 5 on the FMA pipe; here they are 18 mma per token.
#include "nbhd_mma.cuh"

namespace affb {

constexpr int WT_WARPS = 4;
constexpr int WT_STAGES = 3;
constexpr int WT_WPAD = 16 * 8;  // weight elements per stage (16 neighbours x IC <= 8)

__device__ __forceinline__ void cp_async16_n(void* dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes));
}

template <int MT>
struct WtLayout {
  static constexpr int CW = 16 * MT;           // channels per slice
  static constexpr int RS = CW + 8;            // feature row stride (elements)
  static constexpr int STAGE = 16 * RS + WT_WPAD;  // elements per stage
};

template <typename T, int MT>
__global__ void __launch_bounds__(WT_WARPS * 32, 5)
wf_fwd_tc_kernel(const T* __restrict__ w, const T* __restrict__ feat, const int32_t* __restrict__ idx,
                 int B, int No, int M, int IC, int64_t N, int C, bool wvec, T* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using L = WtLayout<MT>;
  constexpr int CW = L::CW, RS = L::RS, STAGE = L::STAGE;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tq = lane & 3;
  T* ring = reinterpret_cast<T*>(smem_raw) + (size_t)warp * WT_STAGES * STAGE;
  const int nslice = C / CW;
  const int KS = (M + 15) >> 4;
  const int ntask = B * No * nslice;  // < 2^31, checked by the host
  const int gw = blockIdx.x * WT_WARPS + warp, nw = gridDim.x * WT_WARPS;
  // gather: an 8-lane group copies one feature row (16-byte chunks lane8 and
  // lane8 + 8); the warp covers rows 4j + (lane >> 3), j < 4, per instruction
  // pair, so each instruction reads four rows of contiguous bytes
  constexpr int CH = CW / 8;  // chunks per row, 2..16
  const int l8 = lane & 7, r4 = lane >> 3;
  // producer cursor: the next (task, step) to gather, its ring slot, the
  // task's feature slice, index and weight rows, and the indices of this
  // lane's four rows in that step (loaded one step ahead)
  int ptask = gw, pks = 0, pslot = 0;
  int myid[4] = {0, 0, 0, 0};
  const T* pfb = nullptr;
  const int32_t* pir = nullptr;
  const T* pwr = nullptr;
  auto set_task = [&]() {
    if (ptask >= ntask) return;
    const int tok = ptask / nslice, sl = ptask - tok * nslice;
    pfb = feat + (int64_t)(tok / No) * N * C + sl * CW + l8 * 8;
    pir = idx + (int64_t)tok * M;
    pwr = w + (int64_t)tok * M * IC;
  };
  auto load_id = [&]() {
    if (ptask < ntask) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int nb = pks * 16 + 4 * j + r4;
        myid[j] = nb < M ? __ldg(pir + nb) : 0;
      }
    }
  };
  set_task();
  load_id();
  auto produce = [&]() {
    if (ptask < ntask) {
      T* dst = ring + pslot * STAGE;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = 4 * j + r4;
        const bool ok = pks * 16 + r < M;
        const T* src = pfb + (int64_t)myid[j] * C;
        T* d = dst + r * RS + l8 * 8;
        if (CH >= 8 || l8 < CH) cp_async16(d, src, ok);
        if (CH > 8 && l8 < CH - 8) cp_async16(d + 64, src + 64, ok);
      }
      // weights of the step's 16 neighbours, zero past M
      T* sw = dst + 16 * RS;
      const int e0 = pks * 16 * IC, etot = M * IC;
      if (wvec) {
        if (lane < 2 * IC) {
          const int e = e0 + lane * 8;
          const int v = etot - e;
          cp_async16_n(sw + lane * 8, pwr + (v > 0 ? e : 0), v >= 8 ? 16 : (v > 0 ? v * 2 : 0));
        }
      } else {
        for (int k = lane; k < 16 * IC; k += 32)
          stf(sw + k, e0 + k < etot ? ldf(pwr + e0 + k) : 0.f);
      }
      pslot = pslot == WT_STAGES - 1 ? 0 : pslot + 1;
      if (++pks == KS) {
        pks = 0;
        ptask += nw;
        set_task();
      }
      load_id();
    }
    cp_commit();
  };
#pragma unroll
  for (int i = 0; i < WT_STAGES - 1; ++i) produce();
  const int mi = lane >> 3;
  int cslot = 0;
  for (int task = gw; task < ntask; task += nw) {
    const int tok = task / nslice, sl = task - tok * nslice;
    float acc[MT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    int last = 0;
    for (int ks = 0; ks < KS; ++ks) {
      produce();
      cp_wait<WT_STAGES - 1>();
      __syncwarp();
      const T* stg = ring + cslot * STAGE;
      // B: weights of neighbours {2tq, 2tq+1, 2tq+8, 2tq+9} of the step, column g
      uint32_t bw[2] = {0u, 0u};
      if (g < IC) {
        const T* sw = stg + 16 * RS + 2 * tq * IC + g;
        bw[0] = pack2<T>(ldf(sw), ldf(sw + IC));
        bw[1] = pack2<T>(ldf(sw + 8 * IC), ldf(sw + 9 * IC));
      }
      const T* st = stg + ((mi >> 1) * 8 + (lane & 7)) * RS + (mi & 1) * 8;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        // A[m = channel][k = neighbour] = F[neighbour][channel]: matrices (c 0-7, nb 0-7),
        // (c 8-15, nb 0-7), (c 0-7, nb 8-15), (c 8-15, nb 8-15)
        uint32_t a[4];
        ldsm_x4_t(a, st + mt * 16);
        MmaType<T>::mma(acc[mt], a, bw);
      }
      __syncwarp();
      last = cslot;
      cslot = cslot == WT_STAGES - 1 ? 0 : cslot + 1;
    }
    // out[tok, ic, slice channels], transposed through the slot just consumed
    // (refilled only by the next produce): [IC][CW + 8] tile, then 16-byte rows
    T* tile = ring + last * STAGE;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = mt * 16 + g + (e >> 1) * 8, ic = 2 * tq + (e & 1);
        if (ic < IC) stf(tile + ic * RS + c, acc[mt][e]);
      }
    }
    __syncwarp();
    T* ob = out + (int64_t)tok * IC * C + sl * CW;
    for (int p = lane; p < IC * (CW / 8); p += 32) {
      const int ic = p / (CW / 8), ch = p - ic * (CW / 8);
      *reinterpret_cast<uint4*>(ob + ic * C + ch * 8) = *reinterpret_cast<const uint4*>(tile + ic * RS + ch * 8);
    }
    __syncwarp();
  }
  cp_wait<0>();
}

template <typename T, int MT>
static int launch_tc(const T* w, const T* feat, const int32_t* idx, int64_t B, int64_t No, int M, int IC,
                     int64_t N, int C, T* out, cudaStream_t st) {
  const size_t smem = (size_t)WT_WARPS * WT_STAGES * WtLayout<MT>::STAGE * sizeof(T);
  auto k = wf_fwd_tc_kernel<T, MT>;
  int per_sm = 0;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
      cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, WT_WARPS * 32, smem) != cudaSuccess) {
    set_error("weighted_features: cannot configure the tensor-core kernel (%zu bytes of shared memory)", smem);
    return AFFB_ERR_CUDA;
  }
  const bool wvec = (M * IC) % 8 == 0 && ((uintptr_t)w & 15) == 0;
  const int64_t ntask = B * No * (C / (16 * MT));
  const int64_t want = (ntask + WT_WARPS - 1) / WT_WARPS;
  const unsigned blocks = (unsigned)imin64(want, (int64_t)sm_count() * (per_sm > 0 ? per_sm : 1));
  k<<<blocks, WT_WARPS * 32, smem, st>>>(w, feat, idx, (int)B, (int)No, M, IC, N, C, wvec, out);
  return AFFB_OK;
}

// Backward, per output token (F its gathered rows, W its weights, D = dout
// of the token, [IC x C]):
//   dW [M x IC] = F . D^T        mma.m16n8k16, A = 16 rows x 16 channels of F
//                                (ldmatrix), B = D^T (registers, per slice)
//   dF [M x C]  = W . D          mma.m16n8k8, A = the 16 x 8 weight tile,
//                                B = 8 x 8 blocks of D (movmatrix.trans of the
//                                dW operand registers)
// and dF is scattered into the fp32 feature gradient with red.add.v2.  Steps
// are (16 neighbours, channel slice of at most 128) with the slices innermost,
// so the dW tile of a neighbour block accumulates over the slices in registers.
__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

template <typename T> struct Mma8;
template <> struct Mma8<__nv_bfloat16> {
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(b));
  }
};
template <> struct Mma8<__half> {
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(b));
  }
};

template <typename T, int MT>
__global__ void __launch_bounds__(WT_WARPS * 32, 4)
wf_bwd_tc_kernel(const T* __restrict__ dout, const T* __restrict__ w, const T* __restrict__ feat,
                 const int32_t* __restrict__ idx, int B, int No, int M, int IC, int64_t N, int C, bool wvec,
                 T* __restrict__ dw, float* __restrict__ dfeat) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using L = WtLayout<MT>;
  constexpr int CW = L::CW, RS = L::RS, STAGE = L::STAGE;
  constexpr int CH = CW / 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tq = lane & 3;
  T* ring = reinterpret_cast<T*>(smem_raw) + (size_t)warp * WT_STAGES * STAGE;
  const int nslice = C / CW;
  const int KS = (M + 15) >> 4;
  const int ntok = B * No;
  const int gw = blockIdx.x * WT_WARPS + warp, nw = gridDim.x * WT_WARPS;
  const int l8 = lane & 7, r4 = lane >> 3;
  // producer cursor: token, neighbour block, slice, ring slot, row pointers
  int ptok = gw, pks = 0, psl = 0, pslot = 0;
  int myid[4] = {0, 0, 0, 0};
  const T* pfb = nullptr;
  const int32_t* pir = nullptr;
  const T* pwr = nullptr;
  auto set_tok = [&]() {
    if (ptok >= ntok) return;
    pfb = feat + (int64_t)(ptok / No) * N * C + l8 * 8;
    pir = idx + (int64_t)ptok * M;
    pwr = w + (int64_t)ptok * M * IC;
  };
  auto load_id = [&]() {
    if (ptok < ntok) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int nb = pks * 16 + 4 * j + r4;
        myid[j] = nb < M ? __ldg(pir + nb) : 0;
      }
    }
  };
  set_tok();
  load_id();
  auto produce = [&]() {
    if (ptok < ntok) {
      T* dst = ring + pslot * STAGE;
      const T* fs = pfb + psl * CW;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = 4 * j + r4;
        const bool ok = pks * 16 + r < M;
        const T* src = fs + (int64_t)myid[j] * C;
        T* d = dst + r * RS + l8 * 8;
        if (CH >= 8 || l8 < CH) cp_async16(d, src, ok);
        if (CH > 8 && l8 < CH - 8) cp_async16(d + 64, src + 64, ok);
      }
      if (psl == 0) {  // weights of the block, once per neighbour block
        T* sw = dst + 16 * RS;
        const int e0 = pks * 16 * IC, etot = M * IC;
        if (wvec) {
          if (lane < 2 * IC) {
            const int e = e0 + lane * 8;
            const int v = etot - e;
            cp_async16_n(sw + lane * 8, pwr + (v > 0 ? e : 0), v >= 8 ? 16 : (v > 0 ? v * 2 : 0));
          }
        } else {
          for (int k = lane; k < 16 * IC; k += 32) stf(sw + k, e0 + k < etot ? ldf(pwr + e0 + k) : 0.f);
        }
      }
      pslot = pslot == WT_STAGES - 1 ? 0 : pslot + 1;
      if (++psl == nslice) {
        psl = 0;
        if (++pks == KS) {
          pks = 0;
          ptok += nw;
          set_tok();
        }
        load_id();
      }
    }
    cp_commit();
  };
#pragma unroll
  for (int i = 0; i < WT_STAGES - 1; ++i) produce();
  int cslot = 0;
  for (int tok = gw; tok < ntok; tok += nw) {
    const T* dor = dout + (int64_t)tok * IC * C + g * C + 2 * tq;
    float* dfb = dfeat + (int64_t)(tok / No) * N * C + 2 * tq;
    const int32_t* ir = idx + (int64_t)tok * M;
    T* dwr = dw + (int64_t)tok * M * IC;
    uint32_t bd[MT][2];  // D^T operands of the current slice: D[g][16 kc + 8 h + 2 tq .. +1]
    int dsl = -1;
    uint32_t aw[2] = {0u, 0u};  // weight tile of the current neighbour block
    for (int ks = 0; ks < KS; ++ks) {
      float dwa[4] = {0.f, 0.f, 0.f, 0.f};
      const int nbg = ks * 16 + g;
      const int id0 = nbg < M ? __ldg(ir + nbg) : -1, id1 = nbg + 8 < M ? __ldg(ir + nbg + 8) : -1;
      for (int sl = 0; sl < nslice; ++sl) {
        if (sl != dsl) {
#pragma unroll
          for (int kc = 0; kc < MT; ++kc)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              bd[kc][h] = g < IC ? __ldg(reinterpret_cast<const uint32_t*>(dor + sl * CW + kc * 16 + h * 8)) : 0u;
          dsl = sl;
        }
        produce();
        cp_wait<WT_STAGES - 1>();
        __syncwarp();
        const T* stg = ring + cslot * STAGE;
        if (sl == 0) {
          // A of W . D: rows g / g + 8 (neighbours), columns 2tq, 2tq + 1 (ic)
          const T* sw = stg + 16 * RS;
          const int c0 = 2 * tq;
          const float w00 = c0 < IC ? ldf(sw + g * IC + c0) : 0.f, w01 = c0 + 1 < IC ? ldf(sw + g * IC + c0 + 1) : 0.f;
          const float w10 = c0 < IC ? ldf(sw + (g + 8) * IC + c0) : 0.f,
                      w11 = c0 + 1 < IC ? ldf(sw + (g + 8) * IC + c0 + 1) : 0.f;
          aw[0] = pack2<T>(w00, w01);
          aw[1] = pack2<T>(w10, w11);
        }
        const T* st = stg + (((lane >> 3) & 1) * 8 + (lane & 7)) * RS + (lane >> 4) * 8;
#pragma unroll
        for (int kc = 0; kc < MT; ++kc) {
          uint32_t a[4];
          ldsm_x4(a, st + kc * 16);
          MmaType<T>::mma(dwa, a, bd[kc]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float df[4] = {0.f, 0.f, 0.f, 0.f};
            Mma8<T>::mma(df, aw, movm_t(bd[kc][h]));
            const int c = sl * CW + kc * 16 + h * 8;
            if (id0 >= 0) red_add_v2(dfb + (int64_t)id0 * C + c, df[0], df[1]);
            if (id1 >= 0) red_add_v2(dfb + (int64_t)id1 * C + c, df[2], df[3]);
          }
        }
        __syncwarp();
        cslot = cslot == WT_STAGES - 1 ? 0 : cslot + 1;
      }
      // dW rows g / g + 8 of the block, columns 2tq, 2tq + 1
      const int ic = 2 * tq;
      if (nbg < M) {
        if (ic < IC) stf(dwr + nbg * IC + ic, dwa[0]);
        if (ic + 1 < IC) stf(dwr + nbg * IC + ic + 1, dwa[1]);
      }
      if (nbg + 8 < M) {
        if (ic < IC) stf(dwr + (nbg + 8) * IC + ic, dwa[2]);
        if (ic + 1 < IC) stf(dwr + (nbg + 8) * IC + ic + 1, dwa[3]);
      }
    }
  }
  cp_wait<0>();
}

template <typename T, int MT>
static int launch_bwd_tc(const T* dout, const T* w, const T* feat, const int32_t* idx, int64_t B, int64_t No, int M,
                         int IC, int64_t N, int C, T* dw, float* dfeat, cudaStream_t st) {
  const size_t smem = (size_t)WT_WARPS * WT_STAGES * WtLayout<MT>::STAGE * sizeof(T);
  auto k = wf_bwd_tc_kernel<T, MT>;
  int per_sm = 0;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
      cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, WT_WARPS * 32, smem) != cudaSuccess) {
    set_error("weighted_features: cannot configure the tensor-core kernel (%zu bytes of shared memory)", smem);
    return AFFB_ERR_CUDA;
  }
  const bool wvec = (M * IC) % 8 == 0 && ((uintptr_t)w & 15) == 0;
  const int64_t ntok = B * No;
  const int64_t want = (ntok + WT_WARPS - 1) / WT_WARPS;
  const unsigned blocks = (unsigned)imin64(want, (int64_t)sm_count() * (per_sm > 0 ? per_sm : 1));
  k<<<blocks, WT_WARPS * 32, smem, st>>>(dout, w, feat, idx, (int)B, (int)No, M, IC, N, C, wvec, dw, dfeat);
  return AFFB_OK;
}

template <typename T>
bool wf_bwd_tc(const T* dout, const T* w, const T* feat, const int32_t* idx, int64_t B, int64_t No, int M, int IC,
               int64_t N, int C, T* dw, float* dfeat, cudaStream_t st, int* err) {
  if (C % 16 != 0 || IC > 8 || M < 1 || ((uintptr_t)feat & 15) != 0 || ((uintptr_t)dout & 3) != 0 ||
      ((uintptr_t)dfeat & 7) != 0)
    return false;
  if (B * No * (C / 16) >= (1ll << 31) || (int64_t)M * IC * C >= (1ll << 31)) return false;
  int mt = 8;
  while (mt > 1 && (C % (16 * mt)) != 0) --mt;
  switch (mt) {
    case 8: *err = launch_bwd_tc<T, 8>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st); break;
    case 7: *err = launch_bwd_tc<T, 7>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st); break;
    case 6: *err = launch_bwd_tc<T, 6>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st); break;
    case 5: *err = launch_bwd_tc<T, 5>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st); break;
    case 4: *err = launch_bwd_tc<T, 4>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st); break;
    case 3: *err = launch_bwd_tc<T, 3>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st); break;
    case 2: *err = launch_bwd_tc<T, 2>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st); break;
    default: *err = launch_bwd_tc<T, 1>(dout, w, feat, idx, B, No, M, IC, N, C, dw, dfeat, st); break;
  }
  return true;
}

template bool wf_bwd_tc<__nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
                                       const int32_t*, int64_t, int64_t, int, int, int64_t, int, __nv_bfloat16*,
                                       float*, cudaStream_t, int*);
template bool wf_bwd_tc<__half>(const __half*, const __half*, const __half*, const int32_t*, int64_t, int64_t, int,
                                int, int64_t, int, __half*, float*, cudaStream_t, int*);

// Forward on the tensor cores when the shape allows it; returns false (nothing
// launched) otherwise.
template <typename T>
bool wf_fwd_tc(const T* w, const T* feat, const int32_t* idx, int64_t B, int64_t No, int M, int IC, int64_t N,
               int C, T* out, cudaStream_t st, int* err) {
  if (C % 16 != 0 || IC > 8 || M < 1 || ((uintptr_t)feat & 15) != 0 || ((uintptr_t)out & 15) != 0) return false;
  // task and token indices are 32-bit; M * IC per token bounded by the caller
  if (B * No * (C / 16) >= (1ll << 31) || (int64_t)M * IC * C >= (1ll << 31)) return false;
  // widest slice of at most 128 channels that divides C
  int mt = 8;
  while (mt > 1 && (C % (16 * mt)) != 0) --mt;
  switch (mt) {
    case 8: *err = launch_tc<T, 8>(w, feat, idx, B, No, M, IC, N, C, out, st); break;
    case 7: *err = launch_tc<T, 7>(w, feat, idx, B, No, M, IC, N, C, out, st); break;
    case 6: *err = launch_tc<T, 6>(w, feat, idx, B, No, M, IC, N, C, out, st); break;
    case 5: *err = launch_tc<T, 5>(w, feat, idx, B, No, M, IC, N, C, out, st); break;
    case 4: *err = launch_tc<T, 4>(w, feat, idx, B, No, M, IC, N, C, out, st); break;
    case 3: *err = launch_tc<T, 3>(w, feat, idx, B, No, M, IC, N, C, out, st); break;
    case 2: *err = launch_tc<T, 2>(w, feat, idx, B, No, M, IC, N, C, out, st); break;
    default: *err = launch_tc<T, 1>(w, feat, idx, B, No, M, IC, N, C, out, st); break;
  }
  return true;
}

template bool wf_fwd_tc<__nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, const int32_t*, int64_t,
                                       int64_t, int, int, int64_t, int, __nv_bfloat16*, cudaStream_t, int*);
template bool wf_fwd_tc<__half>(const __half*, const __half*, const int32_t*, int64_t, int64_t, int, int, int64_t,
                                int, __half*, cudaStream_t, int*);

}  // namespace affb
