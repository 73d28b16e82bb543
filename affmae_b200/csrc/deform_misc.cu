// Secondary deformable-attention operators and the relative-position bias
// gather.  None of these is on the default model path; they complete the
// operator surface of the reference's kernel package.
//
//  * deform_nbidx: fused Shepard weights + weighted gather for precomputed
//    neighbours (FusedDeformAttnFunction, fused_deform_attn.py:79-231 fwd,
//    :252-491 bwd; its backward divides by max(dist - 1e-6, 1e-8)).
//  * msdetrpc: double-weighted gather (MSDETRPCFunction, msdetrpc.py:25-299).
//  * mssample: Shepard weights softmax(-P*sqrt(d2 + 1e-6)) and their
//    gradients (MSSampleFunction, mssample.py:17-297).
//  * pos_bias: bias[b,h,n,m] = table[pe_idx[b,n,m], h], the gather+permute of
//    ClusterAttention._make_pos_bias (src/layers/attention.py:110-124), and
//    its scatter-add backward.
//
// Layout: one warp per output row with lanes over channels (gathers of whole
// value rows are coalesced), or one thread per row for the scalar-only ops.
#include "common.cuh"

namespace affb {

constexpr int MW = 8;  // warps per block
constexpr int KMAX = 16;

// Shepard softmax over K neighbours, logits = -P * dist with
// MODE 0: dist = sqrt(d2) + 1e-6 (fused kernels), MODE 1: sqrt(d2 + 1e-6).
template <int MODE>
__device__ __forceinline__ void shepard_k(const float* __restrict__ sl, const float* __restrict__ kv,
                                          const int32_t* __restrict__ nb, int K, int D, float P,
                                          float* w, float* dist) {
  float mx = -3.4e38f;
  for (int k = 0; k < K; ++k) {
    const float* p = kv + (int64_t)nb[k] * D;
    float d2 = 0.f;
    for (int d = 0; d < D; ++d) {
      const float df = __fsub_rn(sl[d], p[d]);
      d2 = __fadd_rn(d2, __fmul_rn(df, df));
    }
    dist[k] = MODE == 0 ? sqrtf(d2) + 1e-6f : sqrtf(d2 + 1e-6f);
    mx = fmaxf(mx, -P * dist[k]);
  }
  float sum = 0.f;
  for (int k = 0; k < K; ++k) { w[k] = expf(-P * dist[k] - mx); sum += w[k]; }
  for (int k = 0; k < K; ++k) w[k] = w[k] / (sum + 1e-8f);
}

// ---------------------------------------------------------- deform_nbidx
template <typename T>
__global__ void __launch_bounds__(MW * 32)
nbidx_fwd_kernel(const float* __restrict__ sl, const float* __restrict__ kvpos,
                 const int32_t* __restrict__ nb, const float* __restrict__ power,
                 const float* __restrict__ aw, const T* __restrict__ val, int64_t B, int64_t N,
                 int64_t Nkv, int K, int D, int C, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * MW + (threadIdx.x >> 5);
  if (r >= B * N) return;
  const int64_t b = r / N;
  const float P = fmaxf(power[0], 1e-6f);
  float w[KMAX], dist[KMAX];
  shepard_k<0>(sl + r * D, kvpos + b * Nkv * D, nb + r * K, K, D, P, w, dist);
  const float a = aw[r];
  const T* vb = val + b * Nkv * C;
  for (int c = lane; c < C; c += 32) {
    float acc = 0.f;
    for (int k = 0; k < K; ++k) acc = fmaf(a * w[k], ldf(vb + (int64_t)nb[r * K + k] * C + c), acc);
    stf(out + r * C + c, acc);
  }
}

template <typename T>
__global__ void __launch_bounds__(MW * 32)
nbidx_bwd_kernel(const float* __restrict__ sl, const float* __restrict__ kvpos,
                 const int32_t* __restrict__ nb, const float* __restrict__ power,
                 const float* __restrict__ aw, const T* __restrict__ val,
                 const T* __restrict__ dout, int64_t B, int64_t N, int64_t Nkv, int K, int D,
                 int C, float* __restrict__ d_sl, float* __restrict__ d_kv,
                 float* __restrict__ d_pow, float* __restrict__ d_aw, float* __restrict__ d_val) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * MW + (threadIdx.x >> 5);
  if (r >= B * N) return;
  const int64_t b = r / N;
  const float P = fmaxf(power[0], 1e-6f);
  float w[KMAX], dist[KMAX], dot[KMAX];
  const float* kvb = kvpos + b * Nkv * D;
  const int32_t* nr = nb + r * K;
  shepard_k<0>(sl + r * D, kvb, nr, K, D, P, w, dist);
  const float a = aw[r];
  const T* vb = val + b * Nkv * C;
  float* dvb = d_val + b * Nkv * C;
  for (int k = 0; k < K; ++k) dot[k] = 0.f;
  for (int c = lane; c < C; c += 32) {
    const float g = ldf(dout + r * C + c);
    for (int k = 0; k < K; ++k) {
      const int64_t o = (int64_t)nr[k] * C + c;
      dot[k] = fmaf(ldf(vb + o), g, dot[k]);
      red_add(dvb + o, a * w[k] * g);
    }
  }
  float dattn = 0.f, dnw[KMAX], sw = 0.f;
  for (int k = 0; k < K; ++k) {
    dot[k] = warp_sum(dot[k]);
    dattn = fmaf(w[k], dot[k], dattn);
    dnw[k] = a * dot[k];
    sw = fmaf(dnw[k], w[k], sw);
  }
  if (lane != 0) return;
  d_aw[r] = dattn;
  float dp = 0.f;
  float gs[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k = 0; k < K; ++k) {
    const float dl = w[k] * (dnw[k] - sw);
    dp += dl * (-dist[k]);
    const float dd = -P * dl;
    const float den = fmaxf(dist[k] - 1e-6f, 1e-8f);
    for (int d = 0; d < D; ++d) {
      const float diff = sl[r * D + d] - kvb[(int64_t)nr[k] * D + d];
      const float g = dd * diff / den;
      gs[d] += g;
      red_add(d_kv + b * Nkv * D + (int64_t)nr[k] * D + d, -g);
    }
  }
  for (int d = 0; d < D; ++d) d_sl[r * D + d] = gs[d];
  red_add(d_pow, dp);
}

// ---------------------------------------------------------------- msdetrpc
template <typename T>
__global__ void __launch_bounds__(MW * 32)
msdetrpc_fwd_kernel(const int32_t* __restrict__ idx, const T* __restrict__ w,
                    const T* __restrict__ attn, const T* __restrict__ val, int64_t B, int64_t N,
                    int M, int K, int64_t Nv, int C, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * MW + (threadIdx.x >> 5);
  if (r >= B * N) return;
  const int64_t b = r / N;
  const T* vb = val + b * Nv * C;
  for (int c = lane; c < C; c += 32) {
    float acc = 0.f;
    for (int m = 0; m < M; ++m) {
      const float a = ldf(attn + r * M + m);
      for (int k = 0; k < K; ++k) {
        const int64_t e = (r * M + m) * K + k;
        acc = fmaf(a * ldf(w + e), ldf(vb + (int64_t)idx[e] * C + c), acc);
      }
    }
    stf(out + r * C + c, acc);
  }
}

template <typename T>
__global__ void __launch_bounds__(MW * 32)
msdetrpc_bwd_kernel(const T* __restrict__ dout, const int32_t* __restrict__ idx,
                    const T* __restrict__ w, const T* __restrict__ attn, const T* __restrict__ val,
                    int64_t B, int64_t N, int M, int K, int64_t Nv, int C, T* __restrict__ dw,
                    T* __restrict__ dattn, float* __restrict__ dval) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * MW + (threadIdx.x >> 5);
  if (r >= B * N) return;
  const int64_t b = r / N;
  const T* vb = val + b * Nv * C;
  float* dvb = dval + b * Nv * C;
  for (int m = 0; m < M; ++m) {
    const float a = ldf(attn + r * M + m);
    float da = 0.f;
    for (int k = 0; k < K; ++k) {
      const int64_t e = (r * M + m) * K + k;
      const float wk = ldf(w + e);
      const int64_t row = (int64_t)idx[e] * C;
      float dot = 0.f;
      for (int c = lane; c < C; c += 32) {
        const float g = ldf(dout + r * C + c);
        dot = fmaf(ldf(vb + row + c), g, dot);
        red_add(dvb + row + c, a * wk * g);
      }
      dot = warp_sum(dot);
      if (lane == 0) stf(dw + e, a * dot);
      da = fmaf(wk, dot, da);
    }
    if (lane == 0) stf(dattn + r * M + m, da);
  }
}

// ---------------------------------------------------------------- mssample
__global__ void mssample_fwd_kernel(const float* __restrict__ sl, const float* __restrict__ kv,
                                    const int32_t* __restrict__ nb, const float* __restrict__ power,
                                    int64_t B, int64_t N, int64_t Nkv, int K, int D,
                                    float* __restrict__ wout) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B * N) return;
  const int64_t b = r / N;
  const float P = fmaxf(power[0], 1e-6f);
  float w[KMAX], dist[KMAX];
  shepard_k<1>(sl + r * D, kv + b * Nkv * D, nb + r * K, K, D, P, w, dist);
  for (int k = 0; k < K; ++k) wout[r * K + k] = w[k];
}

__global__ void mssample_bwd_kernel(const float* __restrict__ dw, const float* __restrict__ sl,
                                    const float* __restrict__ kv, const int32_t* __restrict__ nb,
                                    const float* __restrict__ power, const float* __restrict__ wsv,
                                    int64_t B, int64_t N, int64_t Nkv, int K, int D,
                                    float* __restrict__ d_sl, float* __restrict__ d_kv,
                                    float* __restrict__ d_pow) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float dp = 0.f;
  if (r < B * N) {
    const int64_t b = r / N;
    const float P = fmaxf(power[0], 1e-6f);
    const float* kvb = kv + b * Nkv * D;
    float sw = 0.f;
    for (int k = 0; k < K; ++k) sw = fmaf(dw[r * K + k], wsv[r * K + k], sw);
    float gs[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < K; ++k) {
      const int64_t p = (int64_t)nb[r * K + k] * D;
      float d2 = 0.f;
      for (int d = 0; d < D; ++d) {
        const float df = __fsub_rn(sl[r * D + d], kvb[p + d]);
        d2 = __fadd_rn(d2, __fmul_rn(df, df));
      }
      const float dist = sqrtf(d2 + 1e-6f);
      const float dl = wsv[r * K + k] * (dw[r * K + k] - sw);
      dp += dl * (-dist);
      const float dd = dl * (-P);
      for (int d = 0; d < D; ++d) {
        const float diff = sl[r * D + d] - kvb[p + d];
        const float g = dd * diff / (dist + 1e-8f);
        gs[d] += g;
        red_add(d_kv + b * Nkv * D + p + d, -g);
      }
    }
    for (int d = 0; d < D; ++d) d_sl[r * D + d] = gs[d];
  }
  dp = warp_sum(dp);
  if ((threadIdx.x & 31) == 0) red_add(d_pow, dp);
}

// ---------------------------------------------------------------- pos bias
template <typename T>
__global__ void pos_bias_fwd_kernel(const T* __restrict__ table, const int64_t* __restrict__ pe,
                                    int64_t T_, int H, int64_t B, int64_t N, int64_t M,
                                    T* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * N * M) return;
  const int64_t b = t / (N * M), nm = t - b * N * M;
  int64_t e = pe[t];
  if (e < 0 || e >= T_) e = e < 0 ? 0 : T_ - 1;  // out-of-range indices are clamped
  for (int h = 0; h < H; ++h) out[(b * H + h) * N * M + nm] = table[e * H + h];
}

template <typename T>
__global__ void pos_bias_bwd_kernel(const T* __restrict__ dbias, const int64_t* __restrict__ pe,
                                    int64_t T_, int H, int64_t B, int64_t N, int64_t M,
                                    float* __restrict__ dtable) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * N * M) return;
  const int64_t b = t / (N * M), nm = t - b * N * M;
  int64_t e = pe[t];
  if (e < 0 || e >= T_) e = e < 0 ? 0 : T_ - 1;
  for (int h = 0; h < H; ++h) red_add(dtable + e * H + h, ldf(dbias + (b * H + h) * N * M + nm));
}

// The same scatter for the reference's relative-position table (T = 255 x 255,
// index (dy + 127) * 255 + dx + 127): neighbour lists name small offsets, so
// most entries fall in the (2R+1)^2 offsets around the centre and all of a
// block's entries for one offset would otherwise hit the same table row in
// L2.  Each block sums those in shared memory and adds each sum to the table
// once; entries outside the window go straight to global memory.
constexpr int PB_TW = 255, PB_R = 16, PB_WIN = 2 * PB_R + 1;

template <typename T>
__global__ void __launch_bounds__(256) pos_bias_bwd_win_kernel(const T* __restrict__ dbias,
                                                               const int64_t* __restrict__ pe, int64_t T_,
                                                               int H, int64_t B, int64_t N, int64_t M,
                                                               float* __restrict__ dtable) {
  extern __shared__ float pb_acc[];  // [PB_WIN * PB_WIN][H]
  for (int i = threadIdx.x; i < PB_WIN * PB_WIN * H; i += blockDim.x) pb_acc[i] = 0.f;
  __syncthreads();
  const int64_t NM = N * M, tot = B * NM;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < tot; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / NM, nm = t - b * NM;
    int64_t e = pe[t];
    if (e < 0 || e >= T_) e = e < 0 ? 0 : T_ - 1;
    const int dy = (int)(e / PB_TW) - PB_TW / 2, dx = (int)(e % PB_TW) - PB_TW / 2;
    const T* src = dbias + b * H * NM + nm;
    if (dx >= -PB_R && dx <= PB_R && dy >= -PB_R && dy <= PB_R) {
      float* a = pb_acc + ((dy + PB_R) * PB_WIN + dx + PB_R) * H;
      for (int h = 0; h < H; ++h) atomicAdd(a + h, ldf(src + h * NM));
    } else {
      for (int h = 0; h < H; ++h) red_add(dtable + e * H + h, ldf(src + h * NM));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < PB_WIN * PB_WIN * H; i += blockDim.x) {
    const float v = pb_acc[i];
    if (v == 0.f) continue;
    const int slot = i / H, h = i - slot * H;
    const int dy = slot / PB_WIN - PB_R, dx = slot % PB_WIN - PB_R;
    red_add(dtable + ((int64_t)(dy + PB_TW / 2) * PB_TW + dx + PB_TW / 2) * H + h, v);
  }
}

static unsigned rows_blocks(int64_t rows) { return (unsigned)((rows + MW - 1) / MW); }

}  // namespace affb

using namespace affb;

extern "C" int affb_deform_nbidx_fwd(const float* sl, const float* kv_pos, const int32_t* nb_idx,
                                     const float* power, const float* attn_w, const void* values,
                                     int dtype, int64_t B, int64_t N, int64_t Nkv, int64_t K,
                                     int D, int64_t C, void* out, void* stream) {
  AFFB_REQUIRE(K >= 1 && K <= KMAX && D >= 1 && D <= 4 && C >= 0 && B >= 0 && N >= 0,
               "deform_nbidx: need 1 <= K <= %d and 1 <= D <= 4", KMAX);
  if (B * N == 0) return AFFB_OK;
  AFFB_DISPATCH(dtype, T,
                nbidx_fwd_kernel<T><<<rows_blocks(B * N), MW * 32, 0, as_stream(stream)>>>(
                    sl, kv_pos, nb_idx, power, attn_w, (const T*)values, B, N, Nkv, (int)K, D,
                    (int)C, (T*)out));
  AFFB_LAUNCH_CHECK("affb_deform_nbidx_fwd");
  return AFFB_OK;
}

extern "C" int affb_deform_nbidx_bwd(const float* sl, const float* kv_pos, const int32_t* nb_idx,
                                     const float* power, const float* attn_w, const void* values,
                                     const void* dout, int dtype, int64_t B, int64_t N,
                                     int64_t Nkv, int64_t K, int D, int64_t C, float* d_sl,
                                     float* d_kvpos, float* d_power, float* d_attn_w,
                                     float* d_values_acc, void* stream) {
  AFFB_REQUIRE(K >= 1 && K <= KMAX && D >= 1 && D <= 4 && C >= 0 && B >= 0 && N >= 0,
               "deform_nbidx: need 1 <= K <= %d and 1 <= D <= 4", KMAX);
  if (B * N == 0) return AFFB_OK;
  AFFB_DISPATCH(dtype, T,
                nbidx_bwd_kernel<T><<<rows_blocks(B * N), MW * 32, 0, as_stream(stream)>>>(
                    sl, kv_pos, nb_idx, power, attn_w, (const T*)values, (const T*)dout, B, N,
                    Nkv, (int)K, D, (int)C, d_sl, d_kvpos, d_power, d_attn_w, d_values_acc));
  AFFB_LAUNCH_CHECK("affb_deform_nbidx_bwd");
  return AFFB_OK;
}

extern "C" int affb_msdetrpc_fwd(const int32_t* idx, const void* w, const void* attn,
                                 const void* val, int dtype, int64_t B, int64_t N, int64_t M,
                                 int64_t K, int64_t Nv, int64_t C, void* out, void* stream) {
  AFFB_REQUIRE(B >= 0 && N >= 0 && M >= 0 && K >= 0 && C >= 0, "msdetrpc: invalid sizes");
  if (B * N == 0) return AFFB_OK;
  AFFB_DISPATCH(dtype, T,
                msdetrpc_fwd_kernel<T><<<rows_blocks(B * N), MW * 32, 0, as_stream(stream)>>>(
                    idx, (const T*)w, (const T*)attn, (const T*)val, B, N, (int)M, (int)K, Nv,
                    (int)C, (T*)out));
  AFFB_LAUNCH_CHECK("affb_msdetrpc_fwd");
  return AFFB_OK;
}

extern "C" int affb_msdetrpc_bwd(const void* dout, const int32_t* idx, const void* w,
                                 const void* attn, const void* val, int dtype, int64_t B,
                                 int64_t N, int64_t M, int64_t K, int64_t Nv, int64_t C, void* dw,
                                 void* dattn, float* dval_acc, void* stream) {
  AFFB_REQUIRE(B >= 0 && N >= 0 && M >= 0 && K >= 0 && C >= 0, "msdetrpc: invalid sizes");
  if (B * N == 0) return AFFB_OK;
  AFFB_DISPATCH(dtype, T,
                msdetrpc_bwd_kernel<T><<<rows_blocks(B * N), MW * 32, 0, as_stream(stream)>>>(
                    (const T*)dout, idx, (const T*)w, (const T*)attn, (const T*)val, B, N, (int)M,
                    (int)K, Nv, (int)C, (T*)dw, (T*)dattn, dval_acc));
  AFFB_LAUNCH_CHECK("affb_msdetrpc_bwd");
  return AFFB_OK;
}

extern "C" int affb_mssample_fwd(const float* sl, const float* kv_pos, const int32_t* nb_idx,
                                 const float* power, int64_t B, int64_t N, int64_t Nkv, int64_t K,
                                 int D, float* w_out, void* stream) {
  AFFB_REQUIRE(K >= 1 && K <= KMAX && D >= 1 && D <= 4,
               "mssample: need 1 <= K <= %d and 1 <= D <= 4", KMAX);
  if (B * N == 0) return AFFB_OK;
  mssample_fwd_kernel<<<(unsigned)((B * N + 255) / 256), 256, 0, as_stream(stream)>>>(
      sl, kv_pos, nb_idx, power, B, N, Nkv, (int)K, D, w_out);
  AFFB_LAUNCH_CHECK("affb_mssample_fwd");
  return AFFB_OK;
}

extern "C" int affb_mssample_bwd(const float* dw, const float* sl, const float* kv_pos,
                                 const int32_t* nb_idx, const float* power, const float* w,
                                 int64_t B, int64_t N, int64_t Nkv, int64_t K, int D, float* d_sl,
                                 float* d_kvpos, float* d_power, void* stream) {
  AFFB_REQUIRE(K >= 1 && K <= KMAX && D >= 1 && D <= 4,
               "mssample: need 1 <= K <= %d and 1 <= D <= 4", KMAX);
  if (B * N == 0) return AFFB_OK;
  mssample_bwd_kernel<<<(unsigned)((B * N + 255) / 256), 256, 0, as_stream(stream)>>>(
      dw, sl, kv_pos, nb_idx, power, w, B, N, Nkv, (int)K, D, d_sl, d_kvpos, d_power);
  AFFB_LAUNCH_CHECK("affb_mssample_bwd");
  return AFFB_OK;
}

extern "C" int affb_pos_bias_fwd(const void* table, const int64_t* pe_idx, int dtype, int64_t T,
                                 int64_t H, int64_t B, int64_t N, int64_t M, void* out,
                                 void* stream) {
  AFFB_REQUIRE(T >= 1 && H >= 1 && B >= 0 && N >= 0 && M >= 0, "pos_bias: invalid sizes");
  const int64_t tot = B * N * M;
  if (tot == 0) return AFFB_OK;
  AFFB_DISPATCH(dtype, Tp,
                pos_bias_fwd_kernel<Tp><<<(unsigned)((tot + 255) / 256), 256, 0, as_stream(stream)>>>(
                    (const Tp*)table, pe_idx, T, (int)H, B, N, M, (Tp*)out));
  AFFB_LAUNCH_CHECK("affb_pos_bias_fwd");
  return AFFB_OK;
}

extern "C" int affb_pos_bias_bwd(const void* dbias, const int64_t* pe_idx, int dtype, int64_t T,
                                 int64_t H, int64_t B, int64_t N, int64_t M, float* dtable_acc,
                                 void* stream) {
  AFFB_REQUIRE(T >= 1 && H >= 1 && B >= 0 && N >= 0 && M >= 0, "pos_bias: invalid sizes");
  const int64_t tot = B * N * M;
  if (tot == 0) return AFFB_OK;
  if (T == (int64_t)PB_TW * PB_TW && H <= 8) {
    const unsigned blocks = (unsigned)imin64((tot + 255) / 256, (int64_t)sm_count() * 8);
    const size_t smem = (size_t)PB_WIN * PB_WIN * H * sizeof(float);
    AFFB_DISPATCH(dtype, Tp,
                  pos_bias_bwd_win_kernel<Tp><<<blocks, 256, smem, as_stream(stream)>>>(
                      (const Tp*)dbias, pe_idx, T, (int)H, B, N, M, dtable_acc));
  } else {
    AFFB_DISPATCH(dtype, Tp,
                  pos_bias_bwd_kernel<Tp><<<(unsigned)((tot + 255) / 256), 256, 0, as_stream(stream)>>>(
                      (const Tp*)dbias, pe_idx, T, (int)H, B, N, M, dtable_acc));
  }
  AFFB_LAUNCH_CHECK("affb_pos_bias_bwd");
  return AFFB_OK;
}
