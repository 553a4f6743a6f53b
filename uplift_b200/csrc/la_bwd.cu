// Backward of the fused Local Attender (training), CUDA cores, sm_100a.
//
// Forward (uplift/uplift.py:801-847): per output pixel p of cell c,
//   l_k = sum_c' W'[k][c'] g[p][c'] + b_k    (W' = W + residual identity)
//   P   = softmax_k(l)                         (one-hot of argmax: hardmax)
//   out[p][ch] = sum_k P_k V[n_k(c)][ch]       (n_k: replicate-clamped offset)
// Backward, given dout:
//   dP_k   = sum_ch dout[p][ch] V[n_k][ch]
//   dl_k   = P_k (dP_k - sum_j P_j dP_j)        (0 for hardmax)
//   dg[p]  = sum_k dl_k W'[k]                   dW[k] += sum_p dl_k g[p]
//   db_k  += sum_p dl_k
//   dV[n][ch] = sum over (p, k) with n_k(p) = n of P_k(p) dout[p][ch]
// Three launches: the softmax weights are recomputed into a caller-provided
// fp32 workspace [B, Ho, Wo, K] (probs_kernel); dlogit_kernel (one thread
// per output pixel, 128 per CTA) forms dP, dl and dg and reduces dW / db
// over its tile in shared memory before one atomic add per entry; and
// dvalue_kernel gathers dV per value pixel (one CTA per value row) by
// enumerating, for every offset, the cells whose clamped neighbour is that
// pixel -- no atomics on the large tensors.  fp32 arithmetic throughout.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>

#include "uplift_la.h"
#include "la_internal.h"

namespace ula {
namespace bwd {

constexpr int kPix = 128;       // output pixels per dlogit CTA (one thread each)
constexpr int kThreads = 256;   // probs / dvalue CTAs
constexpr int kGChunk = 32;     // guide channels staged per dW step
constexpr int kMaxK = UPLIFT_LA_MAX_K;

__device__ __forceinline__ float tof(float x) { return x; }
__device__ __forceinline__ float tof(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float tof(__half x) { return __half2float(x); }
template <typename T> __device__ __forceinline__ T fromf(float x);
template <> __device__ __forceinline__ float fromf<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 fromf<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half fromf<__half>(float x) { return __float2half_rn(x); }

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return min(max(v, lo), hi); }

struct Args {
  const void* dout;   int64_t d_b, d_h, d_w;
  const void* guide;  int64_t g_b, g_h, g_w;
  const void* value;  int64_t v_b, v_h, v_w;
  const float* weight;  // [K][Cg]
  const float* bias;    // [K] or null
  float* probs;         // [B][Ho][Wo][K], dense
  void* dguide;       int64_t dg_b, dg_h, dg_w;
  void* dvalue;       int64_t dv_b, dv_h, dv_w;
  float* dweight;       // [K][Cg], accumulated
  float* dbias;         // [K], accumulated
  int B, Cg, C, H, W, I, Ho, Wo;
  int conv_res, hardmax;
  int8_t dy[kMaxK];
  int8_t dx[kMaxK];
};

// W'[k][c] = W[k][c] (+1 on the residual diagonal) as [Cg][K] in shared memory.
template <int K>
__device__ __forceinline__ void stage_weights(const Args& a, float* s_w, int nthreads) {
  for (int i = threadIdx.x; i < a.Cg * K; i += nthreads) {
    const int c = i / K, k = i - c * K;
    s_w[i] = a.weight[(size_t)k * a.Cg + c] + ((a.conv_res && k == c) ? 1.f : 0.f);
  }
}

template <typename T, int K>
__global__ void __launch_bounds__(kThreads) probs_kernel(const Args a) {
  extern __shared__ float s_w[];  // [Cg][K]
  stage_weights<K>(a, s_w, kThreads);
  __syncthreads();
  const T* __restrict__ guide = static_cast<const T*>(a.guide);
  const int64_t npix = (int64_t)a.B * a.Ho * a.Wo;
  for (int64_t p = (int64_t)blockIdx.x * kThreads + threadIdx.x; p < npix; p += (int64_t)gridDim.x * kThreads) {
    const int x = (int)(p % a.Wo);
    const int64_t r = p / a.Wo;
    const int y = (int)(r % a.Ho);
    const int b = (int)(r / a.Ho);
    const T* gp = guide + b * a.g_b + y * a.g_h + x * a.g_w;
    float l[K];
#pragma unroll
    for (int k = 0; k < K; ++k) l[k] = a.bias != nullptr ? a.bias[k] : 0.f;
    for (int c = 0; c < a.Cg; ++c) {
      const float g = tof(gp[c]);
#pragma unroll
      for (int k = 0; k < K; ++k) l[k] = fmaf(s_w[c * K + k], g, l[k]);
    }
    float* pp = a.probs + p * K;
    if (a.hardmax) {
      int best = 0;
      float bv = l[0];
#pragma unroll
      for (int k = 1; k < K; ++k)
        if (l[k] > bv) { bv = l[k]; best = k; }
#pragma unroll
      for (int k = 0; k < K; ++k) pp[k] = (k == best) ? 1.f : 0.f;
    } else {
      float m = l[0];
#pragma unroll
      for (int k = 1; k < K; ++k) m = fmaxf(m, l[k]);
      float z = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) { l[k] = __expf(l[k] - m); z += l[k]; }
      const float inv = 1.f / z;
#pragma unroll
      for (int k = 0; k < K; ++k) pp[k] = l[k] * inv;
    }
  }
}

template <typename T, int K>
__global__ void __launch_bounds__(kPix) dlogit_kernel(const Args a) {
  extern __shared__ float smem[];
  float* s_w = smem;                         // [Cg][K]
  float* s_dl = s_w + a.Cg * K;              // [kPix][K]
  float* s_g = s_dl + kPix * K;              // [kPix][kGChunk]
  stage_weights<K>(a, s_w, kPix);
  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  const T* __restrict__ guide = static_cast<const T*>(a.guide);
  const T* __restrict__ value = static_cast<const T*>(a.value);
  const int64_t npix = (int64_t)a.B * a.Ho * a.Wo;
  const int64_t p = (int64_t)blockIdx.x * kPix + threadIdx.x;
  const bool valid = p < npix;
  int b = 0, y = 0, x = 0;
  if (valid) {
    x = (int)(p % a.Wo);
    const int64_t r = p / a.Wo;
    y = (int)(r % a.Ho);
    b = (int)(r / a.Ho);
  }
  float dl[K];
#pragma unroll
  for (int k = 0; k < K; ++k) dl[k] = 0.f;
  if (valid && !a.hardmax) {
    const int cy = y / a.I, cx = x / a.I;
    const T* dp = dout + b * a.d_b + y * a.d_h + x * a.d_w;
    const T* vb = value + b * a.v_b;
    int64_t nb[K];
#pragma unroll
    for (int k = 0; k < K; ++k)
      nb[k] = clampi(cy + a.dy[k], 0, a.H - 1) * a.v_h + clampi(cx + a.dx[k], 0, a.W - 1) * a.v_w;
    float dP[K];
#pragma unroll
    for (int k = 0; k < K; ++k) dP[k] = 0.f;
    for (int ch = 0; ch < a.C; ++ch) {
      const float d = tof(dp[ch]);
#pragma unroll
      for (int k = 0; k < K; ++k) dP[k] = fmaf(d, tof(vb[nb[k] + ch]), dP[k]);
    }
    const float* pp = a.probs + p * K;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) s = fmaf(pp[k], dP[k], s);
#pragma unroll
    for (int k = 0; k < K; ++k) dl[k] = pp[k] * (dP[k] - s);
  }
#pragma unroll
  for (int k = 0; k < K; ++k) s_dl[threadIdx.x * K + k] = dl[k];
  __syncthreads();  // s_w staged, s_dl complete
  if (valid && a.dguide != nullptr) {
    T* gp = static_cast<T*>(a.dguide) + b * a.dg_b + y * a.dg_h + x * a.dg_w;
    for (int c = 0; c < a.Cg; ++c) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) acc = fmaf(dl[k], s_w[c * K + k], acc);
      gp[c] = fromf<T>(acc);
    }
  }
  if (a.hardmax || (a.dweight == nullptr && a.dbias == nullptr)) return;
  // dW / db over this tile: guide chunks of kGChunk channels through s_g
  const int64_t p0 = (int64_t)blockIdx.x * kPix;
  const int tile = npix - p0 < kPix ? (int)(npix - p0) : kPix;
  if (a.dbias != nullptr && threadIdx.x < K) {
    float acc = 0.f;
    for (int t = 0; t < tile; ++t) acc += s_dl[t * K + threadIdx.x];
    atomicAdd(a.dbias + threadIdx.x, acc);
  }
  if (a.dweight == nullptr) return;
  for (int c0 = 0; c0 < a.Cg; c0 += kGChunk) {
    const int cn = min(kGChunk, a.Cg - c0);
    __syncthreads();  // previous chunk consumed
    if (valid) {
      const T* gp = guide + b * a.g_b + y * a.g_h + x * a.g_w + c0;
      for (int j = 0; j < cn; ++j) s_g[threadIdx.x * kGChunk + j] = tof(gp[j]);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < K * cn; i += kPix) {
      const int k = i / cn, j = i - k * cn;
      float acc = 0.f;
      for (int t = 0; t < tile; ++t) acc = fmaf(s_dl[t * K + k], s_g[t * kGChunk + j], acc);
      atomicAdd(a.dweight + (size_t)k * a.Cg + c0 + j, acc);
    }
  }
}

// Cells c whose clamped neighbour clamp(c + d) is n along one axis of
// length n_len: [lo, hi] (empty when lo > hi).
__device__ __forceinline__ void cell_range(int n, int d, int n_len, int& lo, int& hi) {
  lo = (n == 0) ? 0 : n - d;
  hi = (n == n_len - 1) ? n_len - 1 : n - d;
  lo = max(lo, 0);
  hi = min(hi, n_len - 1);
}

template <typename T, int K>
__global__ void __launch_bounds__(kThreads) dvalue_kernel(const Args a) {
  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  T* __restrict__ dv = static_cast<T*>(a.dvalue);
  const int row = blockIdx.x;  // (b, ny)
  const int ny = row % a.H, b = row / a.H;
  const int items = a.W * a.C;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    const int nx = i / a.C, ch = i - nx * a.C;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      int ylo, yhi, xlo, xhi;
      cell_range(ny, a.dy[k], a.H, ylo, yhi);
      cell_range(nx, a.dx[k], a.W, xlo, xhi);
      for (int cy = ylo; cy <= yhi; ++cy)
        for (int cx = xlo; cx <= xhi; ++cx)
          for (int iy = 0; iy < a.I; ++iy)
            for (int ix = 0; ix < a.I; ++ix) {
              const int y = cy * a.I + iy, x = cx * a.I + ix;
              const float pk = a.probs[(((int64_t)b * a.Ho + y) * a.Wo + x) * K + k];
              if (pk != 0.f) acc = fmaf(pk, tof(dout[b * a.d_b + y * a.d_h + x * a.d_w + ch]), acc);
            }
    }
    dv[b * a.dv_b + ny * a.dv_h + nx * a.dv_w + ch] = fromf<T>(acc);
  }
}

template <typename T, int K>
int launch(const Args& a, cudaStream_t stream) {
  const int64_t npix = (int64_t)a.B * a.Ho * a.Wo;
  if (npix == 0) return UPLIFT_LA_OK;
  const size_t smem_p = sizeof(float) * (size_t)a.Cg * K;
  const size_t smem_d = sizeof(float) * ((size_t)a.Cg * K + (size_t)kPix * K + (size_t)kPix * kGChunk);
  int dev = 0, optin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return fail(UPLIFT_LA_ERR_CUDA, "device query failed");
  if (smem_d > (size_t)optin) return fail(UPLIFT_LA_ERR_SHAPE, "backward: Cg=%d needs too much shared memory", a.Cg);
  cudaError_t e = cudaFuncSetAttribute(probs_kernel<T, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_p);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(dlogit_kernel<T, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_d);
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const int64_t pblocks = std::min<int64_t>((npix + kThreads - 1) / kThreads, 148ll * 16);
  probs_kernel<T, K><<<(unsigned)pblocks, kThreads, smem_p, stream>>>(a);
  const int64_t dblocks = (npix + kPix - 1) / kPix;
  if (dblocks >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "backward: too many pixels");
  if (a.dguide != nullptr || a.dweight != nullptr || a.dbias != nullptr)
    dlogit_kernel<T, K><<<(unsigned)dblocks, kPix, smem_d, stream>>>(a);
  if (a.dvalue != nullptr && a.B * (int64_t)a.H > 0)
    dvalue_kernel<T, K><<<(unsigned)(a.B * (int64_t)a.H), kThreads, 0, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "backward launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

template <typename T>
int launch_k(const Args& a, int K, cudaStream_t stream) {
  switch (K) {
    case 5: return launch<T, 5>(a, stream);
    case 9: return launch<T, 9>(a, stream);
    case 13: return launch<T, 13>(a, stream);
    case 17: return launch<T, 17>(a, stream);
    case 25: return launch<T, 25>(a, stream);
    default: return fail(UPLIFT_LA_ERR_SHAPE, "backward: K=%d unsupported (5, 9, 13, 17, 25)", K);
  }
}

}  // namespace bwd
}  // namespace ula

extern "C" int uplift_la_backward(const void* dout, const int64_t dout_strides[4],
                                  const void* guide, const int64_t guide_strides[4],
                                  const void* value, const int64_t value_strides[4],
                                  const float* weight, const float* bias,
                                  float* probs,
                                  void* dguide, const int64_t dguide_strides[4],
                                  void* dvalue, const int64_t dvalue_strides[4],
                                  float* dweight, float* dbias,
                                  int B, int Cg, int C, int H, int W, int I, int K,
                                  const int8_t* offsets, int pn, int conv_res, int dtype, int hardmax,
                                  void* stream) {
  using namespace ula;
  using ula::bwd::Args;
  if (dtype != UPLIFT_LA_F32 && dtype != UPLIFT_LA_BF16 && dtype != UPLIFT_LA_F16)
    return fail(UPLIFT_LA_ERR_ARG, "unknown dtype %d", dtype);
  if (B < 0 || Cg < 1 || C < 1 || H < 0 || W < 0 || I < 1)
    return fail(UPLIFT_LA_ERR_SHAPE, "bad sizes B=%d Cg=%d C=%d H=%d W=%d I=%d", B, Cg, C, H, W, I);
  if (K < 1 || K > UPLIFT_LA_MAX_K) return fail(UPLIFT_LA_ERR_SHAPE, "K=%d out of range", K);
  if (pn < 0 || pn > UPLIFT_LA_MAX_PN) return fail(UPLIFT_LA_ERR_OFFSETS, "pn=%d out of range", pn);
  if (offsets == nullptr || dout_strides == nullptr || guide_strides == nullptr || value_strides == nullptr)
    return fail(UPLIFT_LA_ERR_ARG, "null offsets or strides");
  if ((dguide != nullptr && dguide_strides == nullptr) || (dvalue != nullptr && dvalue_strides == nullptr))
    return fail(UPLIFT_LA_ERR_ARG, "null gradient strides");
  const int64_t npix = (int64_t)B * I * H * I * W;
  if (npix > 0 && (dout == nullptr || guide == nullptr || value == nullptr || weight == nullptr || probs == nullptr))
    return fail(UPLIFT_LA_ERR_ARG, "null input pointer");
  if (npix >= ((int64_t)1 << 40)) return fail(UPLIFT_LA_ERR_SHAPE, "too many pixels");
  Args a;
  memset(&a, 0, sizeof(a));
  for (int k = 0; k < K; ++k) {
    const int dy = offsets[2 * k], dx = offsets[2 * k + 1];
    if (dy < -pn || dy > pn || dx < -pn || dx > pn)
      return fail(UPLIFT_LA_ERR_OFFSETS, "offset %d = (%d, %d) exceeds pn=%d", k, dy, dx, pn);
    a.dy[k] = (int8_t)dy;
    a.dx[k] = (int8_t)dx;
  }
  const int64_t* st[5] = {dout_strides, guide_strides, value_strides, dguide_strides, dvalue_strides};
  for (int i = 0; i < 5; ++i)
    if (st[i] != nullptr && st[i][1] != 1 && !(i == 1 || i == 3 ? Cg == 1 : C == 1))
      return fail(UPLIFT_LA_ERR_LAYOUT, "tensors need channel stride 1 (channels_last)");
  a.dout = dout; a.d_b = dout_strides[0]; a.d_h = dout_strides[2]; a.d_w = dout_strides[3];
  a.guide = guide; a.g_b = guide_strides[0]; a.g_h = guide_strides[2]; a.g_w = guide_strides[3];
  a.value = value; a.v_b = value_strides[0]; a.v_h = value_strides[2]; a.v_w = value_strides[3];
  a.weight = weight; a.bias = bias; a.probs = probs;
  a.dguide = dguide;
  if (dguide != nullptr) { a.dg_b = dguide_strides[0]; a.dg_h = dguide_strides[2]; a.dg_w = dguide_strides[3]; }
  a.dvalue = dvalue;
  if (dvalue != nullptr) { a.dv_b = dvalue_strides[0]; a.dv_h = dvalue_strides[2]; a.dv_w = dvalue_strides[3]; }
  a.dweight = dweight; a.dbias = dbias;
  a.B = B; a.Cg = Cg; a.C = C; a.H = H; a.W = W; a.I = I; a.Ho = I * H; a.Wo = I * W;
  a.conv_res = conv_res ? 1 : 0;
  a.hardmax = hardmax ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case UPLIFT_LA_F32: return bwd::launch_k<float>(a, K, s);
    case UPLIFT_LA_BF16: return bwd::launch_k<__nv_bfloat16>(a, K, s);
    default: return bwd::launch_k<__half>(a, K, s);
  }
}
