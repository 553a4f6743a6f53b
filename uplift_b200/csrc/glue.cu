// Resampling and residual kernels around the Local Attender in the UPLiFT
// upsampler's fast mode (C ABI in include/uplift_glue.h).
//
// All three are streaming, HBM-bound NHWC kernels: a thread owns one output
// pixel x one 16-byte channel vector (8 bf16/fp16 or 4 fp32; one element
// when the channel count or alignment does not allow vectors), so a warp
// reads and writes whole contiguous channel runs.  Arithmetic in fp32 with
// a single rounding per result, and source indices computed with PyTorch's
// formulas for F.interpolate, so the results match the eager ops they
// replace:
//   bilinear, align_corners = 0: s = max((d + 0.5) * in / out - 0.5, 0)
//   bilinear, align_corners = 1: s = d * (in - 1) / (out - 1)
//   i0 = (int)s, i1 = i0 + (i0 < in - 1), l1 = s - i0, l0 = 1 - l1
//   out = l0y * (l0x * a + l1x * b) + l1y * (l0x * c + l1x * d)
//   nearest: s = min(floor(d * (in / out)), in - 1)
// References: F.interpolate in uplift/fast.py:219, :229,
// UpsamplingBilinear2d in uplift/uplift.py:228, :335, TVF.resize NEAREST in
// uplift/uplift.py:359, residual_auto in uplift/uplift.py:26-39.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "uplift_glue.h"
#include "la_internal.h"

namespace ula {
namespace glue {

constexpr int kThreads = 256;

template <typename T> struct St;
template <> struct St<float> {
  __device__ __forceinline__ static float f(float x) { return x; }
  __device__ __forceinline__ static float t(float x) { return x; }
};
template <> struct St<__nv_bfloat16> {
  __device__ __forceinline__ static float f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 t(float x) { return __float2bfloat16_rn(x); }
};
template <> struct St<__half> {
  __device__ __forceinline__ static float f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half t(float x) { return __float2half_rn(x); }
};

// VEC consecutive elements, loaded / stored as one 16-byte access when VEC > 1.
template <typename T, int VEC>
struct Vec {
  T e[VEC];
  __device__ __forceinline__ void load(const T* p) {
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(e) = __ldg(reinterpret_cast<const uint4*>(p));
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) e[i] = p[i];
    }
  }
  __device__ __forceinline__ void store(T* p) const {
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(e);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) p[i] = e[i];
    }
  }
};

struct Map {
  const void* src; int64_t s_b, s_h, s_w;
  void* dst;       int64_t d_b, d_h, d_w;
  int C, Hi, Wi, Ho, Wo;
  float scale_h, scale_w;
  int64_t total;  // output pixels x channel vectors
};

// One bilinear source coordinate (PyTorch's area_pixel_compute_source_index).
template <bool ALIGN>
__device__ __forceinline__ void src_coord(int d, float scale, int in, int& i0, int& ip, float& l0, float& l1) {
  float s = ALIGN ? scale * (float)d : scale * ((float)d + 0.5f) - 0.5f;
  if (!ALIGN && s < 0.f) s = 0.f;
  i0 = (int)s;
  ip = (i0 < in - 1) ? 1 : 0;
  l1 = s - (float)i0;
  l0 = 1.f - l1;
}

template <typename T, int VEC, bool ALIGN, bool ACC>
__global__ void __launch_bounds__(kThreads) bilinear_kernel(const Map m) {
  const T* __restrict__ src = static_cast<const T*>(m.src);
  T* __restrict__ dst = static_cast<T*>(m.dst);
  const int nv = m.C / VEC;
  for (int64_t idx = (int64_t)blockIdx.x * kThreads + threadIdx.x; idx < m.total;
       idx += (int64_t)gridDim.x * kThreads) {
    const int v = (int)(idx % nv);
    const int64_t pix = idx / nv;
    const int ox = (int)(pix % m.Wo);
    const int64_t r = pix / m.Wo;
    const int oy = (int)(r % m.Ho);
    const int b = (int)(r / m.Ho);
    int y0, yp, x0, xp;
    float ly0, ly1, lx0, lx1;
    src_coord<ALIGN>(oy, m.scale_h, m.Hi, y0, yp, ly0, ly1);
    src_coord<ALIGN>(ox, m.scale_w, m.Wi, x0, xp, lx0, lx1);
    const T* base = src + b * m.s_b + (int64_t)v * VEC;
    Vec<T, VEC> a, bb, c, d;
    a.load(base + y0 * m.s_h + x0 * m.s_w);
    bb.load(base + y0 * m.s_h + (x0 + xp) * m.s_w);
    c.load(base + (y0 + yp) * m.s_h + x0 * m.s_w);
    d.load(base + (y0 + yp) * m.s_h + (x0 + xp) * m.s_w);
    T* out = dst + b * m.d_b + oy * m.d_h + ox * m.d_w + (int64_t)v * VEC;
    Vec<T, VEC> o;
    if constexpr (ACC) o.load(out);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float val = ly0 * (lx0 * St<T>::f(a.e[e]) + lx1 * St<T>::f(bb.e[e])) +
                        ly1 * (lx0 * St<T>::f(c.e[e]) + lx1 * St<T>::f(d.e[e]));
      // accumulate: the resized value is rounded first, as a separate
      // resize followed by an add would round it
      o.e[e] = ACC ? St<T>::t(St<T>::f(o.e[e]) + St<T>::f(St<T>::t(val))) : St<T>::t(val);
    }
    o.store(out);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads) nearest_kernel(const Map m) {
  const T* __restrict__ src = static_cast<const T*>(m.src);
  T* __restrict__ dst = static_cast<T*>(m.dst);
  const int nv = m.C / VEC;
  for (int64_t idx = (int64_t)blockIdx.x * kThreads + threadIdx.x; idx < m.total;
       idx += (int64_t)gridDim.x * kThreads) {
    const int v = (int)(idx % nv);
    const int64_t pix = idx / nv;
    const int ox = (int)(pix % m.Wo);
    const int64_t r = pix / m.Wo;
    const int oy = (int)(r % m.Ho);
    const int b = (int)(r / m.Ho);
    const int sy = min((int)floorf((float)oy * m.scale_h), m.Hi - 1);
    const int sx = min((int)floorf((float)ox * m.scale_w), m.Wi - 1);
    Vec<T, VEC> a;
    a.load(src + b * m.s_b + sy * m.s_h + sx * m.s_w + (int64_t)v * VEC);
    a.store(dst + b * m.d_b + oy * m.d_h + ox * m.d_w + (int64_t)v * VEC);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads) add_kernel(const Map m) {
  const T* __restrict__ src = static_cast<const T*>(m.src);
  T* __restrict__ dst = static_cast<T*>(m.dst);
  const int nv = m.C / VEC;
  for (int64_t idx = (int64_t)blockIdx.x * kThreads + threadIdx.x; idx < m.total;
       idx += (int64_t)gridDim.x * kThreads) {
    const int v = (int)(idx % nv);
    const int64_t pix = idx / nv;
    const int x = (int)(pix % m.Wo);
    const int64_t r = pix / m.Wo;
    const int y = (int)(r % m.Ho);
    const int b = (int)(r / m.Ho);
    Vec<T, VEC> a, o;
    a.load(src + b * m.s_b + y * m.s_h + x * m.s_w + (int64_t)v * VEC);
    T* out = dst + b * m.d_b + y * m.d_h + x * m.d_w + (int64_t)v * VEC;
    o.load(out);
#pragma unroll
    for (int e = 0; e < VEC; ++e) o.e[e] = St<T>::t(St<T>::f(o.e[e]) + St<T>::f(a.e[e]));
    o.store(out);
  }
}

struct Epi {
  void* dst; int64_t d_b, d_h, d_w;
  const void* bias;
  const void* res; int64_t r_b, r_h, r_w;
  int res_c, C, H, W;
  int64_t total;
};

template <typename T, int VEC, bool RELU>
__global__ void __launch_bounds__(kThreads) bias_act_kernel(const Epi m) {
  T* __restrict__ dst = static_cast<T*>(m.dst);
  const T* __restrict__ bias = static_cast<const T*>(m.bias);
  const T* __restrict__ res = static_cast<const T*>(m.res);
  const int nv = m.C / VEC;
  for (int64_t idx = (int64_t)blockIdx.x * kThreads + threadIdx.x; idx < m.total;
       idx += (int64_t)gridDim.x * kThreads) {
    const int v = (int)(idx % nv);
    const int64_t pix = idx / nv;
    const int x = (int)(pix % m.W);
    const int64_t r = pix / m.W;
    const int y = (int)(r % m.H);
    const int b = (int)(r / m.H);
    const int c0 = v * VEC;
    T* out = dst + b * m.d_b + y * m.d_h + x * m.d_w + c0;
    Vec<T, VEC> o, bv, rv;
    o.load(out);
    if (bias != nullptr) bv.load(bias + c0);
    const bool has_res = res != nullptr && c0 < m.res_c;  // res_c is a multiple of VEC
    if (has_res) rv.load(res + b * m.r_b + y * m.r_h + x * m.r_w + c0);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      float t = St<T>::f(o.e[e]);
      if (bias != nullptr) t = St<T>::f(St<T>::t(t + St<T>::f(bv.e[e])));
      if (RELU) t = fmaxf(t, 0.f);
      if (has_res) t = t + St<T>::f(rv.e[e]);
      o.e[e] = St<T>::t(t);
    }
    o.store(out);
  }
}

template <typename T>
int launch_epi(const Epi& m0, bool vec, bool relu, cudaStream_t stream);

enum class Op { kBilinear, kNearest, kAdd };

int sm_count() {
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    sms[dev] = n;
  }
  return sms[dev];
}

template <typename T, int VEC>
int launch_t(Op op, const Map& m0, bool align, bool acc, cudaStream_t stream) {
  Map m = m0;
  m.total = (int64_t)(m.C / VEC) * m.Ho * m.Wo * (m.total /* batch */);
  if (m.total == 0) return UPLIFT_LA_OK;
  const int64_t blocks = std::min<int64_t>((m.total + kThreads - 1) / kThreads, (int64_t)sm_count() * 16);
  const dim3 grid((unsigned)blocks);
  switch (op) {
    case Op::kBilinear:
      if (align) {
        if (acc) bilinear_kernel<T, VEC, true, true><<<grid, kThreads, 0, stream>>>(m);
        else bilinear_kernel<T, VEC, true, false><<<grid, kThreads, 0, stream>>>(m);
      } else {
        if (acc) bilinear_kernel<T, VEC, false, true><<<grid, kThreads, 0, stream>>>(m);
        else bilinear_kernel<T, VEC, false, false><<<grid, kThreads, 0, stream>>>(m);
      }
      break;
    case Op::kNearest: nearest_kernel<T, VEC><<<grid, kThreads, 0, stream>>>(m); break;
    case Op::kAdd: add_kernel<T, VEC><<<grid, kThreads, 0, stream>>>(m); break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "glue kernel launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

template <typename T>
int launch_v(Op op, const Map& m, bool vec, bool align, bool acc, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  return vec ? launch_t<T, V>(op, m, align, acc, stream) : launch_t<T, 1>(op, m, align, acc, stream);
}

// Validation shared by the three entry points; fills `m` (m.total = B).
int prepare(const char* what, const void* src, const int64_t* ss, const void* dst, const int64_t* ds,
            int B, int C, int Hi, int Wi, int Ho, int Wo, int dtype, Map* m, bool* vec) {
  if (dtype != UPLIFT_LA_F32 && dtype != UPLIFT_LA_BF16 && dtype != UPLIFT_LA_F16)
    return fail(UPLIFT_LA_ERR_ARG, "%s: unknown dtype %d", what, dtype);
  if (ss == nullptr || ds == nullptr) return fail(UPLIFT_LA_ERR_ARG, "%s: null strides", what);
  if (B < 0 || C < 0 || Hi < 0 || Wi < 0 || Ho < 0 || Wo < 0)
    return fail(UPLIFT_LA_ERR_SHAPE, "%s: negative size", what);
  const bool empty = (int64_t)B * C * Ho * Wo == 0;
  if (!empty && (Hi == 0 || Wi == 0)) return fail(UPLIFT_LA_ERR_SHAPE, "%s: empty source", what);
  if (!empty && (src == nullptr || dst == nullptr)) return fail(UPLIFT_LA_ERR_ARG, "%s: null pointer", what);
  if ((C > 1 && ss[1] != 1) || (C > 1 && ds[1] != 1))
    return fail(UPLIFT_LA_ERR_LAYOUT, "%s: channel stride must be 1 (channels_last)", what);
  for (int i = 0; i < 4; ++i)
    if (ss[i] < 0 || ds[i] < 0) return fail(UPLIFT_LA_ERR_LAYOUT, "%s: negative stride", what);
  const int es = dtype == UPLIFT_LA_F32 ? 4 : 2;
  const int ve = 16 / es;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  *vec = C % ve == 0 && a16(src) && a16(dst) && ss[0] % ve == 0 && ss[2] % ve == 0 && ss[3] % ve == 0 &&
         ds[0] % ve == 0 && ds[2] % ve == 0 && ds[3] % ve == 0;
  m->src = src; m->s_b = ss[0]; m->s_h = ss[2]; m->s_w = ss[3];
  m->dst = const_cast<void*>(dst); m->d_b = ds[0]; m->d_h = ds[2]; m->d_w = ds[3];
  m->C = C; m->Hi = Hi; m->Wi = Wi; m->Ho = Ho; m->Wo = Wo;
  m->total = empty ? 0 : B;
  return UPLIFT_LA_OK;
}

template <typename T>
int launch_epi(const Epi& m0, bool vec, bool relu, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  Epi m = m0;
  const int ve = vec ? V : 1;
  m.total = (int64_t)(m.C / ve) * m.H * m.W * m.total;
  if (m.total == 0) return UPLIFT_LA_OK;
  const int64_t blocks = std::min<int64_t>((m.total + kThreads - 1) / kThreads, (int64_t)sm_count() * 16);
  const dim3 grid((unsigned)blocks);
  if (vec) {
    if (relu) bias_act_kernel<T, V, true><<<grid, kThreads, 0, stream>>>(m);
    else bias_act_kernel<T, V, false><<<grid, kThreads, 0, stream>>>(m);
  } else {
    if (relu) bias_act_kernel<T, 1, true><<<grid, kThreads, 0, stream>>>(m);
    else bias_act_kernel<T, 1, false><<<grid, kThreads, 0, stream>>>(m);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "glue kernel launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

int dispatch(Op op, const Map& m, int dtype, bool vec, bool align, bool acc, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case UPLIFT_LA_F32: return launch_v<float>(op, m, vec, align, acc, s);
    case UPLIFT_LA_BF16: return launch_v<__nv_bfloat16>(op, m, vec, align, acc, s);
    default: return launch_v<__half>(op, m, vec, align, acc, s);
  }
}

}  // namespace glue
}  // namespace ula

extern "C" {

int uplift_resize_bilinear(const void* src, const int64_t src_strides[4], void* dst, const int64_t dst_strides[4],
                           int B, int C, int Hi, int Wi, int Ho, int Wo, int align_corners, int accumulate,
                           int dtype, void* stream) {
  using namespace ula::glue;
  Map m;
  bool vec = false;
  int rc = prepare("uplift_resize_bilinear", src, src_strides, dst, dst_strides, B, C, Hi, Wi, Ho, Wo, dtype, &m, &vec);
  if (rc != UPLIFT_LA_OK) return rc;
  if (align_corners) {
    m.scale_h = Ho > 1 ? (float)(Hi - 1) / (float)(Ho - 1) : 0.f;
    m.scale_w = Wo > 1 ? (float)(Wi - 1) / (float)(Wo - 1) : 0.f;
  } else {
    m.scale_h = Ho > 0 ? (float)Hi / (float)Ho : 0.f;
    m.scale_w = Wo > 0 ? (float)Wi / (float)Wo : 0.f;
  }
  return dispatch(Op::kBilinear, m, dtype, vec, align_corners != 0, accumulate != 0, stream);
}

int uplift_resize_nearest(const void* src, const int64_t src_strides[4], void* dst, const int64_t dst_strides[4],
                          int B, int C, int Hi, int Wi, int Ho, int Wo, int dtype, void* stream) {
  using namespace ula::glue;
  Map m;
  bool vec = false;
  int rc = prepare("uplift_resize_nearest", src, src_strides, dst, dst_strides, B, C, Hi, Wi, Ho, Wo, dtype, &m, &vec);
  if (rc != UPLIFT_LA_OK) return rc;
  m.scale_h = Ho > 0 ? (float)Hi / (float)Ho : 0.f;
  m.scale_w = Wo > 0 ? (float)Wi / (float)Wo : 0.f;
  return dispatch(Op::kNearest, m, dtype, vec, false, false, stream);
}

int uplift_add_channels(void* dst, const int64_t dst_strides[4], const void* src, const int64_t src_strides[4],
                        int B, int C, int H, int W, int dtype, void* stream) {
  using namespace ula::glue;
  Map m;
  bool vec = false;
  int rc = prepare("uplift_add_channels", src, src_strides, dst, dst_strides, B, C, H, W, H, W, dtype, &m, &vec);
  if (rc != UPLIFT_LA_OK) return rc;
  m.scale_h = m.scale_w = 1.f;
  return dispatch(Op::kAdd, m, dtype, vec, false, false, stream);
}

int uplift_bias_act(void* dst, const int64_t dst_strides[4], const void* bias, const void* res,
                    const int64_t res_strides[4], int res_channels, int relu, int B, int C, int H, int W,
                    int dtype, void* stream) {
  using namespace ula::glue;
  using ula::fail;
  Map m;
  bool vec = false;
  const int64_t* rs = res != nullptr ? res_strides : dst_strides;
  int rc = prepare("uplift_bias_act", res != nullptr ? res : dst, rs, dst, dst_strides, B, C, H, W, H, W, dtype,
                   &m, &vec);
  if (rc != UPLIFT_LA_OK) return rc;
  if (res != nullptr && (res_channels < 0 || res_channels > C))
    return fail(UPLIFT_LA_ERR_SHAPE, "uplift_bias_act: res_channels=%d outside 0..C=%d", res_channels, C);
  const int ve = dtype == UPLIFT_LA_F32 ? 4 : 8;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  vec = vec && (bias == nullptr || a16(bias)) && (res == nullptr || res_channels % ve == 0);
  Epi e;
  e.dst = dst; e.d_b = m.d_b; e.d_h = m.d_h; e.d_w = m.d_w;
  e.bias = bias;
  e.res = res_channels > 0 ? res : nullptr;
  e.r_b = m.s_b; e.r_h = m.s_h; e.r_w = m.s_w;
  e.res_c = res_channels;
  e.C = C; e.H = H; e.W = W;
  e.total = m.total;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case UPLIFT_LA_F32: return launch_epi<float>(e, vec, relu != 0, s);
    case UPLIFT_LA_BF16: return launch_epi<__nv_bfloat16>(e, vec, relu != 0, s);
    default: return launch_epi<__half>(e, vec, relu != 0, s);
  }
}

}  // extern "C"
