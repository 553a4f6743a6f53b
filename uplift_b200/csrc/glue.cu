// Resampling and residual kernels around the Local Attender in the UPLiFT
// upsampler's fast mode (C ABI in include/uplift_glue.h).
//
// All are streaming, HBM-bound NHWC kernels: one CTA per output row
// (source rows and weights uniform over the CTA), a thread owns one output
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
  int64_t total;  // batch size (0 for an empty problem); one CTA per output row
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
  // one CTA per output row: the source rows and their weights are uniform
  const int row = blockIdx.x;
  const int oy = row % m.Ho, b = row / m.Ho;
  int y0, yp;
  float ly0, ly1;
  src_coord<ALIGN>(oy, m.scale_h, m.Hi, y0, yp, ly0, ly1);
  const T* r0 = src + b * m.s_b + y0 * m.s_h;
  const T* r1 = r0 + yp * m.s_h;
  T* orow = dst + b * m.d_b + oy * m.d_h;
  const int nv = m.C / VEC;
  const int items = m.Wo * nv;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    const int ox = i / nv, c = (i - ox * nv) * VEC;
    int x0, xp;
    float lx0, lx1;
    src_coord<ALIGN>(ox, m.scale_w, m.Wi, x0, xp, lx0, lx1);
    Vec<T, VEC> a, bb, cc, d;
    a.load(r0 + x0 * m.s_w + c);
    bb.load(r0 + (x0 + xp) * m.s_w + c);
    cc.load(r1 + x0 * m.s_w + c);
    d.load(r1 + (x0 + xp) * m.s_w + c);
    T* out = orow + ox * m.d_w + c;
    Vec<T, VEC> o;
    if constexpr (ACC) o.load(out);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float val = ly0 * (lx0 * St<T>::f(a.e[e]) + lx1 * St<T>::f(bb.e[e])) +
                        ly1 * (lx0 * St<T>::f(cc.e[e]) + lx1 * St<T>::f(d.e[e]));
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
  const int row = blockIdx.x;
  const int oy = row % m.Ho, b = row / m.Ho;
  const int sy = min((int)floorf((float)oy * m.scale_h), m.Hi - 1);
  const T* srow = src + b * m.s_b + sy * m.s_h;
  T* orow = dst + b * m.d_b + oy * m.d_h;
  const int nv = m.C / VEC;
  const int items = m.Wo * nv;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    const int ox = i / nv, c = (i - ox * nv) * VEC;
    const int sx = min((int)floorf((float)ox * m.scale_w), m.Wi - 1);
    Vec<T, VEC> a;
    a.load(srow + sx * m.s_w + c);
    a.store(orow + ox * m.d_w + c);
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads) add_kernel(const Map m) {
  const T* __restrict__ src = static_cast<const T*>(m.src);
  T* __restrict__ dst = static_cast<T*>(m.dst);
  const int row = blockIdx.x;
  const int y = row % m.Ho, b = row / m.Ho;
  const T* srow = src + b * m.s_b + y * m.s_h;
  T* orow = dst + b * m.d_b + y * m.d_h;
  const int nv = m.C / VEC;
  const int items = m.Wo * nv;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    const int x = i / nv, c = (i - x * nv) * VEC;
    Vec<T, VEC> a, o;
    a.load(srow + x * m.s_w + c);
    T* out = orow + x * m.d_w + c;
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

// RVEC: the residual is read with 16-byte vectors (its channel count and
// strides allow it); otherwise element by element, only below res_c.
template <typename T, int VEC, bool RELU, bool RVEC>
__global__ void __launch_bounds__(kThreads) bias_act_kernel(const Epi m) {
  T* __restrict__ dst = static_cast<T*>(m.dst);
  const T* __restrict__ bias = static_cast<const T*>(m.bias);
  const T* __restrict__ res = static_cast<const T*>(m.res);
  const int row = blockIdx.x;
  const int y = row % m.H, b = row / m.H;
  T* orow = dst + b * m.d_b + y * m.d_h;
  const T* rrow = res != nullptr ? res + b * m.r_b + y * m.r_h : nullptr;
  const int nv = m.C / VEC;
  const int items = m.W * nv;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    const int x = i / nv, c0 = (i - x * nv) * VEC;
    T* out = orow + x * m.d_w + c0;
    Vec<T, VEC> o, bv, rv;
    o.load(out);
    if (bias != nullptr) bv.load(bias + c0);
    const bool has_res = rrow != nullptr && c0 < m.res_c;
    const T* rp = has_res ? rrow + x * m.r_w + c0 : nullptr;
    if (RVEC && has_res) rv.load(rp);  // res_c is a multiple of VEC
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      float t = St<T>::f(o.e[e]);
      if (bias != nullptr) t = St<T>::f(St<T>::t(t + St<T>::f(bv.e[e])));
      if (RELU) t = fmaxf(t, 0.f);
      if (has_res && c0 + e < m.res_c) t = t + St<T>::f(RVEC ? rv.e[e] : rp[e]);
      o.e[e] = St<T>::t(t);
    }
    o.store(out);
  }
}

template <typename T>
int launch_epi(const Epi& m0, bool vec, bool rvec, bool relu, cudaStream_t stream);

// LayerNorm over the channels of each pixel (+ optional conv bias before,
// ReLU after): one warp per pixel with the pixel's C values in registers
// (VPL vectors of VEC per lane); the per-channel bias and affine terms are
// staged once per CTA in shared memory (fp32, [3][C]).
struct Ln {
  void* dst; int64_t d_b, d_h, d_w;
  const void* pre_bias;
  const void* weight;
  const void* bias;
  float eps;
  int C, H, W;
  int64_t pixels;
};

constexpr int kLnWarps = 8;  // warps per CTA

template <typename T, int VEC, int VPL, bool RELU>
__global__ void __launch_bounds__(kLnWarps * 32) layernorm_kernel(const Ln a) {
  extern __shared__ float ln_smem[];
  T* __restrict__ dst = static_cast<T*>(a.dst);
  const T* __restrict__ pb = static_cast<const T*>(a.pre_bias);
  const T* __restrict__ wt = static_cast<const T*>(a.weight);
  const T* __restrict__ bs = static_cast<const T*>(a.bias);
  float* s_w = ln_smem;
  float* s_b = ln_smem + a.C;
  float* s_p = ln_smem + 2 * a.C;
  for (int c = threadIdx.x; c < a.C; c += kLnWarps * 32) {
    s_w[c] = St<T>::f(wt[c]);
    s_b[c] = St<T>::f(bs[c]);
    s_p[c] = pb != nullptr ? St<T>::f(pb[c]) : 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nvec = a.C / VEC;
  const bool has_pb = pb != nullptr;
  const float inv_c = 1.f / (float)a.C;
  const int64_t wstride = (int64_t)gridDim.x * kLnWarps;
  for (int64_t pix = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5); pix < a.pixels; pix += wstride) {
    const int x = (int)(pix % a.W);
    const int64_t r = pix / a.W;
    const int y = (int)(r % a.H);
    const int bb = (int)(r / a.H);
    T* row = dst + bb * a.d_b + y * a.d_h + x * a.d_w;
    float t[VPL][VEC];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      Vec<T, VEC> xv;
      if (v < nvec) xv.load(row + v * VEC);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        float q = 0.f;
        if (v < nvec) {
          q = St<T>::f(xv.e[e]);
          // the conv output plus its bias, rounded as the eager add would
          if (has_pb) q = St<T>::f(St<T>::t(q + s_p[v * VEC + e]));
        }
        t[j][e] = q;
        sum += q;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mu = sum * inv_c;
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float d = t[j][e] - mu;
        sq += v < nvec ? d * d : 0.f;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float den = sqrtf(sq * inv_c + a.eps);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v >= nvec) continue;
      Vec<T, VEC> ov;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int c = v * VEC + e;
        float o = s_w[c] * ((t[j][e] - mu) / den) + s_b[c];
        if (RELU) o = fmaxf(o, 0.f);
        ov.e[e] = St<T>::t(o);
      }
      ov.store(row + v * VEC);
    }
  }
}

template <typename T, int VEC>
int launch_ln_v(const Ln& a, int vpl, bool relu, cudaStream_t stream) {
  const int64_t blocks64 = std::min<int64_t>((a.pixels + kLnWarps - 1) / kLnWarps, 148ll * 32);
  const dim3 grid((unsigned)blocks64), block(kLnWarps * 32);
  const size_t smem = 3 * sizeof(float) * (size_t)a.C;
#define ULA_LN(V)                                                                           \
  case V:                                                                                   \
    if (relu) layernorm_kernel<T, VEC, V, true><<<grid, block, smem, stream>>>(a);          \
    else layernorm_kernel<T, VEC, V, false><<<grid, block, smem, stream>>>(a);              \
    break;
  switch (vpl) {
    ULA_LN(1) ULA_LN(2) ULA_LN(4) ULA_LN(8) ULA_LN(16)
    default: return fail(UPLIFT_LA_ERR_SHAPE, "uplift_layernorm_act: too many channels");
  }
#undef ULA_LN
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "glue kernel launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

template <typename T>
int launch_ln(const Ln& a, bool vec, bool relu, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  const int ve = vec ? V : 1;
  const int nvec = a.C / ve;
  int vpl = 1;
  while (vpl * 32 < nvec) vpl *= 2;
  return vec ? launch_ln_v<T, V>(a, vpl, relu, stream) : launch_ln_v<T, 1>(a, vpl, relu, stream);
}

enum class Op { kBilinear, kNearest, kAdd };

template <typename T, int VEC>
int launch_t(Op op, const Map& m0, bool align, bool acc, cudaStream_t stream) {
  Map m = m0;
  const int64_t rows = (int64_t)m.Ho * m.total;  // m.total holds the batch
  if (rows == 0 || m.Wo == 0 || m.C == 0) return UPLIFT_LA_OK;
  if (rows >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "glue: too many output rows");
  const dim3 grid((unsigned)rows);
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
  if ((int64_t)C * Wo >= (1ll << 31) || (int64_t)C * Wi >= (1ll << 31))
    return fail(UPLIFT_LA_ERR_SHAPE, "%s: a row exceeds 2^31 elements", what);
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
int launch_epi(const Epi& m0, bool vec, bool rvec, bool relu, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  Epi m = m0;
  const int64_t rows = (int64_t)m.H * m.total;  // m.total holds the batch
  if (rows == 0 || m.W == 0 || m.C == 0) return UPLIFT_LA_OK;
  if (rows >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "glue: too many output rows");
  const dim3 grid((unsigned)rows);
  if (vec && rvec) {
    if (relu) bias_act_kernel<T, V, true, true><<<grid, kThreads, 0, stream>>>(m);
    else bias_act_kernel<T, V, false, true><<<grid, kThreads, 0, stream>>>(m);
  } else if (vec) {
    if (relu) bias_act_kernel<T, V, true, false><<<grid, kThreads, 0, stream>>>(m);
    else bias_act_kernel<T, V, false, false><<<grid, kThreads, 0, stream>>>(m);
  } else {
    if (relu) bias_act_kernel<T, 1, true, false><<<grid, kThreads, 0, stream>>>(m);
    else bias_act_kernel<T, 1, false, false><<<grid, kThreads, 0, stream>>>(m);
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
  bool vec = false, rvec = false;
  // output (and bias) vectors: validated with dst as its own source
  int rc = prepare("uplift_bias_act", dst, dst_strides, dst, dst_strides, B, C, H, W, H, W, dtype, &m, &vec);
  if (rc != UPLIFT_LA_OK) return rc;
  if (res != nullptr) {
    if (res_channels < 0 || res_channels > C)
      return fail(UPLIFT_LA_ERR_SHAPE, "uplift_bias_act: res_channels=%d outside 0..C=%d", res_channels, C);
    if (res_strides == nullptr) return fail(UPLIFT_LA_ERR_ARG, "uplift_bias_act: null residual strides");
    if (res_channels > 1 && res_strides[1] != 1)
      return fail(UPLIFT_LA_ERR_LAYOUT, "uplift_bias_act: residual channel stride must be 1");
    for (int i = 0; i < 4; ++i)
      if (res_strides[i] < 0) return fail(UPLIFT_LA_ERR_LAYOUT, "uplift_bias_act: negative residual stride");
  }
  const int ve = dtype == UPLIFT_LA_F32 ? 4 : 8;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  vec = vec && (bias == nullptr || a16(bias));
  rvec = res != nullptr && res_channels % ve == 0 && a16(res) && res_strides[0] % ve == 0 &&
         res_strides[2] % ve == 0 && res_strides[3] % ve == 0;
  Epi e;
  e.dst = dst; e.d_b = m.d_b; e.d_h = m.d_h; e.d_w = m.d_w;
  e.bias = bias;
  e.res = res_channels > 0 ? res : nullptr;
  e.r_b = res != nullptr ? res_strides[0] : 0;
  e.r_h = res != nullptr ? res_strides[2] : 0;
  e.r_w = res != nullptr ? res_strides[3] : 0;
  e.res_c = res_channels;
  e.C = C; e.H = H; e.W = W;
  e.total = m.total;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case UPLIFT_LA_F32: return launch_epi<float>(e, vec, rvec, relu != 0, s);
    case UPLIFT_LA_BF16: return launch_epi<__nv_bfloat16>(e, vec, rvec, relu != 0, s);
    default: return launch_epi<__half>(e, vec, rvec, relu != 0, s);
  }
}

int uplift_layernorm_act(void* dst, const int64_t dst_strides[4], const void* pre_bias, const void* weight,
                         const void* bias, float eps, int relu, int B, int C, int H, int W, int dtype, void* stream) {
  using namespace ula::glue;
  using ula::fail;
  Map m;
  bool vec = false;
  int rc = prepare("uplift_layernorm_act", dst, dst_strides, dst, dst_strides, B, C, H, W, H, W, dtype, &m, &vec);
  if (rc != UPLIFT_LA_OK) return rc;
  if (m.total > 0 && (weight == nullptr || bias == nullptr))
    return fail(UPLIFT_LA_ERR_ARG, "uplift_layernorm_act: null weight / bias");
  const int ve = dtype == UPLIFT_LA_F32 ? 4 : 8;
  if (C > 16 * 32 * (vec ? ve : 1) || C > 4096)
    return fail(UPLIFT_LA_ERR_SHAPE, "uplift_layernorm_act: C=%d above the register-resident limit", C);
  Ln a;
  a.dst = dst; a.d_b = m.d_b; a.d_h = m.d_h; a.d_w = m.d_w;
  a.pre_bias = pre_bias; a.weight = weight; a.bias = bias; a.eps = eps;
  a.C = C; a.H = H; a.W = W;
  a.pixels = (int64_t)m.total * H * W;
  if (a.pixels == 0 || C == 0) return UPLIFT_LA_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case UPLIFT_LA_F32: return launch_ln<float>(a, vec, relu != 0, s);
    case UPLIFT_LA_BF16: return launch_ln<__nv_bfloat16>(a, vec, relu != 0, s);
    default: return launch_ln<__half>(a, vec, relu != 0, s);
  }
}

}  // extern "C"
