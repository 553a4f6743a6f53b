#pragma once
// Backward of the fused Local Attender (training), sm_100a: kernels and
// launch templates, instantiated per storage type in la_bwd_{f32,bf16,f16}.cu
// (compiled in parallel); the C entry points are in la_bwd.cu.
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
// fp32 workspace [B, Ho, Wo, K] (probs_kernel, a thread per pixel);
// dlogit forms dP, dl and dg and reduces dW / db over the CTA in shared
// memory before one global atomic add per entry -- dlogit_mma_kernel (dP on
// the tensor cores; fp32 through a bf16 hi / lo split) or dlogit_kernel
// (other shapes: a group of 8 lanes per
// unit of CPT children of one cell, lanes over 16-byte channel vectors, so
// each dout row and each neighbour value row is read once per unit); and
// dvalue_window_kernel gathers dV with a sliding window: a thread owns one
// (value row, 16-byte channel vector), sweeps the cells of the row left to
// right and keeps the 2 pn + 1 value pixels a cell can reach in a register
// ring, so each dout child is loaded once per offset row (no atomics on the
// large tensors).  fp32 arithmetic throughout.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <type_traits>

#include "uplift_la.h"
#include "la_internal.h"

namespace ula {
namespace bwd {

constexpr int kThreads = 256;   // threads per CTA: probs, dvalue
constexpr int kDThreads = 128;  // threads per CTA: dlogit
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

// 16-byte vectors of VEC storage elements.
template <typename T, int VEC>
struct V16 {
  alignas(16) T e[VEC];
  __device__ __forceinline__ void load(const T* p) {
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(e) = __ldg(reinterpret_cast<const uint4*>(p));
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) e[i] = p[i];
    }
  }
};

// Softmax (or argmax one-hot) weights of every output pixel; GV guide
// elements per load (16-byte vectors when the guide layout allows).
template <typename T, int K, int GV>
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
    for (int c0 = 0; c0 < a.Cg; c0 += GV) {
      V16<T, GV> gv;
      gv.load(gp + c0);
#pragma unroll
      for (int e = 0; e < GV; ++e) {
        const float g = tof(gv.e[e]);
#pragma unroll
        for (int k = 0; k < K; ++k) l[k] = fmaf(s_w[(c0 + e) * K + k], g, l[k]);
      }
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

// A group of kGroup lanes per unit (CPT children of one cell: the 2 x 2
// children for I = 2, one row of 4 for I = 4, one pixel otherwise), 32 /
// kGroup units per warp; the group's lanes stride over 16-byte channel
// vectors, so each dout row and each neighbour value row is read once per
// unit, and the partial dP sums need log2(kGroup) shuffle steps.  dW / db
// are reduced per unit slot in shared memory (no same-address atomics
// inside a warp), then once per CTA into global memory.
constexpr int kGroup = 8;
constexpr int kSlots = 32 / kGroup;

// Per-slot dW replicas start 8 banks apart, so the four slots of a warp
// (same k, channels sub + 8 j) hit 32 distinct banks.
__host__ __device__ constexpr int dw_slot_stride(int K, int Cg) { return (K * Cg + 31) / 32 * 32 + 8; }

template <int K>
__host__ __device__ constexpr size_t dlogit_smem_floats(int Cg) {
  return (size_t)Cg * K + (size_t)kSlots * dw_slot_stride(K, Cg) + (size_t)kSlots * K;
}

// Four CTAs per SM when the unit holds at most two children (<= 128
// registers), two otherwise.
template <typename T, int K, int CPT, int VEC>
__global__ void __launch_bounds__(kDThreads, CPT <= 2 ? 4 : 2) dlogit_kernel(const Args a) {
  extern __shared__ float smem[];
  const int sstride = dw_slot_stride(K, a.Cg);
  float* s_w = smem;                          // [Cg][K]               W' (residual folded)
  float* s_dw = s_w + a.Cg * K;               // [kSlots][sstride]     this CTA's dW, [K][Cg] per slot
  float* s_db = s_dw + kSlots * sstride;      // [kSlots][K]
  stage_weights<K>(a, s_w, kDThreads);
  for (int i = threadIdx.x; i < kSlots * (sstride + K); i += kDThreads) s_dw[i] = 0.f;
  __syncthreads();
  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  const T* __restrict__ guide = static_cast<const T*>(a.guide);
  const T* __restrict__ value = static_cast<const T*>(a.value);
  const int lane = threadIdx.x & 31, slot = lane / kGroup, sub = lane % kGroup;
  float* my_dw = s_dw + slot * sstride;
  float* my_db = s_db + slot * K;
  const int upc = (a.I * a.I) / CPT;  // units per cell
  const int64_t num_units = (int64_t)a.B * a.H * a.W * upc;
  const int nv = a.C / VEC;
  const bool params = (a.dweight != nullptr || a.dbias != nullptr) && !a.hardmax;
  const int64_t stride = (int64_t)gridDim.x * (kDThreads / 32) * kSlots;
  // warp-uniform trip count: slots past the end run the shuffles on zeros
  for (int64_t u0 = ((int64_t)blockIdx.x * (kDThreads / 32) + (threadIdx.x >> 5)) * kSlots; u0 < num_units;
       u0 += stride) {
    const int64_t u = u0 + slot;
    const bool valid = u < num_units;
    const int64_t uc = valid ? u : num_units - 1;
    const int usub = (int)(uc % upc);
    const int64_t cell = uc / upc;
    const int cx = (int)(cell % a.W);
    const int64_t rr = cell / a.W;
    const int cy = (int)(rr % a.H);
    const int b = (int)(rr / a.H);
    int py[CPT], px[CPT];
#pragma unroll
    for (int t = 0; t < CPT; ++t) {
      const int ch = usub * CPT + t;
      const int ci = ch / a.I;
      py[t] = cy * a.I + ci;
      px[t] = cx * a.I + (ch - ci * a.I);
    }
    float dl[CPT][K];
    if (!a.hardmax) {
      const T* vb = value + b * a.v_b;
      float dP[CPT][K];
      if constexpr (sizeof(T) == 2) {
        // 16-bit storage: children in pairs (t0, t1), one packed FMA updates
        // dP[t0][k] and dP[t1][k] with (d[t0][e], d[t1][e]) * (x, x) -- the
        // same fp32 FMAs in the same order as the scalar form, half the
        // instructions (the converted values land in fresh registers anyway)
        constexpr int CP = (CPT + 1) / 2;
        float2 dP2[CP][K];
#pragma unroll
        for (int t = 0; t < CP; ++t)
#pragma unroll
          for (int k = 0; k < K; ++k) dP2[t][k] = make_float2(0.f, 0.f);
#pragma unroll 1
        for (int v = sub; v < nv; v += kGroup) {
          float d[2 * CP][VEC];
#pragma unroll
          for (int t = 0; t < CPT; ++t) {
            V16<T, VEC> dv;
            dv.load(dout + b * a.d_b + py[t] * a.d_h + px[t] * a.d_w + v * VEC);
#pragma unroll
            for (int e = 0; e < VEC; ++e) d[t][e] = tof(dv.e[e]);
          }
          if (CPT % 2 != 0) {
#pragma unroll
            for (int e = 0; e < VEC; ++e) d[2 * CP - 1][e] = 0.f;
          }
#pragma unroll
          for (int k = 0; k < K; ++k) {
            V16<T, VEC> vv;
            vv.load(vb + clampi(cy + a.dy[k], 0, a.H - 1) * a.v_h + clampi(cx + a.dx[k], 0, a.W - 1) * a.v_w +
                    v * VEC);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              const float x = tof(vv.e[e]);
              const float2 xx = make_float2(x, x);
#pragma unroll
              for (int t = 0; t < CP; ++t)
                dP2[t][k] = __ffma2_rn(make_float2(d[2 * t][e], d[2 * t + 1][e]), xx, dP2[t][k]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < CPT; ++t)
#pragma unroll
          for (int k = 0; k < K; ++k) dP[t][k] = (t % 2 == 0) ? dP2[t / 2][k].x : dP2[t / 2][k].y;
      } else {
#pragma unroll
        for (int t = 0; t < CPT; ++t)
#pragma unroll
          for (int k = 0; k < K; ++k) dP[t][k] = 0.f;
#pragma unroll 1
        for (int v = sub; v < nv; v += kGroup) {
          float d[CPT][VEC];
#pragma unroll
          for (int t = 0; t < CPT; ++t) {
            V16<T, VEC> dv;
            dv.load(dout + b * a.d_b + py[t] * a.d_h + px[t] * a.d_w + v * VEC);
#pragma unroll
            for (int e = 0; e < VEC; ++e) d[t][e] = tof(dv.e[e]);
          }
#pragma unroll
          for (int k = 0; k < K; ++k) {
            V16<T, VEC> vv;
            vv.load(vb + clampi(cy + a.dy[k], 0, a.H - 1) * a.v_h + clampi(cx + a.dx[k], 0, a.W - 1) * a.v_w +
                    v * VEC);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              const float x = tof(vv.e[e]);
#pragma unroll
              for (int t = 0; t < CPT; ++t) dP[t][k] = fmaf(d[t][e], x, dP[t][k]);
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < CPT; ++t)
#pragma unroll
        for (int k = 0; k < K; ++k)
#pragma unroll
          for (int o = kGroup / 2; o > 0; o >>= 1) dP[t][k] += __shfl_xor_sync(0xffffffffu, dP[t][k], o);
#pragma unroll
      for (int t = 0; t < CPT; ++t) {
        const float* pp = a.probs + (((int64_t)b * a.Ho + py[t]) * a.Wo + px[t]) * K;
        float pk[K];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          pk[k] = pp[k];
          s = fmaf(pk[k], dP[t][k], s);
        }
#pragma unroll
        for (int k = 0; k < K; ++k) dl[t][k] = pk[k] * (dP[t][k] - s);
      }
    } else {
#pragma unroll
      for (int t = 0; t < CPT; ++t)
#pragma unroll
        for (int k = 0; k < K; ++k) dl[t][k] = 0.f;
    }
    if (!valid) continue;
    // dguide (the group's lanes over guide channels) and this unit's dW / db
    for (int c = sub; c < a.Cg; c += kGroup) {
      float wacc[K];
#pragma unroll
      for (int k = 0; k < K; ++k) wacc[k] = 0.f;
#pragma unroll
      for (int t = 0; t < CPT; ++t) {
        if (a.dguide != nullptr) {
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < K; ++k) acc = fmaf(dl[t][k], s_w[c * K + k], acc);
          static_cast<T*>(a.dguide)[b * a.dg_b + py[t] * a.dg_h + px[t] * a.dg_w + c] = fromf<T>(acc);
        }
        if (params) {
          const float g = tof(guide[b * a.g_b + py[t] * a.g_h + px[t] * a.g_w + c]);
#pragma unroll
          for (int k = 0; k < K; ++k) wacc[k] = fmaf(dl[t][k], g, wacc[k]);
        }
      }
      if (params) {
#pragma unroll
        for (int k = 0; k < K; ++k) atomicAdd(my_dw + k * a.Cg + c, wacc[k]);
      }
    }
    if (params) {
      for (int k0 = sub; k0 < K; k0 += kGroup) {
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < CPT; ++t)
#pragma unroll
          for (int k = 0; k < K; ++k) acc += (k == k0) ? dl[t][k] : 0.f;
        atomicAdd(my_db + k0, acc);
      }
    }
  }
  if (!params) return;
  __syncthreads();
  for (int i = threadIdx.x; i < K * (a.Cg + 1); i += kDThreads) {
    const bool isw = i < K * a.Cg;
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kSlots; ++q) s += isw ? s_dw[q * sstride + i] : s_db[q * K + (i - K * a.Cg)];
    if (isw && a.dweight != nullptr) atomicAdd(a.dweight + i, s);
    if (!isw && a.dbias != nullptr) atomicAdd(a.dbias + (i - K * a.Cg), s);
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

// dV per value pixel, general form (any offset table): one CTA per value
// row, a thread per (pixel, channel vector), gathering P_k(p) dout[p] over
// the children p of every cell whose offset-k neighbour is this pixel.
template <typename T, int K, int VEC>
__global__ void __launch_bounds__(kThreads) dvalue_kernel(const Args a) {
  __shared__ int s_off[2 * K];  // dy, dx (read with a runtime index below)
  if (threadIdx.x < K) {
    s_off[threadIdx.x] = a.dy[threadIdx.x];
    s_off[K + threadIdx.x] = a.dx[threadIdx.x];
  }
  __syncthreads();
  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  T* __restrict__ dv = static_cast<T*>(a.dvalue);
  const int row = blockIdx.x;  // (b, ny)
  const int ny = row % a.H, b = row / a.H;
  const int nv = a.C / VEC;
  const int items = a.W * nv;
  const T* db = dout + b * a.d_b;
  const float* pb = a.probs + (int64_t)b * a.Ho * a.Wo * K;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    const int nx = i / nv, c0 = (i - nx * nv) * VEC;
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
#pragma unroll 1
    for (int k = 0; k < K; ++k) {
      int ylo, yhi, xlo, xhi;
      cell_range(ny, s_off[k], a.H, ylo, yhi);
      cell_range(nx, s_off[K + k], a.W, xlo, xhi);
      for (int y = ylo * a.I; y < (yhi + 1) * a.I; ++y)
        for (int x = xlo * a.I; x < (xhi + 1) * a.I; ++x) {
          const float pk = pb[((int64_t)y * a.Wo + x) * K + k];
          if (pk != 0.f) {
            V16<T, VEC> d;
            d.load(db + y * a.d_h + x * a.d_w + c0);
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[e] = fmaf(pk, tof(d.e[e]), acc[e]);
          }
        }
    }
    T* out = dv + b * a.dv_b + ny * a.dv_h + nx * a.dv_w + c0;
#pragma unroll
    for (int e = 0; e < VEC; ++e) out[e] = fromf<T>(acc[e]);
  }
}

// The reference's offset tables (uplift/uplift.py:746-760), as the map
// (dy, dx) -> k (-1 where the table has no such offset) and their reach pn.
// Used as compile-time constants by the sliding-window dV kernel when the
// caller passes exactly these tables.
template <int K>
__host__ __device__ constexpr int nbh_pn() { return (K == 5 || K == 9) ? 1 : 2; }

template <int K>
__host__ __device__ constexpr int nbh_k(int dy, int dx) {
  const int ady = dy < 0 ? -dy : dy, adx = dx < 0 ? -dx : dx;
  if (K == 25) return (ady <= 2 && adx <= 2) ? (dy + 2) * 5 + dx + 2 : -1;
  if (K == 9) return (ady <= 1 && adx <= 1) ? (dy + 1) * 3 + dx + 1 : -1;
  if (K == 5) {
    if (dy == 0) return adx <= 1 ? 2 + dx : -1;
    return (ady == 1 && dx == 0) ? (dy < 0 ? 0 : 4) : -1;
  }
  if (K == 13) {
    if (dy == 0) return adx <= 2 ? 6 + dx : -1;
    if (ady == 1) return adx <= 1 ? (dy < 0 ? 1 : 9) + dx + 1 : -1;
    return (ady == 2 && dx == 0) ? (dy < 0 ? 0 : 12) : -1;
  }
  if (K == 17) {
    if (dy == 0) return adx <= 2 ? 8 + dx : -1;
    if (ady == 1) return adx <= 1 ? (dy < 0 ? 3 : 11) + dx + 1 : -1;
    return (ady == 2 && (dx == -2 || dx == 0 || dx == 2)) ? (dy < 0 ? 0 : 14) + (dx + 2) / 2 : -1;
  }
  return -1;
}

// dV with a sliding window (the reference's offset table for K).  A thread
// owns (b, value row ny, channel vector v, segment [x0, x1) of value
// columns) and sweeps the cells cx of [x0 - PN, x1 + PN).  Cell cx
// contributes to the value pixels clamp(cx + dx) in [cx - PN, cx + PN]; ring
// slot s holds the pixel cx - PN + s, so after cell cx the pixel cx - PN is
// complete, is written and the ring shifts by one.  Rows: for each dy the
// cells whose clamped row neighbour is ny (cell_range, a single row away
// from the top and bottom edges); the I x I children of each are loaded once
// and used for every dx of that dy.  Cells within PN of the left or right
// edge take a runtime slot (clamped dx) through a compile-time select.
template <typename T, int K, int VEC, int IT>
__global__ void __launch_bounds__(kThreads, 1) dvalue_window_kernel(const Args a, int seg_len, int nseg) {
  constexpr int PN = nbh_pn<K>();
  constexpr int S = 2 * PN + 1;
  constexpr int ITc = IT > 0 ? IT : 1;  // child grid of the unrolled path
  const int nv = a.C / VEC;
  const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t >= (int64_t)a.B * a.H * nseg * nv) return;
  const int v = (int)(t % nv);
  int64_t r = t / nv;
  const int seg = (int)(r % nseg);
  r /= nseg;
  const int ny = (int)(r % a.H), b = (int)(r / a.H);
  const int x0 = seg * seg_len, x1 = min(a.W, x0 + seg_len);
  if (x0 >= x1) return;
  const T* __restrict__ db = static_cast<const T*>(a.dout) + b * a.d_b + v * VEC;
  const float* __restrict__ pb = a.probs + (int64_t)b * a.Ho * a.Wo * K;
  T* __restrict__ out = static_cast<T*>(a.dvalue) + b * a.dv_b + ny * a.dv_h + v * VEC;
  const int I = IT > 0 ? IT : a.I;
  const bool row_inner = IT > 0 && ny >= PN && ny < a.H - PN;
  // accumulators as channel pairs: one packed FMA (pk, pk) * (d[e], d[e+1])
  // per pair, the same fp32 FMAs as the scalar form
  constexpr int VP = (VEC + 1) / 2;
  float2 ring[S][VP];
#pragma unroll
  for (int s = 0; s < S; ++s)
#pragma unroll
    for (int e = 0; e < VP; ++e) ring[s][e] = make_float2(0.f, 0.f);
  auto accumulate = [&](float2* acc, float pk, const float* d) {
    if (VEC % 2 == 0) {
      const float2 pp = make_float2(pk, pk);
#pragma unroll
      for (int e = 0; e < VP; ++e) acc[e] = __ffma2_rn(pp, make_float2(d[2 * e], d[2 * e + 1]), acc[e]);
    } else {
      acc[0].x = fmaf(pk, d[0], acc[0].x);
    }
  };
  auto store = [&](T* o, const float2* acc) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] = fromf<T>((e % 2 == 0) ? acc[e / 2].x : acc[e / 2].y);
  };

  // ring[slot(dx)] += P_k(child) dout(child) for every dx of offset row i
  auto add_child = [&](auto inner, int i, int cx, int y, int x) {
    V16<T, VEC> dv;
    dv.load(db + y * a.d_h + x * a.d_w);
    float d[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) d[e] = tof(dv.e[e]);
    const float* pp = pb + ((int64_t)y * a.Wo + x) * K;
#pragma unroll
    for (int j = 0; j < S; ++j) {
      const int k = nbh_k<K>(i - PN, j - PN);
      if (k < 0) continue;
      const float pk = pp[k];
      if (decltype(inner)::value) {
        accumulate(ring[j], pk, d);
      } else {
        const int slot = clampi(cx + j - PN, 0, a.W - 1) - cx + PN;
#pragma unroll
        for (int q = 0; q < S; ++q)
          if (q == slot) accumulate(ring[q], pk, d);
      }
    }
  };
  auto step = [&](auto inner, int cx) {
    if (row_inner) {
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int cy = ny - (i - PN);
#pragma unroll
        for (int ch = 0; ch < ITc * ITc; ++ch) add_child(inner, i, cx, cy * ITc + ch / ITc, cx * ITc + ch % ITc);
      }
    } else {
#pragma unroll
      for (int i = 0; i < S; ++i) {
        int lo, hi;
        cell_range(ny, i - PN, a.H, lo, hi);
#pragma unroll 1
        for (int cy = lo; cy <= hi; ++cy)
#pragma unroll 1
          for (int ch = 0; ch < I * I; ++ch) add_child(inner, i, cx, cy * I + ch / I, cx * I + ch % I);
      }
    }
    const int nx = cx - PN;
    if (nx >= x0) store(out + nx * a.dv_w, ring[0]);
#pragma unroll
    for (int s = 0; s + 1 < S; ++s)
#pragma unroll
      for (int e = 0; e < VP; ++e) ring[s][e] = ring[s + 1][e];
#pragma unroll
    for (int e = 0; e < VP; ++e) ring[S - 1][e] = make_float2(0.f, 0.f);
  };
  using Edge = std::integral_constant<bool, false>;
  using Inner = std::integral_constant<bool, true>;
  const int c0 = max(0, x0 - PN), cend = min(a.W, x1 + PN);
  const int i0 = min(max(c0, PN), cend), i1 = max(min(cend, a.W - PN), i0);
  for (int cx = c0; cx < i0; ++cx) step(Edge{}, cx);
#pragma unroll 1
  for (int cx = i0; cx < i1; ++cx) step(Inner{}, cx);
  for (int cx = i1; cx < cend; ++cx) step(Edge{}, cx);
  // pixels the sweep did not reach cx = nx + PN for (right edge of the map)
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int nx = cend - PN + s;
    if (nx >= x0 && nx < x1) store(out + nx * a.dv_w, ring[s]);
  }
}

// ---------------------------------------------------------------------------
// dlogit on tensor cores (I = 2, even Cg <= 64, offsets within +-PN, PN <= 2;
// 16-bit storage with C % 32 == 0, or fp32 with C % 16 == 0).  A warp owns a
// tile of 8 cells of one cell row = 32 output pixels (two rows of 16
// children).  For each offset row
// dy, dP over the tile is one small GEMM
//   D_dy[16 px x 16 window columns] = dout[16 px x C] . V_dy[16 x C]^T
// (window column j = value pixel clamp(cx0 - PN + j) of row clamp(cy + dy)),
// run as mma.sync m16n8k16 with fp32 accumulation: products of 16-bit
// values are exact, so only the summation order differs from the CUDA-core
// kernel.  Operand fragments come straight from global memory as 16-byte
// vectors: thread (g = lane / 4, t = lane % 4) loads channels [8t, 8t + 8)
// of a 32-channel chunk for its A rows (pixels g, g + 8) and its B column
// (window column g); the k-step s of the chunk takes channel pairs 4s and
// 4s + 2 of that vector for the fragment's low and high k halves -- one
// permutation of the channels applied to A and B alike, so the dot products
// are unchanged.  fp32 storage: 16-channel chunks, channels [4t, 4t + 4) per
// thread, each operand pair split into bf16 hi + lo and multiplied as
// hi*hi + hi*lo + lo*hi (about 2^-16 relative per product, the split the
// wide-guide forward kernel uses).  D is staged in shared memory; then a lane per pixel picks
// dP_k = D_dy(k)[pixel][cell + dx(k) + PN] and forms dl (fp32, as the
// CUDA-core kernel); then a lane per guide-channel pair forms dguide and
// accumulates dW / db over all of the warp's tiles in registers.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// fp32 pair (two 32-bit words) -> bf16x2 high part and bf16x2 remainder:
// x = hi + lo to about 2^-16 relative, so hi*hi + hi*lo + lo*hi is an fp32
// product to that accuracy (the dropped lo*lo term is ~2^-16 smaller).
__device__ __forceinline__ void split_bf16x2(uint32_t xa, uint32_t xb, uint32_t& hi, uint32_t& lo) {
  const float a = __uint_as_float(xa), b = __uint_as_float(xb);
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

__device__ __forceinline__ float2 pair_to_float2(float2 v) { return v; }
__device__ __forceinline__ float2 pair_to_float2(__nv_bfloat162 v) { return __bfloat1622float2(v); }
__device__ __forceinline__ float2 pair_to_float2(__half2 v) { return __half22float2(v); }

constexpr int kMmaWarps = 4;   // warps per dlogit_mma CTA
constexpr int kMmaDRow = 20;   // floats per staged D row (16 columns + pad)
constexpr int kMmaStages = 3;  // 32-channel chunks in flight per thread

template <int K>
__host__ __device__ constexpr int kpad4() { return (K + 3) & ~3; }

// 16-byte vectors a thread loads per chunk: 2 x 2 A rows, 2 B columns per dy
template <int PN>
__host__ __device__ constexpr int mma_vecs() { return 4 + 2 * (2 * PN + 1); }

// per-warp shared floats: the chunk ring, reused after the GEMM for the
// staged D (2 x (2 PN + 1) x 16 rows) and dl (32 x KP)
template <int K, int PN>
__host__ __device__ constexpr int mma_warp_floats() {
  return kMmaStages * mma_vecs<PN>() * 32 * 4 > 2 * (2 * PN + 1) * 16 * kMmaDRow + 32 * kpad4<K>()
             ? kMmaStages * mma_vecs<PN>() * 32 * 4
             : 2 * (2 * PN + 1) * 16 * kMmaDRow + 32 * kpad4<K>();
}

// shared floats: dW [K][Cg] and db [K] (each rounded up to 4 floats), W'
// channel pairs [K][32 lanes] (float2), then the warps' regions
template <int K, int PN>
__host__ __device__ constexpr size_t mma_smem_floats(int Cg) {
  return (size_t)((K * Cg + 3) & ~3) + kpad4<K>() + (size_t)K * 64 + (size_t)kMmaWarps * mma_warp_floats<K, PN>();
}

__device__ __forceinline__ void bwd_cp_async16(void* dst_smem, const void* src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void bwd_cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bwd_cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <typename T, int K, int PN>
__global__ void __launch_bounds__(kMmaWarps * 32, 2) dlogit_mma_kernel(const Args a) {
  constexpr int S = 2 * PN + 1;
  constexpr int KP = kpad4<K>();
  constexpr int kWarpFloats = mma_warp_floats<K, PN>();
  constexpr int NV = mma_vecs<PN>();
  using T2 = typename std::conditional<
      std::is_same<T, __nv_bfloat16>::value, __nv_bfloat162,
      typename std::conditional<std::is_same<T, __half>::value, __half2, float2>::type>::type;
  // fp32 storage: 16-channel chunks (one k-step; a thread's 16-byte vector
  // holds channels [4t, 4t + 4)), each operand split into bf16 hi + lo and
  // multiplied with three MMAs; 16-bit storage: 32-channel chunks (two
  // k-steps; channels [8t, 8t + 8)), one MMA each
  constexpr bool kF32 = std::is_same<T, float>::value;
  constexpr int CH = kF32 ? 16 : 32;
  extern __shared__ __align__(16) float smem[];
  float* s_dw = smem;                                  // [K][Cg]
  float* s_db = s_dw + ((K * a.Cg + 3) & ~3);          // [K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float2* s_wp = reinterpret_cast<float2*>(s_db + KP);  // [K][32]: W' of channel pair `lane`
  float* s_D = s_db + KP + K * 64 + warp * kWarpFloats;  // [2][S][16][kMmaDRow]
  float* s_L = s_D + 2 * S * 16 * kMmaDRow;            // [32][KP]
  uint4* ring = reinterpret_cast<uint4*>(s_D) + lane;  // [kMmaStages][NV][32 lanes], this lane's column
  for (int i = threadIdx.x; i < ((K * a.Cg + 3) & ~3) + KP; i += kMmaWarps * 32) smem[i] = 0.f;
  for (int i = threadIdx.x; i < K * 32; i += kMmaWarps * 32) {
    const int k = i / 32, cp = 2 * (i % 32);
    s_wp[i] = cp < a.Cg ? make_float2(a.weight[(size_t)k * a.Cg + cp] + ((a.conv_res && k == cp) ? 1.f : 0.f),
                                      a.weight[(size_t)k * a.Cg + cp + 1] + ((a.conv_res && k == cp + 1) ? 1.f : 0.f))
                        : make_float2(0.f, 0.f);
  }
  __syncthreads();

  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  const T* __restrict__ guide = static_cast<const T*>(a.guide);
  const T* __restrict__ value = static_cast<const T*>(a.value);
  const int g = lane >> 2, t4 = lane & 3;
  const bool params = a.dweight != nullptr || a.dbias != nullptr;
  // guide-channel pair of this lane in the dguide / dW phase
  const int c2 = 2 * lane;
  const bool has_pair = c2 < a.Cg;
  float2 wacc[K];
#pragma unroll
  for (int k = 0; k < K; ++k) wacc[k] = make_float2(0.f, 0.f);
  float bacc = 0.f;  // db[lane] for lane < K

  const int tw = (a.W + 7) / 8;
  const int64_t ntiles = (int64_t)a.B * a.H * tw;
  for (int64_t tile = (int64_t)blockIdx.x * kMmaWarps + warp; tile < ntiles;
       tile += (int64_t)gridDim.x * kMmaWarps) {
    const int tx = (int)(tile % tw);
    const int64_t rr = tile / tw;
    const int cy = (int)(rr % a.H), b = (int)(rr / a.H);
    const int cx0 = tx * 8;
    const T* db = dout + b * a.d_b;
    const T* vb = value + b * a.v_b;

    // ---- D_dy = dout_tile . V_window^T for every dy
    float acc[2][S][2][4];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
      for (int i = 0; i < S; ++i)
#pragma unroll
        for (int ni = 0; ni < 2; ++ni)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[mi][i][ni][q] = 0.f;
    int64_t aoff[2][2];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        aoff[mi][h] = (int64_t)(2 * cy + mi) * a.d_h + (int64_t)min(2 * cx0 + g + 8 * h, a.Wo - 1) * a.d_w + (CH / 4) * t4;
    int64_t bcol[2];
#pragma unroll
    for (int ni = 0; ni < 2; ++ni) bcol[ni] = (int64_t)clampi(cx0 - PN + 8 * ni + g, 0, a.W - 1) * a.v_w + (CH / 4) * t4;
    // chunk ring: each thread copies its own 16-byte vectors (A rows, B
    // columns per dy) kMmaStages - 1 chunks ahead and reads back only those,
    // so no other thread is waited for
    auto issue = [&](int chunk) {
      const int c0 = chunk * CH;
      uint4* dst = ring + (chunk % kMmaStages) * NV * 32;
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int h = 0; h < 2; ++h) bwd_cp_async16(dst + (2 * mi + h) * 32, db + aoff[mi][h] + c0);
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int64_t brow = (int64_t)clampi(cy + i - PN, 0, a.H - 1) * a.v_h + c0;
#pragma unroll
        for (int ni = 0; ni < 2; ++ni) bwd_cp_async16(dst + (4 + 2 * i + ni) * 32, vb + brow + bcol[ni]);
      }
    };
    const int nch = a.C / CH;
#pragma unroll
    for (int q = 0; q < kMmaStages - 1; ++q) {
      if (q < nch) issue(q);
      bwd_cp_async_commit();
    }
#pragma unroll 1
    for (int ch = 0; ch < nch; ++ch) {
      bwd_cp_async_wait<kMmaStages - 2>();  // chunk ch has landed
      if (ch + kMmaStages - 1 < nch) issue(ch + kMmaStages - 1);  // into the slot chunk ch - 1 used
      bwd_cp_async_commit();
      const uint4* src = ring + (ch % kMmaStages) * NV * 32;
      uint4 av[2][2];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int h = 0; h < 2; ++h) av[mi][h] = src[(2 * mi + h) * 32];
#pragma unroll
      for (int i = 0; i < S; ++i) {
        uint4 bv[2];
#pragma unroll
        for (int ni = 0; ni < 2; ++ni) bv[ni] = src[(4 + 2 * i + ni) * 32];
        if constexpr (kF32) {
          // words 0, 1 = channels 4t, 4t + 1 (low k half), words 2, 3 = 4t + 2, 4t + 3
          uint32_t ah[2][2][2], al[2][2][2], bh[2][2], bl[2][2];
#pragma unroll
          for (int mi = 0; mi < 2; ++mi)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int q = 0; q < 2; ++q)
                split_bf16x2(word(av[mi][h], 2 * q), word(av[mi][h], 2 * q + 1), ah[mi][h][q], al[mi][h][q]);
#pragma unroll
          for (int ni = 0; ni < 2; ++ni)
#pragma unroll
            for (int q = 0; q < 2; ++q) split_bf16x2(word(bv[ni], 2 * q), word(bv[ni], 2 * q + 1), bh[ni][q], bl[ni][q]);
#pragma unroll
          for (int mi = 0; mi < 2; ++mi)
#pragma unroll
            for (int ni = 0; ni < 2; ++ni) {
              mma16816<__nv_bfloat16>(acc[mi][i][ni], ah[mi][0][0], ah[mi][1][0], ah[mi][0][1], ah[mi][1][1],
                                      bh[ni][0], bh[ni][1]);
              mma16816<__nv_bfloat16>(acc[mi][i][ni], ah[mi][0][0], ah[mi][1][0], ah[mi][0][1], ah[mi][1][1],
                                      bl[ni][0], bl[ni][1]);
              mma16816<__nv_bfloat16>(acc[mi][i][ni], al[mi][0][0], al[mi][1][0], al[mi][0][1], al[mi][1][1],
                                      bh[ni][0], bh[ni][1]);
            }
        } else {
#pragma unroll
          for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
              for (int ni = 0; ni < 2; ++ni)
                mma16816<T>(acc[mi][i][ni], word(av[mi][0], 2 * s), word(av[mi][1], 2 * s),
                            word(av[mi][0], 2 * s + 1), word(av[mi][1], 2 * s + 1), word(bv[ni], 2 * s),
                            word(bv[ni], 2 * s + 1));
        }
      }
    }
    bwd_cp_async_wait<0>();
    __syncwarp();  // the ring area is rewritten as D below
    // stage D: thread holds rows g, g + 8 and columns 8 ni + 2 t4 + {0, 1}
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
      for (int i = 0; i < S; ++i)
#pragma unroll
        for (int ni = 0; ni < 2; ++ni) {
          float* row = s_D + ((mi * S + i) * 16 + g) * kMmaDRow + 8 * ni + 2 * t4;
          *reinterpret_cast<float2*>(row) = make_float2(acc[mi][i][ni][0], acc[mi][i][ni][1]);
          *reinterpret_cast<float2*>(row + 8 * kMmaDRow) = make_float2(acc[mi][i][ni][2], acc[mi][i][ni][3]);
        }
    __syncwarp();

    // ---- softmax backward, a lane per pixel (pixel = lane: child row
    // lane / 16, child column lane % 16 of the tile)
    {
      const int mi = lane >> 4, m = lane & 15, c = m >> 1;
      const bool valid = cx0 + c < a.W;
      const int x = min(2 * cx0 + m, a.Wo - 1), y = 2 * cy + mi;
      const float* pp = a.probs + (((int64_t)b * a.Ho + y) * a.Wo + x) * K;
      float pk[K], dP[K];
      float sdot = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        pk[k] = pp[k];
        dP[k] = s_D[((mi * S + a.dy[k] + PN) * 16 + m) * kMmaDRow + c + a.dx[k] + PN];
        sdot = fmaf(pk[k], dP[k], sdot);
      }
      float dlv[KP];
#pragma unroll
      for (int k = 0; k < KP; ++k) {
        const int kk = k < K ? k : K - 1;
        dlv[k] = (k < K && valid) ? pk[kk] * (dP[kk] - sdot) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < KP; k += 4)
        *reinterpret_cast<float4*>(s_L + lane * KP + k) = make_float4(dlv[k], dlv[k + 1], dlv[k + 2], dlv[k + 3]);
    }
    __syncwarp();

    // ---- dguide, dW, db: a lane per guide-channel pair, over the 32 pixels
    // (in two halves of 16 pixels, the guide pairs of a half loaded up front:
    // one latency per half)
    float2 wp[K];  // W' of this lane's channel pair
#pragma unroll
    for (int k = 0; k < K; ++k) wp[k] = s_wp[k * 32 + lane];
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      T2 gpre[16];
      if (params && has_pair) {
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int x = min(2 * cx0 + q, a.Wo - 1), y = 2 * cy + half;
          gpre[q] = *reinterpret_cast<const T2*>(guide + b * a.g_b + (int64_t)y * a.g_h + (int64_t)x * a.g_w + c2);
        }
      }
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const int p = 16 * half + q;
        if (cx0 + (q >> 1) >= a.W) continue;  // warp-uniform
        const int x = 2 * cx0 + q, y = 2 * cy + half;
        float dl[KP];
#pragma unroll
        for (int k = 0; k < KP; k += 4) {
          const float4 v4 = *reinterpret_cast<const float4*>(s_L + p * KP + k);
          dl[k] = v4.x; dl[k + 1] = v4.y; dl[k + 2] = v4.z; dl[k + 3] = v4.w;
        }
        if (has_pair) {
          if (a.dguide != nullptr) {
            float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < K; ++k) s2 = __ffma2_rn(make_float2(dl[k], dl[k]), wp[k], s2);
            T2 o2;
            o2.x = fromf<T>(s2.x);
            o2.y = fromf<T>(s2.y);
            *reinterpret_cast<T2*>(static_cast<T*>(a.dguide) + b * a.dg_b + (int64_t)y * a.dg_h +
                                   (int64_t)x * a.dg_w + c2) = o2;
          }
          if (params) {
            const float2 g2 = pair_to_float2(gpre[q]);
#pragma unroll
            for (int k = 0; k < K; ++k) wacc[k] = __ffma2_rn(make_float2(dl[k], dl[k]), g2, wacc[k]);
          }
        }
        if (params && lane < K) bacc += s_L[p * KP + lane];
      }
    }
    __syncwarp();  // s_D / s_L are rewritten by the next tile
  }
  if (!params) return;
  if (has_pair) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      atomicAdd(s_dw + k * a.Cg + c2, wacc[k].x);
      atomicAdd(s_dw + k * a.Cg + c2 + 1, wacc[k].y);
    }
  }
  if (lane < K) atomicAdd(s_db + lane, bacc);
  __syncthreads();
  for (int i = threadIdx.x; i < K * a.Cg; i += kMmaWarps * 32)
    if (a.dweight != nullptr) atomicAdd(a.dweight + i, s_dw[i]);
  if (a.dbias != nullptr && threadIdx.x < K) atomicAdd(a.dbias + threadIdx.x, s_db[threadIdx.x]);
}

struct Plan {
  int mma_pn;    // 1 or 2: tensor-core dlogit (dlogit_mma_kernel<PN>); 0: CUDA-core dlogit
  int dv_tc;     // 1: tensor-core dV (la_bwd_dv.cu)
  int dl_tc;     // 1: tensor-core softmax weights + dlogit (la_bwd_dl.cu) instead of probs + dlogit kernels
  int window;    // 1: sliding-window dV (reference offset table); 0: general dV kernel
  int seg_len;   // value columns per window thread
  int nseg;
};

template <typename T, int K, int CPT, int VEC, int GV>
int launch_cv(const Args& a, const Plan& plan, cudaStream_t stream) {
  const int64_t npix = (int64_t)a.B * a.Ho * a.Wo;
  if (npix == 0) return UPLIFT_LA_OK;
  const size_t smem_p = sizeof(float) * (size_t)a.Cg * K;
  const size_t smem_d = sizeof(float) * dlogit_smem_floats<K>(a.Cg);
  int dev = 0, optin = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return fail(UPLIFT_LA_ERR_CUDA, "device query failed");
  if (smem_d > (size_t)optin) return fail(UPLIFT_LA_ERR_SHAPE, "backward: Cg=%d needs too much shared memory", a.Cg);
  cudaError_t e = cudaFuncSetAttribute(probs_kernel<T, K, GV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_p);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(dlogit_kernel<T, K, CPT, VEC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_d);
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  bool dlogit_done = false;
  if (plan.dl_tc) {
    DlArgs d;
    d.dout = a.dout; d.d_b = a.d_b; d.d_h = a.d_h; d.d_w = a.d_w;
    d.guide = a.guide; d.g_b = a.g_b; d.g_h = a.g_h; d.g_w = a.g_w;
    d.value = a.value; d.v_b = a.v_b; d.v_h = a.v_h; d.v_w = a.v_w;
    d.weight = a.weight; d.bias = a.bias;
    d.probs = a.dvalue != nullptr ? a.probs : nullptr;
    d.dguide = a.dguide; d.dg_b = a.dg_b; d.dg_h = a.dg_h; d.dg_w = a.dg_w;
    d.dweight = a.dweight; d.dbias = a.dbias;
    d.B = a.B; d.Cg = a.Cg; d.C = a.C; d.H = a.H; d.W = a.W; d.I = a.I; d.K = K;
    d.dtype = std::is_same<T, __nv_bfloat16>::value ? UPLIFT_LA_BF16 : UPLIFT_LA_F16;
    d.conv_res = a.conv_res; d.hardmax = a.hardmax;
    for (int k = 0; k < K; ++k) { d.dy[k] = a.dy[k]; d.dx[k] = a.dx[k]; }
    const int rc = dl_tc_launch(d, stream);
    if (rc != UPLIFT_LA_OK) return rc;
    dlogit_done = true;
  } else {
    const int64_t pblocks = std::min<int64_t>((npix + kThreads - 1) / kThreads, (int64_t)sms * 16);
    probs_kernel<T, K, GV><<<(unsigned)pblocks, kThreads, smem_p, stream>>>(a);
  }
  if (!dlogit_done) {
    if (plan.mma_pn > 0 && (a.dguide != nullptr || a.dweight != nullptr || a.dbias != nullptr)) {
      auto kern = plan.mma_pn == 1 ? dlogit_mma_kernel<T, K, 1> : dlogit_mma_kernel<T, K, 2>;
      const size_t smem_m =
          sizeof(float) * (plan.mma_pn == 1 ? mma_smem_floats<K, 1>(a.Cg) : mma_smem_floats<K, 2>(a.Cg));
      if (smem_m > (size_t)optin) return fail(UPLIFT_LA_ERR_SHAPE, "backward: tensor-core dlogit smem");
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_m);
      if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      int occ = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kMmaWarps * 32, smem_m) != cudaSuccess || occ < 1)
        occ = 1;
      const int64_t tiles = (int64_t)a.B * a.H * ((a.W + 7) / 8);
      const int64_t mblocks = std::min<int64_t>((tiles + kMmaWarps - 1) / kMmaWarps, (int64_t)sms * occ);
      kern<<<(unsigned)mblocks, kMmaWarps * 32, smem_m, stream>>>(a);
      dlogit_done = true;
    }
  }
  if (!dlogit_done && (a.dguide != nullptr || a.dweight != nullptr || a.dbias != nullptr)) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, dlogit_kernel<T, K, CPT, VEC>, kDThreads, smem_d) !=
            cudaSuccess || occ < 1)
      occ = 1;
    const int64_t units = (int64_t)a.B * a.H * a.W * ((a.I * a.I) / CPT);
    const int64_t per_cta = (kDThreads / 32) * kSlots;
    const int64_t dblocks = std::min<int64_t>((units + per_cta - 1) / per_cta, (int64_t)sms * occ);
    dlogit_kernel<T, K, CPT, VEC><<<(unsigned)dblocks, kDThreads, smem_d, stream>>>(a);
  }
  if (a.dvalue != nullptr && a.B * (int64_t)a.H > 0) {
    if (plan.dv_tc) {
      DvArgs d;
      d.dout = a.dout; d.d_b = a.d_b; d.d_h = a.d_h; d.d_w = a.d_w;
      d.probs = a.probs;
      d.dvalue = a.dvalue; d.dv_b = a.dv_b; d.dv_h = a.dv_h; d.dv_w = a.dv_w;
      d.B = a.B; d.C = a.C; d.H = a.H; d.W = a.W; d.I = a.I; d.K = K;
      d.dtype = std::is_same<T, __nv_bfloat16>::value ? UPLIFT_LA_BF16 : UPLIFT_LA_F16;
      for (int k = 0; k < K; ++k) { d.dy[k] = a.dy[k]; d.dx[k] = a.dx[k]; }
      const int rc = dv_tc_launch(d, stream);
      if (rc != UPLIFT_LA_OK) return rc;
    } else if (plan.window) {
      const int64_t threads = (int64_t)a.B * a.H * plan.nseg * (a.C / VEC);
      const int64_t blocks = (threads + kThreads - 1) / kThreads;
      if (blocks >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "backward: grid too large");
      const unsigned nb = (unsigned)blocks;
      if (a.I == 2) dvalue_window_kernel<T, K, VEC, 2><<<nb, kThreads, 0, stream>>>(a, plan.seg_len, plan.nseg);
      else dvalue_window_kernel<T, K, VEC, 0><<<nb, kThreads, 0, stream>>>(a, plan.seg_len, plan.nseg);
    } else {
      if (a.B * (int64_t)a.H >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "backward: too many value rows");
      dvalue_kernel<T, K, VEC><<<(unsigned)(a.B * (int64_t)a.H), kThreads, 0, stream>>>(a);
    }
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "backward launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

// Children per dlogit unit: 4 for I = 2 and I = 4 (2 with ULA_BWD_CPT=2),
// 2 for other even I, else 1.  16-byte vectors when the channel counts and
// alignment allow them (vec: dout / value / dvalue; gvec: guide).
inline int unit_children(int I) {
  static const int env = [] {
    const char* s = getenv("ULA_BWD_CPT");
    return s != nullptr ? atoi(s) : 4;
  }();
  if (I % 2 != 0) return 1;
  return (env != 2 && (I == 2 || I == 4)) ? 4 : 2;
}

template <typename T, int K, int CPT, int VEC>
int launch_g(const Args& a, const Plan& plan, bool gvec, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  return gvec ? launch_cv<T, K, CPT, VEC, V>(a, plan, stream) : launch_cv<T, K, CPT, VEC, 1>(a, plan, stream);
}

template <typename T, int K, int VEC>
int launch_c(const Args& a, const Plan& plan, bool gvec, cudaStream_t stream) {
  switch (unit_children(a.I)) {
    case 4: return launch_g<T, K, 4, VEC>(a, plan, gvec, stream);
    case 2: return launch_g<T, K, 2, VEC>(a, plan, gvec, stream);
    default: return launch_g<T, K, 1, VEC>(a, plan, gvec, stream);
  }
}

template <typename T, int K>
int launch(const Args& a, const Plan& plan, bool vec, bool gvec, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  return vec ? launch_c<T, K, V>(a, plan, gvec, stream) : launch_c<T, K, 1>(a, plan, gvec, stream);
}

template <typename T>
int launch_k(const Args& a, const Plan& plan, int K, bool vec, bool gvec, cudaStream_t stream) {
  switch (K) {
    case 5: return launch<T, 5>(a, plan, vec, gvec, stream);
    case 9: return launch<T, 9>(a, plan, vec, gvec, stream);
    case 13: return launch<T, 13>(a, plan, vec, gvec, stream);
    case 17: return launch<T, 17>(a, plan, vec, gvec, stream);
    case 25: return launch<T, 25>(a, plan, vec, gvec, stream);
    default: return fail(UPLIFT_LA_ERR_SHAPE, "backward: K=%d unsupported (5, 9, 13, 17, 25)", K);
  }
}

extern template int launch_k<float>(const Args&, const Plan&, int, bool, bool, cudaStream_t);
extern template int launch_k<__nv_bfloat16>(const Args&, const Plan&, int, bool, bool, cudaStream_t);
extern template int launch_k<__half>(const Args&, const Plan&, int, bool, bool, cudaStream_t);

}  // namespace bwd
}  // namespace ula
