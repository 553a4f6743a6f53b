// CUDA-core Local Attender kernels for B200 (sm_100a): kernel templates
// shared by the per-storage-type instantiation units (la_simt_f32.cu,
// la_simt_bf16.cu, la_simt_f16.cu) and the host front end
// (local_attender.cu), which only sizes and launches them.
//
// Fused UPLiFT Local Attender forward.
//
// One launch computes, for every output pixel of a tile, the 1x1 logit
// projection of the guide (residual folded into the weights), the softmax
// over the K neighbour offsets and the softmax-weighted gather-sum of the
// C-channel value vectors of the parent cell's neighbours.  Reference
// semantics: LocalAttender.forward, uplift/uplift.py:801-847 (projection
// :810-812, replicate-padded neighbour gather :784-798 / :823, softmax over
// K :828, child mapping [B,D,H,I,W,I] :829-830, pooling :835-846).
//
// Work decomposition
//   unit  = CPT output pixels ("children") of one coarse cell that share the
//           K neighbour value vectors (CPT = 4: the 2x2 children of a cell
//           for I = 2, or one row of 4 children for I = 4; CPT = 1 else).
//   tile  = kTilePix output pixels = kTilePix / CPT units, processed by one
//           CTA in two phases:
//     A. logits: two threads per pixel split the guide channels, reduce with
//        one shuffle, add bias, softmax (fp32) -> shared memory.  The
//        per-unit neighbour offsets and output offsets are also staged.
//     B. pooling: a thread owns (unit, 16-byte channel vector); per offset
//        k it loads one value vector (coalesced NHWC, read-only path) and
//        accumulates CPT children with packed fp32 FMA (FFMA2).
//   The grid is persistent (a multiple of the SM count); the projection
//   weights are staged in shared memory once per CTA.  When there are fewer
//   tiles than resident CTAs, each tile is split into channel slices
//   (phase A is repeated per slice, phase B covers the slice's channels).
//
// Staged variant (STAGED, guide rows 16-byte aligned): phase A streams the
// guide through a cp.async ring of 128-byte-per-pixel chunks in shared
// memory (coalesced 128-byte row segments instead of one 16-byte load per
// pixel per thread) and computes the projection register-blocked: a thread
// owns P pixels x all K logits for a quarter (or half) of each chunk's
// channels, with packed FMAs over channel pairs; the partial logits are
// reduced across warps through the (then idle) ring.  For wide guides
// (SD-VAE: Cg = 512) the projection dominates and this path is what keeps
// the kernel near the HBM roofline.
//
// Storage is NHWC (channel stride 1); accumulation is fp32 throughout.

#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <string.h>

#include <algorithm>
#include <type_traits>

#include "uplift_la.h"

namespace ula {

constexpr int kThreads = 256;
constexpr int kTilePix = 128;          // output pixels per tile (2 threads each in phase A)
constexpr int kMaxK = UPLIFT_LA_MAX_K;

struct Params {
  const void* guide;  int64_t g_b, g_h, g_w;
  const void* logits; int64_t l_b, l_k, l_h, l_w;
  const void* value;  int64_t v_b, v_h, v_w;
  void* out;          int64_t o_b, o_h, o_w;
  const float* weight;
  const float* bias;
  int B, Cg, C, H, W, I;
  int conv_res, hardmax, from_logits, guide_vec;
  int units_per_cell;    // I*I / CPT
  int num_units;         // B*H*W*units_per_cell
  int num_tiles;
  int cslices;           // channel slices per tile (work items = num_tiles * cslices)
  int8_t dy[kMaxK];
  int8_t dx[kMaxK];
};

// ---------------------------------------------------------------- storage types
template <typename T> struct Elem;

template <> struct Elem<float> {
  static constexpr int kVec = 4;  // elements per 16-byte vector
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                      __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static float from_f(float x) { return x; }
};

template <> struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 bits.
  __device__ __forceinline__ static void unpack_word(uint32_t w, float& lo, float& hi) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    unpack_word(u.x, f[0], f[1]); unpack_word(u.y, f[2], f[3]);
    unpack_word(u.z, f[4], f[5]); unpack_word(u.w, f[6], f[7]);
  }
  __device__ __forceinline__ static uint32_t pack_word(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack_word(f[0], f[1]), pack_word(f[2], f[3]),
                      pack_word(f[4], f[5]), pack_word(f[6], f[7]));
  }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

template <> struct Elem<__half> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static void unpack_word(uint32_t w, float& lo, float& hi) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    float2 f = __half22float2(h);
    lo = f.x; hi = f.y;
  }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    unpack_word(u.x, f[0], f[1]); unpack_word(u.y, f[2], f[3]);
    unpack_word(u.z, f[4], f[5]); unpack_word(u.w, f[6], f[7]);
  }
  __device__ __forceinline__ static uint32_t pack_word(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack_word(f[0], f[1]), pack_word(f[2], f[3]),
                      pack_word(f[4], f[5]), pack_word(f[6], f[7]));
  }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};

__device__ __forceinline__ uint4 ldg_nc16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return min(max(v, lo), hi); }

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

// 16-byte global -> shared copy, zero-filled when src_bytes == 0 (no read).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Staged guide ring: kStages slots of kTilePix rows x kRowBytes.  Row r of a
// slot holds 8 16-byte units of one pixel's channel chunk; unit u is stored
// at slot (u ^ (r & 7)) so that 8 consecutive pixels reading the same unit
// hit 8 different bank groups.
constexpr int kStages = 4;
constexpr int kRowBytes = 128;
constexpr int kStageBytes = kTilePix * kRowBytes;

// Register blocking of the staged projection: P pixels per thread (two for
// K <= 17, one for K = 25 to bound the accumulators), kWarps / NCS groups of
// 32*P pixels, NCS channel splits (warps sharing pixels, distinct units).
template <int K>
struct StagedMap {
  static constexpr int P = K <= 17 ? 2 : 1;
  static constexpr int NPG = kTilePix / (32 * P);
  static constexpr int NCS = (kThreads / 32) / NPG;
  static constexpr int UPT = 8 / NCS;  // units per thread per chunk
  static_assert(NPG * NCS == kThreads / 32 && UPT * NCS == 8, "staged mapping");
};

// Shared-memory layout (floats / ints), sized on the host by smem_bytes().
template <int K, int CPT>
struct Smem {
  static constexpr int kKP = (K + 3) & ~3;        // padded logit count
  static constexpr int kUnits = kTilePix / CPT;
  // offsets in 4-byte words
  static constexpr int kP = 0;                               // [units][K][CPT] fp32 weights
  static constexpr int kNbr = kP + kUnits * K * CPT;         // [units][K] int32 value offsets
  static constexpr int kOut = (kNbr + kUnits * K + 1) & ~1;  // [units][CPT] int64 out offsets, then
                                                             // [kTilePix] int64 guide-row offsets (staged)
  static constexpr int kBias = kOut + 4 * kUnits * CPT;      // [kKP] (after out and staged guide-row offsets)
  static constexpr int kW = (kBias + kKP + 3) & ~3;          // [Cg][kKP] (projection only)
  static size_t bytes(int Cg, bool from_logits) {
    return 4 * (size_t)(kW + (from_logits ? 0 : Cg * kKP));
  }
  // staged variant: weights [Cgp / VE][K][VE] (Cgp = Cg rounded up to whole
  // chunks), then the guide ring (also holds the [NCS][K][kTilePix]
  // cross-warp reduction, which is smaller)
  __host__ __device__ static size_t ring_offset(int Cgp) { return ((4 * (size_t)(kW + Cgp * K)) + 127) & ~(size_t)127; }
  static size_t staged_bytes(int Cgp) { return ring_offset(Cgp) + (size_t)kStages * kStageBytes; }
  static_assert(StagedMap<K>::NCS * K * kTilePix * 4 <= kStages * kStageBytes, "reduction fits the ring");
};

// Output pixel `pix` of tile `tile` -> (batch, parent cell, pixel); false
// past the last unit.
template <int CPT>
__device__ __forceinline__ bool pixel_coords(const Params& p, int tile, int pix,
                                             int& b, int& cy, int& cx, int& y, int& x) {
  constexpr int NU = kTilePix / CPT;
  const int u = pix / CPT, t = pix - u * CPT;
  const int unit = tile * NU + u;
  if (unit >= p.num_units) return false;
  const int sub = unit % p.units_per_cell;
  const int cell = unit / p.units_per_cell;
  cx = cell % p.W;
  const int rest = cell / p.W;
  cy = rest % p.H;
  b = rest / p.H;
  const int ch = sub * CPT + t;
  const int ci = ch / p.I;
  y = cy * p.I + ci;
  x = cx * p.I + (ch - ci * p.I);
  return true;
}

template <typename T, int K, int CPT, bool VEC, bool STAGED>
__device__ __forceinline__ void la_fwd_body(const Params& p) {
  using E = Elem<T>;
  using S = Smem<K, CPT>;
  using SM = StagedMap<K>;
  constexpr int KP = S::kKP;
  constexpr int NU = S::kUnits;
  constexpr int V = VEC ? E::kVec : 1;
  constexpr int VE = E::kVec;               // elements per 16-byte unit
  constexpr int CH = kRowBytes / sizeof(T);  // channels per staged chunk

  extern __shared__ __align__(128) float smem[];
  float* s_p = smem + S::kP;
  int* s_nbr = reinterpret_cast<int*>(smem + S::kNbr);
  long long* s_out = reinterpret_cast<long long*>(smem + S::kOut);
  float* s_bias = smem + S::kBias;
  float* s_w = smem + S::kW;

  const int tid = threadIdx.x;
  const int nchunks = (p.Cg + CH - 1) / CH;
  char* ring = reinterpret_cast<char*>(smem) + (STAGED ? S::ring_offset(nchunks * CH) : 0);

  // Stage the projection once per CTA.  The residual guide[:, :K] of
  // residual_auto (uplift/uplift.py:26-39) is linear in the guide, so it is
  // folded into the weights: logit = (W + E) g + b with E[k][c] = (k == c).
  if (!p.from_logits) {
    if constexpr (STAGED) {
      // [c / VE][k][c % VE], zero past Cg
      const int n = nchunks * CH * K;
      for (int i = tid; i < n; i += kThreads) {
        const int e = i % VE, k = (i / VE) % K, c = (i / (VE * K)) * VE + e;
        float w = 0.f;
        if (c < p.Cg) {
          w = p.weight[(size_t)k * p.Cg + c];
          if (p.conv_res && k == c) w += 1.f;
        }
        s_w[i] = w;
      }
    } else {
      for (int i = tid; i < p.Cg * KP; i += kThreads) {
        const int c = i / KP, k = i - c * KP;
        float w = 0.f;
        if (k < K) {
          w = p.weight[(size_t)k * p.Cg + c];
          if (p.conv_res && k == c) w += 1.f;
        }
        s_w[i] = w;
      }
    }
    for (int k = tid; k < KP; k += kThreads)
      s_bias[k] = (p.bias != nullptr && k < K) ? p.bias[k] : 0.f;
  }

  const T* __restrict__ gbase = static_cast<const T*>(p.guide);
  const T* __restrict__ lbase = static_cast<const T*>(p.logits);
  const T* __restrict__ vbase = static_cast<const T*>(p.value);
  T* __restrict__ obase = static_cast<T*>(p.out);

  const int num_work = p.num_tiles * p.cslices;
  for (int work = blockIdx.x; work < num_work; work += gridDim.x) {
    const int tile = work / p.cslices;
    const int slice = work - tile * p.cslices;
    __syncthreads();  // previous tile's phase B is done with shared memory

    // ------------------------------------------------- phase A, staged guide
    if constexpr (STAGED) {
      // guide row offset of every pixel of the tile (-1: past the end)
      long long* s_grow = s_out + NU * CPT;
      if (tid < kTilePix) {
        int b, cy, cx, y, x;
        s_grow[tid] = pixel_coords<CPT>(p, tile, tid, b, cy, cx, y, x) ? b * p.g_b + y * p.g_h + x * p.g_w : -1;
      }
      __syncthreads();
      // copy roles: thread copies unit (tid & 7) of pixel rows (tid >> 3) + 32 j
      const int cu = tid & 7;
      auto issue = [&](int chunk, int slot) {
        const int c0 = chunk * CH + cu * VE;
        const uint32_t sbase = smem_u32(ring + slot * kStageBytes);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = (tid >> 3) + 32 * j;
          const long long off = s_grow[r];
          const bool ok = off >= 0 && c0 < p.Cg;
          cp_async16(sbase + r * kRowBytes + ((cu ^ (r & 7)) << 4), ok ? (const void*)(gbase + off + c0) : p.guide,
                     ok ? 16 : 0);
        }
      };

      const int warp = tid >> 5, lane = tid & 31;
      const int cs = warp % SM::NCS;
      const int pbase = (warp / SM::NCS) * 32 * SM::P + lane;
      float2 acc[SM::P][K];
#pragma unroll
      for (int i = 0; i < SM::P; ++i)
#pragma unroll
        for (int k = 0; k < K; ++k) acc[i][k] = make_float2(0.f, 0.f);

#pragma unroll
      for (int st = 0; st < kStages - 1; ++st) {
        if (st < nchunks) issue(st, st);
        cp_async_commit();
      }
      for (int chunk = 0; chunk < nchunks; ++chunk) {
        cp_async_wait<kStages - 2>();
        __syncthreads();  // chunk landed for every thread; slot (chunk - 1) % kStages is free
        if (chunk + kStages - 1 < nchunks) issue(chunk + kStages - 1, (chunk + kStages - 1) % kStages);
        cp_async_commit();
        const char* stage = ring + (chunk % kStages) * kStageBytes;
#pragma unroll
        for (int j = 0; j < SM::UPT; ++j) {
          const int u = cs + j * SM::NCS;
          float g[SM::P][VE];
#pragma unroll
          for (int i = 0; i < SM::P; ++i) {
            const int r = pbase + 32 * i;
            E::unpack(*reinterpret_cast<const uint4*>(stage + r * kRowBytes + ((u ^ (r & 7)) << 4)), g[i]);
          }
          const float* wu = s_w + (chunk * 8 + u) * K * VE;
#pragma unroll
          for (int k = 0; k < K; ++k) {
#pragma unroll
            for (int e4 = 0; e4 < VE; e4 += 4) {
              const float4 w4 = *reinterpret_cast<const float4*>(wu + k * VE + e4);
#pragma unroll
              for (int i = 0; i < SM::P; ++i) {
                acc[i][k] = __ffma2_rn(make_float2(g[i][e4], g[i][e4 + 1]), make_float2(w4.x, w4.y), acc[i][k]);
                acc[i][k] = __ffma2_rn(make_float2(g[i][e4 + 2], g[i][e4 + 3]), make_float2(w4.z, w4.w), acc[i][k]);
              }
            }
          }
        }
      }
      __syncthreads();  // every warp is done reading the ring
      float* red = reinterpret_cast<float*>(ring);  // [NCS][K][kTilePix]
#pragma unroll
      for (int i = 0; i < SM::P; ++i)
#pragma unroll
        for (int k = 0; k < K; ++k) red[(cs * K + k) * kTilePix + pbase + 32 * i] = acc[i][k].x + acc[i][k].y;
      __syncthreads();
    }

    // ------------------------------------------------------------ phase A
    {
      const int pix = tid >> 1, half = tid & 1;
      const int u = pix / CPT, t = pix - u * CPT;
      int b = 0, cy = 0, cx = 0, y = 0, x = 0;
      const bool valid = pixel_coords<CPT>(p, tile, pix, b, cy, cx, y, x);

      float logit[K];
#pragma unroll
      for (int k = 0; k < K; ++k) logit[k] = 0.f;

      if constexpr (STAGED) {
        const float* red = reinterpret_cast<const float*>(ring);
#pragma unroll
        for (int k = 0; k < K; ++k) {
          float a = 0.f;
#pragma unroll
          for (int c = 0; c < SM::NCS; ++c) a += red[(c * K + k) * kTilePix + pix];
          logit[k] = a + s_bias[k];
        }
      } else if (p.from_logits) {
        if (valid && half == 0) {
          const T* lp = lbase + b * p.l_b + y * p.l_h + x * p.l_w;
#pragma unroll
          for (int k = 0; k < K; ++k) logit[k] = E::to_f(lp[k * p.l_k]);
        }
      } else {
        if (valid) {
          const T* gp = gbase + b * p.g_b + y * p.g_h + x * p.g_w;
          if (p.guide_vec) {
            for (int c0 = half * E::kVec; c0 < p.Cg; c0 += 2 * E::kVec) {
              float g[E::kVec];
              E::unpack(ldg_nc16(gp + c0), g);
#pragma unroll
              for (int e = 0; e < E::kVec; ++e) {
                const float* wr = s_w + (c0 + e) * KP;
#pragma unroll
                for (int k4 = 0; k4 < KP; k4 += 4) {
                  const float4 w4 = *reinterpret_cast<const float4*>(wr + k4);
                  if (k4 + 0 < K) logit[k4 + 0] = fmaf(w4.x, g[e], logit[k4 + 0]);
                  if (k4 + 1 < K) logit[k4 + 1] = fmaf(w4.y, g[e], logit[k4 + 1]);
                  if (k4 + 2 < K) logit[k4 + 2] = fmaf(w4.z, g[e], logit[k4 + 2]);
                  if (k4 + 3 < K) logit[k4 + 3] = fmaf(w4.w, g[e], logit[k4 + 3]);
                }
              }
            }
          } else {
            for (int c = half; c < p.Cg; c += 2) {
              const float g = E::to_f(gp[c]);
              const float* wr = s_w + c * KP;
#pragma unroll
              for (int k = 0; k < K; ++k) logit[k] = fmaf(wr[k], g, logit[k]);
            }
          }
        }
        // combine the two channel halves (all lanes participate)
#pragma unroll
        for (int k = 0; k < K; ++k) logit[k] += __shfl_xor_sync(0xffffffffu, logit[k], 1);
#pragma unroll
        for (int k = 0; k < K; ++k) logit[k] += s_bias[k];
      }

      if (half == 0) {
        float* pw = s_p + u * K * CPT + t;
        if (!valid) {
#pragma unroll
          for (int k = 0; k < K; ++k) pw[k * CPT] = 0.f;
        } else if (p.hardmax) {
          // one-hot of the first maximal logit (torch argmax tie rule)
          int best = 0;
          float bv = logit[0];
#pragma unroll
          for (int k = 1; k < K; ++k)
            if (logit[k] > bv) { bv = logit[k]; best = k; }
#pragma unroll
          for (int k = 0; k < K; ++k) pw[k * CPT] = (k == best) ? 1.f : 0.f;
        } else {
          float m = logit[0];
#pragma unroll
          for (int k = 1; k < K; ++k) m = fmaxf(m, logit[k]);
          float s = 0.f;
#pragma unroll
          for (int k = 0; k < K; ++k) { logit[k] = __expf(logit[k] - m); s += logit[k]; }
          const float inv = 1.f / s;
#pragma unroll
          for (int k = 0; k < K; ++k) pw[k * CPT] = logit[k] * inv;
        }
        // per-unit neighbour offsets (replicate padding == clamping) and
        // per-child output offsets
        if (valid) {
          if (t == 0) {
#pragma unroll
            for (int k = 0; k < K; ++k) {
              const int ny = clampi(cy + p.dy[k], 0, p.H - 1);
              const int nx = clampi(cx + p.dx[k], 0, p.W - 1);
              s_nbr[u * K + k] = (int)(ny * p.v_h + nx * p.v_w);
            }
          }
          s_out[u * CPT + t] = b * p.o_b + y * p.o_h + x * p.o_w;
        }
      }
    }
    __syncthreads();

    // ------------------------------------------------------------ phase B
    {
      const int NG = p.C / V;
      const int g0 = (int)((int64_t)slice * NG / p.cslices);
      const int ns = (int)((int64_t)(slice + 1) * NG / p.cslices) - g0;
      const int tile_units = min(NU, p.num_units - tile * NU);
      const int items = tile_units * ns;
      for (int it = tid; it < items; it += kThreads) {
        const int u = it / ns;
        const int gi = g0 + (it - u * ns);
        const int unit = tile * NU + u;
        const int b = (unit / p.units_per_cell) / (p.H * p.W);
        const T* vb = vbase + b * p.v_b + gi * V;
        const int* nb = s_nbr + u * K;
        const float* pw = s_p + u * K * CPT;

        if constexpr (V >= 2) {
          float2 acc[CPT][V / 2];
#pragma unroll
          for (int t = 0; t < CPT; ++t)
#pragma unroll
            for (int e = 0; e < V / 2; ++e) acc[t][e] = make_float2(0.f, 0.f);
#pragma unroll
          for (int k = 0; k < K; ++k) {
            float v[V];
            E::unpack(ldg_nc16(vb + nb[k]), v);
            float pk[CPT];
            if constexpr (CPT == 4) {
              const float4 q = *reinterpret_cast<const float4*>(pw + k * CPT);
              pk[0] = q.x; pk[1] = q.y; pk[2] = q.z; pk[3] = q.w;
            } else {
#pragma unroll
              for (int t = 0; t < CPT; ++t) pk[t] = pw[k * CPT + t];
            }
#pragma unroll
            for (int t = 0; t < CPT; ++t) {
              const float2 pp = make_float2(pk[t], pk[t]);
#pragma unroll
              for (int e = 0; e < V / 2; ++e)
                acc[t][e] = __ffma2_rn(make_float2(v[2 * e], v[2 * e + 1]), pp, acc[t][e]);
            }
          }
#pragma unroll
          for (int t = 0; t < CPT; ++t) {
            float o[V];
#pragma unroll
            for (int e = 0; e < V / 2; ++e) { o[2 * e] = acc[t][e].x; o[2 * e + 1] = acc[t][e].y; }
            T* op = obase + s_out[u * CPT + t] + gi * V;
            *reinterpret_cast<uint4*>(op) = E::pack(o);
          }
        } else {
          float acc[CPT];
#pragma unroll
          for (int t = 0; t < CPT; ++t) acc[t] = 0.f;
#pragma unroll
          for (int k = 0; k < K; ++k) {
            const float v = E::to_f(vb[nb[k]]);
#pragma unroll
            for (int t = 0; t < CPT; ++t) acc[t] = fmaf(pw[k * CPT + t], v, acc[t]);
          }
#pragma unroll
          for (int t = 0; t < CPT; ++t) obase[s_out[u * CPT + t] + gi] = E::from_f(acc[t]);
        }
      }
    }
  }
}

// Two entry points over one body: the per-pixel variant keeps the
// compiler's register choice (about 70, three CTAs per SM); the staged
// variant is held to 128 registers so that two CTAs share an SM and one's
// pooling overlaps the other's projection.
template <typename T, int K, int CPT, bool VEC>
__global__ void __launch_bounds__(kThreads) la_fwd_kernel(const __grid_constant__ Params p) {
  la_fwd_body<T, K, CPT, VEC, false>(p);
}

template <typename T, int K, int CPT, bool VEC>
__global__ void __launch_bounds__(kThreads, 2) la_fwd_staged_kernel(const __grid_constant__ Params p) {
  la_fwd_body<T, K, CPT, VEC, true>(p);
}

using KernelFn = void (*)(Params);

template <typename T, int K, int CPT>
KernelFn pick_vec(bool vec, bool staged) {
  if (staged) return vec ? la_fwd_staged_kernel<T, K, CPT, true> : la_fwd_staged_kernel<T, K, CPT, false>;
  return vec ? la_fwd_kernel<T, K, CPT, true> : la_fwd_kernel<T, K, CPT, false>;
}

template <typename T, int K>
KernelFn pick_cpt(int cpt, bool vec, bool staged) {
  return cpt == 4 ? pick_vec<T, K, 4>(vec, staged) : pick_vec<T, K, 1>(vec, staged);
}

template <typename T>
KernelFn pick_k(int K, int cpt, bool vec, bool staged) {
  switch (K) {
    case 5: return pick_cpt<T, 5>(cpt, vec, staged);
    case 9: return pick_cpt<T, 9>(cpt, vec, staged);
    case 13: return pick_cpt<T, 13>(cpt, vec, staged);
    case 17: return pick_cpt<T, 17>(cpt, vec, staged);
    case 25: return pick_cpt<T, 25>(cpt, vec, staged);
    default: return nullptr;
  }
}

// Kernel for one storage type (defined in la_simt_<type>.cu); nullptr for
// an unsupported K.
KernelFn simt_kernel_f32(int K, int cpt, bool vec, bool staged);
KernelFn simt_kernel_bf16(int K, int cpt, bool vec, bool staged);
KernelFn simt_kernel_f16(int K, int cpt, bool vec, bool staged);

}  // namespace ula
