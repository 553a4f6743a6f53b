// Fused UPLiFT Local Attender forward for B200 (sm_100a).
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
#include "la_internal.h"

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

// ---------------------------------------------------------------- host side
thread_local char g_err[512] = "";
thread_local int g_last_kernel = 0;
int g_policy = UPLIFT_LA_POLICY_AUTO;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

using KernelFn = void (*)(Params);

// Guides at least this wide take the staged projection (measured on B200:
// it wins once the projection is a large share of the work).
#ifndef ULA_STAGED_MIN_CG
#define ULA_STAGED_MIN_CG 128
#endif
constexpr int kStagedMinCg = ULA_STAGED_MIN_CG;
// fp32 guides at least this wide take the tensor-core projection under AUTO.
constexpr int kWideMinCg = 128;

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

// Shared memory of one CTA; `es` = element size (the staged ring holds
// 128-byte chunks, so its weight table is padded to whole chunks).
size_t smem_for(int K, int cpt, int Cg, bool from_logits, bool staged, int es) {
  const int ch = kRowBytes / es;
  const int cgp = (Cg + ch - 1) / ch * ch;
  auto f = [&](auto kk, auto cc) {
    using SS = Smem<decltype(kk)::value, decltype(cc)::value>;
    return staged ? SS::staged_bytes(cgp) : SS::bytes(Cg, from_logits);
  };
  using I1 = std::integral_constant<int, 1>;
  using I4 = std::integral_constant<int, 4>;
#define ULA_SM(KV)                                                          \
  case KV:                                                                  \
    return cpt == 4 ? f(std::integral_constant<int, KV>{}, I4{})            \
                    : f(std::integral_constant<int, KV>{}, I1{});
  switch (K) {
    ULA_SM(5) ULA_SM(9) ULA_SM(13) ULA_SM(17) ULA_SM(25)
    default: return 0;
  }
#undef ULA_SM
}

size_t elem_size(int dtype) { return dtype == UPLIFT_LA_F32 ? 4 : 2; }

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

struct DevInfo {
  int sms = 0;
  size_t max_smem_optin = 0;
};

int device_info(DevInfo* info) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_NO_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
  static DevInfo cache[64];
  if (dev < 64 && cache[dev].sms > 0) { *info = cache[dev]; return UPLIFT_LA_OK; }
  int sms = 0, major = 0, optin = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
  if (major != 10) return fail(UPLIFT_LA_ERR_NO_DEVICE, "device %d has compute capability %d.x; this build targets sm_100a", dev, major);
  info->sms = sms;
  info->max_smem_optin = (size_t)optin;
  if (dev < 64) cache[dev] = *info;
  return UPLIFT_LA_OK;
}

int launch(const Params& p0, int dtype, int K, int cpt, bool vec, bool staged, size_t smem, cudaStream_t stream) {
  Params p = p0;
  if (p.num_units == 0) return UPLIFT_LA_OK;  // empty input: nothing to do
  KernelFn fn = nullptr;
  switch (dtype) {
    case UPLIFT_LA_F32: fn = pick_k<float>(K, cpt, vec, staged); break;
    case UPLIFT_LA_BF16: fn = pick_k<__nv_bfloat16>(K, cpt, vec, staged); break;
    case UPLIFT_LA_F16: fn = pick_k<__half>(K, cpt, vec, staged); break;
    default: return fail(UPLIFT_LA_ERR_ARG, "unknown dtype %d", dtype);
  }
  if (fn == nullptr) return fail(UPLIFT_LA_ERR_SHAPE, "K=%d unsupported (5, 9, 13, 17, 25)", K);

  DevInfo info;
  int rc = device_info(&info);
  if (rc != UPLIFT_LA_OK) return rc;
  if (smem > info.max_smem_optin)
    return fail(UPLIFT_LA_ERR_SHAPE, "guide channels Cg=%d need %zu B of shared memory (max %zu)", p.Cg, smem, info.max_smem_optin);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem);
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "occupancy query: %s", cudaGetErrorString(e));
  if (per_sm < 1) per_sm = 1;
  const int64_t resident = (int64_t)info.sms * per_sm;
  // Fewer tiles than resident CTAs: split each tile's channels into slices
  // (at least 8 vectors each) unless the repeated projection would cost more
  // than the pooling it spreads.
  p.cslices = 1;
  const int ng = vec ? p.C / (16 / (int)elem_size(dtype)) : p.C;
  if (p.num_tiles < resident && (p.from_logits || p.Cg <= p.C)) {
    const int64_t want = (resident + p.num_tiles - 1) / p.num_tiles;
    p.cslices = (int)std::max<int64_t>(1, std::min<int64_t>(want, ng / 8));
  }
  const int grid = (int)std::min<int64_t>((int64_t)p.num_tiles * p.cslices, resident);
  fn<<<grid, kThreads, smem, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

// Strides of size-1 dimensions are arbitrary in torch (a [1, C, 1, 1]
// tensor may report any); replace them with the dense value so alignment
// checks and tensor maps see a canonical NHWC layout.  s = {b, c, h, w}.
void canon_strides(int64_t* s, int C, int H, int W, int B) {
  if (W == 1) s[3] = C;
  if (H == 1) s[2] = s[3] * W;
  if (B == 1) s[0] = s[2] * H;
}

int check_common(const void* value, const int64_t* vs_in, void* out, const int64_t* os_in,
                 int B, int C, int H, int W, int I, int K, const int8_t* offsets, int pn, int dtype,
                 Params* p, int* cpt, bool* vec) {
  if (dtype != UPLIFT_LA_F32 && dtype != UPLIFT_LA_BF16 && dtype != UPLIFT_LA_F16)
    return fail(UPLIFT_LA_ERR_ARG, "unknown dtype %d", dtype);
  if (vs_in == nullptr || os_in == nullptr || offsets == nullptr)
    return fail(UPLIFT_LA_ERR_ARG, "null stride or offset array");
  int64_t vs[4] = {vs_in[0], vs_in[1], vs_in[2], vs_in[3]};
  int64_t os[4] = {os_in[0], os_in[1], os_in[2], os_in[3]};
  canon_strides(vs, C, H, W, B);
  canon_strides(os, C, I * H, I * W, B);
  if (B < 0 || C < 1 || H < 0 || W < 0 || I < 1)
    return fail(UPLIFT_LA_ERR_SHAPE, "bad sizes B=%d C=%d H=%d W=%d I=%d", B, C, H, W, I);
  if (K < 1 || K > kMaxK) return fail(UPLIFT_LA_ERR_SHAPE, "K=%d out of range", K);
  if (pn < 0 || pn > UPLIFT_LA_MAX_PN) return fail(UPLIFT_LA_ERR_OFFSETS, "pn=%d out of range", pn);
  for (int k = 0; k < K; ++k) {
    const int dy = offsets[2 * k], dx = offsets[2 * k + 1];
    if (dy < -pn || dy > pn || dx < -pn || dx > pn)
      return fail(UPLIFT_LA_ERR_OFFSETS, "offset %d = (%d, %d) exceeds pn=%d", k, dy, dx, pn);
    p->dy[k] = (int8_t)dy;
    p->dx[k] = (int8_t)dx;
  }
  if (vs[1] != 1 || os[1] != 1)
    return fail(UPLIFT_LA_ERR_LAYOUT, "value and out need channel stride 1 (channels_last), got %lld / %lld",
                (long long)vs[1], (long long)os[1]);
  const int64_t units64 = (int64_t)B * H * W;
  int upc;
  if (I == 1) { *cpt = 1; upc = 1; }
  else if (I == 2) { *cpt = 4; upc = 1; }
  else if (I == 4) { *cpt = 4; upc = 4; }
  else { *cpt = 1; upc = I * I; }
  if (units64 * upc >= ((int64_t)1 << 31))
    return fail(UPLIFT_LA_ERR_SHAPE, "too many cells (%lld)", (long long)(units64 * upc));
  if ((int64_t)(H > 0 ? H - 1 : 0) * vs[2] + (int64_t)(W > 0 ? W - 1 : 0) * vs[3] + C >= ((int64_t)1 << 31))
    return fail(UPLIFT_LA_ERR_SHAPE, "one value image exceeds 2^31 elements");
  if (B > 0 && H > 0 && W > 0) {
    if (value == nullptr || out == nullptr) return fail(UPLIFT_LA_ERR_ARG, "null value/out pointer");
  }
  const size_t es = elem_size(dtype);
  const int vec_elems = 16 / (int)es;
  *vec = (C % vec_elems == 0) && aligned16(value) && aligned16(out) &&
         (vs[0] % vec_elems == 0) && (vs[2] % vec_elems == 0) && (vs[3] % vec_elems == 0) &&
         (os[0] % vec_elems == 0) && (os[2] % vec_elems == 0) && (os[3] % vec_elems == 0);
  p->value = value; p->v_b = vs[0]; p->v_h = vs[2]; p->v_w = vs[3];
  p->out = out; p->o_b = os[0]; p->o_h = os[2]; p->o_w = os[3];
  p->B = B; p->C = C; p->H = H; p->W = W; p->I = I;
  p->units_per_cell = upc;
  p->num_units = (int)(units64 * upc);
  const int nu = kTilePix / *cpt;
  p->num_tiles = (p->num_units + nu - 1) / nu;
  return UPLIFT_LA_OK;
}

}  // namespace ula

extern "C" {

int uplift_la_forward(const void* guide, const int64_t guide_strides[4],
                      const void* value, const int64_t value_strides[4],
                      const float* weight, const float* bias,
                      void* out, const int64_t out_strides[4],
                      int B, int Cg, int C, int H, int W, int I, int K,
                      const int8_t* offsets, int pn, int conv_res,
                      int dtype, int hardmax, void* stream) {
  using namespace ula;
  Params p;
  memset(&p, 0, sizeof(p));
  int cpt = 1;
  bool vec = false;
  int rc = check_common(value, value_strides, out, out_strides, B, C, H, W, I, K, offsets, pn, dtype, &p, &cpt, &vec);
  if (rc != UPLIFT_LA_OK) return rc;
  if (guide_strides == nullptr) return fail(UPLIFT_LA_ERR_ARG, "null guide strides");
  if (Cg < 1) return fail(UPLIFT_LA_ERR_SHAPE, "Cg=%d", Cg);
  if (guide_strides[1] != 1)
    return fail(UPLIFT_LA_ERR_LAYOUT, "guide needs channel stride 1 (channels_last), got %lld", (long long)guide_strides[1]);
  if (p.num_units > 0 && (guide == nullptr || weight == nullptr))
    return fail(UPLIFT_LA_ERR_ARG, "null guide/weight pointer");
  const int gv = 16 / (int)elem_size(dtype);
  int64_t gs[4] = {guide_strides[0], guide_strides[1], guide_strides[2], guide_strides[3]};
  canon_strides(gs, Cg, I * H, I * W, B);
  p.guide = guide;
  p.g_b = gs[0]; p.g_h = gs[2]; p.g_w = gs[3];
  p.guide_vec = (Cg % gv == 0) && aligned16(guide) && p.g_b % gv == 0 && p.g_h % gv == 0 && p.g_w % gv == 0;
  p.weight = weight;
  p.bias = bias;
  p.Cg = Cg;
  p.conv_res = conv_res ? 1 : 0;
  p.hardmax = hardmax ? 1 : 0;
  p.from_logits = 0;
  if (p.num_units == 0) return UPLIFT_LA_OK;

  const int policy = __atomic_load_n(&g_policy, __ATOMIC_RELAXED);
  if (policy != UPLIFT_LA_POLICY_SIMT && I == 2) {
    TcArgs a;
    a.guide = guide; a.g_b = p.g_b; a.g_h = p.g_h; a.g_w = p.g_w;
    a.value = value; a.v_b = p.v_b; a.v_h = p.v_h; a.v_w = p.v_w;
    a.out = out; a.o_b = p.o_b; a.o_h = p.o_h; a.o_w = p.o_w;
    a.weight = weight; a.bias = bias;
    a.B = B; a.Cg = Cg; a.C = C; a.H = H; a.W = W; a.K = K; a.pn = pn;
    a.conv_res = p.conv_res; a.hardmax = p.hardmax; a.dtype = dtype; a.offsets = offsets;
    const char* why = nullptr;
    if (tc_eligible(a, &why)) {
      rc = tc_launch(a, static_cast<cudaStream_t>(stream));
      if (rc == UPLIFT_LA_OK) g_last_kernel = UPLIFT_LA_KERNEL_TENSOR_CORE;
      return rc;
    }
    // The wide-guide kernel (two-term bf16 split, ~1e-5 relative) pays off
    // where the projection dominates; narrower fp32 guides keep the
    // CUDA-core kernel's fp32 arithmetic unless the tensor cores are asked for.
    const char* why_w = nullptr;
    if (tcw_eligible(a, &why_w) && (policy == UPLIFT_LA_POLICY_TENSOR_CORE || Cg >= kWideMinCg)) {
      rc = tcw_launch(a, static_cast<cudaStream_t>(stream));
      if (rc == UPLIFT_LA_OK) g_last_kernel = UPLIFT_LA_KERNEL_TENSOR_CORE_WIDE;
      return rc;
    }
    if (dtype == UPLIFT_LA_F32) why = why_w;
    if (policy == UPLIFT_LA_POLICY_TENSOR_CORE)
      return fail(UPLIFT_LA_ERR_SHAPE, "tensor-core kernel required but not applicable: %s", why);
  } else if (policy == UPLIFT_LA_POLICY_TENSOR_CORE) {
    return fail(UPLIFT_LA_ERR_SHAPE, "tensor-core kernel required but not applicable: scale I=%d != 2", I);
  }
  const bool staged = p.guide_vec && Cg >= kStagedMinCg;
  const size_t smem = smem_for(K, cpt, Cg, false, staged, (int)elem_size(dtype));
  if (smem == 0) return fail(UPLIFT_LA_ERR_SHAPE, "K=%d unsupported (5, 9, 13, 17, 25)", K);
  rc = launch(p, dtype, K, cpt, vec, staged, smem, static_cast<cudaStream_t>(stream));
  if (rc == UPLIFT_LA_OK) g_last_kernel = staged ? UPLIFT_LA_KERNEL_SIMT_STAGED : UPLIFT_LA_KERNEL_SIMT;
  return rc;
}

int uplift_la_pool(const void* logits, const int64_t logits_strides[4],
                   const void* value, const int64_t value_strides[4],
                   void* out, const int64_t out_strides[4],
                   int B, int C, int H, int W, int I, int K,
                   const int8_t* offsets, int pn,
                   int dtype, int hardmax, void* stream) {
  using namespace ula;
  Params p;
  memset(&p, 0, sizeof(p));
  int cpt = 1;
  bool vec = false;
  int rc = check_common(value, value_strides, out, out_strides, B, C, H, W, I, K, offsets, pn, dtype, &p, &cpt, &vec);
  if (rc != UPLIFT_LA_OK) return rc;
  if (logits_strides == nullptr) return fail(UPLIFT_LA_ERR_ARG, "null logits strides");
  if (p.num_units > 0 && logits == nullptr) return fail(UPLIFT_LA_ERR_ARG, "null logits pointer");
  p.logits = logits;
  p.l_b = logits_strides[0]; p.l_k = logits_strides[1]; p.l_h = logits_strides[2]; p.l_w = logits_strides[3];
  p.hardmax = hardmax ? 1 : 0;
  p.from_logits = 1;
  const size_t smem = smem_for(K, cpt, 0, true, false, (int)elem_size(dtype));
  if (smem == 0) return fail(UPLIFT_LA_ERR_SHAPE, "K=%d unsupported (5, 9, 13, 17, 25)", K);
  rc = launch(p, dtype, K, cpt, vec, false, smem, static_cast<cudaStream_t>(stream));
  if (rc == UPLIFT_LA_OK && p.num_units > 0) g_last_kernel = UPLIFT_LA_KERNEL_SIMT;
  return rc;
}

int uplift_la_set_kernel_policy(int policy) {
  if (policy != UPLIFT_LA_POLICY_AUTO && policy != UPLIFT_LA_POLICY_SIMT && policy != UPLIFT_LA_POLICY_TENSOR_CORE)
    return ula::fail(UPLIFT_LA_ERR_ARG, "unknown kernel policy %d", policy);
  __atomic_store_n(&ula::g_policy, policy, __ATOMIC_RELAXED);
  return UPLIFT_LA_OK;
}

int uplift_la_last_kernel(void) { return ula::g_last_kernel; }

int uplift_la_device_status(int clear) {
  const int a = ula::tc_device_status(clear != 0);
  const int b = ula::tcw_device_status(clear != 0);
  if (a < 0 || b < 0) return -1;
  return a != 0 ? a : b;
}

int uplift_la_test_hook(int fault, unsigned long long wait_limit_ns) {
  return ula::tc_set_test_hook(fault, wait_limit_ns);
}

const char* uplift_la_last_error(void) { return ula::g_err; }

const char* uplift_la_status_string(int status) {
  switch (status) {
    case UPLIFT_LA_OK: return "ok";
    case UPLIFT_LA_ERR_ARG: return "invalid argument";
    case UPLIFT_LA_ERR_SHAPE: return "unsupported or inconsistent shape";
    case UPLIFT_LA_ERR_LAYOUT: return "unsupported layout";
    case UPLIFT_LA_ERR_OFFSETS: return "bad neighbour offsets";
    case UPLIFT_LA_ERR_CUDA: return "CUDA error";
    case UPLIFT_LA_ERR_NO_DEVICE: return "no usable sm_100 device";
    default: return "unknown status";
  }
}

int uplift_la_abi_version(void) { return (1 << 16) | 1; }

}  // extern "C"
