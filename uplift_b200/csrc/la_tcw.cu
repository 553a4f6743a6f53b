// Tensor-core projection for wide fp32 guides (B200, sm_100a).
//
// The SD1.5-VAE attender projects Cg = 512 fp32 guide channels onto K = 17
// logits per output pixel and pools only C = 4 value channels, so the 1x1
// projection -- a [128 px x Cg] . [Cg x K] GEMM per tile -- is the whole
// cost.  On the FP32 FMA pipe it takes ~8.7 K FMA per pixel, which keeps a
// CUDA-core kernel well below the HBM roofline; here it runs on the 5th-gen
// tensor cores (tcgen05, kind::f16) at near-fp32 accuracy with a two-term
// bf16 split of both operands:
//
//     x = x_hi + x_lo + r,   x_hi = bf16(x),  x_lo = bf16(x - x_hi),
//     |r| <= 2^-18 |x|,      g . w = (g_hi + g_lo) . (w_hi + w_lo) + O(2^-17)
//
// All four products are exact in the fp32 accumulators.  The residual
// guide[:, :K] of residual_auto (uplift/uplift.py:26-39) is folded into the
// weights (w + 1 on the diagonal) before the split.
//
// Tile: 4 x 8 coarse cells = 8 x 16 output pixels (M = 128, TMEM lane = pixel).
// The guide streams in 32-channel fp32 chunks (128-byte rows, TMA with the
// 128-byte swizzle).  Per chunk the split warps write [g_hi | g_lo] (2 x 32
// bf16 = 32 TMEM columns) to one of four TMEM A buffers, and one thread
// issues four MMAs with the K dimension stacked,
//
//     D[128 x 2KH] += [g_hi | g_lo] . [[w_hi ; w_lo] ; [w_hi ; w_lo]]^T
//
// (KH = K rounded up to 8; weights K-major in shared memory), so that
// logit k = D[:, k] + D[:, KH + k] + bias.  The kernel is bound by the
// number of MMA instructions per chunk rather than by their width; four is
// half of what a three-product tf32 split needs.  The softmax and the
// pooling of the C <= 32 value channels (replicate-clamped neighbours, read
// through L1) run on the CUDA cores in the epilogue warps.
//
// Roles (448 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: guide chunks into a ring of 8 slots
//   warp 1      TMEM owner + single-thread MMA issuer
//   warps 2-9   split, two groups of four taking alternate chunks
//   warps 10-13 epilogue: logits -> softmax -> pooling -> fp32 stores
// A ring slot is free again as soon as its chunk is in registers.
// Accumulators are double-buffered across tiles, so one tile's epilogue
// overlaps the next tile's MMAs.  Every mbarrier wait is bounded as in the
// bf16 kernel; expiries are recorded in this kernel's status word.
//
// Reference semantics: LocalAttender.forward, uplift/uplift.py:801-847.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>

#include "uplift_la.h"
#include "la_internal.h"
#include "la_tc_common.h"

namespace ula {

__device__ unsigned int g_tcw_status;

namespace tcw {
using namespace tc;

constexpr int kCellsY = 4, kCellsX = 8;  // cells per tile
constexpr int kM = 128;                  // output pixels per tile (8 x 16)
constexpr int kChunkCh = 32;             // fp32 guide channels per chunk (one 128-byte row)
constexpr int kChunkBytes = kM * 128;    // 16 KB
constexpr int kStages = 8;               // even: the two split groups own alternate slots
constexpr int kMaxCg = 512;
constexpr int kMaxC = 32;
constexpr int kLogN = 32;                // K <= 32
constexpr int kAccCols = 64;             // one accumulator set (2KH <= 64 columns)
constexpr int kABufs = 4;                // TMEM A buffers: [g_hi | g_lo], 32 columns each
constexpr int kACol = 2 * kAccCols;      // after the two accumulator sets
constexpr int kTmemCols = 256;
static_assert(kACol + kABufs * 32 <= kTmemCols, "TMEM budget");
constexpr int kThreads = 448;
constexpr int kEpiWarp = 10;             // first epilogue warp
constexpr uint64_t kTimeoutNs = 2000000000ull;

constexpr int kOffBar = 0;
constexpr int kNumBars = kStages * 2 + kABufs * 2 + 2 + 2 + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;  // tmem slot, abort flags
constexpr int kOffBias = kOffMisc + 16;
constexpr int kOffRing = 1024;
constexpr int kOffW = kOffRing + kStages * kChunkBytes;
static_assert(kOffBias + kLogN * 4 <= kOffRing, "header fits below the ring");

// Weight rows per logit half; the weights of two chunks (64 channels) share
// one K-major 128-byte-swizzled tile of 2KH rows.
__host__ __device__ constexpr int kh_of(int K) { return (K + 7) & ~7; }
__host__ __device__ constexpr int wpair_bytes(int K) { return 2 * kh_of(K) * 128; }
__host__ __device__ constexpr int smem_bytes(int K, int nchunks) {
  return kOffW + (nchunks + 1) / 2 * wpair_bytes(K) + 1024;
}

struct Params {
  CUtensorMap gmap;  // guide fp32 [B, 2H, 2W, Cg], box {32, 16, 8, 1}
  const float* value; int64_t v_b, v_h, v_w;
  float* out;         int64_t o_b, o_h, o_w;
  const float* weight;  // [K][Cg]
  const float* bias;    // [K] or null
  int8_t dy[kLogN];
  int8_t dx[kLogN];
  int Cg, C, H, W, nchunks, tiles_x, tiles_y, num_tiles;
  int conv_res, hardmax;
  uint64_t timeout_ns;
  unsigned int* host_status;  // host-visible status word or null
  int test_fault;  // 1: the producer issues no loads (tests the timeout path)
};

__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag, unsigned where,
                                          const WaitLimit& limit) {
  if (mbar_try(b, parity)) return true;  // completed phase: no call into the bounded slow path
  return mbar_wait_status(b, parity, abort_flag, where, limit, &g_tcw_status);
}

// kind::f16 MMA with the A operand read from TMEM (lane = row; a 32-bit
// column holds two consecutive K elements, the lower one in the low half).
__device__ __forceinline__ void mma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread (lane) writes its row.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Two-term bf16 split of x: x_hi = bf16(x), x_lo = bf16(x - x_hi).
__device__ __forceinline__ void split2(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}
__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 a, __nv_bfloat16 b) {
  return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
}

struct TileXY {
  int b, cy0, cx0;
};
__device__ __forceinline__ TileXY tile_of(const Params& p, int t) {
  const int per_img = p.tiles_x * p.tiles_y;
  TileXY r;
  r.b = t / per_img;
  const int rem = t - r.b * per_img;
  const int ty = rem / p.tiles_x;
  r.cy0 = ty * kCellsY;
  r.cx0 = (rem - ty * p.tiles_x) * kCellsX;
  return r;
}

template <int K>
__global__ void __launch_bounds__(kThreads, 1) la_tcw_kernel(const __grid_constant__ Params p) {
  constexpr int KH = kh_of(K), N = 2 * KH;
  constexpr int kWPair = wpair_bytes(K);
  static_assert(N <= kAccCols && N % 16 == 0, "accumulator columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;                  // [kStages] guide chunk landed
  uint64_t* empty = full + kStages;       // [kStages] guide chunk read by a split group
  uint64_t* a_full = empty + kStages;     // [kABufs] [g_hi | g_lo] written to TMEM
  uint64_t* a_empty = a_full + kABufs;    // [kABufs] the chunk's MMAs are done
  uint64_t* acc_full = a_empty + kABufs;  // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  float* sBias = reinterpret_cast<float*>(smem + kOffBias);
  uint8_t* sRing = smem + kOffRing;
  uint8_t* sW = smem + kOffW;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  // ---------------------------------------------------------------- setup
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);  // the 4 split warps of one group
    }
    for (int i = 0; i < kABufs; ++i) {
      mbar_init(&a_full[i], 4);  // the 4 split warps of one group
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // 4 epilogue warps
    }
    mbar_init(drain, 1);
    abort_flag[0] = 0;
    abort_flag[1] = 0;  // stays 0: the flag of waits that must not be aborted
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)), "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // Programmatic dependent launch: nothing above reads global memory.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  // Weights: per pair of chunks (64 channels) a K-major [2KH x 64] bf16 tile
  // with the 128-byte swizzle; rows 0..KH-1 w_hi, rows KH..2KH-1 w_lo
  // (logits >= K and channels >= Cg are zero).
  {
    const int npairs = (p.nchunks + 1) / 2;
    const int n_el = npairs * 64 * KH;
    for (int idx = tid; idx < n_el; idx += kThreads) {
      const int n = idx % KH, c = idx / KH;
      float w = 0.f;
      if (n < K && c < p.Cg) {
        w = p.weight[(size_t)n * p.Cg + c];
        if (p.conv_res && n == c) w += 1.f;
      }
      __nv_bfloat16 hi, lo;
      split2(w, hi, lo);
      const int e = c & 63;
      // rows n and KH + n share the swizzle phase (KH is a multiple of 8)
      uint8_t* base = sW + (c >> 6) * kWPair + ((((e >> 3) ^ (n & 7)) << 4)) + (e & 7) * 2 + (n & 7) * 128;
      *reinterpret_cast<__nv_bfloat16*>(base + (n >> 3) * 1024) = hi;
      *reinterpret_cast<__nv_bfloat16*>(base + ((KH + n) >> 3) * 1024) = lo;
    }
  }
  for (int k = tid; k < kLogN; k += kThreads) sBias[k] = (p.bias != nullptr && k < K) ? p.bias[k] : 0.f;
  fence_proxy_async();  // sW is read by the tensor core (async proxy)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int local_tiles = 0;
  for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) ++local_tiles;
  const WaitLimit tmo{p.timeout_ns, p.host_status};
  const int nch = p.nchunks;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_map(&p.gmap);
      bool ok = true;
      uint32_t g = 0;
      for (int n = 0; n < local_tiles && ok; ++n) {
        const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
        for (int c = 0; c < nch; ++c, ++g) {
          const int slot = g % kStages;
          ok = mbar_wait(&empty[slot], ((g / kStages) & 1) ^ 1, abort_flag, 1, tmo);
          if (!ok) break;
          if (p.test_fault == 1) continue;  // the guide never arrives: consumers time out
          mbar_expect_tx(&full[slot], kChunkBytes);
          tma_load(sRing + slot * kChunkBytes, &p.gmap, &full[slot], c * kChunkCh, 2 * tl.cx0, 2 * tl.cy0, tl.b);
        }
      }
      if (!ok) {  // let issued loads land before the CTA can exit
        const uint64_t t0 = gtimer();
        while (gtimer() - t0 < 200000ull) {}
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kId = idesc_f16(1, 0, kM, N);  // bf16 x bf16 -> fp32, K-major
      const uint32_t aW = su32(sW);
      bool ok = true;
      uint32_t g = 0;
      for (int n = 0; n < local_tiles && ok; ++n) {
        const int s = n & 1;
        ok = mbar_wait(&acc_empty[s], ((n >> 1) & 1) ^ 1, abort_flag, 2, tmo);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + s * kAccCols;
        for (int c = 0; c < nch; ++c, ++g) {
          const int ab = g % kABufs;
          ok = mbar_wait(&a_full[ab], (g / kABufs) & 1, abort_flag, 2, tmo);
          if (!ok) break;
          tc_fence_after();
          // this chunk's 32 channels: bytes 64 * (c & 1) .. + 63 of the pair's rows
          const uint32_t bW = aW + (c >> 1) * kWPair + 64 * (c & 1);
          const uint32_t aBuf = tmem + kACol + ab * 32;
#pragma unroll
          for (int part = 0; part < 2; ++part) {  // g_hi, then g_lo
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {      // 16 channels per K-step
              const uint32_t acc = (c > 0 || part > 0 || ks > 0) ? 1u : 0u;
              mma_bf16_tmem_a(d, aBuf + 16 * part + 8 * ks, mdesc(bW + 32 * ks, 16, 1024, kLayoutSw128), kId, acc);
            }
          }
          tc_commit(&a_empty[ab]);
        }
        if (!ok) break;
        tc_commit(&acc_full[s]);
      }
      // all issued MMAs complete before TMEM can be released (this wait
      // ignores the abort flag: it must not be cut short by another role)
      tc_commit(drain);
      mbar_wait(drain, 0, abort_flag + 1, 2, tmo);
    }
  } else if (warp < kEpiWarp) {
    // ------------------------------------------------------------ split
    // group (warp - 2) / 4 takes the chunks of its parity, so two chunks are
    // split at a time; a warp owns TMEM lane quarter warp % 4, a thread one
    // pixel row.  Ring slots and A buffers alternate with the chunk index
    // (both counts even), so each group only ever waits on its own.
    const int q = warp & 3;
    const int group = (warp - 2) >> 2;
    const int i = 32 * q + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    const uint32_t total = (uint32_t)local_tiles * nch;
    bool ok = true;
    for (uint32_t g = group; g < total && ok; g += 2) {
      const int slot = g % kStages, ab = g % kABufs;
      ok = mbar_wait(&full[slot], (g / kStages) & 1, abort_flag, 3, tmo);
      if (!ok) break;
      const uint8_t* row = sRing + slot * kChunkBytes + i * 128;
      float x[32];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 v = *reinterpret_cast<const float4*>(row + ((u ^ (i & 7)) << 4));
        x[4 * u + 0] = v.x; x[4 * u + 1] = v.y; x[4 * u + 2] = v.z; x[4 * u + 3] = v.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // the row is in registers: the slot may be refilled
      uint32_t a[32];  // columns 0-15: g_hi pairs, 16-31: g_lo pairs
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        __nv_bfloat16 h0, l0, h1, l1;
        split2(x[2 * j], h0, l0);
        split2(x[2 * j + 1], h1, l1);
        a[j] = pack2(h0, h1);
        a[16 + j] = pack2(l0, l1);
      }
      ok = mbar_wait(&a_empty[ab], ((g / kABufs) & 1) ^ 1, abort_flag, 3, tmo);
      if (!ok) break;
      tc_fence_after();
      tmem_st32(lane_base + kACol + ab * 32, a);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[ab]);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int i = 32 * q + lane;  // TMEM lane == pixel of the tile
    const int py = i >> 4, px = i & 15;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    const int C4 = p.C >> 2;
    for (int n = 0; n < local_tiles; ++n) {
      const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
      const int s = n & 1;
      if (!mbar_wait(&acc_full[s], (n >> 1) & 1, abort_flag, 4, tmo)) break;
      tc_fence_after();
      // logit k = D[k] + D[KH + k], read in blocks of 32 columns
      float pk[K];
#pragma unroll
      for (int k = 0; k < K; ++k) pk[k] = sBias[k];
#pragma unroll
      for (int blk = 0; blk < (N + 31) / 32; ++blk) {
        uint32_t r[32];
        tc_ld32(lane_base + s * kAccCols + 32 * blk, r);
        tc_wait_ld();
#pragma unroll
        for (int k = 0; k < K; ++k) {
          if ((k >> 5) == blk) pk[k] += __uint_as_float(r[k & 31]);
          if (((KH + k) >> 5) == blk) pk[k] += __uint_as_float(r[(KH + k) & 31]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[s]);

      if (p.hardmax) {
        int best = 0;
        float bv = pk[0];
#pragma unroll
        for (int k = 1; k < K; ++k)
          if (pk[k] > bv) { bv = pk[k]; best = k; }
#pragma unroll
        for (int k = 0; k < K; ++k) pk[k] = (k == best) ? 1.f : 0.f;
      } else {
        float m = pk[0];
#pragma unroll
        for (int k = 1; k < K; ++k) m = fmaxf(m, pk[k]);
        float z = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) { pk[k] = __expf(pk[k] - m); z += pk[k]; }
        const float inv = 1.f / z;
#pragma unroll
        for (int k = 0; k < K; ++k) pk[k] *= inv;
      }
      const int y = 2 * tl.cy0 + py, x = 2 * tl.cx0 + px;
      if (y < 2 * p.H && x < 2 * p.W) {
        const int cy = y >> 1, cx = x >> 1;
        const float* vb = p.value + tl.b * p.v_b;
        float* op = p.out + tl.b * p.o_b + (int64_t)y * p.o_h + (int64_t)x * p.o_w;
        for (int c4 = 0; c4 < C4; ++c4) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int k = 0; k < K; ++k) {
            const int ny = min(max(cy + p.dy[k], 0), p.H - 1);
            const int nx = min(max(cx + p.dx[k], 0), p.W - 1);
            const float4 v = __ldg(reinterpret_cast<const float4*>(vb + ny * p.v_h + nx * p.v_w) + c4);
            acc.x = fmaf(pk[k], v.x, acc.x);
            acc.y = fmaf(pk[k], v.y, acc.y);
            acc.z = fmaf(pk[k], v.z, acc.z);
            acc.w = fmaf(pk[k], v.w, acc.w);
          }
          reinterpret_cast<float4*>(op)[c4] = acc;
        }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <int K>
int launch_t(const Params& p, int dev, int grid, cudaStream_t stream) {
  auto fn = la_tcw_kernel<K>;
  const int smem = smem_bytes(K, p.nchunks);
  static std::atomic<bool> configured[64] = {};  // racing threads set the same value
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes(K, kMaxCg / kChunkCh));
    if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "tensor-core (wide fp32) kernel launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

}  // namespace tcw

static bool a16w(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool tcw_eligible(const TcArgs& a, const char** why) {
  auto no = [&](const char* m) { if (why) *why = m; return false; };
  if (a.dtype != UPLIFT_LA_F32) return no("storage type is not fp32");
  if (a.Cg % tcw::kChunkCh != 0 || a.Cg < 64 || a.Cg > tcw::kMaxCg) return no("guide channels not a multiple of 32 in 64..512");
  if (a.C % 4 != 0 || a.C > tcw::kMaxC) return no("value channels not a multiple of 4 up to 32");
  if (a.K != 5 && a.K != 9 && a.K != 13 && a.K != 17 && a.K != 25) return no("K not in {5, 9, 13, 17, 25}");
  if (a.B < 1 || a.H < 1 || a.W < 1) return no("empty problem");
  if (a.B > 65535 || a.H > (1 << 20) || a.W > (1 << 20)) return no("too large for the tile grid");
  if (!a16w(a.guide) || !a16w(a.value) || !a16w(a.out)) return no("base pointers not 16-byte aligned");
  const int64_t st[9] = {a.g_b, a.g_h, a.g_w, a.v_b, a.v_h, a.v_w, a.o_b, a.o_h, a.o_w};
  for (int i = 0; i < 9; ++i)
    if (st[i] % 4 != 0 || st[i] <= 0) return no("strides not multiples of 16 bytes");
  return true;
}

int tcw_launch(const TcArgs& a, cudaStream_t stream) {
  using namespace tcw;
  Params p;
  memset(&p, 0, sizeof(p));
  int rc = tc_make_map(&p.gmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.guide, a.Cg, 2 * a.W, 2 * a.H, a.B, a.g_w, a.g_h,
                       a.g_b, kChunkCh, 16, 8);
  if (rc != UPLIFT_LA_OK) return rc;
  p.value = static_cast<const float*>(a.value);
  p.v_b = a.v_b; p.v_h = a.v_h; p.v_w = a.v_w;
  p.out = static_cast<float*>(a.out);
  p.o_b = a.o_b; p.o_h = a.o_h; p.o_w = a.o_w;
  p.weight = a.weight;
  p.bias = a.bias;
  for (int k = 0; k < a.K; ++k) {
    p.dy[k] = a.offsets[2 * k];
    p.dx[k] = a.offsets[2 * k + 1];
  }
  p.Cg = a.Cg;
  p.C = a.C;
  p.H = a.H;
  p.W = a.W;
  p.nchunks = a.Cg / kChunkCh;
  p.tiles_x = (a.W + kCellsX - 1) / kCellsX;
  p.tiles_y = (a.H + kCellsY - 1) / kCellsY;
  const int64_t nt = (int64_t)p.tiles_x * p.tiles_y * a.B;
  if (nt >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "too many tiles");
  p.num_tiles = (int)nt;
  p.conv_res = a.conv_res;
  p.hardmax = a.hardmax;
  p.timeout_ns = tc_test_timeout_ns() != 0 ? tc_test_timeout_ns() : kTimeoutNs;
  p.host_status = host_status_word();
  p.test_fault = tc_test_fault();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(UPLIFT_LA_ERR_NO_DEVICE, "cudaGetDevice failed");
  static std::atomic<int> sm_count[64] = {};
  int sms = (dev >= 0 && dev < 64) ? sm_count[dev].load(std::memory_order_relaxed) : 0;
  if (sms == 0) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (dev >= 0 && dev < 64) sm_count[dev].store(sms, std::memory_order_relaxed);
  }
  const int grid = (int)std::min<int64_t>(nt, cta_budget(sms));
  switch (a.K) {
    case 5: return launch_t<5>(p, dev, grid, stream);
    case 9: return launch_t<9>(p, dev, grid, stream);
    case 13: return launch_t<13>(p, dev, grid, stream);
    case 17: return launch_t<17>(p, dev, grid, stream);
    case 25: return launch_t<25>(p, dev, grid, stream);
    default: return fail(UPLIFT_LA_ERR_SHAPE, "K=%d unsupported", a.K);
  }
}

int tcw_device_status(bool clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tcw_status, sizeof(v));
  if (e != cudaSuccess) {
    fail(UPLIFT_LA_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
    return -1;
  }
  if (clear && v != 0) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_tcw_status, &zero, sizeof(zero));
    if (e != cudaSuccess) {
      fail(UPLIFT_LA_ERR_CUDA, "status clear: %s", cudaGetErrorString(e));
      return -1;
    }
  }
  return (int)v;
}

}  // namespace ula
