// Tensor-core dV of the Local Attender backward for B200 (sm_100a): tcgen05
// MMA with the accumulator in TMEM, TMA loads and stores, mbarrier pipeline.
//
// dV[n] = sum over output pixels p and offsets k with clamp(cell(p) + off_k)
// = n of P_k(p) dout[p] -- the transpose of the forward's pooling
// (uplift/uplift.py:835-837).  Value-centric, so every dV value is written
// once by one CTA (no atomics, no fp32 intermediate tensor):
//
//   a tile = 8 x 16 value pixels (M = 128, TMEM lane = value pixel); the
//   output cells that can reach it lie in 12 cell rows x 20 cell columns
//   around it (|offset| <= 2).  Per cell row (80 output pixels: 2 output
//   rows x 40 output columns) the tile accumulates
//
//       D[128 x C] += Pt[128 x 80] . dout[80 x C]          (5 MMA k-steps)
//
//   where Pt[n][p] = sum of P_k(p) over the offsets k that take p's cell to
//   value pixel n (clamped at the map border like the forward's replicate
//   padding).  dout arrives by TMA as {64 channels, 40 px, 2 rows} boxes
//   with the 128-byte swizzle (the MN-major B operand); Pt is built in
//   shared memory (K-major, no swizzle) by CUDA-core warps from the fp32
//   softmax workspace, rounded to the storage type (as the forward rounds
//   the weights it multiplies by).
//
// Roles (320 threads, one CTA per SM, persistent over tiles): warp 0 TMA
// producer of the dout ring; warp 1 TMEM owner + MMA issuer; warps 2-5 build
// Pt (double-buffered; interior tiles by a gather, a thread per Pt row with
// the next cell row's weights loaded ahead, border tiles by a scatter with
// clamped duplicates summed); warps 6-9 epilogue (TMEM -> storage type -> swizzled
// staging -> TMA store of the warp's 2 value rows).  Every mbarrier wait is
// bounded; on expiry the CTA records the role in this kernel's status word
// (and the registered host word), drains and exits.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>

#include "uplift_la.h"
#include "la_internal.h"
#include "la_tc_common.h"

namespace ula {

__device__ unsigned int g_dv_status;

namespace dvtc {

using namespace ::ula::tc;

constexpr int kTy = 8, kTx = 16;               // value pixels per tile
constexpr int kM = kTy * kTx;                  // 128
constexpr int kPn = 2;                         // offsets within +-2
constexpr int kRegX = kTx + 2 * kPn;           // 20 cell columns reach a tile
constexpr int kKc = 2 * 2 * kRegX;             // 80 output pixels per cell row
constexpr int kChunk = 64;                     // channels per TMA box
constexpr int kMaxC = 384;
constexpr int kBoxBytes = kKc * 128;           // 10 KB: 80 px x 64 channels
constexpr int kStages = 2;                     // dout ring slots
constexpr int kSlotBytes = (kMaxC / kChunk) * kBoxBytes;  // 60 KB
constexpr int kPtBytes = kM * kKc * 2;         // 20 KB
constexpr int kPtSbo = (kKc / 8) * 128;        // 1280 B between 8-row groups of Pt
constexpr int kWarpStage = 32 * 128;           // 4 KB: one epilogue warp's 32 px x 64 ch
constexpr int kThreads = 320;
constexpr int kTmemCols = 512;
constexpr uint64_t kTimeoutNs = 2000000000ull;

constexpr int kOffRing = 0;
constexpr int kOffPt = kOffRing + kStages * kSlotBytes;
constexpr int kOffStage = kOffPt + 2 * kPtBytes;
constexpr int kOffBar = kOffStage + 4 * 2 * kWarpStage;
constexpr int kNumBars = 2 * kStages + 4 + 2 + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + base alignment slack

struct Params {
  CUtensorMap dmap;   // dout  [B, 2H, 2W, C]  box {64, 40, 2, 1}
  CUtensorMap vmap;   // dvalue [B, H, W, C]   box {64, 16, 2, 1}
  const float* probs; // [B][2H][2W][K] fp32
  int8_t dy[UPLIFT_LA_MAX_K];
  int8_t dx[UPLIFT_LA_MAX_K];
  int8_t ktab[(2 * kPn + 1) * (2 * kPn + 1)];  // offset (dy, dx) -> k, or -1
  int gather;                                  // 1: the offsets are distinct (the gather fill applies)
  int B, C, H, W, K, nchunks, tiles_x, tiles_y, num_tiles;
  uint64_t timeout_ns;
  unsigned int* host_status;
};

__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag, unsigned where,
                                          const WaitLimit& limit) {
  if (mbar_try(b, parity)) return true;  // completed phase: no call into the bounded slow path
  return mbar_wait_status(b, parity, abort_flag, where, limit, &g_dv_status);
}

template <typename T> struct St;
template <> struct St<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  __device__ __forceinline__ static uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct St<__half> {
  static constexpr uint32_t kFmt = 0;
  __device__ __forceinline__ static uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

struct Tile {
  int b, vy0, vx0, r0, r1;  // value origin; cell rows [r0, r1) reach it
};
__device__ __forceinline__ Tile tile_of(const Params& p, int t) {
  const int per_img = p.tiles_x * p.tiles_y;
  Tile r;
  r.b = t / per_img;
  const int rem = t - r.b * per_img;
  const int ty = rem / p.tiles_x;
  r.vy0 = ty * kTy;
  r.vx0 = (rem - ty * p.tiles_x) * kTx;
  r.r0 = max(0, r.vy0 - kPn);
  r.r1 = min(p.H, r.vy0 + kTy + kPn);
  return r;
}

template <typename T, int K>
__global__ void __launch_bounds__(kThreads, 1) la_dv_tc_kernel(const __grid_constant__ Params p) {
  using S = St<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sRing = smem + kOffRing;
  uint8_t* sPt = smem + kOffPt;
  uint8_t* sStage = smem + kOffStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;                 // dout slot landed
  uint64_t* empty = full + kStages;      // dout slot consumed by the MMAs
  uint64_t* pt_full = empty + kStages;   // Pt buffer built
  uint64_t* pt_empty = pt_full + 2;      // Pt buffer consumed by the MMAs
  uint64_t* acc_full = pt_empty + 2;     // a tile's accumulator complete
  uint64_t* acc_empty = acc_full + 1;    // the epilogue has read it
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  volatile int* go = reinterpret_cast<volatile int*>(smem + kOffMisc + 16);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&pt_full[i], 4);  // 4 builder warps
      mbar_init(&pt_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);      // 4 epilogue warps
    mbar_init(drain, 1);
    abort_flag[0] = 0;
    abort_flag[1] = 0;            // stays 0: the flag of waits that must not be aborted
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)), "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int local_tiles = 0;
  for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) ++local_tiles;
  const WaitLimit tmo{p.timeout_ns, p.host_status};
  const int half = p.nchunks >= 2 ? (p.nchunks + 1) / 2 : 1;  // 64-channel chunks per MMA (N <= 192)

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_map(&p.dmap);
      bool ok = true;
      uint32_t gc = 0;
      for (int n = 0; n < local_tiles && ok; ++n) {
        const Tile tl = tile_of(p, blockIdx.x + n * gridDim.x);
        for (int cy = tl.r0; cy < tl.r1 && ok; ++cy, ++gc) {
          const int s = gc % kStages;
          ok = mbar_wait(&empty[s], ((gc / kStages) & 1) ^ 1, abort_flag, 1, tmo);
          if (!ok) break;
          mbar_expect_tx(&full[s], p.nchunks * kBoxBytes);
          for (int j = 0; j < p.nchunks; ++j)
            tma_load(sRing + s * kSlotBytes + j * kBoxBytes, &p.dmap, &full[s], j * kChunk, 2 * (tl.vx0 - kPn), 2 * cy,
                     tl.b);
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
      bool ok = true;
      uint32_t gc = 0;
      for (int n = 0; n < local_tiles && ok; ++n) {
        const Tile tl = tile_of(p, blockIdx.x + n * gridDim.x);
        ok = mbar_wait(acc_empty, (n & 1) ^ 1, abort_flag, 2, tmo);
        if (!ok) break;
        tc_fence_after();
        for (int cy = tl.r0; cy < tl.r1 && ok; ++cy, ++gc) {
          const int s = gc % kStages, pb = gc & 1;
          ok = mbar_wait(&full[s], (gc / kStages) & 1, abort_flag, 2, tmo) &&
               mbar_wait(&pt_full[pb], (gc >> 1) & 1, abort_flag, 2, tmo);
          if (!ok) break;
          tc_fence_after();
          const uint32_t aP = su32(sPt + pb * kPtBytes);
          const uint32_t aD = su32(sRing + s * kSlotBytes);
#pragma unroll 1
          for (int j0 = 0; j0 < p.nchunks; j0 += half) {
            const int nj = min(half, p.nchunks - j0);
            const uint32_t idesc = idesc_f16(S::kFmt, 1, kM, kChunk * nj);
#pragma unroll
            for (int ks = 0; ks < kKc / 16; ++ks)
              tc_mma(tmem + kChunk * j0, mdesc(aP + 256 * ks, 128, kPtSbo, kLayoutNone),
                     mdesc(aD + j0 * kBoxBytes + 2048 * ks, kBoxBytes, 1024, kLayoutSw128), idesc,
                     (cy > tl.r0 || ks > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
          tc_commit(&pt_empty[pb]);
        }
        if (!ok) break;
        tc_commit(acc_full);
      }
      // all issued MMAs complete before TMEM can be released (this wait
      // ignores the abort flag: it must not be cut short by another role)
      tc_commit(drain);
      mbar_wait(drain, 0, abort_flag + 1, 2, tmo);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ Pt builders
    // Two ways to fill a cell row's Pt buffer; all four warps take the same
    // one for a tile.
    //  * gather (tiles with no value pixel on the map border, distinct
    //    offsets): thread t owns row t of Pt, value pixel (vy, vx) =
    //    (vy0 + t / 16, vx0 + t % 16).  Cell row cy reaches it only through
    //    the offset row dy = vy - cy, from the 5 cells cx = vx - dx, each with
    //    its 2 x 2 output pixels; no clamping can send anything else there.
    //    The thread writes its whole row (zeros, then the 10 packed pairs), so
    //    nothing is left from earlier cell rows, and the 20 weights of the
    //    next cell row are loaded while this one is written.
    //  * scatter (border tiles, where clamping sends several offsets of one
    //    output pixel to one value pixel): the buffer is zeroed, then thread
    //    t < 80 scatters output pixel t's weights into column t of Pt,
    //    summing the clamped duplicates in fp32.
    // One thread waits on the buffer's barrier and shares the outcome (in
    // a per-buffer word, so a slow reader never sees the next cell row's),
    // so all take the same path.
    const int t = tid - 64;
    const int rny = t >> 4, rnx = t & 15;
    auto interior = [&](const Tile& tl) {
      return p.gather != 0 && tl.vy0 >= 1 && tl.vy0 + kTy <= p.H - 1 && tl.vx0 >= 1 && tl.vx0 + kTx <= p.W - 1;
    };
    // the 20 weights of row t for cell row cy: [cell j][output row][output column]
    auto gather_load = [&](int cy, const Tile& tl, float* g) {
#pragma unroll
      for (int i = 0; i < 20; ++i) g[i] = 0.f;
      const int dyv = tl.vy0 + rny - cy;
      if (dyv < -kPn || dyv > kPn) return;
#pragma unroll
      for (int j = 0; j < 2 * kPn + 1; ++j) {  // cell column vx - dx with dx = kPn - j
        const int k = p.ktab[(dyv + kPn) * (2 * kPn + 1) + (2 * kPn - j)];
        const int cx = tl.vx0 - kPn + rnx + j;
        if (k >= 0 && cx < p.W) {
          const float* pr = p.probs + (((int64_t)tl.b * 2 * p.H + 2 * cy) * (2 * p.W) + 2 * cx) * K + k;
          const int64_t rs = (int64_t)2 * p.W * K;
          g[4 * j + 0] = __ldg(pr);
          g[4 * j + 1] = __ldg(pr + K);
          g[4 * j + 2] = __ldg(pr + rs);
          g[4 * j + 3] = __ldg(pr + rs + K);
        }
      }
    };
    // next stage after (n, cy): the next cell row of the tile, else the next tile's first
    auto next_stage = [&](int& n, int& cy, Tile& tl) {
      if (++cy >= tl.r1) {
        if (++n < local_tiles) {
          tl = tile_of(p, blockIdx.x + n * gridDim.x);
          cy = tl.r0;
        }
      }
    };
    float gcur[20], gnext[20];
    int n = 0, cy = 0;
    Tile tl{};
    bool g_next = false;
    if (local_tiles > 0) {
      tl = tile_of(p, blockIdx.x);
      cy = tl.r0;
      g_next = interior(tl);
      if (g_next) gather_load(cy, tl, gnext);
    }
    uint32_t gc = 0;
    while (n < local_tiles) {
      const int pb = gc & 1;
      if (t == 0) go[pb] = mbar_wait(&pt_empty[pb], ((gc >> 1) & 1) ^ 1, abort_flag, 3, tmo) ? 1 : 0;
      named_bar(1, 128);
      if (go[pb] == 0) break;
      const int ccy = cy;
      const Tile ctl = tl;
      const bool gather = g_next;
      if (gather) {
#pragma unroll
        for (int i = 0; i < 20; ++i) gcur[i] = gnext[i];
      }
      next_stage(n, cy, tl);
      g_next = n < local_tiles && interior(tl);
      if (g_next) gather_load(cy, tl, gnext);  // in flight while this cell row is written
      uint8_t* buf = sPt + pb * kPtBytes;
      if (gather) {
        // row t: 10 groups of 8 K-elements, 128 bytes apart
        uint8_t* row = buf + (t >> 3) * kPtSbo + (t & 7) * 16;
#pragma unroll
        for (int q = 0; q < kKc / 8; ++q) *reinterpret_cast<uint4*>(row + q * 128) = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < 2 * kPn + 1; ++j) {
#pragma unroll
          for (int py = 0; py < 2; ++py) {
            const int pc = py * (2 * kRegX) + 2 * (rnx + j);  // K index (output pixel) of the pair, even
            *reinterpret_cast<uint32_t*>(row + (pc >> 3) * 128 + (pc & 7) * 2) =
                S::pack(gcur[4 * j + 2 * py], gcur[4 * j + 2 * py + 1]);
          }
        }
      } else {
        for (int i = t; i < kPtBytes / 16; i += 128) reinterpret_cast<uint4*>(buf)[i] = make_uint4(0, 0, 0, 0);
        named_bar(1, 128);
        if (t < kKc) {
          const int py = t / (2 * kRegX), px = t - py * (2 * kRegX);
          const int oy = 2 * ccy + py, ox = 2 * (ctl.vx0 - kPn) + px;
          if (ox >= 0 && ox < 2 * p.W) {
            const int cx = ox >> 1;
            const float* pr = p.probs + (((int64_t)ctl.b * 2 * p.H + oy) * (2 * p.W) + ox) * K;
            float pk[K];
            int nk[K];
            bool border = false;
#pragma unroll
            for (int k = 0; k < K; ++k) {
              pk[k] = __ldg(pr + k);
              const int yy = ccy + p.dy[k], xx = cx + p.dx[k];
              border |= yy < 0 || yy >= p.H || xx < 0 || xx >= p.W;
              const int ny = min(max(yy, 0), p.H - 1) - ctl.vy0, nx = min(max(xx, 0), p.W - 1) - ctl.vx0;
              nk[k] = (ny >= 0 && ny < kTy && nx >= 0 && nx < kTx) ? ny * kTx + nx : -1;
            }
            if (border) {  // offsets that clamp onto the same value pixel are summed in fp32
#pragma unroll
              for (int k = 1; k < K; ++k) {
#pragma unroll
                for (int j = 0; j < k; ++j) {
                  if (nk[k] >= 0 && nk[j] == nk[k]) {
                    pk[j] += pk[k];
                    nk[k] = -1;
                  }
                }
              }
            }
            uint8_t* col = buf + (t >> 3) * 128 + (t & 7) * 2;
#pragma unroll
            for (int k = 0; k < K; ++k)
              if (nk[k] >= 0)
                *reinterpret_cast<uint16_t*>(col + (nk[k] >> 3) * kPtSbo + (nk[k] & 7) * 16) = S::bits(pk[k]);
          }
        }
      }
      fence_proxy_async();  // Pt is read by the tensor core (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive(&pt_full[pb]);
      ++gc;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // warp w owns TMEM lanes 32q..32q+31 (q = w % 4) = value rows 2q, 2q + 1
    // of the tile; stores them per 64-channel chunk through its own two
    // staging buffers, so warps never wait for each other
    const int q = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    uint8_t* bufs = sStage + (warp - 6) * 2 * kWarpStage;
    uint32_t jw = 0;
    for (int n = 0; n < local_tiles; ++n) {
      const Tile tl = tile_of(p, blockIdx.x + n * gridDim.x);
      if (!mbar_wait(acc_full, n & 1, abort_flag, 4, tmo)) break;
      tc_fence_after();
      for (int j = 0; j < p.nchunks; ++j) {
        uint32_t r[64];
        tc_ld32(lane_base + kChunk * j, r);
        tc_ld32(lane_base + kChunk * j + 32, r + 32);
        tc_wait_ld();
        if (j + 1 == p.nchunks) {  // the accumulator is free for the next tile
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty);
        }
        uint8_t* buf = bufs + (jw & 1) * kWarpStage;
        ++jw;
        if (lane == 0) bulk_wait_read1();  // the store issued two chunks ago has read `buf`
        __syncwarp();
        uint8_t* row = buf + lane * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* src = r + 8 * c;
          uint4 w;
          w.x = S::pack(__uint_as_float(src[0]), __uint_as_float(src[1]));
          w.y = S::pack(__uint_as_float(src[2]), __uint_as_float(src[3]));
          w.z = S::pack(__uint_as_float(src[4]), __uint_as_float(src[5]));
          w.w = S::pack(__uint_as_float(src[6]), __uint_as_float(src[7]));
          *reinterpret_cast<uint4*>(row + ((c ^ (lane & 7)) << 4)) = w;
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          tma_store(&p.vmap, buf, j * kChunk, tl.vx0, tl.vy0 + 2 * q, tl.b);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <typename T, int K>
int launch_t(const Params& p, int dev, int grid, cudaStream_t stream) {
  auto fn = la_dv_tc_kernel<T, K>;
  static std::atomic<bool> configured[64] = {};  // racing threads set the same value
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev].store(true, std::memory_order_release);
  }
  fn<<<grid, kThreads, kSmemBytes, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "tensor-core dV launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

template <typename T>
int launch_k(const Params& p, int dev, int grid, cudaStream_t stream) {
  switch (p.K) {
    case 5: return launch_t<T, 5>(p, dev, grid, stream);
    case 9: return launch_t<T, 9>(p, dev, grid, stream);
    case 13: return launch_t<T, 13>(p, dev, grid, stream);
    case 17: return launch_t<T, 17>(p, dev, grid, stream);
    case 25: return launch_t<T, 25>(p, dev, grid, stream);
    default: return fail(UPLIFT_LA_ERR_SHAPE, "tensor-core dV: K=%d unsupported", p.K);
  }
}

}  // namespace dvtc

bool dv_tc_eligible(const DvArgs& a, const char** why) {
  auto no = [&](const char* m) { if (why) *why = m; return false; };
  if (a.dtype != UPLIFT_LA_BF16 && a.dtype != UPLIFT_LA_F16) return no("storage type is not bf16/fp16");
  if (a.I != 2) return no("scale I != 2");
  if (a.C % dvtc::kChunk != 0 || a.C > dvtc::kMaxC) return no("channels not a multiple of 64 up to 384");
  if (a.K != 5 && a.K != 9 && a.K != 13 && a.K != 17 && a.K != 25) return no("K not in {5, 9, 13, 17, 25}");
  for (int k = 0; k < a.K; ++k)
    if (a.dy[k] < -dvtc::kPn || a.dy[k] > dvtc::kPn || a.dx[k] < -dvtc::kPn || a.dx[k] > dvtc::kPn)
      return no("offsets beyond +-2");
  if (a.B < 1 || a.H < 1 || a.W < 1) return no("empty problem");
  if (a.B > 65535 || a.H > (1 << 20) || a.W > (1 << 20)) return no("too large for the tile grid");
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!al(a.dout) || !al(a.dvalue)) return no("base pointers not 16-byte aligned");
  const int64_t st[6] = {a.d_b, a.d_h, a.d_w, a.dv_b, a.dv_h, a.dv_w};
  for (int i = 0; i < 6; ++i)
    if (st[i] % 8 != 0 || st[i] <= 0) return no("strides not multiples of 16 bytes");
  return true;
}

int dv_tc_launch(const DvArgs& a, cudaStream_t stream) {
  using namespace dvtc;
  Params p;
  memset(&p, 0, sizeof(p));
  const CUtensorMapDataType dt = a.dtype == UPLIFT_LA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc = tc_make_map(&p.dmap, dt, 2, a.dout, a.C, 2 * a.W, 2 * a.H, a.B, a.d_w, a.d_h, a.d_b, kChunk, 2 * kRegX, 2);
  if (rc == UPLIFT_LA_OK)
    rc = tc_make_map(&p.vmap, dt, 2, a.dvalue, a.C, a.W, a.H, a.B, a.dv_w, a.dv_h, a.dv_b, kChunk, kTx, 2);
  if (rc != UPLIFT_LA_OK) return rc;
  p.probs = a.probs;
  for (int k = 0; k < a.K; ++k) {
    p.dy[k] = a.dy[k];
    p.dx[k] = a.dx[k];
  }
  memset(p.ktab, 0xff, sizeof(p.ktab));
  p.gather = 1;
  for (int k = 0; k < a.K; ++k) {
    int8_t& e = p.ktab[(a.dy[k] + kPn) * (2 * kPn + 1) + (a.dx[k] + kPn)];
    if (e >= 0) p.gather = 0;  // a repeated offset: its weights would have to be summed
    e = (int8_t)k;
  }
  p.B = a.B; p.C = a.C; p.H = a.H; p.W = a.W; p.K = a.K;
  p.nchunks = a.C / kChunk;
  p.tiles_x = (a.W + kTx - 1) / kTx;
  p.tiles_y = (a.H + kTy - 1) / kTy;
  const int64_t nt = (int64_t)p.tiles_x * p.tiles_y * a.B;
  if (nt >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "too many tiles");
  p.num_tiles = (int)nt;
  p.timeout_ns = tc_test_timeout_ns() != 0 ? tc_test_timeout_ns() : kTimeoutNs;
  p.host_status = host_status_word();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(UPLIFT_LA_ERR_NO_DEVICE, "cudaGetDevice failed");
  static std::atomic<int> sm_count[64] = {};
  int sms = (dev >= 0 && dev < 64) ? sm_count[dev].load(std::memory_order_relaxed) : 0;
  if (sms == 0) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (dev >= 0 && dev < 64) sm_count[dev].store(sms, std::memory_order_relaxed);
  }
  const int grid = (int)std::min<int64_t>(nt, cta_budget(sms));
  return a.dtype == UPLIFT_LA_BF16 ? launch_k<__nv_bfloat16>(p, dev, grid, stream)
                                   : launch_k<__half>(p, dev, grid, stream);
}

int dv_device_status(bool clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_dv_status, sizeof(v));
  if (e != cudaSuccess) {
    fail(UPLIFT_LA_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
    return -1;
  }
  if (clear && v != 0) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_dv_status, &zero, sizeof(zero));
    if (e != cudaSuccess) {
      fail(UPLIFT_LA_ERR_CUDA, "status clear: %s", cudaGetErrorString(e));
      return -1;
    }
  }
  return (int)v;
}

}  // namespace ula
