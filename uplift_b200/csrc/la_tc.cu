// Tensor-core Local Attender for B200 (sm_100a): tcgen05 MMA with TMEM
// accumulators, TMA tile loads/stores, mbarrier pipelines, warp-specialised.
//
// For the bf16 / fp16 path with scale I = 2 (every shipped UPLiFT config),
// Cg = 64 guide channels and C a multiple of 64 (<= 384) value channels.
//
// Formulation.  A tile is 4 x 8 coarse cells = 8 x 16 output pixels
// (M = 128).  All K neighbours of all its cells lie in an 8 x 12 window of
// coarse pixels (pn <= 2), so for the tile
//
//     logits[128 x 32]  = G[128 x 64] . W^T[64 x 32]          (MMA 1)
//     A[128 x 96]       = softmax weights scattered to window columns
//     out[128 x C]      = A[128 x 96] . Vwin[96 x C]           (MMA 2)
//
// MMA 2 is a banded GEMM (17 of 96 entries per row are non-zero); on the
// 5th-gen tensor cores the wasted products are cheaper than the FP32 FMA
// pipe doing only the useful ones, so the kernel stays HBM-bound.  The
// softmax weights are rounded to the storage type (bf16 / fp16) as in the
// reference's low-precision path (F.softmax on a bf16 tensor); every sum
// is accumulated in fp32 in TMEM.  Replicate padding: window pixels outside
// the image are zero-filled by TMA and never referenced, because each
// offset is clamped to the image before being mapped to a window column
// (clamped duplicates are merged in fp32 first).
//
// Roles (608 threads = 19 warps, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer of the value windows (64-channel chunks, one
//               ring unit of <= 3 chunks per accumulator half)
//   warp 18     TMA producer of the guide tiles
//   warp 1      TMEM owner + single-thread MMA issuer (logits of unit n+1
//               before the output MMAs of unit n)
//   warps 2-9   two softmax warpgroups (even / odd units): logits -> (+bias,
//               +residual) -> softmax -> A matrix
//   warps 10-17 two epilogue warpgroups, one per 192-column accumulator
//               half: TMEM -> storage type -> smem -> TMA store (or, with
//               the fused final resize, -> bilinear resample -> TMA store)
// Every mbarrier wait is bounded (2 s); on expiry the CTA records the role
// in a device status word (and a host-visible word when one is registered),
// drains its outstanding async work and exits.
//
// Reference semantics: LocalAttender.forward, uplift/uplift.py:801-847.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "uplift_la.h"
#include "la_internal.h"
#include "la_tc_common.h"

namespace ula {

// Status word for in-kernel failures (bounded waits that expired); read and
// cleared through uplift_la_device_status().
__device__ unsigned int g_tc_status;

namespace tc {

// Test hook state (uplift_la_test_hook): a fault mode and a wait limit
// (process-wide; atomics, since any host thread may launch).
std::atomic<int> g_test_fault{0};
std::atomic<unsigned long long> g_test_timeout_ns{0};

constexpr int kCellsY = 4, kCellsX = 8;      // cells per tile
constexpr int kM = 128;                      // output pixels per tile (8 x 16)
constexpr int kWinX = 12, kWin = 96;         // value window 8 x 12 (pn <= 2)
constexpr int kKSteps = kWin / 16;           // MMA-2 K steps
constexpr int kChunk = 64;                   // channels per value / output chunk
constexpr int kMaxC = 384;
constexpr int kUnitChunks = 3;               // value chunks per ring unit (one accumulator half)
constexpr int kNU = 2;                       // value ring units
constexpr int kLogN = 32;                    // MMA-1 N (K <= 32 logits)
constexpr int kLogCol = kMaxC;               // TMEM column of the logit accumulators
constexpr int kTmemCols = 512;
constexpr int kThreads = 608;                // 19 warps
constexpr int kGuideWarp = 18;               // guide-tile producer
constexpr uint64_t kTimeoutNs = 2000000000ull;  // default limit of every mbarrier wait

constexpr int kVBytes = kWin * 128;          // 12 KB: 96 window px x 64 ch
constexpr int kGBytes = kM * 128;            // 16 KB: 128 px x 64 guide ch
constexpr int kStageBytes = kM * 128;        // 16 KB: 128 px x 64 out ch
constexpr int kWBytes = kLogN * 128;         // 4 KB: 32 logits x 64 ch (one guide source)
constexpr int kA2Bytes = kM * kWin * 2;      // 24 KB
constexpr int kA2Sbo = (kWin / 8) * 128;     // 1536 B between 8-row groups of A

constexpr int kOffV = 0;
constexpr int kUnitBytes = kUnitChunks * kVBytes;  // 36 KB
constexpr int kOffG = kOffV + kNU * kUnitBytes;
constexpr int kOffStage = kOffG + 2 * kGBytes;
constexpr int kOffW = kOffStage + 4 * kStageBytes;  // 8 epilogue warps x 2 x 4 KB
constexpr int kOffA2 = kOffW + 2 * kWBytes;  // two sources with the fused guide
constexpr int kOffBar = kOffA2 + 2 * kA2Bytes;
constexpr int kNumBars = 2 + 2 + kNU + kNU + 2 + 2 + 2 + 2 + 2 + 2 + 1;
constexpr int kWarpStage = 32 * 128;         // 4 KB: one epilogue warp's 32 px x 64 ch
constexpr int kOffMisc = kOffBar + kNumBars * 8;   // tmem slot, abort flag
// Fused final resize (RS kernels): each epilogue warpgroup uses its half of
// the staging region for two buffers T of one 8 x 16-pixel, 32-channel
// slice of the tile in storage precision (64-byte pixel rows; 16-byte chunk
// c of row r sits at chunk c ^ ((r >> 1) & 3), so a warp's row writes are
// free of bank conflicts); the resized pixels go straight to global memory.
constexpr int kRsHalfBytes = 2 * kStageBytes;           // 32 KB per warpgroup
constexpr int kRsChunk = 32;                            // channels per resize step
constexpr int kRsTBytes = kM * 64;                      // T: 8 KB
constexpr int kRsOutY = 7, kRsOutX = 14;                // resized pixels per tile
constexpr int kRsOffGo = 2 * kRsTBytes;
static_assert(kRsOffGo + 16 <= kRsHalfBytes, "resize staging exceeds the half region");
constexpr int kOffBias = kOffMisc + 16;
constexpr int kSmemBytes = kOffBias + kLogN * 4 + 1024;  // + base alignment slack

struct Params {
  CUtensorMap gmap;   // guide  [B, 2H, 2W, 64]      box {64, 16, 8, 1}
  CUtensorMap vmap;   // value  [B, H, W, C]         box {64, 12, 8, 1}
  CUtensorMap omap;   // out    [B, 2H, 2W, C]       box {64, 16, 2, 1} (one warp's rows)
  const float* weight;  // [K][64] fp32
  const float* bias;    // [K] fp32 or null
  int8_t dy[kLogN];
  int8_t dx[kLogN];
  int H, W, nchunks, tiles_x, tiles_y, num_tiles;
  int res_k;            // residual channels (min(K, Cg) when conv_res, else 0)
  // fused guide (GF kernels): the guide is never stored.  gmap reads the
  // guide block's activation h and gmap2 its residual input u (64 channels
  // each); guide = w_guide . h + b_guide + u, and the prologue folds it into
  // the projection: logits = [A . w_guide | A] . [h | u] + bias + A . b_guide
  // with A = weight (+ the identity on the first K channels when conv_res).
  CUtensorMap gmap2;
  const float* w_guide;  // [64][64] fp32 (out, in)
  const float* b_guide;  // [64] fp32 or null
  int conv_res;
  int hardmax;
  int margin;           // max |offset| (cells this close to a border may clamp)
  uint64_t timeout_ns;  // limit of every mbarrier wait
  unsigned int* host_status;  // host-visible status word or null
  int test_fault;       // 1: the guide producer issues no loads (tests the timeout path)
  // fused final resize (RS kernels): the attender output [2H, 2W] is never
  // stored; the resized output [Ho, Wo] is written by plain stores.
  int Hi, Wi;           // attender output size (2H, 2W)
  float scale_h, scale_w;  // Hi / Ho, Wi / Wo (align_corners=False)
  void* rs_out; int64_t rs_b, rs_h, rs_w;  // the resized output, element strides (channel stride 1)
};

// Bounded mbarrier wait recording expiries in this kernel's status word.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag, unsigned where,
                                          const WaitLimit& limit) {
  if (mbar_try(b, parity)) return true;  // completed phase: no call into the bounded slow path
  return mbar_wait_status(b, parity, abort_flag, where, limit, &g_tc_status);
}

template <typename T> struct Store;
template <> struct Store<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  __device__ __forceinline__ static uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  __device__ __forceinline__ static float from_bits(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
  // the two values of a packed pair (low half first) as fp32
  __device__ __forceinline__ static float2 unpack2(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr CUtensorMapDataType kMapType = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
};
template <> struct Store<__half> {
  static constexpr uint32_t kFmt = 0;
  __device__ __forceinline__ static uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  __device__ __forceinline__ static float from_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  __device__ __forceinline__ static float2 unpack2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr CUtensorMapDataType kMapType = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
};

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

template <typename T, int K, bool RS, bool GF>
__global__ void __launch_bounds__(kThreads, 1) la_tc_kernel(const __grid_constant__ Params p) {
  // guide tile slots: two single-source tiles, or one slot holding both
  // sources of the fused guide (the softmax never reads it then, so the slot
  // frees as soon as the logits MMA has completed)
  constexpr int kGSlots = GF ? 1 : 2;
  using S = Store<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sV = smem + kOffV;
  uint8_t* sG = smem + kOffG;
  uint8_t* sStage = smem + kOffStage;
  uint8_t* sW = smem + kOffW;
  uint8_t* sA2 = smem + kOffA2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* g_full = bars;
  uint64_t* g_empty = g_full + 2;
  uint64_t* v_full = g_empty + 2;
  uint64_t* v_empty = v_full + kNU;
  uint64_t* log_full = v_empty + kNU;
  uint64_t* log_empty = log_full + 2;
  uint64_t* a2_full = log_empty + 2;
  uint64_t* a2_empty = a2_full + 2;
  uint64_t* out_full = a2_empty + 2;   // per accumulator half
  uint64_t* out_empty = out_full + 2;
  uint64_t* drain = out_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  float* sBias = reinterpret_cast<float*>(smem + kOffBias);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  // ---------------------------------------------------------------- setup
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&g_full[i], 1);
      mbar_init(&g_empty[i], GF ? 1 : 1 + 4);  // logits MMA done (+ 4 softmax warps read the residual)
      mbar_init(&log_full[i], 1);
      mbar_init(&log_empty[i], 4);    // 4 softmax warps
      mbar_init(&a2_full[i], 4);      // 4 softmax warps
      mbar_init(&a2_empty[i], 1);
      mbar_init(&out_full[i], 1);
      mbar_init(&out_empty[i], 4);    // 4 epilogue warps
    }
    for (int i = 0; i < kNU; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
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
  // Programmatic dependent launch: everything above touches no global
  // memory, so it overlaps the tail of the previous kernel in the stream;
  // nothing below may read inputs before that kernel has completed.  The
  // next kernel may start its own prologue as soon as SMs free up.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  // Projection weights in the storage type, K-major with the 128-byte swizzle
  // (row n = logit n, 64 guide channels per 128-byte row).
  if constexpr (!GF) {
    for (int idx = tid; idx < kLogN * 64; idx += kThreads) {
      const int n = idx >> 6, c = idx & 63;
      const float w = (n < K) ? p.weight[n * 64 + c] : 0.f;
      *reinterpret_cast<uint16_t*>(sW + n * 128 + ((((c >> 3) ^ (n & 7)) << 4)) + (c & 7) * 2) = S::bits(w);
    }
    for (int k = tid; k < kLogN; k += kThreads) sBias[k] = (p.bias != nullptr && k < K) ? p.bias[k] : 0.f;
  } else {
    // A = weight (+ identity on the first K channels with conv_res): source 0
    // (h) gets A . w_guide, source 1 (u) gets A, the bias gains A . b_guide;
    // computed in fp32 from copies in the (not yet used) A-matrix buffers,
    // rounded once to the storage type
    float* sWg = reinterpret_cast<float*>(sA2);  // w_guide [64 out][64 in]
    float* sAm = sWg + 64 * 64;                  // A [32][64]
    static_assert((64 * 64 + kLogN * 64) * 4 <= 2 * kA2Bytes, "prologue scratch exceeds the A buffers");
    for (int i = tid; i < 64 * 64; i += kThreads) sWg[i] = p.w_guide[i];
    for (int i = tid; i < kLogN * 64; i += kThreads) {
      const int n = i >> 6, j = i & 63;
      sAm[i] = n < K ? p.weight[n * 64 + j] + ((p.conv_res && j == n) ? 1.f : 0.f) : 0.f;
    }
    __syncthreads();
    for (int idx = tid; idx < 2 * kLogN * 64; idx += kThreads) {
      const int src = idx / (kLogN * 64), n = (idx >> 6) % kLogN, c = idx & 63;
      float w = 0.f;
      if (src == 1) {
        w = sAm[n * 64 + c];
      } else {
#pragma unroll 16
        for (int j = 0; j < 64; ++j) w = fmaf(sAm[n * 64 + j], sWg[j * 64 + c], w);
      }
      *reinterpret_cast<uint16_t*>(sW + src * kWBytes + n * 128 + ((((c >> 3) ^ (n & 7)) << 4)) + (c & 7) * 2) =
          S::bits(w);
    }
    for (int k = tid; k < kLogN; k += kThreads) {
      float bk = 0.f;
      if (k < K) {
        bk = p.bias != nullptr ? p.bias[k] : 0.f;
        if (p.b_guide != nullptr)
          for (int j = 0; j < 64; ++j) bk = fmaf(sAm[k * 64 + j], p.b_guide[j], bk);
      }
      sBias[k] = bk;
    }
  }
  fence_proxy_async();  // sW is read by the tensor core (async proxy)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int local_tiles = 0;
  for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) ++local_tiles;
  const WaitLimit tmo{p.timeout_ns, p.host_status};
  const int half_chunks = (p.nchunks + 1) / 2;

  if (warp == 0 || warp == kGuideWarp) {
    // ------------------------------------------------------------ producers
    // warp 0 streams the value windows through the ring; a separate warp
    // streams the guide tiles so that they are never queued behind a value
    // load that waits for ring space (the logits of tile n+1 gate the MMA
    // issue order)
    if (lane == 0) {
      bool ok = true;
      if (warp == kGuideWarp) {
        prefetch_map(&p.gmap);
        for (int n = 0; n < local_tiles && ok; ++n) {
          const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
          const int s = n % kGSlots;
          ok = mbar_wait(&g_empty[s], ((n / kGSlots) & 1) ^ 1, abort_flag, 1, tmo);
          if (!ok) break;
          if (p.test_fault == 1) continue;  // the guide never arrives: consumers time out
          if constexpr (GF) {  // both sources into the one slot
            mbar_expect_tx(&g_full[0], 2 * kGBytes);
            tma_load(sG, &p.gmap, &g_full[0], 0, 2 * tl.cx0, 2 * tl.cy0, tl.b);
            tma_load(sG + kGBytes, &p.gmap2, &g_full[0], 0, 2 * tl.cx0, 2 * tl.cy0, tl.b);
          } else {
            mbar_expect_tx(&g_full[s], kGBytes);
            tma_load(sG + s * kGBytes, &p.gmap, &g_full[s], 0, 2 * tl.cx0, 2 * tl.cy0, tl.b);
          }
        }
      } else {
        prefetch_map(&p.vmap);
        prefetch_map(&p.omap);
        uint32_t vc = 0;
        for (int n = 0; n < local_tiles && ok; ++n) {
          const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
          // value window, one ring unit per accumulator half (<= 3 chunks of
          // 64 channels, contiguous so that one MMA spans them)
          for (int h = 0; h < 2 && ok; ++h) {
            const int j0 = h * half_chunks, j1 = min(p.nchunks, j0 + half_chunks);
            if (j0 >= j1) continue;
            const int slot = vc % kNU;
            ok = mbar_wait(&v_empty[slot], ((vc / kNU) & 1) ^ 1, abort_flag, 1, tmo);
            if (!ok) break;
            mbar_expect_tx(&v_full[slot], (j1 - j0) * kVBytes);
            for (int j = j0; j < j1; ++j)
              tma_load(sV + slot * kUnitBytes + (j - j0) * kVBytes, &p.vmap, &v_full[slot], j * kChunk,
                       tl.cx0 - 2, tl.cy0 - 2, tl.b);
            ++vc;
          }
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
      constexpr uint32_t kIdLog = idesc_f16(S::kFmt, 0, kM, kLogN);
      const uint32_t aW = su32(sW);
      uint32_t vc = 0;
      bool ok = true;
      auto logits = [&](int n) -> bool {
        const int s = n & 1;
        const uint32_t ph = (n >> 1) & 1;
        const int gs = n % kGSlots;
        if (!mbar_wait(&g_full[gs], (n / kGSlots) & 1, abort_flag, 2, tmo)) return false;
        if (!mbar_wait(&log_empty[s], ph ^ 1, abort_flag, 2, tmo)) return false;
        tc_fence_after();
        const uint32_t aG = su32(sG + gs * kGBytes);
#pragma unroll
        for (int src = 0; src < (GF ? 2 : 1); ++src)
#pragma unroll
          for (int k = 0; k < 4; ++k)  // K = 64 channels per source in steps of 16
            tc_mma(tmem + kLogCol + kLogN * s, mdesc(aG + src * kGBytes + 32 * k, 16, 1024, kLayoutSw128),
                   mdesc(aW + src * kWBytes + 32 * k, 16, 1024, kLayoutSw128), kIdLog, (src | k) > 0);
        tc_commit(&log_full[s]);
        tc_commit(&g_empty[gs]);
        return true;
      };
      if (local_tiles > 0) ok = logits(0);
      for (int n = 0; n < local_tiles && ok; ++n) {
        if (n + 1 < local_tiles) {
          ok = logits(n + 1);
          if (!ok) break;
        }
        const int s = n & 1;
        const uint32_t ph = (n >> 1) & 1;
        ok = mbar_wait(&a2_full[s], ph, abort_flag, 2, tmo);
        if (!ok) break;
        tc_fence_after();
        const uint32_t aA = su32(sA2 + s * kA2Bytes);
        // two accumulator halves so that the epilogue of one overlaps the
        // MMAs of the other
        for (int h = 0; h < 2 && ok; ++h) {
          const int j0 = h * half_chunks, j1 = min(p.nchunks, j0 + half_chunks);
          if (j0 >= j1) continue;
          ok = mbar_wait(&out_empty[h], (n & 1) ^ 1, abort_flag, 2, tmo);
          if (!ok) break;
          tc_fence_after();
          const int slot = vc % kNU;
          ok = mbar_wait(&v_full[slot], (vc / kNU) & 1, abort_flag, 2, tmo);
          if (!ok) break;
          tc_fence_after();
          ++vc;
          const uint32_t aV = su32(sV + slot * kUnitBytes);
          const uint32_t id_out = idesc_f16(S::kFmt, 1, kM, kChunk * (j1 - j0));
#pragma unroll
          for (int ks = 0; ks < kKSteps; ++ks)
            tc_mma(tmem + kChunk * j0, mdesc(aA + 256 * ks, 128, kA2Sbo, kLayoutNone),
                   mdesc(aV + 2048 * ks, kVBytes, 1024, kLayoutSw128), id_out, ks > 0);
          tc_commit(&v_empty[slot]);
          if (!ok) break;
          tc_commit(&out_full[h]);
        }
        if (!ok) break;
        tc_commit(&a2_empty[s]);
      }
      // all issued MMAs complete before TMEM can be released (this wait
      // ignores the abort flag: it must not be cut short by another role)
      tc_commit(drain);
      mbar_wait(drain, 0, abort_flag + 1, 2, tmo);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax
    // two warpgroups: warps 2-5 take the even tiles (slot 0), warps 6-9 the
    // odd tiles (slot 1); each warp owns TMEM lane quarter warp % 4
    const int q = warp & 3;
    const int wg = (warp - 2) >> 2;
    const int i = 32 * q + lane;  // TMEM lane == pixel of the tile
    const int py = i >> 4, px = i & 15;
    const int cr = py >> 1, cc = px >> 1;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    for (int n = wg; n < local_tiles; n += 2) {
      const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
      const int s = n & 1;
      const uint32_t ph = (n >> 1) & 1;
      if (!mbar_wait(&log_full[s], ph, abort_flag, 3, tmo)) break;
      tc_fence_after();
      uint32_t r[32];
      tc_ld32(lane_base + kLogCol + kLogN * s, r);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&log_empty[s]);
      if (!GF && !mbar_wait(&g_full[s], ph, abort_flag, 3, tmo)) break;

      float lg[K];
#pragma unroll
      for (int k = 0; k < K; ++k) lg[k] = __uint_as_float(r[k]) + sBias[k];
      if (!GF && p.res_k > 0) {  // residual_auto: + guide[k] for k < min(K, Cg)
        const uint8_t* grow = sG + s * kGBytes + i * 128;
#pragma unroll
        for (int c8 = 0; c8 < (K + 7) / 8; ++c8) {
          const uint4 v = *reinterpret_cast<const uint4*>(grow + ((c8 ^ (i & 7)) << 4));
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int k = c8 * 8 + e;
            if (k < K && k < p.res_k)
              lg[k] += S::from_bits((uint16_t)(w4[e >> 1] >> ((e & 1) * 16)));
          }
        }
      }
      __syncwarp();
      if (!GF && lane == 0) mbar_arrive(&g_empty[s]);

      float pk[K];
      if (p.hardmax) {
        int best = 0;
        float bv = lg[0];
#pragma unroll
        for (int k = 1; k < K; ++k)
          if (lg[k] > bv) { bv = lg[k]; best = k; }
#pragma unroll
        for (int k = 0; k < K; ++k) pk[k] = (k == best) ? 1.f : 0.f;
      } else {
        float m = lg[0];
#pragma unroll
        for (int k = 1; k < K; ++k) m = fmaxf(m, lg[k]);
        float z = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) { pk[k] = __expf(lg[k] - m); z += pk[k]; }
        const float inv = 1.f / z;
#pragma unroll
        for (int k = 0; k < K; ++k) pk[k] *= inv;
      }
      // window column of every offset after replicate clamping
      const int cy = tl.cy0 + cr, cx = tl.cx0 + cc;
      int idx[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int ny = min(max(cy + p.dy[k], 0), p.H - 1) - (tl.cy0 - 2);
        const int nx = min(max(cx + p.dx[k], 0), p.W - 1) - (tl.cx0 - 2);
        idx[k] = ny * kWinX + nx;
      }
      uint32_t dup = 0;
      const bool border = cy < p.margin || cx < p.margin || cy > p.H - 1 - p.margin || cx > p.W - 1 - p.margin;
      if (border) {  // merge offsets that clamp onto the same pixel
#pragma unroll
        for (int k = 1; k < K; ++k) {
#pragma unroll
          for (int j = 0; j < k; ++j) {
            if (!((dup >> k) & 1u) && !((dup >> j) & 1u) && idx[j] == idx[k]) {
              pk[j] += pk[k];
              dup |= 1u << k;
            }
          }
        }
      }
      if (!mbar_wait(&a2_empty[s], ph ^ 1, abort_flag, 3, tmo)) break;
      // row i of A (K-major, no swizzle: 8x16-byte core matrices; 8-row
      // groups kA2Sbo apart, 8-column groups 128 B apart)
      uint8_t* arow = sA2 + s * kA2Bytes + (i >> 3) * kA2Sbo + (i & 7) * 16;
#pragma unroll
      for (int j = 0; j < kWin / 8; ++j) *reinterpret_cast<uint4*>(arow + j * 128) = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int k = 0; k < K; ++k)
        if (!((dup >> k) & 1u))
          *reinterpret_cast<uint16_t*>(arow + (idx[k] >> 3) * 128 + (idx[k] & 7) * 2) = S::bits(pk[k]);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a2_full[s]);
    }
  } else if constexpr (!RS) {
    // ------------------------------------------------------------ epilogue
    // two warpgroups, one per accumulator half: warps 10-13 drain half 0,
    // warps 14-17 half 1.  Each warp owns TMEM lanes 32q..32q+31 = output
    // rows 2q, 2q+1 of the tile and stores them with its own TMA box from its
    // own staging buffer, so warps never wait for each other.
    const int q = warp & 3;
    const int h = (warp - 10) >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    uint8_t* bufs = sStage + (warp - 10) * 2 * kWarpStage;  // two staging buffers per warp
    uint32_t jw = 0;
    const int j0 = h * half_chunks, j1 = min(p.nchunks, j0 + half_chunks);
    for (int n = 0; n < local_tiles && j0 < j1; ++n) {
      const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
      if (!mbar_wait(&out_full[h], n & 1, abort_flag, 4, tmo)) break;
      tc_fence_after();
      for (int j = j0; j < j1; ++j) {
        uint32_t r[64];
        tc_ld32(lane_base + kChunk * j, r);
        tc_ld32(lane_base + kChunk * j + 32, r + 32);
        tc_wait_ld();
        if (j + 1 == j1) {  // last TMEM read of this half is complete
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&out_empty[h]);
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
          tma_store(&p.omap, buf, j * kChunk, 2 * tl.cx0, 2 * tl.cy0 + 2 * q, tl.b);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  } else {
    // ------------------------------------------------- epilogue + resize
    // The attender output is resampled before it is stored (the bilinear
    // F.interpolate, align_corners=False, of the fast path's final resize).
    // The resize maps 8 input rows / 16 input columns onto exactly 7 / 14
    // output rows / columns (host-checked with the same source-index
    // formula), so a tile's output pixels depend on that tile alone.  Per
    // 32-channel step the warpgroup writes the tile in storage precision
    // (rounded as the stored attender output would be) to T, and 112 of its
    // threads resample it in fp32, each storing one output column x 8
    // channels over 3-4 rows straight to global memory.  T is
    // double-buffered: the threads wait for each other once per step (T
    // complete).  One thread waits on the accumulator barrier and shares the
    // outcome, so all 128 threads always take the same path.
    const int q = warp & 3;
    const int h = (warp - 10) >> 2;
    const int t = tid - (10 + 4 * h) * 32;  // thread in the warpgroup
    const bool leader = t == 0;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    uint8_t* region = sStage + h * kRsHalfBytes;
    volatile int* go = reinterpret_cast<volatile int*>(region + kRsOffGo);
    const int bar_t = 1 + h;
    // resampling work of this thread: output column oc of the tile,
    // 8-channel group cg of the step, output rows [ry0, ry1)
    const bool worker = t < 2 * kRsOutX * 4;
    const int cg = t & 3;
    const int oc = (t >> 2) % kRsOutX;
    const int ry0 = t < kRsOutX * 4 ? 0 : 4;  // output rows 0-3, or 4-6
    const int j0 = h * half_chunks, j1 = min(p.nchunks, j0 + half_chunks);
    const int s0 = j0 * (kChunk / kRsChunk), s1 = j1 * (kChunk / kRsChunk);  // 32-channel steps
    uint32_t step = 0;
    // the lane's pixel (TMEM lane = pixel of the tile) of one 32-channel
    // step into T, rounded to the storage type
    auto pack32 = [&](const uint32_t* r, uint32_t* pk) {  // 32 fp32 -> 16 words of 2 storage values
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = S::pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    };
    auto to_t = [&](uint8_t* sT, const uint32_t* pk) {
      const int row = 32 * q + lane;
      uint8_t* trow = sT + row * 64;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(trow + ((c ^ ((row >> 1) & 3)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    };
    for (int n = 0; n < local_tiles && s0 < s1; ++n) {
      const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
      if (leader) *go = mbar_wait(&out_full[h], n & 1, abort_flag, 4, tmo) ? 1 : 0;
      named_bar(bar_t, 128);
      if (*go == 0) break;
      tc_fence_after();
      // this thread's output column: source columns xa, xa + 1 of the tile
      // (the 7-of-8 pattern the host checked) and PyTorch's fp32 weights
      const int ox = kRsOutX * (tl.cx0 / kCellsX) + oc;
      int x0 = 0, xp = 0;
      float lx0 = 0.f, lx1 = 0.f;
      src_coord_bilinear(ox, p.scale_w, p.Wi, x0, xp, lx0, lx1);
      const int xa = oc + (oc >= 7 ? 1 : 0);
      const float2 lx0v = make_float2(lx0, lx0), lx1v = make_float2(lx1, lx1);
      // vertical weights of this thread's output rows ry0 .. ry0 + 3 (the
      // same for every channel step of the tile)
      float ly0r[4], ly1r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int y0, yp;
        src_coord_bilinear(kRsOutY * (tl.cy0 / kCellsY) + ry0 + i, p.scale_h, p.Hi, y0, yp, ly0r[i], ly1r[i]);
      }
      uint32_t pk[16];
      {
        uint32_t r[32];
        tc_ld32(lane_base + kRsChunk * s0, r);
        tc_wait_ld_regs(r);
        pack32(r, pk);
      }
      if (s0 + 1 == s1) {  // last TMEM read of this half is complete
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&out_empty[h]);
      }
      to_t(region + (step & 1) * kRsTBytes, pk);
      for (int sj = s0; sj < s1; ++sj, ++step) {
        const int b = step & 1;
        const uint8_t* sT = region + b * kRsTBytes;
        named_bar(bar_t, 128);  // T complete (and every thread is past step - 1)
        const bool more = sj + 1 < s1;
        if (worker) {
          // horizontal interpolation of the source rows this thread needs
          // (all loads first), then the vertical one per output row
          // this thread's 8 channels of output column ox, row 7 * ty (+ R0 + i)
          T* orow0 = static_cast<T*>(p.rs_out) + tl.b * p.rs_b + (int64_t)(kRsOutY * (tl.cy0 / kCellsY)) * p.rs_h +
                     (int64_t)ox * p.rs_w + kRsChunk * sj + 8 * cg;
          // horizontal interpolation of source row yl (lx0 * a + lx1 * b)
          auto horiz = [&](int yl, float2* hv) {
            const int pa = yl * 16 + xa, pb = pa + 1;
            const uint4 va = *reinterpret_cast<const uint4*>(sT + pa * 64 + ((cg ^ ((pa >> 1) & 3)) << 4));
            const uint4 vb = *reinterpret_cast<const uint4*>(sT + pb * 64 + ((cg ^ ((pb >> 1) & 3)) << 4));
            const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
            const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              hv[e] = __ffma2_rn(lx0v, S::unpack2(wa[e]), __fmul2_rn(lx1v, S::unpack2(wb[e])));
          };
          // output rows R0 .. R0 + NR - 1 from source rows R0 .. R0 + NR,
          // two horizontally interpolated rows live at a time
          auto sweep = [&](auto r0c, auto nrc) {
            constexpr int R0 = decltype(r0c)::value, NR = decltype(nrc)::value;
            float2 hp[4], hn[4];
            horiz(R0, hp);
#pragma unroll
            for (int i = 0; i < NR; ++i) {
              horiz(R0 + i + 1, hn);
              const float2 ly0v = make_float2(ly0r[i], ly0r[i]), ly1v = make_float2(ly1r[i], ly1r[i]);
              uint32_t o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 v = __ffma2_rn(ly0v, hp[e], __fmul2_rn(ly1v, hn[e]));
                o[e] = S::pack(v.x, v.y);
                hp[e] = hn[e];
              }
              // 16 bytes = 8 channels of one output pixel; a warp writes 8
              // pixels x 64 contiguous bytes per row
              *reinterpret_cast<uint4*>(orow0 + (int64_t)(R0 + i) * p.rs_h) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          };
          if (ry0 == 0) sweep(std::integral_constant<int, 0>{}, std::integral_constant<int, 4>{});
          else sweep(std::integral_constant<int, 4>{}, std::integral_constant<int, 3>{});
        }
        if (more) {  // the next step's columns into the other T buffer (read in step - 1, which every
                     // thread has finished)
          uint32_t r[32];
          tc_ld32(lane_base + kRsChunk * (sj + 1), r);
          tc_wait_ld_regs(r);
          pack32(r, pk);
          if (sj + 2 == s1) {  // last TMEM read of this half is complete
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&out_empty[h]);
          }
          to_t(region + (b ^ 1) * kRsTBytes, pk);
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

// ---------------------------------------------------------------- host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  }
  return fn;
}

}  // namespace tc

// NHWC 4-D map: dims {C, W, H, B}, strides in elements of `es` bytes.
int tc_make_map(CUtensorMap* map, CUtensorMapDataType dt, int es, const void* base, int C, int W, int H, int B,
                int64_t s_w, int64_t s_h, int64_t s_b, int box_c, int box_w, int box_h, CUtensorMapSwizzle swizzle) {
  tc::EncodeTiled enc = tc::encode_fn();
  if (enc == nullptr) return fail(UPLIFT_LA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)s_w * es, (cuuint64_t)s_h * es, (cuuint64_t)s_b * es};
  const cuuint32_t box[4] = {(cuuint32_t)box_c, (cuuint32_t)box_w, (cuuint32_t)box_h, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(UPLIFT_LA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return UPLIFT_LA_OK;
}

namespace tc {

template <typename T, int K, bool RS, bool GF>
int launch_t(const Params& p, int dev, int grid, cudaStream_t stream) {
  auto fn = la_tc_kernel<T, K, RS, GF>;
  // the shared-memory opt-in is per function and device; set it once (two
  // threads racing here both set the same value, which is harmless)
  static std::atomic<bool> configured[64] = {};
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev].store(true, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "tensor-core kernel launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

template <typename T, bool RS, bool GF>
int launch_k(const Params& p, int K, int dev, int grid, cudaStream_t stream) {
  switch (K) {
    case 5: return launch_t<T, 5, RS, GF>(p, dev, grid, stream);
    case 9: return launch_t<T, 9, RS, GF>(p, dev, grid, stream);
    case 13: return launch_t<T, 13, RS, GF>(p, dev, grid, stream);
    case 17: return launch_t<T, 17, RS, GF>(p, dev, grid, stream);
    case 25: return launch_t<T, 25, RS, GF>(p, dev, grid, stream);
    default: return fail(UPLIFT_LA_ERR_SHAPE, "K=%d unsupported", K);
  }
}

template <typename T>
int launch_v(const Params& p, int K, bool rs, bool gf, int dev, int grid, cudaStream_t stream) {
  if (rs) return gf ? launch_k<T, true, true>(p, K, dev, grid, stream) : launch_k<T, true, false>(p, K, dev, grid, stream);
  return gf ? launch_k<T, false, true>(p, K, dev, grid, stream) : launch_k<T, false, false>(p, K, dev, grid, stream);
}

}  // namespace tc

int tc_set_test_hook(int fault, unsigned long long timeout_ns) {
  if (fault < 0 || fault > 1) return fail(UPLIFT_LA_ERR_ARG, "unknown test fault %d", fault);
  tc::g_test_timeout_ns.store(timeout_ns);
  tc::g_test_fault.store(fault);
  return UPLIFT_LA_OK;
}

int tc_test_fault() { return tc::g_test_fault.load(); }
unsigned long long tc_test_timeout_ns() { return tc::g_test_timeout_ns.load(); }

int tc_device_status(bool clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(v));
  if (e != cudaSuccess) {
    fail(UPLIFT_LA_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
    return -1;
  }
  if (clear && v != 0) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(zero));
    if (e != cudaSuccess) {
      fail(UPLIFT_LA_ERR_CUDA, "status clear: %s", cudaGetErrorString(e));
      return -1;
    }
  }
  return (int)v;
}

static bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool tc_eligible(const TcArgs& a, const char** why) {
  auto no = [&](const char* m) { if (why) *why = m; return false; };
  if (a.dtype != UPLIFT_LA_BF16 && a.dtype != UPLIFT_LA_F16) return no("storage type is not bf16/fp16");
  if (a.Cg != 64) return no("guide channels != 64");
  if (a.C % tc::kChunk != 0 || a.C > tc::kMaxC) return no("value channels not a multiple of 64 up to 384");
  if (a.K != 5 && a.K != 9 && a.K != 13 && a.K != 17 && a.K != 25) return no("K not in {5, 9, 13, 17, 25}");
  if (a.pn > 2) return no("pn > 2");
  if (a.B < 1 || a.H < 1 || a.W < 1) return no("empty problem");
  if (a.B > 65535 || a.H > (1 << 20) || a.W > (1 << 20)) return no("too large for the tile grid");
  if (!a16(a.guide) || !a16(a.value) || !a16(a.out)) return no("base pointers not 16-byte aligned");
  const int64_t st[9] = {a.g_b, a.g_h, a.g_w, a.v_b, a.v_h, a.v_w, a.o_b, a.o_h, a.o_w};
  for (int i = 0; i < 9; ++i)
    if (st[i] % 8 != 0 || st[i] <= 0) return no("strides not multiples of 16 bytes");
  if (a.guide2 != nullptr) {
    if (!a16(a.guide2)) return no("residual input not 16-byte aligned");
    if (a.g2_b % 8 != 0 || a.g2_h % 8 != 0 || a.g2_w % 8 != 0 || a.g2_b <= 0 || a.g2_h <= 0 || a.g2_w <= 0)
      return no("residual input strides not multiples of 16 bytes");
    if (a.w_guide == nullptr) return no("no guide block weight");
  }
  return true;
}

bool tc_resize_eligible(const TcArgs& a, const char** why) {
  auto no = [&](const char* m) { if (why) *why = m; return false; };
  using namespace tc;
  const int Hi = 2 * a.H, Wi = 2 * a.W;
  if (a.Ho < 1 || a.Wo < 1) return no("empty output size");
  // tiles of 8 x 16 attender pixels become tiles of 7 x 14 output pixels
  if ((int64_t)a.Ho * 8 != (int64_t)Hi * kRsOutY || (int64_t)a.Wo * 16 != (int64_t)Wi * kRsOutX)
    return no("output size is not 7/8 of the attender output in both dimensions");
  if (a.H % kCellsY != 0 || a.W % kCellsX != 0) return no("attender output not a whole number of 8 x 16 tiles");
  // every output row / column must read its two source rows / columns from
  // the 8 / 16 of its own tile (PyTorch's source-index formula, fp32)
  const float sh = (float)Hi / (float)a.Ho, sw = (float)Wi / (float)a.Wo;
  // (exactly: output row 7m + r reads input rows 8m + r and 8m + r + 1, and
  // output column 14m + c reads 16m + c + (c >= 7) and the one after -- the
  // fixed pattern the kernel's resampling is unrolled for)
  for (int d = 0; d < a.Ho; ++d) {
    int i0, ip;
    float l0, l1;
    src_coord_bilinear(d, sh, Hi, i0, ip, l0, l1);
    const int r = d % kRsOutY;
    if (i0 != (d / kRsOutY) * 2 * kCellsY + r || ip != 1) return no("a resized row does not read rows r, r + 1 of its tile");
  }
  for (int d = 0; d < a.Wo; ++d) {
    int i0, ip;
    float l0, l1;
    src_coord_bilinear(d, sw, Wi, i0, ip, l0, l1);
    const int c = d % kRsOutX;
    if (i0 != (d / kRsOutX) * 2 * kCellsX + c + (c >= 7 ? 1 : 0) || ip != 1)
      return no("a resized column does not read its tile's columns in the 7-of-8 pattern");
  }
  return true;
}

int tc_launch(const TcArgs& a, cudaStream_t stream) {
  using namespace tc;
  Params p;
  memset(&p, 0, sizeof(p));
  const bool rs = a.Ho > 0;
  const CUtensorMapDataType dt = a.dtype == UPLIFT_LA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc = tc_make_map(&p.gmap, dt, 2, a.guide, a.Cg, 2 * a.W, 2 * a.H, a.B, a.g_w, a.g_h, a.g_b, 64, 16, 8);
  if (rc == UPLIFT_LA_OK && a.guide2 != nullptr)
    rc = tc_make_map(&p.gmap2, dt, 2, a.guide2, a.Cg, 2 * a.W, 2 * a.H, a.B, a.g2_w, a.g2_h, a.g2_b, 64, 16, 8);
  if (rc == UPLIFT_LA_OK) rc = tc_make_map(&p.vmap, dt, 2, a.value, a.C, a.W, a.H, a.B, a.v_w, a.v_h, a.v_b, 64, kWinX, 8);
  if (rc == UPLIFT_LA_OK && !rs)
    rc = tc_make_map(&p.omap, dt, 2, a.out, a.C, 2 * a.W, 2 * a.H, a.B, a.o_w, a.o_h, a.o_b, 64, 16, 2);
  if (rc != UPLIFT_LA_OK) return rc;
  p.Hi = 2 * a.H;
  p.Wi = 2 * a.W;
  if (rs) {
    p.rs_out = a.out;
    p.rs_b = a.o_b;
    p.rs_h = a.o_h;
    p.rs_w = a.o_w;
  }
  p.scale_h = rs ? (float)p.Hi / (float)a.Ho : 0.f;
  p.scale_w = rs ? (float)p.Wi / (float)a.Wo : 0.f;
  p.weight = a.weight;
  p.bias = a.bias;
  int margin = 0;
  for (int k = 0; k < a.K; ++k) {
    p.dy[k] = a.offsets[2 * k];
    p.dx[k] = a.offsets[2 * k + 1];
    margin = std::max(margin, std::max(abs((int)p.dy[k]), abs((int)p.dx[k])));
  }
  p.H = a.H;
  p.W = a.W;
  p.nchunks = a.C / kChunk;
  p.tiles_x = (a.W + kCellsX - 1) / kCellsX;
  p.tiles_y = (a.H + kCellsY - 1) / kCellsY;
  const int64_t nt = (int64_t)p.tiles_x * p.tiles_y * a.B;
  if (nt >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "too many tiles");
  p.num_tiles = (int)nt;
  p.res_k = (a.conv_res && a.guide2 == nullptr) ? std::min(a.K, a.Cg) : 0;
  p.w_guide = a.w_guide;
  p.b_guide = a.b_guide;
  p.conv_res = a.conv_res;
  p.timeout_ns = tc_test_timeout_ns() != 0 ? tc_test_timeout_ns() : kTimeoutNs;
  p.host_status = host_status_word();
  p.test_fault = tc_test_fault();
  p.hardmax = a.hardmax;
  p.margin = margin;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(UPLIFT_LA_ERR_NO_DEVICE, "cudaGetDevice failed");
  static std::atomic<int> sm_count[64] = {};
  int sms = (dev >= 0 && dev < 64) ? sm_count[dev].load(std::memory_order_relaxed) : 0;
  if (sms == 0) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (dev >= 0 && dev < 64) sm_count[dev].store(sms, std::memory_order_relaxed);
  }
  const int grid = (int)std::min<int64_t>(nt, cta_budget(sms));
  const bool gf = a.guide2 != nullptr;
  return a.dtype == UPLIFT_LA_BF16 ? launch_v<__nv_bfloat16>(p, a.K, rs, gf, dev, grid, stream)
                                   : launch_v<__half>(p, a.K, rs, gf, dev, grid, stream);
}

}  // namespace ula
