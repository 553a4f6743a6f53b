// Tensor-core dlogit of the Local Attender backward for B200 (sm_100a):
// softmax weights, dP, dl, dguide and dW / db for 16-bit storage, one tile
// of 4 x 8 coarse cells = 8 x 16 output pixels (M = 128, TMEM lane = pixel)
// at a time, as in the forward kernel.  Per tile
//
//   logits[128 x 32] = G[128 x 64] . (W_hi + W_lo)^T       (tcgen05, 8 MMAs)
//   P = softmax(logits + bias + residual)                   (CUDA cores)
//   dPwin[128 x 96]  = dout[128 x C] . Vwin[96 x C]^T       (tcgen05, 4 per 64 ch)
//   dP_k = dPwin[p][window pixel of offset k]; dl = P (dP - <P, dP>)
//   dguide[128 x 64] = (dl_hi + dl_lo) . (W_hi + I) + dl_hi . W_lo
//                                                           (tcgen05, 10 MMAs)
//   dW^T[128 x 64]  += [G | 1]^T . [dl_hi | dl_lo]          (tcgen05, 8 MMAs)
//
// (W_hi / W_lo and dl_hi / dl_lo are the two-term splits of the fp32 weights
// and of dl into the storage type, and I the identity on the residual
// channels, so logits, dW and dguide keep fp32-level accuracy from exact
// 16-bit products with fp32 accumulation.)  dW and db accumulate in TMEM over
// all of a CTA's tiles -- db is the row of the constant ones channel -- and
// are added to global memory once per CTA.  The softmax weights are also
// written to the fp32 workspace the tensor-core dV (la_bwd_dv.cu) reads.
// Reference: autograd through LocalAttender.forward, uplift/uplift.py:801-847.
//
// Roles (480 threads, one CTA per SM, persistent over tiles): warp 0 TMA
// producer (guide tile into one of four slots -- a tile's guide is held from
// its load to its dW, and four slots let the next tiles' guides load while
// that runs; dout and value window in 64-channel chunks through a 3-stage
// ring); warp 1 TMEM owner + front MMA issuer (logits and dP of every tile,
// up to three tiles ahead of the compute warps: three TMEM slots); warp 14
// back MMA issuer (dW and dguide of each tile as its dl arrives, so that
// they never hold up the next tiles' dP); warps 2-9 two compute warpgroups
// (even / odd tiles; a thread per pixel); warps 10-13 dguide epilogue (TMEM
// -> storage type -> swizzled staging -> TMA store) and, at the end, the
// dW / db atomics.  Every mbarrier wait is bounded; on expiry the CTA
// records the role in this kernel's status word (and the registered host
// word), drains and exits.  The wait's completed-phase test is inlined: a
// call into the bounded slow path costs a single-thread issuer hundreds of
// cycles, and the issuers pass about ten waits per tile.

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

__device__ unsigned int g_dl_status;

namespace dltc {

using namespace ::ula::tc;

constexpr int kCellsY = 4, kCellsX = 8;        // cells per tile
constexpr int kM = 128;                        // output pixels per tile
constexpr int kWinX = 12, kWin = 96;           // value window 8 x 12 (pn <= 2)
constexpr int kChunk = 64;
constexpr int kMaxC = 384;
constexpr int kLogN = 32;
constexpr int kThreads = 480;
constexpr int kTmemCols = 512;
constexpr uint64_t kTimeoutNs = 2000000000ull;

constexpr int kGBytes = kM * 128;              // 16 KB: 128 px x 64 ch (guide tile, dout box)
constexpr int kVBytes = kWin * 128;            // 12 KB: 96 px x 64 ch
constexpr int kStageBytes = kGBytes + kVBytes; // 28 KB: dout box + value box
constexpr int kStages = 3;
constexpr int kSlots = 3;                      // logits / dP TMEM slots
constexpr int kGSlots = 4;                     // guide slots: a tile's guide is held from its load to its dW
constexpr int kConstBytes = 16 * 128;          // 2 KB: the ones channel for one 16-pixel K step
constexpr int kWBytes = kLogN * 128;           // 4 KB: 32 logits x 64 ch
constexpr int kDlBytes = kM * 128;             // 16 KB: per pixel [dl_hi x 32 | dl_lo x 32]
constexpr int kWarpStage = 32 * 128;           // 4 KB

constexpr int kOffG = 0;                                  // kGSlots guide slots
constexpr int kOffConst = kOffG + kGSlots * kGBytes;      // the ones channel (db) beside the guide
constexpr int kOffRing = kOffConst + kConstBytes;
constexpr int kOffW = kOffRing + kStages * kStageBytes;   // W_hi, W_lo
constexpr int kOffWg = kOffW + 2 * kWBytes;               // dguide B: [W_hi | W_hi], [W_lo | I]
constexpr int kWgBytes = 64 * 128;                        // 64 guide channels x 64
constexpr int kOffDl = kOffWg + 2 * kWgBytes;             // 2 dl buffers
constexpr int kOffStage = kOffDl + 2 * kDlBytes;
constexpr int kOffBias = kOffStage + 4 * kWarpStage;
constexpr int kOffBar = kOffBias + kLogN * 4;
constexpr int kNumBars = 2 * kGSlots + 4 * kSlots + 2 * kStages + 2 + 2 + 1 + 1 + 1 + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 16 + 1024;
static_assert(kSmemBytes <= 232448, "shared memory");

// TMEM columns
constexpr int kColLog = 0;     // kSlots x 32
constexpr int kColDp = 96;     // kSlots x 96
constexpr int kColDw = 384;    // 64: rows = guide channels (0-63) and the ones channel (64)
constexpr int kColDg = 448;    // 64 (one slot: the epilogue releases it right after its load)
static_assert(kColDp == kSlots * kLogN && kColDw == kColDp + kSlots * kWin && kColDg + 64 == kTmemCols, "TMEM");

struct Params {
  CUtensorMap gmap;   // guide  [B, 2H, 2W, 64]  box {64, 16, 8, 1}
  CUtensorMap dmap;   // dout   [B, 2H, 2W, C]   box {64, 16, 8, 1}
  CUtensorMap vmap;   // value  [B, H, W, C]     box {64, 12, 8, 1}
  CUtensorMap gomap;  // dguide [B, 2H, 2W, 64]  box {64, 16, 2, 1}
  const float* weight;  // [K][64]
  const float* bias;    // [K] or null
  float* probs;         // [B][2H][2W][K] or null
  float* dweight;       // [K][64] or null (accumulated)
  float* dbias;         // [K] or null (accumulated)
  int write_dguide;
  int8_t dy[kLogN];
  int8_t dx[kLogN];
  int H, W, nchunks, tiles_x, tiles_y, num_tiles;
  int res_k, hardmax;
  uint64_t timeout_ns;
  unsigned int* host_status;
};

__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag, unsigned where,
                                          const WaitLimit& limit) {
  if (mbar_try(b, parity)) return true;  // completed phase: no call into the bounded slow path
  return mbar_wait_status(b, parity, abort_flag, where, limit, &g_dl_status);
}

template <typename T> struct St;
template <> struct St<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  __device__ __forceinline__ static uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  __device__ __forceinline__ static float from_bits(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct St<__half> {
  static constexpr uint32_t kFmt = 0;
  __device__ __forceinline__ static uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  __device__ __forceinline__ static float from_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
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

// 128-byte-swizzled K-major row n of a [rows x 64] 16-bit tile: element c.
__device__ __forceinline__ int sw128(int n, int c) { return n * 128 + ((((c >> 3) ^ (n & 7)) << 4)) + (c & 7) * 2; }

template <typename T, int K>
__global__ void __launch_bounds__(kThreads, 1) la_dl_tc_kernel(const __grid_constant__ Params p) {
  using S = St<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sG = smem + kOffG;
  uint8_t* sConst = smem + kOffConst;
  uint8_t* sRing = smem + kOffRing;
  uint8_t* sW = smem + kOffW;
  uint8_t* sWg = smem + kOffWg;
  uint8_t* sDl = smem + kOffDl;
  uint8_t* sStage = smem + kOffStage;
  float* sBias = reinterpret_cast<float*>(smem + kOffBias);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* g_full = bars;
  uint64_t* g_empty = g_full + kGSlots;
  uint64_t* r_full = g_empty + kGSlots;
  uint64_t* r_empty = r_full + kStages;
  uint64_t* log_full = r_empty + kStages;
  uint64_t* log_empty = log_full + kSlots;
  uint64_t* dp_full = log_empty + kSlots;
  uint64_t* dp_empty = dp_full + kSlots;
  uint64_t* dl_full = dp_empty + kSlots;
  uint64_t* dl_empty = dl_full + 2;
  uint64_t* dg_full = dl_empty + 2;
  uint64_t* dg_empty = dg_full + 1;
  uint64_t* dw_done = dg_empty + 1;
  uint64_t* drain = dw_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kGSlots; ++i) {
      mbar_init(&g_full[i], 1);
      mbar_init(&g_empty[i], 1);    // dW MMA of the tile done
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&log_full[i], 1);
      mbar_init(&log_empty[i], 4);  // 4 compute warps
      mbar_init(&dp_full[i], 1);
      mbar_init(&dp_empty[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dl_full[i], 4);
      mbar_init(&dl_empty[i], 1);
    }
    mbar_init(dg_full, 1);
    mbar_init(dg_empty, 4);         // 4 epilogue warps
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&r_full[i], 1);
      mbar_init(&r_empty[i], 1);
    }
    mbar_init(dw_done, 1);
    mbar_init(drain, 2);
    abort_flag[0] = 0;
    abort_flag[1] = 0;  // stays 0: the flag of waits that must not be aborted
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)), "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // constant operands: W_hi / W_lo (K-major, logits: row = logit), the
  // dguide B tiles (K-major, row = guide channel: [W_hi | W_hi] against
  // [dl_hi | dl_lo], [W_lo | I] against dl_hi and dl_lo), the ones channel
  // beside the guide tile (row = pixel, channel 0 = 1), bias
  for (int idx = tid; idx < kLogN * 64; idx += kThreads) {
    const int n = idx >> 6, c = idx & 63;
    const float w = (n < K) ? p.weight[n * 64 + c] : 0.f;
    const uint16_t hi = S::bits(w);
    const uint16_t lo = S::bits(w - S::from_bits(hi));
    *reinterpret_cast<uint16_t*>(sW + sw128(n, c)) = hi;
    *reinterpret_cast<uint16_t*>(sW + kWBytes + sw128(n, c)) = lo;
    *reinterpret_cast<uint16_t*>(sWg + sw128(c, n)) = hi;
    *reinterpret_cast<uint16_t*>(sWg + sw128(c, n + 32)) = hi;
    *reinterpret_cast<uint16_t*>(sWg + kWgBytes + sw128(c, n)) = lo;
    *reinterpret_cast<uint16_t*>(sWg + kWgBytes + sw128(c, n + 32)) =
        (n < p.res_k && n == c) ? S::bits(1.f) : (uint16_t)0;
  }
  for (int idx = tid; idx < 16 * 64; idx += kThreads) {
    const int px = idx >> 6, c = idx & 63;
    *reinterpret_cast<uint16_t*>(sConst + sw128(px, c)) = (c == 0) ? S::bits(1.f) : (uint16_t)0;
  }
  for (int k = tid; k < kLogN; k += kThreads) sBias[k] = (p.bias != nullptr && k < K) ? p.bias[k] : 0.f;
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int local_tiles = 0;
  for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) ++local_tiles;
  const WaitLimit tmo{p.timeout_ns, p.host_status};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_map(&p.gmap);
      prefetch_map(&p.dmap);
      prefetch_map(&p.vmap);
      bool ok = true;
      uint32_t rc = 0;
      for (int n = 0; n < local_tiles && ok; ++n) {
        const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
        const int s = n % kGSlots;
        ok = mbar_wait(&g_empty[s], ((n / kGSlots) & 1) ^ 1, abort_flag, 1, tmo);
        if (!ok) break;
        mbar_expect_tx(&g_full[s], kGBytes);
        tma_load(sG + s * kGBytes, &p.gmap, &g_full[s], 0, 2 * tl.cx0, 2 * tl.cy0, tl.b);
        for (int j = 0; j < p.nchunks && ok; ++j, ++rc) {
          const int st = rc % kStages;
          ok = mbar_wait(&r_empty[st], ((rc / kStages) & 1) ^ 1, abort_flag, 1, tmo);
          if (!ok) break;
          uint8_t* base = sRing + st * kStageBytes;
          mbar_expect_tx(&r_full[st], kStageBytes);
          tma_load(base, &p.dmap, &r_full[st], j * kChunk, 2 * tl.cx0, 2 * tl.cy0, tl.b);
          tma_load(base + kGBytes, &p.vmap, &r_full[st], j * kChunk, tl.cx0 - 2, tl.cy0 - 2, tl.b);
        }
      }
      if (!ok) {  // let issued loads land before the CTA can exit
        const uint64_t t0 = gtimer();
        while (gtimer() - t0 < 200000ull) {}
      }
    }
  } else if (warp == 1 || warp == 14) {
    // ------------------------------------------------------------ MMA issuers
    // warp 1: logits and dP (front) of every tile, as far ahead as the TMEM
    // slots and the loads allow; warp 14: dW and dguide (back), as each
    // tile's dl arrives.  Each commits only its own MMAs.
    if (lane == 0) {
      constexpr uint32_t kIdLog = idesc_f16(S::kFmt, 0, kM, kLogN);
      constexpr uint32_t kIdDp = idesc_f16(S::kFmt, 0, kM, kWin);
      constexpr uint32_t kIdDw = idesc_f16_ab(S::kFmt, 1, 1, kM, 64);
      constexpr uint32_t kIdDg = idesc_f16(S::kFmt, 0, kM, 64);
      const uint32_t aW = su32(sW), aWg = su32(sWg), aConst = su32(sConst);
      uint32_t rc = 0;
      bool ok = true, first_dw = true;
      auto front = [&](int n) -> bool {  // logits and dP of tile n
        const int s = n % kSlots, sg = n % kGSlots;
        const uint32_t ph = (n / kSlots) & 1;
        if (!mbar_wait(&g_full[sg], (n / kGSlots) & 1, abort_flag, 2, tmo)) return false;
        if (!mbar_wait(&log_empty[s], ph ^ 1, abort_flag, 2, tmo)) return false;
        tc_fence_after();
        const uint32_t aG = su32(sG + sg * kGBytes);
#pragma unroll
        for (int src = 0; src < 2; ++src)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma(tmem + kColLog + kLogN * s, mdesc(aG + 32 * k, 16, 1024, kLayoutSw128),
                   mdesc(aW + src * kWBytes + 32 * k, 16, 1024, kLayoutSw128), kIdLog, (src | k) > 0);
        tc_commit(&log_full[s]);
        if (!mbar_wait(&dp_empty[s], ph ^ 1, abort_flag, 2, tmo)) return false;
        tc_fence_after();
        for (int j = 0; j < p.nchunks; ++j, ++rc) {
          const int st = rc % kStages;
          if (!mbar_wait(&r_full[st], (rc / kStages) & 1, abort_flag, 2, tmo)) return false;
          tc_fence_after();
          const uint32_t aD = su32(sRing + st * kStageBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma(tmem + kColDp + kWin * s, mdesc(aD + 32 * k, 16, 1024, kLayoutSw128),
                   mdesc(aD + kGBytes + 32 * k, 16, 1024, kLayoutSw128), kIdDp, (j | k) > 0);
          tc_commit(&r_empty[st]);
        }
        tc_commit(&dp_full[s]);
        return true;
      };
      auto back = [&](int n) -> bool {  // dW and dguide of tile n
        const int sg = n % kGSlots, s = n & 1;
        if (!mbar_wait(&dl_full[s], (n >> 1) & 1, abort_flag, 2, tmo)) return false;
        if (!mbar_wait(dg_empty, (n & 1) ^ 1, abort_flag, 2, tmo)) return false;
        tc_fence_after();
        const uint32_t aG = su32(sG + sg * kGBytes);
        const uint32_t aDl = su32(sDl + s * kDlBytes);
        // dW^T[128 x 64] += [G | 1]^T . [dl_hi | dl_lo]: A MN-major (M =
        // channels in two 64-wide blocks: the guide tile's 16 pixels of the
        // K step, then the 16 rows of the ones tile, the same for every
        // step), B MN-major (N = the 64 dl columns), K = the 128 pixels
#pragma unroll
        for (int ks = 0; ks < kM / 16; ++ks)
          tc_mma(tmem + kColDw, mdesc(aG + 2048 * ks, aConst - (aG + 2048 * ks), 1024, kLayoutSw128),
                 mdesc(aDl + 2048 * ks, kDlBytes, 1024, kLayoutSw128), kIdDw, (first_dw && ks == 0) ? 0u : 1u);
        first_dw = false;
        // dguide[128 x 64]: both operands K-major in 16-column slices; dl
        // slices 0-1 hold dl_hi, 2-3 dl_lo; [W_hi | W_hi] slices 0-3, then
        // W_lo (slices 0-1 of the second tile) against dl_hi and the
        // identity (slices 2-3) against dl_hi and dl_lo
        constexpr int kDgA[10] = {0, 1, 2, 3, 0, 1, 0, 1, 2, 3};
        constexpr int kDgB[10] = {0, 1, 2, 3, 4, 5, 6, 7, 6, 7};
#pragma unroll
        for (int m = 0; m < 10; ++m)
          tc_mma(tmem + kColDg, mdesc(aDl + 32 * kDgA[m], 16, 1024, kLayoutSw128),
                 mdesc(aWg + (kDgB[m] >> 2) * kWgBytes + 32 * (kDgB[m] & 3), 16, 1024, kLayoutSw128), kIdDg,
                 m > 0);
        tc_commit(&dl_empty[s]);
        tc_commit(&g_empty[sg]);
        tc_commit(dg_full);
        return true;
      };
      if (warp == 1) {
        for (int n = 0; n < local_tiles && ok; ++n) ok = front(n);
      } else {
        for (int n = 0; n < local_tiles && ok; ++n) ok = back(n);
        tc_commit(dw_done);  // every dW MMA is complete
      }
      // all issued MMAs complete before TMEM can be released (the drain
      // barrier takes both issuers' commits; the wait ignores the abort
      // flag: it must not be cut short by another role)
      tc_commit(drain);
      if (warp == 1) mbar_wait(drain, 0, abort_flag + 1, 2, tmo);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ compute
    // warps 2-5 take the even tiles, warps 6-9 the odd ones; a thread per
    // pixel (TMEM lane); the tile's cell row is the warp's lane quarter, so
    // every offset's window row is the same across the warp
    const int q = warp & 3;
    const int wg = (warp - 2) >> 2;
    const int i = 32 * q + lane;
    const int py = i >> 4, px = i & 15;
    const int cc = px >> 1;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    for (int n = wg; n < local_tiles; n += 2) {
      const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
      const int s = n % kSlots, sd = n & 1, sg = n % kGSlots;
      const uint32_t ph = (n / kSlots) & 1;
      if (!mbar_wait(&log_full[s], ph, abort_flag, 3, tmo)) break;
      tc_fence_after();
      uint32_t r[32];
      tc_ld32(lane_base + kColLog + kLogN * s, r);
      tc_wait_ld_regs(r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&log_empty[s]);
      if (!mbar_wait(&g_full[sg], (n / kGSlots) & 1, abort_flag, 3, tmo)) break;
      const int oy = 2 * tl.cy0 + py, ox = 2 * tl.cx0 + px;
      const bool inside = oy < 2 * p.H && ox < 2 * p.W;
      float pk[K];
      {
        float lg[K];
#pragma unroll
        for (int k = 0; k < K; ++k) lg[k] = __uint_as_float(r[k]) + sBias[k];
        if (p.res_k > 0) {  // residual_auto: + guide[k] for k < min(K, Cg)
          const uint8_t* grow = sG + sg * kGBytes + i * 128;
#pragma unroll
          for (int c8 = 0; c8 < (K + 7) / 8; ++c8) {
            const uint4 v = *reinterpret_cast<const uint4*>(grow + ((c8 ^ (i & 7)) << 4));
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int k = c8 * 8 + e;
              if (k < K && k < p.res_k) lg[k] += S::from_bits((uint16_t)(w4[e >> 1] >> ((e & 1) * 16)));
            }
          }
        }
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
      }
      if (p.probs != nullptr && inside) {
        float* pp = p.probs + (((int64_t)tl.b * 2 * p.H + oy) * (2 * p.W) + ox) * K;
#pragma unroll
        for (int k = 0; k < K; ++k) pp[k] = pk[k];
      }
      // dP_k = dPwin[pixel][window pixel of offset k] (replicate clamping,
      // as the forward maps offsets to window columns)
      if (!mbar_wait(&dp_full[s], ph, abort_flag, 3, tmo)) break;
      tc_fence_after();
      const int cy = tl.cy0 + q, cx = tl.cx0 + cc;
      float dp[K];
      {
        // window row wr occupies columns 12 wr .. 12 wr + 11 of the slot;
        // they are read as two 16-column loads from the 16-aligned column
        // below 12 wr, and the lane's column picked by compare-and-select
        int cur = -1, o = 0;
        uint32_t row[32];
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const int wr = min(max(cy + p.dy[k], 0), p.H - 1) - (tl.cy0 - 2);   // the same in the whole warp
          const int wc = min(max(cx + p.dx[k], 0), p.W - 1) - (tl.cx0 - 2);
          if (wr != cur) {
            const int a16 = (kWinX * wr) & ~15;
            tc_ld16(lane_base + kColDp + kWin * s + a16, row);
            tc_ld16(lane_base + kColDp + kWin * s + a16 + 16, row + 16);
            tc_wait_ld_regs(row);
            o = kWinX * wr - a16;  // 0, 4, 8 or 12
            cur = wr;
          }
          const int idx = o + wc;  // < 24
          float a8[8];
#pragma unroll
          for (int c = 0; c < 8; ++c)
            a8[c] = __uint_as_float((idx & 16) ? row[16 + c] : ((idx & 8) ? row[8 + c] : row[c]));
          float a4[4], a2[2];
#pragma unroll
          for (int c = 0; c < 4; ++c) a4[c] = (idx & 4) ? a8[4 + c] : a8[c];
#pragma unroll
          for (int c = 0; c < 2; ++c) a2[c] = (idx & 2) ? a4[2 + c] : a4[c];
          dp[k] = (idx & 1) ? a2[1] : a2[0];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dp_empty[s]);
      // dl = P (dP - <P, dP>) (no gradient through the argmax, and none for
      // pixels outside the map)
      float dot = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) dot = fmaf(pk[k], dp[k], dot);
      if (!mbar_wait(&dl_empty[sd], ((n >> 1) & 1) ^ 1, abort_flag, 3, tmo)) break;
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int k2 = 0; k2 < 16; ++k2) {
        float d0 = 0.f, d1 = 0.f;
        const int k0 = 2 * k2, k1 = 2 * k2 + 1;
        if (k0 < K) d0 = (p.hardmax || !inside) ? 0.f : pk[k0] * (dp[k0] - dot);
        if (k1 < K) d1 = (p.hardmax || !inside) ? 0.f : pk[k1] * (dp[k1] - dot);
        hi[k2] = S::pack(d0, d1);
        const float h0 = S::from_bits((uint16_t)(hi[k2] & 0xffffu)), h1 = S::from_bits((uint16_t)(hi[k2] >> 16));
        lo[k2] = S::pack(d0 - h0, d1 - h1);
      }
      uint8_t* drow = sDl + sd * kDlBytes + i * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        *reinterpret_cast<uint4*>(drow + ((c ^ (i & 7)) << 4)) =
            make_uint4(hi[4 * c], hi[4 * c + 1], hi[4 * c + 2], hi[4 * c + 3]);
        *reinterpret_cast<uint4*>(drow + (((c + 4) ^ (i & 7)) << 4)) =
            make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dl_full[sd]);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // dguide: warp w owns TMEM lanes 32q..32q+31 = output rows 2q, 2q + 1 of
    // the tile and stores them through its own two staging buffers
    const int q = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    uint8_t* buf = sStage + (warp - 10) * kWarpStage;
    bool ok = true;
    for (int n = 0; n < local_tiles; ++n) {
      const TileXY tl = tile_of(p, blockIdx.x + n * gridDim.x);
      if (!mbar_wait(dg_full, n & 1, abort_flag, 4, tmo)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[64];
      tc_ld32(lane_base + kColDg, r);
      tc_ld32(lane_base + kColDg + 32, r + 32);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dg_empty);
      if (!p.write_dguide) continue;
      if (lane == 0) bulk_wait_read0();  // the store of the previous tile has read `buf`
      __syncwarp();
      uint8_t* rowp = buf + lane * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t* src = r + 8 * c;
        uint4 w;
        w.x = S::pack(__uint_as_float(src[0]), __uint_as_float(src[1]));
        w.y = S::pack(__uint_as_float(src[2]), __uint_as_float(src[3]));
        w.z = S::pack(__uint_as_float(src[4]), __uint_as_float(src[5]));
        w.w = S::pack(__uint_as_float(src[6]), __uint_as_float(src[7]));
        *reinterpret_cast<uint4*>(rowp + ((c ^ (lane & 7)) << 4)) = w;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_store(&p.gomap, buf, 0, 2 * tl.cx0, 2 * tl.cy0 + 2 * q, tl.b);
        bulk_commit();
      }
    }
    // dW / db: TMEM row c < 64 holds dW^T[c][hi logits | lo logits], row 64
    // (the ones channel) db
    if (ok && local_tiles > 0 && (p.dweight != nullptr || p.dbias != nullptr) &&
        mbar_wait(dw_done, 0, abort_flag, 4, tmo)) {
      tc_fence_after();
      uint32_t r[64];
      tc_ld32(lane_base + kColDw, r);
      tc_ld32(lane_base + kColDw + 32, r + 32);
      tc_wait_ld();
      const int row = 32 * q + lane;
      if (row < 64 && p.dweight != nullptr) {
#pragma unroll
        for (int k = 0; k < K; ++k)
          atomicAdd(p.dweight + k * 64 + row, __uint_as_float(r[k]) + __uint_as_float(r[32 + k]));
      } else if (row == 64 && p.dbias != nullptr) {
#pragma unroll
        for (int k = 0; k < K; ++k) atomicAdd(p.dbias + k, __uint_as_float(r[k]) + __uint_as_float(r[32 + k]));
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
  auto fn = la_dl_tc_kernel<T, K>;
  static std::atomic<bool> configured[64] = {};  // racing threads set the same value
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev].store(true, std::memory_order_release);
  }
  fn<<<grid, kThreads, kSmemBytes, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "tensor-core dlogit launch: %s", cudaGetErrorString(e));
  return UPLIFT_LA_OK;
}

template <typename T>
int launch_k(const Params& p, int K, int dev, int grid, cudaStream_t stream) {
  switch (K) {
    case 5: return launch_t<T, 5>(p, dev, grid, stream);
    case 9: return launch_t<T, 9>(p, dev, grid, stream);
    case 13: return launch_t<T, 13>(p, dev, grid, stream);
    case 17: return launch_t<T, 17>(p, dev, grid, stream);
    case 25: return launch_t<T, 25>(p, dev, grid, stream);
    default: return fail(UPLIFT_LA_ERR_SHAPE, "tensor-core dlogit: K=%d unsupported", K);
  }
}

}  // namespace dltc

bool dl_tc_eligible(const DlArgs& a, const char** why) {
  auto no = [&](const char* m) { if (why) *why = m; return false; };
  if (a.dtype != UPLIFT_LA_BF16 && a.dtype != UPLIFT_LA_F16) return no("storage type is not bf16/fp16");
  if (a.I != 2) return no("scale I != 2");
  if (a.Cg != 64) return no("guide channels != 64");
  if (a.C % dltc::kChunk != 0 || a.C > dltc::kMaxC) return no("channels not a multiple of 64 up to 384");
  if (a.K != 5 && a.K != 9 && a.K != 13 && a.K != 17 && a.K != 25) return no("K not in {5, 9, 13, 17, 25}");
  for (int k = 0; k < a.K; ++k)
    if (a.dy[k] < -2 || a.dy[k] > 2 || a.dx[k] < -2 || a.dx[k] > 2) return no("offsets beyond +-2");
  if (a.B < 1 || a.H < 1 || a.W < 1) return no("empty problem");
  if (a.B > 65535 || a.H > (1 << 20) || a.W > (1 << 20)) return no("too large for the tile grid");
  auto al = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!al(a.dout) || !al(a.guide) || !al(a.value) || !al(a.dguide)) return no("base pointers not 16-byte aligned");
  const int64_t st[9] = {a.d_b, a.d_h, a.d_w, a.g_b, a.g_h, a.g_w, a.v_b, a.v_h, a.v_w};
  for (int i = 0; i < 9; ++i)
    if (st[i] % 8 != 0 || st[i] <= 0) return no("strides not multiples of 16 bytes");
  if (a.dguide != nullptr && (a.dg_b % 8 != 0 || a.dg_h % 8 != 0 || a.dg_w % 8 != 0 || a.dg_b <= 0 || a.dg_h <= 0 ||
                              a.dg_w <= 0))
    return no("dguide strides not multiples of 16 bytes");
  return true;
}

int dl_tc_launch(const DlArgs& a, cudaStream_t stream) {
  using namespace dltc;
  Params p;
  memset(&p, 0, sizeof(p));
  const CUtensorMapDataType dt = a.dtype == UPLIFT_LA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc = tc_make_map(&p.gmap, dt, 2, a.guide, 64, 2 * a.W, 2 * a.H, a.B, a.g_w, a.g_h, a.g_b, 64, 16, 8);
  if (rc == UPLIFT_LA_OK)
    rc = tc_make_map(&p.dmap, dt, 2, a.dout, a.C, 2 * a.W, 2 * a.H, a.B, a.d_w, a.d_h, a.d_b, 64, 16, 8);
  if (rc == UPLIFT_LA_OK)
    rc = tc_make_map(&p.vmap, dt, 2, a.value, a.C, a.W, a.H, a.B, a.v_w, a.v_h, a.v_b, 64, kWinX, 8);
  if (rc == UPLIFT_LA_OK && a.dguide != nullptr)
    rc = tc_make_map(&p.gomap, dt, 2, a.dguide, 64, 2 * a.W, 2 * a.H, a.B, a.dg_w, a.dg_h, a.dg_b, 64, 16, 2);
  if (rc != UPLIFT_LA_OK) return rc;
  p.weight = a.weight;
  p.bias = a.bias;
  p.probs = a.probs;
  p.dweight = a.dweight;
  p.dbias = a.dbias;
  p.write_dguide = a.dguide != nullptr ? 1 : 0;
  for (int k = 0; k < a.K; ++k) {
    p.dy[k] = a.dy[k];
    p.dx[k] = a.dx[k];
  }
  p.H = a.H;
  p.W = a.W;
  p.nchunks = a.C / kChunk;
  p.tiles_x = (a.W + kCellsX - 1) / kCellsX;
  p.tiles_y = (a.H + kCellsY - 1) / kCellsY;
  const int64_t nt = (int64_t)p.tiles_x * p.tiles_y * a.B;
  if (nt >= (1ll << 31)) return fail(UPLIFT_LA_ERR_SHAPE, "too many tiles");
  p.num_tiles = (int)nt;
  p.res_k = a.conv_res ? std::min(a.K, 64) : 0;
  p.hardmax = a.hardmax;
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
  return a.dtype == UPLIFT_LA_BF16 ? launch_k<__nv_bfloat16>(p, a.K, dev, grid, stream)
                                   : launch_k<__half>(p, a.K, dev, grid, stream);
}

int dl_device_status(bool clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_dl_status, sizeof(v));
  if (e != cudaSuccess) {
    fail(UPLIFT_LA_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
    return -1;
  }
  if (clear && v != 0) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_dl_status, &zero, sizeof(zero));
    if (e != cudaSuccess) {
      fail(UPLIFT_LA_ERR_CUDA, "status clear: %s", cudaGetErrorString(e));
      return -1;
    }
  }
  return (int)v;
}

}  // namespace ula
