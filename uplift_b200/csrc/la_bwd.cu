// C entry points of the Local Attender backward (include/uplift_la.h): argument
// checks, the launch plan (tensor-core dlogit, sliding-window dV, vector
// widths) and, for uplift_la_backward_noalloc, the in-library workspace.
// Kernels: la_bwd.cuh.

#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "la_bwd.cuh"

namespace {

// Argument checks shared by both backward entry points (everything except
// the workspace pointer, which only uplift_la_backward takes).
int check_backward_args(const void* dout, const int64_t dout_strides[4], const void* guide,
                        const int64_t guide_strides[4], const void* value, const int64_t value_strides[4],
                        const float* weight, const void* dguide, const int64_t dguide_strides[4],
                        const void* dvalue, const int64_t dvalue_strides[4], int B, int Cg, int C, int H, int W,
                        int I, int K, const int8_t* offsets, int pn, int dtype) {
  using ula::fail;
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
  if (npix > 0 && (dout == nullptr || guide == nullptr || value == nullptr || weight == nullptr))
    return fail(UPLIFT_LA_ERR_ARG, "null input pointer");
  if (npix >= ((int64_t)1 << 40)) return fail(UPLIFT_LA_ERR_SHAPE, "too many pixels");
  for (int k = 0; k < K; ++k) {
    const int dy = offsets[2 * k], dx = offsets[2 * k + 1];
    if (dy < -pn || dy > pn || dx < -pn || dx > pn)
      return fail(UPLIFT_LA_ERR_OFFSETS, "offset %d = (%d, %d) exceeds pn=%d", k, dy, dx, pn);
  }
  const int64_t* st[5] = {dout_strides, guide_strides, value_strides, dguide_strides, dvalue_strides};
  for (int i = 0; i < 5; ++i)
    if (st[i] != nullptr && st[i][1] != 1 && !(i == 1 || i == 3 ? Cg == 1 : C == 1))
      return fail(UPLIFT_LA_ERR_LAYOUT, "tensors need channel stride 1 (channels_last)");
  return UPLIFT_LA_OK;
}

}  // namespace

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
  const int rc = check_backward_args(dout, dout_strides, guide, guide_strides, value, value_strides, weight, dguide,
                                     dguide_strides, dvalue, dvalue_strides, B, Cg, C, H, W, I, K, offsets, pn, dtype);
  if (rc != UPLIFT_LA_OK) return rc;
  const int64_t npix = (int64_t)B * I * H * I * W;
  if (npix > 0 && probs == nullptr) return fail(UPLIFT_LA_ERR_ARG, "null workspace pointer");
  Args a;
  memset(&a, 0, sizeof(a));
  for (int k = 0; k < K; ++k) {
    a.dy[k] = offsets[2 * k];
    a.dx[k] = offsets[2 * k + 1];
  }
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
  // 16-byte channel vectors for dout / value / dvalue when C and alignment allow
  const int ve = dtype == UPLIFT_LA_F32 ? 4 : 8;
  auto a16 = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  bool vec = C % ve == 0 && a16(dout) && a16(value) && a16(dvalue);
  const int64_t vst[6] = {a.d_b, a.d_h, a.d_w, a.v_b, a.v_h, a.v_w};
  for (int i = 0; i < 6; ++i) vec = vec && vst[i] % ve == 0;
  if (dvalue != nullptr) vec = vec && a.dv_b % ve == 0 && a.dv_h % ve == 0 && a.dv_w % ve == 0;
  const bool gvec = Cg % ve == 0 && a16(guide) && a.g_b % ve == 0 && a.g_h % ve == 0 && a.g_w % ve == 0;
  // sliding-window dV when the offsets are the reference's table for K; row
  // segments sized so that about 2048 threads per SM are busy
  bwd::Plan plan{0, 0, 0, 0, W, 1};
  {
    // tensor-core dlogit: I = 2, even Cg <= 64, C % 32 == 0 (16-bit storage)
    // or C % 16 == 0 (fp32), 16-byte dout / value rows, aligned guide / dguide
    // channel pairs, offsets within +-2, softmax (hardmax has no logit gradient);
    // ULA_BWD_MMA=0 selects the CUDA-core dlogit instead (comparisons)
    int maxd = 0;
    for (int k = 0; k < K; ++k) maxd = std::max(maxd, std::max(std::abs((int)a.dy[k]), std::abs((int)a.dx[k])));
    // (fp32: C % 16 == 0 and 8-byte guide pairs)
    const unsigned pair_align = dtype == UPLIFT_LA_F32 ? 7u : 3u;
    auto ap = [pair_align](const void* q) {
      return q == nullptr || (reinterpret_cast<uintptr_t>(q) & pair_align) == 0;
    };
    bool ok = I == 2 && C % (dtype == UPLIFT_LA_F32 ? 16 : 32) == 0 && vec && Cg % 2 == 0 && Cg <= 64 &&
              !hardmax && maxd <= 2 && ap(guide) && a.g_b % 2 == 0 && a.g_h % 2 == 0 && a.g_w % 2 == 0;
    if (dguide != nullptr) ok = ok && ap(dguide) && a.dg_b % 2 == 0 && a.dg_h % 2 == 0 && a.dg_w % 2 == 0;
    static const bool mma_env = [] {
      const char* e = getenv("ULA_BWD_MMA");
      return e == nullptr || atoi(e) != 0;
    }();
    if (ok && mma_env) plan.mma_pn = maxd < 1 ? 1 : maxd;
  }
  bool canonical = true;
  for (int k = 0; k < K; ++k) {
    int kk = -1;
    switch (K) {
      case 5: kk = bwd::nbh_k<5>(a.dy[k], a.dx[k]); break;
      case 9: kk = bwd::nbh_k<9>(a.dy[k], a.dx[k]); break;
      case 13: kk = bwd::nbh_k<13>(a.dy[k], a.dx[k]); break;
      case 17: kk = bwd::nbh_k<17>(a.dy[k], a.dx[k]); break;
      case 25: kk = bwd::nbh_k<25>(a.dy[k], a.dx[k]); break;
      default: break;
    }
    canonical = canonical && kk == k;
  }
  if (canonical && W > 0) {
    plan.window = 1;
    const int pn_k = (K == 5 || K == 9) ? 1 : 2;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t rows = (int64_t)B * H * (C / (vec ? ve : 1));
    const int64_t want = (int64_t)sms * 2048;
    int nseg = rows >= want ? 1 : (int)std::min<int64_t>((want + rows - 1) / rows, W);
    const int min_len = 8 * pn_k;
    if (nseg > 1 && (W + nseg - 1) / nseg < min_len) nseg = std::max(1, W / min_len);
    plan.seg_len = (W + nseg - 1) / nseg;
    plan.nseg = (W + plan.seg_len - 1) / plan.seg_len;
  }
  if (dvalue != nullptr && dtype != UPLIFT_LA_F32) {
    // tensor-core dV: I = 2, 16-bit storage, C a multiple of 64 up to 384,
    // offsets within +-2, aligned NHWC dout / dvalue (ULA_BWD_DV_TC=0 keeps
    // the CUDA-core kernels, for comparisons)
    static const bool dv_env = [] {
      const char* e = getenv("ULA_BWD_DV_TC");
      return e == nullptr || atoi(e) != 0;
    }();
    DvArgs d;
    d.dout = dout; d.d_b = a.d_b; d.d_h = a.d_h; d.d_w = a.d_w;
    d.probs = probs;
    d.dvalue = dvalue; d.dv_b = a.dv_b; d.dv_h = a.dv_h; d.dv_w = a.dv_w;
    d.B = B; d.C = C; d.H = H; d.W = W; d.I = I; d.K = K; d.dtype = dtype;
    for (int k = 0; k < K; ++k) { d.dy[k] = a.dy[k]; d.dx[k] = a.dx[k]; }
    plan.dv_tc = (dv_env && dv_tc_eligible(d, nullptr)) ? 1 : 0;
  }
  if (dtype != UPLIFT_LA_F32) {
    // tensor-core softmax weights + dlogit: I = 2, 16-bit storage, Cg = 64,
    // C a multiple of 64 up to 384, offsets within +-2 (ULA_BWD_DL_TC=0
    // keeps the probs + dlogit kernels, for comparisons)
    static const bool dl_env = [] {
      const char* e = getenv("ULA_BWD_DL_TC");
      return e == nullptr || atoi(e) != 0;
    }();
    DlArgs d;
    d.dout = dout; d.d_b = a.d_b; d.d_h = a.d_h; d.d_w = a.d_w;
    d.guide = guide; d.g_b = a.g_b; d.g_h = a.g_h; d.g_w = a.g_w;
    d.value = value; d.v_b = a.v_b; d.v_h = a.v_h; d.v_w = a.v_w;
    d.weight = weight; d.bias = bias; d.probs = probs;
    d.dguide = dguide; d.dg_b = a.dg_b; d.dg_h = a.dg_h; d.dg_w = a.dg_w;
    d.dweight = dweight; d.dbias = dbias;
    d.B = B; d.Cg = Cg; d.C = C; d.H = H; d.W = W; d.I = I; d.K = K; d.dtype = dtype;
    d.conv_res = a.conv_res; d.hardmax = a.hardmax;
    for (int k = 0; k < K; ++k) { d.dy[k] = a.dy[k]; d.dx[k] = a.dx[k]; }
    plan.dl_tc = (dl_env && dl_tc_eligible(d, nullptr)) ? 1 : 0;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case UPLIFT_LA_F32: return bwd::launch_k<float>(a, plan, K, vec, gvec, s);
    case UPLIFT_LA_BF16: return bwd::launch_k<__nv_bfloat16>(a, plan, K, vec, gvec, s);
    default: return bwd::launch_k<__half>(a, plan, K, vec, gvec, s);
  }
}

// ---------------------------------------------------------------------------
// Allocation-free backward: the softmax-weight workspace lives in a fixed
// array of this library instead of caller memory, for callers that cannot
// allocate device memory (see include/uplift_la.h).  Host code reaches the
// array only through the device address that cudaGetSymbolAddress returns
// for the current device (the array's name on the host is a stand-in, not a
// device address); it is looked up once per device and cached.
namespace {

static __device__ __align__(256) float g_noalloc_probs[UPLIFT_LA_NOALLOC_MAX_PROBS];

constexpr int kNoallocDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoallocDevices] = {};

// Device address of g_noalloc_probs on the current device, or null (error set).
float* noalloc_workspace() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    ula::fail(UPLIFT_LA_ERR_CUDA, "uplift_la_backward_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (dev >= 0 && dev < kNoallocDevices && g_noalloc_ptr[dev] != nullptr) return g_noalloc_ptr[dev];
  float* ptr = nullptr;
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_probs);
  if (e != cudaSuccess || ptr == nullptr) {
    ula::fail(UPLIFT_LA_ERR_CUDA, "uplift_la_backward_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
              cudaGetErrorString(e));
    return nullptr;
  }
  if (dev >= 0 && dev < kNoallocDevices) g_noalloc_ptr[dev] = ptr;
  return ptr;
}

}  // namespace

extern "C" int uplift_la_backward_noalloc(const void* dout, const int64_t dout_strides[4],
                                          const void* guide, const int64_t guide_strides[4],
                                          const void* value, const int64_t value_strides[4],
                                          const float* weight, const float* bias,
                                          void* dguide, const int64_t dguide_strides[4],
                                          void* dvalue, const int64_t dvalue_strides[4],
                                          float* dweight, float* dbias,
                                          int B, int Cg, int C, int H, int W, int I, int K,
                                          const int8_t* offsets, int pn, int conv_res, int dtype, int hardmax,
                                          void* stream) {
  using namespace ula;
  // the arguments first, so that an invalid call names its bad argument
  const int rc = check_backward_args(dout, dout_strides, guide, guide_strides, value, value_strides, weight, dguide,
                                     dguide_strides, dvalue, dvalue_strides, B, Cg, C, H, W, I, K, offsets, pn, dtype);
  if (rc != UPLIFT_LA_OK) return rc;
  // B * (I*H) * (I*W) * K floats, checked factor by factor against the maximum
  const long long cap = UPLIFT_LA_NOALLOC_MAX_PROBS;
  long long need = 1;
  const long long f[6] = {B, I, H, I, W, K};
  for (int i = 0; i < 6 && need > 0; ++i) {
    need = f[i] == 0 ? 0 : (need > cap / f[i] ? cap + 1 : need * f[i]);
  }
  if (need > cap)
    return fail(UPLIFT_LA_ERR_SHAPE,
                "uplift_la_backward_noalloc: workspace B*(I*H)*(I*W)*K exceeds the fixed maximum of %lld floats "
                "(UPLIFT_LA_NOALLOC_MAX_PROBS); use uplift_la_backward with a caller workspace",
                cap);
  float* probs = noalloc_workspace();
  if (probs == nullptr) return UPLIFT_LA_ERR_CUDA;
  return uplift_la_backward(dout, dout_strides, guide, guide_strides, value, value_strides, weight, bias, probs,
                            dguide, dguide_strides, dvalue, dvalue_strides, dweight, dbias, B, Cg, C, H, W, I, K,
                            offsets, pn, conv_res, dtype, hardmax, stream);
}
