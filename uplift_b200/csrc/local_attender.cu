// C-ABI front end of the UPLiFT Local Attender for B200 (sm_100a):
// argument validation, kernel selection (tensor-core kernels in la_tc.cu /
// la_tcw.cu, CUDA-core kernels in la_simt.cuh) and launch.  Reference
// semantics: LocalAttender.forward, uplift/uplift.py:801-847.

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "uplift_la.h"
#include "la_internal.h"
#include "la_simt.cuh"

namespace ula {

// ---------------------------------------------------------------- host side
thread_local char g_err[512] = "";
thread_local int g_last_kernel = 0;
int g_policy = UPLIFT_LA_POLICY_AUTO;
// Host-visible status word registered by uplift_la_set_host_status_word
// (pinned host memory; null = none).
std::atomic<unsigned int*> g_host_status{nullptr};

unsigned int* host_status_word() { return g_host_status.load(std::memory_order_acquire); }

// CTA limit of the persistent tensor-core kernels (uplift_la_set_max_ctas; 0 = none).
std::atomic<int> g_max_ctas{0};

int cta_budget(int sms) {
  const int l = g_max_ctas.load(std::memory_order_relaxed);
  return std::max(1, (l > 0 && l < sms) ? l : sms);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

// Guides at least this wide take the staged projection (measured on B200:
// it wins once the projection is a large share of the work).
#ifndef ULA_STAGED_MIN_CG
#define ULA_STAGED_MIN_CG 128
#endif
constexpr int kStagedMinCg = ULA_STAGED_MIN_CG;
// fp32 guides at least this wide take the tensor-core projection under AUTO.
constexpr int kWideMinCg = 128;

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
  static std::mutex mu;  // launches may come from any host thread
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev].sms > 0) { *info = cache[dev]; return UPLIFT_LA_OK; }
  }
  int sms = 0, major = 0, optin = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return fail(UPLIFT_LA_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
  if (major != 10) return fail(UPLIFT_LA_ERR_NO_DEVICE, "device %d has compute capability %d.x; this build targets sm_100a", dev, major);
  info->sms = sms;
  info->max_smem_optin = (size_t)optin;
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(mu);
    cache[dev] = *info;
  }
  return UPLIFT_LA_OK;
}

int launch(const Params& p0, int dtype, int K, int cpt, bool vec, bool staged, size_t smem, cudaStream_t stream) {
  Params p = p0;
  if (p.num_units == 0) return UPLIFT_LA_OK;  // empty input: nothing to do
  KernelFn fn = nullptr;
  switch (dtype) {
    case UPLIFT_LA_F32: fn = simt_kernel_f32(K, cpt, vec, staged); break;
    case UPLIFT_LA_BF16: fn = simt_kernel_bf16(K, cpt, vec, staged); break;
    case UPLIFT_LA_F16: fn = simt_kernel_f16(K, cpt, vec, staged); break;
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

int uplift_la_forward_resized(const void* guide, const int64_t guide_strides[4],
                              const void* value, const int64_t value_strides[4],
                              const float* weight, const float* bias,
                              void* out, const int64_t out_strides[4],
                              int B, int Cg, int C, int H, int W, int I, int K,
                              const int8_t* offsets, int pn, int conv_res,
                              int dtype, int hardmax, int Ho, int Wo, void* stream) {
  using namespace ula;
  if (dtype != UPLIFT_LA_F32 && dtype != UPLIFT_LA_BF16 && dtype != UPLIFT_LA_F16)
    return fail(UPLIFT_LA_ERR_ARG, "unknown dtype %d", dtype);
  if (guide_strides == nullptr || value_strides == nullptr || out_strides == nullptr || offsets == nullptr)
    return fail(UPLIFT_LA_ERR_ARG, "null stride or offset array");
  if (B < 0 || Cg < 1 || C < 1 || H < 0 || W < 0 || I < 1 || Ho < 1 || Wo < 1)
    return fail(UPLIFT_LA_ERR_SHAPE, "bad sizes B=%d Cg=%d C=%d H=%d W=%d I=%d Ho=%d Wo=%d", B, Cg, C, H, W, I, Ho,
                Wo);
  if (K < 1 || K > kMaxK) return fail(UPLIFT_LA_ERR_SHAPE, "K=%d out of range", K);
  if (pn < 0 || pn > UPLIFT_LA_MAX_PN) return fail(UPLIFT_LA_ERR_OFFSETS, "pn=%d out of range", pn);
  for (int k = 0; k < K; ++k) {
    const int dy = offsets[2 * k], dx = offsets[2 * k + 1];
    if (dy < -pn || dy > pn || dx < -pn || dx > pn)
      return fail(UPLIFT_LA_ERR_OFFSETS, "offset %d = (%d, %d) exceeds pn=%d", k, dy, dx, pn);
  }
  if (guide_strides[1] != 1 || value_strides[1] != 1 || out_strides[1] != 1)
    return fail(UPLIFT_LA_ERR_LAYOUT, "guide, value and out need channel stride 1 (channels_last)");
  if (B == 0) return UPLIFT_LA_OK;
  if (H == 0 || W == 0) return fail(UPLIFT_LA_ERR_SHAPE, "empty value map with a %dx%d output", Ho, Wo);
  if (guide == nullptr || value == nullptr || weight == nullptr || out == nullptr)
    return fail(UPLIFT_LA_ERR_ARG, "null tensor pointer");
  if (__atomic_load_n(&g_policy, __ATOMIC_RELAXED) == UPLIFT_LA_POLICY_SIMT)
    return fail(UPLIFT_LA_ERR_UNSUPPORTED, "fused resize needs the tensor-core kernel (policy SIMT)");
  if (I != 2) return fail(UPLIFT_LA_ERR_UNSUPPORTED, "fused resize: scale I=%d != 2", I);
  int64_t gs[4] = {guide_strides[0], guide_strides[1], guide_strides[2], guide_strides[3]};
  int64_t vs[4] = {value_strides[0], value_strides[1], value_strides[2], value_strides[3]};
  int64_t os[4] = {out_strides[0], out_strides[1], out_strides[2], out_strides[3]};
  canon_strides(gs, Cg, I * H, I * W, B);
  canon_strides(vs, C, H, W, B);
  canon_strides(os, C, Ho, Wo, B);
  TcArgs a;
  a.guide = guide; a.g_b = gs[0]; a.g_h = gs[2]; a.g_w = gs[3];
  a.value = value; a.v_b = vs[0]; a.v_h = vs[2]; a.v_w = vs[3];
  a.out = out; a.o_b = os[0]; a.o_h = os[2]; a.o_w = os[3];
  a.weight = weight; a.bias = bias;
  a.B = B; a.Cg = Cg; a.C = C; a.H = H; a.W = W; a.K = K; a.pn = pn;
  a.conv_res = conv_res ? 1 : 0; a.hardmax = hardmax ? 1 : 0; a.dtype = dtype; a.offsets = offsets;
  a.Ho = Ho; a.Wo = Wo;
  const char* why = nullptr;
  if (!tc_eligible(a, &why) || !tc_resize_eligible(a, &why))
    return fail(UPLIFT_LA_ERR_UNSUPPORTED, "fused resize not applicable: %s", why);
  const int rc = tc_launch(a, static_cast<cudaStream_t>(stream));
  if (rc == UPLIFT_LA_OK) g_last_kernel = UPLIFT_LA_KERNEL_TENSOR_CORE_RESIZE;
  return rc;
}

int uplift_la_forward_fused_guide(const void* act, const int64_t act_strides[4],
                                  const void* res, const int64_t res_strides[4],
                                  const float* w_guide, const float* b_guide,
                                  const void* value, const int64_t value_strides[4],
                                  const float* weight, const float* bias,
                                  void* out, const int64_t out_strides[4],
                                  int B, int Cg, int C, int H, int W, int I, int K,
                                  const int8_t* offsets, int pn, int conv_res,
                                  int dtype, int hardmax, int Ho, int Wo, void* stream) {
  using namespace ula;
  if (dtype != UPLIFT_LA_F32 && dtype != UPLIFT_LA_BF16 && dtype != UPLIFT_LA_F16)
    return fail(UPLIFT_LA_ERR_ARG, "unknown dtype %d", dtype);
  if (act_strides == nullptr || res_strides == nullptr || value_strides == nullptr || out_strides == nullptr ||
      offsets == nullptr)
    return fail(UPLIFT_LA_ERR_ARG, "null stride or offset array");
  const bool resize = Ho > 0 || Wo > 0;
  if (B < 0 || Cg < 1 || C < 1 || H < 0 || W < 0 || I < 1 || (resize && (Ho < 1 || Wo < 1)))
    return fail(UPLIFT_LA_ERR_SHAPE, "bad sizes B=%d Cg=%d C=%d H=%d W=%d I=%d Ho=%d Wo=%d", B, Cg, C, H, W, I, Ho,
                Wo);
  if (K < 1 || K > kMaxK) return fail(UPLIFT_LA_ERR_SHAPE, "K=%d out of range", K);
  if (pn < 0 || pn > UPLIFT_LA_MAX_PN) return fail(UPLIFT_LA_ERR_OFFSETS, "pn=%d out of range", pn);
  for (int k = 0; k < K; ++k) {
    const int dy = offsets[2 * k], dx = offsets[2 * k + 1];
    if (dy < -pn || dy > pn || dx < -pn || dx > pn)
      return fail(UPLIFT_LA_ERR_OFFSETS, "offset %d = (%d, %d) exceeds pn=%d", k, dy, dx, pn);
  }
  if (act_strides[1] != 1 || res_strides[1] != 1 || value_strides[1] != 1 || out_strides[1] != 1)
    return fail(UPLIFT_LA_ERR_LAYOUT, "all tensors need channel stride 1 (channels_last)");
  if (B == 0) return UPLIFT_LA_OK;
  if (H == 0 || W == 0) return fail(UPLIFT_LA_ERR_SHAPE, "empty value map");
  if (act == nullptr || res == nullptr || w_guide == nullptr || value == nullptr || weight == nullptr ||
      out == nullptr)
    return fail(UPLIFT_LA_ERR_ARG, "null tensor pointer");
  if (__atomic_load_n(&g_policy, __ATOMIC_RELAXED) == UPLIFT_LA_POLICY_SIMT)
    return fail(UPLIFT_LA_ERR_UNSUPPORTED, "fused guide needs the tensor-core kernel (policy SIMT)");
  if (I != 2) return fail(UPLIFT_LA_ERR_UNSUPPORTED, "fused guide: scale I=%d != 2", I);
  int64_t gs[4] = {act_strides[0], act_strides[1], act_strides[2], act_strides[3]};
  int64_t rs[4] = {res_strides[0], res_strides[1], res_strides[2], res_strides[3]};
  int64_t vs[4] = {value_strides[0], value_strides[1], value_strides[2], value_strides[3]};
  int64_t os[4] = {out_strides[0], out_strides[1], out_strides[2], out_strides[3]};
  canon_strides(gs, Cg, I * H, I * W, B);
  canon_strides(rs, Cg, I * H, I * W, B);
  canon_strides(vs, C, H, W, B);
  canon_strides(os, C, resize ? Ho : I * H, resize ? Wo : I * W, B);
  TcArgs a;
  a.guide = act; a.g_b = gs[0]; a.g_h = gs[2]; a.g_w = gs[3];
  a.guide2 = res; a.g2_b = rs[0]; a.g2_h = rs[2]; a.g2_w = rs[3];
  a.w_guide = w_guide; a.b_guide = b_guide;
  a.value = value; a.v_b = vs[0]; a.v_h = vs[2]; a.v_w = vs[3];
  a.out = out; a.o_b = os[0]; a.o_h = os[2]; a.o_w = os[3];
  a.weight = weight; a.bias = bias;
  a.B = B; a.Cg = Cg; a.C = C; a.H = H; a.W = W; a.K = K; a.pn = pn;
  a.conv_res = conv_res ? 1 : 0; a.hardmax = hardmax ? 1 : 0; a.dtype = dtype; a.offsets = offsets;
  if (resize) { a.Ho = Ho; a.Wo = Wo; }
  const char* why = nullptr;
  if (!tc_eligible(a, &why) || (resize && !tc_resize_eligible(a, &why)))
    return fail(UPLIFT_LA_ERR_UNSUPPORTED, "fused guide not applicable: %s", why);
  const int rc = tc_launch(a, static_cast<cudaStream_t>(stream));
  if (rc == UPLIFT_LA_OK)
    g_last_kernel = resize ? UPLIFT_LA_KERNEL_TENSOR_CORE_GUIDE_RESIZE : UPLIFT_LA_KERNEL_TENSOR_CORE_GUIDE;
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
  const int c = ula::dv_device_status(clear != 0);
  const int d = ula::dl_device_status(clear != 0);
  if (a < 0 || b < 0 || c < 0 || d < 0) return -1;
  return a != 0 ? a : (b != 0 ? b : (c != 0 ? c : d));
}

int uplift_la_set_host_status_word(unsigned int* word) {
  ula::g_host_status.store(word, std::memory_order_release);
  return UPLIFT_LA_OK;
}

int uplift_la_set_max_ctas(int n) {
  if (n < 0) return ula::fail(UPLIFT_LA_ERR_ARG, "uplift_la_set_max_ctas: n < 0");
  ula::g_max_ctas.store(n, std::memory_order_relaxed);
  return UPLIFT_LA_OK;
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
    case UPLIFT_LA_ERR_UNSUPPORTED: return "no fused kernel for this problem";
    default: return "unknown status";
  }
}

int uplift_la_abi_version(void) { return (1 << 16) | 3; }

}  // extern "C"
