// Internal interface between the C-ABI front end (local_attender.cu) and
// the tensor-core kernels (la_tc.cu, la_tcw.cu).  Not part of the public ABI.
#pragma once

#include <stdint.h>
#include <cuda.h>
#include <cuda_runtime.h>

namespace ula {

// Everything the tensor-core path needs; strides in elements, channel
// stride 1 (NHWC).
struct TcArgs {
  const void* guide; int64_t g_b, g_h, g_w;
  const void* value; int64_t v_b, v_h, v_w;
  void* out;         int64_t o_b, o_h, o_w;
  const float* weight;  // [K, Cg] fp32, device
  const float* bias;    // [K] fp32 or null
  int B, Cg, C, H, W, K, pn;
  int conv_res, hardmax, dtype;
  const int8_t* offsets;  // host [K][2]
  // fused final resize: out is [B, Ho, Wo, C], the bilinear
  // (align_corners=False) resize of the attender output; 0 = no resize
  int Ho = 0, Wo = 0;
  // fused guide: `guide` is the guide block's activation h and guide2 its
  // residual input u (same sizes, Cg channels each); guide = w_guide . h +
  // b_guide + u is folded into the projection.  guide2 = null: plain guide.
  const void* guide2 = nullptr; int64_t g2_b = 0, g2_h = 0, g2_w = 0;
  const float* w_guide = nullptr;  // [Cg][Cg] fp32 (out, in)
  const float* b_guide = nullptr;  // [Cg] fp32 or null
};

// True when the tensor-core kernel supports the problem (sizes, alignment).
bool tc_eligible(const TcArgs& a, const char** why);

// True when the tensor-core kernel can also apply the final bilinear resize
// to a.Ho x a.Wo (see la_tc.cu); checked on top of tc_eligible.
bool tc_resize_eligible(const TcArgs& a, const char** why);

// Launch the tensor-core kernel; returns a UPLIFT_LA_* status.
int tc_launch(const TcArgs& a, cudaStream_t stream);

// Read (and optionally clear) the tensor-core kernel's device status word;
// -1 if the read failed.
int tc_device_status(bool clear);

// Test hook of the tensor-core kernels (see uplift_la_test_hook) and its
// current settings.
int tc_set_test_hook(int fault, unsigned long long timeout_ns);
int tc_test_fault();
unsigned long long tc_test_timeout_ns();

// Tensor-core projection for wide fp32 guides (la_tcw.cu): eligibility,
// launch and status word, as above.
bool tcw_eligible(const TcArgs& a, const char** why);
int tcw_launch(const TcArgs& a, cudaStream_t stream);
int tcw_device_status(bool clear);

// Host-visible status word registered by the caller
// (uplift_la_set_host_status_word), or null; passed to every tensor-core
// launch so that an expired wait is also written there.
unsigned int* host_status_word();
// CTAs for a persistent kernel: min(sms, the uplift_la_set_max_ctas limit), at least 1.
int cta_budget(int sms);

// Tensor-core dV of the backward (la_bwd_dv.cu): dvalue from dout and the
// fp32 softmax workspace; strides in elements, channel stride 1 (NHWC).
struct DvArgs {
  const void* dout;   int64_t d_b, d_h, d_w;
  const float* probs;  // [B][I*H][I*W][K]
  void* dvalue;       int64_t dv_b, dv_h, dv_w;
  int B, C, H, W, I, K, dtype;
  int8_t dy[25], dx[25];
};
bool dv_tc_eligible(const DvArgs& a, const char** why);
int dv_tc_launch(const DvArgs& a, cudaStream_t stream);
int dv_device_status(bool clear);

// Tensor-core dlogit of the backward (la_bwd_dl.cu): softmax weights (into
// the workspace), dguide and dW / db (accumulated) for 16-bit storage.
struct DlArgs {
  const void* dout;   int64_t d_b, d_h, d_w;
  const void* guide;  int64_t g_b, g_h, g_w;
  const void* value;  int64_t v_b, v_h, v_w;
  const float* weight; const float* bias;
  float* probs;        // [B][I*H][I*W][K] or null
  void* dguide;       int64_t dg_b, dg_h, dg_w;  // or null
  float* dweight; float* dbias;                   // or null
  int B, Cg, C, H, W, I, K, dtype, conv_res, hardmax;
  int8_t dy[25], dx[25];
};
bool dl_tc_eligible(const DlArgs& a, const char** why);
int dl_tc_launch(const DlArgs& a, cudaStream_t stream);
int dl_device_status(bool clear);

// Record an error message for uplift_la_last_error().
int fail(int code, const char* fmt, ...);

// NHWC 4-D TMA map (dims {C, W, H, B}, strides in elements of `es` bytes),
// with the 128-byte swizzle unless another is asked for.
int tc_make_map(CUtensorMap* map, CUtensorMapDataType dt, int es, const void* base, int C, int W, int H, int B,
                int64_t s_w, int64_t s_h, int64_t s_b, int box_c, int box_w, int box_h,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

}  // namespace ula
