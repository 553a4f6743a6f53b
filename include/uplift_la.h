/*
 * uplift_la.h -- C ABI of the B200 (sm_100a) UPLiFT Local Attender.
 *
 * The Local Attender upsamples a coarse "value" map [B, C, H, W] to
 * [B, C, I*H, I*W] under the guidance of a fine "guide" map
 * [B, Cg, I*H, I*W].  For every output pixel (y, x) with parent coarse cell
 * (h, w) = (y / I, x / I) it computes
 *
 *     logit[k] = bias[k] + sum_c weight[k][c] * guide[c, y, x]
 *                (+ guide[k, y, x] for k < min(K, Cg) when conv_res)
 *     p        = softmax_k(logit)          (one-hot of the first argmax when hardmax)
 *     out[c, y, x] = sum_k p[k] * value[c, clamp(h + dy[k]), clamp(w + dx[k])]
 *
 * where clamp() to [0, H-1] / [0, W-1] is the replicate padding of the
 * reference.  All arithmetic is fp32; tensors are stored as fp32, bf16 or
 * fp16 (all three of guide / value / out in the same type).
 *
 * Tensors are described by a base pointer and four element strides in the
 * logical order [B, channel, row, col].  The channel stride must be 1
 * (channels_last / NHWC storage, which is what the fast path of the
 * reference uses); other strides are free (sliced or padded tensors work).
 * All pointers are device pointers of the current CUDA device unless noted.
 *
 * No entry point allocates device memory, synchronises the stream or aborts
 * the process: each returns UPLIFT_LA_OK or an error code, and
 * uplift_la_last_error() gives a message for the calling thread.
 */
#ifndef UPLIFT_LA_H_
#define UPLIFT_LA_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* storage types (guide, value, logits and out share one) */
#define UPLIFT_LA_F32  0
#define UPLIFT_LA_BF16 1
#define UPLIFT_LA_F16  2

/* status codes */
#define UPLIFT_LA_OK             0
#define UPLIFT_LA_ERR_ARG        1  /* null pointer, bad enum value         */
#define UPLIFT_LA_ERR_SHAPE      2  /* sizes inconsistent or unsupported    */
#define UPLIFT_LA_ERR_LAYOUT     3  /* channel stride != 1, misalignment    */
#define UPLIFT_LA_ERR_OFFSETS    4  /* |offset| > pn, or pn out of range    */
#define UPLIFT_LA_ERR_CUDA       5  /* a CUDA runtime call or launch failed */
#define UPLIFT_LA_ERR_NO_DEVICE  6  /* no usable sm_100 device              */
#define UPLIFT_LA_ERR_UNSUPPORTED 7 /* no fused kernel applies; nothing was
                                       launched (the caller runs the steps
                                       separately)                          */

/* largest neighbourhood and padding the kernels accept */
#define UPLIFT_LA_MAX_K  25
#define UPLIFT_LA_MAX_PN 4

/*
 * Fused Local Attender forward: 1x1 logit projection (+ residual), softmax
 * over the K neighbour offsets and softmax-weighted gather-sum of the value
 * vectors, in one kernel launch on `stream` (a cudaStream_t; NULL = legacy
 * default stream).
 *
 * Replaces LocalAttender.forward (uplift/uplift.py:801-847) and the fast-path
 * pair _TritonAttenderWrapper.forward (uplift/fast.py:60-64) +
 * TritonLocalAttender.forward (uplift/kernels/triton_attender.py:335-392).
 *
 *   guide   [B, Cg, I*H, I*W]  strides guide_strides (elements)
 *   value   [B, C,  H,   W  ]  strides value_strides
 *   weight  [K, Cg] fp32, row-major (conv1.weight[:, :, 0, 0])
 *   bias    [K] fp32, or NULL for no bias (conv1.bias)
 *   out     [B, C,  I*H, I*W]  strides out_strides, must not alias inputs
 *   offsets host array [K][2] of (dy, dx), |dy|,|dx| <= pn
 *           (LocalAttender.offsets, uplift/uplift.py:746-760)
 *   K       1..UPLIFT_LA_MAX_K; the reference uses 5, 9, 13, 17, 25
 *   I       integer scale factor >= 1
 */
int uplift_la_forward(const void* guide, const int64_t guide_strides[4],
                      const void* value, const int64_t value_strides[4],
                      const float* weight, const float* bias,
                      void* out, const int64_t out_strides[4],
                      int B, int Cg, int C, int H, int W, int I, int K,
                      const int8_t* offsets, int pn, int conv_res,
                      int dtype, int hardmax, void* stream);

/*
 * uplift_la_forward followed by the fast path's final resize, in one launch:
 * out [B, C, Ho, Wo] = F.interpolate(attender output, size=(Ho, Wo),
 * mode="bilinear", align_corners=False), the resize of _OptimizedUPLiFT's
 * last step (uplift/fast.py:218-220).  The attender output itself is never
 * stored: each output tile is resampled in shared memory from the attender
 * values of its tile rounded to the storage type, as the stored tensor would
 * hold them, then interpolated in fp32 with PyTorch's source-index formula
 * (results equal the two separate steps up to the fp32 contraction order,
 * <= 1 storage ulp).  Applies to the tensor-core kernel's problems (bf16 /
 * fp16, I = 2, Cg = 64, C a multiple of 64 up to 384) whose output is 7/8 of
 * the attender output in both dimensions -- 1168 -> 1022 and 512 -> 448 in
 * the DINOv2 upsampler -- with the attender output a whole number of 8 x 16
 * tiles; then every 8 x 16 attender tile maps onto exactly 7 x 14 output
 * pixels and no tile needs another's values.  Otherwise returns
 * UPLIFT_LA_ERR_UNSUPPORTED and launches nothing.  Other arguments as for
 * uplift_la_forward.  No single reference counterpart (it fuses two).
 */
int uplift_la_forward_resized(const void* guide, const int64_t guide_strides[4],
                              const void* value, const int64_t value_strides[4],
                              const float* weight, const float* bias,
                              void* out, const int64_t out_strides[4],
                              int B, int Cg, int C, int H, int W, int I, int K,
                              const int8_t* offsets, int pn, int conv_res,
                              int dtype, int hardmax, int Ho, int Wo, void* stream);

/*
 * The guide produced inside the attender launch.  In the DINOv2 / DINOv3
 * decoders the guide is the output of the last block, a residual DoubleConv
 * whose final layer is a 1x1 convolution with bias
 * (uplift/uplift.py:152-217): guide = w_guide . act + b_guide + res, where
 * `act` is that block's activation before the 1x1 convolution and `res` the
 * first Cg channels of the block's input (residual_auto's truncation,
 * uplift/uplift.py:26-39).  This entry point computes
 * uplift_la_forward(guide, ...) from act and res directly -- the guide is
 * never stored -- by folding the 1x1 convolution and both residuals into
 * the projection: logits = (A . w_guide) act + A res + bias + A b_guide, A =
 * weight plus the identity on the first K channels when conv_res.  The
 * folded [K, 2 Cg] projection is computed in fp32 in the kernel prologue and
 * rounded once to the storage type (the unfused path rounds the guide
 * instead; both are within the storage type's precision).
 *
 *   act, res   [B, Cg, I*H, I*W] (strides; res may be a channel slice)
 *   w_guide    [Cg, Cg] fp32 (out, in): the block's 1x1 conv weight
 *   b_guide    [Cg] fp32 or NULL: its bias
 *   Ho, Wo     0, 0: out is [B, C, I*H, I*W]; else the output also gets the
 *              final resize of uplift_la_forward_resized and is [B, C, Ho, Wo]
 *
 * Applies to the tensor-core kernel's problems (bf16 / fp16, I = 2, Cg = 64,
 * C a multiple of 64 up to 384; with a resize, its conditions too);
 * otherwise returns UPLIFT_LA_ERR_UNSUPPORTED and launches nothing.  No
 * single reference counterpart (it fuses the decoder's last 1x1 conv and
 * residual, uplift/uplift.py:172 and :208-215, into the attender).
 */
int uplift_la_forward_fused_guide(const void* act, const int64_t act_strides[4],
                                  const void* res, const int64_t res_strides[4],
                                  const float* w_guide, const float* b_guide,
                                  const void* value, const int64_t value_strides[4],
                                  const float* weight, const float* bias,
                                  void* out, const int64_t out_strides[4],
                                  int B, int Cg, int C, int H, int W, int I, int K,
                                  const int8_t* offsets, int pn, int conv_res,
                                  int dtype, int hardmax, int Ho, int Wo, void* stream);

/*
 * Softmax-pool from pre-projected logits: the same kernel with the
 * projection replaced by a read of `logits` [B, K, I*H, I*W] (any strides,
 * same storage type as value).  Replaces the Triton fused kernels'
 * interface TritonLocalAttender.forward(att, x, hardmax)
 * (uplift/kernels/triton_attender.py:336) and its PyTorch fallback
 * (uplift/kernels/triton_attender.py:402-431), for every K and I instead of
 * K=17, I in {2,4} only.
 */
int uplift_la_pool(const void* logits, const int64_t logits_strides[4],
                   const void* value, const int64_t value_strides[4],
                   void* out, const int64_t out_strides[4],
                   int B, int C, int H, int W, int I, int K,
                   const int8_t* offsets, int pn,
                   int dtype, int hardmax, void* stream);

/*
 * Backward of uplift_la_forward (training; replaces autograd through the
 * reference's LocalAttender.forward, uplift/uplift.py:801-847, as used by
 * uplift/train_uplift.py).  Given dout [B, C, I*H, I*W] (strides ds), writes
 * dguide [B, Cg, I*H, I*W] and dvalue [B, C, H, W] (storage type; either may
 * be NULL) and ADDS the projection gradients into dweight [K, Cg] and dbias
 * [K] (fp32, caller-zeroed; either may be NULL).  `probs` is a caller-
 * provided fp32 workspace of B*(I*H)*(I*W)*K floats that receives the
 * softmax weights (recomputed from the guide).  Other arguments as for
 * uplift_la_forward; all tensors channel stride 1.  fp32 arithmetic; three
 * kernel launches on `stream`; dweight / dbias accumulate with atomic adds,
 * so their last bits depend on the launch schedule.
 */
int uplift_la_backward(const void* dout, const int64_t dout_strides[4],
                       const void* guide, const int64_t guide_strides[4],
                       const void* value, const int64_t value_strides[4],
                       const float* weight, const float* bias,
                       float* probs,
                       void* dguide, const int64_t dguide_strides[4],
                       void* dvalue, const int64_t dvalue_strides[4],
                       float* dweight, float* dbias,
                       int B, int Cg, int C, int H, int W, int I, int K,
                       const int8_t* offsets, int pn, int conv_res, int dtype, int hardmax,
                       void* stream);

/*
 * uplift_la_backward for callers that cannot allocate device memory: the
 * same arguments and results, minus the `probs` workspace.  It suits a
 * host whose memory pool owns all device memory, a caller that must not let
 * cudaMalloc / cudaFree synchronise the device in the middle of its work,
 * and an FFI binding that has no device allocator.  No counterpart in the
 * reference (its backward is PyTorch autograd, which allocates freely).
 *
 * The workspace is a fixed array of UPLIFT_LA_NOALLOC_MAX_PROBS floats
 * (32 MiB) inside the library, which every GPU that loads the library
 * holds until the process exits.  Calls with B*(I*H)*(I*W)*K above that
 * maximum fail with UPLIFT_LA_ERR_SHAPE and launch nothing (other invalid
 * arguments are reported first, as by uplift_la_backward).  The first call
 * on a device looks the array's device address up (cudaGetSymbolAddress)
 * and keeps it for later calls: make that first call before any stream
 * capture.  The kept address belongs to the device's primary context (the
 * runtime's default); after cudaDeviceReset it is stale, so do not use this
 * entry point again in that process.  All calls share the one
 * array: calls whose kernels overlap on the GPU (other streams, other host
 * threads) race on it, so serialise them.  Every call rewrites the part it
 * reads; dweight / dbias still accumulate into the caller's zeroed outputs.
 * Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
 */
#define UPLIFT_LA_NOALLOC_MAX_PROBS (8 * 1024 * 1024)
int uplift_la_backward_noalloc(const void* dout, const int64_t dout_strides[4],
                               const void* guide, const int64_t guide_strides[4],
                               const void* value, const int64_t value_strides[4],
                               const float* weight, const float* bias,
                               void* dguide, const int64_t dguide_strides[4],
                               void* dvalue, const int64_t dvalue_strides[4],
                               float* dweight, float* dbias,
                               int B, int Cg, int C, int H, int W, int I, int K,
                               const int8_t* offsets, int pn, int conv_res, int dtype, int hardmax,
                               void* stream);

/* Kernel selection for uplift_la_forward (process-wide; default AUTO).
 * AUTO picks a tensor-core kernel (tcgen05 MMA, TMEM accumulators, TMA)
 * when one applies -- bf16/fp16 storage, I = 2, Cg = 64, C a multiple of 64
 * up to 384; or fp32 storage, I = 2, Cg a multiple of 32 in 64..512, C a
 * multiple of 4 up to 32 (the wide-guide split-bf16 projection); 16-byte
 * aligned tensors -- and the CUDA-core kernel otherwise; SIMT always uses
 * the CUDA-core kernel; TENSOR_CORE makes ineligible problems fail with
 * UPLIFT_LA_ERR_SHAPE instead of falling back.  No reference counterpart
 * (the reference has a single Triton kernel family). */
#define UPLIFT_LA_POLICY_AUTO        0
#define UPLIFT_LA_POLICY_SIMT        1
#define UPLIFT_LA_POLICY_TENSOR_CORE 2
int uplift_la_set_kernel_policy(int policy);

/* Kernel launched by the last successful call on the calling thread. */
#define UPLIFT_LA_KERNEL_SIMT        1
#define UPLIFT_LA_KERNEL_TENSOR_CORE 2
#define UPLIFT_LA_KERNEL_SIMT_STAGED 3  /* CUDA-core kernel, guide staged in shared memory */
#define UPLIFT_LA_KERNEL_TENSOR_CORE_WIDE 4  /* fp32, wide guide: split-bf16 tensor-core projection */
#define UPLIFT_LA_KERNEL_TENSOR_CORE_RESIZE 5  /* tensor-core kernel with the fused final resize */
#define UPLIFT_LA_KERNEL_TENSOR_CORE_GUIDE 6   /* tensor-core kernel, guide produced inside */
#define UPLIFT_LA_KERNEL_TENSOR_CORE_GUIDE_RESIZE 7  /* both fusions */
int uplift_la_last_kernel(void);

/* Device status word of the tensor-core kernels: 0 when every launch so far
 * completed its pipeline, else the role (1 producer, 2 MMA, 3 softmax or
 * split, 4 epilogue) whose bounded wait expired first.  Synchronises with
 * the device; `clear` resets the word.  Returns -1 if the read failed. */
int uplift_la_device_status(int clear);

/* Registers a host-visible copy of the device status word: `word` points to
 * 4 bytes of pinned host memory that the device can address (cudaHostAlloc
 * memory under unified addressing; NULL unregisters).  Every later
 * tensor-core launch also writes the failing role's code there when a
 * bounded wait expires, so the host can poll a plain memory read -- no
 * synchronisation, no device call -- and learn that a finished launch left
 * its output incomplete.  The library never clears the word; the caller does.
 * The word must stay allocated while launches that received it can run.
 * Process-wide, all devices.  No reference counterpart (the reference's
 * Triton kernels have no waits that can expire). */
int uplift_la_set_host_status_word(unsigned int* word);

/* Testing only: fault = 1 makes the tensor-core kernels' guide producers issue
 * no loads, so the consumers' bounded waits run out; wait_limit_ns (0 =
 * default 2 s) caps every mbarrier wait.  fault = 0 restores normal
 * operation.  Used to check that an expired wait is reported through
 * uplift_la_device_status() and leaves the context usable.  No reference
 * counterpart. */
int uplift_la_test_hook(int fault, unsigned long long wait_limit_ns);

/* At most n CTAs (0: one per SM, the default) for the persistent
 * tensor-core kernels (forward and backward; each holds a whole SM).  For a
 * caller that runs communication kernels beside them -- an NCCL gather of
 * the previous batch's output, say -- so that those get SMs without
 * delaying the attender's CTAs.  Process-wide, takes effect at the next
 * launch; n < 0 is UPLIFT_LA_ERR_ARG.  No reference counterpart. */
int uplift_la_set_max_ctas(int n);

/* Message for the last non-OK status returned on the calling thread. */
const char* uplift_la_last_error(void);

/* Name of a status code. */
const char* uplift_la_status_string(int status);

/* ABI version: (major << 16) | minor. */
int uplift_la_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* UPLIFT_LA_H_ */
