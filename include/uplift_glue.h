/*
 * uplift_glue.h -- C ABI of the B200 (sm_100a) resampling / residual kernels
 * around the Local Attender in the UPLiFT upsampler's fast mode.
 *
 * These replace the elementwise "glue" between the cuDNN convolutions of the
 * decoder, which in eager PyTorch runs at a small fraction of HBM bandwidth
 * (strided adds, float round trips, separate resize + concatenate passes):
 *
 *   uplift_resize_bilinear  F.interpolate(mode="bilinear", antialias=False)
 *                           as in the fast path's final resize
 *                           (uplift/fast.py:219) and
 *                           UpsamplingBilinear2d (align_corners=True) of the
 *                           up-block residual (uplift/uplift.py:228, :335);
 *                           with `accumulate`, dst += resize(src), the
 *                           residual_auto add of that block fused in
 *   uplift_resize_nearest   F.interpolate(mode="nearest") / TVF.resize
 *                           NEAREST of the skip features in
 *                           noise_and_combine (uplift/uplift.py:354-367,
 *                           uplift/fast.py:229), written straight into a
 *                           channel slice of the concatenation buffer
 *   uplift_add_channels     residual_auto (uplift/uplift.py:26-39): the
 *                           first C channels of dst += those of src, in place
 *   uplift_bias_act         the epilogue of a decoder / encoder convolution
 *                           run without its bias: + bias, ReLU, + residual
 *                           (the folded Conv -> BatchNorm -> ReLU and the
 *                           1x1 conv + residual_auto of _ConvBlock,
 *                           uplift/uplift.py:96-217), in place, in one pass
 *   uplift_layernorm_act    Conv (bias) -> LayerNorm over channels
 *                           ("channels_first", uplift/uplift.py:50-92) ->
 *                           ReLU of the SD1.5-VAE variant's blocks, in place,
 *                           one pass (per-pixel mean and variance over C)
 *
 * Tensors: base pointer + element strides in the order [B, channel, row,
 * col]; the channel stride must be 1 (channels_last / NHWC), other strides
 * are free (channel slices of a wider tensor work).  Arithmetic is fp32
 * ("opmath") with one rounding to the storage type per result, as PyTorch
 * does; source indices follow PyTorch's formulas, so results match
 * F.interpolate / torch.add.  dtype: UPLIFT_LA_F32 / BF16 / F16 from
 * uplift_la.h.  Each call launches one kernel on `stream`, allocates
 * nothing, never synchronises, and returns UPLIFT_LA_OK or an error code
 * (message in uplift_la_last_error()).
 */
#ifndef UPLIFT_GLUE_H_
#define UPLIFT_GLUE_H_

#include <stdint.h>

#include "uplift_la.h"

#ifdef __cplusplus
extern "C" {
#endif

/* dst[B, C, Ho, Wo] (= or +=) bilinear resize of src[B, C, Hi, Wi].
 * align_corners = 0: source = (dst + 0.5) * Hi / Ho - 0.5, clamped at 0;
 * align_corners = 1: source = dst * (Hi - 1) / (Ho - 1).
 * accumulate = 1: dst = dst + round(resize) (residual add of an up-block). */
int uplift_resize_bilinear(const void* src, const int64_t src_strides[4],
                           void* dst, const int64_t dst_strides[4],
                           int B, int C, int Hi, int Wi, int Ho, int Wo,
                           int align_corners, int accumulate, int dtype, void* stream);

/* dst[B, C, Ho, Wo] = nearest resample of src[B, C, Hi, Wi]
 * (source index floor(dst * Hi / Ho) in fp32, PyTorch's "nearest");
 * Ho == Hi, Wo == Wi is a plain (strided) copy. */
int uplift_resize_nearest(const void* src, const int64_t src_strides[4],
                          void* dst, const int64_t dst_strides[4],
                          int B, int C, int Hi, int Wi, int Ho, int Wo,
                          int dtype, void* stream);

/* dst[:, :C] += src[:, :C] over [B, C, H, W], in place. */
int uplift_add_channels(void* dst, const int64_t dst_strides[4],
                        const void* src, const int64_t src_strides[4],
                        int B, int C, int H, int W, int dtype, void* stream);

/* In place over dst[B, C, H, W]: t = dst + bias[c] (rounded), t = max(t, 0)
 * when relu, then t + res[c] (rounded) for c < res_channels; bias (storage
 * type, [C]) and res (strides res_strides) may be NULL.  The roundings are
 * those of the separate eager ops (conv output, + bias, ReLU, + residual). */
int uplift_bias_act(void* dst, const int64_t dst_strides[4], const void* bias,
                    const void* res, const int64_t res_strides[4], int res_channels,
                    int relu, int B, int C, int H, int W, int dtype, void* stream);

/* In place over dst[B, C, H, W], per pixel: t = dst + pre_bias[c] (when
 * given), mu = mean_c t, var = mean_c (t - mu)^2,
 * out = weight[c] * (t - mu) / sqrt(var + eps) + bias[c], max(out, 0) when
 * relu.  pre_bias, weight, bias: [C] in the storage type (weight and bias
 * required).  fp32 arithmetic, one rounding of the result. */
int uplift_layernorm_act(void* dst, const int64_t dst_strides[4], const void* pre_bias,
                         const void* weight, const void* bias, float eps, int relu,
                         int B, int C, int H, int W, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* UPLIFT_GLUE_H_ */
