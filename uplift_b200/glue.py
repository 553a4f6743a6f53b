"""Resampling and residual ops of the upsampler's fast mode, over the C ABI
of include/uplift_glue.h (sm_100a kernels in uplift_b200/csrc/glue.cu).

They replace the eager elementwise glue between the cuDNN convolutions of
the decoder -- the final bilinear resize (uplift/fast.py:219), the up-block
residual UpsamplingBilinear2d + residual_auto (uplift/uplift.py:228, :26-39),
the nearest resample of the skip features and the concatenation of
noise_and_combine (uplift/uplift.py:354-367) -- with single HBM-bound passes
that give the same values (PyTorch's index formulas, fp32 arithmetic, one
rounding per result).  Tensors must be CUDA tensors with channel stride 1
(channels_last); channel slices of wider tensors are fine.  Each op is a
registered torch custom op, so torch.compile traces through it.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _native

_DTYPES = {torch.float32: _native.F32, torch.bfloat16: _native.BF16, torch.float16: _native.F16}


def _check(*ts: torch.Tensor):
    dev = ts[0].device
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("uplift_b200 glue ops run on CUDA (sm_100) tensors only "
                               f"(got a {t.device} tensor; there is no CPU fallback)")
        if t.device != dev or t.dtype != ts[0].dtype:
            raise ValueError("tensors must share device and dtype")
        if t.dim() != 4:
            raise ValueError("expected 4-D [B, C, H, W] tensors")
    if ts[0].dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {ts[0].dtype}")
    return dev


def _cl(t: torch.Tensor) -> torch.Tensor:
    return t if (t.stride(1) == 1 or t.shape[1] == 1) else t.contiguous(memory_format=torch.channels_last)


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def resize_bilinear_raw(x: torch.Tensor, size: Sequence[int], align_corners: bool = False,
                        out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """F.interpolate(x, size, mode="bilinear", align_corners=...) into a new
    channels_last tensor, or added into `out` when accumulate=True."""
    dev = _check(x) if out is None else _check(x, out)
    x = _cl(x)
    B, C, Hi, Wi = x.shape
    Ho, Wo = int(size[0]), int(size[1])
    if out is None:
        out = torch.empty((B, C, Ho, Wo), dtype=x.dtype, device=dev, memory_format=torch.channels_last)
    elif tuple(out.shape) != (B, C, Ho, Wo):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(B, C, Ho, Wo)}")
    with torch.cuda.device(dev):
        rc = _native.load().uplift_resize_bilinear(
            x.data_ptr(), _native.strides(x), out.data_ptr(), _native.strides(out),
            B, C, Hi, Wi, Ho, Wo, int(bool(align_corners)), int(bool(accumulate)), _DTYPES[x.dtype], _stream(dev))
    _native.check(rc, "uplift_resize_bilinear")
    return out


def resize_nearest_into_(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """dst[...] = F.interpolate(src, dst.shape[2:], mode="nearest"); dst may
    be a channel slice of a wider tensor (e.g. a concatenation buffer)."""
    dev = _check(dst, src)
    src = _cl(src)
    B, C, Hi, Wi = src.shape
    if dst.shape[0] != B or dst.shape[1] != C:
        raise ValueError(f"dst {tuple(dst.shape)} does not match src {tuple(src.shape)}")
    with torch.cuda.device(dev):
        rc = _native.load().uplift_resize_nearest(
            src.data_ptr(), _native.strides(src), dst.data_ptr(), _native.strides(dst),
            B, C, Hi, Wi, dst.shape[2], dst.shape[3], _DTYPES[src.dtype], _stream(dev))
    _native.check(rc, "uplift_resize_nearest")
    return dst


def add_channels_raw_(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """dst[:, :c] += src[:, :c] in place, c = min of the channel counts
    (residual_auto of uplift/uplift.py:26-39 with the sum written into dst)."""
    dev = _check(dst, src)
    if dst.shape[0] != src.shape[0] or dst.shape[2:] != src.shape[2:]:
        raise ValueError(f"shape mismatch {tuple(dst.shape)} vs {tuple(src.shape)}")
    src = _cl(src)
    B, _, H, W = dst.shape
    C = min(dst.shape[1], src.shape[1])
    with torch.cuda.device(dev):
        rc = _native.load().uplift_add_channels(
            dst.data_ptr(), _native.strides(dst), src.data_ptr(), _native.strides(src),
            B, C, H, W, _DTYPES[dst.dtype], _stream(dev))
    _native.check(rc, "uplift_add_channels")
    return dst


def bias_act_raw_(y: torch.Tensor, bias: torch.Tensor | None, relu: bool,
                  res: torch.Tensor | None = None) -> torch.Tensor:
    """In place: y = relu?(y + bias[c]) (+ res[:, :c] for the channels both
    have): the epilogue of a convolution run without its bias, with the
    ReLU that follows it and the residual_auto add of its block."""
    dev = _check(y) if res is None else _check(y, res)
    B, C, H, W = y.shape
    b = None
    if bias is not None:
        b = bias.detach()
        if b.dtype != y.dtype or not b.is_contiguous() or b.device != y.device:
            b = b.to(device=y.device, dtype=y.dtype).contiguous()
        if b.numel() != C:
            raise ValueError(f"bias has {b.numel()} entries for {C} channels")
    rc_ch = 0
    if res is not None:
        if res.shape[0] != B or res.shape[2:] != y.shape[2:]:
            raise ValueError(f"residual {tuple(res.shape)} does not match {tuple(y.shape)}")
        res = _cl(res)
        rc_ch = min(C, res.shape[1])
    with torch.cuda.device(dev):
        rc = _native.load().uplift_bias_act(
            y.data_ptr(), _native.strides(y), None if b is None else b.data_ptr(),
            None if res is None else res.data_ptr(), _native.strides(res if res is not None else y),
            rc_ch, int(bool(relu)), B, C, H, W, _DTYPES[y.dtype], _stream(dev))
    _native.check(rc, "uplift_bias_act")
    return y


def _param(t: torch.Tensor | None, like: torch.Tensor, C: int, what: str):
    if t is None:
        return None
    t = t.detach()
    if t.dtype != like.dtype or not t.is_contiguous() or t.device != like.device:
        t = t.to(device=like.device, dtype=like.dtype).contiguous()
    if t.numel() != C:
        raise ValueError(f"{what} has {t.numel()} entries for {C} channels")
    return t


def layernorm_act_raw_(y: torch.Tensor, pre_bias: torch.Tensor | None, weight: torch.Tensor,
                       bias: torch.Tensor, eps: float, relu: bool) -> torch.Tensor:
    """In place: y = relu?(LayerNorm_c(y + pre_bias) * weight + bias), the
    "channels_first" LayerNorm of uplift/uplift.py:50-92 following a conv run
    without its bias (the SD1.5-VAE blocks: Conv -> LayerNorm -> ReLU)."""
    dev = _check(y)
    B, C, H, W = y.shape
    pb = _param(pre_bias, y, C, "pre_bias")
    w = _param(weight, y, C, "weight")
    b = _param(bias, y, C, "bias")
    with torch.cuda.device(dev):
        rc = _native.load().uplift_layernorm_act(
            y.data_ptr(), _native.strides(y), None if pb is None else pb.data_ptr(), w.data_ptr(), b.data_ptr(),
            float(eps), int(bool(relu)), B, C, H, W, _DTYPES[y.dtype], _stream(dev))
    _native.check(rc, "uplift_layernorm_act")
    return y


# ----------------------------------------------------------------- custom ops
@torch.library.custom_op("uplift_b200::resize_bilinear", mutates_args=())
def _resize_bilinear_op(x: torch.Tensor, size: list[int], align_corners: bool) -> torch.Tensor:
    return resize_bilinear_raw(x, size, align_corners)


@_resize_bilinear_op.register_fake
def _(x, size, align_corners):
    return x.new_empty((x.shape[0], x.shape[1], size[0], size[1])).contiguous(memory_format=torch.channels_last)


@torch.library.custom_op("uplift_b200::upsample_add_", mutates_args=("y",))
def _upsample_add_op(y: torch.Tensor, x: torch.Tensor, align_corners: bool) -> None:
    resize_bilinear_raw(x, y.shape[2:], align_corners, out=y, accumulate=True)


@torch.library.custom_op("uplift_b200::nearest_into_", mutates_args=("dst",))
def _nearest_into_op(dst: torch.Tensor, src: torch.Tensor) -> None:
    resize_nearest_into_(dst, src)


@torch.library.custom_op("uplift_b200::add_channels_", mutates_args=("dst",))
def _add_channels_op(dst: torch.Tensor, src: torch.Tensor) -> None:
    add_channels_raw_(dst, src)


@torch.library.custom_op("uplift_b200::bias_act_", mutates_args=("y",))
def _bias_act_op(y: torch.Tensor, bias: Optional[torch.Tensor], relu: bool, res: Optional[torch.Tensor]) -> None:
    bias_act_raw_(y, bias, relu, res)


@torch.library.custom_op("uplift_b200::layernorm_act_", mutates_args=("y",))
def _layernorm_act_op(y: torch.Tensor, pre_bias: Optional[torch.Tensor], weight: torch.Tensor, bias: torch.Tensor,
                      eps: float, relu: bool) -> None:
    layernorm_act_raw_(y, pre_bias, weight, bias, eps, relu)


def layernorm_act_(y, pre_bias, weight, bias, eps, relu=False):
    """y = relu?(LayerNorm over channels of (y + pre_bias)), in place."""
    torch.ops.uplift_b200.layernorm_act_(y, pre_bias, weight, bias, float(eps), bool(relu))
    return y


def bias_act_(y, bias, relu=False, res=None):
    """y = relu?(y + bias) (+ residual), in place (conv epilogue)."""
    torch.ops.uplift_b200.bias_act_(y, bias, bool(relu), res)
    return y


def resize_bilinear(x, size, align_corners=False):
    """Bilinear resize (custom op entry)."""
    return torch.ops.uplift_b200.resize_bilinear(x, [int(size[0]), int(size[1])], bool(align_corners))


def upsample_add_(y, x, align_corners=True):
    """y += bilinear resize of x to y's size, in place (up-block residual)."""
    torch.ops.uplift_b200.upsample_add_(y, x, bool(align_corners))
    return y


def nearest_into_(dst, src):
    """dst = nearest resample of src to dst's size, in place."""
    torch.ops.uplift_b200.nearest_into_(dst, src)
    return dst


def add_channels_(dst, src):
    """dst[:, :c] += src[:, :c], in place."""
    torch.ops.uplift_b200.add_channels_(dst, src)
    return dst
