"""Torch-facing Local Attender operators over the C ABI.

`local_attender` (guide -> logits -> softmax -> pooled values) and
`attender_pool` (pre-projected logits -> pooled values) launch the sm_100a
kernels of libuplift_la.so on the current CUDA stream; `local_attender` is
differentiable (its backward runs the uplift_la_backward kernels).  Both are also
registered as torch custom ops (``torch.ops.uplift_b200.*``) with fake
implementations, so torch.compile traces them without a graph break (the
reference's Triton module takes one, uplift/kernels/triton_attender.py:335).

Inputs are accepted in any layout; the kernels read channels_last (NHWC)
storage, so other layouts are converted first.  The output is channels_last
in the value dtype.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _native

_DTYPES = {torch.float32: _native.F32, torch.bfloat16: _native.BF16, torch.float16: _native.F16}


def _nhwc(t: torch.Tensor) -> torch.Tensor:
    if t.stride(1) == 1 and t.is_contiguous(memory_format=torch.channels_last):
        return t
    if t.stride(1) == 1:  # sliced / padded channels_last view: strides are passed through
        return t
    return t.contiguous(memory_format=torch.channels_last)


def _check_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError(
                "uplift_b200 Local Attender runs on CUDA (sm_100) tensors only; got a "
                f"{t.device} tensor (there is no CPU fallback)")
        if t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def _offsets_flat(offsets) -> list[int]:
    return [int(v) for off in offsets for v in off]


def _scale(Ho: int, Wo: int, H: int, W: int) -> int:
    if H == 0 or W == 0:
        raise ValueError("value map has an empty spatial dimension")
    I = Ho // H
    if I < 1 or I * H != Ho or I * W != Wo:
        raise ValueError(f"output size {Ho}x{Wo} is not an integer multiple of the value size {H}x{W}")
    return I


def local_attender_raw(guide: torch.Tensor, value: torch.Tensor, weight: torch.Tensor,
                       bias: Optional[torch.Tensor], offsets: Sequence, pn: int,
                       conv_res: bool = True, hardmax: bool = False,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Launch uplift_la_forward.  weight: fp32 [K, Cg] (other dtypes/shapes
    are converted), bias: fp32 [K] or None."""
    dev = _check_cuda(guide, value, weight)
    if guide.dtype != value.dtype:
        raise ValueError(f"guide dtype {guide.dtype} != value dtype {value.dtype}")
    if value.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {value.dtype} (float32, bfloat16, float16)")
    if guide.dim() != 4 or value.dim() != 4:
        raise ValueError("guide and value must be 4-D [B, C, H, W]")
    B, C, H, W = value.shape
    Bg, Cg, Ho, Wo = guide.shape
    if Bg != B:
        raise ValueError(f"batch mismatch: guide {Bg} vs value {B}")
    I = _scale(Ho, Wo, H, W)
    K = len(offsets)
    w = weight.detach().reshape(K, -1)
    if w.shape[1] != Cg:
        raise ValueError(f"weight has {w.shape[1]} input channels, guide has {Cg}")
    if w.dtype != torch.float32 or not w.is_contiguous():
        w = w.to(torch.float32).contiguous()
    b = None
    if bias is not None:
        b = bias.detach()
        if b.dtype != torch.float32 or not b.is_contiguous():
            b = b.to(torch.float32).contiguous()
    g = _nhwc(guide)
    v = _nhwc(value)
    if out is None:
        out = torch.empty((B, C, Ho, Wo), dtype=value.dtype, device=dev,
                          memory_format=torch.channels_last)
    lib = _native.load()
    _native.host_status.raise_if_set()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        rc = lib.uplift_la_forward(
            g.data_ptr(), _native.strides(g), v.data_ptr(), _native.strides(v),
            w.data_ptr(), None if b is None else b.data_ptr(),
            out.data_ptr(), _native.strides(out),
            B, Cg, C, H, W, I, K, _native.offsets_array(offsets), int(pn), int(bool(conv_res)),
            _DTYPES[value.dtype], int(bool(hardmax)), stream)
    _native.check(rc, "uplift_la_forward")
    return out


def local_attender_resized_raw(guide: torch.Tensor, value: torch.Tensor, weight: torch.Tensor,
                               bias: Optional[torch.Tensor], offsets: Sequence, pn: int, size: Sequence[int],
                               conv_res: bool = True, hardmax: bool = False) -> torch.Tensor:
    """The attender followed by F.interpolate(size, mode="bilinear",
    align_corners=False): one launch of uplift_la_forward_resized when the
    fused kernel applies (the attender output is never stored), else the
    attender kernel and the glue resize kernel one after the other (same
    values up to the fp32 contraction order of the resize)."""
    dev = _check_cuda(guide, value, weight)
    if guide.dtype != value.dtype:
        raise ValueError(f"guide dtype {guide.dtype} != value dtype {value.dtype}")
    if value.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {value.dtype} (float32, bfloat16, float16)")
    B, C, H, W = value.shape
    Bg, Cg, Ho_a, Wo_a = guide.shape
    if Bg != B:
        raise ValueError(f"batch mismatch: guide {Bg} vs value {B}")
    I = _scale(Ho_a, Wo_a, H, W)
    Ho, Wo = int(size[0]), int(size[1])
    K = len(offsets)
    w = weight.detach().reshape(K, -1)
    if w.shape[1] != Cg:
        raise ValueError(f"weight has {w.shape[1]} input channels, guide has {Cg}")
    if w.dtype != torch.float32 or not w.is_contiguous():
        w = w.to(torch.float32).contiguous()
    b = None
    if bias is not None:
        b = bias.detach()
        if b.dtype != torch.float32 or not b.is_contiguous():
            b = b.to(torch.float32).contiguous()
    g = _nhwc(guide)
    v = _nhwc(value)
    out = torch.empty((B, C, Ho, Wo), dtype=value.dtype, device=dev, memory_format=torch.channels_last)
    lib = _native.load()
    _native.host_status.raise_if_set()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        rc = lib.uplift_la_forward_resized(
            g.data_ptr(), _native.strides(g), v.data_ptr(), _native.strides(v),
            w.data_ptr(), None if b is None else b.data_ptr(),
            out.data_ptr(), _native.strides(out),
            B, Cg, C, H, W, I, K, _native.offsets_array(offsets), int(pn), int(bool(conv_res)),
            _DTYPES[value.dtype], int(bool(hardmax)), Ho, Wo, stream)
    if rc == _native.ERR_UNSUPPORTED:
        from . import glue
        y = local_attender_raw(guide, value, w, b, offsets, pn, conv_res, hardmax)
        return glue.resize_bilinear_raw(y, (Ho, Wo))
    _native.check(rc, "uplift_la_forward_resized")
    return out


def _fp32(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if t is None:
        return None
    t = t.detach()
    return t if (t.dtype == torch.float32 and t.is_contiguous()) else t.to(torch.float32).contiguous()


def local_attender_fused_guide_raw(act: torch.Tensor, res: torch.Tensor, w_guide: torch.Tensor,
                                   b_guide: Optional[torch.Tensor], value: torch.Tensor, weight: torch.Tensor,
                                   bias: Optional[torch.Tensor], offsets: Sequence, pn: int,
                                   conv_res: bool = True, hardmax: bool = False,
                                   size: Optional[Sequence[int]] = None) -> torch.Tensor:
    """The attender of guide = conv1x1(act; w_guide, b_guide) + res[:, :Cg]
    (the decoder's last residual block, uplift/uplift.py:152-217), with the
    guide produced inside the attender launch (uplift_la_forward_fused_guide;
    `size`: also the final resize).  Where the fused kernel does not apply,
    the guide is built by the 1x1 convolution and the conv-epilogue kernel
    and the attender runs on it."""
    dev = _check_cuda(act, res, value, weight)
    B, C, H, W = value.shape
    Cg, Ho_a, Wo_a = act.shape[1], act.shape[2], act.shape[3]
    I = _scale(Ho_a, Wo_a, H, W)
    if res.shape[1] < Cg or tuple(res.shape[2:]) != (Ho_a, Wo_a) or res.shape[0] != B:
        raise ValueError(f"residual input {tuple(res.shape)} does not cover the guide {tuple(act.shape)}")
    K = len(offsets)
    wg = _fp32(w_guide).reshape(Cg, -1)
    if wg.shape[1] != Cg:
        raise ValueError(f"guide block weight {tuple(w_guide.shape)} is not a {Cg}->{Cg} 1x1 convolution")
    bg = _fp32(b_guide)
    w = _fp32(weight).reshape(K, -1)
    b = _fp32(bias)
    a = _nhwc(act)
    r = _nhwc(res)[:, :Cg]
    v = _nhwc(value)
    Ho, Wo = (I * H, I * W) if size is None else (int(size[0]), int(size[1]))
    out = torch.empty((B, C, Ho, Wo), dtype=value.dtype, device=dev, memory_format=torch.channels_last)
    lib = _native.load()
    _native.host_status.raise_if_set()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        rc = lib.uplift_la_forward_fused_guide(
            a.data_ptr(), _native.strides(a), r.data_ptr(), _native.strides(r),
            wg.data_ptr(), None if bg is None else bg.data_ptr(),
            v.data_ptr(), _native.strides(v), w.data_ptr(), None if b is None else b.data_ptr(),
            out.data_ptr(), _native.strides(out), B, Cg, C, H, W, I, K, _native.offsets_array(offsets),
            int(pn), int(bool(conv_res)), _DTYPES[value.dtype], int(bool(hardmax)),
            0 if size is None else Ho, 0 if size is None else Wo, stream)
    if rc == _native.ERR_UNSUPPORTED:
        import torch.nn.functional as F
        from . import glue
        y = F.conv2d(a, w_guide.detach().reshape(Cg, Cg, 1, 1).to(act.dtype)).contiguous(
            memory_format=torch.channels_last)
        guide = glue.bias_act_raw_(y, None if b_guide is None else b_guide.detach().to(act.dtype), False, r)
        if size is None:
            return local_attender_raw(guide, value, w, b, offsets, pn, conv_res, hardmax)
        return local_attender_resized_raw(guide, value, w, b, offsets, pn, size, conv_res, hardmax)
    _native.check(rc, "uplift_la_forward_fused_guide")
    return out


def attender_pool_raw(logits: torch.Tensor, value: torch.Tensor, offsets: Sequence, pn: int,
                      hardmax: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Launch uplift_la_pool on pre-projected logits [B, K, I*H, I*W]."""
    dev = _check_cuda(logits, value)
    if logits.dtype != value.dtype:
        logits = logits.to(value.dtype)
    if value.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {value.dtype} (float32, bfloat16, float16)")
    B, C, H, W = value.shape
    Bl, K, Ho, Wo = logits.shape
    if Bl != B:
        raise ValueError(f"batch mismatch: logits {Bl} vs value {B}")
    if K != len(offsets):
        raise ValueError(f"logits have {K} channels but {len(offsets)} offsets were given")
    I = _scale(Ho, Wo, H, W)
    v = _nhwc(value)
    if out is None:
        out = torch.empty((B, C, Ho, Wo), dtype=value.dtype, device=dev,
                          memory_format=torch.channels_last)
    lib = _native.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        rc = lib.uplift_la_pool(
            logits.data_ptr(), _native.strides(logits), v.data_ptr(), _native.strides(v),
            out.data_ptr(), _native.strides(out), B, C, H, W, I, K,
            _native.offsets_array(offsets), int(pn), _DTYPES[value.dtype], int(bool(hardmax)), stream)
    _native.check(rc, "uplift_la_pool")
    return out


def local_attender_backward_raw(grad: torch.Tensor, guide: torch.Tensor, value: torch.Tensor,
                                weight: torch.Tensor, bias: Optional[torch.Tensor], offsets: Sequence,
                                pn: int, conv_res: bool = True, hardmax: bool = False,
                                need_guide: bool = True, need_value: bool = True, need_params: bool = True):
    """Launch uplift_la_backward: (dguide, dvalue, dweight [K, Cg] fp32,
    dbias [K] fp32); entries not asked for are None."""
    dev = _check_cuda(grad, guide, value)
    B, C, H, W = value.shape
    Cg, Ho, Wo = guide.shape[1], guide.shape[2], guide.shape[3]
    I = _scale(Ho, Wo, H, W)
    K = len(offsets)
    w = weight.detach().reshape(K, -1).to(torch.float32).contiguous()
    b = None if bias is None else bias.detach().to(torch.float32).contiguous()
    d = _nhwc(grad.to(value.dtype))
    g = _nhwc(guide)
    v = _nhwc(value)
    probs = torch.empty((B, Ho, Wo, K), dtype=torch.float32, device=dev)
    dg = torch.empty_like(g, memory_format=torch.channels_last) if need_guide else None
    dv = torch.empty((B, C, H, W), dtype=value.dtype, device=dev,
                     memory_format=torch.channels_last) if need_value else None
    dw = torch.zeros((K, Cg), dtype=torch.float32, device=dev) if need_params else None
    db = torch.zeros((K,), dtype=torch.float32, device=dev) if (need_params and bias is not None) else None
    lib = _native.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        rc = lib.uplift_la_backward(
            d.data_ptr(), _native.strides(d), g.data_ptr(), _native.strides(g), v.data_ptr(), _native.strides(v),
            w.data_ptr(), None if b is None else b.data_ptr(), probs.data_ptr(),
            None if dg is None else dg.data_ptr(), _native.strides(dg if dg is not None else g),
            None if dv is None else dv.data_ptr(), _native.strides(dv if dv is not None else v),
            None if dw is None else dw.data_ptr(), None if db is None else db.data_ptr(),
            B, Cg, C, H, W, I, K, _native.offsets_array(offsets), int(pn), int(bool(conv_res)),
            _DTYPES[value.dtype], int(bool(hardmax)), stream)
    _native.check(rc, "uplift_la_backward")
    return dg, dv, dw, db


# ----------------------------------------------------------------- custom ops
def _pairs(flat: Sequence[int]):
    return [(flat[i], flat[i + 1]) for i in range(0, len(flat), 2)]


@torch.library.custom_op("uplift_b200::local_attender", mutates_args=())
def _local_attender_op(guide: torch.Tensor, value: torch.Tensor, weight: torch.Tensor,
                       bias: Optional[torch.Tensor], offsets: list[int], pn: int,
                       conv_res: bool, hardmax: bool) -> torch.Tensor:
    return local_attender_raw(guide, value, weight, bias, _pairs(offsets), pn, conv_res, hardmax)


@_local_attender_op.register_fake
def _(guide, value, weight, bias, offsets, pn, conv_res, hardmax):
    B, C = value.shape[0], value.shape[1]
    return value.new_empty((B, C, guide.shape[2], guide.shape[3])).contiguous(
        memory_format=torch.channels_last)


def _la_setup_context(ctx, inputs, output):
    guide, value, weight, bias, offsets, pn, conv_res, hardmax = inputs
    ctx.save_for_backward(guide, value, weight, bias)
    ctx.offsets, ctx.pn, ctx.conv_res, ctx.hardmax = offsets, pn, conv_res, hardmax


def _la_backward(ctx, grad):
    guide, value, weight, bias = ctx.saved_tensors
    ng, nv, nw, nb = ctx.needs_input_grad[:4]
    dg, dv, dw, db = local_attender_backward_raw(
        grad, guide, value, weight, bias, _pairs(ctx.offsets), ctx.pn, ctx.conv_res, ctx.hardmax,
        need_guide=ng, need_value=nv, need_params=nw or nb)
    dw = dw.reshape(weight.shape).to(weight.dtype) if nw else None
    db = db.to(bias.dtype) if (nb and db is not None) else None
    return dg, dv, dw, db, None, None, None, None


torch.library.register_autograd("uplift_b200::local_attender", _la_backward, setup_context=_la_setup_context)


@torch.library.custom_op("uplift_b200::local_attender_resized", mutates_args=())
def _local_attender_resized_op(guide: torch.Tensor, value: torch.Tensor, weight: torch.Tensor,
                               bias: Optional[torch.Tensor], offsets: list[int], pn: int, size: list[int],
                               conv_res: bool, hardmax: bool) -> torch.Tensor:
    return local_attender_resized_raw(guide, value, weight, bias, _pairs(offsets), pn, size, conv_res, hardmax)


@_local_attender_resized_op.register_fake
def _(guide, value, weight, bias, offsets, pn, size, conv_res, hardmax):
    B, C = value.shape[0], value.shape[1]
    return value.new_empty((B, C, int(size[0]), int(size[1]))).contiguous(memory_format=torch.channels_last)


@torch.library.custom_op("uplift_b200::local_attender_fused_guide", mutates_args=())
def _local_attender_fused_guide_op(act: torch.Tensor, res: torch.Tensor, w_guide: torch.Tensor,
                                   b_guide: Optional[torch.Tensor], value: torch.Tensor, weight: torch.Tensor,
                                   bias: Optional[torch.Tensor], offsets: list[int], pn: int, conv_res: bool,
                                   hardmax: bool, size: Optional[list[int]]) -> torch.Tensor:
    return local_attender_fused_guide_raw(act, res, w_guide, b_guide, value, weight, bias, _pairs(offsets), pn,
                                          conv_res, hardmax, size)


@_local_attender_fused_guide_op.register_fake
def _(act, res, w_guide, b_guide, value, weight, bias, offsets, pn, conv_res, hardmax, size):
    B, C = value.shape[0], value.shape[1]
    Ho, Wo = (act.shape[2], act.shape[3]) if size is None else (int(size[0]), int(size[1]))
    return value.new_empty((B, C, Ho, Wo)).contiguous(memory_format=torch.channels_last)


@torch.library.custom_op("uplift_b200::attender_pool", mutates_args=())
def _attender_pool_op(logits: torch.Tensor, value: torch.Tensor, offsets: list[int], pn: int,
                      hardmax: bool) -> torch.Tensor:
    return attender_pool_raw(logits, value, _pairs(offsets), pn, hardmax)


@_attender_pool_op.register_fake
def _(logits, value, offsets, pn, hardmax):
    B, C = value.shape[0], value.shape[1]
    return value.new_empty((B, C, logits.shape[2], logits.shape[3])).contiguous(
        memory_format=torch.channels_last)


def local_attender(guide, value, weight, bias, offsets, pn, conv_res=True, hardmax=False):
    """Fused Local Attender (custom op entry; traceable by torch.compile)."""
    return torch.ops.uplift_b200.local_attender(guide, value, weight, bias, _offsets_flat(offsets),
                                                int(pn), bool(conv_res), bool(hardmax))


def local_attender_resized(guide, value, weight, bias, offsets, pn, size, conv_res=True, hardmax=False):
    """Fused Local Attender + final bilinear resize to `size` (custom op
    entry; inference only -- it has no autograd formula)."""
    return torch.ops.uplift_b200.local_attender_resized(guide, value, weight, bias, _offsets_flat(offsets),
                                                        int(pn), [int(size[0]), int(size[1])],
                                                        bool(conv_res), bool(hardmax))


def local_attender_fused_guide(act, res, w_guide, b_guide, value, weight, bias, offsets, pn, conv_res=True,
                               hardmax=False, size=None):
    """Attender with the guide produced inside the launch (custom op entry;
    inference only)."""
    return torch.ops.uplift_b200.local_attender_fused_guide(
        act, res, w_guide, b_guide, value, weight, bias, _offsets_flat(offsets), int(pn), bool(conv_res),
        bool(hardmax), None if size is None else [int(size[0]), int(size[1])])


def attender_pool(logits, value, offsets, pn, hardmax=False):
    """Softmax-pool from pre-projected logits (custom op entry)."""
    return torch.ops.uplift_b200.attender_pool(logits, value, _offsets_flat(offsets), int(pn),
                                               bool(hardmax))
