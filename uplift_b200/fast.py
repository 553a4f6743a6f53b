"""Fast inference mode -- drop-in for the reference's `uplift.fast`.

`make_fast(model, image_size, compile, compile_mode, warmup, device)` keeps
the reference's signature and behaviour (uplift/fast.py:71-133): deep copy,
BatchNorm folding, channels_last, optional torch.compile of the iteration
loop, optional warm-up.  The attender swap differs: the reference swaps in
its Triton kernel only for K = 17 and silently keeps the PyTorch attender
otherwise (uplift/fast.py:106-119); here every K goes to the fused sm_100a
kernel (one launch including conv1 and the residual), and a missing library
raises instead of falling back.

The iteration loop (uplift/fast.py:168-223) runs the encoder / decoder /
refiner convolutions as cuDNN module calls and everything between them on
the sm_100a glue kernels (uplift_b200.glue): residual_auto adds in place
into the fresh conv output, the up-block residual resize fused with its
add, the skip-feature resample written straight into the concatenation
buffer, and the final resize -- each one HBM pass, same values as the
reference's eager ops.
"""
from __future__ import annotations

import copy
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import glue
from . import uplift as U
from .attender import AttenderWrapper, LocalAttender


def make_fast(model: nn.Module, image_size: Optional[int] = None, compile: bool = True,
              compile_mode: str = "max-autotune", warmup: bool = True,
              device: Optional[torch.device] = None, allow_tf32: Optional[bool] = None) -> nn.Module:
    """Optimise a UPLiFT model for inference (see module docstring).

    `allow_tf32` (an addition to the reference's signature): None takes the
    model's own setting (UPLiFT(..., allow_tf32=...)) and, when that is
    None too, does what the reference does -- compile=True switches TF32 on
    globally (uplift/fast.py:122-124).  False gives an fp32-exact fast mode:
    every forward runs with TF32 off (BatchNorm folded, channels_last, fused
    kernels) and the global switches are left as they were; True runs every
    forward with TF32 on, also without touching the globals."""
    if device is None:
        device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    if allow_tf32 is None:
        allow_tf32 = getattr(model, "allow_tf32", None)
    fast = OptimizedUPLiFT(model, device=device)
    fast.allow_tf32 = allow_tf32
    if isinstance(fast.model.attender, LocalAttender):
        fast.model.attender = AttenderWrapper(fast.model.attender).to(device).eval()
    if compile:
        if allow_tf32 is None:
            torch.backends.cuda.matmul.allow_tf32 = True
            torch.backends.cudnn.allow_tf32 = True
        fast._compiled_forward = torch.compile(fast._forward_impl, mode=compile_mode)
    if warmup and image_size is not None and compile:
        _warmup(fast, image_size, device)
    return fast


class OptimizedUPLiFT(nn.Module):
    """Inference wrapper returned by make_fast (uplift/fast.py:140-263)."""

    def __init__(self, model: nn.Module, device: torch.device):
        super().__init__()
        self.model = copy.deepcopy(model)
        self.model.eval()
        self._fold_batchnorm()
        self.model = self.model.to(device=device)
        self.model = self.model.to(memory_format=torch.channels_last)
        self._compiled_forward = None
        self.allow_tf32 = None  # set by make_fast
        # produce the guide inside the attender launch (the decoder's last
        # 1x1 convolution and residual folded into its projection)
        self.fuse_guide = True

    @torch.inference_mode()
    def forward(self, img, x, outsize=None):
        with U.tf32_mode(self.allow_tf32):
            if self._compiled_forward is not None:
                return self._compiled_forward(img, x, outsize)
            return self._forward_impl(img, x, outsize)

    def _forward_impl(self, img, x, outsize=None):
        """The iteration loop of UPLiFT.forward (as the reference's fast path,
        uplift/fast.py:168-223), convolutions as module calls, glue on the
        sm_100a kernels."""
        m = self.model
        ex_feats = None
        steps = []
        for i in range(m.iters):
            if i > 0 and not m.enc_share:
                sf = m.up_factor ** i
                img_i = glue.resize_bilinear(img, (int(img.shape[2] * sf), int(img.shape[3] * sf)))
            else:
                img_i = img
            x_in = x
            if not m.enc_share or ex_feats is None:
                if m.patch_size == 14:
                    img_i = glue.resize_bilinear(img_i, ((img_i.shape[2] * 16) // 14, (img_i.shape[3] * 16) // 14))
                enc_feats = _encoder(m.encoder, img_i)
            else:
                enc_feats = ex_feats
            wrapped = isinstance(m.attender, AttenderWrapper)
            # the decoder's last 1x1 convolution + residual (the guide) is
            # computed inside the attender launch where the kernel allows it
            x = _decoder(m.decoder, x, enc_feats, defer_guide=wrapped and self.fuse_guide)
            # the last attender call also applies the final resize when
            # nothing runs between the two (one launch, the attender output
            # is never stored)
            fuse = (outsize is not None and i == m.iters - 1 and m.refiner is None and wrapped)
            size = tuple(outsize) if fuse else None
            if isinstance(x, _DeferredGuide):
                x = m.attender.forward_fused_guide(x.act, x.res, x.conv, x_in, size=size)
                if fuse:
                    return x
            elif fuse:
                return m.attender(x, x_in, size=size)
            elif m.attender is not None:
                x = m.attender(x, x_in)
            if m.refiner is not None:
                x = _combine(x, enc_feats[m.ref_con], m.ref_ncat_c, m.ref_ncat_s, m.ref_enc_resample)
                x = m.ref_outc(_group(m.refiner, x))
            ex_feats = enc_feats
            steps.append(x)
        if outsize is not None:
            return glue.resize_bilinear(x, outsize)
        if m.return_all_steps:
            return steps
        return x

    def _fold_batchnorm(self):
        """Fuse Conv2d + BatchNorm2d pairs inside Sequentials."""
        for module in self.model.modules():
            if not isinstance(module, nn.Sequential):
                continue
            children = list(module.children())
            out, i = [], 0
            while i < len(children):
                c = children[i]
                if (i + 1 < len(children) and isinstance(c, nn.Conv2d)
                        and isinstance(children[i + 1], nn.BatchNorm2d)):
                    out.append(torch.nn.utils.fuse_conv_bn_eval(c, children[i + 1]))
                    i += 2
                else:
                    out.append(c)
                    i += 1
            for idx, child in enumerate(out):
                module[idx] = child
            while len(module) > len(out):
                del module[len(out)]


# ----------------------------------------------------------------- executor
# Module-by-module mirrors of the forward methods in uplift_b200/uplift.py
# (the reference's uplift/uplift.py:96-531), with the glue on sm_100a
# kernels.  A conv Sequential always returns a fresh tensor, so residual
# sums are written into it in place.

def _cl(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous(memory_format=torch.channels_last)


def _plain_conv(mod) -> bool:
    return type(mod) is nn.Conv2d and mod.padding_mode == "zeros"


# cuDNN's fused convolution + bias + ReLU (one kernel; the bias is added
# before the single rounding of the result, where the eager conv -> + bias ->
# ReLU rounds twice: at most one storage-type ulp apart, like the BatchNorm
# folding of this mode)
_CONV_RELU = getattr(torch, "cudnn_convolution_relu", None)


def _conv_relu(mod, x):
    if _CONV_RELU is not None and not isinstance(mod.padding, str) and x.is_cuda:
        return _CONV_RELU(x, mod.weight, mod.bias, list(mod.stride), list(mod.padding),
                          list(mod.dilation), mod.groups)
    y = _cl(F.conv2d(x, mod.weight, None, mod.stride, mod.padding, mod.dilation, mod.groups))
    return glue.bias_act_(y, mod.bias, True)


def _conv_seq(seq, x, res=None):
    """Run a conv Sequential (Conv [-> ReLU] ... after BatchNorm folding):
    each Conv2d without its bias, then one epilogue pass adding the bias,
    applying the ReLU that follows and, after the last module, adding the
    block residual `res`.  Other modules run as they are.  Returns (y, True)
    when `res` was added."""
    mods = list(seq)
    i, used = 0, False
    while i < len(mods):
        mod = mods[i]
        if (_plain_conv(mod) and i + 1 < len(mods) and type(mods[i + 1]) is U.LayerNorm
                and mods[i + 1].data_format == "channels_first"):
            # Conv -> LayerNorm over channels [-> ReLU]: one pass after the conv
            ln = mods[i + 1]
            relu = i + 2 < len(mods) and type(mods[i + 2]) is nn.ReLU
            nxt = i + (3 if relu else 2)
            y = _cl(F.conv2d(x, mod.weight, None, mod.stride, mod.padding, mod.dilation, mod.groups))
            x = glue.layernorm_act_(y, mod.bias, ln.weight, ln.bias, ln.eps, relu)
            if res is not None and nxt == len(mods):
                x = glue.add_channels_(x, res)
                used = True
            i = nxt
        elif _plain_conv(mod):
            relu = i + 1 < len(mods) and type(mods[i + 1]) is nn.ReLU
            nxt = i + (2 if relu else 1)
            r = res if nxt == len(mods) else None
            if relu and r is None:
                x = _conv_relu(mod, x)
            else:
                y = _cl(F.conv2d(x, mod.weight, None, mod.stride, mod.padding, mod.dilation, mod.groups))
                x = glue.bias_act_(y, mod.bias, relu, r)
            used = used or r is not None
            i = nxt
        else:
            x = mod(x)
            i += 1
    return x, used


def _conv_block(b, x):
    """_ConvBlock.forward: convs (bias, ReLU and the residual_auto add fused
    into their epilogues)."""
    if not b.residual:
        return _conv_seq(b.conv, x)[0]
    xr = b.res_down(x) if b.stride == 2 else x
    y, used = _conv_seq(b.conv, x, xr)
    return y if used else glue.add_channels_(_cl(y), xr)


def _transposed(mod, x):
    """ConvTranspose2d without its bias, then the bias in one vectorised
    pass (torch adds it with a broadcast that does not vectorise)."""
    if type(mod) is not nn.ConvTranspose2d or mod.padding_mode != "zeros":
        return _cl(mod(x))
    y = F.conv_transpose2d(x, mod.weight, None, mod.stride, mod.padding, mod.output_padding, mod.groups,
                           mod.dilation)
    return glue.bias_act_(_cl(y), mod.bias, False)


def _tconv(b, x):
    """TransposeConv.forward: y = up(x) (+ bilinear x, align_corners=True)."""
    y = _transposed(b.up, x)
    if b.residual != "bilinear":
        return y
    if x.shape[1] == y.shape[1]:
        return glue.upsample_add_(y, x, align_corners=True)
    return glue.add_channels_(y, glue.resize_bilinear(x, y.shape[2:], align_corners=True))


def _block(b, x):
    if isinstance(b, U._ConvBlock):
        return _conv_block(b, x)
    if isinstance(b, U.TransposeConv):
        return _tconv(b, x)
    return b(x)


def _group(g, x):
    if g.count == 0:
        return x
    for b in g.blocks:
        x = _block(b, x)
    return x


def _down(d, x):
    if d.down is None:
        return x
    y = d.down(x)
    if d.residual == "bilinear":
        y = glue.add_channels_(_cl(y), d.res_down(x))
    return y


def _up(u, x):
    """UpBlock.forward: transposed conv + bilinear (align_corners=True)
    residual, the resize fused with the add."""
    if u.up is None:
        return x
    y = _transposed(u.up, x)
    if u.residual != "bilinear":
        return y
    return glue.upsample_add_(y, x, align_corners=True)


def _combine(x, f=None, ncat_c=0, ncat_s=1, f_resample="none"):
    """noise_and_combine: [x | resampled f | noise] written into one
    channels_last buffer (no separate resize output, no cat pass).  The
    noise is drawn exactly as the module path draws it."""
    if f is None and ncat_c == 0:
        return x
    B, C1, H, W = x.shape
    C2 = 0 if f is None else f.shape[1]
    buf = torch.empty((B, C1 + C2 + ncat_c, H, W), dtype=x.dtype, device=x.device,
                      memory_format=torch.channels_last)
    glue.nearest_into_(buf[:, :C1], x)  # same size: a copy
    if f is not None:
        if f_resample == "bilinear":
            f = glue.resize_bilinear(f, (H, W))
        glue.nearest_into_(buf[:, C1:C1 + C2], f)
    if ncat_c > 0:
        noise = ncat_s * U._randn([B, ncat_c, H, W], x.device, x.dtype)
        glue.nearest_into_(buf[:, C1 + C2:], noise)
    return buf


def _encoder(e, x):
    feats = [_group(e.block_0, x)]
    x = feats[0]
    for i in range(1, e.down_steps + 1):
        x = _group(getattr(e, f"block_{i}"), _down(getattr(e, f"down_{i}"), x))
        feats.append(x)
    return feats


class _DeferredGuide:
    """The guide left as the last block's activation before its final 1x1
    convolution (`act`), that convolution and the block's residual input
    (`res`, truncated to the guide's channels by the kernel, as
    residual_auto does): guide = conv(act) + res[:, :Cg]."""

    def __init__(self, act, conv, res):
        self.act, self.conv, self.res = act, conv, res


def _guide_tail(b, x):
    """A _DeferredGuide for block `b` on input `x` when the block is a
    residual conv block (stride 1) ending in a Cg -> Cg 1x1 convolution with
    bias whose residual input has at least Cg channels; else None."""
    if not isinstance(b, U._ConvBlock) or not b.residual or b.stride != 1:
        return None
    mods = list(b.conv)
    last = mods[-1] if mods else None
    if not (_plain_conv(last) and tuple(last.kernel_size) == (1, 1) and tuple(last.stride) == (1, 1)
            and last.groups == 1 and last.bias is not None and last.in_channels == last.out_channels
            and x.shape[1] >= last.out_channels):
        return None
    act, _ = _conv_seq(mods[:-1], x)
    return _DeferredGuide(_cl(act), last, x)


def _decoder(d, x, enc_feats, defer_guide=False):
    x = _combine(x, enc_feats[-1], d.ncat_c, d.ncat_s, d.enc_resample)
    for i in range(d.up_steps + 1):
        if i > 0:
            x = _up(getattr(d, f"up_{i}"), x)
            x = _combine(x, enc_feats[-1 - i], d.ncat_c, d.ncat_s, d.enc_resample)
        g = getattr(d, f"block_{i}")
        last = i == d.up_steps
        if last and defer_guide and d.using_attender and g.count > 0:
            for b in g.blocks[:-1]:
                x = _block(b, x)
            tail = _guide_tail(g.blocks[-1], x)
            x = tail if tail is not None else _block(g.blocks[-1], x)
        else:
            x = _group(g, x)
    if d.using_attender:
        return x
    y = d.outc(x)
    return glue.add_channels_(_cl(y), x) if d.residual_outc else y


def _warmup(fast: OptimizedUPLiFT, image_size: int, device: torch.device):
    """One forward at the expected size to trigger compilation."""
    m = fast.model
    dtype = next(m.parameters()).dtype
    lat = image_size // m.patch_size
    with torch.inference_mode():
        fast(torch.randn(1, 3, image_size, image_size, device=device, dtype=dtype),
             torch.randn(1, m.in_channels, lat, lat, device=device, dtype=dtype))
        torch.cuda.synchronize()
    torch.cuda.empty_cache()
