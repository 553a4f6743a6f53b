"""Fast inference mode -- drop-in for the reference's `uplift.fast`.

`make_fast(model, image_size, compile, compile_mode, warmup, device)` keeps
the reference's signature and behaviour (uplift/fast.py:71-133): deep copy,
BatchNorm folding, channels_last, optional torch.compile of the iteration
loop, optional warm-up.  The attender swap differs: the reference swaps in
its Triton kernel only for K = 17 and silently keeps the PyTorch attender
otherwise (uplift/fast.py:106-119); here every K goes to the fused sm_100a
kernel (one launch including conv1 and the residual), and a missing library
raises instead of falling back.
"""
from __future__ import annotations

import copy
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attender import AttenderWrapper, LocalAttender


def make_fast(model: nn.Module, image_size: Optional[int] = None, compile: bool = True,
              compile_mode: str = "max-autotune", warmup: bool = True,
              device: Optional[torch.device] = None) -> nn.Module:
    """Optimise a UPLiFT model for inference (see module docstring)."""
    if device is None:
        device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    fast = OptimizedUPLiFT(model, device=device)
    if isinstance(fast.model.attender, LocalAttender):
        fast.model.attender = AttenderWrapper(fast.model.attender).to(device).eval()
    if compile:
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

    @torch.inference_mode()
    def forward(self, img, x, outsize=None):
        if self._compiled_forward is not None:
            return self._compiled_forward(img, x, outsize)
        return self._forward_impl(img, x, outsize)

    def _forward_impl(self, img, x, outsize=None):
        """The iteration loop of UPLiFT.forward with F.interpolate resizes
        (as the reference's fast path, uplift/fast.py:168-223)."""
        m = self.model
        ex_feats = None
        steps = []
        for i in range(m.iters):
            if i > 0 and not m.enc_share:
                sf = m.up_factor ** i
                img_i = F.interpolate(img, size=(int(img.shape[2] * sf), int(img.shape[3] * sf)),
                                      mode="bilinear", align_corners=False)
            else:
                img_i = img
            x_in = x
            if not m.enc_share or ex_feats is None:
                if m.patch_size == 14:
                    img_i = F.interpolate(img_i, size=((img_i.shape[2] * 16) // 14, (img_i.shape[3] * 16) // 14),
                                          mode="bilinear", align_corners=False)
                enc_feats = m.encoder(img_i)
            else:
                enc_feats = ex_feats
            x = m.decoder(x, enc_feats)
            if m.attender is not None:
                x = m.attender(x, x_in)
            if m.refiner is not None:
                x = self._noise_and_combine_fast(x, enc_feats[m.ref_con], m.ref_ncat_c, m.ref_ncat_s,
                                                 m.ref_enc_resample)
                x = m.ref_outc(m.refiner(x))
            ex_feats = enc_feats
            steps.append(x)
        if outsize is not None:
            return _resize_bilinear(x, outsize)
        if m.return_all_steps:
            return steps
        return x

    @staticmethod
    def _noise_and_combine_fast(x, f=None, ncat_c=0, ncat_s=1, f_resample="none"):
        if f is not None:
            if f_resample == "nearest":
                f = F.interpolate(f, size=(x.shape[2], x.shape[3]), mode="nearest")
            elif f_resample == "bilinear":
                f = F.interpolate(f, size=(x.shape[2], x.shape[3]), mode="bilinear", align_corners=False)
            x = torch.cat([x, f], dim=1)
        if ncat_c > 0:
            x = torch.cat([x, ncat_s * torch.randn([x.shape[0], ncat_c, x.shape[2], x.shape[3]],
                                                   device=x.device, dtype=x.dtype)], dim=1)
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


_INT_MAX = 2**31 - 1


def _resize_bilinear(x, size):
    """F.interpolate(bilinear, align_corners=False), split along the batch
    when the input or output exceeds the 2^31-element limit of torch's
    channels_last bilinear kernel (e.g. 8 x 384 x 1168^2)."""
    out_numel = x.shape[0] * x.shape[1] * size[0] * size[1]
    if max(x.numel(), out_numel) <= _INT_MAX or x.shape[0] == 1:
        return F.interpolate(x, size=size, mode="bilinear", align_corners=False)
    per = max(1, _INT_MAX // max(x[0].numel(), out_numel // x.shape[0]))
    return torch.cat([F.interpolate(x[i:i + per], size=size, mode="bilinear", align_corners=False)
                      for i in range(0, x.shape[0], per)], dim=0)


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
