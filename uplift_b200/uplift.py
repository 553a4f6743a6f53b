"""UPLiFT iterative upsampler -- the caller of the Local Attender.

The encoder / decoder / refiner are plain torch modules (cuDNN convs); the
Local Attender is the fused sm_100a kernel (uplift_b200.attender).  The
module tree and attribute names follow the reference's model
(uplift/uplift.py:96-709) because checkpoint keys depend on them:
`encoder.block_0.blocks.0.conv.0.weight`, `attender.conv1.weight`, ... load
unchanged.  Public API kept: UPLiFT(in_channels, patch_size, cfg, dtype,
low_mem), enable_iterative, return_steps, upsample, forward(img, x,
outsize), compiled.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
import torchvision.transforms.functional as TVF
from torchvision import transforms

from .attender import LocalAttender  # noqa: F401  (re-exported: uplift.uplift.LocalAttender)


def residual_auto(x1, x2):
    """x2 + x1, with x1 truncated or zero-padded to x2's channel count
    (uplift/uplift.py:26-39)."""
    c1, c2 = x1.shape[1], x2.shape[1]
    if c1 == c2:
        return x1 + x2
    if c1 > c2:
        return x1[:, :c2] + x2
    out = x2.clone()
    out[:, :c1] += x1
    return out


def resize_sf(image_batch, sf):
    """Resize by a scale factor (uplift/uplift.py:43-47)."""
    h = int(image_batch.shape[2] * sf)
    w = int(image_batch.shape[3] * sf)
    return TVF.resize(image_batch, [h, w])


class LayerNorm(nn.Module):
    """Layer norm over the channel axis of NCHW maps ("channels_first") or
    the last axis ("channels_last"); parameters `weight`, `bias`."""

    def __init__(self, normalized_shape, eps=1e-6, data_format="channels_last"):
        super().__init__()
        if data_format not in ("channels_last", "channels_first"):
            raise NotImplementedError(data_format)
        self.weight = nn.Parameter(torch.ones(normalized_shape))
        self.bias = nn.Parameter(torch.zeros(normalized_shape))
        self.eps = eps
        self.data_format = data_format
        self.normalized_shape = (normalized_shape,)

    def forward(self, x):
        if self.data_format == "channels_last":
            return F.layer_norm(x, self.normalized_shape, self.weight, self.bias, self.eps)
        mu = x.mean(1, keepdim=True)
        var = (x - mu).pow(2).mean(1, keepdim=True)
        xn = (x - mu) / torch.sqrt(var + self.eps)
        return self.weight[:, None, None] * xn + self.bias[:, None, None]


def _norm(kind, ch):
    return nn.BatchNorm2d(ch) if kind == "batch" else LayerNorm(ch, eps=1e-6, data_format="channels_first")


class IdentityBlock(nn.Module):
    def forward(self, x):
        return x


class _ConvBlock(nn.Module):
    """3x3 conv -> norm -> ReLU, repeated over `widths`, optional trailing
    1x1 conv with bias, optional residual (bilinear-halved when strided)."""

    def __init__(self, in_channels, widths, norm_type="batch", residual=True, stride=1, one_by=True):
        super().__init__()
        assert norm_type in ("batch", "layer") and stride in (1, 2)
        self.residual = residual
        self.norm_type = norm_type
        self.stride = stride
        self.one_by = one_by
        layers, ic = [], in_channels
        for w in widths:
            layers += [nn.Conv2d(ic, w, kernel_size=3, padding=1, bias=False, stride=stride),
                       _norm(norm_type, w), nn.ReLU(inplace=True)]
            ic = w
        if one_by:
            layers.append(nn.Conv2d(ic, ic, kernel_size=1, bias=True))
        self.conv = nn.Sequential(*layers)
        self.res_down = None
        if residual and stride == 2:
            self.res_down = nn.UpsamplingBilinear2d(scale_factor=0.5)

    def forward(self, x):
        y = self.conv(x)
        if not self.residual:
            return y
        xr = self.res_down(x) if self.stride == 2 else x
        return residual_auto(xr, y)


class SingleConv(_ConvBlock):
    """uplift/uplift.py:96-148"""

    def __init__(self, in_channels, h1, norm_type="batch", residual=True, stride=1, one_by=True):
        super().__init__(in_channels, [h1], norm_type, residual, stride, one_by)


class DoubleConv(_ConvBlock):
    """uplift/uplift.py:152-217 (the second 3x3 conv is strided too)."""

    def __init__(self, in_channels, h1, h2, norm_type="batch", residual=True, stride=1, one_by=True):
        super().__init__(in_channels, [h1, h2], norm_type, residual, stride, one_by)


class TransposeConv(nn.Module):
    """uplift/uplift.py:221-235"""

    def __init__(self, in_channels, h1, residual="none"):
        super().__init__()
        assert residual in ("none", "bilinear")
        self.up = nn.ConvTranspose2d(in_channels, h1, kernel_size=2, stride=2)
        self.residual = residual
        if residual == "bilinear":
            self.res_up = nn.UpsamplingBilinear2d(scale_factor=2)

    def forward(self, x):
        y = self.up(x)
        if self.residual == "bilinear":
            y = residual_auto(self.res_up(x), y)
        return y


class BlockGroup(nn.Module):
    """`count` blocks of one type (uplift/uplift.py:238-273)."""

    BLOCKS = ("IdentityBlock", "SingleConv", "DoubleConv", "TransposeConv")

    def __init__(self, in_channels, cfg):
        super().__init__()
        if cfg.block not in self.BLOCKS:
            raise ValueError(f"invalid block type: {cfg.block}")
        self.cfg = cfg
        self.count = cfg.count
        kw = {}
        if cfg.block in ("SingleConv", "DoubleConv"):
            self.residual = getattr(cfg, "residual", True)
            self.stride = getattr(cfg, "stride", 1)
            self.one_by = getattr(cfg, "one_by", True)
            self.norm = getattr(cfg, "norm", "batch")
            kw = dict(norm_type=self.norm, residual=self.residual, stride=self.stride, one_by=self.one_by)
        if self.count > 0:
            blocks, ic = [], in_channels
            for i in range(cfg.count):
                oc = cfg.hc[i]
                if cfg.block == "IdentityBlock":
                    blocks.append(IdentityBlock())
                elif cfg.block == "SingleConv":
                    blocks.append(SingleConv(ic, oc, **kw))
                elif cfg.block == "DoubleConv":
                    blocks.append(DoubleConv(ic, oc, oc, **kw))
                else:
                    blocks.append(TransposeConv(ic, oc))
                ic = oc
            self.blocks = nn.Sequential(*blocks)

    def forward(self, x):
        return self.blocks(x) if self.count > 0 else x


class DownBlock(nn.Module):
    """uplift/uplift.py:280-315"""

    def __init__(self, in_channels, cfg):
        super().__init__()
        self.cfg = cfg
        self.down_op = cfg.down_op
        assert self.down_op in ("conv", "max", "none")
        self.down = None
        self.residual = "none"
        if self.down_op == "none":
            return
        self.factor = cfg.factor
        if self.down_op == "conv":
            self.stride = int(1 / self.factor)
            self.norm_op = nn.BatchNorm2d
            self.down = nn.Sequential(
                nn.Conv2d(in_channels, in_channels, kernel_size=3, padding=1, stride=self.stride),
                nn.BatchNorm2d(in_channels), nn.ReLU(inplace=True))
        else:
            self.down = nn.MaxPool2d(2, 2)
        self.residual = cfg.residual
        assert self.residual in ("bilinear", "none")
        if self.residual == "bilinear":
            self.res_down = nn.UpsamplingBilinear2d(scale_factor=self.factor)

    def forward(self, x):
        if self.down is None:
            return x
        y = self.down(x)
        if self.residual == "bilinear":
            y = residual_auto(self.res_down(x), y)
        return y


class UpBlock(nn.Module):
    """uplift/uplift.py:319-343"""

    def __init__(self, in_channels, cfg):
        super().__init__()
        self.cfg = cfg
        assert cfg.up_op in ("tconv", "none")
        self.up = None
        self.residual = "none"
        if cfg.up_op == "none":
            return
        self.factor = cfg.factor
        self.up = nn.ConvTranspose2d(in_channels, in_channels, kernel_size=self.factor, stride=self.factor)
        self.residual = cfg.residual
        assert self.residual in ("bilinear", "none")
        if self.residual == "bilinear":
            self.res_up = nn.UpsamplingBilinear2d(scale_factor=self.factor)

    def forward(self, x):
        if self.up is None:
            return x
        y = self.up(x)
        if self.residual == "bilinear":
            y = residual_auto(self.res_up(x), y)
        return y


# Noise source of noise_and_combine; tests replace it with seeded noise to
# compare against the reference (which draws torch.randn on the fly).
def _randn(shape, device, dtype):
    return torch.randn(shape, device=device, dtype=dtype)


def noise_and_combine(x, f=None, ncat_c=0, ncat_s=1, f_resample="none"):
    """Concatenate skip features (optionally resized to x) and `ncat_c`
    Gaussian noise channels scaled by `ncat_s` (uplift/uplift.py:354-367)."""
    if f is not None:
        if f_resample == "nearest":
            # TVF.resize(NEAREST) == F.interpolate(mode="nearest") value for
            # value; this skips its fp32 round trip for bf16 / fp16 maps
            f = F.interpolate(f, size=(x.shape[2], x.shape[3]), mode="nearest")
        elif f_resample == "bilinear":
            f = TVF.resize(f, [x.shape[2], x.shape[3]], interpolation=transforms.InterpolationMode.BILINEAR)
        x = torch.cat([x, f], dim=1)
    if ncat_c > 0:
        noise = ncat_s * _randn([x.shape[0], ncat_c, x.shape[2], x.shape[3]], x.device, x.dtype)
        x = torch.cat([x, noise], dim=1)
    return x


class UPLiFTEncoder(nn.Module):
    """Image encoder with 0-4 optional downsampling steps
    (uplift/uplift.py:373-442)."""

    def __init__(self, in_channels, cfg):
        super().__init__()
        self.cfg = cfg
        self.down_steps = cfg.down_steps
        assert self.down_steps in (0, 1, 2, 3, 4)
        self.out_sizes = []
        ic = in_channels
        self.block_0 = BlockGroup(ic, cfg.block_0)
        ic = cfg.block_0.hc[-1]
        self.out_sizes.append(ic)
        for i in range(1, self.down_steps + 1):
            setattr(self, f"down_{i}", DownBlock(ic, getattr(cfg, f"down_{i}")))
            bcfg = getattr(cfg, f"block_{i}")
            setattr(self, f"block_{i}", BlockGroup(ic, bcfg))
            ic = bcfg.hc[-1]
            self.out_sizes.append(ic)

    def get_out_sizes(self):
        return self.out_sizes

    def forward(self, x):
        feats = [self.block_0(x)]
        x = feats[0]
        for i in range(1, self.down_steps + 1):
            x = getattr(self, f"block_{i}")(getattr(self, f"down_{i}")(x))
            feats.append(x)
        return feats


class UPLiFTDecoder(nn.Module):
    """Decoder with 0-4 upsampling steps fed by encoder skips; ends with the
    guide map when an attender follows (uplift/uplift.py:448-531)."""

    def __init__(self, in_channels, out_channels, cfg, enc_channels=None, using_attender=False):
        super().__init__()
        self.cfg = cfg
        self.ncat_c = cfg.ncat_c
        self.ncat_s = cfg.ncat_s
        self.up_steps = cfg.up_steps
        self.using_attender = using_attender
        assert self.up_steps in (0, 1, 2, 3, 4)
        self.enc_channels = [0, 0, 0, 0, 0] if enc_channels is None else enc_channels
        self.enc_resample = getattr(cfg, "enc_resample", "none")
        assert self.enc_resample in ("none", "nearest", "bilinear")
        ic = in_channels + self.enc_channels[-1] + cfg.ncat_c
        self.block_0 = BlockGroup(ic, cfg.block_0)
        ic = cfg.block_0.hc[-1]
        for i in range(1, self.up_steps + 1):
            setattr(self, f"up_{i}", UpBlock(ic, getattr(cfg, f"up_{i}")))
            ic = ic + self.enc_channels[-1 - i] + cfg.ncat_c
            bcfg = getattr(cfg, f"block_{i}")
            setattr(self, f"block_{i}", BlockGroup(ic, bcfg))
            ic = bcfg.hc[-1]
        self.out_channels = ic
        if not using_attender:
            self.outc = nn.Conv2d(ic, out_channels, kernel_size=1)
            self.residual_outc = getattr(cfg, "residual_outc", True)
            self.out_channels = out_channels

    def forward(self, x, enc_feats):
        x = noise_and_combine(x, enc_feats[-1], self.ncat_c, self.ncat_s, self.enc_resample)
        x = self.block_0(x)
        for i in range(1, self.up_steps + 1):
            x = getattr(self, f"up_{i}")(x)
            x = noise_and_combine(x, enc_feats[-1 - i], self.ncat_c, self.ncat_s, self.enc_resample)
            x = getattr(self, f"block_{i}")(x)
        if self.using_attender:
            return x
        y = self.outc(x)
        return residual_auto(x, y) if self.residual_outc else y


class tf32_mode:
    """Scope the TF32 switches of cuDNN convolutions and matmuls to a block:
    allow=True / False sets both for the block and restores the previous
    values after it; allow=None leaves them as they are.  The switches are
    process-wide, so blocks that run at the same time in several host
    threads see each other's settings."""

    def __init__(self, allow: Optional[bool]):
        self.allow = allow
        self._old = None

    def __enter__(self):
        if self.allow is not None:
            self._old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
            torch.backends.cuda.matmul.allow_tf32 = bool(self.allow)
            torch.backends.cudnn.allow_tf32 = bool(self.allow)
        return self

    def __exit__(self, *exc):
        if self._old is not None:
            torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = self._old
            self._old = None
        return False


class UPLiFT(nn.Module):
    """Iterative feature upsampler (uplift/uplift.py:537-709).  Each
    iteration: encoder (once with enc_share) -> decoder -> guide -> fused
    Local Attender (value = previous features) -> optional refiner.

    `allow_tf32` (not in the reference, which leaves PyTorch's global
    switches alone): None keeps the global settings (PyTorch's default lets
    cuDNN convolutions round fp32 operands to TF32); False runs every
    forward with TF32 off -- the fp32-exact mode the fp32 parity
    requirement (1e-4) needs -- and True with TF32 on; either way the global
    switches are restored after the call."""

    def __init__(self, in_channels, patch_size, cfg, dtype: torch.dtype = torch.float32, low_mem=False,
                 allow_tf32: Optional[bool] = None):
        super().__init__()
        self.allow_tf32 = allow_tf32
        self.in_channels = in_channels
        self.patch_size = patch_size
        self.cfg = cfg
        self.up_factor = cfg.up_factor
        self.target_dtype = dtype
        self.low_mem = low_mem
        self.using_attender = hasattr(cfg, "attender") and cfg.attender != -1
        self.encoder = UPLiFTEncoder(3, cfg.encoder)
        enc_channels = self.encoder.get_out_sizes()
        self.decoder = UPLiFTDecoder(in_channels, in_channels, cfg.decoder, enc_channels,
                                     using_attender=self.using_attender)
        self.attender = None
        if self.using_attender:
            self.attender = LocalAttender(self.decoder.out_channels, cfg.attender, low_mem=low_mem)
        self.enc_share = getattr(cfg, "enc_share", False)
        self.refiner = None
        if hasattr(cfg, "refiner"):
            self.ref_ncat_c = cfg.refiner.ncat_c
            self.ref_ncat_s = cfg.refiner.ncat_s
            self.ref_enc_resample = cfg.refiner.enc_resample
            self.ref_con = getattr(cfg.refiner, "ref_con", -1 - cfg.decoder.up_steps)
            ref_ic = in_channels + cfg.refiner.ncat_c + enc_channels[self.ref_con]
            self.refiner = BlockGroup(ref_ic, cfg.refiner.block_0)
            self.ref_outc = nn.Conv2d(cfg.refiner.block_0.hc[-1], in_channels, kernel_size=1)
        self.iters = 1
        self.return_all_steps = False
        self._apply_dtype()

    def enable_iterative(self, iters):
        assert iters > 0
        self.iters = iters

    def return_steps(self, setting):
        self.return_all_steps = setting

    def encode(self, img):
        if self.patch_size == 14:  # ViT patch-14 pre-scale to a multiple of 16
            img = TVF.resize(img, [(img.shape[2] * 16) // 14, (img.shape[3] * 16) // 14])
        return self.encoder(img)

    def upsample(self, img, x, cur_iter=0, ex_feats=None):
        x_in = x
        enc_feats = ex_feats if (self.enc_share and ex_feats is not None) else self.encode(img)
        x = self.decoder(x, enc_feats)
        if self.attender is not None:
            x = self.attender(x, x_in)
        if self.refiner is not None:
            x = noise_and_combine(x, enc_feats[self.ref_con], self.ref_ncat_c, self.ref_ncat_s,
                                  self.ref_enc_resample)
            x = self.ref_outc(self.refiner(x))
        return x, enc_feats

    def forward(self, img, x, outsize=None):
        with tf32_mode(self.allow_tf32):
            return self._forward(img, x, outsize)

    def _forward(self, img, x, outsize=None):
        steps = []
        ex_feats = None
        for i in range(self.iters):
            img_i = resize_sf(img, self.up_factor ** i) if (i > 0 and not self.enc_share) else img
            x, ex_feats = self.upsample(img_i, x, i, ex_feats)
            steps.append(x)
        if outsize is not None:
            return TVF.resize(x, outsize, interpolation=transforms.InterpolationMode.BILINEAR)
        if self.return_all_steps:
            return steps
        return x

    def _apply_dtype(self):
        for module in self.modules():
            for p in module.parameters(recurse=False):
                p.data = p.data.to(self.target_dtype)
            for name, buf in module._buffers.items():
                if buf is not None:
                    module._buffers[name] = buf.to(self.target_dtype)

    def compiled(self, backend: str, mode: str, fullgraph: bool, dynamic: bool,
                 device="cuda", set_tf32: bool = True, warmup: Callable | None = None) -> nn.Module:
        """torch.compile the whole module (uplift/uplift.py:656-709); the
        attender is a registered custom op, so it stays in the graph."""
        if device is not None:
            super().to(device)
        self._apply_dtype()
        self.eval()
        if set_tf32 and torch.cuda.is_available():
            torch.backends.cuda.matmul.allow_tf32 = True
            torch.backends.cudnn.allow_tf32 = True
        comp = torch.compile(self, backend=backend, mode=mode, fullgraph=fullgraph, dynamic=dynamic)
        if warmup is not None:
            with torch.inference_mode():
                args, kwargs = warmup()
                comp(*args, **kwargs)
        return comp
