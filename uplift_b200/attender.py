"""Drop-in Local Attender modules backed by the sm_100a kernels.

`LocalAttender` keeps the constructor, attributes, parameter names and
forward signature of the reference module (uplift/uplift.py:740-847), so
state_dicts and callers work unchanged.  Its forward is one fused kernel
launch; the reference's K-fold neighbour stack and [B,C,K,H,I,W,I] product
are never materialised, which also makes `low_mem` a no-op for memory.

`FusedLocalAttender` is the counterpart of the reference's Triton module
(uplift/kernels/triton_attender.py:317-400): forward(att, x, hardmax) on
pre-projected logits, for every K in {5, 9, 13, 17, 25} and any integer I.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from . import ops

# (offsets, pn) per neighbourhood size.  The offsets and their order define
# the logit channel order, so they are the reference's tables
# (uplift/uplift.py:746-760), written out here as data.
NEIGHBOURHOODS: dict[int, tuple[tuple[tuple[int, int], ...], int]] = {
    5: (((-1, 0), (0, -1), (0, 0), (0, 1), (1, 0)), 1),
    9: (tuple((dy, dx) for dy in (-1, 0, 1) for dx in (-1, 0, 1)), 1),
    13: (((-2, 0), (-1, -1), (-1, 0), (-1, 1), (0, -2), (0, -1), (0, 0), (0, 1), (0, 2),
          (1, -1), (1, 0), (1, 1), (2, 0)), 2),
    17: (((-2, -2), (-2, 0), (-2, 2), (-1, -1), (-1, 0), (-1, 1), (0, -2), (0, -1), (0, 0),
          (0, 1), (0, 2), (1, -1), (1, 0), (1, 1), (2, -2), (2, 0), (2, 2)), 2),
    25: (tuple((dy, dx) for dy in (-2, -1, 0, 1, 2) for dx in (-2, -1, 0, 1, 2)), 2),
}


def neighbourhood(num_connected: int):
    try:
        offsets, pn = NEIGHBOURHOODS[num_connected]
    except KeyError:
        raise ValueError(f"LocalAttender: invalid num_connected {num_connected} "
                         f"(supported: {sorted(NEIGHBOURHOODS)})") from None
    return [tuple(o) for o in offsets], pn


def _fp32_projection(owner, conv1, K):
    """conv1's weight [K, Cg] and bias [K] in fp32 for the kernel, converted
    once and cached on `owner` until the parameters change (checked by data
    pointer and version counter); under torch.compile the raw parameters are
    passed and converted inside the op."""
    w, b = conv1.weight, conv1.bias
    if torch.compiler.is_compiling():
        return w, b
    key = (w.data_ptr(), w._version, w.dtype, w.device, None if b is None else (b.data_ptr(), b._version))
    if key != owner._proj_key:
        wf = w.detach().to(torch.float32).reshape(K, -1).contiguous()
        bf = None if b is None else b.detach().to(torch.float32).contiguous()
        owner._proj = (wf, bf)
        owner._proj_key = key
    return owner._proj


class LocalAttender(nn.Module):
    """Local-attention pooling of a coarse value map guided by a fine guide map.

    guide [B, Cg, I*H, I*W] and value [B, C, H, W] -> [B, C, I*H, I*W].
    Same settings as the reference (uplift/uplift.py:724-728): in_channels =
    Cg, num_connected = K, conv_res = residual on the 1x1 conv, low_mem
    (accepted; the fused kernel never needs the extra memory).

    Differences from the reference, by design: an invalid num_connected
    raises ValueError instead of exiting the process; the output has the
    value dtype in low_mem mode too (the reference returns fp32 there,
    uplift/uplift.py:840); the output is channels_last; tensors must be on
    an sm_100 CUDA device.
    """

    def __init__(self, in_channels, num_connected=5, conv_res=True, low_mem=False):
        super().__init__()
        self.in_channels = in_channels
        self.num_connected = num_connected
        offsets, pn = neighbourhood(num_connected)
        self.offsets = offsets
        self.pn = pn
        self.conv1 = nn.Conv2d(in_channels, num_connected, kernel_size=1)
        self.conv_res = conv_res
        self.pad = nn.ReplicationPad2d(self.pn)
        self.low_mem = low_mem
        self._proj_key = None
        self._proj = None

    def show_offsets(self):
        """Print the offset pattern on a (3+2pn)^2 grid (uplift/uplift.py:774-781)."""
        k = 3 + 2 * self.pn
        c = self.pn + 1
        vis = np.zeros([k, k])
        for dy, dx in self.offsets:
            vis[c + dy, c + dx] = 1
        print(vis)

    def make_offsets(self, x):
        """[B, C, H, W] -> [B, C, K, H, W] stack of replicate-padded shifts
        (the reference's helper, uplift/uplift.py:784-798; not used by forward)."""
        H, W = x.shape[2], x.shape[3]
        xp = self.pad(x)
        views = [xp[:, :, self.pn + dy:self.pn + dy + H, self.pn + dx:self.pn + dx + W]
                 for dy, dx in self.offsets]
        return torch.stack(views, dim=2)

    def _projection(self):
        return _fp32_projection(self, self.conv1, self.num_connected)

    def forward(self, guide, value, hardmax=False):
        if torch.is_grad_enabled() and (guide.requires_grad or value.requires_grad
                                        or self.conv1.weight.requires_grad):
            # training: the live parameters, so autograd reaches conv1
            w, b = self.conv1.weight, self.conv1.bias
        else:
            w, b = self._projection()
        return ops.local_attender(guide, value, w, b, self.offsets, self.pn,
                                  conv_res=self.conv_res, hardmax=hardmax)


class FusedLocalAttender(nn.Module):
    """Softmax (or hardmax) pooling from pre-projected logits.

    forward(att [B, K, I*H, I*W], x [B, C, H, W], hardmax=False) ->
    [B, C, I*H, I*W]; the interface of the reference's fused Triton module
    (uplift/kernels/triton_attender.py:336), without its K=17 / I in {2, 4}
    restriction and without a PyTorch fallback.
    """

    def __init__(self, num_connected: int = 17):
        super().__init__()
        offsets, pn = neighbourhood(num_connected)
        self.num_connected = num_connected
        self.offsets = offsets
        self.pn = pn

    def forward(self, att, x, hardmax=False):
        return ops.attender_pool(att, x, self.offsets, self.pn, hardmax=hardmax)


class AttenderWrapper(nn.Module):
    """Fast-mode attender: the original conv1 (+ residual) fused with the
    pooling in one launch.  Same forward(guide, value, hardmax) as the
    reference's _TritonAttenderWrapper (uplift/fast.py:46-64), for any K."""

    def __init__(self, attender: LocalAttender):
        super().__init__()
        self.conv1 = attender.conv1
        self.conv_res = attender.conv_res
        self.num_connected = attender.num_connected
        self.offsets = attender.offsets
        self.pn = attender.pn
        self._proj_key = None
        self._proj = None

    def forward(self, guide, value, hardmax=False, size=None):
        """`size` (an addition to the reference's wrapper): the output also
        goes through the fast path's final bilinear resize to `size`
        (uplift/fast.py:218-220), fused into the attender launch where the
        tensor-core kernel allows it."""
        w, b = _fp32_projection(self, self.conv1, self.num_connected)
        if size is not None:
            return ops.local_attender_resized(guide, value, w, b, self.offsets, self.pn, size,
                                              conv_res=self.conv_res, hardmax=hardmax)
        return ops.local_attender(guide, value, w, b, self.offsets, self.pn,
                                  conv_res=self.conv_res, hardmax=hardmax)

    def forward_fused_guide(self, act, res, guide_conv, value, hardmax=False, size=None):
        """forward(guide, value) for guide = guide_conv(act) + res[:, :Cg]
        -- the decoder's last residual block with its final 1x1 convolution
        (uplift/uplift.py:152-217) -- without storing the guide: the 1x1
        convolution and both residuals are folded into the attender's
        projection in the same launch (`size`: also the final resize)."""
        w, b = _fp32_projection(self, self.conv1, self.num_connected)
        return ops.local_attender_fused_guide(act, res, guide_conv.weight, guide_conv.bias, value, w, b,
                                              self.offsets, self.pn, conv_res=self.conv_res, hardmax=hardmax,
                                              size=size)
