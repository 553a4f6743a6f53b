"""The guide produced inside the attender launch
(uplift_la_forward_fused_guide): the decoder's last residual block ends in
a 1x1 convolution with bias, guide = w_guide . act + b_guide + res[:, :Cg]
(uplift/uplift.py:152-217, residual_auto :26-39), and the attender's
projection (+ residual) folds it in, so the guide is never stored.

Checked against the double-precision oracle of the unfused computation
(guide in fp64, then the attender), against the unfused GPU path (guide
rounded to bf16 by the 1x1 convolution, then the attender kernel), with the
fused final resize too, and end to end in make_fast."""
import pytest
import torch
import torch.nn.functional as F

from conftest import TOL, normwise_err
from oracle import c_oracle
from uplift_b200 import _native, ops
from uplift_b200.attender import neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
# the folded [K, 2 Cg] projection is rounded once to bf16 (the unfused path
# rounds the guide instead); measured against the fp64 oracle it stays
# within the tensor-core kernel's own bound
GF_TOL = 1e-2


def _case(B, H, W, C, K, dt, seed, res_channels=64):
    g = torch.Generator().manual_seed(seed)
    cl = torch.channels_last
    act = torch.relu(torch.randn(B, 64, 2 * H, 2 * W, generator=g)).to(dt)
    wide = torch.randn(B, res_channels, 2 * H, 2 * W, generator=g).to(dt)
    value = torch.randn(B, C, H, W, generator=g).to(dt)
    w_guide = (torch.randn(64, 64, generator=g) * 0.125).to(dt).float()
    b_guide = (torch.randn(64, generator=g) * 0.1).to(dt).float()
    weight = (torch.randn(K, 64, generator=g) * 0.3).to(dt).float()
    bias = torch.randn(K, generator=g) * 0.5
    return dict(act=act.to(DEV).contiguous(memory_format=cl), wide=wide.to(DEV).contiguous(memory_format=cl),
                value=value.to(DEV).contiguous(memory_format=cl), w_guide=w_guide.to(DEV),
                b_guide=b_guide.to(DEV), weight=weight.to(DEV), bias=bias.to(DEV), K=K)


def _oracle(c, conv_res=True, with_bias=True):
    """fp64 guide from the block's inputs, then the fp64 attender oracle."""
    act = c["act"].double().cpu()
    res = c["wide"][:, :64].double().cpu()
    guide = torch.einsum("oc,bchw->bohw", c["w_guide"].double().cpu(), act) + res
    if with_bias:
        guide = guide + c["b_guide"].double().cpu().view(1, -1, 1, 1)
    offsets, _ = neighbourhood(c["K"])
    return c_oracle.forward(guide.float(), c["value"].cpu(), c["weight"].cpu(), c["bias"].cpu(), offsets,
                            conv_res=conv_res)


def _fused(c, conv_res=True, with_bias=True, size=None, hardmax=False):
    offsets, pn = neighbourhood(c["K"])
    return ops.local_attender_fused_guide_raw(c["act"], c["wide"], c["w_guide"],
                                              c["b_guide"] if with_bias else None, c["value"], c["weight"],
                                              c["bias"], offsets, pn, conv_res, hardmax, size)


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
def test_fused_guide_vs_double_oracle(K, cuda_lib):
    # (B, H, W, C, residual channels): ragged tiles, residual as a slice of a
    # wider block input (the DINOv2 decoder's 192-channel concatenation)
    for i, (B, H, W, C, rc) in enumerate([(2, 6, 9, 128, 64), (1, 8, 16, 384, 192), (3, 5, 7, 64, 96)]):
        c = _case(B, H, W, C, K, torch.bfloat16, seed=20 * K + i, res_channels=rc)
        for conv_res, with_bias in ((True, True), (False, True), (True, False)):
            out = _fused(c, conv_res, with_bias)
            torch.cuda.synchronize()
            assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE_GUIDE
            err = normwise_err(out, _oracle(c, conv_res, with_bias))
            assert err <= GF_TOL <= TOL[torch.bfloat16], (K, B, H, W, C, rc, conv_res, with_bias, err)
    assert _native.device_status(clear=True) == 0


def test_fused_guide_vs_unfused_gpu_path(cuda_lib):
    """Against the path it replaces on the GPU: the 1x1 convolution (cuDNN),
    the conv epilogue (+ bias + residual, rounded to bf16) and the attender."""
    from uplift_b200 import glue
    c = _case(2, 16, 24, 384, 17, torch.bfloat16, seed=7, res_channels=192)
    offsets, pn = neighbourhood(17)
    y = F.conv2d(c["act"], c["w_guide"].to(torch.bfloat16).view(64, 64, 1, 1)).contiguous(
        memory_format=torch.channels_last)
    guide = glue.bias_act_(y, c["b_guide"].to(torch.bfloat16), False, c["wide"])
    exp = ops.local_attender_raw(guide, c["value"], c["weight"], c["bias"], offsets, pn)
    got = _fused(c)
    assert normwise_err(got, exp) <= TOL[torch.bfloat16]


def test_fused_guide_with_fused_resize(cuda_lib):
    c = _case(2, 8, 16, 192, 17, torch.bfloat16, seed=8, res_channels=192)
    out = _fused(c, size=(14, 28))
    torch.cuda.synchronize()
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE_GUIDE_RESIZE
    exp = F.interpolate(_oracle(c).double(), size=(14, 28), mode="bilinear", align_corners=False)
    assert out.shape == (2, 192, 14, 28)
    assert normwise_err(out, exp) <= GF_TOL


def test_fused_guide_falls_back_where_the_kernel_does_not_apply(cuda_lib):
    """fp32 (no tensor-core kernel for a 64-channel fp32 guide): the guide is
    built by the convolution + epilogue and the attender runs on it (the
    convolution with TF32 off, as the fp32-exact fast mode runs it)."""
    from uplift_b200.uplift import tf32_mode
    c = _case(1, 5, 6, 48, 17, torch.float32, seed=9)
    with tf32_mode(False):
        out = _fused(c)
    assert _native.last_kernel() in _native.KERNELS_CUDA_CORE
    assert normwise_err(out, _oracle(c)) <= TOL[torch.float32]


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_make_fast_produces_the_guide_inside_the_attender(dt, cuda_lib):
    """The fast-mode executor defers the decoder's last 1x1 convolution to
    the attender launch; with it off, the same executor stores the guide.
    bf16: equal within the bf16 requirement (different rounding points);
    fp32: the fused kernel does not apply, so the fallback runs the same ops
    as the unfused executor and the outputs are identical."""
    from uplift_b200 import uplift as U
    from uplift_b200.configs import get_config
    from uplift_b200.fast import make_fast
    cfg = get_config("dinov2-s14")
    torch.manual_seed(0)
    m = U.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, dtype=dt, allow_tf32=False).eval().to(DEV)
    m.enable_iterative(2)
    fast = make_fast(m, compile=False, device=torch.device(DEV))
    g = torch.Generator().manual_seed(4)
    img = torch.rand(2, 3, 224, 224, generator=g).to(DEV, dt)
    feats = torch.randn(2, 384, 16, 16, generator=g).to(DEV, dt)
    fused = fast(img, feats)
    kern = _native.last_kernel()
    fused_rs = fast(img, feats, (56, 56))
    kern_rs = _native.last_kernel()
    fast.fuse_guide = False
    plain = fast(img, feats)
    plain_rs = fast(img, feats, (56, 56))
    if dt == torch.bfloat16:
        assert kern == _native.KERNEL_TENSOR_CORE_GUIDE and kern_rs == _native.KERNEL_TENSOR_CORE_GUIDE_RESIZE
        assert normwise_err(fused, plain) <= TOL[dt] and normwise_err(fused_rs, plain_rs) <= TOL[dt]
    else:
        assert torch.equal(fused, plain) and torch.equal(fused_rs, plain_rs)
