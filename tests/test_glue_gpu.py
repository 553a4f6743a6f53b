"""The fast-mode glue kernels (include/uplift_glue.h) against the eager
PyTorch ops they replace: F.interpolate bilinear / nearest and
residual_auto (uplift/uplift.py:26-39)."""
import pytest
import torch
import torch.nn.functional as F

from uplift_b200 import glue
from uplift_b200.uplift import residual_auto

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def _rand(shape, dt, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dt).to(DEV).contiguous(memory_format=torch.channels_last)


def _ulp_close(a, b, dt):
    """Equal up to one rounding of the storage type (fp32 opmath may
    contract differently from torch's compiled kernel)."""
    a, b = a.float(), b.float()
    eps = {torch.float32: 2e-6, torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10}[dt]
    return bool(((a - b).abs() <= eps * b.abs().clamp_min(1.0)).all())


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("align", [False, True])
def test_bilinear_matches_interpolate(dt, align, cuda_lib):
    cases = [((2, 8, 7, 9), (13, 17)), ((1, 64, 37, 41), (20, 23)), ((2, 3, 146, 146), (167, 167)),
             ((1, 384, 73, 73), (64, 64)), ((2, 12, 1, 5), (4, 10)), ((1, 7, 5, 6), (5, 6))]
    for i, (shape, size) in enumerate(cases):
        x = _rand(shape, dt, seed=i)
        got = glue.resize_bilinear(x, size, align_corners=align)
        exp = F.interpolate(x, size=size, mode="bilinear", align_corners=align)
        assert got.shape == exp.shape and got.dtype == dt
        assert _ulp_close(got, exp, dt), (shape, size)


@pytest.mark.parametrize("dt", DTYPES)
def test_upsample_add_matches_block_residual(dt, cuda_lib):
    """UpBlock / TransposeConv residual: y + UpsamplingBilinear2d(x), fused."""
    x = _rand((2, 64, 19, 23), dt, seed=1)
    y = _rand((2, 64, 38, 46), dt, seed=2)
    exp = residual_auto(torch.nn.UpsamplingBilinear2d(scale_factor=2)(x), y)
    got = glue.upsample_add_(y.clone(), x, align_corners=True)
    assert _ulp_close(got, exp, dt)


@pytest.mark.parametrize("dt", DTYPES)
def test_nearest_into_slice_is_exact(dt, cuda_lib):
    f = _rand((2, 128, 64, 64), dt, seed=3)
    x = _rand((2, 96, 16, 16), dt, seed=4)
    buf = torch.empty((2, 96 + 128, 16, 16), dtype=dt, device=DEV, memory_format=torch.channels_last)
    glue.nearest_into_(buf[:, :96], x)
    glue.nearest_into_(buf[:, 96:], f)
    exp = torch.cat([x, F.interpolate(f, size=(16, 16), mode="nearest")], dim=1)
    assert torch.equal(buf, exp)
    for size in ((23, 17), (64, 64), (100, 128)):  # non-integer ratios, identity, upsampling
        out = torch.empty((2, 128) + size, dtype=dt, device=DEV).contiguous(memory_format=torch.channels_last)
        assert torch.equal(glue.nearest_into_(out, f), F.interpolate(f, size=size, mode="nearest"))


@pytest.mark.parametrize("dt", DTYPES)
def test_add_channels_is_residual_auto(dt, cuda_lib):
    for c1, c2 in ((64, 64), (512, 64), (3, 16), (5, 8)):  # equal, truncate, zero-pad, scalar path
        x1 = _rand((2, c1, 9, 11), dt, seed=c1)
        y = _rand((2, c2, 9, 11), dt, seed=c2 + 1)
        exp = residual_auto(x1, y)
        got = glue.add_channels_(y.clone(), x1)
        assert torch.equal(got, exp), (c1, c2)


def test_strided_views_and_nchw_inputs(cuda_lib):
    dt = torch.bfloat16
    big = _rand((2, 80, 30, 30), dt, seed=7)
    view = big[:, 8:72, 3:27, 2:28]  # channel slice with channels_last strides
    exp = F.interpolate(view.contiguous(), size=(48, 52), mode="bilinear", align_corners=False)
    assert _ulp_close(glue.resize_bilinear(view, (48, 52)), exp, dt)
    nchw = torch.randn(2, 16, 10, 12, device=DEV, dtype=dt)  # converted to channels_last
    assert _ulp_close(glue.resize_bilinear(nchw, (20, 24)), F.interpolate(nchw, size=(20, 24), mode="bilinear"), dt)


def test_final_resize_beyond_int32_elements(cuda_lib):
    """The fast path's final resize at 1022 px with 384 channels exceeds 2^31
    elements for B >= 5 (torch's NHWC kernel refuses it); 64-bit indexing
    here, checked image by image against F.interpolate."""
    dt = torch.bfloat16
    x = torch.empty((5, 384, 1168, 1168), dtype=dt, device=DEV, memory_format=torch.channels_last)
    x.normal_()
    out = glue.resize_bilinear(x, (1022, 1022))
    assert out.numel() < 2 ** 31 < x.numel()
    for b in (0, 4):
        exp = F.interpolate(x[b:b + 1], size=(1022, 1022), mode="bilinear", align_corners=False)
        assert _ulp_close(out[b:b + 1], exp, dt)
    del x, out
    torch.cuda.empty_cache()


def test_errors(cuda_lib):
    with pytest.raises(RuntimeError, match="CUDA"):
        glue.resize_bilinear(torch.randn(1, 4, 4, 4), (8, 8))
    a = _rand((1, 4, 4, 4), torch.float32, 0)
    with pytest.raises(ValueError):
        glue.add_channels_(a, _rand((1, 4, 5, 4), torch.float32, 1))


@pytest.mark.parametrize("dt", DTYPES)
def test_bias_act_is_conv_epilogue(dt, cuda_lib):
    """conv (no bias) -> + bias -> ReLU -> + residual_auto, in one pass, equal
    to the eager sequence of the conv with its bias."""
    g = torch.Generator().manual_seed(11)
    conv = torch.nn.Conv2d(24, 16, 3, padding=1).to(DEV).to(dt).to(memory_format=torch.channels_last)
    with torch.no_grad():
        for relu in (False, True):
            for c_res in (None, 16, 24, 8):  # no residual, equal, truncated, zero-padded
                x = _rand((2, 24, 13, 11), dt, seed=5)
                res = None if c_res is None else _rand((2, c_res, 13, 11), dt, seed=c_res)
                exp = conv(x)
                if relu:
                    exp = torch.relu(exp)
                if res is not None:
                    exp = residual_auto(res, exp)
                y = F.conv2d(x, conv.weight, None, 1, 1).contiguous(memory_format=torch.channels_last)
                got = glue.bias_act_(y, conv.bias, relu, res)
                assert torch.equal(got, exp), (relu, c_res)


def test_bias_act_partial_residual_vector(cuda_lib):
    """A 3-channel residual (the image, into the encoder's first block) with
    16-byte output vectors: the partial residual is read element-wise."""
    dt = torch.bfloat16
    y0 = _rand((2, 16, 33, 35), dt, seed=21)
    img = _rand((2, 3, 33, 35), dt, seed=22)
    bias = torch.randn(16, device=DEV).to(dt)
    exp = residual_auto(img, y0 + bias.view(1, -1, 1, 1))
    got = glue.bias_act_(y0.clone(), bias, False, img)
    assert torch.equal(got, exp)


@pytest.mark.parametrize("dt", DTYPES)
def test_layernorm_act_matches_module(dt, cuda_lib):
    """Conv (no bias) + fused bias / channels-first LayerNorm / ReLU against
    the eager Conv -> LayerNorm -> ReLU of the SD1.5-VAE blocks."""
    from uplift_b200.uplift import LayerNorm
    for cin, c in ((16, 512), (8, 64), (12, 24), (4, 3)):  # vector paths of several widths, scalar path
        conv = torch.nn.Conv2d(cin, c, 3, padding=1).to(DEV).to(dt).to(memory_format=torch.channels_last)
        ln = LayerNorm(c, eps=1e-6, data_format="channels_first").to(DEV).to(dt)
        with torch.no_grad():
            ln.weight.normal_()
            ln.bias.normal_()
            x = _rand((2, cin, 9, 13), dt, seed=c)
            for relu in (False, True):
                # reference: the same LayerNorm in fp32 on the rounded conv
                # output (eager fp16 / bf16 would round every intermediate;
                # the kernel computes in fp32 and rounds once)
                t = conv(x).float()
                mu = t.mean(1, keepdim=True)
                var = (t - mu).pow(2).mean(1, keepdim=True)
                exp = ln.weight.float()[:, None, None] * ((t - mu) / torch.sqrt(var + ln.eps)) \
                    + ln.bias.float()[:, None, None]
                if relu:
                    exp = torch.relu(exp)
                y = F.conv2d(x, conv.weight, None, 1, 1).contiguous(memory_format=torch.channels_last)
                got = glue.layernorm_act_(y, conv.bias, ln.weight, ln.bias, ln.eps, relu)
                tol = {torch.float32: 1e-5, torch.bfloat16: 2 ** -8, torch.float16: 2 ** -11}[dt]
                err = ((got.float() - exp).abs() / exp.abs().clamp_min(1.0)).max().item()
                assert err <= tol, (cin, c, relu, err)
