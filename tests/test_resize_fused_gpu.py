"""The Local Attender with the fast path's final resize fused into its launch
(uplift_la_forward_resized): the attender output followed by
F.interpolate(size, mode="bilinear", align_corners=False) of
_OptimizedUPLiFT's last step (uplift/fast.py:218-220), for output sizes
7/8 of the attender output (1168 -> 1022 and 512 -> 448 in the DINOv2
upsampler).  Checked against the same two steps run separately (equal up
to one rounding of the storage type: the fp32 contraction order of the
interpolation may differ), against torch's own F.interpolate of the
unfused output, and against the double-precision oracle."""
import pytest
import torch
import torch.nn.functional as F

from conftest import TOL, normwise_err
from oracle import c_oracle
from uplift_b200 import _native, ops
from uplift_b200.attender import AttenderWrapper, LocalAttender, neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ULP = {torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10}


def _ulp_close(a, b, dt):
    """Equal up to one rounding of the storage type (values below 1 in
    absolute terms)."""
    a, b = a.float(), b.float()
    return bool(((a - b).abs() <= ULP[dt] * b.abs().clamp_min(1.0)).all())


def _inputs(B, H, W, C, K, dt, seed, Cg=64):
    g = torch.Generator().manual_seed(seed)
    guide = torch.randn(B, Cg, 2 * H, 2 * W, generator=g).to(dt)
    value = torch.randn(B, C, H, W, generator=g).to(dt)
    weight = (torch.randn(K, Cg, generator=g) * 0.3).to(dt).float()
    bias = torch.randn(K, generator=g) * 0.5
    cl = torch.channels_last
    return (guide.to(DEV).contiguous(memory_format=cl), value.to(DEV).contiguous(memory_format=cl),
            weight.to(DEV), bias.to(DEV))


def _size(H, W):
    return (2 * H * 7) // 8, (2 * W * 7) // 8


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
def test_fused_resize_equals_two_steps(K, dt, cuda_lib):
    # (B, H, W, C): several tiles, one tile, one or several 64-channel chunks
    for i, (B, H, W, C) in enumerate([(2, 8, 16, 64), (1, 4, 8, 384), (3, 12, 24, 192), (1, 16, 8, 128)]):
        guide, value, w, b = _inputs(B, H, W, C, K, dt, seed=10 * K + i)
        offsets, pn = neighbourhood(K)
        size = _size(H, W)
        for conv_res, hardmax in ((True, False), (False, False), (True, True)):
            fused = ops.local_attender_resized_raw(guide, value, w, b, offsets, pn, size, conv_res, hardmax)
            torch.cuda.synchronize()
            assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE_RESIZE
            y = ops.local_attender_raw(guide, value, w, b, offsets, pn, conv_res, hardmax)
            exp = F.interpolate(y, size=size, mode="bilinear", align_corners=False)
            assert fused.shape == exp.shape == (B, C) + size and fused.dtype == dt
            assert fused.is_contiguous(memory_format=torch.channels_last)
            assert _ulp_close(fused, exp, dt), (B, H, W, C, conv_res, hardmax)
    assert _native.device_status(clear=True) == 0


def test_fused_resize_vs_double_oracle(cuda_lib):
    """Against the fp64 oracle of the attender, interpolated in fp64: the
    bf16 requirement (2e-2 normwise) and the tensor-core kernel's own bound."""
    K, dt = 17, torch.bfloat16
    guide, value, w, b = _inputs(2, 8, 24, 128, K, dt, seed=3)
    offsets, pn = neighbourhood(K)
    size = _size(8, 24)
    fused = ops.local_attender_resized_raw(guide, value, w, b, offsets, pn, size)
    att = c_oracle.forward(guide.cpu(), value.cpu(), w.cpu(), b.cpu(), offsets).double()
    exp = F.interpolate(att, size=size, mode="bilinear", align_corners=False)
    err = normwise_err(fused, exp)
    assert err <= 8e-3 <= TOL[dt], err


def test_ineligible_sizes_fall_back_to_two_launches(cuda_lib):
    """Output sizes that are not 7/8 of the attender output, ragged tiles, or
    fp32 storage: the entry point returns UNSUPPORTED and launches nothing;
    the torch op then runs the attender and the resize kernel."""
    K = 17
    offsets, pn = neighbourhood(K)
    for (H, W, C, dt, size) in [(8, 16, 64, torch.bfloat16, (20, 30)),    # not 7/8
                                (6, 16, 64, torch.bfloat16, (10, 28)),    # 12 rows: not whole tiles
                                (8, 16, 48, torch.bfloat16, (14, 28)),    # C not a multiple of 64
                                (8, 16, 64, torch.float32, (14, 28))]:    # fp32
        guide, value, w, b = _inputs(1, H, W, C, K, dt, seed=H + W + C)
        lib = _native.load()
        out = torch.empty((1, C) + size, dtype=dt, device=DEV, memory_format=torch.channels_last)
        rc = lib.uplift_la_forward_resized(
            guide.data_ptr(), _native.strides(guide), value.data_ptr(), _native.strides(value),
            w.data_ptr(), b.data_ptr(), out.data_ptr(), _native.strides(out), 1, 64, C, H, W, 2, K,
            _native.offsets_array(offsets), pn, 1, {torch.bfloat16: _native.BF16, torch.float32: _native.F32}[dt],
            0, size[0], size[1], None)
        assert rc == _native.ERR_UNSUPPORTED, lib.uplift_la_last_error().decode()
        got = ops.local_attender_resized_raw(guide, value, w, b, offsets, pn, size)
        y = ops.local_attender_raw(guide, value, w, b, offsets, pn)
        exp = F.interpolate(y, size=size, mode="bilinear", align_corners=False)
        assert torch.equal(got, exp) or normwise_err(got, exp) <= 1e-6 or \
            bool(((got.float() - exp.float()).abs() <= 2 ** -7 * exp.float().abs().clamp_min(1.0)).all())


def test_wrapper_and_custom_op(cuda_lib):
    """AttenderWrapper(size=...) and the traced custom op give the fused result."""
    torch.manual_seed(0)
    la = LocalAttender(64, 17).to(DEV).to(torch.bfloat16).eval()
    wrap = AttenderWrapper(la).eval()
    guide, value, _, _ = _inputs(2, 8, 16, 128, 17, torch.bfloat16, seed=9)
    with torch.no_grad():
        got = wrap(guide, value, size=(14, 28))
        exp = F.interpolate(la(guide, value), size=(14, 28), mode="bilinear", align_corners=False)
        compiled = torch.compile(lambda g, v: wrap(g * 1.0, v, size=(14, 28)), fullgraph=True)
        got_c = compiled(guide, value)
    assert _ulp_close(got, exp, torch.bfloat16)
    assert torch.equal(got_c, got)


def test_fast_mode_upsampler_uses_the_fused_resize(cuda_lib):
    """make_fast's last iteration applies the resize inside the attender
    launch when the output size allows it; the result equals the unfused
    executor followed by the resize."""
    from uplift_b200 import uplift as U
    from uplift_b200.configs import get_config
    from uplift_b200.fast import make_fast
    from uplift_b200 import glue
    cfg = get_config("dinov2-s14")
    torch.manual_seed(0)
    m = U.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, dtype=torch.bfloat16).eval().to(DEV)
    m.enable_iterative(2)
    fast = make_fast(m, compile=False, device=torch.device(DEV))
    g = torch.Generator().manual_seed(4)
    img = torch.rand(2, 3, 224, 224, generator=g).to(DEV, torch.bfloat16)
    feats = torch.randn(2, 384, 16, 16, generator=g).to(DEV, torch.bfloat16)
    full = fast(img, feats)                       # 64 x 64, no resize
    out = fast(img, feats, (56, 56))              # 64 -> 56 = 7/8: fused (with the guide fused too)
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE_GUIDE_RESIZE
    fast.fuse_guide = False
    assert _ulp_close(fast(img, feats, (56, 56)), glue.resize_bilinear(fast(img, feats), (56, 56)),
                      torch.bfloat16)
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE  # the plain call ran last
    fast.fuse_guide = True
    exp = glue.resize_bilinear(full, (56, 56))
    assert out.shape == (2, 384, 56, 56)
    assert _ulp_close(out, exp, torch.bfloat16)
    other = fast(img, feats, (60, 60))            # not 7/8: attender, then the resize kernel
    assert _ulp_close(other, glue.resize_bilinear(full, (60, 60)), torch.bfloat16)


def test_fused_resize_dinov2_1022_last_level(cuda_lib):
    """The last level of the 1022 px upsampler at full size (B=8, value
    384 x 584^2, attender output 1168^2 = 4.19 G elements, past 2^31,
    resized to 1022^2): the fused launch equals torch's F.interpolate of the
    unfused attender output, compared on the device."""
    K, dt = 17, torch.bfloat16
    B, H, W, C = 8, 584, 584, 384
    g = torch.Generator(device=DEV).manual_seed(11)
    cl = torch.channels_last
    guide = torch.randn(B, 64, 2 * H, 2 * W, generator=g, device=DEV).to(dt).contiguous(memory_format=cl)
    value = torch.randn(B, C, H, W, generator=g, device=DEV).to(dt).contiguous(memory_format=cl)
    w = (torch.randn(K, 64, generator=g, device=DEV) * 0.3).to(dt).float()
    b = torch.randn(K, generator=g, device=DEV) * 0.5
    offsets, pn = neighbourhood(K)
    fused = ops.local_attender_resized_raw(guide, value, w, b, offsets, pn, (1022, 1022))
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE_RESIZE
    y = ops.local_attender_raw(guide, value, w, b, offsets, pn)
    del guide
    bad = 0
    for i in range(B):  # per image: bounded temporaries, < 2^31 elements per interpolate
        e = F.interpolate(y[i:i + 1], size=(1022, 1022), mode="bilinear", align_corners=False).float()
        a = fused[i:i + 1].float()
        bad += int(((a - e).abs() > 2 ** -7 * e.abs().clamp_min(1.0)).sum())
    assert bad == 0
    assert _native.device_status(clear=True) == 0
