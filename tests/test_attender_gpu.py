"""Parity of the sm_100a Local Attender kernels with the oracle and with the
reference's own outputs (golden vectors), through the C ABI."""
import pytest
import torch

from conftest import TOL, dtype_of, normwise_err
from oracle import c_oracle
from oracle import local_attender_oracle as lao
from uplift_b200 import _native, ops
from uplift_b200.attender import FusedLocalAttender, LocalAttender, neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _la_from_case(case):
    K, Cg = case["weight"].shape
    la = LocalAttender(Cg, K, conv_res=case["conv_res"], low_mem=case["low_mem"])
    with torch.no_grad():
        la.conv1.weight.copy_(case["weight"].float().view(K, Cg, 1, 1))
        la.conv1.bias.copy_(case["bias"].float())
    return la.to(DEV).to(case["guide"].dtype)


@pytest.mark.parametrize("layout", ["nchw", "channels_last"])
def test_golden_reference_cases(golden_cases, cuda_lib, layout):
    for case in golden_cases:
        dt = dtype_of(case["dtype"])
        fmt = torch.channels_last if layout == "channels_last" else torch.contiguous_format
        v = case["value"].to(DEV).contiguous(memory_format=fmt)
        if case["mode"] == "forward":
            la = _la_from_case(case)
            g = case["guide"].to(DEV).contiguous(memory_format=fmt)
            out = la(g, v)
        else:
            att = case["logits"].to(DEV).contiguous(memory_format=fmt)
            out = FusedLocalAttender(case["K"])(att, v, hardmax=case["hardmax"])
        ref = case["out"]
        assert out.shape == ref.shape, case["name"]
        assert out.dtype == dt, case["name"]
        err = normwise_err(out, ref)
        assert err <= TOL[dt], (case["name"], err)
        if case["hardmax"]:
            assert torch.equal(out.cpu().contiguous(), ref.to(dt)), case["name"]


def test_golden_against_double_oracle(golden_cases, cuda_lib):
    """Tighter check than the reference tolerance: the kernel computes in
    fp32 from the stored inputs, so against the double oracle only the final
    rounding to the storage type remains."""
    for case in golden_cases:
        if case["mode"] != "forward":
            continue
        dt = dtype_of(case["dtype"])
        la = _la_from_case(case)
        out = la(case["guide"].to(DEV), case["value"].to(DEV))
        exp = c_oracle.forward(case["guide"], case["value"], case["weight"], case["bias"],
                               case["offsets"], conv_res=case["conv_res"])
        tol = {torch.float32: 1e-5, torch.bfloat16: 4e-3, torch.float16: 5e-4}[dt]
        if _native.last_kernel() == _native.KERNEL_TENSOR_CORE_WIDE:
            tol = 3e-5  # two-term bf16 split of the fp32 projection (~2^-17 per product)
        assert normwise_err(out, exp) <= tol, (case["name"], normwise_err(out, exp))


def test_config1_standalone(golden_config1, cuda_lib):
    from golden.make_golden import config1_inputs
    guide, value, weight, bias = config1_inputs()
    offsets, pn = neighbourhood(9)
    out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV),
                                 offsets, pn).cpu()
    assert list(out.shape) == golden_config1["out_shape"]
    assert normwise_err(out[:, ::8], golden_config1["out_every8"]) <= TOL[torch.float32]
    assert abs(out.double().sum().item() - golden_config1["out_sum"]) <= 1e-5 * golden_config1["out_abs_sum"]


def _rand_case(K, I, dt, B, Cg, C, H, W, seed, conv_res=True, wscale=0.3):
    g = torch.Generator().manual_seed(seed)
    guide = torch.randn(B, Cg, I * H, I * W, generator=g).to(dt)
    value = torch.randn(B, C, H, W, generator=g).to(dt)
    weight = torch.randn(K, Cg, generator=g) * wscale
    bias = torch.randn(K, generator=g) * 0.5
    return guide, value, weight, bias


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
@pytest.mark.parametrize("I", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
def test_sweep_vs_double_oracle(K, I, dt, cuda_lib):
    offsets, pn = neighbourhood(K)
    for (B, Cg, C, H, W) in [(2, 32, 48, 7, 9), (1, 12, 20, 3, 2), (3, 8, 8, 1, 5)]:
        seed = K * 1000 + I * 10 + B
        guide, value, weight, bias = _rand_case(K, I, dt, B, Cg, C, H, W, seed, conv_res=True)
        for conv_res in (True, False):
            out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV),
                                         offsets, pn, conv_res=conv_res)
            exp = c_oracle.forward(guide, value, weight, bias, offsets, conv_res=conv_res)
            tol = {torch.float32: 1e-5, torch.bfloat16: 4e-3, torch.float16: 5e-4}[dt]
            assert normwise_err(out, exp) <= tol, (B, Cg, C, H, W, conv_res, normwise_err(out, exp))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_hardmax_selects_exact_neighbour(dt, cuda_lib):
    K, I = 17, 2
    offsets, pn = neighbourhood(K)
    guide, value, weight, bias = _rand_case(K, I, dt, 2, 16, 24, 6, 7, 99)
    out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV),
                                 offsets, pn, hardmax=True).cpu()
    exp = c_oracle.forward(guide, value, weight, bias, offsets, hardmax=True)
    assert torch.equal(out.contiguous(), exp.to(dt))


def test_strided_views_and_streams(cuda_lib):
    """Sliced channels_last views go through the stride path; a side stream
    is honoured."""
    K, I, dt = 17, 2, torch.bfloat16
    offsets, pn = neighbourhood(K)
    guide, value, weight, bias = _rand_case(K, I, dt, 2, 64, 40, 8, 6, 5)
    big_v = torch.zeros(2, 48, 10, 8, dtype=dt).contiguous(memory_format=torch.channels_last).to(DEV)
    big_v[:, 4:44, 1:9, 1:7] = value.to(DEV)
    v_view = big_v[:, 4:44, 1:9, 1:7]
    assert v_view.stride(1) == 1
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = ops.local_attender_raw(guide.to(DEV), v_view, weight.to(DEV), bias.to(DEV), offsets, pn)
    s.synchronize()
    exp = c_oracle.forward(guide, value, weight, bias, offsets)
    assert normwise_err(out, exp) <= 4e-3


def test_odd_channels_scalar_path(cuda_lib):
    for dt, C, Cg in [(torch.bfloat16, 3, 5), (torch.float32, 7, 3), (torch.float16, 9, 17)]:
        offsets, pn = neighbourhood(13)
        guide, value, weight, bias = _rand_case(13, 2, dt, 2, Cg, C, 5, 4, C)
        out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV),
                                     offsets, pn)
        exp = c_oracle.forward(guide, value, weight, bias, offsets)
        tol = {torch.float32: 1e-5, torch.bfloat16: 4e-3, torch.float16: 5e-4}[dt]
        assert normwise_err(out, exp) <= tol


def test_errors_are_raised(cuda_lib):
    la = LocalAttender(16, 9).to(DEV)
    with pytest.raises(ValueError, match="integer multiple"):
        la(torch.randn(1, 16, 5, 4, device=DEV), torch.randn(1, 3, 2, 2, device=DEV))
    with pytest.raises(ValueError, match="dtype"):
        la(torch.randn(1, 16, 4, 4, device=DEV), torch.randn(1, 3, 2, 2, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="CUDA"):
        la(torch.randn(1, 16, 4, 4, device=DEV), torch.randn(1, 3, 2, 2))


def test_empty_batch(cuda_lib):
    la = LocalAttender(16, 17).to(DEV)
    out = la(torch.randn(0, 16, 8, 8, device=DEV), torch.randn(0, 5, 4, 4, device=DEV))
    assert out.shape == (0, 5, 8, 8)


# ---------------------------------------------------------------- full size
DINO_LEVELS = [(32, 64), (64, 128), (128, 256), (256, 512)]  # coarse -> fine, 448 px iters=4


@pytest.mark.slow
def test_dinov2_iters4_shapes_full_size(cuda_lib):
    """The four attender calls of the DINOv2-S/14 448 px iters=4 upsampler at
    B=8, bf16 (K=17, Cg=64, C=384): size-independent properties on the full
    tensors, and the oracle on bands of rows."""
    K, dt, B = 17, torch.bfloat16, 8
    offsets, pn = neighbourhood(K)
    g = torch.Generator(device=DEV).manual_seed(0)
    weight = torch.randn(K, 64, device=DEV, generator=g) * 0.02
    bias = torch.zeros(K, device=DEV)
    for (h, ho) in DINO_LEVELS:
        value = torch.randn(B, 384, h, h, device=DEV, generator=g).to(dt).contiguous(memory_format=torch.channels_last)
        guide = torch.randn(B, 64, ho, ho, device=DEV, generator=g).to(dt).contiguous(memory_format=torch.channels_last)
        out = ops.local_attender_raw(guide, value, weight, bias, offsets, pn)
        assert out.shape == (B, 384, ho, ho) and out.is_contiguous(memory_format=torch.channels_last)
        assert torch.isfinite(out).all()
        # convex combination: each output lies within its neighbourhood's range
        vmax, vmin = value.float().amax(), value.float().amin()
        assert out.float().amax() <= vmax + 1e-2 and out.float().amin() >= vmin - 1e-2
        # constant value map -> constant output (weights sum to one)
        const = torch.full_like(value, 1.5)
        oc = ops.local_attender_raw(guide, const, weight, bias, offsets, pn)
        assert (oc.float() - 1.5).abs().max().item() <= 1e-2
        # linearity in the value map
        v2 = torch.randn(value.shape, device=DEV, generator=g).to(dt).contiguous(memory_format=torch.channels_last)
        o2 = ops.local_attender_raw(guide, v2, weight, bias, offsets, pn)
        osum = ops.local_attender_raw(guide, (value.float() + v2.float()).to(dt), weight, bias, offsets, pn)
        assert normwise_err(osum, out.float() + o2.float()) <= 2e-2
        # oracle on two bands of coarse rows of image 3 (top border and middle)
        for r0 in (0, h // 2):
            r1 = min(h, r0 + 4)
            lo, hi = max(0, r0 - pn), min(h, r1 + pn)
            v_c = value[3:4, :, lo:hi].float().cpu()
            g_c = guide[3:4, :, lo * 2:hi * 2].float().cpu()
            exp = c_oracle.forward(g_c, v_c, weight.cpu(), bias.cpu(), offsets)
            got = out[3:4, :, r0 * 2:r1 * 2].float().cpu()
            ref = exp[:, :, (r0 - lo) * 2:(r1 - lo) * 2]
            # 8e-3: AUTO runs the tensor-core kernel here, which rounds the
            # softmax weights to bf16 like the reference's bf16 path
            assert normwise_err(got, ref) <= 8e-3, (h, r0)
        del value, guide, out, oc, o2, osum, v2, const
    torch.cuda.empty_cache()


def test_sdvae_shape_fp32(cuda_lib):
    """SD1.5-VAE attender: Cg=512, C=4, K=17, fp32 (one 128->256 level, B=2)."""
    K = 17
    offsets, pn = neighbourhood(K)
    guide, value, weight, bias = _rand_case(K, 2, torch.float32, 2, 512, 4, 128, 128, 3, wscale=0.05)
    out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV), offsets, pn)
    exp = c_oracle.forward(guide, value, weight, bias, offsets)
    assert normwise_err(out, exp) <= TOL[torch.float32]


def test_torch_oracle_full_chunked_bf16(cuda_lib):
    """The reference-order bf16 oracle on a mid-size DINOv2 level (one image)."""
    K, dt = 17, torch.bfloat16
    offsets, pn = neighbourhood(K)
    guide, value, weight, bias = _rand_case(K, 2, dt, 1, 64, 384, 32, 32, 11, wscale=0.02)
    weight, bias = weight.to(dt), bias.to(dt)  # a bf16 model's conv1 parameters
    out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV), offsets, pn)
    exp = lao.local_attender_chunked(guide, value, weight, bias)
    assert normwise_err(out, exp) <= TOL[dt]
