"""Parity of the CUDA-core kernel's staged-guide projection (guides of 128 or
more channels, 16-byte aligned rows: the SD1.5-VAE attender has Cg = 512)
with the double-precision oracle, through the C ABI."""
import pytest
import torch

from conftest import TOL, normwise_err
from oracle import c_oracle
from uplift_b200 import _native, ops
from uplift_b200.attender import neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
# fp32 compute from the stored inputs: only the final rounding differs
TIGHT = {torch.float32: 1e-5, torch.bfloat16: 4e-3, torch.float16: 5e-4}


def _case(K, I, dt, B, Cg, C, H, W, seed, wscale=0.05):
    g = torch.Generator().manual_seed(seed)
    guide = torch.randn(B, Cg, I * H, I * W, generator=g).to(dt)
    value = torch.randn(B, C, H, W, generator=g).to(dt)
    weight = torch.randn(K, Cg, generator=g) * wscale
    bias = torch.randn(K, generator=g) * 0.5
    return guide, value, weight, bias


def _run(guide, value, weight, bias, K, **kw):
    """CUDA-core policy: some of these fp32 shapes would otherwise take the
    wide-guide tensor-core kernel."""
    offsets, pn = neighbourhood(K)
    with _native.kernel_policy(_native.POLICY_SIMT):
        out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV), offsets, pn, **kw)
        kernel = _native.last_kernel()
    return out, kernel


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
def test_staged_sweep_vs_double_oracle(K, dt, cuda_lib):
    # Cg 136 / 520 end in a partial 128-byte chunk; C 12 is vectorised, 7 is not
    for (I, B, Cg, C, H, W) in [(2, 2, 128, 12, 7, 9), (1, 1, 136, 7, 5, 4), (3, 1, 520, 12, 3, 5),
                                (2, 3, 136, 20, 13, 13)]:
        guide, value, weight, bias = _case(K, I, dt, B, Cg, C, H, W, seed=K * 100 + Cg + I)
        offsets, _ = neighbourhood(K)
        for conv_res in (True, False):
            out, kernel = _run(guide, value, weight, bias, K, conv_res=conv_res)
            assert kernel == _native.KERNEL_SIMT_STAGED
            exp = c_oracle.forward(guide, value, weight, bias, offsets, conv_res=conv_res)
            err = normwise_err(out, exp)
            assert err <= TIGHT[dt], (I, B, Cg, C, H, W, conv_res, err)


def test_staged_sdvae_level_fp32(cuda_lib):
    """SD1.5-VAE attender level (Cg=512, C=4, K=17, fp32, 64->128, B=4):
    the reference tolerance and the tight bound."""
    K = 17
    guide, value, weight, bias = _case(K, 2, torch.float32, 4, 512, 4, 64, 64, seed=7, wscale=0.02)
    out, kernel = _run(guide, value, weight, bias, K)
    assert kernel == _native.KERNEL_SIMT_STAGED
    exp = c_oracle.forward(guide, value, weight, bias, neighbourhood(K)[0])
    assert normwise_err(out, exp) <= TIGHT[torch.float32] <= TOL[torch.float32]


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_staged_hardmax_exact(dt, cuda_lib):
    K = 17
    guide, value, weight, bias = _case(K, 2, dt, 2, 256, 24, 6, 7, seed=5, wscale=0.3)
    out, kernel = _run(guide, value, weight, bias, K, hardmax=True)
    assert kernel == _native.KERNEL_SIMT_STAGED
    exp = c_oracle.forward(guide, value, weight, bias, neighbourhood(K)[0], hardmax=True)
    assert torch.equal(out.cpu().contiguous(), exp.to(dt))


def test_staged_guide_views(cuda_lib):
    """An aligned channel slice of a wider guide stays on the staged path;
    a slice that breaks 16-byte row alignment takes the per-pixel path; both
    match the oracle."""
    K, dt = 13, torch.float32
    guide, value, weight, bias = _case(K, 2, dt, 2, 160, 16, 6, 5, seed=3)
    offsets, _ = neighbourhood(K)
    exp = c_oracle.forward(guide, value, weight, bias, offsets)
    for start, expect in ((8, _native.KERNEL_SIMT_STAGED), (1, _native.KERNEL_SIMT)):
        big = torch.zeros(2, 172, 12, 10, dtype=dt).contiguous(memory_format=torch.channels_last).to(DEV)
        big[:, start:start + 160] = guide.to(DEV)
        view = big[:, start:start + 160]
        assert view.stride(1) == 1
        out, kernel = _run(view, value, weight, bias, K)
        assert kernel == expect, start
        assert normwise_err(out, exp) <= TIGHT[dt], start


def test_narrow_guide_stays_unstaged(cuda_lib):
    guide, value, weight, bias = _case(9, 2, torch.float32, 1, 64, 32, 4, 4, seed=1)
    _, kernel = _run(guide, value, weight, bias, 9)
    assert kernel == _native.KERNEL_SIMT
