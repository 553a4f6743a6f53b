"""Parity of the tensor-core projection kernel for wide fp32 guides (two-term
bf16 split of guide and weights; the SD1.5-VAE attender has Cg = 512, C = 4)
with the double-precision oracle, through the C ABI."""
import pytest
import torch

from conftest import TOL, normwise_err
from oracle import c_oracle
from uplift_b200 import _native, ops
from uplift_b200.attender import LocalAttender, neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
# the split represents each operand to 2^-18 relative, each product to
# ~2^-17; logits and outputs land well inside the fp32 requirement (1e-4)
TIGHT = 3e-5


def _case(K, B, Cg, C, H, W, seed, wscale=0.05):
    g = torch.Generator().manual_seed(seed)
    guide = torch.randn(B, Cg, 2 * H, 2 * W, generator=g)
    value = torch.randn(B, C, H, W, generator=g)
    weight = torch.randn(K, Cg, generator=g) * wscale
    bias = torch.randn(K, generator=g) * 0.5
    return guide, value, weight, bias


def _run(policy, guide, value, weight, bias, K, **kw):
    offsets, pn = neighbourhood(K)
    with _native.kernel_policy(policy):
        out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV), offsets, pn, **kw)
        torch.cuda.synchronize()
        kernel = _native.last_kernel()
    return out, kernel


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
def test_tcw_vs_double_oracle(K, cuda_lib):
    # partial tiles (H, W not multiples of 4 / 8), 1x1 maps, several chunk counts
    shapes = [(1, 64, 4, 4, 8), (2, 96, 8, 5, 9), (1, 512, 4, 1, 1), (3, 128, 32, 3, 17), (1, 512, 12, 9, 11)]
    for i, (B, Cg, C, H, W) in enumerate(shapes):
        guide, value, weight, bias = _case(K, B, Cg, C, H, W, seed=100 * K + i)
        offsets, _ = neighbourhood(K)
        for conv_res in (True, False):
            out, kernel = _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, K, conv_res=conv_res)
            assert kernel == _native.KERNEL_TENSOR_CORE_WIDE
            exp = c_oracle.forward(guide, value, weight, bias, offsets, conv_res=conv_res)
            err = normwise_err(out, exp)
            assert err <= TIGHT, (B, Cg, C, H, W, conv_res, err)
    assert _native.device_status(clear=True) == 0


def test_tcw_sdvae_level(cuda_lib):
    """An SD1.5-VAE attender level (Cg=512, C=4, K=17, value 64x64 -> 128x128,
    B=4): the tensor-core result equals the CUDA-core kernel's and the oracle's."""
    K = 17
    guide, value, weight, bias = _case(K, 4, 512, 4, 64, 64, seed=7, wscale=0.02)
    tc, k1 = _run(_native.POLICY_AUTO, guide, value, weight, bias, K)
    simt, k2 = _run(_native.POLICY_SIMT, guide, value, weight, bias, K)
    assert k1 == _native.KERNEL_TENSOR_CORE_WIDE and k2 in _native.KERNELS_CUDA_CORE
    assert normwise_err(tc, simt) <= TIGHT
    print("tcw vs fp64 oracle:", normwise_err(tc, c_oracle.forward(guide, value, weight, bias, neighbourhood(K)[0])))
    exp = c_oracle.forward(guide, value, weight, bias, neighbourhood(K)[0])
    assert normwise_err(tc, exp) <= TIGHT <= TOL[torch.float32]


def test_tcw_hardmax_exact(cuda_lib):
    K = 17
    guide, value, weight, bias = _case(K, 2, 256, 8, 6, 10, seed=5, wscale=0.3)
    out, kernel = _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, K, hardmax=True)
    assert kernel == _native.KERNEL_TENSOR_CORE_WIDE
    exp = c_oracle.forward(guide, value, weight, bias, neighbourhood(K)[0], hardmax=True)
    assert torch.equal(out.cpu().contiguous(), exp)


def test_tcw_module_and_views(cuda_lib):
    """LocalAttender(512, 17) in fp32 on NCHW inputs and on sliced
    channels_last views of the value / output."""
    torch.manual_seed(0)
    la = LocalAttender(512, 17).to(DEV)
    guide, value, _, _ = _case(17, 2, 512, 8, 7, 9, seed=9)
    out = la(guide.to(DEV), value.to(DEV))
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE_WIDE
    w = la.conv1.weight.detach().cpu().view(17, 512)
    b = la.conv1.bias.detach().cpu()
    exp = c_oracle.forward(guide, value, w, b, neighbourhood(17)[0])
    assert normwise_err(out, exp) <= TIGHT
    big = torch.zeros(2, 16, 9, 11).contiguous(memory_format=torch.channels_last).to(DEV)
    big[:, 4:12, 1:8, 1:10] = value.to(DEV)
    view = big[:, 4:12, 1:8, 1:10]
    out2 = la(guide.to(DEV), view)
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE_WIDE
    assert normwise_err(out2, exp) <= TIGHT


def test_tcw_ineligible_shapes_fall_back(cuda_lib):
    guide, value, weight, bias = _case(17, 1, 512, 36, 4, 4, seed=1)  # C=36 > 32
    with pytest.raises(ValueError, match="tensor-core kernel required"):
        _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, 17)
    out, kernel = _run(_native.POLICY_AUTO, guide, value, weight, bias, 17)
    assert kernel in _native.KERNELS_CUDA_CORE
    exp = c_oracle.forward(guide, value, weight, bias, neighbourhood(17)[0])
    assert normwise_err(out, exp) <= TIGHT


def test_tcw_expired_wait_is_reported_and_context_survives(cuda_lib):
    """Failure detection without a GPU fault, as for the bf16 kernel: the
    test hook stops the guide producer, the split warps' bounded waits
    (20 ms) run out, the kernel records the role, drains and exits, and a
    normal launch in the same context is correct."""
    lib = _native.load()
    guide, value, weight, bias = _case(17, 1, 256, 4, 8, 16, seed=21)
    offsets, _ = neighbourhood(17)
    assert _native.device_status(clear=True) == 0
    _native.check(lib.uplift_la_test_hook(1, 20_000_000), "test hook")
    try:
        _, kernel = _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, 17)  # synchronises
        status = _native.device_status(clear=True)
        host_word = _native.host_status.value()
        _native.host_status.clear()  # this test reads the device copy itself
    finally:
        lib.uplift_la_test_hook(0, 0)
    assert kernel == _native.KERNEL_TENSOR_CORE_WIDE
    assert status in (1, 2, 3, 4), status
    assert host_word in (1, 2, 3, 4), host_word
    out, _ = _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, 17)
    exp = c_oracle.forward(guide, value, weight, bias, offsets)
    assert normwise_err(out, exp) <= TIGHT
    assert _native.device_status(clear=True) == 0
