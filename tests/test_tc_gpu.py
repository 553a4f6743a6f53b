"""Parity of the tensor-core (tcgen05 / TMEM / TMA) Local Attender kernel
with the double-precision oracle and with the CUDA-core kernel."""
import pytest
import torch

from conftest import TOL, normwise_err
from oracle import c_oracle
from uplift_b200 import _native, ops
from uplift_b200.attender import LocalAttender, neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(B, H, W, C, K, dt, seed, Cg=64):
    g = torch.Generator().manual_seed(seed)
    guide = torch.randn(B, Cg, 2 * H, 2 * W, generator=g).to(dt)
    value = torch.randn(B, C, H, W, generator=g).to(dt)
    # a bf16 / fp16 model's conv1 weights are stored in that type
    weight = (torch.randn(K, Cg, generator=g) * 0.3).to(dt).float()
    bias = torch.randn(K, generator=g) * 0.5
    return guide, value, weight, bias


def _run(policy, guide, value, weight, bias, K, **kw):
    offsets, pn = neighbourhood(K)
    with _native.kernel_policy(policy):
        out = ops.local_attender_raw(guide.to(DEV), value.to(DEV), weight.to(DEV), bias.to(DEV),
                                     offsets, pn, **kw)
        torch.cuda.synchronize()
        kernel = _native.last_kernel()
    return out, kernel


# the tensor-core path rounds the softmax weights to the storage type (as
# the reference's bf16 path does); against the fp64 oracle that costs at most
# about one storage ulp of the weights
TC_TOL = {torch.bfloat16: 8e-3, torch.float16: 1.5e-3}


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_tc_vs_double_oracle(K, dt, cuda_lib):
    shapes = [(1, 4, 8, 64), (2, 5, 9, 128), (1, 1, 1, 64), (3, 3, 17, 64), (1, 12, 7, 384), (2, 2, 3, 192)]
    for i, (B, H, W, C) in enumerate(shapes):
        guide, value, weight, bias = _inputs(B, H, W, C, K, dt, seed=100 * K + i)
        offsets, _ = neighbourhood(K)
        for conv_res in (True, False):
            out, kernel = _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, K, conv_res=conv_res)
            assert kernel == _native.KERNEL_TENSOR_CORE
            exp = c_oracle.forward(guide, value, weight, bias, offsets, conv_res=conv_res)
            err = normwise_err(out, exp)
            assert err <= TC_TOL[dt], (B, H, W, C, conv_res, err)
    assert _native.device_status(clear=True) == 0


def test_tc_hardmax_exact(cuda_lib):
    guide, value, weight, bias = _inputs(2, 6, 10, 64, 17, torch.bfloat16, seed=3)
    out, kernel = _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, 17, hardmax=True)
    assert kernel == _native.KERNEL_TENSOR_CORE
    offsets, _ = neighbourhood(17)
    exp = c_oracle.forward(guide, value, weight, bias, offsets, hardmax=True)
    assert torch.equal(out.cpu().contiguous(), exp.to(torch.bfloat16))


def test_tc_matches_simt_and_reference_tolerance(golden_cases, cuda_lib):
    """Golden reference cases eligible for the tensor-core path, both kernels."""
    n = 0
    for case in golden_cases:
        if case["mode"] != "forward" or case["dtype"] != "torch.bfloat16" or case["I"] != 2:
            continue
        K, Cg = case["weight"].shape
        if Cg != 64 or case["value"].shape[1] % 64 != 0:
            continue
        la = LocalAttender(Cg, K, conv_res=case["conv_res"])
        with torch.no_grad():
            la.conv1.weight.copy_(case["weight"].float().view(K, Cg, 1, 1))
            la.conv1.bias.copy_(case["bias"].float())
        la = la.to(DEV).to(torch.bfloat16)
        with _native.kernel_policy(_native.POLICY_TENSOR_CORE):
            out = la(case["guide"].to(DEV), case["value"].to(DEV))
        assert normwise_err(out, case["out"]) <= TOL[torch.bfloat16], case["name"]
        n += 1
    assert n >= 0


def test_tc_selected_for_dinov2_shapes(cuda_lib):
    """AUTO uses the tensor-core kernel for the DINOv2-S/14 attender shape."""
    la = LocalAttender(64, 17).to(DEV).to(torch.bfloat16)
    out = la(torch.randn(2, 64, 64, 64, device=DEV, dtype=torch.bfloat16),
             torch.randn(2, 384, 32, 32, device=DEV, dtype=torch.bfloat16))
    torch.cuda.synchronize()
    assert out.shape == (2, 384, 64, 64)
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE


def test_tc_full_size_vs_simt(cuda_lib):
    """Last DINOv2 level at B=8 (value 384x256^2 -> 512^2): both kernels agree
    and the oracle agrees on a band of rows."""
    guide, value, weight, bias = _inputs(8, 256, 256, 384, 17, torch.bfloat16, seed=9)
    tc, k1 = _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, 17)
    simt, k2 = _run(_native.POLICY_SIMT, guide, value, weight, bias, 17)
    assert k1 == _native.KERNEL_TENSOR_CORE and k2 in _native.KERNELS_CUDA_CORE
    assert normwise_err(tc, simt.float()) <= 1e-2
    offsets, pn = neighbourhood(17)
    for b, r0 in ((5, 0), (2, 120), (7, 252)):
        r1 = min(256, r0 + 4)
        lo, hi = max(0, r0 - pn), min(256, r1 + pn)
        exp = c_oracle.forward(guide[b:b + 1, :, 2 * lo:2 * hi], value[b:b + 1, :, lo:hi], weight, bias, offsets)
        got = tc[b:b + 1, :, 2 * r0:2 * r1].float().cpu()
        assert normwise_err(got, exp[:, :, 2 * (r0 - lo):2 * (r1 - lo)]) <= TC_TOL[torch.bfloat16]
    assert _native.device_status(clear=True) == 0


def test_policy_errors(cuda_lib):
    guide, value, weight, bias = _inputs(1, 4, 4, 48, 17, torch.bfloat16, seed=1)  # C=48: ineligible
    with pytest.raises(ValueError, match="tensor-core kernel required"):
        _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, 17)
    out, kernel = _run(_native.POLICY_AUTO, guide, value, weight, bias, 17)
    assert kernel in _native.KERNELS_CUDA_CORE


def test_cta_limit_leaves_results_unchanged(cuda_lib):
    """uplift_la_set_max_ctas caps the persistent kernels' grid (for running
    communication kernels beside them): every tile is computed the same way
    by whichever CTA takes it, so the forward and the backward are bitwise
    identical under a cap of 37 CTAs."""
    guide, value, weight, bias = _inputs(2, 20, 36, 384, 17, torch.bfloat16, seed=31)
    offsets, pn = neighbourhood(17)
    cl = torch.channels_last
    g, v = guide.to(DEV).contiguous(memory_format=cl), value.to(DEV).contiguous(memory_format=cl)
    dout = torch.randn(2, 384, 40, 72, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    dout = dout.to(DEV).contiguous(memory_format=cl)

    def run():
        out = ops.local_attender_raw(g, v, weight.to(DEV), bias.to(DEV), offsets, pn)
        dg, dv, dw, db = ops.local_attender_backward_raw(dout, g, v, weight.to(DEV), bias.to(DEV), offsets, pn)
        torch.cuda.synchronize()
        return out, dg, dv
    full = run()
    try:
        _native.set_max_ctas(37)
        capped = run()
    finally:
        _native.set_max_ctas(0)
    for a, b in zip(full, capped):
        assert torch.equal(a, b)


def test_expired_wait_is_reported_and_context_survives(cuda_lib):
    """Failure detection without a GPU fault: the test hook makes the guide
    producer issue no loads, so the consumers' bounded waits (limited to
    20 ms here) run out.  The kernel must record the role in the device
    status word, drain and exit; the context must stay usable."""
    lib = _native.load()
    guide, value, weight, bias = _inputs(1, 8, 16, 64, 17, torch.bfloat16, seed=21)
    offsets, _ = neighbourhood(17)
    assert _native.device_status(clear=True) == 0
    _native.check(lib.uplift_la_test_hook(1, 20_000_000), "test hook")
    try:
        _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, 17)  # synchronises
        status = _native.device_status(clear=True)
        host_word = _native.host_status.value()
        _native.host_status.clear()  # this test reads the device copy itself
    finally:
        lib.uplift_la_test_hook(0, 0)
    assert status in (1, 2, 3, 4), status
    assert host_word in (1, 2, 3, 4), host_word
    out, kernel = _run(_native.POLICY_TENSOR_CORE, guide, value, weight, bias, 17)
    exp = c_oracle.forward(guide, value, weight, bias, offsets)
    assert normwise_err(out, exp) <= TC_TOL[torch.bfloat16]
    assert _native.device_status(clear=True) == 0


def test_expired_wait_reaches_python_through_the_module(cuda_lib):
    """The product path surfaces an expired wait by itself: the launch that
    gave up writes the host-visible status word, and the module's next call
    raises ExpiredWaitError (no device_status() call by the user); the call
    after that runs normally and is correct."""
    lib = _native.load()
    guide, value, weight, bias = _inputs(1, 8, 16, 64, 17, torch.bfloat16, seed=22)
    torch.manual_seed(0)
    la = LocalAttender(64, 17).to(DEV).to(torch.bfloat16)
    with torch.no_grad():
        la.conv1.weight.copy_(weight.reshape(17, 64, 1, 1))
        la.conv1.bias.copy_(bias)
    g, v = guide.to(DEV), value.to(DEV)
    with torch.no_grad():
        la(g, v)  # registers the host status word
        torch.cuda.synchronize()
        _native.check(lib.uplift_la_test_hook(1, 20_000_000), "test hook")
        try:
            la(g, v)
            torch.cuda.synchronize()
        finally:
            lib.uplift_la_test_hook(0, 0)
        with pytest.raises(_native.ExpiredWaitError):
            la(g, v)
        out = la(g, v)
        torch.cuda.synchronize()
    offsets, _ = neighbourhood(17)
    exp = c_oracle.forward(guide, value, la.conv1.weight.detach().float().reshape(17, 64).cpu(),
                           la.conv1.bias.detach().float().cpu(), offsets)
    assert normwise_err(out, exp) <= TC_TOL[torch.bfloat16]
    assert _native.host_status.value() == 0
    assert _native.device_status(clear=True) == 0
