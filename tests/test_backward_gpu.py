"""Backward of the fused Local Attender (uplift_la_backward through the
`uplift_b200::local_attender` custom op's autograd) against fp64 autograd
through the oracle, which restates the reference's differentiable module
(uplift/uplift.py:801-847)."""
import pytest
import torch

from conftest import normwise_err
from oracle import local_attender_oracle as lao
from uplift_b200 import ops
from uplift_b200.attender import LocalAttender, neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _case(K, I, B, Cg, C, H, W, seed, dt=torch.float32, wscale=0.3):
    g = torch.Generator().manual_seed(seed)
    guide = torch.randn(B, Cg, I * H, I * W, generator=g).to(dt)
    value = torch.randn(B, C, H, W, generator=g).to(dt)
    weight = (torch.randn(K, Cg, generator=g) * wscale).to(dt)
    bias = (torch.randn(K, generator=g) * 0.5).to(dt)
    gout = torch.randn(B, C, I * H, I * W, generator=g)
    return guide, value, weight, bias, gout


def _oracle_grads(guide, value, weight, bias, gout, K, conv_res, hardmax):
    offsets, pn = neighbourhood(K)
    ts = [t.double().requires_grad_() for t in (guide, value, weight, bias)]
    out = lao.local_attender(*ts, conv_res=conv_res, hardmax=hardmax, offsets=offsets, pn=pn)
    (out * gout.double()).sum().backward()
    return [t.grad for t in ts]


def _kernel_grads(guide, value, weight, bias, gout, K, conv_res, hardmax):
    offsets, pn = neighbourhood(K)
    ts = [t.to(DEV).requires_grad_() for t in (guide, value, weight, bias)]
    out = ops.local_attender(*ts, offsets, pn, conv_res=conv_res, hardmax=hardmax)
    (out.float() * gout.to(DEV)).sum().backward()
    return [t.grad.float().cpu() for t in ts]


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
def test_gradients_vs_fp64_autograd(K, cuda_lib):
    for (I, B, Cg, C, H, W) in [(2, 2, 16, 12, 5, 7), (1, 1, 24, 8, 6, 5), (3, 2, 8, 6, 3, 4), (2, 1, 32, 20, 1, 9)]:
        for conv_res in (True, False):
            case = _case(K, I, B, Cg, C, H, W, seed=K * 10 + I)
            exp = _oracle_grads(*case, K, conv_res, False)
            got = _kernel_grads(*case, K, conv_res, False)
            for name, e, g in zip(("guide", "value", "weight", "bias"), exp, got):
                err = normwise_err(g, e)
                assert err <= 1e-4, (K, I, B, Cg, C, H, W, conv_res, name, err)


def test_hardmax_gradient(cuda_lib):
    """argmax selection: no gradient into the logits (guide, weight, bias);
    the value gradient routes each output to its selected neighbour."""
    K = 17
    case = _case(K, 2, 2, 16, 12, 6, 7, seed=3)
    exp = _oracle_grads(*case, K, True, True)
    got = _kernel_grads(*case, K, True, True)
    assert normwise_err(got[1], exp[1]) <= 1e-5
    for g in (got[0], got[2], got[3]):
        assert float(g.abs().max()) == 0.0


def test_bf16_gradients(cuda_lib):
    K = 17
    case = _case(K, 2, 2, 64, 48, 6, 8, seed=9, dt=torch.bfloat16, wscale=0.05)
    exp = _oracle_grads(*case, K, True, False)
    got = _kernel_grads(*case, K, True, False)
    for name, e, g in zip(("guide", "value", "weight", "bias"), exp, got):
        assert normwise_err(g, e) <= 2e-2, name


def test_module_training_step(cuda_lib):
    """LocalAttender in a training step: autograd reaches conv1 through the
    fused kernel, and an SGD step matches the same step through the oracle."""
    torch.manual_seed(0)
    K, Cg, C = 17, 64, 32
    la = LocalAttender(Cg, K).to(DEV)
    ref_w = la.conv1.weight.detach().cpu().double().clone().requires_grad_()
    ref_b = la.conv1.bias.detach().cpu().double().clone().requires_grad_()
    g = torch.Generator().manual_seed(4)
    guide = torch.randn(2, Cg, 16, 20, generator=g)
    value = torch.randn(2, C, 8, 10, generator=g)
    target = torch.randn(2, C, 16, 20, generator=g)
    loss = ((la(guide.to(DEV), value.to(DEV)) - target.to(DEV)) ** 2).mean()
    loss.backward()
    offsets, pn = neighbourhood(K)
    ref = lao.local_attender(guide.double(), value.double(), ref_w.reshape(K, Cg), ref_b, offsets=offsets, pn=pn)
    ((ref - target.double()) ** 2).mean().backward()
    assert normwise_err(la.conv1.weight.grad.cpu().reshape(K, Cg), ref_w.grad.reshape(K, Cg)) <= 1e-4
    assert normwise_err(la.conv1.bias.grad.cpu(), ref_b.grad) <= 1e-4
    with torch.no_grad():  # inference afterwards still takes the cached fp32 projection path
        out = la(guide.to(DEV), value.to(DEV))
    assert not out.requires_grad


@pytest.mark.parametrize("K", [9, 17, 25])
def test_gradients_permuted_offsets(K, cuda_lib):
    """An offset table in another order than the reference's takes the
    general dV kernel (runtime offsets) instead of the sliding window."""
    offsets, pn = neighbourhood(K)
    perm = torch.randperm(K, generator=torch.Generator().manual_seed(K)).tolist()
    offsets = [offsets[i] for i in perm]
    for (I, B, Cg, C, H, W) in [(2, 2, 16, 12, 5, 7), (1, 1, 8, 6, 4, 3)]:
        guide, value, weight, bias, gout = _case(K, I, B, Cg, C, H, W, seed=K + I)
        ts = [t.double().requires_grad_() for t in (guide, value, weight, bias)]
        out = lao.local_attender(*ts, offsets=offsets, pn=pn)
        (out * gout.double()).sum().backward()
        tg = [t.to(DEV).requires_grad_() for t in (guide, value, weight, bias)]
        o = ops.local_attender(*tg, offsets, pn)
        (o.float() * gout.to(DEV)).sum().backward()
        for name, e, g in zip(("guide", "value", "weight", "bias"), [t.grad for t in ts], [t.grad for t in tg]):
            assert normwise_err(g.float().cpu(), e) <= 1e-4, (K, I, name)


@pytest.mark.parametrize("I", [4, 6])
def test_gradients_other_factors(I, cuda_lib):
    """Units of four children in a row (I = 4) and of two (I = 6)."""
    K = 17
    for dt, tol in ((torch.float32, 1e-4), (torch.bfloat16, 2e-2)):
        case = _case(K, I, 2, 32, 16, 3, 4, seed=I, dt=dt, wscale=0.05)
        exp = _oracle_grads(*case, K, True, False)
        got = _kernel_grads(*case, K, True, False)
        for name, e, g in zip(("guide", "value", "weight", "bias"), exp, got):
            assert normwise_err(g, e) <= tol, (I, dt, name)


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
def test_gradients_tensor_core_dlogit(K, dt, cuda_lib):
    """I = 2, even Cg <= 64, C a multiple of 32 (16-bit) or 16 (fp32): dP runs
    on the tensor cores (tiles of 8 cells; ragged right edge, single rows,
    one-cell maps; fp32 through a bf16 hi/lo split of both operands).  dW / db
    are fp32 outputs, held to the fp32 bound; dguide / dvalue to the storage
    type's rounding (fp32: the fp32 bound)."""
    tol_store = {torch.bfloat16: 1e-2, torch.float16: 2e-3, torch.float32: 1e-4}[dt]
    for (B, Cg, C, H, W) in [(2, 64, 32, 5, 11), (1, 16, 64, 1, 3), (1, 8, 96, 3, 8), (1, 2, 32, 2, 1),
                             (1, 64, 64, 4, 17)]:
        for conv_res in (True, False):
            case = list(_case(K, 2, B, Cg, C, H, W, seed=K + C + W, dt=dt, wscale=0.05))
            case[4] = case[4].to(dt).float()  # the kernel receives dout in the storage type
            case[2], case[3] = case[2].float(), case[3].float()  # fp32 parameters: fp32 gradients
            exp = _oracle_grads(*case, K, conv_res, False)
            got = _kernel_grads(*case, K, conv_res, False)
            for name, e, g, tol in zip(("guide", "value", "weight", "bias"), exp, got,
                                       (tol_store, tol_store, 1e-4, 1e-4)):
                err = normwise_err(g, e)
                assert err <= tol, (K, dt, B, Cg, C, H, W, conv_res, name, err)


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gradients_value_wide_channels(K, dt, cuda_lib):
    """dV of 16-bit storage with 128-256 channels: ragged row ends, single
    rows, clamped edges, the reference's and a permuted offset table (the
    sliding-window and the general dV kernel), hardmax."""
    tol_store = 1e-2 if dt == torch.bfloat16 else 2e-3
    offsets, pn = neighbourhood(K)
    perm = torch.randperm(K, generator=torch.Generator().manual_seed(7 * K)).tolist()
    for table in (offsets, [offsets[i] for i in perm]):
        for (B, Cg, C, H, W, hardmax) in [(2, 16, 128, 5, 19, False), (1, 8, 256, 1, 3, False),
                                          (1, 64, 128, 4, 33, False), (1, 16, 128, 3, 7, True)]:
            case = list(_case(K, 2, B, Cg, C, H, W, seed=K + C + W, dt=dt, wscale=0.05))
            case[4] = case[4].to(dt).float()
            case[2], case[3] = case[2].float(), case[3].float()
            ts = [t.double().requires_grad_() for t in case[:4]]
            out = lao.local_attender(*ts, hardmax=hardmax, offsets=table, pn=pn)
            (out * case[4].double()).sum().backward()
            tg = [t.to(DEV).requires_grad_() for t in case[:4]]
            o = ops.local_attender(*tg, table, pn, hardmax=hardmax)
            (o.float() * case[4].to(DEV)).sum().backward()
            err = normwise_err(tg[1].grad.float().cpu(), ts[1].grad)
            assert err <= tol_store, (K, dt, B, Cg, C, H, W, hardmax, err)
