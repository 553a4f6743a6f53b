"""The tensor-core dlogit of the backward (la_bwd_dl.cu) for 16-bit storage:
logits, softmax weights, dP = dout . value window, dl = P (dP - <P, dP>),
dguide = dl . (W + I) and dW / db = sum over pixels of dl . [guide | 1], all
per tile of 128 output pixels on the tensor cores.  The gradient of the
projection through LocalAttender.forward (uplift/uplift.py:801-847) is
checked against fp64 autograd through the oracle (every K, ragged tiles,
1-6 channel chunks, with and without the residual, permuted offset tables,
hardmax, fp16), and against the probs + dlogit kernels it replaces
(ULA_BWD_DL_TC=0, read once per process, so that run is a child process)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from conftest import normwise_err
from oracle import local_attender_oracle as lao
from uplift_b200 import ops
from uplift_b200.attender import neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ROOT = Path(__file__).resolve().parent.parent
# dguide is rounded once to the storage type; dW and db are fp32 sums of
# exact 16-bit products (two-term splits of dl and W); dvalue as the
# tensor-core dV (P rounded to the storage type)
TOL = {torch.bfloat16: {"guide": 4e-3, "value": 1e-2, "weight": 1e-4, "bias": 1e-4},
       torch.float16: {"guide": 1e-3, "value": 2e-3, "weight": 1e-4, "bias": 1e-4}}


def _case(K, B, C, H, W, seed, dt, wscale=0.3):
    g = torch.Generator().manual_seed(seed)
    guide = torch.randn(B, 64, 2 * H, 2 * W, generator=g).to(dt)
    value = torch.randn(B, C, H, W, generator=g).to(dt)
    weight = torch.randn(K, 64, generator=g) * wscale
    bias = torch.randn(K, generator=g) * 0.5
    gout = torch.randn(B, C, 2 * H, 2 * W, generator=g).to(dt)
    return guide, value, weight, bias, gout


def _oracle(case, offsets, pn, conv_res, hardmax):
    guide, value, weight, bias, gout = case
    ts = [t.double().requires_grad_() for t in (guide, value, weight, bias)]
    out = lao.local_attender(*ts, conv_res=conv_res, hardmax=hardmax, offsets=offsets, pn=pn)
    (out * gout.double()).sum().backward()
    return [t.grad for t in ts]


def _kernel(case, offsets, pn, conv_res, hardmax):
    guide, value, weight, bias, gout = case
    cl = torch.channels_last
    grads = ops.local_attender_backward_raw(
        gout.to(DEV).contiguous(memory_format=cl), guide.to(DEV).contiguous(memory_format=cl),
        value.to(DEV).contiguous(memory_format=cl), weight.to(DEV), bias.to(DEV), offsets, pn,
        conv_res=conv_res, hardmax=hardmax, need_guide=True, need_value=True, need_params=True)
    torch.cuda.synchronize()
    return [g.float().cpu() for g in grads]


def _check(case, offsets, pn, conv_res, hardmax, dt, tag):
    exp = _oracle(case, offsets, pn, conv_res, hardmax)
    got = _kernel(case, offsets, pn, conv_res, hardmax)
    for name, e, g in zip(("guide", "value", "weight", "bias"), exp, got):
        if hardmax and name != "value":
            assert float(g.abs().max()) == 0.0, (tag, name)
            continue
        err = normwise_err(g, e)
        assert err <= TOL[dt][name], (tag, name, err)


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
def test_tc_dlogit_vs_fp64_autograd(K, cuda_lib):
    offsets, pn = neighbourhood(K)
    # (B, C, H, W): ragged tiles (H % 4, W % 8), a single cell row, 1-6
    # chunks (a 1 x 1 map is left out: every offset clamps to the one value
    # pixel, so the logit gradients are zero up to rounding and have no
    # relative error to check)
    for i, (B, C, H, W) in enumerate([(2, 64, 5, 7), (1, 384, 9, 17), (2, 128, 8, 16), (1, 192, 1, 2),
                                      (1, 320, 12, 40)]):
        for conv_res in (True, False):
            case = _case(K, B, C, H, W, seed=K * 11 + i, dt=torch.bfloat16)
            _check(case, offsets, pn, conv_res, False, torch.bfloat16, (K, B, C, H, W, conv_res))
    from uplift_b200 import _native
    assert _native.device_status(clear=True) == 0


def test_tc_dlogit_permuted_offsets_hardmax_fp16(cuda_lib):
    offsets, pn = neighbourhood(17)
    perm = offsets[5:] + offsets[:5]
    for dt in (torch.bfloat16, torch.float16):
        case = _case(17, 2, 128, 10, 19, seed=5, dt=dt, wscale=0.05)
        for offs, hard in ((perm, False), (offsets, True), (perm, True)):
            _check(case, offs, pn, True, hard, dt, (dt, hard))


SCRIPT = r"""
import sys, torch
sys.path.insert(0, {root!r})
from uplift_b200 import ops
from uplift_b200.attender import neighbourhood
g = torch.Generator(device="cuda:0").manual_seed(21)
cl = torch.channels_last
B, C, H, W = 2, 384, 128, 128
guide = torch.randn(B, 64, 2 * H, 2 * W, generator=g, device="cuda:0").to(torch.bfloat16).contiguous(memory_format=cl)
value = torch.randn(B, C, H, W, generator=g, device="cuda:0").to(torch.bfloat16).contiguous(memory_format=cl)
dout = torch.randn(B, C, 2 * H, 2 * W, generator=g, device="cuda:0").to(torch.bfloat16).contiguous(memory_format=cl)
w = torch.randn(17, 64, generator=g, device="cuda:0") * 0.1
b = torch.randn(17, generator=g, device="cuda:0") * 0.5
offsets, pn = neighbourhood(17)
dg, dv, dw, db = ops.local_attender_backward_raw(dout, guide, value, w, b, offsets, pn)
torch.save([t.cpu() for t in (dg, dv, dw, db)], {out!r})
"""


def test_tc_dlogit_matches_the_probs_and_dlogit_kernels_on_a_dinov2_level(tmp_path, cuda_lib):
    """The 128^2 -> 256^2 level of the 448 px upsampler (B=2): the tensor-core
    dlogit and the kernels it replaces on the same inputs, each in its own
    process.  They sum in different orders (which shows the tensor-core
    kernel ran), within the rounding of each output."""
    outs = {}
    for tag, env in (("tc", "1"), ("simt", "0")):
        out = tmp_path / f"dl_{tag}.pt"
        proc = subprocess.run([sys.executable, "-c", SCRIPT.format(root=str(ROOT), out=str(out))],
                              env=dict(os.environ, ULA_BWD_DL_TC=env), capture_output=True, text=True, timeout=600)
        assert proc.returncode == 0, proc.stderr[-3000:]
        outs[tag] = torch.load(out, weights_only=False)
    for name, a, b, tol in zip(("guide", "value", "weight", "bias"), outs["tc"], outs["simt"],
                               (4e-3, 1e-2, 1e-4, 1e-4)):
        err = normwise_err(a.float(), b.float())
        assert err <= tol, (name, err)
    assert not torch.equal(outs["tc"][2], outs["simt"][2])
