"""The tensor-core dV of the backward (la_bwd_dv.cu): value-centric tiles of
8 x 16 value pixels, dV = Pt . dout accumulated in TMEM over the output cell
rows that reach the tile, Pt (the softmax weights, rounded to the storage
type) built in shared memory.  It is the transpose of the forward's pooling
(uplift/uplift.py:835-837), so it is checked against fp64 autograd through
the oracle (every K, ragged tiles, 1-6 channel chunks, permuted offset
tables, hardmax, fp16; border tiles through the scatter fill of Pt,
interior tiles through the gather fill), and against the CUDA-core dV
kernel it replaces
(ULA_BWD_DV_TC=0, read once per process, so that run is a child process)."""
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
# P is rounded to the storage type before the products (as the forward does)
TOL16 = {torch.bfloat16: 1e-2, torch.float16: 2e-3}


def _case(K, B, C, H, W, seed, dt, wscale=0.3):
    g = torch.Generator().manual_seed(seed)
    guide = torch.randn(B, 64, 2 * H, 2 * W, generator=g).to(dt)
    value = torch.randn(B, C, H, W, generator=g).to(dt)
    weight = (torch.randn(K, 64, generator=g) * wscale).to(dt)
    bias = (torch.randn(K, generator=g) * 0.5).to(dt)
    gout = torch.randn(B, C, 2 * H, 2 * W, generator=g).to(dt)
    return guide, value, weight, bias, gout


def _oracle_dv(case, offsets, pn, hardmax):
    guide, value, weight, bias, gout = case
    ts = [t.double().requires_grad_() for t in (guide, value, weight, bias)]
    out = lao.local_attender(*ts, conv_res=True, hardmax=hardmax, offsets=offsets, pn=pn)
    (out * gout.double()).sum().backward()
    return ts[1].grad


def _kernel_dv(case, offsets, pn, hardmax):
    guide, value, weight, bias, gout = case
    cl = torch.channels_last
    _, dv, _, _ = ops.local_attender_backward_raw(
        gout.to(DEV).contiguous(memory_format=cl), guide.to(DEV).contiguous(memory_format=cl),
        value.to(DEV).contiguous(memory_format=cl), weight.to(DEV).float(), bias.to(DEV).float(), offsets, pn,
        conv_res=True, hardmax=hardmax, need_guide=False, need_value=True, need_params=False)
    torch.cuda.synchronize()
    return dv


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
def test_tc_dv_vs_fp64_autograd(K, cuda_lib):
    offsets, pn = neighbourhood(K)
    # (B, C, H, W): ragged tiles (H % 8, W % 16), tiny maps, 1-6 chunks;
    # the last three have interior tiles (no value pixel on the map border:
    # the gather fill of Pt), the smallest such maps among them
    for i, (B, C, H, W) in enumerate([(2, 64, 5, 7), (1, 384, 9, 17), (2, 128, 8, 16), (1, 192, 1, 1),
                                      (1, 320, 12, 40), (2, 64, 17, 33), (1, 128, 24, 50), (1, 384, 33, 70)]):
        case = _case(K, B, C, H, W, seed=K * 7 + i, dt=torch.bfloat16)
        err = normwise_err(_kernel_dv(case, offsets, pn, False), _oracle_dv(case, offsets, pn, False))
        assert err <= TOL16[torch.bfloat16], (K, B, C, H, W, err)


def test_tc_dv_permuted_offsets_hardmax_fp16(cuda_lib):
    offsets, pn = neighbourhood(17)
    perm = offsets[9:] + offsets[:9]
    for dt in (torch.bfloat16, torch.float16):
        for shape in ((2, 128, 10, 19), (1, 128, 26, 49)):  # border tiles only; interior tiles too
            case = _case(17, *shape, seed=3, dt=dt, wscale=0.05)
            for offs, hard in ((perm, False), (offsets, True), (perm, True)):
                err = normwise_err(_kernel_dv(case, offs, pn, hard), _oracle_dv(case, offs, pn, hard))
                assert err <= TOL16[dt], (dt, shape, hard, err)


SCRIPT = r"""
import sys, torch
sys.path.insert(0, {root!r})
from uplift_b200 import ops
from uplift_b200.attender import neighbourhood
g = torch.Generator(device="cuda:0").manual_seed(12)
cl = torch.channels_last
B, C, H, W = 2, 384, 256, 256
guide = torch.randn(B, 64, 2 * H, 2 * W, generator=g, device="cuda:0").to(torch.bfloat16).contiguous(memory_format=cl)
value = torch.randn(B, C, H, W, generator=g, device="cuda:0").to(torch.bfloat16).contiguous(memory_format=cl)
dout = torch.randn(B, C, 2 * H, 2 * W, generator=g, device="cuda:0").to(torch.bfloat16).contiguous(memory_format=cl)
w = torch.randn(17, 64, generator=g, device="cuda:0") * 0.1
b = torch.randn(17, generator=g, device="cuda:0") * 0.5
offsets, pn = neighbourhood(17)
_, dv, _, _ = ops.local_attender_backward_raw(dout, guide, value, w, b, offsets, pn, need_guide=False,
                                              need_value=True, need_params=False)
torch.save(dv.cpu(), {out!r})
"""


def test_tc_dv_matches_cuda_core_dv_on_a_dinov2_level(tmp_path, cuda_lib):
    """The 256^2 -> 512^2 level of the 448 px upsampler (B=2): the
    tensor-core dV and the CUDA-core dV on the same inputs, each in its own
    process.  They round P at different points, so they differ (which shows
    the tensor-core kernel ran) by no more than that rounding."""
    outs = {}
    for tag, env in (("tc", "1"), ("simt", "0")):
        out = tmp_path / f"dv_{tag}.pt"
        proc = subprocess.run([sys.executable, "-c", SCRIPT.format(root=str(ROOT), out=str(out))],
                              env=dict(os.environ, ULA_BWD_DV_TC=env), capture_output=True, text=True, timeout=600)
        assert proc.returncode == 0, proc.stderr[-3000:]
        outs[tag] = torch.load(out, weights_only=False)
    err = normwise_err(outs["tc"], outs["simt"])
    assert 0 < err <= 1e-2, err
