"""The tensor-core kernel's small-grid mode: below a number of tiles per SM
each tile is split into its two accumulator halves, which different CTAs
compute.  The arithmetic per output value is unchanged, so the split and
unsplit launches must agree bit for bit; both are also checked against the
double-precision oracle.  The threshold is read once per process, so each
setting runs in its own process."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from conftest import normwise_err
from oracle import c_oracle
from uplift_b200.attender import neighbourhood

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

SCRIPT = r"""
import sys, torch
sys.path.insert(0, {root!r})
from uplift_b200 import _native, ops
from uplift_b200.attender import neighbourhood
cases = torch.load({inp!r}, weights_only=False)
outs = []
for c in cases:
    offsets, pn = neighbourhood(c["K"])
    dev = "cuda:0"
    cl = torch.channels_last
    g = c["guide"].to(dev).contiguous(memory_format=cl)
    v = c["value"].to(dev).contiguous(memory_format=cl)
    with _native.kernel_policy(_native.POLICY_TENSOR_CORE):
        if c.get("size"):
            y = ops.local_attender_resized_raw(g, v, c["w"].to(dev), c["b"].to(dev), offsets, pn, c["size"])
        else:
            y = ops.local_attender_raw(g, v, c["w"].to(dev), c["b"].to(dev), offsets, pn)
    outs.append(y.cpu())
assert _native.device_status(clear=True) == 0
torch.save(outs, {out!r})
"""


def _cases():
    g = torch.Generator().manual_seed(31)
    cases = []
    # (B, H, W, C, K, size): one to a few hundred tiles, ragged edges, 2-6 chunks
    for (B, H, W, C, K, size) in [(1, 4, 8, 128, 17, None), (2, 9, 13, 384, 17, None), (3, 16, 16, 256, 9, None),
                                  (8, 32, 32, 384, 17, None), (2, 8, 16, 384, 25, (14, 28)),
                                  (1, 20, 12, 192, 5, None)]:
        cases.append(dict(guide=torch.randn(B, 64, 2 * H, 2 * W, generator=g).to(torch.bfloat16),
                          value=torch.randn(B, C, H, W, generator=g).to(torch.bfloat16),
                          w=(torch.randn(K, 64, generator=g) * 0.3).to(torch.bfloat16).float(),
                          b=torch.randn(K, generator=g) * 0.5, K=K, size=size))
    return cases


def _run(tmp_path, cases, threshold, tag):
    inp, out = tmp_path / "cases.pt", tmp_path / f"out_{tag}.pt"
    if not inp.exists():
        torch.save(cases, inp)
    env = dict(os.environ, ULA_TC_SPLIT_TILES_PER_SM=str(threshold))
    proc = subprocess.run([sys.executable, "-c", SCRIPT.format(root=str(ROOT), inp=str(inp), out=str(out))],
                          env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-3000:]
    return torch.load(out, weights_only=False)


def test_split_and_unsplit_agree_bitwise(tmp_path, cuda_lib):
    cases = _cases()
    split = _run(tmp_path, cases, 1 << 20, "split")   # every launch split
    whole = _run(tmp_path, cases, 0, "whole")         # no launch split
    for c, a, b in zip(cases, split, whole):
        assert torch.equal(a, b), (tuple(c["value"].shape), c["K"], c["size"])
        if c["size"] is None:
            exp = c_oracle.forward(c["guide"], c["value"], c["w"], c["b"], neighbourhood(c["K"])[0])
            assert normwise_err(a, exp) <= 8e-3
