"""The fused attender is a registered torch custom op: torch.compile traces a
model containing it without graph breaks (the reference's Triton module is
@torch.compiler.disable, uplift/kernels/triton_attender.py:335)."""
import pytest
import torch

from uplift_b200.attender import LocalAttender

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_local_attender_compiles_fullgraph(cuda_lib):
    torch.manual_seed(0)
    la = LocalAttender(64, 17).to(DEV).to(torch.bfloat16)
    guide = torch.randn(2, 64, 32, 48, device=DEV, dtype=torch.bfloat16)
    value = torch.randn(2, 384, 16, 24, device=DEV, dtype=torch.bfloat16)

    def f(g, v):
        return la(g * 1.0, v) + 0.0  # surrounding ops keep the op inside a real graph

    compiled = torch.compile(f, fullgraph=True)  # a graph break raises here
    with torch.no_grad():
        out = compiled(guide, value)
        ref = la(guide, value)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
