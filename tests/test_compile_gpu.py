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


def test_make_fast_compiled_matches_plain(cuda_lib):
    """make_fast with torch.compile (BN folding, channels_last, compiled
    iteration loop with the fused attender inside) matches the plain model."""
    from uplift_b200 import uplift as U
    from uplift_b200.configs import get_config
    from uplift_b200.fast import make_fast
    cfg = get_config("dinov2-s14")
    torch.manual_seed(0)
    m = U.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, dtype=torch.bfloat16).eval().to(DEV)
    m.enable_iterative(2)
    g = torch.Generator().manual_seed(3)
    img = torch.rand(2, 3, 112, 112, generator=g).to(DEV, torch.bfloat16)
    feats = torch.randn(2, 384, 8, 8, generator=g).to(DEV, torch.bfloat16)
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    # allow_tf32=True: TF32 inside the fast forward only, the globals untouched
    fast = make_fast(m, compile=True, compile_mode="default", warmup=False, device=torch.device(DEV),
                     allow_tf32=True)
    with torch.no_grad():
        ref = m(img, feats)
    out = fast(img, feats)
    torch.cuda.synchronize()
    assert (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32) == old
    err = ((out.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
    assert out.shape == ref.shape and err <= 2e-2, err  # bf16 convs, folded BatchNorm
