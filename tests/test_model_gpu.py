"""End-to-end parity of the upsampler (reference iteration loop around the
fused attender) with outputs of the reference model itself (fp32, seeded
noise), and of make_fast with the plain model."""
import pytest
import torch

from conftest import GOLDEN, normwise_err
from golden.make_golden import SeededNoise
from uplift_b200 import uplift as U
from uplift_b200.configs import get_config
from uplift_b200.fast import make_fast

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def model_golden():
    return torch.load(GOLDEN / "model_cases.pt", weights_only=False)


def _model(variant, iters):
    """fp32 model in the fp32-exact mode (TF32 off inside every forward;
    make_fast inherits the setting)."""
    cfg = get_config(variant)
    torch.manual_seed(0)
    m = U.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, allow_tf32=False).eval()
    m.enable_iterative(iters)
    return m.to(DEV)


def test_upsampler_matches_reference(model_golden, cuda_lib, monkeypatch):
    for case in model_golden["cases"]:
        model = _model(case["variant"], case["iters"])
        monkeypatch.setattr(U, "_randn", SeededNoise(case["noise_seed"]))
        with torch.no_grad():
            y = model(case["img"].to(DEV), case["feats"].to(DEV), case["outsize"])
        y = y[:, ::case["channel_step"]].float().cpu()
        assert y.shape == case["out"].shape
        err = normwise_err(y, case["out"])
        assert err <= 1e-4, (case["variant"], case["outsize"], err)


def test_make_fast_matches_plain(model_golden, cuda_lib):
    case = model_golden["cases"][0]  # DINOv2 arch, no final resize
    model = _model(case["variant"], case["iters"])
    fast = make_fast(model, compile=False, device=torch.device(DEV))
    with torch.no_grad():
        y_plain = model(case["img"].to(DEV), case["feats"].to(DEV))
    y_fast = fast(case["img"].to(DEV), case["feats"].to(DEV))
    # BatchNorm folding changes rounding only
    assert normwise_err(y_fast, y_plain) <= 1e-4


def test_bf16_upsampler_runs_tensor_core_path(cuda_lib):
    from uplift_b200 import _native
    cfg = get_config("dinov2-s14")
    torch.manual_seed(0)
    m = U.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, dtype=torch.bfloat16).eval().to(DEV)
    m.enable_iterative(2)
    img = torch.rand(2, 3, 112, 112, device=DEV, dtype=torch.bfloat16)
    feats = torch.randn(2, 384, 8, 8, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        y = m(img, feats)
    torch.cuda.synchronize()
    assert y.shape == (2, 384, 32, 32) and torch.isfinite(y.float()).all()
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE


def test_low_mem_equals_parallel_and_bf16_iterates(cuda_lib):
    """DINOv3-S+/16 architecture, bf16: low_mem=True gives the same output as
    the parallel path (the fused kernel never materialises the K-fold
    tensor, so the flag only exists for API compatibility) and the model runs
    for iters > 1 (the reference's low_mem returns fp32 there and the next
    bf16 conv fails, uplift/uplift.py:840)."""
    cfg = get_config("dinov3-splus16")
    outs = []
    for low_mem in (False, True):
        torch.manual_seed(0)
        m = U.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, dtype=torch.bfloat16,
                     low_mem=low_mem).eval().to(DEV)
        m.enable_iterative(3)
        g = torch.Generator().manual_seed(5)
        img = torch.rand(2, 3, 128, 128, generator=g).to(DEV, torch.bfloat16)
        feats = torch.randn(2, 384, 8, 8, generator=g).to(DEV, torch.bfloat16)
        with torch.no_grad():
            outs.append(m(img, feats))
    assert outs[0].shape == (2, 384, 64, 64) and outs[0].dtype == torch.bfloat16
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("variant", ["dinov2-s14", "dinov3-splus16", "sd15-vae"])
def test_fast_executor_matches_plain_all_variants(variant, cuda_lib, monkeypatch):
    """The fast-mode executor (convs without bias + fused epilogues, glue
    kernels, concatenation buffers, refiner and noise channels for SD1.5-VAE)
    against the module path, fp32, same seeded noise in both, no final resize
    (the plain path's TVF resize antialiases, the fast path's does not, as in
    the reference)."""
    cfg = get_config(variant)
    torch.manual_seed(0)
    m = U.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, allow_tf32=False).eval().to(DEV)
    m.enable_iterative(2)
    g = torch.Generator().manual_seed(5)
    side = 64 if variant == "sd15-vae" else 112
    lat = side // cfg.backbone.patch
    img = torch.rand(2, 3, side, side, generator=g).to(DEV)
    feats = torch.randn(2, cfg.backbone.channel, lat, lat, generator=g).to(DEV)
    fast = make_fast(m, compile=False, device=torch.device(DEV))
    monkeypatch.setattr(U, "_randn", SeededNoise(77))
    with torch.no_grad():
        y_plain = m(img, feats)
    monkeypatch.setattr(U, "_randn", SeededNoise(77))
    y_fast = fast(img, feats)
    assert y_fast.shape == y_plain.shape
    assert normwise_err(y_fast, y_plain) <= 1e-4, normwise_err(y_fast, y_plain)
