"""The upsampler (caller of the attender) mirrors the reference module tree:
same state_dict keys, shapes and -- built under the same seed -- the same
initial parameters, for the three released variants.  CPU only (the model
is only constructed, never run)."""
import hashlib

import pytest
import torch

from conftest import GOLDEN
from uplift_b200.configs import VARIANTS, get_config, load_config
from uplift_b200.uplift import UPLiFT


def _sha(t):
    return hashlib.sha256(t.detach().float().contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.fixture(scope="module")
def model_golden():
    return torch.load(GOLDEN / "model_cases.pt", weights_only=False)


@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_state_dict_matches_reference(variant, model_golden):
    ref = model_golden["params"][variant]
    cfg = get_config(variant)
    torch.manual_seed(0)
    model = UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift)
    sd = model.state_dict()
    assert list(sd.keys()) == ref["__keys__"]
    for k, v in sd.items():
        if not v.dtype.is_floating_point:
            continue
        shape, sha = ref[k]
        assert list(v.shape) == shape, k
        assert _sha(v) == sha, f"{k}: initial values differ from the reference's under seed 0"


def test_config_yaml_loader(tmp_path):
    p = tmp_path / "c.yaml"
    p.write_text("uplift:\n  attender: 17\n  encoder:\n    down_steps: 0\n    block_0: {block: SingleConv, count: 1, hc: [8]}\n")
    cfg = load_config(p)
    assert cfg.uplift.attender == 17 and cfg.uplift.encoder.block_0.hc == [8]


def test_hub_signatures():
    import hubconf
    with pytest.raises(NotImplementedError, match="include_extractor=False"):
        hubconf.uplift_dinov2_s14(pretrained=False)
    m = hubconf.uplift_sd15_vae(pretrained=False, include_extractor=False)
    assert isinstance(m, UPLiFT) and m.attender.num_connected == 17
    with pytest.raises(ValueError, match="Unknown variant"):
        hubconf.uplift("nope", pretrained=False, include_extractor=False)


def test_tf32_mode_scopes_the_switches():
    """allow_tf32 on the model and on make_fast sets TF32 for the forward
    only and leaves PyTorch's global switches as they were; None (the
    reference's behaviour) touches nothing."""
    from uplift_b200.fast import make_fast
    from uplift_b200.uplift import tf32_mode
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    try:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = True, True
        with tf32_mode(False):
            assert (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32) == (False, False)
        assert (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32) == (True, True)
        with tf32_mode(None):
            assert (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32) == (True, True)
        cfg = get_config("dinov2-s14")
        torch.manual_seed(0)
        model = UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift, allow_tf32=False)
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = False, True
        fast = make_fast(model, compile=False, warmup=False, device=torch.device("cpu"))
        assert fast.allow_tf32 is False  # inherited from the model
        fast = make_fast(model, compile=False, warmup=False, device=torch.device("cpu"), allow_tf32=True)
        assert fast.allow_tf32 is True
        assert (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32) == (False, True)
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def test_bf16_upsampler_fixture_inputs_regenerate():
    """The inputs of the bf16 upsampler goldens come back from their seeds
    bit for bit (the GPU test regenerates them instead of storing them)."""
    import sys
    sys.path.insert(0, str(GOLDEN))
    from make_golden_bf16_upsampler import inputs, sha
    gold = torch.load(GOLDEN / "upsampler_bf16_bands.pt", weights_only=False)
    assert len(gold["cases"]) == 3
    for case in gold["cases"]:
        img, feats = inputs(case["img_px"], case["feat_px"], 384, case["seed"])
        assert sha(img) == case["img_sha"] and sha(feats) == case["feats_sha"]
        assert case["bands"].shape[0] == 3 and case["channel_sum"].shape == (384,)
