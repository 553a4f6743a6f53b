"""Model loading with the reference's hub signatures (hubconf.py:4-39,
uplift/hub_loader.py:64-113).

Only the upsampler itself is built here (`include_extractor=False`); the
timm / diffusers backbone extractors are outside this package.  Pretrained
weights are fetched with huggingface_hub when it and the network are
available; `pretrained=False` builds a random-init model.
"""
from __future__ import annotations

import torch

from .configs import VARIANTS, get_config
from .uplift import UPLiFT

HF_ORG = "UPLiFT-upsampler"
_FILES = {
    "dinov2-s14": ("uplift_dinov2-s14", "uplift_dinov2-s14.safetensors"),
    "dinov3-splus16": ("uplift_dinov3-splus16", "uplift_dinov3-splus16.safetensors"),
    "sd15-vae": ("uplift_sd1.5vae", "uplift_sd1.5vae.safetensors"),
}


def _download_weights(variant: str, cache_dir=None) -> str:
    from huggingface_hub import hf_hub_download
    repo, fname = _FILES[variant]
    return hf_hub_download(repo_id=f"{HF_ORG}/{repo}", filename=fname, cache_dir=cache_dir)


def load_model(variant: str, pretrained: bool = True, include_extractor: bool = True,
               fast: bool = False, **kwargs):
    """UPLiFT model of a released variant; see module docstring."""
    if variant not in VARIANTS:
        raise ValueError(f"Unknown variant '{variant}'. Choose from: {list(VARIANTS)}")
    if include_extractor:
        raise NotImplementedError(
            "backbone extractors (timm / diffusers) are not part of uplift_b200; "
            "load with include_extractor=False and pass backbone features to the model")
    cfg = get_config(variant)
    model = UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift,
                   dtype=kwargs.pop("dtype", torch.float32), low_mem=kwargs.pop("low_mem", False))
    if "iters" in kwargs:
        model.enable_iterative(kwargs.pop("iters"))
    if pretrained:
        from safetensors.torch import load_file
        model.load_state_dict(load_file(_download_weights(variant)))
    if fast:
        from .fast import make_fast
        model = make_fast(model, **kwargs)
    return model
