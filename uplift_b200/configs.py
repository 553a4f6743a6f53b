"""Architecture configurations of the three released UPLiFT variants.

The hyper-parameters (channel widths, block types, counts, attender size,
noise channels) define the parameter shapes of the released checkpoints, so
they equal those of the reference's configs (uplift/configs/
uplift_dinov2-s14.yaml, uplift_dinov3-splus16.yaml, uplift_sd1.5vae.yaml,
sections `backbone` and `uplift`).  Training, dataset and logging sections
are not needed by inference and are left out.

`load_config(path)` also reads a reference-style YAML file (PyYAML) into the
same attribute-access form, for users with their own configs.
"""
from __future__ import annotations

import copy
from types import SimpleNamespace


def _group(block, norm, hc):
    return {"block": block, "norm": norm, "count": len(hc), "hc": list(hc)}


def _no_down():
    return {"down_op": "none", "factor": 1.0, "residual": "none"}


def _vit_uplift():
    """DINOv2-S/14 and DINOv3-S+/16 share the upsampler architecture."""
    enc = {"down_steps": 4}
    for i, hc in enumerate([16, 32, 64, 128, 128]):
        enc[f"block_{i}"] = _group("SingleConv", "batch", [hc])
        if i > 0:
            enc[f"down_{i}"] = _no_down()
    dec = {"up_steps": 1, "ncat_c": 0, "ncat_s": 1, "enc_resample": "nearest",
           "block_0": _group("DoubleConv", "batch", [64]),
           "up_1": {"up_op": "tconv", "factor": 2, "residual": "bilinear"},
           "block_1": _group("DoubleConv", "batch", [64])}
    return {"up_factor": 2, "attender": 17, "enc_share": True, "encoder": enc, "decoder": dec}


def _sdvae_uplift():
    enc = {"down_steps": 4}
    for i, hc in enumerate([64, 128, 256, 512, 512]):
        enc[f"block_{i}"] = _group("SingleConv", "layer", [hc, hc])
        if i > 0:
            enc[f"down_{i}"] = _no_down()
    dec = {"up_steps": 1, "ncat_c": 4, "ncat_s": 1, "enc_resample": "nearest",
           "block_0": _group("SingleConv", "layer", [512]),
           "up_1": {"up_op": "tconv", "factor": 2, "residual": "bilinear"},
           "block_1": _group("SingleConv", "layer", [512, 512])}
    ref = {"enc_resample": "nearest", "ncat_c": 4, "ncat_s": 1, "ref_con": -1,
           "block_0": _group("SingleConv", "layer", [512] * 12)}
    return {"up_factor": 2, "no_UEP": True, "attender": 17, "enc_share": True,
            "encoder": enc, "decoder": dec, "refiner": ref}


VARIANTS = {
    "dinov2-s14": {"backbone": {"channel": 384, "patch": 14, "stride": 14,
                                "model_type": "vit_small_patch14_dinov2.lvd142m",
                                "diff_pipe_name": None},
                   "uplift": _vit_uplift()},
    "dinov3-splus16": {"backbone": {"channel": 384, "patch": 16, "stride": 16,
                                    "model_type": "vit_small_plus_patch16_dinov3.lvd1689m",
                                    "diff_pipe_name": None},
                       "uplift": _vit_uplift()},
    "sd15-vae": {"backbone": {"channel": 4, "patch": 8, "stride": 8, "model_type": None,
                              "diff_pipe_name": "stable-diffusion-v1-5/stable-diffusion-v1-5"},
                 "uplift": _sdvae_uplift()},
}


def to_namespace(d):
    if isinstance(d, dict):
        return SimpleNamespace(**{k: to_namespace(v) for k, v in d.items()})
    if isinstance(d, list):
        return [to_namespace(v) for v in d]
    return d


def get_config(variant: str):
    """Attribute-access config ({backbone, uplift}) of a released variant."""
    if variant not in VARIANTS:
        raise ValueError(f"Unknown variant '{variant}'. Choose from: {list(VARIANTS)}")
    return to_namespace(copy.deepcopy(VARIANTS[variant]))


def load_config(path):
    """Read a reference-style YAML config into attribute-access form."""
    import yaml
    with open(path) as f:
        return to_namespace(yaml.safe_load(f))
