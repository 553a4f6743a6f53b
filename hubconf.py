"""torch.hub entry points with the reference's signatures (hubconf.py:4-39 of
mwalmer-umd/UPLiFT), backed by uplift_b200.  See uplift_b200/hub.py."""
dependencies = ["torch"]


def uplift(variant="dinov2-s14", pretrained=True, include_extractor=True, fast=False, **kwargs):
    """Load an UPLiFT upsampler ("dinov2-s14", "dinov3-splus16", "sd15-vae")."""
    from uplift_b200.hub import load_model
    return load_model(variant, pretrained, include_extractor, fast=fast, **kwargs)


def uplift_dinov2_s14(pretrained=True, include_extractor=True, fast=False, **kwargs):
    return uplift("dinov2-s14", pretrained, include_extractor, fast=fast, **kwargs)


def uplift_dinov3_splus16(pretrained=True, include_extractor=True, fast=False, **kwargs):
    return uplift("dinov3-splus16", pretrained, include_extractor, fast=fast, **kwargs)


def uplift_sd15_vae(pretrained=True, include_extractor=True, fast=False, **kwargs):
    return uplift("sd15-vae", pretrained, include_extractor, fast=fast, **kwargs)
