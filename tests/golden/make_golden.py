"""Generate the Local Attender golden vectors by EXECUTING THE REFERENCE.

Run where a checkout of the reference is available, naming it with --ref
or the UPLIFT_REFERENCE environment variable:

    python tests/golden/make_golden.py --ref <reference checkout>

It loads uplift/uplift.py (LocalAttender, uplift/uplift.py:740-847) and
uplift/kernels/triton_attender.py (TritonLocalAttender._fallback_forward,
:402-431, the only reference code with `hardmax`) by file path, runs them on
the CPU on seeded inputs, and writes

    tests/golden/la_cases.pt      small cases, inputs + outputs
    tests/golden/la_config1.pt    standalone config (K=9, fp32, B=1, value
                                  384x32x32, guide 64x64x64): input hashes,
                                  every 8th output channel, output checksums
    tests/golden/model_cases.pt   the full UPLiFT upsampler (uplift/uplift.py:
                                  537-643) of the three released variants:
                                  per-parameter shape + sha256 under seed 0,
                                  and small fp32 forward cases (seeded noise
                                  replaces torch.randn in noise_and_combine)

The committed fixtures pin both the CPU oracle and the CUDA kernels to the
reference.  Nothing on the GPU side reads the reference at run time.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import importlib.util
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def load_module(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def tensor_sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


def config1_inputs():
    """Seeded inputs of the standalone fp32 config: value 1x384x32x32 and
    guide 1x64x64x64 N(0,1), conv1 weight N(0, 0.02), zero bias, seed 0."""
    g = torch.Generator().manual_seed(0)
    value = torch.randn(1, 384, 32, 32, generator=g)
    guide = torch.randn(1, 64, 64, 64, generator=g)
    weight = torch.randn(9, 64, generator=g) * 0.02
    bias = torch.zeros(9)
    return guide, value, weight, bias


# name, K, I, Cg, C, B, H, W, dtype, conv_res, low_mem
FORWARD_CASES = [
    ("k5_i2_f32", 5, 2, 16, 12, 2, 5, 7, torch.float32, True, False),
    ("k9_i2_f32", 9, 2, 16, 12, 2, 5, 7, torch.float32, True, False),
    ("k13_i2_f32", 13, 2, 16, 12, 2, 5, 7, torch.float32, True, False),
    ("k17_i2_f32", 17, 2, 16, 12, 2, 5, 7, torch.float32, True, False),   # Cg < K: zero-pad residual
    ("k25_i2_f32", 25, 2, 16, 12, 2, 5, 7, torch.float32, True, False),
    ("k17_i2_f32_cg_eq_k", 17, 2, 17, 8, 1, 4, 4, torch.float32, True, False),
    ("k17_i2_f32_cg64", 17, 2, 64, 24, 1, 6, 5, torch.float32, True, False),
    ("k9_i2_f32_nores", 9, 2, 16, 12, 2, 5, 7, torch.float32, False, False),
    ("k17_i1_f32", 17, 1, 24, 8, 2, 6, 5, torch.float32, True, False),
    ("k17_i3_f32", 17, 3, 24, 8, 1, 4, 3, torch.float32, True, False),
    ("k17_i4_f32", 17, 4, 24, 40, 1, 4, 3, torch.float32, True, False),
    ("k5_i4_f32", 5, 4, 8, 4, 2, 3, 2, torch.float32, True, False),
    ("k25_i2_f32_1x1", 25, 2, 8, 6, 3, 1, 1, torch.float32, True, False),
    ("k13_i2_f32_1xw", 13, 2, 8, 6, 1, 1, 9, torch.float32, True, False),
    ("k17_i2_f32_c4_cg512", 17, 2, 512, 4, 1, 4, 4, torch.float32, True, False),  # SD-VAE-like
    ("k17_i2_f32_lowmem", 17, 2, 16, 12, 2, 5, 7, torch.float32, True, True),
    ("k17_i2_bf16", 17, 2, 64, 32, 2, 6, 6, torch.bfloat16, True, False),
    ("k9_i2_bf16", 9, 2, 64, 40, 1, 5, 8, torch.bfloat16, True, False),
    ("k17_i2_bf16_lowmem", 17, 2, 64, 32, 1, 4, 4, torch.bfloat16, True, True),  # returns fp32
    ("k17_i4_bf16", 17, 4, 64, 16, 1, 3, 3, torch.bfloat16, True, False),
    ("k9_i2_f16", 9, 2, 32, 16, 1, 4, 5, torch.float16, True, False),
    ("k17_i2_bf16_c3", 17, 2, 16, 3, 1, 4, 4, torch.bfloat16, True, False),      # odd C: scalar path
    ("k17_i2_f32_empty", 17, 2, 16, 8, 0, 4, 4, torch.float32, True, False),
]

# name, I, C, B, H, W, dtype, hardmax
POOL_CASES = [
    ("pool_k17_i2_f32_soft", 2, 5, 2, 4, 3, torch.float32, False),
    ("pool_k17_i2_f32_hard", 2, 5, 2, 4, 3, torch.float32, True),
    ("pool_k17_i4_f32_hard", 4, 8, 1, 3, 3, torch.float32, True),
    ("pool_k17_i1_bf16_hard", 1, 16, 1, 5, 6, torch.bfloat16, True),
    ("pool_k17_i2_bf16_soft", 2, 16, 1, 5, 6, torch.bfloat16, False),
]


def namespace(d):
    from types import SimpleNamespace
    if isinstance(d, dict):
        return SimpleNamespace(**{k: namespace(v) for k, v in d.items()})
    if isinstance(d, list):
        return [namespace(v) for v in d]
    return d


class SeededNoise:
    """Deterministic stand-in for torch.randn inside noise_and_combine: draws
    from its own CPU generator in call order, then moves to the device."""

    def __init__(self, seed):
        self.g = torch.Generator().manual_seed(seed)
        self._randn = torch.randn  # the real one, even while torch.randn is patched

    def __call__(self, shape, device=None, dtype=None):
        return self._randn(list(shape), generator=self.g).to(device=device, dtype=dtype)


MODEL_VARIANTS = {"dinov2-s14": "uplift_dinov2-s14.yaml", "dinov3-splus16": "uplift_dinov3-splus16.yaml",
                  "sd15-vae": "uplift_sd1.5vae.yaml"}


def model_golden(ref: Path, up):
    import yaml
    out = {"params": {}, "cases": []}
    cfgs = {}
    for variant, fname in MODEL_VARIANTS.items():
        cfg = namespace(yaml.safe_load(open(ref / "uplift" / "configs" / fname)))
        cfgs[variant] = cfg
        torch.manual_seed(0)
        model = up.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift)
        out["params"][variant] = {k: (list(v.shape), tensor_sha(v.detach().float()))
                                  for k, v in model.state_dict().items() if v.dtype.is_floating_point}
        out["params"][variant]["__keys__"] = list(model.state_dict().keys())
    # forward cases (fp32, eval mode)
    specs = [("dinov2-s14", 1, 56, 4, 2, None, 11), ("dinov2-s14", 2, 56, 4, 2, [30, 30], 12),
             ("sd15-vae", 1, 32, 4, 2, None, 13)]
    for variant, B, img_px, feat_px, iters, outsize, seed in specs:
        cfg = cfgs[variant]
        torch.manual_seed(0)
        model = up.UPLiFT(cfg.backbone.channel, cfg.backbone.patch, cfg.uplift).eval()
        model.enable_iterative(iters)
        g = torch.Generator().manual_seed(seed)
        lo = -1.0 if variant == "sd15-vae" else 0.0
        img = torch.rand(B, 3, img_px, img_px, generator=g) * (1 - lo) + lo
        feats = torch.randn(B, cfg.backbone.channel, feat_px, feat_px, generator=g)
        real_randn = torch.randn
        noise = SeededNoise(seed + 1000)
        try:
            torch.randn = lambda *a, **k: noise(a[0], k.get("device"), k.get("dtype")) if a and isinstance(a[0], list) else real_randn(*a, **k)
            with torch.no_grad():
                y = model(img, feats, outsize)
        finally:
            torch.randn = real_randn
        step = 4 if y.numel() > 200_000 else 1  # keep the fixture small: every 4th channel
        out["cases"].append(dict(variant=variant, B=B, iters=iters, outsize=outsize, img=img, feats=feats,
                                 noise_seed=seed + 1000, channel_step=step, out=y[:, ::step].clone()))
        print(f"model {variant:14s} out {tuple(y.shape)}")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("UPLIFT_REFERENCE"),
                    help="reference checkout (default: $UPLIFT_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("name the reference checkout with --ref or UPLIFT_REFERENCE")
    ref = Path(args.ref)
    up = load_module("ref_uplift_model", ref / "uplift" / "uplift.py")
    tri = load_module("ref_triton_attender", ref / "uplift" / "kernels" / "triton_attender.py")

    cases = []
    gen = torch.Generator().manual_seed(1234)
    for (name, K, I, Cg, C, B, H, W, dt, conv_res, low_mem) in FORWARD_CASES:
        la = up.LocalAttender(Cg, K, conv_res=conv_res, low_mem=low_mem)
        weight = torch.randn(K, Cg, generator=gen) * 0.3
        bias = torch.randn(K, generator=gen) * 0.5
        with torch.no_grad():
            la.conv1.weight.copy_(weight.view(K, Cg, 1, 1))
            la.conv1.bias.copy_(bias)
        la = la.to(dt)
        guide = torch.randn(B, Cg, I * H, I * W, generator=gen).to(dt)
        value = torch.randn(B, C, H, W, generator=gen).to(dt)
        with torch.no_grad():
            out = la(guide, value)
        cases.append(dict(name=name, mode="forward", K=K, I=I, dtype=str(dt), conv_res=conv_res,
                          low_mem=low_mem, hardmax=False, offsets=list(la.offsets), pn=la.pn,
                          guide=guide, value=value, weight=la.conv1.weight.detach().reshape(K, Cg).clone(),
                          bias=la.conv1.bias.detach().clone(), out=out.clone()))
        print(f"{name:28s} out {tuple(out.shape)} {out.dtype}")

    tla = tri.TritonLocalAttender(17)
    for (name, I, C, B, H, W, dt, hardmax) in POOL_CASES:
        att = (torch.randn(B, 17, I * H, I * W, generator=gen) * 2.0).to(dt)
        value = torch.randn(B, C, H, W, generator=gen).to(dt)
        with torch.no_grad():
            out = tla._fallback_forward(att, value, hardmax)
        cases.append(dict(name=name, mode="pool", K=17, I=I, dtype=str(dt), conv_res=False,
                          low_mem=False, hardmax=hardmax, offsets=list(up.LocalAttender(1, 17).offsets),
                          pn=2, logits=att, value=value, out=out.clone()))
        print(f"{name:28s} out {tuple(out.shape)} {out.dtype}")

    meta = dict(torch=torch.__version__, generator="tests/golden/make_golden.py",
                reference_files=["uplift/uplift.py", "uplift/kernels/triton_attender.py"])
    torch.save(dict(meta=meta, cases=cases), HERE / "la_cases.pt")

    # standalone config: LocalAttender(64, 9), fp32, B=1
    guide, value, weight, bias = config1_inputs()
    la = up.LocalAttender(64, 9)
    with torch.no_grad():
        la.conv1.weight.copy_(weight.view(9, 64, 1, 1))
        la.conv1.bias.copy_(bias)
        out = la(guide, value)
    cfg1 = dict(meta=meta, K=9, offsets=list(la.offsets), pn=la.pn,
                sha=dict(guide=tensor_sha(guide), value=tensor_sha(value), weight=tensor_sha(weight)),
                out_every8=out[:, ::8].clone(),
                out_sum=float(out.double().sum()), out_abs_sum=float(out.double().abs().sum()),
                out_shape=list(out.shape))
    torch.save(cfg1, HERE / "la_config1.pt")
    print("config1", tuple(out.shape), cfg1["out_sum"])

    mg = model_golden(ref, up)
    mg["meta"] = meta
    torch.save(mg, HERE / "model_cases.pt")


if __name__ == "__main__":
    sys.exit(main())
