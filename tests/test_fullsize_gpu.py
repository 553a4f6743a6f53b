"""The attender at the sizes of the 1022 px DINOv2 upsampler (features 73^2,
iters=4), B=8 images per GPU, bf16: the first level (73^2 -> 146^2, ragged
tiles in both directions) and the last (584^2 -> 1168^2: an output of
8 x 384 x 1168^2 = 4.19 G elements, past 2^31), each against the
double-precision oracle on bands of output rows at the top, the middle and
the bottom of the first and the last image (every band spans the full
width, so the last, ragged column tiles are included).  A band is computed
by the oracle from its value rows plus the +-pn halo, which gives exactly
the whole-image result on those rows."""
import pytest
import torch

from conftest import normwise_err
from oracle import c_oracle
from uplift_b200 import _native, ops
from uplift_b200.attender import neighbourhood

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TC_TOL = 8e-3  # the tensor-core kernel's bound against the fp64 oracle (bf16)


def _band_oracle(guide, value, w, b, offsets, pn, b_idx, r0, r1):
    """Oracle output rows [r0, r1) (output coordinates, I = 2) of image b_idx."""
    H = value.shape[2]
    c0, c1 = r0 // 2, (r1 + 1) // 2
    lo, hi = max(0, c0 - pn), min(H, c1 + pn)
    g = guide[b_idx:b_idx + 1, :, 2 * lo:2 * hi].cpu()
    v = value[b_idx:b_idx + 1, :, lo:hi].cpu()
    full = c_oracle.forward(g, v, w.cpu(), b.cpu(), offsets)
    return full[:, :, r0 - 2 * lo:r1 - 2 * lo]


@pytest.mark.parametrize("side", [73, 584])
def test_dinov2_1022_levels_vs_oracle_bands(side, cuda_lib):
    K, dt, B, C = 17, torch.bfloat16, 8, 384
    offsets, pn = neighbourhood(K)
    g = torch.Generator(device=DEV).manual_seed(side)
    cl = torch.channels_last
    guide = torch.randn(B, 64, 2 * side, 2 * side, generator=g, device=DEV).to(dt).contiguous(memory_format=cl)
    value = torch.randn(B, C, side, side, generator=g, device=DEV).to(dt).contiguous(memory_format=cl)
    w = (torch.randn(K, 64, generator=g, device=DEV) * 0.3).to(dt).float()
    b = torch.randn(K, generator=g, device=DEV) * 0.5
    out = ops.local_attender_raw(guide, value, w, b, offsets, pn)
    torch.cuda.synchronize()
    assert _native.last_kernel() == _native.KERNEL_TENSOR_CORE
    assert out.shape == (B, C, 2 * side, 2 * side)
    Ho = 2 * side
    for b_idx in (0, B - 1):
        for r0 in (0, Ho // 2 - 5, Ho - 8):
            r1 = r0 + 8
            exp = _band_oracle(guide, value, w, b, offsets, pn, b_idx, r0, r1)
            got = out[b_idx:b_idx + 1, :, r0:r1]
            err = normwise_err(got, exp)
            assert err <= TC_TOL, (side, b_idx, r0, err)
    assert torch.isfinite(out[B - 1, :, -2:, -2:].float()).all()  # the last elements, past 2^31
    assert _native.device_status(clear=True) == 0
