"""CPU oracle for the UPLiFT Local Attender -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path (``uplift_b200``) never
calls it and fails loudly when its CUDA library is missing.

It restates, with torch CPU tensor ops in the storage dtype of the inputs,
the reference's non-fast Local Attender:

* offset tables and padding numbers   -- uplift/uplift.py:746-760
* residual_auto (truncate / zero-pad) -- uplift/uplift.py:26-39
* conv1 1x1 projection + residual     -- uplift/uplift.py:765, :810-812
* replicate-padded neighbour gather   -- uplift/uplift.py:784-798, :823
* softmax over K, child mapping       -- uplift/uplift.py:828-830
* parallel pooling                    -- uplift/uplift.py:835-837
* serial low_mem pooling (fp32 accumulator, returns fp32)
                                      -- uplift/uplift.py:840-846
* hardmax (one-hot of argmax) of the Triton module's fallback
                                      -- uplift/kernels/triton_attender.py:421-424

The op sequence (conv -> add -> softmax -> product -> sum over K) is the
reference's, so bf16 inputs are rounded at the same points as in the
reference.  Parity of this restatement is pinned against golden vectors
produced by executing the reference itself (tests/golden/make_golden.py,
checked by tests/test_oracle_golden.py).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

# (offsets, pn) per neighbourhood size; order matters (it is the K axis order
# of the logits).  uplift/uplift.py:746-760.
OFFSETS: dict[int, tuple[list[tuple[int, int]], int]] = {
    5: ([(-1, 0), (0, -1), (0, 0), (0, 1), (1, 0)], 1),
    9: ([(dy, dx) for dy in (-1, 0, 1) for dx in (-1, 0, 1)], 1),
    13: ([(-2, 0)] + [(-1, d) for d in (-1, 0, 1)] + [(0, d) for d in (-2, -1, 0, 1, 2)]
         + [(1, d) for d in (-1, 0, 1)] + [(2, 0)], 2),
    17: ([(-2, d) for d in (-2, 0, 2)] + [(-1, d) for d in (-1, 0, 1)]
         + [(0, d) for d in (-2, -1, 0, 1, 2)] + [(1, d) for d in (-1, 0, 1)]
         + [(2, d) for d in (-2, 0, 2)], 2),
    25: ([(dy, dx) for dy in (-2, -1, 0, 1, 2) for dx in (-2, -1, 0, 1, 2)], 2),
}


def residual_auto(x1: torch.Tensor, x2: torch.Tensor) -> torch.Tensor:
    """x2 plus x1 truncated or zero-padded to x2's channel count
    (uplift/uplift.py:26-39)."""
    c1, c2 = x1.shape[1], x2.shape[1]
    if c1 == c2:
        return x1 + x2
    if c1 > c2:
        return x1[:, :c2] + x2
    padded = torch.zeros_like(x2)
    padded[:, :c1] = x1
    return padded + x2


def neighbour_stack(value: torch.Tensor, offsets, pn: int) -> torch.Tensor:
    """[B, C, H, W] -> [B, C, K, H, W]: the value map shifted by each offset
    with replicate padding (uplift/uplift.py:784-798), written as a clamped
    index gather."""
    _, _, H, W = value.shape
    rows = torch.arange(H)
    cols = torch.arange(W)
    shifted = []
    for dy, dx in offsets:
        assert abs(dy) <= pn and abs(dx) <= pn
        ry = (rows + dy).clamp(0, H - 1)
        rx = (cols + dx).clamp(0, W - 1)
        shifted.append(value.index_select(2, ry).index_select(3, rx))
    return torch.stack(shifted, dim=2)


def project_logits(guide, weight, bias, conv_res=True):
    """conv1 (1x1, bias) + residual_auto (uplift/uplift.py:810-812).
    weight is [K, Cg] or [K, Cg, 1, 1]; bias [K] or None."""
    K = weight.shape[0]
    w4 = weight.reshape(K, -1, 1, 1).to(guide.dtype)
    b = None if bias is None else bias.to(guide.dtype)
    att = F.conv2d(guide, w4, b)
    if conv_res:
        att = residual_auto(guide, att)
    return att


def pool(att, value, offsets, pn, low_mem=False, hardmax=False):
    """Softmax over K and softmax-weighted neighbour sum
    (uplift/uplift.py:813-847); hardmax as in
    uplift/kernels/triton_attender.py:421-424."""
    B, C, H, W = value.shape
    K = att.shape[1]
    Ho, Wo = att.shape[2], att.shape[3]
    I = Ho // H
    assert I * H == Ho and I * W == Wo, "output size must be an integer multiple of the value size"
    x = neighbour_stack(value, offsets, pn).unsqueeze(4).unsqueeze(6)  # [B,C,K,H,1,W,1]
    if hardmax:
        a = F.one_hot(att.argmax(dim=1), num_classes=K).permute(0, 3, 1, 2).to(value.dtype)
    else:
        a = F.softmax(att, dim=1)
    a = a.reshape(B, K, H, I, W, I).unsqueeze(1)  # [B,1,K,H,I,W,I]
    if not low_mem:
        return (x * a).sum(dim=2).reshape(B, C, Ho, Wo)
    res = torch.zeros([B, C, Ho, Wo])  # fp32 accumulator, as the reference
    for k in range(K):
        res += (x[:, :, k] * a[:, :, k]).reshape(B, C, Ho, Wo)
    return res


def local_attender(guide, value, weight, bias, K=None, conv_res=True, low_mem=False,
                   hardmax=False, offsets=None, pn=None):
    """Full Local Attender forward on CPU tensors (NCHW or channels_last).
    Returns [B, C, I*H, I*W] in value.dtype (fp32 when low_mem, like the
    reference)."""
    K = weight.shape[0] if K is None else K
    if offsets is None:
        offsets, pn = OFFSETS[K]
    att = project_logits(guide, weight, bias, conv_res)
    return pool(att, value, offsets, pn, low_mem=low_mem, hardmax=hardmax)


def local_attender_chunked(guide, value, weight, bias, conv_res=True, hardmax=False,
                           rows_per_chunk=8, offsets=None, pn=None, out_dtype=None):
    """Same result as local_attender (parallel pooling), computed one image
    and one band of coarse rows at a time so that full-size shapes fit in
    host memory.  Each band is given its +-pn halo rows of value, so the
    replicate padding only acts at the true image border."""
    K = weight.shape[0]
    if offsets is None:
        offsets, pn = OFFSETS[K]
    B, C, H, W = value.shape
    I = guide.shape[2] // H
    out = torch.empty(B, C, I * H, I * W, dtype=out_dtype or value.dtype)
    for b in range(B):
        for h0 in range(0, H, rows_per_chunk):
            h1 = min(H, h0 + rows_per_chunk)
            lo, hi = max(0, h0 - pn), min(H, h1 + pn)
            v = value[b:b + 1, :, lo:hi]
            # rows of the band inside the halo-extended crop; crop rows outside
            # [h0, h1) are computed and discarded.
            g = guide[b:b + 1, :, lo * I:hi * I]
            att = project_logits(g, weight, bias, conv_res)
            o = pool(att, v, offsets, pn, hardmax=hardmax)
            out[b:b + 1, :, h0 * I:h1 * I] = o[:, :, (h0 - lo) * I:(h1 - lo) * I]
    return out
