"""Pin the CPU oracles to golden vectors produced by executing the reference
(tests/golden/make_golden.py).  CPU only."""
import hashlib

import pytest
import torch

from conftest import normwise_err, dtype_of
from oracle import local_attender_oracle as lao
from oracle import c_oracle
from golden.make_golden import config1_inputs


def _run_torch_oracle(case):
    if case["mode"] == "forward":
        return lao.local_attender(case["guide"], case["value"], case["weight"], case["bias"],
                                  K=case["K"], conv_res=case["conv_res"], low_mem=case["low_mem"])
    return lao.pool(case["logits"], case["value"], case["offsets"], case["pn"],
                    hardmax=case["hardmax"])


def test_offset_tables_match_reference(golden_cases):
    seen = set()
    for case in golden_cases:
        K = case["K"]
        if K in seen:
            continue
        seen.add(K)
        offsets, pn = lao.OFFSETS[K]
        assert [tuple(o) for o in case["offsets"]] == offsets
        assert case["pn"] == pn
    assert seen == {5, 9, 13, 17, 25}


def test_torch_oracle_matches_reference(golden_cases):
    """Same op sequence as the reference: identical up to summation order."""
    for case in golden_cases:
        out = _run_torch_oracle(case)
        ref = case["out"]
        assert out.shape == ref.shape, case["name"]
        assert out.dtype == ref.dtype, case["name"]
        dt = dtype_of(case["dtype"])
        tol = 1e-6 if (dt == torch.float32 or case["low_mem"]) else 8e-3
        assert normwise_err(out, ref) <= tol, (case["name"], normwise_err(out, ref))


def test_c_oracle_matches_reference(golden_cases):
    """The double-precision C restatement agrees with the reference to the
    reference's own rounding (fp32: ~1e-6; bf16/fp16 reference rounds its
    softmax weights and products)."""
    for case in golden_cases:
        if case["mode"] == "forward":
            out = c_oracle.forward(case["guide"], case["value"], case["weight"], case["bias"],
                                   case["offsets"], conv_res=case["conv_res"])
        else:
            out = c_oracle.forward(None, case["value"], None, None, case["offsets"],
                                   hardmax=case["hardmax"], logits=case["logits"])
        ref = case["out"]
        dt = dtype_of(case["dtype"])
        tol = {torch.float32: 2e-6, torch.bfloat16: 1.5e-2, torch.float16: 2e-3}[dt]
        assert out.shape == ref.shape
        assert normwise_err(out, ref) <= tol, (case["name"], normwise_err(out, ref))


def test_hardmax_is_exact_selection(golden_cases):
    for case in golden_cases:
        if not case["hardmax"]:
            continue
        out = c_oracle.forward(None, case["value"], None, None, case["offsets"], hardmax=True,
                               logits=case["logits"])
        # the reference's hardmax output is one neighbour value per pixel, exactly
        assert torch.equal(out.to(case["out"].dtype), case["out"]), case["name"]


def test_config1_golden(golden_config1):
    """Standalone fp32 config (K=9, value 384x32x32, guide 64x64x64)."""
    guide, value, weight, bias = config1_inputs()
    sha = lambda t: hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
    assert sha(guide) == golden_config1["sha"]["guide"], "torch CPU RNG changed; regenerate fixtures"
    assert sha(value) == golden_config1["sha"]["value"]
    assert sha(weight) == golden_config1["sha"]["weight"]
    out = lao.local_attender(guide, value, weight, bias, K=9)
    assert list(out.shape) == golden_config1["out_shape"]
    assert normwise_err(out[:, ::8], golden_config1["out_every8"]) <= 1e-6
    assert abs(out.double().sum().item() - golden_config1["out_sum"]) <= 1e-6 * golden_config1["out_abs_sum"]
    out_c = c_oracle.forward(guide, value, weight, bias, golden_config1["offsets"])
    assert normwise_err(out_c[:, ::8], golden_config1["out_every8"]) <= 2e-6


def test_chunked_oracle_equals_whole():
    g = torch.Generator().manual_seed(7)
    guide = torch.randn(2, 16, 22, 14, generator=g)
    value = torch.randn(2, 6, 11, 7, generator=g)
    weight = torch.randn(17, 16, generator=g) * 0.3
    bias = torch.randn(17, generator=g)
    whole = lao.local_attender(guide, value, weight, bias)
    chunked = lao.local_attender_chunked(guide, value, weight, bias, rows_per_chunk=3)
    assert normwise_err(chunked, whole) <= 1e-6


@pytest.mark.parametrize("K", [5, 9, 13, 17, 25])
def test_c_oracle_constant_value_is_identity(K):
    """Softmax weights sum to one: a constant value map comes back unchanged."""
    g = torch.Generator().manual_seed(K)
    guide = torch.randn(1, 8, 6, 8, generator=g)
    value = torch.full((1, 3, 3, 4), 2.5)
    weight = torch.randn(K, 8, generator=g)
    offsets, _ = lao.OFFSETS[K]
    out = c_oracle.forward(guide, value, weight, None, offsets)
    assert torch.allclose(out, torch.full_like(out, 2.5), atol=1e-6)
