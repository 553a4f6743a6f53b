"""The C-ABI library builds for sm_100a, loads, and exports what
include/*.h declare.  CPU only: argument validation runs before any
CUDA call, so no kernel is launched here."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from uplift_b200 import _native
from uplift_b200.attender import LocalAttender, NEIGHBOURHOODS, neighbourhood

INCLUDE = Path(__file__).resolve().parent.parent / "include"


def declared_functions():
    names = set()
    for header in sorted(INCLUDE.glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(uplift_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    return _native.load(build_if_missing=True)


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert names, "no declarations parsed"
    assert sorted(_native.EXPORTED) == names
    for name in names:
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings(lib):
    assert lib.uplift_la_abi_version() >> 16 == 1
    assert lib.uplift_la_status_string(0) == b"ok"
    assert lib.uplift_la_status_string(_native.ERR_LAYOUT) == b"unsupported layout"


def test_library_is_sm100a_only():
    """The shared object carries sm_100a code (nvcc -gencode compute_100a)."""
    from uplift_b200 import build
    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def _call_forward(lib, **kw):
    s = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    args = dict(guide=None, gs=s, value=None, vs=s, weight=None, bias=None, out=None, os=s,
                B=1, Cg=8, C=4, H=2, W=2, I=2, K=9, offsets=_native.offsets_array(neighbourhood(9)[0]),
                pn=1, conv_res=1, dtype=0, hardmax=0, stream=None)
    args.update(kw)
    return lib.uplift_la_forward(args["guide"], args["gs"], args["value"], args["vs"], args["weight"],
                                 args["bias"], args["out"], args["os"], args["B"], args["Cg"], args["C"],
                                 args["H"], args["W"], args["I"], args["K"], args["offsets"], args["pn"],
                                 args["conv_res"], args["dtype"], args["hardmax"], args["stream"])


def test_validation_errors_without_launch(lib):
    assert _call_forward(lib, dtype=7) == _native.ERR_ARG
    assert _call_forward(lib, K=40) == _native.ERR_SHAPE
    assert _call_forward(lib, I=0) == _native.ERR_SHAPE
    bad = _native.offsets_array([(3, 0)] * 9)
    assert _call_forward(lib, offsets=bad) == _native.ERR_OFFSETS
    nchw = (ctypes.c_int64 * 4)(16, 4, 2, 1)  # channel stride != 1
    assert _call_forward(lib, vs=nchw) == _native.ERR_LAYOUT
    assert b"channel stride" in lib.uplift_la_last_error()
    # valid arguments but null data pointers for a non-empty problem
    s = (ctypes.c_int64 * 4)(32, 1, 16, 8)
    assert _call_forward(lib, vs=s, os=s, gs=s) == _native.ERR_ARG


def test_cta_limit_is_validated(lib):
    """uplift_la_set_max_ctas: n < 0 is an argument error; 0 restores one CTA
    per SM (host-side state only, no device touched)."""
    assert lib.uplift_la_set_max_ctas(-1) == _native.ERR_ARG
    assert lib.uplift_la_set_max_ctas(37) == _native.OK
    assert lib.uplift_la_set_max_ctas(0) == _native.OK


def test_empty_problem_is_a_noop(lib):
    """B = 0: validated and returns OK without touching a device."""
    s = (ctypes.c_int64 * 4)(32, 1, 16, 8)
    assert _call_forward(lib, B=0, vs=s, os=s, gs=s) == _native.OK


def test_python_errors_are_raised(lib):
    with pytest.raises(ValueError, match="unknown dtype"):
        _native.check(_call_forward(lib, dtype=9), "uplift_la_forward")


def test_no_cpu_fallback():
    la = LocalAttender(16, 17)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        la(torch.randn(1, 16, 4, 4), torch.randn(1, 8, 2, 2))


def test_module_api_matches_reference_surface():
    la = LocalAttender(64, 17)
    assert la.num_connected == 17 and la.pn == 2 and la.conv_res and not la.low_mem
    assert list(la.state_dict().keys()) == ["conv1.weight", "conv1.bias"]
    assert tuple(la.conv1.weight.shape) == (17, 64, 1, 1)
    assert len(la.offsets) == 17
    stack = la.make_offsets(torch.randn(2, 3, 5, 4))
    assert stack.shape == (2, 3, 17, 5, 4)
    with pytest.raises(ValueError):
        LocalAttender(8, 7)
    for K, (offs, pn) in NEIGHBOURHOODS.items():
        assert len(offs) == K and max(max(abs(a), abs(b)) for a, b in offs) == pn
