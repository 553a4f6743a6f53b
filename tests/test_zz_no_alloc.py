"""uplift_la_backward_noalloc: the backward for callers that cannot allocate
device memory (a host whose pool owns all device memory, code that must not
let cudaMalloc / cudaFree synchronise the device, an FFI binding without a
device allocator).  Its softmax-weight workspace is a fixed array inside the
library, shared by every call, so each call must give the same gradients as
uplift_la_backward with a caller workspace, also when the previous call left
other contents in the array.  Collected last on purpose: the array is
module-global state of the library."""
import ctypes

import pytest
import torch

from conftest import normwise_err
from uplift_b200 import _native
from uplift_b200.attender import neighbourhood

DEV = "cuda:0"
_DT = {torch.float32: _native.F32, torch.bfloat16: _native.BF16, torch.float16: _native.F16}


def _case(K, I, B, Cg, C, H, W, dt, seed):
    g = torch.Generator().manual_seed(seed)
    cl = torch.channels_last
    return dict(
        guide=torch.randn(B, Cg, I * H, I * W, generator=g).to(dt).to(DEV).contiguous(memory_format=cl),
        value=torch.randn(B, C, H, W, generator=g).to(dt).to(DEV).contiguous(memory_format=cl),
        dout=torch.randn(B, C, I * H, I * W, generator=g).to(dt).to(DEV).contiguous(memory_format=cl),
        weight=(torch.randn(K, Cg, generator=g) * 0.1).to(DEV),
        bias=(torch.randn(K, generator=g) * 0.5).to(DEV),
        K=K, I=I)


def _grads(lib, c, noalloc):
    """One backward through the C ABI; the test (the caller) allocates the
    inputs and outputs, and the workspace only for the allocating entry."""
    g, v, d, w, b, K, I = c["guide"], c["value"], c["dout"], c["weight"], c["bias"], c["K"], c["I"]
    B, C, H, W = v.shape
    Cg = g.shape[1]
    offsets, pn = neighbourhood(K)
    offsets = c.get("offsets", offsets)
    hardmax = int(c.get("hardmax", False))
    dg = torch.empty_like(g, memory_format=torch.channels_last)
    dv = torch.empty_like(v, memory_format=torch.channels_last)
    dw = torch.zeros(K, Cg, device=DEV)
    db = torch.zeros(K, device=DEV)
    common = [d.data_ptr(), _native.strides(d), g.data_ptr(), _native.strides(g), v.data_ptr(), _native.strides(v),
              w.data_ptr(), b.data_ptr()]
    tail = [dg.data_ptr(), _native.strides(dg), dv.data_ptr(), _native.strides(dv), dw.data_ptr(), db.data_ptr(),
            B, Cg, C, H, W, I, K, _native.offsets_array(offsets), pn, 1, _DT[v.dtype], hardmax,
            torch.cuda.current_stream().cuda_stream]
    if noalloc:
        rc = lib.uplift_la_backward_noalloc(*common, *tail)
    else:
        probs = torch.empty(B * I * H * I * W * K, device=DEV)
        rc = lib.uplift_la_backward(*common, probs.data_ptr(), *tail)
    assert rc == _native.OK, lib.uplift_la_last_error().decode()
    torch.cuda.synchronize()
    return dg, dv, dw, db


@pytest.mark.gpu
def test_noalloc_matches_backward_on_two_calls(cuda_lib):
    """Calls in a row (a larger bf16 problem, then a smaller fp32 one over
    the first call's leftovers in the shared array, then a permuted offset
    table -- the general dV kernel -- with hardmax, which reads the array in
    other patterns) against the allocating entry point on the same inputs."""
    permuted = _case(17, 2, 1, 32, 24, 9, 11, torch.float32, seed=3)
    offsets, _ = neighbourhood(17)
    permuted["offsets"] = offsets[5:] + offsets[:5]
    permuted["hardmax"] = True
    cases = [_case(17, 2, 2, 64, 48, 20, 18, torch.bfloat16, seed=1),
             _case(9, 3, 1, 24, 16, 7, 9, torch.float32, seed=2),
             permuted]
    for c in cases:
        got = _grads(cuda_lib, c, noalloc=True)
        exp = _grads(cuda_lib, c, noalloc=False)
        for name, x, y in zip(("dguide", "dvalue", "dweight", "dbias"), got, exp):
            # dguide / dvalue come from the same deterministic kernels; dW / db
            # are reduced with atomic adds, so only their order may differ
            assert normwise_err(x.float(), y.float()) <= 1e-6, (c["K"], name)


def test_noalloc_rejects_workspace_above_maximum(cuda_lib):
    """B*(I*H)*(I*W)*K above the fixed maximum fails with a clear error
    before any CUDA call (so this runs without a GPU too; the pointers are
    placeholders that nothing dereferences)."""
    s = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    K, I = 17, 2
    offsets, pn = neighbourhood(K)
    H = W = 512  # 1 x 1024 x 1024 x 17 floats > 8 Mi floats
    p = 256
    rc = cuda_lib.uplift_la_backward_noalloc(p, s, p, s, p, s, p, None, None, s, None, s, None, None,
                                             1, 64, 8, H, W, I, K, _native.offsets_array(offsets), pn, 1,
                                             _native.F32, 0, None)
    assert rc == _native.ERR_SHAPE
    msg = cuda_lib.uplift_la_last_error().decode()
    assert "maximum" in msg and str(_native.NOALLOC_MAX_PROBS) in msg


def test_noalloc_reports_bad_arguments_before_the_size_limit(cuda_lib):
    """An invalid call that is also too large names its bad argument (here
    an unknown storage type), not the workspace limit."""
    s = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    offsets, pn = neighbourhood(17)
    p = 256
    rc = cuda_lib.uplift_la_backward_noalloc(p, s, p, s, p, s, p, None, None, s, None, s, None, None,
                                             1, 64, 8, 512, 512, 2, 17, _native.offsets_array(offsets), pn, 1,
                                             7, 0, None)
    assert rc == _native.ERR_ARG
    assert "dtype" in cuda_lib.uplift_la_last_error().decode()
