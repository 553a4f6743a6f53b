"""ctypes binding of the C ABI in include/uplift_la.h.

This is the only way the package reaches the GPU kernels.  Loading fails
loudly (RuntimeError) when the library is missing: there is no CPU or
PyTorch fallback anywhere in the product path.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

from . import build as _build

F32, BF16, F16 = 0, 1, 2
OK, ERR_ARG, ERR_SHAPE, ERR_LAYOUT, ERR_OFFSETS, ERR_CUDA, ERR_NO_DEVICE, ERR_UNSUPPORTED = range(8)
MAX_K = 25
MAX_PN = 4
NOALLOC_MAX_PROBS = 8 * 1024 * 1024  # floats, UPLIFT_LA_NOALLOC_MAX_PROBS

# every symbol include/uplift_la.h declares
EXPORTED = (
    "uplift_la_forward",
    "uplift_la_forward_resized",
    "uplift_la_forward_fused_guide",
    "uplift_la_pool",
    "uplift_la_last_error",
    "uplift_la_status_string",
    "uplift_la_abi_version",
    "uplift_la_set_kernel_policy",
    "uplift_la_last_kernel",
    "uplift_la_device_status",
    "uplift_la_test_hook",
    "uplift_la_set_host_status_word",
    "uplift_la_set_max_ctas",
    "uplift_la_backward",
    "uplift_la_backward_noalloc",
    # include/uplift_glue.h
    "uplift_resize_bilinear",
    "uplift_resize_nearest",
    "uplift_add_channels",
    "uplift_bias_act",
    "uplift_layernorm_act",
)
POLICY_AUTO, POLICY_SIMT, POLICY_TENSOR_CORE = 0, 1, 2
KERNEL_SIMT, KERNEL_TENSOR_CORE, KERNEL_SIMT_STAGED, KERNEL_TENSOR_CORE_WIDE = 1, 2, 3, 4
KERNEL_TENSOR_CORE_RESIZE = 5
KERNEL_TENSOR_CORE_GUIDE, KERNEL_TENSOR_CORE_GUIDE_RESIZE = 6, 7
KERNELS_CUDA_CORE = (KERNEL_SIMT, KERNEL_SIMT_STAGED)

_lib = None
_lock = threading.Lock()

_I64_4 = ctypes.c_int64 * 4


def lib_path() -> Path:
    """The in-tree library, or the file named by UPLIFT_LA_LIBRARY."""
    override = os.environ.get("UPLIFT_LA_LIBRARY")
    return Path(override) if override else _build.lib_path()


def load(build_if_missing: bool = False):
    """Load libuplift_la.so once; raise RuntimeError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not path.exists():
            if build_if_missing:
                _build.build()
            else:
                raise RuntimeError(
                    f"uplift_b200 CUDA library not found at {path}; build it with "
                    "`python -m uplift_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(str(path))
        vp, i, i64p = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)
        i8p, fp = ctypes.POINTER(ctypes.c_int8), ctypes.c_void_p
        lib.uplift_la_forward.restype = i
        lib.uplift_la_forward.argtypes = [vp, i64p, vp, i64p, fp, fp, vp, i64p,
                                          i, i, i, i, i, i, i, i8p, i, i, i, i, vp]
        lib.uplift_la_forward_resized.restype = i
        lib.uplift_la_forward_resized.argtypes = [vp, i64p, vp, i64p, fp, fp, vp, i64p,
                                                  i, i, i, i, i, i, i, i8p, i, i, i, i, i, i, vp]
        lib.uplift_la_forward_fused_guide.restype = i
        lib.uplift_la_forward_fused_guide.argtypes = [vp, i64p, vp, i64p, fp, fp, vp, i64p, fp, fp, vp, i64p,
                                                      i, i, i, i, i, i, i, i8p, i, i, i, i, i, i, vp]
        lib.uplift_la_pool.restype = i
        lib.uplift_la_pool.argtypes = [vp, i64p, vp, i64p, vp, i64p,
                                       i, i, i, i, i, i, i8p, i, i, i, vp]
        lib.uplift_la_last_error.restype = ctypes.c_char_p
        lib.uplift_la_last_error.argtypes = []
        lib.uplift_la_status_string.restype = ctypes.c_char_p
        lib.uplift_la_status_string.argtypes = [i]
        lib.uplift_la_abi_version.restype = i
        lib.uplift_la_abi_version.argtypes = []
        lib.uplift_la_set_kernel_policy.restype = i
        lib.uplift_la_set_kernel_policy.argtypes = [i]
        lib.uplift_la_last_kernel.restype = i
        lib.uplift_la_last_kernel.argtypes = []
        lib.uplift_la_device_status.restype = i
        lib.uplift_la_device_status.argtypes = [i]
        lib.uplift_la_test_hook.restype = i
        lib.uplift_la_test_hook.argtypes = [i, ctypes.c_ulonglong]
        lib.uplift_la_set_host_status_word.restype = i
        lib.uplift_la_set_host_status_word.argtypes = [vp]
        lib.uplift_la_set_max_ctas.restype = i
        lib.uplift_la_set_max_ctas.argtypes = [i]
        lib.uplift_la_backward.restype = i
        lib.uplift_la_backward.argtypes = [vp, i64p, vp, i64p, vp, i64p, fp, fp, fp, vp, i64p, vp, i64p,
                                           fp, fp, i, i, i, i, i, i, i, i8p, i, i, i, i, vp]
        lib.uplift_la_backward_noalloc.restype = i
        lib.uplift_la_backward_noalloc.argtypes = [vp, i64p, vp, i64p, vp, i64p, fp, fp, vp, i64p, vp, i64p,
                                                   fp, fp, i, i, i, i, i, i, i, i8p, i, i, i, i, vp]
        lib.uplift_resize_bilinear.restype = i
        lib.uplift_resize_bilinear.argtypes = [vp, i64p, vp, i64p, i, i, i, i, i, i, i, i, i, vp]
        lib.uplift_resize_nearest.restype = i
        lib.uplift_resize_nearest.argtypes = [vp, i64p, vp, i64p, i, i, i, i, i, i, i, vp]
        lib.uplift_add_channels.restype = i
        lib.uplift_add_channels.argtypes = [vp, i64p, vp, i64p, i, i, i, i, i, vp]
        lib.uplift_bias_act.restype = i
        lib.uplift_bias_act.argtypes = [vp, i64p, vp, vp, i64p, i, i, i, i, i, i, i, vp]
        lib.uplift_layernorm_act.restype = i
        lib.uplift_layernorm_act.argtypes = [vp, i64p, vp, vp, vp, ctypes.c_float, i, i, i, i, i, i, vp]
        _lib = lib
    return _lib


def strides(t) -> "ctypes.Array":
    return _I64_4(*[int(s) for s in t.stride()])


def offsets_array(offsets):
    flat = [int(v) for off in offsets for v in off]
    return (ctypes.c_int8 * len(flat))(*flat)


def check(rc: int, what: str) -> None:
    """Turn a status code into a Python exception."""
    if rc == OK:
        return
    lib = load()
    msg = lib.uplift_la_last_error().decode(errors="replace")
    name = lib.uplift_la_status_string(rc).decode()
    text = f"{what}: {name} ({rc}): {msg}"
    if rc in (ERR_ARG, ERR_SHAPE, ERR_LAYOUT, ERR_OFFSETS):
        raise ValueError(text)
    raise RuntimeError(text)


class kernel_policy:
    """Context manager selecting the kernel family (AUTO / SIMT / TENSOR_CORE)."""

    def __init__(self, policy: int):
        self.policy = policy

    def __enter__(self):
        check(load().uplift_la_set_kernel_policy(self.policy), "uplift_la_set_kernel_policy")
        return self

    def __exit__(self, *exc):
        load().uplift_la_set_kernel_policy(POLICY_AUTO)
        return False


def last_kernel() -> int:
    return load().uplift_la_last_kernel()


def set_max_ctas(n: int) -> None:
    """Cap the persistent tensor-core kernels at n CTAs (0: one per SM), so
    that communication kernels running beside them get SMs of their own
    (uplift_la_set_max_ctas)."""
    check(load().uplift_la_set_max_ctas(int(n)), "uplift_la_set_max_ctas")


def device_status(clear: bool = True) -> int:
    """0 if every tensor-core launch completed its pipeline (synchronises)."""
    return load().uplift_la_device_status(int(clear))


ROLES = {1: "producer", 2: "MMA issuer", 3: "softmax / split", 4: "epilogue"}


class ExpiredWaitError(RuntimeError):
    """A tensor-core launch gave up on a bounded wait: the tiles it had not
    finished were never written, so that launch's output is incomplete."""


class HostStatus:
    """The host-visible status word of the tensor-core kernels
    (uplift_la_set_host_status_word): one pinned int32 that a launch whose
    bounded wait expired writes the failing role into.  Registered on the
    first kernel launch of the process; `raise_if_set()` is a plain memory
    read (no synchronisation), called before every launch, so an expiry
    surfaces as ExpiredWaitError at the first call after the failed kernel
    has finished."""

    def __init__(self):
        self._buf = None
        self._word = None

    def ensure(self):
        if self._buf is None:
            import torch
            with _lock:
                if self._buf is None:
                    buf = torch.zeros(1, dtype=torch.int32, pin_memory=True)
                    check(load().uplift_la_set_host_status_word(buf.data_ptr()),
                          "uplift_la_set_host_status_word")
                    self._word = ctypes.c_uint32.from_address(buf.data_ptr())
                    self._buf = buf

    def value(self) -> int:
        return 0 if self._word is None else int(self._word.value)

    def clear(self) -> None:
        if self._word is not None:
            self._word.value = 0

    def raise_if_set(self) -> None:
        if self._word is None:
            import torch
            if not torch.cuda.is_current_stream_capturing():  # no host allocation inside a capture
                self.ensure()
            return
        code = self._word.value
        if code:
            self._word.value = 0
            load().uplift_la_device_status(1)  # clear the device copy too (error path: synchronises)
            raise ExpiredWaitError(
                f"a Local Attender tensor-core launch on this process gave up after a bounded wait "
                f"(role: {ROLES.get(code, code)}); its output is incomplete and must not be used")


host_status = HostStatus()
