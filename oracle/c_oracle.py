"""ctypes binding of the double-precision C oracle (oracle/la_oracle.c) --
test infrastructure only."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import torch

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libla_oracle.so"
_lib = None


def build() -> Path:
    """Compile the C oracle with gcc (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        src = _HERE / "la_oracle.c"
        if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        fp = ctypes.POINTER(ctypes.c_float)
        lib.la_oracle_forward.restype = ctypes.c_int
        lib.la_oracle_forward.argtypes = [fp, fp, fp, fp, fp, fp] + [ctypes.c_int] * 7 + [
            ctypes.POINTER(ctypes.c_int8), ctypes.c_int, ctypes.c_int]
        _lib = lib
    return _lib


def _f32(t):
    if t is None:
        return None, None
    a = np.ascontiguousarray(t.detach().to(torch.float32).contiguous().numpy())
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def forward(guide, value, weight, bias, offsets, conv_res=True, hardmax=False, logits=None):
    """fp32 result of the double-precision oracle, as an NCHW torch tensor.
    Inputs are CPU tensors of any float dtype (rounded values are used as
    given); weight is [K, Cg] (or [K, Cg, 1, 1]); offsets a list of (dy, dx)."""
    lib = _load()
    B, C, H, W = value.shape
    K = len(offsets)
    if logits is not None:
        Ho, Wo = logits.shape[2], logits.shape[3]
        Cg = 0
    else:
        Ho, Wo = guide.shape[2], guide.shape[3]
        Cg = guide.shape[1]
    I = Ho // H if H else 1
    g_a, g_p = _f32(guide) if logits is None else (None, None)
    v_a, v_p = _f32(value)
    w_a, w_p = _f32(weight.reshape(K, -1)) if logits is None else (None, None)
    b_a, b_p = _f32(bias) if (bias is not None and logits is None) else (None, None)
    l_a, l_p = _f32(logits)
    out = np.empty((B, C, Ho, Wo), dtype=np.float32)
    off = np.asarray(offsets, dtype=np.int8).reshape(-1)
    rc = lib.la_oracle_forward(g_p, v_p, w_p, b_p, l_p,
                               out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                               B, Cg, C, H, W, I, K,
                               off.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)),
                               int(bool(conv_res)), int(bool(hardmax)))
    if rc != 0:
        raise ValueError(f"la_oracle_forward failed ({rc})")
    del g_a, v_a, w_a, b_a, l_a
    return torch.from_numpy(out)
