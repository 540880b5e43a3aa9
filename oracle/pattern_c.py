"""ctypes binding of ``oracle/pattern_ref.c`` (the C restatement of the pattern).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle_pattern.so")
_lib = None


def build() -> str:
    """Compile the C restatement with ``make`` (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or (
                os.path.getmtime(_SO) < os.path.getmtime(os.path.join(_HERE, "pattern_ref.c"))):
            build()
        lib = ctypes.CDLL(_SO)
        lib.esa_oracle_pattern.argtypes = [
            ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        lib.esa_oracle_pattern.restype = None
        lib.esa_oracle_audit.argtypes = [
            ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.POINTER(ctypes.c_int64)]
        lib.esa_oracle_audit.restype = ctypes.c_int64
        _lib = lib
    return _lib


def elastic_indices(positions, num_heads, attn_length, layer_idx, num_hidden_layers):
    """Same contract as :func:`oracle.pattern.elastic_indices`, computed in C."""
    lib = _load()
    pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int64))
    n = pos.shape[0]
    idx = np.empty((num_heads, n, attn_length), dtype=np.int64)
    mask = np.empty((num_heads, n, attn_length), dtype=np.int64)
    lib.esa_oracle_pattern(num_heads, n, pos.ctypes.data, attn_length, layer_idx,
                           num_hidden_layers, idx.ctypes.data, mask.ctypes.data)
    return idx, mask


def audit_monotone(num_heads, seq_len, attn_length, layer_idx, num_hidden_layers):
    """(violations, max_step) of the raw per-slot index columns over rows 0..L-1."""
    lib = _load()
    step = ctypes.c_int64(0)
    bad = lib.esa_oracle_audit(num_heads, seq_len, attn_length, layer_idx,
                               num_hidden_layers, ctypes.byref(step))
    return int(bad), int(step.value)
