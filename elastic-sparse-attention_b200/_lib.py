"""ctypes binding of libesa_b200.so (the C ABI declared in include/esa_b200.h).

The shared library is built in-tree next to this file (``csrc/Makefile``).
There is no fallback: if the library is missing or a call fails, the error
is raised.  Calls pass raw device pointers plus the current torch CUDA
stream; torch only provides memory and streams.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libesa_b200.so")

ESA_OK = 0
FLAG_GATHER_ONLY = 1
FLAG_F32_DKV = 2     # esa_backward writes dk / dv as float32
DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

# Every symbol exported by include/esa_b200.h.
EXPORTED = ("esa_version", "esa_last_error", "esa_device_errors", "esa_forward_writes_probs",
            "esa_pattern",
            "esa_pattern_audit", "esa_forward", "esa_backward_workspace_size", "esa_backward",
            "esa_key_plan_size", "esa_key_plan_build",
            "esa_backward_noalloc", "esa_trace_enable", "esa_trace_count", "esa_trace_read",
            "esa_probe_gather", "esa_copy_rows",
            # decoder-layer harness (include/esa_layer.h)
            "esa_rmsnorm_forward", "esa_rmsnorm_backward_workspace_size", "esa_rmsnorm_backward",
            "esa_rope_apply", "esa_swiglu_forward", "esa_swiglu_backward")

# ESA_DEVERR_* bits of the per-device error word
DEVERR_KV_RANGE = 1
DEVERR_TIMEOUT = 2
DEVERR_QUERY_RANGE = 4
DEVERR_PLAN = 8


class EsaTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride_b", ctypes.c_int64),
                ("stride_h", ctypes.c_int64), ("stride_s", ctypes.c_int64)]


class EsaRows(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("dst", ctypes.c_void_p),
                ("src_dtype", ctypes.c_int32), ("dst_dtype", ctypes.c_int32),
                ("row_elems", ctypes.c_int64), ("count", ctypes.c_int64 * 3),
                ("src_stride", ctypes.c_int64 * 3), ("dst_stride", ctypes.c_int64 * 3)]


class EsaProblem(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("batch", ctypes.c_int32),
                ("num_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("attn_length", ctypes.c_int32),
                ("layer_idx", ctypes.c_int32), ("num_hidden_layers", ctypes.c_int32),
                ("q_len", ctypes.c_int64), ("kv_len", ctypes.c_int64),
                ("kv_offset", ctypes.c_int64), ("kv_rows", ctypes.c_int64),
                ("row_offset", ctypes.c_int64), ("rows", ctypes.c_void_p),
                ("scale", ctypes.c_float), ("flags", ctypes.c_int32),
                ("dropout_p", ctypes.c_float), ("head_offset", ctypes.c_int32),
                ("dropout_seed", ctypes.c_uint64), ("weights", ctypes.c_void_p),
                ("probs", ctypes.c_void_p), ("pattern_heads", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("key_plan", ctypes.c_void_p),
                ("key_plan_bytes", ctypes.c_uint64)]


class EsaError(RuntimeError):
    """A libesa_b200 entry point returned an error code."""


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load libesa_b200.so once; raise if it is absent (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise EsaError(
                f"libesa_b200.so not found at {LIB_PATH}; build it with "
                "`make -C elastic-sparse-attention_b200/csrc` (or __graft_entry__.build()). "
                "This implementation has no CPU or Triton fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        i32, i64 = ctypes.c_int32, ctypes.c_int64
        lib.esa_version.restype = ctypes.c_int
        lib.esa_last_error.restype = ctypes.c_char_p
        lib.esa_forward_writes_probs.argtypes = [ctypes.POINTER(EsaProblem)]
        lib.esa_forward_writes_probs.restype = ctypes.c_int
        lib.esa_device_errors.argtypes = [i32, ctypes.POINTER(i32), P]
        lib.esa_device_errors.restype = ctypes.c_int
        lib.esa_pattern.argtypes = [i32, i32, i32, i32, i64, P, i64, i64, P, P, P]
        lib.esa_pattern.restype = ctypes.c_int
        lib.esa_pattern_audit.argtypes = [i32, i32, i32, i32, i64, P, P]
        lib.esa_pattern_audit.restype = ctypes.c_int
        lib.esa_forward.argtypes = [ctypes.POINTER(EsaProblem), EsaTensor, EsaTensor, EsaTensor,
                                    EsaTensor, P, P]
        lib.esa_forward.restype = ctypes.c_int
        lib.esa_backward_workspace_size.argtypes = [ctypes.POINTER(EsaProblem)]
        lib.esa_backward_workspace_size.restype = ctypes.c_size_t
        lib.esa_backward.argtypes = [ctypes.POINTER(EsaProblem), EsaTensor, EsaTensor, EsaTensor,
                                     EsaTensor, P, EsaTensor, EsaTensor, EsaTensor, EsaTensor,
                                     P, P, P, ctypes.c_size_t, P]
        lib.esa_backward.restype = ctypes.c_int
        lib.esa_key_plan_size.argtypes = [ctypes.POINTER(EsaProblem)]
        lib.esa_key_plan_size.restype = ctypes.c_size_t
        lib.esa_key_plan_build.argtypes = [ctypes.POINTER(EsaProblem), P, ctypes.c_size_t, P]
        lib.esa_key_plan_build.restype = ctypes.c_int
        lib.esa_trace_enable.argtypes = [i32]
        lib.esa_trace_enable.restype = ctypes.c_int
        lib.esa_trace_count.restype = ctypes.c_int
        lib.esa_trace_read.argtypes = [i32, ctypes.POINTER(ctypes.c_char_p),
                                       ctypes.POINTER(ctypes.c_float)]
        lib.esa_trace_read.restype = ctypes.c_int
        lib.esa_probe_gather.argtypes = [i32, ctypes.POINTER(EsaProblem), EsaTensor, EsaTensor,
                                         P, P]
        lib.esa_probe_gather.restype = ctypes.c_int
        lib.esa_copy_rows.argtypes = [ctypes.POINTER(EsaRows), P]
        lib.esa_copy_rows.restype = ctypes.c_int
        F = ctypes.c_float
        lib.esa_rmsnorm_forward.argtypes = [i32, i64, i32, P, P, P, P, F, P, P, P]
        lib.esa_rmsnorm_forward.restype = ctypes.c_int
        lib.esa_rmsnorm_backward_workspace_size.argtypes = [i64, i32]
        lib.esa_rmsnorm_backward_workspace_size.restype = ctypes.c_size_t
        lib.esa_rmsnorm_backward.argtypes = [i32, i64, i32, P, P, P, P, P, P, P, P,
                                             ctypes.c_size_t, P]
        lib.esa_rmsnorm_backward.restype = ctypes.c_int
        lib.esa_rope_apply.argtypes = [i32, i32, i64, i32, EsaTensor, i32, EsaTensor, i32, P, P,
                                       i32, P]
        lib.esa_rope_apply.restype = ctypes.c_int
        lib.esa_swiglu_forward.argtypes = [i32, i64, i32, P, P, P]
        lib.esa_swiglu_forward.restype = ctypes.c_int
        lib.esa_swiglu_backward.argtypes = [i32, i64, i32, P, P, P, P, P]
        lib.esa_swiglu_backward.restype = ctypes.c_int
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != ESA_OK:
        msg = load().esa_last_error().decode(errors="replace")
        raise EsaError(f"{what} failed (code {rc}): {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def tensor4(t: torch.Tensor) -> EsaTensor:
    """[B, H, L, D] tensor with a contiguous last axis -> EsaTensor."""
    if t.stride(-1) != 1:
        raise ValueError("the head_dim axis must be contiguous")
    return EsaTensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def problem(*, dtype: torch.dtype, batch: int, num_heads: int, num_kv_heads: int, head_dim: int,
            attn_length: int, layer_idx: int, num_hidden_layers: int, q_len: int, kv_len: int,
            kv_offset: int = 0, kv_rows: int | None = None, row_offset: int = 0,
            rows: torch.Tensor | None = None, scale: float, flags: int = 0,
            dropout_p: float = 0.0, dropout_seed: int = 0,
            weights: torch.Tensor | None = None,
            probs: torch.Tensor | None = None, head_offset: int = 0,
            pattern_heads: int = 0, key_plan: torch.Tensor | None = None) -> EsaProblem:
    if dtype not in DTYPES:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, bfloat16 or float16")
    return EsaProblem(DTYPES[dtype], batch, num_heads, num_kv_heads, head_dim, attn_length,
                      layer_idx, num_hidden_layers, q_len, kv_len, kv_offset,
                      kv_len if kv_rows is None else kv_rows, row_offset, ptr(rows), scale, flags,
                      dropout_p, head_offset, dropout_seed, ptr(weights), ptr(probs),
                      pattern_heads, 0, ptr(key_plan),
                      0 if key_plan is None else key_plan.numel())


def trace_records() -> list[tuple[str, float]]:
    """(kernel name, milliseconds) of every launch recorded since
    esa_trace_enable(1); waits for each record's end event."""
    lib = load()
    out = []
    for i in range(lib.esa_trace_count()):
        name, ms = ctypes.c_char_p(), ctypes.c_float()
        check(lib.esa_trace_read(i, ctypes.byref(name), ctypes.byref(ms)), "esa_trace_read")
        out.append((name.value.decode(), float(ms.value)))
    return out
