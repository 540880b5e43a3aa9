"""Tensor-level calls of the decoder-layer harness kernels (include/esa_layer.h):
RMSNorm with a fused residual add, rotary embedding in place, SwiGLU.

Like ``ops``, torch only allocates memory and provides the stream; every
kernel is in libesa_b200.so and there is no fallback.
"""
from __future__ import annotations

import torch

from . import _lib
from .ops import _check_device, _on


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype not in _lib.DTYPES:
        raise TypeError(f"unsupported dtype {t.dtype}")
    return _lib.DTYPES[t.dtype]


def _rows(t: torch.Tensor, dim: int) -> int:
    if not t.is_contiguous() or t.shape[-1] != dim:
        raise ValueError("row operands must be contiguous with the feature axis last")
    return t.numel() // dim


def rmsnorm_forward(x: torch.Tensor, weight: torch.Tensor, eps: float,
                    residual: torch.Tensor | None = None):
    """(h, y, rstd): h = x + residual (x itself without a residual), y =
    h * rstd * weight, rstd float32 per row."""
    dev = _check_device(x, weight)
    dim = x.shape[-1]
    n = _rows(x, dim)
    y = torch.empty_like(x)
    rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=dev)
    h = x
    if residual is not None:
        if residual.shape != x.shape or residual.dtype != x.dtype:
            raise ValueError("residual must match x")
        _rows(residual, dim)
        h = torch.empty_like(x)
    lib = _lib.load()
    with _on(dev):
        _lib.check(lib.esa_rmsnorm_forward(
            _dtype_code(x), n, dim, x.data_ptr(), _lib.ptr(residual),
            h.data_ptr() if residual is not None else None, weight.data_ptr(), eps,
            y.data_ptr(), rstd.data_ptr(), _lib.stream_handle(dev)), "esa_rmsnorm_forward")
    return h, y, rstd


def rmsnorm_backward(h: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor,
                     dy: torch.Tensor, dh_in: torch.Tensor | None = None):
    """(dh, dweight) of :func:`rmsnorm_forward`; dh includes dh_in."""
    dev = _check_device(h, weight, rstd, dy)
    dim = h.shape[-1]
    n = _rows(h, dim)
    dy = dy.contiguous()
    if dh_in is not None:
        dh_in = dh_in.contiguous()
    dh = torch.empty_like(h)
    dw = torch.empty_like(weight)
    lib = _lib.load()
    need = lib.esa_rmsnorm_backward_workspace_size(n, dim)
    ws = torch.empty(max(int(need), 16), dtype=torch.uint8, device=dev)
    with _on(dev):
        _lib.check(lib.esa_rmsnorm_backward(
            _dtype_code(h), n, dim, h.data_ptr(), weight.data_ptr(), rstd.data_ptr(),
            dy.data_ptr(), _lib.ptr(dh_in), dh.data_ptr(), dw.data_ptr(), ws.data_ptr(),
            ws.numel(), _lib.stream_handle(dev)), "esa_rmsnorm_backward")
    return dh, dw


def rope_inv_freq(head_dim: int, base: float, device) -> torch.Tensor:
    """1 / base^(2i / head_dim) for i < head_dim / 2, float32 (the usual
    Llama-style table: integer exponents 0, 2, ... divided by head_dim)."""
    exps = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
    return (1.0 / (base ** exps)).to(device=device, dtype=torch.float32)


def rope_(q: torch.Tensor, k: torch.Tensor | None, inv_freq: torch.Tensor,
          positions: torch.Tensor | None = None, inverse: bool = False) -> None:
    """Rotate q [B, Hq, L, D] and k [B, Hk, L, D] (strided views with a
    contiguous D axis, e.g. parts of a QKV projection buffer) in place.
    ``inverse`` rotates back (the backward, applied to gradients)."""
    dev = _check_device(q, inv_freq)
    B, Hq, L, D = q.shape
    if k is not None and (k.shape[0] != B or k.shape[2] != L or k.shape[3] != D or
                          k.dtype != q.dtype):
        raise ValueError("q and k must share batch, length, head_dim and dtype")
    if positions is not None:
        positions = positions.to(device=dev, dtype=torch.int64).contiguous()
        if positions.numel() != L:
            raise ValueError("positions must hold one entry per row")
    empty = _lib.EsaTensor(None, 0, 0, 0)
    lib = _lib.load()
    with _on(dev):
        _lib.check(lib.esa_rope_apply(
            _dtype_code(q), B, L, D, _lib.tensor4(q), Hq,
            _lib.tensor4(k) if k is not None else empty, k.shape[1] if k is not None else 0,
            _lib.ptr(positions), inv_freq.data_ptr(), 1 if inverse else 0,
            _lib.stream_handle(dev)), "esa_rope_apply")


def swiglu_forward(gate_up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up for rows [gate | up] of width 2 * ffn."""
    dev = _check_device(gate_up)
    ffn = gate_up.shape[-1] // 2
    n = _rows(gate_up, 2 * ffn)
    out = torch.empty(gate_up.shape[:-1] + (ffn,), dtype=gate_up.dtype, device=dev)
    lib = _lib.load()
    with _on(dev):
        _lib.check(lib.esa_swiglu_forward(_dtype_code(gate_up), n, ffn, gate_up.data_ptr(),
                                          out.data_ptr(), _lib.stream_handle(dev)),
                   "esa_swiglu_forward")
    return out


def swiglu_backward(gate_up: torch.Tensor, dout: torch.Tensor, recompute: bool = True):
    """(d gate_up, forward output recomputed or None)."""
    dev = _check_device(gate_up, dout)
    ffn = gate_up.shape[-1] // 2
    n = _rows(gate_up, 2 * ffn)
    dout = dout.contiguous()
    dgu = torch.empty_like(gate_up)
    out = (torch.empty(gate_up.shape[:-1] + (ffn,), dtype=gate_up.dtype, device=dev)
           if recompute else None)
    lib = _lib.load()
    with _on(dev):
        _lib.check(lib.esa_swiglu_backward(_dtype_code(gate_up), n, ffn, gate_up.data_ptr(),
                                           dout.data_ptr(), dgu.data_ptr(), _lib.ptr(out),
                                           _lib.stream_handle(dev)), "esa_swiglu_backward")
    return dgu, out
