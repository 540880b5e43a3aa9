"""Tensor-level calls into libesa_b200 (forward, backward, pattern, audit).

Each function allocates its outputs and workspace with torch (the C ABI never
allocates), then launches on the current CUDA stream of the input's device.
"""
from __future__ import annotations

import contextlib
import ctypes
from dataclasses import dataclass

import torch

from . import _lib

# Positions are handled in exact float32 arithmetic only below 2^24.
MAX_POSITION = 1 << 24


@dataclass(frozen=True)
class PatternSpec:
    """The elastic pattern of one layer (reference __init__ arguments, :375-386).

    ``pattern_heads`` / ``head_offset``: the tensors of a call hold query heads
    [head_offset, head_offset + Hq) of a layer with ``pattern_heads`` query
    heads (the module's num_attention_heads); 0 / 0 = they hold every head.
    Used to split one layer's heads over GPUs or launches."""
    layer_idx: int
    num_hidden_layers: int
    attention_length: int
    pattern_heads: int = 0
    head_offset: int = 0

    def heads(self, pattern_heads: int, head_offset: int) -> "PatternSpec":
        """The same layer's pattern for the query heads [head_offset, ...) of
        ``pattern_heads``."""
        return PatternSpec(self.layer_idx, self.num_hidden_layers, self.attention_length,
                           pattern_heads, head_offset)


def _aligned(t: torch.Tensor) -> bool:
    es = t.element_size()
    return (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
            and all((s * es) % 16 == 0 for s in t.stride()[:3]))


def as_kernel_operand(t: torch.Tensor) -> torch.Tensor:
    """Return ``t`` if the kernels can read it in place, else a contiguous copy
    (the reference always calls ``.contiguous()``, :244-245)."""
    return t if _aligned(t) else t.contiguous()


def _check_device(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    if dev.type != "cuda":
        raise RuntimeError("elastic sparse attention (B200) runs on CUDA tensors only; "
                           "there is no CPU fallback")
    for t in ts[1:]:
        if t.device != dev:
            raise RuntimeError("all operands must be on the same CUDA device")
    return dev


def pattern_indices(num_heads: int, spec: PatternSpec, n_rows: int, device: torch.device,
                    rows: torch.Tensor | None = None, row_offset: int = 0,
                    clamp_len: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """(idx, mask) int64 [H, n_rows, w] built on ``device`` by the pattern kernel."""
    lib = _lib.load()
    w = spec.attention_length
    idx = torch.empty((num_heads, n_rows, w), dtype=torch.int64, device=device)
    mask = torch.empty_like(idx)
    if rows is not None:
        rows = rows.to(device=device, dtype=torch.int64).contiguous()
    with torch.cuda.device(device):
        _lib.check(lib.esa_pattern(num_heads, w, spec.layer_idx, spec.num_hidden_layers, n_rows,
                                   _lib.ptr(rows), row_offset, clamp_len, idx.data_ptr(),
                                   mask.data_ptr(), _lib.stream_handle(device)), "esa_pattern")
    return idx, mask


def pattern_audit(num_heads: int, spec: PatternSpec, seq_len: int, device: torch.device) -> int:
    """Number of decreasing steps in the per-slot index columns (0 expected)."""
    lib = _lib.load()
    count = torch.zeros(1, dtype=torch.int64, device=device)
    with torch.cuda.device(device):
        _lib.check(lib.esa_pattern_audit(num_heads, spec.attention_length, spec.layer_idx,
                                         spec.num_hidden_layers, seq_len, count.data_ptr(),
                                         _lib.stream_handle(device)), "esa_pattern_audit")
    return int(count.item())


def _on(dev: torch.device):
    """Make ``dev`` current for a library call (no-op when it already is)."""
    return contextlib.nullcontext() if dev.index == torch.cuda.current_device() \
        else torch.cuda.device(dev)


def device_errors(device=None, clear: bool = True) -> int:
    """ESA_DEVERR_* bits the kernels recorded on ``device`` (default: the
    current device) since the last reset, after the work queued so far on its
    current stream; resets them when ``clear``.  Synchronises that stream."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flags = ctypes.c_int32(0)
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.esa_device_errors(1 if clear else 0, ctypes.byref(flags),
                                         _lib.stream_handle(dev)), "esa_device_errors")
    return int(flags.value)


def _problem(q, k, spec: PatternSpec, scale: float, rows, row_offset: int, kv_len: int,
             kv_offset: int, flags: int = 0, dropout_p: float = 0.0, dropout_seed: int = 0,
             weights=None, probs=None, key_plan=None):
    B, Hq, Lq, D = q.shape
    return _lib.problem(dtype=q.dtype, batch=B, num_heads=Hq, num_kv_heads=k.shape[1], head_dim=D,
                        attn_length=spec.attention_length, layer_idx=spec.layer_idx,
                        num_hidden_layers=spec.num_hidden_layers, q_len=Lq, kv_len=kv_len,
                        kv_offset=kv_offset, kv_rows=k.shape[2], row_offset=row_offset,
                        rows=rows, scale=scale, flags=flags, dropout_p=dropout_p,
                        dropout_seed=dropout_seed, weights=weights, probs=probs,
                        head_offset=spec.head_offset, pattern_heads=spec.pattern_heads,
                        key_plan=key_plan)


def key_plan(q, k, spec: PatternSpec, row_offset: int = 0, kv_len: int | None = None,
             kv_offset: int = 0) -> torch.Tensor | None:
    """The backward key side's precomputed user lists for this layer and these
    shapes / offsets (a uint8 device buffer), or None when its backward takes
    no plan.  Independent of the batch size and of the data: build it once and
    pass it to every :func:`backward` of the layer with the same shapes."""
    dev = _check_device(q, k)
    pb = _problem(q, k, spec, 1.0, None, row_offset, k.shape[2] if kv_len is None else kv_len,
                  kv_offset)
    lib = _lib.load()
    need = int(lib.esa_key_plan_size(ctypes.byref(pb)))
    if need == 0:
        return None
    plan = torch.empty(need, dtype=torch.uint8, device=dev)
    with _on(dev):
        _lib.check(lib.esa_key_plan_build(ctypes.byref(pb), plan.data_ptr(), need,
                                          _lib.stream_handle(dev)), "esa_key_plan_build")
    return plan


def probs_buffer(q, k, spec: PatternSpec, rows: torch.Tensor | None = None, row_offset: int = 0,
                 kv_len: int | None = None, kv_offset: int = 0, dropout_p: float = 0.0,
                 return_weights: bool = False) -> torch.Tensor | None:
    """A float32 [B, Hq, w, Lq] buffer for the forward to leave its softmax
    probabilities in, so that the backward skips recomputing the scores; None
    when the forward path for this problem does not write them."""
    B, Hq, Lq, _ = q.shape
    if return_weights or dropout_p > 0:
        return None   # those run the gather kernels, which do not write probs
    pb = _problem(q, k, spec, 1.0, rows, row_offset, k.shape[2] if kv_len is None else kv_len,
                  kv_offset)
    if _lib.load().esa_forward_writes_probs(ctypes.byref(pb)) != 1:
        return None
    return torch.empty((B, Hq, spec.attention_length, Lq), dtype=torch.float32, device=q.device)


def forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec: PatternSpec, scale: float,
            rows: torch.Tensor | None = None, row_offset: int = 0, kv_len: int | None = None,
            kv_offset: int = 0, out: torch.Tensor | None = None, gather_only: bool = False,
            dropout_p: float = 0.0, dropout_seed: int = 0, return_weights: bool = False,
            probs: torch.Tensor | None = None):
    """Forward pass.  Returns (o [B, Hq, Lq, D] as a view of a [B, Lq, Hq, D]
    buffer, lse float32 [B, Hq, Lq] base 2) and, with ``return_weights``, the
    softmax weights after dropout [B, Hq, Lq, w] in the input dtype.
    ``gather_only`` keeps sliding-window layers on the CUDA-core kernel (for
    cross-checking the two paths).  ``probs`` (from :func:`probs_buffer`)
    receives the probabilities for :func:`backward`."""
    dev = _check_device(q, k, v)
    B, Hq, Lq, D = q.shape
    if out is None:
        out = torch.empty((B, Lq, Hq, D), dtype=q.dtype, device=dev).transpose(1, 2)
    lse = torch.empty((B, Hq, Lq), dtype=torch.float32, device=dev)
    weights = (torch.empty((B, Hq, Lq, spec.attention_length), dtype=q.dtype, device=dev)
               if return_weights else None)
    if probs is not None:
        _check_probs(probs, q, spec)
    pb = _problem(q, k, spec, scale, rows, row_offset, k.shape[2] if kv_len is None else kv_len,
                  kv_offset, _lib.FLAG_GATHER_ONLY if gather_only else 0, dropout_p,
                  dropout_seed, weights, probs)
    lib = _lib.load()
    with _on(dev):
        _lib.check(lib.esa_forward(ctypes.byref(pb), _lib.tensor4(q), _lib.tensor4(k),
                                   _lib.tensor4(v), _lib.tensor4(out), lse.data_ptr(),
                                   _lib.stream_handle(dev)), "esa_forward")
    return (out, lse, weights) if return_weights else (out, lse)


def backward(q, k, v, o, lse, dout, spec: PatternSpec, scale: float,
             rows: torch.Tensor | None = None, row_offset: int = 0, kv_len: int | None = None,
             kv_offset: int = 0, sorted_rows=None, row_perm=None, workspace=None,
             dropout_p: float = 0.0, dropout_seed: int = 0, dq=None, dk=None, dv=None,
             probs: torch.Tensor | None = None, gather_only: bool = False,
             key_plan: torch.Tensor | None = None, dkv_fp32: bool = False):
    """Backward pass.  Returns (dq, dk, dv) in the input dtype.  With dropout,
    pass the forward's dropout_p and dropout_seed (the keep mask is rebuilt).
    dq / dk / dv may be given as (strided) views to write the gradients into,
    e.g. the q / k / v parts of one fused QKV gradient buffer.  ``gather_only``
    keeps sliding-window layers off the tensor-core backward (cross-checks).
    ``key_plan`` (from :func:`key_plan` for the same problem) spares the key
    side its pattern searches.  ``dkv_fp32``: dk / dv are float32 (the
    unrounded sums, for callers that add partial key gradients of several
    calls); dq stays in the input dtype."""
    dev = _check_device(q, k, v, o, lse, dout)
    kv_dtype = torch.float32 if dkv_fp32 else k.dtype
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k, dtype=kv_dtype) if dk is None else dk
    dv = torch.empty_like(v, dtype=kv_dtype) if dv is None else dv
    for g, ref, dt in ((dq, q, q.dtype), (dk, k, kv_dtype), (dv, v, kv_dtype)):
        if g.shape != ref.shape or g.dtype != dt or g.device != ref.device:
            raise ValueError("gradient buffers must match the shapes of q, k, v and their dtypes "
                             "(float32 for dk / dv with dkv_fp32)")
    if probs is not None:
        _check_probs(probs, q, spec)
    if key_plan is not None and (key_plan.dtype != torch.uint8 or key_plan.device != dev
                                 or not key_plan.is_contiguous()):
        raise ValueError("key_plan must be the contiguous uint8 buffer from key_plan()")
    flags = (_lib.FLAG_GATHER_ONLY if gather_only else 0) | (_lib.FLAG_F32_DKV if dkv_fp32 else 0)
    pb = _problem(q, k, spec, scale, rows, row_offset, k.shape[2] if kv_len is None else kv_len,
                  kv_offset, flags, dropout_p, dropout_seed, None, probs, key_plan)
    lib = _lib.load()
    need = lib.esa_backward_workspace_size(ctypes.byref(pb))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    with _on(dev):
        _lib.check(lib.esa_backward(ctypes.byref(pb), _lib.tensor4(q), _lib.tensor4(k),
                                    _lib.tensor4(v), _lib.tensor4(o), lse.data_ptr(),
                                    _lib.tensor4(dout), _lib.tensor4(dq), _lib.tensor4(dk),
                                    _lib.tensor4(dv), _lib.ptr(sorted_rows), _lib.ptr(row_perm),
                                    workspace.data_ptr(), workspace.numel(),
                                    _lib.stream_handle(dev)), "esa_backward")
    return dq, dk, dv


def _check_probs(probs: torch.Tensor, q: torch.Tensor, spec: PatternSpec) -> None:
    B, Hq, Lq, _ = q.shape
    if (probs.dtype != torch.float32 or probs.shape != (B, Hq, spec.attention_length, Lq)
            or not probs.is_contiguous() or probs.device != q.device):
        raise ValueError("probs must be a contiguous float32 [B, Hq, w, q_len] tensor "
                         "(see probs_buffer)")


def backward_workspace_bytes(q, k, spec: PatternSpec, kv_len: int | None = None) -> int:
    pb = _problem(q, k, spec, 1.0, None, 0, k.shape[2] if kv_len is None else kv_len, 0)
    return int(_lib.load().esa_backward_workspace_size(ctypes.byref(pb)))


def copy_rows(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """``dst.copy_(src)`` for two 4-D views [n0, n1, n2, row] of the same shape
    whose last dimension is contiguous (``esa_copy_rows``): a 16-bit copy, or
    fp32 ``src`` rounded to a 16-bit ``dst``.  The sequence split moves its K /
    V rows and partial dK / dV between [B, S, H, D] tensors and per-head-group
    [rows, B, heads, D] buffers with it.  Returns ``dst``."""
    if dst.dim() != 4 or src.shape != dst.shape:
        raise ValueError(f"copy_rows: 4-D views of one shape expected, got {tuple(src.shape)} "
                         f"-> {tuple(dst.shape)}")
    if src.stride(-1) != 1 or dst.stride(-1) != 1:
        raise ValueError("copy_rows: the last dimension must be contiguous")
    dev = _check_device(dst, src)
    if dst.numel() == 0:
        return dst
    r = _lib.EsaRows()
    r.src, r.dst = src.data_ptr(), dst.data_ptr()
    r.src_dtype, r.dst_dtype = _lib.DTYPES[src.dtype], _lib.DTYPES[dst.dtype]
    r.row_elems = src.shape[3]
    for i in range(3):
        r.count[i], r.src_stride[i], r.dst_stride[i] = src.shape[i], src.stride(i), dst.stride(i)
    with _on(dev):
        _lib.check(_lib.load().esa_copy_rows(ctypes.byref(r), _lib.stream_handle(dev)),
                   "esa_copy_rows")
    return dst
