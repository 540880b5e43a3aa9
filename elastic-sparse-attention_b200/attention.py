"""Drop-in ``ElasticSparseAttention`` module backed by hand-written sm_100a kernels.

Mirrors ``elastic_sparse_attention.py:345-765`` of HighCWu/elastic-sparse-attention:
the same constructor arguments and validation errors, the same
``forward(query_states, key_states, value_states, cache_position=None)``
signature and the same ``(attn_output [B, q_len, H*D], attn_weights)`` result.

Differences, all deliberate:

* Every ``implementation`` value ("triton", "naive", "dense") is accepted and
  validated as in the reference (:412-417) and runs on the CUDA kernels; there
  is no Triton, no PyTorch fallback and no CPU path.  As in the reference,
  ``implementation="naive"`` returns the softmax weights ``[B, H, q_len, w]``
  (:673-680, here not differentiable) and the others return ``None``
  (:622, :726).
* The pattern is computed inside the kernels from (position, head, slot), so
  nothing of size ``[H, max_seq_len, w]`` is built at construction (the
  reference builds it on the CPU, :454-468).  ``sparse_attention_indices``,
  ``sparse_causal_mask`` and ``full_attention_mask`` are still available, built
  lazily on the GPU on first access, bit-exact with the reference buffers.
* ``attention_dropout`` is applied where the reference applies it: in
  training mode for the "naive" (:674) and "dense" (:721) implementations;
  the "triton" implementation ignores it, as the reference's Triton kernel
  does.  The keep mask comes from an in-kernel counter-based generator
  (Philox4x32-10) seeded from torch's CPU generator, so it differs from
  torch.dropout's mask but has the same distribution and scaling.
"""
from __future__ import annotations

import logging
import threading
from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import ops
from .ops import PatternSpec

logger = logging.getLogger(__name__)

_audit_lock = threading.Lock()
_audited: dict[tuple, int] = {}   # (H, w, layer, nl) -> longest audited sequence length


def _ensure_monotone(num_heads: int, spec: PatternSpec, seq_len: int, device: torch.device):
    """The backward's key-side enumeration needs every per-slot index column to
    be non-decreasing along positions; check it once per pattern and length
    (over all of the pattern's heads when the call holds a subset of them)."""
    num_heads = spec.pattern_heads or num_heads
    key = (num_heads, spec.attention_length, spec.layer_idx, spec.num_hidden_layers)
    with _audit_lock:
        if _audited.get(key, 0) >= seq_len:
            return
    bad = ops.pattern_audit(num_heads, spec, seq_len, device)
    if bad:
        raise RuntimeError(
            f"elastic pattern {key} has {bad} decreasing index steps up to length {seq_len}; "
            "the backward kernel's transposed enumeration does not support it")
    with _audit_lock:
        _audited[key] = max(_audited.get(key, 0), seq_len)


class KeyPlanCache:
    """The key plan (:func:`ops.key_plan`) of one layer, built at the first
    backward of a shape and kept while the shape repeats, like the reference
    module keeps its index buffers (:454-468).  One plan is held at a time: a
    call with other shapes replaces it."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self._key = None
        self._plan = None

    def get(self, q: torch.Tensor, k: torch.Tensor, spec: PatternSpec, row_offset: int = 0,
            kv_len: Optional[int] = None, kv_offset: int = 0,
            build=None) -> Optional[torch.Tensor]:
        """The plan for these shapes and offsets (``build``: the function that
        makes it, :func:`ops.key_plan` by default)."""
        if not self.enabled:
            return None
        key = (q.device, q.dtype, tuple(q.shape[1:]), tuple(k.shape[1:3]), spec, row_offset,
               kv_len, kv_offset)
        if key != self._key:
            self._key, self._plan = None, None   # release the old plan first
            self._plan = (build or ops.key_plan)(q, k, spec, row_offset=row_offset,
                                                 kv_len=kv_len, kv_offset=kv_offset)
            self._key = key
        return self._plan

    def clear(self) -> None:
        self._key, self._plan = None, None


class ElasticSparseAttentionFunction(torch.autograd.Function):
    """Autograd boundary (reference ``ElasticSparseAttentionFunction``, :235-339).

    ``apply(q, k, v, pattern, sm_scale, num_kv_groups, rows=None)``: instead of
    materialised ``sparse_indices`` / ``sparse_mask`` tensors, ``pattern`` is the
    :class:`PatternSpec` they are generated from and ``rows`` the optional query
    positions (``cache_position``).  ``plans`` (a :class:`KeyPlanCache`)
    supplies the backward's key plan.  Returns o ``[B, H, q_len, D]``.
    """

    @staticmethod
    def forward(ctx, q, k, v, pattern: PatternSpec, sm_scale: float, num_kv_groups: int,
                rows: Optional[torch.Tensor] = None, dropout_p: float = 0.0,
                dropout_seed: int = 0, return_weights: bool = False,
                plans: Optional[KeyPlanCache] = None):
        if q.shape[1] != k.shape[1] * num_kv_groups:
            raise ValueError("num_kv_groups does not match the query / key head counts")
        q, k, v = (ops.as_kernel_operand(t) for t in (q, k, v))
        # the forward's probabilities, kept for the backward where that path writes them
        probs = ops.probs_buffer(q, k, pattern, rows=rows, dropout_p=dropout_p,
                                 return_weights=return_weights)
        res = ops.forward(q, k, v, pattern, sm_scale, rows=rows, dropout_p=dropout_p,
                          dropout_seed=dropout_seed, return_weights=return_weights, probs=probs)
        o, lse = res[0], res[1]
        ctx.save_for_backward(q, k, v, o, lse, rows, probs)
        ctx.pattern = pattern
        ctx.sm_scale = sm_scale
        ctx.dropout = (dropout_p, dropout_seed)
        ctx.plans = plans
        if return_weights:
            ctx.mark_non_differentiable(res[2])
            return o, res[2]
        return o

    @staticmethod
    def backward(ctx, do, *unused):
        q, k, v, o, lse, rows, probs = ctx.saved_tensors
        do = ops.as_kernel_operand(do)
        spec = ctx.pattern
        sorted_rows = perm = None
        if rows is not None:
            sorted_rows, perm = torch.sort(rows, stable=True)
            seq = int(sorted_rows[-1].item()) + 1 if rows.numel() else 0
        else:
            seq = q.shape[2]
        _ensure_monotone(q.shape[1], spec, max(seq, 2), q.device)
        plan = ctx.plans.get(q, k, spec) if ctx.plans is not None and rows is None else None
        dq, dk, dv = ops.backward(q, k, v, o, lse, do, spec, ctx.sm_scale, rows=rows,
                                  sorted_rows=sorted_rows, row_perm=perm,
                                  dropout_p=ctx.dropout[0], dropout_seed=ctx.dropout[1],
                                  probs=probs, key_plan=plan)
        return dq, dk, dv, None, None, None, None, None, None, None, None


def _forward_without_grad(q, k, v, pattern: PatternSpec, sm_scale: float, num_kv_groups: int,
                          rows: Optional[torch.Tensor], dropout_p: float, dropout_seed: int,
                          return_weights: bool):
    """The forward of :class:`ElasticSparseAttentionFunction` for calls that
    need no gradient (same results, no autograd bookkeeping)."""
    if q.shape[1] != k.shape[1] * num_kv_groups:
        raise ValueError("num_kv_groups does not match the query / key head counts")
    q, k, v = (ops.as_kernel_operand(t) for t in (q, k, v))
    res = ops.forward(q, k, v, pattern, sm_scale, rows=rows, dropout_p=dropout_p,
                      dropout_seed=dropout_seed, return_weights=return_weights)
    return (res[0], res[2]) if return_weights else res[0]


class ElasticSparseAttention(nn.Module):
    """Elastic sparse attention with GQA; see the module docstring for the contract.

    Args follow the reference (:375-386): ``layer_idx``, ``num_hidden_layers``,
    ``num_attention_heads``, ``head_dim``, ``attention_length`` (w),
    ``max_seq_len``, ``num_key_value_heads=None`` (MHA), ``attention_dropout=0.0``,
    ``implementation="triton"``.
    """

    def __init__(self, layer_idx: int, num_hidden_layers: int, num_attention_heads: int,
                 head_dim: int, attention_length: int, max_seq_len: int,
                 num_key_value_heads: Optional[int] = None, attention_dropout: float = 0.0,
                 implementation: str = "triton"):
        super().__init__()
        valid_implementations = ["triton", "naive", "dense"]
        if implementation not in valid_implementations:
            raise ValueError(
                f"Invalid implementation '{implementation}'. Must be one of "
                f"{valid_implementations}.")
        self.layer_idx = layer_idx
        self.num_hidden_layers = num_hidden_layers
        self.num_attention_heads = num_attention_heads
        self.head_dim = head_dim
        self.attention_length = attention_length
        self.attention_dropout = attention_dropout
        self.implementation = implementation
        self.max_seq_len = max_seq_len
        self.num_key_value_heads = (num_key_value_heads if num_key_value_heads is not None
                                    else num_attention_heads)
        if self.num_attention_heads % self.num_key_value_heads != 0:
            raise ValueError(
                f"`num_attention_heads` ({self.num_attention_heads}) must be divisible by "
                f"`num_key_value_heads` ({self.num_key_value_heads}) for GQA.")
        self.num_kv_groups = self.num_attention_heads // self.num_key_value_heads
        self.scaling = self.head_dim ** -0.5
        if max_seq_len > ops.MAX_POSITION:
            raise ValueError(f"max_seq_len ({max_seq_len}) above {ops.MAX_POSITION} is not "
                             "supported (float32 position arithmetic)")
        if attention_dropout > 0 and implementation == "triton":
            logger.warning("attention_dropout=%s is not applied by implementation='triton' (as "
                           "in the reference's Triton kernel)", attention_dropout)
        self.pattern = PatternSpec(layer_idx, num_hidden_layers, attention_length)
        self._buffers_cache: dict = {}
        # the backward's key plan for the current shapes (set .enabled = False
        # to trade its memory, ~4 bytes per (query, head, slot), for the key
        # side's pattern searches)
        self.key_plans = KeyPlanCache()

    # -- pattern buffers (lazy; reference :446-468) --------------------------
    def _pattern_device(self) -> torch.device:
        if not torch.cuda.is_available():
            raise RuntimeError("pattern buffers are built by a CUDA kernel; no GPU is visible")
        return torch.device("cuda", torch.cuda.current_device())

    def _create_elastic_sparse_indices(self, seq_len: int, device=None):
        """(indices, mask) int64 [H, seq_len, w], reference :470-535 (built on the GPU)."""
        dev = self._pattern_device() if device is None else torch.device(device)
        return ops.pattern_indices(self.num_attention_heads, self.pattern, seq_len, dev)

    def _cached_pattern(self):
        dev = self._pattern_device()
        key = ("sparse", dev)
        if key not in self._buffers_cache:
            self._buffers_cache[key] = self._create_elastic_sparse_indices(self.max_seq_len, dev)
        return self._buffers_cache[key]

    @property
    def sparse_attention_indices(self) -> torch.Tensor:
        return self._cached_pattern()[0]

    @property
    def sparse_causal_mask(self) -> torch.Tensor:
        return self._cached_pattern()[1]

    @property
    def full_attention_mask(self) -> torch.Tensor:
        """Dense bool [1, H, L, L] mask (reference :537-572); O(L^2) memory."""
        dev = self._pattern_device()
        key = ("full", dev)
        if key not in self._buffers_cache:
            L = self.max_seq_len
            idx, mask = self._cached_pattern()
            full = torch.zeros(self.num_attention_heads, L, L, dtype=torch.bool, device=dev)
            h = torch.arange(self.num_attention_heads, device=dev).view(-1, 1, 1).expand_as(idx)
            qpos = torch.arange(L, device=dev).view(1, -1, 1).expand_as(idx)
            m = mask.bool()
            full[h[m], qpos[m], idx.clamp(0, L - 1)[m]] = True
            self._buffers_cache[key] = full.unsqueeze(0)
        return self._buffers_cache[key]

    def _get_prepared_indices_and_mask(self, kv_seq_len: int):
        """Slices of the pattern buffers for ``kv_seq_len`` (reference :574-590)."""
        if kv_seq_len > self.max_seq_len:
            raise ValueError(
                f"Input sequence length ({kv_seq_len}) exceeds the maximum length initialized "
                f"in the module ({self.max_seq_len}).")
        return self.sparse_attention_indices[:, :kv_seq_len, :], \
            self.sparse_causal_mask[:, :kv_seq_len, :]

    # -- forward (reference :728-765) ----------------------------------------
    def forward(self, query_states: torch.Tensor, key_states: torch.Tensor,
                value_states: torch.Tensor, cache_position: Optional[torch.LongTensor] = None,
                ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        q_seq_len = query_states.shape[2]
        kv_seq_len = key_states.shape[2]
        if kv_seq_len > self.max_seq_len:
            raise ValueError(
                f"Input sequence length ({kv_seq_len}) exceeds the maximum length initialized "
                f"in the module ({self.max_seq_len}).")
        needs_grad = torch.is_grad_enabled() and (
            query_states.requires_grad or key_states.requires_grad or value_states.requires_grad)
        rows = None
        if cache_position is not None:
            rows = self._prepare_rows(cache_position, q_seq_len, kv_seq_len,
                                      query_states.device, checked=needs_grad)
        elif q_seq_len > kv_seq_len:
            raise ValueError(f"q_len ({q_seq_len}) > kv_len ({kv_seq_len}) needs cache_position")
        dropout_p = (self.attention_dropout if self.training and
                     self.implementation in ("naive", "dense") else 0.0)
        seed = int(torch.randint(0, 2 ** 62, (1,)).item()) if dropout_p > 0 else 0
        want_weights = self.implementation == "naive"
        if needs_grad:
            res = ElasticSparseAttentionFunction.apply(
                query_states, key_states, value_states, self.pattern, self.scaling,
                self.num_kv_groups, rows, dropout_p, seed, want_weights, self.key_plans)
        else:
            # inference: no autograd node, nothing saved
            res = _forward_without_grad(query_states, key_states, value_states, self.pattern,
                                        self.scaling, self.num_kv_groups, rows, dropout_p, seed,
                                        want_weights)
        attn_output, attn_weights = (res[0], res[1]) if want_weights else (res, None)
        batch_size, _, q_len, head_dim = query_states.shape
        hidden_dim = self.num_attention_heads * head_dim
        attn_output = attn_output.transpose(1, 2).reshape(batch_size, q_len, hidden_dim)
        return attn_output, attn_weights

    @staticmethod
    def _prepare_rows(cache_position, q_seq_len: int, kv_seq_len: int, device,
                      checked: bool = True) -> torch.Tensor:
        """Query positions for ``cache_position`` as the reference indexes the
        ``[:kv_len]`` slice of its buffers (:607-608): negative entries wrap,
        out-of-range entries raise IndexError.

        A host-side ``cache_position`` is checked on the host.  A device tensor
        is checked with one device->host read when a backward will follow
        (``checked``) and no CUDA graph is being captured.  Otherwise (decode
        under ``no_grad``, graph capture) nothing waits for the GPU: the forward
        kernel wraps negative entries itself, writes zeros for out-of-range
        rows and records ``ESA_DEVERR_QUERY_RANGE``, read with
        ``ops.device_errors()``."""
        rows = torch.as_tensor(cache_position)
        if rows.dtype != torch.int64:
            rows = rows.to(torch.int64)
        rows = rows.reshape(-1)
        if rows.numel() != q_seq_len:
            raise ValueError(f"cache_position has {rows.numel()} entries for q_len {q_seq_len}")
        if not rows.is_cuda:
            rows = torch.where(rows < 0, rows + kv_seq_len, rows)
            if rows.numel() and (int(rows.min()) < 0 or int(rows.max()) >= kv_seq_len):
                raise IndexError(f"cache_position out of range for kv_len {kv_seq_len}")
            return rows.to(device).contiguous()
        if not checked:
            return rows.to(device).contiguous()
        rows = torch.where(rows < 0, rows + kv_seq_len, rows)
        if (rows.numel() and not torch.cuda.is_current_stream_capturing()
                and bool(((rows < 0) | (rows >= kv_seq_len)).any())):
            raise IndexError(f"cache_position out of range for kv_len {kv_seq_len}")
        return rows.to(device).contiguous()

    def extra_repr(self) -> str:
        return (f"layer_idx={self.layer_idx}, num_hidden_layers={self.num_hidden_layers}, "
                f"heads={self.num_attention_heads}/{self.num_key_value_heads}, "
                f"head_dim={self.head_dim}, attention_length={self.attention_length}, "
                f"max_seq_len={self.max_seq_len}")
