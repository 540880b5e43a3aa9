"""numpy restatement of the elastic sparse index / causal-mask generator.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``elastic_sparse_attention.py:470-535`` (``_create_elastic_sparse_indices``)
operation by operation.  torch evaluates every step of that function in
float32 with one rounding per operation (``long (x) python-float`` and
``long / int`` promote to float32, no fused multiply-add on the CPU path), and
``Tensor.round`` is round-half-to-even, which is what ``np.rint`` does.  So
each line below is one float32 numpy operation, in the reference's order:

    a    = layer / (nl - 1)            (python double; nl == 1 -> layer / 1)    :488-489
    E    = max(w - 1, i) + 1                                                    :483, :495
    pd   = f32(w * (1 - a)) + f32(E) * f32(a)                                   :496
    st   = max(0, rint(f32(E) - pd))                                            :497
    sp   = f32(E - st) / f32(w)                                                 :498-499
    ov_k = st + rint(f32(k) * sp),  k = 0..w                                    :503-506
    base = ov[:w],  shifted = ov[1:] - 1                                        :510-511
    t_h  = f32(h) / f32(H - 1)         (H == 1 -> 0)                            :515-516
    idx  = rint(f32(base) * (1 - t_h) + f32(shifted) * t_h)                     :521-526
    mask = idx <= i;  idx[~mask] = 0                                            :532-533
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def layer_alpha(layer_idx: int, num_hidden_layers: int) -> float:
    """alpha as the reference computes it (python double), ``:488-489``."""
    denominator = num_hidden_layers - 1 if num_hidden_layers > 1 else 1
    return layer_idx / denominator


def row_params(positions: np.ndarray, attn_length: int, layer_idx: int,
               num_hidden_layers: int) -> tuple[np.ndarray, np.ndarray]:
    """Per query position: (start ``st`` int64, spacing ``sp`` float32), ``:482-499``."""
    w = attn_length
    a = layer_alpha(layer_idx, num_hidden_layers)
    pos = np.asarray(positions, dtype=np.int64)
    end = np.maximum(w - 1, pos)
    E = (end + 1).astype(F32)
    c = F32(w * (1 - a))                       # python double, rounded once to f32
    pd = c + E * F32(a)                        # two f32 roundings, no FMA
    st = np.rint(E - pd)
    st = np.maximum(st, F32(0)).astype(np.int64)
    win = (end + 1 - st).astype(F32)
    sp = win / F32(w)
    return st, sp


def oversized(positions: np.ndarray, attn_length: int, layer_idx: int,
              num_hidden_layers: int) -> np.ndarray:
    """``attention_indices_oversized`` [n, w+1] int64, ``:503-506``."""
    st, sp = row_params(positions, attn_length, layer_idx, num_hidden_layers)
    k = np.arange(attn_length + 1, dtype=np.int64).astype(F32)
    rel = np.rint(k[None, :] * sp[:, None]).astype(np.int64)
    return st[:, None] + rel


def head_weights(num_heads: int) -> np.ndarray:
    """Interpolation weight t_h per query head (float32), ``:515-516``."""
    h = np.arange(num_heads, dtype=np.int64)
    if num_heads > 1:
        return h.astype(F32) / F32(num_heads - 1)
    return np.zeros(num_heads, dtype=F32)


def elastic_indices(positions, num_heads: int, attn_length: int, layer_idx: int,
                    num_hidden_layers: int) -> tuple[np.ndarray, np.ndarray]:
    """(idx, mask), both int64 ``[H, n, w]``, for the given query positions.

    With ``positions = arange(L)`` this equals the reference's
    ``_create_elastic_sparse_indices(L)`` bit for bit (``:470-535``); a row
    depends only on its own position, so any subset of rows is the
    corresponding slice of the reference buffers.
    """
    pos = np.asarray(positions, dtype=np.int64)
    ov = oversized(pos, attn_length, layer_idx, num_hidden_layers)
    base = ov[:, :attn_length].astype(F32)
    shifted = (ov[:, 1:] - 1).astype(F32)
    t = head_weights(num_heads)[:, None, None]
    one_minus_t = F32(1) - t
    val = base[None] * one_minus_t + shifted[None] * t
    idx = np.rint(val).astype(np.int64)
    mask = idx <= pos[None, :, None]
    idx = np.where(mask, idx, 0)
    return idx, mask.astype(np.int64)


def prepared_indices(num_heads: int, attn_length: int, layer_idx: int,
                     num_hidden_layers: int, max_seq_len: int, q_len: int,
                     kv_len: int, cache_position=None):
    """What ``_triton_forward`` hands to the kernel (``:574-615``).

    Raises ``ValueError`` when ``kv_len > max_seq_len`` (``:579-584``); rows are
    ``[:q_len]`` or ``cache_position`` of the ``[:kv_len]`` slice
    (``:602-611``); indices are clamped to ``[0, kv_len - 1]`` (``:615``).
    """
    if kv_len > max_seq_len:
        raise ValueError(
            f"Input sequence length ({kv_len}) exceeds the maximum length initialized "
            f"in the module ({max_seq_len}).")
    if cache_position is None:
        rows = np.arange(min(q_len, kv_len), dtype=np.int64)
    else:
        rows = np.asarray(cache_position, dtype=np.int64)
        # torch indexing of the [:kv_len] slice: negative rows wrap, rows >= kv_len raise
        rows = np.where(rows < 0, rows + kv_len, rows)
        if np.any(rows < 0) or np.any(rows >= kv_len):
            raise IndexError("cache_position out of range of the sliced pattern")
    idx, mask = elastic_indices(rows, num_heads, attn_length, layer_idx, num_hidden_layers)
    idx = np.clip(idx, 0, kv_len - 1)
    return idx, mask, rows


def full_mask(seq_len: int, num_heads: int, attn_length: int, layer_idx: int,
              num_hidden_layers: int) -> np.ndarray:
    """Dense bool ``[H, L, L]`` mask (``_create_full_sparse_mask``, ``:537-572``)."""
    idx, mask = elastic_indices(np.arange(seq_len), num_heads, attn_length, layer_idx,
                                num_hidden_layers)
    out = np.zeros((num_heads, seq_len, seq_len), dtype=bool)
    h = np.broadcast_to(np.arange(num_heads)[:, None, None], idx.shape)
    q = np.broadcast_to(np.arange(seq_len)[None, :, None], idx.shape)
    k = np.clip(idx, 0, seq_len - 1)
    m = mask.astype(bool)
    out[h[m], q[m], k[m]] = True
    return out


def active_blocks_per_tile(num_heads: int, seq_len: int, attn_length: int, layer_idx: int,
                           num_hidden_layers: int, block: int = 128,
                           rows: np.ndarray | None = None) -> np.ndarray:
    """Number of (``block``-query tile, ``block``-key block) pairs holding >= 1
    valid entry, per head, as ``[H, n_tiles]`` int64.

    This is the accounting unit of the "effective TFLOP/s over active blocks"
    metric: ``4 * D * block * block`` FLOPs per active pair (forward).
    """
    n_tiles = (seq_len + block - 1) // block
    tiles = np.arange(n_tiles) if rows is None else np.asarray(rows)
    out = np.zeros((num_heads, len(tiles)), dtype=np.int64)
    for n, t in enumerate(tiles):
        pos = np.arange(t * block, min(seq_len, (t + 1) * block))
        idx, mask = elastic_indices(pos, num_heads, attn_length, layer_idx, num_hidden_layers)
        kb = np.where(mask.astype(bool), idx // block, -1)
        for h in range(num_heads):
            u = np.unique(kb[h])
            out[h, n] = int(np.count_nonzero(u >= 0))
    return out
