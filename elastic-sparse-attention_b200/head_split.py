"""Elastic sparse attention with one layer's heads split over GPUs.

Every (query, head) pair attends to its own w keys and the K/V heads of a GQA
group are read only by that group's query heads, so splitting a layer by
whole GQA groups needs no communication: rank r of N holds KV heads
[r * Hkv / N, (r + 1) * Hkv / N) and their G query heads each, and computes
them with the pattern of those heads (the head interpolation weight
t = h / (H - 1) of the reference, elastic_sparse_attention.py:515-516, uses
the layer-wide head index h, passed to the kernels as the call's head
offset).  The result on each rank is exactly its slice of the single-GPU
result.  No reference counterpart: the reference runs on one device, and its
Triton grid (Lq, H, B) (:261) is the axis split here.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .attention import ElasticSparseAttentionFunction, KeyPlanCache, _forward_without_grad
from .ops import PatternSpec, MAX_POSITION


def head_share(num_attention_heads: int, num_key_value_heads: int, rank: int,
               world_size: int) -> tuple[int, int, int, int]:
    """(first query head, query heads, first KV head, KV heads) of ``rank``."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside a group of {world_size}")
    if num_attention_heads % num_key_value_heads:
        raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
    if num_key_value_heads % world_size:
        raise ValueError(f"num_key_value_heads ({num_key_value_heads}) must be divisible by the "
                         f"number of ranks ({world_size}) to split whole GQA groups")
    g = num_attention_heads // num_key_value_heads
    kv = num_key_value_heads // world_size
    return rank * kv * g, kv * g, rank * kv, kv


class HeadShardedElasticSparseAttention(nn.Module):
    """This rank's share of one layer's heads.

    Pattern arguments as ``ElasticSparseAttention`` (reference :375-386), with
    ``num_attention_heads`` / ``num_key_value_heads`` the layer's totals.
    ``rank`` / ``world_size`` default to the process group's.
    ``forward(q, k, v)`` takes this rank's heads, q [B, Hq / N, L, D] and k/v
    [B, Hkv / N, L, D] (``head_share`` gives which), and returns
    [B, L, Hq / N * D]: the columns of the reference output that belong to
    those heads.  Gradients flow as in ``ElasticSparseAttention``.
    """

    def __init__(self, layer_idx: int, num_hidden_layers: int, num_attention_heads: int,
                 head_dim: int, attention_length: int, max_seq_len: int,
                 num_key_value_heads: Optional[int] = None, rank: Optional[int] = None,
                 world_size: Optional[int] = None, group=None):
        super().__init__()
        if rank is None or world_size is None:
            import torch.distributed as dist
            if not dist.is_initialized():
                raise ValueError("rank / world_size are needed without a process group")
            rank = dist.get_rank(group) if rank is None else rank
            world_size = dist.get_world_size(group) if world_size is None else world_size
        if max_seq_len > MAX_POSITION:
            raise ValueError(f"max_seq_len ({max_seq_len}) above {MAX_POSITION} is not supported")
        self.num_attention_heads = num_attention_heads
        self.num_key_value_heads = num_key_value_heads or num_attention_heads
        self.head0, self.local_heads, self.kv_head0, self.local_kv_heads = head_share(
            num_attention_heads, self.num_key_value_heads, rank, world_size)
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.scaling = head_dim ** -0.5
        self.num_kv_groups = num_attention_heads // self.num_key_value_heads
        self.pattern = PatternSpec(layer_idx, num_hidden_layers, attention_length).heads(
            num_attention_heads, self.head0)
        self.key_plans = KeyPlanCache()

    def forward(self, query_states: torch.Tensor, key_states: torch.Tensor,
                value_states: torch.Tensor) -> torch.Tensor:
        B, Hq, L, D = query_states.shape
        if Hq != self.local_heads or key_states.shape[1] != self.local_kv_heads:
            raise ValueError(f"this rank holds {self.local_heads} query / {self.local_kv_heads} "
                             f"KV heads, got {Hq} / {key_states.shape[1]}")
        if key_states.shape[2] > self.max_seq_len:
            raise ValueError(f"Input sequence length ({key_states.shape[2]}) exceeds the maximum "
                             f"length initialized in the module ({self.max_seq_len}).")
        if L > key_states.shape[2]:
            raise ValueError(f"q_len ({L}) > kv_len ({key_states.shape[2]})")
        needs_grad = torch.is_grad_enabled() and (
            query_states.requires_grad or key_states.requires_grad or value_states.requires_grad)
        if needs_grad:
            out = ElasticSparseAttentionFunction.apply(query_states, key_states, value_states,
                                                       self.pattern, self.scaling,
                                                       self.num_kv_groups, None, 0.0, 0, False,
                                                       self.key_plans)
        else:
            out = _forward_without_grad(query_states, key_states, value_states, self.pattern,
                                        self.scaling, self.num_kv_groups, None, 0.0, 0, False)
        return out.transpose(1, 2).reshape(B, L, Hq * D)
