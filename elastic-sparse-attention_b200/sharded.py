"""Sequence-sharded elastic sparse attention over a process group.

Query rows (and the K/V rows of the same positions) are split evenly across
the ranks of a group: rank r owns positions [r*S, (r+1)*S).  For a layer with
dilation alpha, the queries of rank r read keys from a contiguous range
[lo_r, (r+1)*S): every (head, slot) index column is non-decreasing along
positions (the property the backward relies on; audited by
``esa_pattern_audit``), so the smallest key any of r's queries reads is the
smallest valid index of its first row, and every row above it up to r*S is
read by some head and slot.

Forward:  fetch rows [lo_r, r*S) of K and V from their owners (NCCL grouped
          send/recv into one [rows, B, Hkv, D] buffer that also holds the
          local rows), then run the forward with row_offset = r*S and
          kv_offset = lo_r (the C ABI's offsets; indices are clamped to the
          global length as the reference does).
Backward: the local backward yields dQ for the local rows and partial dK/dV
          for every row of the buffer; the partials for remote rows go back to
          their owners (the reverse exchange) and are summed in fp32.

No reference counterpart: the reference runs on one device.  The layout of
the local shards is sequence-major, [B, S, H, D] (what an HF-style attention
layer produces), read in place by the kernels through strides.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops as cuda_ops
from .ops import PatternSpec

_plan_lock = threading.Lock()
_plan_cache: dict = {}


@dataclass(frozen=True)
class ShardPlan:
    """Who owns which rows and which key rows each rank reads."""
    world: int
    rows_per_rank: int        # S
    lo: tuple                 # lo[r]: first key position rank r reads

    def owned(self, r: int) -> tuple[int, int]:
        return r * self.rows_per_rank, (r + 1) * self.rows_per_rank

    def pieces_needed(self, r: int) -> list[tuple[int, int, int]]:
        """(owner q, start, stop) of the remote key rows rank r reads."""
        a0, _ = self.owned(r)
        out = []
        for q in range(r):
            qa, qb = self.owned(q)
            a, b = max(self.lo[r], qa), min(a0, qb)
            if a < b:
                out.append((q, a, b))
        return out

    def pieces_sent(self, q: int) -> list[tuple[int, int, int]]:
        """(reader r, start, stop) of rank q's rows that higher ranks read."""
        out = []
        for r in range(q + 1, self.world):
            for (owner, a, b) in self.pieces_needed(r):
                if owner == q:
                    out.append((r, a, b))
        return out


def make_plan(num_heads: int, spec: PatternSpec, rows_per_rank: int, world: int,
              device: torch.device, ops=cuda_ops) -> ShardPlan:
    """lo[r] = smallest valid key index of row r*S over all heads and slots."""
    key = (num_heads, spec, rows_per_rank, world)
    with _plan_lock:
        if key in _plan_cache:
            return _plan_cache[key]
    rows = torch.arange(world, dtype=torch.int64, device=device) * rows_per_rank
    idx, mask = ops.pattern_indices(num_heads, spec, world, device, rows=rows)
    big = torch.iinfo(torch.int64).max
    lo = torch.where(mask.bool(), idx, torch.full_like(idx, big)).amin(dim=(0, 2)).cpu().tolist()
    lo = tuple(min(int(v), r * rows_per_rank) for r, v in enumerate(lo))
    plan = ShardPlan(world, rows_per_rank, lo)
    with _plan_lock:
        _plan_cache[key] = plan
    return plan


def _exchange(plan: ShardPlan, rank: int, group, local: torch.Tensor, buf: torch.Tensor,
              lo: int):
    """Fill buf ([rows, ...], row 0 = position lo) with the remote rows rank
    `rank` reads, and send the rows of `local` ([S, ...]) that higher ranks
    read.  One grouped batch of NCCL / gloo point-to-point operations."""
    a0, _ = plan.owned(rank)
    p2p = []
    for (q, a, b) in plan.pieces_needed(rank):
        p2p.append(dist.P2POp(dist.irecv, buf[a - lo:b - lo], group=group, group_peer=q))
    sends = []
    for (r, a, b) in plan.pieces_sent(rank):
        piece = local[a - a0:b - a0].contiguous()
        sends.append(piece)
        p2p.append(dist.P2POp(dist.isend, piece, group=group, group_peer=r))
    if p2p:
        for req in dist.batch_isend_irecv(p2p):
            req.wait()


def _reverse_exchange(plan: ShardPlan, rank: int, group, dbuf: torch.Tensor, lo: int,
                      acc: torch.Tensor):
    """Send the partial gradients of remote rows (dbuf rows below r*S) to their
    owners; receive the partials of the local rows from higher ranks and add
    them into acc ([S, ...], fp32)."""
    a0, _ = plan.owned(rank)
    p2p, recvs = [], []
    for (q, a, b) in plan.pieces_needed(rank):
        p2p.append(dist.P2POp(dist.isend, dbuf[a - lo:b - lo].contiguous(), group=group,
                                   group_peer=q))
    for (r, a, b) in plan.pieces_sent(rank):
        t = torch.empty((b - a,) + tuple(dbuf.shape[1:]), dtype=dbuf.dtype, device=dbuf.device)
        recvs.append((t, a, b))
        p2p.append(dist.P2POp(dist.irecv, t, group=group, group_peer=r))
    if p2p:
        for req in dist.batch_isend_irecv(p2p):
            req.wait()
    for (t, a, b) in recvs:
        acc[a - a0:b - a0] += t.float()


class _ShardedFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, spec: PatternSpec, scale: float, plan: ShardPlan, rank: int,
                group, ops):
        # q [B, S, Hq, D], k/v [B, S, Hkv, D] (sequence-major shards)
        B, S, Hq, D = q.shape
        Hkv = k.shape[2]
        a0, b0 = plan.owned(rank)
        lo = plan.lo[rank]
        rows = b0 - lo
        L = plan.world * plan.rows_per_rank
        # [rows, B, Hkv, D]: row slices are contiguous for the exchange
        kbuf = torch.empty((rows, B, Hkv, D), dtype=k.dtype, device=k.device)
        vbuf = torch.empty_like(kbuf)
        kbuf[a0 - lo:] = k.transpose(0, 1)
        vbuf[a0 - lo:] = v.transpose(0, 1)
        _exchange(plan, rank, group, k.transpose(0, 1), kbuf, lo)
        _exchange(plan, rank, group, v.transpose(0, 1), vbuf, lo)
        qv = q.transpose(1, 2)                       # [B, Hq, S, D] view
        kv_k = kbuf.permute(1, 2, 0, 3)              # [B, Hkv, rows, D] view
        kv_v = vbuf.permute(1, 2, 0, 3)
        probs = None
        if hasattr(ops, "probs_buffer"):
            # the forward leaves its probabilities for the backward (no score pass)
            probs = ops.probs_buffer(qv, kv_k, spec, row_offset=a0, kv_len=L, kv_offset=lo)
        o, lse = ops.forward(qv, kv_k, kv_v, spec, scale, row_offset=a0, kv_len=L, kv_offset=lo,
                             **({"probs": probs} if probs is not None else {}))
        ctx.save_for_backward(q, kbuf, vbuf, o, lse, probs)
        ctx.meta = (spec, scale, plan, rank, group, ops)
        return o.transpose(1, 2)                     # [B, S, Hq, D]

    @staticmethod
    def backward(ctx, do):
        if do.stride(-1) != 1:
            do = do.contiguous()
        q, kbuf, vbuf, o, lse, probs = ctx.saved_tensors
        spec, scale, plan, rank, group, ops = ctx.meta
        a0, _ = plan.owned(rank)
        lo = plan.lo[rank]
        L = plan.world * plan.rows_per_rank
        dq, dkb, dvb = ops.backward(q.transpose(1, 2), kbuf.permute(1, 2, 0, 3),
                                    vbuf.permute(1, 2, 0, 3), o, lse, do.transpose(1, 2), spec,
                                    scale, row_offset=a0, kv_len=L, kv_offset=lo,
                                    **({"probs": probs} if probs is not None else {}))
        # partial dK/dV per buffer row, back in the [rows, B, Hkv, D] order
        dk_rows = dkb.permute(2, 0, 1, 3)
        dv_rows = dvb.permute(2, 0, 1, 3)
        dk_acc = dk_rows[a0 - lo:].float()
        dv_acc = dv_rows[a0 - lo:].float()
        _reverse_exchange(plan, rank, group, dk_rows, lo, dk_acc)
        _reverse_exchange(plan, rank, group, dv_rows, lo, dv_acc)
        dk = dk_acc.to(kbuf.dtype).transpose(0, 1)   # [B, S, Hkv, D]
        dv = dv_acc.to(vbuf.dtype).transpose(0, 1)
        return dq.transpose(1, 2), dk, dv, None, None, None, None, None, None


class SequenceShardedElasticSparseAttention(torch.nn.Module):
    """Elastic sparse attention with the sequence split over a process group.

    Same pattern arguments as ``ElasticSparseAttention``.  ``forward(q, k, v)``
    takes this rank's shards in sequence-major layout, q [B, S, Hq, D] and k/v
    [B, S, Hkv, D], where S = seq_len / world and rank r holds positions
    [r*S, (r+1)*S), and returns [B, S, Hq * D].  ``ops`` is the kernel backend
    (the CUDA library by default).
    """

    def __init__(self, layer_idx: int, num_hidden_layers: int, num_attention_heads: int,
                 head_dim: int, attention_length: int, max_seq_len: int,
                 num_key_value_heads: int | None = None, group=None, ops=cuda_ops):
        super().__init__()
        self.spec = PatternSpec(layer_idx, num_hidden_layers, attention_length)
        self.num_attention_heads = num_attention_heads
        self.num_key_value_heads = num_key_value_heads or num_attention_heads
        if num_attention_heads % self.num_key_value_heads:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.scaling = head_dim ** -0.5
        self.group = group
        self.ops = ops

    def plan(self, rows_per_rank: int, device) -> ShardPlan:
        world = dist.get_world_size(self.group)
        return make_plan(self.num_attention_heads, self.spec, rows_per_rank, world, device,
                         self.ops)

    def forward(self, q, k, v):
        B, S, Hq, D = q.shape
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        if S * world > self.max_seq_len:
            raise ValueError(f"sequence length {S * world} exceeds max_seq_len {self.max_seq_len}")
        plan = self.plan(S, q.device)
        if self.ops is cuda_ops and torch.is_grad_enabled():
            from .attention import _ensure_monotone
            _ensure_monotone(Hq, self.spec, max(S * world, 2), q.device)
        out = _ShardedFunction.apply(q, k, v, self.spec, self.scaling, plan, rank, self.group,
                                     self.ops)
        return out.reshape(B, S, Hq * D)
