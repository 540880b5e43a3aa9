"""Sequence-sharded elastic sparse attention over a process group.

Query rows (and the K/V rows of the same positions) are split evenly across
the ranks of a group: rank r owns positions [r*S, (r+1)*S).  For a layer with
dilation alpha, the queries of rank r read keys from a contiguous range
[lo_r, (r+1)*S): every (head, slot) index column is non-decreasing along
positions (the property the backward relies on; audited by
``esa_pattern_audit``), so the smallest key any of r's queries reads is the
smallest valid index of its first row, and every row above it up to r*S is
read by some head and slot.

The KV heads are processed in head groups (whole GQA groups), so that the
transfers of one group overlap the kernels of the previous one:

Forward:  for every head group, one grouped batch of NCCL send/recv fetches
          rows [lo_r, r*S) of its K and V from their owners into a per-group
          [rows, heads, D] buffer that also holds the local rows; all batches
          are issued at once on the communicator's stream, and the compute
          stream waits for group g's batch just before group g's forward
          (row_offset = r*S, kv_offset = lo_r: the C ABI's offsets; indices
          are clamped to the global length as the reference does).
Backward: group g's backward yields dQ for the local rows and partial dK/dV
          for every buffer row; the partials of remote rows go back to their
          owners in one batch per group, issued right after that group's
          kernels, so they travel while the next group computes; the owners
          add them to their local partials in fp32.

The NCCL traffic of a rank is the remote K/V rows its queries read (at most
all rows below its shard, at alpha = 1) and the same rows of partial dK/dV
back.  No reference counterpart: the reference runs on one device.  The layout
of the local shards is sequence-major, [B, S, H, D] (what an HF-style
attention layer produces), read in place by the kernels through strides.
"""
from __future__ import annotations

import threading
import time
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops as cuda_ops
from .ops import PatternSpec

_plan_lock = threading.Lock()
_plan_cache: dict = {}

# One scratch buffer per device for the backward's temporaries (the fp32
# partial dK / dV of the buffer rows and the kernels' workspace): the layers'
# backwards run one after another and each ends by waiting for its transfers,
# so they can share it, and the caching allocator does not have to find room
# for ~10 GB of differently sized blocks per layer.
_scratch_lock = threading.Lock()
_scratch: dict = {}


def _scratch_bytes(device: torch.device, nbytes: int) -> torch.Tensor:
    """A uint8 buffer of at least nbytes on device (256-byte aligned start),
    shared by every sequence-sharded backward on that device."""
    nbytes = (nbytes + 255) // 256 * 256
    with _scratch_lock:
        buf = _scratch.get(device)
        if buf is None or buf.numel() < nbytes:
            _scratch.pop(device, None)
            del buf
            buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
            _scratch[device] = buf
        return buf


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


# ---------------------------------------------------------------------------
# Optional per-step timing of one rank (profile_step): CUDA events on the
# compute stream around the kernels and around each wait for a transfer.  The
# record list is process-wide: the backward runs on autograd's own thread.
# ---------------------------------------------------------------------------
class _Timing:
    records = None
    host_ms = None   # host time spent issuing NCCL batches (dict), while profiling


_timing = _Timing()


class _Span:
    def __init__(self, kind: str):
        self.kind = kind
        self.rec = _timing.records

    def __enter__(self):
        if self.rec is not None:
            self.a = torch.cuda.Event(enable_timing=True)
            self.a.record()
        return self

    def __exit__(self, *exc):
        if self.rec is not None:
            b = torch.cuda.Event(enable_timing=True)
            b.record()
            self.rec.append((self.kind, self.a, b))


def profile_step(step, device) -> dict:
    """Runs step() once and splits this rank's device time (compute stream)
    into kernels, waits for NCCL transfers, layout copies (K/V into the
    per-group buffers, dK/dV back to [B, S, H, D]), fp32 sums of the partial
    dK/dV, and the rest (gaps between launches, allocation, torch ops of the
    caller); milliseconds."""
    torch.cuda.synchronize(device)
    _timing.records = []
    _timing.host_ms = {"nccl_issue": 0.0}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        e0.record()
        t0 = time.perf_counter()
        step()
        host = (time.perf_counter() - t0) * 1e3
        e1.record()
        torch.cuda.synchronize(device)
        recs = _timing.records
        nccl_issue = _timing.host_ms["nccl_issue"]
    finally:
        _timing.records = None
        _timing.host_ms = None
    total = e0.elapsed_time(e1)
    # host_ms: the host's time to issue the step (close to step_ms means the
    # GPU waited for the host); nccl_issue_host_ms: of it, inside NCCL calls
    out = {"step_ms": round(total, 3), "host_ms": round(host, 3),
           "nccl_issue_host_ms": round(nccl_issue, 3)}
    kinds = ("kernels", "exchange_wait", "layout", "reduce")
    for kind in kinds:
        out[kind + "_ms"] = round(sum(a.elapsed_time(b) for k, a, b in recs if k == kind), 3)
    out["other_ms"] = round(total - sum(out[k + "_ms"] for k in kinds), 3)
    return out


def _batch(p2p):
    """Issue one grouped batch of point-to-point operations; [] if none."""
    if not p2p:
        return []
    if _timing.host_ms is None:
        return dist.batch_isend_irecv(p2p)
    t0 = time.perf_counter()
    works = dist.batch_isend_irecv(p2p)
    _timing.host_ms["nccl_issue"] += (time.perf_counter() - t0) * 1e3
    return works


def _wait(works):
    with _Span("exchange_wait"):
        for w in works:
            w.wait()


def _fetch(plan: ShardPlan, rank: int, group, bufs, lo: int):
    """Issue (do not wait for) the fetch of the remote rows of every buffer in
    bufs ([rows, ...], row 0 = position lo, the local rows already in place)
    and the sends of this rank's rows that higher ranks read (taken from the
    local part of the same buffers).  Peers are ranks of `group`."""
    a0, _ = plan.owned(rank)
    p2p = []
    for buf in bufs:
        for (q, a, b) in plan.pieces_needed(rank):
            p2p.append(dist.P2POp(dist.irecv, buf[a - lo:b - lo], group=group, group_peer=q))
        for (r, a, b) in plan.pieces_sent(rank):
            p2p.append(dist.P2POp(dist.isend, buf[a - lo:b - lo], group=group, group_peer=r))
    return _batch(p2p)


def _return_partials(plan: ShardPlan, rank: int, group, dbufs, lo: int, space=None):
    """Issue the sends of the partial gradients of remote rows (rows below
    r*S of each buffer in dbufs) to their owners and the receives of the
    partials of this rank's rows from higher ranks; returns (works, [(buffer
    index, tensor, start, stop)] of the receives).  The receives are carved
    from ``space`` (a flat tensor of the buffers' dtype, ``len(dbufs)`` x the
    rows of pieces_sent x a buffer row) when given, else allocated."""
    p2p, recvs = [], []
    used = 0
    for i, dbuf in enumerate(dbufs):
        for (q, a, b) in plan.pieces_needed(rank):
            p2p.append(dist.P2POp(dist.isend, dbuf[a - lo:b - lo], group=group, group_peer=q))
        for (r, a, b) in plan.pieces_sent(rank):
            shape = (b - a,) + tuple(dbuf.shape[1:])
            if space is None:
                t = torch.empty(shape, dtype=dbuf.dtype, device=dbuf.device)
            else:
                n = (b - a) * dbuf[0].numel()
                t = space[used:used + n].view(shape)
                used += n
            recvs.append((i, t, a, b))
            p2p.append(dist.P2POp(dist.irecv, t, group=group, group_peer=r))
    return _batch(p2p), recvs


def _copy_rows(ops, dst: torch.Tensor, src: torch.Tensor) -> None:
    """dst.copy_(src) for [n0, n1, n2, row] views: the library's row-copy
    kernel (16-byte vectors, HBM-bound) when ``ops`` has it and the views are
    16-byte aligned; torch's strided copy otherwise (kernel-less test ops, or
    odd caller tensors)."""
    es_s, es_d = src.element_size(), dst.element_size()
    if (hasattr(ops, "copy_rows") and src.is_cuda and src.stride(-1) == 1
            and dst.stride(-1) == 1 and src.shape[-1] % 8 == 0
            and src.data_ptr() % 16 == 0 and dst.data_ptr() % 16 == 0
            and all((st * es_s) % 16 == 0 for st in src.stride()[:3])
            and all((st * es_d) % 16 == 0 for st in dst.stride()[:3])):
        ops.copy_rows(dst, src)
    else:
        dst.copy_(src)


def group_count(num_kv_heads: int, wanted: int) -> int:
    """Largest count <= wanted that divides num_kv_heads."""
    n = max(1, min(wanted, num_kv_heads))
    while num_kv_heads % n:
        n -= 1
    return n


class _ShardedFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, spec: PatternSpec, scale: float, plan: ShardPlan, rank: int,
                group, ops, ngroups: int, key_plans=None):
        # q [B, S, Hq, D], k/v [B, S, Hkv, D] (sequence-major shards)
        B, S, Hq, D = q.shape
        Hkv = k.shape[2]
        G = Hq // Hkv
        hg = Hkv // ngroups                              # KV heads per head group
        a0, b0 = plan.owned(rank)
        lo = plan.lo[rank]
        rows = b0 - lo
        L = plan.world * plan.rows_per_rank
        # per head group: [rows, B, hg, D]; row slices are contiguous for the transfers
        with _Span("layout"):
            kbuf = torch.empty((ngroups, rows, B, hg, D), dtype=k.dtype, device=k.device)
            vbuf = torch.empty_like(kbuf)
            # [B, S, Hkv, D] -> [ngroups, S, B, hg * D] rows of the buffers
            for t, buf in ((k, kbuf), (v, vbuf)):
                _copy_rows(ops, buf[:, a0 - lo:].flatten(3, 4),
                           t.unflatten(2, (ngroups, hg)).flatten(3, 4).permute(2, 1, 0, 3))
        works = [_fetch(plan, rank, group, (kbuf[g], vbuf[g]), lo) for g in range(ngroups)]
        out = torch.empty_like(q)                        # [B, S, Hq, D]
        lses, probs = [], []
        for g in range(ngroups):
            h0 = g * hg * G
            sg = spec.heads(Hq, h0)
            qv = q[:, :, h0:h0 + hg * G].transpose(1, 2)  # [B, hg*G, S, D] view
            kv_k = kbuf[g].permute(1, 2, 0, 3)              # [B, hg, rows, D] view
            kv_v = vbuf[g].permute(1, 2, 0, 3)
            pr = (ops.probs_buffer(qv, kv_k, sg, row_offset=a0, kv_len=L, kv_offset=lo)
                  if hasattr(ops, "probs_buffer") else None)
            _wait(works[g])
            with _Span("kernels"):
                _, lse = ops.forward(qv, kv_k, kv_v, sg, scale, row_offset=a0, kv_len=L,
                                     kv_offset=lo, out=out[:, :, h0:h0 + hg * G].transpose(1, 2),
                                     **({"probs": pr} if pr is not None else {}))
            lses.append(lse)
            probs.append(pr)
        ctx.save_for_backward(q, kbuf, vbuf, out, *lses,
                              *[p for p in probs if p is not None])
        ctx.has_probs = [p is not None for p in probs]
        ctx.meta = (spec, scale, plan, rank, group, ops, ngroups)
        ctx.key_plans = key_plans if hasattr(ops, "key_plan") else None
        return out

    @staticmethod
    def backward(ctx, do):
        if do.stride(-1) != 1:
            do = do.contiguous()
        spec, scale, plan, rank, group, ops, ngroups = ctx.meta
        saved = ctx.saved_tensors
        q, kbuf, vbuf, out = saved[:4]
        lses = saved[4:4 + ngroups]
        it = iter(saved[4 + ngroups:])
        probs = [next(it) if h else None for h in ctx.has_probs]
        B, S, Hq, D = q.shape
        hg = kbuf.shape[3]
        G = Hq // (hg * ngroups)
        a0, _ = plan.owned(rank)
        lo = plan.lo[rank]
        L = plan.world * plan.rows_per_rank
        dq = torch.empty_like(q)
        # partial dK / dV in fp32: the partials of a key from several ranks
        # are added unrounded and rounded once, as in the one-GPU key side;
        # they and the kernels' workspace live in the device's shared scratch
        nkv = kbuf.numel()
        g_q = q[:, :, :hg * G].transpose(1, 2)
        g_k = kbuf[0].permute(1, 2, 0, 3)
        ws_bytes = (ops.backward_workspace_bytes(g_q, g_k, spec, kv_len=L)
                    if hasattr(ops, "backward_workspace_bytes") else 0)
        ws_bytes = (ws_bytes + 255) // 256 * 256
        # the fp32 partials of this rank's rows that higher ranks return: all
        # groups' receives are in flight together, each group's dK and dV
        sent_rows = sum(b - a for (_, a, b) in plan.pieces_sent(rank))
        recv_elems = 2 * sent_rows * kbuf[0, 0].numel()    # per group
        recv_at = 2 * nkv * 4 + ws_bytes
        scratch = _scratch_bytes(kbuf.device, recv_at + ngroups * recv_elems * 4)
        dkb = scratch[:nkv * 4].view(torch.float32).view(kbuf.shape)
        dvb = scratch[nkv * 4:2 * nkv * 4].view(torch.float32).view(kbuf.shape)
        ws = scratch[2 * nkv * 4:2 * nkv * 4 + ws_bytes] if ws_bytes else None
        recv_space = scratch[recv_at:recv_at + ngroups * recv_elems * 4].view(torch.float32)
        pending = []
        for g in range(ngroups):
            h0 = g * hg * G
            sl = slice(h0, h0 + hg * G)
            sg = spec.heads(Hq, h0)
            # the group's key plan (built at the first backward of this shape)
            kp = None
            if ctx.key_plans is not None:
                kp = ctx.key_plans[g].get(q[:, :, sl].transpose(1, 2), kbuf[g].permute(1, 2, 0, 3),
                                          sg, row_offset=a0, kv_len=L, kv_offset=lo,
                                          build=ops.key_plan)
            with _Span("kernels"):
                ops.backward(q[:, :, sl].transpose(1, 2), kbuf[g].permute(1, 2, 0, 3),
                             vbuf[g].permute(1, 2, 0, 3), out[:, :, sl].transpose(1, 2), lses[g],
                             do[:, :, sl].transpose(1, 2), sg, scale, row_offset=a0, kv_len=L,
                             kv_offset=lo, dq=dq[:, :, sl].transpose(1, 2),
                             dk=dkb[g].permute(1, 2, 0, 3), dv=dvb[g].permute(1, 2, 0, 3),
                             dkv_fp32=True,
                             **({"probs": probs[g]} if probs[g] is not None else {}),
                             **({"workspace": ws} if ws is not None else {}),
                             **({"key_plan": kp} if kp is not None else {}))
            pending.append(_return_partials(
                plan, rank, group, (dkb[g], dvb[g]), lo,
                recv_space[g * recv_elems:(g + 1) * recv_elems]))
        # local rows: own partials plus the fp32 partials returned by higher
        # ranks (only the rows they read, a suffix of this rank's rows)
        dk_loc, dv_loc = dkb[:, a0 - lo:], dvb[:, a0 - lo:]   # [ngroups, S, B, hg, D]
        for g, (works, recvs) in enumerate(pending):
            _wait(works)
            with _Span("reduce"):
                for (i, t, a, b) in recvs:
                    (dk_loc if i == 0 else dv_loc)[g, a - a0:b - a0] += t
        # [ngroups, S, B, hg, D] fp32 -> [B, S, Hkv, D] in the input dtype, one rounding
        with _Span("layout"):
            dk = torch.empty((B, S, ngroups, hg, D), dtype=kbuf.dtype, device=kbuf.device)
            dv = torch.empty_like(dk)
            for dst, src in ((dk, dk_loc), (dv, dv_loc)):
                _copy_rows(ops, dst.flatten(3, 4).permute(2, 1, 0, 3), src.flatten(3, 4))
            dk, dv = dk.view(B, S, ngroups * hg, D), dv.view(B, S, ngroups * hg, D)
        return dq, dk, dv, None, None, None, None, None, None, None, None


class SequenceShardedElasticSparseAttention(torch.nn.Module):
    """Elastic sparse attention with the sequence split over a process group.

    Same pattern arguments as ``ElasticSparseAttention``.  ``forward(q, k, v)``
    takes this rank's shards in sequence-major layout, q [B, S, Hq, D] and k/v
    [B, S, Hkv, D], where S = seq_len / world and rank r holds positions
    [r*S, (r+1)*S), and returns [B, S, Hq * D].  ``head_groups``: KV heads
    are processed in this many groups (fewer if it does not divide
    num_key_value_heads) so that transfers overlap kernels.  ``ops`` is the
    kernel backend (the CUDA library by default).
    """

    def __init__(self, layer_idx: int, num_hidden_layers: int, num_attention_heads: int,
                 head_dim: int, attention_length: int, max_seq_len: int,
                 num_key_value_heads: int | None = None, group=None, ops=cuda_ops,
                 head_groups: int = 4):
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
        self.head_groups = group_count(self.num_key_value_heads, head_groups)
        # key plans: of the one-rank path (a group of one), and of each head
        # group's backward call in the split
        from .attention import KeyPlanCache
        self.key_plans = KeyPlanCache()
        self.group_key_plans = [KeyPlanCache() for _ in range(self.head_groups)]

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
        if Hq != self.num_attention_heads or k.shape[2] != self.num_key_value_heads:
            raise ValueError("head counts of q / k do not match the module")
        if world == 1 and self.ops is cuda_ops:
            # nothing to exchange: the one-GPU path on the [B, S, H, D] shards
            # read in place (no per-group buffers), with the layer's key plan
            from .attention import ElasticSparseAttentionFunction, _forward_without_grad
            G = Hq // k.shape[2]
            qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
            if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad
                                            or v.requires_grad):
                o = ElasticSparseAttentionFunction.apply(qt, kt, vt, self.spec, self.scaling, G,
                                                         None, 0.0, 0, False, self.key_plans)
            else:
                o = _forward_without_grad(qt, kt, vt, self.spec, self.scaling, G, None, 0.0, 0,
                                          False)
            return o.transpose(1, 2).reshape(B, S, Hq * D)
        plan = self.plan(S, q.device)
        if self.ops is cuda_ops and torch.is_grad_enabled():
            from .attention import _ensure_monotone
            _ensure_monotone(Hq, self.spec, max(S * world, 2), q.device)
        out = _ShardedFunction.apply(q, k, v, self.spec, self.scaling, plan, rank, self.group,
                                     self.ops, self.head_groups, self.group_key_plans)
        return out.reshape(B, S, Hq * D)
