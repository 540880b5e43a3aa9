"""Chunked fp32 torch restatement of the reference's "naive" attention path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``ElasticSparseAttention._naive_forward`` (``elastic_sparse_attention.py:624-680``):
GQA by ``repeat_interleave`` (``:632-634``), ``take_along_dim`` gathers of the
``w`` key/value rows of every query (``:655-660``), scaled scores (``:664-665``),
``masked_fill(finfo.min)`` of masked slots (``:669``), softmax in float32
(``:673``) and the weighted sum of gathered values (``:678``).  The only
difference is bookkeeping: query rows are processed in chunks so that the
``[B, H, n, w, D]`` gathers fit in memory (each output row depends only on its
own index row, so chunking changes nothing numerically).  Gradients come from
torch autograd through the same ops, exactly like the reference's fallback
(the reference's naive path has no hand-written backward).

The reference's naive path calls ``_get_prepared_indices_and_mask(q_len,
kv_len)`` with one argument too many (``:638`` vs ``:574``); the prepared
indices here are computed by :func:`oracle.pattern.prepared_indices`, which
follows ``_triton_forward``'s slicing and clamping (``:600-615``).
"""
from __future__ import annotations

import math

import torch


def _gather_rows(x: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """x [B, H, Lkv, D], idx [H, n, w] -> [B, H, n, w, D] (``:655-660``)."""
    B, H, _, D = x.shape
    ix = idx.unsqueeze(0).unsqueeze(-1).expand(B, -1, -1, -1, D)
    return torch.take_along_dim(x.unsqueeze(2), ix, dim=3)


def naive_chunk(q, k, v, idx, mask, scale: float):
    """One chunk of query rows: q [B,H,n,D], k/v [B,H,Lkv,D] (already repeated).

    Returns (out [B,H,n,D], weights [B,H,n,w]) in q's dtype, as ``:662-680``.
    """
    gk = _gather_rows(k, idx)
    gv = _gather_rows(v, idx)
    scores = torch.matmul(q.unsqueeze(3), gk.transpose(-1, -2)).squeeze(3)
    scores = scores * scale
    scores = scores.masked_fill(mask.unsqueeze(0) < 1, torch.finfo(scores.dtype).min)
    w = torch.softmax(scores, dim=-1, dtype=torch.float32).type_as(q)
    out = torch.matmul(w.unsqueeze(-2), gv).squeeze(-2)
    return out, w


def _chunk_rows(B, H, w, D, budget_elems=1 << 26):
    per_row = max(1, B * H * w * D * 2)
    return max(1, budget_elems // per_row)


def naive_forward(q, k, v, idx, mask, scale: float, num_kv_groups: int,
                  chunk: int | None = None, return_weights: bool = False):
    """Forward over all query rows. q [B,Hq,n,D]; k,v [B,Hkv,Lkv,D];
    idx/mask [Hq, n, w] prepared (sliced + clamped) int64 tensors."""
    if num_kv_groups > 1:
        k = k.repeat_interleave(num_kv_groups, dim=1)
        v = v.repeat_interleave(num_kv_groups, dim=1)
    B, H, n, D = q.shape
    w = idx.shape[-1]
    step = chunk or _chunk_rows(B, H, w, D)
    outs, ws = [], []
    for r0 in range(0, n, step):
        r1 = min(n, r0 + step)
        o, a = naive_chunk(q[:, :, r0:r1], k, v, idx[:, r0:r1], mask[:, r0:r1], scale)
        outs.append(o)
        if return_weights:
            ws.append(a)
    out = torch.cat(outs, dim=2)
    return (out, torch.cat(ws, dim=2)) if return_weights else (out, None)


def naive_forward_backward(q, k, v, do, idx, mask, scale: float, num_kv_groups: int,
                           chunk: int | None = None):
    """Forward output and (dq, dk, dv) by autograd through the naive ops.

    Chunked over query rows; dk/dv accumulate across chunks in float32 (each
    chunk's autograd already sums its own scatter-adds).
    """
    B, Hq, n, D = q.shape
    w = idx.shape[-1]
    step = chunk or max(1, _chunk_rows(B, Hq, w, D) // 4)
    out = torch.empty_like(q)
    dq = torch.empty_like(q)
    dk = torch.zeros(k.shape, dtype=torch.float32, device=k.device)
    dv = torch.zeros(v.shape, dtype=torch.float32, device=v.device)
    for r0 in range(0, n, step):
        r1 = min(n, r0 + step)
        qc = q[:, :, r0:r1].detach().clone().requires_grad_(True)
        kc = k.detach().clone().requires_grad_(True)
        vc = v.detach().clone().requires_grad_(True)
        kk, vv = kc, vc
        if num_kv_groups > 1:
            kk = kc.repeat_interleave(num_kv_groups, dim=1)
            vv = vc.repeat_interleave(num_kv_groups, dim=1)
        o, _ = naive_chunk(qc, kk, vv, idx[:, r0:r1], mask[:, r0:r1], scale)
        gq, gk, gv = torch.autograd.grad(o, (qc, kc, vc), do[:, :, r0:r1])
        out[:, :, r0:r1] = o.detach()
        dq[:, :, r0:r1] = gq
        dk += gk.float()
        dv += gv.float()
    return out, dq, dk.to(k.dtype), dv.to(v.dtype)


def default_scale(head_dim: int) -> float:
    """``self.scaling = head_dim ** -0.5`` (``:444``)."""
    return head_dim ** -0.5


def lse_rows(q, k, idx, mask, scale: float, num_kv_groups: int):
    """Per-row log-sum-exp of the masked scaled scores (float64), [B, Hq, n]."""
    if num_kv_groups > 1:
        k = k.repeat_interleave(num_kv_groups, dim=1)
    gk = _gather_rows(k.double(), idx)
    s = torch.matmul(q.double().unsqueeze(3), gk.transpose(-1, -2)).squeeze(3) * scale
    s = s.masked_fill(mask.unsqueeze(0) < 1, -math.inf)
    return torch.logsumexp(s, dim=-1)


def naive_forward_backward_manual(q, k, v, do, idx, mask, scale: float, num_kv_groups: int,
                                  chunk: int = 1024):
    """The same forward and gradients as :func:`naive_forward_backward`, with
    the backward written out by hand (the exact ops autograd performs through
    ``:664-678``: softmax backward ``p * (g - sum(p * g))``, matmul backward,
    and the scatter-add that ``take_along_dim`` backward does).  Computes in
    float32 on the inputs' device, so it can check full-size GPU results.
    Returns (out, dq, dk, dv) as float32 tensors.
    """
    B, Hq, n, D = q.shape
    Hkv, Lkv = k.shape[1], k.shape[2]
    w = idx.shape[-1]
    dev = q.device
    qf, dof = q.float(), do.float()
    kr, vr = k.float(), v.float()
    if num_kv_groups > 1:
        kr = kr.repeat_interleave(num_kv_groups, dim=1)
        vr = vr.repeat_interleave(num_kv_groups, dim=1)
    out = torch.empty((B, Hq, n, D), dtype=torch.float32, device=dev)
    dq = torch.empty_like(out)
    dkr = torch.zeros((B, Hq * Lkv, D), dtype=torch.float32, device=dev)
    dvr = torch.zeros_like(dkr)
    hoff = (torch.arange(Hq, device=dev) * Lkv).view(Hq, 1, 1)
    neg = torch.finfo(torch.float32).min
    for r0 in range(0, n, chunk):
        r1 = min(n, r0 + chunk)
        ix, mk = idx[:, r0:r1].to(dev), mask[:, r0:r1].to(dev)
        gk = _gather_rows(kr, ix)
        gv = _gather_rows(vr, ix)
        qc, dc = qf[:, :, r0:r1], dof[:, :, r0:r1]
        s = torch.einsum("bhcd,bhcwd->bhcw", qc, gk) * scale
        s = s.masked_fill(mk.unsqueeze(0) < 1, neg)
        p = torch.softmax(s, dim=-1)
        out[:, :, r0:r1] = torch.einsum("bhcw,bhcwd->bhcd", p, gv)
        dp = torch.einsum("bhcd,bhcwd->bhcw", dc, gv)
        ds = p * (dp - (p * dp).sum(-1, keepdim=True)) * scale
        dq[:, :, r0:r1] = torch.einsum("bhcw,bhcwd->bhcd", ds, gk)
        flat = (ix + hoff).reshape(-1)
        c = r1 - r0
        dkr.index_add_(1, flat, torch.einsum("bhcw,bhcd->bhcwd", ds, qc).reshape(B, Hq * c * w, D))
        dvr.index_add_(1, flat, torch.einsum("bhcw,bhcd->bhcwd", p, dc).reshape(B, Hq * c * w, D))
        del gk, gv, s, p, dp, ds
    dk = dkr.view(B, Hkv, num_kv_groups, Lkv, D).sum(2)
    dv = dvr.view(B, Hkv, num_kv_groups, Lkv, D).sum(2)
    return out, dq, dk, dv


def naive_forward_backward_keep(q, k, v, do, idx, mask, scale: float, num_kv_groups: int,
                                keep, p: float):
    """Naive path with dropout given as an explicit keep mask [B, H, n, w]:
    weights = softmax(scores) * keep / (1 - p) (``torch.dropout`` semantics,
    ``:674``), out = weights . V, gradients by autograd.  float32 throughout.
    Returns (out, weights, dq, dk, dv)."""
    qf, kf, vf = (t.detach().float().clone().requires_grad_(True) for t in (q, k, v))
    kk, vv = kf, vf
    if num_kv_groups > 1:
        kk = kf.repeat_interleave(num_kv_groups, dim=1)
        vv = vf.repeat_interleave(num_kv_groups, dim=1)
    gk, gv = _gather_rows(kk, idx), _gather_rows(vv, idx)
    s = torch.einsum("bhcd,bhcwd->bhcw", qf, gk) * scale
    s = s.masked_fill(mask.unsqueeze(0) < 1, torch.finfo(torch.float32).min)
    w = torch.softmax(s, dim=-1) * keep.float() / (1.0 - p)
    out = torch.einsum("bhcw,bhcwd->bhcd", w, gv)
    dq, dk, dv = torch.autograd.grad(out, (qf, kf, vf), do.float())
    return out.detach(), w.detach(), dq, dk, dv
