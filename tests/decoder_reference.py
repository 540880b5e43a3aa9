"""Plain-torch float32 restatement of the decoder stack in
``elastic-sparse-attention_b200/decoder.py`` (test helper): the same layer
order and formulas written with ordinary torch ops, attention by the oracle's
restatement of the reference's naive path, gradients by autograd."""
from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import naive, pattern


def rmsnorm(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope(x, positions, inv_freq):
    """x [B, H, L, D]; rotate-half convention with angle f32(p) * inv_freq."""
    ang = positions.float()[:, None] * inv_freq[None, :]          # [L, D/2]
    cos, sin = ang.cos(), ang.sin()
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def swiglu(gu):
    g, u = gu.chunk(2, dim=-1)
    return F.silu(g) * u


def reference_loss(params: dict, input_ids, labels, cfg: dict):
    """params: float32 tensors named like the module's parameters."""
    B, L = input_ids.shape
    Hq, Hkv, D, nl, w, eps = cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["nl"], cfg["w"], cfg["eps"]
    positions = torch.arange(L, device=input_ids.device)
    inv_freq = cfg["inv_freq"]
    h = F.embedding(input_ids, params["embed"])
    for i in range(nl):
        pre = f"layers.{i}."
        y = rmsnorm(h, params[pre + "input_norm"], eps)
        qkv = (y @ params[pre + "qkv_proj"].t()).view(B, L, Hq + 2 * Hkv, D)
        q = rope(qkv[:, :, :Hq].transpose(1, 2), positions, inv_freq)
        k = rope(qkv[:, :, Hq:Hq + Hkv].transpose(1, 2), positions, inv_freq)
        v = qkv[:, :, Hq + Hkv:].transpose(1, 2)
        idx, mask, _ = pattern.prepared_indices(Hq, w, i, nl, L, L, L)
        o, _ = naive.naive_forward(q, k, v, torch.from_numpy(idx).to(q.device),
                                   torch.from_numpy(mask).to(q.device), D ** -0.5, Hq // Hkv)
        h = h + o.transpose(1, 2).reshape(B, L, Hq * D) @ params[pre + "o_proj"].t()
        y2 = rmsnorm(h, params[pre + "post_attention_norm"], eps)
        h = h + swiglu(y2 @ params[pre + "gate_up_proj"].t()) @ params[pre + "down_proj"].t()
    yf = rmsnorm(h, params["final_norm"], eps)
    logits = yf @ params["lm_head"].t()
    return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]),
                           labels[:, 1:].reshape(-1))
