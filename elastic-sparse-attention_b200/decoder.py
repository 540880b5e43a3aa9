"""Decoder-layer stack around elastic sparse attention (the C4 configuration).

The reference ships the attention module only (it is meant to sit inside an
external decoder layer), so this harness has no reference counterpart.  It is
a pre-norm Llama-style stack: token embedding, per layer RMSNorm -> fused QKV
projection -> rotary embedding -> elastic sparse attention (layer_idx = layer
number, num_hidden_layers = the stack depth) -> output projection -> residual
add -> RMSNorm -> SwiGLU MLP -> residual add, then a final RMSNorm, the LM
head and the mean next-token cross entropy.

Built for B200 without layout copies:

* The QKV projection writes one [B, L, Hq + 2 Hkv, D] buffer.  RoPE rotates
  its q and k parts in place and the attention kernels read q, k, v straight
  from it through strides; the attention output is written as [B, L, Hq, D],
  the output projection's input, with no transpose.  In the backward the
  attention kernels write dQ, dK, dV into the parts of one gradient buffer of
  the same layout, the inverse rotation runs in place on it, and it feeds the
  projection's weight and input gradients directly (the module path
  ``transpose(1, 2).contiguous()`` of the reference's callers, :244 / :763,
  never happens).
* Residual adds are fused into the following RMSNorm; SwiGLU runs on the
  fused gate/up projection output and recomputes its output in the backward
  instead of keeping it.
* The LM head and loss run over row chunks and produce their gradients in the
  forward, so the [L, vocab] logits never exist in full.
* GEMMs are cuBLAS through torch (bf16 in, fp32 accumulate).

``activation_checkpointing=True`` recomputes each layer in the backward
(keeps only its input), for lengths whose activations do not fit.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F
import torch.utils.checkpoint

from . import layer_ops, ops
from .attention import KeyPlanCache, _ensure_monotone
from .ops import PatternSpec


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps: float):
        x = x.contiguous()
        _, y, rstd = layer_ops.rmsnorm_forward(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx, dw = layer_ops.rmsnorm_backward(x, w, rstd, dy)
        return dx, dw, None


class _AddRMSNorm(torch.autograd.Function):
    """(h, y) = (a + b, rmsnorm(a + b) * w)."""

    @staticmethod
    def forward(ctx, a, b, w, eps: float):
        h, y, rstd = layer_ops.rmsnorm_forward(a.contiguous(), w, eps, residual=b.contiguous())
        ctx.save_for_backward(h, w, rstd)
        return h, y

    @staticmethod
    def backward(ctx, dh, dy):
        h, w, rstd = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(h)
        dx, dw = layer_ops.rmsnorm_backward(h, w, rstd, dy, dh_in=dh)
        return dx, dx, dw, None


class _AttentionBlock(torch.autograd.Function):
    """a = attention(rope(y Wqkv^T)) Wo^T with the layouts described above."""

    @staticmethod
    def forward(ctx, y, wqkv, wo, spec: PatternSpec, heads: tuple, inv_freq, positions,
                plans=None):
        Hq, Hkv, D = heads
        B, L, d = y.shape
        qkv = torch.matmul(y, wqkv.t())                       # [B, L, (Hq + 2 Hkv) D]
        q, k, v = _split_heads(qkv, B, L, Hq, Hkv, D)
        layer_ops.rope_(q, k, inv_freq, positions)
        scale = D ** -0.5
        probs = ops.probs_buffer(q, k, spec)                  # kept for the backward
        o, lse = ops.forward(q, k, v, spec, scale, probs=probs)   # o: view of [B, L, Hq, D]
        o_rows = o.transpose(1, 2).reshape(B, L, Hq * D)      # a view, no copy
        a = torch.matmul(o_rows, wo.t())
        ctx.save_for_backward(y, wqkv, wo, qkv, o_rows, lse, inv_freq, positions, probs)
        ctx.meta = (spec, heads, scale)
        ctx.plans = plans
        return a

    @staticmethod
    def backward(ctx, da):
        y, wqkv, wo, qkv, o_rows, lse, inv_freq, positions, probs = ctx.saved_tensors
        spec, (Hq, Hkv, D), scale = ctx.meta
        B, L, d = y.shape
        da = da.contiguous()
        do_rows = torch.matmul(da, wo)                        # [B, L, Hq D]
        dwo = torch.matmul(da.reshape(-1, d).t(), o_rows.reshape(-1, Hq * D))
        q, k, v = _split_heads(qkv, B, L, Hq, Hkv, D)
        o = o_rows.view(B, L, Hq, D).transpose(1, 2)
        dqkv = torch.empty_like(qkv)
        dq, dk, dv = _split_heads(dqkv, B, L, Hq, Hkv, D)
        _ensure_monotone(Hq, spec, max(L, 2), y.device)
        plan = ctx.plans.get(q, k, spec) if ctx.plans is not None else None
        ops.backward(q, k, v, o, lse, do_rows.view(B, L, Hq, D).transpose(1, 2), spec, scale,
                     dq=dq, dk=dk, dv=dv, probs=probs, key_plan=plan)
        del do_rows
        layer_ops.rope_(dq, dk, inv_freq, positions, inverse=True)
        dy = torch.matmul(dqkv, wqkv)
        dwqkv = torch.matmul(dqkv.reshape(-1, dqkv.shape[-1]).t(), y.reshape(-1, d))
        return dy, dwqkv, dwo, None, None, None, None, None


def _split_heads(qkv, B, L, Hq, Hkv, D):
    """q [B, Hq, L, D], k / v [B, Hkv, L, D] views of a [B, L, (Hq+2Hkv) D] buffer."""
    x = qkv.view(B, L, Hq + 2 * Hkv, D)
    return (x[:, :, :Hq].transpose(1, 2), x[:, :, Hq:Hq + Hkv].transpose(1, 2),
            x[:, :, Hq + Hkv:].transpose(1, 2))


class _MLPBlock(torch.autograd.Function):
    """out = swiglu(y Wgu^T) Wd^T, rows of Wgu = [gate; up]."""

    @staticmethod
    def forward(ctx, y, wgu, wd):
        gu = torch.matmul(y, wgu.t())
        m = layer_ops.swiglu_forward(gu)
        out = torch.matmul(m, wd.t())
        ctx.save_for_backward(y, wgu, wd, gu)
        return out

    @staticmethod
    def backward(ctx, dout):
        y, wgu, wd, gu = ctx.saved_tensors
        d = y.shape[-1]
        dout = dout.contiguous()
        dm = torch.matmul(dout, wd)
        dgu, m = layer_ops.swiglu_backward(gu, dm, recompute=True)
        del dm
        dwd = torch.matmul(dout.reshape(-1, d).t(), m.reshape(-1, m.shape[-1]))
        del m
        dy = torch.matmul(dgu, wgu)
        dwgu = torch.matmul(dgu.reshape(-1, dgu.shape[-1]).t(), y.reshape(-1, d))
        return dy, dwgu, dwd


class _LMHeadCrossEntropy(torch.autograd.Function):
    """Mean cross entropy of softmax(y W^T) against targets (-100 = ignored),
    over row chunks; the gradients are formed in the forward."""

    @staticmethod
    def forward(ctx, y, w, targets, chunk: int):
        d = y.shape[-1]
        y2 = y.reshape(-1, d)
        t = targets.reshape(-1)
        n = y2.shape[0]
        dy = torch.empty_like(y2)
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        loss_sum = torch.zeros((), dtype=torch.float32, device=y.device)
        count = (t != -100).sum()
        for s in range(0, n, chunk):
            yc, tc = y2[s:s + chunk], t[s:s + chunk]
            logits = torch.matmul(yc, w.t()).float()
            lse = torch.logsumexp(logits, dim=-1)
            valid = tc != -100
            tcl = tc.clamp_min(0)
            tgt = logits.gather(1, tcl[:, None])[:, 0]
            loss_sum += ((lse - tgt) * valid).sum()
            p = logits.sub_(lse[:, None]).exp_()              # softmax, in place
            p[torch.arange(p.shape[0], device=p.device), tcl] -= 1.0
            p.mul_(valid[:, None])
            g = p.to(y.dtype)
            del p, logits
            dy[s:s + chunk] = torch.matmul(g, w)
            dw += torch.matmul(g.t(), yc).float()
        inv = 1.0 / count.clamp_min(1).float()
        ctx.save_for_backward(dy, dw, inv)
        ctx.shape = y.shape
        ctx.w_dtype = w.dtype
        return loss_sum * inv

    @staticmethod
    def backward(ctx, dloss):
        dy, dw, inv = ctx.saved_tensors
        s = dloss * inv
        return (dy * s.to(dy.dtype)).view(ctx.shape), (dw * s).to(ctx.w_dtype), None, None


class ElasticDecoderLayerWeights(nn.Module):
    """The parameters of one decoder layer (pre-norm, fused QKV and gate/up)."""

    def __init__(self, hidden: int, Hq: int, Hkv: int, D: int, ffn: int, dtype, device):
        super().__init__()
        kw = dict(dtype=dtype, device=device)
        self.input_norm = nn.Parameter(torch.ones(hidden, **kw))
        self.qkv_proj = nn.Parameter(torch.empty((Hq + 2 * Hkv) * D, hidden, **kw))
        self.o_proj = nn.Parameter(torch.empty(hidden, Hq * D, **kw))
        self.post_attention_norm = nn.Parameter(torch.ones(hidden, **kw))
        self.gate_up_proj = nn.Parameter(torch.empty(2 * ffn, hidden, **kw))
        self.down_proj = nn.Parameter(torch.empty(hidden, ffn, **kw))


class ElasticDecoderStack(nn.Module):
    """Token ids -> next-token loss (or final hidden states) through
    ``num_hidden_layers`` decoder layers with elastic sparse attention.

    Defaults are the C4 configuration: 4 layers, hidden 4096, 32 heads of
    128, SwiGLU 11008, RoPE base 10000, vocabulary 32000, attention_length 64.
    Weights are random N(0, 0.02) (norm weights 1) in ``dtype``.
    """

    def __init__(self, vocab_size: int = 32000, hidden_size: int = 4096,
                 num_hidden_layers: int = 4, num_attention_heads: int = 32,
                 num_key_value_heads: int | None = None, head_dim: int | None = None,
                 intermediate_size: int = 11008, rope_theta: float = 10000.0,
                 rms_norm_eps: float = 1e-6, attention_length: int = 64,
                 max_seq_len: int = 262144, activation_checkpointing: bool = False,
                 loss_chunk_rows: int = 8192, dtype=torch.bfloat16, device=None, seed: int = 0):
        super().__init__()
        self.Hq = num_attention_heads
        self.Hkv = num_key_value_heads or num_attention_heads
        if self.Hq % self.Hkv:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        self.D = head_dim or hidden_size // num_attention_heads
        self.hidden = hidden_size
        self.ffn = intermediate_size
        self.eps = rms_norm_eps
        self.max_seq_len = max_seq_len
        self.checkpointing = activation_checkpointing
        self.loss_chunk_rows = loss_chunk_rows
        self.specs = [PatternSpec(i, num_hidden_layers, attention_length)
                      for i in range(num_hidden_layers)]
        # per layer: the backward's key plan for the current shapes
        self.key_plans = [KeyPlanCache() for _ in range(num_hidden_layers)]
        kw = dict(dtype=dtype, device=device)
        self.embed = nn.Parameter(torch.empty(vocab_size, hidden_size, **kw))
        self.layers = nn.ModuleList(
            ElasticDecoderLayerWeights(hidden_size, self.Hq, self.Hkv, self.D, intermediate_size,
                                       dtype, device) for _ in range(num_hidden_layers))
        self.final_norm = nn.Parameter(torch.ones(hidden_size, **kw))
        self.lm_head = nn.Parameter(torch.empty(vocab_size, hidden_size, **kw))
        self.register_buffer("inv_freq", layer_ops.rope_inv_freq(self.D, rope_theta, device),
                             persistent=False)
        g = torch.Generator(device="cpu").manual_seed(seed)
        with torch.no_grad():
            for p in self.parameters():
                if p.dim() == 2:
                    p.copy_(torch.randn(p.shape, generator=g) * 0.02)

    def _layer(self, i: int, h, y, positions):
        lw = self.layers[i]
        a = _AttentionBlock.apply(y, lw.qkv_proj, lw.o_proj, self.specs[i],
                                  (self.Hq, self.Hkv, self.D), self.inv_freq, positions,
                                  self.key_plans[i])
        h, y2 = _AddRMSNorm.apply(h, a, lw.post_attention_norm, self.eps)
        m = _MLPBlock.apply(y2, lw.gate_up_proj, lw.down_proj)
        next_w = self.layers[i + 1].input_norm if i + 1 < len(self.layers) else self.final_norm
        return _AddRMSNorm.apply(h, m, next_w, self.eps)

    def forward(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None,
                positions: torch.Tensor | None = None):
        """input_ids [B, L] -> mean next-token cross entropy against labels
        (shifted by one, -100 ignored), or the final normalised hidden states
        [B, L, hidden] when labels is None."""
        B, L = input_ids.shape
        if L > self.max_seq_len:
            raise ValueError(f"sequence length {L} exceeds max_seq_len {self.max_seq_len}")
        if positions is None:
            positions = torch.arange(L, device=input_ids.device)
        h = F.embedding(input_ids, self.embed)
        y = _RMSNorm.apply(h, self.layers[0].input_norm, self.eps)
        for i in range(len(self.layers)):
            if self.checkpointing and torch.is_grad_enabled():
                h, y = torch.utils.checkpoint.checkpoint(self._layer, i, h, y, positions,
                                                         use_reentrant=False)
            else:
                h, y = self._layer(i, h, y, positions)
        if labels is None:
            return y
        targets = torch.full_like(labels, -100)
        targets[:, :-1] = labels[:, 1:]
        return _LMHeadCrossEntropy.apply(y, self.lm_head, targets, self.loss_chunk_rows)

    def flops_per_token(self, seq_len: int) -> float:
        """Dense GEMM FLOPs per token of one forward + backward (3 x 2 x
        params in the projections and the LM head), without attention."""
        d, f = self.hidden, self.ffn
        per_layer = d * (self.Hq + 2 * self.Hkv) * self.D + self.Hq * self.D * d + 3 * d * f
        return 6.0 * (len(self.layers) * per_layer + self.lm_head.shape[0] * d)
