"""GPU: the decoder-layer harness kernels (RMSNorm with residual add, RoPE,
SwiGLU) against plain torch float32 formulas, and the decoder stack (loss and
every parameter gradient) against a plain-torch float32 restatement whose
attention is the oracle's restatement of the reference's naive path.

Tolerances: float32 kernels within 1e-5 relative of the float32 formulas
(1e-4 for reductions over rows); 16-bit kernels within one output rounding
(2^-8 relative for bf16, 2^-11 for fp16, plus 1e-6 absolute).  The stack in
float32 within 1e-4 (loss) and 1e-3 (gradients, relative to each gradient's
largest entry); in bf16 within 2e-2 (loss) and 6e-2 (gradients).
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
REL = {torch.float32: 1e-5, torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}


def close(got, want, dtype, what, rel=None, atol=1e-6):
    rel = REL[dtype] if rel is None else rel
    err = (got.float() - want.float()).abs()
    bound = atol + rel * want.float().abs() * 1.01 + rel * 1e-3 * want.float().abs().max()
    worst = (err - bound).max().item()
    assert worst <= 0, f"{what}: max err {err.max().item():.3e} exceeds bound by {worst:.3e}"


@pytest.fixture(scope="module")
def lops():
    import elastic_sparse_attention_b200 as esa
    return esa.layer_ops


DTYPES = [torch.float32, torch.bfloat16, torch.float16]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,dim", [(37, 64), (1000, 4096), (5, 256), (300, 2048)])
@pytest.mark.parametrize("with_res", [False, True])
def test_rmsnorm_forward_backward(lops, dtype, rows, dim, with_res):
    if dim // (16 // torch.empty((), dtype=dtype).element_size()) > 1024:
        pytest.skip("dim above one vector per thread")
    g = torch.Generator().manual_seed(rows + dim)
    x = torch.randn(rows, dim, generator=g).to(DEV, dtype)
    r = torch.randn(rows, dim, generator=g).to(DEV, dtype) if with_res else None
    w = (1 + 0.1 * torch.randn(dim, generator=g)).to(DEV, dtype)
    dy = torch.randn(rows, dim, generator=g).to(DEV, dtype)
    dh_in = torch.randn(rows, dim, generator=g).to(DEV, dtype) if with_res else None
    h, y, rstd = lops.rmsnorm_forward(x, w, 1e-6, residual=r)
    hr = (x.float() + r.float()).to(dtype) if with_res else x
    assert torch.equal(h, hr)
    hf = hr.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
    close(y, ref.detach(), dtype, "rmsnorm y")
    close(rstd, torch.rsqrt(hr.float().pow(2).mean(-1) + 1e-6), torch.float32, "rstd", rel=1e-5)
    ref.backward(dy.float())
    dh, dw = lops.rmsnorm_backward(h, w, rstd, dy, dh_in=dh_in)
    want_dh = hf.grad + (dh_in.float() if with_res else 0)
    close(dh, want_dh, dtype, "rmsnorm dh", atol=1e-5)
    # dw sums over rows: float32 rounding of the sum order, then one output rounding
    close(dw, wf.grad, dtype, "rmsnorm dw", rel=max(REL[dtype], 1e-4), atol=1e-4)


def rope_ref(x, positions, inv_freq, inverse=False):
    ang = positions.float()[:, None] * inv_freq[None, :]
    cos, sin = ang.cos(), ang.sin()
    if inverse:
        sin = -sin
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("Hq,Hkv,D,L", [(4, 2, 64, 50), (32, 32, 128, 300), (8, 1, 16, 7)])
def test_rope_in_place_on_fused_qkv(lops, dtype, Hq, Hkv, D, L):
    if dtype != torch.float32 and D < 16:
        pytest.skip("half-row below 16 bytes")
    B = 2
    g = torch.Generator().manual_seed(Hq + D + L)
    qkv = torch.randn(B, L, Hq + 2 * Hkv, D, generator=g).to(DEV, dtype)
    orig = qkv.clone()
    q = qkv[:, :, :Hq].transpose(1, 2)
    k = qkv[:, :, Hq:Hq + Hkv].transpose(1, 2)
    inv = lops.rope_inv_freq(D, 10000.0, DEV)
    pos = torch.arange(L, device=DEV) * 97 + 11        # large positions: large angles
    lops.rope_(q, k, inv, positions=pos)
    want_q = rope_ref(orig[:, :, :Hq].transpose(1, 2), pos, inv)
    want_k = rope_ref(orig[:, :, Hq:Hq + Hkv].transpose(1, 2), pos, inv)
    close(q, want_q, dtype, "rope q", atol=1e-5)
    close(k, want_k, dtype, "rope k", atol=1e-5)
    assert torch.equal(qkv[:, :, Hq + Hkv:], orig[:, :, Hq + Hkv:])   # v untouched
    lops.rope_(q, k, inv, positions=pos, inverse=True)
    tol = 1e-5 if dtype == torch.float32 else 4 * REL[dtype]
    assert (qkv.float() - orig.float()).abs().max().item() <= tol * orig.float().abs().max().item()
    # default positions 0..L-1
    q2 = orig[:, :, :Hq].transpose(1, 2).contiguous()
    lops.rope_(q2, None, inv)
    close(q2, rope_ref(orig[:, :, :Hq].transpose(1, 2), torch.arange(L, device=DEV), inv), dtype,
          "rope default positions", atol=1e-5)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,ffn", [(33, 64), (513, 11008), (4, 8)])
def test_swiglu_forward_backward(lops, dtype, rows, ffn):
    if ffn * torch.empty((), dtype=dtype).element_size() % 16:
        pytest.skip("row width below 16 bytes")
    g = torch.Generator().manual_seed(rows + ffn)
    gu = (3 * torch.randn(rows, 2 * ffn, generator=g)).to(DEV, dtype)
    dout = torch.randn(rows, ffn, generator=g).to(DEV, dtype)
    out = lops.swiglu_forward(gu)
    guf = gu.float().requires_grad_(True)
    gate, up = guf.chunk(2, dim=-1)
    ref = torch.nn.functional.silu(gate) * up
    close(out, ref.detach(), dtype, "swiglu out", rel=max(REL[dtype], 2e-6))
    ref.backward(dout.float())
    dgu, out2 = lops.swiglu_backward(gu, dout)
    assert torch.equal(out2, out)
    close(dgu, guf.grad, dtype, "swiglu dgate_up", rel=max(REL[dtype], 2e-6), atol=1e-5)


def _stack_and_reference(dtype, cfg):
    import elastic_sparse_attention_b200 as esa
    from decoder_reference import reference_loss
    m = esa.ElasticDecoderStack(vocab_size=cfg["V"], hidden_size=cfg["d"],
                                num_hidden_layers=cfg["nl"], num_attention_heads=cfg["Hq"],
                                num_key_value_heads=cfg["Hkv"], intermediate_size=cfg["F"],
                                attention_length=cfg["w"], max_seq_len=cfg["L"],
                                loss_chunk_rows=cfg["chunk"], dtype=dtype, device=DEV, seed=3,
                                activation_checkpointing=cfg.get("ckpt", False))
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg["V"], (cfg["B"], cfg["L"]), generator=g).to(DEV)
    loss = m(ids, labels=ids)
    loss.backward()
    params = {n: p.detach().float().clone().requires_grad_(True) for n, p in m.named_parameters()}
    rcfg = dict(Hq=cfg["Hq"], Hkv=cfg["Hkv"], D=cfg["d"] // cfg["Hq"], nl=cfg["nl"], w=cfg["w"],
                eps=1e-6, inv_freq=m.inv_freq)
    ref = reference_loss(params, ids, ids, rcfg)
    ref.backward()
    return m, loss, ref, params


CFG = dict(V=512, d=256, nl=3, Hq=4, Hkv=2, F=384, w=16, L=300, B=2, chunk=128)


@pytest.mark.parametrize("ckpt", [False, True])
def test_decoder_stack_fp32_matches_reference(ckpt):
    m, loss, ref, params = _stack_and_reference(torch.float32, dict(CFG, ckpt=ckpt))
    assert abs(loss.item() - ref.item()) <= 1e-4 * abs(ref.item())
    for n, p in m.named_parameters():
        want = params[n].grad
        err = (p.grad.float() - want).abs().max().item()
        assert err <= 1e-3 * want.abs().max().item() + 1e-7, f"{n}: {err:.3e}"


def test_decoder_stack_bf16_matches_reference():
    cfg = dict(CFG, L=520, w=64, d=512, Hq=4, Hkv=4, F=1024, nl=4)
    m, loss, ref, params = _stack_and_reference(torch.bfloat16, cfg)
    assert abs(loss.item() - ref.item()) <= 2e-2 * abs(ref.item())
    for n, p in m.named_parameters():
        want = params[n].grad
        err = (p.grad.float() - want).abs().max().item()
        assert err <= 6e-2 * want.abs().max().item(), f"{n}: {err:.3e}"
        cos = torch.nn.functional.cosine_similarity(p.grad.float().flatten(), want.flatten(), dim=0)
        assert cos.item() > 0.995, f"{n}: cosine {cos.item():.4f}"
