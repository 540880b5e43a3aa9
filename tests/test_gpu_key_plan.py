"""GPU: the backward's key plan (precomputed user lists of the tensor-core key
side) against the key side that searches the pattern itself.

Within a tile the plan lists the users in the key kernel's own order, so
for layers without summed long-run chunks dK / dV are bit-identical; where a
column holds summed chunks (layer 7 here: slot 0 of the first heads keeps
one key over whole 1024-query chunks) the pieces are summed in another
order, so those are compared within the parity tolerance of the oracle
comparator instead.  dQ does not depend on the plan.
"""
import numpy as np
import pytest
import torch

from oracle import compare, naive, pattern

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def randn(*shape, dtype, gen):
    return torch.randn(*shape, generator=gen).to(DEV, dtype)


def _fwd_bwd(ops, q, k, v, do, spec, plan=None, **kw):
    scale = q.shape[-1] ** -0.5
    pr = ops.probs_buffer(q, k, spec, row_offset=kw.get("row_offset", 0),
                          kv_len=kw.get("kv_len"), kv_offset=kw.get("kv_offset", 0))
    o, lse = ops.forward(q, k, v, spec, scale, probs=pr, **kw)
    return ops.backward(q, k, v, o, lse, do, spec, scale, probs=pr, key_plan=plan, **kw)


@pytest.mark.parametrize("dtype,Hq,Hkv,D,L,layer", [
    (torch.bfloat16, 8, 2, 128, 5000, 1), (torch.bfloat16, 8, 2, 128, 5000, 4),
    (torch.bfloat16, 8, 2, 128, 5000, 7), (torch.float16, 4, 4, 128, 3000, 3),
    (torch.bfloat16, 6, 2, 64, 4100, 5), (torch.bfloat16, 16, 2, 128, 2048, 6),
    (torch.float16, 4, 2, 64, 300, 2)])
def test_planned_key_side_matches_search(esa, dtype, Hq, Hkv, D, L, layer):
    ops = esa.ops
    g = torch.Generator().manual_seed(Hq * 7 + D + layer + L)
    q, do = randn(1, Hq, L, D, dtype=dtype, gen=g), randn(1, Hq, L, D, dtype=dtype, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dtype, gen=g), randn(1, Hkv, L, D, dtype=dtype, gen=g)
    spec = ops.PatternSpec(layer, 8, 64)
    plan = ops.key_plan(q, k, spec)
    assert plan is not None
    ops.device_errors()
    dq0, dk0, dv0 = _fwd_bwd(ops, q, k, v, do, spec)
    dq1, dk1, dv1 = _fwd_bwd(ops, q, k, v, do, spec, plan)
    assert ops.device_errors() == 0
    assert torch.equal(dq0, dq1)
    if layer == 7 and L >= 1024:
        for a, b, t in ((dk1, dk0, "dk"), (dv1, dv0, "dv")):
            ok, mx, mean = compare.within(a.float(), b.float(), dtype)
            assert ok, (t, mx, mean)
    else:
        assert torch.equal(dk0, dk1) and torch.equal(dv0, dv1)


def test_planned_key_side_against_oracle_with_offsets(esa):
    """A sequence-split rank's call (row_offset, kv_offset, K/V sliced to the
    rank's key range) and a head-split call (head_offset / pattern_heads) with
    their plans, against the fp32 oracle."""
    ops = esa.ops
    g = torch.Generator().manual_seed(91)
    dt = torch.bfloat16
    B, Hq, Hkv, L, D, w, layer = 1, 8, 2, 8192, 128, 64, 5
    q, do = randn(B, Hq, L, D, dtype=dt, gen=g), randn(B, Hq, L, D, dtype=dt, gen=g)
    k, v = randn(B, Hkv, L, D, dtype=dt, gen=g), randn(B, Hkv, L, D, dtype=dt, gen=g)
    spec = ops.PatternSpec(layer, 8, w)
    scale = D ** -0.5
    # rank 1 of a 2-way sequence split: queries [S, L), keys from lo
    S = L // 2
    idx, mask, _ = pattern.prepared_indices(Hq, w, layer, 8, L, S, L, np.arange(S, L))
    lo = int(idx[mask.astype(bool)].min())
    qr, dor, kr, vr = q[:, :, S:], do[:, :, S:], k[:, :, lo:], v[:, :, lo:]
    kw = dict(row_offset=S, kv_len=L, kv_offset=lo)
    plan = ops.key_plan(qr, kr, spec, **kw)
    dq, dk, dv = _fwd_bwd(ops, qr, kr, vr, dor, spec, plan, **kw)
    _, rdq, rdk, rdv = naive.naive_forward_backward_manual(
        qr.float(), k.float(), v.float(), dor.float(), torch.from_numpy(idx).to(DEV),
        torch.from_numpy(mask).to(DEV), scale, Hq // Hkv, chunk=2048)
    for got, want, t in ((dq, rdq, "dq"), (dk, rdk[:, :, lo:], "dk"), (dv, rdv[:, :, lo:], "dv")):
        ok, mx, mean = compare.within(got, want, dt)
        assert ok, ("sequence split", t, mx, mean)
    # the second half of the heads, as a head-split share, equals the
    # all-heads call's slices
    dq_all, dk_all, dv_all = _fwd_bwd(ops, q, k, v, do, spec, ops.key_plan(q, k, spec))
    sub = spec.heads(Hq, Hq // 2)
    qs, dos = q[:, Hq // 2:].contiguous(), do[:, Hq // 2:].contiguous()
    ks, vs = k[:, Hkv // 2:].contiguous(), v[:, Hkv // 2:].contiguous()
    dqs, dks, dvs = _fwd_bwd(ops, qs, ks, vs, dos, sub, ops.key_plan(qs, ks, sub))
    assert torch.equal(dqs, dq_all[:, Hq // 2:])
    assert torch.equal(dks, dk_all[:, Hkv // 2:]) and torch.equal(dvs, dv_all[:, Hkv // 2:])
    assert ops.device_errors() == 0


def test_plan_of_another_problem_is_rejected(esa):
    """A plan of the same size but another layer: the key side records
    ESA_DEVERR_PLAN and writes nothing (no fault); a plan of another size is
    refused before any launch."""
    ops = esa.ops
    g = torch.Generator().manual_seed(5)
    dt = torch.bfloat16
    q, do = randn(1, 8, 2048, 128, dtype=dt, gen=g), randn(1, 8, 2048, 128, dtype=dt, gen=g)
    k, v = randn(1, 2, 2048, 128, dtype=dt, gen=g), randn(1, 2, 2048, 128, dtype=dt, gen=g)
    spec3, spec5 = ops.PatternSpec(3, 8, 64), ops.PatternSpec(5, 8, 64)
    plan5 = ops.key_plan(q, k, spec5)
    ops.device_errors()
    _fwd_bwd(ops, q, k, v, do, spec3, plan5)
    assert ops.device_errors() == esa._lib.DEVERR_PLAN
    short = ops.key_plan(q[:, :, :1024], k[:, :, :1024], spec3)
    with pytest.raises(esa._lib.EsaError, match="key_plan"):
        _fwd_bwd(ops, q, k, v, do, spec3, short)


def test_module_builds_and_reuses_its_plan(esa):
    """The module builds its plan at the first backward and reuses it; the
    gradients equal those of the module with the plan disabled."""
    g = torch.Generator().manual_seed(17)
    dt = torch.bfloat16
    B, Hq, Hkv, L, D = 1, 8, 2, 3000, 128
    q, k, v = (randn(B, h, L, D, dtype=dt, gen=g) for h in (Hq, Hkv, Hkv))
    do = randn(B, L, Hq * D, dtype=dt, gen=g)
    grads = []
    for enabled in (True, False):
        m = esa.ElasticSparseAttention(4, 8, Hq, D, 64, L, num_key_value_heads=Hkv)
        m.key_plans.enabled = enabled
        for _ in range(2):
            qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
            out, _ = m(qq, kk, vv)
            out.backward(do)
        plan = m.key_plans._plan
        assert (plan is not None) == enabled
        grads.append((qq.grad, kk.grad, vv.grad))
    for a, b in zip(*grads):
        assert torch.equal(a, b)
