"""GPU: forward and backward of the CUDA path against the reference's outputs
(fixtures) and against the pinned oracle.

Tolerances (``oracle/compare.py``): fp32 inputs
within max-abs 1e-4 of the fp32 fallback; bf16/fp16 outputs and gradients
within max-abs 2e-2 and mean-abs 2e-3 of an fp32 fallback run on the same
(rounded) inputs, an element's error being the smaller of its distance to the
fp32 result and to that result rounded to the output dtype (the kernels store
16-bit values, which from |x| = 8 up are more than 2e-2 apart in bf16).
"""
import numpy as np
import pytest
import torch

from oracle import compare, naive, pattern

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
F32_TOL = compare.F32_MAX


def run_module(esa, q, k, v, do, layer, nl, w, max_seq_len=None, cache_position=None):
    B, Hq, n, D = q.shape
    m = esa.ElasticSparseAttention(layer, nl, Hq, D, w, max_seq_len or k.shape[2],
                                   num_key_value_heads=k.shape[1])
    qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    out, weights = m(qq, kk, vv, cache_position=cache_position)
    assert weights is None
    assert out.shape == (B, n, Hq * D) and out.dtype == q.dtype
    out.backward(do.transpose(1, 2).reshape(B, n, Hq * D))
    o = out.detach().view(B, n, Hq, D).transpose(1, 2)
    return o, qq.grad, kk.grad, vv.grad


def run_oracle(q, k, v, do, layer, nl, w, cache_position=None, chunk=1024):
    B, Hq, n, D = q.shape
    L = k.shape[2]
    cp = None if cache_position is None else cache_position.cpu().numpy()
    idx, mask, _ = pattern.prepared_indices(Hq, w, layer, nl, L, n, L, cp)
    return naive.naive_forward_backward_manual(
        q.float(), k.float(), v.float(), do.float(), torch.from_numpy(idx).to(q.device),
        torch.from_numpy(mask).to(q.device), D ** -0.5, Hq // k.shape[1], chunk=chunk)


HALF_ULP = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}


def assert_close(got, want, dtype, what):
    ok, mx, mean = compare.within(got, want, dtype)
    assert ok, (what, mx, mean)


def randn(*shape, dtype=torch.float32, scale=1.0, gen=None):
    return (torch.randn(*shape, generator=gen) * scale).to(DEV, dtype)


# ---------------------------------------------------------------------------
# Against the reference's own outputs (fixtures from make_golden.py)
# ---------------------------------------------------------------------------
def test_against_reference_fixtures(esa, naive_small):
    meta_all, arrays = naive_small
    for meta in meta_all:
        name, layer = meta["name"], meta["layer"]
        dtype = torch.float32 if meta["dtype"] == "float32" else torch.bfloat16
        q, k, v, do = (torch.from_numpy(arrays[f"{name}_{t}"]).to(DEV) for t in "q k v do".split())
        cp = meta["cache_position"]
        cpt = None if cp is None else torch.tensor(cp, device=DEV)
        o, dq, dk, dv = run_module(esa, q.to(dtype), k.to(dtype), v.to(dtype), do.to(dtype), layer,
                                   meta["nl"], meta["w"], max_seq_len=meta["L"], cache_position=cpt)
        pre = f"{name}_l{layer}"
        B, Hq, n, D = q.shape
        ref_o = torch.from_numpy(arrays[pre + "_out"]).view(B, n, Hq, D).transpose(1, 2).to(DEV)
        if dtype == torch.float32:
            assert_close(o, ref_o, dtype, pre + " out")
            for g, t in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
                assert_close(g, torch.from_numpy(arrays[f"{pre}_{t}"]).to(DEV), dtype, pre + " " + t)
        else:
            # the fixture's bf16 run is itself a bf16 computation; compare with the
            # fp32 oracle instead and check the bf16 fixture is in the same band
            ro, rdq, rdk, rdv = run_oracle(q.to(dtype), k.to(dtype), v.to(dtype), do.to(dtype),
                                           layer, meta["nl"], meta["w"])
            for g, r, t in ((o, ro, "out"), (dq, rdq, "dq"), (dk, rdk, "dk"), (dv, rdv, "dv")):
                assert_close(g, r, dtype, pre + " " + t)
            assert (ref_o.float() - ro).abs().max().item() < 5e-2


def test_c1_full(esa, c1_rows):
    """C1: B1 H4 L4096 D64 fp32, q/k/v ~ N(0,1) from seed 0, w=64, 8 layers;
    elementwise against the oracle and against the reference rows."""
    torch.manual_seed(0)
    B, H, L, D = 1, 4, 4096, 64
    q, k, v = torch.randn(B, H, L, D), torch.randn(B, H, L, D), torch.randn(B, H, L, D)
    do = torch.randn(B, H, L, D)
    q, k, v, do = (t.to(DEV) for t in (q, k, v, do))
    rows = torch.from_numpy(c1_rows["rows"]).to(DEV)
    for layer in range(8):
        o, dq, dk, dv = run_module(esa, q, k, v, do, layer, 8, 64)
        ro, rdq, rdk, rdv = run_oracle(q, k, v, do, layer, 8, 64)
        assert_close(o, ro, torch.float32, f"l{layer} out")
        assert_close(dq, rdq, torch.float32, f"l{layer} dq")
        assert_close(dk, rdk, torch.float32, f"l{layer} dk")
        assert_close(dv, rdv, torch.float32, f"l{layer} dv")
        ref = torch.from_numpy(c1_rows[f"l{layer}"]).to(DEV)
        got = o.transpose(1, 2).reshape(B, L, H * D)[0, rows]
        assert (got - ref).abs().max().item() <= F32_TOL


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [8, 16, 32, 64, 128, 256])
def test_dtypes_and_head_dims(esa, dtype, D):
    if dtype == torch.float32 and D == 256:
        pytest.skip("fp32 kernels cover head_dim <= 128")
    g = torch.Generator().manual_seed(D)
    B, Hq, Hkv, L = 2, 4, 2, 300
    q, k, v, do = (randn(B, Hq if i in (0, 3) else Hkv, L, D, dtype=dtype, gen=g)
                   for i in range(4))
    for layer in (0, 4, 7):
        o, dq, dk, dv = run_module(esa, q, k, v, do, layer, 8, 64)
        ref = run_oracle(q, k, v, do, layer, 8, 64)
        for got, want, t in zip((o, dq, dk, dv), ref, ("out", "dq", "dk", "dv")):
            assert_close(got, want, dtype, f"{dtype} D{D} l{layer} {t}")


@pytest.mark.parametrize("w,G,nl", [(7, 1, 3), (16, 2, 4), (100, 4, 6), (33, 8, 2), (64, 32, 8),
                                    (1, 1, 1), (256, 2, 8)])
def test_lengths_and_groups(esa, w, G, nl):
    g = torch.Generator().manual_seed(w * 7 + G)
    B, Hkv, L, D = 1, 2, 515, 64
    Hq = Hkv * G
    q, k, v, do = (randn(B, h, L, D, gen=g) for h in (Hq, Hkv, Hkv, Hq))
    for layer in sorted({0, nl // 2, nl - 1}):
        o, dq, dk, dv = run_module(esa, q, k, v, do, layer, nl, w)
        ref = run_oracle(q, k, v, do, layer, nl, w)
        for got, want, t in zip((o, dq, dk, dv), ref, ("out", "dq", "dk", "dv")):
            assert_close(got, want, torch.float32, f"w{w} G{G} l{layer} {t}")


@pytest.mark.parametrize("cache_position", [[299], [0, 17, 299], [250, 3, 3, 128, 64, 299],
                                            [-1, -300, 5]])
def test_decode_cache_position(esa, cache_position):
    """Decode rows (reference :602-608), unsorted and repeated positions,
    negative positions wrapping like torch indexing."""
    g = torch.Generator().manual_seed(11)
    B, Hq, Hkv, L, D = 2, 8, 2, 300, 64
    n = len(cache_position)
    q, do = randn(B, Hq, n, D, gen=g), randn(B, Hq, n, D, gen=g)
    k, v = randn(B, Hkv, L, D, gen=g), randn(B, Hkv, L, D, gen=g)
    cp = torch.tensor(cache_position, device=DEV)
    for layer in (0, 5):
        o, dq, dk, dv = run_module(esa, q, k, v, do, layer, 8, 64, max_seq_len=512,
                                   cache_position=cp)
        wrapped = torch.where(cp < 0, cp + L, cp)
        ref = run_oracle(q, k, v, do, layer, 8, 64, cache_position=wrapped)
        for got, want, t in zip((o, dq, dk, dv), ref, ("out", "dq", "dk", "dv")):
            assert_close(got, want, torch.float32, f"decode l{layer} {t}")


def test_cache_position_out_of_range(esa):
    """Host cache_position and calls that need a backward raise IndexError
    like the reference; a device cache_position under no_grad is not read
    back: its out-of-range rows come out zero and set ESA_DEVERR_QUERY_RANGE."""
    m = esa.ElasticSparseAttention(3, 4, 2, 32, 16, 64)
    q = torch.randn(1, 2, 3, 32, device=DEV)
    k = torch.randn(1, 2, 10, 32, device=DEV)
    esa.ops.device_errors()
    with pytest.raises(IndexError):
        m(q, k, k, cache_position=torch.tensor([10, 0, 1]))
    with pytest.raises(IndexError):
        m(q.requires_grad_(True), k, k, cache_position=torch.tensor([1, -11, 2], device=DEV))
    q = q.detach()
    with torch.no_grad():
        good, _ = m(q, k, k, cache_position=torch.tensor([9, 4, -3], device=DEV))
        assert esa.ops.device_errors() == 0
        out, _ = m(q, k, k, cache_position=torch.tensor([9, 10, -3], device=DEV))
        assert esa.ops.device_errors() == esa._lib.DEVERR_QUERY_RANGE
        assert esa.ops.device_errors() == 0   # reset by the previous read
        out2, _ = m(q, k, k, cache_position=torch.tensor([-11, 4, 7], device=DEV))
        assert esa.ops.device_errors(clear=False) == esa._lib.DEVERR_QUERY_RANGE
        assert esa.ops.device_errors() == esa._lib.DEVERR_QUERY_RANGE
    assert torch.equal(out[:, 0], good[:, 0]) and torch.equal(out[:, 2], good[:, 2])
    assert torch.count_nonzero(out[:, 1]) == 0 and torch.count_nonzero(out2[:, 0]) == 0
    assert torch.equal(out2[:, 1], good[:, 1])
    # a negative device position wraps in the kernel like torch indexing
    ref = run_oracle(q, k, k, q, 3, 4, 16, cache_position=torch.tensor([9, 4, 7], device=DEV))[0]
    assert_close(good.view(1, 3, 2, 32).transpose(1, 2), ref, torch.float32, "wrapped rows")


def test_prefill_shorter_than_cache(esa):
    """q_len < kv_len without cache_position uses pattern rows [0, q_len) (:610-611)."""
    g = torch.Generator().manual_seed(5)
    q, do = randn(1, 4, 100, 64, gen=g), randn(1, 4, 100, 64, gen=g)
    k, v = randn(1, 4, 250, 64, gen=g), randn(1, 4, 250, 64, gen=g)
    o, dq, dk, dv = run_module(esa, q, k, v, do, 3, 8, 64)
    ref = run_oracle(q, k, v, do, 3, 8, 64)
    for got, want, t in zip((o, dq, dk, dv), ref, ("out", "dq", "dk", "dv")):
        assert_close(got, want, torch.float32, "prefill " + t)


def test_strided_inputs(esa):
    """q/k/v as [B, L, H, D] tensors viewed as [B, H, L, D] (HF layout), read in
    place; misaligned views fall back to one contiguous copy."""
    g = torch.Generator().manual_seed(9)
    B, L, Hq, Hkv, D = 2, 200, 8, 4, 64
    q = randn(B, L, Hq, D, dtype=torch.bfloat16, gen=g).transpose(1, 2)
    k = randn(B, L, Hkv, D, dtype=torch.bfloat16, gen=g).transpose(1, 2)
    v = randn(B, L, Hkv, D, dtype=torch.bfloat16, gen=g).transpose(1, 2)
    do = randn(B, Hq, L, D, dtype=torch.bfloat16, gen=g)
    o, dq, dk, dv = run_module(esa, q, k, v, do, 6, 8, 64)
    assert dq.stride() == q.stride()
    ref = run_oracle(q, k, v, do, 6, 8, 64)
    for got, want, t in zip((o, dq, dk, dv), ref, ("out", "dq", "dk", "dv")):
        assert_close(got, want, torch.bfloat16, "strided " + t)
    base = randn(B * Hq * L * D + 1, dtype=torch.bfloat16, gen=g)
    qm = base[1:].view(B, Hq, L, D)   # 2-byte offset: not 16-byte aligned
    o2, *_ = run_module(esa, qm, k, v, do, 6, 8, 64)
    o3, *_ = run_module(esa, qm.contiguous(), k, v, do, 6, 8, 64)
    assert torch.equal(o2, o3)


def test_empty_query(esa):
    m = esa.ElasticSparseAttention(0, 4, 2, 32, 16, 64)
    out, _ = m(torch.randn(1, 2, 0, 32, device=DEV), torch.randn(1, 2, 8, 32, device=DEV),
               torch.randn(1, 2, 8, 32, device=DEV), cache_position=torch.zeros(0, dtype=torch.long, device=DEV))
    assert out.shape == (1, 0, 64)


def test_deterministic(esa):
    """No atomics: two runs give bit-identical outputs and gradients."""
    g = torch.Generator().manual_seed(1)
    q, k, v, do = (randn(1, h, 2048, 128, dtype=torch.bfloat16, gen=g) for h in (16, 4, 4, 16))
    a = run_module(esa, q, k, v, do, 7, 8, 64)
    b = run_module(esa, q, k, v, do, 7, 8, 64)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_c2_forward_full_size(esa):
    """C2: B=2, H=32, L=32768, D=128 bf16, N(0,1) * D^-0.25, forward, all rows
    of three layers against the fp32 oracle."""
    g = torch.Generator().manual_seed(0)
    B, H, L, D = 2, 32, 32768, 128
    s = D ** -0.25
    q, k, v = (randn(B, H, L, D, dtype=torch.bfloat16, scale=s, gen=g) for _ in range(3))
    for layer in (0, 3, 7):
        spec = esa.PatternSpec(layer, 8, 64)
        o, lse = esa.ops.forward(q, k, v, spec, D ** -0.5)
        idx, mask, _ = pattern.prepared_indices(H, 64, layer, 8, L, L, L)
        ro, _ = naive.naive_forward(q.float(), k.float(), v.float(), torch.from_numpy(idx).to(DEV),
                                    torch.from_numpy(mask).to(DEV), D ** -0.5, 1, chunk=2048)
        assert_close(o, ro, torch.bfloat16, f"C2 l{layer}")
        del o, ro


def test_c3_forward_backward_full_size(esa):
    """C3: B=1, Hq=32, Hkv=8, L=131072, D=128 bf16, q/k/v/dO ~ N(0,1): full
    outputs and gradients of the window layer, a mid-depth dilated layer and
    the last layer against the fp32 oracle, plus the checksum identity
    <dQ, Q> == <dK, K> (both equal sum dS * q.k)."""
    g = torch.Generator().manual_seed(0)
    B, Hq, Hkv, L, D = 1, 32, 8, 131072, 128
    q, k, v, do = (randn(B, h, L, D, dtype=torch.bfloat16, gen=g) for h in (Hq, Hkv, Hkv, Hq))
    for layer in (0, 3, 7):
        o, dq, dk, dv = run_module(esa, q, k, v, do, layer, 8, 64)
        ro, rdq, rdk, rdv = run_oracle(q, k, v, do, layer, 8, 64, chunk=2048)
        for got, want, t in zip((o, dq, dk, dv), (ro, rdq, rdk, rdv), ("out", "dq", "dk", "dv")):
            assert_close(got, want, torch.bfloat16, f"C3 l{layer} {t}")
        lhs = (rdq.double() * q.double()).sum()
        rhs = (rdk.double() * k.double()).sum()
        assert abs(lhs - rhs).item() <= 1e-3 * max(1.0, abs(lhs).item())
        ours = (dq.double() * q.double()).sum() - (dk.double() * k.double()).sum()
        assert abs(ours).item() <= 2e-2 * max(1.0, abs(lhs).item())
        # sum over keys of dV equals sum over queries of dO (softmax rows sum to 1)
        sv = dv.double().sum(dim=(2,)).sum(dim=1)
        so = do.double().sum(dim=(2,)).sum(dim=1)
        assert torch.allclose(sv, so, atol=1.0, rtol=2e-2)
        del o, dq, dk, dv, ro, rdq, rdk, rdv
        torch.cuda.empty_cache()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G,w,L,q_len", [(4, 64, 1000, 1000), (4, 97, 333, 333), (8, 64, 517, 517),
                                         (2, 64, 700, 700), (2, 65, 130, 130), (4, 64, 50, 50),
                                         (4, 16, 600, 300), (12, 40, 257, 257)])
def test_window_tensor_core_path(esa, dtype, G, w, L, q_len):
    """Layer 0 (a causal window of w keys) runs on the tcgen05 kernel for
    head_dim 128; it must agree with the CUDA-core gather kernel and with the
    fp32 oracle, including ragged tails, prefill (q_len < kv_len) and windows
    longer than the sequence."""
    g = torch.Generator().manual_seed(G * 1000 + w)
    Hkv, D = 2, 128
    Hq = Hkv * G
    q = randn(1, Hq, q_len, D, dtype=dtype, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dtype, gen=g), randn(1, Hkv, L, D, dtype=dtype, gen=g)
    spec = esa.PatternSpec(0, 8, w)
    o_tc, lse_tc = esa.ops.forward(q, k, v, spec, D ** -0.5)
    o_g, lse_g = esa.ops.forward(q, k, v, spec, D ** -0.5, gather_only=True)
    assert (lse_tc - lse_g).abs().max().item() < 1e-2
    assert (o_tc.float() - o_g.float()).abs().max().item() < 2e-2
    idx, mask, _ = pattern.prepared_indices(Hq, w, 0, 8, L, q_len, L)
    ro, _ = naive.naive_forward(q.float(), k.float(), v.float(), torch.from_numpy(idx).to(DEV),
                                torch.from_numpy(mask).to(DEV), D ** -0.5, G)
    assert_close(o_tc, ro, dtype, f"window G{G} w{w} L{L}")
    lse_ref = naive.lse_rows(q, k, torch.from_numpy(idx).to(DEV), torch.from_numpy(mask).to(DEV),
                             D ** -0.5, G)
    assert (lse_tc.double() / 1.4426950408889634 - lse_ref).abs().max().item() < 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G,w,D,L,layer", [(1, 64, 128, 700, 5), (2, 33, 64, 515, 3), (4, 64, 128, 1000, 7),
                                           (8, 7, 128, 300, 2), (32, 64, 64, 260, 6), (4, 50, 128, 4099, 1)])
def test_tile_forward_matches_gather_forward(esa, dtype, G, w, D, L, layer):
    """The slot-major tile forward (16-bit data, w <= 64) against the per-pair
    gather forward and the fp32 oracle, including odd w and ragged tiles."""
    g = torch.Generator().manual_seed(G * 31 + w + D)
    Hkv = max(2, 8 // G)   # > 4096 (row, head) pairs: above the latency kernel's range
    Hq = Hkv * G
    q = randn(1, Hq, L, D, dtype=dtype, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dtype, gen=g), randn(1, Hkv, L, D, dtype=dtype, gen=g)
    spec = esa.PatternSpec(layer, 8, w)
    o_t, lse_t = esa.ops.forward(q, k, v, spec, D ** -0.5)
    o_g, lse_g = esa.ops.forward(q, k, v, spec, D ** -0.5, gather_only=True)
    assert (lse_t - lse_g).abs().max().item() < 1e-3
    assert (o_t.float() - o_g.float()).abs().max().item() < 2e-2
    idx, mask, _ = pattern.prepared_indices(Hq, w, layer, 8, L, L, L)
    ro, _ = naive.naive_forward(q.float(), k.float(), v.float(), torch.from_numpy(idx).to(DEV),
                                torch.from_numpy(mask).to(DEV), D ** -0.5, G, chunk=1024)
    assert_close(o_t, ro, dtype, f"tile G{G} w{w} D{D} L{L}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G,w,D,L,layer", [(1, 64, 128, 700, 5), (2, 33, 64, 515, 3),
                                           (4, 64, 128, 1000, 7), (8, 7, 128, 300, 2)])
def test_tile_backward_against_oracle(esa, dtype, G, w, D, L, layer):
    """Query-side tile backward (16-bit data, w <= 64, >= 256 rows) through the
    module: all three gradients against the fp32 oracle."""
    g = torch.Generator().manual_seed(G * 17 + w + D)
    Hkv = 2
    Hq = Hkv * G
    q, do = randn(1, Hq, L, D, dtype=dtype, gen=g), randn(1, Hq, L, D, dtype=dtype, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dtype, gen=g), randn(1, Hkv, L, D, dtype=dtype, gen=g)
    o, dq, dk, dv = run_module(esa, q, k, v, do, layer, 8, w)
    ref = run_oracle(q, k, v, do, layer, 8, w)
    for got, want, t in zip((o, dq, dk, dv), ref, ("out", "dq", "dk", "dv")):
        assert_close(got, want, dtype, f"tile bwd G{G} w{w} D{D} {t}")


def test_naive_implementation_returns_reference_weights(esa, naive_small):
    """implementation="naive" returns attn_weights like the reference's naive
    path (:673-680); compared with the weights the reference itself produced."""
    meta_all, arrays = naive_small
    for meta in meta_all:
        name, layer = meta["name"], meta["layer"]
        dtype = torch.float32 if meta["dtype"] == "float32" else torch.bfloat16
        q, k, v = (torch.from_numpy(arrays[f"{name}_{t}"]).to(DEV, dtype) for t in "qkv")
        cp = meta["cache_position"]
        m = esa.ElasticSparseAttention(layer, meta["nl"], meta["Hq"], meta["D"], meta["w"], meta["L"],
                                       num_key_value_heads=meta["Hkv"], implementation="naive")
        out, weights = m(q, k, v, cache_position=None if cp is None else torch.tensor(cp, device=DEV))
        ref = torch.from_numpy(arrays[f"{name}_l{layer}_weights"]).to(DEV)
        assert weights.shape == ref.shape and weights.dtype == dtype
        tol = 1e-5 if dtype == torch.float32 else 2e-2
        assert (weights.float() - ref).abs().max().item() <= tol, name
        assert esa.ElasticSparseAttention(layer, meta["nl"], meta["Hq"], meta["D"], meta["w"],
                                          meta["L"], num_key_value_heads=meta["Hkv"],
                                          implementation="dense")(q, k, v, cache_position=None if cp is None else torch.tensor(cp, device=DEV))[1] is None


@pytest.mark.parametrize("dtype,p", [(torch.float32, 0.3), (torch.bfloat16, 0.1)])
def test_dropout_matches_oracle_with_same_mask(esa, dtype, p):
    """Training-mode dropout of the naive implementation: the keep mask is
    recovered from the returned weights, and outputs and gradients equal the
    oracle run with that mask (so forward and backward use one mask)."""
    g = torch.Generator().manual_seed(21)
    B, Hq, Hkv, L, D, layer = 1, 4, 2, 400, 64, 5
    q, do = randn(B, Hq, L, D, dtype=dtype, gen=g), randn(B, Hq, L, D, dtype=dtype, gen=g)
    k, v = randn(B, Hkv, L, D, dtype=dtype, gen=g), randn(B, Hkv, L, D, dtype=dtype, gen=g)
    m = esa.ElasticSparseAttention(layer, 8, Hq, D, 64, L, num_key_value_heads=Hkv,
                                   attention_dropout=p, implementation="naive").train()
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    out, weights = m(qq, kk, vv)
    out.backward(do.transpose(1, 2).reshape(B, L, Hq * D))
    idx, mask, _ = pattern.prepared_indices(Hq, 64, layer, 8, L, L, L)
    ti, tm = torch.from_numpy(idx).to(DEV), torch.from_numpy(mask).to(DEV)
    keep = (weights != 0) & (tm.unsqueeze(0) > 0)
    frac = 1.0 - keep.float().sum().item() / tm.sum().item()
    assert abs(frac - p) < 0.02, frac
    ro, rw, rdq, rdk, rdv = naive.naive_forward_backward_keep(q, k, v, do, ti, tm, D ** -0.5,
                                                              Hq // Hkv, keep, p)
    o = out.detach().view(B, L, Hq, D).transpose(1, 2)
    assert_close(weights, rw, dtype, "weights")
    for got, want, t in ((o, ro, "out"), (qq.grad, rdq, "dq"), (kk.grad, rdk, "dk"),
                         (vv.grad, rdv, "dv")):
        assert_close(got, want, dtype, f"dropout {t}")
    # eval mode and the triton implementation apply no dropout
    m.eval()
    o_eval, _ = m(q, k, v)
    o_tri, w_tri = esa.ElasticSparseAttention(layer, 8, Hq, D, 64, L, num_key_value_heads=Hkv,
                                              attention_dropout=p).train()(q, k, v)
    assert w_tri is None and torch.allclose(o_eval.float(), o_tri.float(), atol=2e-2)


@pytest.mark.parametrize("dtype,D", [(torch.float32, 128), (torch.float32, 8), (torch.bfloat16, 256),
                                     (torch.bfloat16, 128), (torch.float16, 64), (torch.bfloat16, 16)])
@pytest.mark.parametrize("w,layer,nl", [(64, 7, 8), (5, 2, 4), (300, 3, 8), (32, 0, 8), (1000, 5, 6)])
def test_decode_kernel_matches_gather_and_oracle(esa, dtype, D, w, layer, nl):
    """Few-pair forwards (decode rows) run the latency kernel, whose slots are
    split over the warps of a CTA (several sub-chunks per warp once w > 256):
    against the per-pair gather kernel and the fp32 oracle, output and lse."""
    g = torch.Generator().manual_seed(w + D)
    B, Hq, Hkv, L = 2, 8, 2, 1500
    rows = [L - 1, 0, 777, 31, 1499, 1200]
    q = randn(B, Hq, len(rows), D, dtype=dtype, gen=g)
    k, v = randn(B, Hkv, L, D, dtype=dtype, gen=g), randn(B, Hkv, L, D, dtype=dtype, gen=g)
    spec = esa.PatternSpec(layer, nl, w)
    rt = torch.tensor(rows, device=DEV)
    o_d, lse_d = esa.ops.forward(q, k, v, spec, D ** -0.5, rows=rt)
    o_g, lse_g = esa.ops.forward(q, k, v, spec, D ** -0.5, rows=rt, gather_only=True)
    # the gather kernel sums weights rounded to the input type, this one fp32 weights
    lse_tol = 1e-4 if dtype == torch.float32 else 1e-2
    assert (lse_d - lse_g).abs().max().item() < lse_tol
    idx, mask, _ = pattern.prepared_indices(Hq, w, layer, nl, L, len(rows), L, np.array(rows))
    ti, tm = torch.from_numpy(idx).to(DEV), torch.from_numpy(mask).to(DEV)
    ro, _ = naive.naive_forward(q.float(), k.float(), v.float(), ti, tm, D ** -0.5, Hq // Hkv)
    assert_close(o_d, ro, dtype, f"decode {dtype} D{D} w{w}")
    assert_close(o_g, ro, dtype, f"gather {dtype} D{D} w{w}")
    lse_ref = naive.lse_rows(q, k, ti, tm, D ** -0.5, Hq // Hkv)
    assert (lse_d.double() / 1.4426950408889634 - lse_ref).abs().max().item() < lse_tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G,w,D,L,layer", [(4, 64, 128, 1000, 7), (2, 33, 64, 2100, 3),
                                           (1, 64, 128, 700, 5), (8, 7, 128, 515, 2)])
def test_saved_probs_forward_backward(esa, dtype, G, w, D, L, layer):
    """The tile forward leaves the normalised probabilities (slot-major fp32)
    for the backward, which then skips recomputing the scores: the
    probabilities match the oracle's softmax weights, the forward outputs are
    unchanged, and the gradients match both the recomputing backward and the
    oracle."""
    g = torch.Generator().manual_seed(G * 5 + w + L)
    Hkv = max(2, 8 // G)
    Hq = Hkv * G
    q, do = randn(1, Hq, L, D, dtype=dtype, gen=g), randn(1, Hq, L, D, dtype=dtype, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dtype, gen=g), randn(1, Hkv, L, D, dtype=dtype, gen=g)
    spec = esa.PatternSpec(layer, 8, w)
    scale = D ** -0.5
    pr = esa.ops.probs_buffer(q, k, spec)
    assert pr is not None and pr.shape == (1, Hq, w, L) and pr.dtype == torch.float32
    o1, lse1 = esa.ops.forward(q, k, v, spec, scale, probs=pr)
    o0, lse0 = esa.ops.forward(q, k, v, spec, scale)
    assert torch.equal(o1, o0) and torch.equal(lse1, lse0)
    idx, mask, _ = pattern.prepared_indices(Hq, w, layer, 8, L, L, L)
    ti, tm = torch.from_numpy(idx).to(DEV), torch.from_numpy(mask).to(DEV)
    _, w_ref = naive.naive_forward(q.float(), k.float(), v.float(), ti, tm, scale, G,
                                   chunk=1024, return_weights=True)
    err = (pr.permute(0, 1, 3, 2) - w_ref).abs().max().item()
    assert err < 4e-3, err     # weights rounded to the input type once in the forward
    g1 = esa.ops.backward(q, k, v, o1, lse1, do, spec, scale, probs=pr)
    g0 = esa.ops.backward(q, k, v, o0, lse0, do, spec, scale)
    ref = naive.naive_forward_backward_manual(q.float(), k.float(), v.float(), do.float(), ti, tm,
                                              scale, G)
    for a, b_, r_, t in zip(g1, g0, ref[1:], ("dq", "dk", "dv")):
        assert_close(a, r_, dtype, f"saved probs {t}")
        assert (a.float() - b_.float()).abs().max().item() < 2e-2
    # no probabilities where the forward does not write them (layer 0: tensor cores)
    if D == 128 and G in (2, 4, 8):
        assert esa.ops.probs_buffer(q, k, esa.PatternSpec(0, 8, 64)) is None


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G,w,L,q_len", [(4, 64, 1000, 1000), (4, 97, 333, 333), (8, 64, 517, 517),
                                         (2, 64, 700, 700), (2, 65, 130, 130), (4, 64, 50, 50),
                                         (4, 16, 600, 300), (12, 40, 257, 257), (4, 64, 4099, 4099)])
def test_window_tensor_core_backward(esa, dtype, G, w, L, q_len):
    """Layer 0 backward on the tcgen05 kernels (dQ query-major, dK/dV
    key-major over all heads of a group): against the CUDA-core backward and
    the fp32 oracle, including ragged tiles, prefill (q_len < kv_len), GQA
    group sizes 2..12 and windows longer than the sequence."""
    g = torch.Generator().manual_seed(G * 77 + w + L)
    Hkv, D = 2, 128
    Hq = Hkv * G
    q, do = randn(1, Hq, q_len, D, dtype=dtype, gen=g), randn(1, Hq, q_len, D, dtype=dtype, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dtype, gen=g), randn(1, Hkv, L, D, dtype=dtype, gen=g)
    spec = esa.PatternSpec(0, 8, w)
    o, lse = esa.ops.forward(q, k, v, spec, D ** -0.5)
    esa.ops.device_errors()
    g_tc = esa.ops.backward(q, k, v, o, lse, do, spec, D ** -0.5)
    assert esa.ops.device_errors() == 0
    g_ga = esa.ops.backward(q, k, v, o, lse, do, spec, D ** -0.5, gather_only=True)
    idx, mask, _ = pattern.prepared_indices(Hq, w, 0, 8, L, q_len, L)
    ref = naive.naive_forward_backward_manual(q.float(), k.float(), v.float(), do.float(),
                                              torch.from_numpy(idx).to(DEV),
                                              torch.from_numpy(mask).to(DEV), D ** -0.5, G)
    for a, b_, r_, t in zip(g_tc, g_ga, ref[1:], ("dq", "dk", "dv")):
        assert_close(a, r_, dtype, f"window bwd G{G} w{w} L{L} {t}")
        # the two paths round differently: within one output ulp of each other
        assert ((a.float() - b_.float()).abs() - 2 * HALF_ULP[dtype] * b_.float().abs()).max().item() < 2e-2, t


@pytest.mark.parametrize("dtype,G,L,perm,D", [(torch.bfloat16, 4, 5000, False, 64),
                                              (torch.bfloat16, 4, 5000, False, 128),
                                              (torch.float16, 2, 4100, False, 128),
                                              (torch.float32, 2, 4100, False, 64),
                                              (torch.float32, 4, 3000, True, 64)])
def test_long_runs_split_into_chunks(esa, dtype, G, L, perm, D):
    """alpha = 1 (last layer): head 0's slot 0 sends every query to key 0, and
    other heads' slot 0 has runs of thousands of queries.  Full 1024-slot
    chunks of such runs are summed by the chunk kernel and added by the key
    side (the tensor-core key kernel for 16-bit data in query order, the FMA
    one otherwise); gradients must match the oracle, also with unsorted query
    rows (cache_position, sorted on the host with a permutation)."""
    g = torch.Generator().manual_seed(L + G)
    Hkv, nl = 2, 8
    Hq = Hkv * G
    q, do = randn(1, Hq, L, D, dtype=dtype, gen=g), randn(1, Hq, L, D, dtype=dtype, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dtype, gen=g), randn(1, Hkv, L, D, dtype=dtype, gen=g)
    cp = torch.randperm(L, generator=g).to(DEV) if perm else None
    o, dq, dk, dv = run_module(esa, q, k, v, do, nl - 1, nl, 64, cache_position=cp)
    ref = run_oracle(q, k, v, do, nl - 1, nl, 64, cache_position=cp)
    for got, want, t in zip((o, dq, dk, dv), ref, ("out", "dq", "dk", "dv")):
        assert_close(got, want, dtype, f"long runs {dtype} G{G} L{L} {t}")


@pytest.mark.parametrize("dtype,G,D,layer", [(torch.bfloat16, 4, 128, 5), (torch.float16, 1, 128, 3),
                                             (torch.bfloat16, 8, 64, 7), (torch.bfloat16, 2, 128, 1),
                                             (torch.bfloat16, 3, 128, 4)])
def test_key_side_tensor_core_matches_fma_kernel(esa, dtype, G, D, layer):
    """The tensor-core key side (bf16 / fp16, D = 64 / 128, two query heads of
    a group per launch with fp32 sums between launches -- G = 3 ends with a
    one-head launch -- and (p, dS) as hi + lo terms) against the FMA key
    kernel (``gather_only``) on a longer sequence than the oracle cases: dK /
    dV within two output ulps of each other."""
    from elastic_sparse_attention_b200 import ops
    g = torch.Generator().manual_seed(G * 31 + D + layer)
    Hkv, L, w = 2, 6000, 64
    Hq = Hkv * G
    q, do = randn(1, Hq, L, D, dtype=dtype, gen=g), randn(1, Hq, L, D, dtype=dtype, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dtype, gen=g), randn(1, Hkv, L, D, dtype=dtype, gen=g)
    spec = ops.PatternSpec(layer, 8, w)
    scale = D ** -0.5
    o, lse = ops.forward(q, k, v, spec, scale)
    _, dk_tc, dv_tc = ops.backward(q, k, v, o, lse, do, spec, scale)
    _, dk_ga, dv_ga = ops.backward(q, k, v, o, lse, do, spec, scale, gather_only=True)
    assert ops.device_errors() == 0
    for a, b_, t in ((dk_tc, dk_ga, "dk"), (dv_tc, dv_ga, "dv")):
        diff = (a.float() - b_.float()).abs() - 2 * HALF_ULP[dtype] * b_.float().abs()
        assert diff.max().item() <= 1e-3, (t, diff.max().item())


@pytest.mark.parametrize("layer", [0, 3, 7])
def test_sequence_split_kernel_offsets(esa, layer):
    """The kernel arguments of the sequence split, on one GPU: L = 65536 split
    4 ways into virtual ranks; rank r calls ops.forward / ops.backward on its
    query rows [r*S, (r+1)*S) with row_offset = r*S and K/V sliced to
    [lo_r, (r+1)*S), kv_offset = lo_r (its first key, from the split's plan).
    Per rank, the output, dQ and the partial dK/dV of the buffer rows are
    compared with the oracle run on the same query rows against the whole
    K/V, which also shows that no key below lo_r is read."""
    from elastic_sparse_attention_b200 import sharded
    g = torch.Generator().manual_seed(40 + layer)
    B, Hq, Hkv, L, D, w, world = 1, 8, 2, 65536, 128, 64, 4
    S = L // world
    dt = torch.bfloat16
    q, do = randn(B, Hq, L, D, dtype=dt, gen=g), randn(B, Hq, L, D, dtype=dt, gen=g)
    k, v = randn(B, Hkv, L, D, dtype=dt, gen=g), randn(B, Hkv, L, D, dtype=dt, gen=g)
    spec = esa.PatternSpec(layer, 8, w)
    plan = sharded.make_plan(Hq, spec, S, world, torch.device(DEV))
    scale = D ** -0.5
    esa.ops.device_errors()
    for r in range(world):
        a0, b0 = r * S, (r + 1) * S
        lo = plan.lo[r]
        assert lo <= a0
        qr, dor, kr, vr = q[:, :, a0:b0], do[:, :, a0:b0], k[:, :, lo:b0], v[:, :, lo:b0]
        pr = esa.ops.probs_buffer(qr, kr, spec, row_offset=a0, kv_len=L, kv_offset=lo)
        o, lse = esa.ops.forward(qr, kr, vr, spec, scale, row_offset=a0, kv_len=L, kv_offset=lo,
                                 probs=pr)
        dq, dk, dv = esa.ops.backward(qr, kr, vr, o, lse, dor, spec, scale, row_offset=a0,
                                      kv_len=L, kv_offset=lo, probs=pr)
        idx, mask, _ = pattern.prepared_indices(Hq, w, layer, 8, L, S, L, np.arange(a0, b0))
        ro, rdq, rdk, rdv = naive.naive_forward_backward_manual(
            qr.float(), k.float(), v.float(), dor.float(), torch.from_numpy(idx).to(DEV),
            torch.from_numpy(mask).to(DEV), scale, Hq // Hkv, chunk=2048)
        if lo > 0:
            assert rdk[:, :, :lo].abs().max().item() == 0 and rdv[:, :, :lo].abs().max().item() == 0
        for got, want, t in ((o, ro, "out"), (dq, rdq, "dq"), (dk, rdk[:, :, lo:b0], "dk"),
                             (dv, rdv[:, :, lo:b0], "dv")):
            assert_close(got, want, dt, f"split l{layer} rank {r} {t}")
        del o, lse, dq, dk, dv, ro, rdq, rdk, rdv, pr
    assert esa.ops.device_errors() == 0


@pytest.mark.parametrize("dtype,layer,D", [(torch.bfloat16, 5, 128), (torch.float32, 3, 64),
                                           (torch.bfloat16, 0, 128)])
def test_head_split_matches_all_heads(esa, dtype, layer, D):
    """A call on a subset of the query heads (PatternSpec.heads: the heads
    [head_offset, head_offset + Hq) of a pattern over pattern_heads heads,
    whole GQA groups with their K/V heads) gives exactly the slices of the
    call on all heads: outputs, lse, gradients, and the dropout mask."""
    g = torch.Generator().manual_seed(70 + layer)
    B, Hq, Hkv, L, w = 1, 8, 4, 1100, 64   # > 4096 (row, head) pairs per share: no latency kernel
    G = Hq // Hkv
    q, do = randn(B, Hq, L, D, dtype=dtype, gen=g), randn(B, Hq, L, D, dtype=dtype, gen=g)
    k, v = randn(B, Hkv, L, D, dtype=dtype, gen=g), randn(B, Hkv, L, D, dtype=dtype, gen=g)
    spec = esa.PatternSpec(layer, 8, w)
    scale = D ** -0.5
    o, lse = esa.ops.forward(q, k, v, spec, scale)
    dq, dk, dv = esa.ops.backward(q, k, v, o, lse, do, spec, scale)
    _, _, wts = esa.ops.forward(q, k, v, spec, scale, dropout_p=0.2, dropout_seed=5,
                                return_weights=True)
    for kv0 in range(0, Hkv, 2):   # two shares of two KV heads each
        h0, h1 = kv0 * G, (kv0 + 2) * G
        sub = spec.heads(Hq, h0)
        qs, dos = q[:, h0:h1].contiguous(), do[:, h0:h1].contiguous()
        ks, vs = k[:, kv0:kv0 + 2].contiguous(), v[:, kv0:kv0 + 2].contiguous()
        os_, lses = esa.ops.forward(qs, ks, vs, sub, scale)
        dqs, dks, dvs = esa.ops.backward(qs, ks, vs, os_, lses, dos, sub, scale)
        assert torch.equal(os_, o[:, h0:h1]) and torch.equal(lses, lse[:, h0:h1])
        assert torch.equal(dqs, dq[:, h0:h1])
        assert torch.equal(dks, dk[:, kv0:kv0 + 2]) and torch.equal(dvs, dv[:, kv0:kv0 + 2])
        _, _, ws = esa.ops.forward(qs, ks, vs, sub, scale, dropout_p=0.2, dropout_seed=5,
                                   return_weights=True)
        assert torch.equal(ws, wts[:, h0:h1])


def test_head_sharded_module_matches_full_module(esa):
    """HeadShardedElasticSparseAttention on each of 4 emulated ranks (one GPU)
    gives its heads' columns of the full module's output and its heads'
    gradients, bit for bit."""
    g = torch.Generator().manual_seed(12)
    B, Hq, Hkv, L, D, layer = 1, 16, 4, 1500, 128, 6
    dt = torch.bfloat16
    q, do = randn(B, Hq, L, D, dtype=dt, gen=g), randn(B, Hq, L, D, dtype=dt, gen=g)
    k, v = randn(B, Hkv, L, D, dtype=dt, gen=g), randn(B, Hkv, L, D, dtype=dt, gen=g)
    full = run_module(esa, q, k, v, do, layer, 8, 64)
    world = 4
    for r in range(world):
        h0, nh, kv0, nkv = esa.head_share(Hq, Hkv, r, world)
        m = esa.HeadShardedElasticSparseAttention(layer, 8, Hq, D, 64, L, num_key_value_heads=Hkv,
                                                  rank=r, world_size=world)
        qq = q[:, h0:h0 + nh].clone().requires_grad_(True)
        kk = k[:, kv0:kv0 + nkv].clone().requires_grad_(True)
        vv = v[:, kv0:kv0 + nkv].clone().requires_grad_(True)
        out = m(qq, kk, vv)
        out.backward(do[:, h0:h0 + nh].transpose(1, 2).reshape(B, L, nh * D))
        o = out.detach().view(B, L, nh, D).transpose(1, 2)
        assert torch.equal(o, full[0][:, h0:h0 + nh])
        assert torch.equal(qq.grad, full[1][:, h0:h0 + nh])
        assert torch.equal(kk.grad, full[2][:, kv0:kv0 + nkv])
        assert torch.equal(vv.grad, full[3][:, kv0:kv0 + nkv])


def test_gather_probe_modes(esa):
    """The gather probe (measurement aid) runs in every mode on a tile-kernel
    problem, records no device error, and refuses an unknown mode."""
    import ctypes
    g = torch.Generator().manual_seed(3)
    dt = torch.bfloat16
    q = randn(1, 8, 2048, 128, dtype=dt, gen=g)
    k, v = randn(1, 2, 2048, 128, dtype=dt, gen=g), randn(1, 2, 2048, 128, dtype=dt, gen=g)
    lib = esa._lib.load()
    pb = esa.ops._problem(q, k, esa.PatternSpec(5, 8, 64), 128 ** -0.5, None, 0, 2048, 0)
    sink = torch.zeros(4, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    esa.ops.device_errors()
    for mode in range(4):
        rc = lib.esa_probe_gather(mode, ctypes.byref(pb), esa._lib.tensor4(k), esa._lib.tensor4(v),
                                  sink.data_ptr(), stream)
        assert rc == 0, lib.esa_last_error()
    torch.cuda.synchronize()
    assert esa.ops.device_errors() == 0
    assert lib.esa_probe_gather(4, ctypes.byref(pb), esa._lib.tensor4(k), esa._lib.tensor4(v),
                                sink.data_ptr(), stream) == -1


@pytest.mark.parametrize("layer,G,D,gather_only", [(5, 4, 128, False), (3, 1, 64, False),
                                                   (0, 4, 128, False), (6, 2, 128, True)])
def test_fp32_key_gradients(esa, layer, G, D, gather_only):
    """ESA_FLAG_F32_DKV (``dkv_fp32``): every key-side writer (tensor-core key
    kernel with and without fp32 sums between launches, the FMA key kernel,
    the window layer's dK/dV kernel) writes the unrounded sums; rounded to the
    input dtype they are the 16-bit results bit for bit, and dq is unchanged."""
    g = torch.Generator().manual_seed(layer * 5 + G)
    dt, Hkv, L, w = torch.bfloat16, 2, 2100, 64
    q, do = randn(1, Hkv * G, L, D, dtype=dt, gen=g), randn(1, Hkv * G, L, D, dtype=dt, gen=g)
    k, v = randn(1, Hkv, L, D, dtype=dt, gen=g), randn(1, Hkv, L, D, dtype=dt, gen=g)
    spec = esa.PatternSpec(layer, 8, w)
    scale = D ** -0.5
    o, lse = esa.ops.forward(q, k, v, spec, scale, gather_only=gather_only)
    dq, dk, dv = esa.ops.backward(q, k, v, o, lse, do, spec, scale, gather_only=gather_only)
    dq32, dk32, dv32 = esa.ops.backward(q, k, v, o, lse, do, spec, scale, gather_only=gather_only,
                                        dkv_fp32=True)
    assert dk32.dtype == torch.float32 and dv32.dtype == torch.float32
    assert torch.equal(dq32, dq)
    assert torch.equal(dk32.to(dt), dk) and torch.equal(dv32.to(dt), dv)
    assert esa.ops.device_errors() == 0


def test_graft_smoke(esa):
    """The repository's smoke check (module forward + backward of a dilated
    and the sliding-window layer against the oracle) as part of the suite."""
    import __graft_entry__
    __graft_entry__.smoke()
