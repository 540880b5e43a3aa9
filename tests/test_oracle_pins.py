"""CPU: pin the oracle against outputs of the reference itself (tests/golden).

The fixtures were produced by ``tests/golden/make_golden.py`` from the
reference's own module and scripts; these tests check the restatements in
``oracle/`` reproduce them, so the GPU parity tests can trust the oracle.
"""
import hashlib

import numpy as np
import pytest
import torch

from conftest import parse_key
from oracle import holes, naive, pattern, pattern_c


def _digest(idx, mask):
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(idx, dtype="<i8").tobytes())
    h.update(np.ascontiguousarray(mask, dtype="<i8").tobytes())
    return h.hexdigest()


def test_small_patterns_bit_exact(pattern_small):
    keys = sorted(k[:-4] for k in pattern_small if k.endswith("_idx"))
    assert len(keys) >= 12
    for key in keys:
        L, H, w, nl, layer = parse_key(key)
        idx, mask = pattern.elastic_indices(np.arange(L), H, w, layer, nl)
        np.testing.assert_array_equal(idx, pattern_small[key + "_idx"], err_msg=key)
        np.testing.assert_array_equal(mask, pattern_small[key + "_mask"], err_msg=key)
        ci, cm = pattern_c.elastic_indices(np.arange(L), H, w, layer, nl)
        np.testing.assert_array_equal(ci, idx, err_msg=key)
        np.testing.assert_array_equal(cm, mask, err_msg=key)


@pytest.mark.parametrize("prefix", ["L4096_H4_w64_nl8", "L4096_H32_w64_nl4"])
def test_digests_numpy(pattern_digests, prefix):
    keys = [k for k in pattern_digests["digests"] if k.startswith(prefix + "_")]
    assert keys
    for key in keys:
        L, H, w, nl, layer = parse_key(key)
        idx, mask = pattern.elastic_indices(np.arange(L), H, w, layer, nl)
        assert _digest(idx, mask) == pattern_digests["digests"][key], key


@pytest.mark.parametrize("key", ["L32768_H32_w64_nl8_l1", "L32768_H32_w64_nl8_l5",
                                 "L131072_H32_w64_nl8_l0", "L131072_H32_w64_nl8_l7",
                                 "L1048576_H2_w64_nl8_l3", "L1048576_H2_w64_nl8_l6"])
def test_digests_c_large(pattern_digests, key):
    L, H, w, nl, layer = parse_key(key)
    idx, mask = pattern_c.elastic_indices(np.arange(L), H, w, layer, nl)
    assert _digest(idx, mask) == pattern_digests["digests"][key]


def test_generator_copies_agree(pattern_digests):
    """The module's generator, check_attn_hole's copy and vis_attn_mask's copy
    (its mask inverted) agree, as recorded from the reference's own code."""
    agree = pattern_digests["generator_agreement"]
    assert len(agree) >= 6
    for key, flags in agree.items():
        assert all(flags.values()), (key, flags)


def test_hole_known_answers(holes_cases):
    """check_attn_hole.py's three __main__ cases (plus two small ones)."""
    assert {(c["attn_length"], c["position_id"], c["unreachable"]) for c in holes_cases[:3]} == \
        {(64, 131071, 0), (64, 4095, 0), (16, 32767, 501)}
    for c in holes_cases:
        got = holes.unreachable_count(c["seq_len"], c["num_hidden_layers"],
                                      c["num_attention_heads"], c["attn_length"], c["position_id"])
        assert got == c["unreachable"], c


@pytest.mark.parametrize("L,H,w,nl", [(4096, 4, 64, 8), (4096, 32, 64, 4), (2000, 5, 16, 3),
                                      (700, 3, 100, 6)])
def test_pattern_invariants(L, H, w, nl):
    """Causality (vis_attn_mask.py:97), full rows from i >= w-1, ascending
    valid indices with no repeats."""
    for layer in range(nl):
        idx, mask = pattern.elastic_indices(np.arange(L), H, w, layer, nl)
        m = mask.astype(bool)
        pos = np.arange(L)[None, :, None]
        assert not np.any(m & (idx > pos))
        assert m[:, w - 1:, :].all()
        v = np.where(m, idx, -1)
        d = np.diff(v, axis=-1)
        assert np.all((d > 0) | (v[..., 1:] == -1) | (v[..., :-1] == -1))


@pytest.mark.parametrize("H,L,w,nl", [(4, 4096, 64, 8), (32, 32768, 64, 8), (32, 131072, 64, 8),
                                      (32, 262144, 64, 4), (16, 1048576, 64, 8)])
def test_slot_columns_monotone(H, L, w, nl):
    """The key-side enumeration of the backward needs every (head, slot)
    index column non-decreasing along positions (and it steps by at most 1)."""
    for layer in range(nl):
        bad, step = pattern_c.audit_monotone(H, L, w, layer, nl)
        assert bad == 0, (layer, bad)
        assert step <= 2, (layer, step)


def _run_case(meta, arrays, dtype=torch.float32):
    name, layer = meta["name"], meta["layer"]
    q = torch.from_numpy(arrays[f"{name}_q"]).to(dtype)
    k = torch.from_numpy(arrays[f"{name}_k"]).to(dtype)
    v = torch.from_numpy(arrays[f"{name}_v"]).to(dtype)
    do = torch.from_numpy(arrays[f"{name}_do"]).to(dtype)
    Hq, Hkv, L = meta["Hq"], meta["Hkv"], meta["L"]
    idx, mask, _ = pattern.prepared_indices(Hq, meta["w"], layer, meta["nl"], L, q.shape[2], L,
                                            meta["cache_position"])
    out, dq, dk, dv = naive.naive_forward_backward(
        q, k, v, do, torch.from_numpy(idx), torch.from_numpy(mask), naive.default_scale(meta["D"]),
        Hq // Hkv, chunk=17)
    return out, dq, dk, dv


def test_naive_oracle_matches_reference(naive_small):
    meta_all, arrays = naive_small
    for meta in meta_all:
        if meta["dtype"] != "float32":
            continue
        out, dq, dk, dv = _run_case(meta, arrays)
        pre = f"{meta['name']}_l{meta['layer']}"
        B, Hq, n, D = out.shape
        ref_out = arrays[pre + "_out"].reshape(B, n, Hq, D).transpose(0, 2, 1, 3)
        np.testing.assert_allclose(out.numpy(), ref_out, atol=1e-6, rtol=0, err_msg=pre)
        np.testing.assert_allclose(dq.numpy(), arrays[pre + "_dq"], atol=1e-5, rtol=0, err_msg=pre)
        np.testing.assert_allclose(dk.numpy(), arrays[pre + "_dk"], atol=1e-5, rtol=0, err_msg=pre)
        np.testing.assert_allclose(dv.numpy(), arrays[pre + "_dv"], atol=1e-5, rtol=0, err_msg=pre)
        if pre + "_dense_out" in arrays:
            np.testing.assert_allclose(arrays[pre + "_dense_out"], arrays[pre + "_out"], atol=1e-5)


def test_naive_oracle_bf16_close_to_reference_bf16(naive_small):
    meta_all, arrays = naive_small
    for meta in meta_all:
        if meta["dtype"] != "bfloat16":
            continue
        out, *_ = _run_case(meta, arrays, torch.bfloat16)
        pre = f"{meta['name']}_l{meta['layer']}"
        B, Hq, n, D = out.shape
        ref_out = arrays[pre + "_out"].reshape(B, n, Hq, D).transpose(0, 2, 1, 3)
        np.testing.assert_allclose(out.float().numpy(), ref_out, atol=2e-2)


def test_c1_oracle_rows(c1_rows):
    """C1 (B1 H4 L4096 D64 fp32, seed 0, w=64, 8 layers): the oracle's output
    equals the reference naive output on the recorded rows."""
    torch.manual_seed(0)
    B, H, L, D = 1, 4, 4096, 64
    q, k, v = torch.randn(B, H, L, D), torch.randn(B, H, L, D), torch.randn(B, H, L, D)
    rows = c1_rows["rows"]
    for layer in (0, 3, 7):
        idx, mask, _ = pattern.prepared_indices(H, 64, layer, 8, L, L, L)
        sel = torch.from_numpy(rows)
        out, _ = naive.naive_forward(q[:, :, sel], k, v, torch.from_numpy(idx[:, rows]),
                                     torch.from_numpy(mask[:, rows]), D ** -0.5, 1)
        got = out.transpose(1, 2).reshape(len(rows), H * D).numpy()
        np.testing.assert_allclose(got, c1_rows[f"l{layer}"], atol=1e-6, rtol=0)


@pytest.mark.parametrize("B,Hq,Hkv,L,D,w,layer,nl,cpos", [
    (1, 4, 2, 150, 16, 16, 2, 4, None), (2, 3, 1, 90, 32, 7, 1, 3, None),
    (1, 2, 2, 128, 32, 64, 5, 8, [127, 3, 64, 64])])
def test_manual_backward_equals_autograd(B, Hq, Hkv, L, D, w, layer, nl, cpos):
    """The hand-written backward of the oracle (used for full-size GPU checks)
    equals autograd through the naive ops (itself pinned to the reference)."""
    g = torch.Generator().manual_seed(7)
    n = L if cpos is None else len(cpos)
    q, k, v = (torch.randn(B, Hq, n, D, generator=g), torch.randn(B, Hkv, L, D, generator=g),
               torch.randn(B, Hkv, L, D, generator=g))
    do = torch.randn(B, Hq, n, D, generator=g)
    idx, mask, _ = pattern.prepared_indices(Hq, w, layer, nl, L, n, L, cpos)
    ti, tm = torch.from_numpy(idx), torch.from_numpy(mask)
    a = naive.naive_forward_backward(q, k, v, do, ti, tm, D ** -0.5, Hq // Hkv)
    b = naive.naive_forward_backward_manual(q, k, v, do, ti, tm, D ** -0.5, Hq // Hkv, chunk=33)
    for x, y in zip(a, b):
        np.testing.assert_allclose(x.numpy(), y.numpy(), atol=2e-5, rtol=0)
