"""GPU: the device pattern kernel is bit-exact with the reference buffers."""
import hashlib

import numpy as np
import pytest
import torch

from conftest import parse_key
from oracle import pattern, pattern_c

pytestmark = pytest.mark.gpu


def _digest_dev(idx: torch.Tensor, mask: torch.Tensor) -> str:
    h = hashlib.sha256()
    h.update(idx.cpu().numpy().astype("<i8").tobytes())
    h.update(mask.cpu().numpy().astype("<i8").tobytes())
    return h.hexdigest()


def test_small_patterns(esa, pattern_small):
    dev = torch.device("cuda", 0)
    for key in sorted(k[:-4] for k in pattern_small if k.endswith("_idx")):
        L, H, w, nl, layer = parse_key(key)
        idx, mask = esa.ops.pattern_indices(H, esa.PatternSpec(layer, nl, w), L, dev)
        np.testing.assert_array_equal(idx.cpu().numpy(), pattern_small[key + "_idx"], err_msg=key)
        np.testing.assert_array_equal(mask.cpu().numpy(), pattern_small[key + "_mask"], err_msg=key)


def test_digests(esa, pattern_digests):
    """Every recorded digest of the reference buffers, up to L=131072 x 32 heads
    and L=2^20 x 2 heads, all layers."""
    dev = torch.device("cuda", 0)
    for key, want in sorted(pattern_digests["digests"].items()):
        L, H, w, nl, layer = parse_key(key)
        idx, mask = esa.ops.pattern_indices(H, esa.PatternSpec(layer, nl, w), L, dev)
        assert _digest_dev(idx, mask) == want, key
        del idx, mask
        torch.cuda.empty_cache()


def test_module_buffers(esa):
    m = esa.ElasticSparseAttention(5, 8, 4, 64, 64, 1000)
    ref_idx, ref_mask = pattern.elastic_indices(np.arange(1000), 4, 64, 5, 8)
    np.testing.assert_array_equal(m.sparse_attention_indices.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(m.sparse_causal_mask.cpu().numpy(), ref_mask)
    idx, mask = m._get_prepared_indices_and_mask(300)
    assert idx.shape == (4, 300, 64)
    full = m.full_attention_mask
    ref_full = pattern.full_mask(1000, 4, 64, 5, 8)
    np.testing.assert_array_equal(full[0].cpu().numpy(), ref_full)


@pytest.mark.parametrize("rows,clamp", [([0, 5, 63, 64, 999, 998, 1], 0),
                                        ([3, 500, 999], 200), (None, 100)])
def test_rows_and_clamp(esa, rows, clamp):
    """Prepared (sliced + clamped) indices as _triton_forward builds them (:600-615)."""
    dev = torch.device("cuda", 0)
    spec = esa.PatternSpec(6, 8, 64)
    r = torch.tensor(rows, device=dev) if rows is not None else None
    n = len(rows) if rows is not None else 100
    idx, mask = esa.ops.pattern_indices(32, spec, n, dev, rows=r, clamp_len=clamp)
    pos = np.array(rows) if rows is not None else np.arange(n)
    ri, rm = pattern.elastic_indices(pos, 32, 64, 6, 8)
    if clamp:
        ri = np.clip(ri, 0, clamp - 1)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_array_equal(mask.cpu().numpy(), rm)


def test_large_rows_against_c_oracle(esa):
    """C5-sized positions (L = 2^20, 16 heads): sampled rows vs the C restatement."""
    dev = torch.device("cuda", 0)
    pos = np.sort(np.random.default_rng(3).choice(1 << 20, 4096, replace=False))
    for layer in range(8):
        spec = esa.PatternSpec(layer, 8, 64)
        idx, mask = esa.ops.pattern_indices(16, spec, len(pos), dev,
                                            rows=torch.from_numpy(pos).to(dev))
        ri, rm = pattern_c.elastic_indices(pos, 16, 64, layer, 8)
        np.testing.assert_array_equal(idx.cpu().numpy(), ri)
        np.testing.assert_array_equal(mask.cpu().numpy(), rm)


@pytest.mark.parametrize("H,L,w,nl", [(32, 131072, 64, 8), (16, 1 << 20, 64, 8), (4, 5000, 7, 3)])
def test_device_audit(esa, H, L, w, nl):
    dev = torch.device("cuda", 0)
    for layer in range(nl):
        assert esa.ops.pattern_audit(H, esa.PatternSpec(layer, nl, w), L, dev) == 0
