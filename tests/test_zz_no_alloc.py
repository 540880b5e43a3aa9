"""GPU: esa_backward_noalloc, the backward entry point that allocates nothing.

Callers that cannot allocate device memory -- a plugin inside a host
application that owns all GPU allocations, or a serving loop that must not
allocate once it runs -- call esa_backward_noalloc, which takes its workspace
from a 16 MiB array built into the library instead of from the caller.  These
tests call it through the C ABI (ctypes) and check it against esa_backward
with a caller-provided workspace, on consecutive calls (the array keeps the
previous call's contents).  The file name sorts last so that a run stopping at
its first failure has already run every other test; the tests also pass when
this file runs alone in a fresh process.
"""
import ctypes

import pytest
import torch

from test_gpu_attention import assert_close

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _noalloc_fn(esa):
    lib = esa._lib.load()
    fn = lib.esa_backward_noalloc
    T, P = esa._lib.EsaTensor, ctypes.c_void_p
    fn.argtypes = [ctypes.POINTER(esa._lib.EsaProblem), T, T, T, T, P, T, T, T, T, P, P, P]
    fn.restype = ctypes.c_int
    return fn


def _case(esa, dtype, B, Hq, Hkv, L, D, layer, seed, rows=None):
    g = torch.Generator().manual_seed(seed)
    n = L if rows is None else len(rows)
    q = torch.randn(B, Hq, n, D, generator=g).to(DEV, dtype)
    k = torch.randn(B, Hkv, L, D, generator=g).to(DEV, dtype)
    v = torch.randn(B, Hkv, L, D, generator=g).to(DEV, dtype)
    do = torch.randn(B, Hq, n, D, generator=g).to(DEV, dtype)
    spec = esa.PatternSpec(layer, 8, 64)
    r = None if rows is None else torch.tensor(rows, device=DEV)
    o, lse = esa.ops.forward(q, k, v, spec, D ** -0.5, rows=r)
    return spec, r, (q, k, v, o, lse, do)


def _run_noalloc(esa, fn, spec, r, tensors, sorted_rows=None, perm=None):
    q, k, v, o, lse, do = tensors
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    pb = esa.ops._problem(q, k, spec, q.shape[-1] ** -0.5, r, 0, k.shape[2], 0)
    t4 = esa._lib.tensor4
    rc = fn(ctypes.byref(pb), t4(q), t4(k), t4(v), t4(o), lse.data_ptr(), t4(do), t4(dq), t4(dk),
            t4(dv), esa._lib.ptr(sorted_rows), esa._lib.ptr(perm),
            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, esa._lib.load().esa_last_error().decode()
    return dq, dk, dv


def test_noalloc_backward_matches_workspace_backward(esa):
    fn = _noalloc_fn(esa)
    cases = [
        dict(dtype=torch.bfloat16, B=1, Hq=8, Hkv=2, L=1000, D=128, layer=5, seed=1),
        dict(dtype=torch.float32, B=2, Hq=4, Hkv=4, L=300, D=64, layer=7, seed=2),
        dict(dtype=torch.bfloat16, B=1, Hq=8, Hkv=2, L=1000, D=128, layer=5, seed=1),
    ]
    for c in cases:   # consecutive calls: the shared array keeps the last call's bytes
        spec, r, t = _case(esa, **c)
        want = esa.ops.backward(*t[:5], t[5], spec, c["D"] ** -0.5)
        got = _run_noalloc(esa, fn, spec, r, t)
        torch.cuda.synchronize()
        for g_, w_ in zip(got, want):
            assert_close(g_, w_, c["dtype"], f"noalloc {c}")


def test_noalloc_backward_decode_rows(esa):
    """Unsorted cache_position rows: the caller passes the sorted positions and
    the permutation, as with esa_backward."""
    fn = _noalloc_fn(esa)
    rows = [250, 3, 3, 128, 64, 299]
    for _ in range(2):
        spec, r, t = _case(esa, torch.float32, 2, 8, 2, 300, 64, 5, seed=3, rows=rows)
        srt, perm = torch.sort(r, stable=True)
        want = esa.ops.backward(*t[:5], t[5], spec, 64 ** -0.5, rows=r, sorted_rows=srt,
                                row_perm=perm)
        got = _run_noalloc(esa, fn, spec, r, t, sorted_rows=srt, perm=perm)
        torch.cuda.synchronize()
        for g_, w_ in zip(got, want):
            assert_close(g_, w_, torch.float32, "noalloc decode")


def test_noalloc_rejects_problems_above_the_array(esa):
    fn = _noalloc_fn(esa)
    # 32 heads x 64 slots x 4096 rows x 8 bytes = 64 MiB of workspace > 16 MiB
    pb = esa._lib.problem(dtype=torch.bfloat16, batch=1, num_heads=32, num_kv_heads=8,
                          head_dim=128, attn_length=64, layer_idx=3, num_hidden_layers=8,
                          q_len=4096, kv_len=4096, scale=128 ** -0.5)
    t = esa._lib.EsaTensor(1 << 20, 4096, 1024, 128)
    rc = fn(ctypes.byref(pb), t, t, t, t, 1 << 20, t, t, t, t, None, None, None)
    assert rc == -4
    assert "more than the" in esa._lib.load().esa_last_error().decode()
