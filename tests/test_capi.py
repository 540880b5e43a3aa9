"""CPU: the C-ABI library loads, exports every symbol the header declares, its
struct layout matches the ctypes mirror, and argument validation reports
errors without touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "esa_b200.h")
HEADERS = (HEADER, os.path.join(ROOT, "include", "esa_layer.h"))


def header_functions():
    names = set()
    for path in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(path).read(), flags=re.S)
        names |= set(re.findall(r"\b(esa_[a-z_0-9]+)\s*\(", text))
    return sorted(names)


def test_library_exports_header_symbols(esa):
    lib = esa._lib.load()
    names = header_functions()
    assert set(names) == set(esa._lib.EXPORTED), names
    for name in names:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", esa._lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (esa_\w+)", out))
    assert set(names) <= exported


def test_struct_layout_matches_header(tmp_path, esa):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "esa_b200.h"\n'
        "int main(void){\n"
        ' printf("%zu %zu %zu %zu %zu %zu %zu\\n", sizeof(esa_problem_t),'
        " offsetof(esa_problem_t, q_len), offsetof(esa_problem_t, rows),"
        " offsetof(esa_problem_t, scale), sizeof(esa_tensor_t),"
        " offsetof(esa_tensor_t, stride_s), offsetof(esa_problem_t, row_offset));\n"
        ' printf(" %zu %zu %zu %zu %zu\\n", offsetof(esa_problem_t, dropout_seed),'
        " offsetof(esa_problem_t, weights), offsetof(esa_problem_t, probs),"
        " offsetof(esa_problem_t, head_offset), offsetof(esa_problem_t, pattern_heads));\n"
        ' printf(" %zu %zu\\n", offsetof(esa_problem_t, key_plan),'
        " offsetof(esa_problem_t, key_plan_bytes));\n"
        " return 0; }\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)],
                   check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    P, T = esa._lib.EsaProblem, esa._lib.EsaTensor
    want = [ctypes.sizeof(P), P.q_len.offset, P.rows.offset, P.scale.offset, ctypes.sizeof(T),
            T.stride_s.offset, P.row_offset.offset, P.dropout_seed.offset, P.weights.offset,
            P.probs.offset, P.head_offset.offset, P.pattern_heads.offset, P.key_plan.offset,
            P.key_plan_bytes.offset]
    assert got == want


def _problem(esa, **kw):
    base = dict(dtype=esa._lib.DTYPES[__import__("torch").bfloat16], batch=1, num_heads=4,
                num_kv_heads=2, head_dim=128, attn_length=64, layer_idx=3, num_hidden_layers=8,
                q_len=16, kv_len=16, kv_offset=0, kv_rows=16, row_offset=0, rows=None,
                scale=128 ** -0.5, flags=0, dropout_p=0.0, head_offset=0, dropout_seed=0,
                weights=None, probs=None, pattern_heads=0, reserved=0, key_plan=None,
                key_plan_bytes=0)
    base.update(kw)
    return esa._lib.EsaProblem(**base)


def _plan_bytes(segs, ntiles, seg_users, seg_heavy):
    a = lambda x: (x + 255) // 256 * 256
    return a(32 * 8) + 2 * a(segs * (ntiles + 1) * 4) + a(segs * seg_users * 4) + \
        a(segs * seg_heavy * 4)


def test_key_plan_size(esa):
    """The key plan's size (host-side: no device work) and where it applies:
    one segment per (KV head, launch of 2 query heads of a group), a tile per
    4 keys, at most one record per (query, head, slot)."""
    lib = esa._lib.load()
    size = lambda **kw: lib.esa_key_plan_size(ctypes.byref(_problem(esa, **kw)))
    L = 4096
    # G = 2: one launch per KV head
    assert size(q_len=L, kv_len=L, kv_rows=L) == _plan_bytes(2, L // 4, 2 * 64 * L, 2 * 64 * 4)
    # G = 4 (8 query / 2 KV heads): two launches of 2 heads per KV head
    assert size(num_heads=8, q_len=L, kv_len=L, kv_rows=L) == \
        _plan_bytes(4, L // 4, 2 * 64 * L, 2 * 64 * 4)
    # MHA: one head per launch
    assert size(num_kv_heads=4, q_len=L, kv_len=L, kv_rows=L) == \
        _plan_bytes(4, L // 4, 64 * L, 64 * 4)
    # no plan: the tensor-core window backward (layer 0, G = 4), fp32, other
    # head_dim, explicit rows, the gather-only flag, an empty call
    assert size(num_heads=8, layer_idx=0, q_len=L, kv_len=L, kv_rows=L) == 0
    assert size(dtype=esa._lib.DTYPES[__import__("torch").float32], q_len=L, kv_len=L,
                kv_rows=L) == 0
    assert size(head_dim=32, q_len=L, kv_len=L, kv_rows=L) == 0
    assert size(rows=1 << 20, q_len=L, kv_len=L, kv_rows=L) == 0
    assert size(flags=1, q_len=L, kv_len=L, kv_rows=L) == 0
    assert size(q_len=0) == 0


def test_backward_rejects_mismatched_key_plan(esa):
    lib = esa._lib.load()
    L = 4096
    pb = _problem(esa, q_len=L, kv_len=L, kv_rows=L, key_plan=1 << 20, key_plan_bytes=12345)
    t = esa._lib.EsaTensor(1 << 20, 4096, 1024, 128)
    ws = lib.esa_backward_workspace_size(ctypes.byref(pb))
    rc = lib.esa_backward(ctypes.byref(pb), t, t, t, t, 1 << 20, t, t, t, t, None, None,
                          1 << 20, ws, None)
    assert rc == -1 and "key_plan" in lib.esa_last_error().decode()


@pytest.mark.parametrize("kw,code,frag", [
    (dict(num_kv_heads=3), -1, "divisible"),
    (dict(head_dim=48), -2, "head_dim"), (dict(head_dim=4), -2, "head_dim"),
    (dict(attn_length=0), -2, "attention_length"),
    (dict(attn_length=4096), -2, "attention_length"),
    (dict(kv_len=1 << 25), -2, "2^24"),
    (dict(dtype=7), -1, "dtype"),
    (dict(scale=float("inf")), -1, "scale"),
    (dict(head_offset=1), -1, "head_offset"),
    (dict(head_offset=2, pattern_heads=5), -1, "head_offset"),
    (dict(head_offset=-1, pattern_heads=8), -1, "head_offset"),
])
def test_forward_rejects_bad_problems(esa, kw, code, frag):
    lib = esa._lib.load()
    pb = _problem(esa, **kw)
    t = esa._lib.EsaTensor(16, 0, 0, 0)
    rc = lib.esa_forward(ctypes.byref(pb), t, t, t, t, 16, None)
    assert rc == code
    assert frag in lib.esa_last_error().decode()


def test_forward_rejects_misaligned_tensor(esa):
    lib = esa._lib.load()
    pb = _problem(esa)
    good = esa._lib.EsaTensor(1 << 20, 4096, 1024, 128)
    bad = esa._lib.EsaTensor((1 << 20) + 2, 4096, 1024, 128)
    assert lib.esa_forward(ctypes.byref(pb), bad, good, good, good, 1 << 20, None) == -1
    assert "16-byte" in lib.esa_last_error().decode()
    odd = esa._lib.EsaTensor(1 << 20, 4096, 1024, 3)
    assert lib.esa_forward(ctypes.byref(pb), good, odd, good, good, 1 << 20, None) == -1
    assert "strides" in lib.esa_last_error().decode()


def test_backward_workspace_and_checks(esa):
    lib = esa._lib.load()
    pb = _problem(esa)
    need = lib.esa_backward_workspace_size(ctypes.byref(pb))
    # (p, dS) per (batch, head, slot, row) + fp32 dK/dV accumulators for GQA
    assert need == (1 * 4 * 64 * 16 * 8) + (2 * 1 * 2 * 16 * 128 * 4)
    t = esa._lib.EsaTensor(1 << 20, 4096, 1024, 128)
    rc = lib.esa_backward(ctypes.byref(pb), t, t, t, t, 1 << 20, t, t, t, t, None, None,
                          1 << 20, need - 1, None)
    assert rc == -4 and "workspace" in lib.esa_last_error().decode()
    rc = lib.esa_backward(ctypes.byref(pb), t, t, t, t, 1 << 20, t, t, t, t, 1 << 21, None,
                          1 << 20, need, None)
    assert rc == -1 and "together" in lib.esa_last_error().decode()


def test_empty_query_is_a_noop(esa):
    lib = esa._lib.load()
    pb = _problem(esa, q_len=0)
    t = esa._lib.EsaTensor(16, 0, 0, 0)
    assert lib.esa_forward(ctypes.byref(pb), t, t, t, t, 16, None) == 0


def test_pattern_rejects_bad_rows(esa):
    lib = esa._lib.load()
    assert lib.esa_pattern(4, 64, 0, 8, 1 << 25, None, 0, 0, 16, 16, None) == -1
    assert lib.esa_pattern(4, 0, 0, 8, 16, None, 0, 0, 16, 16, None) == -1
    assert lib.esa_pattern(4, 64, 0, 8, 0, None, 0, 0, None, None, None) == 0


@pytest.mark.parametrize("kw,want", [
    (dict(), 0),                                          # 16 rows: the latency kernel
    (dict(q_len=4096, kv_len=4096, kv_rows=4096), 1),     # tile kernel
    (dict(q_len=4096, kv_len=4096, kv_rows=4096, layer_idx=0), 0),   # tensor-core window
    (dict(q_len=4096, kv_len=4096, kv_rows=4096, dtype=0), 0),       # fp32: gather kernels
    (dict(q_len=4096, kv_len=4096, kv_rows=4096, dropout_p=0.1), 0),
    (dict(q_len=4096, kv_len=4096, kv_rows=4096, attn_length=65), 0),
    (dict(num_kv_heads=3), -1),
])
def test_forward_writes_probs_query(esa, kw, want):
    """Which forward paths leave their probabilities for the backward (a host
    decision, no GPU needed)."""
    lib = esa._lib.load()
    assert lib.esa_forward_writes_probs(ctypes.byref(_problem(esa, **kw))) == want


def test_rows_struct_layout_matches_header(tmp_path, esa):
    src = tmp_path / "rows.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "esa_b200.h"\n'
        "int main(void){\n"
        ' printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(esa_rows_t), offsetof(esa_rows_t, src_dtype),'
        " offsetof(esa_rows_t, row_elems), offsetof(esa_rows_t, count),"
        " offsetof(esa_rows_t, src_stride), offsetof(esa_rows_t, dst_stride));\n"
        " return 0; }\n")
    exe = tmp_path / "rows"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)],
                   check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    R = esa._lib.EsaRows
    assert got == [ctypes.sizeof(R), R.src_dtype.offset, R.row_elems.offset, R.count.offset,
                   R.src_stride.offset, R.dst_stride.offset]


def _rows(esa, **kw):
    r = esa._lib.EsaRows()
    r.src, r.dst, r.src_dtype, r.dst_dtype, r.row_elems = 1 << 20, 1 << 21, 1, 1, 64
    for i, (n, s, d) in enumerate([(2, 4096, 4096), (3, 256, 256), (4, 64, 64)]):
        r.count[i], r.src_stride[i], r.dst_stride[i] = n, s, d
    for key, val in kw.items():
        if isinstance(val, tuple):
            getattr(r, key)[val[0]] = val[1]
        else:
            setattr(r, key, val)
    return r


@pytest.mark.parametrize("kw,code,frag", [
    (dict(src_dtype=1, dst_dtype=2), -2, "dtypes"),
    (dict(src_dtype=2, dst_dtype=0), -2, "dtypes"),
    (dict(src_dtype=0, dst_dtype=0), -2, "dtypes"),
    (dict(row_elems=60), -1, "multiple of 8"),
    (dict(row_elems=0), -1, "multiple of 8"),
    (dict(src_stride=(1, 260)), -1, "16-byte"),
    (dict(dst_stride=(2, 4)), -1, "16-byte"),
    (dict(count=(0, -1)), -1, "negative"),
    (dict(src=(1 << 20) + 8), -1, "misaligned"),
    (dict(dst=None), -1, "null"),
])
def test_copy_rows_rejects_bad_descriptors(esa, kw, code, frag):
    """Checked before any CUDA call (no GPU needed)."""
    lib = esa._lib.load()
    r = _rows(esa, **kw)
    assert lib.esa_copy_rows(ctypes.byref(r), None) == code
    assert frag in lib.esa_last_error().decode()


def test_copy_rows_empty_grid_is_a_noop(esa):
    lib = esa._lib.load()
    assert lib.esa_copy_rows(ctypes.byref(_rows(esa, count=(1, 0))), None) == 0
    # fp32 -> bf16 with fp32 strides that are 16-byte multiples (4 elements)
    r = _rows(esa, src_dtype=0, dst_dtype=1, src_stride=(2, 4), count=(2, 0))
    assert lib.esa_copy_rows(ctypes.byref(r), None) == 0
