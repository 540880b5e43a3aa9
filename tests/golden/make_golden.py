"""Generate the golden fixtures in this directory from the reference itself.

Run in a container where the reference checkout is present (it is not needed,
and not read, anywhere else):

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

Everything written here comes from executing the reference's own code:

* ``pattern_small.npz``  explicit ``sparse_attention_indices`` /
  ``sparse_causal_mask`` buffers of ``ElasticSparseAttention`` for small
  configurations (``elastic_sparse_attention.py:465-468``).
* ``pattern_digests.json``  SHA-256 of those buffers (int64, little endian,
  indices then mask) for the benchmark-sized configurations, plus agreement
  flags between the module's generator and the two copies in
  ``check_attn_hole.py:5-51`` and ``vis_attn_mask.py:17-61``.
* ``holes.json``  unreachable-position counts of the receptive-field check of
  ``check_attn_hole.py:53-180`` for its three ``__main__`` cases
  (``:185-234``), computed on the CPU with the reference's own generator.
* ``naive_small.npz``  inputs, outputs and autograd gradients of the
  reference's ``implementation="naive"`` path (``:624-680``) and outputs of
  ``implementation="dense"`` (``:682-726``) for small seeded cases.  The naive
  path needs one harness-side shim: it calls
  ``_get_prepared_indices_and_mask(q_len, kv_len)`` (``:638``) on a method
  that takes only ``kv_len`` (``:574``), so the shim drops the first argument.
* ``c1_rows.npz``  sampled output rows of the naive path at the CPU-runnable
  configuration (B=1, H=4, L=4096, D=64, fp32, seed 0, w=64, 8 layers).
"""
from __future__ import annotations

import argparse
import ast
import hashlib
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(path):
    sys.path.insert(0, path)
    import elastic_sparse_attention as esa  # noqa: E402
    import check_attn_hole as cah  # noqa: E402
    # vis_attn_mask imports matplotlib at module level; pull out only its
    # generator and config class by parsing the file.
    src = open(os.path.join(path, "vis_attn_mask.py")).read()
    tree = ast.parse(src)
    keep = [n for n in tree.body
            if isinstance(n, (ast.ClassDef, ast.FunctionDef))
            and n.name in ("MockConfig", "_create_elastic_sparse_indices")]
    ns = {"torch": torch, "Tuple": __import__("typing").Tuple}
    exec(compile(ast.Module(body=keep, type_ignores=[]), "vis_attn_mask.py", "exec"), ns)
    return esa, cah, ns


def shim_naive(module):
    orig = module._get_prepared_indices_and_mask
    module._get_prepared_indices_and_mask = lambda *args: orig(args[-1])
    return module


def digest(idx: torch.Tensor, mask: torch.Tensor) -> str:
    h = hashlib.sha256()
    h.update(idx.to(torch.int64).contiguous().numpy().astype("<i8").tobytes())
    h.update(mask.to(torch.int64).contiguous().numpy().astype("<i8").tobytes())
    return h.hexdigest()


SMALL_PATTERNS = [
    # (L, H, w, nl, layers)
    (256, 4, 16, 4, [0, 1, 2, 3]),
    (130, 3, 64, 8, [0, 4, 7]),
    (200, 1, 32, 1, [0]),
    (300, 2, 7, 3, [1]),
    (512, 8, 32, 12, [0, 6, 11]),
    (96, 5, 100, 2, [1]),
]

DIGEST_PATTERNS = [
    (4096, 4, 64, 8, list(range(8))),
    (4096, 32, 64, 4, list(range(4))),
    (32768, 32, 64, 8, list(range(8))),
    (131072, 32, 64, 8, list(range(8))),
    (1048576, 2, 64, 8, list(range(8))),
]


def make_patterns(esa, cah, vis):
    arrays = {}
    for (L, H, w, nl, layers) in SMALL_PATTERNS:
        for layer in layers:
            m = esa.ElasticSparseAttention(layer, nl, H, 16, w, L, implementation="naive")
            key = f"L{L}_H{H}_w{w}_nl{nl}_l{layer}"
            arrays[key + "_idx"] = m.sparse_attention_indices.numpy().astype(np.int32)
            arrays[key + "_mask"] = m.sparse_causal_mask.numpy().astype(np.int8)
    np.savez_compressed(os.path.join(HERE, "pattern_small.npz"), **arrays)

    digests = {}
    for (L, H, w, nl, layers) in DIGEST_PATTERNS:
        for layer in layers:
            t0 = time.time()
            m = esa.ElasticSparseAttention(layer, nl, H, 16, w, L, implementation="naive")
            key = f"L{L}_H{H}_w{w}_nl{nl}_l{layer}"
            digests[key] = digest(m.sparse_attention_indices, m.sparse_causal_mask)
            del m
            print("digest", key, f"{time.time() - t0:.1f}s", flush=True)

    # agreement of the three generator copies at the configurations the
    # reference's scripts use (vis: L=512, 8 heads, k=32, 12 layers; holes: w=64)
    agree = {}
    for (L, H, w, nl, layer) in [(512, 8, 32, 12, 0), (512, 8, 32, 12, 6), (512, 8, 32, 12, 11),
                                 (4096, 4, 64, 8, 3), (4096, 8, 64, 8, 7), (4096, 8, 16, 8, 5)]:
        m = esa.ElasticSparseAttention(layer, nl, H, 16, w, L, implementation="naive")
        mi, mm = m.sparse_attention_indices, m.sparse_causal_mask
        ci, cm = cah.create_elastic_sparse_indices_for_validation(L, layer, nl, H, w,
                                                                   torch.device("cpu"))
        vi, vm = vis["_create_elastic_sparse_indices"](vis["MockConfig"](nl, H, w), layer, L, "cpu")
        agree[f"L{L}_H{H}_w{w}_nl{nl}_l{layer}"] = {
            "check_attn_hole_equal": bool(torch.equal(ci * cm, mi) and torch.equal(cm, mm)),
            "vis_indices_equal_where_valid": bool(torch.equal(vi * mm, mi)),
            "vis_mask_is_complement": bool(torch.equal(vm.long(), 1 - mm)),
        }
    with open(os.path.join(HERE, "pattern_digests.json"), "w") as f:
        json.dump({"digests": digests, "generator_agreement": agree}, f, indent=1, sort_keys=True)


def hole_count(cah, seq_len, nl, H, w, pos):
    """check_attn_hole.py:88-171 on the CPU, with the reference's generator."""
    dev = torch.device("cpu")
    history = pos + 1
    reach = torch.zeros(history, dtype=torch.bool)
    idx, mask = cah.create_elastic_sparse_indices_for_validation(seq_len, nl - 1, nl, H, w, dev)
    reach[idx[:, pos, :][mask[:, pos, :].bool()].unique()] = True
    reach[pos] = True
    for layer in range(nl - 2, -1, -1):
        idx, mask = cah.create_elastic_sparse_indices_for_validation(seq_len, layer, nl, H, w, dev)
        src = torch.where(reach)[0]
        new = idx[:, src, :][mask[:, src, :].bool()].unique()
        reach[new[new < history]] = True
        if int(reach.sum()) == history:
            break
    return int(history - reach.sum())


def make_holes(cah):
    cases = [(131072, 8, 8, 64, 131071), (131072, 8, 8, 64, 4095), (131072, 8, 8, 16, 32767),
             (4096, 4, 4, 16, 4095), (8192, 6, 4, 8, 8191)]
    out = []
    for (L, nl, H, w, pos) in cases:
        t0 = time.time()
        n = hole_count(cah, L, nl, H, w, pos)
        out.append({"seq_len": L, "num_hidden_layers": nl, "num_attention_heads": H,
                    "attn_length": w, "position_id": pos, "unreachable": n})
        print("holes", out[-1], f"{time.time() - t0:.1f}s", flush=True)
    with open(os.path.join(HERE, "holes.json"), "w") as f:
        json.dump(out, f, indent=1)


NAIVE_CASES = [
    # name, B, Hq, Hkv, L, D, w, nl, layers, dtype, cache_position
    ("mha_f32", 1, 2, 2, 128, 32, 64, 8, [0, 3, 7], torch.float32, None),
    ("gqa_f32", 2, 4, 2, 96, 16, 16, 4, [2], torch.float32, None),
    ("w7_f32", 1, 3, 1, 80, 16, 7, 3, [1], torch.float32, None),
    ("decode_f32", 1, 2, 2, 128, 32, 64, 8, [5], torch.float32, [127, 3, 64]),
    ("mha_bf16", 1, 2, 2, 96, 32, 32, 8, [6], torch.bfloat16, None),
]


def make_naive(esa):
    arrays = {}
    meta = []
    for (name, B, Hq, Hkv, L, D, w, nl, layers, dtype, cpos) in NAIVE_CASES:
        g = torch.Generator().manual_seed(0)
        q = torch.randn(B, Hq, L if cpos is None else len(cpos), D, generator=g)
        k = torch.randn(B, Hkv, L, D, generator=g)
        v = torch.randn(B, Hkv, L, D, generator=g)
        do = torch.randn(B, Hq, q.shape[2], D, generator=g)
        arrays[f"{name}_q"], arrays[f"{name}_k"] = q.numpy(), k.numpy()
        arrays[f"{name}_v"], arrays[f"{name}_do"] = v.numpy(), do.numpy()
        for layer in layers:
            m = shim_naive(esa.ElasticSparseAttention(layer, nl, Hq, D, w, L, num_key_value_heads=Hkv,
                                                      implementation="naive"))
            qq, kk, vv = (t.to(dtype).detach().clone().requires_grad_(True) for t in (q, k, v))
            cp = None if cpos is None else torch.tensor(cpos, dtype=torch.long)
            out, weights = m(qq, kk, vv, cache_position=cp)
            qlen = q.shape[2]
            out.backward(do.to(dtype).transpose(1, 2).reshape(B, qlen, Hq * D))
            pre = f"{name}_l{layer}"
            arrays[pre + "_out"] = out.detach().float().numpy()
            arrays[pre + "_weights"] = weights.detach().float().numpy()
            arrays[pre + "_dq"] = qq.grad.float().numpy()
            arrays[pre + "_dk"] = kk.grad.float().numpy()
            arrays[pre + "_dv"] = vv.grad.float().numpy()
            if cpos is None:
                md = esa.ElasticSparseAttention(layer, nl, Hq, D, w, L, num_key_value_heads=Hkv,
                                                implementation="dense")
                od, _ = md(q.to(dtype), k.to(dtype), v.to(dtype))
                arrays[pre + "_dense_out"] = od.detach().float().numpy()
            meta.append({"name": name, "layer": layer, "B": B, "Hq": Hq, "Hkv": Hkv, "L": L, "D": D,
                         "w": w, "nl": nl, "dtype": str(dtype).replace("torch.", ""),
                         "cache_position": cpos})
    np.savez_compressed(os.path.join(HERE, "naive_small.npz"), **arrays)
    with open(os.path.join(HERE, "naive_small.json"), "w") as f:
        json.dump(meta, f, indent=1)


def make_c1_rows(esa):
    """C1: B=1, H=4, L=4096, D=64, fp32, q/k/v ~ N(0,1) from seed 0, w=64, 8 layers."""
    torch.manual_seed(0)
    B, H, L, D = 1, 4, 4096, 64
    q = torch.randn(B, H, L, D)
    k = torch.randn(B, H, L, D)
    v = torch.randn(B, H, L, D)
    rows = np.unique(np.concatenate([np.arange(0, 70), np.arange(4030, 4096),
                                     np.random.default_rng(1).integers(0, L, 120)]))
    arrays = {"rows": rows}
    for layer in range(8):
        m = shim_naive(esa.ElasticSparseAttention(layer, 8, H, D, 64, L, implementation="naive"))
        with torch.no_grad():
            out, _ = m(q, k, v)
        arrays[f"l{layer}"] = out[0, rows].numpy()
        print("c1 layer", layer, flush=True)
    np.savez_compressed(os.path.join(HERE, "c1_rows.npz"), **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default="patterns,holes,naive,c1")
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    esa, cah, vis = load_reference(args.reference)
    only = args.only.split(",")
    if "patterns" in only:
        make_patterns(esa, cah, vis)
    if "holes" in only:
        make_holes(cah)
    if "naive" in only:
        make_naive(esa)
    if "c1" in only:
        make_c1_rows(esa)


if __name__ == "__main__":
    main()
