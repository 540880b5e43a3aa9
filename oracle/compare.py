"""Comparison of kernel outputs with the fp32 oracle (test infrastructure).

Only tests/, __graft_entry__.smoke() and bench.py's baseline legs use this
package; the product path never imports it.

Tolerances of the parity contract: fp32 within max-abs 1e-4 of the fp32
restatement of the reference's fallback path (elastic_sparse_attention.py
:624-680); bf16 / fp16 outputs and gradients within max-abs 2e-2 and
mean-abs 2e-3 of it.  A 16-bit result is a stored value: from |x| = 8 up
(bf16) even the correctly rounded value is more than 2e-2 from the fp32
value.  So an element's error is the smaller of its distance to the fp32
oracle (the contract as written) and its distance to the oracle rounded to
the output dtype (the storage-aware form), both held to the same flat
bounds.  In the rounded form, an oracle value that sits (within 1e-4
relative) on the midpoint between two neighbouring 16-bit values may round
either way, and the element counts as exact.
"""
from __future__ import annotations

import torch

F32_MAX = 1e-4
LOW_MAX, LOW_MEAN = 2e-2, 2e-3
MIDPOINT_REL = 1e-4


def errors(got: torch.Tensor, want: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Elementwise error of ``got`` against the fp32 oracle ``want``: for
    16-bit results the smaller of |got - oracle| and |got - oracle rounded to
    dtype| (rounding-midpoint ties counted as exact)."""
    want = want.float()
    got = got.float()
    direct = (got - want).abs()
    if dtype == torch.float32:
        return direct
    want_r = want.to(dtype).float()
    rounded = (got - want_r).abs()
    tie = (want - 0.5 * (got + want_r)).abs() <= MIDPOINT_REL * want.abs()
    rounded = torch.where(tie, torch.zeros_like(rounded), rounded)
    return torch.minimum(direct, rounded)


def within(got: torch.Tensor, want: torch.Tensor, dtype: torch.dtype) -> tuple[bool, float, float]:
    """(passes, max error, mean error) under the contract's bounds for ``dtype``."""
    err = errors(got, want, dtype)
    mx = err.max().item() if err.numel() else 0.0
    mean = err.mean().item() if err.numel() else 0.0
    if dtype == torch.float32:
        return mx <= F32_MAX, mx, mean
    return (mx <= LOW_MAX and mean <= LOW_MEAN), mx, mean
