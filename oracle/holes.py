"""Receptive-field ("attention hole") check, restated on the CPU.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``check_attn_hole.py:53-180``: start from the target row's direct keys
at the last layer (``:102-114``), then walk layers ``nl-2 .. 0`` adding every
valid key of every currently reachable row (``:134-156``), stopping early on
full coverage (``:161-163``).  The returned count is ``history_len -
reachable`` (``:170-171``).  The generator used is the C restatement of
``create_elastic_sparse_indices_for_validation`` (``check_attn_hole.py:5-51``),
whose valid set equals the module's (its mask adds ``idx >= 0``, which always
holds).
"""
from __future__ import annotations

import numpy as np

from . import pattern_c


def unreachable_count(seq_len: int, num_hidden_layers: int, num_heads: int,
                      attn_length: int, position_id: int | None = None,
                      rows_per_call: int = 1 << 15) -> int:
    target = seq_len - 1 if position_id is None else position_id
    if not 0 <= target < seq_len:
        raise ValueError(f"position_id must be between 0 and {seq_len - 1}")
    history = target + 1
    reach = np.zeros(history, dtype=bool)

    def keys_of(rows: np.ndarray, layer: int) -> np.ndarray:
        found = []
        for r0 in range(0, len(rows), rows_per_call):
            part = rows[r0:r0 + rows_per_call]
            idx, mask = pattern_c.elastic_indices(part, num_heads, attn_length, layer,
                                                  num_hidden_layers)
            found.append(np.unique(idx[mask.astype(bool)]))
        return np.unique(np.concatenate(found)) if found else np.zeros(0, np.int64)

    last = num_hidden_layers - 1
    reach[keys_of(np.array([target]), last)] = True
    reach[target] = True
    for layer in range(num_hidden_layers - 2, -1, -1):
        src = np.nonzero(reach)[0]
        new = keys_of(src, layer)
        reach[new[new < history]] = True
        if reach.all():
            break
    return int(history - reach.sum())
