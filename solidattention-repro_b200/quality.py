"""Selection quality from the dense audit (host side, numpy).

Follows audit_dense_selection (cpp/src/pipeline_main.cpp:502-574) per
(sequence-layer, KV head): the selected mass is the dense attention mass of
the selected blocks (plus the always-attended open tail); the oracle set is
the forced blocks ([0, init) and the last `local`) filled up to the budget by
the remaining blocks in descending mass (a stable sort, ties to the lower
block), and the oracle recall is the fraction of that set the selection
holds. With planted hot blocks, hot recall is the fraction of them selected.
"""
from __future__ import annotations

import numpy as np


def selection_quality(mass, selected, counts, num_sealed, budget: int, init: int, local: int,
                      hot=None) -> dict:
    """mass [S*L][KH][table+1]; selected [S*L][groups][budget]; counts
    [S*L][groups]; num_sealed [S*L]; hot (optional) [S*L][KH][n_hot] block ids.
    KV head h uses selection group h * groups // KH."""
    mass = np.asarray(mass, np.float64)
    selected = np.asarray(selected)
    counts = np.asarray(counts)
    n_sl, kh, width = mass.shape
    groups = selected.shape[1]
    sel_mass, recall, hot_recall = [], [], []
    for sl in range(n_sl):
        nb = int(num_sealed[sl])
        if nb <= 0:
            continue
        eff = min(budget, nb)
        n_init = min(init, nb)
        n_local = min(local, nb)
        forced = set(range(n_init)) | set(range(nb - n_local, nb))
        for h in range(kh):
            g = h * groups // kh
            ids = selected[sl, g, :int(counts[sl, g])].astype(np.int64)
            m = mass[sl, h, :nb]
            sel_mass.append(float(m[ids].sum() + mass[sl, h, width - 1]))
            order = np.argsort(-m, kind="stable")
            oracle = set(forced)
            for b in order:
                if len(oracle) >= eff:
                    break
                oracle.add(int(b))
            recall.append(len(oracle & set(ids.tolist())) / max(1, len(oracle)))
            if hot is not None:
                hb = [int(x) for x in np.asarray(hot)[sl, h] if 0 <= int(x) < nb]
                if hb:
                    hot_recall.append(len(set(hb) & set(ids.tolist())) / len(hb))
    out = {"selected_mass": float(np.mean(sel_mass)) if sel_mass else None,
           "oracle_recall": float(np.mean(recall)) if recall else None,
           "units": len(sel_mass)}
    if hot is not None:
        out["hot_recall"] = float(np.mean(hot_recall)) if hot_recall else None
    return out
