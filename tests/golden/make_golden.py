"""Generate the golden vectors under tests/golden/ from the reference itself.

Run in a container that has the reference tree (its root given by --reference,
else SA_REFERENCE_ROOT, else a checkout named `reference` beside this
repository) and the compiled
reference (oracle/_ref, built by `python __graft_entry__.py build`):

    python tests/golden/make_golden.py [--reference <reference root>]

Outputs (small, committed; the GPU box has no reference tree):

* golden_ref.npz -- the outputs of the reference's own C++
  (cpp/src/attention_reference.cpp, cpp/src/selection.cpp, compiled from its
  sources) on the seeded cases of cases.py: attention, shared/per-KV-head
  selection (ids and scores), representatives (values and chosen offsets),
  with a SHA-256 of each case's inputs;
* python_twins.json -- the reference's Python twins on their own test inputs
  (tests/test_selection.py, tests/test_kv_lifecycle.py) and on a small seeded
  case: local_causal_token_scores masses, select_blocks picks, LayerTail seal
  indices and tail lengths.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def make_ref_vectors(ref) -> dict:
    """Outputs of the compiled reference on the seeded cases, plus input digests."""
    from cases import (ATTENTION, REPRESENTATIVES, SCALE, SELECTION, attention_case, digest,
                       representatives_case, selection_case)

    out = {}
    for i in range(len(ATTENTION)):
        kv, q, tokens, qh, kh = attention_case(i)
        out[f"attn{i}_sha"] = np.array(digest(kv, q))
        out[f"attn{i}_out"] = ref.attention(kv, q, tokens, qh, kh, 128, SCALE).ravel()
    for i in range(len(SELECTION)):
        q, reps, qh, group, blocks, budget, init, local = selection_case(i)
        ids, scores = ref.select_grouped(q, reps, qh, group, blocks, 128, budget, init, local)
        out[f"sel{i}_sha"] = np.array(digest(q, reps))
        out[f"sel{i}_ids"] = ids
        out[f"sel{i}_scores"] = scores
    for i in range(len(REPRESENTATIVES)):
        kv, pq, tokens, qh, kh, window, topk = representatives_case(i)
        vals, offs = ref.build_representatives(pq, kv, tokens, qh, kh, 128, 32, window, topk)
        out[f"rep{i}_sha"] = np.array(digest(kv, pq))
        out[f"rep{i}_values"] = vals
        out[f"rep{i}_offsets"] = offs
    return out


def make_python_twins(reference: Path) -> dict:
    sys.path.insert(0, str(reference / "src"))
    import torch
    from solidattention_lab.kv_lifecycle import LayerTail
    from solidattention_lab.selection import local_causal_token_scores, select_blocks

    res = {}
    # tests/test_selection.py:6-12 -- window 1: every key receives mass 1
    q = torch.tensor([[[10.0, 0.0], [0.0, 10.0]]])
    res["window1_scores"] = local_causal_token_scores(q, q.clone(), local_window=1).tolist()
    # tests/test_selection.py:15-23 -- GQA heads are not averaged before scoring
    query = torch.tensor([[[[1.0, 0.0]], [[0.0, 1.0]]]])
    reps = torch.tensor([[[1.0, 0.0], [0.0, 0.1]], [[0.0, 0.1], [0.0, 1.0]]])
    res["gqa_select"] = {"query": query[0, :, 0].tolist(), "reps": reps.tolist(),
                         "chosen": select_blocks(query, reps, 1, 0, 0)}
    # a seeded case: received masses of 4 query heads over 64 tokens, window 8,
    # head_dim 16
    g = torch.Generator().manual_seed(5)
    qq = torch.randn(4, 64, 16, generator=g).half().float()
    kk = torch.randn(2, 64, 16, generator=g).half().float()
    res["masses_case"] = {"query": qq.numpy().astype(np.float16).view(np.uint16).ravel().tolist(),
                          "key": kk.numpy().astype(np.float16).view(np.uint16).ravel().tolist(),
                          "window": 8,
                          "scores": local_causal_token_scores(qq, kk, 8).numpy().ravel().tolist()}
    # tests/test_kv_lifecycle.py:13-37 -- the seal boundary and planted indices
    tail = LayerTail(q_heads=4, kv_heads=2, head_dim=2, local_tokens=32, block_tokens=32, repr_topk=4)
    key = torch.randn(1, 2, 63, 2, generator=g)
    tail.append(key, key.clone())
    tail.add_attention_mass(torch.ones(4, 63))
    res["tail63"] = {"sealed": len(tail.seal_ready()), "length": tail.length}
    tail = LayerTail(q_heads=4, kv_heads=2, head_dim=2, local_tokens=32, block_tokens=32, repr_topk=4)
    key = torch.arange(1 * 2 * 64 * 2, dtype=torch.float32).view(1, 2, 64, 2)
    tail.append(key, -key)
    score = torch.zeros(4, 64)
    score[:, 7], score[:, 9], score[:, 11], score[:, 13] = 10, 9, 8, 7
    tail.add_attention_mass(score)
    sealed = tail.seal_ready()
    res["tail64"] = {"sealed": len(sealed), "length": tail.length,
                     "indices": sealed[0].representative_indices.tolist(),
                     "planted_scores": score[0, :32].tolist()}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    args = ap.parse_args()
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(HERE))
    import oracle

    root = oracle.reference_root_dir(args.reference)
    if root is None:
        raise SystemExit("the reference tree was not found (--reference or SA_REFERENCE_ROOT)")
    oracle.build(root)
    ref = oracle.reference()
    if ref is None:
        raise SystemExit("oracle/_ref was not built: the reference tree is required")
    np.savez_compressed(HERE / "golden_ref.npz", **make_ref_vectors(ref))
    (HERE / "python_twins.json").write_text(json.dumps(make_python_twins(Path(root))))
    print("wrote", HERE / "golden_ref.npz", HERE / "python_twins.json")


if __name__ == "__main__":
    main()
