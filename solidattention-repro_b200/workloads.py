"""Synthetic decode workloads with the shapes of the path's benchmark configs.

No dataset is involved: every input is seeded synthetic data generated on
the device (torch's CUDA generator; values FP16 N(0,1), rounded to nearest
even), the same recipe for every config:

* prompt KV: FP16 N(0,1) rows for Nb sealed 32-token blocks per
  (sequence, layer);
* planted hot blocks: for each (layer, KV head) a seeded set of non-forced
  blocks whose keys get +0.5 * q_hat, q_hat = the L2-normalised mean of the
  KV head's G base decode queries (FP32 add, then RNE to FP16);
* representatives: the online-seal build (window 32, top-4) of every block
  from seeded N(0,1) FP16 per-token prompt queries;
* decode step s: query = fp16(0.8 * q_base + 0.6 * z_s), z_s ~ N(0,1) (so
  the query stays N(0,1) and correlated with the planted blocks); the new
  token's K/V are FP16 N(0,1); tokens pre-filled into the open tails follow
  the same recipe from their own seeded stream.

Each generator function below produces one piece for one (sequence, layer)
from its own seed, so any subset of sequences, layers or KV heads can be
rebuilt on its own with the values the whole workload has.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np
import torch

from . import DecodeContext

BLOCK = 32
D = 128


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    query_heads: int
    kv_heads: int
    layers: int
    seqs: int
    context_blocks: int   # sealed blocks at the start (context / 32)
    budget_blocks: int
    init_blocks: int
    local_blocks: int
    hot_blocks: int
    out_fp16: bool = True
    # variable context: when > 0, sequence b's context is a seeded uniform
    # draw in [context_min_blocks, context_blocks] blocks (context_blocks is
    # then the maximum); batch = sequences of the whole box
    context_min_blocks: int = 0
    batch: int = 1

    def sequence_blocks(self, global_seq: int) -> int:
        """Sealed blocks of sequence `global_seq` at the start of decoding."""
        if self.context_min_blocks <= 0:
            return self.context_blocks
        tokens = np.random.default_rng(7_000_003 + global_seq).integers(
            self.context_min_blocks * BLOCK, self.context_blocks * BLOCK + 1)
        return int(max(self.context_min_blocks, min(self.context_blocks, round(tokens / BLOCK))))

    @property
    def group(self) -> int:
        return self.query_heads // self.kv_heads

    def selected_kv_bytes(self, tail_tokens: int = 0) -> int:
        """Algorithmic selected-KV bytes of one decode step (all layers, seqs)."""
        per_token = 2 * self.kv_heads * D * 2
        sel = min(self.budget_blocks, self.context_blocks)
        return self.seqs * self.layers * (sel * BLOCK + tail_tokens) * per_token

    def rep_bytes(self, blocks: int | None = None) -> int:
        """Algorithmic representative bytes scanned by one step's scoring."""
        nb = self.context_blocks if blocks is None else blocks
        return self.seqs * self.layers * self.query_heads * nb * D * 4


# The path's benchmark configs (context in 32-token blocks, budgets in blocks).
CONFIGS = {
    "cfg1": Workload("cfg1-qwen3-0.6b-1layer-2k-budget512", 16, 8, 1, 1, 64, 16, 1, 2, 0),
    "cfg2": Workload("cfg2-qwen3-0.6b-28layer-16k-budget2048", 16, 8, 28, 1, 512, 64, 1, 4, 8),
    "cfg3": Workload("cfg3-qwen3-8b-36layer-32k-budget4096", 32, 8, 36, 1, 1024, 128, 1, 4, 16),
    "cfg5": Workload("cfg5-qwen3-8b-36layer-128k-budget8192", 32, 8, 36, 1, 4096, 256, 1, 8, 32),
    # batch of 64 sequences with 8K..32K contexts, 8 sequences per GPU (the
    # per-GPU share of the batch on 8 GPUs; the whole batch needs >180 GB)
    "cfg4": Workload("cfg4-qwen3-8b-36layer-batch64-8k-32k-budget2048", 32, 8, 36, 8, 1024, 64, 1,
                     4, 0, context_min_blocks=256, batch=64),
}


def _seed_base(seed: int) -> int:
    return seed * 1000003


def base_queries(w: Workload, seed: int, global_seq: int, device: torch.device) -> torch.Tensor:
    """The sequence's base decode queries [layers][QH][D] FP32 (FP16 values)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(_seed_base(seed) + 17 + 104729 * global_seq)
    return torch.randn(w.layers, w.query_heads, D, device=device, generator=gen).half().float()


def hot_blocks(w: Workload, seed: int, global_seq: int) -> np.ndarray:
    """Planted hot block ids [layers][KH][hot] of a sequence (sorted per row),
    drawn from the non-forced blocks."""
    nb = w.sequence_blocks(global_seq)
    hot = np.zeros((w.layers, w.kv_heads, w.hot_blocks), np.int64)
    rng = np.random.default_rng((seed, global_seq))
    candidates = np.arange(w.init_blocks, nb - w.local_blocks)
    for layer in range(w.layers):
        for h in range(w.kv_heads):
            ids = rng.choice(candidates, size=min(w.hot_blocks, len(candidates)), replace=False)
            hot[layer, h, :len(ids)] = np.sort(ids)
    return hot


def prompt_kv(w: Workload, seed: int, global_seq: int, layer: int, q_base_layer: torch.Tensor,
              hot: np.ndarray, device: torch.device) -> torch.Tensor:
    """Token-major prompt rows [nb*32][2][KH][D] FP16 of one (sequence, layer),
    every KV head, with the hot blocks of `hot` [KH][n] planted (+0.5*q_hat on
    their keys; q_hat from q_base_layer [QH][D])."""
    nb = w.sequence_blocks(global_seq)
    gen = torch.Generator(device=device)
    gen.manual_seed(_seed_base(seed) + (global_seq * w.layers + layer) * 7919 + 1)
    kv = torch.randn(nb * BLOCK, 2, w.kv_heads, D, device=device, generator=gen).half()
    for h in range(w.kv_heads):
        ids = hot[h]
        if w.hot_blocks == 0 or len(ids) == 0:
            continue
        grp = q_base_layer[h * w.group:(h + 1) * w.group].mean(0)
        q_hat = grp / grp.norm()
        rows = (torch.as_tensor(ids, device=device)[:, None] * BLOCK +
                torch.arange(BLOCK, device=device)[None, :]).reshape(-1)
        kv[rows, 0, h] = (kv[rows, 0, h].float() + 0.5 * q_hat).half()
    return kv


def prompt_queries(w: Workload, seed: int, global_seq: int, layer: int,
                   device: torch.device) -> torch.Tensor:
    """Per-token prompt queries [QH][nb*32][D] FP32 (FP16 values) of one
    (sequence, layer): the input of its representatives' build."""
    nb = w.sequence_blocks(global_seq)
    gen = torch.Generator(device=device)
    gen.manual_seed(_seed_base(seed) + (global_seq * w.layers + layer) * 7919 + 2)
    return torch.randn(w.query_heads, nb * BLOCK, D, device=device, generator=gen).half().float()


def tail_tokens(w: Workload, seed: int, global_seq: int, q_base: torch.Tensor, count: int,
                device: torch.device):
    """`count` already-decoded tail tokens of a sequence, every layer: queries
    [count][layers][QH][D] FP32 (the decode recipe around q_base [layers][QH][D])
    and K/V rows [count][layers][2][KH][D] FP16."""
    gen = torch.Generator(device=device)
    gen.manual_seed(_seed_base(seed) + 31337 + 104729 * global_seq)
    z = torch.randn(count, w.layers, w.query_heads, D, device=device, generator=gen)
    q = (0.8 * q_base[None] + 0.6 * z).half().float()
    kv = torch.randn(count, w.layers, 2, w.kv_heads, D, device=device, generator=gen).half()
    return q, kv


def tail_for_seal_at_end(steps: int, warmup: int = 0) -> int:
    """Tokens to pre-fill into every open tail so that the last of `warmup`
    untimed plus `steps` timed decode steps fills the tail and seals it (a
    32-token block seals on the step that appends its 32nd token)."""
    return (-(warmup + steps)) % BLOCK


def seal_steps(initial_tail: int, first: int, count: int) -> int:
    """Seals among decode steps [first, first + count) of a context whose tails
    started with `initial_tail` tokens."""
    return sum(1 for i in range(first, first + count) if (initial_tail + i) % BLOCK == BLOCK - 1)


def make_context(w: Workload, decode_steps: int, device: torch.device, seed: int = 0,
                 kv_heads_slice: tuple[int, int] | None = None,
                 seq_offset: int = 0, initial_tail: int = 0,
                 layer_ids: list[int] | None = None) -> tuple[DecodeContext, dict]:
    """Build a DecodeContext holding workload `w`, ready for `decode_steps` steps.

    kv_heads_slice=(first, count) keeps only those KV heads (and their query
    heads) on this device: the KV-head sharding of a long single sequence.
    seq_offset = the global batch index of this context's first sequence
    (sequence sharding of a batch: context lengths follow the global index).
    initial_tail (0..31) = tokens already decoded into every open tail.
    layer_ids = the workload layers this context holds (all by default); a
    subset gets exactly those layers' values.
    Returns (ctx, info) with the base queries, hot block ids and per-sequence
    context blocks.
    """
    if not 0 <= initial_tail < BLOCK:
        raise ValueError("initial_tail must be in [0, 32)")
    layer_ids = list(range(w.layers)) if layer_ids is None else list(layer_ids)
    kh0, khn = kv_heads_slice or (0, w.kv_heads)
    q0, q1 = kh0 * w.group, (kh0 + khn) * w.group
    qh = khn * w.group
    L = len(layer_ids)
    extra = (decode_steps + initial_tail) // BLOCK + 2
    seq_nb = [w.sequence_blocks(seq_offset + s) for s in range(w.seqs)]
    table_blocks = max(seq_nb) + extra
    ctx = DecodeContext(query_heads=qh, kv_heads=khn, layers=L, seqs=w.seqs,
                        pool_blocks=L * sum(nb + extra + 1 for nb in seq_nb),
                        table_blocks=table_blocks, budget_blocks=w.budget_blocks,
                        init_blocks=w.init_blocks, local_blocks=w.local_blocks,
                        out_fp16=w.out_fp16, device=device)
    # Every draw is seeded by (seed, global sequence index, layer), so a
    # sequence shard, a KV-head shard or a layer subset sees exactly the
    # values of the whole batch. Base decode queries cover the full head set.
    q_base = torch.empty(w.seqs, L, qh, D, device=device)
    hot = np.zeros((w.seqs, L, w.kv_heads, w.hot_blocks), np.int64)
    tail_q = torch.empty(initial_tail, w.seqs, L, qh, D, device=device)
    tail_kv = torch.empty(initial_tail, w.seqs, L, 2, khn, D, dtype=torch.float16, device=device)
    for s in range(w.seqs):
        gs = seq_offset + s
        nb = seq_nb[s]
        qb_full = base_queries(w, seed, gs, device)
        q_base[s] = qb_full[layer_ids, q0:q1]
        hot_all = hot_blocks(w, seed, gs)
        hot[s] = hot_all[layer_ids]
        for li, layer in enumerate(layer_ids):
            phys = ctx.prefill(s, li, nb)
            base = int(phys[0])
            assert (phys[:nb] == np.arange(base, base + nb)).all()
            kv = prompt_kv(w, seed, gs, layer, qb_full[layer], hot_all[layer], device)
            kv = kv[:, :, kh0:kh0 + khn]
            ctx.pool[base:base + nb] = kv.reshape(nb, BLOCK, 2, khn, D).permute(0, 3, 2, 1, 4)
            del kv
            pq = prompt_queries(w, seed, gs, layer, device)[q0:q1].contiguous()
            ctx.build_reps(s, li, 0, nb, pq, window=32, topk=4, per_block=True)
            del pq
        if initial_tail:
            tq, tkv = tail_tokens(w, seed, gs, qb_full, initial_tail, device)
            tail_q[:, s] = tq[:, layer_ids, q0:q1]
            tail_kv[:, s] = tkv[:, layer_ids, :, kh0:kh0 + khn]
    for t in range(initial_tail):
        ctx.append(tail_q[t].contiguous(), tail_kv[t].contiguous())
    ctx.sync()
    return ctx, {"q_base": q_base, "hot": hot, "qh_local": qh, "kv_heads_local": khn,
                 "seq_blocks": seq_nb, "initial_tail": initial_tail, "layer_ids": layer_ids,
                 "tail_q": tail_q, "tail_kv": tail_kv}


def decode_inputs(w: Workload, info: dict, steps: int, device: torch.device, seed: int = 0,
                  kv_heads_slice: tuple[int, int] | None = None):
    """Per-step queries [steps][S][L][QH][D] FP32 and new K/V [steps][S][L][2][KH][D] FP16
    (L = the context's layers, info["layer_ids"])."""
    kh0, khn = kv_heads_slice or (0, w.kv_heads)
    layer_ids = info.get("layer_ids", list(range(w.layers)))
    gen = torch.Generator(device=device)
    gen.manual_seed(_seed_base(seed) + 99)
    q_base = info["q_base"]
    z = torch.randn(steps, w.seqs, w.layers, w.query_heads, D, device=device, generator=gen)
    z = z[:, :, layer_ids, kh0 * w.group:(kh0 + khn) * w.group]
    queries = (0.8 * q_base[None] + 0.6 * z).half().float().contiguous()
    kv = torch.randn(steps, w.seqs, w.layers, 2, w.kv_heads, D, device=device, generator=gen).half()
    kv = kv[:, :, layer_ids, :, kh0:kh0 + khn].contiguous()
    return queries, kv


def scale() -> float:
    return 1.0 / math.sqrt(D)
